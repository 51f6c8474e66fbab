"""Native host runtime classes (C++ scheduler and KV block pool, csrc/runtime)."""
from .ops._ext import require as _require

_m = _require()
Scheduler = _m.Scheduler
SchedulerConfig = _m.SchedulerConfig
SamplingCfg = _m.SamplingCfg
StepPlan = _m.StepPlan
