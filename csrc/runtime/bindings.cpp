// pybind11 bindings of the native host runtime (scheduler + block pool).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "scheduler.h"

namespace py = pybind11;
using namespace b200::rt;

static StepBuffers buffers_from(py::dict d) {
  auto p32 = [&](const char* k) { return reinterpret_cast<int32_t*>(d[k].cast<uintptr_t>()); };
  StepBuffers b;
  b.input_ids = p32("input_ids");
  b.positions = p32("positions");
  b.slot_mapping = p32("slot_mapping");
  b.cu_q = p32("cu_q");
  b.seq_lens = p32("seq_lens");
  b.block_tables = p32("block_tables");
  b.logits_idx = p32("logits_idx");
  b.temperature = reinterpret_cast<float*>(d["temperature"].cast<uintptr_t>());
  b.top_k = p32("top_k");
  b.top_p = reinterpret_cast<float*>(d["top_p"].cast<uintptr_t>());
  b.min_p = reinterpret_cast<float*>(d["min_p"].cast<uintptr_t>());
  b.seeds = reinterpret_cast<int64_t*>(d["seeds"].cast<uintptr_t>());
  b.steps = p32("steps");
  b.state_slots = d.contains("state_slots") ? p32("state_slots") : nullptr;
  b.tree_mask = d.contains("tree_mask")
                    ? reinterpret_cast<int64_t*>(d["tree_mask"].cast<uintptr_t>())
                    : nullptr;
  b.max_tokens = d["max_tokens"].cast<int>();
  b.max_reqs = d["max_reqs"].cast<int>();
  return b;
}

void register_runtime(py::module_& m) {
  py::class_<SamplingCfg>(m, "SamplingCfg")
      .def(py::init<>())
      .def_readwrite("max_tokens", &SamplingCfg::max_tokens)
      .def_readwrite("min_tokens", &SamplingCfg::min_tokens)
      .def_readwrite("ignore_eos", &SamplingCfg::ignore_eos)
      .def_readwrite("eos_id", &SamplingCfg::eos_id)
      .def_readwrite("stop_ids", &SamplingCfg::stop_ids)
      .def_readwrite("temperature", &SamplingCfg::temperature)
      .def_readwrite("top_k", &SamplingCfg::top_k)
      .def_readwrite("top_p", &SamplingCfg::top_p)
      .def_readwrite("min_p", &SamplingCfg::min_p)
      .def_readwrite("seed", &SamplingCfg::seed)
      .def_readwrite("no_prefix_cache", &SamplingCfg::no_prefix_cache)
      .def_readwrite("priority", &SamplingCfg::priority);

  py::class_<SchedulerConfig>(m, "SchedulerConfig")
      .def(py::init<>())
      .def_readwrite("block_size", &SchedulerConfig::block_size)
      .def_readwrite("max_num_seqs", &SchedulerConfig::max_num_seqs)
      .def_readwrite("max_num_batched_tokens", &SchedulerConfig::max_num_batched_tokens)
      .def_readwrite("max_model_len", &SchedulerConfig::max_model_len)
      .def_readwrite("max_blocks_per_seq", &SchedulerConfig::max_blocks_per_seq)
      .def_readwrite("chunked_prefill", &SchedulerConfig::chunked_prefill)
      .def_readwrite("prefix_caching", &SchedulerConfig::prefix_caching)
      .def_readwrite("long_prefill_threshold", &SchedulerConfig::long_prefill_threshold)
      .def_readwrite("priority_policy", &SchedulerConfig::priority_policy);

  py::class_<StepPlan>(m, "StepPlan")
      .def_readonly("num_tokens", &StepPlan::num_tokens)
      .def_readonly("num_reqs", &StepPlan::num_reqs)
      .def_readonly("num_decodes", &StepPlan::num_decodes)
      .def_readonly("num_prefills", &StepPlan::num_prefills)
      .def_readonly("num_prefill_tokens", &StepPlan::num_prefill_tokens)
      .def_readonly("num_samples", &StepPlan::num_samples)
      .def_readonly("max_seq_len", &StepPlan::max_seq_len)
      .def_readonly("num_preempted", &StepPlan::num_preempted)
      .def_readonly("all_greedy", &StepPlan::all_greedy)
      .def_readonly("any_filter", &StepPlan::any_filter)
      .def_readonly("sample_req_ids", &StepPlan::sample_req_ids)
      .def_readonly("sample_counts", &StepPlan::sample_counts)
      .def_readonly("num_spec_tokens", &StepPlan::num_spec_tokens)
      .def_readonly("tree", &StepPlan::tree)
      .def_readonly("req_ids", &StepPlan::req_ids);

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init([](const SchedulerConfig& c, int num_blocks, py::dict bufs) {
             return new Scheduler(c, num_blocks, buffers_from(bufs));
           }),
           py::arg("config"), py::arg("num_blocks"), py::arg("buffers"))
      .def("add_request", &Scheduler::add_request)
      .def("abort_request", &Scheduler::abort_request)
      .def("schedule", &Scheduler::schedule, py::call_guard<py::gil_scoped_release>())
      .def("update",
           [](Scheduler& s, uintptr_t sampled_ptr, int n) {
             return s.update(reinterpret_cast<const int64_t*>(sampled_ptr), n);
           })
      .def("has_unfinished", &Scheduler::has_unfinished)
      .def("num_waiting", &Scheduler::num_waiting)
      .def("num_running", &Scheduler::num_running)
      .def("num_free_blocks", &Scheduler::num_free_blocks)
      .def("step_index", &Scheduler::step_index)
      .def("output_tokens", &Scheduler::output_tokens)
      .def("forget", &Scheduler::forget)
      .def("propose_ngram", &Scheduler::propose_ngram, py::arg("k"), py::arg("n_min") = 1,
           py::arg("n_max") = 4)
      .def("set_draft", &Scheduler::set_draft)
      .def("set_draft_tree", &Scheduler::set_draft_tree, py::arg("id"), py::arg("tokens"),
           py::arg("parents"))
      .def("propose_ngram_tree", &Scheduler::propose_ngram_tree, py::arg("k"),
           py::arg("n_min") = 1, py::arg("n_max") = 4, py::arg("width") = 2)
      .def("take_kv_moves", &Scheduler::take_kv_moves)
      .def("last_path", &Scheduler::last_path)
      .def("reserve_slots", &Scheduler::reserve_slots)
      .def("block_ids", &Scheduler::block_ids)
      .def("decode_request_ids", &Scheduler::decode_request_ids)
      .def("tokens_range", &Scheduler::tokens_range)
      .def("num_tokens", &Scheduler::num_tokens)
      .def("spec_accepted", &Scheduler::spec_accepted)
      .def("spec_proposed", &Scheduler::spec_proposed)
      .def("prefix_cache_hits", &Scheduler::prefix_cache_hits)
      .def("prefix_cache_queries", &Scheduler::prefix_cache_queries)
      .def("request_info", [](const Scheduler& s, int64_t id) -> py::object {
        const Request* r = s.get(id);
        if (!r) return py::none();
        py::dict d;
        d["num_prompt"] = r->num_prompt;
        d["num_output"] = r->num_output();
        d["num_computed"] = r->num_computed;
        d["num_cached_prefix"] = r->num_cached_prefix;
        d["status"] = (int)r->status;
        d["reason"] = (int)r->reason;
        d["first_token_step"] = r->first_token_step;
        d["finish_step"] = r->finish_step;
        d["num_preemptions"] = r->num_preemptions;
        d["num_blocks"] = (int)r->blocks.size();
        d["state_slot"] = r->state_slot;
        d["draft"] = r->draft;
        d["draft_parent"] = r->draft_parent;
        return d;
      });
}
