"""vLLM itself with this package as its platform plugin, on a B200: ``vllm.LLM`` on a 2-layer
Llama-architecture model (random weights) runs its attention, KV-cache writes and norms on
this package's kernels, and its prompt log-probabilities match stock vLLM's (the same model
and weights without the plugin) at bf16 resolution.

The plugin is made discoverable the way an installed wheel would be: a ``*.dist-info`` with
the package's entry points (``vllm.platform_plugins`` / ``vllm.general_plugins``) on the
child's ``PYTHONPATH``.  Each run is a child process (vLLM's engine in-process,
``VLLM_ENABLE_V1_MULTIPROCESSING=0``) under a timeout."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
pytest.importorskip("vllm")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import json, os, sys
import torch
from vllm import LLM, SamplingParams
path, use_plugin = sys.argv[1], sys.argv[2] == "1"
launches0 = None
if use_plugin:
    import vllm_musa_b200._C as C
    launches0 = C.launch_count()
llm = LLM(model=path, load_format="dummy", dtype="bfloat16", max_model_len=512,
          gpu_memory_utilization=0.25, enforce_eager=True, seed=0, max_num_seqs=8,
          skip_tokenizer_init=True)
g = torch.Generator().manual_seed(3)
prompts = [{"prompt_token_ids": torch.randint(0, 4000, (n,), generator=g).tolist()}
           for n in (17, 130, 70)]
sp = SamplingParams(temperature=0.0, max_tokens=4, prompt_logprobs=0, logprobs=0,
                    ignore_eos=True, detokenize=False)
outs = llm.generate(prompts, sp, use_tqdm=False)
plp = [[next(iter(d.values())).logprob for d in o.prompt_logprobs[1:]] for o in outs]
res = {"prompt_logprobs": plp, "tokens": [list(o.outputs[0].token_ids) for o in outs],
       "platform": type(__import__("vllm.platforms", fromlist=["current_platform"])
                        .current_platform).__name__}
if use_plugin:
    res["launches"] = C.launch_count() - launches0
print("RESULT " + json.dumps(res), flush=True)
'''


def _dist_info(d):
    di = os.path.join(d, "vllm_musa_b200_plugin-0.1.dist-info")
    os.makedirs(di, exist_ok=True)
    with open(os.path.join(di, "METADATA"), "w") as f:
        f.write("Metadata-Version: 2.1\nName: vllm-musa-b200-plugin\nVersion: 0.1\n")
    with open(os.path.join(di, "entry_points.txt"), "w") as f:
        f.write("[vllm.platform_plugins]\nb200 = vllm_musa_b200:b200_platform_plugin\n\n"
                "[vllm.general_plugins]\nb200_custom_ops = vllm_musa_b200:register_custom_ops\n")


def _run(model_dir, plugin_dir, use_plugin):
    env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0", TOKENIZERS_PARALLELISM="false")
    env["PYTHONPATH"] = os.pathsep.join(([plugin_dir] if use_plugin else []) + [ROOT])
    if not use_plugin:
        env["VLLM_PLUGINS"] = ""  # no general plugins either
    r = subprocess.run(["timeout", "-k", "20", "420", sys.executable, "-c", CHILD, model_dir,
                        "1" if use_plugin else "0"], env=env, cwd=ROOT, capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_vllm_llm_runs_on_b200_plugin(tmp_path):
    model = tmp_path / "llama2l"
    model.mkdir()
    (model / "config.json").write_text(json.dumps({
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": 4096,
        "hidden_size": 1024, "intermediate_size": 2816, "num_hidden_layers": 2,
        "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 64,
        "rms_norm_eps": 1e-5, "rope_theta": 10000.0, "max_position_embeddings": 2048,
        "tie_word_embeddings": False, "torch_dtype": "bfloat16"}))
    plugins = str(tmp_path / "plugins")
    _dist_info(plugins)
    ours = _run(str(model), plugins, True)
    stock = _run(str(model), plugins, False)
    assert ours["platform"] == "B200Platform" and stock["platform"] != "B200Platform"
    assert ours["launches"] > 0  # this package's kernels ran inside vLLM
    for a, b in zip(ours["prompt_logprobs"], stock["prompt_logprobs"]):
        assert len(a) == len(b)
        assert max(abs(x - y) for x, y in zip(a, b)) < 0.05
