"""The CUDA extension registers every op schema at import (no GPU needed): a malformed schema
aborts the process, so import it in a child process and check the ops are there."""
import glob
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_extension_imports_and_registers_ops():
    if not glob.glob(os.path.join(ROOT, "vllm_musa_b200", "_C*.so")):
        pytest.skip("extension not built in-tree")
    code = ("import torch, vllm_musa_b200._C; o = torch.ops.b200; "
            "[getattr(o, n) for n in ('paged_decode', 'paged_prefill', 'mamba2_scan', "
            "'gated_rmsnorm', 'w4_dequant', 'row_fp8_qdq', 'causal_conv1d', 'gemm_grouped_bf16')]")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
