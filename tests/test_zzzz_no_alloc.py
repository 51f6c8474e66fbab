"""Allocation-free decode entry point, called through its exported C symbol.

Some callers cannot allocate GPU memory at the point where they run attention: hosts that
cap this library's device memory at a fixed budget, and runtimes that link the library without
the PyTorch allocator.  ``b200_paged_decode_noalloc`` serves them from a static device scratch
array; these tests check it against the regular entry point (torch.ops.b200.paged_decode with
a torch-allocated workspace) on two calls in a row, with and without split-KV scratch, that a
warm call changes the device's free memory by nothing, and that oversize requests and
unsupported geometry are refused with their documented codes.
The file sorts last so a stop-at-first-failure run has executed every other test first.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, ERR_TOO_LARGE, ERR_ARGS = 0, 1, 3


def _lib():
    import vllm_musa_b200._C as C
    lib = ctypes.CDLL(C.__file__)
    fn = lib.b200_paged_decode_noalloc
    fn.restype = ctypes.c_int
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fn.argtypes = [P, I64, P, I64, P, P, I, P, I64, P, I, I, I, I, I, I, I, ctypes.c_float, P, P]
    return fn


def _case(seed, lens, D=128, Hq=32, Hkv=8, bs=64):
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    nb = sum((l + bs - 1) // bs for l in lens) + 2
    kc = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16).cuda()
    vc = torch.randn(nb, Hkv, bs, D, generator=g).to(torch.bfloat16).cuda()
    perm = torch.randperm(nb, generator=g)
    W = max((l + bs - 1) // bs for l in lens) + 1
    bt = torch.zeros(B, W, dtype=torch.int32)
    used = 0
    for b, l in enumerate(lens):
        n = (l + bs - 1) // bs
        bt[b, :n] = perm[used:used + n].to(torch.int32)
        used += n
    q = torch.randn(B, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16).cuda()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32).cuda()


def _call(fn, q, kc, vc, bt, sl, Hq, Hkv, max_len, splits, out, status):
    D = kc.shape[-1]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), kc.data_ptr(),
              vc.data_ptr(), kc.shape[0], bt.data_ptr(), bt.stride(0), sl.data_ptr(), q.shape[0],
              Hq, Hkv, D, kc.shape[2], max_len, splits, 1.0 / math.sqrt(D),
              status.data_ptr(), stream)


def test_noalloc_decode_matches_regular_entry_point():
    from vllm_musa_b200 import ops
    fn = _lib()
    Hq, Hkv, max_len, splits = 32, 8, 2048, 4
    status = torch.ones(1, dtype=torch.int32, device="cuda")
    for seed, lens in ((1, [1, 70, 640, 2000, 129, 3]), (2, [1500, 5, 64, 65])):
        q, kc, vc, bt, sl = _case(seed, lens)
        out = torch.empty(len(lens), Hq * 128, dtype=torch.bfloat16, device="cuda")
        rc = _call(fn, q, kc, vc, bt, sl, Hq, Hkv, max_len, splits, out, status)
        assert rc == OK
        ref = ops.paged_decode(q, kc, vc, bt, sl, Hq, Hkv, 1.0 / math.sqrt(128), max_len,
                               num_splits=splits)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)


def test_noalloc_decode_rejects_oversize():
    fn = _lib()
    lens = [8] * 512
    q, kc, vc, bt, sl = _case(3, lens)
    out = torch.empty(len(lens), 32 * 128, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    # 512 x 32 heads x 64 splits x 128 fp32 partials = 512 MiB > 16 MiB scratch
    rc = _call(fn, q, kc, vc, bt, sl, 32, 8, 8192, 64, out, status)
    assert rc == ERR_TOO_LARGE


def test_noalloc_decode_allocates_nothing_and_serves_one_split():
    """After a warm-up (module load, the regular path, the entry point's per-device set-up),
    further calls leave the device's free memory unchanged, with split scratch (4 splits) and
    without it (1 split), and both match the regular entry point."""
    from vllm_musa_b200 import ops
    fn = _lib()
    Hq, Hkv, max_len = 32, 8, 2048
    lens = [1, 300, 2000, 64]
    q, kc, vc, bt, sl = _case(4, lens)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = {s_: torch.empty(len(lens), Hq * 128, dtype=torch.bfloat16, device="cuda")
            for s_ in (1, 4)}
    refs = {s_: ops.paged_decode(q, kc, vc, bt, sl, Hq, Hkv, 1.0 / math.sqrt(128), max_len,
                                 num_splits=s_) for s_ in (1, 4)}
    assert _call(fn, q, kc, vc, bt, sl, Hq, Hkv, max_len, 4, outs[4], status) == OK
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for s_ in (4, 1, 4):
        assert _call(fn, q, kc, vc, bt, sl, Hq, Hkv, max_len, s_, outs[s_], status) == OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert int(status.item()) == 0
    for s_ in (1, 4):
        torch.testing.assert_close(outs[s_].float(), refs[s_].float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("D,Hq,Hkv,bs", [(96, 32, 8, 64), (128, 20, 8, 64), (128, 64, 2, 64),
                                         (128, 32, 8, 24)])
def test_noalloc_decode_rejects_unsupported_geometry(D, Hq, Hkv, bs):
    """head_dim outside {64, 128, 256}, a query-head count that is not a multiple of the KV
    heads, a GQA group above 16 and a block size that is not a multiple of 16 are refused
    with ERR_ARGS before anything is launched."""
    fn = _lib()
    lens = [5, 40]
    q, kc, vc, bt, sl = _case(5, lens, D=D, Hq=Hq, Hkv=Hkv, bs=bs)
    out = torch.empty(len(lens), Hq * D, dtype=torch.bfloat16, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call(fn, q, kc, vc, bt, sl, Hq, Hkv, 256, 2, out, status) == ERR_ARGS
