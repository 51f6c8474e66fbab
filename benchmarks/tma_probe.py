"""TMA -> shared-memory throughput per CTA and per GPU (the measurements behind the GEMM's
K-atoms-per-stage rule).  Builds tma_probe.cu with nvcc into a temporary directory and prints
one JSON line per configuration.

    python benchmarks/tma_probe.py
"""
import ctypes
import json
import os
import subprocess
import sys
import tempfile

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def build() -> ctypes.CDLL:
    out = os.path.join(tempfile.mkdtemp(), "tma_probe.so")
    subprocess.check_call(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared",
                           "-Xcompiler", "-fPIC", "-I" + os.path.join(os.path.dirname(HERE), "csrc"),
                           os.path.join(HERE, "tma_probe.cu"), "-o", out])
    lib = ctypes.CDLL(out)
    lib.run_tbw.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.POINTER(ctypes.c_float), ctypes.c_void_p, ctypes.c_int]
    return lib


def main():
    lib = build()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    big = torch.empty(6 << 30, dtype=torch.uint8, device="cuda")

    def run(grid, box_rows, per_stage, stages, mode, nprod=1):
        copy = box_rows * 128
        per = grid * nprod * copy * per_stage
        iters = max(16, (2 << 30) // per) if mode == 0 else (5 << 30) // per
        ms = ctypes.c_float()
        rc = lib.run_tbw(big.data_ptr(), (32 << 20) if mode == 0 else (6 << 30), grid, box_rows,
                         per_stage, stages, iters, mode, ctypes.byref(ms), err.data_ptr(), nprod)
        torch.cuda.synchronize()
        nbytes = per * iters
        print(json.dumps(dict(src="L2" if mode == 0 else "HBM", ctas=grid, producers=nprod,
                              box_kib=copy // 1024, boxes_per_stage=per_stage, stages=stages,
                              us=round(ms.value * 1e3, 1),
                              GBps_per_cta=round(nbytes / grid / (ms.value * 1e-3) / 1e9, 1),
                              TBps=round(nbytes / (ms.value * 1e-3) / 1e12, 3), rc=rc,
                              err=int(err.item()))), flush=True)

    for box in (64, 128, 256):
        for per in (1, 2, 4):
            kib = box * 128 * per // 1024
            if kib > 96:
                continue
            for grid in (1, 148):
                run(grid, box, per, max(2, min(12, 192 // kib)), 0)
    for nprod in (1, 2, 4):
        run(1, 128, 1, max(2, 12 // nprod), 0, nprod)
    for box, per in ((128, 1), (256, 1), (128, 2)):
        kib = box * 128 * per // 1024
        run(148, box, per, max(2, min(12, 192 // kib)), 1)


if __name__ == "__main__":
    main()
