"""Microbenchmark of one NVFP4 projection: the tcgen05 verify GEMM
(cb_verify_gemm_nvfp4) or the CUDA-core GEMV (cb_gemv_nvfp4) on random
weights of one (N, K) shape, M token rows, L2 flushed before every launch.

    python -m cirrus_s_1a_b200.microbench --n 32000 --k 768 --m 8 --iters 20 [--gemv]

Prints one JSON line: mean launch time (CUDA events) and achieved GB/s of the
packed weight bytes.  The shapes of the reference's weight-stream benchmark are
768x768, 4096x768 (gate_up), 768x2048 (down) and 32000x768 (LM head).
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import statistics

import torch

from . import _lib
from .engine import PackedMatrix


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=32000)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--m", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--gemv", action="store_true", help="time the CUDA-core GEMV instead")
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(0)
    pm = PackedMatrix([torch.randn(args.n, args.k, generator=g) * 0.02], dev)
    x = torch.randn(args.m, args.k, generator=g).to(dev)
    xb = x.to(torch.bfloat16).view(torch.int16).contiguous()
    y = torch.empty(args.m, pm.rows, device=dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    L = _lib.lib()
    ms = pm.struct()
    st = torch.cuda.current_stream(dev).cuda_stream

    def launch():
        if args.gemv:
            _lib.check(L.cb_gemv_nvfp4(C.byref(ms), x.data_ptr(), args.k, args.m, y.data_ptr(), pm.rows, args.n, st),
                       "cb_gemv_nvfp4")
        else:
            _lib.check(L.cb_verify_gemm_nvfp4(C.byref(ms), xb.data_ptr(), args.k, args.m, y.data_ptr(), pm.rows,
                                              args.n, None, st), "cb_verify_gemm_nvfp4")

    times = []
    for i in range(args.warmup + args.iters):
        flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        b.synchronize()
        if i >= args.warmup:
            times.append(a.elapsed_time(b) * 1e3)
    us = statistics.mean(times)
    print(json.dumps({"kernel": "gemv_nvfp4" if args.gemv else "verify_gemm (tcgen05)", "n": args.n, "k": args.k,
                      "m": args.m, "us": us, "bytes": pm.real_bytes, "gbs": pm.real_bytes / (us * 1e-6) / 1e9,
                      "flops": 2 * args.m * args.n * args.k}))


if __name__ == "__main__":
    main()
