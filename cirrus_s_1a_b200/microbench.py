"""Microbenchmark of one NVFP4 projection: the tensor-core GEMM
(cb_gemm_nvfp4: input preparation + tcgen05 GEMM) or the CUDA-core GEMV
(cb_gemv_nvfp4) on random weights of one (N, K) shape, M token rows, L2
flushed before every launch.

    python -m cirrus_s_1a_b200.microbench --n 32000 --k 768 --m 8 --iters 20 [--gemv]
        [--pre rmsnorm] [--epi add|swiglu] [--warm]

--pre / --epi select the GEMM's RMSNorm prologue and residual-add / SwiGLU
epilogue; --warm times 20 back-to-back launches in one CUDA graph without the
L2 flush (the per-launch cost inside a step whose weights are still in L2).

With --gdn it times the chunked Gated DeltaNet prefill instead (one layer:
--batch sequences x 12 heads x --tokens tokens, Dk = Dv = 64, the C2
distributions of the reference benchmark):

    python -m cirrus_s_1a_b200.microbench --gdn --batch 1 --tokens 4096

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
    ap.add_argument("--pre", choices=("none", "rmsnorm"), default="none")
    ap.add_argument("--epi", choices=("store", "add", "swiglu"), default="store")
    ap.add_argument("--warm", action="store_true", help="20 launches per CUDA graph replay, no L2 flush")
    ap.add_argument("--gdn", action="store_true", help="time the chunked Gated DeltaNet prefill instead")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--tokens", type=int, default=4096)
    args = ap.parse_args()
    if args.gdn:
        gdn(args)
        return
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(0)
    pm = PackedMatrix([torch.randn(args.n, args.k, generator=g) * 0.02], dev)
    x = torch.randn(args.m, args.k, generator=g).to(dev)
    norm_w = (1.0 + 0.1 * torch.randn(args.k, generator=g)).to(dev)
    pre = {"none": _lib.CB_GEMM_PRE_NONE, "rmsnorm": _lib.CB_GEMM_PRE_RMSNORM}[args.pre]
    epi = {"store": _lib.CB_GEMM_EPI_STORE, "add": _lib.CB_GEMM_EPI_ADD, "swiglu": _lib.CB_GEMM_EPI_SWIGLU}[args.epi]
    rows_out = args.n // 2 if args.epi == "swiglu" else args.n
    y = torch.zeros(args.m, pm.rows, device=dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    L = _lib.lib()
    ms = pm.struct()
    nb = L.cb_gemm_scratch_bytes(args.k, args.m)
    scratch = torch.empty(max(nb, 16), dtype=torch.uint8, device=dev)
    side = torch.cuda.Stream(dev)
    reps = 20 if args.warm else 1

    def launch(st):
        for _ in range(reps):
            if args.gemv:
                _lib.check(L.cb_gemv_nvfp4(C.byref(ms), x.data_ptr(), args.k, args.m, y.data_ptr(), pm.rows, args.n,
                                           st), "cb_gemv_nvfp4")
            else:
                _lib.check(L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), args.k, args.m, pre,
                                           norm_w.data_ptr() if args.pre == "rmsnorm" else None, 1e-6, y.data_ptr(),
                                           pm.rows, rows_out, epi, scratch.data_ptr(), nb, None, st), "cb_gemm_nvfp4")

    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        launch(side.cuda_stream)  # eager warm-up (kernel attributes), then one captured step
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            launch(side.cuda_stream)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    times = []
    for i in range(args.warmup + args.iters):
        if not args.warm:
            flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        if i >= args.warmup:
            times.append(a.elapsed_time(b) * 1e3 / reps)
    us = statistics.mean(times)
    print(json.dumps({"kernel": "gemv_nvfp4" if args.gemv else "gemm_nvfp4 (tcgen05)", "n": args.n, "k": args.k,
                      "m": args.m, "pre": args.pre, "epi": args.epi, "l2": "warm" if args.warm else "flushed",
                      "us": us, "bytes": pm.real_bytes, "gbs": pm.real_bytes / (us * 1e-6) / 1e9,
                      "flops": 2 * args.m * args.n * args.k}))


def gdn(args) -> None:
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(0)
    B, T, H, D = args.batch, args.tokens, 12, 64
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).to(dev)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).to(dev)
    v = torch.randn(B, T, H, D, generator=g).to(dev)
    gl = torch.sigmoid(torch.randn(B, T, H, generator=g) + 3.0).log().to(dev)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g)).to(dev)
    S0 = (torch.randn(B, H, D, D, generator=g) * 0.1).to(dev)
    S = torch.empty_like(S0)
    out = torch.empty(B, T, H, D, device=dev)
    L = _lib.lib()
    st = torch.cuda.current_stream(dev).cuda_stream
    times = []
    for i in range(args.warmup + args.iters):
        S.copy_(S0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _lib.check(L.cb_gdn_chunk_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), gl.data_ptr(), beta.data_ptr(),
                                          B, T, H, D, D, C.c_float(D ** -0.5), S.data_ptr(), out.data_ptr(), st),
                   "cb_gdn_chunk_prefill")
        b.record()
        b.synchronize()
        if i >= args.warmup:
            times.append(a.elapsed_time(b) * 1e3)
    us = statistics.mean(times)
    # per chunk and head: 6 products of 64^3 and the 64^2 x 64 solve, 2 flops per FMA
    flops = 2.0 * B * H * ((T + 63) // 64) * (6 * 64 ** 3 + 64 ** 3)
    print(json.dumps({"kernel": "gdn_chunk_prefill", "batch": B, "tokens": T, "heads": H, "us": us,
                      "tokens_per_s": B * T / (us * 1e-6), "gflops": flops / (us * 1e-6) / 1e9}))


if __name__ == "__main__":
    main()
