#!/usr/bin/env python3
"""Decode benchmark of the B200 cirrus-s-1a path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): one tau=1 decode step of one sequence at 32K context
(cache holds 32767 tokens, the step appends the 32768th) with the benchmark
shapes (d 768, vocab 32000, 9 GDN + 3 SWA self layers, 6 cross layers,
12 q / 4 kv heads of 64, window 2048, indexer 4 x 64, top-k 512), random
NVFP4 weights (seed 0) and a synthetic cache (bf16 K/V ~ N(0, 1), E4M3
indexer keys of N(0, 1), GDN state ~ N(0, 0.1)).  Each step restores the
position to 32767, so every timed step does exactly the 32K-context work.
L2 is flushed (512 MB write) between timed steps, outside the timed region.

One JSON line on rank 0:
  value        tokens/s of all ranks, device-timed (CUDA events) graph replay
  e2e          the same through the public DecodeGraph API with the token id
               copied in from pinned host memory and the argmax token copied
               back every step
  roofline     the dominant kernel, the persistent decode kernel (one launch
               is one whole step): the step's algorithmic bytes / its CUDA-event
               time vs the measured HBM copy bandwidth; ``traffic`` is the DRAM
               read + write of one launch from an ncu capture of this workload
  weight_stream_kernel  the NVFP4 weight stream alone (every projection of a
               step, M = 1) as one persistent launch (the reference's headline
               microbenchmark, configs[1])
  weight_stream  the same as separate GEMV launches in one CUDA graph
  weight_stream_by_M  the weight stream at M = 2 .. 64 token rows through the
               tensor-core GEMM, the CUDA-core GEMV and (M <= 8) the stream kernel
  batched      step time of B sequences x T tokens (B = 8, 64; T = 1, 5); more
               than 16 token rows run on the tensor-core GEMM
  spec_decode  configs[4] on this GPU: 64 sequences at 32K, prompt-lookup drafts
               of 4, greedy acceptance with on-device rewind (SpecDecoder)
  prefill      prompt tokens / s of the prefill path (512 and 32K tokens at
               batch 1, 8 x 4096)
  cpu_baseline the oracle restatement of the reference forward on the host
               cores (rank 0, N = 1, a bounded number of 32K-context steps)

``--impl reference`` times only that CPU restatement (rank 0) and prints its
own line.  Multi-GPU: one process per GPU under torchrun; every rank decodes
its own sequence (no collective on the data path), the timing is the max over
ranks and ``value`` sums the ranks' tokens.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (batch 1, τ=1, 32K ctx) per B200 + HBM GB/s vs 8 TB/s; box tok/s 1/2/4/8"
# DRAM bytes (read + write) of one persistent-kernel launch at this workload,
# from an ncu capture (dram__bytes_read.sum + dram__bytes_write.sum), and the
# SHA-256 prefix of the kernel source it was captured from: a changed source
# reports traffic null until it is captured again.
STEP_TRAFFIC = {"bytes": 95_820_800 + 3_996_416, "source": "cirrus_s_1a_b200/csrc/decode_mk.cu",
                "sha256_16": "e152670d4e85d71d"}
CPU_ARM_WHY = ("the reference is a Python package that cannot travel to the GPU box, so the CPU arm runs the "
               "oracle: the reference forward restated operation by operation (oracle/model.py), checked against "
               "fixtures generated from the reference itself (tests/golden), with the B200 storage casts")
PUBLISHED_TOK_S = 1815.0  # reference: decode tok/s at 32K, tau=1 (GB10, measured stream + roofline remainder)
CTX = 32768
FLUSH_BYTES = 512 << 20


def workload_config(world: int) -> dict:
    """The ``config`` of both arms' lines (the same workload)."""
    return {"workload": "cirrus-s-1a decode step, batch 1, tau=1, ctx 32768 (benchmark shapes, random NVFP4 "
                        "weights seed 0, synthetic cache)",
            "batch_per_gpu": 1, "ctx": CTX, "weights": "nvfp4 (e2m1 + e4m3/16 + f32)", "kv": "bf16",
            "indexer_keys": "e4m3", "l2": "flushed between timed steps (512 MB write)",
            "parallelism": f"replicas x{world} (independent sequences)"}


def step_traffic():
    """(bytes, note) of the recorded ncu traffic, bytes None when the kernel source changed since."""
    import hashlib

    path = os.path.join(ROOT, STEP_TRAFFIC["source"])
    sha = hashlib.sha256(open(path, "rb").read()).hexdigest()[:16] if os.path.exists(path) else ""
    if sha == STEP_TRAFFIC["sha256_16"]:
        return STEP_TRAFFIC["bytes"], f"ncu capture of {STEP_TRAFFIC['source']} @ {sha}"
    return None, f"no ncu capture of the current {STEP_TRAFFIC['source']} ({sha})"


def _peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi samples of one GPU during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id, self.rows, self.proc = gpu_id, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[3:]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows),
                "window": "1.2 s of the same steps right before the timed steps, and the timed steps"}


def step_bytes(cfg, weight_bytes: float, ctx: int) -> dict:
    """Algorithmic bytes of one tau=1 batch-1 decode step at context ``ctx``."""
    H, dk, dv = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v
    kinds = cfg.self_layer_kinds
    n_gdn, n_swa = kinds.count("gdn"), kinds.count("swa")
    C = 2 * H * dk + H * dv
    kv_row = cfg.n_kv_heads * cfg.head_dim * 2  # bf16
    return {
        "weights": weight_bytes,
        "gdn_state_rw": 2 * n_gdn * H * dk * dv * 4,
        "conv_state_rw": 2 * n_gdn * (cfg.gdn_conv_size - 1) * C * 4,
        "swa_kv": n_swa * min(ctx, cfg.swa_window) * 2 * kv_row,
        "indexer_keys": ctx * cfg.indexer_dim,
        "topk_kv_gather": min(ctx, cfg.sparse_topk + 1) * 2 * kv_row,
    }


def weight_stream_graph(eng, M: int = 1, tensor_cores: bool = False):
    """CUDA graph of one product per projection matrix of the model (the
    reference's "decode-step weight stream", configs[1]) for M token rows:
    the CUDA-core GEMV, or the tensor-core GEMM (input preparation + tcgen05)."""
    import ctypes as C

    import torch

    from cirrus_s_1a_b200 import _lib
    from cirrus_s_1a_b200.engine import PackedMatrix

    mats = [m for m in eng.model._keep if isinstance(m, PackedMatrix)]
    dev = eng.device
    kmax = max(m.k for m in mats)
    x = torch.randn(M, kmax, device=dev)
    y = torch.empty(M, max(m.rows for m in mats), device=dev)
    L0 = _lib.lib()
    nb = L0.cb_gemm_scratch_bytes((kmax + 63) // 64 * 64, M)
    scratch = torch.empty(max(nb, 16), dtype=torch.uint8, device=dev)
    ldy = y.shape[1]
    structs = [m.struct() for m in mats]
    L = _lib.lib()
    side = torch.cuda.Stream(dev)

    def run(st):
        for s in structs:
            if tensor_cores:
                _lib.check(L.cb_gemm_nvfp4(C.byref(s), x.data_ptr(), kmax, M, _lib.CB_GEMM_PRE_NONE, None, 0.0,
                                           y.data_ptr(), ldy, s.rows, _lib.CB_GEMM_EPI_STORE, scratch.data_ptr(), nb,
                                           None, st), "gemm")
            else:
                _lib.check(L.cb_gemv_nvfp4(C.byref(s), x.data_ptr(), kmax, M, y.data_ptr(), ldy, s.rows, st), "gemv")

    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        run(side.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            run(side.cuda_stream)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    real = sum(m.real_bytes for m in mats)
    g.keep = (x, y, scratch)  # buffers the captured launches use
    return g, len(structs), real


def weight_stream_kernel_graph(eng, M: int = 1):
    """CUDA graph of the one-launch weight stream (cb_weight_stream_nvfp4) over the
    same projection matrices as ``weight_stream_graph``."""
    import ctypes as C

    import torch

    from cirrus_s_1a_b200 import _lib
    from cirrus_s_1a_b200.engine import PackedMatrix

    L = _lib.lib()
    mats = [m for m in eng.model._keep if isinstance(m, PackedMatrix)]
    dev = eng.device
    arr = (_lib.CbMatrix * len(mats))(*[m.struct() for m in mats])
    plan = torch.empty(L.cb_stream_plan_bytes(len(mats)), dtype=torch.uint8, device=dev)
    rows = C.c_int64(0)
    _lib.check(L.cb_stream_plan(arr, len(mats), plan.data_ptr(), plan.numel(), C.byref(rows),
                                torch.cuda.current_stream(dev).cuda_stream), "cb_stream_plan")
    kmax = max(m.k for m in mats)
    x = torch.randn(M, kmax, device=dev)
    y = torch.empty(M, rows.value, device=dev)
    side = torch.cuda.Stream(dev)

    def run(st):
        _lib.check(L.cb_weight_stream_nvfp4(plan.data_ptr(), len(mats), rows.value // 16, x.data_ptr(), kmax, kmax,
                                            M, y.data_ptr(), rows.value, None, st), "cb_weight_stream_nvfp4")

    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        run(side.cuda_stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            run(side.cuda_stream)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g.keep = (plan, x, y)
    return g, len(mats), sum(m.real_bytes for m in mats)


def time_graph(g, flush, stream, warmup: int, iters: int) -> float:
    """Mean CUDA-event time (ms) of a graph replay with L2 flushed before each."""
    import torch

    out = []
    for i in range(warmup + iters):
        flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g.replay()
        b.record(stream)
        b.synchronize()
        if i >= warmup:
            out.append(a.elapsed_time(b))
    return statistics.mean(out)


def cpu_baseline(cfg, sd, cache, ctx: int, budget_s: float, max_steps: int) -> dict:
    """Oracle (the reference forward restated on the CPU) decode steps at ``ctx``."""
    import torch

    from oracle import model as om

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    p = om.quantized_params(sd)
    ref = cache.to_reference()
    oc = om.OracleCache(ref["layers"], ref["shared"], ref["pos"])
    ids = torch.tensor([[17]])
    om.forward(p, cfg, ids, cache=oc, n_logits=1, casts=om.B200)  # warm-up
    n, t0 = 0, time.perf_counter()
    while n < max_steps and (n == 0 or time.perf_counter() - t0 < budget_s):
        om.forward(p, cfg, ids, cache=oc, n_logits=1, casts=om.B200)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} oracle decode steps (batch 1, tau=1) at ctx {ctx}, torch CPU fp32, "
                      f"{threads} threads, {dt:.1f} s"}


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    import torch

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from oracle import model as om

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=0)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    p = om.quantized_params(sd)
    # synthetic 32K cache built directly in the reference Cache layout (CPU)
    g = torch.Generator().manual_seed(1)
    H, dk, dv, KC = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v, cfg.gdn_conv_size
    C = 2 * H * dk + H * dv
    n = CTX - 1
    layers = []
    for kind in cfg.self_layer_kinds:
        if kind == "gdn":
            layers.append({"conv": torch.randn(1, KC - 1, C, generator=g), "S": torch.randn(1, H, dk, dv, generator=g) * 0.1})
        else:
            shp = (1, cfg.swa_window, cfg.n_kv_heads, cfg.head_dim)
            layers.append({"k": torch.randn(shp, generator=g).bfloat16().float(),
                           "v": torch.randn(shp, generator=g).bfloat16().float()})
    shp = (1, n, cfg.n_kv_heads, cfg.head_dim)
    shared = {"k": torch.randn(shp, generator=g).bfloat16().float(), "v": torch.randn(shp, generator=g).bfloat16().float(),
              "ik": torch.randn(1, n, cfg.indexer_dim, generator=g).to(torch.float8_e4m3fn).float()}
    oc = om.OracleCache(layers, shared, n)
    ids = torch.tensor([[17]])
    for _ in range(args.warmup):
        om.forward(p, cfg, ids, cache=oc, n_logits=1, casts=om.B200)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        om.forward(p, cfg, ids, cache=oc, n_logits=1, casts=om.B200)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = args.steps / tot
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": workload_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} oracle decode steps at ctx {CTX} (torch CPU fp32, "
                                       f"{threads} threads)",
                             "why_port": CPU_ARM_WHY},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


SPEC_BATCH, SPEC_DRAFT, SPEC_STEPS = 64, 4, 12


def spec_decode(eng, dev, stream, flush, args, rank: int) -> dict:
    """BASELINE configs[4] on this GPU: SPEC_BATCH independent sequences at 32K
    context, each with a 32K-token prompt-lookup history (the n-gram-repeating
    stream of ``synthetic.random_prompt``; the cache itself is the synthetic
    32K fill), greedy decoding with prompt-lookup drafts of up to SPEC_DRAFT
    tokens (``SpecDecoder``: device drafter, one verify forward, device
    acceptance and rewind, one CUDA graph per step).  Device-timed over
    SPEC_STEPS steps after warm-up, L2 flushed before each step; the metric is
    emitted (accepted + bonus) tokens per second."""
    import torch

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.speculative import SpecDecoder

    from cirrus_s_1a_b200.shard import shard_bounds

    cfg = eng.cfg
    world = int(os.environ.get("WORLD_SIZE", "1"))
    # this rank's contiguous shard of the global batch of SPEC_BATCH * world sequences
    s0, s1 = shard_bounds(SPEC_BATCH * world, world, rank)
    B, T = s1 - s0, 1 + SPEC_DRAFT
    max_new = (args.warmup + SPEC_STEPS + 2) * T + 8
    cache = eng.new_cache(B, max_ctx=CTX + max_new + 2 * T)
    synthetic.fill_cache(cache, CTX, seed=3 + rank)
    prompts = [synthetic.random_prompt(CTX - 1, cfg.vocab_size, seed=1000 + s) for s in range(s0, s1)]
    first = [p[-1] for p in prompts]  # any token: the synthetic cache has no real prompt to predict from
    dec = SpecDecoder(eng, cache, max_draft=SPEC_DRAFT)
    dec.start(prompts, max_new, first_tokens=first)
    dec.capture()
    for _ in range(args.warmup):
        flush.random_(0, 255)
        dec.step()
    e0 = int(dec.emitted.item())
    ms = 0.0
    for _ in range(SPEC_STEPS):
        flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dec.step()
        b.record(stream)
        b.synchronize()
        ms += a.elapsed_time(b)
    emitted = int(dec.emitted.item()) - e0
    out = {"workload": f"configs[4]: {B} sequences per GPU at ctx {CTX}, prompt-lookup drafts of up to {SPEC_DRAFT} "
                       "tokens (n-gram 2..4 over a 32K n-gram-repeating token history), greedy acceptance with "
                       "on-device rewind, random weights",
           "batch_per_gpu": B, "draft": SPEC_DRAFT, "steps": SPEC_STEPS, "ms": ms, "emitted": float(emitted),
           "ms_per_step": ms / SPEC_STEPS, "tokens_per_step": emitted / SPEC_STEPS,
           "tokens_per_s": emitted / (ms * 1e-3),
           "note": "random weights: the model's greedy tokens rarely continue the copied spans, so few drafts "
                   "are accepted; tokens_per_step near the batch size is the expected outcome"}
    del dec, cache
    torch.cuda.empty_cache()
    return out


def prefill_bench(eng, dev, stream) -> dict:
    """Prompt prefill through the public forward (cb_forward in 128-token chunks on
    the prefill kernels): configs[0]'s 512-token prompt and a 32K prompt at batch 1,
    and 8 x 4096; one warm-up, then one device-timed prefill each."""
    import torch

    from cirrus_s_1a_b200 import synthetic

    out = []
    for B, P in ((1, 512), (1, CTX), (8, 4096)):
        ids = torch.tensor([synthetic.random_prompt(P, eng.cfg.vocab_size, seed=50 + b) for b in range(B)],
                           device=dev)
        ms = 0.0
        for it in range(2):
            cache = eng.new_cache(B, max_ctx=P + 64)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            eng(ids, cache=cache, n_logits=1)
            b.record(stream)
            b.synchronize()
            ms = a.elapsed_time(b)
            del cache
        out.append({"batch": B, "prompt": P, "ms": ms, "tokens_per_s": B * P / (ms * 1e-3)})
        torch.cuda.empty_cache()
    return {"note": "prompt tokens / s through CirrusB200.forward (n_logits=1), device-timed, random weights",
            "runs": out}


def profile_stream(M: int) -> None:
    """The one-launch weight stream (cb_weight_stream_nvfp4) over the model's 78
    projections with M input rows, two graph replays with L2 flushed before each
    (for a profiler: the second launch is the one to capture)."""
    import torch

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    eng = CirrusB200(cfg, synthetic.random_state_dict(cfg, seed=0), device="cuda:0", max_ctx=256)
    g, n_mats, nbytes = weight_stream_kernel_graph(eng, M)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda:0")
    for _ in range(2):
        flush.random_(0, 255)
        g.replay()
    torch.cuda.synchronize()
    print(json.dumps({"profile_stream": {"M": M, "matrices": n_mats, "bytes": nbytes}}), flush=True)


def profile_step(B: int, T: int) -> None:
    """Two eager steps of B sequences x T tokens at ctx 32K (the batched
    workload), each inside an NVTX range 'step' (`ncu --nvtx --nvtx-include
    "step/"` lists only their launches)."""
    import torch

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    eng = CirrusB200(cfg, synthetic.random_state_dict(cfg, seed=0), device="cuda:0", max_ctx=CTX + 64)
    cache = eng.new_cache(B)
    synthetic.fill_cache(cache, CTX, 1)
    ids = torch.randint(0, cfg.vocab_size, (B, T), device="cuda:0")
    for _ in range(2):
        cache.pos_dev.fill_(CTX - 1)
        cache.pos_host = [CTX - 1] * B
        torch.cuda.nvtx.range_push("step")
        eng(ids, cache=cache, n_logits=1)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    print(json.dumps({"profile_step": {"batch": B, "T": T, "ctx": CTX}}), flush=True)


def profile_prefill(B: int, P: int) -> None:
    """One warm-up prefill and one prefill inside an NVTX range 'prefill' (B
    prompts of P tokens), for a profiler's launch list."""
    import torch

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    eng = CirrusB200(cfg, synthetic.random_state_dict(cfg, seed=0), device="cuda:0", max_ctx=P + 64)
    ids = torch.tensor([synthetic.random_prompt(P, cfg.vocab_size, seed=s) for s in range(B)], device="cuda:0")
    for it in range(2):
        cache = eng.new_cache(B, max_ctx=P + 64)
        torch.cuda.synchronize()
        if it:
            torch.cuda.nvtx.range_push("prefill")
        eng(ids, cache=cache, n_logits=1)
        if it:
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    print(json.dumps({"profile_prefill": {"batch": B, "prompt": P}}), flush=True)


def trace_step(B: int, T: int) -> None:
    """Per-phase timing of the persistent kernel (CTA 0's %globaltimer stamps at
    every grid barrier and its sub-phase marks) for B sequences x T tokens at
    32K, L2 flushed before each of 6 steps; prints one JSON line grouped by phase type."""
    import ctypes as C

    import torch

    from cirrus_s_1a_b200 import _lib, synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200, DecodeGraph

    cfg = baseline_config()
    eng = CirrusB200(cfg, synthetic.random_state_dict(cfg, seed=0), device="cuda:0", max_ctx=CTX + 64)
    names = []
    for kind in cfg.self_layer_kinds:
        names += ["gdn" if kind == "gdn" else "swa_head", "ffn_self"]
    names += ["shared_proj", "append_scores", "compaction", "resolve"]
    names += ["cross_head", "ffn_cross"] * cfg.n_cross_layers + ["lm_head"]
    cache = eng.new_cache(B)
    synthetic.fill_cache(cache, CTX - 8, seed=1)
    g = DecodeGraph(eng, cache, T=T, n_logits=T, want_logits=False)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda:0")
    us = []
    for _ in range(6):
        cache.pos_dev.fill_(CTX - 8)
        flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        us.append(a.elapsed_time(b) * 1e3)
    ws = eng.workspace(B, T, cache.max_ctx)
    buf = (C.c_uint64 * 512)()
    n = _lib.lib().cb_read_trace(C.byref(eng.model.desc), B, T, cache.max_ctx, ws.data_ptr(), buf, 512,
                                 torch.cuda.current_stream().cuda_stream)
    v = list(buf[:n])
    agg = {}
    for p, name in enumerate(names):  # barrier 1 ends the set-up; phase p ends at barrier p + 2
        start, arrive, leave = v[2 * (p + 1)], v[2 * (p + 2) - 1], v[2 * (p + 2)]
        marks = [(v[256 + 6 * p + i] - start) / 1e3 if start <= v[256 + 6 * p + i] <= arrive else 0.0
                 for i in range(6)]
        e = agg.setdefault(name, {"count": 0, "work_us": 0.0, "wait_us": 0.0, "marks_us": [0.0] * 6})
        e["count"] += 1
        e["work_us"] += (arrive - start) / 1e3
        e["wait_us"] += (leave - arrive) / 1e3
        for i, m in enumerate(marks):
            e["marks_us"][i] += m
    for e in agg.values():
        c = e["count"]
        e["work_us"], e["wait_us"] = e["work_us"] / c, e["wait_us"] / c
        e["marks_us"] = [m / c for m in e["marks_us"]]
    print(json.dumps({"trace_step": {"batch": B, "T": T, "ctx": CTX, "step_us_median": sorted(us)[len(us) // 2],
                                     "per_phase": agg}}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-step", metavar="BxT", default=None,
                    help="run two eager batched steps (B sequences x T tokens) inside NVTX ranges named 'step' "
                         "for a profiler's launch list, then exit")
    ap.add_argument("--trace-step", metavar="BxT", default=None,
                    help="print the persistent kernel's per-phase timing for B sequences x T tokens, then exit")
    ap.add_argument("--profile-stream", metavar="M", type=int, default=None,
                    help="run the one-launch weight stream twice with M input rows (for a profiler), then exit")
    ap.add_argument("--profile-prefill", metavar="BxP", default=None,
                    help="run a warm-up prefill and one prefill (B prompts of P tokens) inside an NVTX range "
                         "named 'prefill', then exit")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_step:
        profile_step(*(int(v) for v in args.profile_step.lower().split("x")))
        return
    if args.trace_step:
        trace_step(*(int(v) for v in args.trace_step.lower().split("x")))
        return
    if args.profile_stream:
        profile_stream(args.profile_stream)
        return
    if args.profile_prefill:
        profile_prefill(*(int(v) for v in args.profile_prefill.lower().split("x")))
        return

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch

    from cirrus_s_1a_b200 import _lib, synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200, DecodeGraph

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=0)
    eng = CirrusB200(cfg, sd, device=dev, max_ctx=CTX + 64)
    cache = eng.new_cache(1)
    synthetic.fill_cache(cache, CTX, seed=1 + rank)

    L = _lib.lib()
    n0 = L.cb_launch_count()
    graph = DecodeGraph(eng, cache, T=1, n_logits=1, want_logits=False)
    launches_per_step = (L.cb_launch_count() - n0) // 2  # warm-up launch + captured launch
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    tok = torch.tensor([[17]], dtype=torch.int64)

    def reset():
        cache.pos_dev.fill_(CTX - 1)
        cache.pos_host = [CTX - 1]
        flush.random_(0, 255)

    # ------------------------------------------------ device-timed steps
    graph.ids.copy_(tok)
    for _ in range(args.warmup):
        reset()
        graph.replay()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    sampler = ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}")
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    # nvidia-smi samples every 200 ms: keep the GPU on this same workload for
    # about a second before the timed steps so the samples cover the load the
    # timed region runs under (and the timed region itself when it is long)
    sampler.start()
    t_probe = time.perf_counter()
    while time.perf_counter() - t_probe < 1.2:
        for _ in range(20):
            reset()
            graph.replay()
        torch.cuda.synchronize(dev)
    for i in range(args.steps):
        reset()
        torch.cuda.nvtx.range_push("cb_step")
        evs[i][0].record(stream)
        graph.replay()
        evs[i][1].record(stream)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    if world > 1:
        torch.distributed.barrier()
    t_steps = [a.elapsed_time(b) for a, b in evs]
    t_total_ms = sum(t_steps)

    # ------------------------------------------------ end to end (public API)
    ids_host = torch.tensor([[17]], dtype=torch.int64).pin_memory()
    out_host = torch.zeros(1, dtype=torch.int32).pin_memory()
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        reset()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.ids.copy_(ids_host, non_blocking=True)
        graph.replay()
        out_host.copy_(graph.argmax.view(-1), non_blocking=True)
        b.record(stream)
        b.synchronize()
        ids_host[0, 0] = int(out_host[0])  # the next step consumes the token just produced
        if i >= args.warmup:
            e2e_ms.append(a.elapsed_time(b))
    e2e_total = sum(e2e_ms)

    # ------------------------------------------------ weight stream roofline
    sgraph, _, _ = weight_stream_kernel_graph(eng, 1)
    s_ms = time_graph(sgraph, flush, stream, args.warmup, args.steps)
    del sgraph
    wgraph, n_mats, wbytes = weight_stream_graph(eng)
    w_ms = []
    for i in range(args.warmup + args.steps):
        flush.random_(0, 255)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        wgraph.replay()
        b.record(stream)
        b.synchronize()
        if i >= args.warmup:
            w_ms.append(a.elapsed_time(b))

    # ------------------------------------------------ weight stream at M token rows: tensor-core GEMM vs GEMV
    verify = {}
    for M in (2, 8, 16, 32, 64):
        row = {}
        for kind, tc in (("tcgen05", True), ("cuda_core", False)):
            vg, _, vbytes = weight_stream_graph(eng, M=M, tensor_cores=tc)
            v_ms = []
            for i in range(args.warmup + max(args.steps // 5, 3)):
                flush.random_(0, 255)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                vg.replay()
                b.record(stream)
                b.synchronize()
                if i >= args.warmup:
                    v_ms.append(a.elapsed_time(b))
            us = statistics.mean(v_ms) * 1e3
            row[kind] = {"us": us, "achieved_gbs": vbytes / (us * 1e-6) / 1e9,
                         "frac": vbytes / (us * 1e-6) / 1e9 / _peaks()["hbm_gbs"]}
            del vg
        if M <= 8:
            sg, _, sbytes = weight_stream_kernel_graph(eng, M)
            us = time_graph(sg, flush, stream, args.warmup, max(args.steps // 5, 3)) * 1e3
            row["stream_kernel"] = {"us": us, "achieved_gbs": sbytes / (us * 1e-6) / 1e9,
                                    "frac": sbytes / (us * 1e-6) / 1e9 / _peaks()["hbm_gbs"]}
            del sg
        verify[str(M)] = row

    # ------------------------------------------------ batched steps (B sequences x T tokens)
    batched = []
    del graph
    for Bb, Tb in ((8, 1), (1, 5), (64, 1), (64, 5)):
        bcache = eng.new_cache(Bb)
        synthetic.fill_cache(bcache, CTX, 1)
        bg = DecodeGraph(eng, bcache, T=Tb, n_logits=Tb, want_logits=False)
        b_ms = []
        for i in range(args.warmup + 3):
            bcache.pos_dev.fill_(CTX - 1)
            flush.random_(0, 255)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            bg.replay()
            b.record(stream)
            b.synchronize()
            if i >= args.warmup:
                b_ms.append(a.elapsed_time(b))
        ms_b = statistics.mean(b_ms)
        batched.append({"batch": Bb, "T": Tb, "ms_per_step": ms_b, "tokens_per_s": Bb * Tb / (ms_b * 1e-3),
                        "path": "persistent" if Bb * Tb <= 8 else "one launch per op"})
        del bg, bcache
        torch.cuda.empty_cache()

    # ------------------------------------------------ batched speculative decoding
    spec = spec_decode(eng, dev, stream, flush, args, rank)
    prefill = prefill_bench(eng, dev, stream) if world == 1 else None

    tot = torch.tensor([t_total_ms, e2e_total, spec["ms"], spec["emitted"]], dtype=torch.float64, device=dev)
    if world > 1:  # the slowest rank's times; the tokens of every rank
        mx = tot[:3].clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        em = tot[3:].clone()
        torch.distributed.all_reduce(em, op=torch.distributed.ReduceOp.SUM)
        tot = torch.cat((mx, em))
    t_total_ms, e2e_total = float(tot[0]), float(tot[1])
    spec["box_tokens_per_s"] = float(tot[3]) / (float(tot[2]) * 1e-3)
    spec["n_gpus"] = world
    spec.pop("emitted")
    peaks = _peaks()
    w_avg_s = statistics.mean(w_ms) * 1e-3
    sb = step_bytes(cfg, float(eng.model.weight_real_bytes), CTX)
    step_total = sum(sb.values())
    ms_step = t_total_ms / args.steps
    value = world * args.steps / (t_total_ms * 1e-3)
    traffic, traffic_note = step_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "f32", "data": "synthetic",
        "config": workload_config(world),
        "roofline": {"bound": "hbm", "kernel": "decode_mk_kernel<1> (one launch = one decode step)",
                     "achieved": step_total / (ms_step * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": step_total / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"],
                     "traffic": traffic, "traffic_source": traffic_note, "bytes": step_total, "parts": sb,
                     "us": ms_step * 1e3,
                     "peak_source": peaks["source"]},
        "weight_stream_kernel": {"bound": "hbm", "kernel": f"weight_stream_kernel<1> (one persistent launch over the "
                                 f"{n_mats} projection matrices, M=1)", "us": s_ms * 1e3,
                                 "achieved": wbytes / (s_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                 "frac": wbytes / (s_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], "bytes": wbytes},
        "weight_stream": {"bound": "hbm", "kernel": f"gemv_nvfp4 ({n_mats} launches, M=1, one CUDA graph)",
                          "achieved": wbytes / w_avg_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": wbytes / w_avg_s / 1e9 / peaks["hbm_gbs"], "bytes": wbytes,
                          "us": w_avg_s * 1e6},
        "weight_stream_by_M": {"bytes": wbytes, "unit": "GB/s", "note": f"{n_mats} projections per pass, L2 "
                               "flushed, M token rows; tcgen05 = cb_gemm_nvfp4 (input preparation + tcgen05 GEMM, 2 "
                               "launches per projection), cuda_core = cb_gemv_nvfp4; cb_forward uses the GEMM from "
                               "17 token rows", "by_M": verify},
        "batched": {"note": "per GPU, ctx 32768, L2 flushed, T tokens per sequence per step (T=5: a verify "
                               "of 1 + 4 draft tokens), device-timed CUDA-graph replay", "steps": batched},
        "spec_decode": spec,
        "prefill": prefill,
        "e2e": {"value": world * args.steps / (e2e_total * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 4, "ms_per_step": e2e_total / args.steps},
        "gpu_launches": launches_per_step * args.steps,
        "launches_per_step": launches_per_step,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, sd, cache, CTX, args.cpu_budget_s, 50)
        line["cpu_baseline"]["why_port"] = CPU_ARM_WHY
    if rank == 0:
        print(json.dumps(line), flush=True)
    del wgraph
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
