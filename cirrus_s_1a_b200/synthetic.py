"""Seeded synthetic weights, prompts and caches (no checkpoints or datasets exist offline).

``random_state_dict`` draws a full parameter set with the reference's key
names, shapes and initial distributions (``cirrus/model/model.py:85-90``:
every Linear and the embedding N(0, 0.02); ``layers.py:93`` conv taps
N(0, 1/sqrt(k)); ``layers.py:147-149`` A_log = log U(1, 16) and dt_bias =
softplus^-1 of a log-uniform step in [1e-3, 1e-1]; norm weights one).  The
draw order is this module's own, so the values differ from the reference's
RNG stream; every consumer (bench, tests, oracle) loads the same dict.

``random_prompt`` builds the benchmark's n-gram-repeating token stream: a
uniform stream in which a fraction of 8-token spans are copies of earlier spans.
"""

from __future__ import annotations

import math

import torch


def linear_shapes(cfg) -> dict:
    """Reference state_dict names -> shapes for every Linear weight (model.py / layers.py)."""
    d, ffn = cfg.d_model, cfg.ffn_hidden
    H, dk, dv = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v
    out = {}
    for i, kind in enumerate(cfg.self_layer_kinds):
        p = f"self_layers.{i}."
        if kind == "gdn":
            out[p + "mixer.qkv.weight"] = (2 * H * dk + H * dv, d)
            out[p + "mixer.gate.weight"] = (H * dv, d)
            out[p + "mixer.ab.weight"] = (2 * H, d)
            out[p + "mixer.o_proj.weight"] = (d, H * dv)
        else:
            out[p + "mixer.q_proj.weight"] = (cfg.q_dim, d)
            out[p + "mixer.kv_proj.weight"] = (2 * cfg.kv_dim, d)
            out[p + "mixer.gate.weight"] = (cfg.n_q_heads, d)
            out[p + "mixer.o_proj.weight"] = (d, cfg.q_dim)
        out[p + "ffn.gate_up.weight"] = (2 * ffn, d)
        out[p + "ffn.down.weight"] = (d, ffn)
    out["shared.kv_proj.weight"] = (2 * cfg.kv_dim, d)
    if cfg.sparse_topk is not None:
        out["shared.idx_k.weight"] = (cfg.indexer_dim, d)
        out["shared.idx_q.weight"] = (cfg.indexer_heads * cfg.indexer_dim, d)
        out["shared.idx_w.weight"] = (cfg.indexer_heads, d)
    for j in range(cfg.n_cross_layers):
        p = f"cross_layers.{j}."
        out[p + "mixer.q_proj.weight"] = (cfg.q_dim, d)
        out[p + "mixer.gate.weight"] = (cfg.n_q_heads, d)
        out[p + "mixer.o_proj.weight"] = (d, cfg.q_dim)
        out[p + "ffn.gate_up.weight"] = (2 * ffn, d)
        out[p + "ffn.down.weight"] = (d, ffn)
    out["lm_head.weight"] = (cfg.vocab_size, d)
    for m in range(cfg.n_mtp_heads):
        p = f"mtp.{m}."
        out[p + "proj.weight"] = (d, 2 * d)
        out[p + "ffn.gate_up.weight"] = (2 * ffn, d)
        out[p + "ffn.down.weight"] = (d, ffn)
    return out


def norm_shapes(cfg) -> dict:
    d = cfg.d_model
    out = {}
    for i, kind in enumerate(cfg.self_layer_kinds):
        p = f"self_layers.{i}."
        out[p + "norm1.weight"] = (d,)
        out[p + "norm2.weight"] = (d,)
        if kind == "gdn":
            out[p + "mixer.o_norm.weight"] = (cfg.gdn_head_dim_v,)
        else:
            out[p + "mixer.q_norm.weight"] = (cfg.head_dim,)
            out[p + "mixer.k_norm.weight"] = (cfg.head_dim,)
    out["shared.norm.weight"] = (d,)
    out["shared.k_norm.weight"] = (cfg.head_dim,)
    for j in range(cfg.n_cross_layers):
        p = f"cross_layers.{j}."
        out[p + "norm1.weight"] = (d,)
        out[p + "norm2.weight"] = (d,)
        out[p + "mixer.q_norm.weight"] = (cfg.head_dim,)
    out["final_norm.weight"] = (d,)
    for m in range(cfg.n_mtp_heads):
        p = f"mtp.{m}."
        for n in ("norm_h", "norm_e", "ffn_norm"):
            out[p + n + ".weight"] = (d,)
    return out


def random_state_dict(cfg, seed: int = 0, norm_jitter: float = 0.0) -> dict:
    """float32 CPU tensors keyed like the reference ``CirrusModel.state_dict()``.

    ``norm_jitter`` > 0 draws norm weights as 1 + N(0, jitter) instead of ones,
    which makes parity tests sensitive to which norm weight is applied where.
    """
    g = torch.Generator().manual_seed(seed)
    sd: dict = {}
    for name, shape in linear_shapes(cfg).items():
        sd[name] = torch.randn(shape, generator=g) * 0.02
    sd["embed.weight"] = sd["lm_head.weight"]  # tied (model.py:76-77)
    for name, shape in norm_shapes(cfg).items():
        sd[name] = torch.ones(shape) + (torch.randn(shape, generator=g) * norm_jitter if norm_jitter else 0.0)
    C = 2 * cfg.gdn_heads * cfg.gdn_head_dim_k + cfg.gdn_heads * cfg.gdn_head_dim_v
    for i, kind in enumerate(cfg.self_layer_kinds):
        if kind != "gdn":
            continue
        p = f"self_layers.{i}.mixer."
        sd[p + "conv.weight"] = torch.randn((C, cfg.gdn_conv_size), generator=g) / math.sqrt(cfg.gdn_conv_size)
        sd[p + "A_log"] = torch.log(torch.rand(cfg.gdn_heads, generator=g) * 15.0 + 1.0)
        dt = torch.exp(torch.rand(cfg.gdn_heads, generator=g) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
        sd[p + "dt_bias"] = dt + torch.log(-torch.expm1(-dt))
    sd["draft_ids"] = torch.arange(min(cfg.mtp_draft_vocab, cfg.vocab_size))
    return sd


def fill_cache(cache, ctx: int, seed: int, ties: str | None = None) -> None:
    """Seeded synthetic decode state at context ``ctx`` for every sequence of a
    ``DeviceCache`` (the stand-in for a real ``ctx``-token prompt): GDN state
    N(0, 0.1), conv windows N(0, 1), SWA ring and shared K/V bf16 N(0, 1),
    indexer keys E4M3 of N(0, 1); positions are set to ``ctx - 1``, so the next
    one-token forward sees ``ctx`` keys.

    ``ties`` makes the indexer scores tie heavily, so that the most-recent-first
    tie rule decides the selection: ``"repeat"`` zeroes every key (score exactly
    0 after the ReLU) and then copies 64 random keys to ctx/8 positions, so every
    nonzero score belongs to a run of about 64 exactly equal scores and the k-th
    largest is always tied; ``"zero"`` keeps 0.5% of the keys random and zeroes
    the rest, so fewer than k keys score above 0 and the threshold falls inside
    the run of zeros.
    """
    g = torch.Generator(device=cache.kv_k.device).manual_seed(seed)
    dev = cache.kv_k.device
    cache.gdn_state.normal_(0.0, 0.1, generator=g)
    cache.gdn_conv.normal_(0.0, 1.0, generator=g)
    for t in (cache.swa_k, cache.swa_v):
        t.copy_(torch.randn(t.shape, generator=g, device=dev).to(torch.bfloat16))
    for t in (cache.kv_k, cache.kv_v):
        t[:, :ctx].copy_(torch.randn(t[:, :ctx].shape, generator=g, device=dev).to(torch.bfloat16))
    di = cache.model.cfg.indexer_dim
    ik = torch.randn((cache.batch, ctx, di), generator=g, device=dev)
    if ties is not None:
        if ties not in ("repeat", "zero"):
            raise ValueError("ties must be None, 'repeat' or 'zero'")
        keep = torch.rand((cache.batch, ctx, 1), generator=g, device=dev) < (0.0 if ties == "repeat" else 0.005)
        ik = ik * keep
        if ties == "repeat":
            src = torch.randn((cache.batch, 64, di), generator=g, device=dev)
            for b in range(cache.batch):
                rows = torch.randint(0, ctx, (ctx // 8,), generator=g, device=dev)
                ik[b, rows] = src[b, torch.randint(0, 64, (ctx // 8,), generator=g, device=dev)]
    cache.kv_ik[:, :ctx, :di].copy_(ik.to(torch.float8_e4m3fn).view(torch.uint8))
    cache.pos_dev.fill_(ctx - 1)
    cache.pos_host = [ctx - 1] * cache.batch


def random_prompt(n: int, vocab: int, seed: int = 0, copy_frac: float = 0.25, span: int = 8) -> list:
    """``n`` token ids: uniform over the vocabulary, except that each 8-token span
    is, with probability ``copy_frac``, a copy of an earlier span."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, vocab, (n,), generator=g)
    u = torch.rand(n // span + 1, generator=g)
    src = torch.rand(n // span + 1, generator=g)
    for s in range(1, n // span):
        if u[s] < copy_frac:
            start = s * span
            j = int(src[s] * (start - span + 1))
            toks[start:start + span] = toks[j:j + span].clone()
    return toks.tolist()
