"""torch-CPU restatement of the cirrus-s-1a forward pass.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Follows ``cirrus/model/model.py:99-176`` and ``cirrus/model/layers.py:33-339``
operation by operation, on a plain dict of tensors named like the reference
``state_dict`` (so a reference checkpoint loads unchanged).  The cache has the
reference's structure (``model.py:41-51``): one dict per self layer
(GDN ``{"conv", "S"}``, SWA ``{"k", "v"}`` holding the last ``swa_window`` keys)
plus ``shared = {"k", "v", "ik"}`` over all tokens, and ``pos``.

Differences from the reference, both optional and off by default:

* ``Casts(kv_bf16=True)`` rounds every attention K/V row to bfloat16 when it is
  produced (SWA window and shared cache), ``Casts(ik_fp8=True)`` rounds every
  indexer key to E4M3 (saturating).  These are the storage formats of the
  B200 cache; with them on, the oracle computes with exactly the stored values.
* SWA always uses the cache branch (``layers.py:233-240``) with an empty cache
  for a prompt; the reference's tests pin that the block-wise prompt path
  (``layers.py:195-210``) gives the same result.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch
import torch.nn.functional as F

from oracle import nvfp4

LINEAR_SUFFIXES = (
    ".qkv.weight", ".gate.weight", ".ab.weight", ".o_proj.weight", ".q_proj.weight", ".kv_proj.weight",
    ".gate_up.weight", ".down.weight", ".idx_k.weight", ".idx_q.weight", ".idx_w.weight", ".proj.weight",
)


@dataclass(frozen=True)
class Casts:
    kv_bf16: bool = False
    ik_fp8: bool = False


EXACT = Casts()
B200 = Casts(kv_bf16=True, ik_fp8=True)


@dataclass
class OracleCache:
    layers: list = field(default_factory=list)
    shared: dict = field(default_factory=dict)
    pos: int = 0

    def clone(self) -> "OracleCache":
        cl = lambda d: {k: v.clone() for k, v in d.items()}  # noqa: E731
        return OracleCache([cl(l) for l in self.layers], cl(self.shared), self.pos)


@dataclass
class OracleOutput:
    logits: torch.Tensor
    hidden: torch.Tensor
    cache: OracleCache | None = None
    topk: torch.Tensor | None = None  # selection mask [B, nq, Tk] when sparse


def is_linear(name: str) -> bool:
    return name == "lm_head.weight" or any(name.endswith(s) for s in LINEAR_SUFFIXES)


def quantized_params(sd: dict, tensor_scale: float = 1.0) -> dict:
    """Every Linear weight replaced by dequant(quant(W)) (NVFP4, numpy codec);
    the tied embedding follows the LM head.  Other tensors are copied."""
    out = {}
    for name, t in sd.items():
        if is_linear(name):
            w = nvfp4.fake_quant(t.detach().float().cpu().numpy(), tensor_scale)
            out[name] = torch.from_numpy(w).to(t.dtype)
        else:
            out[name] = t.detach().clone()
    if "lm_head.weight" in out:
        out["embed.weight"] = out["lm_head.weight"]
    return out


# ---------------------------------------------------------------- layers
def _acc(x):
    return x if x.dtype == torch.float64 else x.float()


def rmsnorm(x, w, eps):
    """layers.py:39-44."""
    dt = x.dtype
    x = _acc(x)
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return (x * _acc(w)).to(dt)


def linear(x, w):
    return F.linear(x, w)


def inv_freq(cfg) -> torch.Tensor:
    """layers.py:67-70."""
    rot = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
    return 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / max(rot, 1)))


def rope(x, pos, cfg):
    """Partial interleaved rotary, layers.py:72-82.  x [B, T, H, D], pos [T]."""
    inv = inv_freq(cfg)
    rot = inv.numel() * 2
    if rot == 0:
        return x
    freqs = _acc(pos)[:, None] * inv[None, :]
    cos = freqs.cos()[None, :, None, :]
    sin = freqs.sin()[None, :, None, :]
    xr, xp = _acc(x[..., :rot]), x[..., rot:]
    x1, x2 = xr[..., 0::2], xr[..., 1::2]
    out = torch.stack((x1 * cos - x2 * sin, x1 * sin + x2 * cos), dim=-1).flatten(-2)
    return torch.cat((out.to(x.dtype), xp), dim=-1)


def short_conv(x, w, cache):
    """layers.py:95-104.  x [B, T, C], w [C, K], cache [B, K-1, C] or None."""
    B, T, C = x.shape
    K = w.shape[1]
    if cache is None:
        cache = x.new_zeros(B, K - 1, C)
    xx = torch.cat((cache, x), dim=1)
    y = (xx.unfold(1, K, 1) * w).sum(-1)
    return F.silu(y), xx[:, -(K - 1):]


def gated_delta_rule(q, k, v, g, beta, scale, state=None):
    """Exact recurrence, layers.py:108-129.  State S[b, h, k, v]."""
    B, T, H, Dk = k.shape
    Dv = v.shape[-1]
    S = q.new_zeros(B, H, Dk, Dv, dtype=torch.promote_types(q.dtype, torch.float32)) if state is None else _acc(state)
    out = []
    for t in range(T):
        S = S * _acc(g[:, t]).exp()[..., None, None]
        kt, vt = _acc(k[:, t]), _acc(v[:, t])
        pred = torch.einsum("bhkv,bhk->bhv", S, kt)
        delta = _acc(beta[:, t])[..., None] * (vt - pred)
        S = S + torch.einsum("bhk,bhv->bhkv", kt, delta)
        out.append(torch.einsum("bhkv,bhk->bhv", S, _acc(q[:, t]) * scale))
    return torch.stack(out, dim=1).to(v.dtype), S


def gdn(p, pre, x, cache, cfg):
    """GatedDeltaNet.forward, layers.py:151-174 (exact recurrent path)."""
    B, T, _ = x.shape
    H, dk, dv = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v
    conv_state = cache.get("conv") if cache else None
    S0 = cache.get("S") if cache else None
    qkv, conv_state = short_conv(linear(x, p[pre + "qkv.weight"]), p[pre + "conv.weight"], conv_state)
    qk = H * dk
    q, k, v = qkv.split([qk, qk, H * dv], dim=-1)
    q = F.normalize(_acc(q.view(B, T, H, dk)), dim=-1).to(x.dtype)
    k = F.normalize(_acc(k.view(B, T, H, dk)), dim=-1).to(x.dtype)
    v = v.view(B, T, H, dv)
    a, b = _acc(linear(x, p[pre + "ab.weight"])).chunk(2, dim=-1)
    g = -_acc(p[pre + "A_log"]).exp() * F.softplus(a + _acc(p[pre + "dt_bias"]))
    beta = b.sigmoid()
    o, S = gated_delta_rule(q, k, v, g, beta, dk**-0.5, S0)
    o = rmsnorm(o, p[pre + "o_norm.weight"], cfg.norm_eps) * F.silu(linear(x, p[pre + "gate.weight"])).view(B, T, H, dv)
    return linear(o.reshape(B, T, -1), p[pre + "o_proj.weight"]), {"conv": conv_state, "S": S}


def _round_bf16(x):
    return x.to(torch.bfloat16).to(x.dtype)


def _round_e4m3(x):
    a = x.detach().float().cpu().numpy()
    return torch.from_numpy(nvfp4.e4m3_decode(nvfp4.e4m3_encode(a))).to(x.dtype)


def attend(q, k, v, mask, n_rep):
    """layers.py:183-192 with an explicit boolean mask [B or 1, T, Tk]."""
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    if n_rep > 1:
        k, v = k.repeat_interleave(n_rep, dim=1), v.repeat_interleave(n_rep, dim=1)
    o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask[:, None])
    return o.transpose(1, 2)


def swa(p, pre, x, pos, cache, cfg, casts):
    """SlidingWindowAttention.forward cache branch, layers.py:227-246."""
    B, T, _ = x.shape
    Hq, Hkv, hd = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    q = rmsnorm(linear(x, p[pre + "q_proj.weight"]).view(B, T, Hq, hd), p[pre + "q_norm.weight"], cfg.norm_eps)
    k, v = linear(x, p[pre + "kv_proj.weight"]).view(B, T, 2, Hkv, hd).unbind(2)
    q, k = rope(q, pos, cfg), rope(rmsnorm(k, p[pre + "k_norm.weight"], cfg.norm_eps), pos, cfg)
    if casts.kv_bf16:
        k, v = _round_bf16(k), _round_bf16(v)
    if cache:
        k = torch.cat((cache["k"], k), dim=1)
        v = torch.cat((cache["v"], v), dim=1)
    Tk = k.shape[1]
    kpos = torch.arange(int(pos[-1]) - Tk + 1, int(pos[-1]) + 1)
    diff = pos[:, None] - kpos[None, :]
    mask = ((diff >= 0) & (diff < cfg.swa_window))[None]
    o = attend(q, k, v, mask, Hq // Hkv)
    o = o * linear(x, p[pre + "gate.weight"]).sigmoid()[..., None]
    keep = cfg.swa_window
    return linear(o.reshape(B, T, -1), p[pre + "o_proj.weight"]), {"k": k[:, -keep:], "v": v[:, -keep:]}


def shared_kv(p, h, pos, cfg, casts):
    """SharedKV.forward, layers.py:265-279."""
    B, T, _ = h.shape
    Hkv, hd = cfg.n_kv_heads, cfg.head_dim
    x = rmsnorm(h, p["shared.norm.weight"], cfg.norm_eps)
    k, v = linear(x, p["shared.kv_proj.weight"]).view(B, T, 2, Hkv, hd).unbind(2)
    k = rope(rmsnorm(k, p["shared.k_norm.weight"], cfg.norm_eps), pos, cfg)
    if casts.kv_bf16:
        k, v = _round_bf16(k), _round_bf16(v)
    out = {"k": k, "v": v}
    if cfg.sparse_topk is not None:
        ik = linear(x, p["shared.idx_k.weight"])
        out["ik"] = _round_e4m3(ik) if casts.ik_fp8 else ik
        out["iq"] = linear(x, p["shared.idx_q.weight"]).view(B, T, cfg.indexer_heads, cfg.indexer_dim)
        out["iw"] = linear(x, p["shared.idx_w.weight"])
    return out


def indexer_scores(iq, iw, ik):
    """layers.py:282-288."""
    s = torch.einsum("bthd,bsd->bths", _acc(iq), _acc(ik)).relu()
    return torch.einsum("bths,bth->bts", s, _acc(iw))


def topk_mask(scores, causal, k):
    """layers.py:291-309 (stable sort of the flipped row: most recent key wins ties)."""
    Tk = scores.shape[-1]
    if k >= Tk:
        return causal
    s = scores.masked_fill(~causal, float("-inf"))
    order = s.flip(-1).sort(dim=-1, descending=True, stable=True).indices[..., :k]
    idx = Tk - 1 - order
    sel = torch.zeros(s.shape, dtype=torch.bool).scatter(-1, idx, True)
    diag = torch.zeros_like(sel)
    diag[..., :, -scores.shape[-2]:] = torch.eye(scores.shape[-2], dtype=torch.bool)
    return (sel | diag) & causal


def cross_attn(p, pre, x, pos, k, v, mask, cfg):
    """CrossAttention.forward, layers.py:325-331."""
    B, T, _ = x.shape
    Hq, hd = cfg.n_q_heads, cfg.head_dim
    q = rope(rmsnorm(linear(x, p[pre + "q_proj.weight"]).view(B, T, Hq, hd), p[pre + "q_norm.weight"], cfg.norm_eps),
             pos, cfg)
    o = attend(q, k, v, mask, Hq // cfg.n_kv_heads)
    o = o * linear(x, p[pre + "gate.weight"]).sigmoid()[..., None]
    return linear(o.reshape(B, T, -1), p[pre + "o_proj.weight"])


def swiglu(p, pre, x):
    """layers.py:52-54."""
    g, u = linear(x, p[pre + "gate_up.weight"]).chunk(2, dim=-1)
    return linear(F.silu(g) * u, p[pre + "down.weight"])


# ----------------------------------------------------------------- model
def forward(p: dict, cfg, input_ids: torch.Tensor, cache: OracleCache | None = None, use_cache: bool = False,
            n_logits: int | None = None, casts: Casts = EXACT) -> OracleOutput:
    """CirrusModel.forward, model.py:99-176 (inference: no labels)."""
    B, T = input_ids.shape
    start = cache.pos if cache is not None else 0
    pos = torch.arange(start, start + T)
    want_cache = use_cache or cache is not None
    eps = cfg.norm_eps

    h = p["embed.weight"][input_ids]
    new_layers = []
    for i, kind in enumerate(cfg.self_layer_kinds):
        pre = f"self_layers.{i}."
        lc = cache.layers[i] if cache is not None else None
        xin = rmsnorm(h, p[pre + "norm1.weight"], eps)
        if kind == "gdn":
            y, nc = gdn(p, pre + "mixer.", xin, lc, cfg)
        else:
            y, nc = swa(p, pre + "mixer.", xin, pos, lc, cfg, casts)
        h = h + y
        h = h + swiglu(p, pre + "ffn.", rmsnorm(h, p[pre + "norm2.weight"], eps))
        new_layers.append(nc)

    skv = shared_kv(p, h, pos, cfg, casts)
    if cache is not None and cache.shared:
        skv = {k: torch.cat((cache.shared[k], v), dim=1) for k, v in skv.items() if k in ("k", "v", "ik")} | {
            k: v for k, v in skv.items() if k in ("iq", "iw")}
    k_all, v_all = skv["k"], skv["v"]
    Tk = k_all.shape[1]

    nq = T if n_logits is None else min(n_logits, T)
    x, qpos = h[:, -nq:], pos[-nq:]
    kpos = torch.arange(Tk)
    mask = (kpos[None, :] <= qpos[:, None])[None]
    sel = None
    if cfg.sparse_topk is not None:
        scores = indexer_scores(skv["iq"][:, -nq:], skv["iw"][:, -nq:], skv["ik"])
        mask = topk_mask(scores, mask, cfg.sparse_topk)
        sel = mask
    for j in range(cfg.n_cross_layers):
        pre = f"cross_layers.{j}."
        x = x + cross_attn(p, pre + "mixer.", rmsnorm(x, p[pre + "norm1.weight"], eps), qpos, k_all, v_all, mask, cfg)
        x = x + swiglu(p, pre + "ffn.", rmsnorm(x, p[pre + "norm2.weight"], eps))

    hn = rmsnorm(x, p["final_norm.weight"], eps)
    logits = linear(hn, p["lm_head.weight"])
    out = OracleOutput(logits=logits, hidden=x, topk=sel)
    if want_cache:
        out.cache = OracleCache(new_layers, {k: skv[k] for k in ("k", "v", "ik") if k in skv}, start + T)
    return out


def mtp_draft(p: dict, cfg, h_last: torch.Tensor, token: int, n: int | None = None, draft_ids=None) -> list:
    """CirrusModel.mtp_draft, model.py:230-245, for the first MTP module."""
    if cfg.n_mtp_heads == 0:
        return []
    n = cfg.mtp_passes if n is None else n
    eps = cfg.norm_eps
    ids = torch.arange(min(cfg.mtp_draft_vocab, cfg.vocab_size)) if draft_ids is None else draft_ids
    W = p["embed.weight"][ids]
    h, tok, out = h_last[:, None], torch.tensor([[token]]), []
    for _ in range(n):
        e = p["embed.weight"][tok]
        xx = linear(torch.cat((rmsnorm(h, p["mtp.0.norm_h.weight"], eps), rmsnorm(e, p["mtp.0.norm_e.weight"], eps)), -1),
                    p["mtp.0.proj.weight"])
        h = xx + swiglu(p, "mtp.0.ffn.", rmsnorm(xx, p["mtp.0.ffn_norm.weight"], eps))
        idx = (rmsnorm(h, p["final_norm.weight"], eps)[:, -1] @ W.T).argmax(-1)
        tok = ids[idx].view(1, 1)
        out.append(int(tok))
    return out


def greedy(p: dict, cfg, prompt: list, max_new: int, casts: Casts = EXACT) -> list:
    """generate.greedy, generate.py:28-40."""
    out = forward(p, cfg, torch.tensor([prompt]), use_cache=True, n_logits=1, casts=casts)
    gen = []
    while True:
        tok = int(out.logits[0, -1].argmax())
        gen.append(tok)
        if len(gen) >= max_new:
            return gen
        out = forward(p, cfg, torch.tensor([[tok]]), cache=out.cache, n_logits=1, casts=casts)


__all__ = ["Casts", "EXACT", "B200", "OracleCache", "OracleOutput", "forward", "greedy", "mtp_draft",
           "quantized_params", "is_linear", "topk_mask", "indexer_scores", "gated_delta_rule", "short_conv",
           "rope", "rmsnorm", "inv_freq"]
