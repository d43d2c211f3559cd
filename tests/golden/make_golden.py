"""Generate the golden fixtures by running the REFERENCE implementation.

Run from the repository root in a container where the reference checkout is
available (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/cirrus-s-1a

It imports the reference's own modules (``cirrus.model.model``,
``cirrus.model.layers``, ``cirrus.model.generate``, and the NVFP4 dequant of
``scripts/bench_spark.py``) and writes small ``.pt`` files next to this
script.  The oracle tests load only these files, so they run anywhere.

The reference has no NVFP4 quantiser; ``_quant_torch`` below states the
benchmark recipe (absmax/6 -> E4M3 via torch's float8 cast, E2M1 by an
explicit threshold list) independently of ``oracle/nvfp4.py``, so the oracle
test cross-checks the two.
"""

from __future__ import annotations

import argparse
import os
import sys
from dataclasses import replace

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _quant_torch(w: torch.Tensor) -> torch.Tensor:
    """Fake-quantise float32 [N, K] to NVFP4 values (tensor scale 1)."""
    N, K = w.shape
    b = w.float().reshape(N, K // 16, 16)
    s = (b.abs().amax(-1) / 6.0).to(torch.float8_e4m3fn).float()
    q = torch.where(s[..., None] > 0, b / s[..., None].clamp_min(1e-30), torch.zeros_like(b))
    a = q.abs()
    # nearest E2M1 magnitude, ties to the even code (codes 0..7 = 0, .5, 1, 1.5, 2, 3, 4, 6)
    mag = torch.full_like(a, 6.0)
    mag = torch.where(a <= 5.0, torch.full_like(a, 4.0), mag)
    mag = torch.where(a < 3.5, torch.full_like(a, 3.0), mag)
    mag = torch.where(a <= 2.5, torch.full_like(a, 2.0), mag)
    mag = torch.where(a < 1.75, torch.full_like(a, 1.5), mag)
    mag = torch.where(a <= 1.25, torch.full_like(a, 1.0), mag)
    mag = torch.where(a < 0.75, torch.full_like(a, 0.5), mag)
    mag = torch.where(a <= 0.25, torch.zeros_like(a), mag)
    val = torch.where(torch.signbit(q), -mag, mag)
    return (val * s[..., None]).reshape(N, K)


def _quantize_sd(sd: dict) -> dict:
    lin = (".qkv.weight", ".gate.weight", ".ab.weight", ".o_proj.weight", ".q_proj.weight", ".kv_proj.weight",
           ".gate_up.weight", ".down.weight", ".idx_k.weight", ".idx_q.weight", ".idx_w.weight", ".proj.weight")
    out = {}
    for k, v in sd.items():
        if k == "lm_head.weight" or any(k.endswith(s) for s in lin):
            out[k] = _quant_torch(v.float()).to(v.dtype)
        else:
            out[k] = v.clone()
    out["embed.weight"] = out["lm_head.weight"]
    return out


def _cache_to_dict(c) -> dict:
    return {"layers": [{k: v.clone() for k, v in l.items()} for l in c.layers],
            "shared": {k: v.clone() for k, v in c.shared.items()}, "pos": c.pos}


def debug_fixture(ref) -> dict:
    from cirrus.config import get_config
    from cirrus.model.generate import greedy, speculative_greedy
    from cirrus.model.model import CirrusModel

    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    try:
        out: dict = {}
        for variant, over in (("sparse", {}), ("dense", {"sparse_topk": None})):
            torch.manual_seed(0)
            cfg = replace(get_config("cirrus-s-1a-debug"), **over)
            m = CirrusModel(cfg).eval()
            sd32 = {k: v.float() for k, v in m.state_dict().items()}
            m.load_state_dict({k: (v.double() if v.is_floating_point() else v) for k, v in sd32.items()})
            g = torch.Generator().manual_seed(1)
            ids = torch.randint(0, cfg.vocab_size, (1, 20), generator=g)
            rec: dict = {"state_dict": sd32, "ids": ids}
            with torch.no_grad():
                rec["full_logits"] = m(ids).logits
                rec["last_logits_n1"] = m(ids, n_logits=1).logits
                o = m(ids[:, :11], use_cache=True)
                rec["prefill11_cache"] = _cache_to_dict(o.cache)
                steps, cache = [o.logits], o.cache
                for t in range(11, 20):
                    o = m(ids[:, t:t + 1], cache=cache)
                    steps.append(o.logits)
                    cache = o.cache
                rec["incremental_logits"] = torch.cat(steps, 1)
                rec["final_cache"] = _cache_to_dict(cache)
                # verify-style step: 4 tokens at once on top of the 11-token prefix
                o = m(ids[:, :11], use_cache=True)
                ov = m(ids[:, 11:15], cache=o.cache, n_logits=4)
                rec["verify4_logits"] = ov.logits
                V = cfg.vocab_size
                base = torch.randint(0, V, (12,), generator=g).tolist()
                prompt = base + torch.randint(0, V, (5,), generator=g).tolist() + base[:4]
                rec["gen_prompt"] = prompt
                rec["greedy"] = greedy(m, prompt, 30)[0]
                rec["spec_mtp"] = speculative_greedy(m, prompt, 30)[0]
                rec["spec_nomtp"] = speculative_greedy(m, prompt, 30, use_mtp=False)[0]
                # NVFP4 fake-quantised weights through the same reference model
                sdq = _quantize_sd(sd32)
                m.load_state_dict({k: (v.double() if v.is_floating_point() else v) for k, v in sdq.items()})
                rec["q_full_logits"] = m(ids).logits
                rec["q_greedy"] = greedy(m, prompt, 30)[0]
                out[variant] = rec
        return out
    finally:
        torch.set_default_dtype(old)


def units_fixture() -> dict:
    from cirrus.model.layers import PartialRotary, ShortConv, gated_delta_rule_ref, indexer_scores, topk_mask

    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    try:
        g = torch.Generator().manual_seed(2)
        out: dict = {}
        B, T, H, Dk, Dv = 2, 9, 3, 16, 8
        q = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(B, T, H, Dk, generator=g), dim=-1)
        v, gg, beta = torch.randn(B, T, H, Dv, generator=g), -torch.rand(B, T, H, generator=g), torch.rand(B, T, H, generator=g)
        S0 = torch.randn(B, H, Dk, Dv, generator=g) * 0.1
        o, S = gated_delta_rule_ref(q, k, v, gg, beta, Dk**-0.5, S0)
        out["gdn"] = dict(q=q, k=k, v=v, g=gg, beta=beta, S0=S0, scale=Dk**-0.5, o=o, S=S)

        torch.manual_seed(3)
        conv = ShortConv(5, 4)
        x = torch.randn(1, 7, 5, generator=g)
        y_full, c_full = conv(x, None)
        y1, c1 = conv(x[:, :3], None)
        out["conv"] = dict(w=conv.weight.detach().clone(), x=x, y=y_full, cache=c_full, y1=y1, c1=c1)

        rope = PartialRotary(64, 0.5, 1e6)
        xr = torch.randn(1, 6, 4, 64, generator=g).float()
        pos = torch.tensor([0, 1, 777, 32767, 65535, 131071])
        out["rope"] = dict(x=xr, pos=pos, y=rope(xr, pos))

        iq = torch.randn(1, 3, 4, 64, generator=g).float()
        iw = torch.randn(1, 3, 4, generator=g).float()
        ik = torch.randn(1, 300, 64, generator=g).float()
        out["indexer"] = dict(iq=iq, iw=iw, ik=ik, s=indexer_scores(iq, iw, ik))

        cases = []
        for seed, (Tq, Tk, kk) in enumerate(((1, 40, 8), (4, 40, 8), (12, 12, 4), (3, 600, 64), (5, 9, 6))):
            gs = torch.Generator().manual_seed(100 + seed)
            sc = torch.randn(1, Tq, Tk, generator=gs).clamp_min(0.0).float()
            sc[..., ::3] = 0.0
            qpos = torch.arange(Tk - Tq, Tk)
            causal = (torch.arange(Tk)[None, :] <= qpos[:, None])[None]
            cases.append(dict(scores=sc, causal=causal, k=kk, mask=topk_mask(sc, causal, kk)))
        out["topk"] = cases
        return out
    finally:
        torch.set_default_dtype(old)


def nvfp4_fixture(ref) -> dict:
    sys.path.insert(0, os.path.join(ref, "scripts"))
    import bench_spark

    g = torch.Generator().manual_seed(4)
    codes = torch.randint(0, 16, (32, 64), dtype=torch.uint8, generator=g)
    scales = (torch.rand(32, 4, generator=g) * 0.9 + 0.1).to(torch.float8_e4m3fn).view(torch.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    w = torch.randn(24, 64, generator=g) * 0.02
    return dict(codes=codes, scales=scales, packed=packed,
                dequant=bench_spark.dequant_codes(codes, scales, 1.0),
                dequant_packed_g05=bench_spark.dequant_ref(packed, scales, 0.5),
                w=w, w_q=_quant_torch(w))


def baseline_fixture() -> dict:
    sys.path.insert(0, REPO)
    from cirrus.config import get_config
    from cirrus.model.model import CirrusModel

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config

    bc = baseline_config()
    cfg = replace(get_config("cirrus-s-1a"), vocab_size=bc.vocab_size, gdn_heads=bc.gdn_heads,
                  gdn_head_dim_k=bc.gdn_head_dim_k, gdn_head_dim_v=bc.gdn_head_dim_v, n_q_heads=bc.n_q_heads,
                  n_kv_heads=bc.n_kv_heads, head_dim=bc.head_dim, swa_window=bc.swa_window,
                  sparse_topk=bc.sparse_topk, indexer_heads=bc.indexer_heads, indexer_dim=bc.indexer_dim)
    torch.manual_seed(0)
    m = CirrusModel(cfg).eval()
    sd = synthetic.random_state_dict(bc, seed=0)
    sdq = _quantize_sd(sd)
    m.load_state_dict(sdq)
    prompt = synthetic.random_prompt(48, cfg.vocab_size, seed=1)
    rec: dict = {"prompt": prompt, "num_params": m.num_params()}
    with torch.no_grad():
        o = m(torch.tensor([prompt]), use_cache=True, n_logits=1)
        rec["prefill_logits"] = o.logits[0, -1].clone()
        rec["prefill_hidden"] = o.hidden[0, -1].clone()
        toks = [int(o.logits[0, -1].argmax())]
        cache = o.cache
        for _ in range(3):
            o = m(torch.tensor([[toks[-1]]]), cache=cache, n_logits=1)
            cache = o.cache
            toks.append(int(o.logits[0, -1].argmax()))
        rec["greedy4"] = toks
        rec["step_logits"] = o.logits[0, -1].clone()
        draft = [toks[-1], prompt[5], prompt[6], prompt[7]]
        ov = m(torch.tensor([draft]), cache=cache, n_logits=4)
        rec["verify_in"] = draft
        rec["verify_argmax"] = ov.logits[0].argmax(-1).tolist()
        rec["verify_logits_first_last"] = torch.stack((ov.logits[0, 0], ov.logits[0, -1])).clone()
        rec["S_layer0_head0"] = cache.layers[0]["S"][0, 0].clone()
        rec["conv_layer0"] = cache.layers[0]["conv"][0].clone()
        rec["shared_ik_last"] = cache.shared["ik"][0, -4:].clone()
    return rec


def _token_stream(n: int, vocab: int, seed: int) -> list:
    """Uniform ids in which a quarter of the 8-token spans copy an earlier span."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, vocab, (n,), generator=g)
    for s in range(1, n // 8):
        if float(torch.rand((), generator=g)) < 0.25:
            j = int(torch.randint(0, s * 8 - 7, (), generator=g))
            toks[s * 8:s * 8 + 8] = toks[j:j + 8].clone()
    return toks.tolist()


def decoding_fixture() -> dict:
    """The reference's prompt-lookup drafter, greedy acceptance and draft choice
    (cirrus/decoding/prompt_lookup.py) on seeded token streams."""
    from cirrus.decoding.prompt_lookup import PromptLookupDrafter, accept_greedy, choose_draft

    drafts, streams = [], []
    for seed, (n, vocab) in enumerate(((400, 50), (600, 7), (300, 1000), (200, 3))):
        stream = _token_stream(n, vocab, seed)
        streams.append(stream)
        for cfg in ((2, 4, 4), (2, 4, 8), (1, 3, 5), (3, 3, 2)):
            mn, mx, k = cfg
            d = PromptLookupDrafter(max_ngram=mx, min_ngram=mn, max_draft=k)
            d.extend(stream[:1])
            for L in range(2, n + 1):
                d.extend(stream[L - 1:L])
                if L % 7 == 0 or L < 12:
                    drafts.append({"stream": seed, "len": L, "min_ngram": mn, "max_ngram": mx, "k": k,
                                   "draft": d.draft(k)})
    g = torch.Generator().manual_seed(11)
    accepts = []
    for _ in range(200):
        nd = int(torch.randint(0, 9, (), generator=g))
        draft = torch.randint(0, 4, (nd,), generator=g).tolist()
        target = torch.randint(0, 4, (nd + 1,), generator=g).tolist()
        accepts.append({"draft": draft, "target": target, "out": accept_greedy(draft, target)})
    chooses = []
    for _ in range(100):
        lk = torch.randint(0, 9, (int(torch.randint(0, 5, (), generator=g)),), generator=g).tolist()
        mt = torch.randint(0, 9, (int(torch.randint(0, 3, (), generator=g)),), generator=g).tolist()
        chooses.append({"lookup": lk, "mtp": mt, "out": choose_draft(lk, mt)})
    return {"streams": streams, "drafts": drafts, "accepts": accepts, "chooses": chooses}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--parts", default="debug,units,nvfp4,baseline,decoding",
                    help="comma-separated fixtures to write")
    args = ap.parse_args()
    ref = os.path.abspath(args.reference)
    sys.path.insert(0, ref)
    import cirrus.model.layers as L

    L._fla_chunk_gdr = None  # the exact recurrence, as scripts/bench_spark.py:968 does
    parts = set(args.parts.split(","))
    if "debug" in parts:
        torch.save(debug_fixture(ref), os.path.join(HERE, "debug_ref.pt"))
    if "units" in parts:
        torch.save(units_fixture(), os.path.join(HERE, "units_ref.pt"))
    if "nvfp4" in parts:
        torch.save(nvfp4_fixture(ref), os.path.join(HERE, "nvfp4_ref.pt"))
    if "baseline" in parts:
        torch.save(baseline_fixture(), os.path.join(HERE, "baseline_ref.pt"))
    if "decoding" in parts:
        torch.save(decoding_fixture(), os.path.join(HERE, "decoding_ref.pt"))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".pt"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
