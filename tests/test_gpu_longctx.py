"""Parity of the benchmarked configuration: the B200 forward at 32K and 128K
context compared with the CPU oracle, and the persistent kernel's top-k
selections compared bit for bit with the reference tie rule.

* Top-k (``layers.py:291-309``; the reference's own tie test is
  ``tests/test_model.py:100-111``): after one forward the selections of every
  query row are read back from the workspace (``cb_workspace_layout``) together
  with the indexer query and weights the kernel used; the oracle recomputes
  the scores in the same fixed float32 order (``oracle/indexer.py``) and
  selects with the reference rule.  The selections must be identical.  The
  synthetic caches make ties dominate (``synthetic.fill_cache(ties=...)``):
  runs of repeated keys around the k-th largest score, or a threshold inside a
  run of exactly-zero scores covering almost every key.
* Logits: a tau=1 step and a 5-token verify from a synthetic 32K cache on
  both GPU paths, against the oracle stepped from the exported cache
  (1e-2 relative / 2e-2 absolute).
* SWA ring wrap at window 2048: decode past position 2064 (window + 16 ring slots).
* configs[0] as written: a 512-token prompt and 128 greedy steps, teacher-forced
  with the oracle's tokens so that every step's logits are compared; the GPU's
  argmax must equal the oracle's except where the oracle's top-2 margin is
  below 2e-2 (a documented near-tie).
* 128K context at batch 16 (one launch per op), and a cache with
  max_ctx just above 131072, where the persistent kernel does not apply.
"""

import numpy as np
import pytest
import torch

from oracle import indexer as oi
from oracle import model as om

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2
CTX = 32768


def _engine(cfg, sd, max_ctx, path="auto"):
    from cirrus_s_1a_b200.engine import CirrusB200

    return CirrusB200(cfg, sd, max_ctx=max_ctx, path=path)


def _setup(seed=0):
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=seed, norm_jitter=0.1)
    return cfg, sd


def _close(a, b, what):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    torch.testing.assert_close(a, b, rtol=RTOL, atol=ATOL, msg=lambda m: f"{what}: max abs err {err}\n{m}")


def _oracle_cache(cache, b=0):
    ref = cache.to_reference(b)
    return om.OracleCache(ref["layers"], ref["shared"], ref["pos"])


def _check_selections(eng, cache, T, nq, pos_before):
    """Every query row's selection equals the oracle rule on the kernel's own scores."""
    cfg = eng.cfg
    m = eng.model.desc
    Hi, Di, k = cfg.indexer_heads, cfg.indexer_dim, cfg.sparse_topk
    inter = eng.intermediates(cache, T)
    proj = inter["proj"].cpu()
    sel_idx, sel_cnt = inter["sel_idx"].cpu(), inter["sel_cnt"].cpu()
    Tc = min(T, 8)
    for b in range(cache.batch):
        n_keys = pos_before[b] + T
        ik = cache.kv_ik[b, :n_keys, :Di].contiguous().cpu().view(torch.float8_e4m3fn).float().numpy()
        for j in range(nq):
            t = Tc - nq + j
            row = proj[b * Tc + t]
            iq = row[m.sh_off_iq:m.sh_off_iq + Hi * Di].numpy().reshape(Hi, Di)
            iw = row[m.sh_off_iw:m.sh_off_iw + Hi].numpy()
            p = pos_before[b] + t
            scores = oi.indexer_scores(iq, iw, ik[:p + 1])
            want = oi.topk_select(scores, k)
            r = b * nq + j
            got = sel_idx[r, :int(sel_cnt[r])].numpy()
            assert len(got) == len(want), (b, j, len(got), len(want))
            assert np.array_equal(got, want), (b, j, np.setdiff1d(want, got)[:8], np.setdiff1d(got, want)[:8])
            yield scores, want


@pytest.mark.parametrize("ties", ["repeat", "zero", None])
@pytest.mark.parametrize("T", [1, 5])
def test_persistent_topk_selection_is_bit_exact_at_32k(ties, T):
    from cirrus_s_1a_b200 import synthetic

    cfg, sd = _setup(seed=3)
    eng = _engine(cfg, sd, CTX + 64)
    cache = eng.new_cache(1)
    synthetic.fill_cache(cache, CTX, seed=5, ties=ties)
    before = list(cache.pos_host)
    ids = torch.randint(0, cfg.vocab_size, (1, T), generator=torch.Generator().manual_seed(7))
    eng(ids, cache=cache, n_logits=T)
    assert eng.read_status(cache, T) == 0
    for scores, want in _check_selections(eng, cache, T, T, before):
        kth = np.sort(scores)[::-1][cfg.sparse_topk - 1]
        if ties == "zero":
            assert kth == 0.0  # the threshold lies inside the run of zero scores
        if ties is not None:
            assert (scores == kth).sum() > 1  # the k-th score is tied


@pytest.mark.parametrize("path", ["auto", "multi"])
def test_step_and_verify_match_oracle_at_32k(path):
    from cirrus_s_1a_b200 import synthetic

    cfg, sd = _setup(seed=4)
    p = om.quantized_params(sd)
    eng = _engine(cfg, sd, CTX + 64, path)
    cache = eng.new_cache(1)
    synthetic.fill_cache(cache, CTX - 8, seed=6)
    oc = _oracle_cache(cache)
    tok = 123
    for s in range(2):
        o = eng(torch.tensor([[tok]]), cache=cache, n_logits=1)
        r = om.forward(p, cfg, torch.tensor([[tok]]), cache=oc, n_logits=1, casts=om.B200)
        oc = r.cache
        _close(o.logits, r.logits, f"32K step {s}")
        tok = int(r.logits[0, -1].argmax())
    draft = [tok, 5, 77, 901, 12]
    snap, oc_snap = cache.clone(), oc.clone()
    o = eng(torch.tensor([draft]), cache=cache, n_logits=5)
    r = om.forward(p, cfg, torch.tensor([draft]), cache=oc, n_logits=5, casts=om.B200)
    _close(o.logits, r.logits, "32K verify of 5")
    _close(o.hidden, r.hidden, "32K verify hidden")
    assert eng.read_status(cache, 5) == 0
    # a snapshot taken before the verify (the reference's rewind, generate.py:71-77)
    # still decodes like the oracle after the verify has overwritten scratch rows
    o = eng(torch.tensor([draft[:2]]), cache=snap, n_logits=1)
    r = om.forward(p, cfg, torch.tensor([draft[:2]]), cache=oc_snap, n_logits=1, casts=om.B200)
    _close(o.logits, r.logits, "32K re-run from the snapshot")


@pytest.mark.parametrize("path", ["auto", "multi"])
def test_swa_ring_wraps_at_window_2048(path):
    from cirrus_s_1a_b200 import synthetic

    cfg, sd = _setup(seed=8)
    assert cfg.swa_window == 2048
    p = om.quantized_params(sd)
    eng = _engine(cfg, sd, 4096, path)
    cache = eng.new_cache(1)
    synthetic.fill_cache(cache, 2060, seed=9)  # positions 2059.. cross the 2064-slot ring
    oc = _oracle_cache(cache)
    tok = 44
    for s in range(6):
        o = eng(torch.tensor([[tok]]), cache=cache, n_logits=1)
        r = om.forward(p, cfg, torch.tensor([[tok]]), cache=oc, n_logits=1, casts=om.B200)
        oc = r.cache
        _close(o.logits, r.logits, f"wrap step {s} at position {cache.pos - 1}")
        tok = int(r.logits[0, -1].argmax())
    assert cache.pos > 2064
    draft = [tok, 3, 1000, 31999, 8]
    o = eng(torch.tensor([draft]), cache=cache, n_logits=5)
    r = om.forward(p, cfg, torch.tensor([draft]), cache=oc, n_logits=5, casts=om.B200)
    _close(o.logits, r.logits, "wrap verify of 5")
    exp = cache.to_reference()
    for i, (a, b) in enumerate(zip(exp["layers"], r.cache.layers)):
        if "k" in a:  # the SWA window keys, in position order, against the oracle's window
            torch.testing.assert_close(a["k"], b["k"].float(), rtol=2e-2, atol=2e-2, msg=f"layer {i} window keys")


@pytest.mark.parametrize("path", ["auto", "multi"])
def test_configs0_prompt512_greedy128(path):
    """512-token prompt (ids uniform, seed 0), 128 greedy steps."""
    cfg, sd = _setup(seed=0)
    p = om.quantized_params(sd)
    eng = _engine(cfg, sd, 1024, path)
    prompt = torch.randint(0, cfg.vocab_size, (1, 512), generator=torch.Generator().manual_seed(0))
    o = eng(prompt, use_cache=True, n_logits=1)
    r = om.forward(p, cfg, prompt, use_cache=True, n_logits=1, casts=om.B200)
    _close(o.logits, r.logits, "prefill 512")
    cache, oc = o.cache, r.cache
    agree, near_ties = 0, 0
    for s in range(128):
        lg = r.logits[0, -1]
        top2 = lg.topk(2).values
        want = int(lg.argmax())
        got = int(o.logits[0, -1].argmax())
        if got == want:
            agree += 1
        else:
            assert float(top2[0] - top2[1]) < ATOL, f"step {s}: GPU {got} != oracle {want}"
            near_ties += 1
        o = eng(torch.tensor([[want]]), cache=cache, n_logits=1)
        r = om.forward(p, cfg, torch.tensor([[want]]), cache=oc, n_logits=1, casts=om.B200)
        oc = r.cache
        _close(o.logits, r.logits, f"greedy step {s}")
    assert agree >= 120, (agree, near_ties)
    assert eng.read_status(cache) == 0


def test_128k_batch16_and_fallback_above_131072():
    """batch 16 at 128K (one launch per op: batch * T > 8) and a
    batch-1 cache with max_ctx above 131072 (past the persistent kernel's
    selection bitmap), both against the oracle."""
    from cirrus_s_1a_b200 import synthetic

    cfg, sd = _setup(seed=12)
    p = om.quantized_params(sd)
    eng = _engine(cfg, sd, 131072)
    cache = eng.new_cache(16)
    synthetic.fill_cache(cache, 131072 - 8, seed=13)
    before = list(cache.pos_host)
    ocs = [_oracle_cache(cache, b) for b in (0, 11)]
    toks = torch.randint(0, cfg.vocab_size, (16, 1), generator=torch.Generator().manual_seed(2))
    o = eng(toks, cache=cache, n_logits=1)
    assert eng.read_status(cache) == 0
    for b, oc in zip((0, 11), ocs):
        r = om.forward(p, cfg, toks[b:b + 1], cache=oc, n_logits=1, casts=om.B200)
        _close(o.logits[b], r.logits[0], f"128K batch-16 row {b}")
    assert sum(1 for _ in _check_selections(eng, cache, 1, 1, before)) == 16
    del cache
    torch.cuda.empty_cache()

    eng2 = _engine(cfg, sd, 131072 + 64)
    c2 = eng2.new_cache(1)
    synthetic.fill_cache(c2, 131072 + 40, seed=14)
    before = list(c2.pos_host)
    oc = _oracle_cache(c2)
    tok = torch.tensor([[77]])
    o = eng2(tok, cache=c2, n_logits=1)
    r = om.forward(p, cfg, tok, cache=oc, n_logits=1, casts=om.B200)
    _close(o.logits, r.logits, "max_ctx 131136 (multi-kernel fallback)")
    assert sum(1 for _ in _check_selections(eng2, c2, 1, 1, before)) == 1
