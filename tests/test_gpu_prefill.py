"""Prompt prefill on the prefill kernels (cb_forward with T > CB_MAX_T at the
benchmark shapes: tensor-core GEMMs, chunked Gated DeltaNet with the conv,
gating and gated RMSNorm fused, block-wise SWA over the ring) against the
oracle's restatement of ``CirrusModel.forward`` on the same NVFP4 weights with
the B200 storage casts.

Prompts span several CB_PREFILL_CHUNK chunks, including one longer than the
SWA window (the ring wraps inside the prefill and the block attention masks
keys that left the window) and one whose cross-decoder top-k selects 512 of
more than 512 keys.  Tolerances as for the decode path: logits within 1e-2
relative / 2e-2 absolute; the caches the prefill leaves behind (GDN state,
conv windows, SWA ring, shared K/V) within 2e-2."""

import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2


def _setup(seed=0, max_ctx=4096):
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=seed, norm_jitter=0.1)
    return cfg, CirrusB200(cfg, sd, max_ctx=max_ctx), om.quantized_params(sd)


def _close(a, b, what, rtol=RTOL, atol=ATOL):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol, msg=lambda m: f"{what}: max abs err {err}\n{m}")


def _check_cache(cache, cref, b=0):
    exp = cache.to_reference(b)
    assert exp["pos"] == cref.pos
    for i, (x, y) in enumerate(zip(exp["layers"], cref.layers)):
        for key in x:
            ref = y[key][b:b + 1].float() if y[key].shape[0] > 1 else y[key].float()
            _close(x[key], ref, f"layer {i} {key}", rtol=2e-2, atol=2e-2)
    for key in ("k", "v"):
        ref = cref.shared[key][b:b + 1] if cref.shared[key].shape[0] > 1 else cref.shared[key]
        _close(exp["shared"][key], ref, f"shared {key}", rtol=5e-2, atol=5e-2)


def test_multi_chunk_prompt_all_logits():
    """300 tokens = chunks of 128, 128, 44; logits of every position."""
    from cirrus_s_1a_b200 import synthetic

    cfg, eng, p = _setup(seed=1)
    prompt = synthetic.random_prompt(300, cfg.vocab_size, seed=5)
    ids = torch.tensor([prompt])
    o_ref = om.forward(p, cfg, ids, use_cache=True, casts=om.B200)
    o = eng(ids, use_cache=True)
    _close(o.logits, o_ref.logits, "logits")
    _close(o.hidden, o_ref.hidden, "hidden")
    _check_cache(o.cache, o_ref.cache)
    cache, cref = o.cache, o_ref.cache
    for s in range(4):  # decode continues from the prefilled cache
        tok = int(o_ref.logits[0, -1].argmax())
        o_ref = om.forward(p, cfg, torch.tensor([[tok]]), cache=cref, n_logits=1, casts=om.B200)
        o = eng(torch.tensor([[tok]]), cache=cache, n_logits=1)
        cref, cache = o_ref.cache, o.cache
        _close(o.logits, o_ref.logits, f"decode {s}")
    assert eng.read_status(cache) == 0


@pytest.mark.parametrize("n", [9, 127, 128, 129])
def test_chunk_boundaries(n):
    from cirrus_s_1a_b200 import synthetic

    cfg, eng, p = _setup(seed=2, max_ctx=512)
    ids = torch.tensor([synthetic.random_prompt(n, cfg.vocab_size, seed=n)])
    o_ref = om.forward(p, cfg, ids, use_cache=True, n_logits=3, casts=om.B200)
    o = eng(ids, use_cache=True, n_logits=3)
    _close(o.logits, o_ref.logits, f"logits n={n}")
    _check_cache(o.cache, o_ref.cache)


def test_prompt_longer_than_window():
    """2300 tokens: the SWA ring wraps during the prefill (window 2048), the top-k
    of the last query selects 512 + 1 of 2300 keys; then two decode steps."""
    from cirrus_s_1a_b200 import synthetic

    cfg, eng, p = _setup(seed=3)
    prompt = synthetic.random_prompt(2300, cfg.vocab_size, seed=7)
    ids = torch.tensor([prompt])
    o_ref = om.forward(p, cfg, ids, use_cache=True, n_logits=2, casts=om.B200)
    o = eng(ids, use_cache=True, n_logits=2)
    _close(o.logits, o_ref.logits, "logits")
    _check_cache(o.cache, o_ref.cache)
    cache, cref = o.cache, o_ref.cache
    for s in range(2):
        tok = int(o_ref.logits[0, -1].argmax())
        o_ref = om.forward(p, cfg, torch.tensor([[tok]]), cache=cref, n_logits=1, casts=om.B200)
        o = eng(torch.tensor([[tok]]), cache=cache, n_logits=1)
        cref, cache = o_ref.cache, o.cache
        _close(o.logits, o_ref.logits, f"decode {s}")


def test_batched_prompts_match_individual_runs():
    from cirrus_s_1a_b200 import synthetic

    cfg, eng, p = _setup(seed=4, max_ctx=512)
    prompts = [synthetic.random_prompt(200, cfg.vocab_size, seed=s) for s in (20, 21, 22)]
    o = eng(torch.tensor(prompts), use_cache=True, n_logits=1)
    for b, pr in enumerate(prompts):
        r = om.forward(p, cfg, torch.tensor([pr]), use_cache=True, n_logits=1, casts=om.B200)
        _close(o.logits[b:b + 1], r.logits, f"sequence {b}")
        _check_cache(o.cache, r.cache, b)
