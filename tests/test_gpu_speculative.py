"""Speculative decoding on the B200 (``cirrus_s_1a_b200.speculative``) and the
device MTP draft head, against the oracle and against plain greedy decoding.

* ``cb_prompt_lookup_draft``: the drafts of a batch of token histories equal
  the reference rule (``oracle/decoding.py``, pinned to
  ``cirrus/decoding/prompt_lookup.py`` by ``tests/golden/decoding_ref.pt``),
  including the per-sequence budget cap and the padding of the verify input.
* ``SpecDecoder``: with ``max_draft = 0`` it is greedy decoding and emits the
  same tokens as token-by-token eager forwards; with drafts it emits the same
  tokens as greedy (the reference's invariant, ``tests/test_model.py:89-97``),
  rewinding partial acceptances from the per-token GDN snapshots.  Where the
  greedy run's own top-2 logit margin is below 2e-2 the two may part (a
  documented near-tie: the verify forward computes the same position with a
  different token width).
* ``CirrusB200.mtp_draft``: the drafted tokens equal the oracle's
  ``mtp_draft`` (``cirrus/model/model.py:230-245``) from the same hidden state.
"""

import numpy as np
import pytest
import torch

from oracle import decoding as od
from oracle import model as om

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _engine(name, seed=3, max_ctx=512):
    from dataclasses import replace

    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config, get_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = {"debug": get_config("cirrus-s-1a-debug"), "baseline": baseline_config(),
           "debug_dense": replace(get_config("cirrus-s-1a-debug"), sparse_topk=None)}[name]
    sd = synthetic.random_state_dict(cfg, seed=seed, norm_jitter=0.1)
    return CirrusB200(cfg, sd, max_ctx=max_ctx), sd


def test_device_drafter_matches_reference_rule():
    from cirrus_s_1a_b200 import _lib

    L = _lib.lib()
    rng = np.random.default_rng(0)
    B, ld, T = 12, 700, 6
    toks = np.zeros((B, ld), dtype=np.int32)
    lens = np.zeros(B, dtype=np.int32)
    budget = np.zeros(B, dtype=np.int32)
    for b in range(B):
        n = int(rng.integers(1, ld - 10))
        vocab = int(rng.choice([3, 7, 50, 1000]))
        toks[b, :n] = rng.integers(0, vocab, n)
        lens[b] = n
        budget[b] = int(rng.choice([0, 1, 2, 3, 100]))
    for mn, mx, md in ((2, 4, 5), (1, 3, 3), (3, 4, 8)):
        dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
        t, l_, bu = dev(toks), dev(lens), dev(budget)
        ids = torch.full((B, T), -1, dtype=torch.int64, device="cuda")
        dl = torch.full((B,), -1, dtype=torch.int32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        _lib.check(L.cb_prompt_lookup_draft(t.data_ptr(), ld, l_.data_ptr(), bu.data_ptr(), B, mn, mx, md,
                                            ids.data_ptr(), T, dl.data_ptr(), st), "draft")
        ids, dl = ids.cpu().numpy(), dl.cpu().numpy()
        for b in range(B):
            hist = toks[b, :lens[b]].tolist()
            cap = min(md, T - 1, int(budget[b]) - 1)
            want = od.lookup_draft(hist, cap, mn, mx) if cap > 0 else []
            assert dl[b] == len(want), (b, mn, mx, md)
            assert ids[b, 0] == hist[-1]
            assert ids[b, 1:1 + len(want)].tolist() == want
            assert (ids[b, 1 + len(want):] == hist[-1]).all()


def _eager_greedy(eng, prompts, n):
    """Token-by-token greedy with logits (for the near-tie margins)."""
    o = eng(torch.tensor(prompts), use_cache=True, n_logits=1)
    cache, toks, margins = o.cache, [[] for _ in prompts], [[] for _ in prompts]
    for _ in range(n):
        lg = o.logits[:, -1].float().cpu()
        top2 = lg.topk(2, dim=-1).values
        nxt = lg.argmax(-1)
        for b in range(len(prompts)):
            toks[b].append(int(nxt[b]))
            margins[b].append(float(top2[b, 0] - top2[b, 1]))
        o = eng(nxt.view(-1, 1), cache=cache, n_logits=1)
    return toks, margins


def _agree(got, want, margins, what):
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b:
            assert margins[i] < ATOL, f"{what}: token {i}: {a} != {b}, greedy margin {margins[i]}"
            return i
    assert len(got) == len(want), what
    return len(got)


@pytest.mark.parametrize("name,batch", [("debug", 2), ("debug_dense", 3), ("baseline", 1), ("baseline", 3)])
def test_spec_decoder_emits_the_greedy_tokens(name, batch):
    from cirrus_s_1a_b200.speculative import SpecDecoder

    eng, _ = _engine(name)
    vocab = eng.cfg.vocab_size
    g = torch.Generator().manual_seed(5)
    prompts = []
    for _ in range(batch):
        base = torch.randint(0, vocab, (10,), generator=g).tolist()
        prompts.append(base + torch.randint(0, vocab, (6,), generator=g).tolist() + base[:5])
    n = 40
    want, margins = _eager_greedy(eng, prompts, n)

    greedy = SpecDecoder(eng, eng.new_cache(batch), max_draft=0)
    greedy.start(prompts, n)
    greedy.capture()
    got_g, st_g = greedy.run()
    spec = SpecDecoder(eng, eng.new_cache(batch), max_draft=4)
    spec.start(prompts, n)
    spec.capture()
    got_s, st_s = spec.run()
    for b in range(batch):
        assert len(got_g[b]) == n and len(got_s[b]) == n
        _agree(got_g[b], want[b], margins[b], f"device greedy seq {b}")
        _agree(got_s[b], want[b], margins[b], f"speculative seq {b}")
    assert st_g.tokens == batch * n
    assert st_s.steps <= st_g.steps
    assert eng.read_status(spec.cache, spec.T) == 0


def test_spec_decoder_rewinds_partial_acceptance():
    """A prompt that is one span repeated makes the drafter propose long drafts
    that the (random) model mostly rejects: every step rewinds, and the tokens
    still follow greedy."""
    from cirrus_s_1a_b200.speculative import SpecDecoder

    eng, _ = _engine("baseline", seed=7)
    g = torch.Generator().manual_seed(9)
    span = torch.randint(0, eng.cfg.vocab_size, (6,), generator=g).tolist()
    prompts = [span * 5 + span[:3]]
    want, margins = _eager_greedy(eng, prompts, 24)
    spec = SpecDecoder(eng, eng.new_cache(1), max_draft=7)
    spec.start(prompts, 24)
    got, stats = spec.run(check_every=1)
    _agree(got[0], want[0], margins[0], "repeated-span prompt")
    assert stats.tokens == 24


@pytest.mark.parametrize("name", ["debug", "baseline"])
def test_mtp_draft_matches_oracle(name):
    eng, sd = _engine(name, seed=4)
    cfg = eng.cfg
    p = om.quantized_params(sd)
    g = torch.Generator().manual_seed(2)
    for trial in range(3):
        prompt = torch.randint(0, cfg.vocab_size, (1, 12), generator=g)
        r = om.forward(p, cfg, prompt, use_cache=True, n_logits=1, casts=om.B200)
        tok = int(r.logits[0, -1].argmax())
        want = om.mtp_draft(p, cfg, r.hidden[:, -1], tok, draft_ids=sd["draft_ids"])
        got = eng.mtp_draft(r.hidden[:, -1], torch.tensor([tok]))
        assert len(got) == cfg.mtp_passes
        assert got == want, (trial, got, want)


@pytest.mark.parametrize("name", ["debug", "baseline"])
def test_reference_verifier_loop_runs_over_the_engine(name):
    """The reference's decoding loops (restated in oracle.decoding, pinned to the
    reference's own token sequences on CPU) driven over CirrusB200 with their
    default arguments -- speculative_greedy's max_draft 8 and MTP drafts from
    CirrusB200.mtp_draft, cache.clone() snapshots and re-runs on partial
    acceptance: the tokens are the greedy tokens, up to documented near-ties."""
    eng, _ = _engine(name, seed=6)
    vocab = eng.cfg.vocab_size
    g = torch.Generator().manual_seed(11)
    base = torch.randint(0, vocab, (9,), generator=g).tolist()
    prompt = base + torch.randint(0, vocab, (7,), generator=g).tolist() + base[:4]
    n = 24
    want, margins = _eager_greedy(eng, [prompt], n)
    assert od.greedy_loop(eng, prompt, n) == want[0]
    got, steps = od.speculative_loop(eng, prompt, n)
    assert len(got) == n
    _agree(got, want[0], margins[0], "reference speculative loop")
    assert steps <= n
