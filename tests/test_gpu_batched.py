"""Steps of many sequences at once (cb_forward with batch * T > 16 rows): the
tensor-core GEMM for every projection, block-wise SWA for decode and verify
steps of 32+ rows, the batched indexer / top-k and cross attention, against the
oracle run one sequence at a time on the same NVFP4 weights with the B200
storage casts.  Tolerances as for the single-sequence path: logits within 1e-2
relative / 2e-2 absolute."""

import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-2


def _close(a, b, what):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    torch.testing.assert_close(a, b, rtol=RTOL, atol=ATOL, msg=lambda m: f"{what}: max abs err {err}\n{m}")


@pytest.mark.parametrize("B,T", [(33, 1), (8, 5)])
def test_many_sequences_decode_and_verify_match_oracle(B, T):
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=8, norm_jitter=0.1)
    eng = CirrusB200(cfg, sd, max_ctx=256)
    p = om.quantized_params(sd)
    prompts = [synthetic.random_prompt(40, cfg.vocab_size, seed=100 + b) for b in range(B)]
    o = eng(torch.tensor(prompts), use_cache=True, n_logits=1)
    g = torch.Generator().manual_seed(1)
    steps = [torch.randint(0, cfg.vocab_size, (B, T), generator=g) for _ in range(2)]
    outs = []
    for ids in steps:
        o = eng(ids, cache=o.cache, n_logits=T)
        outs.append(o.logits)
    check = sorted({0, 1, B // 2, B - 1})
    for b in check:
        r = om.forward(p, cfg, torch.tensor([prompts[b]]), use_cache=True, n_logits=1, casts=om.B200)
        for s, ids in enumerate(steps):
            r = om.forward(p, cfg, ids[b:b + 1], cache=r.cache, n_logits=T, casts=om.B200)
            _close(outs[s][b:b + 1], r.logits, f"sequence {b} step {s}")
    assert eng.read_status(o.cache, T) == 0
