"""Failure detection of the persistent kernel, and per-device launch state.

The persistent decode kernel separates its phases with grid barriers whose
waits are bounded (``%globaltimer``).  The host can shorten the limit and, for
tests, make one barrier incomplete (``cb_set_wait_limit``: CTA 0 skips one
arrival).  Every wait on that barrier then runs out: the kernel writes
CB_ERR_TIMEOUT to the status word and every CTA returns, so the launch ends
promptly, the context stays usable and the cache position is not advanced.
Nothing here faults or traps the GPU: the failure is a counter that the host
told one CTA not to increment.

The last test drives two GPUs from one process (skipped with fewer than two):
kernel attributes are set per device, so both devices run the persistent
kernel and agree bit for bit.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

CB_ERR_TIMEOUT = 8


def _engine(device="cuda:0", max_ctx=256):
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=2, norm_jitter=0.1)
    return CirrusB200(cfg, sd, device=device, max_ctx=max_ctx)


@pytest.mark.parametrize("barrier", [1, 7, 40])
def test_stalled_barrier_times_out_and_returns(barrier):
    eng = _engine()
    prompt = torch.randint(0, eng.cfg.vocab_size, (1, 24), generator=torch.Generator().manual_seed(1))
    o = eng(prompt, use_cache=True, n_logits=1)
    cache = o.cache
    tok = int(o.logits[0, -1].argmax())
    snap = cache.clone()
    ref = eng(torch.tensor([[tok]]), cache=cache.clone(), n_logits=1).logits.clone()
    assert eng.read_status(cache) == 0

    pos_before = cache.pos_dev.clone()
    eng.set_wait_limit(cache, 1_000_000, stall_barrier=barrier)  # 1 ms, one barrier left incomplete
    ids = torch.tensor([[tok]], device=eng.device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.launch(cache, ids, 1, 1, None, None, None)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert eng.read_status(cache) == CB_ERR_TIMEOUT
    assert elapsed < 0.1, elapsed  # every CTA gave up after about 1 ms
    assert torch.equal(cache.pos_dev, pos_before)  # the step was not committed

    # the context is still usable: clear the hook and the status, rerun the step
    # from the snapshot (the aborted launch may have advanced recurrent state)
    eng.set_wait_limit(cache, 0, stall_barrier=0)
    eng.clear_status(cache)
    out = eng(torch.tensor([[tok]]), cache=snap, n_logits=1)
    assert eng.read_status(snap) == 0
    assert torch.equal(out.logits, ref)


def test_default_limit_is_restored_and_long_steps_pass():
    eng = _engine(max_ctx=4096)
    cache = eng.new_cache(1)
    from cirrus_s_1a_b200 import synthetic

    synthetic.fill_cache(cache, 4000, seed=3)
    eng.set_wait_limit(cache, 5_000_000)  # 5 ms: far above a step's longest phase
    o = eng(torch.tensor([[9]]), cache=cache, n_logits=1)
    assert eng.read_status(cache) == 0
    assert torch.isfinite(o.logits).all()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_devices_in_one_process():
    outs = []
    for dev in ("cuda:0", "cuda:1"):
        eng = _engine(device=dev)
        prompt = torch.randint(0, eng.cfg.vocab_size, (1, 16), generator=torch.Generator().manual_seed(4))
        with torch.cuda.device(dev):
            o = eng(prompt, use_cache=True, n_logits=1)
            o = eng(torch.tensor([[int(o.logits[0, -1].argmax())]]), cache=o.cache, n_logits=1)
            assert eng.read_status(o.cache) == 0
        outs.append(o.logits.cpu())
    assert torch.equal(outs[0], outs[1])
