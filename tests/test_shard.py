"""Sequence sharding launcher (``cirrus_s_1a_b200.shard``) on CPU ranks.

Two ``gloo`` ranks (spawned processes, rendezvous on 127.0.0.1) each decode
their contiguous shard of a global batch with a stand-in decoder, coordinate
through the process group's store and report to rank 0, which adds up the
tokens.  Failures are made on the host: a rank that raises between steps, and
a rank that exits without reporting.
"""

import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from cirrus_s_1a_b200.shard import ShardCoordinator, run_shard, shard_bounds

N_SEQ, STEPS, VOCAB = 13, 6, 101


@pytest.mark.parametrize("n_seq,world", [(0, 1), (1, 1), (13, 2), (64, 8), (7, 8), (512, 3)])
def test_shard_bounds_cover_each_sequence_once(n_seq, world):
    seen = []
    sizes = []
    for r in range(world):
        a, b = shard_bounds(n_seq, world, r)
        assert a <= b
        if r > 0:
            assert a == shard_bounds(n_seq, world, r - 1)[1]  # contiguous
        seen += list(range(a, b))
        sizes.append(b - a)
    assert seen == list(range(n_seq))
    assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_requests():
    for args in ((4, 0, 0), (4, 2, 2), (4, 2, -1), (-1, 2, 0)):
        with pytest.raises(ValueError):
            shard_bounds(*args)


def _decode(start, stop, between_steps, fail_at=None, exit_at=None):
    """Stand-in decoder: sequence s emits one token per step (next = sum of the
    last three mod VOCAB); returns (tokens, seconds)."""
    seqs = {s: [s % VOCAB, (3 * s) % VOCAB, (7 * s + 1) % VOCAB] for s in range(start, stop)}
    tokens = 0
    for step in range(STEPS):
        if fail_at is not None and step == fail_at:
            raise RuntimeError(f"injected failure at step {step}")
        if exit_at is not None and step == exit_at:
            os._exit(0)  # leaves without reporting, between steps
        for s, t in seqs.items():
            t.append(sum(t[-3:]) % VOCAB)
            tokens += 1
        if not between_steps(step + 1):
            break
    return tokens, 0.001 * (step + 1)


def _rank_main(rank, world, port, out_dir, mode):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    store = dist.distributed_c10d._get_default_store()
    coord = ShardCoordinator(store, rank, world, timeout_s=8.0)
    result = {"rank": rank}
    try:
        if rank == 1 and mode == "raise":
            work = lambda a, b, hook: _decode(a, b, hook, fail_at=2)  # noqa: E731
        elif rank == 1 and mode == "exit":
            work = lambda a, b, hook: _decode(a, b, hook, exit_at=2)  # noqa: E731
        else:
            work = _decode
        if rank == 0 and mode == "raise":
            # rank 0 runs slower so that the peer's failure is published before it finishes
            def work(a, b, hook):
                import time

                def slow(step):
                    time.sleep(0.3)
                    return hook(step)

                return _decode(a, b, slow)
        try:
            start, stop, tokens, _ = run_shard(coord, N_SEQ, work, stop_on_peer_failure=(mode == "raise"))
            result.update(start=start, stop=stop, tokens=tokens)
        except RuntimeError as exc:
            result["error"] = str(exc)
        if mode == "ok":
            # the data path has no collective; the job may still use the group for its own plumbing
            t = torch.tensor([float(result.get("tokens", 0))])
            dist.all_reduce(t)
            result["allreduce_tokens"] = float(t)
        if rank == 0:
            g = coord.gather()
            result["gather"] = {"tokens": g.tokens, "failed": g.failed, "lost": g.lost, "ok": g.ok,
                                "ranks": {str(k): v["status"] for k, v in g.ranks.items()}}
    finally:
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(result, f)
        if mode != "exit":
            dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(tmp_path, mode):
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, join=True,
                       start_method="spawn")
    out = {}
    for r in range(2):
        p = tmp_path / f"rank{r}.json"
        if p.exists():
            out[r] = json.loads(p.read_text())
    return out


def test_two_ranks_decode_their_shards_and_rank0_sums_tokens(tmp_path):
    out = _spawn(tmp_path, "ok")
    a0, b0 = shard_bounds(N_SEQ, 2, 0)
    a1, b1 = shard_bounds(N_SEQ, 2, 1)
    assert (out[0]["start"], out[0]["stop"], out[1]["start"], out[1]["stop"]) == (a0, b0, a1, b1)
    assert out[0]["tokens"] == (b0 - a0) * STEPS and out[1]["tokens"] == (b1 - a1) * STEPS
    g = out[0]["gather"]
    assert g["ok"] and g["tokens"] == N_SEQ * STEPS
    assert out[0]["allreduce_tokens"] == N_SEQ * STEPS


def test_failed_rank_is_reported_and_peer_stops_between_steps(tmp_path):
    out = _spawn(tmp_path, "raise")
    assert "injected failure" in out[1]["error"]
    g = out[0]["gather"]
    assert g["failed"] == [1] and g["lost"] == [] and not g["ok"]
    assert g["ranks"]["1"].startswith("failed: RuntimeError: injected failure")
    # rank 0 saw the failure at a step boundary and stopped early with whole steps only
    a0, b0 = shard_bounds(N_SEQ, 2, 0)
    assert 0 < out[0]["tokens"] < (b0 - a0) * STEPS and out[0]["tokens"] % (b0 - a0) == 0


def test_rank_that_exits_without_reporting_is_lost(tmp_path):
    try:
        out = _spawn(tmp_path, "exit")
    except mp.ProcessExitedException:
        pytest.fail("a rank exiting with status 0 must not fail the launcher")
    assert 1 not in out  # rank 1 left before writing anything
    g = out[0]["gather"]
    assert g["lost"] == [1] and g["failed"] == [] and g["tokens"] == (shard_bounds(N_SEQ, 2, 0)[1]) * STEPS
