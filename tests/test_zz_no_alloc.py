"""The allocation-free indexer top-k entry point (cb_indexer_topk_noalloc).

Some callers cannot allocate device memory when they call this library -- a
serving process whose memory planner hands out every device byte at start-up,
or a binding in another language that only receives the input and output
buffers from its host runtime.  For them the top-k score scratch lives in a
static array inside the library.  This test calls the new entry point through
the C ABI twice in a row, with different inputs each time (the array keeps the
previous call's scores), and checks that it selects exactly the keys the
existing entry point selects with a caller-provided scratch buffer.  It also
checks that a request larger than the static array is refused.

This file is named so that pytest collects it last."""

import numpy as np
import pytest
import torch

from oracle import nvfp4

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _case(seed, rows, Hi, Di, max_ctx, k):
    rng = np.random.default_rng(seed)
    ik = nvfp4.e4m3_encode(rng.normal(0, 1, (2, max_ctx, Di)).astype(np.float32))
    ik[:, 200:900] = ik[:, 100:101]  # exact ties
    ik[:, 3000:5000:3] = 0
    ld = Hi * Di + Hi
    q = rng.normal(0, 1, (rows, ld)).astype(np.float32)
    qpos = rng.integers(0, max_ctx, rows).astype(np.int32)
    qpos[0], qpos[1] = k - 1, max_ctx - 1  # every key kept / the longest row
    seq = rng.integers(0, 2, rows).astype(np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    return t(q), t(ik), t(seq), t(qpos), ld


def _run(L, noalloc, q, ik, seq, qpos, ld, Hi, Di, max_ctx, k, rows):
    st = torch.cuda.current_stream().cuda_stream
    sel = torch.full((rows, k + 1), -7, dtype=torch.int32, device=DEV)
    cnt = torch.full((rows,), -7, dtype=torch.int32, device=DEV)
    args = (q.data_ptr(), q.data_ptr() + 4 * Hi * Di, ld, ik.data_ptr(), max_ctx, Hi, Di, seq.data_ptr(),
            qpos.data_ptr(), rows, k)
    if noalloc:
        rc = L.cb_indexer_topk_noalloc(*args, sel.data_ptr(), cnt.data_ptr(), st)
    else:
        scores = torch.empty(rows, max_ctx, dtype=torch.float32, device=DEV)
        rc = L.cb_indexer_topk(*args, scores.data_ptr(), sel.data_ptr(), cnt.data_ptr(), st)
    assert rc == 0
    torch.cuda.synchronize()
    return sel.cpu(), cnt.cpu()


def test_noalloc_topk_matches_allocating_entry_point():
    from cirrus_s_1a_b200 import _lib

    L = _lib.lib()
    Hi, Di, k = 4, 64, 512
    # calls in a row; the last one fills the static scratch exactly (32 * 32768 = 2^20 scores)
    for seed, (rows, max_ctx) in ((1, (6, 32768)), (2, (9, 20000)), (3, (32, 32768))):
        assert rows * max_ctx <= _lib.CB_NOALLOC_MAX_SCORES
        case = _case(seed, rows, Hi, Di, max_ctx, k)
        sel_a, cnt_a = _run(L, False, *case, Hi, Di, max_ctx, k, rows)
        sel_b, cnt_b = _run(L, True, *case, Hi, Di, max_ctx, k, rows)
        assert torch.equal(cnt_a, cnt_b)
        for r in range(rows):
            n = int(cnt_a[r])
            assert torch.equal(sel_a[r, :n], sel_b[r, :n]), (seed, r)


def test_noalloc_topk_refuses_requests_beyond_its_scratch():
    from cirrus_s_1a_b200 import _lib

    L = _lib.lib()
    rows, max_ctx = 33, 32768  # 33 * 32768 > CB_NOALLOC_MAX_SCORES
    assert rows * max_ctx > _lib.CB_NOALLOC_MAX_SCORES
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    p = dummy.data_ptr()
    rc = L.cb_indexer_topk_noalloc(p, p, 260, p, max_ctx, 4, 64, p, p, rows, 512, p, p,
                                   torch.cuda.current_stream().cuda_stream)
    assert rc == 7
    assert L.cb_status_string(rc).startswith(b"rows * max_ctx exceeds")
