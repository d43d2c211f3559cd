"""Chunked Gated DeltaNet prefill (cb_gdn_chunk_prefill) against the oracle's
exact token-by-token recurrence (gated_delta_rule, layers.py:108-129) in
float64, on the C2 input distributions: state N(0, 0.1), q and k N(0, 1)
L2-normalised, v N(0, 1), alpha = sigmoid(N(3, 1)) (g = log alpha),
beta = sigmoid(N(0, 1)); lengths that end inside a chunk, several sequences
and heads, and a start state carried in."""

import ctypes as C

import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def L():
    from cirrus_s_1a_b200 import _lib

    return _lib.lib()


def _inputs(B, T, H, seed, D=64):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g, dtype=torch.float64), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g, dtype=torch.float64), dim=-1)
    v = torch.randn(B, T, H, D, generator=g, dtype=torch.float64)
    alpha = torch.sigmoid(torch.randn(B, T, H, generator=g, dtype=torch.float64) + 3.0)
    beta = torch.sigmoid(torch.randn(B, T, H, generator=g, dtype=torch.float64))
    S0 = torch.randn(B, H, D, D, generator=g, dtype=torch.float64) * 0.1
    # the kernel reads fp32: compare against the recurrence on the same fp32 values
    return [t.float().double() for t in (q, k, v, alpha.log(), beta, S0)]


def _run(L, q, k, v, gl, beta, S0, scale):
    B, T, H, D = k.shape
    dq, dk, dv, dg, db = (t.float().contiguous().to(DEV) for t in (q, k, v, gl, beta))
    S = S0.float().contiguous().to(DEV)
    out = torch.full((B, T, H, D), float("nan"), device=DEV)
    rc = L.cb_gdn_chunk_prefill(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(), B, T, H, D,
                                D, C.c_float(scale), S.data_ptr(), out.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return out.double().cpu(), S.double().cpu()


@pytest.mark.parametrize("B,T,H", [(1, 1, 1), (1, 63, 2), (2, 64, 3), (2, 130, 3), (1, 300, 12)])
def test_gdn_chunk_prefill_matches_recurrence(L, B, T, H):
    q, k, v, gl, beta, S0 = _inputs(B, T, H, seed=B * 1000 + T * 10 + H)
    scale = 64 ** -0.5
    o_ref, S_ref = om.gated_delta_rule(q, k, v, gl, beta, scale, state=S0)
    o, S = _run(L, q, k, v, gl, beta, S0, scale)
    eo = ((o - o_ref).abs().max() / o_ref.abs().max()).item()
    es = ((S - S_ref).abs().max() / S_ref.abs().max()).item()
    assert eo < 2e-5 and es < 2e-5, (B, T, H, eo, es)


def test_gdn_chunk_prefill_4096_tokens(L):
    """C2 prefill: 4096 tokens in 64-token chunks, 12 heads."""
    q, k, v, gl, beta, S0 = _inputs(1, 4096, 12, seed=42)
    scale = 64 ** -0.5
    o_ref, S_ref = om.gated_delta_rule(q, k, v, gl, beta, scale, state=S0)
    o, S = _run(L, q, k, v, gl, beta, S0, scale)
    eo = ((o - o_ref).abs().max() / o_ref.abs().max()).item()
    es = ((S - S_ref).abs().max() / S_ref.abs().max()).item()
    assert eo < 1e-4 and es < 1e-4, (eo, es)


def test_gdn_chunk_prefill_continues_a_split_sequence(L):
    """Two calls over [0, 100) and [100, 230) equal one call over [0, 230)."""
    q, k, v, gl, beta, S0 = _inputs(1, 230, 4, seed=9)
    scale = 64 ** -0.5
    o_all, S_all = _run(L, q, k, v, gl, beta, S0, scale)
    o1, S1 = _run(L, q[:, :100], k[:, :100], v[:, :100], gl[:, :100], beta[:, :100], S0, scale)
    o2, S2 = _run(L, q[:, 100:], k[:, 100:], v[:, 100:], gl[:, 100:], beta[:, 100:], S1, scale)
    o_cat = torch.cat([o1, o2], dim=1)
    assert ((o_cat - o_all).abs().max() / o_all.abs().max()).item() < 2e-5
    assert ((S2 - S_all).abs().max() / S_all.abs().max()).item() < 2e-5
