"""Many-token tensor-core GEMM (cb_gemm_nvfp4: tcgen05.mma kind::f16 into
tensor memory, f16 weights exact, f16 head + tail activations prepared by a
first launch into caller scratch) against a
float64 matmul of the float32 inputs and the oracle's dequantised NVFP4
weights: the model's (N, K) shapes, token counts from 1 to 320 (several token
tiles, ragged last tile), the RMSNorm prologue, the residual add and the fused
SwiGLU epilogue; the rows_out bound, argument checks and the status word."""

import ctypes as C

import pytest
import torch

from oracle import nvfp4

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TOL = 2e-5  # relative to the largest output: exact weights, ~22-bit inputs, fp32 accumulation


@pytest.fixture(scope="module")
def L():
    from cirrus_s_1a_b200 import _lib

    return _lib.lib()


def _st():
    return torch.cuda.current_stream().cuda_stream


def _scratch(L, k, m):
    n = L.cb_gemm_scratch_bytes(k, m)
    buf = torch.empty(max(n, 16), dtype=torch.uint8, device=DEV)
    return buf, buf.data_ptr(), n


def _packed(n, k, seed):
    from cirrus_s_1a_b200.engine import PackedMatrix

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    pm = PackedMatrix([w], torch.device(DEV))
    deq = torch.from_numpy(nvfp4.fake_quant(w.numpy())).double()
    return pm, deq, g


def _rms(x, nw, eps):
    x = x.double()
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * nw.double()


@pytest.mark.parametrize("shape", [(768, 768), (2304, 768), (768, 2048), (24, 768), (32000, 768), (48, 64),
                                   (144, 128), (1024, 4096)])
def test_gemm_store_vs_f64(L, shape):
    from cirrus_s_1a_b200 import _lib

    n, k = shape
    pm, deq, g = _packed(n, k, 7 * n + k)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ms = pm.struct()
    for M in (1, 5, 32, 33, 64, 100) if n < 32000 else (1, 64):
        x = torch.randn(M, k, generator=g)
        xd = x.to(DEV)
        y = torch.full((M, pm.rows), float("nan"), device=DEV)
        buf, sp, sb = _scratch(L, k, M)
        rc = L.cb_gemm_nvfp4(C.byref(ms), xd.data_ptr(), k, M, _lib.CB_GEMM_PRE_NONE, None, 0.0,
                             y.data_ptr(), pm.rows, n, _lib.CB_GEMM_EPI_STORE, sp, sb, status.data_ptr(), _st())
        assert rc == 0, rc
        torch.cuda.synchronize()
        ref = x.double() @ deq.T
        got = y[:, :n].double().cpu()
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        assert err < TOL, (shape, M, err)
        assert torch.isnan(y[:, n:]).all()  # rows_out bounds the writes
    assert int(status.item()) == 0


@pytest.mark.parametrize("M", [3, 64, 320])
def test_gemm_rmsnorm_add(L, M):
    from cirrus_s_1a_b200 import _lib

    n, k, eps = 768, 768, 1e-6
    pm, deq, g = _packed(n, k, 11 + M)
    x = torch.randn(M, k, generator=g) * 3.0
    nw = 1.0 + 0.1 * torch.randn(k, generator=g)
    y0 = torch.randn(M, n, generator=g)
    y = y0.clone().to(DEV)
    xd, nwd = x.to(DEV), nw.to(DEV)  # held in names: a temporary's memory could be reused before the launch
    ms = pm.struct()
    buf, sp, sb = _scratch(L, k, M)
    rc = L.cb_gemm_nvfp4(C.byref(ms), xd.data_ptr(), k, M, _lib.CB_GEMM_PRE_RMSNORM, nwd.data_ptr(),
                         eps, y.data_ptr(), n, n, _lib.CB_GEMM_EPI_ADD, sp, sb, None, _st())
    assert rc == 0
    torch.cuda.synchronize()
    ref = y0.double() + _rms(x, nw, eps) @ deq.T
    err = ((y.double().cpu() - ref).abs().max() / ref.abs().max()).item()
    assert err < TOL, err


@pytest.mark.parametrize("M", [1, 40, 130])
def test_gemm_swiglu(L, M):
    """gate_up [2F, K] with the SwiGLU epilogue = silu(x W_g^T) * (x W_u^T) (layers.py:52-54)."""
    from cirrus_s_1a_b200 import _lib

    F, k, eps = 2048, 768, 1e-6
    pm, deq, g = _packed(2 * F, k, 5 + M)
    x = torch.randn(M, k, generator=g)
    nw = 1.0 + 0.1 * torch.randn(k, generator=g)
    y = torch.full((M, F + 16), float("nan"), device=DEV)
    xd, nwd = x.to(DEV), nw.to(DEV)
    ms = pm.struct()
    buf, sp, sb = _scratch(L, k, M)
    rc = L.cb_gemm_nvfp4(C.byref(ms), xd.data_ptr(), k, M, _lib.CB_GEMM_PRE_RMSNORM, nwd.data_ptr(),
                         eps, y.data_ptr(), F + 16, F, _lib.CB_GEMM_EPI_SWIGLU, sp, sb, None, _st())
    assert rc == 0
    torch.cuda.synchronize()
    h = _rms(x, nw, eps) @ deq.T
    ref = torch.nn.functional.silu(h[:, :F]) * h[:, F:]
    got = y[:, :F].double().cpu()
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    assert err < 5 * TOL, err
    assert torch.isnan(y[:, F:]).all()


def test_gemm_matches_gemv(L):
    """Same products as the CUDA-core GEMV (both exact in the weights, fp32 accumulation)."""
    from cirrus_s_1a_b200 import _lib

    n, k, M = 2304, 768, 16
    pm, _, g = _packed(n, k, 99)
    x = torch.randn(M, k, generator=g).to(DEV)
    y1 = torch.empty(M, n, device=DEV)
    y2 = torch.empty(M, n, device=DEV)
    ms = pm.struct()
    buf, sp, sb = _scratch(L, k, M)
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), k, M, 0, None, 0.0, y1.data_ptr(), n, n, 0, sp, sb, None,
                           _st()) == 0
    assert L.cb_gemv_nvfp4(C.byref(ms), x.data_ptr(), k, M, y2.data_ptr(), n, n, _st()) == 0
    torch.cuda.synchronize()
    assert ((y1 - y2).abs().max() / y2.abs().max()).item() < TOL


def test_gemm_rejects_bad_arguments(L):
    from cirrus_s_1a_b200 import _lib

    pm, _, _ = _packed(64, 64, 1)
    ms = pm.struct()
    x = torch.zeros(4, 64, device=DEV)
    y = torch.zeros(4, 64, device=DEV)
    buf, sp, sb = _scratch(L, 64, 4)
    E_ARG, E_SHAPE, E_WS = 1, 2, 4
    # unaligned x, ldx not a multiple of 4, rows_out above the rows, zero tokens, bad modes, RMSNorm without weights
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr() + 4, 64, 2, 0, None, 0.0, y.data_ptr(), 64, 64, 0, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 66, 2, 0, None, 0.0, y.data_ptr(), 64, 64, 0, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 80, 80, 0, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 0, 0, None, 0.0, y.data_ptr(), 64, 64, 0, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 5, None, 0.0, y.data_ptr(), 64, 64, 0, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 64, 64, 7, sp, sb, None,
                           _st()) == E_ARG
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, _lib.CB_GEMM_PRE_RMSNORM, None, 0.0, y.data_ptr(), 64,
                           64, 0, sp, sb, None, _st()) == E_ARG
    # SwiGLU needs F = rows / 2 a multiple of 64
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 64, 32,
                           _lib.CB_GEMM_EPI_SWIGLU, sp, sb, None, _st()) == E_SHAPE
    # scratch smaller than cb_gemm_scratch_bytes, or none
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 64, 64, 0, sp, sb - 16, None,
                           _st()) == E_WS
    assert L.cb_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 64, 64, 0, None, sb, None,
                           _st()) == E_ARG
    # K must be a multiple of 64
    pm2, _, _ = _packed(32, 48, 2)
    ms2 = pm2.struct()
    assert L.cb_gemm_nvfp4(C.byref(ms2), x.data_ptr(), 64, 2, 0, None, 0.0, y.data_ptr(), 64, 32, 0, sp, sb, None,
                           _st()) == E_SHAPE
