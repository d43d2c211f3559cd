"""Tensor-core verify GEMM (cb_verify_gemm_nvfp4, tcgen05.mma kind::f16 into
tensor memory) against a float64 matmul of bf16 inputs and the oracle's
dequantised NVFP4 weights, for token widths 1..16 and the model's (N, K)
shapes; plus the rows_out bound, the row-width limit and the status word."""

import ctypes as C

import pytest
import torch

from oracle import nvfp4

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def L():
    from cirrus_s_1a_b200 import _lib

    return _lib.lib()


def _st():
    return torch.cuda.current_stream().cuda_stream


def _bf16_bits(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).view(torch.int16).contiguous()


@pytest.mark.parametrize("shape", [(768, 768), (4096, 768), (768, 2048), (2304, 768), (24, 768), (32000, 768),
                                   (48, 64), (144, 128)])
def test_verify_gemm_vs_f64(L, shape):
    from cirrus_s_1a_b200.engine import PackedMatrix

    n, k = shape
    g = torch.Generator().manual_seed(7 * n + k)
    w = torch.randn(n, k, generator=g) * 0.02
    pm = PackedMatrix([w], torch.device(DEV))
    deq = torch.from_numpy(nvfp4.fake_quant(w.numpy())).double()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    for M in (1, 2, 4, 5, 8, 16):
        x = torch.randn(M, k, generator=g)
        xb = _bf16_bits(x).to(DEV)
        y = torch.full((M, pm.rows), float("nan"), device=DEV)
        ms = pm.struct()
        rc = L.cb_verify_gemm_nvfp4(C.byref(ms), xb.data_ptr(), k, M, y.data_ptr(), pm.rows, n, status.data_ptr(),
                                    _st())
        assert rc == 0, rc
        torch.cuda.synchronize()
        ref = x.to(torch.bfloat16).double() @ deq.T
        got = y[:, :n].double().cpu()
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        assert err < 1e-5, (shape, M, err)     # exact products, fp32 accumulation
        assert torch.isnan(y[:, n:]).all()     # rows_out bounds the writes
    assert int(status.item()) == 0


def test_verify_gemm_matches_cuda_core_gemv(L):
    """The tensor-core path and the CUDA-core GEMV agree on the same bf16 inputs."""
    from cirrus_s_1a_b200.engine import PackedMatrix

    n, k = 1024, 768
    g = torch.Generator().manual_seed(11)
    pm = PackedMatrix([torch.randn(n, k, generator=g) * 0.02], torch.device(DEV))
    x = torch.randn(8, k, generator=g).to(torch.bfloat16)
    y1 = torch.empty(8, n, device=DEV)
    y2 = torch.empty(8, n, device=DEV)
    ms = pm.struct()
    assert L.cb_verify_gemm_nvfp4(C.byref(ms), x.view(torch.int16).to(DEV).data_ptr(), k, 8, y1.data_ptr(), n, n,
                                  None, _st()) == 0
    assert L.cb_gemv_nvfp4(C.byref(ms), x.float().to(DEV).data_ptr(), k, 8, y2.data_ptr(), n, n, _st()) == 0
    torch.cuda.synchronize()
    err = ((y1 - y2).abs().max() / y2.abs().max()).item()
    assert err < 1e-5, err


def test_verify_gemm_rejects_bad_arguments(L):
    from cirrus_s_1a_b200.engine import PackedMatrix

    pm = PackedMatrix([torch.randn(32, 64) * 0.02], torch.device(DEV))
    ms = pm.struct()
    x = torch.zeros(17, 64, dtype=torch.int16, device=DEV)
    y = torch.zeros(17, 32, device=DEV)
    assert L.cb_verify_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 17, y.data_ptr(), 32, 32, None, _st()) == 1
    assert L.cb_verify_gemm_nvfp4(C.byref(ms), x.data_ptr(), 64, 0, y.data_ptr(), 32, 32, None, _st()) == 1
    pm32 = PackedMatrix([torch.randn(32, 32) * 0.02], torch.device(DEV))
    ms32 = pm32.struct()
    assert L.cb_verify_gemm_nvfp4(C.byref(ms32), x.data_ptr(), 64, 2, y.data_ptr(), 32, 32, None, _st()) == 2
