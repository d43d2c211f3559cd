"""The one-launch NVFP4 weight stream (cb_weight_stream_nvfp4): every matrix of a
list of the model's projection shapes against a float64 matmul of the oracle's
dequantised weights and against the CUDA-core GEMV, for 1..8 token rows; the
plan's argument checks."""

import ctypes as C

import pytest
import torch

from oracle import nvfp4

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SHAPES = [(768, 768), (4096, 768), (768, 2048), (3104, 768), (1296, 768), (32000, 768), (16, 768)]


def _st():
    return torch.cuda.current_stream().cuda_stream


def test_weight_stream_matches_f64_and_gemv():
    from cirrus_s_1a_b200 import _lib
    from cirrus_s_1a_b200.engine import PackedMatrix

    L = _lib.lib()
    g = torch.Generator().manual_seed(3)
    mats, deqs = [], []
    for n, k in SHAPES:
        w = torch.randn(n, k, generator=g) * 0.02
        mats.append(PackedMatrix([w], torch.device(DEV)))
        deqs.append(torch.from_numpy(nvfp4.fake_quant(w.numpy())).double())
    arr = (_lib.CbMatrix * len(mats))(*[m.struct() for m in mats])
    plan = torch.empty(L.cb_stream_plan_bytes(len(mats)), dtype=torch.uint8, device=DEV)
    rows = C.c_int64(0)
    assert L.cb_stream_plan(arr, len(mats), plan.data_ptr(), plan.numel(), C.byref(rows), _st()) == 0
    assert rows.value == sum(m.rows for m in mats)
    tiles = rows.value // 16
    kmax = 2048
    for M in (1, 2, 4, 5, 8):
        x = torch.randn(M, kmax, generator=g)
        xd = x.to(DEV)
        y = torch.full((M, rows.value), float("nan"), device=DEV)
        status = torch.zeros(1, dtype=torch.int32, device=DEV)
        rc = L.cb_weight_stream_nvfp4(plan.data_ptr(), len(mats), tiles, xd.data_ptr(), kmax, kmax, M, y.data_ptr(),
                                      rows.value, status.data_ptr(), _st())
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        off = 0
        for (n, k), pm, deq in zip(SHAPES, mats, deqs):
            ref = x[:, :k].double() @ deq.T
            got = y[:, off:off + n].double().cpu()
            err = ((got - ref).abs().max() / ref.abs().max()).item()
            assert err < 2e-6, ((n, k), M, err)
            ms = pm.struct()
            yg = torch.empty(M, pm.rows, device=DEV)
            assert L.cb_gemv_nvfp4(C.byref(ms), xd.data_ptr(), kmax, M, yg.data_ptr(), pm.rows, n, _st()) == 0
            torch.cuda.synchronize()
            assert ((yg[:, :n] - y[:, off:off + n]).abs().max() / yg[:, :n].abs().max()).item() < 2e-6
            off += pm.rows


def test_weight_stream_rejects_bad_plans():
    from cirrus_s_1a_b200 import _lib
    from cirrus_s_1a_b200.engine import PackedMatrix

    L = _lib.lib()
    good = PackedMatrix([torch.randn(32, 768) * 0.02], torch.device(DEV))
    bad_k = PackedMatrix([torch.randn(32, 96) * 0.02], torch.device(DEV))  # K not a multiple of 256
    plan = torch.empty(4096, dtype=torch.uint8, device=DEV)
    rows = C.c_int64(0)
    arr = (_lib.CbMatrix * 2)(good.struct(), bad_k.struct())
    assert L.cb_stream_plan(arr, 2, plan.data_ptr(), plan.numel(), C.byref(rows), _st()) == 2
    assert L.cb_stream_plan(arr, 0, plan.data_ptr(), plan.numel(), C.byref(rows), _st()) == 1
    assert L.cb_stream_plan(arr, 1, plan.data_ptr(), 1, C.byref(rows), _st()) == 1
    x = torch.zeros(9, 768, device=DEV)
    y = torch.zeros(9, 32, device=DEV)
    assert L.cb_weight_stream_nvfp4(plan.data_ptr(), 1, 2, x.data_ptr(), 768, 768, 9, y.data_ptr(), 32, None,
                                    _st()) == 1  # more than 8 rows
