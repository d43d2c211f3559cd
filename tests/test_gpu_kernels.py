"""Kernel-level parity on the B200 through the C ABI: NVFP4 quantiser and tile
packer (bit-exact vs the numpy oracle), GEMV (vs a float64 matmul of the
oracle's dequantised weights), embedding gather (exact), argmax, indexer
scores and top-k selection (bit-exact vs the oracle), GDN step (vs the
oracle's recurrence)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import indexer as oidx
from oracle import model as om
from oracle import nvfp4

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def L():
    from cirrus_s_1a_b200 import _lib

    return _lib.lib()


def _st():
    return torch.cuda.current_stream().cuda_stream


def _edge_weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    w[0, :16] = 0.0                                   # zero block -> zero scale
    w[1, :16] = torch.linspace(-1, 1, 16)
    w[2, :16] = -0.0
    w[3, :] = torch.randn(k, generator=g) * 300.0     # large scales (saturation region)
    w[4, :16] = torch.tensor([6, 5, 3.5, 2.5, 1.75, 1.25, .75, .25, -6, -5, -3.5, -2.5, -1.75, -1.25, -.75, -.25]) / 100
    return w


def test_quantize_bitexact_vs_oracle(L):
    for (n, k, seed) in ((64, 768, 0), (40, 2048, 1), (16, 64, 2)):
        w = _edge_weights(n, k, seed)
        wd = w.to(DEV).contiguous()
        codes = torch.empty(n, k // 2, dtype=torch.uint8, device=DEV)
        scales = torch.empty(n, k // 16, dtype=torch.uint8, device=DEV)
        assert L.cb_nvfp4_quantize(wd.data_ptr(), n, k, 1.0, codes.data_ptr(), scales.data_ptr(), _st()) == 0
        oc, os_ = nvfp4.quantize(w.numpy())
        torch.cuda.synchronize()
        assert np.array_equal(scales.cpu().numpy(), os_)
        assert np.array_equal(codes.cpu().numpy(), nvfp4.pack_standard(oc))
    # a non-unit tensor scale
    w = _edge_weights(32, 256, 3)
    wd = w.to(DEV).contiguous()
    codes = torch.empty(32, 128, dtype=torch.uint8, device=DEV)
    scales = torch.empty(32, 16, dtype=torch.uint8, device=DEV)
    assert L.cb_nvfp4_quantize(wd.data_ptr(), 32, 256, 0.37, codes.data_ptr(), scales.data_ptr(), _st()) == 0
    oc, os_ = nvfp4.quantize(w.numpy(), 0.37)
    assert np.array_equal(scales.cpu().numpy(), os_)
    assert np.array_equal(codes.cpu().numpy(), nvfp4.pack_standard(oc))


def _tiles_np(codes_std, scales, n, k):
    nt = (n + 15) // 16
    out = []
    for t in range(nt):
        c = np.zeros((16, k // 2), np.uint8)
        s = np.zeros((16, k // 16), np.uint8)
        r = min(16, n - 16 * t)
        c[:r] = codes_std[16 * t:16 * t + r]
        s[:r] = scales[16 * t:16 * t + r]
        out.append(np.concatenate([c.ravel(), s.ravel()]))
    return np.concatenate(out)


def test_pack_tiles_layout(L):
    n, k = 37, 512
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    scales = rng.integers(0, 127, (n, k // 16), dtype=np.uint8)
    cd, sd = torch.from_numpy(codes).to(DEV), torch.from_numpy(scales).to(DEV)
    nt = (n + 15) // 16
    tiles = torch.full((nt * 16 * (k // 2 + k // 16),), 0xAB, dtype=torch.uint8, device=DEV)
    assert L.cb_nvfp4_pack_tiles(cd.data_ptr(), sd.data_ptr(), n, k, tiles.data_ptr(), _st()) == 0
    assert np.array_equal(tiles.cpu().numpy(), _tiles_np(codes, scales, n, k))


def _packed(weights):
    from cirrus_s_1a_b200.engine import PackedMatrix

    return PackedMatrix(weights, torch.device(DEV))


@pytest.mark.parametrize("shape", [(768, 768), (4096, 768), (768, 2048), (24, 768), (32000, 768), (48, 64)])
def test_gemv_vs_oracle_dequant(L, shape):
    n, k = shape
    g = torch.Generator().manual_seed(n + k)
    w = torch.randn(n, k, generator=g) * 0.02
    pm = _packed([w])
    deq = torch.from_numpy(nvfp4.fake_quant(w.numpy())).double()
    for M in (1, 2, 3, 5, 8, 11):
        x = torch.randn(M, k, generator=g)
        y = torch.full((M, pm.rows), float("nan"), device=DEV)
        ms = pm.struct()
        assert L.cb_gemv_nvfp4(C.byref(ms), x.to(DEV).data_ptr(), k, M, y.data_ptr(), pm.rows, n, _st()) == 0
        ref = x.double() @ deq.T
        got = y[:, :n].double().cpu()
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        assert err < 2e-6, (shape, M, err)
        assert torch.isnan(y[:, n:]).all()  # rows_out bounds the writes


def test_embed_gathers_exact_dequant_rows(L):
    from cirrus_s_1a_b200._lib import I32

    n, k = 300, 768
    w = torch.randn(n, k, generator=torch.Generator().manual_seed(5)) * 0.02
    pm = _packed([w])
    ids = torch.tensor([0, 299, 17, 17, 150], dtype=torch.int64, device=DEV)
    h = torch.empty(5, k, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ms = pm.struct()
    assert L.cb_embed(C.byref(ms), ids.data_ptr(), 5, h.data_ptr(), status.data_ptr(), _st()) == 0
    deq = nvfp4.fake_quant(w.numpy())
    assert np.array_equal(h.cpu().numpy(), deq[ids.cpu().numpy()])
    assert int(status.item()) == 0
    bad = torch.tensor([5, 100000], dtype=torch.int64, device=DEV)
    assert L.cb_embed(C.byref(ms), bad.data_ptr(), 2, h.data_ptr(), status.data_ptr(), _st()) == 0
    assert int(status.item()) == 6 and float(h[1].abs().sum()) == 0.0
    del I32


def test_argmax_first_max(L):
    x = torch.randn(7, 32000, device=DEV)
    x[3, 5] = 100.0
    x[3, 9] = 100.0  # tie: first index wins
    out = torch.empty(7, dtype=torch.int32, device=DEV)
    assert L.cb_argmax(x.data_ptr(), 7, 32000, 32000, out.data_ptr(), _st()) == 0
    ref = x.argmax(-1)
    assert out.cpu().tolist()[3] == 5
    assert out.cpu().tolist() == ref.cpu().tolist()


def _e4m3_bytes(x: np.ndarray) -> np.ndarray:
    return nvfp4.e4m3_encode(x.astype(np.float32))


@pytest.mark.parametrize("Hi,Di,k", [(4, 64, 512), (2, 8, 6), (4, 64, 64)])
def test_indexer_topk_bitexact(L, Hi, Di, k):
    rng = np.random.default_rng(Hi * 100 + Di + k)
    max_ctx = 6000
    B = 2
    ik = _e4m3_bytes(rng.normal(0, 1, (B, max_ctx, Di)))
    # many exact ties: repeated key rows and keys that score exactly 0
    ik[:, 100:400] = ik[:, 50:51]
    ik[:, 1000:3000:2] = 0
    qpos = np.array([5, k - 1, k, k + 1, 777, 5999, 4000, 2500], np.int32)
    seq = np.array([0, 1, 0, 1, 0, 1, 1, 0], np.int32)
    rows = len(qpos)
    iq = rng.normal(0, 1, (rows, Hi * Di + Hi)).astype(np.float32)  # iw packed after iq in each row
    ld = Hi * Di + Hi
    d_ik = torch.from_numpy(ik).to(DEV)
    d_iq = torch.from_numpy(iq).to(DEV)
    d_seq, d_qpos = torch.from_numpy(seq).to(DEV), torch.from_numpy(qpos).to(DEV)
    scores = torch.full((rows, max_ctx), float("nan"), device=DEV)
    sel = torch.full((rows, k + 1), -1, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(rows, dtype=torch.int32, device=DEV)
    rc = L.cb_indexer_topk(d_iq.data_ptr(), d_iq.data_ptr() + 4 * Hi * Di, ld, d_ik.data_ptr(), max_ctx, Hi, Di,
                           d_seq.data_ptr(), d_qpos.data_ptr(), rows, k, scores.data_ptr(), sel.data_ptr(),
                           cnt.data_ptr(), _st())
    assert rc == 0
    scores, sel, cnt = scores.cpu().numpy(), sel.cpu().numpy(), cnt.cpu().numpy()
    ikf = nvfp4.e4m3_decode(ik)
    for r in range(rows):
        n = qpos[r] + 1
        q = iq[r, :Hi * Di].reshape(Hi, Di)
        w = iq[r, Hi * Di:]
        ref_s = oidx.indexer_scores(q, w, ikf[seq[r], :n])
        ref_sel = oidx.topk_select(ref_s, k)
        assert cnt[r] == len(ref_sel), r
        assert np.array_equal(sel[r, :cnt[r]], ref_sel), r
        if n > k:
            assert np.array_equal(scores[r, :n].view(np.uint32), ref_s.view(np.uint32)), r


def _gdn_reference(proj, conv_state, S, p, cfg, li, T):
    """Torch restatement of the GDN mixer from its in_proj output (layers.py:155-173)."""
    H, dk, dv = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v
    B = proj.shape[0] // T
    pr = proj.view(B, T, -1)
    qkv_raw = pr[..., :2 * H * dk + H * dv]
    pre = f"self_layers.{li}.mixer."
    qkv, conv_new = om.short_conv(qkv_raw, p[pre + "conv.weight"], conv_state)
    q, k, v = qkv.split([H * dk, H * dk, H * dv], dim=-1)
    q = torch.nn.functional.normalize(q.view(B, T, H, dk), dim=-1)
    k = torch.nn.functional.normalize(k.view(B, T, H, dk), dim=-1)
    v = v.view(B, T, H, dv)
    return q, k, v, conv_new


def test_gdn_step_vs_oracle(L):
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config
    from cirrus_s_1a_b200.engine import CirrusB200

    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=3, norm_jitter=0.1)
    eng = CirrusB200(cfg, sd, max_ctx=64)
    m = eng.model
    H, dk, dv, KC = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v, cfg.gdn_conv_size
    Cc = 2 * H * dk + H * dv
    li = 1
    ldp = m.desc.self_layers[li].in_proj.rows
    g = torch.Generator().manual_seed(7)
    for T in (1, 3, 8):
        B = 2
        proj = torch.randn(B * T, ldp, generator=g)
        conv0 = torch.randn(B, KC - 1, Cc, generator=g)
        S0 = torch.randn(B, H, dk, dv, generator=g) * 0.1
        d_proj, d_conv, d_S = proj.to(DEV), conv0.clone().to(DEV), S0.clone().to(DEV)
        out = torch.zeros(B * T, H * dv, device=DEV)
        rc = L.cb_gdn_step(C.byref(m.desc), li, d_proj.data_ptr(), ldp, B, T, d_S.data_ptr(), H * dk * dv,
                           d_conv.data_ptr(), (KC - 1) * Cc, out.data_ptr(), H * dv, _st())
        assert rc == 0
        q, k, v, conv_new = _gdn_reference(proj, conv0, S0, sd, cfg, li, T)
        pre = f"self_layers.{li}.mixer."
        a = proj[:, m.desc.gdn_off_a:m.desc.gdn_off_a + H].view(B, T, H)
        b = proj[:, m.desc.gdn_off_b:m.desc.gdn_off_b + H].view(B, T, H)
        gg = -sd[pre + "A_log"].exp() * torch.nn.functional.softplus(a + sd[pre + "dt_bias"])
        o, S = om.gated_delta_rule(q, k, v, gg, b.sigmoid(), dk**-0.5, S0)
        gate = proj[:, m.desc.gdn_off_gate:m.desc.gdn_off_gate + H * dv].view(B, T, H, dv)
        o = om.rmsnorm(o, sd[pre + "o_norm.weight"], cfg.norm_eps) * torch.nn.functional.silu(gate)
        torch.testing.assert_close(out.cpu().view(B, T, H, dv), o, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(d_S.cpu(), S, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(d_conv.cpu(), conv_new, rtol=0, atol=0)
