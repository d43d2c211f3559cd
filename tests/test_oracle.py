"""Pin the CPU oracle against the reference's own outputs (golden fixtures
written by tests/golden/make_golden.py from the reference implementation)."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import indexer as oidx
from oracle import model as om
from oracle import nvfp4


# ------------------------------------------------------------------ NVFP4
def test_e4m3_all_codes_roundtrip():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    vals = nvfp4.e4m3_decode(codes)
    back = nvfp4.e4m3_encode(vals)
    # +0 and -0 keep their sign bit
    assert np.array_equal(back, codes)
    ref = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(vals, ref)


def test_e4m3_encode_matches_torch_cast():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 0.01, 20000), rng.normal(0, 50, 20000), rng.uniform(-448, 448, 5000)])
    x = x.astype(np.float32)
    ours = nvfp4.e4m3_encode(x)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)
    # saturation (torch's cast gives NaN above the range; the codec saturates)
    assert nvfp4.e4m3_decode(nvfp4.e4m3_encode(np.float32([1e6, -1e6]))).tolist() == [448.0, -448.0]


def test_e2m1_ties_and_saturation():
    x = np.float32([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.25, -5.0, 0.26, -0.74, 1e9])
    vals = nvfp4.E2M1_LUT[nvfp4.e2m1_encode(x)]
    assert vals.tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, -0.0, -4.0, 0.5, -0.5, 6.0]


def test_e2m1_threshold_encoder_equals_table_rne():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.normal(0, 2, 100000), rng.uniform(-8, 8, 100000),
                        np.float32([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 6.5, -0.0, 0.0])]).astype(np.float32)
    x = np.concatenate([x, np.nextafter(x, np.float32(np.inf)), np.nextafter(x, np.float32(-np.inf))])
    assert np.array_equal(nvfp4.e2m1_encode(x), nvfp4.e2m1_encode_table(x))


def test_dequant_matches_reference_benchmark_dequant():
    g = golden("nvfp4_ref.pt")
    ours = nvfp4.dequantize(g["codes"].numpy(), g["scales"].numpy())
    assert np.array_equal(ours, g["dequant"].numpy())
    codes = nvfp4.unpack_standard(g["packed"].numpy())
    assert np.array_equal(codes, g["codes"].numpy())
    ours05 = nvfp4.dequantize(codes, g["scales"].numpy(), 0.5)
    assert np.array_equal(ours05, g["dequant_packed_g05"].numpy())
    assert np.array_equal(nvfp4.pack_standard(codes), g["packed"].numpy())


def test_quantizer_matches_independent_restatement():
    g = golden("nvfp4_ref.pt")
    assert np.array_equal(nvfp4.fake_quant(g["w"].numpy()), g["w_q"].numpy())


def test_quantizer_zero_block_and_range():
    w = np.zeros((2, 32), np.float32)
    w[1, 16:] = np.linspace(-1, 1, 16)
    codes, scales = nvfp4.quantize(w)
    assert codes[0].max() == 0 and scales[0].max() == 0
    deq = nvfp4.dequantize(codes, scales)
    sval = nvfp4.e4m3_decode(scales[1, 1])
    # the widest E2M1 gap is 2 (between 4 and 6), so the error is at most one scale unit
    assert np.abs(deq[1, 16:] - w[1, 16:]).max() <= sval + 1e-6
    assert np.abs(deq[1]).max() == pytest.approx(1.0, rel=0.07)


# ------------------------------------------------------------------ units
def test_gdn_recurrence_matches_reference():
    u = golden("units_ref.pt")["gdn"]
    o, S = om.gated_delta_rule(u["q"], u["k"], u["v"], u["g"], u["beta"], u["scale"], u["S0"])
    torch.testing.assert_close(o, u["o"], rtol=0, atol=1e-12)
    torch.testing.assert_close(S, u["S"], rtol=0, atol=1e-12)


def test_short_conv_matches_reference():
    u = golden("units_ref.pt")["conv"]
    y, c = om.short_conv(u["x"], u["w"], None)
    torch.testing.assert_close(y, u["y"], rtol=0, atol=1e-12)
    torch.testing.assert_close(c, u["cache"], rtol=0, atol=0)
    y1, c1 = om.short_conv(u["x"][:, :3], u["w"], None)
    y2, _ = om.short_conv(u["x"][:, 3:], u["w"], c1)
    torch.testing.assert_close(torch.cat((y1, y2), 1), u["y"], rtol=0, atol=1e-12)


def test_rope_matches_reference():
    u = golden("units_ref.pt")["rope"]

    class C:
        head_dim, partial_rotary, rope_theta = 64, 0.5, 1e6

    torch.testing.assert_close(om.rope(u["x"], u["pos"], C), u["y"], rtol=0, atol=0)


def test_indexer_scores_fixed_order_close_to_reference():
    u = golden("units_ref.pt")["indexer"]
    torch.testing.assert_close(om.indexer_scores(u["iq"], u["iw"], u["ik"]), u["s"], rtol=0, atol=0)
    for t in range(3):
        s = oidx.indexer_scores(u["iq"][0, t].numpy(), u["iw"][0, t].numpy(), u["ik"][0].numpy())
        np.testing.assert_allclose(s, u["s"][0, t].numpy(), rtol=1e-5, atol=1e-5)


def test_topk_rule_matches_reference_masks():
    for case in golden("units_ref.pt")["topk"]:
        sc, causal, k, mask = case["scores"], case["causal"], case["k"], case["mask"]
        assert torch.equal(om.topk_mask(sc, causal, k), mask)
        Tq, Tk = sc.shape[1], sc.shape[2]
        for t in range(Tq):
            n = Tk - Tq + t + 1
            sel = oidx.topk_select(sc[0, t, :n].numpy(), k)
            ref = torch.nonzero(mask[0, t]).flatten().numpy()
            assert np.array_equal(sel, ref), (case["k"], t)


def test_topk_negative_zero_ties_with_positive_zero():
    s = np.float32([0.0, -0.0, 0.0, -0.0, 1.0, -1.0, 0.0])
    # k=3: 1.0 (idx 4), then zeros most-recent-first: idx 6, 3 (-0 counts as 0); diag 6 is in
    assert oidx.topk_select(s, 3).tolist() == [3, 4, 6]
    mask = om.topk_mask(torch.from_numpy(s)[None, None], torch.ones(1, 1, 7, dtype=torch.bool), 3)
    assert torch.nonzero(mask[0, 0]).flatten().tolist() == [3, 4, 6]


# ------------------------------------------------------------ debug model
def _sd(rec, dtype=torch.float64):
    return {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in rec["state_dict"].items()}


def _debug_cfg(variant):
    from dataclasses import replace

    from cirrus_s_1a_b200.config import get_config

    return replace(get_config("cirrus-s-1a-debug"), **({} if variant == "sparse" else {"sparse_topk": None}))


@pytest.mark.parametrize("variant", ["sparse", "dense"])
def test_debug_model_full_and_incremental(variant):
    rec = golden("debug_ref.pt")[variant]
    cfg, p, ids = _debug_cfg(variant), _sd(rec), rec["ids"]
    full = om.forward(p, cfg, ids).logits
    torch.testing.assert_close(full, rec["full_logits"], rtol=0, atol=1e-10)
    torch.testing.assert_close(om.forward(p, cfg, ids, n_logits=1).logits, rec["last_logits_n1"], rtol=0, atol=1e-10)
    o = om.forward(p, cfg, ids[:, :11], use_cache=True)
    for i, l in enumerate(rec["prefill11_cache"]["layers"]):
        for k, v in l.items():
            torch.testing.assert_close(o.cache.layers[i][k], v, rtol=0, atol=1e-10)
    steps, cache = [o.logits], o.cache
    for t in range(11, 20):
        o = om.forward(p, cfg, ids[:, t:t + 1], cache=cache)
        steps.append(o.logits)
        cache = o.cache
    torch.testing.assert_close(torch.cat(steps, 1), rec["incremental_logits"], rtol=0, atol=1e-10)
    for k, v in rec["final_cache"]["shared"].items():
        torch.testing.assert_close(cache.shared[k], v, rtol=0, atol=1e-10)
    o = om.forward(p, cfg, ids[:, :11], use_cache=True)
    ov = om.forward(p, cfg, ids[:, 11:15], cache=o.cache, n_logits=4)
    torch.testing.assert_close(ov.logits, rec["verify4_logits"], rtol=0, atol=1e-10)


@pytest.mark.parametrize("variant", ["sparse", "dense"])
def test_debug_model_greedy_and_quantized(variant):
    rec = golden("debug_ref.pt")[variant]
    cfg, p = _debug_cfg(variant), _sd(rec)
    assert om.greedy(p, cfg, rec["gen_prompt"], 30) == rec["greedy"]
    pq = om.quantized_params(rec["state_dict"])
    pq = {k: (v.double() if v.is_floating_point() else v) for k, v in pq.items()}
    torch.testing.assert_close(om.forward(pq, cfg, rec["ids"]).logits, rec["q_full_logits"], rtol=0, atol=1e-10)
    assert om.greedy(pq, cfg, rec["gen_prompt"], 30) == rec["q_greedy"]


def test_debug_mtp_draft_runs():
    rec = golden("debug_ref.pt")["sparse"]
    cfg, p = _debug_cfg("sparse"), _sd(rec)
    o = om.forward(p, cfg, torch.tensor([rec["gen_prompt"]]), use_cache=True, n_logits=1)
    d = om.mtp_draft(p, cfg, o.hidden[:, -1], int(o.logits[0, -1].argmax()))
    assert len(d) == cfg.mtp_passes and all(0 <= t < cfg.vocab_size for t in d)


# --------------------------------------------------------- baseline shapes
def test_baseline_shapes_oracle_matches_reference():
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config

    rec = golden("baseline_ref.pt")
    cfg = baseline_config()
    sd = synthetic.random_state_dict(cfg, seed=0)
    assert sum(v.numel() for k, v in sd.items() if k not in ("embed.weight", "draft_ids")) == rec["num_params"]
    p = om.quantized_params(sd)
    prompt = rec["prompt"]
    o = om.forward(p, cfg, torch.tensor([prompt]), use_cache=True, n_logits=1)
    torch.testing.assert_close(o.logits[0, -1], rec["prefill_logits"], rtol=1e-4, atol=1e-4)
    toks = [int(o.logits[0, -1].argmax())]
    cache = o.cache
    for _ in range(3):
        o = om.forward(p, cfg, torch.tensor([[toks[-1]]]), cache=cache, n_logits=1)
        cache = o.cache
        toks.append(int(o.logits[0, -1].argmax()))
    assert toks == rec["greedy4"]
    torch.testing.assert_close(o.logits[0, -1], rec["step_logits"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(cache.layers[0]["S"][0, 0], rec["S_layer0_head0"], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(cache.shared["ik"][0, -4:], rec["shared_ik_last"], rtol=1e-4, atol=1e-5)
    ov = om.forward(p, cfg, torch.tensor([rec["verify_in"]]), cache=cache, n_logits=4)
    assert ov.logits[0].argmax(-1).tolist() == rec["verify_argmax"]
    torch.testing.assert_close(torch.stack((ov.logits[0, 0], ov.logits[0, -1])), rec["verify_logits_first_last"],
                               rtol=1e-4, atol=1e-4)


# ---------------------------------------------------------------- decoding
def test_decoding_oracle_matches_reference_drafter():
    """oracle/decoding.py against the reference's PromptLookupDrafter,
    accept_greedy and choose_draft (fixtures from cirrus/decoding/prompt_lookup.py)."""
    from oracle import decoding as od

    rec = golden("decoding_ref.pt")
    assert len(rec["drafts"]) > 300
    nonempty = 0
    for c in rec["drafts"]:
        toks = rec["streams"][c["stream"]][:c["len"]]
        got = od.lookup_draft(toks, c["k"], c["min_ngram"], c["max_ngram"])
        assert got == c["draft"], c
        nonempty += bool(got)
    assert nonempty > 100
    for c in rec["accepts"]:
        n, emit = c["out"]
        assert od.accept_greedy(c["draft"], c["target"]) == (n, list(emit))
    for c in rec["chooses"]:
        assert od.choose_draft(c["lookup"], c["mtp"]) == list(c["out"])


class _OracleModel:
    """The oracle forward behind the reference model's inference surface."""

    def __init__(self, p, cfg):
        self.p, self.cfg = p, cfg

    def __call__(self, ids, cache=None, use_cache=False, n_logits=None):
        return om.forward(self.p, self.cfg, ids, cache=cache, use_cache=use_cache, n_logits=n_logits)

    def mtp_draft(self, h_last, token):
        ids = self.p["draft_ids"].long()  # the fixture stores every tensor as float
        return om.mtp_draft(self.p, self.cfg, h_last, int(token.reshape(-1)[0]), draft_ids=ids)


@pytest.mark.parametrize("variant", ["sparse", "dense"])
def test_verifier_loops_reproduce_reference_token_sequences(variant):
    """oracle.decoding.greedy_loop / speculative_loop over the float64 oracle model
    emit the tokens the reference's greedy / speculative_greedy emitted (default
    max_draft 8 with MTP drafts, and without MTP) on the same model and prompt."""
    from oracle import decoding as od

    rec = golden("debug_ref.pt")[variant]
    model = _OracleModel(_sd(rec), _debug_cfg(variant))
    prompt = rec["gen_prompt"]
    assert od.greedy_loop(model, prompt, 30) == rec["greedy"]
    assert od.speculative_loop(model, prompt, 30)[0] == rec["spec_mtp"]
    assert od.speculative_loop(model, prompt, 30, use_mtp=False)[0] == rec["spec_nomtp"]
