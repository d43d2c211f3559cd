"""CPU tests of the host side: the C ABI library loads and exports every symbol
the header declares, the ctypes structs match the C layout, the decoding
helpers reproduce the reference's greedy / speculative tokens (driven by the
oracle model, no GPU), and the synthetic inputs have the stated shapes."""

import ctypes as C
import os
import re
import shutil
import subprocess
import tempfile

import pytest
import torch

from conftest import ROOT, golden
from oracle import model as om

HEADER = os.path.join(ROOT, "include", "cirrus_b200.h")


@pytest.fixture(scope="module")
def built_lib():
    from cirrus_s_1a_b200 import _lib
    from cirrus_s_1a_b200.build import build

    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        build()
    if not os.path.exists(_lib.LIB_PATH):
        pytest.skip("library not built and no nvcc")
    return _lib.lib()


def _header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(cb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_symbol(built_lib):
    from cirrus_s_1a_b200 import _lib

    names = _header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(built_lib, n), n
    assert set(names) == set(_lib.EXPORTS)
    assert built_lib.cb_abi_version() == 2
    assert built_lib.cb_status_string(5) == b"context full (position >= max_ctx)"


def test_host_argument_checks_fail_without_launching(built_lib):
    # null pointers / bad sizes are rejected before any CUDA call (no GPU needed)
    assert built_lib.cb_nvfp4_quantize(None, 4, 16, 1.0, None, None, None) == 1
    assert built_lib.cb_nvfp4_quantize(1, 4, 15, 1.0, 1, 1, None) == 1
    assert built_lib.cb_argmax(None, 1, 1, 1, None, None) == 1
    assert built_lib.cb_forward(None, None, None, 0, None, 1, 1, None, None, None, None) == 1
    assert built_lib.cb_workspace_bytes(None, 1, 1, 1) == 0
    assert built_lib.cb_verify_gemm_nvfp4(None, None, 0, 1, None, 0, 0, None, None) == 1
    assert built_lib.cb_gdn_chunk_prefill(None, None, None, None, None, 1, 1, 1, 64, 64, 1.0, None, None, None) == 1


def test_ctypes_structs_match_c_layout(built_lib):
    from cirrus_s_1a_b200 import _lib

    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("no gcc")
    structs = {"CbMatrix": _lib.CbMatrix, "CbSelfLayer": _lib.CbSelfLayer, "CbCrossLayer": _lib.CbCrossLayer,
               "CbModel": _lib.CbModel, "CbCache": _lib.CbCache, "CbWorkspaceLayout": _lib.CbWorkspaceLayout}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "cirrus_b200.h"', "int main(void){"]
    for name, cls in structs.items():
        lines.append(f'printf("{name} %zu\\n", sizeof({name}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{name}.{fname} %zu\\n", offsetof({name}, {fname}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "l.c"), os.path.join(d, "l")
        open(src, "w").write("\n".join(lines))
        subprocess.run([gcc, "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split("\n")
    got = dict(l.split() for l in out if l)
    for name, cls in structs.items():
        assert int(got[name]) == C.sizeof(cls), name
        for fname, _ in cls._fields_:
            assert int(got[f"{name}.{fname}"]) == getattr(cls, fname).offset, (name, fname)


# ----------------------------------------------------------- decoding logic
class OracleModel:
    """CPU stand-in with the CirrusModel call signature (drives the host-side
    decoding helpers without a GPU)."""

    def __init__(self, cfg, p):
        self.cfg, self.p = cfg, p

    def __call__(self, input_ids, cache=None, use_cache=False, n_logits=None):
        return om.forward(self.p, self.cfg, input_ids, cache=cache, use_cache=use_cache, n_logits=n_logits)

    def mtp_draft(self, h_last, token, n=None):
        return om.mtp_draft(self.p, self.cfg, h_last, int(token), n)


def test_greedy_and_speculative_reproduce_reference_tokens():
    from dataclasses import replace

    from cirrus_s_1a_b200 import generate as G
    from cirrus_s_1a_b200.config import get_config

    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    try:
        rec = golden("debug_ref.pt")["sparse"]
        p = {k: (v.double() if v.is_floating_point() else v) for k, v in rec["state_dict"].items()}
        m = OracleModel(replace(get_config("cirrus-s-1a-debug")), p)
        prompt = rec["gen_prompt"]
        assert G.greedy(m, prompt, 30)[0] == rec["greedy"]
        assert G.speculative_greedy(m, prompt, 30, use_mtp=False)[0] == rec["spec_nomtp"]
        assert G.speculative_greedy(m, prompt, 30)[0] == rec["spec_mtp"]
    finally:
        torch.set_default_dtype(old)


def test_drafter_and_acceptance_rules():
    from cirrus_s_1a_b200.generate import PromptLookupDrafter, accept_greedy, choose_draft

    d = PromptLookupDrafter(max_ngram=3, min_ngram=2, max_draft=4)
    d.extend([7, 8, 1, 2, 3, 4, 5, 9, 7, 8])
    assert d.draft() == [1, 2, 3, 4]
    d = PromptLookupDrafter(max_ngram=1, min_ngram=1, max_draft=1)
    d.extend([3, 5, 3, 6, 3])
    assert d.draft() == [6]  # the latest occurrence wins
    d = PromptLookupDrafter(max_ngram=3, min_ngram=1, max_draft=2)
    d.extend([5, 1, 6, 6, 2, 1, 9, 9, 5, 1])
    assert d.draft() == [6, 6]  # longest seen n-gram (5, 1)
    assert PromptLookupDrafter().draft() == []
    assert accept_greedy([1, 2, 3], [1, 2, 4, 0]) == (2, [1, 2, 4])
    assert accept_greedy([], [7]) == (0, [7])
    with pytest.raises(ValueError):
        accept_greedy([1, 2], [1, 2])
    assert choose_draft([4, 5, 6], [1, 1]) == [4, 5, 6]
    assert choose_draft([4], [1, 1]) == [1, 1]
    assert choose_draft([4], []) == [4]
    with pytest.raises(ValueError):
        PromptLookupDrafter(max_ngram=1, min_ngram=2)


def test_synthetic_inputs():
    from cirrus_s_1a_b200 import synthetic
    from cirrus_s_1a_b200.config import baseline_config, get_config

    cfg = get_config("cirrus-s-1a-debug")
    sd = synthetic.random_state_dict(cfg, seed=0)
    assert sd["embed.weight"] is sd["lm_head.weight"]
    assert sd["self_layers.0.mixer.qkv.weight"].shape == (2 * 2 * 16 + 2 * 16, 64)
    bc = baseline_config()
    lin = synthetic.linear_shapes(bc)
    assert sum(n * k for n, k in lin.values()) > 150e6
    toks = synthetic.random_prompt(4096, 32000, seed=0)
    assert len(toks) == 4096 and min(toks) >= 0 and max(toks) < 32000
    seen, copied = set(), 0
    for start in range(0, 4096, 8):
        copied += tuple(toks[start:start + 8]) in seen
        for j in range(max(0, start - 7), start + 1):  # every 8-gram that ends before the next span
            seen.add(tuple(toks[j:j + 8]))
    assert 0.15 < copied / 512 < 0.35
