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
    assert built_lib.cb_abi_version() == 3
    assert built_lib.cb_status_string(5) == b"context full (position >= max_ctx)"


def test_host_argument_checks_fail_without_launching(built_lib):
    # null pointers / bad sizes are rejected before any CUDA call (no GPU needed)
    assert built_lib.cb_nvfp4_quantize(None, 4, 16, 1.0, None, None, None) == 1
    assert built_lib.cb_nvfp4_quantize(1, 4, 15, 1.0, 1, 1, None) == 1
    assert built_lib.cb_argmax(None, 1, 1, 1, None, None) == 1
    assert built_lib.cb_forward(None, None, None, 0, None, 1, 1, None, None, None, None) == 1
    assert built_lib.cb_workspace_bytes(None, 1, 1, 1) == 0
    assert built_lib.cb_gemm_nvfp4(None, None, 0, 1, 0, None, 0.0, None, 0, 0, 0, None, 0, None, None) == 1
    assert built_lib.cb_gemm_scratch_bytes(768, 64) == 12 * 16384 and built_lib.cb_gemm_scratch_bytes(100, 1) == 0
    assert built_lib.cb_gdn_chunk_prefill(None, None, None, None, None, 1, 1, 1, 64, 64, 1.0, None, None, None) == 1


def test_ctypes_structs_match_c_layout(built_lib):
    from cirrus_s_1a_b200 import _lib

    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("no gcc")
    structs = {"CbMatrix": _lib.CbMatrix, "CbSelfLayer": _lib.CbSelfLayer, "CbCrossLayer": _lib.CbCrossLayer,
               "CbModel": _lib.CbModel, "CbCache": _lib.CbCache, "CbWorkspaceLayout": _lib.CbWorkspaceLayout,
               "CbSliced": _lib.CbSliced, "CbMtp": _lib.CbMtp}
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


REFERENCE = os.environ.get("CIRRUS_REFERENCE", "/root/reference")


def _reference_generate():
    """The reference's own decoding loop (cirrus/model/generate.py), imported
    read-only from a checkout when one is present; the test is skipped otherwise."""
    import importlib
    import sys

    if not os.path.isdir(os.path.join(REFERENCE, "cirrus")):
        pytest.skip("reference checkout not present")
    if REFERENCE not in sys.path:
        sys.path.append(REFERENCE)
    return importlib.import_module("cirrus.model.generate")


def test_reference_decoding_loop_drives_the_oracle_to_the_reference_tokens():
    """The reference's greedy / speculative_greedy (MTP drafts on, the default)
    over a CPU stand-in with CirrusB200's call signature reproduce the tokens the
    reference model produced (golden fixture)."""
    from dataclasses import replace

    from cirrus_s_1a_b200.config import get_config

    G = _reference_generate()
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


def test_drop_in_surface_matches_the_reference_model():
    """CirrusB200 exposes what the reference's decoding loop calls
    (generate.py:30, 39, 64-77): the forward signature and defaults of
    CirrusModel.forward (model.py:99-110) for inference, mtp_draft (model.py:231)
    and an Output with logits / hidden / cache; the cache has clone()."""
    import inspect

    _reference_generate()
    from cirrus.model import model as RM

    from cirrus_s_1a_b200.engine import CirrusB200, DeviceCache, Output

    ref = inspect.signature(RM.CirrusModel.forward).parameters
    ours = inspect.signature(CirrusB200.forward).parameters
    for name in ("input_ids", "cache", "use_cache", "labels", "n_logits"):
        assert name in ours, name
        assert ours[name].default == ref[name].default, name
    assert list(ours)[:6] == list(ref)[:6]
    rm = inspect.signature(RM.CirrusModel.mtp_draft).parameters
    om_ = inspect.signature(CirrusB200.mtp_draft).parameters
    assert list(om_) == list(rm) and om_["n"].default == rm["n"].default
    assert [f for f in Output.__dataclass_fields__] == [f for f in RM.Output.__dataclass_fields__]
    assert callable(getattr(DeviceCache, "clone")) and isinstance(DeviceCache.pos, property)


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
