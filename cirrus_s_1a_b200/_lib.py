"""ctypes binding of ``libcirrus_b200.so`` (the C ABI of ``include/cirrus_b200.h``).

The library is loaded from this package directory only.  Importing this
module never builds anything; a missing library is an error, never a
fallback: there is no CPU path.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcirrus_b200.so")

CB_MAX_SELF = 32
CB_MAX_CROSS = 16
CB_MAX_T = 8
CB_TILE_ROWS = 16
CB_SWA_EXTRA = 16
CB_PREFILL_CHUNK = 128
CB_LAYER_GDN, CB_LAYER_SWA = 0, 1

STATUS = {0: "ok", 1: "invalid argument", 2: "shape not supported", 3: "CUDA launch failed",
          4: "workspace too small", 5: "context full (position >= max_ctx)", 6: "token id outside the vocabulary",
          7: "rows * max_ctx exceeds the static scratch of cb_indexer_topk_noalloc",
          8: "a bounded wait in the persistent kernel timed out"}
CB_PATH_AUTO, CB_PATH_MULTI_KERNEL = 0, 1
CB_NOALLOC_MAX_SCORES = 1 << 20
CB_GEMM_PRE_NONE, CB_GEMM_PRE_RMSNORM = 0, 1
CB_GEMM_EPI_STORE, CB_GEMM_EPI_ADD, CB_GEMM_EPI_SWIGLU = 0, 1, 2

EXPORTS = ("cb_abi_version", "cb_status_string", "cb_nvfp4_quantize", "cb_nvfp4_pack_tiles", "cb_gemv_nvfp4",
           "cb_embed", "cb_argmax", "cb_gdn_step", "cb_indexer_topk", "cb_workspace_bytes", "cb_forward",
           "cb_read_status", "cb_clear_status", "cb_launch_count", "cb_indexer_topk_noalloc", "cb_read_trace",
           "cb_gdn_chunk_prefill", "cb_set_wait_limit",
           "cb_workspace_layout", "cb_nvfp4_slice_bytes", "cb_nvfp4_pack_slices", "cb_prompt_lookup_draft",
           "cb_spec_accept", "cb_mtp_workspace_bytes", "cb_mtp_draft", "cb_gemm_nvfp4", "cb_gemm_scratch_bytes",
           "cb_stream_plan_bytes", "cb_stream_plan", "cb_weight_stream_nvfp4")

P = C.c_void_p
I32 = C.c_int32


class CbMatrix(C.Structure):
    _fields_ = [("tiles", P), ("tile_scale", P), ("rows", I32), ("k", I32)]


class CbSliced(C.Structure):
    _fields_ = [("data", P), ("tensor_scale", P), ("rows", I32), ("k", I32), ("width", I32)]


class CbSelfLayer(C.Structure):
    _fields_ = [("kind", I32), ("slot", I32), ("norm1", P), ("norm2", P), ("in_proj", CbMatrix),
                ("o_proj", CbMatrix), ("gate_up", CbMatrix), ("down", CbMatrix), ("conv_w", P), ("A_log", P),
                ("dt_bias", P), ("o_norm", P), ("q_norm", P), ("k_norm", P), ("o_proj_ks", CbSliced),
                ("down_ks", CbSliced)]


class CbCrossLayer(C.Structure):
    _fields_ = [("norm1", P), ("norm2", P), ("q_gate", CbMatrix), ("o_proj", CbMatrix), ("gate_up", CbMatrix),
                ("down", CbMatrix), ("q_norm", P), ("down_ks", CbSliced)]


class CbModel(C.Structure):
    _fields_ = [
        ("d_model", I32), ("vocab_size", I32), ("n_self_layers", I32), ("n_cross_layers", I32),
        ("gdn_heads", I32), ("gdn_dk", I32), ("gdn_dv", I32), ("conv_size", I32),
        ("n_q_heads", I32), ("n_kv_heads", I32), ("head_dim", I32), ("rot_dim", I32),
        ("swa_window", I32), ("sparse_topk", I32),
        ("indexer_heads", I32), ("indexer_dim", I32), ("ffn_hidden", I32),
        ("norm_eps", C.c_float),
        ("forward_path", I32),
        ("inv_freq", P),
        ("gdn_off_gate", I32), ("gdn_off_a", I32), ("gdn_off_b", I32),
        ("swa_off_kv", I32), ("swa_off_gate", I32),
        ("sh_off_ik", I32), ("sh_off_iq", I32), ("sh_off_iw", I32),
        ("cr_off_gate", I32),
        ("self_layers", CbSelfLayer * CB_MAX_SELF),
        ("shared_norm", P), ("shared_k_norm", P), ("shared_proj", CbMatrix),
        ("cross_layers", CbCrossLayer * CB_MAX_CROSS),
        ("final_norm", P), ("lm_head", CbMatrix),
    ]


class CbMtp(C.Structure):
    _fields_ = [("norm_h", P), ("norm_e", P), ("ffn_norm", P), ("proj", CbMatrix), ("gate_up", CbMatrix),
                ("down", CbMatrix), ("draft_head", CbMatrix), ("draft_ids", P), ("n_draft", I32)]


class CbCache(C.Structure):
    _fields_ = [("batch", I32), ("max_ctx", I32), ("swa_slots", I32), ("n_gdn", I32), ("n_swa", I32),
                ("pos", P), ("gdn_state", P), ("gdn_conv", P), ("swa_k", P), ("swa_v", P), ("kv_k", P),
                ("kv_v", P), ("kv_ik", P), ("snap_state", P), ("snap_conv", P)]


class CbWorkspaceLayout(C.Structure):
    _fields_ = [("bytes", C.c_uint64), ("proj", C.c_uint64), ("sel_idx", C.c_uint64), ("sel_cnt", C.c_uint64),
                ("ld_proj", I32), ("sel_ld", I32), ("rows", I32)]


class CbError(RuntimeError):
    pass


_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CbError(f"{LIB_PATH} is missing: build it with `python -m cirrus_s_1a_b200.build` "
                          "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        L.cb_abi_version.restype = C.c_int
        L.cb_status_string.restype = C.c_char_p
        L.cb_status_string.argtypes = [C.c_int]
        L.cb_nvfp4_quantize.argtypes = [P, I32, I32, C.c_float, P, P, P]
        L.cb_nvfp4_pack_tiles.argtypes = [P, P, I32, I32, P, P]
        L.cb_nvfp4_slice_bytes.restype = C.c_int64
        L.cb_nvfp4_slice_bytes.argtypes = [I32, I32]
        L.cb_nvfp4_pack_slices.argtypes = [P, P, I32, I32, I32, P, P]
        L.cb_gemv_nvfp4.argtypes = [C.POINTER(CbMatrix), P, I32, I32, P, I32, I32, P]
        L.cb_gemm_nvfp4.argtypes = [C.POINTER(CbMatrix), P, I32, I32, I32, P, C.c_float, P, I32, I32, I32, P,
                                    C.c_size_t, P, P]
        L.cb_gemm_scratch_bytes.restype = C.c_size_t
        L.cb_gemm_scratch_bytes.argtypes = [I32, I32]
        L.cb_stream_plan_bytes.restype = C.c_size_t
        L.cb_stream_plan_bytes.argtypes = [I32]
        L.cb_stream_plan.argtypes = [C.POINTER(CbMatrix), I32, P, C.c_size_t, C.POINTER(C.c_int64), P]
        L.cb_weight_stream_nvfp4.argtypes = [P, I32, I32, P, I32, I32, I32, P, C.c_int64, P, P]
        L.cb_gdn_chunk_prefill.argtypes = [P, P, P, P, P, I32, I32, I32, I32, I32, C.c_float, P, P, P]
        L.cb_embed.argtypes = [C.POINTER(CbMatrix), P, I32, P, P, P]
        L.cb_argmax.argtypes = [P, I32, I32, I32, P, P]
        L.cb_gdn_step.argtypes = [C.POINTER(CbModel), I32, P, I32, I32, I32, P, C.c_int64, P, C.c_int64, P, I32, P]
        L.cb_indexer_topk.argtypes = [P, P, I32, P, I32, I32, I32, P, P, I32, I32, P, P, P, P]
        L.cb_indexer_topk_noalloc.argtypes = [P, P, I32, P, I32, I32, I32, P, P, I32, I32, P, P, P]
        L.cb_workspace_bytes.restype = C.c_size_t
        L.cb_workspace_bytes.argtypes = [C.POINTER(CbModel), I32, I32, I32]
        L.cb_forward.argtypes = [C.POINTER(CbModel), C.POINTER(CbCache), P, C.c_size_t, P, I32, I32, P, P, P, P]
        L.cb_read_status.argtypes = [P, C.POINTER(I32), P]
        L.cb_mtp_workspace_bytes.restype = C.c_size_t
        L.cb_mtp_workspace_bytes.argtypes = [C.POINTER(CbModel), C.POINTER(CbMtp)]
        L.cb_mtp_draft.argtypes = [C.POINTER(CbModel), C.POINTER(CbMtp), P, P, I32, P, P, C.c_size_t, P]
        L.cb_prompt_lookup_draft.argtypes = [P, I32, P, P, I32, I32, I32, I32, P, I32, P, P]
        L.cb_spec_accept.argtypes = [C.POINTER(CbModel), C.POINTER(CbCache), P, P, P, I32, P, I32, P, P, P, P]
        L.cb_clear_status.argtypes = [P, P]
        L.cb_set_wait_limit.argtypes = [P, C.c_uint64, I32, P]
        L.cb_workspace_layout.argtypes = [C.POINTER(CbModel), I32, I32, I32, C.POINTER(CbWorkspaceLayout)]
        L.cb_read_trace.argtypes = [C.POINTER(CbModel), I32, I32, I32, P, P, I32, P]
        L.cb_launch_count.restype = C.c_int64
        L.cb_launch_count.argtypes = []
        for name in EXPORTS:
            if name not in ("cb_status_string", "cb_workspace_bytes", "cb_launch_count", "cb_nvfp4_slice_bytes",
                            "cb_mtp_workspace_bytes", "cb_gemm_scratch_bytes", "cb_stream_plan_bytes"):
                getattr(L, name).restype = C.c_int
        if L.cb_abi_version() != 3:
            raise CbError("libcirrus_b200.so ABI version mismatch")
        _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise CbError(f"{what}: {STATUS.get(rc, 'error')} (code {rc})")


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
