"""Drop-in B200 model: ``CirrusB200`` behaves like the reference ``CirrusModel``
for inference (``cirrus/model/model.py:99-176``): ``model(input_ids, cache=...,
use_cache=..., n_logits=...)`` returns an ``Output`` whose ``logits``,
``hidden`` and ``cache`` the reference's ``greedy`` / ``speculative_greedy``
(``cirrus/model/generate.py:28-89``) consume unchanged.

All compute runs in ``libcirrus_b200.so`` (sm_100a); torch only owns device
memory and streams.  There is no CPU path: without a CUDA device or without
the built library the constructor raises.

Weights: every Linear is quantised on the GPU to NVFP4 (absmax/6 E4M3 block
scales, E2M1 codes, float32 tensor scale) and packed into 16-row tiles;
matrices that read the same input are concatenated (GDN qkv|gate|ab, SWA
q|kv|gate, shared kv|idx_k|idx_q|idx_w, cross q|gate).  The embedding is the
tied LM head (``model.py:76-77``), gathered from the same NVFP4 tiles.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from cirrus_s_1a_b200 import _lib
from cirrus_s_1a_b200._lib import (CB_LAYER_GDN, CB_LAYER_SWA, CB_MAX_T, CB_PREFILL_CHUNK, CB_SWA_EXTRA, CbCache,
                                   CbMatrix, CbModel,
                                   CbMtp, CbSliced)


def pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def tile_bytes(k: int) -> int:
    return 16 * (k // 2 + k // 16)


def inv_freq_of(cfg) -> torch.Tensor:
    """Rotary inverse frequencies exactly as ``layers.py:67-70`` computes them (float32)."""
    rot = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
    return 1.0 / (cfg.rope_theta ** (torch.arange(0, rot, 2, dtype=torch.float32) / max(rot, 1)))


def _stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class PackedMatrix:
    """One or more NVFP4 matrices concatenated row-wise in tile layout."""

    def __init__(self, weights: list, device, tensor_scale: float = 1.0):
        k = weights[0].shape[1]
        if any(w.shape[1] != k for w in weights) or k % 16:
            raise ValueError("concatenated matrices must share K (a multiple of 16)")
        self.k = k
        self.offsets = []
        rows = 0
        for w in weights:
            self.offsets.append(rows)
            rows += pad16(w.shape[0])
        self.rows = rows
        self.real_rows = sum(w.shape[0] for w in weights)
        self.real_bytes = self.real_rows * k * 9 // 16  # E2M1 codes + E4M3 scales of the real rows
        self.tiles = torch.zeros(rows // 16 * tile_bytes(k), dtype=torch.uint8, device=device)
        self.tile_scale = torch.full((rows // 16,), float(tensor_scale), dtype=torch.float32, device=device)
        L = _lib.lib()
        st = _stream_ptr(device)
        for w, off in zip(weights, self.offsets):
            n = w.shape[0]
            wd = w.detach().to(device=device, dtype=torch.float32).contiguous()
            codes = torch.empty(n, k // 2, dtype=torch.uint8, device=device)
            scales = torch.empty(n, k // 16, dtype=torch.uint8, device=device)
            _lib.check(L.cb_nvfp4_quantize(wd.data_ptr(), n, k, float(tensor_scale), codes.data_ptr(),
                                           scales.data_ptr(), st), "cb_nvfp4_quantize")
            dst = self.tiles.data_ptr() + off // 16 * tile_bytes(k)
            _lib.check(L.cb_nvfp4_pack_tiles(codes.data_ptr(), scales.data_ptr(), n, k, dst, st),
                       "cb_nvfp4_pack_tiles")

    def struct(self) -> CbMatrix:
        return CbMatrix(self.tiles.data_ptr(), self.tile_scale.data_ptr(), self.rows, self.k)


class SlicedMatrix:
    """A column-sliced NVFP4 copy of one matrix (``CbSliced``): the persistent
    kernel's split-K phases read one slice of ``width`` columns per CTA."""

    def __init__(self, weight, width: int, device, tensor_scale: float = 1.0):
        n, k = weight.shape
        L = _lib.lib()
        self.width, self.rows, self.k = width, n, k
        sb = L.cb_nvfp4_slice_bytes(n, width)
        if sb <= 0 or k % width or k % 16:
            raise ValueError(f"cannot slice a [{n}, {k}] matrix into {width}-column slices")
        st = _stream_ptr(device)
        wd = weight.detach().to(device=device, dtype=torch.float32).contiguous()
        codes = torch.empty(n, k // 2, dtype=torch.uint8, device=device)
        scales = torch.empty(n, k // 16, dtype=torch.uint8, device=device)
        _lib.check(L.cb_nvfp4_quantize(wd.data_ptr(), n, k, float(tensor_scale), codes.data_ptr(), scales.data_ptr(),
                                       st), "cb_nvfp4_quantize")
        self.data = torch.empty(k // width * sb, dtype=torch.uint8, device=device)
        _lib.check(L.cb_nvfp4_pack_slices(codes.data_ptr(), scales.data_ptr(), n, k, width, self.data.data_ptr(), st),
                   "cb_nvfp4_pack_slices")
        self.scale = torch.full((1,), float(tensor_scale), dtype=torch.float32, device=device)

    def struct(self) -> CbSliced:
        return CbSliced(self.data.data_ptr(), self.scale.data_ptr(), self.rows, self.k, self.width)


class DeviceModel:
    """NVFP4 weights of one model on one CUDA device plus its ``CbModel`` descriptor."""

    def __init__(self, cfg, sd: dict, device, tensor_scale: float = 1.0, path: str = "auto"):
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        f32 = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
        self._keep: list = []
        kinds = cfg.self_layer_kinds
        if len(kinds) > _lib.CB_MAX_SELF or cfg.n_cross_layers > _lib.CB_MAX_CROSS:
            raise ValueError("too many layers for the descriptor")
        m = CbModel()
        m.d_model, m.vocab_size = cfg.d_model, cfg.vocab_size
        m.n_self_layers, m.n_cross_layers = len(kinds), cfg.n_cross_layers
        m.gdn_heads, m.gdn_dk, m.gdn_dv, m.conv_size = (cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v,
                                                        cfg.gdn_conv_size)
        m.n_q_heads, m.n_kv_heads, m.head_dim = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
        m.rot_dim = int(cfg.head_dim * cfg.partial_rotary) // 2 * 2
        m.swa_window = cfg.swa_window
        m.sparse_topk = 0 if cfg.sparse_topk is None else cfg.sparse_topk
        m.indexer_heads, m.indexer_dim, m.ffn_hidden = cfg.indexer_heads, cfg.indexer_dim, cfg.ffn_hidden
        m.norm_eps = cfg.norm_eps
        m.forward_path = {"auto": _lib.CB_PATH_AUTO, "multi": _lib.CB_PATH_MULTI_KERNEL}[path]
        inv = f32(inv_freq_of(cfg))
        self._keep.append(inv)
        m.inv_freq = inv.data_ptr()

        def keep(t):
            t = f32(t)
            self._keep.append(t)
            return t.data_ptr()

        def pack(*names):
            pm = PackedMatrix([sd[n] for n in names], dev, tensor_scale)
            self._keep.append(pm)
            return pm

        def sliced(name, width):
            sm = SlicedMatrix(sd[name], width, dev, tensor_scale)
            self._keep.append(sm)
            return sm.struct()

        H, dk, dv = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v
        n_gdn = n_swa = 0
        gdn_offs = swa_offs = None
        for i, kind in enumerate(kinds):
            p = f"self_layers.{i}."
            L = m.self_layers[i]
            L.norm1, L.norm2 = keep(sd[p + "norm1.weight"]), keep(sd[p + "norm2.weight"])
            if kind == "gdn":
                L.kind, L.slot = CB_LAYER_GDN, n_gdn
                n_gdn += 1
                ab = sd[p + "mixer.ab.weight"]
                # a = first H rows, b = next H rows (ab(x).chunk(2), layers.py:161): separate 16-row segments
                pm = PackedMatrix([sd[p + "mixer.qkv.weight"], sd[p + "mixer.gate.weight"], ab[:H], ab[H:]], dev,
                                  tensor_scale)
                self._keep.append(pm)
                gdn_offs = pm.offsets
                L.in_proj = pm.struct()
                L.o_proj = pack(p + "mixer.o_proj.weight").struct()
                if dv % 16 == 0:
                    L.o_proj_ks = sliced(p + "mixer.o_proj.weight", dv // 8)
                L.conv_w = keep(sd[p + "mixer.conv.weight"])
                L.A_log = keep(sd[p + "mixer.A_log"])
                L.dt_bias = keep(sd[p + "mixer.dt_bias"])
                L.o_norm = keep(sd[p + "mixer.o_norm.weight"])
            else:
                L.kind, L.slot = CB_LAYER_SWA, n_swa
                n_swa += 1
                pm = pack(p + "mixer.q_proj.weight", p + "mixer.kv_proj.weight", p + "mixer.gate.weight")
                swa_offs = pm.offsets
                L.in_proj = pm.struct()
                L.o_proj = pack(p + "mixer.o_proj.weight").struct()
                L.q_norm = keep(sd[p + "mixer.q_norm.weight"])
                L.k_norm = keep(sd[p + "mixer.k_norm.weight"])
            L.gate_up = pack(p + "ffn.gate_up.weight").struct()
            L.down = pack(p + "ffn.down.weight").struct()
            L.down_ks = sliced(p + "ffn.down.weight", 16)
        if gdn_offs is not None:
            m.gdn_off_gate, m.gdn_off_a, m.gdn_off_b = gdn_offs[1], gdn_offs[2], gdn_offs[3]
        if swa_offs is not None:
            m.swa_off_kv, m.swa_off_gate = swa_offs[1], swa_offs[2]
        self.n_gdn, self.n_swa = n_gdn, n_swa

        names = ["shared.kv_proj.weight"]
        if cfg.sparse_topk is not None:
            names += ["shared.idx_k.weight", "shared.idx_q.weight", "shared.idx_w.weight"]
        pm = pack(*names)
        m.shared_proj = pm.struct()
        if cfg.sparse_topk is not None:
            m.sh_off_ik, m.sh_off_iq, m.sh_off_iw = pm.offsets[1], pm.offsets[2], pm.offsets[3]
        m.shared_norm = keep(sd["shared.norm.weight"])
        m.shared_k_norm = keep(sd["shared.k_norm.weight"])
        for j in range(cfg.n_cross_layers):
            p = f"cross_layers.{j}."
            L = m.cross_layers[j]
            L.norm1, L.norm2 = keep(sd[p + "norm1.weight"]), keep(sd[p + "norm2.weight"])
            pm = pack(p + "mixer.q_proj.weight", p + "mixer.gate.weight")
            m.cr_off_gate = pm.offsets[1]
            L.q_gate = pm.struct()
            L.o_proj = pack(p + "mixer.o_proj.weight").struct()
            L.gate_up = pack(p + "ffn.gate_up.weight").struct()
            L.down = pack(p + "ffn.down.weight").struct()
            L.down_ks = sliced(p + "ffn.down.weight", 16)
            L.q_norm = keep(sd[p + "mixer.q_norm.weight"])
        m.final_norm = keep(sd["final_norm.weight"])
        self.lm_head = pack("lm_head.weight")
        m.lm_head = self.lm_head.struct()
        self.desc = m
        # the first MTP module and the FR-Spec draft head (the embedding rows of draft_ids)
        self.mtp = None
        if getattr(cfg, "n_mtp_heads", 0) > 0 and "mtp.0.proj.weight" in sd:
            ids = sd.get("draft_ids", torch.arange(min(cfg.mtp_draft_vocab, cfg.vocab_size)))
            ids = ids.detach().to(torch.int64).cpu()
            t = CbMtp()
            t.norm_h, t.norm_e = keep(sd["mtp.0.norm_h.weight"]), keep(sd["mtp.0.norm_e.weight"])
            t.ffn_norm = keep(sd["mtp.0.ffn_norm.weight"])
            t.proj = pack("mtp.0.proj.weight").struct()
            t.gate_up = pack("mtp.0.ffn.gate_up.weight").struct()
            t.down = pack("mtp.0.ffn.down.weight").struct()
            head = PackedMatrix([sd["lm_head.weight"].detach().float()[ids]], dev, tensor_scale)
            self._keep.append(head)
            t.draft_head = head.struct()
            self.draft_ids = ids.to(device=dev, dtype=torch.int32)
            t.draft_ids, t.n_draft = self.draft_ids.data_ptr(), int(ids.numel())
            self.mtp = t
        packed = [x for x in self._keep if isinstance(x, PackedMatrix)]
        if self.mtp is not None:  # the decode step streams every weight but the MTP module and its draft head
            mtp_ptrs = {self.mtp.proj.tiles, self.mtp.gate_up.tiles, self.mtp.down.tiles, self.mtp.draft_head.tiles}
            packed = [x for x in packed if x.tiles.data_ptr() not in mtp_ptrs]
        self.weight_bytes = sum(x.tiles.numel() for x in packed)
        self.weight_real_bytes = sum(x.real_bytes for x in packed)
        torch.cuda.synchronize(dev)


class DeviceCache:
    """Decode state of ``batch`` sequences on the device (the reference ``Cache``,
    ``model.py:41-51``).

    ``clone()`` copies the recurrent state (GDN S and conv windows) and the
    positions, and shares the append-only K/V storage: rows at positions
    >= pos are scratch, so restoring a snapshot after a discarded verify
    forward (``generate.py:71-77``) is exact.  A clone and its source must not
    both be advanced past the fork point.
    """

    def __init__(self, model: DeviceModel, batch: int, max_ctx: int, _share: "DeviceCache | None" = None):
        cfg, dev = model.cfg, model.device
        self.model, self.batch, self.max_ctx = model, batch, max_ctx
        # window + CB_PREFILL_CHUNK slots: a prompt chunk appends all its keys before its attention
        self.swa_slots = cfg.swa_window + max(CB_SWA_EXTRA, CB_PREFILL_CHUNK)
        H, dk, dv, KC = cfg.gdn_heads, cfg.gdn_head_dim_k, cfg.gdn_head_dim_v, cfg.gdn_conv_size
        C_ = 2 * H * dk + H * dv
        if _share is None:
            self.pos_dev = torch.zeros(batch, dtype=torch.int32, device=dev)
            self.gdn_state = torch.zeros(batch, max(model.n_gdn, 1), H, dk, dv, dtype=torch.float32, device=dev)
            self.gdn_conv = torch.zeros(batch, max(model.n_gdn, 1), KC - 1, C_, dtype=torch.float32, device=dev)
            kvh, hd = cfg.n_kv_heads, cfg.head_dim
            self.swa_k = torch.zeros(batch, max(model.n_swa, 1), self.swa_slots, kvh, hd, dtype=torch.bfloat16,
                                     device=dev)
            self.swa_v = torch.zeros_like(self.swa_k)
            self.kv_k = torch.zeros(batch, max_ctx, kvh, hd, dtype=torch.bfloat16, device=dev)
            self.kv_v = torch.zeros_like(self.kv_k)
            self.kv_ik = torch.zeros(batch, max_ctx, max(cfg.indexer_dim, 1), dtype=torch.uint8, device=dev)
            self.pos_host = [0] * batch
        else:
            self.pos_dev = _share.pos_dev.clone()
            self.gdn_state = _share.gdn_state.clone()
            self.gdn_conv = _share.gdn_conv.clone()
            self.swa_k, self.swa_v = _share.swa_k, _share.swa_v
            self.kv_k, self.kv_v, self.kv_ik = _share.kv_k, _share.kv_v, _share.kv_ik
            self.pos_host = list(_share.pos_host)
        self.snap_state = self.snap_conv = None
        self._struct = None

    def enable_snapshots(self, tokens: int) -> None:
        """Allocate per-token GDN snapshots for verify forwards of up to ``tokens``
        tokens (``CbCache.snap_state`` / ``snap_conv``): a forward then also
        records the recurrent state after each of its first ``tokens - 1`` tokens."""
        if tokens > CB_MAX_T:
            raise ValueError(f"a verify forward takes at most {CB_MAX_T} tokens")
        n = max(tokens - 1, 1)
        self.snap_state = torch.zeros((n,) + tuple(self.gdn_state.shape), dtype=torch.float32,
                                      device=self.gdn_state.device)
        self.snap_conv = torch.zeros((n,) + tuple(self.gdn_conv.shape), dtype=torch.float32,
                                     device=self.gdn_conv.device)
        self._struct = None

    @property
    def pos(self) -> int:
        """Tokens in the cache (the reference's ``Cache.pos``; sequence 0 when batched)."""
        return self.pos_host[0]

    def clone(self) -> "DeviceCache":
        return DeviceCache(self.model, self.batch, self.max_ctx, _share=self)

    def struct(self) -> CbCache:
        if self._struct is None:
            s = CbCache()
            s.batch, s.max_ctx, s.swa_slots = self.batch, self.max_ctx, self.swa_slots
            s.n_gdn, s.n_swa = max(self.model.n_gdn, 1), max(self.model.n_swa, 1)
            s.pos, s.gdn_state, s.gdn_conv = (self.pos_dev.data_ptr(), self.gdn_state.data_ptr(),
                                              self.gdn_conv.data_ptr())
            s.swa_k, s.swa_v = self.swa_k.data_ptr(), self.swa_v.data_ptr()
            s.kv_k, s.kv_v, s.kv_ik = self.kv_k.data_ptr(), self.kv_v.data_ptr(), self.kv_ik.data_ptr()
            if self.snap_state is not None:
                s.snap_state, s.snap_conv = self.snap_state.data_ptr(), self.snap_conv.data_ptr()
            self._struct = s
        return self._struct

    # ------------------------------------------------ reference-format view
    def to_reference(self, b: int = 0) -> dict:
        """The reference ``Cache`` contents of sequence ``b`` as CPU float32 tensors:
        ``{"layers": [...], "shared": {"k", "v", "ik"}, "pos": int}``."""
        cfg = self.model.cfg
        pos = self.pos_host[b]
        layers, gi, si = [], 0, 0
        for kind in cfg.self_layer_kinds:
            if kind == "gdn":
                layers.append({"conv": self.gdn_conv[b, gi].float().cpu()[None],
                               "S": self.gdn_state[b, gi].float().cpu()[None]})
                gi += 1
            else:
                n = min(pos, cfg.swa_window)
                slots = [(p % self.swa_slots) for p in range(pos - n, pos)]
                idx = torch.tensor(slots, dtype=torch.long, device=self.swa_k.device)
                layers.append({"k": self.swa_k[b, si].index_select(0, idx).float().cpu()[None],
                               "v": self.swa_v[b, si].index_select(0, idx).float().cpu()[None]})
                si += 1
        shared = {"k": self.kv_k[b, :pos].float().cpu()[None], "v": self.kv_v[b, :pos].float().cpu()[None]}
        if cfg.sparse_topk is not None:
            raw = self.kv_ik[b, :pos].contiguous().cpu()
            shared["ik"] = raw.view(torch.float8_e4m3fn).float()[None]
        return {"layers": layers, "shared": shared, "pos": pos}


@dataclass
class Output:
    """``model.py:54-59``."""
    logits: torch.Tensor | None
    hidden: torch.Tensor
    cache: DeviceCache | None = None
    loss: torch.Tensor | None = None
    metrics: dict = field(default_factory=dict)


class CirrusB200:
    """Inference drop-in for ``CirrusModel`` on one B200.

    ``CirrusB200(cfg, state_dict)`` takes a reference ``state_dict`` (float
    weights; the reference key names) and quantises every Linear to NVFP4.
    ``path="auto"`` runs a chunk of up to 8 rows (batch * tokens) as one
    persistent launch and larger chunks as one launch per op; ``path="multi"``
    always uses one launch per op.
    """

    def __init__(self, cfg, state_dict: dict, device="cuda", max_ctx: int | None = None, tensor_scale: float = 1.0,
                 path: str = "auto"):
        if not torch.cuda.is_available():
            raise _lib.CbError("CirrusB200 needs a CUDA device (there is no CPU path)")
        _lib.lib()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_ctx = max_ctx or cfg.max_seq_len
        with torch.cuda.device(self.device):
            self.model = DeviceModel(cfg, state_dict, self.device, tensor_scale, path)
        self.draft_ids = state_dict.get("draft_ids", torch.arange(min(cfg.mtp_draft_vocab, cfg.vocab_size)))
        self._ws: dict = {}

    # ----------------------------------------------------------- helpers
    def new_cache(self, batch: int = 1, max_ctx: int | None = None) -> DeviceCache:
        return DeviceCache(self.model, batch, max_ctx or self.max_ctx)

    def workspace(self, batch: int, T: int, max_ctx: int) -> torch.Tensor:
        Tc = min(T, CB_PREFILL_CHUNK)  # cb_forward runs longer inputs in chunks of at most this many tokens
        key = (batch, Tc, max_ctx)
        ws = self._ws.get(key)
        if ws is None:
            nbytes = _lib.lib().cb_workspace_bytes(C.byref(self.model.desc), batch, Tc, max_ctx)
            if nbytes == 0:
                raise _lib.CbError("cb_workspace_bytes failed")
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._ws[key] = ws
        return ws

    def launch(self, cache: DeviceCache, ids_dev: torch.Tensor, T: int, n_logits: int, logits, hidden, argmax,
               stream: int | None = None) -> None:
        """Enqueue one ``cb_forward`` (no synchronisation; capturable)."""
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        st = stream if stream is not None else _stream_ptr(self.device)
        rc = _lib.lib().cb_forward(C.byref(self.model.desc), C.byref(cache.struct()), ws.data_ptr(), ws.numel(),
                                   ids_dev.data_ptr(), T, n_logits, _lib.ptr(logits), _lib.ptr(hidden),
                                   _lib.ptr(argmax), st)
        _lib.check(rc, "cb_forward")

    def intermediates(self, cache: DeviceCache, T: int = 1) -> dict:
        """Views into the workspace of the last forward on this cache's shape
        (``cb_workspace_layout``): ``proj`` float32 [batch*Tc, ld] (the shared
        projection: k | v | idx_k | idx_q | idx_w), ``sel_idx`` int32 [rows, k+1]
        and ``sel_cnt`` int32 [rows] (the keys each query row selected)."""
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        lay = _lib.CbWorkspaceLayout()
        _lib.check(_lib.lib().cb_workspace_layout(C.byref(self.model.desc), cache.batch, T, cache.max_ctx,
                                                  C.byref(lay)), "cb_workspace_layout")
        rows = lay.rows

        def view(off, n, dtype):
            return ws[off:off + 4 * n].view(dtype)

        return {"proj": view(lay.proj, rows * lay.ld_proj, torch.float32).view(rows, lay.ld_proj),
                "sel_idx": view(lay.sel_idx, rows * lay.sel_ld, torch.int32).view(rows, lay.sel_ld),
                "sel_cnt": view(lay.sel_cnt, rows, torch.int32)}

    def set_wait_limit(self, cache: DeviceCache, limit_ns: int, stall_barrier: int = 0, T: int = 1) -> None:
        """Bounded-wait limit of the persistent kernel on this cache's workspace
        (``cb_set_wait_limit``; 0 = the default 200 ms).  ``stall_barrier`` > 0
        makes one barrier of every later launch incomplete (fault injection for tests)."""
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        _lib.check(_lib.lib().cb_set_wait_limit(ws.data_ptr(), int(limit_ns), int(stall_barrier),
                                                _stream_ptr(self.device)), "cb_set_wait_limit")

    def clear_status(self, cache: DeviceCache, T: int = 1) -> None:
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        _lib.check(_lib.lib().cb_clear_status(ws.data_ptr(), _stream_ptr(self.device)), "cb_clear_status")

    def read_status(self, cache: DeviceCache, T: int = 1) -> int:
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        out = _lib.I32(0)
        _lib.check(_lib.lib().cb_read_status(ws.data_ptr(), C.byref(out), _stream_ptr(self.device)), "status")
        return int(out.value)

    def phase_trace(self, cache: DeviceCache, T: int = 1) -> list:
        """Per-phase timing of the last persistent launch on this cache's workspace:
        a list of (phase index, CTA-0 work us, barrier wait us) from %globaltimer stamps."""
        ws = self.workspace(cache.batch, T, cache.max_ctx)
        buf = (C.c_uint64 * 512)()
        n = _lib.lib().cb_read_trace(C.byref(self.model.desc), cache.batch, min(T, CB_MAX_T), cache.max_ctx,
                                     ws.data_ptr(), buf, 512, _stream_ptr(self.device))
        if n < 0:
            raise _lib.CbError("cb_read_trace failed")
        vals = list(buf[:n])
        out, prev = [], vals[0]
        for i in range(1, n // 2):
            arrive, leave = vals[2 * i - 1], vals[2 * i]
            if arrive == 0 or leave < arrive or arrive < prev:
                break
            out.append((i, (arrive - prev) / 1e3, (leave - arrive) / 1e3))
            prev = leave
        return out

    # ----------------------------------------------------------- MTP draft
    @torch.no_grad()
    def mtp_draft(self, h_last: torch.Tensor, token, n: int | None = None) -> list:
        """``CirrusModel.mtp_draft`` (``model.py:230-245``): ``n`` (default
        ``cfg.mtp_passes``) draft tokens after ``token`` from the first MTP module
        and the FR-Spec draft head, computed on the device (``cb_mtp_draft``).
        ``h_last``: [1, d] hidden that predicted ``token`` (``Output.hidden[:, -1]``)."""
        t = self.model.mtp
        if t is None:
            return []
        n = self.cfg.mtp_passes if n is None else int(n)
        L = _lib.lib()
        dev = self.device
        with torch.cuda.device(dev):
            h = h_last.detach().to(device=dev, dtype=torch.float32).reshape(-1).contiguous()
            if h.numel() != self.cfg.d_model:
                raise ValueError("h_last must hold one d_model vector")
            tok = torch.as_tensor(token).reshape(-1)[:1].to(device=dev, dtype=torch.int32)
            out = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
            if getattr(self, "_mtp_ws", None) is None:
                nbytes = L.cb_mtp_workspace_bytes(C.byref(self.model.desc), C.byref(t))
                self._mtp_ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            _lib.check(L.cb_mtp_draft(C.byref(self.model.desc), C.byref(t), h.data_ptr(), tok.data_ptr(), n,
                                      out.data_ptr(), self._mtp_ws.data_ptr(), self._mtp_ws.numel(),
                                      _stream_ptr(dev)), "cb_mtp_draft")
            return out[:n].tolist()

    # ----------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, cache: DeviceCache | None = None, use_cache: bool = False,
                labels=None, n_logits: int | None = None, **unused) -> Output:
        """``CirrusModel.forward`` for inference (``model.py:99-176``)."""
        if labels is not None:
            raise NotImplementedError("training (labels) is outside the B200 decode path")
        if input_ids.dim() != 2:
            raise ValueError("input_ids must be [B, T]")
        B, T = input_ids.shape
        want_cache = use_cache or cache is not None
        if cache is None:
            cache = self.new_cache(B)
        elif cache.batch != B:
            raise ValueError(f"cache holds {cache.batch} sequences, input has {B}")
        if max(cache.pos_host) + T > cache.max_ctx:
            raise _lib.CbError(f"context full: {max(cache.pos_host)} + {T} > max_ctx {cache.max_ctx}")
        nq = T if n_logits is None else max(1, min(n_logits, T))
        with torch.cuda.device(self.device):
            ids = input_ids.to(self.device, torch.int64, non_blocking=True).contiguous()
            logits = torch.empty(B, nq, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
            hidden = torch.empty(B, nq, self.cfg.d_model, dtype=torch.float32, device=self.device)
            self.launch(cache, ids, T, nq, logits, hidden, None)
        cache.pos_host = [p + T for p in cache.pos_host]
        return Output(logits=logits, hidden=hidden, cache=cache if want_cache else None)

    __call__ = forward

    def eval(self):
        return self


class DecodeGraph:
    """One captured ``cb_forward`` for a fixed (batch, T, n_logits) on one cache:
    ``step(ids)`` copies the ids in, replays the graph and leaves the results in
    ``logits`` / ``hidden`` / ``argmax`` (device tensors)."""

    def __init__(self, engine: CirrusB200, cache: DeviceCache, T: int = 1, n_logits: int = 1,
                 want_logits: bool = True):
        self.engine, self.cache, self.T, self.nq = engine, cache, T, n_logits
        dev = engine.device
        B = cache.batch
        self.ids = torch.zeros(B, T, dtype=torch.int64, device=dev)
        self.logits = (torch.empty(B, n_logits, engine.cfg.vocab_size, dtype=torch.float32, device=dev)
                       if want_logits else None)
        self.hidden = torch.empty(B, n_logits, engine.cfg.d_model, dtype=torch.float32, device=dev)
        self.argmax = torch.zeros(B, n_logits, dtype=torch.int32, device=dev)
        engine.workspace(B, T, cache.max_ctx)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        saved = (cache.pos_dev.clone(), cache.gdn_state.clone(), cache.gdn_conv.clone())
        with torch.cuda.stream(side):
            # warm-up launch (sets kernel attributes), then capture
            engine.launch(cache, self.ids, T, n_logits, self.logits, self.hidden, self.argmax, side.cuda_stream)
            with torch.cuda.graph(self.graph, stream=side):
                engine.launch(cache, self.ids, T, n_logits, self.logits, self.hidden, self.argmax,
                              side.cuda_stream)
        torch.cuda.current_stream(dev).wait_stream(side)
        # undo the warm-up launch's state changes (K/V rows past pos are scratch)
        cache.pos_dev.copy_(saved[0])
        cache.gdn_state.copy_(saved[1])
        cache.gdn_conv.copy_(saved[2])
        torch.cuda.synchronize(dev)

    def replay(self) -> None:
        self.graph.replay()
        self.cache.pos_host = [p + self.T for p in self.cache.pos_host]

    def step(self, ids: torch.Tensor) -> None:
        self.ids.copy_(ids, non_blocking=True)
        self.replay()
