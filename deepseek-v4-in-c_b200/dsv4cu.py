"""Python binding of libdsv4cu.so (the B200 hot-path library) via ctypes.

Two surfaces, mirroring the C ABI:

* ``HostAPI``: the reference engine's own operator entry points (``dsv4_mmq_n``,
  ``fp8_n``, ``dsv4_route``, ``dsv4_topk`` ...) over host numpy arrays, exactly as
  the reference's C host code calls them (include/dsv4_compat.h).
* ``Device``: the native ``dsv4cu_*`` entry points over device memory (torch
  CUDA tensors are used only as device allocations) on a CUDA stream
  (include/dsv4cu.h).

There is no fallback: if the shared library is missing or fails to load, every
entry point raises. Build it with ``make -C deepseek-v4-in-c_b200``.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsv4cu.so")

WF32, WBF16, WFP8, WFP4 = 0, 1, 2, 3


class DSV4CUError(RuntimeError):
    pass


class QMat(C.Structure):
    """DSV4QMat / dsv4cu_qmat (src/00_base/dsv4_weights.h:34-40)."""
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("wdt", C.c_int),
                ("rows", C.c_int), ("cols", C.c_int),
                ("blk_r", C.c_int), ("blk_c", C.c_int)]


class Expert(C.Structure):
    """DSV4ExpertW / dsv4cu_expert: {w1, w3, w2} (src/00_base/dsv4_weights.h:101-104)."""
    _fields_ = [("w1", QMat), ("w3", QMat), ("w2", QMat)]


class TrunkTensor(C.Structure):
    """DSV4TrunkTensor / dsv4cu_trunk_tensor (src/50_loader/dsv4_trunk.h:20-27)."""
    _fields_ = [("slot", C.c_int32), ("dtype", C.c_int32), ("rows", C.c_int32), ("cols", C.c_int32),
                ("wdt", C.c_int32), ("blk_r", C.c_int32), ("blk_c", C.c_int32),
                ("off", C.c_int64), ("nbytes", C.c_int64)]


_lib = None


def lib() -> C.CDLL:
    """Load libdsv4cu.so once; raise if it is absent (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise DSV4CUError(f"{LIB_PATH} is missing; build with make -C {HERE}")
        # RTLD_LOCAL: the library exports the reference's own symbol names
        # (dsv4_mmq_n, ...); loaded globally they would take the place of the
        # reference's kernels inside any reference library loaded afterwards.
        L = C.CDLL(LIB_PATH, mode=C.RTLD_LOCAL)
        vp, i, f, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
        sig = {
            "dsv4cu_last_error": (C.c_char_p, []),
            "dsv4cu_ctx_create": (i, [C.POINTER(vp), i]),
            "dsv4cu_ctx_destroy": (None, [vp]),
            "dsv4cu_ctx_reserve": (i, [vp, sz]),
            "dsv4cu_ctx_workspace_bytes": (sz, [vp]),
            "dsv4cu_ctx_status": (i, [vp, vp, C.POINTER(i)]),
            "dsv4cu_ctx_inject": (i, [vp, i]),
            "dsv4cu_mmq_workspace": (sz, [vp, i]),
            "dsv4cu_mmq": (i, [vp, vp, vp, vp, i, vp]),
            "dsv4cu_gemm_bf16w": (i, [vp, vp, vp, vp, i, i, vp]),
            "dsv4cu_gemm_bf16w_workspace": (sz, [vp, i, i]),
            "dsv4cu_gemv_workspace": (sz, [vp, i]),
            "dsv4cu_gemv": (i, [vp, vp, vp, vp, i, vp]),
            "dsv4cu_gemv_ev": (i, [vp, vp, vp, vp, i, vp, vp]),
            "dsv4cu_route": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, i, f, i, vp]),
            "dsv4cu_swiglu": (i, [vp, vp, vp, i, f, vp]),
            "dsv4cu_moe_create": (i, [C.POINTER(vp), vp, i, vp, i, i]),
            "dsv4cu_moe_destroy": (None, [vp]),
            "dsv4cu_moe_set_path": (i, [vp, i]),
            "dsv4cu_moe_workspace": (sz, [vp, i, i]),
            "dsv4cu_moe_decode": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, f, f, i, vp, vp, vp]),
            "dsv4cu_moe_prefill_workspace": (sz, [vp, i, i, i]),
            "dsv4cu_moe_prefill": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, f, f, i, i, vp, vp, vp]),
            "dsv4cu_moe_prefill_ev": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, f, f, i, i, vp, vp, vp, vp]),
            "dsv4cu_moe_decode_ev": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, f, f, i, vp, vp, vp, vp]),
            "dsv4cu_moe_decode_host": (i, [vp, vp, vp, vp, vp, i, f, f, i, vp]),
            "dsv4cu_moe_rows_workspace": (sz, [vp, i]),
            "dsv4cu_moe_rows": (i, [vp, vp, vp, vp, C.c_long, vp, i, f, vp]),
            "dsv4cu_ep_pack": (i, [vp, vp, vp, vp, vp, vp, i, i, i, i, i, vp]),
            "dsv4cu_ep_tail": (i, [vp, i, vp, i, i, i, vp, vp]),
            "dsv4cu_ep_combine": (i, [vp, vp, vp, vp, vp, i, i, i, vp]),
            "dsv4cu_ep_create": (i, [C.POINTER(vp), i, i, i, i, i, i]),
            "dsv4cu_ep_handle": (i, [vp, vp]),
            "dsv4cu_ep_connect": (i, [vp, vp]),
            "dsv4cu_ep_workspace": (sz, [vp, vp, i]),
            "dsv4cu_ep_forward": (i, [vp, vp, vp, vp, vp, vp, i, f, f, vp, vp, vp, vp]),
            "dsv4cu_ep_destroy": (None, [vp]),
            "dsv4cu_attn_create": (i, [C.POINTER(vp), vp, vp]),
            "dsv4cu_attn_destroy": (None, [vp]),
            "dsv4cu_attn_step": (i, [vp, vp, vp, vp, i, vp]),
            "dsv4cu_attn_block": (i, [vp, vp, vp, i, vp]),
            "dsv4cu_attn_n_compressed": (i, [vp]),
            "dsv4cu_attn_fill_context": (i, [vp, i, C.c_ulonglong, vp]),
            "dsv4cu_ffn_create": (i, [C.POINTER(vp), vp]),
            "dsv4cu_ffn_destroy": (None, [vp]),
            "dsv4cu_ffn_block": (i, [vp, vp, vp, i, vp, vp]),
            "dsv4cu_layer_step": (i, [vp, vp, vp, vp, i, i, vp]),
            "dsv4cu_mat_create": (i, [C.POINTER(vp), vp, vp]),
            "dsv4cu_mat_destroy": (None, [vp]),
            "dsv4cu_mat_workspace": (sz, [vp, i, i]),
            "dsv4cu_mat_gemm": (i, [vp, vp, vp, vp, i, i, vp]),
            "dsv4cu_mat_gemm_cfg": (i, [vp, vp, vp, vp, i, i, i, i, vp]),
            "dsv4cu_mat_gemm_ev": (i, [vp, vp, vp, vp, i, i, vp, vp]),
            "dsv4cu_indexer_score": (i, [vp, vp, vp, vp, i, i, i, vp]),
            "dsv4cu_indexer_score_fp8": (i, [vp, vp, vp, vp, vp, vp, i, i, i, i, vp]),
            "dsv4cu_indexer_set_path": (i, [i]),
            "dsv4cu_sparse_attn_set_path": (i, [i]),
            "dsv4cu_gemm_bf16w_set_path": (i, [i]),
            "dsv4cu_topk": (i, [vp, vp, vp, i, i, vp]),
            "dsv4cu_sparse_attn": (i, [vp, vp, vp, vp, i, vp, vp, i, i, i, f, vp]),
            "dsv4cu_indexer_offset": (i, [vp, i, i, vp]),
            "dsv4cu_argmax": (i, [vp, vp, i, i, vp]),
            "dsv4cu_rmsnorm": (i, [vp, vp, vp, i, i, f, vp]),
            "dsv4cu_hc_post": (i, [vp, vp, vp, vp, vp, i, i, i, vp]),
            "dsv4cu_hc_pre": (i, [vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, i, f, f, vp]),
            "dsv4cu_hc_head": (i, [vp, vp, vp, vp, vp, i, i, i, f, f, vp]),
            "dsv4cu_compress_step": (i, [vp, vp, vp, vp, vp, vp, i, i, i, vp]),
            "dsv4cu_rope_apply": (i, [vp, vp, i, i, i, i, vp, vp, vp, i, i, i, vp]),
            "dsv4cu_experts_load": (i, [C.POINTER(vp), vp, C.c_char_p, C.c_char_p, i, i, i, i, i, vp]),
            "dsv4cu_experts_free": (None, [vp]),
            "dsv4cu_experts_index": (i, [C.c_char_p, C.POINTER(i), C.POINTER(i), i, i, C.POINTER(C.c_int64)]),
            "dsv4cu_trunk_manifest": (i, [C.c_char_p, C.POINTER(i), i, C.POINTER(C.c_int64), C.POINTER(i),
                                          C.POINTER(TrunkTensor), i]),
            "dsv4cu_trunk_load": (i, [C.POINTER(vp), C.c_char_p, i, i, vp]),
            "dsv4cu_trunk_slot": (i, [vp, i, i, C.POINTER(TrunkTensor), C.POINTER(vp)]),
            "dsv4cu_trunk_qmat": (i, [vp, i, i, C.POINTER(QMat)]),
            "dsv4cu_trunk_widen": (i, [vp, i, i, vp, vp]),
            "dsv4cu_trunk_resident_bytes": (C.c_int64, [vp]),
            "dsv4cu_trunk_free": (None, [vp]),
            "dsv4cu_head": (i, [vp, vp, vp, vp, vp, i, vp]),
            "dsv4cu_quantize_fp8": (i, [vp, vp, vp, i, i, vp]),
            "dsv4cu_quantize_fp4": (i, [vp, vp, vp, i, i, vp]),
            "dsv4cu_fill_normal": (i, [vp, sz, C.c_uint64, f, f, vp]),
            "dsv4cu_round_bf16": (i, [vp, sz, vp]),
            # host-pointer reference ABI
            "dsv4_mmq_n": (None, [vp, vp, vp, i]),
            "dsv4_mmq": (None, [vp, vp, vp]),
            "bf16_n": (None, [vp, vp, vp, i, i, i]),
            "fp8_n": (None, [vp, vp, vp, vp, i, i, i, i, i]),
            "fp4_n": (None, [vp, vp, vp, vp, i, i, i, i, i]),
            "dsv4_swiglu": (None, [vp, vp, vp, i, f]),
            "dsv4_rmsnorm": (None, [vp, vp, vp, i, f]),
            "dsv4_route": (None, [vp, vp, vp, vp, vp, vp, i, i, i, f]),
            "dsv4_expert_forward": (None, [vp, vp, vp, vp, vp, vp, i, f]),
            "dsv4_sparse_attn": (None, [vp, vp, vp, vp, vp, i, i, i, f, vp]),
            "dsv4_window_idxs": (i, [vp, i, i]),
            "dsv4_indexer_score": (None, [vp, vp, vp, vp, i, i, i]),
            "dsv4_topk": (i, [vp, vp, i, i]),
            "dsv4_indexer_offset": (None, [vp, i, i]),
            "dsv4_prefill_vk_init": (i, [C.POINTER(vp), vp, vp, vp]),
            "dsv4_prefill_vk_free": (None, [vp]),
            "dsv4_prefill_vk_gemm": (i, [vp, vp, vp, vp, i]),
            "dsv4_prefill_vk_expert_fused": (i, [vp, vp, vp, vp, vp, vp, i, i, f, vp, vp]),
            "dsv4cu_host_forget": (None, [vp]),
            "dsv4cu_host_forget_all": (None, []),
            "dsv4cu_host_verify": (None, [i]),
            "dsv4cu_host_registry_count": (sz, []),
            "dsv4cu_host_registry_bytes": (sz, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().dsv4cu_last_error().decode(errors="replace")


def check(rc: int, what: str = "dsv4cu") -> None:
    if rc != 0:
        raise DSV4CUError(f"{what}: status {rc}: {last_error()}")


def _event_handles(events):
    """cudaEvent_t handles of torch.cuda.Event objects; torch creates the
    driver event on first record, so an unrecorded event is recorded once
    on the current stream first."""
    for e in events:
        if not e.cuda_event:
            e.record()
    return (C.c_void_p * len(events))(*[e.cuda_event for e in events])


def _p(a):
    """Host pointer of a numpy array (or None)."""
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------------ host ABI
class HostAPI:
    """The reference's operator entry points over host arrays."""

    def __init__(self):
        self.L = lib()

    def mmq(self, x: np.ndarray, m: QMat) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, m.rows), np.float32)
        self.L.dsv4_mmq_n(_p(y), _p(x), C.byref(m), nt)
        return y

    def fp8_n(self, x, W, S, rows, cols, blk_r, blk_c):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, rows), np.float32)
        self.L.fp8_n(_p(y), _p(x), _p(W), _p(S), cols, rows, blk_r, blk_c, nt)
        return y

    def fp4_n(self, x, W, S, rows, cols, blk_r, blk_c):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, rows), np.float32)
        self.L.fp4_n(_p(y), _p(x), _p(W), _p(S), cols, rows, blk_r, blk_c, nt)
        return y

    def bf16_n(self, x, W, rows, cols):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, rows), np.float32)
        self.L.bf16_n(_p(y), _p(x), _p(W), cols, rows, nt)
        return y

    def route(self, logits, topk, route_scale, bias=None, tid2eid=None, token_id=0):
        ne = logits.shape[0]
        scores = np.ascontiguousarray(logits, np.float32).copy()
        orig = np.zeros(ne, np.float32)
        idx = np.zeros(topk, np.int32)
        wts = np.zeros(topk, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        t = None if tid2eid is None else np.ascontiguousarray(tid2eid, np.int64)
        self.L.dsv4_route(_p(idx), _p(wts), _p(scores), _p(orig), _p(b), _p(t), token_id, ne,
                          topk, route_scale)
        return idx, wts, scores, orig

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        self.L.dsv4_rmsnorm(_p(y), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return y

    def swiglu(self, gate, up, limit):
        g = np.ascontiguousarray(gate, np.float32)
        u = np.ascontiguousarray(up, np.float32)
        y = np.zeros_like(g)
        self.L.dsv4_swiglu(_p(y), _p(g), _p(u), g.size, limit)
        return y

    def expert_forward(self, x, w3: list, inter, limit):
        e = Expert(*w3)
        out = np.zeros(w3[2].rows, np.float32)
        scr = np.zeros(3 * inter, np.float32)
        self.L.dsv4_expert_forward(_p(out), _p(np.ascontiguousarray(x, np.float32)), C.addressof(e),
                                   _p(scr), _p(scr[inter:]), _p(scr[2 * inter:]), inter, limit)
        return out, scr[:inter].copy(), scr[inter:2 * inter].copy(), scr[2 * inter:].copy()

    def indexer_score(self, q, kv, weights):
        h, d = q.shape
        n = kv.shape[0]
        out = np.zeros(n, np.float32)
        self.L.dsv4_indexer_score(_p(out), _p(np.ascontiguousarray(q, np.float32)),
                                  _p(np.ascontiguousarray(kv, np.float32)),
                                  _p(np.ascontiguousarray(weights, np.float32)), h, d, n)
        return out

    def topk(self, scores, k):
        s = np.ascontiguousarray(scores, np.float32)
        out = np.full(max(1, min(k, s.size)), -7, np.int32)
        r = self.L.dsv4_topk(_p(out), _p(s), s.size, k)
        return out[:max(r, 0)], r

    def indexer_offset(self, idxs, offset):
        a = np.ascontiguousarray(idxs, np.int32).copy()
        self.L.dsv4_indexer_offset(_p(a), a.size, offset)
        return a

    def window_idxs(self, pos, win):
        out = np.zeros(max(win, 1), np.int32)
        n = self.L.dsv4_window_idxs(_p(out), pos, win)
        return out[:win], n

    def sparse_attn(self, q, kv, sink, idxs, scale):
        h, d = q.shape
        o = np.zeros((h, d), np.float32)
        scr = np.zeros(h * max(1, len(idxs)), np.float32)
        self.L.dsv4_sparse_attn(_p(o), _p(np.ascontiguousarray(q, np.float32)),
                                _p(np.ascontiguousarray(kv, np.float32)),
                                _p(np.ascontiguousarray(sink, np.float32)),
                                _p(np.ascontiguousarray(idxs, np.int32)), h, d, len(idxs), scale,
                                _p(scr))
        return o

    def forget_all(self):
        self.L.dsv4cu_host_forget_all()

    def forget(self, host_ptr: int):
        self.L.dsv4cu_host_forget(host_ptr)

    def verify(self, full: bool):
        """Exact (every byte per call) or sampled content check of mirrored weights."""
        self.L.dsv4cu_host_verify(1 if full else 0)


# ---------------------------------------------------------------- device ABI
class AttnCfg(C.Structure):
    """dsv4cu_attn_cfg (include/dsv4cu.h)."""
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_heads", "head_dim", "q_lora", "o_lora", "o_groups", "qk_rope",
                                       "sliding_window", "index_n_heads", "index_head_dim", "index_topk", "hc_mult",
                                       "hc_sinkhorn_iters")] + \
               [("rms_eps", C.c_float), ("hc_eps", C.c_float), ("compress_ratio", C.c_int), ("max_pos", C.c_int)]


class AttnWeights(C.Structure):
    """dsv4cu_attn_weights (include/dsv4cu.h): device pointers."""
    _fields_ = [(n, QMat) for n in ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "comp_wkv", "comp_wgate", "idx_wq_b",
                                    "idx_wproj")] + \
               [(n, C.c_void_p) for n in ("q_norm", "kv_norm", "sink", "comp_ape", "comp_norm", "attn_norm", "hc_fn",
                                          "hc_base", "hc_scale", "cs", "sn")]


class FfnDesc(C.Structure):
    """dsv4cu_ffn_desc (include/dsv4cu.h): device pointers."""
    _fields_ = [("moe", C.c_void_p), ("gate", QMat), ("bias", C.c_void_p), ("tid2eid", C.c_void_p),
                ("ffn_norm", C.c_void_p), ("hc_fn", C.c_void_p), ("hc_base", C.c_void_p), ("hc_scale", C.c_void_p)] + \
               [(n, C.c_int) for n in ("hidden", "hc_mult", "hc_sinkhorn_iters", "n_experts", "topk", "nt_max")] + \
               [(n, C.c_float) for n in ("rms_eps", "hc_eps", "route_scale", "swiglu_limit")] + \
               [("ep", C.c_void_p)]


class Device:
    """The native dsv4cu_* entry points on one CUDA device."""

    def __init__(self, device: int = 0):
        import torch
        self.torch = torch
        self.L = lib()
        self.device = device
        h = C.c_void_p()
        torch.cuda.set_device(device)
        check(self.L.dsv4cu_ctx_create(C.byref(h), device), "ctx_create")
        self.ctx = h

    def close(self):
        if self.ctx:
            self.L.dsv4cu_ctx_destroy(self.ctx)
            self.ctx = None

    def stream(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    INJECT_WITHHOLD_STAGE = 1

    def inject(self, what: int):
        """Arm a test-only fault for the next dsv4cu_gemv (dsv4cu_ctx_inject)."""
        check(self.L.dsv4cu_ctx_inject(self.ctx, what), "dsv4cu_ctx_inject")

    def status_code(self) -> int:
        """Synchronise and return (and clear) the context's device status word."""
        code = C.c_int(0)
        self.L.dsv4cu_ctx_status(self.ctx, self.stream(), C.byref(code))
        return code.value

    def check_status(self):
        """Raise if a kernel of this context hit a bounded-wait timeout."""
        code = C.c_int(0)
        check(self.L.dsv4cu_ctx_status(self.ctx, self.stream(), C.byref(code)), "device status")

    @staticmethod
    def ptr(t):
        return None if t is None else t.data_ptr()

    def qmat(self, w, s, wdt, rows, cols, blk_r=0, blk_c=0) -> QMat:
        return QMat(self.ptr(w), self.ptr(s), wdt, rows, cols, blk_r, blk_c)

    def mmq(self, y, x, m: QMat, nt: int):
        check(self.L.dsv4cu_mmq(self.ctx, self.ptr(y), self.ptr(x), C.byref(m), nt, self.stream()),
              "dsv4cu_mmq")

    def gemm_bf16w(self, y, x, m: QMat, nt: int, terms: int = 1):
        """Exact-weight GEMM on the bf16 tensor cores (dsv4cu_gemm_bf16w), 1 or 2 bf16 activation terms."""
        check(self.L.dsv4cu_gemm_bf16w(self.ctx, self.ptr(y), self.ptr(x), C.byref(m), nt, terms, self.stream()),
              "dsv4cu_gemm_bf16w")

    def gemv(self, y, x, m: QMat, nt: int, events=None):
        """Decode GEMV (dsv4cu_gemv / dsv4cu_gemv_ev): one or two tokens streamed."""
        if events is None:
            check(self.L.dsv4cu_gemv(self.ctx, self.ptr(y), self.ptr(x), C.byref(m), nt, self.stream()),
                  "dsv4cu_gemv")
        else:
            check(self.L.dsv4cu_gemv_ev(self.ctx, self.ptr(y), self.ptr(x), C.byref(m), nt, self.stream(),
                                        _event_handles(events)), "dsv4cu_gemv_ev")

    def mat_create(self, m: QMat):
        """Prepare a packed matrix for the tensor-core GEMM (dsv4cu_mat_create)."""
        h = C.c_void_p()
        check(self.L.dsv4cu_mat_create(C.byref(h), C.byref(m), self.stream()), "dsv4cu_mat_create")
        return h

    def mat_destroy(self, h):
        self.L.dsv4cu_mat_destroy(h)

    def mat_gemm(self, h, y, x, nt: int, terms: int = 3, nb: int = 0, kb: int = 0, events=None):
        if events is not None:
            evp = _event_handles(events)
            check(self.L.dsv4cu_mat_gemm_ev(self.ctx, h, self.ptr(y), self.ptr(x), nt, terms, self.stream(), evp),
                  "dsv4cu_mat_gemm_ev")
        elif nb or kb:
            check(self.L.dsv4cu_mat_gemm_cfg(self.ctx, h, self.ptr(y), self.ptr(x), nt, terms, nb, kb,
                                             self.stream()), "dsv4cu_mat_gemm_cfg")
        else:
            check(self.L.dsv4cu_mat_gemm(self.ctx, h, self.ptr(y), self.ptr(x), nt, terms, self.stream()),
                  "dsv4cu_mat_gemm")

    def route(self, idx, wts, scores, orig, logits, topk, route_scale, nt, bias=None,
              tid2eid=None, token_ids=None):
        ne = logits.shape[-1]
        check(self.L.dsv4cu_route(self.ptr(idx), self.ptr(wts), self.ptr(scores), self.ptr(orig),
                                  self.ptr(logits), self.ptr(bias), self.ptr(tid2eid),
                                  self.ptr(token_ids), ne, topk, route_scale, nt, self.stream()),
              "dsv4cu_route")

    def experts_load(self, model_dir: str, index_dir: str, layer: int, first: int, count: int, hidden: int,
                     inter: int):
        """Routed experts [first, first + count) of `layer` from a pack into HBM:
        (store handle, list of Expert descriptors)."""
        h = C.c_void_p()
        arr = (Expert * count)()
        check(self.L.dsv4cu_experts_load(C.byref(h), arr, model_dir.encode(), index_dir.encode(), layer, first,
                                         count, hidden, inter, self.stream()), "experts_load")
        return h, list(arr)

    def experts_free(self, h):
        self.L.dsv4cu_experts_free(h)

    def trunk_load(self, pack_dir: str, first: int = 0, count: int = 0):
        """Layers [first, first + count) (count 0: to the last) of trunk.bin into
        HBM (dsv4cu_trunk_load); returns an opaque handle."""
        h = C.c_void_p()
        check(self.L.dsv4cu_trunk_load(C.byref(h), pack_dir.encode(), first, count, self.stream()), "trunk_load")
        return h

    def trunk_slot(self, h, layer: int, slot: int):
        """(record, device address) of a resident tensor (dsv4cu_trunk_slot)."""
        d, p = TrunkTensor(), C.c_void_p()
        check(self.L.dsv4cu_trunk_slot(h, layer, slot, C.byref(d), C.byref(p)), "trunk_slot")
        return d, p.value

    def trunk_qmat(self, h, layer: int, slot: int) -> QMat:
        """Device descriptor of a packed matrix and its scales (dsv4cu_trunk_qmat)."""
        q = QMat()
        check(self.L.dsv4cu_trunk_qmat(h, layer, slot, C.byref(q)), "trunk_qmat")
        return q

    def trunk_widen(self, h, layer: int, slot: int, dst):
        """A vector widened to f32 into the device tensor dst (dsv4cu_trunk_widen)."""
        check(self.L.dsv4cu_trunk_widen(h, layer, slot, self.ptr(dst), self.stream()), "trunk_widen")

    def trunk_resident_bytes(self, h) -> int:
        return int(self.L.dsv4cu_trunk_resident_bytes(h))

    def trunk_free(self, h):
        self.L.dsv4cu_trunk_free(h)

    def moe_create(self, experts: list, shared: Expert | None, hidden: int, inter: int):
        """Prepare a MoE layer (dsv4cu_moe_create); returns an opaque handle."""
        arr = (Expert * len(experts))(*experts)
        h = C.c_void_p()
        check(self.L.dsv4cu_moe_create(C.byref(h), C.addressof(arr), len(experts),
                                       None if shared is None else C.addressof(shared), hidden, inter),
              "dsv4cu_moe_create")
        return h

    MOE_PATH = {"auto": 0, "tensor": 1, "stream": 2}

    def moe_set_path(self, layer, path: str):
        """Decode path of a layer (dsv4cu_moe_set_path): "auto", "tensor" or "stream"."""
        check(self.L.dsv4cu_moe_set_path(layer, self.MOE_PATH[path]), "dsv4cu_moe_set_path")

    def moe_destroy(self, layer):
        self.L.dsv4cu_moe_destroy(layer)

    def moe_prefill(self, layer, out, x, logits, topk, route_scale, limit, nt, terms=3, idx_out=None,
                    wts_out=None, bias=None, tid2eid=None, token_ids=None, events=None):
        args = (self.ctx, layer, self.ptr(out), self.ptr(x), self.ptr(logits), self.ptr(bias), self.ptr(tid2eid),
                self.ptr(token_ids), topk, route_scale, limit, nt, terms, self.ptr(idx_out), self.ptr(wts_out),
                self.stream())
        if events is None:
            check(self.L.dsv4cu_moe_prefill(*args), "dsv4cu_moe_prefill")
        else:
            evp = _event_handles(events)
            check(self.L.dsv4cu_moe_prefill_ev(*args, evp), "dsv4cu_moe_prefill_ev")

    def moe_decode(self, layer, out, x, logits, topk, route_scale, limit, nt, idx_out=None, wts_out=None,
                   bias=None, tid2eid=None, token_ids=None, stream=None, events=None):
        st = self.stream() if stream is None else stream
        args = (self.ctx, layer, self.ptr(out), self.ptr(x), self.ptr(logits), self.ptr(bias),
                self.ptr(tid2eid), self.ptr(token_ids), topk, route_scale, limit, nt, self.ptr(idx_out),
                self.ptr(wts_out), st)
        if events is None:
            check(self.L.dsv4cu_moe_decode(*args), "dsv4cu_moe_decode")
        else:
            evp = _event_handles(events)
            check(self.L.dsv4cu_moe_decode_ev(*args, evp), "dsv4cu_moe_decode_ev")

    def moe_decode_host(self, layer, out, x, logits, topk, route_scale, limit, nt):
        """dsv4cu_moe_decode_host on host tensors / arrays (pinned for asynchronous copies)."""
        hp = (lambda a: a.data_ptr()) if hasattr(x, "data_ptr") else (lambda a: a.ctypes.data)
        check(self.L.dsv4cu_moe_decode_host(self.ctx, layer, hp(out), hp(x), hp(logits), topk, route_scale, limit,
                                            nt, self.stream()), "dsv4cu_moe_decode_host")

    def attn_create(self, cfg: AttnCfg, weights: AttnWeights):
        """One layer's device attention (dsv4cu_attn_create); weights stay referenced."""
        h = C.c_void_p()
        check(self.L.dsv4cu_attn_create(C.byref(h), C.byref(cfg), C.byref(weights)), "dsv4cu_attn_create")
        return h

    def attn_step(self, a, out, x, pos: int):
        check(self.L.dsv4cu_attn_step(self.ctx, a, self.ptr(out), self.ptr(x), pos, self.stream()),
              "dsv4cu_attn_step")

    def attn_block(self, a, h, pos: int):
        check(self.L.dsv4cu_attn_block(self.ctx, a, self.ptr(h), pos, self.stream()), "dsv4cu_attn_block")

    def attn_fill_context(self, a, pos: int, seed: int):
        check(self.L.dsv4cu_attn_fill_context(a, pos, seed, self.stream()), "dsv4cu_attn_fill_context")

    def attn_destroy(self, a):
        self.L.dsv4cu_attn_destroy(a)

    def ffn_create(self, desc: FfnDesc):
        h = C.c_void_p()
        check(self.L.dsv4cu_ffn_create(C.byref(h), C.byref(desc)), "dsv4cu_ffn_create")
        return h

    def ffn_block(self, f, h, nt: int = 1, token_ids=None):
        check(self.L.dsv4cu_ffn_block(self.ctx, f, self.ptr(h), nt, self.ptr(token_ids), self.stream()),
              "dsv4cu_ffn_block")

    def layer_step(self, a, f, h, pos: int, token_id: int = 0):
        check(self.L.dsv4cu_layer_step(self.ctx, a, f, self.ptr(h), pos, token_id, self.stream()),
              "dsv4cu_layer_step")

    def ffn_destroy(self, f):
        self.L.dsv4cu_ffn_destroy(f)

    EP_HANDLE_BYTES = 128

    def ep_create(self, rank: int, world: int, nt_max: int, hidden: int, topk: int, experts_per_rank: int):
        """Rank-local state of the peer-memory expert-parallel step (dsv4cu_ep_create)."""
        h = C.c_void_p()
        check(self.L.dsv4cu_ep_create(C.byref(h), rank, world, nt_max, hidden, topk, experts_per_rank),
              "dsv4cu_ep_create")
        return h

    def ep_handle(self, ep) -> bytes:
        """This rank's exported handle (dsv4cu_ep_handle), to be all-gathered."""
        blob = (C.c_char * self.EP_HANDLE_BYTES)()
        check(self.L.dsv4cu_ep_handle(ep, blob), "dsv4cu_ep_handle")
        return bytes(blob)

    def ep_connect(self, ep, handles: list):
        """Map the peers' buffers from every rank's handle, in rank order (dsv4cu_ep_connect)."""
        joined = b"".join(handles)
        buf = (C.c_char * len(joined)).from_buffer_copy(joined)
        check(self.L.dsv4cu_ep_connect(ep, buf), "dsv4cu_ep_connect")

    def ep_forward(self, ep, layer, out, x, logits, nt, route_scale, limit, idx=None, wts=None, events=None):
        """One expert-parallel layer step (dsv4cu_ep_forward); events: 7 torch.cuda.Event or None."""
        evp = None if events is None else _event_handles(events)
        check(self.L.dsv4cu_ep_forward(self.ctx, ep, layer, self.ptr(out), self.ptr(x), self.ptr(logits), nt,
                                       route_scale, limit, self.ptr(idx), self.ptr(wts), self.stream(), evp),
              "dsv4cu_ep_forward")

    def ep_destroy(self, ep):
        self.L.dsv4cu_ep_destroy(ep)

    def moe_rows(self, layer, y, x, ldx, ids, nrows, limit):
        """y[r] = expert ids[r] (n_experts = the shared expert) on row r of x (dsv4cu_moe_rows)."""
        check(self.L.dsv4cu_moe_rows(self.ctx, layer, self.ptr(y), self.ptr(x), ldx, self.ptr(ids), nrows, limit,
                                     self.stream()), "dsv4cu_moe_rows")

    def ep_pack(self, send, counts, pair_slot, x, idx, nt, topk, hidden, experts_per_rank, n_ranks):
        check(self.L.dsv4cu_ep_pack(self.ctx, self.ptr(send), self.ptr(counts), self.ptr(pair_slot), self.ptr(x),
                                    self.ptr(idx), nt, topk, hidden, experts_per_rank, n_ranks, self.stream()),
              "dsv4cu_ep_pack")

    def ep_tail(self, recv, nrecv, x, nt, hidden, shared_id, ids):
        check(self.L.dsv4cu_ep_tail(self.ptr(recv), nrecv, self.ptr(x), nt, hidden, shared_id, self.ptr(ids),
                                    self.stream()), "dsv4cu_ep_tail")

    def ep_combine(self, out, back, pair_slot, wts, shared, nt, topk, hidden):
        check(self.L.dsv4cu_ep_combine(self.ptr(out), self.ptr(back), self.ptr(pair_slot), self.ptr(wts),
                                       self.ptr(shared), nt, topk, hidden, self.stream()), "dsv4cu_ep_combine")

    def indexer_score(self, out, q, kv, w, n_heads, head_dim, n_pos):
        check(self.L.dsv4cu_indexer_score(self.ptr(out), self.ptr(q), self.ptr(kv), self.ptr(w),
                                          n_heads, head_dim, n_pos, self.stream()),
              "dsv4cu_indexer_score")

    def indexer_score_fp8(self, out, q8, qs, k8, ks, w, n_heads, head_dim, n_pos, k_stride):
        check(self.L.dsv4cu_indexer_score_fp8(self.ptr(out), self.ptr(q8), self.ptr(qs),
                                              self.ptr(k8), self.ptr(ks), self.ptr(w), n_heads,
                                              head_dim, n_pos, k_stride, self.stream()),
              "dsv4cu_indexer_score_fp8")

    INDEXER_PATH = {"auto": 0, "fp64": 1}

    def indexer_set_path(self, path: str):
        """Kernel of the exact FP8 score (dsv4cu_indexer_set_path): "auto" (int8
        tensor-core digits) or "fp64" (FP64 tensor cores)."""
        check(self.L.dsv4cu_indexer_set_path(self.INDEXER_PATH[path]), "dsv4cu_indexer_set_path")

    ATTN_PATH = {"auto": 0, "fp32": 1, "cluster8": 2}

    BF16W_PATH = {"auto": 0, "convert": 1, "predequant": 2}

    def gemm_bf16w_set_path(self, path: str):
        """Where the exact-weight GEMM dequantizes (dsv4cu_gemm_bf16w_set_path):
        "auto", "convert" (converter warps per token tile) or "predequant" (one
        bf16 copy of the matrix per call); the results are the same bits."""
        check(self.L.dsv4cu_gemm_bf16w_set_path(self.BF16W_PATH[path]), "dsv4cu_gemm_bf16w_set_path")

    def sparse_attn_set_path(self, path: str):
        """Chunk kernel of the sparse attention (dsv4cu_sparse_attn_set_path):
        "auto" (bf16 tensor cores where the shape allows), "fp32" or "cluster8"
        (the tensor-core kernel in 8-CTA clusters)."""
        check(self.L.dsv4cu_sparse_attn_set_path(self.ATTN_PATH[path]), "dsv4cu_sparse_attn_set_path")

    def topk(self, idx, scores, n, k):
        check(self.L.dsv4cu_topk(self.ctx, self.ptr(idx), self.ptr(scores), n, k, self.stream()),
              "dsv4cu_topk")

    def rmsnorm(self, y, x, w, n: int, nt: int = 1, eps: float = 1e-6):
        check(self.L.dsv4cu_rmsnorm(self.ptr(y), self.ptr(x), self.ptr(w), n, nt, eps, self.stream()), "rmsnorm")

    def rope_apply(self, v, nt, nh, head_dim, rd, cs, sn, pos, inverse=0):
        """In place on v [nt][nh][head_dim]; cs / sn device [n_pos][table_half]; pos device int32 [nt]."""
        check(self.L.dsv4cu_rope_apply(self.ctx, self.ptr(v), nt, nh, head_dim, rd, self.ptr(cs), self.ptr(sn),
                                       self.ptr(pos), cs.shape[1], cs.shape[0], inverse, self.stream()),
              "rope_apply")

    def hc_pre(self, y, post, comb, mixes, x, fn, base, scale, nt: int, hc: int, hidden: int, iters: int = 20,
               norm_eps: float = 1e-6, hc_eps: float = 1e-6):
        check(self.L.dsv4cu_hc_pre(self.ptr(y), self.ptr(post), self.ptr(comb), self.ptr(mixes), self.ptr(x),
                                   self.ptr(fn), self.ptr(base), self.ptr(scale), nt, hc, hidden, iters, norm_eps,
                                   hc_eps, self.stream()), "hc_pre")

    def hc_head(self, y, x, fn, base, scale, nt: int, hc: int, hidden: int, norm_eps: float = 1e-6,
                hc_eps: float = 1e-6):
        check(self.L.dsv4cu_hc_head(self.ptr(y), self.ptr(x), self.ptr(fn), self.ptr(base), self.ptr(scale), nt, hc,
                                    hidden, norm_eps, hc_eps, self.stream()), "hc_head")

    def compress_step(self, out, kv_in, score_in, ape, kv_state, score_state, pos: int, ratio: int, head_dim: int):
        r = self.L.dsv4cu_compress_step(self.ptr(out), self.ptr(kv_in), self.ptr(score_in), self.ptr(ape),
                                        self.ptr(kv_state), self.ptr(score_state), pos, ratio, head_dim, self.stream())
        if r < 0:
            check(r, "compress_step")
        return r

    def hc_post(self, y, x, residual, post, comb, nt: int, hc: int, hidden: int):
        check(self.L.dsv4cu_hc_post(self.ptr(y), self.ptr(x), self.ptr(residual), self.ptr(post), self.ptr(comb), nt,
                                    hc, hidden, self.stream()), "hc_post")

    def argmax(self, best, logits, n: int, nt: int = 1):
        check(self.L.dsv4cu_argmax(self.ptr(best), self.ptr(logits), n, nt, self.stream()), "argmax")

    def head(self, logits, best, x, m: QMat, nt: int = 1):
        check(self.L.dsv4cu_head(self.ctx, self.ptr(logits), self.ptr(best), self.ptr(x), C.byref(m), nt,
                                 self.stream()), "head")

    def sparse_attn(self, o, q, kv, kv_bf16, sink, idxs, h, d, topk, scale):
        check(self.L.dsv4cu_sparse_attn(self.ctx, self.ptr(o), self.ptr(q), self.ptr(kv), kv_bf16,
                                        self.ptr(sink), self.ptr(idxs), h, d, topk, scale,
                                        self.stream()), "dsv4cu_sparse_attn")

    def quantize_fp8(self, w, s, src, rows, cols):
        check(self.L.dsv4cu_quantize_fp8(self.ptr(w), self.ptr(s), self.ptr(src), rows, cols,
                                         self.stream()), "quantize_fp8")

    def quantize_fp4(self, w, s, src, rows, cols):
        check(self.L.dsv4cu_quantize_fp4(self.ptr(w), self.ptr(s), self.ptr(src), rows, cols,
                                         self.stream()), "quantize_fp4")

    def fill_normal(self, dst, seed, mean, std):
        check(self.L.dsv4cu_fill_normal(self.ptr(dst), dst.numel(), seed, mean, std,
                                        self.stream()), "fill_normal")

    def round_bf16(self, x):
        check(self.L.dsv4cu_round_bf16(self.ptr(x), x.numel(), self.stream()), "round_bf16")


def trunk_manifest(pack_dir: str, layer: int = -1):
    """Host only: (n_layers, run, records) of a pack's trunk.idx; for layer >= 0
    run = (file offset, bytes, widened bytes) and records its TrunkTensor list,
    else both None."""
    L = lib()
    nl, nt = C.c_int(), C.c_int()
    run = (C.c_int64 * 3)()
    if layer < 0:
        check(L.dsv4cu_trunk_manifest(pack_dir.encode(), C.byref(nl), -1, None, None, None, 0), "trunk_manifest")
        return nl.value, None, None
    check(L.dsv4cu_trunk_manifest(pack_dir.encode(), C.byref(nl), layer, run, C.byref(nt), None, 0), "trunk_manifest")
    arr = (TrunkTensor * max(1, nt.value))()
    check(L.dsv4cu_trunk_manifest(pack_dir.encode(), C.byref(nl), layer, run, C.byref(nt), arr, nt.value),
          "trunk_manifest")
    return nl.value, tuple(run), [arr[i] for i in range(nt.value)]


def experts_index(index_dir: str, layer: int = -1, expert: int = -1):
    """Host only: (n_layers, n_experts, records) of a pack's experts.idx;
    records = six (shard, offset, bytes) for (layer, expert), or None."""
    L = lib()
    nl, ne = C.c_int(), C.c_int()
    loc = (C.c_int64 * 18)()
    want = layer >= 0
    check(L.dsv4cu_experts_index(index_dir.encode(), C.byref(nl), C.byref(ne), layer, expert,
                                 loc if want else None), "experts_index")
    recs = [tuple(loc[3 * t:3 * t + 3]) for t in range(6)] if want else None
    return nl.value, ne.value, recs
