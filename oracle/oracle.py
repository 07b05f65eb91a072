"""CPU checkers for the CUDA library: TEST INFRASTRUCTURE ONLY.

Two checkers, both plain C, loaded with ctypes:

* ``Oracle`` wraps ``oracle/liboracle.so``: this repository's C restatement of
  the reference algorithms (``oracle/dsv4_oracle.c``; every function cites the
  reference lines it restates).
* ``RefLib`` wraps ``oracle/_ref/libdsv4ref.so``: the reference's own CPU kernels
  compiled from its sources by ``oracle/Makefile``. It exists only where the
  reference tree was available at build time; callers must tolerate its absence.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may use
this module. The product library never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdsv4ref.so")
LAYER_SO = os.path.join(HERE, "_ref", "libdsv4layer.so")
TRUNK_SO = os.path.join(HERE, "_ref", "libdsv4trunk.so")
# The reference source tree: set by the caller (DSV4_REFERENCE_TREE or build(ref_tree=...));
# without it only the restatement is built.
REF_TREE = os.environ.get("DSV4_REFERENCE_TREE")

WF32, WBF16, WFP8, WFP4 = 0, 1, 2, 3


class QMat(C.Structure):
    """Same layout as the reference DSV4QMat (src/00_base/dsv4_weights.h:34-40)."""
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("wdt", C.c_int),
                ("rows", C.c_int), ("cols", C.c_int),
                ("blk_r", C.c_int), ("blk_c", C.c_int)]


def build(ref_tree: str | None = None) -> None:
    """Compile the restatement (always) and, given the reference source tree
    (ref_tree or DSV4_REFERENCE_TREE), the reference library and its unit
    tests. Builds the checkers; does not run them."""
    subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    tree = ref_tree or REF_TREE
    if tree and os.path.isdir(os.path.join(tree, "src", "10_compute")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={tree}"], check=True)
        # the reference's own unit tests linked against the CUDA library (run only by the GPU tests)
        if os.path.exists(os.path.join(HERE, "..", "deepseek-v4-in-c_b200", "libdsv4cu.so")):
            subprocess.run(["make", "-s", "-C", HERE, "units", f"REF={tree}"], check=True)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def qmat(w: np.ndarray, s, wdt: int, rows: int, cols: int, blk_r=0, blk_c=0) -> QMat:
    return QMat(w.ctypes.data, None if s is None else s.ctypes.data, wdt, rows, cols,
                blk_r, blk_c)


class _Common:
    """Calls shared by the restatement and the reference library (same ABI
    shapes; the restatement prefixes its symbols with ``orc_``)."""

    def __init__(self, lib, prefix):
        self.lib = lib
        self.pf = prefix
        f = self.fn
        f("indexer_score").restype = None
        f("topk").restype = C.c_int
        f("sparse_attn").restype = None
        f("route").restype = None
        f("swiglu").restype = None
        f("rmsnorm").restype = None
        f("rope_apply").restype = None
        f("hc_post").restype = None
        f("hc_pre").restype = None
        f("compress_step").restype = C.c_int

    def fn(self, name):
        return getattr(self.lib, self.pf + name)

    def route(self, logits, topk, route_scale, bias=None, tid2eid=None, token_id=0):
        ne = logits.shape[0]
        scores = np.ascontiguousarray(logits, dtype=np.float32).copy()
        orig = np.zeros(ne, np.float32)
        idx = np.zeros(topk, np.int32)
        wts = np.zeros(topk, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        t = None if tid2eid is None else np.ascontiguousarray(tid2eid, np.int64)
        self.fn("route")(_p(idx), _p(wts), _p(scores), _p(orig), _p(b), _p(t),
                         C.c_int(token_id), C.c_int(ne), C.c_int(topk),
                         C.c_float(route_scale))
        return idx, wts, scores, orig

    def swiglu(self, gate, up, limit):
        y = np.zeros_like(gate, dtype=np.float32)
        self.fn("swiglu")(_p(y), _p(np.ascontiguousarray(gate, np.float32)),
                          _p(np.ascontiguousarray(up, np.float32)), C.c_int(gate.size),
                          C.c_float(limit))
        return y

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        self.fn("rmsnorm")(_p(y), _p(x), _p(np.ascontiguousarray(w, np.float32)), C.c_int(x.size),
                           C.c_float(eps))
        return y

    def rope_apply(self, v, rd, cs, sn, pos, inverse=0):
        """v [head_dim] (a copy is rotated and returned); cs / sn [positions][half]."""
        v = np.ascontiguousarray(v, np.float32).copy()
        cs = np.ascontiguousarray(cs, np.float32)
        self.fn("rope_apply")(_p(v), C.c_int(v.size), C.c_int(rd), _p(cs), _p(np.ascontiguousarray(sn, np.float32)),
                              C.c_int(pos), C.c_int(cs.shape[1]), C.c_int(inverse))
        return v

    def hc_pre(self, x, fn, base, scale, iters, norm_eps, hc_eps):
        """x [hc][hidden], fn [(2 + hc) hc][hc hidden], base [(2 + hc) hc], scale [3]
        -> (y [hidden], post [hc], comb [hc][hc], mixes [(2 + hc) hc])."""
        x = np.ascontiguousarray(x, np.float32)
        hc, hidden = x.shape
        mix = (2 + hc) * hc
        y = np.zeros(hidden, np.float32)
        post = np.zeros(hc, np.float32)
        comb = np.zeros((hc, hc), np.float32)
        mixes = np.zeros(mix, np.float32)
        fn = np.ascontiguousarray(fn, np.float32)
        base = np.ascontiguousarray(base, np.float32)
        scale = np.ascontiguousarray(scale, np.float32)
        if self.pf == "orc_":
            self.fn("hc_pre")(_p(y), _p(post), _p(comb), _p(mixes), _p(x), _p(fn), _p(base), _p(scale), C.c_int(hc),
                              C.c_int(hidden), C.c_int(iters), C.c_float(norm_eps), C.c_float(hc_eps))
        else:       # the reference takes a DSV4HcW {fn, base, scale} (src/00_base/dsv4_weights.h:116-121)
            w = (C.c_void_p * 3)(fn.ctypes.data, base.ctypes.data, scale.ctypes.data)
            self.fn("hc_pre")(_p(y), _p(post), _p(comb), _p(mixes), _p(x), w, C.c_int(hc), C.c_int(hidden),
                              C.c_int(iters), C.c_float(norm_eps), C.c_float(hc_eps))
        return y, post, comb, mixes

    def hc_head(self, x, fn, base, scale, norm_eps, hc_eps):
        """The restatement only (hc_head is static in the reference's CLI)."""
        x = np.ascontiguousarray(x, np.float32)
        hc, hidden = x.shape
        y = np.zeros(hidden, np.float32)
        self.lib.orc_hc_head.restype = None
        self.lib.orc_hc_head(_p(y), _p(x), _p(np.ascontiguousarray(fn, np.float32)),
                             _p(np.ascontiguousarray(base, np.float32)), _p(np.ascontiguousarray(scale, np.float32)),
                             C.c_int(hc), C.c_int(hidden), C.c_float(norm_eps), C.c_float(hc_eps))
        return y

    def compress_step(self, kv_in, score_in, ape, kv_state, score_state, pos, ratio, head_dim):
        """Updates kv_state / score_state in place; returns (emitted, out [head_dim])."""
        out = np.zeros(head_dim, np.float32)
        r = self.fn("compress_step")(_p(out), _p(np.ascontiguousarray(kv_in, np.float32)),
                                     _p(np.ascontiguousarray(score_in, np.float32)),
                                     _p(np.ascontiguousarray(ape, np.float32)), _p(kv_state), _p(score_state),
                                     C.c_int(pos), C.c_int(ratio), C.c_int(head_dim))
        return r, out

    def hc_post(self, x, residual, post, comb):
        """x [hidden], residual [hc][hidden], post [hc], comb [hc][hc] -> y [hc][hidden]."""
        residual = np.ascontiguousarray(residual, np.float32)
        hc, hidden = residual.shape
        y = np.zeros((hc, hidden), np.float32)
        self.fn("hc_post")(_p(y), _p(np.ascontiguousarray(x, np.float32)), _p(residual),
                           _p(np.ascontiguousarray(post, np.float32)), _p(np.ascontiguousarray(comb, np.float32)),
                           C.c_int(hc), C.c_int(hidden))
        return y

    def indexer_score(self, q, kv, weights):
        h, d = q.shape
        n = kv.shape[0]
        out = np.zeros(n, np.float32)
        self.fn("indexer_score")(_p(out), _p(np.ascontiguousarray(q, np.float32)),
                                 _p(np.ascontiguousarray(kv, np.float32)),
                                 _p(np.ascontiguousarray(weights, np.float32)),
                                 C.c_int(h), C.c_int(d), C.c_int(n))
        return out

    def topk(self, scores, k):
        scores = np.ascontiguousarray(scores, np.float32)
        out = np.full(max(1, min(k, scores.size)), -7, np.int32)
        r = self.fn("topk")(_p(out), _p(scores), C.c_int(scores.size), C.c_int(k))
        return out[:max(r, 0)]


class Oracle(_Common):
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(with_ref=False)
        lib = C.CDLL(path)
        super().__init__(lib, "orc_")
        lib.orc_e8m0.restype = C.c_float
        lib.orc_e8m0.argtypes = [C.c_uint8]
        lib.orc_e4m3.restype = C.c_float
        lib.orc_e4m3.argtypes = [C.c_uint8]
        lib.orc_e2m1.restype = C.c_float
        lib.orc_e2m1.argtypes = [C.c_uint8]
        lib.orc_fp4_at.restype = C.c_float
        lib.orc_fp4_at.argtypes = [C.c_void_p, C.c_int64]
        lib.orc_mmq_n.restype = C.c_int
        lib.orc_dot_f32d.restype = C.c_double
        lib.orc_window_idxs.restype = C.c_int
        lib.orc_expert_buckets.restype = C.c_int

    def mmq(self, x, m: QMat, nt=None):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, m.rows), np.float32)
        r = self.lib.orc_mmq_n(_p(y), _p(x), C.byref(m), C.c_int(nt))
        if r != 0:
            raise ValueError(f"oracle: unknown weight format {m.wdt}")
        return y

    def expert_forward(self, x, w3: list, inter: int, limit: float):
        arr = (QMat * 3)(*w3)
        out = np.zeros(w3[2].rows, np.float32)
        self.lib.orc_expert_forward(_p(out), _p(np.ascontiguousarray(x, np.float32)), arr,
                                    C.c_int(inter), C.c_float(limit))
        return out

    def moe_decode(self, x, logits, experts: list, shared: list, topk, route_scale,
                   hidden, inter, limit, bias=None, tid2eid=None, token_id=0):
        ne = len(experts)
        arr = (QMat * (3 * ne))(*[q for e in experts for q in e])
        sh = (QMat * 3)(*shared)
        out = np.zeros(hidden, np.float32)
        idx = np.zeros(topk, np.int32)
        wts = np.zeros(topk, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        t = None if tid2eid is None else np.ascontiguousarray(tid2eid, np.int64)
        self.lib.orc_moe_decode(_p(out), _p(idx), _p(wts),
                                _p(np.ascontiguousarray(x, np.float32)),
                                _p(np.ascontiguousarray(logits, np.float32)), _p(b), _p(t),
                                C.c_int(token_id), arr, sh, C.c_int(ne), C.c_int(topk),
                                C.c_float(route_scale), C.c_int(hidden), C.c_int(inter),
                                C.c_float(limit))
        return out, idx, wts

    def sparse_attn(self, q, kv, sink, idxs, scale):
        h, d = q.shape
        o = np.zeros((h, d), np.float32)
        self.lib.orc_sparse_attn(_p(o), _p(np.ascontiguousarray(q, np.float32)),
                                 _p(np.ascontiguousarray(kv, np.float32)),
                                 _p(np.ascontiguousarray(sink, np.float32)),
                                 _p(np.ascontiguousarray(idxs, np.int32)), C.c_int(h),
                                 C.c_int(d), C.c_int(len(idxs)), C.c_float(scale))
        return o

    def window_idxs(self, pos, win):
        out = np.zeros(win, np.int32)
        n = self.lib.orc_window_idxs(_p(out), C.c_int(pos), C.c_int(win))
        return out, n

    def indexer_offset(self, idxs, offset):
        a = np.ascontiguousarray(idxs, np.int32).copy()
        self.lib.orc_indexer_offset(_p(a), C.c_int(a.size), C.c_int(offset))
        return a

    def expert_buckets(self, topk_idx, n_experts):
        ti = np.ascontiguousarray(topk_idx, np.int32)
        n, topk = ti.shape
        count = np.zeros(n_experts, np.int32)
        off = np.zeros(n_experts + 1, np.int32)
        tok = np.zeros(n * topk, np.int32)
        ks = np.zeros(n * topk, np.int32)
        d = self.lib.orc_expert_buckets(_p(count), _p(off), _p(tok), _p(ks), _p(ti),
                                        C.c_int(n), C.c_int(topk), C.c_int(n_experts))
        return count, off, tok, ks, d


class RefLib(_Common):
    """The reference's own kernels (oracle/_ref/libdsv4ref.so)."""

    def __init__(self, path: str = REF_SO):
        lib = C.CDLL(path)
        super().__init__(lib, "dsv4_")
        lib.dsv4_cfg_init.restype = None

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def mmq(self, x, m: QMat):
        x = np.ascontiguousarray(x, np.float32)
        nt = x.shape[0] if x.ndim == 2 else 1
        y = np.zeros((nt, m.rows), np.float32)
        self.lib.dsv4_mmq_n(_p(y), _p(x), C.byref(m), C.c_int(nt))
        return y

    def matmul_fp8_exact(self, x, m: QMat):
        """tests/unit/ref_kernels.c:53-76, the exact-table FP8 reference."""
        y = np.zeros(m.rows, np.float32)
        self.lib.dsv4_matmul_fp8_f32(_p(y), _p(np.ascontiguousarray(x, np.float32)),
                                     C.c_void_p(m.w), C.c_void_p(m.s), C.c_int(m.cols),
                                     C.c_int(m.rows), C.c_int(m.blk_r), C.c_int(m.blk_c))
        return y

    def expert_forward(self, x, w3: list, inter: int, limit: float):
        """src/10_compute/dsv4_ops.c:85-93 through the reference's own matmuls.
        DSV4ExpertW is {w1, w3, w2} (src/00_base/dsv4_weights.h:101-104)."""
        arr = (QMat * 3)(*w3)
        out = np.zeros(w3[2].rows, np.float32)
        scratch = np.zeros(inter * 3, np.float32)
        self.lib.dsv4_expert_forward(_p(out), _p(np.ascontiguousarray(x, np.float32)), arr,
                                     _p(scratch), _p(scratch[inter:]), _p(scratch[2 * inter:]),
                                     C.c_int(inter), C.c_float(limit))
        return out

    def sparse_attn(self, q, kv, sink, idxs, scale):
        h, d = q.shape
        o = np.zeros((h, d), np.float32)
        scratch = np.zeros(h * max(1, len(idxs)), np.float32)
        self.lib.dsv4_sparse_attn(_p(o), _p(np.ascontiguousarray(q, np.float32)),
                                  _p(np.ascontiguousarray(kv, np.float32)),
                                  _p(np.ascontiguousarray(sink, np.float32)),
                                  _p(np.ascontiguousarray(idxs, np.int32)), C.c_int(h),
                                  C.c_int(d), C.c_int(len(idxs)), C.c_float(scale),
                                  _p(scratch))
        return o


class RefLayer:
    """The reference's attention block on its own CPU kernels (oracle/_ref/
    libdsv4layer.so: src/70_decode/dsv4_layer_attn.c behind layer_ref.c), one
    layer with seeded random weights. Test infrastructure only.

    dims: hidden, n_heads, head_dim, q_lora, o_lora, o_groups, qk_rope,
    sliding_window, index_n_heads, index_head_dim, index_topk, hc_mult."""

    MATS = ("wq_a", "wq_b", "wkv", "wo_a", "wo_b", "comp_wkv", "comp_wgate", "idx_wq_b", "idx_wproj")
    VECS = ("q_norm", "kv_norm", "sink", "comp_ape", "comp_norm", "attn_norm", "hc_fn", "hc_base", "hc_scale",
            "cs", "sn")

    def __init__(self, dims, ratio: int, max_pos: int, seed: int, path: str = LAYER_SO):
        self.lib = L = C.CDLL(path)
        L.lr_create.restype = C.c_void_p
        L.lr_create.argtypes = [C.POINTER(C.c_int), C.c_int, C.c_int, C.c_ulonglong]
        L.lr_free.argtypes = [C.c_void_p]
        L.lr_qmat.argtypes = [C.c_void_p, C.c_int, C.POINTER(QMat)]
        L.lr_vec.restype = C.POINTER(C.c_float)
        L.lr_vec.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int)]
        L.lr_attention.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.lr_attn_block.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.lr_n_compressed.argtypes = [C.c_void_p]
        L.lr_kv_cache.restype = C.POINTER(C.c_float)
        L.lr_kv_cache.argtypes = [C.c_void_p]
        self.dims = list(dims)
        L.lr_trap_crashes()
        arr = (C.c_int * 12)(*self.dims)
        self.h = L.lr_create(arr, ratio, max_pos, seed)
        if not self.h:
            raise RuntimeError("lr_create failed")
        self.ratio, self.max_pos = ratio, max_pos

    @staticmethod
    def available(path: str = LAYER_SO) -> bool:
        return os.path.exists(path)

    def close(self):
        if self.h:
            self.lib.lr_free(self.h)
            self.h = None

    def qmat(self, name):
        """(QMat with host pointers, weight bytes, scale bytes or None) of a matrix, or None."""
        m = QMat()
        if not self.lib.lr_qmat(self.h, self.MATS.index(name), C.byref(m)):
            return None
        esz = {WBF16: 2, WFP8: 1}[m.wdt]
        w = np.ctypeslib.as_array(C.cast(m.w, C.POINTER(C.c_uint8)), shape=(m.rows * m.cols * esz,))
        s = None
        if m.s:
            n = ((m.rows + m.blk_r - 1) // m.blk_r) * ((m.cols + m.blk_c - 1) // m.blk_c)
            s = np.ctypeslib.as_array(C.cast(m.s, C.POINTER(C.c_uint8)), shape=(n,))
        return m, w, s

    def vec(self, name):
        n = C.c_int(0)
        p = self.lib.lr_vec(self.h, self.VECS.index(name), C.byref(n))
        if not p or n.value == 0:
            return None
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def attention(self, x, pos: int):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.dims[0], np.float32)
        self.lib.lr_attention(self.h, _p(out), _p(x), pos)
        return out

    def attn_block(self, h, pos: int):
        h = np.ascontiguousarray(h, np.float32).copy()
        self.lib.lr_attn_block(self.h, _p(h), pos)
        return h

    def n_compressed(self) -> int:
        return self.lib.lr_n_compressed(self.h)

    def ffn_create(self, n_experts: int, topk: int, inter: int, route_scale: float, limit: float, bias: bool,
                   seed: int):
        """The FFN half's weights (BF16 gate, FP4 experts, FP8 shared expert, ffn_norm, mHC)."""
        L = self.lib
        L.lr_ffn_create.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int,
                                    C.c_ulonglong]
        L.lr_expert_qmat.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(QMat)]
        L.lr_ffn_vec.restype = C.POINTER(C.c_float)
        L.lr_ffn_vec.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_int)]
        L.lr_ffn_block.argtypes = [C.c_void_p, C.c_void_p]
        L.lr_layer.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.lr_ffn_create(self.h, n_experts, topk, inter, route_scale, limit, 1 if bias else 0, seed)
        self.n_experts, self.topk, self.inter = n_experts, topk, inter

    def expert_qmat(self, e: int, m: int):
        """(QMat, weight bytes, scale bytes or None) of matrix m of expert e (n_experts: shared; -1: gate)."""
        q = QMat()
        if not self.lib.lr_expert_qmat(self.h, e, m, C.byref(q)):
            return None
        nb = {WBF16: q.rows * q.cols * 2, WFP8: q.rows * q.cols, WFP4: q.rows * q.cols // 2}[q.wdt]
        w = np.ctypeslib.as_array(C.cast(q.w, C.POINTER(C.c_uint8)), shape=(nb,))
        s = None
        if q.s:
            n = ((q.rows + q.blk_r - 1) // q.blk_r) * ((q.cols + q.blk_c - 1) // q.blk_c)
            s = np.ctypeslib.as_array(C.cast(q.s, C.POINTER(C.c_uint8)), shape=(n,))
        return q, w, s

    def ffn_vec(self, which: str):
        n = C.c_int(0)
        p = self.lib.lr_ffn_vec(self.h, ("bias", "ffn_norm", "hc_fn", "hc_base", "hc_scale").index(which),
                                C.byref(n))
        if not p or n.value == 0:
            return None
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def ffn_block(self, h):
        h = np.ascontiguousarray(h, np.float32).copy()
        self.lib.lr_ffn_block(self.h, _p(h))
        return h

    def layer(self, h, pos: int):
        h = np.ascontiguousarray(h, np.float32).copy()
        self.lib.lr_layer(self.h, _p(h), pos)
        return h


class RefTrunkTensor(C.Structure):
    """The record trunk_ref.c fills (the reference's DSV4TrunkTensor fields)."""
    _fields_ = [("slot", C.c_int32), ("dtype", C.c_int32), ("rows", C.c_int32), ("cols", C.c_int32),
                ("wdt", C.c_int32), ("blk_r", C.c_int32), ("blk_c", C.c_int32),
                ("off", C.c_int64), ("nbytes", C.c_int64)]


def ref_trunk_available(path: str = TRUNK_SO) -> bool:
    return os.path.exists(path)


def ref_trunk_manifest(pack_dir: str, layer: int = -1, path: str = TRUNK_SO):
    """The reference's own trunk.idx reader (src/50_loader/dsv4_trunk_manifest.c:
    24-110 behind oracle/trunk_ref.c): None when it rejects the index, else
    (n_layers, run, records) as tuples, run / records None for layer < 0."""
    lib = C.CDLL(path)
    f = lib.ref_trunk_manifest
    f.restype = C.c_int
    f.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.c_int, C.POINTER(C.c_int64), C.POINTER(C.c_int),
                  C.POINTER(RefTrunkTensor), C.c_int]
    nl, nt = C.c_int(), C.c_int()
    run = (C.c_int64 * 3)()
    if f(pack_dir.encode(), C.byref(nl), layer, run, C.byref(nt), None, 0) != 0:
        return None
    if layer < 0:
        return nl.value, None, None
    arr = (RefTrunkTensor * max(1, nt.value))()
    f(pack_dir.encode(), C.byref(nl), layer, run, C.byref(nt), arr, nt.value)
    recs = [(t.slot, t.off, t.nbytes, t.dtype, t.rows, t.cols, t.wdt, t.blk_r, t.blk_c)
            for t in arr[:nt.value]]
    return nl.value, tuple(run), recs
