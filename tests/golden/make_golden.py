"""Generate the golden vectors in tests/golden/ from the REFERENCE's own kernels.

Runs oracle/_ref/libdsv4ref.so (the reference's src/10_compute compiled from
its own sources by oracle/Makefile) on seeded inputs and stores inputs and
outputs as .npz fixtures. The fixtures travel with the repository, so the GPU
tests can check against the reference where the reference tree is absent.

    python tests/golden/make_golden.py      # needs oracle/_ref/libdsv4ref.so
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "deepseek-v4-in-c_b200")]

import oracle  # noqa: E402
import pack  # noqa: E402


def rand_fp8_codes(rng, n):
    b = rng.integers(0, 256, n, dtype=np.uint8)
    return np.where((b & 0x7F) == 0x7F, b & 0xFE, b).astype(np.uint8)


def matmul_cases(ref: oracle.RefLib, rng):
    out = {}
    # FP8 128x128, rows not a multiple of 16 or 128, nt = 1 and 3
    R, K = 300, 512
    W = rand_fp8_codes(rng, R * K).reshape(R, K)
    S = rng.integers(118, 134, (-(-R // 128)) * (K // 128), dtype=np.uint8)
    x = pack.bf16_round(rng.standard_normal((3, K)).astype(np.float32))
    m = oracle.qmat(W, S, oracle.WFP8, R, K, 128, 128)
    out.update(fp8_W=W, fp8_S=S, fp8_x=x, fp8_y=ref.mmq(x, m))
    # FP8 generic block width 100 (K = 256), as test_matmul.c:468-484
    Kg = 256
    Wg = rand_fp8_codes(rng, 37 * Kg).reshape(37, Kg)
    Sg = np.full(1 * 3, 127, np.uint8)
    xg = ((rng.integers(0, 65536, Kg) - 32768) * 1e-3).astype(np.float32)
    mg = oracle.qmat(Wg, Sg, oracle.WFP8, 37, Kg, 128, 100)
    out.update(fp8g_W=Wg, fp8g_S=Sg, fp8g_x=xg[None], fp8g_y=ref.mmq(xg[None], mg))
    # FP4 1x32, K = 1024; and a K = 160 tail geometry
    for tag, R4, K4, nt in (("fp4", 257, 1024, 2), ("fp4t", 3, 160, 1)):
        W4 = rng.integers(0, 256, R4 * K4 // 2, dtype=np.uint8).reshape(R4, K4 // 2)
        S4 = rng.integers(120, 132, R4 * (K4 // 32), dtype=np.uint8)
        x4 = pack.bf16_round(rng.standard_normal((nt, K4)).astype(np.float32))
        m4 = oracle.qmat(W4, S4, oracle.WFP4, R4, K4, 1, 32)
        out.update({f"{tag}_W": W4, f"{tag}_S": S4, f"{tag}_x": x4, f"{tag}_y": ref.mmq(x4, m4)})
    # BF16
    Wb = pack.bf16_bits(rng.standard_normal((64, 512)).astype(np.float32) * 0.05)
    xb = rng.standard_normal((2, 512)).astype(np.float32)
    mb = oracle.qmat(Wb, None, oracle.WBF16, 64, 512)
    out.update(bf16_W=Wb, bf16_x=xb, bf16_y=ref.mmq(xb, mb))
    return out


def route_cases(ref, rng):
    T, E, K = 64, 256, 8
    logits = pack.bf16_round(rng.standard_normal((T, E)).astype(np.float32))
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    tid2eid = rng.integers(0, E, (97, K)).astype(np.int64)
    out = dict(logits=logits, bias=bias, tid2eid=tid2eid)
    for tag, b, t in (("plain", None, None), ("bias", bias, None), ("hash", None, tid2eid)):
        res = [ref.route(logits[i], K, 1.5, b, t, token_id=(i * 7) % 97) for i in range(T)]
        out[f"{tag}_idx"] = np.stack([r[0] for r in res])
        out[f"{tag}_wts"] = np.stack([r[1] for r in res])
        out[f"{tag}_scores"] = np.stack([r[2] for r in res])
        out[f"{tag}_orig"] = np.stack([r[3] for r in res])
    return out


def indexer_cases(ref, rng):
    H, D, N = 64, 128, 300
    q = rng.standard_normal((H, D)).astype(np.float32)
    kv = rng.standard_normal((N, D)).astype(np.float32)
    w = rng.standard_normal(H).astype(np.float32)
    out = dict(q=q, kv=kv, w=w, score=ref.indexer_score(q, kv, w))
    # FP8 keys/queries with power-of-two scales, dequantized exactly
    q8, qsc = quant_rows(rng.standard_normal((H, D)).astype(np.float32))
    k8, ksc = quant_rows(rng.standard_normal((N, D)).astype(np.float32))
    qf = (pack.E4M3[q8] * qsc[:, None]).astype(np.float32)
    kf = (pack.E4M3[k8] * ksc[:, None]).astype(np.float32)
    out.update(q8=q8, qsc=qsc, k8=k8, ksc=ksc, score8=ref.indexer_score(qf, kf, w))
    # odd head_dim (tail of the 16-chain tree)
    q3 = rng.standard_normal((5, 21)).astype(np.float32)
    k3 = rng.standard_normal((40, 21)).astype(np.float32)
    w3 = rng.standard_normal(5).astype(np.float32)
    out.update(q3=q3, k3=k3, w3=w3, score3=ref.indexer_score(q3, k3, w3))
    return out


def quant_rows(a):
    """e4m3 codes with one power-of-two fp32 scale per row."""
    amax = np.abs(a).max(axis=1)
    f, E = np.frexp(amax)
    e = E - 9 + (f > 0.875)
    sc = np.ldexp(np.ones_like(amax), e).astype(np.float32)
    v = np.ldexp(a, -e[:, None]).astype(np.float32)
    codes = pack._rne_grid(v, pack._E4M3_POS).astype(np.uint8)
    codes = np.where(np.signbit(v), codes | 0x80, codes).astype(np.uint8)
    return codes, sc


def topk_cases(ref, rng):
    out = {}
    for j, n in enumerate((1, 2, 5, 16, 64, 257, 1000, 4000)):
        s = ((rng.integers(0, 256, n) - 128) * 0.01).astype(np.float32)
        s[::7] = 0.5                       # ties at the boundary
        if n > 3:
            s[3] = -0.0
            s[1] = 0.0                     # +0 and -0 tie
        for k in (1, 3, min(n // 2, 1024), min(n, 1024)):
            if k <= 0:
                continue
            out[f"s{j}_k{k}_scores"] = s
            out[f"s{j}_k{k}_idx"] = ref.topk(s, k)
    return out


def attn_cases(ref, rng):
    H, D, N, T = 8, 64, 200, 40
    q = rng.standard_normal((H, D)).astype(np.float32)
    kv = rng.standard_normal((N, D)).astype(np.float32)
    sink = rng.standard_normal(H).astype(np.float32)
    idx = rng.integers(0, N, T).astype(np.int32)
    idx[::5] = -1
    o = ref.sparse_attn(q, kv, sink, idx, 1.0 / np.sqrt(D))
    return dict(q=q, kv=kv, sink=sink, idx=idx, o=o)


def expert_cases(ref, rng):
    hid, inter = 512, 256
    out = {}
    for tag, fmt in (("fp4", oracle.WFP4), ("fp8", oracle.WFP8)):
        mats = []
        for rows, cols, name in ((inter, hid, "w1"), (inter, hid, "w3"), (hid, inter, "w2")):
            w = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
            if fmt == oracle.WFP4:
                W, S = pack.quantize_fp4(w)
                q = oracle.qmat(W, S, fmt, rows, cols, 1, 32)
            else:
                W, S = pack.quantize_fp8(w)
                q = oracle.qmat(W, S, fmt, rows, cols, 128, 128)
            out[f"{tag}_{name}_W"] = W
            out[f"{tag}_{name}_S"] = S
            mats.append((W, S, q))
        x = pack.bf16_round(rng.standard_normal(hid).astype(np.float32))
        out[f"{tag}_x"] = x
        out[f"{tag}_out"] = ref.expert_forward(x, [m[2] for m in mats], inter, 10.0)
    return out


def main():
    if not oracle.RefLib.available():
        sys.exit("oracle/_ref/libdsv4ref.so not built (make -C oracle ref)")
    ref = oracle.RefLib()
    rng = np.random.default_rng(20261201)
    for name, fn in (("matmul", matmul_cases), ("route", route_cases), ("indexer", indexer_cases),
                     ("topk", topk_cases), ("attn", attn_cases), ("expert", expert_cases)):
        data = fn(ref, rng)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        print(name, sum(v.nbytes for v in data.values()), "bytes")


if __name__ == "__main__":
    main()
