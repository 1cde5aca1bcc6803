"""Generate tests/golden/ref_ops.npz from the reference's OWN scalar oracles.

Run in a checkout where the reference tree is present:
    python tests/golden/make_golden.py
It compiles oracle/_ref/libref_oracle.so from the reference headers
(native/operator_reference.h, native/projection_reference.h,
native/attention_reference.h) via oracle/Makefile, feeds seeded random inputs
through them and stores inputs + reference outputs. The committed fixture pins
the in-repo oracle (oracle/qwen_oracle.cpp) without the reference tree.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "ref_ops.npz"


def main():
    path = O.build_ref()
    if path is None:
        raise SystemExit("reference tree not found: cannot regenerate golden fixtures")
    R = C.CDLL(str(path))
    R.ref_last_error.restype = C.c_char_p
    D, F = C.POINTER(C.c_double), C.POINTER(C.c_float)

    def ok(rc):
        if rc:
            raise RuntimeError(R.ref_last_error().decode())

    rng = np.random.default_rng(20261201)
    out = {}
    f32 = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731

    # RMSNorm (operator_reference.h:11-14)
    for i, (rows, width) in enumerate([(3, 64), (2, 256), (1, 2048)]):
        x, w = f32(rows, width), (1 + 0.1 * rng.standard_normal(width)).astype(np.float32)
        y = np.zeros(rows * width)
        ok(R.ref_rms(O.ptr(x), x.size, O.ptr(w), w.size, width, C.c_double(1e-6), O.ptr(y, C.c_double)))
        out.update({f"rms{i}_x": x, f"rms{i}_w": w, f"rms{i}_y": y})
    # SiLU
    x = (4 * f32(257)).astype(np.float32)
    y = np.zeros(x.size)
    ok(R.ref_silu(O.ptr(x), x.size, O.ptr(y, C.c_double)))
    out.update(silu_x=x, silu_y=y)
    # RoPE (operator_reference.h:15-18); its bounds allow tokens <= 8, offset <= 512 - tokens.
    for i, (heads, tokens, dim, rot, off, theta) in enumerate(
            [(2, 3, 64, 16, 5, 1e7), (4, 8, 256, 64, 504, 1e7), (1, 1, 4, 4, 3, 1e4)]):
        x = f32(heads, tokens, dim)
        y = np.zeros(x.size)
        ok(R.ref_rope(O.ptr(x), heads, tokens, dim, rot, off, C.c_double(theta), O.ptr(y, C.c_double)))
        out.update({f"rope{i}_x": x, f"rope{i}_geo": np.array([heads, tokens, dim, rot, off]),
                    f"rope{i}_theta": np.array(theta), f"rope{i}_y": y})
    # Gated delta rule + causal conv (operator_reference.h:19-45)
    for i, (T, hk, hv, dk, dv, K) in enumerate([(1, 1, 2, 4, 4, 4), (5, 2, 4, 16, 8, 4),
                                                (8, 2, 4, 64, 64, 4)]):
        ch = 2 * hk * dk + hv * dv
        args = dict(qkv=f32(T, ch), hist=f32(K - 1, ch), conv=(0.3 * f32(ch, K)).astype(np.float32),
                    a=f32(T, hv), b=f32(T, hv), alog=(0.5 * f32(hv)).astype(np.float32),
                    dt=(0.5 * f32(hv)).astype(np.float32), init=(0.1 * f32(hv, dv, dk)).astype(np.float32))
        act, hist, o, st = (np.zeros(T * ch), np.zeros((K - 1) * ch), np.zeros(T * hv * dv),
                            np.zeros(hv * dv * dk))
        ok(R.ref_delta(*(O.ptr(args[k]) for k in ("qkv", "hist", "conv", "a", "b", "alog", "dt", "init")),
                       T, hk, hv, dk, dv, K, *(O.ptr(a, C.c_double) for a in (act, hist, o, st))))
        for k, v in args.items():
            out[f"delta{i}_{k}"] = v
        out.update({f"delta{i}_geo": np.array([T, hk, hv, dk, dv, K]), f"delta{i}_act": act,
                    f"delta{i}_hist_out": hist, f"delta{i}_out": o, f"delta{i}_state": st})
    # Routing weights for a valid top-k selection (operator_reference.h:47-57)
    for i, (rows, experts, top) in enumerate([(4, 16, 2), (8, 256, 8)]):
        lg = f32(rows, experts)
        sel = np.argsort(-lg, axis=1, kind="stable")[:, :top].astype(np.int32)
        pr, w = np.zeros(rows * experts), np.zeros(rows * top)
        ok(R.ref_routing(O.ptr(lg), O.ptr(sel, C.c_int), rows, experts, top, O.ptr(pr, C.c_double),
                         O.ptr(w, C.c_double)))
        out.update({f"route{i}_logits": lg, f"route{i}_sel": sel, f"route{i}_p": pr, f"route{i}_w": w})
    # Affine projection (projection_reference.h:8-22), widths 2..8, groups 32..128
    for i, (rows, outs, width, group, bits) in enumerate(
            [(3, 16, 256, 64, 4), (8, 32, 512, 64, 4), (2, 8, 128, 32, 3), (1, 5, 256, 128, 8),
             (4, 7, 192, 64, 6)]):
        x = f32(rows, width)
        words = width * bits // 32
        packed = rng.integers(0, 2**32, size=(outs, words), dtype=np.uint64).astype(np.uint32)
        sc = (0.01 * f32(outs, width // group)).astype(np.float32)
        bi = (0.05 * f32(outs, width // group)).astype(np.float32)
        y = np.zeros(rows * outs)
        ok(R.ref_projection(O.ptr(x), O.ptr(packed, C.c_uint32), O.ptr(sc), O.ptr(bi), rows, outs,
                            width, group, bits, O.ptr(y, C.c_double)))
        out.update({f"proj{i}_x": x, f"proj{i}_packed": packed, f"proj{i}_sc": sc,
                    f"proj{i}_bi": bi, f"proj{i}_geo": np.array([rows, outs, width, group, bits]),
                    f"proj{i}_y": y})
    # Causal GQA attention (attention_reference.h:8-21)
    for i, (heads, kvh, tokens, offset, dim) in enumerate([(4, 1, 1, 37, 64), (16, 2, 3, 20, 256),
                                                           (8, 2, 5, 0, 32)]):
        n = offset + tokens
        q, k, v = f32(heads, tokens, dim), f32(kvh, n, dim), f32(kvh, n, dim)
        o = np.zeros(q.size)
        ok(R.ref_attention(O.ptr(q), O.ptr(k), O.ptr(v), heads, kvh, tokens, offset, dim,
                           O.ptr(o, C.c_double)))
        out.update({f"attn{i}_q": q, f"attn{i}_k": k, f"attn{i}_v": v,
                    f"attn{i}_geo": np.array([heads, kvh, tokens, offset, dim]), f"attn{i}_o": o})
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
