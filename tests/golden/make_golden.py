"""Regenerates the golden fixtures in this folder (reference_tests.npz).

lisa-rs runs only on Metal and its Rust tests cannot be built here, so the
fixtures are the CPU expectations the reference's own tests compute, restated
in numpy from their source and fed the same deterministic inputs:

* tests/attn_sliced.rs:21-25 ``gen_f16`` inputs (seeds 1/2/3 for q/K/V,
  truncating f32->bf16 of src/format/dtype.rs:42-47) and its CPU reference
  ``cpu_expected`` (tests/attn_sliced.rs:114-130) for
  ctx in {1, 16, 63, 64, 129, 1000}, every head, dims 0, 37, ..., 222
  (the reference checks ``(0..HD).step_by(37)``). Tolerance there: 1e-4.
* tests/attn_cache.rs:194-292 block-3 causality case: capacity 6, base 3,
  query/K/V patterns %37, %41, %43, expected for rows 0..2, every head,
  dims {0, 73, 255}. Tolerance there: 2e-5.

The arithmetic follows the Rust: f32 folds in token/dim order (np.cumsum in
float32 is a sequential fold), f32 exp, f32 division.

Run:  python tests/golden/make_golden.py   (writes reference_tests.npz)
"""
from __future__ import annotations

import os

import numpy as np

QH, KVH, HD = 24, 4, 256
OSTRIDE = QH * HD
SLICED_CTX = [1, 16, 63, 64, 129, 1000]
SLICED_DIMS = list(range(0, HD, 37))
B3_CAP, B3_BASE, B3_DIMS = 6, 3, [0, 73, HD - 1]


def trunc_bf16(x: np.ndarray) -> np.ndarray:
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def gen_f16(seed: int, items: int) -> np.ndarray:
    """tests/attn_sliced.rs:21-25."""
    i = np.arange(items, dtype=np.int64)
    vals = ((i * seed * 13 % 131).astype(np.float32) - np.float32(65.0)) * np.float32(0.01) + np.float32(seed % 7)
    return trunc_bf16(vals.astype(np.float32))


def block3_inputs():
    """tests/attn_cache.rs:201-209."""
    iq = np.arange(3 * OSTRIDE)
    ik = np.arange(KVH * B3_CAP * HD)
    q = trunc_bf16(((iq % 37).astype(np.float32) - np.float32(18.0)) * np.float32(0.01))
    k = trunc_bf16(((ik % 41).astype(np.float32) - np.float32(20.0)) * np.float32(0.008))
    v = trunc_bf16(((ik % 43).astype(np.float32) - np.float32(21.0)) * np.float32(0.006))
    return q, k, v


def cpu_softmax_expected(q_row: np.ndarray, keys: np.ndarray, vals: np.ndarray, dims) -> np.ndarray:
    """The CPU softmax of tests/attn_sliced.rs:114-130 / attn_cache.rs:261-291
    for one (row, head): q_row f32 [256], keys/vals f32 [ctx, 256]."""
    prods = (q_row[None, :] * keys).astype(np.float32)
    scores = np.cumsum(prods, axis=1, dtype=np.float32)[:, -1] * np.float32(0.0625)
    mx = np.float32(scores.max())
    w = np.exp((scores - mx).astype(np.float32)).astype(np.float32)
    denom = np.cumsum(w, dtype=np.float32)[-1]
    out = []
    for d in dims:
        acc = np.cumsum((w * vals[:, d]).astype(np.float32), dtype=np.float32)[-1]
        out.append(np.float32(acc / denom))
    return np.array(out, np.float32)


def make_sliced():
    exp = np.zeros((len(SLICED_CTX), QH, len(SLICED_DIMS)), np.float32)
    for ci, ctx in enumerate(SLICED_CTX):
        q = bf(gen_f16(1, OSTRIDE)).reshape(QH, HD)
        k = bf(gen_f16(2, KVH * ctx * HD)).reshape(KVH, ctx, HD)
        v = bf(gen_f16(3, KVH * ctx * HD)).reshape(KVH, ctx, HD)
        for h in range(QH):
            kvh = h // (QH // KVH)
            exp[ci, h] = cpu_softmax_expected(q[h], k[kvh], v[kvh], SLICED_DIMS)
    return exp


def make_block3():
    qb, kb, vb = block3_inputs()
    q = bf(qb).reshape(3, QH, HD)
    k = bf(kb).reshape(KVH, B3_CAP, HD)
    v = bf(vb).reshape(KVH, B3_CAP, HD)
    exp = np.zeros((3, QH, len(B3_DIMS)), np.float32)
    for r in range(3):
        ctx = B3_BASE + r + 1
        for h in range(QH):
            kvh = h // (QH // KVH)
            exp[r, h] = cpu_softmax_expected(q[r, h], k[kvh, :ctx], v[kvh, :ctx], B3_DIMS)
    return exp


def main(path: str | None = None) -> str:
    path = path or os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_tests.npz")
    np.savez_compressed(
        path,
        sliced_ctx=np.array(SLICED_CTX, np.int32),
        sliced_dims=np.array(SLICED_DIMS, np.int32),
        sliced_expected=make_sliced(),
        block3_cap=np.int32(B3_CAP),
        block3_base=np.int32(B3_BASE),
        block3_dims=np.array(B3_DIMS, np.int32),
        block3_expected=make_block3(),
    )
    return path


if __name__ == "__main__":
    print(main())
