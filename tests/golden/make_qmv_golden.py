"""Regenerates qmv_reference_tests.npz: the affine-u4 QMV known-answer cases
of lisa-rs's own tests, restated in numpy from their source with the same
deterministic inputs and their CPU expectations (an f32 fold over k in
order, weight = q * scale + bias in f32):

* tests/qmv.rs:5-113 ``qmv_matches_affine_reference_with_tail_rows``:
  M = 1, N = 19, K = 128, x = (k - 63) * 0.003, packed nibble
  (word * 3 + nibble * 5) % 16, scale 0.0125, bias -0.08. Tolerance 2e-4.
* tests/qmv.rs:115-220 ``qmv_wide3_matches_three_affine_references_with_tail_rows``:
  M = 3, x = (k - 61 + row * 7) * 0.0025, nibble (word * 7 + nibble * 3) % 16,
  scale 0.011, bias -0.075. Tolerance 2e-4.
f32 -> bf16 is the truncation of src/format/dtype.rs:42-47.

Run:  python tests/golden/make_qmv_golden.py   (writes qmv_reference_tests.npz)
"""
from __future__ import annotations

import os

import numpy as np


def trunc_bf16(x) -> np.ndarray:
    return (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf(b) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def packed_words(n: int, k: int, mul_w: int, mul_n: int) -> np.ndarray:
    idx = np.arange(n * k // 8, dtype=np.uint64)
    word = np.zeros_like(idx)
    for nib in range(8):
        word |= ((idx * mul_w + nib * mul_n) % 16) << np.uint64(4 * nib)
    return word.astype(np.uint32).reshape(n, k // 8)


def expected_fold(x_bits, packed, scale_bits, bias_bits):
    """The reference tests' CPU loop: per (input row, output row) an f32 fold
    over k of x * (q * scale + bias)."""
    m_rows, k = x_bits.shape
    n = packed.shape[0]
    q = ((packed[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF).reshape(n, k).astype(np.float32)
    s = np.repeat(bf(scale_bits).reshape(n, k // 64), 64, axis=1)
    b = np.repeat(bf(bias_bits).reshape(n, k // 64), 64, axis=1)
    w = (q * s + b).astype(np.float32)
    x = bf(x_bits)
    out = np.zeros((m_rows, n), np.float32)
    for mi in range(m_rows):
        prod = (x[mi][None, :] * w).astype(np.float32)
        out[mi] = np.cumsum(prod, axis=1, dtype=np.float32)[:, -1]
    return out


def build():
    n, k = 19, 128
    x1 = trunc_bf16((np.arange(k, dtype=np.float32) - 63.0) * np.float32(0.003)).reshape(1, k)
    p1 = packed_words(n, k, 3, 5)
    s1 = np.full(n * k // 64, trunc_bf16(np.float32(0.0125)), np.uint16)
    b1 = np.full(n * k // 64, trunc_bf16(np.float32(-0.08)), np.uint16)
    m = 3
    rows = np.arange(m * k) // k
    cols = np.arange(m * k) % k
    x3 = trunc_bf16((cols.astype(np.float32) - 61.0 + rows.astype(np.float32) * 7.0) * np.float32(0.0025)).reshape(m, k)
    p3 = packed_words(n, k, 7, 3)
    s3 = np.full(n * k // 64, trunc_bf16(np.float32(0.011)), np.uint16)
    b3 = np.full(n * k // 64, trunc_bf16(np.float32(-0.075)), np.uint16)
    return {
        "m1_x": x1, "m1_packed": p1, "m1_scales": s1, "m1_biases": b1,
        "m1_expected": expected_fold(x1, p1, s1, b1),
        "m3_x": x3, "m3_packed": p3, "m3_scales": s3, "m3_biases": b3,
        "m3_expected": expected_fold(x3, p3, s3, b3),
    }


if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "qmv_reference_tests.npz")
    np.savez_compressed(out, **build())
    print("wrote", out)
