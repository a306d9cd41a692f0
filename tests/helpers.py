"""Shared test helpers: seeded synthetic inputs with the BASELINE.json
distributions, oracle runs, and the north-star tolerance check."""
from __future__ import annotations

import numpy as np

import oracle as O

QH, KVH, HD = 24, 4, 256
QROW, KROW, OROW = QH * 512, KVH * HD, QH * HD
ATOL, RTOL = 8e-3, 1e-2  # north-star tolerance on bf16 outputs


def bf16_round(x: np.ndarray) -> np.ndarray:
    return O.bf16_to_f32(O.f32_to_bf16(np.asarray(x, np.float32)))


def norm_weights(rng: np.random.Generator):
    """1 + N(0, 0.02) as bf16 bits."""
    qn = O.f32_to_bf16((1.0 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    kn = O.f32_to_bf16((1.0 + 0.02 * rng.standard_normal(HD)).astype(np.float32))
    return qn, kn


def layer_inputs(rng: np.random.Generator, rows: int):
    """q_gate [rows, 12288], k, v [rows, 1024]: N(0,1) rounded to bf16 (f32 arrays)."""
    q = bf16_round(rng.standard_normal((rows, QROW)).astype(np.float32))
    k = bf16_round(rng.standard_normal((rows, KROW)).astype(np.float32))
    v = bf16_round(rng.standard_normal((rows, KROW)).astype(np.float32))
    return q, k, v


def random_cache(rng: np.random.Generator, capacity: int, filled: int):
    """K/V caches [4, capacity, 256] bf16 bits; rows < filled ~ N(0,1)
    (post-norm, post-RoPE values drawn directly), the rest zero."""
    kc = np.zeros((KVH, capacity, HD), np.uint16)
    vc = np.zeros((KVH, capacity, HD), np.uint16)
    if filled:
        kc[:, :filled] = O.f32_to_bf16(rng.standard_normal((KVH, filled, HD)).astype(np.float32))
        vc[:, :filled] = O.f32_to_bf16(rng.standard_normal((KVH, filled, HD)).astype(np.float32))
    return kc, vc


def assert_close_bf16(got_bits: np.ndarray, want_bits: np.ndarray, what: str = ""):
    g = O.bf16_to_f32(got_bits).astype(np.float64)
    w = O.bf16_to_f32(want_bits).astype(np.float64)
    assert np.all(np.isfinite(g)), f"{what}: non-finite output"
    err = np.abs(g - w)
    bad = err > np.maximum(ATOL, RTOL * np.abs(w))
    assert not bad.any(), (f"{what}: {bad.sum()} of {bad.size} outside tolerance; max abs err "
                           f"{err.max():.3e} at {np.unravel_index(err.argmax(), err.shape)}")
    return float(err.max())


def projection_logits(gated_bits: np.ndarray, seed: int = 1234, n_out: int = 1024) -> np.ndarray:
    """A seeded synthetic projection of each row: [rows, 6144] @ W[6144, n_out]."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((OROW, n_out)).astype(np.float64)
    return O.bf16_to_f32(gated_bits).reshape(-1, OROW).astype(np.float64) @ w


def argmax_projection(gated_bits: np.ndarray, seed: int = 1234, n_out: int = 1024) -> np.ndarray:
    return np.argmax(projection_logits(gated_bits, seed, n_out), axis=1)


FLIP_LOG: list[dict] = []  # every argmax disagreement seen in this process (what, row, gap, perturbation)


def assert_argmax_agrees(got_bits: np.ndarray, want_bits: np.ndarray, what: str = "", exact: bool = True) -> int:
    """The north star's exact-argmax check on a synthetic projection of every
    row. exact=True (every BASELINE config): no row may disagree. exact=False
    (off-config edge cases): a row may only disagree where the oracle's own
    top two logits are closer than twice the logit perturbation between the
    two outputs (a tie at the output tolerance), at most 1 % of rows. Every
    disagreement is logged in FLIP_LOG and printed with its gap; returns the
    number of disagreeing rows."""
    lg, lw = projection_logits(got_bits), projection_logits(want_bits)
    ag, aw = lg.argmax(1), lw.argmax(1)
    diff = ag != aw
    rows = np.nonzero(diff)[0]
    pert = np.abs(lg - lw).max(1)
    for r in rows:
        rec = {"what": what, "row": int(r), "gap": float(lw[r, aw[r]] - lw[r, ag[r]]), "perturbation": float(pert[r])}
        FLIP_LOG.append(rec)
        print(f"argmax flip: {rec}")
    if exact:
        assert not diff.any(), f"{what}: argmax differs in {diff.sum()} of {diff.size} rows: {FLIP_LOG[-len(rows):]}"
        return 0
    gap = lw[rows, aw[rows]] - lw[rows, ag[rows]]
    bad = gap > 2 * pert[rows]
    assert not bad.any(), f"{what}: argmax differs beyond ties in rows {rows[bad][:10]}"
    assert diff.sum() <= max(1, 0.01 * diff.size), f"{what}: too many tie flips ({diff.sum()})"
    return int(diff.sum())
