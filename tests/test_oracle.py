"""CPU: pin the oracle against the reference tests' own CPU expectations
(tests/golden/reference_tests.npz, from tests/golden/make_golden.py) and
check its internal consistency the way lisa-rs's tests do."""
import os

import numpy as np
import pytest

import oracle as O
from helpers import HD, KVH, KROW, QH, QROW, layer_inputs, norm_weights, random_cache

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_tests.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def gen_f16(seed, items):
    import make_golden

    return make_golden.gen_f16(seed, items)


@pytest.mark.parametrize("sliced", [True, False])
def test_sliced_golden(gold, sliced):
    """tests/attn_sliced.rs:132-191: sliced and serial attention vs the CPU
    softmax for ctx in {1,16,63,64,129,1000}, tolerance 1e-4."""
    for ci, ctx in enumerate(gold["sliced_ctx"]):
        ctx = int(ctx)
        q = gen_f16(1, QH * HD)
        k = gen_f16(2, KVH * ctx * HD).reshape(KVH, ctx, HD)
        v = gen_f16(3, KVH * ctx * HD).reshape(KVH, ctx, HD)
        out = O.sdpa(q, k, v, ctx - 1, sliced=sliced)[0][:, gold["sliced_dims"]]
        assert np.abs(out - gold["sliced_expected"][ci]).max() < 1e-4, ctx


def test_sliced_batch3_row2_bit_identical():
    """tests/attn_sliced.rs:186-187: row 2 of a batch-3 dispatch equals the
    standalone M=1 row bit for bit."""
    for ctx in [16, 63, 64, 129, 1000]:
        q = gen_f16(1, QH * HD)
        k = gen_f16(2, KVH * ctx * HD).reshape(KVH, ctx, HD)
        v = gen_f16(3, KVH * ctx * HD).reshape(KVH, ctx, HD)
        single = O.sdpa(q, k, v, ctx - 1, sliced=True)[0]
        triple = O.sdpa(np.tile(q, 3), k, v, ctx - 3, sliced=True)[2]
        assert np.array_equal(single.view(np.uint32), triple.view(np.uint32))


def test_block3_causal_golden(gold):
    """tests/attn_cache.rs:194-292: block-3 rows are causal over old and new
    cache rows (capacity 6, base 3), tolerance 2e-5."""
    import make_golden

    qb, kb, vb = make_golden.block3_inputs()
    out = O.sdpa(qb.reshape(3, QH, HD), kb.reshape(KVH, 6, HD), vb.reshape(KVH, 6, HD), 3, sliced=False)
    assert np.abs(out[:, :, gold["block3_dims"]] - gold["block3_expected"]).max() < 2e-5


def test_persistent_cache_matches_legacy_batch():
    """tests/attn_cache.rs:14-192: q/k norm+RoPE, KV append and cached decode of
    the last token equal the legacy batch path's last row (max abs 2e-5)."""
    L = 16
    iq = np.arange(L * QROW)
    ik = np.arange(L * KROW)
    q = (((iq % 113).astype(np.float32) - 56.0) * np.float32(0.01)).astype(np.float32).reshape(L, QROW)
    k = (((ik % 97).astype(np.float32) - 48.0) * np.float32(0.012)).astype(np.float32).reshape(L, KROW)
    v = (((ik % 89).astype(np.float32) - 44.0) * np.float32(0.008)).astype(np.float32).reshape(L, KROW)
    gain = O.f32_to_bf16_trunc(np.ones(HD, np.float32))
    legacy = O.legacy_batch(q, k, v, gain, gain)
    kc = np.zeros((KVH, L, HD), np.uint16)
    vc = np.zeros((KVH, L, HD), np.uint16)
    for pos in range(L):
        O.kv_append(k[pos], v[pos], pos, gain, kc, vc)
    query, _ = O.q_prologue(q[L - 1], L - 1, gain)
    out = O.sdpa(query, kc, vc, L - 1, sliced=False)[0]
    assert np.abs(out - legacy[L - 1]).max() < 2e-5


def test_serial_and_sliced_agree_on_random_layer():
    rng = np.random.default_rng(7)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, 3)
    kc, vc = random_cache(rng, 700, 697)
    kc2, vc2 = kc.copy(), vc.copy()
    a = O.attention_layer(q, k, v, 697, qn, kn, kc, vc, sliced=True)
    b = O.attention_layer(q, k, v, 697, qn, kn, kc2, vc2, sliced=False)
    assert np.array_equal(kc, kc2) and np.array_equal(vc, vc2)
    fa, fb = O.bf16_to_f32(a), O.bf16_to_f32(b)
    assert np.abs(fa - fb).max() <= 2 ** -7 * np.abs(fb).max() + 1e-6


def test_append_skips_rows_past_capacity():
    """attention.metal:172: a row at pos >= capacity is not stored."""
    rng = np.random.default_rng(3)
    _, kn = norm_weights(rng)
    _, k, v = layer_inputs(rng, 3)
    kc, vc = random_cache(rng, 5, 0)
    O.kv_append(k, v, 3, kn, kc, vc)
    assert kc[:, 3].any() and kc[:, 4].any() and not kc[:, :3].any()


def test_rope_position_zero_is_identity_rotation():
    rng = np.random.default_rng(4)
    qn, _ = norm_weights(rng)
    q, _, _ = layer_inputs(rng, 1)
    query, gate = O.q_prologue(q, 0, qn)
    x = O.bf16_to_f32(O.f32_to_bf16(q[0].reshape(QH, 512)[:, :HD]))
    inv = 1.0 / np.sqrt((x * x).sum(1, keepdims=True) / 256.0 + 1e-6)
    want = x * inv * O.bf16_to_f32(qn)[None]
    assert np.abs(O.bf16_to_f32(query[0]) - want).max() < 2e-2
    assert np.array_equal(gate[0], O.bf16_to_f32(O.f32_to_bf16(q[0].reshape(QH, 512)[:, HD:])))


def test_qmv_oracle_matches_reference_kat():
    """tests/qmv.rs:5-220: the affine-u4 QMV known-answer cases (M=1 and the
    3-row wide variant, N=19 with a tail, K=128) at the reference tolerance."""
    g = np.load(os.path.join(os.path.dirname(GOLD), "qmv_reference_tests.npz"))
    for pre in ("m1", "m3"):
        got = O.q4_qmv(g[pre + "_x"], g[pre + "_packed"], g[pre + "_scales"], g[pre + "_biases"])
        assert np.abs(got - g[pre + "_expected"]).max() < 2e-4, pre
