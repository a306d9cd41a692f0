"""GPU parity of the tcgen05 chunked-prefill path (C ABI) against the oracle."""
import numpy as np
import pytest

import oracle as O
from helpers import (HD, KROW, OROW, QROW, assert_argmax_agrees, assert_close_bf16, layer_inputs, norm_weights,
                     random_cache)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, load_cache, read_cache, to_bits, weights  # noqa: E402


def gpu_prefill(q, k, v, qn, kn, chunks, capacity, dtype=torch.float32):
    r = lisa_attn.AttnRunner(1, capacity)
    w = weights(qn, kn)
    outs = []
    pos = 0
    for m in chunks:
        tq, tk, tv = dev_inputs(q[pos:pos + m], k[pos:pos + m], v[pos:pos + m], dtype)
        outs.append(to_bits(r.forward_prefill(0, tq, tk, tv, w)))
        r.advance(m)
        pos += m
    torch.cuda.synchronize()
    r.check_device_error()
    return np.concatenate(outs), r


def oracle_rows(q, k, v, qn, kn, capacity, sample):
    """Oracle gated output for the sampled rows of a full prefix."""
    n = q.shape[0]
    kc = np.zeros((4, capacity, HD), np.uint16)
    vc = np.zeros((4, capacity, HD), np.uint16)
    O.kv_append(k, v, 0, kn, kc, vc)
    out = {}
    for row in sample:
        query, gate = O.q_prologue(q[row], row, qn)
        o = O.sdpa(query, kc, vc, row, sliced=False)
        out[row] = O.gate_out(o.reshape(1, OROW), gate.reshape(1, OROW))[0]
    return out, kc, vc


@pytest.mark.parametrize("chunks", [[1], [7], [128], [129], [300, 200, 13, 1], [256, 256, 256, 256]])
def test_prefill_matches_oracle(chunks):
    n = sum(chunks)
    rng = np.random.default_rng(1000 + n + len(chunks))
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, n)
    got, r = gpu_prefill(q, k, v, qn, kn, chunks, n + 3)
    kc = np.zeros((4, n + 3, HD), np.uint16)
    vc = np.zeros((4, n + 3, HD), np.uint16)
    want = []
    pos = 0
    for m in chunks:
        want.append(O.attention_layer(q[pos:pos + m], k[pos:pos + m], v[pos:pos + m], pos, qn, kn, kc, vc,
                                      sliced=False))
        pos += m
    want = np.concatenate(want)
    assert_close_bf16(got, want, f"prefill {chunks}")
    assert_argmax_agrees(got, want, f"prefill {chunks}", exact=False)
    gk, gv = read_cache(r, 0)
    assert np.array_equal(gv[:, :n], vc[:, :n])
    kd = np.abs(O.bf16_to_f32(gk[:, :n]) - O.bf16_to_f32(kc[:, :n]))
    assert kd.max() <= 2 ** -7 * np.abs(O.bf16_to_f32(kc[:, :n])).max()


def test_config2_prefill_4096_in_512_chunks():
    """4096 tokens from an empty cache, 8 chunks of 512;
    every one of the 4096 rows against the oracle, and the whole cache."""
    n = 4096
    rng = np.random.default_rng(0x5EED + 2)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, n)
    got, r = gpu_prefill(q, k, v, qn, kn, [512] * 8, n)
    kc = np.zeros((4, n, HD), np.uint16)
    vc = np.zeros((4, n, HD), np.uint16)
    want = np.concatenate([O.attention_layer(q[b:b + 512], k[b:b + 512], v[b:b + 512], b, qn, kn, kc, vc,
                                             sliced=False) for b in range(0, n, 512)])
    assert_close_bf16(got, want, "config 2, all rows")
    flips = assert_argmax_agrees(got, want, "config 2", exact=False)
    print(f"config 2: {flips} argmax tie flips over {n} rows")
    gk, gv = read_cache(r, 0)
    assert np.array_equal(gv, vc)
    kd = np.abs(O.bf16_to_f32(gk) - O.bf16_to_f32(kc))
    assert kd.max() <= 2 ** -7 * np.abs(O.bf16_to_f32(kc)).max()


def test_prefill_chunk_at_32k_then_decode_at_last_position():
    """A 512-row chunk at base 32256 of a 32768-capacity context over a
    filled cache (key tiles up to 256 deep, TMA coordinates near the top of
    the cache), all rows against the oracle; then the last position is
    trimmed and decoded again (M=1 at 32767) over what the prefill wrote."""
    cap, base, m = 32768, 32256, 512
    rng = np.random.default_rng(0x5EED + 32)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc, vc = random_cache(rng, cap, base)
    r = lisa_attn.AttnRunner(1, cap)
    load_cache(r, 0, kc, vc)
    r.restore_position(base)
    q, k, v = layer_inputs(rng, m)
    got = to_bits(r.forward_prefill(0, *dev_inputs(q, k, v), w))
    r.advance(m)
    want = O.attention_layer(q, k, v, base, qn, kn, kc, vc, sliced=False)
    assert_close_bf16(got, want, "chunk at 32256")
    assert_argmax_agrees(got, want, "chunk at 32256", exact=False)
    r.trim_state(1)
    assert r.position() == cap - 1
    q1, k1, v1 = layer_inputs(rng, 1)
    got1 = to_bits(r.forward_decode(0, *dev_inputs(q1, k1, v1), w))
    r.check_device_error()
    want1 = O.attention_layer(q1, k1, v1, cap - 1, qn, kn, kc, vc, sliced=True)
    assert_close_bf16(got1, want1, "decode at 32767")
    assert_argmax_agrees(got1, want1, "decode at 32767")


def test_prefill_then_decode_continues():
    """A prefill followed by M=1 decode uses the cache the prefill wrote."""
    n = 700
    rng = np.random.default_rng(77)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, n + 1)
    _, r = gpu_prefill(q[:n], k[:n], v[:n], qn, kn, [512, 188], n + 1)
    got = to_bits(r.forward_decode(0, *dev_inputs(q[n:], k[n:], v[n:]), weights(qn, kn)))
    want, _, _ = oracle_rows(q, k, v, qn, kn, n + 1, [n])
    assert_close_bf16(got[0], want[n], "decode after prefill")


def test_prefill_bf16_inputs_identical():
    rng = np.random.default_rng(78)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, 200)
    a, _ = gpu_prefill(q, k, v, qn, kn, [200], 200, torch.float32)
    b, _ = gpu_prefill(q, k, v, qn, kn, [200], 200, torch.bfloat16)
    assert np.array_equal(a, b)


def test_prefill_errors():
    rng = np.random.default_rng(79)
    qn, kn = norm_weights(rng)
    r = lisa_attn.AttnRunner(1, 600)
    q, k, v = layer_inputs(rng, 513)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.prefill_layer(0, 0, 513, *dev_inputs(q, k, v), weights(qn, kn))
    assert e.value.status == lisa_attn.EINVAL
    q, k, v = layer_inputs(rng, 100)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.prefill_layer(0, 550, 100, *dev_inputs(q, k, v), weights(qn, kn))
    assert e.value.status == lisa_attn.ENOSPC
