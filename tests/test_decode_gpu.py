"""GPU parity of the split-KV decode / verify path (C ABI) against the oracle,
plus the lisa-rs invariants: M=1 == M=3 rows bit for bit, the trim/commit
rollback contract, bounds errors."""
import numpy as np
import pytest

import oracle as O
from helpers import (HD, KVH, OROW, assert_argmax_agrees, assert_close_bf16, layer_inputs, norm_weights,
                     random_cache)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, load_cache, read_cache, to_bits, weights  # noqa: E402


def run_case(seed, capacity, base, rows, dtype=torch.float32):
    """GPU and oracle on the same seeded layer; returns (gpu bits, oracle bits,
    gpu caches, oracle caches)."""
    rng = np.random.default_rng(seed)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, rows)
    kc, vc = random_cache(rng, capacity, base)
    r = lisa_attn.AttnRunner(1, capacity)
    load_cache(r, 0, kc, vc)
    tq, tk, tv = dev_inputs(q, k, v, dtype)
    out = r.decode_layer(0, base, rows, tq, tk, tv, weights(qn, kn))
    torch.cuda.synchronize()
    r.check_device_error()
    gk, gv = read_cache(r, 0)
    want = O.attention_layer(q, k, v, base, qn, kn, kc, vc, sliced=True)
    return to_bits(out), want, (gk, gv), (kc, vc)


def test_config0_decode_ctx2048():
    """M=1 at position 2047 over a 2047-row cache."""
    got, want, (gk, gv), (kc, vc) = run_case(0x5EED, 2048, 2047, 1)
    assert_close_bf16(got, want, "config0")
    assert_argmax_agrees(got, want, "argmax")
    assert np.array_equal(gv, vc)  # V append is a pure rounding
    kd = np.abs(O.bf16_to_f32(gk[:, 2047]) - O.bf16_to_f32(kc[:, 2047]))
    assert kd.max() <= 2 ** -7 * np.abs(O.bf16_to_f32(kc[:, 2047])).max()
    assert np.array_equal(gk[:, :2047], kc[:, :2047])


def test_bf16_and_f32_inputs_identical():
    a, *_ = run_case(11, 600, 555, 1, torch.float32)
    b, *_ = run_case(11, 600, 555, 1, torch.bfloat16)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("ctx", [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 255, 1000, 16384, 16385, 32768])
def test_decode_context_edges(ctx):
    got, want, *_ = run_case(100 + ctx, ctx + 5, ctx - 1, 1)
    assert_close_bf16(got, want, f"ctx={ctx}")


@pytest.mark.parametrize("base", [0, 1, 125, 126, 127, 8189])
def test_verify_m3(base):
    """BASELINE config 1 (base 8189) and chunk-boundary straddles."""
    got, want, *_ = run_case(200 + base, base + 3, base, 3)
    assert_close_bf16(got, want, f"verify base={base}")
    assert_argmax_agrees(got, want, f"verify base={base}")


@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4, 5])
def test_config1_verify_trim_rerun(seed):
    """BASELINE config 1 as written: M=3 verify at positions 8189..8191 over an
    8189-token cache; then the KV is trimmed to a seeded accepted prefix of 1,
    2 or 3 rows (commit_verified_prefix) and the verify re-runs at the new
    position; both verifies against the oracle, whose cache received only the
    accepted rows of the first."""
    rng = np.random.default_rng(0x5EED + 1 + 100 * seed)
    accepted = int(rng.integers(1, 4))
    base = 8189
    cap = base + 6
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc, vc = random_cache(rng, cap, base)
    r = lisa_attn.AttnRunner(1, cap)
    load_cache(r, 0, kc, vc)
    r.restore_position(base)
    qa, ka, va = layer_inputs(rng, 3)
    got_a = to_bits(r.verify_block3(0, *dev_inputs(qa, ka, va), w))
    r.advance(3, verify=True)
    kco, vco = kc.copy(), vc.copy()
    want_a = O.attention_layer(qa, ka, va, base, qn, kn, kco, vco, sliced=True)
    assert_close_bf16(got_a, want_a, "config 1 first verify")
    assert_argmax_agrees(got_a, want_a, "config 1 first verify")
    r.commit_verified_prefix(accepted)
    assert r.position() == base + accepted
    # the oracle's cache holds only the accepted rows (rejected rows are
    # overwritten by the re-run, as in runner.rs:911-944)
    kco, vco = kc.copy(), vc.copy()
    O.attention_layer(qa[:accepted], ka[:accepted], va[:accepted], base, qn, kn, kco, vco, sliced=True)
    qb, kb, vb = layer_inputs(rng, 3)
    got_b = to_bits(r.verify_block3(0, *dev_inputs(qb, kb, vb), w))
    r.advance(3, verify=True)
    r.check_device_error()
    want_b = O.attention_layer(qb, kb, vb, base + accepted, qn, kn, kco, vco, sliced=True)
    assert_close_bf16(got_b, want_b, f"config 1 re-run after accepting {accepted}")
    assert_argmax_agrees(got_b, want_b, f"config 1 re-run after accepting {accepted}")
    gk, gv = read_cache(r, 0)
    assert np.array_equal(gv[:, :base + accepted + 3], vco[:, :base + accepted + 3])


@pytest.mark.parametrize("base", [3, 126, 127, 128, 1000, 8189])
def test_verify_rows_bit_identical_to_sequential_decode(base):
    """tests/attn_sliced.rs:186-187, strengthened to all three rows: verify rows
    equal the same rows decoded one at a time, bit for bit, and leave the same
    cache."""
    rng = np.random.default_rng(300 + base)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, 3)
    kc, vc = random_cache(rng, base + 3, base)
    w = weights(qn, kn)
    r3 = lisa_attn.AttnRunner(1, base + 3)
    load_cache(r3, 0, kc, vc)
    tq, tk, tv = dev_inputs(q, k, v)
    out3 = to_bits(r3.decode_layer(0, base, 3, tq, tk, tv, w))
    r1 = lisa_attn.AttnRunner(1, base + 3)
    load_cache(r1, 0, kc, vc)
    rows = []
    for i in range(3):
        tq, tk, tv = dev_inputs(q[i:i + 1], k[i:i + 1], v[i:i + 1])
        rows.append(to_bits(r1.decode_layer(0, base + i, 1, tq, tk, tv, w)))
    assert np.array_equal(out3, np.concatenate(rows))
    assert np.array_equal(read_cache(r3, 0)[0], read_cache(r1, 0)[0])


@pytest.mark.parametrize("accepted", [1, 2, 3])
def test_verify_commit_rollback_then_decode(accepted):
    """speculative/mod.rs:156-167: verify 3 rows, commit_verified_prefix(rows),
    decode the next token; equal to a fresh sequential run that only saw the
    accepted rows (stale KV rows are overwritten, runner.rs:911-944)."""
    base = 777
    rng = np.random.default_rng(400 + accepted)
    qn, kn = norm_weights(rng)
    q3, k3, v3 = layer_inputs(rng, 3)
    qx, kx, vx = layer_inputs(rng, 1)
    kc, vc = random_cache(rng, base + 8, base)
    w = weights(qn, kn)
    r = lisa_attn.AttnRunner(1, base + 8)
    load_cache(r, 0, kc, vc)
    r.restore_position(base)
    r.verify_block3(0, *dev_inputs(q3, k3, v3), w)
    r.advance(3, verify=True)
    assert r.position() == base + 3
    r.commit_verified_prefix(accepted)
    assert r.position() == base + accepted
    got = to_bits(r.forward_decode(0, *dev_inputs(qx, kx, vx), w))
    r.advance(1)

    fresh = lisa_attn.AttnRunner(1, base + 8)
    load_cache(fresh, 0, kc, vc)
    fresh.restore_position(base)
    for i in range(accepted):
        fresh.forward_decode(0, *dev_inputs(q3[i:i + 1], k3[i:i + 1], v3[i:i + 1]), w)
        fresh.advance(1)
    want = to_bits(fresh.forward_decode(0, *dev_inputs(qx, kx, vx), w))
    assert np.array_equal(got, want)
    # and against the oracle
    kco, vco = kc.copy(), vc.copy()
    for i in range(accepted):
        O.attention_layer(q3[i], k3[i], v3[i], base + i, qn, kn, kco, vco)
    assert_close_bf16(got, O.attention_layer(qx, kx, vx, base + accepted, qn, kn, kco, vco), "rollback")


def test_position_contract_errors():
    r = lisa_attn.AttnRunner(2, 64)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.commit_verified_prefix(1)
    assert e.value.status == lisa_attn.ESTATE
    r.advance(3, verify=True)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.commit_verified_prefix(4)
    assert e.value.status == lisa_attn.EINVAL
    with pytest.raises(lisa_attn.LisaError):  # consumed by the failed commit (take())
        r.commit_verified_prefix(1)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.trim_state(4)
    assert e.value.status == lisa_attn.ESTATE
    r.trim_state(2)
    assert r.position() == 1
    with pytest.raises(lisa_attn.LisaError):
        r.set_position(5)
    r.set_position(0)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.restore_position(65)
    assert e.value.status == lisa_attn.ENOSPC
    r.restore_position(63)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.advance(3, verify=True)
    assert e.value.status == lisa_attn.ENOSPC


def test_dispatch_argument_errors():
    rng = np.random.default_rng(5)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    r = lisa_attn.AttnRunner(1, 64)
    q, k, v = layer_inputs(rng, 2)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.decode_layer(0, 0, 2, *dev_inputs(q, k, v), w)
    assert e.value.status == lisa_attn.EINVAL
    q, k, v = layer_inputs(rng, 3)
    with pytest.raises(lisa_attn.LisaError) as e:
        r.decode_layer(0, 62, 3, *dev_inputs(q, k, v), w)
    assert e.value.status == lisa_attn.ENOSPC
    with pytest.raises(lisa_attn.LisaError) as e:
        r.decode_layer(1, 0, 3, *dev_inputs(q, k, v), w)
    assert e.value.status == lisa_attn.EINVAL
    lib = lisa_attn.load_library()
    out = torch.empty((3, OROW), dtype=torch.bfloat16, device="cuda")
    assert lib.lisa_attn_decode(r.handle, 0, 0, 3, 0, None, None, None, None, None, 1e-6, out.data_ptr(),
                                None) == lisa_attn.EINVAL
    assert lib.lisa_attn_decode(r.handle, 0, 0, 3, 7, out.data_ptr(), out.data_ptr(), out.data_ptr(),
                                out.data_ptr(), out.data_ptr(), 1e-6, out.data_ptr(), None) == lisa_attn.EINVAL
    r.check_device_error()


def test_checkpoint_restore_roundtrip():
    """MtpRunner::checkpoint_state / restore_state (runner.rs:2376-2441)."""
    rng = np.random.default_rng(9)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    r = lisa_attn.AttnRunner(1, 300)
    kc, vc = random_cache(rng, 300, 200)
    load_cache(r, 0, kc, vc)
    r.restore_position(200)
    snap = r.checkpoint_state()
    q, k, v = layer_inputs(rng, 1)
    a = to_bits(r.forward_decode(0, *dev_inputs(q, k, v), w))
    r.advance(1)
    q2, k2, v2 = layer_inputs(rng, 1)
    r.forward_decode(0, *dev_inputs(q2, k2, v2), w)
    r.restore_state(snap)
    assert r.position() == 200
    b = to_bits(r.forward_decode(0, *dev_inputs(q, k, v), w))
    assert np.array_equal(a, b)
    r.reset_state()
    assert r.position() == 0
    assert not read_cache(r, 0)[0].any()


def test_multi_layer_offsets():
    """Each layer has its own cache at cache_index * 4 * cap * 256 * 2 bytes
    (runner.rs:1463-1464)."""
    rng = np.random.default_rng(10)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    r = lisa_attn.AttnRunner(3, 500)
    caches = [random_cache(rng, 500, 400) for _ in range(3)]
    for i, (kc, vc) in enumerate(caches):
        load_cache(r, i, kc, vc)
    q, k, v = layer_inputs(rng, 1)
    for i, (kc, vc) in enumerate(caches):
        got = to_bits(r.decode_layer(i, 400, 1, *dev_inputs(q, k, v), w))
        assert_close_bf16(got, O.attention_layer(q, k, v, 400, qn, kn, kc.copy(), vc.copy()), f"layer {i}")
