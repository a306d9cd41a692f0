"""GPU: lisa_attn_decode_noalloc, the decode entry point for callers that may
not allocate device memory while they run (engines that reserve all GPU memory
in a pool at start-up). It must give the same gated output as
lisa_attn_decode on the same cache and inputs, for two calls in a row (the
second call reuses the fixed scratch the first one left behind).

This file is collected last on purpose, so a run that stops at the first
failure has run every other test before it."""
import ctypes

import numpy as np
import pytest

from helpers import OROW, assert_close_bf16, layer_inputs, norm_weights, random_cache

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, load_cache, to_bits, weights  # noqa: E402


def _noalloc(lib, kc, vc, cap, base, rows, q, k, v, w, out):
    dt = lisa_attn.DTYPE_BF16 if q.dtype == torch.bfloat16 else lisa_attn.DTYPE_F32
    return lib.lisa_attn_decode_noalloc(kc.data_ptr(), vc.data_ptr(), cap, base, rows, dt,
                                        q.data_ptr(), k.data_ptr(), v.data_ptr(), w.q_norm.data_ptr(),
                                        w.k_norm.data_ptr(), ctypes.c_float(1e-6), out.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_decode_on_two_calls():
    lib = lisa_attn.load_library()
    cap = 5000
    rng = np.random.default_rng(2024)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc0, vc0 = random_cache(rng, cap, 4000)
    ref = lisa_attn.AttnRunner(1, cap)      # existing entry point, context-owned cache
    load_cache(ref, 0, kc0, vc0)
    own = lisa_attn.AttnRunner(1, cap)      # a cache owned by "the caller"
    load_cache(own, 0, kc0, vc0)
    k_own, v_own = own.kv_cache(0)
    for base, rows in [(3999, 1), (4000, 3)]:   # two calls in a row
        q, k, v = layer_inputs(rng, rows)
        tq, tk, tv = dev_inputs(q, k, v)
        want = to_bits(ref.decode_layer(0, base, rows, tq, tk, tv, w))
        out = torch.empty((rows, OROW), dtype=torch.bfloat16, device="cuda")
        assert _noalloc(lib, k_own, v_own, cap, base, rows, tq, tk, tv, w, out) == lisa_attn.OK
        torch.cuda.synchronize()
        got = to_bits(out)
        assert_close_bf16(got, want, f"noalloc base={base} rows={rows}")
    torch.cuda.synchronize()
    assert torch.equal(k_own, ref.kv_cache(0)[0]) and torch.equal(v_own, ref.kv_cache(0)[1])


def test_noalloc_rejects_requests_beyond_its_scratch():
    lib = lisa_attn.load_library()
    cap = lisa_attn.NOALLOC_MAX_POSITIONS + 8
    kc = torch.zeros((4, cap, 256), dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    rng = np.random.default_rng(1)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    tq, tk, tv = dev_inputs(*layer_inputs(rng, 1))
    out = torch.empty((1, OROW), dtype=torch.bfloat16, device="cuda")
    assert _noalloc(lib, kc, vc, cap, lisa_attn.NOALLOC_MAX_POSITIONS, 1, tq, tk, tv, w, out) == lisa_attn.E2BIG
    assert _noalloc(lib, kc, vc, cap, cap - 1, 3, tq, tk, tv, w, out) == lisa_attn.ENOSPC
    assert _noalloc(lib, kc, vc, cap, 10, 2, tq, tk, tv, w, out) == lisa_attn.EINVAL


@pytest.mark.parametrize("cap,filled,calls", [
    # the largest request the fixed scratch holds (base + rows == 16384), twice
    (16384, 16381, [(16381, 3), (16383, 1)]),
    # a verify whose rows straddle a 448-position chunk boundary, then M=1
    (1000, 446, [(446, 3), (449, 1)]),
])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_noalloc_edges_match_decode(cap, filled, calls, dtype):
    lib = lisa_attn.load_library()
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    rng = np.random.default_rng(cap + filled)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc0, vc0 = random_cache(rng, cap, filled)
    ref = lisa_attn.AttnRunner(1, cap)
    load_cache(ref, 0, kc0, vc0)
    own = lisa_attn.AttnRunner(1, cap)
    load_cache(own, 0, kc0, vc0)
    k_own, v_own = own.kv_cache(0)
    for base, rows in calls:
        tq, tk, tv = dev_inputs(*layer_inputs(rng, rows), tdt)
        want = to_bits(ref.decode_layer(0, base, rows, tq, tk, tv, w))
        out = torch.empty((rows, OROW), dtype=torch.bfloat16, device="cuda")
        assert _noalloc(lib, k_own, v_own, cap, base, rows, tq, tk, tv, w, out) == lisa_attn.OK
        assert lib.lisa_attn_noalloc_check_device_error() == lisa_attn.OK
        assert np.array_equal(to_bits(out), want), f"base={base} rows={rows}"


def test_noalloc_reports_device_timeout_then_recovers():
    """A bounded wait that runs out inside a no-alloc call is reported by
    lisa_attn_noalloc_check_device_error (the call itself returned before the
    kernel ran); the next call is correct."""
    lib = lisa_attn.load_library()
    cap = 3000
    rng = np.random.default_rng(77)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc0, vc0 = random_cache(rng, cap, 2500)
    ref = lisa_attn.AttnRunner(1, cap)
    load_cache(ref, 0, kc0, vc0)
    own = lisa_attn.AttnRunner(1, cap)
    load_cache(own, 0, kc0, vc0)
    k_own, v_own = own.kv_cache(0)
    tq, tk, tv = dev_inputs(*layer_inputs(rng, 1))
    out = torch.empty((1, OROW), dtype=torch.bfloat16, device="cuda")
    assert lib.lisa_attn_debug_wait_fault(1000, 1) == lisa_attn.OK
    try:
        assert _noalloc(lib, k_own, v_own, cap, 2500, 1, tq, tk, tv, w, out) == lisa_attn.OK
        assert lib.lisa_attn_noalloc_check_device_error() == lisa_attn.ETIMEOUT
    finally:
        assert lib.lisa_attn_debug_wait_fault(0, 0) == lisa_attn.OK
    assert lib.lisa_attn_noalloc_check_device_error() == lisa_attn.OK
    want = to_bits(ref.decode_layer(0, 2500, 1, tq, tk, tv, w))
    assert _noalloc(lib, k_own, v_own, cap, 2500, 1, tq, tk, tv, w, out) == lisa_attn.OK
    assert lib.lisa_attn_noalloc_check_device_error() == lisa_attn.OK
    assert np.array_equal(to_bits(out), want)
