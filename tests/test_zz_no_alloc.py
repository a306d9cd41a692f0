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
    return lib.lisa_attn_decode_noalloc(kc.data_ptr(), vc.data_ptr(), cap, base, rows, lisa_attn.DTYPE_F32,
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
