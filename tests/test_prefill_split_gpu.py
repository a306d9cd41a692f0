"""GPU parity of the split prefill grid: (query pair, head) units run as two
clusters over consecutive key ranges whose partials merge (the first cluster
to finish stores its unnormalised O, max and sum; the second folds them in).
Forced on with lisa_attn_debug_prefill_split(ALWAYS) so small chunks take the
merge path; the deep chunk also runs with the planner's own choice and with
splitting off."""
import numpy as np
import pytest

import oracle as O
from helpers import HD, assert_argmax_agrees, assert_close_bf16, layer_inputs, norm_weights, random_cache

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, load_cache, to_bits, weights  # noqa: E402
from test_prefill_gpu import gpu_prefill  # noqa: E402

AUTO, NEVER, ALWAYS = 0, 1, 2


@pytest.fixture
def split_mode():
    lib = lisa_attn.load_library()
    yield lambda mode: lib.lisa_attn_debug_prefill_split(mode)
    lib.lisa_attn_debug_prefill_split(AUTO)


def test_split_mode_api(split_mode):
    assert split_mode(ALWAYS) == AUTO
    assert split_mode(NEVER) == ALWAYS
    assert split_mode(7) == lisa_attn.EINVAL
    assert split_mode(-1) == lisa_attn.EINVAL
    assert split_mode(AUTO) == NEVER


def oracle_chunks(q, k, v, qn, kn, chunks, capacity):
    kc = np.zeros((4, capacity, HD), np.uint16)
    vc = np.zeros((4, capacity, HD), np.uint16)
    want, pos = [], 0
    for m in chunks:
        want.append(O.attention_layer(q[pos:pos + m], k[pos:pos + m], v[pos:pos + m], pos, qn, kn, kc, vc,
                                      sliced=False))
        pos += m
    return np.concatenate(want)


@pytest.mark.parametrize("chunks", [[512] * 8, [300, 200, 13, 1], [512, 129], [256, 256, 256, 256, 1]])
def test_forced_split_matches_oracle(split_mode, chunks):
    """Every row of every chunk against the oracle, and the same bits on a
    second run (the merge is symmetric in its two segments, so which one
    finishes first does not show)."""
    split_mode(ALWAYS)
    n = sum(chunks)
    rng = np.random.default_rng(0x5EED + 2 + n)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, n)
    got, _ = gpu_prefill(q, k, v, qn, kn, chunks, n, torch.bfloat16)
    again, _ = gpu_prefill(q, k, v, qn, kn, chunks, n, torch.bfloat16)
    assert np.array_equal(got, again)
    want = oracle_chunks(q, k, v, qn, kn, chunks, n)
    assert_close_bf16(got, want, f"split {chunks}")
    assert_argmax_agrees(got, want, f"split {chunks}", exact=False)


def test_forced_split_f32_and_bf16_inputs_identical(split_mode):
    split_mode(ALWAYS)
    rng = np.random.default_rng(79)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, 1024)
    a, _ = gpu_prefill(q, k, v, qn, kn, [512, 512], 1024, torch.float32)
    b, _ = gpu_prefill(q, k, v, qn, kn, [512, 512], 1024, torch.bfloat16)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("mode", [AUTO, NEVER, ALWAYS])
def test_deep_chunk_each_mode(split_mode, mode):
    """A 512-row chunk at base 16384 over a filled cache (the planner splits
    it: 129-tile units) with the planner's choice, splitting off and forced."""
    split_mode(mode)
    cap, base, m = 16896, 16384, 512
    rng = np.random.default_rng(0x5EED + 16)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    kc, vc = random_cache(rng, cap, base)
    r = lisa_attn.AttnRunner(1, cap)
    load_cache(r, 0, kc, vc)
    r.restore_position(base)
    q, k, v = layer_inputs(rng, m)
    got = to_bits(r.forward_prefill(0, *dev_inputs(q, k, v), w))
    torch.cuda.synchronize()
    r.check_device_error()
    want = O.attention_layer(q, k, v, base, qn, kn, kc, vc, sliced=False)
    assert_close_bf16(got, want, f"chunk at {base}, mode {mode}")
    assert_argmax_agrees(got, want, f"chunk at {base}, mode {mode}", exact=False)
