"""GPU parity of lisa_attn_decode_batch (one M=1 decode step of one layer for
many sequences in three launches) against lisa_attn_decode run per sequence
and against the oracle: BASELINE config 3's shape (64 sequences, seeded
contexts, several layers) at reduced context lengths, chunk-boundary
contexts, f32 and bf16 inputs, and the argument errors."""
import numpy as np
import pytest

import oracle as O
from helpers import KROW, OROW, QROW, assert_argmax_agrees, assert_close_bf16, layer_inputs, norm_weights

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, to_bits, weights  # noqa: E402


def _fill(runner, layers, filled, gen):
    for layer in range(layers):
        kc, vc = runner.kv_cache(layer)
        for c in (kc, vc):
            c.zero_()
            c[:, :filled].copy_(torch.randn((4, filled, 256), generator=gen, device="cuda").to(torch.bfloat16))


def _case(ctxs, layers, seed, dtype=torch.float32, check_oracle=()):
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    n = len(ctxs)
    runs = [lisa_attn.AttnRunner(layers, c + 2) for c in ctxs]   # batched
    refs = [lisa_attn.AttnRunner(layers, c + 2) for c in ctxs]   # one call per sequence
    for a, b, c in zip(runs, refs, ctxs):
        _fill(a, layers, c - 1, gen)
        for layer in range(layers):
            for x, y in zip(a.kv_cache(layer), b.kv_cache(layer)):
                y.copy_(x)
    bases = [c - 1 for c in ctxs]
    bd = lisa_attn.BatchDecoder(n, sum(c + 2 for c in ctxs))
    for layer in range(layers):
        q, k, v = layer_inputs(rng, n)
        tq, tk, tv = dev_inputs(q, k, v, dtype)
        kc_before = [r.kv_cache(layer) for r in runs]
        host_caches = [(to_bits(kk).copy(), to_bits(vv).copy()) for kk, vv in kc_before] if check_oracle else None
        got = to_bits(bd.decode(runs, layer, bases, tq, tk, tv, w))
        bd.check_device_error()
        for i, (r, base) in enumerate(zip(refs, bases)):
            want = to_bits(r.decode_layer(layer, base, 1, tq[i:i + 1], tk[i:i + 1], tv[i:i + 1], w))
            assert_close_bf16(got[i:i + 1], want, f"seq {i} ctx {ctxs[i]} layer {layer}")
            ka, va = runs[i].kv_cache(layer)
            kb, vb = r.kv_cache(layer)
            assert torch.equal(va, vb), f"V append seq {i}"
            dk = (ka.float() - kb.float()).abs().max().item()
            assert dk <= 2 ** -7 * kb.float().abs().max().item(), f"K append seq {i}"
        for i in check_oracle:
            kh, vh = host_caches[i]
            want = O.attention_layer(q[i:i + 1], k[i:i + 1], v[i:i + 1], bases[i], qn, kn, kh, vh, sliced=True)
            assert_close_bf16(got[i:i + 1], want, f"oracle seq {i}")
            assert assert_argmax_agrees(got[i:i + 1], want, "argmax") == 0
    return got


def test_batch_chunk_edges():
    _case([1, 2, 63, 64, 65, 447, 448, 449, 896, 897, 1000, 5000, 16385], 2, 11, check_oracle=(0, 7, 12))


def test_batch_bf16_inputs():
    _case([100, 3000, 7777], 1, 12, dtype=torch.bfloat16, check_oracle=(1,))


def test_config3_shape_64_sequences():
    """Config 3's batch: 64 sequences with seeded contexts (U[1024, 32768]
    scaled down by 8 to keep the test small), 3 stacked layers."""
    rng = np.random.default_rng(0x5EED + 3)
    ctxs = (rng.integers(1024, 32769, size=64) // 8).tolist()
    _case(ctxs, 3, 13, check_oracle=(0, 31, 63))


def test_batch_errors():
    lib = lisa_attn.load_library()
    rng = np.random.default_rng(14)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    runs = [lisa_attn.AttnRunner(1, 1000) for _ in range(2)]
    tq, tk, tv = dev_inputs(*layer_inputs(rng, 2))
    bd = lisa_attn.BatchDecoder(2, 1000)  # too little scratch for two 1000-position sequences at the end
    with pytest.raises(lisa_attn.LisaError) as e:
        bd.decode(runs, 0, [999, 999], tq, tk, tv, w)
    assert e.value.status == lisa_attn.E2BIG
    bd = lisa_attn.BatchDecoder(2, 2000)
    with pytest.raises(lisa_attn.LisaError) as e:
        bd.decode(runs, 0, [1000, 5], tq, tk, tv, w)
    assert e.value.status == lisa_attn.ENOSPC
    with pytest.raises(lisa_attn.LisaError) as e:
        bd.decode(runs, 1, [5, 5], tq, tk, tv, w)
    assert e.value.status == lisa_attn.EINVAL
    bd.decode(runs, 0, [5, 900], tq, tk, tv, w)
    bd.check_device_error()
    assert lib.lisa_attn_batch_create(0, 0, 10, None) == lisa_attn.EINVAL
