"""GPU: the failure channel of the decode kernels. Every mbarrier wait in the
kernels is bounded; when one runs out the kernel records LISA_ETIMEOUT in an
error word and returns. These tests make a wait run out on purpose through the
test hook lisa_attn_debug_wait_fault (1 ms limit, load warp withholds every
copy: nothing is in flight and nothing is accessed out of bounds), check that
each entry point's error query reports it, and that the next normal call on the
same context / workspace is correct."""
import numpy as np
import pytest

import oracle as O
from helpers import OROW, assert_close_bf16, layer_inputs, norm_weights, random_cache

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
import lisa_split  # noqa: E402
from gpu_util import dev_inputs, load_cache, to_bits, weights  # noqa: E402


class injected_timeout:
    def __enter__(self):
        lib = lisa_attn.load_library()
        assert lib.lisa_attn_debug_wait_fault(1000, 1) == lisa_attn.OK
        return self

    def __exit__(self, *exc):
        assert lisa_attn.load_library().lisa_attn_debug_wait_fault(0, 0) == lisa_attn.OK


def test_debug_hook_argument_checks():
    lib = lisa_attn.load_library()
    assert lib.lisa_attn_debug_wait_fault(0, 1) == lisa_attn.EINVAL
    assert lib.lisa_attn_debug_wait_fault(20_000_000, 0) == lisa_attn.EINVAL
    assert lib.lisa_attn_debug_wait_fault(0, 0) == lisa_attn.OK


@pytest.mark.parametrize("rows", [1, 3])
def test_context_decode_reports_timeout_then_recovers(rows):
    rng = np.random.default_rng(900 + rows)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    base = 2000
    kc, vc = random_cache(rng, base + 3, base)
    r = lisa_attn.AttnRunner(1, base + 3)
    load_cache(r, 0, kc, vc)
    q, k, v = layer_inputs(rng, rows)
    tq, tk, tv = dev_inputs(q, k, v)
    r.check_device_error()
    with injected_timeout():
        r.decode_layer(0, base, rows, tq, tk, tv, w)  # launches fine; the kernel gives up
        with pytest.raises(lisa_attn.LisaError) as e:
            r.check_device_error()
        assert e.value.status == lisa_attn.ETIMEOUT
    r.check_device_error()  # the flag was cleared
    got = to_bits(r.decode_layer(0, base, rows, tq, tk, tv, w))
    r.check_device_error()
    want = O.attention_layer(q, k, v, base, qn, kn, kc.copy(), vc.copy(), sliced=True)
    assert_close_bf16(got, want, "after timeout")


def test_window_decode_reports_timeout_then_recovers():
    rng = np.random.default_rng(950)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    base = 1500
    dec = lisa_split.SplitKVDecoder(lisa_split.Window(0, 0, base + 1), max_rows=1)
    kc, vc = random_cache(rng, base + 1, base)
    dec.k.copy_(torch.from_numpy(kc.view(np.int16)).cuda().view(torch.bfloat16))
    dec.v.copy_(torch.from_numpy(vc.view(np.int16)).cuda().view(torch.bfloat16))
    q, k, v = layer_inputs(rng, 1)
    tq, tk, tv = dev_inputs(q, k, v)
    with injected_timeout():
        lisa_attn.decode_window(dec.k, dec.v, 0, base, 1, tq, tk, tv, w, dec.part_o[:1], dec.part_ml[:1],
                                dec.workspace)
        with pytest.raises(lisa_attn.LisaError) as e:
            lisa_attn.window_check_device_error(dec.workspace)
        assert e.value.status == lisa_attn.ETIMEOUT
    got = to_bits(dec.decode(base, tq, tk, tv, w))
    lisa_attn.window_check_device_error(dec.workspace)
    want = O.attention_layer(q, k, v, base, qn, kn, kc.copy(), vc.copy(), sliced=True)
    assert_close_bf16(got, want, "window after timeout")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_contexts_on_two_devices_in_one_process():
    """The kernels' dynamic shared-memory attribute is a per-device setting:
    decode and prefill must work on a second GPU after the first has run."""
    rng = np.random.default_rng(960)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, 200)
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            w = lisa_attn.AttentionWeights(*(torch.from_numpy(a.view(np.int16)).to(f"cuda:{dev}")
                                             .view(torch.bfloat16) for a in (qn, kn)))
            r = lisa_attn.AttnRunner(1, 256, device=dev)
            conv = [torch.from_numpy(a).to(f"cuda:{dev}") for a in (q, k, v)]
            a = to_bits(r.forward_prefill(0, *conv, w))
            r.advance(200)
            b = to_bits(r.forward_decode(0, *(t[:1].contiguous() for t in conv), w))
            torch.cuda.synchronize(dev)
            r.check_device_error()
            outs.append((a, b))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


def test_batch_decode_reports_timeout_then_recovers():
    rng = np.random.default_rng(970)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    runs = [lisa_attn.AttnRunner(1, 3000) for _ in range(3)]
    bases = [100, 2000, 2999]
    for r, b in zip(runs, bases):
        kc, vc = random_cache(rng, 3000, b)
        load_cache(r, 0, kc, vc)
    q, k, v = layer_inputs(rng, 3)
    tq, tk, tv = dev_inputs(q, k, v)
    bd = lisa_attn.BatchDecoder(3, 9000)
    with injected_timeout():
        bd.decode(runs, 0, bases, tq, tk, tv, w)
        with pytest.raises(lisa_attn.LisaError) as e:
            bd.check_device_error()
        assert e.value.status == lisa_attn.ETIMEOUT
    got = to_bits(bd.decode(runs, 0, bases, tq, tk, tv, w))
    bd.check_device_error()
    for i, r in enumerate(runs):
        ref = to_bits(r.decode_layer(0, bases[i], 1, tq[i:i + 1], tk[i:i + 1], tv[i:i + 1], w))
        assert_close_bf16(got[i:i + 1], ref, f"seq {i}")
