"""GPU, without torch: the device bridge of the C ABI (streams, events, device
and pinned host buffers, copies) is enough to run decode, verify and prefill
from host buffers, as a Rust host would through its extern "C" block. Only
ctypes, numpy and the library are used here (the oracle is the checker)."""
import ctypes

import numpy as np
import pytest

import oracle as O
from helpers import KROW, OROW, QROW, assert_close_bf16, layer_inputs, norm_weights, random_cache

pytestmark = pytest.mark.gpu

import lisa_attn  # noqa: E402

P = ctypes.c_void_p


def ok(status):
    assert status == lisa_attn.OK, status


class Dev:
    """Device-side copy of host arrays through pinned staging buffers."""

    def __init__(self, lib, stream):
        self.lib, self.stream, self.bufs, self.hosts = lib, stream, [], []

    def pinned(self, nbytes):
        h = P()
        ok(self.lib.lisa_attn_host_alloc(nbytes, ctypes.byref(h)))
        self.hosts.append(h)
        return h

    def upload(self, arr):
        arr = np.ascontiguousarray(arr)
        d = P()
        ok(self.lib.lisa_attn_buffer_alloc(0, arr.nbytes, ctypes.byref(d)))
        self.bufs.append(d)
        h = self.pinned(arr.nbytes)
        ctypes.memmove(h, arr.ctypes.data, arr.nbytes)
        ok(self.lib.lisa_attn_copy_h2d(d, h, arr.nbytes, self.stream))
        return d

    def alloc(self, nbytes):
        d = P()
        ok(self.lib.lisa_attn_buffer_alloc(0, nbytes, ctypes.byref(d)))
        self.bufs.append(d)
        return d

    def download(self, d, shape, dtype):
        out = np.empty(shape, dtype)
        h = self.pinned(out.nbytes)
        ok(self.lib.lisa_attn_copy_d2h(h, d, out.nbytes, self.stream))
        ok(self.lib.lisa_attn_stream_synchronize(self.stream))
        ctypes.memmove(out.ctypes.data, h, out.nbytes)
        return out

    def close(self):
        for d in self.bufs:
            ok(self.lib.lisa_attn_buffer_free(d))
        for h in self.hosts:
            ok(self.lib.lisa_attn_host_free(h))


def test_decode_verify_prefill_through_the_device_bridge():
    lib = lisa_attn.load_library()
    n = ctypes.c_int()
    ok(lib.lisa_attn_dev_count(ctypes.byref(n)))
    assert n.value >= 1
    name = ctypes.create_string_buffer(128)
    total, sms = ctypes.c_uint64(), ctypes.c_int()
    ok(lib.lisa_attn_dev_info(0, name, 128, ctypes.byref(total), ctypes.byref(sms)))
    assert total.value > 0 and sms.value > 0
    stream, e0, e1 = P(), P(), P()
    ok(lib.lisa_attn_stream_create(0, ctypes.byref(stream)))
    ok(lib.lisa_attn_event_create(0, 1, ctypes.byref(e0)))
    ok(lib.lisa_attn_event_create(0, 1, ctypes.byref(e1)))
    dev = Dev(lib, stream)
    rng = np.random.default_rng(4321)
    qn, kn = norm_weights(rng)
    dqn, dkn = dev.upload(qn), dev.upload(kn)
    cap, base = 3000, 2500
    ctx = P()
    ok(lib.lisa_attn_create(0, 1, cap, ctypes.byref(ctx)))
    kc, vc = random_cache(rng, cap, base)
    kp, vp = P(), P()
    ok(lib.lisa_attn_kv_cache(ctx, 0, ctypes.byref(kp), ctypes.byref(vp)))
    for dst, arr in ((kp, kc), (vp, vc)):
        h = dev.pinned(arr.nbytes)
        ctypes.memmove(h, arr.ctypes.data, arr.nbytes)
        ok(lib.lisa_attn_copy_h2d(dst, h, arr.nbytes, stream))
    ok(lib.lisa_attn_restore_position(ctx, base))

    # decode (M=1), timed with the bridge's events
    q, k, v = layer_inputs(rng, 1)
    dq, dk, dv = dev.upload(q), dev.upload(k), dev.upload(v)
    dout = dev.alloc(OROW * 2)
    ok(lib.lisa_attn_event_record(e0, stream))
    ok(lib.lisa_attn_decode(ctx, 0, base, 1, lisa_attn.DTYPE_F32, dq, dk, dv, dqn, dkn, ctypes.c_float(1e-6), dout,
                            stream))
    ok(lib.lisa_attn_event_record(e1, stream))
    ok(lib.lisa_attn_event_synchronize(e1))
    ms = ctypes.c_float()
    ok(lib.lisa_attn_event_elapsed_ms(e0, e1, ctypes.byref(ms)))
    assert ms.value > 0
    got = dev.download(dout, (1, OROW), np.uint16)
    ok(lib.lisa_attn_advance(ctx, 1, 0))
    want = O.attention_layer(q, k, v, base, qn, kn, kc, vc, sliced=True)
    assert_close_bf16(got, want, "bridge decode")

    # verify (M=3) on a second stream ordered after the first by an event
    s2 = P()
    ok(lib.lisa_attn_stream_create(0, ctypes.byref(s2)))
    ok(lib.lisa_attn_event_record(e0, stream))
    ok(lib.lisa_attn_stream_wait_event(s2, e0))
    q3, k3, v3 = layer_inputs(rng, 3)
    dq3, dk3, dv3 = dev.upload(q3), dev.upload(k3), dev.upload(v3)
    ok(lib.lisa_attn_stream_synchronize(stream))
    dout3 = dev.alloc(3 * OROW * 2)
    ok(lib.lisa_attn_decode(ctx, 0, base + 1, 3, lisa_attn.DTYPE_F32, dq3, dk3, dv3, dqn, dkn, ctypes.c_float(1e-6),
                            dout3, s2))
    ok(lib.lisa_attn_stream_synchronize(s2))
    got3 = dev.download(dout3, (3, OROW), np.uint16)
    want3 = O.attention_layer(q3, k3, v3, base + 1, qn, kn, kc, vc, sliced=True)
    assert_close_bf16(got3, want3, "bridge verify")

    # prefill of 300 rows on a fresh context, then the device error word
    pctx = P()
    ok(lib.lisa_attn_create(0, 1, 512, ctypes.byref(pctx)))
    qp, kp_, vp_ = layer_inputs(rng, 300)
    dqp, dkp, dvp = dev.upload(qp), dev.upload(kp_), dev.upload(vp_)
    doutp = dev.alloc(300 * OROW * 2)
    ok(lib.lisa_attn_memset(doutp, 0, 300 * OROW * 2, stream))
    ok(lib.lisa_attn_prefill_chunk(pctx, 0, 0, 300, lisa_attn.DTYPE_F32, dqp, dkp, dvp, dqn, dkn,
                                   ctypes.c_float(1e-6), doutp, stream))
    gotp = dev.download(doutp, (300, OROW), np.uint16)
    kz = np.zeros((4, 512, 256), np.uint16)
    vz = np.zeros((4, 512, 256), np.uint16)
    wantp = O.attention_layer(qp, kp_, vp_, 0, qn, kn, kz, vz, sliced=False)
    assert_close_bf16(gotp, wantp, "bridge prefill")
    ok(lib.lisa_attn_check_device_error(ctx))
    ok(lib.lisa_attn_check_device_error(pctx))

    ok(lib.lisa_attn_destroy(ctx))
    ok(lib.lisa_attn_destroy(pctx))
    dev.close()
    for e in (e0, e1):
        ok(lib.lisa_attn_event_destroy(e))
    ok(lib.lisa_attn_stream_destroy(s2))
    ok(lib.lisa_attn_stream_destroy(stream))


def test_bridge_argument_errors_without_device_work():
    lib = lisa_attn.load_library()
    p = P()
    assert lib.lisa_attn_buffer_alloc(0, 0, ctypes.byref(p)) == lisa_attn.EINVAL
    assert lib.lisa_attn_buffer_alloc(999, 16, ctypes.byref(p)) == lisa_attn.EINVAL
    assert lib.lisa_attn_buffer_free(None) == lisa_attn.EINVAL
    assert lib.lisa_attn_event_record(None, None) == lisa_attn.EINVAL
    assert lib.lisa_attn_copy_h2d(None, None, 16, None) == lisa_attn.EINVAL
    assert lib.lisa_attn_dev_info(-1, None, 0, None, None) == lisa_attn.EINVAL
