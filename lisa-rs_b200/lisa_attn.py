"""Host-side mirror of the lisa-rs attention dispatch over the C ABI in
include/lisa_attn.h (liblisa_attn.so, built for sm_100a).

``AttnRunner`` keeps the method names and position semantics of the
attention slice of ``QwenRunner`` / ``MtpRunner`` (lisa-rs
src/model/runner.rs): ``forward_decode`` / ``verify_block3`` /
``forward_prefill`` run one attention layer, ``advance`` ends a forward,
``commit_verified_prefix``, ``trim_state``, ``set_position``,
``restore_state``, ``reset_state`` and ``checkpoint_state`` follow
runner.rs:423-503, 911-944 and 2376-2545. Errors raise ``LisaError`` with the
C status, as the reference returns ``Err(String)``.

Tensors are torch CUDA tensors (torch is only the device-memory allocator
here). There is no CPU path: if the CUDA library is missing, loading fails.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblisa_attn.so")

QH, KVH, HD = 24, 4, 256
QROW, KROW, OROW = QH * 512, KVH * HD, QH * HD
PREFILL_MAX_ROWS = 512

OK, EINVAL, ENOSPC, ESTATE, ETIMEOUT, ECUDA, E2BIG = 0, -22, -28, -71, -62, -1000, -7
NOALLOC_MAX_POSITIONS = 16384
XCHG_HANDLE_BYTES = 64
BATCH_MAX_SEQS = 128
DTYPE_F32, DTYPE_BF16 = 0, 1
_NAMES = {E2BIG: "E2BIG", EINVAL: "EINVAL", ENOSPC: "ENOSPC", ESTATE: "ESTATE", ETIMEOUT: "ETIMEOUT", ECUDA: "ECUDA"}

# name -> (restype, argtypes); mirrors include/lisa_attn.h
_P, _u32, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "lisa_attn_create": (_i32, [_i32, _i32, _u32, ctypes.POINTER(_P)]),
    "lisa_attn_destroy": (_i32, [_P]),
    "lisa_attn_kv_cache": (_i32, [_P, _i32, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "lisa_attn_capacity": (_u32, [_P]),
    "lisa_attn_n_layers": (_i32, [_P]),
    "lisa_attn_decode": (_i32, [_P, _i32, _u32, _i32, _i32, _P, _P, _P, _P, _P, _f32, _P, _P]),
    "lisa_attn_prefill_chunk": (_i32, [_P, _i32, _u32, _i32, _i32, _P, _P, _P, _P, _P, _f32, _P, _P]),
    "lisa_attn_position": (_u32, [_P]),
    "lisa_attn_advance": (_i32, [_P, _i32, _i32]),
    "lisa_attn_commit_verified_prefix": (_i32, [_P, _i32]),
    "lisa_attn_trim_state": (_i32, [_P, _u32]),
    "lisa_attn_set_position": (_i32, [_P, _u32]),
    "lisa_attn_restore_position": (_i32, [_P, _u32]),
    "lisa_attn_reset_state": (_i32, [_P, _P]),
    "lisa_attn_snapshot_bytes": (_sz, [_P]),
    "lisa_attn_kv_snapshot": (_i32, [_P, _P, _sz, ctypes.POINTER(_u32), _P]),
    "lisa_attn_kv_restore": (_i32, [_P, _P, _sz, _u32, _P]),
    "lisa_attn_check_device_error": (_i32, [_P]),
    "lisa_attn_window_workspace_bytes": (_sz, [_u32, _i32]),
    "lisa_attn_decode_window": (_i32, [_P, _P, _u32, _u32, _u32, _i32, _i32, _P, _P, _P, _P, _P, _f32, _P, _P,
                                       _P, _sz, _P]),
    "lisa_attn_merge_windows": (_i32, [_i32, _i32, _P, _P, _i32, _P, _P, _P]),
    "lisa_attn_window_check_device_error": (_i32, [_P, _P]),
    "lisa_attn_batch_create": (_i32, [_i32, _i32, ctypes.c_uint64, ctypes.POINTER(_P)]),
    "lisa_attn_batch_destroy": (_i32, [_P]),
    "lisa_attn_decode_batch": (_i32, [_P, _i32, _P, _i32, _P, _i32, _P, _P, _P, _P, _P, _f32, _P, _P]),
    "lisa_attn_batch_check_device_error": (_i32, [_P, _P]),
    "lisa_attn_xchg_create": (_i32, [_i32, _i32, _i32, _i32, _u32, ctypes.POINTER(_P)]),
    "lisa_attn_xchg_handle": (_i32, [_P, _P]),
    "lisa_attn_xchg_open": (_i32, [_P, _P]),
    "lisa_attn_xchg_decode": (_i32, [_P, _P, _P, _u32, _u32, _i32, _i32, _P, _P, _P, _P, _P, _f32, _P, _P]),
    "lisa_attn_xchg_check_device_error": (_i32, [_P, _P]),
    "lisa_attn_xchg_destroy": (_i32, [_P]),
    "lisa_attn_decode_noalloc": (_i32, [_P, _P, _u32, _u32, _i32, _i32, _P, _P, _P, _P, _P, _f32, _P, _P]),
    "lisa_attn_noalloc_check_device_error": (_i32, []),
    "lisa_attn_debug_wait_fault": (_i32, [_u32, _i32]),
    "lisa_attn_debug_prefill_split": (_i32, [_i32]),
    "lisa_attn_debug_prefill_plan": (_i32, [_u32, _i32, _i32, _i32, _P, _P, _P, _i32]),
    "lisa_attn_qmv_u4": (_i32, [_i32, _P, _i32, _i32, _P, _P]),
    "lisa_attn_gdn_recurrence": (_i32, [_i32, _i32, _i32, _P, _P, _P, _P, _P, _P, _P, _P, _sz, _P]),
    "lisa_attn_st_open": (_i32, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "lisa_attn_st_close": (_i32, [_P]),
    "lisa_attn_st_count": (_i32, [_P]),
    "lisa_attn_st_find": (_i32, [_P, ctypes.c_char_p]),
    "lisa_attn_st_info": (_i32, [_P, _i32, ctypes.c_char_p, _sz, ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_uint64),
                                 _i32, ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_uint64),
                                 ctypes.POINTER(ctypes.c_uint64)]),
    "lisa_attn_st_host_ptr": (_i32, [_P, _i32, ctypes.POINTER(_P)]),
    "lisa_attn_st_upload": (_i32, [_P, _i32, _P, _sz, _P]),
    "lisa_attn_dev_count": (_i32, [ctypes.POINTER(_i32)]),
    "lisa_attn_dev_info": (_i32, [_i32, ctypes.c_char_p, _sz, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_i32)]),
    "lisa_attn_dev_select": (_i32, [_i32]),
    "lisa_attn_buffer_alloc": (_i32, [_i32, _sz, ctypes.POINTER(_P)]),
    "lisa_attn_buffer_free": (_i32, [_P]),
    "lisa_attn_host_alloc": (_i32, [_sz, ctypes.POINTER(_P)]),
    "lisa_attn_host_free": (_i32, [_P]),
    "lisa_attn_stream_create": (_i32, [_i32, ctypes.POINTER(_P)]),
    "lisa_attn_stream_destroy": (_i32, [_P]),
    "lisa_attn_stream_synchronize": (_i32, [_P]),
    "lisa_attn_event_create": (_i32, [_i32, _i32, ctypes.POINTER(_P)]),
    "lisa_attn_event_destroy": (_i32, [_P]),
    "lisa_attn_event_record": (_i32, [_P, _P]),
    "lisa_attn_stream_wait_event": (_i32, [_P, _P]),
    "lisa_attn_event_synchronize": (_i32, [_P]),
    "lisa_attn_event_elapsed_ms": (_i32, [_P, _P, ctypes.POINTER(_f32)]),
    "lisa_attn_copy_h2d": (_i32, [_P, _P, _sz, _P]),
    "lisa_attn_copy_d2h": (_i32, [_P, _P, _sz, _P]),
    "lisa_attn_copy_d2d": (_i32, [_P, _P, _sz, _P]),
    "lisa_attn_memset": (_i32, [_P, _i32, _sz, _P]),
    "lisa_attn_build_info": (ctypes.c_char_p, []),
}

_lib = None


class LisaError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {_NAMES.get(status, status)} ({status})")
        self.status = status


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads liblisa_attn.so and binds every declared entry point. Raises
    OSError if the library has not been built (no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise OSError(f"{path} not built; run `make -C {_HERE}` (or __graft_entry__.build())")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(fn: str, status: int) -> None:
    if status != OK:
        raise LisaError(fn, status)


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    raise TypeError(f"q/k/v must be float32 or bfloat16, got {t.dtype}")


def _stream_ptr(stream) -> int | None:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class AttentionWeights:
    """The attention-layer weights the path reads: q_norm and k_norm gains
    (bf16 [256]); cf. AttentionWeights in runner.rs:93-101."""

    def __init__(self, q_norm, k_norm):
        import torch

        assert q_norm.dtype == torch.bfloat16 and k_norm.dtype == torch.bfloat16
        assert q_norm.numel() == HD and k_norm.numel() == HD
        self.q_norm = q_norm.contiguous()
        self.k_norm = k_norm.contiguous()


class AttnRunner:
    """KV cache + position contract of the attention layers of one model
    (n_layers = 16 for the target, 1 for the MTP drafter)."""

    def __init__(self, n_layers: int, capacity: int, device: int | None = None, eps: float = 1e-6):
        import torch

        self.lib = load_library()
        self.device = torch.cuda.current_device() if device is None else device
        self.eps = eps
        h = _P()
        _check("lisa_attn_create", self.lib.lisa_attn_create(self.device, n_layers, capacity, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.lisa_attn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- state ----
    @property
    def handle(self):
        return self._h

    @property
    def capacity(self) -> int:
        return self.lib.lisa_attn_capacity(self._h)

    @property
    def n_layers(self) -> int:
        return self.lib.lisa_attn_n_layers(self._h)

    def position(self) -> int:
        return self.lib.lisa_attn_position(self._h)

    def kv_cache(self, layer: int):
        """(k, v) as torch bf16 views [4, capacity, 256] of the layer's cache."""
        import torch

        k, v = _P(), _P()
        _check("lisa_attn_kv_cache", self.lib.lisa_attn_kv_cache(self._h, layer, ctypes.byref(k), ctypes.byref(v)))
        return _wrap_device(k.value, (KVH, self.capacity, HD), self.device), _wrap_device(
            v.value, (KVH, self.capacity, HD), self.device)

    # ---- dispatch ----
    def _layer_call(self, fn, layer, base, rows, q_gate, k, v, w: AttentionWeights, out, stream):
        import torch

        dt = _dtype_code(q_gate)
        assert k.dtype == q_gate.dtype and v.dtype == q_gate.dtype
        for t in (q_gate, k, v):
            assert t.is_cuda and t.is_contiguous()
        assert q_gate.numel() == rows * QROW and k.numel() == rows * KROW and v.numel() == rows * KROW
        if out is None:
            out = torch.empty((rows, OROW), dtype=torch.bfloat16, device=q_gate.device)
        status = getattr(self.lib, fn)(self._h, layer, base, rows, dt, _ptr(q_gate), _ptr(k), _ptr(v),
                                       _ptr(w.q_norm), _ptr(w.k_norm), self.eps, _ptr(out), _stream_ptr(stream))
        _check(fn, status)
        return out

    def decode_layer(self, layer, base, rows, q_gate, k, v, w, out=None, stream=None):
        """One attention layer at explicit base (rows 1 or 3)."""
        return self._layer_call("lisa_attn_decode", layer, base, rows, q_gate, k, v, w, out, stream)

    def prefill_layer(self, layer, base, rows, q_gate, k, v, w, out=None, stream=None):
        return self._layer_call("lisa_attn_prefill_chunk", layer, base, rows, q_gate, k, v, w, out, stream)

    def forward_decode(self, layer, q_gate, k, v, w, out=None, stream=None):
        """encode_attention with batch 1 at the current position (runner.rs:1426)."""
        return self.decode_layer(layer, self.position(), 1, q_gate, k, v, w, out, stream)

    def verify_block3(self, layer, q_gate, k, v, w, out=None, stream=None):
        """encode_attention with batch 3 at the current position."""
        return self.decode_layer(layer, self.position(), 3, q_gate, k, v, w, out, stream)

    def forward_prefill(self, layer, q_gate, k, v, w, out=None, stream=None):
        """encode_prefill_attention for one chunk of <= 512 rows (runner.rs:1962)."""
        rows = q_gate.numel() // QROW
        return self.prefill_layer(layer, self.position(), rows, q_gate, k, v, w, out, stream)

    def advance(self, rows: int, verify: bool = False) -> None:
        _check("lisa_attn_advance", self.lib.lisa_attn_advance(self._h, rows, int(verify)))

    def commit_verified_prefix(self, rows: int) -> None:
        _check("lisa_attn_commit_verified_prefix", self.lib.lisa_attn_commit_verified_prefix(self._h, rows))

    def trim_state(self, count: int) -> None:
        _check("lisa_attn_trim_state", self.lib.lisa_attn_trim_state(self._h, count))

    def set_position(self, position: int) -> None:
        _check("lisa_attn_set_position", self.lib.lisa_attn_set_position(self._h, position))

    def restore_position(self, position: int) -> None:
        _check("lisa_attn_restore_position", self.lib.lisa_attn_restore_position(self._h, position))

    def reset_state(self, stream=None) -> None:
        _check("lisa_attn_reset_state", self.lib.lisa_attn_reset_state(self._h, _stream_ptr(stream)))

    def checkpoint_state(self, stream=None):
        """MtpRunner::checkpoint_state: device copy of all K/V + position."""
        import torch

        n = self.lib.lisa_attn_snapshot_bytes(self._h)
        buf = torch.empty(n, dtype=torch.uint8, device=f"cuda:{self.device}")
        pos = _u32()
        _check("lisa_attn_kv_snapshot",
               self.lib.lisa_attn_kv_snapshot(self._h, _ptr(buf), n, ctypes.byref(pos), _stream_ptr(stream)))
        return buf, pos.value

    def restore_state(self, checkpoint, stream=None) -> None:
        buf, pos = checkpoint
        _check("lisa_attn_kv_restore",
               self.lib.lisa_attn_kv_restore(self._h, _ptr(buf), buf.numel(), pos, _stream_ptr(stream)))

    def check_device_error(self) -> None:
        _check("lisa_attn_check_device_error", self.lib.lisa_attn_check_device_error(self._h))


def _wrap_device(ptr: int, shape, device: int):
    """A torch bf16 tensor view of device memory owned by the library."""
    import torch

    class _Holder:
        pass

    n = 1
    for s in shape:
        n *= s
    holder = _Holder()
    holder.__cuda_array_interface__ = {
        "shape": (n,), "typestr": "<u2", "data": (ptr, False), "version": 3, "strides": None}
    with torch.cuda.device(device):
        t = torch.as_tensor(holder, device=f"cuda:{device}")
    return t.view(torch.bfloat16).view(*shape)


# ---- split-KV windows (multi-GPU long context) --------------------------------

def window_workspace_bytes(window_rows: int, rows: int) -> int:
    return load_library().lisa_attn_window_workspace_bytes(window_rows, rows)


def decode_window(k_cache, v_cache, kv_lo, base, rows, q_gate, k, v, w, part_o, part_ml, workspace,
                  eps=1e-6, stream=None):
    lib = load_library()
    window_rows = k_cache.shape[1]
    _check("lisa_attn_decode_window",
           lib.lisa_attn_decode_window(_ptr(k_cache), _ptr(v_cache), window_rows, kv_lo, base, rows,
                                       _dtype_code(q_gate), _ptr(q_gate), _ptr(k), _ptr(v), _ptr(w.q_norm),
                                       _ptr(w.k_norm), eps, _ptr(part_o), _ptr(part_ml), _ptr(workspace),
                                       workspace.numel() * workspace.element_size(), _stream_ptr(stream)))


def window_check_device_error(workspace, stream=None):
    """Raises LisaError(ETIMEOUT) if the last decode_window call on this
    workspace had a device wait give up."""
    _check("lisa_attn_window_check_device_error",
           load_library().lisa_attn_window_check_device_error(_ptr(workspace), _stream_ptr(stream)))


def merge_windows(n_parts, rows, part_o, part_ml, q_gate, out, stream=None):
    lib = load_library()
    _check("lisa_attn_merge_windows",
           lib.lisa_attn_merge_windows(n_parts, rows, _ptr(part_o), _ptr(part_ml), _dtype_code(q_gate),
                                       _ptr(q_gate), _ptr(out), _stream_ptr(stream)))


class WindowExchange:
    """This rank's end of a split-KV exchange (lisa_attn_xchg_*): a receive
    region in device memory that every rank of the sequence writes its window
    partials into. Construct on every rank, all-gather ``handle()`` bytes in
    rank order with any host transport, then ``open(handles)``."""

    def __init__(self, world: int, rank: int, window_rows: int, max_rows: int = 3, device: int | None = None):
        import torch

        self.lib = load_library()
        self.device = torch.cuda.current_device() if device is None else device
        h = _P()
        _check("lisa_attn_xchg_create",
               self.lib.lisa_attn_xchg_create(self.device, world, rank, max_rows, window_rows, ctypes.byref(h)))
        self._h = h
        self.world, self.rank, self.max_rows = world, rank, max_rows

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(XCHG_HANDLE_BYTES)
        _check("lisa_attn_xchg_handle", self.lib.lisa_attn_xchg_handle(self._h, buf))
        return buf.raw

    def open(self, handles: list[bytes]) -> None:
        assert len(handles) == self.world and all(len(b) == XCHG_HANDLE_BYTES for b in handles)
        blob = ctypes.create_string_buffer(b"".join(handles), XCHG_HANDLE_BYTES * self.world)
        _check("lisa_attn_xchg_open", self.lib.lisa_attn_xchg_open(self._h, blob))

    def decode(self, k_cache, v_cache, kv_lo, base, rows, q_gate, k, v, w, out, eps=1e-6, stream=None):
        _check("lisa_attn_xchg_decode",
               self.lib.lisa_attn_xchg_decode(self._h, _ptr(k_cache), _ptr(v_cache), kv_lo, base, rows,
                                              _dtype_code(q_gate), _ptr(q_gate), _ptr(k), _ptr(v), _ptr(w.q_norm),
                                              _ptr(w.k_norm), eps, _ptr(out), _stream_ptr(stream)))
        return out

    def check_device_error(self, stream=None) -> None:
        _check("lisa_attn_xchg_check_device_error",
               self.lib.lisa_attn_xchg_check_device_error(self._h, _stream_ptr(stream)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.lisa_attn_xchg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchDecoder:
    """lisa_attn_decode_batch: one M=1 decode step of one layer for many
    sequences (each an AttnRunner with its own KV cache) in three launches.
    Scratch for up to ``max_seqs`` sequences whose capacities sum to at most
    ``max_total_positions``."""

    def __init__(self, max_seqs: int, max_total_positions: int, device: int | None = None, eps: float = 1e-6):
        import torch

        self.lib = load_library()
        self.device = torch.cuda.current_device() if device is None else device
        self.eps = eps
        h = _P()
        _check("lisa_attn_batch_create",
               self.lib.lisa_attn_batch_create(self.device, max_seqs, max_total_positions, ctypes.byref(h)))
        self._h = h
        self._keep = None

    def decode(self, runners, layer, bases, q_gate, k, v, w, out=None, stream=None):
        """q_gate [n, 12288], k, v [n, 1024] (f32 or bf16), row i for
        runners[i] at position bases[i]; returns gated bf16 [n, 6144]."""
        import torch

        n = len(runners)
        assert len(bases) == n and q_gate.numel() == n * QROW and k.numel() == n * KROW and v.numel() == n * KROW
        if out is None:
            out = torch.empty((n, OROW), dtype=torch.bfloat16, device=q_gate.device)
        ctxs = (_P * n)(*[r.handle.value for r in runners])
        bs = (_u32 * n)(*bases)
        self._keep = (ctxs, bs)
        _check("lisa_attn_decode_batch",
               self.lib.lisa_attn_decode_batch(self._h, n, ctxs, layer, bs, _dtype_code(q_gate), _ptr(q_gate),
                                               _ptr(k), _ptr(v), _ptr(w.q_norm), _ptr(w.k_norm), self.eps,
                                               _ptr(out), _stream_ptr(stream)))
        return out

    def check_device_error(self, stream=None) -> None:
        _check("lisa_attn_batch_check_device_error",
               self.lib.lisa_attn_batch_check_device_error(self._h, _stream_ptr(stream)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.lisa_attn_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- affine-u4 projections (QMV) ----------------------------------------------

class Q4Proj(ctypes.Structure):
    """lisa_attn_q4_proj: one affine-u4 projection (device pointers) and its output."""
    _fields_ = [("packed", _P), ("scales", _P), ("biases", _P), ("out", _P), ("n", _i32)]


def qmv_u4(x, projections, out=None, stream=None):
    """x bf16 [rows, k]; projections: list of (packed uint32 [n, k/8] (int32
    tensor), scales bf16 [n, k/64], biases bf16 [n, k/64]). Returns the f32
    outputs [rows, n] (one per projection), computed by one launch of
    lisa_attn_qmv_u4 (the fused q/k/v QMV of the decode step)."""
    import torch

    rows, k = x.shape
    outs = out or [torch.empty((rows, pk.shape[0]), dtype=torch.float32, device=x.device)
                   for pk, _, _ in projections]
    arr = (Q4Proj * len(projections))(*[
        Q4Proj(_ptr(pk), _ptr(sc), _ptr(bi), _ptr(o), pk.shape[0]) for (pk, sc, bi), o in zip(projections, outs)])
    _check("lisa_attn_qmv_u4",
           load_library().lisa_attn_qmv_u4(len(projections), arr, rows, k, _ptr(x.contiguous()), _stream_ptr(stream)))
    return outs


# ---- safetensors shards and the weight index ----------------------------------

ST_DTYPES = ["BOOL", "U8", "U16", "I16", "F16", "BF16", "U32", "I32", "F32", "U64", "F64"]


class Shard:
    """One memory-mapped safetensors file (lisa_attn_st_*; the reference's
    format::safetensor::Shard, src/format/safetensor.rs:17-41)."""

    def __init__(self, path: str):
        self.lib = load_library()
        h = _P()
        _check("lisa_attn_st_open", self.lib.lisa_attn_st_open(os.fsencode(path), ctypes.byref(h)))
        self._h = h
        self.path = path
        self.tensors = {}
        for i in range(self.lib.lisa_attn_st_count(h)):
            name = ctypes.create_string_buffer(512)
            dt, nd = _i32(), _i32()
            shape = (ctypes.c_uint64 * 8)()
            off, nb = ctypes.c_uint64(), ctypes.c_uint64()
            _check("lisa_attn_st_info", self.lib.lisa_attn_st_info(h, i, name, 512, ctypes.byref(dt), shape, 8,
                                                                   ctypes.byref(nd), ctypes.byref(off),
                                                                   ctypes.byref(nb)))
            self.tensors[name.value.decode()] = {"index": i, "dtype": ST_DTYPES[dt.value],
                                                 "shape": [shape[j] for j in range(nd.value)],
                                                 "offset": off.value, "len": nb.value}

    def host_bytes(self, name: str) -> bytes:
        t = self.tensors[name]
        p = _P()
        _check("lisa_attn_st_host_ptr", self.lib.lisa_attn_st_host_ptr(self._h, t["index"], ctypes.byref(p)))
        return ctypes.string_at(p.value, t["len"])

    def upload(self, name: str, dst, stream=None) -> None:
        t = self.tensors[name]
        _check("lisa_attn_st_upload", self.lib.lisa_attn_st_upload(
            self._h, t["index"], _ptr(dst), dst.numel() * dst.element_size(), _stream_ptr(stream)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.lisa_attn_st_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class WeightIndex:
    """Tensor name -> (shard, slot) over several shards, as
    model::weights::WeightIndex (src/model/weights.rs:16-81): a name present in
    two shards is an error; rows(name, first, count) slices along dim 0."""

    def __init__(self, paths):
        self.shards = [Shard(p) for p in paths]
        self.slots = {}
        for si, sh in enumerate(self.shards):
            for name, t in sh.tensors.items():
                if name in self.slots:
                    raise ValueError(f"duplicate tensor {name}")
                self.slots[name] = (si, t)

    def __len__(self):
        return len(self.slots)

    def slot(self, name):
        s = self.slots.get(name)
        return None if s is None else s[1]

    def bytes(self, name):
        s = self.slots.get(name)
        return None if s is None else self.shards[s[0]].host_bytes(name)

    def rows(self, name, first, count):
        t = self.slot(name)
        if t is None or not t["shape"]:
            return None
        n = t["shape"][0]
        if first + count > n or t["len"] % n:
            return None
        rb = t["len"] // n
        return self.bytes(name)[first * rb:(first + count) * rb]

    def device_tensor(self, name, device=None, stream=None):
        """Upload one tensor into a new torch device tensor of its dtype
        (U32 as int32, BF16 as bfloat16)."""
        import torch

        t = self.slot(name)
        if t is None:
            raise KeyError(name)
        dt = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "U32": torch.int32,
              "I32": torch.int32, "U8": torch.uint8, "BOOL": torch.bool, "I16": torch.int16, "U16": torch.int16,
              "F64": torch.float64, "U64": torch.int64}[t["dtype"]]
        out = torch.empty(t["shape"], dtype=dt, device=device if device is not None else "cuda")
        self.shards[self.slots[name][0]].upload(name, out, stream)
        return out

    def q4_projection(self, prefix, device=None):
        """An affine-u4 linear layer stored as <prefix>.weight (U32 [n, k/8]),
        <prefix>.scales and <prefix>.biases (BF16 [n, k/64]), as MLX writes
        them; returns device tensors (packed, scales, biases) for qmv_u4."""
        w, s, b = (self.slot(prefix + suf) for suf in (".weight", ".scales", ".biases"))
        if w is None or s is None or b is None:
            raise KeyError(prefix)
        if w["dtype"] != "U32" or s["dtype"] != "BF16" or b["dtype"] != "BF16" or len(w["shape"]) != 2:
            raise ValueError(f"{prefix}: not an affine-u4 projection")
        n, k8 = w["shape"]
        if s["shape"] != [n, k8 // 8] or b["shape"] != [n, k8 // 8]:
            raise ValueError(f"{prefix}: scales/biases shape does not match group size 64")
        return tuple(self.device_tensor(prefix + suf, device) for suf in (".weight", ".scales", ".biases"))


def gdn_recurrence(conv_out, q_norm, k_norm, beta, decay, state, y, value_heads=48, repeat=3, slots=None,
                   stream=None):
    """lisa_attn_gdn_recurrence over conv_out.shape[0] tokens (f32 tensors);
    updates `state` in place and writes `y`; `slots` [steps, value_heads*128*128]
    receives the state after every token when given."""
    steps = conv_out.shape[0]
    stride = slots[0].numel() if slots is not None else 0
    _check("lisa_attn_gdn_recurrence", load_library().lisa_attn_gdn_recurrence(
        steps, value_heads, repeat, _ptr(conv_out), _ptr(q_norm), _ptr(k_norm), _ptr(beta), _ptr(decay),
        _ptr(state), _ptr(y), _ptr(slots), stride, _stream_ptr(stream)))
