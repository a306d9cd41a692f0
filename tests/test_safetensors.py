"""CPU: the safetensors reader of the C ABI (lisa_attn_st_*) and the weight
index mirror, against files written here byte by byte. Follows the
reference's own test (src/format/safetensor.rs:93-132 parses_synthetic_shard)
and src/model/weights.rs (duplicate names, row slices); the malformed cases
return LISA_EINVAL where the reference panics."""
import ctypes
import json
import struct

import numpy as np
import pytest

import lisa_attn


def write_shard(path, tensors, metadata=None, raw_header=None, data=None):
    """tensors: name -> (dtype name, shape, bytes)."""
    header, blob, off = {}, b"", 0
    for name, (dt, shape, b) in tensors.items():
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blob += b
        off += len(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = raw_header if raw_header is not None else json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + (blob if data is None else data))
    return 8 + len(h)


def test_parses_synthetic_shard(tmp_path):
    """safetensor.rs:97-131: two tensors tiling a 40-byte data region."""
    header = b'{"a":{"dtype":"F32","shape":[2,3],"data_offsets":[0,24]},"b":{"dtype":"BF16","shape":[8],"data_offsets":[24,40]}}'
    p = tmp_path / "s.safetensors"
    p.write_bytes(struct.pack("<Q", len(header)) + header + bytes(40))
    sh = lisa_attn.Shard(str(p))
    assert set(sh.tensors) == {"a", "b"}
    assert sh.tensors["a"]["offset"] == 0 and sh.tensors["a"]["len"] == 24
    assert sh.tensors["b"]["offset"] == 24 and sh.tensors["b"]["len"] == 16
    assert sh.tensors["a"]["dtype"] == "F32" and sh.tensors["a"]["shape"] == [2, 3]


def test_values_metadata_and_escapes(tmp_path):
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    w = np.arange(40, dtype=np.uint32).reshape(5, 8)
    p = tmp_path / "m.safetensors"
    write_shard(p, {"layer.0/a \\\"q\"": ("F32", a.shape, a.tobytes()), "w": ("U32", w.shape, w.tobytes())},
                metadata={"format": "mlx", "nested": {"x": [1, 2.5e3, True, None]}})
    sh = lisa_attn.Shard(str(p))
    assert set(sh.tensors) == {'layer.0/a \\"q"', "w"}  # __metadata__ skipped
    assert np.array_equal(np.frombuffer(sh.host_bytes("w"), np.uint32).reshape(5, 8), w)
    assert np.array_equal(np.frombuffer(sh.host_bytes('layer.0/a \\"q"'), np.float32).reshape(3, 4), a)
    lib = lisa_attn.load_library()
    assert lib.lisa_attn_st_find(sh._h, b"w") >= 0
    assert lib.lisa_attn_st_find(sh._h, b"nope") == lisa_attn.EINVAL


@pytest.mark.parametrize("case", ["truncated_header", "bad_json", "beyond_file", "shape_mismatch", "unknown_dtype",
                                  "reversed_offsets", "short_file"])
def test_malformed_files_are_rejected(tmp_path, case):
    p = tmp_path / "bad.safetensors"
    good = b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}}'
    if case == "truncated_header":
        p.write_bytes(struct.pack("<Q", 1000) + good + bytes(8))
    elif case == "bad_json":
        h = b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]}'
        p.write_bytes(struct.pack("<Q", len(h)) + h + bytes(8))
    elif case == "beyond_file":
        p.write_bytes(struct.pack("<Q", len(good)) + good + bytes(4))
    elif case == "shape_mismatch":
        h = b'{"a":{"dtype":"F32","shape":[3],"data_offsets":[0,8]}}'
        p.write_bytes(struct.pack("<Q", len(h)) + h + bytes(8))
    elif case == "unknown_dtype":
        h = b'{"a":{"dtype":"Q4","shape":[2],"data_offsets":[0,8]}}'
        p.write_bytes(struct.pack("<Q", len(h)) + h + bytes(8))
    elif case == "reversed_offsets":
        h = b'{"a":{"dtype":"F32","shape":[0],"data_offsets":[8,0]}}'
        p.write_bytes(struct.pack("<Q", len(h)) + h + bytes(8))
    else:
        p.write_bytes(b"\x01\x00")
    lib = lisa_attn.load_library()
    h = ctypes.c_void_p()
    assert lib.lisa_attn_st_open(str(p).encode(), ctypes.byref(h)) == lisa_attn.EINVAL


def test_weight_index_over_shards(tmp_path):
    """weights.rs: slots over several shards, duplicate names rejected,
    rows() slices along dim 0 (None past the end)."""
    emb = np.arange(6 * 10, dtype=np.uint32).reshape(6, 10)
    norm = np.arange(5, dtype=np.uint16)
    write_shard(tmp_path / "s1.safetensors", {"embed": ("U32", emb.shape, emb.tobytes())})
    write_shard(tmp_path / "s2.safetensors", {"norm": ("BF16", norm.shape, norm.tobytes())})
    idx = lisa_attn.WeightIndex([str(tmp_path / "s1.safetensors"), str(tmp_path / "s2.safetensors")])
    assert len(idx) == 2 and idx.slot("norm")["dtype"] == "BF16"
    assert np.array_equal(np.frombuffer(idx.rows("embed", 2, 3), np.uint32).reshape(3, 10), emb[2:5])
    assert idx.rows("embed", 5, 2) is None and idx.slot("missing") is None
    write_shard(tmp_path / "s3.safetensors", {"norm": ("BF16", norm.shape, norm.tobytes())})
    with pytest.raises(ValueError):
        lisa_attn.WeightIndex([str(tmp_path / "s2.safetensors"), str(tmp_path / "s3.safetensors")])
