"""GPU: lisa_attn_qmv_u4, the affine-u4 QMV (q4_qmv_fast / fused3,
src/kernels/shaders/qmv.metal:1-133) for the decode and verify shapes,
against the reference's own known-answer cases (tests/qmv.rs) and the numpy
oracle at the model's projection sizes; and the fused q/k/v QMV feeding the
attention decode, against the oracle chain."""
import os

import numpy as np
import pytest

import oracle as O
from helpers import KROW, QROW, assert_argmax_agrees, assert_close_bf16, norm_weights, random_cache

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_bf16, to_bits, weights  # noqa: E402

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qmv_reference_tests.npz")
HIDDEN = 5120  # src/model/mod.rs:7


def dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def random_proj(rng, n, k):
    packed = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
    scales = O.f32_to_bf16((0.01 + 0.01 * rng.random((n, k // 64))).astype(np.float32))
    biases = O.f32_to_bf16((-0.08 * rng.random((n, k // 64))).astype(np.float32))
    return packed, scales, biases


def run(x_bits, projs):
    x = dev_bf16(x_bits)
    dev = [(dev_u32(p), dev_bf16(s), dev_bf16(b)) for p, s, b in projs]
    outs = lisa_attn.qmv_u4(x, dev)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("pre", ["m1", "m3"])
def test_reference_known_answers(pre):
    g = np.load(GOLD)
    (got,) = run(g[pre + "_x"], [(g[pre + "_packed"], g[pre + "_scales"], g[pre + "_biases"])])
    assert np.abs(got - g[pre + "_expected"]).max() < 2e-4  # the reference's tolerance


@pytest.mark.parametrize("rows", [1, 2, 3, 4])
def test_fused_qkv_projection_sizes(rows):
    """q_proj (12288 rows: 24 heads x (256 query + 256 gate)), k_proj and
    v_proj (1024 rows) of the 5120-wide hidden state in one launch."""
    rng = np.random.default_rng(60 + rows)
    x = O.f32_to_bf16(rng.standard_normal((rows, HIDDEN)).astype(np.float32))
    projs = [random_proj(rng, n, HIDDEN) for n in (QROW, KROW, KROW)]
    got = run(x, projs)
    for (p, s, b), g in zip(projs, got):
        want = O.q4_qmv(x, p, s, b)
        err = np.abs(g - want).max()
        assert err <= 2e-5 * np.abs(want).max() + 1e-4, err


@pytest.mark.parametrize("n,k,rows", [(19, 128, 3), (33, 64, 3), (100, 6144, 3), (5120, 6144, 3), (5120, 6144, 1),
                                      (7, 8192, 2)])
def test_odd_shapes(n, k, rows):
    """Tail rows, K not a multiple of 1024, the o_proj shape (5120 x 6144)."""
    rng = np.random.default_rng(n + k)
    x = O.f32_to_bf16(rng.standard_normal((rows, k)).astype(np.float32))
    proj = random_proj(rng, n, k)
    (got,) = run(x, [proj])
    want = O.q4_qmv(x, *proj)
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max() + 1e-4


def test_qmv_then_attention_decode_chain():
    """The decode step around the attention layer: fused q/k/v QMV of the
    hidden state, then lisa_attn_decode on its f32 outputs, against the
    oracle's QMV and attention."""
    rng = np.random.default_rng(77)
    x = O.f32_to_bf16(rng.standard_normal((1, HIDDEN)).astype(np.float32))
    projs = [random_proj(rng, n, HIDDEN) for n in (QROW, KROW, KROW)]
    qg_d, k_d, v_d = lisa_attn.qmv_u4(dev_bf16(x), [(dev_u32(p), dev_bf16(s), dev_bf16(b)) for p, s, b in projs])
    qn, kn = norm_weights(rng)
    base = 3000
    kc, vc = random_cache(rng, base + 1, base)
    r = lisa_attn.AttnRunner(1, base + 1)
    kk, vv = r.kv_cache(0)
    kk.copy_(dev_bf16(kc).view(kk.shape))
    vv.copy_(dev_bf16(vc).view(vv.shape))
    got = to_bits(r.decode_layer(0, base, 1, qg_d, k_d, v_d, weights(qn, kn)))
    q, k, v = (O.q4_qmv(x, *pr) for pr in projs)
    want = O.attention_layer(q, k, v, base, qn, kn, kc, vc, sliced=True)
    assert_close_bf16(got, want, "qmv -> attention")
    assert assert_argmax_agrees(got, want, "qmv -> attention") == 0


def test_qmv_argument_errors():
    lib = lisa_attn.load_library()
    x = torch.zeros((1, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((1, 8), dtype=torch.float32, device="cuda")
    pk = torch.zeros((8, 16), dtype=torch.int32, device="cuda")
    sb = torch.zeros((8, 2), dtype=torch.bfloat16, device="cuda")
    P = lisa_attn.Q4Proj
    good = (P * 1)(P(pk.data_ptr(), sb.data_ptr(), sb.data_ptr(), out.data_ptr(), 8))
    assert lib.lisa_attn_qmv_u4(1, good, 1, 128, x.data_ptr(), None) == lisa_attn.OK
    assert lib.lisa_attn_qmv_u4(1, good, 5, 128, x.data_ptr(), None) == lisa_attn.EINVAL   # rows > 4
    assert lib.lisa_attn_qmv_u4(1, good, 1, 96, x.data_ptr(), None) == lisa_attn.EINVAL    # k % 64
    assert lib.lisa_attn_qmv_u4(0, good, 1, 128, x.data_ptr(), None) == lisa_attn.EINVAL
    assert lib.lisa_attn_qmv_u4(1, good, 1, 128, x.data_ptr() + 2, None) == lisa_attn.EINVAL  # misaligned x
    x8 = torch.zeros((3, 8192), dtype=torch.bfloat16, device="cuda")
    assert lib.lisa_attn_qmv_u4(1, good, 3, 8192, x8.data_ptr(), None) == lisa_attn.EINVAL  # x too large
    bad = (P * 1)(P(pk.data_ptr() + 4, sb.data_ptr(), sb.data_ptr(), out.data_ptr(), 8))
    assert lib.lisa_attn_qmv_u4(1, bad, 1, 128, x.data_ptr(), None) == lisa_attn.EINVAL    # misaligned
    torch.cuda.synchronize()


def test_q4_projection_loaded_from_a_safetensors_shard(tmp_path):
    """An MLX affine-u4 projection written as <name>.weight/.scales/.biases
    into a shard, loaded through the weight index onto the device and run by
    the QMV, against the oracle on the file's bytes."""
    import struct, json
    rng = np.random.default_rng(91)
    n, k = 300, 1024
    packed, scales, biases = random_proj(rng, n, k)
    tens = {"model.layers.3.self_attn.q_proj.weight": ("U32", packed), "model.layers.3.self_attn.q_proj.scales":
            ("BF16", scales), "model.layers.3.self_attn.q_proj.biases": ("BF16", biases)}
    header, blob = {}, b""
    for name, (dt, a) in tens.items():
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [len(blob), len(blob) + a.nbytes]}
        blob += a.tobytes()
    h = json.dumps(header).encode()
    path = tmp_path / "q.safetensors"
    path.write_bytes(struct.pack("<Q", len(h)) + h + blob)
    idx = lisa_attn.WeightIndex([str(path)])
    proj = idx.q4_projection("model.layers.3.self_attn.q_proj")
    x = O.f32_to_bf16(rng.standard_normal((1, k)).astype(np.float32))
    (got,) = lisa_attn.qmv_u4(dev_bf16(x), [proj])
    want = O.q4_qmv(x, packed, scales, biases)
    assert np.abs(got.cpu().numpy() - want).max() <= 2e-5 * np.abs(want).max() + 1e-4
