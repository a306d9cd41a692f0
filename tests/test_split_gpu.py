"""GPU: the split-KV window entry points (lisa_attn_decode_window +
lisa_attn_merge_windows) with G windows emulated on one GPU, against the
single-context decode and the oracle; BASELINE config 4 (262144 positions,
M=1 and the M=3 verify variant) split into 2, 4 and 8 windows."""
import numpy as np
import pytest

import lisa_split
import oracle as O
from helpers import HD, KVH, OROW, QH, assert_argmax_agrees, assert_close_bf16, layer_inputs, norm_weights

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import lisa_attn  # noqa: E402
from gpu_util import dev_inputs, load_cache, to_bits, weights  # noqa: E402


def run_windows(kc_full, vc_full, base, rows, q, k, v, w, world):
    """Decode with the cache split into `world` windows; returns gated bits and
    the windows' caches (with the appended rows)."""
    cap = base + rows
    plan = lisa_split.plan_windows(cap, world)
    part_o = torch.empty((world, rows, QH, HD), dtype=torch.float32, device="cuda")
    part_ml = torch.empty((world, rows, QH, 2), dtype=torch.float32, device="cuda")
    tq, tk, tv = dev_inputs(q, k, v)
    caches = []
    for win in plan:
        n = max(win.rows, 1)
        kw = torch.zeros((KVH, n, HD), dtype=torch.bfloat16, device="cuda")
        vw = torch.zeros_like(kw)
        if win.rows:
            kw.copy_(kc_full[:, win.lo:win.lo + win.rows])
            vw.copy_(vc_full[:, win.lo:win.lo + win.rows])
        ws = torch.empty(lisa_attn.window_workspace_bytes(n, rows), dtype=torch.uint8, device="cuda")
        lisa_attn.decode_window(kw, vw, win.lo, base, rows, tq, tk, tv, w, part_o[win.rank], part_ml[win.rank], ws)
        caches.append((win, kw, vw))
    out = torch.empty((rows, OROW), dtype=torch.bfloat16, device="cuda")
    lisa_attn.merge_windows(world, rows, part_o, part_ml, tq, out)
    torch.cuda.synchronize()
    return to_bits(out), caches


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("rows", [1, 3])
def test_windows_match_single_context(world, rows):
    rng = np.random.default_rng(500 + world * 10 + rows)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    base = 3000
    q, k, v = layer_inputs(rng, rows)
    kc = torch.randn((KVH, base + rows, HD), device="cuda").to(torch.bfloat16)
    vc = torch.randn((KVH, base + rows, HD), device="cuda").to(torch.bfloat16)
    kc[:, base:] = 0
    vc[:, base:] = 0
    got, caches = run_windows(kc, vc, base, rows, q, k, v, w, world)
    r = lisa_attn.AttnRunner(1, base + rows)
    rk, rv = r.kv_cache(0)
    rk.copy_(kc)
    rv.copy_(vc)
    want = to_bits(r.decode_layer(0, base, rows, *dev_inputs(q, k, v), w))
    assert_close_bf16(got, want, f"world={world} rows={rows}")
    # the appended rows landed in the windows that own them, identical to the context's
    for win, kw, vw in caches:
        if win.rows:
            assert torch.equal(kw[:, :win.rows], rk[:, win.lo:win.lo + win.rows])
            assert torch.equal(vw[:, :win.rows], rv[:, win.lo:win.lo + win.rows])


@pytest.mark.parametrize("rows", [1, 3])
def test_config4_262144_split_8(rows):
    """262144 positions (new row at 262143, or rows at
    262141..262143 for verify), split over 8 windows, against the oracle."""
    rng = np.random.default_rng(0x5EED + 4 + rows)
    qn, kn = norm_weights(rng)
    w = weights(qn, kn)
    cap = 262144
    base = cap - rows
    q, k, v = layer_inputs(rng, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(77 + rows)
    kc = torch.randn((KVH, cap, HD), device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn((KVH, cap, HD), device="cuda", generator=g).to(torch.bfloat16)
    got, _ = run_windows(kc, vc, base, rows, q, k, v, w, 8)
    kh = kc.cpu().view(torch.int16).numpy().view(np.uint16).copy()
    vh = vc.cpu().view(torch.int16).numpy().view(np.uint16).copy()
    want = O.attention_layer(q, k, v, base, qn, kn, kh, vh, sliced=True)
    assert_close_bf16(got, want, f"config4 rows={rows}")


def test_window_argument_errors():
    lib = lisa_attn.load_library()
    kw = torch.zeros((KVH, 256, HD), dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(lisa_attn.window_workspace_bytes(256, 1), dtype=torch.uint8, device="cuda")
    po = torch.empty((1, QH, HD), dtype=torch.float32, device="cuda")
    pm = torch.empty((1, QH, 2), dtype=torch.float32, device="cuda")
    qg = torch.zeros((1, QH * 512), dtype=torch.float32, device="cuda")
    kv = torch.zeros((1, KVH * HD), dtype=torch.float32, device="cuda")
    nw = torch.ones(HD, dtype=torch.bfloat16, device="cuda")
    args = [kw.data_ptr(), kw.data_ptr(), 256, 0, 10, 1, 0, qg.data_ptr(), kv.data_ptr(), kv.data_ptr(),
            nw.data_ptr(), nw.data_ptr(), 1e-6, po.data_ptr(), pm.data_ptr(), ws.data_ptr(), ws.numel(), None]
    assert lib.lisa_attn_decode_window(*args) == lisa_attn.OK
    bad = list(args)
    bad[16] = ws.numel() - 1  # workspace too small
    assert lib.lisa_attn_decode_window(*bad) == lisa_attn.EINVAL
    bad = list(args)
    bad[5] = 4  # rows outside 1..3
    assert lib.lisa_attn_decode_window(*bad) == lisa_attn.EINVAL
    bad = list(args)
    bad[15] = ws.data_ptr() + 8  # misaligned workspace
    assert lib.lisa_attn_decode_window(*bad) == lisa_attn.EINVAL
    torch.cuda.synchronize()


def _exchange_case(rng, base, rows):
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, rows)
    kc = torch.randn((KVH, base + rows, HD), device="cuda").to(torch.bfloat16)
    vc = torch.randn((KVH, base + rows, HD), device="cuda").to(torch.bfloat16)
    kc[:, base:] = 0
    vc[:, base:] = 0
    return qn, kn, q, k, v, kc, vc


@pytest.mark.parametrize("rows", [1, 3])
def test_exchange_world1_matches_context_and_replays_in_a_graph(rows):
    """lisa_attn_xchg_decode with one rank: the split, the publishing combine
    and the bounded-wait merge against the single-context decode; then the
    same step captured in a CUDA graph and replayed several times (the step
    counter lives on the device), every replay equal to the eager result."""
    rng = np.random.default_rng(800 + rows)
    base = 5000
    qn, kn, q, k, v, kc, vc = _exchange_case(rng, base, rows)
    w = weights(qn, kn)
    dec = lisa_split.SplitKVDecoder(lisa_split.Window(0, 0, base + rows), max_rows=3)
    dec.k.copy_(kc)
    dec.v.copy_(vc)
    tq, tk, tv = dev_inputs(q, k, v)
    got = to_bits(dec.decode(base, tq, tk, tv, w))
    dec.check_device_error()
    r = lisa_attn.AttnRunner(1, base + rows)
    rk, rv = r.kv_cache(0)
    rk.copy_(kc)
    rv.copy_(vc)
    want = to_bits(r.decode_layer(0, base, rows, tq, tk, tv, w))
    assert_close_bf16(got, want, f"exchange world=1 rows={rows}")
    assert torch.equal(dec.k, rk) and torch.equal(dec.v, rv)
    out = torch.empty((rows, OROW), dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        dec.decode(base, tq, tk, tv, w, out, stream=s)  # warm-up on the capture stream
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            dec.decode(base, tq, tk, tv, w, out, stream=s)
    for _ in range(5):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(to_bits(out), got)
    dec.check_device_error()


def _exchange_rank(rank, world, port, base, rows, seed, result_dir):
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    rng = np.random.default_rng(seed)
    qn, kn = norm_weights(rng)
    q, k, v = layer_inputs(rng, rows)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kc = torch.randn((KVH, base + rows, HD), device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn((KVH, base + rows, HD), device="cuda", generator=g).to(torch.bfloat16)
    kc[:, base:] = 0
    vc[:, base:] = 0
    win = lisa_split.plan_windows(base + rows, world)[rank]
    dec = lisa_split.SplitKVDecoder(win, max_rows=3)
    if win.rows:
        dec.k[:, :win.rows].copy_(kc[:, win.lo:win.lo + win.rows])
        dec.v[:, :win.rows].copy_(vc[:, win.lo:win.lo + win.rows])
    w = weights(qn, kn)
    tq, tk, tv = dev_inputs(q, k, v)
    outs = []
    for _ in range(3):  # several steps: both receive parities and the flags' step numbers
        outs.append(to_bits(dec.decode(base, tq, tk, tv, w)))
    dec.check_device_error()
    np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.stack(outs))
    if rank == 0:
        r = lisa_attn.AttnRunner(1, base + rows)
        rk, rv = r.kv_cache(0)
        rk.copy_(kc)
        rv.copy_(vc)
        np.save(os.path.join(result_dir, "single.npy"), to_bits(r.decode_layer(0, base, rows, tq, tk, tv, w)))
        kh = kc.cpu().view(torch.int16).numpy().view(np.uint16).copy()
        vh = vc.cpu().view(torch.int16).numpy().view(np.uint16).copy()
        np.save(os.path.join(result_dir, "oracle.npy"), O.attention_layer(q, k, v, base, qn, kn, kh, vh, sliced=True))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
@pytest.mark.parametrize("rows", [1, 3])
def test_exchange_across_gpus(rows, tmp_path):
    """Config 4's exchange on real GPUs (one process per GPU, peer stores over
    NVLink, no NVLS): every rank's gated output equals the single-GPU
    context decode of the whole sequence, on three consecutive steps."""
    import socket

    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    base = 20000
    mp.spawn(_exchange_rank, args=(world, port, base, rows, 4242 + rows, str(tmp_path)), nprocs=world, join=True)
    # Against the reference math (the oracle), on every rank and step. The
    # single-GPU decode is checked too, but its chunks start at other
    # positions than the windows' (P is rounded to bf16 per chunk), so the two
    # GPU paths may differ by a bf16 step or two in rare elements.
    want = np.load(tmp_path / "oracle.npy")
    single = np.load(tmp_path / "single.npy")
    assert_close_bf16(single, want, "single GPU")
    first = np.load(tmp_path / "rank0.npy")
    for rank in range(world):
        outs = np.load(tmp_path / f"rank{rank}.npy")
        for step, o in enumerate(outs):
            assert np.array_equal(o, first[0]), f"rank {rank} step {step} differs from rank 0 step 0"
        assert_close_bf16(outs[0], want, f"rank {rank}")
    assert assert_argmax_agrees(first[0], want, "exchange") == 0
