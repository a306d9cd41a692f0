"""CPU: the multi-GPU host logic — window and sequence plans, and the
all-gather of window partials over a world_size-2 gloo group, merged by
log-sum-exp, against the oracle's single-window attention."""
import os

import numpy as np
import pytest

import lisa_split
import oracle as O
from helpers import HD, KVH, QH, layer_inputs, norm_weights, random_cache


def test_plan_windows_cover_and_align():
    for cap, world in [(262144, 8), (262144, 3), (1000, 4), (5, 8), (128, 1)]:
        ws = lisa_split.plan_windows(cap, world)
        assert len(ws) == world and [w.rank for w in ws] == list(range(world))
        lo = 0
        for w in ws:
            assert w.lo == lo and w.rows >= 0
            if w.rows and w.lo + w.rows < cap:
                assert w.rows % 128 == 0
            lo += w.rows
        assert lo == cap


def test_plan_sequences_partition_and_balance():
    rng = np.random.default_rng(3)
    ctx = rng.integers(1024, 32769, size=64).tolist()
    for world in (1, 2, 4, 8):
        plan = lisa_split.plan_sequences(ctx, world)
        flat = sorted(i for p in plan for i in p)
        assert flat == list(range(64))
        loads = [sum(ctx[i] for i in p) for p in plan]
        assert max(loads) - min(loads) <= max(ctx)


def window_partial(query_bits, kc, vc, lo, n, ctx_r):
    """Normalised O, max and sum of one window [lo, lo+n) for each (row, head):
    the quantities lisa_attn_decode_window returns (f64 reference)."""
    rows = query_bits.shape[0]
    q = O.bf16_to_f32(query_bits).astype(np.float64)
    o = np.zeros((rows, QH, HD))
    ml = np.zeros((rows, QH, 2))
    for r in range(rows):
        hi = min(lo + n, ctx_r[r])
        for h in range(QH):
            kvh = h // (QH // KVH)
            if hi <= lo:
                ml[r, h] = (-np.inf, 0.0)
                continue
            k = O.bf16_to_f32(kc[kvh, lo:hi]).astype(np.float64)
            v = O.bf16_to_f32(vc[kvh, lo:hi]).astype(np.float64)
            s = k @ q[r, h] * 0.0625
            m = s.max()
            p = np.exp(s - m)
            o[r, h] = p @ v / p.sum()
            ml[r, h] = (m, p.sum())
    return o.astype(np.float32), ml.astype(np.float32)


def merge(all_o, all_ml):
    gm = all_ml[..., 0].max(0)
    w = np.where(all_ml[..., 1] > 0, np.exp(all_ml[..., 0] - gm) * all_ml[..., 1], 0.0)
    return (w[..., None] * all_o).sum(0) / w.sum(0)[..., None]


def _rank_main(rank, world, port, q, kc, vc, base, result_path):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ctx_r = [base + r + 1 for r in range(q.shape[0])]
    win = lisa_split.plan_windows(base + q.shape[0], world)[rank]
    po, pm = window_partial(q, kc, vc, win.lo, win.rows, ctx_r)
    all_o, all_ml = lisa_split.gather_partials(torch.from_numpy(po), torch.from_numpy(pm))
    if rank == 0:
        np.save(result_path, merge(all_o.numpy().astype(np.float64), all_ml.numpy().astype(np.float64)))
    dist.barrier()
    dist.destroy_process_group()


def test_gather_and_merge_over_gloo_world2(tmp_path):
    import socket

    import torch.multiprocessing as mp

    rng = np.random.default_rng(11)
    qn, kn = norm_weights(rng)
    qg, k, v = layer_inputs(rng, 3)
    base = 700
    kc, vc = random_cache(rng, base + 3, base)
    O.kv_append(k, v, base, kn, kc, vc)
    query, _ = O.q_prologue(qg, base, qn)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "merged.npy")
    mp.spawn(_rank_main, args=(2, port, query, kc, vc, base, out), nprocs=2, join=True)
    merged = np.load(out)
    want = O.sdpa(query, kc, vc, base, sliced=False)
    assert np.abs(merged - want).max() < 1e-4


def _monitor_rank(rank, world, port, mode, result_path):
    import datetime
    import json
    import time

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0, timeout=datetime.timedelta(seconds=10))
    mon = lisa_split.PeerMonitor(store, rank, world, interval=0.05, stale_after=1.0)
    po = torch.full((1, QH, HD), float(rank))
    pm = torch.zeros((1, QH, 2))
    for _ in range(3):  # steps with every rank present
        mon.check()
        all_o, _ = lisa_split.gather_partials(po, pm)
        assert all_o.shape[0] == world
    dist.barrier()
    if rank == 1:
        if mode == "leave":
            mon.leave()
        os._exit(0)  # between steps: nothing of this rank is in flight
    # rank 0 goes on stepping: the check before the launch must stop it
    t0 = time.monotonic()
    res = {"raised": False}
    while time.monotonic() - t0 < 10.0:
        try:
            mon.check()
        except lisa_split.PeerLost as e:
            res = {"raised": True, "why": str(e), "after_s": time.monotonic() - t0}
            break
        time.sleep(0.02)
    # a collective issued anyway ends with an error instead of hanging
    t1 = time.monotonic()
    try:
        lisa_split.gather_partials(po, pm)
        res["collective"] = "returned"
    except Exception as e:
        res["collective"] = type(e).__name__
    res["collective_s"] = time.monotonic() - t1
    with open(result_path, "w") as f:
        json.dump(res, f)
    os._exit(0)


@pytest.mark.parametrize("mode", ["leave", "vanish"])
def test_rank_departure_between_steps_is_reported_not_hung(mode, tmp_path):
    """SplitKVDecoder's host-side failure detection on gloo CPU ranks: rank 1
    leaves between steps (announced, or silently); rank 0's next pre-launch
    check raises PeerLost within seconds, and a collective issued anyway
    fails (process-group timeout or closed peer) instead of hanging."""
    import json
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "res.json")
    mp.spawn(_monitor_rank, args=(2, port, mode, out), nprocs=2, join=True)
    res = json.load(open(out))
    assert res["raised"], res
    assert res["after_s"] < 5.0, res
    assert res["collective"] != "returned" and res["collective_s"] < 30.0, res
