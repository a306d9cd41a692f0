"""Multi-GPU partitioning of the attention decode path (one process per GPU,
torch.distributed for the plumbing).

lisa-rs drives a single Apple GPU and has no multi-device code; these are the
two ways the B200 build spreads the path over the GPUs of one node:

* Batched decode (independent sequences): ``plan_sequences`` assigns whole
  sequences to ranks (longest-processing-time first, balanced by context
  length). Ranks never exchange data.
* One long sequence: its KV positions are split into contiguous windows, one
  per rank (``plan_windows``). Every rank runs ``lisa_attn_decode_window`` on
  its window and gets per-(row, head) partials (normalised O, max, sum); one
  all-gather of those partials (24*rows*(256+2) floats per rank) and
  ``lisa_attn_merge_windows`` give every rank the gated output.
  ``SplitKVDecoder`` wraps this.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

QH, KVH, HD = 24, 4, 256


@dataclass(frozen=True)
class Window:
    rank: int
    lo: int    # first global position held
    rows: int  # positions held (window capacity)


def plan_windows(capacity: int, world: int, align: int = 128) -> list[Window]:
    """Contiguous windows covering positions [0, capacity), one per rank, sizes
    multiples of `align` except the last (the rank that appends new rows)."""
    if world < 1 or capacity < 1:
        raise ValueError("world and capacity must be positive")
    per = -(-capacity // world)
    per = -(-per // align) * align
    out = []
    lo = 0
    for r in range(world):
        rows = max(0, min(per, capacity - lo))
        out.append(Window(r, lo, rows))
        lo += rows
    return out


def plan_sequences(ctx_lens: list[int], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of sequence indices to ranks,
    balancing the sum of context lengths (the KV bytes each rank streams)."""
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(ctx_lens)), key=lambda i: -ctx_lens[i]):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + ctx_lens[i], r))
    for seqs in out:
        seqs.sort()
    return out


def gather_partials(part_o, part_ml, group=None):
    """Host-transport form of the window exchange (any torch.distributed
    backend, e.g. gloo ranks on CPU): one all-gather of each rank's partials
    packed as [rows, 24, 256 + 2] (O, max, sum) into one [world, ...] buffer;
    returns stacked (O, (max, sum)) in rank order (the merge order). The GPU
    path exchanges the same records through peer memory (WindowExchange)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return part_o.unsqueeze(0), part_ml.unsqueeze(0)  # a single window
    world = dist.get_world_size(group)
    packed = torch.cat([part_o, part_ml], dim=-1).contiguous()
    out = torch.empty((world * packed.shape[0],) + tuple(packed.shape[1:]), dtype=packed.dtype,
                      device=packed.device)
    dist.all_gather_into_tensor(out, packed, group=group)
    out = out.view((world,) + tuple(packed.shape))
    return out[..., :HD].contiguous(), out[..., HD:].contiguous()


class PeerLost(RuntimeError):
    """A rank of the split-KV group left or stopped answering between steps."""


class PeerMonitor:
    """Host-side liveness of the ranks that share one split-KV sequence.

    Every rank runs a heartbeat thread that bumps ``hb/<rank>`` in a
    torch.distributed Store every ``interval`` seconds and watches the other
    ranks' counters; a rank that calls ``leave()`` writes ``left/<rank>``. A
    peer whose counter has not moved for ``stale_after`` seconds, that left,
    or a store that stopped answering marks the group lost. ``check()`` (one
    attribute read, called before every step's launch) then raises PeerLost,
    so no rank launches a step whose exchange a departed peer would never
    complete."""

    def __init__(self, store, rank: int, world: int, interval: float = 0.1, stale_after: float = 2.0,
                 prefix: str = "lisa_split"):
        import threading

        self.store, self.rank, self.world = store, rank, world
        self.interval, self.stale_after, self.prefix = interval, stale_after, prefix
        self.lost: str | None = None
        self._stop = threading.Event()
        self._beat = 0
        self.store.set(self._key("hb", rank), "0")
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _key(self, kind: str, r: int) -> str:
        return f"{self.prefix}/{kind}/{r}"

    def _run(self):
        import time

        last = {r: (None, time.monotonic()) for r in range(self.world) if r != self.rank}
        while not self._stop.is_set():
            try:
                self._beat += 1
                self.store.set(self._key("hb", self.rank), str(self._beat))
                for r in last:
                    if self.store.check([self._key("left", r)]):
                        self.lost = f"rank {r} left"
                        return
                    val = self.store.get(self._key("hb", r)) if self.store.check([self._key("hb", r)]) else None
                    now = time.monotonic()
                    if val != last[r][0]:
                        last[r] = (val, now)
                    elif now - last[r][1] > self.stale_after:
                        self.lost = f"rank {r} stopped its heartbeat"
                        return
            except Exception as e:  # the store itself went away (its host rank exited)
                self.lost = f"store unreachable: {type(e).__name__}"
                return
            self._stop.wait(self.interval)

    def check(self) -> None:
        if self.lost is not None:
            raise PeerLost(self.lost)

    def leave(self) -> None:
        """Announce a clean departure between steps, then stop beating."""
        self._stop.set()
        try:
            self.store.set(self._key("left", self.rank), "1")
        except Exception:
            pass

    def close(self) -> None:
        self._stop.set()


class SplitKVDecoder:
    """One attention layer of one long sequence whose KV cache is split over
    the ranks of `group` (this rank holds ``window``; one process per GPU).
    decode() appends the new rows inside the owning window, attends, exchanges
    the window partials through peer memory (lisa_attn_xchg_decode: split,
    combine with peer stores, bounded-wait merge) and returns the gated bf16
    output [rows, 6144] on every rank. ``monitor`` (a PeerMonitor) is checked
    before every launch."""

    def __init__(self, window: Window, device=None, max_rows: int = 3, group=None, monitor=None):
        import torch
        import torch.distributed as dist

        import lisa_attn

        self.window = window
        self.group = group
        self.monitor = monitor
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        rows = max(window.rows, 1)
        self.k = torch.zeros((KVH, rows, HD), dtype=torch.bfloat16, device=self.device)
        self.v = torch.zeros_like(self.k)
        multi = dist.is_available() and dist.is_initialized()
        world = dist.get_world_size(group) if multi else 1
        rank = dist.get_rank(group) if multi else 0
        self.xchg = lisa_attn.WindowExchange(world, rank, rows, max_rows, device=self.device.index)
        handles = [None] * world
        if multi:
            dist.all_gather_object(handles, self.xchg.handle(), group=group)
        else:
            handles = [self.xchg.handle()]
        self.xchg.open(handles)
        if multi:
            dist.barrier(group=group)  # every rank has mapped every region before the first step
        # window workspace for the separate-call form (decode_window / merge_windows)
        self.workspace = torch.empty(lisa_attn.window_workspace_bytes(rows, max_rows), dtype=torch.uint8,
                                     device=self.device)
        self.part_o = torch.empty((max_rows, QH, HD), dtype=torch.float32, device=self.device)
        self.part_ml = torch.empty((max_rows, QH, 2), dtype=torch.float32, device=self.device)

    def decode(self, base: int, q_gate, k, v, w, out=None, stream=None):
        import torch

        if self.monitor is not None:
            self.monitor.check()
        rows = q_gate.numel() // (QH * 512)
        if out is None:
            out = torch.empty((rows, QH * HD), dtype=torch.bfloat16, device=self.device)
        return self.xchg.decode(self.k, self.v, self.window.lo, base, rows, q_gate, k, v, w, out, stream=stream)

    def check_device_error(self, stream=None) -> None:
        self.xchg.check_device_error(stream)
