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
    """All-gather of the window partials of every rank: returns stacked
    tensors [world, ...] in rank order (the merge order)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return part_o.unsqueeze(0), part_ml.unsqueeze(0)  # a single window
    world = dist.get_world_size(group)
    out_o = [torch.empty_like(part_o) for _ in range(world)]
    out_ml = [torch.empty_like(part_ml) for _ in range(world)]
    dist.all_gather(out_o, part_o.contiguous(), group=group)
    dist.all_gather(out_ml, part_ml.contiguous(), group=group)
    return torch.stack(out_o), torch.stack(out_ml)


class SplitKVDecoder:
    """One attention layer of one long sequence whose KV cache is split over
    the ranks of `group` (this rank holds ``window``). decode() appends the new
    rows inside the owning window, attends, exchanges partials and returns the
    gated bf16 output [rows, 6144] on every rank."""

    def __init__(self, window: Window, device=None, max_rows: int = 3, group=None):
        import torch

        import lisa_attn

        self.window = window
        self.group = group
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        rows = max(window.rows, 1)
        self.k = torch.zeros((KVH, rows, HD), dtype=torch.bfloat16, device=self.device)
        self.v = torch.zeros_like(self.k)
        ws = lisa_attn.window_workspace_bytes(rows, max_rows)
        self.workspace = torch.empty(ws, dtype=torch.uint8, device=self.device)
        self.part_o = torch.empty((max_rows, QH, HD), dtype=torch.float32, device=self.device)
        self.part_ml = torch.empty((max_rows, QH, 2), dtype=torch.float32, device=self.device)

    def decode(self, base: int, q_gate, k, v, w, out=None, stream=None):
        import torch

        import lisa_attn

        rows = q_gate.numel() // (QH * 512)
        po, pm = self.part_o[:rows], self.part_ml[:rows]
        lisa_attn.decode_window(self.k, self.v, self.window.lo, base, rows, q_gate, k, v, w, po, pm,
                                self.workspace, stream=stream)
        all_o, all_ml = gather_partials(po, pm, self.group)
        if out is None:
            out = torch.empty((rows, QH * HD), dtype=torch.bfloat16, device=self.device)
        lisa_attn.merge_windows(all_o.shape[0], rows, all_o, all_ml, q_gate, out, stream=stream)
        return out
