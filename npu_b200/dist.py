"""Multi-GPU partitioning of the attention hot path (one process per GPU).

The reference runs on a single device (pyxrt.device(0), npu/fa.py:183-188) and
its only work split is over its 4 AIE tiles (npu/fa.py:92-124). Here:

* Batched prefill / decode: independent (batch, KV head) units or whole
  sequences are sharded across ranks; there is no collective on the data path.
* A single long sequence (context-parallel prefill): query rows are cut into
  2G chunks and rank g owns chunks g and 2G-1-g (zig-zag), which balances the
  causal work; each rank holds K/V for the positions of its own chunks, and
  one NCCL all-gather over NVLink assembles the full K/V before the local
  attention. No reduction is needed: every rank owns the complete softmax of
  its rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch


def shard_units(B: int, Hkv: int, world: int, rank: int) -> list[tuple[int, int, int]]:
    """Contiguous share of the B*Hkv (batch, KV head) units for `rank`, as
    (batch, kv_lo, kv_hi) segments. Units are ordered batch-major, so when
    world divides B every rank gets whole batches."""
    n = B * Hkv
    lo, hi = rank * n // world, (rank + 1) * n // world
    segs = []
    u = lo
    while u < hi:
        b, hk = divmod(u, Hkv)
        end = min(hi, (b + 1) * Hkv)
        segs.append((b, hk, hk + (end - u)))
        u = end
    return segs


def shard_sequences(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of decode sequences to ranks, balancing
    the total KV length (the bytes each rank streams)."""
    bins: list[list[int]] = [[] for _ in range(world)]
    load = [0] * world
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        bins[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(b) for b in bins]


def zigzag_chunks(T: int, world: int, rank: int) -> list[tuple[int, int]]:
    """Row ranges [start, end) of the two zig-zag chunks rank owns: the
    sequence is cut into 2*world chunks; rank g gets chunks g and 2*world-1-g."""
    n = 2 * world
    if T % n:
        raise ValueError(f"T={T} must be divisible by 2*world={n}")
    c = T // n
    return [(rank * c, (rank + 1) * c), ((n - 1 - rank) * c, (n - rank) * c)]


def causal_flops_rows(rows: tuple[int, int], D: int, Hq: int, B: int = 1) -> int:
    """Algorithmic FLOPs of causal attention for query rows [r0, r1) starting
    at position r0 with keys 0..r (4*D per query-key pair per head)."""
    r0, r1 = rows
    keys = (r1 * (r1 + 1) - r0 * (r0 + 1)) // 2
    return 4 * B * Hq * D * keys


@dataclass
class ContextParallelPrefill:
    """Zig-zag context-parallel causal prefill of one long sequence.

    Each rank passes q_local [B, Hq, 2c, D] and k_local / v_local
    [B, Hkv, 2c, D]: the rows of its two chunks (zigzag_chunks) back to back.
    `run` all-gathers K and V into [B, Hkv, T, D] and returns this rank's
    output rows [B, Hq, 2c, D]. `attn_fn(q, k, v, start_pos)` is the
    attention kernel (npu_b200.api.prefill by default, which then writes both
    chunks' rows straight into `out`).

    The gather runs in two halves. Rank g's first chunk is chunk g, so the
    first chunks of all ranks are rows [0, T/2) in rank order; its second
    chunk is chunk 2G-1-g, so the second chunks are rows [T/2, T) in reverse
    rank order. A rank's first chunk needs keys from the first half only: its
    attention runs while the second half is still being gathered, and the
    second chunk (which needs every key before it) runs after it.
    """

    T: int
    world: int
    rank: int
    group: Optional[object] = None
    attn_fn: Optional[Callable] = None

    def __post_init__(self):
        self.chunks = zigzag_chunks(self.T, self.world, self.rank)
        self.c = self.T // (2 * self.world)
        self.launches_per_run = 2

    def _gather_half(self, k_part: torch.Tensor, v_part: torch.Tensor, async_op: bool):
        """All ranks' [B, H, c, D] K and V parts -> [world, 2, B, H, c, D] in
        rank order (one collective for K and V together)."""
        import torch.distributed as dist

        send = torch.stack([k_part, v_part])
        flat = torch.empty((self.world * 2,) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        work = dist.all_gather_into_tensor(flat, send, group=self.group, async_op=async_op)
        return flat.view((self.world,) + tuple(send.shape)), work

    def _place(self, full: torch.Tensor, recv: torch.Tensor, second: bool) -> None:
        """Copy one gathered half into its rows of full [2, B, H, T, D]: rank
        g's first chunk is chunk g, its second chunk is chunk 2G-1-g."""
        _, B, H, T, D = full.shape
        w, c = self.world, self.c
        src = recv.permute(1, 2, 3, 0, 4, 5)  # [2, B, H, world, c, D]
        if second:
            src = src.flip(3)
        half = full[:, :, :, w * c:] if second else full[:, :, :, :w * c]
        half.view(2, B, H, w, c, D).copy_(src)

    def gather_kv(self, k_local: torch.Tensor, v_local: torch.Tensor):
        """Blocking gather of the whole sequence's K and V [B, H, T, D]."""
        B, H, two_c, D = k_local.shape
        assert two_c == 2 * self.c
        c = self.c
        full = torch.empty((2, B, H, self.T, D), dtype=k_local.dtype, device=k_local.device)
        r1, _ = self._gather_half(k_local[:, :, :c], v_local[:, :, :c], async_op=False)
        r2, _ = self._gather_half(k_local[:, :, c:], v_local[:, :, c:], async_op=False)
        self._place(full, r1, second=False)
        self._place(full, r2, second=True)
        return full[0], full[1]

    def run(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
            out: Optional[torch.Tensor] = None, **kw) -> torch.Tensor:
        B, H, two_c, D = k_local.shape
        assert two_c == 2 * self.c
        c = self.c
        full = torch.empty((2, B, H, self.T, D), dtype=k_local.dtype, device=k_local.device)
        r1, w1 = self._gather_half(k_local[:, :, :c], v_local[:, :, :c], async_op=True)
        r2, w2 = self._gather_half(k_local[:, :, c:], v_local[:, :, c:], async_op=True)
        if self.attn_fn is None:
            from .api import prefill

            if out is None:
                out = torch.empty(q_local.shape, dtype=kw.get("out_dtype", torch.float32), device=q_local.device)

            def attend(slot, k, v, start):
                return prefill(q_local[:, :, slot * c:(slot + 1) * c], k, v, start_pos=start, causal=True,
                               out=out[:, :, slot * c:(slot + 1) * c], **kw)
        else:
            def attend(slot, k, v, start):
                return self.attn_fn(q_local[:, :, slot * c:(slot + 1) * c], k, v, start, **kw)

        outs = []
        for slot, (work, recv) in enumerate(((w1, r1), (w2, r2))):
            work.wait()  # NCCL: the current stream waits; the host does not
            self._place(full, recv, second=slot == 1)
            r0, r1_ = self.chunks[slot]
            outs.append(attend(slot, full[0, :, :, :r1_], full[1, :, :, :r1_], r0))
        if self.attn_fn is None:
            return out
        return torch.cat(outs, dim=2)
