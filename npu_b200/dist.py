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
    attention kernel (npu_b200.api.prefill by default).
    """

    T: int
    world: int
    rank: int
    group: Optional[object] = None
    attn_fn: Optional[Callable] = None

    def __post_init__(self):
        self.chunks = zigzag_chunks(self.T, self.world, self.rank)
        self.c = self.T // (2 * self.world)

    def gather_kv(self, k_local: torch.Tensor, v_local: torch.Tensor):
        import torch.distributed as dist

        B, H, two_c, D = k_local.shape
        assert two_c == 2 * self.c
        kv = torch.stack([k_local, v_local])  # [2, B, H, 2c, D]
        flat = torch.empty((self.world * 2,) + tuple(kv.shape[1:]), dtype=kv.dtype, device=kv.device)
        dist.all_gather_into_tensor(flat, kv.contiguous(), group=self.group)
        buf = flat.view((self.world,) + tuple(kv.shape))
        full = torch.empty((2, B, H, self.T, D), dtype=kv.dtype, device=kv.device)
        c, n = self.c, 2 * self.world
        for r in range(self.world):
            for slot, chunk in enumerate((r, n - 1 - r)):
                full[:, :, :, chunk * c:(chunk + 1) * c] = buf[r, :, :, :, slot * c:(slot + 1) * c]
        return full[0], full[1]

    def run(self, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor, **kw) -> torch.Tensor:
        attn = self.attn_fn
        if attn is None:
            from .api import prefill

            def attn(q, k, v, start_pos, **kw2):
                return prefill(q, k, v, start_pos=start_pos, causal=True, **kw2)

        k_full, v_full = self.gather_kv(k_local, v_local)
        outs = []
        for slot, (r0, r1) in enumerate(self.chunks):
            qs = q_local[:, :, slot * self.c:(slot + 1) * self.c]
            outs.append(attn(qs, k_full[:, :, :r1], v_full[:, :, :r1], r0, **kw))
        return torch.cat(outs, dim=2)
