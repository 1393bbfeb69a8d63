"""Device-resident KV cache for the attention path.

The reference keeps, per layer, a (k, v) pair of [B, Hkv, T_cached, D] tensors
that every step grows with torch.cat and then expands with repeat_interleave
(smollm.py:68-77, 198-208); its NPU decode route pads Tk to a bucket
(smollm.py:17-20, 144). Here the cache is allocated once at its maximum length
and written in place by npu_b200.api.rope_append, and the prefill/decode
kernels read it directly with per-sequence positions, GQA heads unexpanded.

Positions live on the device in two int32 vectors, so a step needs no host
synchronisation: every layer's append reads the step's start positions from
one and writes start + T into the other (the same value from each layer), the
attention reads lengths from the second, and `advance` copies the second into
the first on the device. The buffers never move, so a step can be captured in
a CUDA graph and replayed.
"""
from __future__ import annotations

import torch


class KVCache:
    """k, v: [n_layers, B, Hkv, max_len, head_dim] bf16 on `device`."""

    def __init__(self, n_layers: int, batch: int, n_kv_heads: int, max_len: int, head_dim: int,
                 device: torch.device):
        if min(n_layers, batch, n_kv_heads, max_len, head_dim) <= 0:
            raise ValueError("KVCache dimensions must be positive")
        shape = (n_layers, batch, n_kv_heads, max_len, head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self._pos = torch.zeros((2, batch), dtype=torch.int32, device=device)
        self.max_len = max_len
        self.batch = batch

    @property
    def start(self) -> torch.Tensor:
        """int32 [B]: position of each sequence's next token (device)."""
        return self._pos[0]

    @property
    def end(self) -> torch.Tensor:
        """int32 [B]: positions after the step in progress (what the appends
        write and the attention reads as sequence lengths)."""
        return self._pos[1]

    def layer(self, i: int):
        return self.k[i], self.v[i]

    def advance(self) -> None:
        """Finish a step: the lengths written by this step become the next
        start (a device copy on the current stream)."""
        self._pos[0].copy_(self._pos[1])

    def reset(self, lengths=None) -> None:
        """Empty the cache (or set per-sequence lengths, e.g. after a prefill
        computed elsewhere); the stored K/V rows are left as they are."""
        if lengths is None:
            self._pos.zero_()
        else:
            self._pos[0].copy_(torch.as_tensor(lengths, dtype=torch.int32))
            self._pos[1].copy_(self._pos[0])

    def lengths(self) -> list:
        """Host copy of the current lengths (synchronises)."""
        return [int(x) for x in self.start.tolist()]
