"""Qwen3.5/3.6 gated attention on the B200 kernels (the reference's
attn_forward, qwen/forward.py:133-239, for one attention block).

Reference: RMSNorm -> q projection holding [q_h | gate_h] per head -> per-head
Q/K RMSNorm -> partial RoPE (first 64 of 256 lanes) -> repeat_interleave to
16 heads and torch.cat into a cache of expanded heads -> dense attention in
fp32 -> out * sigmoid(gate) -> output projection.

Here:
  * the q and k/v projections are two cuBLAS GEMMs (wk and wv stacked);
  * one b2a_qk_norm_rope_append launch normalises and rotates q and k and
    appends k, v to a device-resident KVCache with the 2 KV heads unexpanded
    (GQA 8:1 read natively by the attention kernels, 8x less cache);
  * b2a_prefill_gated (T > 1) / b2a_decode_gated (T = 1) apply sigmoid(gate)
    in the attention kernels' output stores and write O straight into the
    [B, T, Hq * D] layout the output projection takes (no transpose copy);
  * the output projection is a cuBLAS GEMM.
The gate is read in place from the q projection (a strided view).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import api
from .kvcache import KVCache


@dataclass
class QwenAttnConfig:
    """Attention hyper-parameters (the attention fields of qwen/model.py:29-50)."""

    d_model: int = 2048
    n_head: int = 16
    n_head_kv: int = 2
    head_dim: int = 256
    rope_dim: int = 64
    rms_eps: float = 1e-6
    rope_theta: float = 10000000.0
    max_pos: int = 32768


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """qwen/forward.py:58-61: fp32 statistics, result in x's dtype."""
    xf = x.float()
    return ((xf * xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()) * w.float()).to(x.dtype)


def partial_rope_tables(rope_dim: int, max_pos: int, theta: float, dtype, device):
    """cos/sin [max_pos, rope_dim] as build_partial_rope_cache (qwen/forward.py:64-78)."""
    inv = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float32, device=device) / rope_dim))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous()


class QwenGatedAttentionB200:
    """One gated attention block over a KVCache (layer index `layer` in it)."""

    def __init__(self, attn_norm, wq, wk, wv, wo, q_norm, k_norm, cfg: QwenAttnConfig, device: torch.device,
                 dtype: Optional[torch.dtype] = None):
        dtype = dtype or wq.dtype
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("the block runs in float32 or bfloat16")
        Hq, Hkv, Dh = cfg.n_head, cfg.n_head_kv, cfg.head_dim
        if tuple(wq.shape) != (2 * Hq * Dh, cfg.d_model) or tuple(wo.shape) != (cfg.d_model, Hq * Dh):
            raise ValueError("wq must be [2 * n_head * head_dim, d_model] and wo [d_model, n_head * head_dim]")

        def t(x):
            return x.to(device=device, dtype=dtype).contiguous()

        self.cfg, self.device, self.dtype = cfg, device, dtype
        self.attn_norm, self.wq, self.wo = t(attn_norm), t(wq), t(wo)
        self.wkv = torch.cat([t(wk), t(wv)], dim=0).contiguous()
        self.q_norm, self.k_norm = t(q_norm), t(k_norm)
        self.cos, self.sin = partial_rope_tables(cfg.rope_dim, cfg.max_pos, cfg.rope_theta, dtype, device)
        self._ws = None

    def new_cache(self, batch: int, max_len: int, n_layers: int = 1) -> KVCache:
        return KVCache(n_layers, batch, self.cfg.n_head_kv, max_len, self.cfg.head_dim, self.device)

    @torch.no_grad()
    def attention(self, x: torch.Tensor, cache: KVCache, layer: int = 0) -> torch.Tensor:
        """Gated attention output before the output projection, [B, T, Hq * D]
        in the block dtype. Appends this step's k, v to the cache (the caller
        advances the cache once per step, after its last layer)."""
        c = self.cfg
        B, T, _ = x.shape
        Hq, Hkv, Dh = c.n_head, c.n_head_kv, c.head_dim
        h = _rms_norm(x, self.attn_norm, c.rms_eps)
        qf = F.linear(h, self.wq).view(B, T, Hq, 2, Dh)        # per head [q | gate]
        kv = F.linear(h, self.wkv)
        q, gate = qf[:, :, :, 0], qf[:, :, :, 1]                 # [B, T, Hq, Dh] views
        k = kv[..., :Hkv * Dh].view(B, T, Hkv, Dh)
        v = kv[..., Hkv * Dh:].view(B, T, Hkv, Dh)
        k_cache, v_cache = cache.layer(layer)
        q_rot = api.rope_append(q, k, v, self.cos, self.sin, k_cache, v_cache,
                                start_pos_per_batch=cache.start, seqlens_out=cache.end,
                                q_norm=self.q_norm, k_norm=self.k_norm, norm_eps=c.rms_eps,
                                rope_dim=c.rope_dim)
        out = torch.empty((B, T, Hq, Dh), dtype=x.dtype, device=x.device)
        if T == 1:
            if self._ws is None or self._ws.numel() < api.decode_workspace_bytes(B, Hq, Hkv, Dh, cache.max_len):
                self._ws = torch.empty(api.decode_workspace_bytes(B, Hq, Hkv, Dh, cache.max_len),
                                       dtype=torch.uint8, device=x.device)
            api.decode(q_rot[:, :, 0], k_cache, v_cache, cache.end, out_dtype=x.dtype, out=out[:, 0],
                       workspace=self._ws, gate=gate[:, 0])
        else:
            api.prefill(q_rot, k_cache, v_cache, start_pos_per_batch=cache.start, scale=1.0 / math.sqrt(Dh),
                        causal=True, out_dtype=x.dtype, out=out.transpose(1, 2), gate=gate.transpose(1, 2))
        return out.view(B, T, Hq * Dh)

    @torch.no_grad()
    def forward(self, x: torch.Tensor, cache: KVCache, layer: int = 0) -> torch.Tensor:
        """attn_forward's output [B, T, d_model] (before the residual add)."""
        return F.linear(self.attention(x, cache, layer), self.wo)
