"""Qwen3.5/3.6 gated attention restated from the reference (test oracle).

Follows qwen/forward.py: rms_norm (:58-61), build_partial_rope_cache (:64-78),
apply_partial_rope (:81-95) and attn_forward (:133-239): per-head Q/K RMSNorm,
partial rotary on the first rope_dim lanes of each head, GQA by
repeat_interleave, a cache of expanded heads grown with torch.cat, softmax in
fp32, output gated by sigmoid(q_gate) before the output projection. The real
weights come from a GGUF file that is not available offline; `make_layer`
draws seeded random ones with the reference's shapes (the q projection holds
[q_h | gate_h] per head, interleaved, qwen/forward.py:159-162,185-188).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class QwenAttnConfig:
    """The attention fields of qwen/model.py:29-50 (Qwen3.6 geometry:
    n_head 16, n_head_kv 2, head_dim 256, rope_dim 64, qwen/forward.py:6-9);
    d_model, eps and theta are stand-ins for the GGUF metadata."""

    d_model: int = 2048
    n_head: int = 16
    n_head_kv: int = 2
    head_dim: int = 256
    rope_dim: int = 64
    rms_eps: float = 1e-6
    rope_theta: float = 10000000.0


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """qwen/forward.py:58-61: fp32 statistics, result in x's dtype."""
    xf = x.float()
    return ((xf * xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()) * w.float()).to(x.dtype)


def partial_rope_tables(rope_dim: int, max_pos: int, theta: float, dtype=torch.float32, device="cpu"):
    """qwen/forward.py:64-78: cos/sin [max_pos, rope_dim], halves duplicated."""
    inv = 1.0 / (theta ** (torch.arange(0, rope_dim, 2, dtype=torch.float32, device=device) / rope_dim))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def partial_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, rope_dim: int) -> torch.Tensor:
    """qwen/forward.py:81-95: x [B, T, H, Dh], cos/sin [T, rope_dim]; rotate-half
    on x[..., :rope_dim], the other lanes pass through."""
    xr, xp = x[..., :rope_dim], x[..., rope_dim:]
    h = rope_dim // 2
    rot = torch.cat([-xr[..., h:], xr[..., :h]], dim=-1)
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat([xr * c + rot * s, xp], dim=-1)


@dataclass
class QwenAttnLayer:
    attn_norm: torch.Tensor   # [d_model]
    wq: torch.Tensor          # [2 * n_head * head_dim, d_model]: per head [q | gate]
    wk: torch.Tensor          # [n_head_kv * head_dim, d_model]
    wv: torch.Tensor
    wo: torch.Tensor          # [d_model, n_head * head_dim]
    q_norm: torch.Tensor      # [head_dim]
    k_norm: torch.Tensor


def make_layer(cfg: QwenAttnConfig, seed: int = 0, dtype=torch.float32, std: float = 0.02) -> QwenAttnLayer:
    g = torch.Generator().manual_seed(seed)

    def w(*shape, scale=std, base=0.0):
        return (base + torch.randn(*shape, generator=g) * scale).to(dtype)

    Hq, Hkv, Dh, D = cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.d_model
    return QwenAttnLayer(attn_norm=w(D, scale=0.1, base=1.0), wq=w(2 * Hq * Dh, D), wk=w(Hkv * Dh, D),
                         wv=w(Hkv * Dh, D), wo=w(D, Hq * Dh), q_norm=w(Dh, scale=0.1, base=1.0),
                         k_norm=w(Dh, scale=0.1, base=1.0))


def attn_forward(x: torch.Tensor, layer: QwenAttnLayer, cfg: QwenAttnConfig, cos: torch.Tensor,
                 sin: torch.Tensor, kv_cache, start_pos: int, pre_proj: bool = False):
    """qwen/forward.py:133-239 (CPU branch). Returns (out [B, T, d_model],
    (k, v) cache of expanded heads [B, Tk, Hq, Dh]); with pre_proj the gated
    attention output [B, T, Hq * Dh] before the output projection."""
    B, T, _ = x.shape
    Hq, Hkv, Dh, rd = cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.rope_dim
    h = rms_norm(x, layer.attn_norm, cfg.rms_eps)
    q_full = F.linear(h, layer.wq).view(B, T, Hq, 2, Dh)
    q, q_gate = q_full[..., 0, :], q_full[..., 1, :]
    k = F.linear(h, layer.wk).view(B, T, Hkv, Dh)
    v = F.linear(h, layer.wv).view(B, T, Hkv, Dh)
    q = rms_norm(q, layer.q_norm, cfg.rms_eps)
    k = rms_norm(k, layer.k_norm, cfg.rms_eps)
    q = partial_rope(q, cos[start_pos:start_pos + T], sin[start_pos:start_pos + T], rd)
    k = partial_rope(k, cos[start_pos:start_pos + T], sin[start_pos:start_pos + T], rd)
    k = k.repeat_interleave(Hq // Hkv, dim=2)
    v = v.repeat_interleave(Hq // Hkv, dim=2)
    if kv_cache is not None:
        k = torch.cat([kv_cache[0], k], dim=1)
        v = torch.cat([kv_cache[1], v], dim=1)
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    scores = torch.matmul(qt, kt.transpose(-2, -1)) / (Dh ** 0.5)
    Tk = kt.shape[-2]
    if T > 1:
        rows = torch.arange(T) + start_pos
        cols = torch.arange(Tk)
        scores = scores.masked_fill(cols[None, :] > rows[:, None], float("-inf"))
    attn = F.softmax(scores.float(), dim=-1).to(q.dtype)
    out = torch.matmul(attn, vt).transpose(1, 2).contiguous()
    out = (out * torch.sigmoid(q_gate)).view(B, T, Hq * Dh)
    return (out if pre_proj else F.linear(out, layer.wo)), (k, v)


# Golden cases run through the reference's own attn_forward by
# tests/golden/make_golden.py (qwen_attn.npz). The head geometry is Qwen3.6's
# (16 / 2 heads, head_dim 256, rope_dim 64, theta 1e7); d_model is 256 to keep
# the fixture small (it only sizes the projections around the attention).
# Weights and inputs are regenerated from these seeds at test time, and their
# SHA-256 fingerprints are stored next to the outputs.
QWEN_GOLDEN_CASES = {
    # tag: (dtype, batch, prefill tokens, decode steps, weight seed, input seed)
    "f32": (torch.float32, 2, 300, 4, 31, 32),
    "bf16": (torch.bfloat16, 1, 40, 2, 33, 34),
}
QWEN_GOLDEN_MAX_POS = 1024


def golden_config() -> QwenAttnConfig:
    return QwenAttnConfig(d_model=256)


def golden_case(tag: str):
    """(cfg, layer, prefill x, [decode x per step]) for one golden case."""
    dtype, B, T, steps, wseed, xseed = QWEN_GOLDEN_CASES[tag]
    cfg = golden_config()
    layer = make_layer(cfg, seed=wseed, dtype=dtype)
    g = torch.Generator().manual_seed(xseed)
    x = torch.randn(B, T, cfg.d_model, generator=g).to(dtype)
    xs = [torch.randn(B, 1, cfg.d_model, generator=g).to(dtype) for _ in range(steps)]
    return cfg, layer, x, xs


def fingerprint(*tensors: torch.Tensor) -> str:
    """SHA-256 over the raw bytes of the tensors (bf16 as its bit pattern)."""
    import hashlib

    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()


def layer_tensors(layer: QwenAttnLayer) -> list:
    return [layer.attn_norm, layer.wq, layer.wk, layer.wv, layer.wo, layer.q_norm, layer.k_norm]
