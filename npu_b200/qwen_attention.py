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

`attn_forward` at the end of this file keeps the reference function's own
signature and tuple cache of expanded heads (a one-import drop-in for
qwen/forward.py) and runs the same attention kernels on that cache.
"""
from __future__ import annotations

import math
import weakref
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


# Device copies of layers' attention weights, by id() of the layer object and
# dropped when that object is collected (layer classes such as dataclasses
# are not hashable, so a weak-key dictionary cannot hold them).
_LAYER_WEIGHTS: dict = {}


def _layer_on_device(layer, device: torch.device, dtype: torch.dtype) -> dict:
    """The layer's attention weights on `device` in `dtype`: the tensors
    themselves when they already are, else copies made on first use and kept
    while the layer object lives (later in-place changes to the layer's host
    weights are not seen)."""
    names = ("attn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm")
    if all(getattr(layer, n).device == device and getattr(layer, n).dtype == dtype for n in names):
        return {n: getattr(layer, n) for n in names}
    lid = id(layer)
    per_layer = _LAYER_WEIGHTS.get(lid)
    if per_layer is None:
        per_layer = _LAYER_WEIGHTS[lid] = {}
        try:
            weakref.finalize(layer, _LAYER_WEIGHTS.pop, lid, None)
        except TypeError:  # not weak-referenceable: the copies live until exit
            pass
    key = (str(device), dtype)
    if key not in per_layer:
        per_layer[key] = {n: getattr(layer, n).to(device=device, dtype=dtype).contiguous() for n in names}
    return per_layer[key]


@torch.no_grad()
def attn_forward(x: torch.Tensor, layer, cfg, cos: torch.Tensor, sin: torch.Tensor, kv_cache, start_pos: int,
                 device: Optional[torch.device] = None):
    """Drop-in for the reference's attn_forward (qwen/forward.py:133-239):
    same arguments (x [B, T, d_model]; `layer` with attn_norm, wq holding
    [q_h | gate_h] per head, wk, wv, wo, q_norm, k_norm; `cfg` with n_head,
    n_head_kv, head_dim, rope_dim, rms_eps; the cos / sin tables of
    build_partial_rope_cache; the (k, v) cache of expanded heads [B, Tk,
    n_head, head_dim] or None; the absolute position of x's first token) and
    the same results: the block output [B, T, d_model] on x's device and dtype,
    and the new (k, v) cache, grown by torch.cat as in the reference.

    Projections, the per-head Q/K RMSNorm, the partial RoPE and the cache
    concatenation run as torch ops on `device` (default: the current CUDA
    device), in x's dtype as in the reference. The attention itself runs on
    the B200 kernels with the sigmoid gate fused into their output stores:
    b2a_prefill_gated for T > 1 (causal from start_pos), b2a_decode_gated for
    T = 1 (every cached key, no mask, qwen/forward.py:211-216). The kernels read
    one copy of each KV head from the expanded cache (a head stride of
    n_head / n_head_kv heads), so GQA costs no extra cache traffic. The
    returned cache lives on `device` as bf16 (the kernels' input type); a
    caller passes it back unchanged, as the reference's forward does."""
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("attn_forward needs a CUDA device (no CPU path)")
        device = torch.device("cuda", torch.cuda.current_device())
    B, T, _ = x.shape
    Hq, Hkv, Dh, rd = cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.rope_dim
    rep = Hq // Hkv
    dtype = x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32
    w = _layer_on_device(layer, device, dtype)
    xd = x.to(device=device, dtype=dtype)
    h = _rms_norm(xd, w["attn_norm"], cfg.rms_eps)
    q_full = F.linear(h, w["wq"]).view(B, T, Hq, 2, Dh)
    q, q_gate = q_full[..., 0, :], q_full[..., 1, :]
    k = F.linear(h, w["wk"]).view(B, T, Hkv, Dh)
    v = F.linear(h, w["wv"]).view(B, T, Hkv, Dh)
    q = _rms_norm(q, w["q_norm"], cfg.rms_eps)
    k = _rms_norm(k, w["k_norm"], cfg.rms_eps)
    cs = cos[start_pos:start_pos + T].to(device=device, dtype=dtype)
    sn = sin[start_pos:start_pos + T].to(device=device, dtype=dtype)

    def rope(t):  # qwen/forward.py:81-95: rotate-half on the first rd lanes
        tr, tp = t[..., :rd], t[..., rd:]
        half = rd // 2
        rot = torch.cat([-tr[..., half:], tr[..., :half]], dim=-1)
        return torch.cat([tr * cs[None, :, None, :] + rot * sn[None, :, None, :], tp], dim=-1)

    q, k = rope(q), rope(k)
    k = k.to(torch.bfloat16).repeat_interleave(rep, dim=2)
    v = v.to(torch.bfloat16).repeat_interleave(rep, dim=2)
    if kv_cache is not None:
        k = torch.cat([kv_cache[0].to(device=device, dtype=torch.bfloat16), k], dim=1)
        v = torch.cat([kv_cache[1].to(device=device, dtype=torch.bfloat16), v], dim=1)
    Tk = k.shape[1]
    # One copy of each KV head: heads 0, rep, 2 rep, ... of the expanded cache.
    kh = k[:, :, ::rep].transpose(1, 2)   # [B, Hkv, Tk, Dh], strided view
    vh = v[:, :, ::rep].transpose(1, 2)
    qb = q.to(torch.bfloat16)
    out = torch.empty((B, T, Hq, Dh), dtype=dtype, device=device)
    if T == 1:
        seqlens = torch.full((B,), Tk, dtype=torch.int32, device=device)
        api.decode(qb[:, 0], kh, vh, seqlens, scale=1.0 / math.sqrt(Dh), out_dtype=dtype, out=out[:, 0],
                   gate=q_gate[:, 0])
    else:
        api.prefill(qb.transpose(1, 2), kh, vh, start_pos=start_pos, scale=1.0 / math.sqrt(Dh), causal=True,
                    out_dtype=dtype, out=out.transpose(1, 2), gate=q_gate.transpose(1, 2))
    y = F.linear(out.view(B, T, Hq * Dh), w["wo"])
    return y.to(device=x.device, dtype=x.dtype), (k, v)
