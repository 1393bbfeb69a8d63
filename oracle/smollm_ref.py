"""SmolLM2-135M forward restated from the reference's smollm.py (test oracle).

This is the caller side of the drop-in boundary: the same layer computation
(smollm.py:168-253) and the same attention hook — when a layer's
`npu` dict holds "attention" and T > 1 (or decode attention is enabled), the
layer flattens (batch, head, query block) into a run_batch call
(smollm.py:129-166); otherwise it runs the CPU attention (smollm.py:222-234).
Weights come from `make_state_dict`, a seeded random init with the HF key
names (the real checkpoint is not available offline).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

BUCKETS_TK = (32, 64, 128, 256, 512, 1024, 2048, 4096, 8192)  # smollm.py:20


@dataclass
class Config:  # smollm.py:23-34
    dim: int = 576
    n_layers: int = 30
    n_heads: int = 9
    n_kv_heads: int = 3
    head_dim: int = 64
    ffn_dim: int = 1536
    vocab: int = 49152
    max_pos: int = 8192
    rope_theta: float = 100000.0
    rms_eps: float = 1e-5


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMSNorm returned in x's dtype (smollm.py:37-42)."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def rope_tables(head_dim: int, max_pos: int, theta: float, dtype, device):
    """cos/sin [max_pos, head_dim], halves duplicated (smollm.py:45-50)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x * cos + rotate_half(x) * sin, rotate_half = [-x2, x1] (smollm.py:53-58)."""
    half = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., half:], x[..., :half]], dim=-1) * sin


def bucket_tk(tk: int) -> int:
    """Smallest decode bucket >= tk (smollm.py:61-65)."""
    for b in BUCKETS_TK:
        if b >= tk:
            return b
    raise ValueError(f"Tk={tk} exceeds max bucket {BUCKETS_TK[-1]}")


def make_state_dict(cfg: Config, seed: int = 0, dtype=torch.float32, std: float = 0.02) -> dict:
    """Seeded N(0, std) weights with HF key names; norm weights are 1."""
    g = torch.Generator().manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(dtype)

    D, Hd = cfg.dim, cfg.head_dim
    sd = {"model.embed_tokens.weight": w(cfg.vocab, D)}
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = w(cfg.n_heads * Hd, D)
        sd[p + "self_attn.k_proj.weight"] = w(cfg.n_kv_heads * Hd, D)
        sd[p + "self_attn.v_proj.weight"] = w(cfg.n_kv_heads * Hd, D)
        sd[p + "self_attn.o_proj.weight"] = w(D, cfg.n_heads * Hd)
        sd[p + "mlp.gate_proj.weight"] = w(cfg.ffn_dim, D)
        sd[p + "mlp.up_proj.weight"] = w(cfg.ffn_dim, D)
        sd[p + "mlp.down_proj.weight"] = w(D, cfg.ffn_dim)
        sd[p + "input_layernorm.weight"] = torch.ones(D, dtype=dtype)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(D, dtype=dtype)
    sd["model.norm.weight"] = torch.ones(D, dtype=dtype)
    return sd


class Layer:
    """One decoder block; `npu` / `npu_decode_attention` are the hook
    attributes SmolLM.enable_npu sets (smollm.py:98-101, :297-320)."""

    def __init__(self, sd: dict, i: int):
        p = f"model.layers.{i}."
        self.wq = sd[p + "self_attn.q_proj.weight"]
        self.wk = sd[p + "self_attn.k_proj.weight"]
        self.wv = sd[p + "self_attn.v_proj.weight"]
        self.wo = sd[p + "self_attn.o_proj.weight"]
        self.w_gate = sd[p + "mlp.gate_proj.weight"]
        self.w_up = sd[p + "mlp.up_proj.weight"]
        self.w_down = sd[p + "mlp.down_proj.weight"]
        self.ln1 = sd[p + "input_layernorm.weight"]
        self.ln2 = sd[p + "post_attention_layernorm.weight"]
        self.npu = None
        self.npu_decode = None
        self.npu_decode_cpu = False
        self.npu_decode_attention = False

    def _fa_attention(self, q, k_exp, v_exp, start_pos, B, T, Tk, Hq, Dh, bucket_kv=False):
        """Flatten (B, Hq, query block) into one run_batch call
        (smollm.py:129-166): pad T to BR and Tk to BC (or a decode bucket),
        duplicate the expanded K/V per query block, start_rows = i*BR+start_pos."""
        attn = self.npu["attention"]
        BR, BC = attn.BR, attn.BC
        Tq_pad = -(-T // BR) * BR
        Tk_pad = bucket_tk(Tk) if bucket_kv else -(-Tk // BC) * BC
        n_q = Tq_pad // BR
        if Tq_pad > T:
            q = torch.cat([q, q.new_zeros(B, Hq, Tq_pad - T, Dh)], dim=2)
        if Tk_pad > Tk:
            pad = k_exp.new_zeros(B, Hq, Tk_pad - Tk, Dh)
            k_exp = torch.cat([k_exp, pad], dim=2)
            v_exp = torch.cat([v_exp, pad], dim=2)
        N = B * Hq * n_q
        q_stack = q.reshape(B, Hq, n_q, BR, Dh).reshape(N, BR, Dh).contiguous()
        k_stack = k_exp[:, :, None].expand(B, Hq, n_q, Tk_pad, Dh).reshape(N, Tk_pad, Dh).contiguous()
        v_stack = v_exp[:, :, None].expand(B, Hq, n_q, Tk_pad, Dh).reshape(N, Tk_pad, Dh).contiguous()
        start_rows = [i * BR + start_pos for _ in range(B * Hq) for i in range(n_q)]
        o = attn.run_batch(q_stack, k_stack, v_stack, start_rows, causal=True).float()
        o = o.reshape(B, Hq, Tq_pad, Dh)[:, :, :T]
        return o.transpose(1, 2).contiguous().reshape(B, T, Hq * Dh)

    def forward(self, x, cos, sin, cfg: Config, past, start_pos: int):
        """smollm.py:168-253 (unfused projections, CPU attention or the hook)."""
        B, T, _ = x.shape
        Hq, Hkv, Dh = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        h = rms_norm(x, self.ln1, cfg.rms_eps)
        q = F.linear(h, self.wq).view(B, T, Hq, Dh).transpose(1, 2)
        k = F.linear(h, self.wk).view(B, T, Hkv, Dh).transpose(1, 2)
        v = F.linear(h, self.wv).view(B, T, Hkv, Dh).transpose(1, 2)
        cs, sn = cos[start_pos:start_pos + T], sin[start_pos:start_pos + T]
        q, k = rope(q, cs, sn), rope(k, cs, sn)
        if past is not None:
            k = torch.cat([past[0], k], dim=2)
            v = torch.cat([past[1], v], dim=2)
        new_cache = (k, v)
        k_exp = k.repeat_interleave(Hq // Hkv, dim=1)
        v_exp = v.repeat_interleave(Hq // Hkv, dim=1)
        Tk = k_exp.shape[2]
        if self.npu is not None and "attention" in self.npu and (T > 1 or self.npu_decode_attention):
            o = self._fa_attention(q, k_exp, v_exp, start_pos, B, T, Tk, Hq, Dh,
                                   bucket_kv=(T == 1 and self.npu_decode_attention))
        else:
            att = torch.matmul(q, k_exp.transpose(-2, -1)) / math.sqrt(Dh)
            if T > 1:
                row = torch.arange(T, device=x.device)[:, None] + start_pos
                col = torch.arange(Tk, device=x.device)[None, :]
                att = att + torch.where(col <= row, 0.0, float("-inf")).to(att.dtype)
            att = F.softmax(att.float(), dim=-1).to(x.dtype)
            o = torch.matmul(att, v_exp).transpose(1, 2).contiguous().view(B, T, Hq * Dh)
        x = x + F.linear(o, self.wo)
        h = rms_norm(x, self.ln2, cfg.rms_eps)
        x = x + F.linear(F.silu(F.linear(h, self.w_gate)) * F.linear(h, self.w_up), self.w_down)
        return x, new_cache


class SmolLM:
    """smollm.py:256-357: embedding, 30 layers, final norm, tied head."""

    def __init__(self, sd: dict, cfg: Config):
        self.cfg = cfg
        self.embed = sd["model.embed_tokens.weight"]
        self.layers = [Layer(sd, i) for i in range(cfg.n_layers)]
        self.final_norm = sd["model.norm.weight"]
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.max_pos, cfg.rope_theta, self.embed.dtype,
                                         self.embed.device)

    def to(self, device) -> "SmolLM":
        for name in ("embed", "final_norm", "cos", "sin"):
            setattr(self, name, getattr(self, name).to(device))
        for layer in self.layers:
            for name in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "ln1", "ln2"):
                setattr(layer, name, getattr(layer, name).to(device))
        return self

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cache=None, start_pos: int = 0):
        if cache is None:
            cache = [None] * self.cfg.n_layers
        x = self.embed[ids]
        new_cache = [None] * self.cfg.n_layers
        for i, layer in enumerate(self.layers):
            x, new_cache[i] = layer.forward(x, self.cos, self.sin, self.cfg, cache[i], start_pos)
        x = rms_norm(x, self.final_norm, self.cfg.rms_eps)
        return F.linear(x, self.embed), new_cache
