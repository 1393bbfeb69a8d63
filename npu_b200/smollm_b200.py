"""SmolLM2 forward with the attention path and its callers on the B200 kernels.

The reference's layer (smollm.py:168-253) projects q, k and v, rotates q and k
(apply_rope), grows the layer's (k, v) cache with torch.cat, expands GQA heads
with repeat_interleave and then runs attention on the CPU or through
run_batch. Here the same layer math runs as:

  * one fused QKV projection (wq, wk, wv stacked: a single cuBLAS GEMM);
  * b2a_rope_append: rotation of q and k and an in-place append of k and v
    into a device-resident KVCache, in one launch, heads never expanded;
  * b2a_prefill (T > 1, causal from each sequence's cache position) or
    b2a_decode (T = 1) reading the cache directly;
  * output projection, RMSNorms and the SwiGLU MLP in torch, as in the
    reference.

Sequence positions stay on the device (KVCache), so a decode step issues no
host synchronisation. Weights use the reference's HF key names
(smollm.py:84-93, :256-265). The model may run in fp32 (the reference's NPU
configuration) or bf16; attention always takes bf16 Q/K/V.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import api
from .kvcache import KVCache
from .profiler import profile


@dataclass
class SmolLMConfig:
    """Architecture hyper-parameters (the fields of smollm.py:23-34)."""

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
    """RMSNorm computed in fp32, returned in x's dtype (smollm.py:37-42)."""
    xf = x.float()
    return ((xf * xf.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()) * w.float()).to(x.dtype)


def rope_tables(head_dim: int, max_pos: int, theta: float, dtype, device):
    """Rotary cos/sin [max_pos, head_dim] as build_rope_cache (smollm.py:45-50):
    fp32 angles, halves duplicated, cast to the model dtype."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    ang = torch.outer(torch.arange(max_pos, dtype=torch.float32, device=device), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous()


class SmolLMB200:
    """Decoder stack over a KVCache; forward(ids, cache) -> logits."""

    def __init__(self, sd: dict, cfg: SmolLMConfig, device: torch.device, dtype: Optional[torch.dtype] = None,
                 fuse_wo: bool = True):
        """fuse_wo: single-token steps run the output projection and residual
        add inside the decode combine kernel (b2a_decode_proj) instead of a
        separate GEMM."""
        dtype = dtype or sd["model.embed_tokens.weight"].dtype
        self.fuse_wo = fuse_wo
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("the model runs in float32 or bfloat16")
        self.cfg, self.device, self.dtype = cfg, device, dtype

        def w(key):
            return sd[key].to(device=device, dtype=dtype).contiguous()

        self.embed = w("model.embed_tokens.weight")
        self.final_norm = w("model.norm.weight")
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"model.layers.{i}."
            self.layers.append({
                "wqkv": torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                   w(p + "self_attn.v_proj.weight")], dim=0).contiguous(),
                "wo": w(p + "self_attn.o_proj.weight"),
                "w_gate": w(p + "mlp.gate_proj.weight"),
                "w_up": w(p + "mlp.up_proj.weight"),
                "w_down": w(p + "mlp.down_proj.weight"),
                "ln1": w(p + "input_layernorm.weight"),
                "ln2": w(p + "post_attention_layernorm.weight"),
            })
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.max_pos, cfg.rope_theta, dtype, device)
        self._ws = None

    def new_cache(self, batch: int, max_len: int) -> KVCache:
        if max_len > self.cfg.max_pos:
            raise ValueError(f"max_len {max_len} exceeds the rotary table length {self.cfg.max_pos}")
        return KVCache(self.cfg.n_layers, batch, self.cfg.n_kv_heads, max_len, self.cfg.head_dim, self.device)

    def _workspace(self, B: int, Lmax: int) -> torch.Tensor:
        c = self.cfg
        need = api.decode_workspace_bytes(B, c.n_heads, c.n_kv_heads, c.head_dim, Lmax)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def _attention(self, lw: dict, h: torch.Tensor, cache: KVCache, i: int, x: torch.Tensor):
        """Attention of layer i; returns the new residual stream (x plus the
        output projection of the attention)."""
        c = self.cfg
        B, T, _ = h.shape
        Hq, Hkv, Dh = c.n_heads, c.n_kv_heads, c.head_dim
        with profile("qkv"):
            qkv = F.linear(h, lw["wqkv"])                                # [B, T, (Hq + 2 Hkv) Dh]
        q = qkv[..., :Hq * Dh].view(B, T, Hq, Dh)
        k = qkv[..., Hq * Dh:(Hq + Hkv) * Dh].view(B, T, Hkv, Dh)
        v = qkv[..., (Hq + Hkv) * Dh:].view(B, T, Hkv, Dh)
        k_cache, v_cache = cache.layer(i)
        with profile("rope"):
            q_rot = api.rope_append(q, k, v, self.cos, self.sin, k_cache, v_cache,
                                    start_pos_per_batch=cache.start, seqlens_out=cache.end)
        if T == 1:
            if self.fuse_wo and x.is_contiguous():
                # Attention, output projection and residual add in one decode
                # (the combine kernel adds o @ wo.T into x in place).
                with profile("attn"):
                    api.decode_proj(q_rot[:, :, 0], k_cache, v_cache, cache.end, lw["wo"], x.view(B, -1),
                                    workspace=self._workspace(B, cache.max_len))
                return x
            with profile("attn"):
                o = api.decode(q_rot[:, :, 0], k_cache, v_cache, cache.end, out_dtype=h.dtype,
                               workspace=self._workspace(B, cache.max_len))
            with profile("wo"):
                return x + F.linear(o.reshape(B, 1, Hq * Dh), lw["wo"])
        # The kernel writes O straight into the [B, T, Hq * Dh] layout the
        # output projection reads (a strided [B, Hq, T, Dh] view of it).
        o = torch.empty((B, T, Hq, Dh), dtype=h.dtype, device=h.device)
        with profile("attn"):
            api.prefill(q_rot, k_cache, v_cache, start_pos_per_batch=cache.start, scale=1.0 / math.sqrt(Dh),
                        causal=True, out_dtype=h.dtype, out=o.transpose(1, 2))
        with profile("wo"):
            return x + F.linear(o.view(B, T, Hq * Dh), lw["wo"])

    @torch.no_grad()
    def capture_decode(self, cache: KVCache, warmup: int = 2):
        """A CUDA graph of one single-token step over `cache` (every layer's
        norm, projections, rope_append, decode attention and MLP: ~12
        launches per layer replayed as one). Returns step(ids [B, 1]) ->
        logits [B, 1, vocab] (a buffer the next replay overwrites). Warm-up and
        capture run real steps; the cache's positions are restored afterwards,
        so the rows they wrote (at most warmup + 1 past each sequence's
        length, which must fit in max_len) are overwritten by the next tokens
        and never read.
        """
        B = cache.batch
        ids_buf = torch.zeros((B, 1), dtype=torch.long, device=self.device)
        self._workspace(B, cache.max_len)  # allocate outside the capture
        saved = cache._pos.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.forward(ids_buf, cache)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.forward(ids_buf, cache)
        cache._pos.copy_(saved)

        def step(ids: torch.Tensor) -> torch.Tensor:
            ids_buf.copy_(ids)
            graph.replay()
            return out

        step.graph = graph
        return step

    @torch.no_grad()
    def capture_prefill(self, cache: KVCache, T: int, warmup: int = 2):
        """A CUDA graph of one T-token prefill step over `cache` (every layer's
        norms, fused QKV GEMM, rope_append, prefill attention, output
        projection and MLP replayed as one launch), the prefill counterpart of
        capture_decode. Returns step(ids [B, T]) -> logits [B, T, vocab] (a
        buffer the next replay overwrites); each replay appends at the
        cache's current positions and advances them, like forward. Warm-up and
        capture run real steps and the positions are restored afterwards, so
        the rows they wrote are overwritten by the next replay."""
        B = cache.batch
        ids_buf = torch.zeros((B, T), dtype=torch.long, device=self.device)
        saved = cache._pos.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                cache._pos.copy_(saved)
                self.forward(ids_buf, cache)
        torch.cuda.current_stream(self.device).wait_stream(side)
        cache._pos.copy_(saved)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.forward(ids_buf, cache)
        cache._pos.copy_(saved)

        def step(ids: torch.Tensor) -> torch.Tensor:
            ids_buf.copy_(ids)
            graph.replay()
            return out

        step.graph = graph
        return step

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cache: KVCache) -> torch.Tensor:
        """Logits [B, T, vocab] for tokens ids [B, T] placed after each
        sequence's cached prefix; appends them to the cache."""
        c = self.cfg
        if ids.dim() != 2 or ids.shape[0] != cache.batch:
            raise ValueError("ids must be [B, T] with B = cache.batch")
        x = self.embed[ids.to(self.device)]
        # Op names follow the reference forward's profile() blocks
        # (smollm.py:179-251), with "attn" for its attn_npu / attn_cpu.
        for i, lw in enumerate(self.layers):
            with profile("rms1"):
                h = rms_norm(x, lw["ln1"], c.rms_eps)
            x = self._attention(lw, h, cache, i, x)
            with profile("rms2"):
                h = rms_norm(x, lw["ln2"], c.rms_eps)
            with profile("gate_up"):
                gu = F.silu(F.linear(h, lw["w_gate"])) * F.linear(h, lw["w_up"])
            with profile("w_down"):
                x = x + F.linear(gu, lw["w_down"])
        cache.advance()
        x = rms_norm(x, self.final_norm, c.rms_eps)
        return F.linear(x, self.embed)
