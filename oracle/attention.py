"""fp32 CPU restatement of the reference's attention arithmetic (test oracle).

Each function names the reference lines it follows. Inputs are typically bf16
and are upcast to fp32, as the reference does (npu/fa_ref.py:69-73,
npu/fa_ref.py:138).
"""
from __future__ import annotations

import math
from typing import Sequence

import torch

NEG_INF = float("-inf")


def expand_kv(k: torch.Tensor, n_rep: int) -> torch.Tensor:
    """GQA expansion [B, Hkv, T, D] -> [B, Hkv*n_rep, T, D]: each KV head is
    repeated n_rep times consecutively (repeat_interleave over heads,
    smollm.py:205-207, qwen/forward.py:194-197)."""
    if n_rep == 1:
        return k
    B, H, T, D = k.shape
    return k[:, :, None].expand(B, H, n_rep, T, D).reshape(B, H * n_rep, T, D)


def causal_mask(tq: int, tk: int, start_pos: int) -> torch.Tensor:
    """Boolean [tq, tk], True where key c is hidden from query row r:
    c > start_pos + r (npu/fa_ref.py:57-60, :105-107)."""
    rows = torch.arange(tq)[:, None] + start_pos
    cols = torch.arange(tk)[None, :]
    return cols > rows


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, start_pos: int = 0,
                    causal: bool = True, scale: float | None = None) -> torch.Tensor:
    """Materialised-score attention, fp32: the CPU path of smollm.py:222-234 and
    _torch_causal_attention (npu/fa_ref.py:134-145). q [B, Hq, Tq, D],
    k/v [B, Hkv, Tk, D] with Hq a multiple of Hkv (expanded here).

    Rows whose keys are all masked come out as 0, the convention of
    flash_attention_ref (npu/fa_ref.py:125-128); softmax alone would give NaN.
    """
    B, Hq, Tq, D = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    kf = expand_kv(k.float(), Hq // Hkv)
    vf = expand_kv(v.float(), Hq // Hkv)
    sc = (1.0 / math.sqrt(D)) if scale is None else scale
    s = torch.matmul(q.float(), kf.transpose(-2, -1)) * sc
    if causal:
        s = s.masked_fill(causal_mask(Tq, Tk, start_pos), NEG_INF)
    dead = torch.isneginf(s).all(dim=-1, keepdim=True)
    p = torch.softmax(s.masked_fill(dead, 0.0), dim=-1).masked_fill(dead, 0.0)
    return torch.matmul(p, vf)


def flash_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, Br: int, Bc: int,
                        causal: bool = True, start_pos: int = 0,
                        scale: float | None = None) -> torch.Tensor:
    """Block-streaming online-softmax forward (FA-2), fp32, restating
    flash_attention_ref (npu/fa_ref.py:42-131): per query block, running max m,
    running sum l and accumulator O over key blocks; alpha = exp(m - m_new)
    with fully masked rows guarded to 0 (npu/fa_ref.py:111-123); final O / l
    with l == 0 rows left at 0 (npu/fa_ref.py:125-128). Tail blocks are clipped.
    Vectorised over (batch, head); q/k/v share the head count (the caller
    expands GQA first, as the reference does)."""
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    assert k.shape == (B, H, Tk, D) and v.shape == (B, H, Tk, D)
    sc = (1.0 / math.sqrt(D)) if scale is None else scale
    qf, kf, vf = q.float(), k.float(), v.float()
    out = torch.zeros((B, H, Tq, D), dtype=torch.float32)
    for r0 in range(0, Tq, Br):
        r1 = min(r0 + Br, Tq)
        qi = qf[:, :, r0:r1]
        m = torch.full((B, H, r1 - r0), NEG_INF)
        l = torch.zeros((B, H, r1 - r0))
        acc = torch.zeros((B, H, r1 - r0, D))
        for c0 in range(0, Tk, Bc):
            c1 = min(c0 + Bc, Tk)
            s = torch.matmul(qi, kf[:, :, c0:c1].transpose(-2, -1)) * sc
            if causal:
                hide = (torch.arange(c0, c1)[None, :] > (torch.arange(r0, r1)[:, None] + start_pos))
                s = s.masked_fill(hide, NEG_INF)
            m_new = torch.maximum(m, s.amax(dim=-1))
            dead = torch.isneginf(m_new)
            alpha = torch.where(dead, torch.zeros_like(m), torch.exp(m - m_new))
            p = torch.where(dead[..., None], torch.zeros_like(s), torch.exp(s - m_new[..., None]))
            l = alpha * l + p.sum(dim=-1)
            acc = alpha[..., None] * acc + torch.matmul(p, vf[:, :, c0:c1])
            m = m_new
        live = l > 0
        acc = acc / torch.where(live, l, torch.ones_like(l))[..., None]
        out[:, :, r0:r1] = torch.where(live[..., None], acc, torch.zeros_like(acc))
    return out


def run_batch_ref(Q_stack: torch.Tensor, K_stack: torch.Tensor, V_stack: torch.Tensor,
                  start_rows: Sequence[int], causal: bool = True) -> torch.Tensor:
    """What NpuAttention.run_batch (npu/fa.py:206-323) returns, in fp32: block n
    is Q_stack[n] [BR, D] against K/V_stack[n] [TK, D] with its rows at
    absolute positions start_rows[n] + r (the header start_row,
    npu/fa.py:270-272, npu/fa_kernel.cc:72-74)."""
    N = Q_stack.shape[0]
    out = torch.empty(Q_stack.shape, dtype=torch.float32)
    for n in range(N):
        out[n] = dense_attention(Q_stack[n][None, None], K_stack[n][None, None], V_stack[n][None, None],
                                 start_pos=int(start_rows[n]), causal=causal)[0, 0]
    return out


def decode_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
               seqlens: Sequence[int], scale: float | None = None) -> torch.Tensor:
    """Single-token decode: sequence b's query [Hq, D] against its first
    seqlens[b] cached keys, no mask (smollm.py:224-234 with T=1, where the mask
    is only applied for T > 1). q [B, Hq, D], caches [B, Hkv, Lmax, D] -> fp32
    [B, Hq, D]; an empty sequence gives 0."""
    B, Hq, D = q.shape
    out = torch.zeros((B, Hq, D), dtype=torch.float32)
    for b in range(B):
        L = int(seqlens[b])
        if L <= 0:
            continue
        out[b] = dense_attention(q[b][None, :, None], k_cache[b:b + 1, :, :L], v_cache[b:b + 1, :, :L],
                                 causal=False, scale=scale)[0, :, 0]
    return out


def prefill_rows_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, b: int, h: int,
                     rows: Sequence[int], start_pos: int = 0, causal: bool = True,
                     scale: float | None = None, positions: Sequence[int] | None = None) -> torch.Tensor:
    """fp32 attention for selected query rows of one (batch, query head): used
    to check large problems on a sample of rows. Row r sits at absolute
    position start_pos + r, or positions[i] for the i-th row when given (so q
    may hold only the sampled rows). Returns [len(rows), D]."""
    Hq, D = q.shape[1], q.shape[3]
    hk = h // (Hq // k.shape[1])
    sc = (1.0 / math.sqrt(D)) if scale is None else scale
    qr = q[b, h, list(rows)].float()
    kf = k[b, hk].float()
    vf = v[b, hk].float()
    s = (qr @ kf.T) * sc
    if causal:
        if positions is not None:
            pos = torch.as_tensor(list(positions))[:, None]
        else:
            pos = torch.as_tensor(list(rows))[:, None] + start_pos
        s = s.masked_fill(torch.arange(kf.shape[0])[None, :] > pos, NEG_INF)
    dead = torch.isneginf(s).all(dim=-1, keepdim=True)
    p = torch.softmax(s.masked_fill(dead, 0.0), dim=-1).masked_fill(dead, 0.0)
    return p @ vf


def attention_flops(B: int, Hq: int, D: int, Tq: int, Tk: int, start_pos: int = 0, causal: bool = True) -> int:
    """Algorithmic FLOPs = 4 * B * Hq * D * sum over rows of unmasked keys
    (QK^T and PV, 2 FLOPs per multiply-add; masked work not counted)."""
    if not causal:
        return 4 * B * Hq * D * Tq * Tk
    import numpy as np

    keys = np.clip(np.arange(Tq, dtype=np.int64) + start_pos + 1, 0, Tk).sum()
    return 4 * B * Hq * D * int(keys)
