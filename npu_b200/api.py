"""Torch-facing native API over the C ABI: causal GQA prefill and split-KV decode.

These are the B200 entry points behind the reference-compatible wrapper in
npu_b200.fa (NpuAttention.run_batch). Tensors must already be CUDA bf16 with a
contiguous head dimension; nothing here falls back to a CPU path.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda_bf16(name: str, t: torch.Tensor, ndim: int) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU path exists)")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bfloat16, got {t.dtype}")
    if t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} needs a contiguous last (head_dim) dimension")


def prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    start_pos: int = 0,
    start_pos_per_batch: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    causal: bool = True,
    out_dtype: torch.dtype = torch.float32,
    out: Optional[torch.Tensor] = None,
    return_lse: bool = False,
):
    """Attention forward for q [B, Hq, Tq, D] against k/v [B, Hkv, Tk, D].

    Row r of q sits at absolute position start + r (start = start_pos, or
    start_pos_per_batch[b] if given as an int32 CUDA tensor [B]). With causal,
    key c is masked iff c > start + r; rows with no key output 0 — the
    semantics of flash_attention_ref (npu/fa_ref.py:42-131). Query head h uses
    KV head h // (Hq // Hkv). Returns o [B, Hq, Tq, D] in out_dtype (and the
    natural-log LSE [B, Hq, Tq] if return_lse).
    """
    _need_cuda_bf16("q", q, 4)
    _need_cuda_bf16("k", k, 4)
    _need_cuda_bf16("v", v, 4)
    B, Hq, Tq, D = q.shape
    Bk, Hkv, Tk, Dk = k.shape
    if (Bk, Dk) != (B, D) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, Hq, Tq, D), dtype=out_dtype, device=q.device)
    elif out.dtype != out_dtype or tuple(out.shape) != (B, Hq, Tq, D) or out.stride(-1) != 1:
        raise ValueError("out must match [B, Hq, Tq, D], out_dtype and a contiguous last dim")
    lse = torch.empty((B, Hq, Tq), dtype=torch.float32, device=q.device) if return_lse else None
    spb = None
    if start_pos_per_batch is not None:
        spb = start_pos_per_batch
        if spb.dtype != torch.int32 or spb.device != q.device or spb.numel() != B or not spb.is_contiguous():
            raise ValueError("start_pos_per_batch must be a contiguous int32 tensor [B] on q's device")
    lib = _lib.load()
    with torch.cuda.device(q.device):
        rc = lib.b2a_prefill(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None,
            B, Hq, Hkv, Tq, Tk, D,
            _lib.ll3(*q.stride()[:3]), _lib.ll3(*k.stride()[:3]), _lib.ll3(*v.stride()[:3]),
            _lib.ll3(*out.stride()[:3]),
            int(start_pos), spb.data_ptr() if spb is not None else None,
            float(scale), 1 if causal else 0, 1 if out_dtype == torch.float32 else 0,
            _stream_ptr(q.device),
        )
    _lib.check(rc, "b2a_prefill")
    return (out, lse) if return_lse else out


def decode_workspace_bytes(B: int, Hq: int, Hkv: int, D: int, Lmax: int, split_len: int = 0) -> int:
    return int(_lib.load().b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split_len))


def decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    seqlens: torch.Tensor,
    *,
    scale: Optional[float] = None,
    out_dtype: torch.dtype = torch.float32,
    split_len: int = 0,
    workspace: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One query token per sequence: q [B, Hq, D] against caches [B, Hkv, Lmax, D].

    Sequence b attends to keys 0 .. seqlens[b]-1 with no mask (the T=1 path of
    smollm.py:222-234). seqlens is an int32 CUDA tensor [B]. The split-KV
    scratch is taken from `workspace` (a uint8 CUDA tensor) or allocated here
    through torch's caching allocator.
    """
    _need_cuda_bf16("q", q, 3)
    _need_cuda_bf16("k_cache", k_cache, 4)
    _need_cuda_bf16("v_cache", v_cache, 4)
    B, Hq, D = q.shape
    Bk, Hkv, Lmax, Dk = k_cache.shape
    if (Bk, Dk) != (B, D) or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k_cache.shape)} v{tuple(v_cache.shape)}")
    if seqlens.dtype != torch.int32 or seqlens.device != q.device or seqlens.numel() != B:
        raise ValueError("seqlens must be an int32 tensor [B] on q's device")
    seqlens = seqlens.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = _lib.load()
    if split_len == 0:
        split_len = int(lib.b2a_decode_default_split(B, Hkv, Lmax))
    need = int(lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split_len))
    if need == 0:
        raise _lib.B2AError(_lib.B2A_ERR_INVALID_ARG, "b2a_decode_workspace_bytes")
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty((B, Hq, D), dtype=out_dtype, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.b2a_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seqlens.data_ptr(), out.data_ptr(),
            B, Hq, Hkv, Lmax, D,
            _lib.ll2(*q.stride()[:2]), _lib.ll3(*k_cache.stride()[:3]), _lib.ll3(*v_cache.stride()[:3]),
            _lib.ll2(*out.stride()[:2]),
            float(scale), int(split_len), 1 if out.dtype == torch.float32 else 0,
            workspace.data_ptr(), need, _stream_ptr(q.device),
        )
    _lib.check(rc, "b2a_decode")
    return out


def device_error(clear: bool = True, device: Optional[torch.device] = None) -> int:
    """Status the kernels left in the device error word (synchronises)."""
    import ctypes

    device = device or torch.device("cuda", torch.cuda.current_device())
    st = ctypes.c_int(0)
    with torch.cuda.device(device):
        _lib.check(_lib.load().b2a_get_device_error(ctypes.byref(st), 1 if clear else 0, _stream_ptr(device)),
                   "b2a_get_device_error")
    return st.value
