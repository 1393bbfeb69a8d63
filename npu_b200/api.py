"""Torch-facing native API over the C ABI: causal GQA prefill, split-KV decode
and the fused RoPE + KV-cache append that feeds them.

These are the B200 entry points behind the reference-compatible wrapper in
npu_b200.fa (NpuAttention.run_batch). Tensors are CUDA bf16 with a contiguous
head dimension, except for prefill_host, which takes host bf16 tensors and
moves them itself; nothing here falls back to a CPU path.
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


def _check_gate(gate: torch.Tensor, shape: tuple, device: torch.device) -> None:
    if not isinstance(gate, torch.Tensor) or gate.device != device:
        raise ValueError("gate must be a CUDA tensor on q's device")
    if gate.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("gate must be float32 or bfloat16")
    if tuple(gate.shape) != tuple(shape) or gate.stride(-1) != 1:
        raise ValueError(f"gate must be {list(shape)} with a contiguous last dim, got {tuple(gate.shape)}")


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
    gate: Optional[torch.Tensor] = None,
):
    """Attention forward for q [B, Hq, Tq, D] against k/v [B, Hkv, Tk, D].

    Row r of q sits at absolute position start + r (start = start_pos, or
    start_pos_per_batch[b] if given as an int32 CUDA tensor [B]). With causal,
    key c is masked iff c > start + r; rows with no key output 0 — the
    semantics of flash_attention_ref (npu/fa_ref.py:42-131). Query head h uses
    KV head h // (Hq // Hkv). Returns o [B, Hq, Tq, D] in out_dtype (and the
    natural-log LSE [B, Hq, Tq] if return_lse). With `gate` ([B, Hq, Tq, D],
    fp32 or bf16, any strides with a contiguous last dim) the output is
    attention * sigmoid(gate), fused into the kernel's stores (Qwen's gated
    attention, qwen/forward.py:223-226).
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
    if gate is not None:
        _check_gate(gate, (B, Hq, Tq, D), q.device)
    with torch.cuda.device(q.device):
        if gate is None:
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
        else:
            rc = lib.b2a_prefill_gated(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(), out.data_ptr(),
                lse.data_ptr() if lse is not None else None,
                B, Hq, Hkv, Tq, Tk, D,
                _lib.ll3(*q.stride()[:3]), _lib.ll3(*k.stride()[:3]), _lib.ll3(*v.stride()[:3]),
                _lib.ll3(*gate.stride()[:3]), _lib.ll3(*out.stride()[:3]),
                1 if gate.dtype == torch.bfloat16 else 0,
                int(start_pos), spb.data_ptr() if spb is not None else None,
                float(scale), 1 if causal else 0, 1 if out_dtype == torch.float32 else 0,
                _stream_ptr(q.device),
            )
    _lib.check(rc, "b2a_prefill")
    return (out, lse) if return_lse else out


def prefill_host_workspace_bytes(B: int, Hq: int, Hkv: int, Tq: int, Tk: int, D: int,
                                 out_fp32: bool = False, n_chunks: int = 0) -> int:
    return int(_lib.load().b2a_prefill_host_workspace_bytes(B, Hq, Hkv, Tq, Tk, D, 1 if out_fp32 else 0,
                                                            n_chunks))


def prefill_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    start_pos: int = 0,
    start_pos_per_batch=None,
    scale: Optional[float] = None,
    causal: bool = True,
    out_dtype: torch.dtype = torch.bfloat16,
    out: Optional[torch.Tensor] = None,
    n_chunks: int = 0,
    device: Optional[torch.device] = None,
    workspace: Optional[torch.Tensor] = None,
    sync: bool = True,
) -> torch.Tensor:
    """`prefill` for tensors in HOST memory (b2a_prefill_host): q [B, Hq, Tq, D]
    and k/v [B, Hkv, Tk, D] contiguous bf16 CPU tensors, result o [B, Hq, Tq, D]
    on the host (page-locked when allocated here). The work is cut into
    n_chunks pieces whose uploads, kernels and downloads overlap on the GPU
    `device` (default: the current one). start_pos_per_batch, if given, is a
    host sequence / CPU int32 tensor [B]. With sync=False the call returns once
    the copies and kernels are queued on the device's current stream; the
    inputs must then stay untouched and `out` unread until that stream is
    synchronised. Page-locked inputs (`tensor.pin_memory()`) are needed for the
    copies to overlap; pageable ones give the same result, serialised.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor) or t.is_cuda:
            raise ValueError(f"{name} must be a CPU tensor (use prefill for device tensors)")
        if t.dtype != torch.bfloat16 or t.dim() != 4 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous 4-d bfloat16 tensor, got {t.dtype} {tuple(t.shape)}")
    B, Hq, Tq, D = q.shape
    Bk, Hkv, Tk, Dk = k.shape
    if (Bk, Dk) != (B, D) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is not None and (out.is_cuda or out.dtype != out_dtype or tuple(out.shape) != (B, Hq, Tq, D)
                            or not out.is_contiguous()):
        raise ValueError("out must be a contiguous CPU tensor [B, Hq, Tq, D] of out_dtype")
    spb = None
    if start_pos_per_batch is not None:
        if isinstance(start_pos_per_batch, torch.Tensor) and start_pos_per_batch.is_cuda:
            raise ValueError("start_pos_per_batch must be on the host")
        spb = torch.as_tensor(start_pos_per_batch, dtype=torch.int32).contiguous()
        if spb.numel() != B:
            raise ValueError("start_pos_per_batch must be a host sequence of B int32 positions")
    if device is None:
        if not torch.cuda.is_available():
            raise RuntimeError("prefill_host needs a CUDA device (no CPU path)")
        device = torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if out is None:
        out = torch.empty((B, Hq, Tq, D), dtype=out_dtype, pin_memory=True)
    out_fp32 = out_dtype == torch.float32
    lib = _lib.load()
    need = int(lib.b2a_prefill_host_workspace_bytes(B, Hq, Hkv, Tq, Tk, D, 1 if out_fp32 else 0, n_chunks))
    if need == 0:
        _lib.check(_lib.B2A_ERR_INVALID_ARG, "b2a_prefill_host_workspace_bytes")
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    elif not workspace.is_cuda or workspace.device != device or workspace.numel() < need:
        raise ValueError(f"workspace must be a CUDA uint8 tensor of >= {need} bytes on {device}")
    with torch.cuda.device(device):
        rc = lib.b2a_prefill_host(
            q.data_ptr(), k.data_ptr() if Tk else None, v.data_ptr() if Tk else None, out.data_ptr(),
            B, Hq, Hkv, Tq, Tk, D, int(start_pos), spb.data_ptr() if spb is not None else None,
            float(scale), 1 if causal else 0, 1 if out_fp32 else 0, int(n_chunks),
            workspace.data_ptr(), workspace.numel(), _stream_ptr(device),
        )
        _lib.check(rc, "b2a_prefill_host")
        if sync:
            torch.cuda.current_stream(device).synchronize()
    return out


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
    gate: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One query token per sequence: q [B, Hq, D] against caches [B, Hkv, Lmax, D].

    Sequence b attends to keys 0 .. seqlens[b]-1 with no mask (the T=1 path of
    smollm.py:222-234). seqlens is an int32 CUDA tensor [B]. The split-KV
    scratch is taken from `workspace` (a uint8 CUDA tensor) or allocated here
    through torch's caching allocator. With `gate` ([B, Hq, D], fp32 or bf16)
    the output is attention * sigmoid(gate), fused into the combine kernel.
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
    if gate is not None:
        _check_gate(gate, (B, Hq, D), q.device)
    with torch.cuda.device(q.device):
        if gate is None:
            rc = lib.b2a_decode(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seqlens.data_ptr(), out.data_ptr(),
                B, Hq, Hkv, Lmax, D,
                _lib.ll2(*q.stride()[:2]), _lib.ll3(*k_cache.stride()[:3]), _lib.ll3(*v_cache.stride()[:3]),
                _lib.ll2(*out.stride()[:2]),
                float(scale), int(split_len), 1 if out.dtype == torch.float32 else 0,
                workspace.data_ptr(), need, _stream_ptr(q.device),
            )
        else:
            rc = lib.b2a_decode_gated(
                q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seqlens.data_ptr(), gate.data_ptr(),
                out.data_ptr(), B, Hq, Hkv, Lmax, D,
                _lib.ll2(*q.stride()[:2]), _lib.ll3(*k_cache.stride()[:3]), _lib.ll3(*v_cache.stride()[:3]),
                _lib.ll2(*gate.stride()[:2]), _lib.ll2(*out.stride()[:2]),
                1 if gate.dtype == torch.bfloat16 else 0,
                float(scale), int(split_len), 1 if out.dtype == torch.float32 else 0,
                workspace.data_ptr(), need, _stream_ptr(q.device),
            )
    _lib.check(rc, "b2a_decode")
    return out


def decode_proj(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    seqlens: torch.Tensor,
    wo: torch.Tensor,
    x: torch.Tensor,
    *,
    scale: Optional[float] = None,
    split_len: int = 0,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Decode attention fused with the output projection and residual add
    (b2a_decode_proj): x += attention(q, caches) @ wo.T, in place.

    q [B, Hq, D] and the caches as `decode`; wo [dim, Hq * D] (the F.linear
    weight of the output projection, fp32 or bf16, last dim contiguous); x the
    residual stream [B, dim] (fp32 or bf16, last dim contiguous), returned.
    The attention output is rounded to x's dtype before the projection, as
    the unfused `x + F.linear(o, wo)` would see it; every output has one
    writer and a fixed summation order (reproducible results).
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
    for name, t in (("wo", wo), ("x", x)):
        if not isinstance(t, torch.Tensor) or t.device != q.device or t.dim() != 2 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a 2-d CUDA tensor on q's device with a contiguous last dim")
        if t.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"{name} must be float32 or bfloat16")
    dim = wo.shape[0]
    if wo.shape[1] != Hq * D or tuple(x.shape) != (B, dim):
        raise ValueError(f"wo must be [dim, {Hq * D}] and x [{B}, dim], got wo{tuple(wo.shape)} x{tuple(x.shape)}")
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
    with torch.cuda.device(q.device):
        rc = lib.b2a_decode_proj(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seqlens.data_ptr(), wo.data_ptr(),
            wo.stride(0), 1 if wo.dtype == torch.float32 else 0, dim, x.data_ptr(), x.stride(0),
            1 if x.dtype == torch.float32 else 0, B, Hq, Hkv, Lmax, D,
            _lib.ll2(*q.stride()[:2]), _lib.ll3(*k_cache.stride()[:3]), _lib.ll3(*v_cache.stride()[:3]),
            float(scale), int(split_len), workspace.data_ptr(), need, _stream_ptr(q.device),
        )
    _lib.check(rc, "b2a_decode_proj")
    return x


def rope_append(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    start_pos: int = 0,
    start_pos_per_batch: Optional[torch.Tensor] = None,
    seqlens_out: Optional[torch.Tensor] = None,
    q_out: Optional[torch.Tensor] = None,
    q_norm: Optional[torch.Tensor] = None,
    k_norm: Optional[torch.Tensor] = None,
    norm_eps: float = 1e-6,
    rope_dim: Optional[int] = None,
) -> torch.Tensor:
    """Rotate q and k and append k, v to a device-resident cache, in place.

    q [B, T, Hq, D], k and v [B, T, Hkv, D] (fp32 or bf16, last dim
    contiguous; typically views of one fused QKV projection) are rotated with
    the rotary tables cos/sin [max_pos, D] (same dtype, rotate-half form of
    smollm.py:53-58) at positions p_b + t, p_b = start_pos_per_batch[b] or
    start_pos. k and v land in rows p_b .. p_b + T - 1 of k_cache/v_cache
    [B, Hkv, Lmax, D] bf16; seqlens_out (int32 [B], optional) receives
    p_b + T. Returns q rotated as [B, Hq, T, D] bf16, the layout prefill and
    decode take.

    Qwen's gated-attention prologue (qwen/forward.py:178-204): q_norm /
    k_norm ([D], q's dtype) RMS-normalise each q / k head first (eps
    norm_eps), and rope_dim < D rotates only the first rope_dim lanes (cos/sin
    are then [max_pos, rope_dim]).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not t.is_cuda or t.dim() != 4 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a CUDA [B, T, H, D] tensor with a contiguous last dim")
    if q.dtype not in (torch.float32, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must share one dtype, float32 or bfloat16")
    if cos.dtype != q.dtype or sin.dtype != q.dtype or not cos.is_contiguous() or not sin.is_contiguous():
        raise ValueError("cos/sin must be contiguous [max_pos, D] tensors in q's dtype")
    _need_cuda_bf16("k_cache", k_cache, 4)
    _need_cuda_bf16("v_cache", v_cache, 4)
    B, T, Hq, D = q.shape
    Hkv = k.shape[2]
    Bc, Hc, Lmax, Dc = k_cache.shape
    if tuple(k.shape) != (B, T, Hkv, D) or tuple(v.shape) != (B, T, Hkv, D):
        raise ValueError(f"shape mismatch q{tuple(q.shape)} k{tuple(k.shape)} v{tuple(v.shape)}")
    if (Bc, Hc, Dc) != (B, Hkv, D) or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError(f"cache shape {tuple(k_cache.shape)} does not fit k{tuple(k.shape)}")
    rope_dim = D if rope_dim is None else int(rope_dim)
    if cos.dim() != 2 or cos.shape[1] != rope_dim or tuple(sin.shape) != tuple(cos.shape):
        raise ValueError("cos/sin must be [max_pos, rope_dim]")
    for name, w in (("q_norm", q_norm), ("k_norm", k_norm)):
        if w is not None and (w.dtype != q.dtype or w.device != q.device or tuple(w.shape) != (D,)
                              or not w.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous [D] tensor in q's dtype on q's device")
    spb = None
    if start_pos_per_batch is not None:
        spb = start_pos_per_batch
        if spb.dtype != torch.int32 or spb.device != q.device or spb.numel() != B or not spb.is_contiguous():
            raise ValueError("start_pos_per_batch must be a contiguous int32 tensor [B] on q's device")
    if seqlens_out is not None:
        if (seqlens_out.dtype != torch.int32 or seqlens_out.device != q.device or seqlens_out.numel() != B
                or not seqlens_out.is_contiguous()):
            raise ValueError("seqlens_out must be a contiguous int32 tensor [B] on q's device")
    if q_out is None:
        q_out = torch.empty((B, Hq, T, D), dtype=torch.bfloat16, device=q.device)
    elif q_out.dtype != torch.bfloat16 or tuple(q_out.shape) != (B, Hq, T, D) or not q_out.is_contiguous():
        raise ValueError("q_out must be a contiguous bf16 [B, Hq, T, D] tensor")
    lib = _lib.load()
    with torch.cuda.device(q.device):
        rc = lib.b2a_qk_norm_rope_append(
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            _lib.ll3(*q.stride()[:3]), _lib.ll3(*k.stride()[:3]), _lib.ll3(*v.stride()[:3]),
            1 if q.dtype == torch.bfloat16 else 0,
            q_norm.data_ptr() if q_norm is not None else None,
            k_norm.data_ptr() if k_norm is not None else None, float(norm_eps),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], rope_dim,
            q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
            _lib.ll3(*k_cache.stride()[:3]), _lib.ll3(*v_cache.stride()[:3]),
            B, T, Hq, Hkv, D, Lmax, int(start_pos),
            spb.data_ptr() if spb is not None else None,
            seqlens_out.data_ptr() if seqlens_out is not None else None,
            _stream_ptr(q.device),
        )
    _lib.check(rc, "b2a_qk_norm_rope_append")
    return q_out


def device_error(clear: bool = True, device: Optional[torch.device] = None) -> int:
    """Status the kernels left in the device error word (synchronises)."""
    import ctypes

    device = device or torch.device("cuda", torch.cuda.current_device())
    st = ctypes.c_int(0)
    with torch.cuda.device(device):
        _lib.check(_lib.load().b2a_get_device_error(ctypes.byref(st), 1 if clear else 0, _stream_ptr(device)),
                   "b2a_get_device_error")
    return st.value
