"""Parity of the split-KV decode kernels with the fp32 oracle (max|Δ| <= 2e-2)."""
import math

import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _case(B, Hq, Hkv, Lmax, D, lens, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g).bfloat16()
    kc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16()
    vc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16()
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("B,Hq,Hkv,Lmax,D,lens,split", [
    (1, 1, 1, 64, 64, [1], 64),
    (2, 8, 2, 200, 64, [63, 200], 64),
    (3, 9, 3, 300, 64, [64, 65, 300], 128),
    (4, 32, 4, 1024, 128, [1, 500, 1000, 1024], 0),
    (2, 16, 1, 513, 128, [513, 257], 128),
    (3, 16, 2, 700, 256, [700, 1, 333], 192),
    (5, 12, 4, 4200, 128, [4200, 4097, 4096, 2049, 7], 0),
    (2, 4, 4, 128, 128, [0, 128], 64),
])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_decode_matches_oracle(cuda_dev, B, Hq, Hkv, Lmax, D, lens, split, out_dtype):
    from npu_b200 import api

    q, kc, vc, sl = _case(B, Hq, Hkv, Lmax, D, lens, B * 31 + Lmax + D, cuda_dev)
    out = api.decode(q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev), sl.to(cuda_dev), split_len=split,
                     out_dtype=out_dtype)
    ref = A.decode_ref(q, kc, vc, lens)
    assert (out.float().cpu() - ref).abs().max().item() <= TOL
    for b, L in enumerate(lens):
        if L == 0:
            assert torch.all(out[b] == 0)


def test_decode_config4_shape_sampled(cuda_dev):
    """Config 4 geometry (Hq=32, Hkv=4, D=128, L ~ U[1024, 32768]) on 16
    sequences, all heads checked."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, Lmax, D = 16, 32, 4, 32768, 128
    lens = torch.randint(1024, 32769, (B,), generator=g, dtype=torch.int32)
    q = torch.randn(B, Hq, D, generator=g).bfloat16().to(cuda_dev)
    kc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16().to(cuda_dev)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16().to(cuda_dev)
    out = api.decode(q, kc, vc, lens.to(cuda_dev), scale=1 / math.sqrt(128))
    ref = A.decode_ref(q.cpu(), kc.cpu(), vc.cpu(), lens.tolist())
    assert (out.cpu() - ref).abs().max().item() <= TOL


def test_decode_strided_cache_and_query(cuda_dev):
    """A cache stored [B, Lmax, Hkv, D] (position-major) and a query stored
    [B, 1, Hq, D] are accepted through their strides."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(9)
    B, Hq, Hkv, Lmax, D = 3, 8, 2, 333, 64
    kb = torch.randn(B, Lmax, Hkv, D, generator=g).bfloat16().to(cuda_dev)
    vb = torch.randn(B, Lmax, Hkv, D, generator=g).bfloat16().to(cuda_dev)
    qb = torch.randn(B, 1, Hq, D, generator=g).bfloat16().to(cuda_dev)
    lens = [333, 100, 65]
    out = api.decode(qb[:, 0], kb.transpose(1, 2), vb.transpose(1, 2),
                     torch.tensor(lens, dtype=torch.int32, device=cuda_dev), split_len=64)
    ref = A.decode_ref(qb[:, 0].cpu(), kb.transpose(1, 2).cpu(), vb.transpose(1, 2).cpu(), lens)
    assert (out.cpu() - ref).abs().max().item() <= TOL


def test_decode_length_beyond_cache_is_reported(cuda_dev):
    """A seqlen larger than the cache is clamped on the device and reported
    through the device error word, not read out of bounds."""
    from npu_b200 import api

    q, kc, vc, _ = _case(1, 4, 1, 128, 64, [128], 3, cuda_dev)
    api.device_error(clear=True)
    out = api.decode(q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev),
                     torch.tensor([500], dtype=torch.int32, device=cuda_dev), split_len=64)
    from npu_b200 import _lib

    assert api.device_error(clear=True) == _lib.B2A_ERR_DEVICE_BAD_LEN
    ref = A.decode_ref(q, kc, vc, [128])
    assert (out.cpu() - ref).abs().max().item() <= TOL


def test_config4_all_128_sequences(cuda_dev):
    """Config 4 at its benchmarked size: 128 sequences, lengths ~ U[1024,
    32768] (seed 0 as in the bench), 32 query / 4 KV heads, D=128, 32k-key
    caches, the default split length. Every output is finite; the shortest,
    the longest and six more sequences are checked against the oracle."""
    from npu_b200 import api

    B, Hq, Hkv, D, Lmax = 128, 32, 4, 128, 32768
    lens = torch.randint(1024, Lmax + 1, (B,), generator=torch.Generator().manual_seed(0))
    g = torch.Generator(device=cuda_dev).manual_seed(44)
    q = torch.randn(B, Hq, D, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    kc = torch.randn(B, Hkv, Lmax, D, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    sl = lens.to(torch.int32).to(cuda_dev)
    out = api.decode(q, kc, vc, sl, scale=1 / math.sqrt(D), out_dtype=torch.bfloat16)
    assert api.device_error() == 0
    assert torch.isfinite(out.float()).all()
    pick = sorted({int(lens.argmin()), int(lens.argmax()), 0, 1, 37, 64, 100, 127})
    for b in pick:
        L = int(lens[b])
        ref = A.decode_ref(q[b:b + 1].cpu(), kc[b:b + 1, :, :L].cpu(), vc[b:b + 1, :, :L].cpu(), [L],
                           scale=1 / math.sqrt(D))
        err = (out[b:b + 1].float().cpu() - ref).abs().max().item()
        assert err <= TOL, (b, L, err)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("B,Hq,Hkv,D,dim", [(3, 9, 3, 64, 576), (2, 16, 2, 256, 512)])
def test_decode_proj_matches_decode_then_projection(cuda_dev, dtype, B, Hq, Hkv, D, dim):
    """b2a_decode_proj (attention, output projection and residual add in the
    combine kernel) against b2a_decode followed by x + F.linear(o, wo), and
    against the fp32 oracle; SmolLM's (9/3 heads, 64, 576) and a Qwen-like
    (16/2 heads, 256) geometry."""
    import torch.nn.functional as F

    from npu_b200 import api

    Lmax = 700
    lens = [1, 350, 700][:B]
    q, kc, vc, sl = _case(B, Hq, Hkv, Lmax, D, lens, 61, cuda_dev)
    q, kc, vc, sl = q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev), sl.to(cuda_dev)
    g = torch.Generator().manual_seed(62)
    x0 = torch.randn(B, dim, generator=g).to(dtype).to(cuda_dev)
    wo = (torch.randn(dim, Hq * D, generator=g) * 0.05).to(dtype).to(cuda_dev)
    o = api.decode(q, kc, vc, sl, out_dtype=dtype)
    want = (x0.float() + F.linear(o.reshape(B, Hq * D).float(), wo.float()))
    x = x0.clone()
    api.decode_proj(q, kc, vc, sl, wo, x)
    assert api.device_error() == 0
    scale = max(1.0, want.abs().max().item())
    # fp32: summation order only; bf16: the residual add rounded once
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert (x.float() - want).abs().max().item() <= tol * scale
    # one writer per output and a fixed summation order: reproducible
    x2 = x0.clone()
    api.decode_proj(q, kc, vc, sl, wo, x2)
    assert torch.equal(x, x2)
    ref_o = A.decode_ref(q.cpu(), kc.cpu(), vc.cpu(), lens)
    ref = x0.float().cpu() + ref_o.reshape(B, Hq * D) @ wo.float().cpu().T
    assert (x.float().cpu() - ref).abs().max().item() <= (TOL if dtype == torch.float32 else 6e-2) * scale


@pytest.mark.parametrize("gate_dtype", [torch.float32, torch.bfloat16])
def test_gated_decode_head_dim_128(cuda_dev, gate_dtype):
    """b2a_decode_gated at D=128 (the gate fused into the combine kernel) with
    a strided gate view, against the oracle times sigmoid(gate)."""
    from npu_b200 import api

    B, Hq, Hkv, D, Lmax = 3, 16, 2, 128, 900
    lens = [1, 450, 900]
    q, kc, vc, sl = _case(B, Hq, Hkv, Lmax, D, lens, 71, cuda_dev)
    q, kc, vc, sl = q.to(cuda_dev), kc.to(cuda_dev), vc.to(cuda_dev), sl.to(cuda_dev)
    gate_full = torch.randn(B, Hq, 2, D, generator=torch.Generator().manual_seed(72)).to(gate_dtype).to(cuda_dev)
    gate = gate_full[:, :, 1]
    out = api.decode(q, kc, vc, sl, gate=gate)
    assert api.device_error() == 0
    ref = A.decode_ref(q.cpu(), kc.cpu(), vc.cpu(), lens) * torch.sigmoid(gate.float().cpu())
    assert (out.cpu() - ref).abs().max().item() <= TOL
