"""Parity of the sm_100a prefill kernel with the fp32 oracle (max|Δ| <= 2e-2,
the north-star tolerance), through the C ABI via npu_b200.api / NpuAttention."""
import math

import numpy as np
import pytest
import torch

from conftest import from_bits
from oracle import attention as A

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rand(shape, gen, dev):
    return torch.randn(*shape, generator=gen).to(torch.bfloat16).to(dev)


def test_umma_layouts(cuda_dev):
    """One 128^3 tcgen05 MMA per operand layout: K-major B, MN-major B, and
    MN-major B with A read from tensor memory."""
    from npu_b200 import _lib

    g = torch.Generator().manual_seed(0)
    a = torch.randn(128, 128, generator=g).bfloat16()
    b = torch.randn(128, 128, generator=g).bfloat16()
    for mn in (0, 1, 2):
        c = torch.zeros(128, 128, dtype=torch.float32, device=cuda_dev)
        ad, bd = a.to(cuda_dev), b.to(cuda_dev)
        rc = _lib.load().b2a_diag_umma_gemm(ad.data_ptr(), bd.data_ptr(), c.data_ptr(), mn,
                                            torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        ref = a.float() @ (b.float() if mn else b.float().T)
        assert (c.cpu() - ref).abs().max().item() < 1e-2, f"b_mn_major={mn}"


@pytest.mark.parametrize("i", range(5))
def test_reference_selftest_grid(cuda_dev, fa_golden, i):
    """The reference's own self-test shapes (npu/fa_ref.py:148-167)."""
    from npu_b200 import api

    g = fa_golden
    q, k, v = (from_bits(g[f"selftest{i}_{n}"]).to(cuda_dev) for n in "qkv")
    sp = int(g[f"selftest{i}_meta"][3])
    out = api.prefill(q, k, v, start_pos=sp, causal=True)
    ref = g[f"selftest{i}_fa_32_32"]
    assert np.abs(out.cpu().numpy() - ref).max() <= TOL


def test_config1_gqa(cuda_dev, fa_golden):
    """Config 1: B=1, T=128, 9/3 heads, D=64, fp32 out vs the reference's
    torch fp32 attention (golden)."""
    from npu_b200 import api

    g = fa_golden
    q, k, v = (from_bits(g[f"cfg1_{n}"]).to(cuda_dev) for n in "qkv")
    out = api.prefill(q, k, v, scale=1.0 / 8)
    assert np.abs(out.cpu().numpy() - g["cfg1_dense"]).max() <= TOL


def test_chunked_prefill_golden(cuda_dev, fa_golden):
    from npu_b200 import api

    g = fa_golden
    q, k, v = (from_bits(g[f"chunk_{n}"]).to(cuda_dev) for n in "qkv")
    assert np.abs(api.prefill(q, k, v, start_pos=80).cpu().numpy() - g["chunk_fa_16_32"]).max() <= TOL
    out = api.prefill(q, k, v, causal=False).cpu().numpy()
    assert np.abs(out - g["chunk_nomask_fa_32_32"]).max() <= TOL


CASES = [
    # B, Hq, Hkv, Tq, Tk, D, start_pos, causal
    (1, 1, 1, 1, 1, 64, 0, True),
    (1, 2, 1, 17, 17, 64, 0, True),
    (2, 4, 2, 127, 127, 128, 0, True),
    (1, 4, 4, 128, 128, 128, 0, True),
    (1, 2, 1, 129, 129, 64, 0, True),
    (1, 2, 2, 255, 300, 128, 45, True),
    (2, 8, 1, 256, 256, 64, 0, True),
    (1, 8, 2, 257, 257, 128, 0, True),
    (1, 3, 1, 300, 1000, 64, 700, True),
    (2, 4, 4, 200, 333, 128, 0, False),
    (1, 2, 1, 1000, 1000, 128, 0, True),
    (1, 32, 4, 512, 512, 128, 0, True),
    # head_dim 256 (Qwen3.6 geometry, one-tile kernel with 64-key blocks)
    (1, 2, 1, 1, 1, 256, 0, True),
    (1, 4, 2, 65, 65, 256, 0, True),
    (2, 16, 2, 129, 129, 256, 0, True),
    (1, 8, 1, 200, 700, 256, 500, True),
    (1, 2, 2, 300, 333, 256, 0, False),
    (1, 16, 2, 1000, 1000, 256, 0, True),
]


@pytest.mark.parametrize("B,Hq,Hkv,Tq,Tk,D,sp,causal", CASES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_prefill_matches_oracle(cuda_dev, B, Hq, Hkv, Tq, Tk, D, sp, causal, out_dtype):
    from npu_b200 import api

    g = torch.Generator().manual_seed(B * 1000 + Tq * 7 + Tk + D)
    q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
    out = api.prefill(q, k, v, start_pos=sp, causal=causal, out_dtype=out_dtype)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu(), start_pos=sp, causal=causal)
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= TOL, err
    assert torch.isfinite(out).all()


def test_strided_bthd_inputs(cuda_dev):
    """q/k/v as [B, T, H, D] buffers viewed as [B, H, T, D] (the layout the
    projections produce before transpose(1, 2), smollm.py:195-197)."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(5)
    B, T, Hq, Hkv, D = 2, 300, 8, 2, 64
    qb = _rand((B, T, Hq, D), g, cuda_dev)
    kb = _rand((B, T, Hkv, D), g, cuda_dev)
    vb = _rand((B, T, Hkv, D), g, cuda_dev)
    q, k, v = qb.transpose(1, 2), kb.transpose(1, 2), vb.transpose(1, 2)
    out = api.prefill(q, k, v)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu())
    assert (out.cpu() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("D", [64, 128])
def test_bf16_output_into_strided_bthd_buffer(cuda_dev, D):
    """bf16 output written into a [B, T, H, D] buffer viewed as [B, H, T, D]
    (the layout the output projection reads), with a ragged T: the rows past T
    of the last query block must not be written, the rest of the buffer stays
    untouched."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(15 + D)
    B, T, Hq, Hkv = 2, 300, 8, 2
    q, k, v = _rand((B, Hq, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev)
    buf = torch.full((B, T + 5, Hq, D), 7.0, dtype=torch.bfloat16, device=cuda_dev)
    out = buf[:, :T].transpose(1, 2)
    api.prefill(q, k, v, out_dtype=torch.bfloat16, out=out)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu())
    assert (out.float().cpu() - ref).abs().max().item() <= TOL
    assert torch.all(buf[:, T:] == 7.0)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T", [300, 1100])
def test_output_16_byte_aligned_only(cuda_dev, out_dtype, T):
    """An output 16 bytes past a 32-byte boundary takes the 16-byte store path
    (the 32-byte vector stores need 32-byte alignment); one-tile (T=300) and
    two-tile (T=1100) work items. The words around the output stay as they
    were."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(77 + T)
    B, Hq, Hkv, D = 1, 4, 2, 128
    q, k, v = _rand((B, Hq, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev)
    n = B * Hq * T * D
    pad = 16 // torch.tensor([], dtype=out_dtype).element_size()
    flat = torch.full((n + 2 * pad,), 3.0, dtype=out_dtype, device=cuda_dev)
    assert flat.data_ptr() % 32 == 0
    out = flat[pad:pad + n].view(B, Hq, T, D)
    api.prefill(q, k, v, out_dtype=out_dtype, out=out)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu())
    assert (out.float().cpu() - ref).abs().max().item() <= TOL
    assert torch.all(flat[:pad] == 3.0) and torch.all(flat[pad + n:] == 3.0)


def test_fully_masked_rows_and_empty_keys(cuda_dev):
    from npu_b200 import api

    g = torch.Generator().manual_seed(6)
    q = _rand((1, 2, 64, 64), g, cuda_dev)
    k = _rand((1, 2, 64, 64), g, cuda_dev)
    out = api.prefill(q, k, k, start_pos=-10)
    ref = A.dense_attention(q.cpu(), k.cpu(), k.cpu(), start_pos=-10)
    assert torch.all(out[:, :, :10] == 0)
    assert (out.cpu() - ref).abs().max().item() <= TOL
    out = api.prefill(q, k, k, start_pos=-1_000_000)
    assert torch.all(out == 0)
    empty = k[:, :, :0]
    out = api.prefill(q, empty, empty)
    assert torch.all(out == 0)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_running_max_jumps(cuda_dev, D):
    """Scores that climb in steps above the lazy-rescale threshold (2^8 in
    the exp2 domain) at random keys, so a row's running max moves inside the
    first and inside the second 64-key half of key blocks: exercises the
    rescale of P already written for the block and of O."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(11 + D)
    B, Hq, Hkv, T = 1, 2, 1, 1024
    sl2 = math.log2(math.e) / math.sqrt(D)
    spikes = (torch.rand(T, generator=g) < 1 / 40).float()
    x = 12.0 * torch.cumsum(spikes, 0) + torch.randn(T, generator=g)  # target S * scale * log2(e)
    q = torch.ones(B, Hq, T, D).to(torch.bfloat16).to(cuda_dev)
    k = (x / (D * sl2)).view(1, 1, T, 1).expand(B, Hkv, T, D).to(torch.bfloat16).to(cuda_dev)
    v = _rand((B, Hkv, T, D), g, cuda_dev)
    out, lse = api.prefill(q, k, v, return_lse=True)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu())
    assert (out.cpu() - ref).abs().max().item() <= TOL
    s = (q[0].float().cpu() @ A.expand_kv(k.cpu().float(), Hq // Hkv)[0].transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(A.causal_mask(T, T, 0), float("-inf"))
    assert (lse[0].cpu() - torch.logsumexp(s, dim=-1)).abs().max().item() < 1e-3 * s.abs().max().item()


def test_per_batch_start_positions_and_lse(cuda_dev):
    from npu_b200 import api

    g = torch.Generator().manual_seed(7)
    B, Hq, Hkv, Tq, Tk, D = 3, 4, 2, 100, 400, 128
    q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
    sps = [0, 150, 300]
    out, lse = api.prefill(q, k, v, start_pos_per_batch=torch.tensor(sps, dtype=torch.int32, device=cuda_dev),
                           return_lse=True)
    for b, sp in enumerate(sps):
        ref = A.dense_attention(q[b:b + 1].cpu(), k[b:b + 1].cpu(), v[b:b + 1].cpu(), start_pos=sp)
        assert (out[b:b + 1].cpu() - ref).abs().max().item() <= TOL
        s = (q[b].float().cpu() @ A.expand_kv(k[b:b + 1].cpu().float(), 2)[0].transpose(-1, -2)) / math.sqrt(D)
        s = s.masked_fill(A.causal_mask(Tq, Tk, sp), float("-inf"))
        ref_lse = torch.logsumexp(s, dim=-1)
        assert (lse[b].cpu() - ref_lse).abs().max().item() < 1e-3


def test_npu_attention_run_batch_contract(cuda_dev):
    """run_batch as smollm.py:157-163 drives it: host tensors in, per-block
    start rows, dummy blocks at -1e6 (npu/fa.py:236) -> zeros, bf16 out."""
    from npu_b200 import NpuAttention

    attn = NpuAttention(D=64)
    g = torch.Generator().manual_seed(8)
    N, BR, TK, D = 6, attn.BR, 256, 64
    Q = torch.randn(N, BR, D, generator=g).bfloat16()
    K = torch.randn(N, TK, D, generator=g).bfloat16()
    V = torch.randn(N, TK, D, generator=g).bfloat16()
    rows = [0, 128, 0, 128, 37, -1_000_000]
    out = attn.run_batch(Q, K, V, rows, causal=True)
    assert out.device.type == "cpu" and out.dtype == torch.bfloat16 and out.shape == (N, BR, D)
    ref = A.run_batch_ref(Q, K, V, rows)
    assert (out.float() - ref).abs().max().item() <= TOL
    assert torch.all(out[5] == 0)
    one = attn.run_one(Q[2], K[2], V[2], start_row=0, causal=False)
    ref1 = A.dense_attention(Q[2][None, None], K[2][None, None], V[2][None, None], causal=False)[0, 0]
    assert (one.float() - ref1).abs().max().item() <= TOL
    with pytest.raises(AssertionError):
        attn.run_batch(Q, K[:, :100], V[:, :100], rows)  # TK % BC != 0


@pytest.mark.parametrize("T", [2048, 8192])
def test_config3_sampled_rows(cuda_dev, T):
    """Config 3 geometry (B=64 trimmed to 4, Hq=32, Hkv=4, D=128) at full T:
    first, last, tile-boundary and diagonal rows against the oracle."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(T)
    B, Hq, Hkv, D = 4, 32, 4, 128
    q, k, v = _rand((B, Hq, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev), _rand((B, Hkv, T, D), g, cuda_dev)
    out = api.prefill(q, k, v, scale=1 / math.sqrt(128))
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    rows = [0, 1, 127, 128, 255, 256, T // 2, T - 129, T - 2, T - 1]
    for b, h in [(0, 0), (1, 7), (3, 31), (2, 12)]:
        ref = A.prefill_rows_ref(qc, kc, vc, b, h, rows)
        assert (out[b, h, rows].cpu() - ref).abs().max().item() <= TOL
    assert torch.isfinite(out).all()


def test_no_device_error_left(cuda_dev):
    from npu_b200 import api

    assert api.device_error(clear=True) == 0


def test_d256_per_batch_starts_ragged_pairs_and_lse(cuda_dev):
    """Head dim 256: per-batch start positions including a negative one
    (leading rows fully masked), query lengths that end inside a 128-row
    tile (300) or below one tile (100), and the LSE."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(21)
    for Tq in (300, 100):
        B, Hq, Hkv, Tk, D = 3, 4, 2, 520, 256
        q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
        sps = [-40, 0, Tk - Tq]
        out, lse = api.prefill(q, k, v, start_pos_per_batch=torch.tensor(sps, dtype=torch.int32, device=cuda_dev),
                               return_lse=True)
        for b, sp in enumerate(sps):
            ref = A.dense_attention(q[b:b + 1].cpu(), k[b:b + 1].cpu(), v[b:b + 1].cpu(), start_pos=sp)
            assert (out[b:b + 1].cpu() - ref).abs().max().item() <= TOL, (Tq, b)
            s = (q[b].float().cpu() @ A.expand_kv(k[b:b + 1].cpu().float(), 2)[0].transpose(-1, -2)) / math.sqrt(D)
            s = s.masked_fill(A.causal_mask(Tq, Tk, sp), float("-inf"))
            ref_lse = torch.logsumexp(s, dim=-1)
            got = lse[b].cpu()
            live = torch.isfinite(ref_lse)
            assert torch.all(torch.isneginf(got[~live]))
            assert (got[live] - ref_lse[live]).abs().max().item() < 1e-3, (Tq, b)
        assert torch.all(out[0, :, :40] == 0)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_two_tile_items_without_keys_and_chunked_batches(cuda_dev, out_dtype):
    """Two-tile CTAs (Tq > 1024) over 2 x 48 heads x 5 query blocks with
    per-batch start positions: query blocks with no visible key at all
    (batch 0, start -500: the first block), blocks where only the second
    128-row tile sees keys (the second block), a chunked batch (start 200,
    Tq < Tk), the LSE, and the same geometry without the causal mask; all
    compared in full against the oracle."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(31)
    B, Hq, Hkv, Tq, Tk, D = 2, 48, 8, 1100, 1300, 128
    q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
    sps = [-500, 200]
    out, lse = api.prefill(q, k, v, start_pos_per_batch=torch.tensor(sps, dtype=torch.int32, device=cuda_dev),
                           out_dtype=out_dtype, return_lse=True)
    assert api.device_error() == 0
    for b, sp in enumerate(sps):
        ref = A.dense_attention(q[b:b + 1].cpu(), k[b:b + 1].cpu(), v[b:b + 1].cpu(), start_pos=sp)
        assert (out[b:b + 1].float().cpu() - ref).abs().max().item() <= TOL, b
        s = (q[b].float().cpu() @ A.expand_kv(k[b:b + 1].cpu().float(), Hq // Hkv)[0].transpose(-1, -2)) / math.sqrt(D)
        s = s.masked_fill(A.causal_mask(Tq, Tk, sp), float("-inf"))
        ref_lse = torch.logsumexp(s, dim=-1)
        live = torch.isfinite(ref_lse)
        assert torch.all(torch.isneginf(lse[b].cpu()[~live]))
        assert (lse[b].cpu()[live] - ref_lse[live]).abs().max().item() < 1e-3, b
    assert torch.all(out[0, :, :500] == 0)
    # Non-causal, same geometry: every item has all key blocks.
    out2 = api.prefill(q, k, v, causal=False, out_dtype=out_dtype)
    ref2 = A.dense_attention(q.cpu(), k.cpu(), v.cpu(), causal=False)
    assert (out2.float().cpu() - ref2).abs().max().item() <= TOL


def test_config5_geometry_sampled_rows(cuda_dev):
    """Config 5 head geometry (16 query / 2 KV heads, D=256, scale 1/16) on a
    16k-token causal prefill: sampled rows against the oracle."""
    from npu_b200 import api

    T = 16384
    g = torch.Generator().manual_seed(5)
    q, k, v = _rand((1, 16, T, 256), g, cuda_dev), _rand((1, 2, T, 256), g, cuda_dev), _rand((1, 2, T, 256), g, cuda_dev)
    out = api.prefill(q, k, v, scale=1 / 16)
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    rows = [0, 63, 64, 127, 128, 4097, T // 2, T - 65, T - 1]
    for h in (0, 7, 8, 15):
        ref = A.prefill_rows_ref(qc, kc, vc, 0, h, rows, scale=1 / 16)
        assert (out[0, h, rows].cpu() - ref).abs().max().item() <= TOL
    assert torch.isfinite(out).all()


def test_config5_full_length_sampled_rows(cuda_dev):
    """Config 5 at its benchmarked length, T=131072 (16 query / 2 KV heads,
    D=256, scale 1/16, one sequence): the first row, the middle, the last row
    and both sides of each of the last four 128-row tile boundaries, i.e. the
    end of a 1024-block causal key walk, against the oracle."""
    from npu_b200 import api

    T = 131072
    g = torch.Generator(device=cuda_dev).manual_seed(55)
    q = torch.randn(1, 16, T, 256, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    k = torch.randn(1, 2, T, 256, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    v = torch.randn(1, 2, T, 256, generator=g, device=cuda_dev, dtype=torch.bfloat16)
    out = api.prefill(q, k, v, scale=1 / 16, out_dtype=torch.bfloat16)
    assert api.device_error() == 0
    rows = [0, 1, 65535, 65536]
    for j in range(1, 5):
        rows += [T - 128 * j - 1, T - 128 * j]
    rows += [T - 1]
    rows = sorted(set(rows))
    kc, vc = k.cpu(), v.cpu()
    qr = q[:, :, rows].cpu()  # only the sampled rows leave the device
    for h in (0, 7, 8, 15):
        ref = A.prefill_rows_ref(qr, kc, vc, 0, h, range(len(rows)), scale=1 / 16, positions=rows)
        err = (out[0, h, rows].float().cpu() - ref).abs().max().item()
        assert err <= TOL, (h, err)
    assert not torch.isnan(out).any()


@pytest.mark.parametrize("Tq", [600, 1300])
@pytest.mark.parametrize("Hq,Hkv", [(8, 2), (6, 2), (16, 16)])
def test_two_tile_items_head_pairs_and_row_pairs(cuda_dev, Hq, Hkv, Tq):
    """Work items by query length and GQA group: with an even group (8/2)
    queries of 513-3072 rows run as two query heads of one KV head over the
    same 128 rows (Tq 600 and 1300); odd groups (6/2 with group 3; 16/16 with
    group 1) run one-tile CTAs up to 1024 rows (Tq 600) and two 128-row
    blocks of one head beyond (Tq 1300). Ragged query length, a chunked start
    and the LSE, all rows against the oracle."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(40 + Hq + Tq)
    B, Tk, D, sp = 2, Tq + 200, 128, 200
    q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
    out, lse = api.prefill(q, k, v, start_pos=sp, return_lse=True)
    assert api.device_error() == 0
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu(), start_pos=sp)
    assert (out.cpu() - ref).abs().max().item() <= TOL
    s = (q.float().cpu() @ A.expand_kv(k.cpu().float(), Hq // Hkv).transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(A.causal_mask(Tq, Tk, sp), float("-inf"))
    assert (lse.cpu() - torch.logsumexp(s, dim=-1)).abs().max().item() < 1e-3


@pytest.mark.parametrize("Tq,out_dtype,gate_dtype", [(300, torch.bfloat16, torch.bfloat16),
                                                     (1300, torch.float32, torch.float32),
                                                     (2100, torch.bfloat16, torch.float32)])
def test_gated_prefill_head_dim_128(cuda_dev, Tq, out_dtype, gate_dtype):
    """b2a_prefill_gated on the D <= 128 kernel (one-tile CTAs at Tq=300,
    head-pair items at 1300 and 2100): output =
    attention * sigmoid(gate), the gate a strided view with a head stride of
    2 D as in Qwen's [q_h | gate_h] projection."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(Tq)
    B, Hq, Hkv, D = 2, 8, 2, 128
    Tk = Tq + 64
    q, k, v = _rand((B, Hq, Tq, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev), _rand((B, Hkv, Tk, D), g, cuda_dev)
    gate_full = torch.randn(B, Tq, Hq, 2, D, generator=g).to(gate_dtype).to(cuda_dev)
    gate = gate_full[:, :, :, 1].transpose(1, 2)  # [B, Hq, Tq, D], strided
    out = api.prefill(q, k, v, start_pos=64, gate=gate, out_dtype=out_dtype)
    assert api.device_error() == 0
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu(), start_pos=64) * torch.sigmoid(gate.float().cpu())
    assert (out.float().cpu() - ref).abs().max().item() <= TOL
