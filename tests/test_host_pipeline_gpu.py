"""b2a_prefill_host: host-memory Q/K/V in, host O out, with chunked uploads,
kernels and downloads overlapping on three streams. Every chunk runs the
same kernel on the same rows as one whole-problem launch, so the result must
equal api.prefill's bit for bit; the oracle check pins the values."""
import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu


def _host(shape, g, pin=True):
    t = torch.randn(*shape, generator=g).bfloat16()
    return t.pin_memory() if pin else t


def _device_ref(q, k, v, dev, **kw):
    from npu_b200 import api

    o = api.prefill(q.to(dev), k.to(dev), v.to(dev), **kw)
    torch.cuda.synchronize(dev)
    return o.cpu()


@pytest.mark.parametrize("B,Hq,Hkv,T,D,n_chunks", [
    (6, 8, 2, 300, 128, 4),    # whole-batch chunks, ragged last chunk (2+2+2 -> 3 chunks of 2)
    (5, 8, 2, 257, 64, 3),     # 10 units / 3 -> 2 batches per chunk, last chunk 1 batch
    (1, 16, 4, 640, 128, 0),   # one batch: chunks are single KV heads
    (2, 8, 8, 129, 256, 5),    # D = 256, MHA, 16 units in chunks of 4 (one head group)
])
def test_prefill_host_matches_device_prefill(cuda_dev, B, Hq, Hkv, T, D, n_chunks):
    from npu_b200 import api

    g = torch.Generator().manual_seed(B * 1000 + T)
    q, k, v = _host((B, Hq, T, D), g), _host((B, Hkv, T, D), g), _host((B, Hkv, T, D), g)
    o = api.prefill_host(q, k, v, n_chunks=n_chunks, device=cuda_dev)
    assert not o.is_cuda and o.dtype == torch.bfloat16 and o.is_pinned()
    ref = _device_ref(q, k, v, cuda_dev, out_dtype=torch.bfloat16)
    assert torch.equal(o, ref)
    if B * Hq * T <= 6 * 8 * 300:
        err = (o.float() - A.dense_attention(q, k, v)).abs().max().item()
        assert err <= 2e-2
    assert api.device_error() == 0


def test_prefill_host_per_batch_start_positions_fp32(cuda_dev):
    """Chunked prefill (Tq < Tk) with a start row per batch, the run_batch
    case of smollm.py:129-166; whole-batch chunks read the positions from
    the workspace copy, head chunks from the host array."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(11)
    B, Hq, Hkv, Tq, Tk, D = 4, 8, 2, 96, 320, 128
    q, k, v = _host((B, Hq, Tq, D), g), _host((B, Hkv, Tk, D), g), _host((B, Hkv, Tk, D), g)
    starts = [224, 0, 100, 17]
    sp_dev = torch.tensor(starts, dtype=torch.int32, device=cuda_dev)
    ref = _device_ref(q, k, v, cuda_dev, start_pos_per_batch=sp_dev, out_dtype=torch.float32)
    for n_chunks in (2, 8):  # 2: whole batches; 8 units -> 1 KV head per chunk
        o = api.prefill_host(q, k, v, start_pos_per_batch=starts, out_dtype=torch.float32, n_chunks=n_chunks,
                             device=cuda_dev)
        assert o.dtype == torch.float32
        assert torch.equal(o, ref), n_chunks
    for b, sp in enumerate(starts):
        want = A.dense_attention(q[b:b + 1], k[b:b + 1], v[b:b + 1], start_pos=sp)
        assert (o[b:b + 1] - want).abs().max().item() <= 2e-2


def test_prefill_host_pageable_and_async(cuda_dev):
    """Pageable inputs give the same result; with sync=False the output is
    complete once the stream is synchronised, and a reused caller workspace
    and output buffer work across calls."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, T, D = 3, 4, 1, 200, 64
    q, k, v = _host((B, Hq, T, D), g, pin=False), _host((B, Hkv, T, D), g, pin=False), \
        _host((B, Hkv, T, D), g, pin=False)
    ref = _device_ref(q, k, v, cuda_dev, out_dtype=torch.bfloat16)
    assert torch.equal(api.prefill_host(q, k, v, n_chunks=3, device=cuda_dev), ref)
    ws = torch.empty(api.prefill_host_workspace_bytes(B, Hq, Hkv, T, T, D, n_chunks=3), dtype=torch.uint8,
                     device=cuda_dev)
    out = torch.empty((B, Hq, T, D), dtype=torch.bfloat16).pin_memory()
    qp, kp, vp = q.pin_memory(), k.pin_memory(), v.pin_memory()
    for _ in range(3):
        out.zero_()
        api.prefill_host(qp, kp, vp, out=out, n_chunks=3, device=cuda_dev, workspace=ws, sync=False)
        torch.cuda.current_stream(cuda_dev).synchronize()
        assert torch.equal(out, ref)


def test_prefill_host_no_keys_and_errors(cuda_dev):
    from npu_b200 import _lib, api

    g = torch.Generator().manual_seed(6)
    q = _host((2, 4, 33, 128), g)
    e = torch.empty(2, 2, 0, 128, dtype=torch.bfloat16)
    o = api.prefill_host(q, e, e, device=cuda_dev)
    assert torch.count_nonzero(o) == 0
    with pytest.raises(ValueError):
        api.prefill_host(q.to(cuda_dev), e, e)
    small = torch.empty(16, dtype=torch.uint8, device=cuda_dev)
    with pytest.raises(ValueError):
        api.prefill_host(q, e, e, device=cuda_dev, workspace=small)
    # The library itself rejects a short workspace without queueing anything.
    lib = _lib.load()
    rc = lib.b2a_prefill_host(q.data_ptr(), None, None, o.data_ptr(), 2, 4, 2, 33, 0, 128, 0, None, 0.1, 1, 0,
                              0, small.data_ptr(), 16, torch.cuda.current_stream(cuda_dev).cuda_stream)
    assert rc == _lib.B2A_ERR_WORKSPACE


def test_run_batch_host_inputs_go_through_the_host_pipeline(cuda_dev):
    """NpuAttention.run_batch with host stacks (the reference's call) returns
    host results equal to the device path and within tolerance of the oracle."""
    from npu_b200.fa import NpuAttention

    g = torch.Generator().manual_seed(9)
    N, BR, TK, D = 12, 128, 256, 64
    Q = torch.randn(N, BR, D, generator=g)
    K = torch.randn(N, TK, D, generator=g)
    V = torch.randn(N, TK, D, generator=g)
    rows = [128 * (n % 2) for n in range(N)]
    attn = NpuAttention(BR=BR, BC=32, D=D, device=cuda_dev)
    out = attn.run_batch(Q, K, V, rows, causal=True)
    assert not out.is_cuda and out.shape == (N, BR, D)
    dev_out = attn.run_batch(Q.to(cuda_dev), K.to(cuda_dev), V.to(cuda_dev), rows, causal=True)
    assert torch.equal(out, dev_out.cpu())
    ref = A.run_batch_ref(Q.bfloat16().float(), K.bfloat16().float(), V.bfloat16().float(), rows)
    assert (out.float() - ref).abs().max().item() <= 2e-2
