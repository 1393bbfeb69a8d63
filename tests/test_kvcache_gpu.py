"""Fused RoPE + in-place KV-cache append (b2a_rope_append) and the SmolLM
forward that runs on it (npu_b200.smollm_b200), against the reference's
per-step apply_rope + torch.cat path (smollm.py:186-208) restated in
oracle/smollm_ref.py."""
import pytest
import torch

from oracle.smollm_ref import Config, SmolLM, make_state_dict, rope, rope_tables

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_append_bit_exact(cuda_dev, D, dtype):
    from npu_b200 import api

    g = torch.Generator().manual_seed(D)
    B, T, Hq, Hkv, Lmax, max_pos = 3, 5, 6, 2, 40, 64
    qkv = torch.randn(B, T, (Hq + 2 * Hkv) * D, generator=g).to(dtype)  # one fused projection output
    q = qkv[..., :Hq * D].view(B, T, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hkv) * D].view(B, T, Hkv, D)
    v = qkv[..., (Hq + Hkv) * D:].view(B, T, Hkv, D)
    cos, sin = rope_tables(D, max_pos, 10000.0, dtype, "cpu")
    starts = [0, 7, 35]
    kc = torch.zeros(B, Hkv, Lmax, D, dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    seq = torch.full((B,), -1, dtype=torch.int32, device=cuda_dev)
    spb = torch.tensor(starts, dtype=torch.int32, device=cuda_dev)
    qd = qkv.to(cuda_dev)
    q_out = api.rope_append(qd[..., :Hq * D].view(B, T, Hq, D), qd[..., Hq * D:(Hq + Hkv) * D].view(B, T, Hkv, D),
                            qd[..., (Hq + Hkv) * D:].view(B, T, Hkv, D), cos.to(cuda_dev), sin.to(cuda_dev),
                            kc, vc, start_pos_per_batch=spb, seqlens_out=seq)
    assert api.device_error() == 0
    assert seq.tolist() == [s + T for s in starts]
    kc, vc, q_out = kc.cpu(), vc.cpu(), q_out.cpu()
    for b, s in enumerate(starts):
        cs, sn = cos[s:s + T], sin[s:s + T]
        ref_q = rope(q[b].transpose(0, 1), cs, sn).to(torch.bfloat16)     # [Hq, T, D]
        ref_k = rope(k[b].transpose(0, 1), cs, sn).to(torch.bfloat16)
        assert torch.equal(q_out[b], ref_q)
        assert torch.equal(kc[b, :, s:s + T], ref_k)
        assert torch.equal(vc[b, :, s:s + T], v[b].transpose(0, 1).to(torch.bfloat16))
        untouched = torch.ones(Lmax, dtype=torch.bool)
        untouched[s:s + T] = False
        assert torch.all(kc[b, :, untouched] == 0) and torch.all(vc[b, :, untouched] == 0)


def test_rope_append_position_checks(cuda_dev):
    from npu_b200 import api, _lib

    B, T, H, D, Lmax = 2, 4, 2, 64, 16
    x = torch.randn(B, T, H, D, device=cuda_dev)
    cos, sin = rope_tables(D, 32, 10000.0, torch.float32, cuda_dev)
    kc = torch.zeros(B, H, Lmax, D, dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    with pytest.raises(_lib.B2AError):
        api.rope_append(x, x, x, cos, sin, kc, vc, start_pos=Lmax - T + 1)  # host-checked
    api.device_error()
    spb = torch.tensor([0, Lmax - T + 1], dtype=torch.int32, device=cuda_dev)  # device-checked
    api.rope_append(x, x, x, cos, sin, kc, vc, start_pos_per_batch=spb)
    assert api.device_error() == _lib.B2A_ERR_DEVICE_BAD_LEN
    # Only the row past the end (position 16) was dropped; the others landed.
    assert torch.all(kc[1, :, :Lmax - T + 1].float() == 0)
    assert torch.all(kc[1, :, Lmax - T + 1:].float().abs().sum(-1) > 0)
    assert torch.all(kc[0, :, :T].float().abs().sum(-1) > 0)


@pytest.fixture(scope="module")
def ref_model():
    return SmolLM(make_state_dict(Config(), seed=0), Config())


def test_smollm_prefill_then_decode_on_device_cache(cuda_dev, ref_model):
    """Prefill 96 tokens, then 6 single-token steps, each teacher-forced with
    the reference's greedy token; top-1 and logits against the reference's
    CPU path with its torch.cat cache."""
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig

    model = SmolLMB200(make_state_dict(Config(), seed=0), SmolLMConfig(), cuda_dev)
    ids = torch.randint(0, Config().vocab, (2, 96), generator=torch.Generator().manual_seed(3))
    ref_logits, ref_cache = ref_model.forward(ids)
    cache = model.new_cache(batch=2, max_len=512)
    logits = model.forward(ids.to(cuda_dev), cache).float().cpu()
    pos = 96
    for step in range(7):
        last, ref_last = logits[:, -1], ref_logits[:, -1]
        assert torch.equal(last.argmax(-1), ref_last.argmax(-1)), step
        assert (last - ref_last).abs().max().item() < 0.25, step
        nxt = ref_last.argmax(-1, keepdim=True)
        if step == 6:
            break
        ref_logits, ref_cache = ref_model.forward(nxt, cache=ref_cache, start_pos=pos)
        logits = model.forward(nxt.to(cuda_dev), cache).float().cpu()
        pos += 1
    assert cache.lengths() == [pos, pos]
    from npu_b200 import api
    assert api.device_error() == 0


def test_smollm_decode_step_as_cuda_graph(cuda_dev):
    """A whole single-token step (30 layers, ~360 launches) captured once and
    replayed: same logits as the eager step on an identical cache."""
    from npu_b200 import api
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig

    model = SmolLMB200(make_state_dict(Config(), seed=0), SmolLMConfig(), cuda_dev)
    ids = torch.randint(0, Config().vocab, (2, 40), generator=torch.Generator().manual_seed(9)).to(cuda_dev)
    eager_cache, graph_cache = model.new_cache(2, 128), model.new_cache(2, 128)
    model.forward(ids, eager_cache)
    model.forward(ids, graph_cache)
    step = model.capture_decode(graph_cache)
    assert graph_cache.lengths() == [40, 40]
    tok = ids[:, -1:]
    for _ in range(5):
        ref = model.forward(tok, eager_cache)
        got = step(tok)
        assert torch.allclose(got, ref, atol=1e-4, rtol=0)
        tok = ref[:, -1].argmax(-1, keepdim=True)
    assert graph_cache.lengths() == eager_cache.lengths() == [45, 45]
    assert api.device_error() == 0


def test_smollm_prefill_step_as_cuda_graph(cuda_dev):
    """A whole 64-token prefill step (30 layers) captured once and replayed
    twice on a cache: each replay appends at the cache's positions like the
    eager forward and gives the same logits."""
    from npu_b200 import api
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig

    model = SmolLMB200(make_state_dict(Config(), seed=0), SmolLMConfig(), cuda_dev)
    g = torch.Generator().manual_seed(10)
    ids = [torch.randint(0, Config().vocab, (2, 64), generator=g).to(cuda_dev) for _ in range(2)]
    eager_cache, graph_cache = model.new_cache(2, 256), model.new_cache(2, 256)
    step = model.capture_prefill(graph_cache, 64)
    assert graph_cache.lengths() == [0, 0]
    for chunk in ids:
        ref = model.forward(chunk, eager_cache)
        got = step(chunk)
        assert torch.allclose(got, ref, atol=1e-4, rtol=0)
    assert graph_cache.lengths() == eager_cache.lengths() == [128, 128]
    assert api.device_error() == 0


def test_profiler_times_the_forward_ops_on_the_device(cuda_dev):
    """With the profiler on, a SmolLM forward on the B200 path records device
    time (CUDA events) for each op name of the reference's profile() blocks
    (smollm.py:179-251), 30 calls each, and the logits do not change."""
    from npu_b200.profiler import PROF
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig

    model = SmolLMB200(make_state_dict(Config(), seed=0), SmolLMConfig(), cuda_dev)
    ids = torch.randint(0, Config().vocab, (1, 64), generator=torch.Generator().manual_seed(3)).to(cuda_dev)
    ref = model.forward(ids, model.new_cache(1, 128))
    PROF.reset()
    PROF.enable()
    try:
        got = model.forward(ids, model.new_cache(1, 128))
        st = PROF.stats()
    finally:
        PROF.disable()
        PROF.reset()
    assert torch.equal(got, ref)
    for name in ("rms1", "qkv", "rope", "attn", "wo", "rms2", "gate_up", "w_down"):
        assert st[name]["calls"] == 30, name
        assert st[name]["device_ms"] is not None and st[name]["device_ms"] > 0, name


def test_smollm_decode_with_fused_output_projection(cuda_dev):
    """Single-token steps with the output projection and residual add fused
    into the decode combine kernel (b2a_decode_proj, the default) give the
    logits of the unfused path (b2a_decode, then the wo GEMM) over a prefill
    and 6 decode steps, and the same greedy tokens."""
    from npu_b200 import api
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig

    sd = make_state_dict(Config(), seed=0)
    fused = SmolLMB200(sd, SmolLMConfig(), cuda_dev)
    plain = SmolLMB200(sd, SmolLMConfig(), cuda_dev, fuse_wo=False)
    assert fused.fuse_wo and not plain.fuse_wo
    ids = torch.randint(0, Config().vocab, (2, 50), generator=torch.Generator().manual_seed(12)).to(cuda_dev)
    cf, cp = fused.new_cache(2, 128), plain.new_cache(2, 128)
    lf, lp = fused.forward(ids, cf), plain.forward(ids, cp)
    assert torch.equal(lf, lp)  # prefill takes the same path in both
    tf = tp = lf[:, -1:].argmax(-1)
    for _ in range(6):
        lf, lp = fused.forward(tf, cf), plain.forward(tp, cp)
        assert (lf - lp).abs().max().item() < 1e-3
        tf, tp = lf[:, -1:].argmax(-1), lp[:, -1:].argmax(-1)
        assert torch.equal(tf, tp)
    assert api.device_error() == 0
