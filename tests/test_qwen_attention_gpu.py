"""Qwen3.5/3.6 gated attention (qwen/forward.py:133-239) on the B200 path —
fused per-head Q/K RMSNorm + partial RoPE + KV append, attention with the
sigmoid gate fused into its output stores — against outputs of the
reference's own attn_forward (tests/golden/qwen_attn.npz) and against its CPU
restatement in oracle/qwen_ref.py (seeded random weights; the GGUF checkpoint
is not available offline)."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN, from_bits

from oracle import qwen_ref as R

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _block(cuda_dev, dtype=torch.float32):
    from npu_b200.qwen_attention import QwenAttnConfig, QwenGatedAttentionB200

    rc = R.QwenAttnConfig()
    layer = R.make_layer(rc, seed=5, dtype=dtype)
    cfg = QwenAttnConfig(d_model=rc.d_model, n_head=rc.n_head, n_head_kv=rc.n_head_kv, head_dim=rc.head_dim,
                         rope_dim=rc.rope_dim, rms_eps=rc.rms_eps, rope_theta=rc.rope_theta, max_pos=4096)
    blk = QwenGatedAttentionB200(layer.attn_norm, layer.wq, layer.wk, layer.wv, layer.wo, layer.q_norm,
                                 layer.k_norm, cfg, cuda_dev)
    cos, sin = R.partial_rope_tables(rc.rope_dim, 4096, rc.rope_theta, dtype)
    return rc, layer, blk, cos, sin


def test_qwen_prologue_norm_and_partial_rope(cuda_dev):
    from npu_b200 import api

    rc, layer, blk, cos, sin = _block(cuda_dev)
    g = torch.Generator().manual_seed(2)
    B, T, Hq, Hkv, D = 2, 7, rc.n_head, rc.n_head_kv, rc.head_dim
    qf = torch.randn(B, T, Hq, 2, D, generator=g)
    k = torch.randn(B, T, Hkv, D, generator=g)
    v = torch.randn(B, T, Hkv, D, generator=g)
    kc = torch.zeros(B, Hkv, 64, D, dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    qd = qf.to(cuda_dev)
    q_rot = api.rope_append(qd[:, :, :, 0], k.to(cuda_dev), v.to(cuda_dev), blk.cos, blk.sin, kc, vc,
                            start_pos=20, q_norm=blk.q_norm, k_norm=blk.k_norm, norm_eps=rc.rms_eps,
                            rope_dim=rc.rope_dim)
    assert api.device_error() == 0
    cs, sn = cos[20:20 + T], sin[20:20 + T]
    ref_q = R.partial_rope(R.rms_norm(qf[:, :, :, 0], layer.q_norm, rc.rms_eps), cs, sn, rc.rope_dim)
    ref_k = R.partial_rope(R.rms_norm(k, layer.k_norm, rc.rms_eps), cs, sn, rc.rope_dim)
    assert (q_rot.float().cpu() - ref_q.transpose(1, 2)).abs().max().item() < 2e-2
    assert (kc[:, :, 20:20 + T].float().cpu() - ref_k.transpose(1, 2)).abs().max().item() < 2e-2
    assert torch.equal(vc[:, :, 20:20 + T].cpu(), v.transpose(1, 2).to(torch.bfloat16))
    # lanes past rope_dim are only normalised
    assert (q_rot[..., rc.rope_dim:].float().cpu()
            - R.rms_norm(qf[:, :, :, 0], layer.q_norm, rc.rms_eps).transpose(1, 2)[..., rc.rope_dim:]).abs().max() < 2e-2


def test_qwen_gated_attention_prefill_then_decode(cuda_dev):
    rc, layer, blk, cos, sin = _block(cuda_dev)
    g = torch.Generator().manual_seed(4)
    B, T = 2, 300
    x = torch.randn(B, T, rc.d_model, generator=g)
    cache = blk.new_cache(batch=B, max_len=512)
    ref, ref_cache = R.attn_forward(x, layer, rc, cos, sin, None, 0, pre_proj=True)
    out = blk.attention(x.to(cuda_dev), cache)
    cache.advance()
    assert (out.cpu() - ref).abs().max().item() <= TOL
    pos = T
    for step in range(3):
        xs = torch.randn(B, 1, rc.d_model, generator=g)
        ref, ref_cache = R.attn_forward(xs, layer, rc, cos, sin, ref_cache, pos, pre_proj=True)
        out = blk.attention(xs.to(cuda_dev), cache)
        cache.advance()
        assert (out.cpu() - ref).abs().max().item() <= TOL, step
        pos += 1
    # One more step through the whole block (output projection included).
    xs = torch.randn(B, 1, rc.d_model, generator=g)
    ref_full, ref_cache = R.attn_forward(xs, layer, rc, cos, sin, ref_cache, pos)
    full = blk.forward(xs.to(cuda_dev), cache)
    cache.advance()
    pos += 1
    assert (full.cpu() - ref_full).abs().max().item() <= TOL * max(1.0, ref_full.abs().max().item())
    assert cache.lengths() == [pos, pos]
    from npu_b200 import api
    assert api.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attn_forward_drop_in_matches_reference_signature(cuda_dev, dtype):
    """npu_b200.qwen_attention.attn_forward called exactly as qwen/forward.py
    calls its own attn_forward (host tensors, the reference layer object and
    config, cos/sin tables, a tuple cache of expanded heads grown step by
    step): a 300-token prefill from position 0, then four one-token decode
    steps feeding the returned cache back in."""
    from npu_b200.qwen_attention import attn_forward

    rc = R.QwenAttnConfig()
    layer = R.make_layer(rc, seed=9, dtype=dtype)
    cos, sin = R.partial_rope_tables(rc.rope_dim, 1024, rc.rope_theta, dtype)
    g = torch.Generator().manual_seed(10)
    B, T = 2, 300
    x = torch.randn(B, T, rc.d_model, generator=g).to(dtype)
    ref, ref_cache = R.attn_forward(x, layer, rc, cos, sin, None, 0)
    out, cache = attn_forward(x, layer, rc, cos, sin, None, 0, device=cuda_dev)
    assert out.device == x.device and out.dtype == x.dtype and out.shape == ref.shape
    scale = max(1.0, ref.float().abs().max().item())
    assert (out.float() - ref.float()).abs().max().item() <= TOL * scale
    assert cache[0].shape == ref_cache[0].shape and cache[1].shape == ref_cache[1].shape
    pos = T
    for step in range(4):
        xs = torch.randn(B, 1, rc.d_model, generator=g).to(dtype)
        ref, ref_cache = R.attn_forward(xs, layer, rc, cos, sin, ref_cache, pos)
        out, cache = attn_forward(xs, layer, rc, cos, sin, cache, pos, device=cuda_dev)
        scale = max(1.0, ref.float().abs().max().item())
        assert (out.float() - ref.float()).abs().max().item() <= TOL * scale, step
        pos += 1
    assert cache[0].shape == ref_cache[0].shape == (B, pos, rc.n_head, rc.head_dim)
    for mine, theirs in zip(cache, ref_cache):
        assert mine.shape == theirs.shape
        assert (mine.float().cpu() - theirs.float()).abs().max().item() < 5e-2 * max(1.0, theirs.float().abs().max())


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_attn_forward_drop_in_matches_reference_golden(cuda_dev, tag):
    """The drop-in attn_forward against the outputs the reference's own
    qwen/forward.py attn_forward produced on the same seeded weights and
    inputs: the prefill from position 0 (300 tokens, batch 2, fp32; 40 tokens
    in bf16), then the single-token decode steps through the returned cache."""
    from npu_b200.qwen_attention import attn_forward

    g = dict(np.load(GOLDEN / "qwen_attn.npz"))
    cfg, layer, x, xs = R.golden_case(tag)
    assert R.fingerprint(*R.layer_tensors(layer)) == str(g[f"qwen_{tag}_weights_sha256"])
    assert R.fingerprint(x, *xs) == str(g[f"qwen_{tag}_inputs_sha256"])
    dtype = x.dtype
    cos, sin = R.partial_rope_tables(cfg.rope_dim, R.QWEN_GOLDEN_MAX_POS, cfg.rope_theta, dtype)

    def check(got, key):
        a = g[key]
        want = (from_bits(a) if dtype == torch.bfloat16 else torch.from_numpy(a.copy())).float()
        scale = max(1.0, want.abs().max().item())
        err = (got.float().cpu() - want).abs().max().item()
        assert err <= TOL * scale, (key, err)

    out, cache = attn_forward(x, layer, cfg, cos, sin, None, 0, device=cuda_dev)
    assert out.dtype == dtype and out.device == x.device
    check(out, f"qwen_{tag}_prefill_out")
    pos = x.shape[1]
    for i, xi in enumerate(xs):
        out, cache = attn_forward(xi, layer, cfg, cos, sin, cache, pos, device=cuda_dev)
        check(out, f"qwen_{tag}_decode{i}_out")
        pos += 1
    rows = g[f"qwen_{tag}_cache_rows"].tolist()
    for j, key in enumerate(("cache_k", "cache_v")):
        a = g[f"qwen_{tag}_{key}"]
        want = (from_bits(a) if dtype == torch.bfloat16 else torch.from_numpy(a.copy())).float()
        got = cache[j][:, rows].float().cpu()  # bf16 cache: one rounding of the reference's values
        assert (got - want).abs().max().item() <= 1e-2 * max(1.0, want.abs().max().item()), key
