"""The CPU oracle against the golden vectors the reference itself produced
(tests/golden/make_golden.py ran npu/fa_ref.py and smollm.py)."""
import math

import numpy as np
import pytest
import torch

from conftest import from_bits
from oracle import attention as A


@pytest.mark.parametrize("i", range(5))
def test_selftest_grid_matches_reference(fa_golden, i):
    g = fa_golden
    q, k, v = (from_bits(g[f"selftest{i}_{n}"]) for n in "qkv")
    tq, tk, d, sp = (int(x) for x in g[f"selftest{i}_meta"])
    dense = A.dense_attention(q, k, v, start_pos=sp)
    assert np.abs(dense.numpy() - g[f"selftest{i}_dense"]).max() < 1e-5
    for Br, Bc in [(8, 16), (16, 32), (32, 32)]:
        fa = A.flash_attention_ref(q, k, v, Br=Br, Bc=Bc, causal=True, start_pos=sp)
        assert np.abs(fa.numpy() - g[f"selftest{i}_fa_{Br}_{Bc}"]).max() < 1e-5


def test_config1_gqa_matches_reference(fa_golden):
    g = fa_golden
    q, k, v = (from_bits(g[f"cfg1_{n}"]) for n in "qkv")
    dense = A.dense_attention(q, k, v)  # native GQA 9/3, expanded inside
    assert np.abs(dense.numpy() - g["cfg1_dense"]).max() < 1e-5
    fa = A.flash_attention_ref(q, A.expand_kv(k, 3), A.expand_kv(v, 3), Br=32, Bc=32)
    assert np.abs(fa.numpy() - g["cfg1_fa_32_32"]).max() < 1e-5


def test_chunked_and_unmasked_match_reference(fa_golden):
    g = fa_golden
    q, k, v = (from_bits(g[f"chunk_{n}"]) for n in "qkv")
    assert np.abs(A.dense_attention(q, k, v, start_pos=80).numpy() - g["chunk_fa_16_32"]).max() < 1e-5
    assert np.abs(A.dense_attention(q, k, v, causal=False).numpy() - g["chunk_nomask_fa_32_32"]).max() < 1e-5


def test_fully_masked_rows_are_zero():
    torch.manual_seed(3)
    q = torch.randn(1, 2, 8, 64).bfloat16()
    k = torch.randn(1, 2, 16, 64).bfloat16()
    v = torch.randn(1, 2, 16, 64).bfloat16()
    out = A.dense_attention(q, k, v, start_pos=-4)  # rows 0..3 see no key
    assert torch.all(out[:, :, :4] == 0)
    fa = A.flash_attention_ref(q, k, v, Br=4, Bc=8, start_pos=-4)
    assert torch.allclose(out, fa, atol=1e-5)
    assert torch.all(fa[:, :, :4] == 0)


def test_run_batch_ref_is_blockwise_dense():
    torch.manual_seed(1)
    N, BR, TK, D = 5, 32, 96, 64
    Q = torch.randn(N, BR, D).bfloat16()
    K = torch.randn(N, TK, D).bfloat16()
    V = torch.randn(N, TK, D).bfloat16()
    rows = [0, 32, 64, 17, -1_000_000]
    out = A.run_batch_ref(Q, K, V, rows)
    for n in range(N):
        ref = A.flash_attention_ref(Q[n][None, None], K[n][None, None], V[n][None, None], 16, 32,
                                    start_pos=rows[n])[0, 0]
        assert torch.allclose(out[n], ref, atol=1e-5)
    assert torch.all(out[4] == 0)  # the reference's dummy-block convention (npu/fa.py:236)


def test_decode_ref_equals_last_row_of_causal_prefill():
    torch.manual_seed(2)
    B, Hq, Hkv, Lmax, D = 3, 8, 2, 40, 64
    q = torch.randn(B, Hq, D).bfloat16()
    kc = torch.randn(B, Hkv, Lmax, D).bfloat16()
    vc = torch.randn(B, Hkv, Lmax, D).bfloat16()
    lens = [1, 23, 40]
    out = A.decode_ref(q, kc, vc, lens)
    for b, L in enumerate(lens):
        ref = A.dense_attention(q[b][None, :, None], kc[b:b + 1, :, :L], vc[b:b + 1, :, :L], start_pos=L - 1)
        assert torch.allclose(out[b], ref[0, :, 0], atol=1e-6)
    assert torch.all(A.decode_ref(q, kc, vc, [0, 0, 0]) == 0)


def test_prefill_rows_ref_matches_dense():
    torch.manual_seed(4)
    q = torch.randn(2, 8, 70, 64).bfloat16()
    k = torch.randn(2, 2, 90, 64).bfloat16()
    v = torch.randn(2, 2, 90, 64).bfloat16()
    dense = A.dense_attention(q, k, v, start_pos=20)
    rows = [0, 5, 69]
    got = A.prefill_rows_ref(q, k, v, 1, 5, rows, start_pos=20)
    assert torch.allclose(got, dense[1, 5, rows], atol=1e-6)


def test_flop_count_closed_form():
    assert A.attention_flops(1, 1, 64, 4, 4) == 4 * 64 * (1 + 2 + 3 + 4)
    T = 512
    assert A.attention_flops(64, 32, 128, T, T) == 4 * 64 * 32 * 128 * T * (T + 1) // 2
    assert A.attention_flops(1, 1, 8, 3, 10, causal=False) == 4 * 8 * 30


@pytest.mark.slow
def test_smollm_oracle_matches_reference_logits(smollm_golden):
    from oracle.smollm_ref import Config, SmolLM, make_state_dict

    model = SmolLM(make_state_dict(Config(), seed=0), Config())
    for T in (64, 128):
        ids = torch.from_numpy(smollm_golden[f"smollm_T{T}_ids"])
        logits, _ = model.forward(ids)
        ref = smollm_golden[f"smollm_T{T}_last_logits"]
        last = logits[0, -1].numpy()
        assert np.abs(last - ref).max() < 1e-4
        assert int(last.argmax()) == int(ref.argmax())


def test_smollm_hook_routes_attention_through_run_batch():
    """With an oracle-backed run_batch in layer.npu["attention"], the hooked
    forward equals the CPU-attention forward (the drop-in contract)."""
    from oracle.smollm_ref import Config, SmolLM, make_state_dict

    cfg = Config(n_layers=2)
    model = SmolLM(make_state_dict(cfg, seed=0), cfg)
    ids = torch.randint(0, cfg.vocab, (1, 45), generator=torch.Generator().manual_seed(1))
    base, _ = model.forward(ids)

    class FakeAttn:
        BR, BC = 32, 32
        calls = 0

        def run_batch(self, Q, K, V, start_rows, causal=True):
            FakeAttn.calls += 1
            return A.run_batch_ref(Q, K, V, start_rows, causal).to(torch.bfloat16)

    for layer in model.layers:
        layer.npu = {"attention": FakeAttn()}
    hooked, _ = model.forward(ids)
    assert FakeAttn.calls == cfg.n_layers
    assert torch.allclose(hooked, base, atol=5e-2)
    assert int(hooked[0, -1].argmax()) == int(base[0, -1].argmax())


def _qwen_golden():
    from conftest import GOLDEN
    return dict(np.load(GOLDEN / "qwen_attn.npz"))


def _as_torch(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return from_bits(a) if dtype == torch.bfloat16 else torch.from_numpy(a.copy())


@pytest.mark.parametrize("tag", ["f32", "bf16"])
def test_qwen_oracle_matches_reference_attn_forward(tag):
    """oracle/qwen_ref.py against outputs of the reference's own
    qwen/forward.py attn_forward (tests/golden/make_golden.py): a prefill from
    position 0 and single-token decode steps through the returned cache."""
    from oracle import qwen_ref as R

    g = _qwen_golden()
    cfg, layer, x, xs = R.golden_case(tag)
    dtype = x.dtype
    # the seeded weights and inputs are the ones the reference ran on
    assert R.fingerprint(*R.layer_tensors(layer)) == str(g[f"qwen_{tag}_weights_sha256"])
    assert R.fingerprint(x, *xs) == str(g[f"qwen_{tag}_inputs_sha256"])
    cos, sin = R.partial_rope_tables(cfg.rope_dim, R.QWEN_GOLDEN_MAX_POS, cfg.rope_theta, dtype)
    rows = g[f"qwen_{tag}_cache_rows"].tolist()
    assert torch.equal(cos[rows], _as_torch(g[f"qwen_{tag}_cos_rows"], dtype))
    assert torch.equal(sin[rows], _as_torch(g[f"qwen_{tag}_sin_rows"], dtype))
    # fp32: the restatement reorders nothing that matters beyond rounding;
    # bf16: one bf16 step of the largest output
    tol = 1e-5 if dtype == torch.float32 else 1.0 / 128

    def close(got, key):
        want = _as_torch(g[key], dtype).float()
        scale = max(1.0, want.abs().max().item())
        assert (got.float() - want).abs().max().item() <= tol * scale, key

    with torch.no_grad():
        y, cache = R.attn_forward(x, layer, cfg, cos, sin, None, 0)
        close(y, f"qwen_{tag}_prefill_out")
        pos = x.shape[1]
        for i, xi in enumerate(xs):
            y, cache = R.attn_forward(xi, layer, cfg, cos, sin, cache, pos)
            close(y, f"qwen_{tag}_decode{i}_out")
            pos += 1
    assert cache[0].shape[1] == pos
    close(cache[0][:, rows], f"qwen_{tag}_cache_k")
    close(cache[1][:, rows], f"qwen_{tag}_cache_v")
