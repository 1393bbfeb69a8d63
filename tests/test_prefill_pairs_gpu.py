"""The opt-in SM-pair prefill (head dim 128, even GQA group: two CTAs of a
cluster share every M = 256 UMMA, each loading half of K and V). Selected by
the environment variable B2A_PREFILL_SM_PAIRS (a row threshold), which the
library reads on every call. It must give the one-SM kernel's output bit for
bit, and the fp32 oracle's within the north-star tolerance."""
import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _rand(shape, gen, dev):
    return torch.randn(*shape, generator=gen).to(torch.bfloat16).to(dev)


# (B, Hq, Hkv, Tq, Tk, start_pos, causal): tails, Tq < Tk with a start
# position, a negative start (rows without keys), non-causal, ragged rows.
CASES = [
    (2, 8, 2, 256, 256, 0, True),
    (1, 8, 4, 300, 300, 0, True),
    (2, 4, 2, 129, 700, 500, True),
    (1, 4, 1, 200, 200, -130, True),
    (1, 8, 2, 333, 250, 0, False),
    (1, 32, 4, 1100, 1100, 0, True),
]


@pytest.mark.parametrize("B,Hq,Hkv,Tq,Tk,sp,causal", CASES)
def test_sm_pairs_match_one_sm_kernel_and_oracle(cuda_dev, monkeypatch, B, Hq, Hkv, Tq, Tk, sp, causal):
    from npu_b200 import api

    g = torch.Generator().manual_seed(Tq * 13 + Tk + B)
    q, k, v = _rand((B, Hq, Tq, 128), g, cuda_dev), _rand((B, Hkv, Tk, 128), g, cuda_dev), \
        _rand((B, Hkv, Tk, 128), g, cuda_dev)
    monkeypatch.delenv("B2A_PREFILL_SM_PAIRS", raising=False)
    one, lse1 = api.prefill(q, k, v, start_pos=sp, causal=causal, out_dtype=torch.float32, return_lse=True)
    monkeypatch.setenv("B2A_PREFILL_SM_PAIRS", "1")
    pair, lse2 = api.prefill(q, k, v, start_pos=sp, causal=causal, out_dtype=torch.float32, return_lse=True)
    monkeypatch.delenv("B2A_PREFILL_SM_PAIRS")
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(pair, one), (pair - one).abs().max().item()
    assert torch.equal(lse2, lse1)
    ref = A.dense_attention(q.cpu(), k.cpu(), v.cpu(), start_pos=sp, causal=causal)
    assert (pair.cpu() - ref).abs().max().item() <= TOL


def test_sm_pairs_threshold_and_bf16_output(cuda_dev, monkeypatch):
    """Below the threshold the one-SM kernel runs; at it, the pairs. Both give
    the same bf16 output (config 3 heads, 2048 rows)."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(7)
    q, k, v = _rand((2, 32, 2048, 128), g, cuda_dev), _rand((2, 4, 2048, 128), g, cuda_dev), \
        _rand((2, 4, 2048, 128), g, cuda_dev)
    monkeypatch.setenv("B2A_PREFILL_SM_PAIRS", "4096")
    below = api.prefill(q, k, v, out_dtype=torch.bfloat16)
    monkeypatch.setenv("B2A_PREFILL_SM_PAIRS", "2048")
    at = api.prefill(q, k, v, out_dtype=torch.bfloat16)
    monkeypatch.delenv("B2A_PREFILL_SM_PAIRS")
    torch.cuda.synchronize()
    assert api.device_error() == 0
    assert torch.equal(at, below)
    rows = [0, 1, 127, 128, 255, 256, 1023, 2047]
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    for b, h in ((0, 0), (1, 31), (0, 9)):
        ref = A.prefill_rows_ref(qc, kc, vc, b, h, rows)
        assert (at[b, h, rows].float().cpu() - ref).abs().max().item() <= TOL
