"""Config 2: SmolLM2-135M 30-layer causal prefill with the B200 kernel swapped
in for every layer through layer.npu["attention"] (smollm.py:212-221); the
top-1 token at position T-1 must equal the CPU path's (smollm.py:222-234).

The model runs in fp32 with bf16 Q/K/V into the kernel, as the reference's NPU
path does (npu/fa.py:267,287-289): the reference caller casts the attention
result with .float() (smollm.py:163), so a bf16 model cannot take that route.
"""
import pytest
import torch

from oracle.smollm_ref import Config, SmolLM, make_state_dict

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cpu_model():
    return SmolLM(make_state_dict(Config(), seed=0), Config())


def _ids(T: int) -> torch.Tensor:
    return torch.randint(0, Config().vocab, (1, T), generator=torch.Generator().manual_seed(1))


def test_config2_top1_model_on_gpu(cuda_dev, cpu_model):
    from npu_b200 import enable_attention

    ids = _ids(1024)
    ref_logits, _ = cpu_model.forward(ids)
    gpu_model = SmolLM(make_state_dict(Config(), seed=0), Config()).to(cuda_dev)
    shared = enable_attention(gpu_model)
    assert all(layer.npu["attention"] is shared for layer in gpu_model.layers)
    logits, cache = gpu_model.forward(ids.to(cuda_dev))
    last, ref_last = logits[0, -1].float().cpu(), ref_logits[0, -1]
    assert int(last.argmax()) == int(ref_last.argmax())
    assert (last - ref_last).abs().max().item() < 0.25  # the reference accepts 2.75e-1 (plans/01-fa-decode.md:154)
    assert len(cache) == 30 and cache[0][0].shape == (1, 3, 1024, 64)


def test_run_batch_with_host_resident_model(cuda_dev, cpu_model):
    """The reference's own deployment: the model on the CPU, only attention on
    the accelerator (run_batch receives and returns host tensors)."""
    from npu_b200 import NpuAttention

    ids = _ids(200)
    ref_logits, _ = cpu_model.forward(ids)
    attn = NpuAttention(D=64)
    for layer in cpu_model.layers:
        layer.npu = {"attention": attn}
    try:
        logits, _ = cpu_model.forward(ids)
    finally:
        for layer in cpu_model.layers:
            layer.npu = None
    assert int(logits[0, -1].argmax()) == int(ref_logits[0, -1].argmax())
    assert (logits[0, -1] - ref_logits[0, -1]).abs().max().item() < 0.25


def test_decode_attention_through_run_batch(cuda_dev, cpu_model):
    """T=1 decode routed through run_batch with Tk buckets
    (npu_decode_attention, smollm.py:144,212-221) after a prefill."""
    from npu_b200 import NpuAttention

    ids = _ids(100)
    _, cache = cpu_model.forward(ids)
    nxt = torch.tensor([[123]])
    ref_logits, _ = cpu_model.forward(nxt, cache=cache, start_pos=100)
    attn = NpuAttention(D=64)
    for layer in cpu_model.layers:
        layer.npu = {"attention": attn}
        layer.npu_decode_attention = True
    try:
        logits, _ = cpu_model.forward(nxt, cache=cache, start_pos=100)
    finally:
        for layer in cpu_model.layers:
            layer.npu = None
            layer.npu_decode_attention = False
    assert int(logits[0, -1].argmax()) == int(ref_logits[0, -1].argmax())
    assert (logits[0, -1] - ref_logits[0, -1]).abs().max().item() < 0.25
