"""Failure reporting on the GPU without a GPU fault: every wait in the
kernels is bounded; when one runs out the kernel raises its CTA's abort flag,
records B2A_ERR_DEVICE_TIMEOUT in the device error word and exits, and the
CUDA context stays usable. A diagnostic kernel waits on an mbarrier that
nothing ever arrives on (with a ~1 ms bound instead of the kernels' ~2 s)."""
import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda_dev):
    from npu_b200 import _lib, api

    lib = _lib.load()
    api.device_error()  # start from a clear error word
    stream = torch.cuda.current_stream(cuda_dev).cuda_stream
    assert lib.b2a_diag_wait_timeout(2_000_000, stream) == 0
    assert api.device_error(clear=False) == _lib.B2A_ERR_DEVICE_TIMEOUT
    assert api.device_error() == _lib.B2A_ERR_DEVICE_TIMEOUT  # read and clear
    assert api.device_error() == 0
    # The context is intact: a normal prefill runs and is correct.
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 200, 128, generator=g).bfloat16().to(cuda_dev)
    k = torch.randn(1, 2, 200, 128, generator=g).bfloat16().to(cuda_dev)
    out = api.prefill(q, k, k)
    assert (out.cpu() - A.dense_attention(q.cpu(), k.cpu(), k.cpu())).abs().max().item() <= 2e-2
    assert api.device_error() == 0


def test_bad_sequence_length_is_reported_not_faulted(cuda_dev):
    """A decode sequence length beyond the cache is clamped on the device and
    reported as B2A_ERR_DEVICE_BAD_LEN."""
    from npu_b200 import _lib, api

    api.device_error()
    g = torch.Generator().manual_seed(4)
    q = torch.randn(2, 8, 64, generator=g).bfloat16().to(cuda_dev)
    kc = torch.randn(2, 2, 128, 64, generator=g).bfloat16().to(cuda_dev)
    lens = torch.tensor([100, 500], dtype=torch.int32, device=cuda_dev)
    api.decode(q, kc, kc, lens)
    assert api.device_error() == _lib.B2A_ERR_DEVICE_BAD_LEN
    assert api.device_error() == 0
