"""b2a_decode_noalloc — the decode entry point for callers that cannot
allocate device memory (it uses a fixed scratch buffer inside the library
instead of a caller workspace). Called through the C ABI and compared with
b2a_decode, the entry point that takes a caller workspace, on two calls in a
row with different geometries (the second call reuses the buffer the first
one left behind). Kept in its own file, collected last."""
import math

import pytest
import torch

from npu_b200 import _lib

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _inputs(B, Hq, Hkv, Lmax, D, seed, dev):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g).bfloat16().to(dev)
    kc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16().to(dev)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g).bfloat16().to(dev)
    lens = torch.randint(1, Lmax + 1, (B,), generator=g, dtype=torch.int32).to(dev)
    return q, kc, vc, lens


def _strides(q, kc, vc, o):
    return (_lib.ll2(*q.stride()[:2]), _lib.ll3(*kc.stride()[:3]), _lib.ll3(*vc.stride()[:3]),
            _lib.ll2(*o.stride()[:2]))


def _noalloc(q, kc, vc, lens, split=0):
    B, Hq, D = q.shape
    Hkv, Lmax = kc.shape[1], kc.shape[2]
    o = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    rc = _lib.load().b2a_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), o.data_ptr(), B, Hq, Hkv, Lmax, D,
        *_strides(q, kc, vc, o), 1.0 / math.sqrt(D), split, 1, torch.cuda.current_stream().cuda_stream)
    return rc, o


def _with_workspace(q, kc, vc, lens, split=0):
    lib = _lib.load()
    B, Hq, D = q.shape
    Hkv, Lmax = kc.shape[1], kc.shape[2]
    o = torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    need = lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split)
    ws = torch.empty(need, dtype=torch.uint8, device=q.device)
    rc = lib.b2a_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), o.data_ptr(), B, Hq, Hkv,
                        Lmax, D, *_strides(q, kc, vc, o), 1.0 / math.sqrt(D), split, 1, ws.data_ptr(), need,
                        torch.cuda.current_stream().cuda_stream)
    return rc, o


def test_noalloc_matches_workspace_decode_twice(cuda_dev):
    first = _inputs(4, 32, 4, 4096, 128, 11, cuda_dev)
    second = _inputs(3, 9, 3, 1000, 64, 12, cuda_dev)
    for q, kc, vc, lens in (first, second):
        rc, got = _noalloc(q, kc, vc, lens)
        assert rc == _lib.B2A_OK, _lib.strerror(rc)
        rc2, want = _with_workspace(q, kc, vc, lens)
        assert rc2 == _lib.B2A_OK
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() <= TOL


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_dev):
    q, kc, vc, lens = _inputs(2, 8, 2, 256, 64, 13, cuda_dev)
    lib = _lib.load()
    # 128 sequences x 4 KV heads x 512 splits of 64 keys needs ~1 GB of scratch.
    need = lib.b2a_decode_workspace_bytes(128, 32, 4, 128, 32768, 64)
    assert need > 16 * 1024 * 1024
    o = torch.empty(128, 32, 128, dtype=torch.float32, device=cuda_dev)
    rc = lib.b2a_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), o.data_ptr(),
                                128, 32, 4, 32768, 128, _lib.ll2(32 * 128, 128),
                                _lib.ll3(4 * 32768 * 128, 32768 * 128, 128),
                                _lib.ll3(4 * 32768 * 128, 32768 * 128, 128), _lib.ll2(32 * 128, 128),
                                0.088, 64, 1, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.B2A_ERR_WORKSPACE
