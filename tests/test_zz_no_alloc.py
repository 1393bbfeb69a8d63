"""b2a_decode_noalloc — the decode entry point for callers that cannot
allocate device memory (it uses a fixed scratch buffer inside the library
instead of a caller workspace). Called through the C ABI and compared with
b2a_decode, the entry point that takes a caller workspace: the two run the
same kernels with the same split length, so their outputs must be identical
bit for bit, on two calls in a row with different geometries (the second call
reuses the buffer the first one left behind). One case is also checked
against the fp32 oracle. Kept in its own file, collected last."""
import math

import pytest
import torch

from npu_b200 import _lib
from oracle.attention import decode_ref

pytestmark = pytest.mark.gpu
TOL = 2e-2
CAP = _lib.B2A_NOALLOC_SCRATCH_BYTES


def _inputs(B, Hq, Hkv, Lmax, D, seed, dev, lo=1):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g, device=dev).bfloat16()
    kc = torch.randn(B, Hkv, Lmax, D, generator=g, device=dev, dtype=torch.bfloat16)
    vc = torch.randn(B, Hkv, Lmax, D, generator=g, device=dev, dtype=torch.bfloat16)
    lens = torch.randint(lo, Lmax + 1, (B,), generator=g, device=dev, dtype=torch.int32)
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
    for i, (q, kc, vc, lens) in enumerate((first, second)):
        rc, got = _noalloc(q, kc, vc, lens)
        assert rc == _lib.B2A_OK, _lib.strerror(rc)
        rc2, want = _with_workspace(q, kc, vc, lens)
        assert rc2 == _lib.B2A_OK
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert torch.equal(got, want), (i, (got - want).abs().max().item())
        if i == 0:
            ref = decode_ref(q.cpu(), kc.cpu(), vc.cpu(), lens.cpu().tolist())
            assert (got.cpu() - ref).abs().max().item() <= TOL


def test_noalloc_lengthens_the_default_split_to_fit(cuda_dev):
    """Config 4's geometry (128 sequences, 32/4 heads, D=128, 32k-key caches):
    the speed-tuned default split needs more than the fixed scratch, so the
    entry point doubles it until the partials fit and still gives b2a_decode's
    result for that split."""
    lib = _lib.load()
    B, Hq, Hkv, Lmax, D = 128, 32, 4, 32768, 128
    split = lib.b2a_decode_default_split(B, Hkv, Lmax)
    assert lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split) > CAP
    while lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, split) > CAP:
        split *= 2
    assert split < Lmax
    q, kc, vc, lens = _inputs(B, Hq, Hkv, Lmax, D, 21, cuda_dev, lo=1024)
    rc, got = _noalloc(q, kc, vc, lens)
    assert rc == _lib.B2A_OK, _lib.strerror(rc)
    rc2, want = _with_workspace(q, kc, vc, lens, split)
    assert rc2 == _lib.B2A_OK
    torch.cuda.synchronize()
    assert torch.equal(got, want), (got - want).abs().max().item()
    for b in (0, int(torch.argmax(lens).item())):
        ref = decode_ref(q[b:b + 1].cpu(), kc[b:b + 1].cpu(), vc[b:b + 1].cpu(), [int(lens[b])])
        assert (got[b:b + 1].cpu() - ref).abs().max().item() <= TOL


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_dev):
    """Real tensors of the declared geometry, so nothing could read out of
    bounds even if the size check moved after the launch."""
    lib = _lib.load()
    # An explicit split of 64 keys: 16 x 8 KV heads x 64 splits x 4 heads x
    # 256 fp32 partials, about 33 MB.
    B, Hq, Hkv, Lmax, D = 16, 32, 8, 4096, 256
    assert lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, 64) > CAP
    q, kc, vc, lens = _inputs(B, Hq, Hkv, Lmax, D, 13, cuda_dev)
    rc, _ = _noalloc(q, kc, vc, lens, split=64)
    assert rc == _lib.B2A_ERR_WORKSPACE
    # Default split: even one split per sequence needs B * Hq * D * 4 bytes.
    B, Hq, Hkv, Lmax, D = 128, 128, 8, 64, 256
    assert lib.b2a_decode_workspace_bytes(B, Hq, Hkv, D, Lmax, 64) > CAP
    q, kc, vc, lens = _inputs(B, Hq, Hkv, Lmax, D, 14, cuda_dev)
    rc, _ = _noalloc(q, kc, vc, lens)
    assert rc == _lib.B2A_ERR_WORKSPACE
    torch.cuda.synchronize()
