"""The C-ABI library without a GPU: it loads, exports every declared symbol,
and rejects bad arguments before touching CUDA. No compute is launched."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from npu_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))
FAKE = 0x10000  # 16-byte aligned, never dereferenced: validation fails first


def declared_symbols():
    names = set()
    for h in HEADERS:
        names |= set(re.findall(r"B2A_API\s+[\w\s\*]+?\b(b2a_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_headers_declare_the_abi():
    names = declared_symbols()
    for want in ("b2a_prefill", "b2a_decode", "b2a_decode_workspace_bytes", "b2a_strerror",
                 "b2a_get_device_error", "b2a_decode_default_split", "b2a_version"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_strerror_and_version():
    lib = _lib.load()
    for code in range(0, -12, -1):
        text = lib.b2a_strerror(code).decode()
        assert text and "unknown" not in text
    assert "unknown" in lib.b2a_strerror(-99).decode()
    assert lib.b2a_version() >= 100


def _prefill(**over):
    args = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, lse=None, B=1, Hq=8, Hkv=2, Tq=64, Tk=64, D=128,
                qs=(8 * 64 * 128, 64 * 128, 128), ks=(2 * 64 * 128, 64 * 128, 128),
                vs=(2 * 64 * 128, 64 * 128, 128), os=(8 * 64 * 128, 64 * 128, 128),
                sp=0, spb=None, scale=0.125, causal=1, fp32=1)
    args.update(over)
    a = args
    return _lib.load().b2a_prefill(a["q"], a["k"], a["v"], a["o"], a["lse"], a["B"], a["Hq"], a["Hkv"], a["Tq"],
                                   a["Tk"], a["D"], _lib.ll3(*a["qs"]), _lib.ll3(*a["ks"]), _lib.ll3(*a["vs"]),
                                   _lib.ll3(*a["os"]), a["sp"], a["spb"], a["scale"], a["causal"], a["fp32"],
                                   None)


def test_prefill_argument_validation():
    assert _prefill(q=None) == _lib.B2A_ERR_INVALID_ARG
    assert _prefill(B=0) == _lib.B2A_ERR_INVALID_ARG
    assert _prefill(Tq=0) == _lib.B2A_ERR_INVALID_ARG
    assert _prefill(scale=0.0) == _lib.B2A_ERR_INVALID_ARG
    assert _prefill(scale=float("nan")) == _lib.B2A_ERR_INVALID_ARG
    assert _prefill(D=96) == _lib.B2A_ERR_HEAD_DIM
    assert _prefill(D=512) == _lib.B2A_ERR_HEAD_DIM
    assert _prefill(Hkv=3) == _lib.B2A_ERR_GQA
    assert _prefill(q=FAKE + 2) == _lib.B2A_ERR_ALIGNMENT
    assert _prefill(qs=(8 * 64 * 128, 64 * 128, 100)) == _lib.B2A_ERR_ALIGNMENT
    assert _prefill(lse=FAKE + 2) == _lib.B2A_ERR_ALIGNMENT


def test_prefill_valid_args_without_gpu_report_cuda_error():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    assert _prefill() in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)


def test_decode_workspace_arithmetic():
    lib = _lib.load()
    # B=128, Hq=32, Hkv=4, D=128, Lmax=32768, split 2048 -> 16 splits, group 8
    n = 128 * 4 * 16 * 8
    want = ((n * 128 * 4 + 255) // 256) * 256 + ((n * 4 + 255) // 256) * 256
    assert lib.b2a_decode_workspace_bytes(128, 32, 4, 128, 32768, 2048) == want
    assert lib.b2a_decode_workspace_bytes(128, 32, 4, 128, 32768, 100) == 0  # not a multiple of 64
    assert lib.b2a_decode_workspace_bytes(1, 32, 1, 128, 64, 64) == 0       # group 32 > 16
    assert lib.b2a_decode_workspace_bytes(1, 8, 2, 96, 64, 64) == 0         # head_dim
    s = lib.b2a_decode_default_split(128, 4, 32768)
    assert s % 64 == 0 and 512 <= s <= 4096
    assert lib.b2a_decode_default_split(1, 1, 100) == 512


def test_decode_argument_validation():
    lib = _lib.load()

    def call(**over):
        a = dict(q=FAKE, k=FAKE, v=FAKE, sl=FAKE, o=FAKE, B=2, Hq=8, Hkv=2, L=256, D=128, split=64,
                 ws=FAKE, wsb=1 << 30, scale=0.1)
        a.update(over)
        return lib.b2a_decode(a["q"], a["k"], a["v"], a["sl"], a["o"], a["B"], a["Hq"], a["Hkv"], a["L"], a["D"],
                              _lib.ll2(8 * 128, 128), _lib.ll3(2 * 256 * 128, 256 * 128, 128),
                              _lib.ll3(2 * 256 * 128, 256 * 128, 128), _lib.ll2(8 * 128, 128),
                              a["scale"], a["split"], 1, a["ws"], a["wsb"], None)

    assert call(sl=None) == _lib.B2A_ERR_INVALID_ARG
    assert call(D=80) == _lib.B2A_ERR_HEAD_DIM
    assert call(Hkv=3) == _lib.B2A_ERR_GQA
    assert call(split=100) == _lib.B2A_ERR_INVALID_ARG
    assert call(k=FAKE + 8) == _lib.B2A_ERR_ALIGNMENT
    assert call(ws=None) == _lib.B2A_ERR_WORKSPACE
    assert call(wsb=16) == _lib.B2A_ERR_WORKSPACE
    if not torch.cuda.is_available():
        assert call() in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)


def test_python_api_refuses_cpu_tensors():
    from npu_b200 import api

    q = torch.zeros(1, 2, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        api.prefill(q, q, q)
    with pytest.raises(ValueError, match="CUDA"):
        api.decode(q[:, :, 0], q, q, torch.zeros(1, dtype=torch.int32))


def test_b2a_error_carries_status_text():
    err = _lib.B2AError(_lib.B2A_ERR_GQA, "b2a_prefill")
    assert err.code == _lib.B2A_ERR_GQA and "multiple" in str(err)


def _rope(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, qs=(5 * 8 * 64, 8 * 64, 64), ks=(5 * 2 * 64, 2 * 64, 64),
             vs=(5 * 2 * 64, 2 * 64, 64), bf16=0, cos=FAKE, sin=FAKE, max_pos=64, q_out=FAKE, kc=FAKE, vc=FAKE,
             kcs=(2 * 32 * 64, 32 * 64, 64), vcs=(2 * 32 * 64, 32 * 64, 64), B=1, T=5, Hq=8, Hkv=2, D=64,
             Lmax=32, sp=0, spb=None, seq=None)
    a.update(over)
    return _lib.load().b2a_rope_append(
        a["q"], a["k"], a["v"], _lib.ll3(*a["qs"]), _lib.ll3(*a["ks"]), _lib.ll3(*a["vs"]), a["bf16"], a["cos"],
        a["sin"], a["max_pos"], a["q_out"], a["kc"], a["vc"], _lib.ll3(*a["kcs"]), _lib.ll3(*a["vcs"]), a["B"],
        a["T"], a["Hq"], a["Hkv"], a["D"], a["Lmax"], a["sp"], a["spb"], a["seq"], None)


def test_rope_append_argument_validation():
    assert _rope(q=None) == _lib.B2A_ERR_INVALID_ARG
    assert _rope(T=0) == _lib.B2A_ERR_INVALID_ARG
    assert _rope(D=96) == _lib.B2A_ERR_HEAD_DIM
    assert _rope(sp=28) == _lib.B2A_ERR_INVALID_ARG       # 28 + 5 > Lmax
    assert _rope(sp=-1) == _lib.B2A_ERR_INVALID_ARG
    assert _rope(max_pos=4) == _lib.B2A_ERR_INVALID_ARG   # positions past the rotary table
    assert _rope(q=FAKE + 8) == _lib.B2A_ERR_ALIGNMENT    # fp32 sources need 16-byte alignment
    assert _rope(bf16=1, qs=(5 * 8 * 64, 8 * 64, 68)) == _lib.B2A_ERR_ALIGNMENT  # bf16: 16-byte strides
    assert _rope(kcs=(2 * 32 * 64, 32 * 64, 66)) == _lib.B2A_ERR_ALIGNMENT
    assert _rope(kc=FAKE + 4) == _lib.B2A_ERR_ALIGNMENT


def _qk_rope(**over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, qs=(5 * 16 * 512, 16 * 512, 512), ks=(5 * 2 * 256, 2 * 256, 256),
             vs=(5 * 2 * 256, 2 * 256, 256), bf16=0, qn=FAKE, kn=FAKE, eps=1e-6, cos=FAKE, sin=FAKE, max_pos=64,
             rd=64, q_out=FAKE, kc=FAKE, vc=FAKE, kcs=(2 * 32 * 256, 32 * 256, 256), vcs=(2 * 32 * 256, 32 * 256, 256),
             B=1, T=5, Hq=16, Hkv=2, D=256, Lmax=32, sp=0, spb=None, seq=None)
    a.update(over)
    return _lib.load().b2a_qk_norm_rope_append(
        a["q"], a["k"], a["v"], _lib.ll3(*a["qs"]), _lib.ll3(*a["ks"]), _lib.ll3(*a["vs"]), a["bf16"], a["qn"],
        a["kn"], a["eps"], a["cos"], a["sin"], a["max_pos"], a["rd"], a["q_out"], a["kc"], a["vc"],
        _lib.ll3(*a["kcs"]), _lib.ll3(*a["vcs"]), a["B"], a["T"], a["Hq"], a["Hkv"], a["D"], a["Lmax"], a["sp"],
        a["spb"], a["seq"], None)


def test_qk_norm_rope_append_argument_validation():
    assert _qk_rope(rd=48) == _lib.B2A_ERR_INVALID_ARG      # not a power of two
    assert _qk_rope(rd=8) == _lib.B2A_ERR_INVALID_ARG       # below 16
    assert _qk_rope(rd=512) == _lib.B2A_ERR_INVALID_ARG     # above D
    assert _qk_rope(eps=float("nan")) == _lib.B2A_ERR_INVALID_ARG
    assert _qk_rope(qn=FAKE + 4) == _lib.B2A_ERR_ALIGNMENT
    assert _qk_rope(rd=0, cos=None, sin=None, sp=40) == _lib.B2A_ERR_INVALID_ARG   # past Lmax
    if not torch.cuda.is_available():
        assert _qk_rope() in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)
        assert _qk_rope(rd=0, cos=None, sin=None, qn=None, kn=None) in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)


def _a256(x):
    return (x + 255) // 256 * 256


def test_prefill_host_workspace_arithmetic():
    lib = _lib.load()
    # Config 3 geometry; the default 32 chunks hold 2 whole batches each:
    # 2 slots of q/k/v/o + B ints.
    B, Hq, Hkv, T, D = 64, 32, 4, 8192, 128
    per = 2 * Hkv  # units per chunk
    slot = _a256(per * 8 * T * D * 2) + 2 * _a256(per * T * D * 2) + _a256(per * 8 * T * D * 2)
    assert lib.b2a_prefill_host_workspace_bytes(B, Hq, Hkv, T, T, D, 0, 0) == 2 * slot + _a256(B * 4)
    assert lib.b2a_prefill_host_workspace_bytes(B, Hq, Hkv, T, T, D, 0, 32) == 2 * slot + _a256(B * 4)
    # 16 chunks of 4 batches, fp32 output (o region doubled).
    per = 4 * Hkv
    slot32 = _a256(per * 8 * T * D * 2) + 2 * _a256(per * T * D * 2) + _a256(per * 8 * T * D * 4)
    assert lib.b2a_prefill_host_workspace_bytes(B, Hq, Hkv, T, T, D, 1, 16) == 2 * slot32 + _a256(B * 4)
    # One batch, fewer units than chunks: chunks are single KV heads.
    one = _a256(8 * 512 * 64 * 2) + 2 * _a256(512 * 64 * 2) + _a256(8 * 512 * 64 * 2)
    assert lib.b2a_prefill_host_workspace_bytes(1, 32, 4, 512, 512, 64, 0, 0) == 2 * one + 256
    for bad in ((0, 8, 2, 64, 64, 128, 0, 0), (1, 8, 3, 64, 64, 128, 0, 0), (1, 8, 2, 64, 64, 96, 0, 0),
                (1, 8, 2, 0, 64, 128, 0, 0), (1, 8, 2, 64, -1, 128, 0, 0), (1, 8, 2, 64, 64, 128, 0, -1)):
        assert lib.b2a_prefill_host_workspace_bytes(*bad) == 0, bad


def test_prefill_host_argument_validation():
    lib = _lib.load()

    def call(**over):
        a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, B=2, Hq=8, Hkv=2, Tq=64, Tk=64, D=128, sp=0, spb=None,
                 scale=0.125, causal=1, fp32=0, n=0, ws=FAKE * 16, wsb=1 << 30)
        a.update(over)
        return lib.b2a_prefill_host(a["q"], a["k"], a["v"], a["o"], a["B"], a["Hq"], a["Hkv"], a["Tq"],
                                    a["Tk"], a["D"], a["sp"], a["spb"], a["scale"], a["causal"], a["fp32"],
                                    a["n"], a["ws"], a["wsb"], None)

    assert call(D=96) == _lib.B2A_ERR_HEAD_DIM
    assert call(Hkv=3) == _lib.B2A_ERR_GQA
    assert call(B=0) == _lib.B2A_ERR_INVALID_ARG
    assert call(q=None) == _lib.B2A_ERR_INVALID_ARG
    assert call(k=None) == _lib.B2A_ERR_INVALID_ARG
    assert call(scale=0.0) == _lib.B2A_ERR_INVALID_ARG
    assert call(ws=None) == _lib.B2A_ERR_WORKSPACE
    assert call(wsb=1024) == _lib.B2A_ERR_WORKSPACE
    assert call(ws=FAKE * 16 + 16) == _lib.B2A_ERR_WORKSPACE  # workspace must be 256-byte aligned
    if not torch.cuda.is_available():
        assert call() in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)


def test_prefill_host_python_argument_checks():
    """npu_b200.api.prefill_host validates its host tensors before touching
    CUDA: device tensors, other dtypes, non-contiguous or mismatched shapes,
    and start positions of the wrong length are refused."""
    from npu_b200 import api

    q = torch.zeros(2, 4, 16, 64, dtype=torch.bfloat16)
    k = torch.zeros(2, 2, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        api.prefill_host(q.float(), k, k)
    with pytest.raises(ValueError):
        api.prefill_host(q.transpose(1, 2), k, k)  # not contiguous
    with pytest.raises(ValueError):
        api.prefill_host(q, k[:, :, :8], k)        # k / v shapes differ
    with pytest.raises(ValueError):
        api.prefill_host(q, k[:1], k[:1])          # batch mismatch
    with pytest.raises(ValueError):
        api.prefill_host(q, k, k, out_dtype=torch.float16)
    with pytest.raises(ValueError):
        api.prefill_host(q, k, k, start_pos_per_batch=[0, 1, 2])
    with pytest.raises(ValueError):
        api.prefill_host(q, k, k, out=torch.empty(2, 4, 16, 64, dtype=torch.float32))  # out dtype
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            api.prefill_host(q, k, k)  # no device: no CPU path


def test_noalloc_scratch_constant_and_checks_without_gpu():
    """b2a_decode_noalloc: the Python mirror of B2A_NOALLOC_SCRATCH_BYTES
    matches the header, and a problem that cannot fit the fixed scratch is
    rejected before any CUDA call (FAKE pointers are never dereferenced)."""
    text = (ROOT / "include" / "b2attn.h").read_text()
    m = re.search(r"#define\s+B2A_NOALLOC_SCRATCH_BYTES\s+\((\d+)u\s*\*\s*(\d+)u\s*\*\s*(\d+)u\)", text)
    assert m, "B2A_NOALLOC_SCRATCH_BYTES not found in b2attn.h"
    assert int(m[1]) * int(m[2]) * int(m[3]) == _lib.B2A_NOALLOC_SCRATCH_BYTES
    lib = _lib.load()

    def call(B, Hq, Hkv, L, D, split):
        return lib.b2a_decode_noalloc(FAKE, FAKE, FAKE, FAKE, FAKE, B, Hq, Hkv, L, D,
                                      _lib.ll2(Hq * D, D), _lib.ll3(Hkv * L * D, L * D, D),
                                      _lib.ll3(Hkv * L * D, L * D, D), _lib.ll2(Hq * D, D), 0.1, split, 1, None)

    # an explicit split whose partials exceed the scratch
    assert lib.b2a_decode_workspace_bytes(16, 32, 8, 256, 4096, 64) > _lib.B2A_NOALLOC_SCRATCH_BYTES
    assert call(16, 32, 8, 4096, 256, 64) == _lib.B2A_ERR_WORKSPACE
    # default split: even one split per sequence needs B*Hq*D*4 bytes > 16 MiB
    assert lib.b2a_decode_workspace_bytes(128, 128, 8, 256, 64, 64) > _lib.B2A_NOALLOC_SCRATCH_BYTES
    assert call(128, 128, 8, 64, 256, 0) == _lib.B2A_ERR_WORKSPACE
    if not torch.cuda.is_available():
        # config-4 geometry fits once the split is lengthened; without a GPU the
        # call then stops at the device lookup
        assert call(128, 32, 4, 32768, 128, 0) in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)


def test_decode_proj_argument_validation():
    """b2a_decode_proj rejects a missing or misaligned projection weight or
    residual stream before any CUDA call."""
    lib = _lib.load()

    def call(wo=FAKE, wo_ld=8 * 128, w32=0, dim=576, x=FAKE, x_sb=576, x32=1, D=128, split=64):
        return lib.b2a_decode_proj(FAKE, FAKE, FAKE, FAKE, wo, wo_ld, w32, dim, x, x_sb, x32, 2, 8, 2, 256, D,
                                   _lib.ll2(8 * 128, 128), _lib.ll3(2 * 256 * 128, 256 * 128, 128),
                                   _lib.ll3(2 * 256 * 128, 256 * 128, 128), 0.1, split, FAKE, 1 << 30, None)

    assert call(wo=None) == _lib.B2A_ERR_INVALID_ARG
    assert call(x=None) == _lib.B2A_ERR_INVALID_ARG
    assert call(dim=0) == _lib.B2A_ERR_INVALID_ARG
    assert call(wo_ld=100) == _lib.B2A_ERR_INVALID_ARG       # < Hq * D
    assert call(x_sb=500) == _lib.B2A_ERR_INVALID_ARG        # < dim
    assert call(wo=FAKE + 8) == _lib.B2A_ERR_ALIGNMENT
    assert call(wo_ld=8 * 128 + 4) == _lib.B2A_ERR_ALIGNMENT  # bf16 rows not 16-byte aligned
    assert call(x=FAKE + 2) == _lib.B2A_ERR_ALIGNMENT         # fp32 x
    assert call(D=96) == _lib.B2A_ERR_HEAD_DIM
    if not torch.cuda.is_available():
        assert call() in (_lib.B2A_ERR_CUDA, _lib.B2A_ERR_DEVICE)
