"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/BojanFaletic-NPU

It imports the reference's own code — npu/fa_ref.py (flash_attention_ref,
_torch_causal_attention) and smollm.py (SmolLM) — runs it on seeded inputs,
and stores inputs and outputs in tests/golden/*.npz. The tests then check the
oracle in oracle/ against these files; nothing at test time reads the
reference checkout.
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().copy()


def load_module(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses look their module up here
    spec.loader.exec_module(mod)
    return mod


def fa_ref_cases(fa_ref) -> dict:
    """The reference self-test grid (npu/fa_ref.py:148-167): seed 0, B=1, H=9,
    D=64, shapes (Tq, Tk) with start_pos = Tk - Tq, three (Br, Bc) pairs; plus
    a non-causal case and a start_pos > 0 causal case."""
    out = {}
    torch.manual_seed(0)
    shapes = [(16, 16), (32, 32), (17, 17), (64, 64), (5, 20)]
    for i, (tq, tk) in enumerate(shapes):
        q = torch.randn(1, 9, tq, 64, dtype=torch.bfloat16)
        k = torch.randn(1, 9, tk, 64, dtype=torch.bfloat16)
        v = torch.randn(1, 9, tk, 64, dtype=torch.bfloat16)
        sp = tk - tq
        out[f"selftest{i}_q"] = bf16_bits(q)
        out[f"selftest{i}_k"] = bf16_bits(k)
        out[f"selftest{i}_v"] = bf16_bits(v)
        out[f"selftest{i}_meta"] = np.array([tq, tk, 64, sp], dtype=np.int64)
        out[f"selftest{i}_dense"] = fa_ref._torch_causal_attention(q, k, v, start_pos=sp).numpy()
        for Br, Bc in [(8, 16), (16, 32), (32, 32)]:
            out[f"selftest{i}_fa_{Br}_{Bc}"] = fa_ref.flash_attention_ref(
                q, k, v, Br=Br, Bc=Bc, causal=True, start_pos=sp).numpy()
    # Config 1 geometry: B=1, T=128, 9 query heads over 3 KV heads, D=64, seed 0.
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 9, 128, 64, generator=g).to(torch.bfloat16)
    k = torch.randn(1, 3, 128, 64, generator=g).to(torch.bfloat16)
    v = torch.randn(1, 3, 128, 64, generator=g).to(torch.bfloat16)
    ke, ve = k.repeat_interleave(3, dim=1), v.repeat_interleave(3, dim=1)
    out["cfg1_q"], out["cfg1_k"], out["cfg1_v"] = bf16_bits(q), bf16_bits(k), bf16_bits(v)
    out["cfg1_dense"] = fa_ref._torch_causal_attention(q, ke, ve, start_pos=0).numpy()
    out["cfg1_fa_32_32"] = fa_ref.flash_attention_ref(q, ke, ve, Br=32, Bc=32, causal=True).numpy()
    # Chunked prefill: 48 new rows after 80 cached keys, non-multiple tiles.
    q2 = torch.randn(1, 4, 48, 128, generator=g).to(torch.bfloat16)
    k2 = torch.randn(1, 4, 128, 128, generator=g).to(torch.bfloat16)
    v2 = torch.randn(1, 4, 128, 128, generator=g).to(torch.bfloat16)
    out["chunk_q"], out["chunk_k"], out["chunk_v"] = bf16_bits(q2), bf16_bits(k2), bf16_bits(v2)
    out["chunk_fa_16_32"] = fa_ref.flash_attention_ref(q2, k2, v2, Br=16, Bc=32, causal=True,
                                                       start_pos=80).numpy()
    out["chunk_nomask_fa_32_32"] = fa_ref.flash_attention_ref(q2, k2, v2, Br=32, Bc=32, causal=False).numpy()
    return out


def smollm_cases(smollm, Config, make_state_dict) -> dict:
    """Last-position logits of the reference smollm.py forward (CPU attention
    path) on the seeded random-init model, at T = 64 and T = 128."""
    out = {}
    cfg = smollm.Config()
    sd = make_state_dict(Config(), seed=0)
    model = smollm.SmolLM(sd, cfg)
    for T in (64, 128):
        ids = torch.randint(0, cfg.vocab, (1, T), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            logits, _ = model.forward(ids)
        out[f"smollm_T{T}_ids"] = ids.numpy()
        out[f"smollm_T{T}_last_logits"] = logits[0, -1].numpy()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    ref = Path(a.reference)
    sys.path.insert(0, str(ref))  # smollm.py imports npu.profiler
    sys.path.insert(0, str(REPO))
    torch.set_num_threads(max(1, torch.get_num_threads()))
    fa_ref = load_module("ref_fa_ref", ref / "npu" / "fa_ref.py")
    np.savez_compressed(HERE / "fa_ref_cases.npz", **fa_ref_cases(fa_ref))
    smollm = load_module("ref_smollm", ref / "smollm.py")
    from oracle.smollm_ref import Config, make_state_dict

    np.savez_compressed(HERE / "smollm_logits.npz", **smollm_cases(smollm, Config, make_state_dict))
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
