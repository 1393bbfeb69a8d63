"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once where the reference checkout is available:

    python tests/golden/make_golden.py --reference /path/to/BojanFaletic-NPU

It imports the reference's own code — npu/fa_ref.py (flash_attention_ref,
_torch_causal_attention), smollm.py (SmolLM) and qwen/forward.py
(attn_forward, AttnLayer, with qwen/model.py's Config) — runs it on seeded
inputs, and stores inputs and outputs in tests/golden/*.npz. The tests then check the
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


def qwen_cases(qf, qm) -> dict:
    """The reference's gated attention (qwen/forward.py:133-239) on seeded
    random weights: a prefill from position 0, then single-token decode steps
    that feed the returned cache back in, exactly as the reference's forward
    loop does. The weights and inputs come from oracle.qwen_ref.golden_case
    (seeded, regenerated at test time); their SHA-256 fingerprints are stored.
    Stored outputs: every step's block output, and sampled rows of the final
    (k, v) cache of expanded heads."""
    from oracle import qwen_ref as R

    out = {}
    for tag in R.QWEN_GOLDEN_CASES:
        cfg, layer, x, xs = R.golden_case(tag)
        dtype = x.dtype
        ref_cfg = qm.Config(arch="qwen35moe", n_layer=1, n_ctx_train=R.QWEN_GOLDEN_MAX_POS, d_model=cfg.d_model,
                            n_head=cfg.n_head, n_head_kv=cfg.n_head_kv, head_dim=cfg.head_dim,
                            rms_eps=cfg.rms_eps, rope_theta=cfg.rope_theta, rope_dim=cfg.rope_dim, n_expert=1,
                            n_expert_used=1, d_expert_ff=1, vocab_size=1, bos_id=0, eos_id=0, pad_id=None,
                            is_attention=[True])
        ref_layer = qf.AttnLayer(i=0, attn_norm=layer.attn_norm, post_norm=torch.ones_like(layer.attn_norm),
                                 wq=layer.wq, wk=layer.wk, wv=layer.wv, wo=layer.wo, q_norm=layer.q_norm,
                                 k_norm=layer.k_norm)
        cos, sin = qf.build_partial_rope_cache(cfg.rope_dim, R.QWEN_GOLDEN_MAX_POS, cfg.rope_theta, dtype=dtype)
        keep = bf16_bits if dtype == torch.bfloat16 else (lambda t: t.numpy().copy())
        with torch.no_grad():
            y, cache = qf.attn_forward(x, ref_layer, ref_cfg, cos, sin, None, 0)
            out[f"qwen_{tag}_prefill_out"] = keep(y)
            pos = x.shape[1]
            for i, xi in enumerate(xs):
                y, cache = qf.attn_forward(xi, ref_layer, ref_cfg, cos, sin, cache, pos)
                out[f"qwen_{tag}_decode{i}_out"] = keep(y)
                pos += 1
        rows = sorted({0, 1, 127, 128, x.shape[1] - 1, x.shape[1], pos - 1} & set(range(pos)))
        out[f"qwen_{tag}_cache_rows"] = np.array(rows, dtype=np.int64)
        out[f"qwen_{tag}_cache_k"] = keep(cache[0][:, rows].contiguous())
        out[f"qwen_{tag}_cache_v"] = keep(cache[1][:, rows].contiguous())
        out[f"qwen_{tag}_cos_rows"] = keep(cos[rows].contiguous())
        out[f"qwen_{tag}_sin_rows"] = keep(sin[rows].contiguous())
        out[f"qwen_{tag}_weights_sha256"] = np.array(R.fingerprint(*R.layer_tensors(layer)))
        out[f"qwen_{tag}_inputs_sha256"] = np.array(R.fingerprint(x, *xs))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    ap.add_argument("--only", choices=["fa_ref", "smollm", "qwen"], action="append",
                    help="write only these fixtures (default: all)")
    a = ap.parse_args()
    want = set(a.only or ["fa_ref", "smollm", "qwen"])
    ref = Path(a.reference)
    sys.path.insert(0, str(ref))  # smollm.py imports npu.profiler
    sys.path.insert(0, str(REPO))
    torch.set_num_threads(max(1, torch.get_num_threads()))
    if "fa_ref" in want:
        fa_ref = load_module("ref_fa_ref", ref / "npu" / "fa_ref.py")
        np.savez_compressed(HERE / "fa_ref_cases.npz", **fa_ref_cases(fa_ref))
    if "smollm" in want:
        smollm = load_module("ref_smollm", ref / "smollm.py")
        from oracle.smollm_ref import Config, make_state_dict

        np.savez_compressed(HERE / "smollm_logits.npz", **smollm_cases(smollm, Config, make_state_dict))
    if "qwen" in want:
        import qwen.forward as qf  # qwen/forward.py imports qwen.model (gguf) by package name
        import qwen.model as qm

        np.savez_compressed(HERE / "qwen_attn.npz", **qwen_cases(qf, qm))
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
