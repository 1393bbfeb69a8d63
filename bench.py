"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): causal GQA prefill attention throughput, algorithmic
TFLOP/s, on config 3 at T=8192 (B=64, Hq=32, Hkv=4, D=128, bf16,
scale 1/sqrt(128)); the (batch x KV-head) units are split across the N GPUs
with no collective (strong scaling: total work fixed). A step is one launch
over the whole batch. `decode` reports config 4 (128 sequences, one query
token, lengths ~ U[1024, 32768], HBM GB/s) the same way; `sweep` reports the
config 3 prefill at T=512 and T=2048; `long_context` reports config 5 (one
131072-token sequence, D=256; zig-zag context parallel with a NCCL K/V
all-gather when N > 1).

Timing: W untimed steps, then K steps bracketed by barrier + synchronize,
CUDA events on the launching stream, max over ranks. Inputs are larger than
the 126 MB L2 (Q alone is 4.3 GB at T=8192), so no flush is needed.
`--impl reference` times the CPU restatement of the reference's attention
(dense fp32 attention of smollm.py:222-234) on a bounded sample instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "causal-prefill attn TFLOP/s + decode attn HBM GB/s at 1/2/4/8 B200"
CFG3 = dict(B=64, Hq=32, Hkv=4, D=128)
CFG4 = dict(B=128, Hq=32, Hkv=4, D=128, Lmin=1024, Lmax=32768)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ----------------------------------------------------------------- helpers
def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def prefill_flops(B: int, Hq: int, D: int, T: int) -> int:
    """4 * B * Hq * D * T(T+1)/2: QK^T and PV over the unmasked keys."""
    return 4 * B * Hq * D * T * (T + 1) // 2


def decode_lengths(seed: int = 0) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(CFG4["Lmin"], CFG4["Lmax"] + 1, (CFG4["B"],), generator=g).tolist()


class ClockSampler:
    """nvidia-smi sampling during the timed region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: str):
        self.proc = None
        self.gpus = gpus

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", self.gpus], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


class Dist:
    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}")
        self.pg = None

    def init(self):
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        return torch.device("cuda", self.local)

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def timed(fn, steps: int, warmup: int, dist: Dist, per_launch: bool = True):
    """Run fn() warmup times, then time `steps` calls. Returns (total_ms
    (max over ranks), mean per-call device ms on this rank)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(st)
    for i in range(steps):
        ev[i][0].record(st)
        fn()
        ev[i][1].record(st)
    t1.record(st)
    torch.cuda.synchronize()
    dist.barrier()
    total = t0.elapsed_time(t1)
    per = sum(a.elapsed_time(b) for a, b in ev) / steps
    return dist.max(total), per


# ----------------------------------------------------------------- our arm
def run_ours(a, dist: Dist) -> dict | None:
    from npu_b200 import api

    dev = dist.init()
    pk, pk_src = peaks()
    world, rank = dist.world, dist.rank
    B, Hq, Hkv, D = a.batch, CFG3["Hq"], CFG3["Hkv"], CFG3["D"]
    T = a.T
    scale = 1.0 / math.sqrt(D)
    b_lo, b_hi = rank * B // world, (rank + 1) * B // world
    Bl = b_hi - b_lo
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    q = torch.randn(Bl, Hq, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(Bl, Hkv, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(Bl, Hkv, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    o = torch.empty(Bl, Hq, T, D, device=dev, dtype=torch.bfloat16)

    def step():
        api.prefill(q, k, v, scale=scale, out=o, out_dtype=torch.bfloat16)

    gpus = ",".join(str(i) for i in range(world))
    sampler = ClockSampler(gpus) if (rank == 0 and "prefill" in a.legs) else None
    if sampler:
        sampler.__enter__()
    if "prefill" in a.legs:
        total_ms, per_ms = timed(step, a.steps, a.warmup, dist)
    else:
        total_ms = per_ms = float("nan")
    if sampler:
        sampler.__exit__(None, None, None)
    flops_all = prefill_flops(B, Hq, D, T)
    flops_rank = prefill_flops(Bl, Hq, D, T)
    value = flops_all * a.steps / (total_ms * 1e-3) / 1e12
    achieved = flops_rank / (per_ms * 1e-3) / 1e12
    peak = float(pk["bf16_tflops"])
    err = api.device_error()

    # End to end: pinned host buffers, H2D of q/k/v and D2H of o every step.
    e2e = None
    if a.e2e and "prefill" in a.legs:
        hq = q.cpu().pin_memory()
        hk = k.cpu().pin_memory()
        hv = v.cpu().pin_memory()
        ho = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)

        ws = torch.empty(api.prefill_host_workspace_bytes(Bl, Hq, Hkv, T, T, D), dtype=torch.uint8, device=dev)

        def e2e_step():
            # b2a_prefill_host: chunked H2D / kernel / D2H on three streams,
            # ordered on the current stream (timed by its events).
            api.prefill_host(hq, hk, hv, scale=scale, out=ho, out_dtype=torch.bfloat16, device=dev,
                             workspace=ws, sync=False)

        e_steps = max(1, min(a.steps, a.e2e_steps))
        e_total, _ = timed(e2e_step, e_steps, 1, dist)
        e2e = {"value": flops_all * e_steps / (e_total * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": (hq.numel() + hk.numel() + hv.numel()) * 2 * world,
               "d2h_bytes_per_step": ho.numel() * 2 * world, "steps": e_steps,
               "api": "npu_b200.prefill_host (C ABI b2a_prefill_host) with pinned host buffers"}
        del hq, hk, hv, ho, ws
    del q, k, v, o
    torch.cuda.empty_cache()

    sweep = []
    for Ts in (a.sweep if "sweep" in a.legs else []):
        qs = torch.randn(Bl, Hq, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        ks = torch.randn(Bl, Hkv, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        vs = torch.randn(Bl, Hkv, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        os_ = torch.empty(Bl, Hq, Ts, D, device=dev, dtype=torch.bfloat16)
        tot, per = timed(lambda: api.prefill(qs, ks, vs, scale=scale, out=os_, out_dtype=torch.bfloat16),
                         a.steps, a.warmup, dist)
        f = prefill_flops(B, Hq, D, Ts)
        sweep.append({"T": Ts, "value": f * a.steps / (tot * 1e-3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_step": tot / a.steps,
                      "frac_of_peak": (prefill_flops(Bl, Hq, D, Ts) / (per * 1e-3) / 1e12) / peak})
        del qs, ks, vs, os_
    torch.cuda.empty_cache()

    decode = run_decode(a, dist, dev, pk) if (a.decode and "decode" in a.legs) else None
    long_ctx = run_long_context(a, dist, dev, pk) if (a.long and "long" in a.legs) else None

    cpu = None
    if rank == 0 and world == 1 and a.cpu_baseline and "prefill" in a.legs:
        cpu = cpu_prefill_sample(T, a.cpu_units)

    if rank != 0:
        return None
    traffic = load_traffic("prefill_T%d" % T, B=Bl)
    line = {
        "metric": METRIC,
        "value_is": f"causal GQA prefill attention, algorithmic TFLOP/s, config 3 T={T}",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16, generated on device)",
        "config": {"workload": f"config3_causal_gqa_prefill_T{T}", "B": B, "Hq": Hq, "Hkv": Hkv, "D": D,
                   "T": T, "causal": True, "scale": scale, "out": "bf16",
                   "parallelism": f"dp{world} over (batch x kv_head), no collective",
                   "l2": "inputs larger than L2 (Q is %.1f GB)" % (B * Hq * T * D * 2 / 1e9)},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{pk_src} bf16_tflops (burst)",
                     "frac_of_sustained": achieved / float(pk.get("bf16_tflops_sustained", peak)),
                     "kernel": "fa_prefill_kernel<128>", "traffic": traffic,
                     "flops_per_launch": flops_rank, "launch_ms": per_ms},
        "e2e": e2e,
        "gpu_launches": a.steps,
        "clocks": sampler.summary() if sampler else None,
        "device_error": err,
        "sweep": sweep,
        "decode": decode,
        "long_context": long_ctx,
        "cpu_baseline": cpu,
    }
    return line


def run_decode(a, dist: Dist, dev, pk) -> dict:
    from npu_b200 import api

    from npu_b200.dist import shard_sequences

    lens = decode_lengths(0)[: a.decode_batch]
    mine = shard_sequences(lens, dist.world)[dist.rank]
    Bm, Hq, Hkv, D, Lmax = len(mine), CFG4["Hq"], CFG4["Hkv"], CFG4["D"], CFG4["Lmax"]
    g = torch.Generator(device=dev).manual_seed(2000 + dist.rank)
    q = torch.randn(Bm, Hq, D, device=dev, generator=g, dtype=torch.bfloat16)
    kc = torch.randn(Bm, Hkv, Lmax, D, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(Bm, Hkv, Lmax, D, device=dev, generator=g, dtype=torch.bfloat16)
    sl = torch.tensor([lens[i] for i in mine], dtype=torch.int32, device=dev)
    o = torch.empty(Bm, Hq, D, device=dev, dtype=torch.bfloat16)
    split = int(api._lib.load().b2a_decode_default_split(Bm, Hkv, Lmax))
    ws = torch.empty(api.decode_workspace_bytes(Bm, Hq, Hkv, D, Lmax, split), dtype=torch.uint8, device=dev)
    scale = 1.0 / math.sqrt(D)

    def step():
        api.decode(q, kc, vc, sl, scale=scale, out=o, workspace=ws, split_len=split)

    total_ms, per_ms = timed(step, a.steps, a.warmup, dist)
    kv_all = sum(lens) * Hkv * D * 2 * 2
    qo_all = len(lens) * Hq * D * 2 * 2
    kv_rank = sum(lens[i] for i in mine) * Hkv * D * 2 * 2 + Bm * Hq * D * 2 * 2
    value = (kv_all + qo_all) * a.steps / (total_ms * 1e-3) / 1e9
    achieved = kv_rank / (per_ms * 1e-3) / 1e9
    peak = float(pk["hbm_gbs"])
    del q, kc, vc, o, ws
    torch.cuda.empty_cache()
    return {"metric": "split-KV decode attention HBM GB/s (config 4)", "value": value, "unit": "GB/s",
            "ms_per_step": total_ms / a.steps, "split_len": split, "sum_len": sum(lens),
            "algorithmic_bytes_per_step": kv_all + qo_all, "gpu_launches": 2 * a.steps,
            "scaling": "strong", "parallelism": f"dp{dist.world} over sequences (greedy by length)",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "kernel": "decode_split_kernel<128> + decode_combine_kernel",
                         "traffic": load_traffic("decode_cfg4", keys=sum(lens[i] for i in mine)),
                         "launch_ms": per_ms}}


def run_long_context(a, dist: Dist, dev, pk) -> dict:
    """Config 5: one sequence of T=131072, 16 query / 2 KV heads, D=256, causal.
    One GPU runs it whole; N GPUs split the query rows zig-zag (rank g owns
    chunks g and 2N-1-g) and all-gather K/V with NCCL once per step."""
    from npu_b200 import api
    from npu_b200.dist import ContextParallelPrefill, causal_flops_rows

    T, Hq, Hkv, D = a.long_T, 16, 2, 256
    scale = 1.0 / 16
    world, rank = dist.world, dist.rank
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    rows = T if world == 1 else T // world
    q = torch.randn(1, Hq, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(1, Hkv, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(1, Hkv, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    if world == 1:
        o = torch.empty_like(q)

        def step():
            api.prefill(q, k, v, scale=scale, out=o, out_dtype=torch.bfloat16)

        mine = causal_flops_rows((0, T), D, Hq)
        launches = 1
    else:
        cp = ContextParallelPrefill(T, world, rank, group=None)

        def step():
            cp.run(q, k, v, scale=scale, out_dtype=torch.bfloat16)

        mine = sum(causal_flops_rows(c, D, Hq) for c in cp.chunks)
        launches = 2
    total_ms, per_ms = timed(step, a.steps, a.warmup, dist)
    flops = causal_flops_rows((0, T), D, Hq)
    peak = float(pk["bf16_tflops"])
    achieved = mine / (per_ms * 1e-3) / 1e12
    del q, k, v
    torch.cuda.empty_cache()
    return {"metric": "long-context causal prefill attention TFLOP/s (config 5)", "value":
            flops * a.steps / (total_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": total_ms / a.steps,
            "T": T, "Hq": Hq, "Hkv": Hkv, "D": D, "gpu_launches": launches * a.steps,
            "parallelism": "single GPU" if world == 1 else f"zig-zag context parallel x{world}, NCCL all-gather of K/V",
            "rank0_frac_of_peak": achieved / peak, "scaling": "strong",
            # Rank 0's algorithmic FLOPs over its step time: one kernel launch
            # at 1 GPU; at N GPUs the step also holds the K/V all-gather.
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": "measured bf16_tflops (burst)",
                         "frac_of_sustained": achieved / float(pk.get("bf16_tflops_sustained", peak)),
                         "kernel": "fa_prefill_d256_kernel", "traffic": None, "launch_ms": per_ms,
                         "flops_per_launch": mine}}


def load_traffic(key: str, **kw):
    """DRAM bytes per launch from the committed ncu summary (or None)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        entry = json.loads(p.read_text()).get(key)
    except Exception:
        return None
    if not entry:
        return None
    if "bytes_per_batch" in entry and "B" in kw:
        return entry["bytes_per_batch"] * kw["B"]
    if "bytes_per_key" in entry and "keys" in kw:
        return entry["bytes_per_key"] * kw["keys"]
    return entry.get("bytes_per_launch")


# ----------------------------------------------------------------- CPU arm
def cpu_unit_prefill(T: int, seed: int) -> float:
    """Dense fp32 attention of one (batch, KV group) unit of config 3 — the
    reference's CPU attention (smollm.py:222-234) — head by head to bound
    memory. Returns seconds."""
    from oracle.attention import dense_attention

    Hq, Hkv, D = CFG3["Hq"], CFG3["Hkv"], CFG3["D"]
    grp = Hq // Hkv
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, grp, T, D, generator=g).bfloat16()
    k = torch.randn(1, 1, T, D, generator=g).bfloat16()
    v = torch.randn(1, 1, T, D, generator=g).bfloat16()
    t0 = time.perf_counter()
    for h in range(grp):
        dense_attention(q[:, h:h + 1], k, v, causal=True, scale=1.0 / math.sqrt(D))
    return time.perf_counter() - t0


def cpu_prefill_sample(T: int, units: int) -> dict:
    cores = torch.get_num_threads()
    secs = sum(cpu_unit_prefill(T, 7 + u) for u in range(units))
    grp = CFG3["Hq"] // CFG3["Hkv"]
    f = prefill_flops(1, grp, CFG3["D"], T) * units
    return {"value": f / secs / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{units} (batch, kv-head) unit(s) of config 3 at T={T} ({grp} query heads each), "
                      f"dense fp32 torch attention (oracle restatement of smollm.py:222-234), {secs:.1f} s"}


def run_reference(a) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    T = a.T
    for w in range(a.warmup):
        cpu_unit_prefill(min(T, 2048), 100 + w)
    t_total = 0.0
    for s in range(a.steps):
        t_total += cpu_unit_prefill(T, 200 + s)
    grp = CFG3["Hq"] // CFG3["Hkv"]
    f = prefill_flops(1, grp, CFG3["D"], T) * a.steps
    value = f / t_total / 1e12
    sample = (f"each step: one (batch, kv-head) unit of config 3 at T={T} ({grp} query heads), dense fp32 "
              "torch attention on the host cores (oracle restatement of smollm.py:222-234)")
    return {"impl": "reference", "metric": METRIC,
            "value_is": f"causal GQA prefill attention, algorithmic TFLOP/s, config 3 T={T} (CPU sample)",
            "value": value, "unit": "TFLOP/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": t_total * 1e3 / a.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"config3_causal_gqa_prefill_T{T}", **CFG3, "T": T},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--T", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=CFG3["B"], help="config-3 batch (64; smaller only for profiling)")
    ap.add_argument("--decode-batch", type=int, default=CFG4["B"], help="config-4 sequences (128)")
    ap.add_argument("--legs", type=lambda s: set(x for x in s.split(",") if x),
                    default={"prefill", "sweep", "decode", "long"}, help="subset of prefill,sweep,decode,long")
    ap.add_argument("--sweep", type=lambda s: [int(x) for x in s.split(",") if x], default=[512, 2048])
    ap.add_argument("--no-decode", dest="decode", action="store_false")
    ap.add_argument("--no-long", dest="long", action="store_false")
    ap.add_argument("--long-T", type=int, default=131072)
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-units", type=int, default=2)
    a = ap.parse_args()
    if a.warmup < 3 and a.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if a.impl == "reference":
        line = run_reference(a)
        if line:
            print(json.dumps(line), flush=True)
        return
    dist = Dist(a.gpus)
    try:
        line = run_ours(a, dist)
    finally:
        dist.close()
    if line:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
