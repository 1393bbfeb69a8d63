"""Benchmark of the B200 attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): causal GQA prefill attention throughput, algorithmic
TFLOP/s, on config 3 at T=8192 (B=64, Hq=32, Hkv=4, D=128, bf16, scale
1/sqrt(128)). Work is sharded by independent (batch x KV-head) units with no
collective, reported as weak scaling: every rank runs a full B=64 batch, so
the timed region (and the power regime it runs in) is the same at every N,
and `value` is all ranks' FLOPs over the slowest rank's time. A step is one
launch over the rank's batch.

Sub-lines in the same JSON object:
  sweep         config 3 at T=512 and T=2048 (weak, as the headline)
  decode        config 4: 128 sequences x one query token, lengths ~
                U[1024, 32768], HBM GB/s; weak (128 sequences per rank) with
                a `strong` sub-object that splits one 128-sequence batch
                across the ranks (greedy by length)
  long_context  config 5: one 131072-token sequence, D=256, 16/2 heads; zig-zag
                context parallel with an NCCL K/V all-gather when N > 1
                (strong scaling: one sequence)
  config1       SmolLM2 one-layer prefill attention (B=1, T=128, 9/3 heads,
                D=64), device and end-to-end timings beside the CPU
                restatements of fa_ref.py's flash_attention_ref and the dense
                attention (replicas only)
  chatbot       bench_chatbot.py's sweep on the B200 path (1 GPU): prefill,
                decode step and sustained decode at L = 16 .. 2048 with top-1
                against the CPU forward timed beside it
  config2       SmolLM2-135M 30-layer prefill forward at T=1024 on the GPU
                (fp32 and bf16 weights) with the top-1 token checked against
                the CPU forward, which is timed beside it; and one layer's
                attention through the reference's own call surface
                (NpuAttention(BR=32, BC=32, D=64).run_batch on host stacks)
                beside the CPU attention of smollm.py:222-234 (replicas only)
  e2e           the headline metric through npu_b200.prefill_host (C ABI
                b2a_prefill_host) with pinned host buffers, H2D of q/k/v and
                D2H of o inside every timed step; one B=64 batch split across
                the ranks; with a `roofline` against the host-link bandwidth
                measured in the same run with every rank copying at once

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
CFG5 = dict(T=131072, Hq=16, Hkv=2, D=256)
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


def decode_bytes(lens, Hq: int, Hkv: int, D: int) -> int:
    """K+V bytes of every cached key (counted once for the group of query
    heads that reads it) plus q and o, bf16."""
    return sum(lens) * Hkv * D * 2 * 2 + len(lens) * Hq * D * 2 * 2


def visible_gpu_ids(world: int) -> str:
    """nvidia-smi ids of the GPUs the ranks use (CUDA_VISIBLE_DEVICES order)."""
    vis = [x.strip() for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip()]
    return ",".join(vis[:world]) if len(vis) >= world else ",".join(str(i) for i in range(world))


class ClockSampler:
    """nvidia-smi sampling during the timed region (200 ms period), per GPU."""

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
        sm, mx, reasons, power = [], 0.0, set(), []
        per_gpu: dict[str, list] = {}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (getattr(self, "out", "") or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                clk = float(f[1])
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            sm.append(clk)
            per_gpu.setdefault(f[0], []).append(clk)
            try:
                power.append(float(f[3]))
            except ValueError:
                pass
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "per_gpu_sm_mhz": {k: statistics.median(v) for k, v in per_gpu.items()},
                "power_w_max": max(power) if power else None}


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


def timed(fn, steps: int, warmup: int, dist: Dist):
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


def host_link_bound(dist: Dist, dev, nbytes: int = 512 << 20, reps: int = 4) -> dict:
    """Pinned host<->device bandwidth with every rank copying at once (the
    e2e path's pattern), measured three ways: H2D alone, D2H alone, and both
    directions together. Rates are whole-job (all ranks) over the slowest
    rank's device time. `value` is the two-direction aggregate."""
    h_src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    h_dst = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    d_dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d_src = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    cur = torch.cuda.current_stream(dev)

    def once(h2d: bool, d2h: bool):
        up.wait_stream(cur)
        down.wait_stream(cur)
        if h2d:
            with torch.cuda.stream(up):
                d_dst.copy_(h_src, non_blocking=True)
        if d2h:
            with torch.cuda.stream(down):
                h_dst.copy_(d_src, non_blocking=True)
        cur.wait_stream(up)
        cur.wait_stream(down)

    rates = {}
    for name, h2d, d2h in (("both", True, True), ("h2d", True, False), ("d2h", False, True)):
        total_ms, _ = timed(lambda: once(h2d, d2h), reps, 1, dist)
        rates[name] = dist.world * (int(h2d) + int(d2h)) * nbytes * reps / (total_ms * 1e-3) / 1e9
    del h_src, h_dst, d_dst, d_src
    return {"value": rates["both"], "unit": "GB/s", "what": "pinned H2D + D2H at once on every rank, aggregate",
            "h2d_alone_gbs": rates["h2d"], "d2h_alone_gbs": rates["d2h"],
            "bytes_per_rank_per_direction": nbytes, "reps": reps, "ranks": dist.world}


def host_link_time_s(link: dict, h2d_bytes: float, d2h_bytes: float) -> float:
    """Least time the host link needs for a step's copies (whole job): each
    direction at most at its rate alone, both together at most at the
    two-direction aggregate."""
    return max(h2d_bytes / (link["h2d_alone_gbs"] * 1e9), d2h_bytes / (link["d2h_alone_gbs"] * 1e9),
               (h2d_bytes + d2h_bytes) / (link["value"] * 1e9))


# ----------------------------------------------------------------- our arm
def run_ours(a, dist: Dist) -> dict | None:
    from npu_b200 import api

    dev = dist.init()
    pk, pk_src = peaks()
    world, rank = dist.world, dist.rank
    B, Hq, Hkv, D = a.batch, CFG3["Hq"], CFG3["Hkv"], CFG3["D"]
    T = a.T
    scale = 1.0 / math.sqrt(D)
    peak = float(pk["bf16_tflops"])
    # Weak scaling: every rank runs its own full config-3 batch.
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    q = torch.randn(B, Hq, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(B, Hkv, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(B, Hkv, T, D, device=dev, generator=g, dtype=torch.bfloat16)
    o = torch.empty(B, Hq, T, D, device=dev, dtype=torch.bfloat16)

    def step():
        api.prefill(q, k, v, scale=scale, out=o, out_dtype=torch.bfloat16)

    sampler = ClockSampler(visible_gpu_ids(world)) if (rank == 0 and "prefill" in a.legs) else None
    if sampler:
        sampler.__enter__()
    if "prefill" in a.legs:
        total_ms, per_ms = timed(step, a.steps, a.warmup, dist)
    else:
        total_ms = per_ms = float("nan")
    if sampler:
        sampler.__exit__(None, None, None)
    flops_rank = prefill_flops(B, Hq, D, T)
    value = world * flops_rank * a.steps / (total_ms * 1e-3) / 1e12
    achieved = flops_rank / (per_ms * 1e-3) / 1e12
    err = api.device_error()
    del q, k, v, o
    torch.cuda.empty_cache()

    e2e = run_e2e(a, dist, dev) if (a.e2e and "prefill" in a.legs) else None

    sweep = []
    for Ts in (a.sweep if "sweep" in a.legs else []):
        qs = torch.randn(B, Hq, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        ks = torch.randn(B, Hkv, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        vs = torch.randn(B, Hkv, Ts, D, device=dev, generator=g, dtype=torch.bfloat16)
        os_ = torch.empty(B, Hq, Ts, D, device=dev, dtype=torch.bfloat16)
        tot, per = timed(lambda: api.prefill(qs, ks, vs, scale=scale, out=os_, out_dtype=torch.bfloat16),
                         a.steps, a.warmup, dist)
        f = prefill_flops(B, Hq, D, Ts)
        entry = {"T": Ts, "value": world * f * a.steps / (tot * 1e-3) / 1e12, "unit": "TFLOP/s",
                 "ms_per_step": tot / a.steps, "scaling": "weak",
                 "frac_of_peak": (f / (per * 1e-3) / 1e12) / peak}
        if rank == 0 and world == 1 and a.cpu_baseline:
            # T=512: the whole batch (every (batch, KV head) unit); longer: a sample
            entry["cpu_baseline"] = cpu_prefill_sample(Ts, B * Hkv if Ts <= 512 else a.cpu_units)
        sweep.append(entry)
        del qs, ks, vs, os_
    torch.cuda.empty_cache()

    decode = run_decode(a, dist, dev, pk) if "decode" in a.legs else None
    long_ctx = run_long_context(a, dist, dev, pk) if "long" in a.legs else None
    cfg1 = run_config1(a, dist, dev) if "config1" in a.legs else None
    cfg2 = run_config2(a, dist, dev) if "config2" in a.legs else None
    chat = run_chatbot(a, dist, dev) if "chatbot" in a.legs else None

    cpu = None
    if rank == 0 and world == 1 and a.cpu_baseline and "prefill" in a.legs:
        cpu = cpu_prefill_sample(T, a.cpu_units)

    if rank != 0:
        return None
    traffic = load_traffic("prefill_T%d" % T, B=B)
    line = {
        "metric": METRIC,
        "value_is": f"causal GQA prefill attention, algorithmic TFLOP/s, config 3 T={T}, all ranks",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": total_ms / a.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16, generated on device)",
        "config": {"workload": f"config3_causal_gqa_prefill_T{T}", "B_per_rank": B, "B_total": B * world,
                   "Hq": Hq, "Hkv": Hkv, "D": D, "T": T, "causal": True, "scale": scale, "out": "bf16",
                   "parallelism": f"dp{world} over (batch x kv_head) units, no collective, B={B} per rank",
                   "l2": "inputs larger than L2 (Q is %.1f GB per rank)" % (B * Hq * T * D * 2 / 1e9)},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": f"{pk_src} bf16_tflops (burst)",
                     "frac_of_sustained": achieved / float(pk.get("bf16_tflops_sustained", peak)),
                     "kernel": "fa_prefill_kernel<128, 2, false>", "traffic": traffic,
                     "flops_per_launch": flops_rank, "launch_ms": per_ms},
        "e2e": e2e,
        "gpu_launches": a.steps,
        "clocks": sampler.summary() if sampler else None,
        "device_error": err,
        "sweep": sweep,
        "decode": decode,
        "long_context": long_ctx,
        "config1": cfg1,
        "config2": cfg2,
        "chatbot": chat,
        "cpu_baseline": cpu,
    }
    return line


def run_e2e(a, dist: Dist, dev) -> dict:
    """Config 3 through the host-buffer entry point: one B=64 batch split
    across the ranks by (batch x KV head) units, pinned host q/k/v/o, every
    copy inside the timed steps; roofline against the host link measured
    here with all ranks copying at once."""
    from npu_b200 import api

    world, rank = dist.world, dist.rank
    B, Hq, Hkv, D, T = a.batch, CFG3["Hq"], CFG3["Hkv"], CFG3["D"], a.T
    link = host_link_bound(dist, dev)
    b_lo, b_hi = rank * B // world, (rank + 1) * B // world
    Bl = b_hi - b_lo
    g = torch.Generator().manual_seed(4000 + rank)
    hq = torch.randn(Bl, Hq, T, D, generator=g, dtype=torch.bfloat16).pin_memory()
    hk = torch.randn(Bl, Hkv, T, D, generator=g, dtype=torch.bfloat16).pin_memory()
    hv = torch.randn(Bl, Hkv, T, D, generator=g, dtype=torch.bfloat16).pin_memory()
    ho = torch.empty((Bl, Hq, T, D), dtype=torch.bfloat16, pin_memory=True)
    ws = torch.empty(api.prefill_host_workspace_bytes(Bl, Hq, Hkv, T, T, D), dtype=torch.uint8, device=dev)
    scale = 1.0 / math.sqrt(D)

    def e2e_step():
        # b2a_prefill_host: chunked H2D / kernel / D2H on three streams,
        # ordered on the current stream (timed by its events).
        api.prefill_host(hq, hk, hv, scale=scale, out=ho, out_dtype=torch.bfloat16, device=dev,
                         workspace=ws, sync=False)

    steps = max(1, min(a.steps, a.e2e_steps))
    total, _ = timed(e2e_step, steps, max(1, min(a.warmup, 3)), dist)
    h2d = (B * Hq * T * D + 2 * B * Hkv * T * D) * 2
    d2h = B * Hq * T * D * 2
    step_s = total / steps * 1e-3
    moved = (h2d + d2h) / step_s / 1e9
    # The copies' own lower bound for this byte mix (more H2D than D2H), as
    # an effective rate: achieved / peak = bound time / step time.
    link_peak = (h2d + d2h) / host_link_time_s(link, h2d, d2h) / 1e9
    del hq, hk, hv, ho, ws
    return {"value": prefill_flops(B, Hq, D, T) * steps / (total * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps, "ms_per_step": total / steps,
            "work": f"one config-3 batch (B={B}, T={T}) split across {world} rank(s)",
            "api": "npu_b200.prefill_host (C ABI b2a_prefill_host) with pinned host buffers",
            "roofline": {"bound": "host_link", "achieved": moved, "peak": link_peak, "unit": "GB/s",
                         "frac": moved / link_peak, "peak_source": link,
                         "peak_is": "step bytes over max(H2D bytes / H2D-alone rate, D2H bytes / D2H-alone "
                                    "rate, all bytes / both-directions rate), rates measured in this run"}}


def run_decode(a, dist: Dist, dev, pk) -> dict:
    """Config 4. Weak: every rank decodes all 128 sequences (its own data).
    Strong: the same 128 lengths split across the ranks by length."""
    from npu_b200 import api
    from npu_b200.dist import shard_sequences

    lens = decode_lengths(0)[: a.decode_batch]
    Hq, Hkv, D, Lmax = CFG4["Hq"], CFG4["Hkv"], CFG4["D"], CFG4["Lmax"]
    scale = 1.0 / math.sqrt(D)
    g = torch.Generator(device=dev).manual_seed(2000 + dist.rank)
    Bm = len(lens)
    q = torch.randn(Bm, Hq, D, device=dev, generator=g, dtype=torch.bfloat16)
    kc = torch.randn(Bm, Hkv, Lmax, D, device=dev, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(Bm, Hkv, Lmax, D, device=dev, generator=g, dtype=torch.bfloat16)
    o = torch.empty(Bm, Hq, D, device=dev, dtype=torch.bfloat16)
    peak = float(pk["hbm_gbs"])

    def measure(idx):
        n = len(idx)
        sl = torch.tensor([lens[i] for i in idx], dtype=torch.int32, device=dev)
        qi, ki, vi, oi = (q[:n], kc[:n], vc[:n], o[:n])
        split = int(api._lib.load().b2a_decode_default_split(n, Hkv, Lmax))
        ws = torch.empty(api.decode_workspace_bytes(n, Hq, Hkv, D, Lmax, split), dtype=torch.uint8, device=dev)

        def call():
            api.decode(qi, ki, vi, sl, scale=scale, out=oi, workspace=ws, split_len=split)

        # A decode step is replayed from a CUDA graph (its two launches, as a
        # serving loop captures its decode step): at 16 sequences per GPU the
        # kernels take ~0.09 ms, less than the Python call that enqueues them.
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            call()
        total_ms, per_ms = timed(graph.replay, a.steps, a.warmup, dist)
        del graph
        return total_ms, per_ms, split, decode_bytes([lens[i] for i in idx], Hq, Hkv, D)

    tot_w, per_w, split_w, bytes_rank = measure(list(range(Bm)))
    mine = shard_sequences(lens, dist.world)[dist.rank]
    tot_s, per_s, split_s, bytes_mine = measure(mine)
    bytes_all = decode_bytes(lens, Hq, Hkv, D)
    achieved = bytes_rank / (per_w * 1e-3) / 1e9

    # End to end through the public call: every step uploads this step's
    # query (pinned host -> device), decodes against the device-resident
    # caches and downloads the output; copies and kernels on one stream.
    hq = q.cpu().pin_memory()
    ho = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
    sl_all = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws_e = torch.empty(api.decode_workspace_bytes(Bm, Hq, Hkv, D, Lmax, split_w), dtype=torch.uint8, device=dev)

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        api.decode(q, kc, vc, sl_all, scale=scale, out=o, workspace=ws_e, split_len=split_w)
        ho.copy_(o, non_blocking=True)

    tot_e, _ = timed(e2e_step, a.steps, a.warmup, dist)
    e2e = {"value": dist.world * bytes_rank * a.steps / (tot_e * 1e-3) / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": hq.numel() * 2 * dist.world, "d2h_bytes_per_step": ho.numel() * 2 * dist.world,
           "ms_per_step": tot_e / a.steps,
           "api": "npu_b200.decode with the query uploaded from and the output read back to pinned host memory "
                  "every step (caches resident on the device)"}
    del hq, ho, ws_e
    del q, kc, vc, o
    torch.cuda.empty_cache()
    cpu = None
    if dist.rank == 0 and dist.world == 1 and a.cpu_baseline:
        cpu = cpu_decode_sample(lens, a.cpu_decode_seqs)
    return {"metric": "split-KV decode attention HBM GB/s (config 4)",
            "value": dist.world * bytes_rank * a.steps / (tot_w * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": tot_w / a.steps, "split_len": split_w, "sum_len": sum(lens),
            "algorithmic_bytes_per_step_per_rank": bytes_rank, "gpu_launches": 4 * a.steps, "scaling": "weak",
            "step": "the decode call (split + combine kernels) replayed from a CUDA graph",
            "parallelism": f"dp{dist.world}, 128 sequences per rank, no collective",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "kernel": "decode_split_kernel<128> + decode_combine_kernel",
                         "traffic": load_traffic("decode_cfg4", keys=sum(lens)), "launch_ms": per_w},
            "strong": {"value": bytes_all * a.steps / (tot_s * 1e-3) / 1e9, "unit": "GB/s",
                       "ms_per_step": tot_s / a.steps, "split_len_rank0": split_s,
                       "sequences_rank0": len(mine), "scaling": "strong",
                       "parallelism": f"128 sequences over {dist.world} rank(s), greedy by length",
                       "rank0_frac_of_peak": bytes_mine / (per_s * 1e-3) / 1e9 / peak},
            "e2e": e2e, "cpu_baseline": cpu}


def run_long_context(a, dist: Dist, dev, pk) -> dict:
    """Config 5: one sequence of T=131072, 16 query / 2 KV heads, D=256, causal.
    One GPU runs it whole; N GPUs split the query rows zig-zag (rank g owns
    chunks g and 2N-1-g) and all-gather K/V with NCCL once per step."""
    from npu_b200 import api
    from npu_b200.dist import ContextParallelPrefill, causal_flops_rows

    T, Hq, Hkv, D = a.long_T, CFG5["Hq"], CFG5["Hkv"], CFG5["D"]
    scale = 1.0 / 16
    world, rank = dist.world, dist.rank
    g = torch.Generator(device=dev).manual_seed(3000 + rank)
    rows = T if world == 1 else T // world
    q = torch.randn(1, Hq, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(1, Hkv, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(1, Hkv, rows, D, device=dev, generator=g, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    if world == 1:
        def step():
            api.prefill(q, k, v, scale=scale, out=o, out_dtype=torch.bfloat16)

        mine = causal_flops_rows((0, T), D, Hq)
        launches = 1
    else:
        cp = ContextParallelPrefill(T, world, rank, group=None)

        def step():
            cp.run(q, k, v, scale=scale, out=o, out_dtype=torch.bfloat16)

        mine = sum(causal_flops_rows(c, D, Hq) for c in cp.chunks)
        launches = cp.launches_per_run
    total_ms, per_ms = timed(step, a.steps, a.warmup, dist)
    flops = causal_flops_rows((0, T), D, Hq)
    peak = float(pk["bf16_tflops"])
    achieved = mine / (per_ms * 1e-3) / 1e12
    del q, k, v, o
    torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and a.cpu_baseline:
        cpu = cpu_long_sample(T, a.cpu_long_blocks)
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
                         "kernel": "fa_prefill_d256_kernel",
                         "traffic": load_traffic("long_T%d" % T) if world == 1 else None,
                         "launch_ms": per_ms, "flops_per_launch": mine},
            "cpu_baseline": cpu}


def run_config1(a, dist: Dist, dev) -> dict:
    """Config 1: SmolLM2 one-layer causal prefill attention, B=1, T=128, 9/3
    heads, D=64, scale 1/8, fp32 output. Launch-latency bound; timed on the
    device and end to end (host q/k/v in, host o out)."""
    from npu_b200 import api

    g = torch.Generator().manual_seed(0)
    qh = torch.randn(1, 9, 128, 64, generator=g).bfloat16()
    kh = torch.randn(1, 3, 128, 64, generator=g).bfloat16()
    vh = torch.randn(1, 3, 128, 64, generator=g).bfloat16()
    q, k, v = qh.to(dev), kh.to(dev), vh.to(dev)
    o = torch.empty(1, 9, 128, 64, device=dev)
    f = prefill_flops(1, 9, 64, 128)
    reps = 50 * a.steps
    tot, per = timed(lambda: api.prefill(q, k, v, scale=0.125, out=o), reps, max(a.warmup, 10), dist)
    # The same launches replayed from a CUDA graph (no host work between
    # them): the kernel's own time per launch.
    n_graph = 50
    for _ in range(3):
        api.prefill(q, k, v, scale=0.125, out=o)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(n_graph):
            api.prefill(q, k, v, scale=0.125, out=o)
    tot_g, _ = timed(graph.replay, a.steps, a.warmup, dist)
    per_graph = tot_g / (a.steps * n_graph)
    del graph
    qp, kp, vp = qh.pin_memory(), kh.pin_memory(), vh.pin_memory()
    op = torch.empty(1, 9, 128, 64, pin_memory=True)

    def e2e_step():
        api.prefill_host(qp, kp, vp, scale=0.125, out=op, out_dtype=torch.float32, device=dev, sync=False)

    tot_e, _ = timed(e2e_step, reps, max(a.warmup, 10), dist)
    line = {"workload": "config1 SmolLM2 one-layer prefill attention, B=1, T=128, 9/3 heads, D=64",
            "parallelism": "replicas only (too small to shard)", "flops": f,
            "device_us_per_launch": per * 1e3, "device_tflops": f / (per * 1e-3) / 1e12,
            "graph_us_per_launch": per_graph * 1e3, "graph_tflops": f / (per_graph * 1e-3) / 1e12,
            "note": "eager launches are bound by host-side call overhead; the graph replay shows the kernel",
            "e2e_us_per_call": tot_e / reps * 1e3, "e2e_api": "npu_b200.prefill_host (pinned host buffers)",
            "gpu_launches": 2 * reps + n_graph * a.steps}
    if dist.rank == 0 and dist.world == 1 and a.cpu_baseline:
        line["cpu_baseline"] = cpu_config1(qh, kh, vh)
    return line


def run_config2(a, dist: Dist, dev) -> dict:
    """Config 2: SmolLM2-135M, 30 layers, T=1024, seeded N(0, 0.02) weights
    (norm weights 1), ids uniform over the vocab (seed 1). The B200 forward
    (fused QKV GEMM, rope + cache append kernel, prefill kernel) in fp32 and
    bf16, top-1 at position T-1 against the CPU forward of the reference's
    layer (fp32, CPU attention); and one layer's attention through the
    reference call surface with host stacks."""
    from npu_b200 import NpuAttention
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig
    from oracle.smollm_ref import Config, SmolLM, make_state_dict

    cfg = Config()
    T = 1024
    ids = torch.randint(0, cfg.vocab, (1, T), generator=torch.Generator().manual_seed(1))
    sd = make_state_dict(cfg, seed=0)
    out = {"workload": "config2 SmolLM2-135M 30-layer prefill forward, T=1024, random-init weights",
           "parallelism": "replicas only (too small to shard)",
           "attention_flops_per_forward": 30 * prefill_flops(1, 9, 64, T)}
    fwd = {}
    for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        model = SmolLMB200(sd, SmolLMConfig(), dev, dtype=dt)
        cache = model.new_cache(batch=1, max_len=T)
        ids_d = ids.to(dev)

        def step():
            cache.reset()
            return model.forward(ids_d, cache)

        tot, per = timed(step, a.steps, a.warmup, dist)
        logits = step()[0, -1].float().cpu()
        cache.reset()
        graph_step = model.capture_prefill(cache, T)
        tot_g, per_g = timed(lambda: (cache.reset(), graph_step(ids_d)), a.steps, a.warmup, dist)
        g_logits = graph_step(ids_d)[0, -1].float().cpu()
        fwd[name] = {"ms_per_forward": per, "tokens_per_s": T / (per * 1e-3), "top1": int(logits.argmax()),
                     "graph_ms_per_forward": per_g, "graph_top1": int(g_logits.argmax()),
                     "gpu_launches_per_forward": 30 * 2}
        del model, cache, graph_step
    out["forward_gpu"] = fwd
    # One layer's attention through run_batch with the reference's own
    # object and stacks (model on the host): q/k/v as layer 0 produces them.
    attn = NpuAttention(BR=32, BC=32, D=64, n_cores=4)  # smollm.py:318
    g = torch.Generator().manual_seed(2)
    q = torch.randn(1, 9, T, 64, generator=g)
    kx = torch.randn(1, 3, T, 64, generator=g).repeat_interleave(3, dim=1)
    vx = torch.randn(1, 3, T, 64, generator=g).repeat_interleave(3, dim=1)
    n_q = T // 32
    Q = q.view(1, 9, n_q, 32, 64).reshape(9 * n_q, 32, 64).contiguous()
    K = kx.unsqueeze(2).expand(1, 9, n_q, T, 64).reshape(9 * n_q, T, 64).contiguous()
    V = vx.unsqueeze(2).expand(1, 9, n_q, T, 64).reshape(9 * n_q, T, 64).contiguous()
    rows = [i * 32 for _ in range(9) for i in range(n_q)]
    for _ in range(max(a.warmup, 2)):
        attn.run_batch(Q, K, V, rows)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        attn.run_batch(Q, K, V, rows)
    rb_ms = (time.perf_counter() - t0) * 1e3 / a.steps
    out["run_batch_layer"] = {
        "what": "one layer's attention, NpuAttention(BR=32, BC=32, D=64).run_batch on the host stacks "
                "smollm.py:157-161 builds (288 blocks, K/V duplicated per block), host result",
        "ms_per_call_wall": rb_ms, "h2d_bytes_per_call": 3 * 9 * T * 64 * 2, "d2h_bytes_per_call": 9 * T * 64 * 2,
        "note": "wall clock on the host (the call synchronises); K/V uploaded once per (batch, head)"}
    if dist.rank == 0 and dist.world == 1 and a.cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        ref = SmolLM(sd, cfg)
        t0 = time.perf_counter()
        ref_logits, _ = ref.forward(ids)
        cpu_fwd = time.perf_counter() - t0
        ref_top1 = int(ref_logits[0, -1].argmax())
        out["cpu_baseline"] = {"ms_per_forward": cpu_fwd * 1e3, "tokens_per_s": T / cpu_fwd, "top1": ref_top1,
                               "cores": torch.get_num_threads(), "kind": "port",
                               "sample": "one full 30-layer T=1024 forward, fp32, CPU attention "
                                         "(restatement of smollm.py:168-253)"}
        for name in fwd:
            fwd[name]["top1_matches_cpu"] = fwd[name]["top1"] == ref_top1
        t0 = time.perf_counter()
        for _ in range(3):
            att = torch.matmul(q, kx.transpose(-2, -1)) / 8.0
            att = att + torch.triu(torch.full((T, T), float("-inf")), diagonal=1)
            torch.matmul(torch.softmax(att.float(), dim=-1), vx)
        out["cpu_baseline"]["attention_layer_ms"] = (time.perf_counter() - t0) * 1e3 / 3
    return out


def run_chatbot(a, dist: Dist, dev) -> dict | None:
    """The reference's chatbot benchmark (bench_chatbot.py:61-136) on the B200
    path: at each context length L, top-1 at position L-1 against the CPU
    forward (correctness first), prefill latency, one decode step with the
    context at L, and sustained greedy decode tok/s over `decode_n` tokens
    (the decode step replayed as one CUDA graph). SmolLM2-135M with seeded
    random weights (no checkpoint offline), fp32 as the reference's NPU
    configuration; prompts as bench_chatbot.py:29-32 (seed 12345 + L). The CPU
    side is the reference's layer restated (oracle), timed on all host cores,
    up to `chatbot_cpu_max_L`. One GPU only (replicas would add nothing)."""
    if dist.world != 1:
        return None
    from npu_b200.smollm_b200 import SmolLMB200, SmolLMConfig
    from oracle.smollm_ref import Config, SmolLM, make_state_dict

    torch.set_num_threads(os.cpu_count() or 1)
    cfg = Config()
    sd = make_state_dict(cfg, seed=0)
    gpu = SmolLMB200(sd, SmolLMConfig(), dev)
    cpu = SmolLM(sd, cfg) if a.cpu_baseline else None
    n = a.chatbot_decode_n
    rows = []

    def dev_ms(fn, iters):
        ts = []
        for _ in range(iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    def wall_ms(fn, iters):
        ts = []
        for _ in range(iters):
            t0 = time.perf_counter()
            fn()
            ts.append((time.perf_counter() - t0) * 1e3)
        return statistics.median(ts)

    for L in a.chatbot_lengths:
        ids = torch.randint(0, min(cfg.vocab, 32000), (1, L), generator=torch.Generator().manual_seed(12345 + L))
        ids_d = ids.to(dev)
        cache = gpu.new_cache(batch=1, max_len=L + n + 8)

        def prefill():
            cache.reset()
            return gpu.forward(ids_d, cache)

        logits = prefill()[0, -1].float().cpu()
        prefill()
        p_ms = dev_ms(prefill, a.steps)
        prefill()
        nxt = ids_d[:, -1:]
        saved = cache._pos.clone()

        def step():
            cache._pos.copy_(saved)
            return gpu.forward(nxt, cache)

        step()
        s_ms = dev_ms(step, a.steps)
        cache._pos.copy_(saved)
        graph_step = gpu.capture_decode(cache)

        def decode_n():
            cache._pos.copy_(saved)
            tok = nxt
            for _ in range(n):
                tok = graph_step(tok)[:, -1].argmax(-1, keepdim=True)

        decode_n()
        d_ms = dev_ms(decode_n, max(1, a.steps // 2))
        row = {"L": L, "prefill_ms": p_ms, "step_ms": s_ms, "decode_tok_s": n / (d_ms * 1e-3),
               "top1": int(logits.argmax())}
        del graph_step
        if cpu is not None and L <= a.chatbot_cpu_max_L:
            with torch.no_grad():
                ref_logits, ref_cache = cpu.forward(ids)
            ref = ref_logits[0, -1]
            row["top1_matches_cpu"] = int(ref.argmax()) == row["top1"]
            row["max_logit_delta"] = (logits - ref).abs().max().item()
            it = 1 if L >= 1024 else 2
            row["cpu_prefill_ms"] = wall_ms(lambda: cpu.forward(ids), it)
            nid = ids[:, -1:]
            row["cpu_step_ms"] = wall_ms(lambda: cpu.forward(nid, cache=ref_cache, start_pos=L), 3)

            def cpu_decode():
                c, tok, pos = ref_cache, nid, L
                for _ in range(n):
                    lg, c = cpu.forward(tok, cache=c, start_pos=pos)
                    tok = lg[:, -1].argmax(-1, keepdim=True)
                    pos += 1

            row["cpu_decode_tok_s"] = n / (wall_ms(cpu_decode, 1) * 1e-3)
        rows.append(row)
        del cache
    torch.cuda.empty_cache()
    out = {"what": "bench_chatbot.py on the B200 path: TTFT (prefill), inter-token step, sustained greedy "
                   "decode (CUDA graph per step), top-1 against the CPU forward",
           "model": "SmolLM2-135M, seeded random weights, fp32", "decode_n": n, "rows": rows}
    if cpu is not None:
        checked = [r for r in rows if "top1_matches_cpu" in r]
        out["correctness"] = f"{sum(r['top1_matches_cpu'] for r in checked)}/{len(checked)} lengths match top-1"
        out["cpu_cores"] = torch.get_num_threads()
    return out


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


def cpu_decode_sample(lens, n_seq: int) -> dict:
    """Config 4 on the host: the reference's single-token attention per
    sequence (smollm.py:205-234 with T=1: repeat_interleave of the KV heads,
    scores, fp32 softmax, weighted sum) over the first n_seq sequences'
    caches, in the model's fp32 (caches upcast once, outside the timing)."""
    Hq, Hkv, D = CFG4["Hq"], CFG4["Hkv"], CFG4["D"]
    grp = Hq // Hkv
    sel = lens[:n_seq]
    g = torch.Generator().manual_seed(77)
    cases = [(torch.randn(Hq, 1, D, generator=g).bfloat16().float(),
              torch.randn(Hkv, L, D, generator=g).bfloat16().float(),
              torch.randn(Hkv, L, D, generator=g).bfloat16().float()) for L in sel]
    t0 = time.perf_counter()
    for q, k, v in cases:
        ke, ve = k.repeat_interleave(grp, dim=0), v.repeat_interleave(grp, dim=0)
        s = torch.matmul(q, ke.transpose(-2, -1)) / math.sqrt(D)   # [Hq, 1, L]
        torch.matmul(torch.softmax(s.float(), dim=-1), ve)
    secs = time.perf_counter() - t0
    return {"value": decode_bytes(sel, Hq, Hkv, D) / secs / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n_seq} of the 128 config-4 sequences (sum L = {sum(sel)}), dense fp32 "
                                      f"attention per sequence (smollm.py:205-234 at T=1), {secs:.2f} s; bytes "
                                      "counted as the GPU's (bf16 K/V once per KV head)"}


def cpu_long_sample(T: int, blocks: int) -> dict:
    """Config 5 on the host: `blocks` 128-row query blocks spread over the
    sequence, each against its whole causal prefix, dense fp32 (the CPU path
    of smollm.py:222-234 restricted to the sampled rows); extrapolated as
    TFLOP/s over the sampled rows' causal FLOPs."""
    Hq, Hkv, D = CFG5["Hq"], CFG5["Hkv"], CFG5["D"]
    grp = Hq // Hkv
    g = torch.Generator().manual_seed(88)
    k = torch.randn(Hkv, T, D, generator=g).bfloat16().float()
    v = torch.randn(Hkv, T, D, generator=g).bfloat16().float()
    starts = [((2 * i + 1) * T) // (2 * blocks) // 128 * 128 for i in range(blocks)]
    qs = [torch.randn(Hkv, grp, 128, D, generator=g).bfloat16().float() for _ in starts]
    flops = 0
    t0 = time.perf_counter()
    for s0, q in zip(starts, qs):
        P = s0 + 128
        for h in range(Hkv):
            s = torch.matmul(q[h], k[h, :P].T) / 16.0                        # [grp, 128, P]
            mask = torch.arange(P)[None, :] > (torch.arange(128)[:, None] + s0)
            s.masked_fill_(mask, float("-inf"))
            torch.matmul(torch.softmax(s, dim=-1), v[h, :P])
        flops += 4 * Hq * D * sum(s0 + r + 1 for r in range(128))
    secs = time.perf_counter() - t0
    return {"value": flops / secs / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{blocks} query blocks of 128 rows at positions {starts} of T={T}, each against its "
                      f"full causal prefix, dense fp32 (smollm.py:222-234), {secs:.1f} s"}


def cpu_config1(q, k, v) -> dict:
    """Config 1 on the host: the oracle's dense attention (smollm.py:222-234,
    npu/fa_ref.py:134-145) and its flash_attention_ref restatement
    (npu/fa_ref.py:42-131, Br = Bc = 32) on the same bf16 inputs."""
    from oracle.attention import dense_attention, expand_kv, flash_attention_ref

    torch.set_num_threads(os.cpu_count() or 1)
    reps = 50
    dense_attention(q, k, v, scale=0.125)
    t0 = time.perf_counter()
    for _ in range(reps):
        dense_attention(q, k, v, scale=0.125)
    dense_ms = (time.perf_counter() - t0) * 1e3 / reps
    ke, ve = expand_kv(k, 3), expand_kv(v, 3)
    t0 = time.perf_counter()
    for _ in range(5):
        flash_attention_ref(q, ke, ve, Br=32, Bc=32, causal=True, scale=0.125)
    fa_ms = (time.perf_counter() - t0) * 1e3 / 5
    return {"dense_ms": dense_ms, "flash_attention_ref_ms": fa_ms, "cores": torch.get_num_threads(),
            "kind": "port", "sample": "whole config-1 problem, fp32 on the host"}


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
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"config3_causal_gqa_prefill_T{T}", **CFG3, "T": T, "causal": True,
                       "scale": 1.0 / math.sqrt(CFG3["D"]), "out": "f32"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


ALL_LEGS = {"prefill", "sweep", "decode", "long", "config1", "config2", "chatbot"}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--T", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=CFG3["B"], help="config-3 batch per rank (64)")
    ap.add_argument("--decode-batch", type=int, default=CFG4["B"], help="config-4 sequences (128)")
    ap.add_argument("--legs", type=lambda s: set(x for x in s.split(",") if x), default=set(ALL_LEGS),
                    help="subset of " + ",".join(sorted(ALL_LEGS)))
    ap.add_argument("--sweep", type=lambda s: [int(x) for x in s.split(",") if x], default=[512, 2048])
    ap.add_argument("--long-T", type=int, default=CFG5["T"])
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-units", type=int, default=2)
    ap.add_argument("--cpu-decode-seqs", type=int, default=16)
    ap.add_argument("--cpu-long-blocks", type=int, default=4)
    ap.add_argument("--chatbot-lengths", type=lambda s: [int(x) for x in s.split(",") if x],
                    default=[16, 64, 256, 1024, 2048])
    ap.add_argument("--chatbot-decode-n", type=int, default=16)
    ap.add_argument("--chatbot-cpu-max-L", type=int, default=2048)
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
