"""Per-op profiler for the B200 path, with the reference's interface
(npu/profiler.py:1-78: `PROF.enable()`, `with profile(name): ...`,
`PROF.report()`, `PROF.reset()`; zero cost when disabled).

The reference times each op with the host clock, which is what its
synchronous NPU dispatches take. Work here is asynchronous on a CUDA stream,
so a host clock would time the launches, not the kernels. Each `profile`
block therefore records a pair of CUDA events on the current stream (device
time between them, resolved lazily when the report is made, so timing adds no
synchronisation) and opens an NVTX range of the same name, which shows up in
Nsight Systems / Nsight Compute (`ncu --nvtx --nvtx-include <name>/`). The
host wall time of the block is kept as well; without a CUDA device only the
host time is recorded.

    from npu_b200.profiler import PROF, profile

    PROF.enable()
    with profile("attn"):
        out = npu_b200.prefill(q, k, v)
    PROF.report()          # per-op device ms, host ms, calls, share
"""
from __future__ import annotations

import time
from collections import defaultdict

import torch


class _Profiler:
    __slots__ = ("enabled", "nvtx", "_host_ns", "_cnt", "_pending", "_dev_ms")

    def __init__(self):
        self.enabled = False
        self.nvtx = True
        self._host_ns: dict[str, int] = defaultdict(int)
        self._cnt: dict[str, int] = defaultdict(int)
        self._pending: list = []          # (name, start event, end event)
        self._dev_ms: dict[str, float] = defaultdict(float)

    def enable(self, nvtx: bool = True):
        self.enabled = True
        self.nvtx = nvtx

    def disable(self):
        self.enabled = False

    def reset(self):
        self._host_ns.clear()
        self._cnt.clear()
        self._pending.clear()
        self._dev_ms.clear()

    def add(self, name: str, ns: int, events=None):
        self._host_ns[name] += ns
        self._cnt[name] += 1
        if events is not None:
            self._pending.append((name, events[0], events[1]))

    def _resolve(self) -> None:
        """Fold recorded event pairs into device milliseconds (waits for the
        last recorded event, once)."""
        if not self._pending:
            return
        self._pending[-1][2].synchronize()
        for name, e0, e1 in self._pending:
            self._dev_ms[name] += e0.elapsed_time(e1)
        self._pending.clear()

    def stats(self) -> dict:
        """{name: {"device_ms", "host_ms", "calls"}} (device_ms is None for ops
        recorded without a CUDA device)."""
        self._resolve()
        out = {}
        for name, ns in self._host_ns.items():
            out[name] = {"device_ms": self._dev_ms[name] if name in self._dev_ms else None,
                         "host_ms": ns / 1e6, "calls": self._cnt[name]}
        return out

    def report(self, total_label: str = "total") -> None:
        st = self.stats()
        if not st:
            print("[profiler] no samples recorded")
            return

        def key(v):
            return v["device_ms"] if v["device_ms"] is not None else v["host_ms"]

        rows = sorted(st.items(), key=lambda kv: -key(kv[1]))
        total = key(st[total_label]) if total_label in st else sum(key(v) for v in st.values())
        print(f"{'op':<24} {'device_ms':>10} {'host_ms':>10} {'calls':>7} {'ms/call':>10} {'%':>6}")
        for name, v in rows:
            ms = key(v)
            dev = f"{v['device_ms']:10.2f}" if v["device_ms"] is not None else f"{'-':>10}"
            pct = 100.0 * ms / total if total > 0 else 0.0
            print(f"{name:<24} {dev} {v['host_ms']:>10.2f} {v['calls']:>7d} {ms / v['calls']:>10.3f} {pct:>5.1f}%")


PROF = _Profiler()


class _TimerCM:
    __slots__ = ("name", "t0", "ev", "nvtx")

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        self.ev = None
        self.nvtx = PROF.nvtx and torch.cuda.is_available()
        # No timing events inside a CUDA graph capture: host time and NVTX only.
        if torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing():
            self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.ev[0].record()
        if self.nvtx:
            torch.cuda.nvtx.range_push(self.name)
        self.t0 = time.perf_counter_ns()
        return self

    def __exit__(self, *exc):
        dt = time.perf_counter_ns() - self.t0
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        if self.ev is not None:
            self.ev[1].record()
        PROF.add(self.name, dt, self.ev)
        return False


class _NoopCM:
    __slots__ = ()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NOOP = _NoopCM()


def profile(name: str):
    """Context manager timing the block under `name` when PROF is enabled."""
    return _TimerCM(name) if PROF.enabled else _NOOP
