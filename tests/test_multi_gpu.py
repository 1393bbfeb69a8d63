"""Multi-GPU paths on real GPUs (skipped with fewer than 2): the zig-zag
context-parallel prefill with its NCCL K/V all-gather, and batch sharding.
Each rank checks the rows it owns against the fp32 oracle (sampled at every
chunk edge) and against the single-GPU kernel on the same inputs. The test
runs on every GPU the box has (2 to 8 ranks), with NVLS off."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TOL = 2e-2
T_CP = 16384  # divisible by 2 * world for world = 2..8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, result):
    import datetime

    import torch.distributed as dist

    from npu_b200 import api
    from npu_b200.dist import ContextParallelPrefill, shard_units
    from oracle.attention import prefill_rows_ref

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = torch.Generator().manual_seed(0)
        Hq, Hkv, D = 16, 2, 256
        qc = torch.randn(1, Hq, T, D, generator=g).bfloat16()
        kc = torch.randn(1, Hkv, T, D, generator=g).bfloat16()
        vc = torch.randn(1, Hkv, T, D, generator=g).bfloat16()
        q, k, v = qc.to(dev), kc.to(dev), vc.to(dev)
        cp = ContextParallelPrefill(T, world, rank)
        pick = lambda t: torch.cat([t[:, :, a:b] for a, b in cp.chunks], dim=2).contiguous()
        out = cp.run(pick(q), pick(k), pick(v), scale=1 / 16)
        assert api.device_error() == 0
        full = api.prefill(q, k, v, scale=1 / 16)
        err_vs_kernel = (out - pick(full)).abs().max().item()
        # Oracle rows: first, second, middle, second-to-last and last row of
        # each of this rank's chunks, for a query head of each KV head.
        err_vs_oracle = 0.0
        n_rows = 0
        for slot, (a, b) in enumerate(cp.chunks):
            rows = sorted({a, a + 1, (a + b) // 2, b - 2, b - 1})
            local = [r - a + slot * cp.c for r in rows]
            for h in (0, 9):
                ref = prefill_rows_ref(qc, kc, vc, 0, h, rows, scale=1 / 16)
                got = out[0, h, local].float().cpu()
                err_vs_oracle = max(err_vs_oracle, (got - ref).abs().max().item())
                n_rows += len(rows)

        # Batched prefill sharded by (batch, KV head) units: no collective.
        B, Hq3, Hkv3, D3, T3 = 4, 8, 2, 128, 512
        g3 = torch.Generator().manual_seed(1)
        q3 = torch.randn(B, Hq3, T3, D3, generator=g3).bfloat16().to(dev)
        k3 = torch.randn(B, Hkv3, T3, D3, generator=g3).bfloat16().to(dev)
        v3 = torch.randn(B, Hkv3, T3, D3, generator=g3).bfloat16().to(dev)
        ref3 = api.prefill(q3, k3, v3)
        grp = Hq3 // Hkv3
        err_sh = 0.0
        for b, lo, hi in shard_units(B, Hkv3, world, rank):
            o = api.prefill(q3[b:b + 1, lo * grp:hi * grp], k3[b:b + 1, lo:hi], v3[b:b + 1, lo:hi])
            err_sh = max(err_sh, (o - ref3[b:b + 1, lo * grp:hi * grp]).abs().max().item())
        torch.cuda.synchronize()
        result[rank] = (err_vs_oracle, n_rows, err_vs_kernel, err_sh, api.device_error())
    finally:
        dist.destroy_process_group()


def test_context_parallel_and_sharding_on_all_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T_CP, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    assert len(result) == world
    for rank, (err_or, n_rows, err_k, err_sh, dev_err) in sorted(result.items()):
        print(f"world {world} rank {rank}: {n_rows} oracle rows max|d| {err_or:.3e}, "
              f"vs 1-GPU kernel {err_k:.3e}, sharded prefill {err_sh:.3e}")
        assert err_or <= TOL, (rank, err_or)
        assert err_k <= TOL, (rank, err_k)
        assert err_sh <= TOL, (rank, err_sh)
        assert dev_err == 0
