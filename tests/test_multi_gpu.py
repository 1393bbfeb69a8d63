"""Multi-GPU paths on real GPUs (skipped with fewer than 2): the zig-zag
context-parallel prefill with its NCCL K/V all-gather, and batch sharding,
each checked against the single-GPU kernel on the same inputs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, T, result):
    import datetime

    import torch.distributed as dist

    from npu_b200 import api
    from npu_b200.dist import ContextParallelPrefill, shard_units

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        g = torch.Generator().manual_seed(0)
        Hq, Hkv, D = 16, 2, 256
        q = torch.randn(1, Hq, T, D, generator=g).bfloat16().to(dev)
        k = torch.randn(1, Hkv, T, D, generator=g).bfloat16().to(dev)
        v = torch.randn(1, Hkv, T, D, generator=g).bfloat16().to(dev)
        full = api.prefill(q, k, v, scale=1 / 16)
        cp = ContextParallelPrefill(T, world, rank)
        pick = lambda t: torch.cat([t[:, :, a:b] for a, b in cp.chunks], dim=2).contiguous()
        out = cp.run(pick(q), pick(k), pick(v), scale=1 / 16)
        err_cp = (out - pick(full)).abs().max().item()

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
        result[rank] = (err_cp, err_sh, api.device_error())
    finally:
        dist.destroy_process_group()


def test_context_parallel_and_sharding_on_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 4096, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    assert len(result) == world
    for rank, (err_cp, err_sh, dev_err) in result.items():
        assert err_cp <= TOL, (rank, err_cp)
        assert err_sh <= TOL, (rank, err_sh)
        assert dev_err == 0
