"""Host-side multi-GPU logic on CPU: partitioning, and the zig-zag
context-parallel prefill as world_size-2 gloo ranks with the oracle standing
in for the kernel (the exchange and reassembly are what is under test)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from npu_b200 import dist as D


def test_shard_units_cover_everything_once():
    for B, H, W in [(64, 4, 1), (64, 4, 8), (3, 4, 5), (1, 2, 4), (7, 3, 2)]:
        seen = []
        for r in range(W):
            for b, lo, hi in D.shard_units(B, H, W, r):
                assert 0 <= lo < hi <= H
                seen += [(b, h) for h in range(lo, hi)]
        assert sorted(seen) == [(b, h) for b in range(B) for h in range(H)]
    assert D.shard_units(64, 4, 8, 3) == [(b, 0, 4) for b in range(24, 32)]


def test_shard_sequences_balances_length():
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1024, 32769, (128,), generator=g).tolist()
    for W in (1, 2, 4, 8):
        bins = D.shard_sequences(lens, W)
        assert sorted(i for b in bins for i in b) == list(range(128))
        loads = [sum(lens[i] for i in b) for b in bins]
        assert max(loads) - min(loads) <= max(lens)
        if W > 1:
            assert max(loads) / (sum(lens) / W) < 1.02


def test_zigzag_balances_causal_work():
    T, world, D_, H = 131072, 8, 256, 16
    work = [sum(D.causal_flops_rows(c, D_, H) for c in D.zigzag_chunks(T, world, r)) for r in range(world)]
    assert max(work) == min(work)
    total = D.causal_flops_rows((0, T), D_, H)
    assert sum(work) == total
    rows = sorted(r for g in range(world) for c in D.zigzag_chunks(T, world, g) for r in range(c[0], c[1], 4096))
    assert rows == list(range(0, T, 4096))
    with pytest.raises(ValueError):
        D.zigzag_chunks(100, 8, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_worker(rank, world, port, T, result):
    import datetime

    import torch.distributed as dist

    from oracle.attention import dense_attention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(0)
        B, Hq, Hkv, Dh = 1, 4, 2, 32
        q = torch.randn(B, Hq, T, Dh, generator=g).bfloat16()
        k = torch.randn(B, Hkv, T, Dh, generator=g).bfloat16()
        v = torch.randn(B, Hkv, T, Dh, generator=g).bfloat16()
        cp = D.ContextParallelPrefill(T, world, rank,
                                      attn_fn=lambda q_, k_, v_, sp: dense_attention(q_, k_, v_, start_pos=sp))
        sl = [slice(a, b) for a, b in cp.chunks]
        pick = lambda t: torch.cat([t[:, :, s] for s in sl], dim=2)
        out = cp.run(pick(q), pick(k), pick(v))
        ref = pick(dense_attention(q, k, v))
        result[rank] = float((out - ref).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_prefill_gloo(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_cp_worker, args=(r, world, port, 64, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len(result) == world
    assert max(result.values()) < 1e-5


def _dead_peer_worker(rank, world, port, result):
    """Rank 1 joins the group and exits without reaching the collective;
    rank 0's K/V all-gather must fail within the group's timeout, not hang."""
    import datetime
    import os
    import time

    import torch.distributed as dist

    from npu_b200.dist import ContextParallelPrefill

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # dies between steps, with nothing in flight
    cp = ContextParallelPrefill(256, world, rank)
    k = torch.zeros(1, 1, 2 * cp.c, 64)
    t0 = time.time()
    try:
        cp.gather_kv(k, k)
        result[rank] = ("no error", time.time() - t0)
    except Exception as e:  # gloo reports the lost peer (closed connection or timeout)
        result[rank] = (type(e).__name__, time.time() - t0)


def test_dead_peer_is_detected_on_the_host():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    result = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert 0 in result, "rank 0 neither finished nor failed"
    err, secs = result[0]
    assert err != "no error"
    assert secs < 60
