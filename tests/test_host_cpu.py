"""Host-side logic that needs no GPU."""
import gc

import torch

from oracle import qwen_ref as R


def test_qwen_drop_in_weight_copies_follow_the_layer_object():
    """attn_forward keeps device copies of a layer's weights while the layer
    object lives, reuses them across calls, and drops them with the layer."""
    from npu_b200 import qwen_attention as m

    rc = R.QwenAttnConfig(d_model=64, n_head=2, n_head_kv=1, head_dim=64, rope_dim=16)
    layer = R.make_layer(rc, seed=1)
    before = len(m._LAYER_WEIGHTS)
    w = m._layer_on_device(layer, torch.device("cpu"), torch.bfloat16)
    assert m._layer_on_device(layer, torch.device("cpu"), torch.bfloat16) is w
    assert w["wq"].dtype == torch.bfloat16 and torch.equal(w["wq"], layer.wq.to(torch.bfloat16))
    assert len(m._LAYER_WEIGHTS) == before + 1
    del layer, w
    gc.collect()
    assert len(m._LAYER_WEIGHTS) == before
    # Weights already on the target device and dtype are used as they are.
    same = R.make_layer(rc, seed=2, dtype=torch.bfloat16)
    assert m._layer_on_device(same, torch.device("cpu"), torch.bfloat16)["wo"] is same.wo


def _reference_stacks(B, Hq, T, Tk, BR, D, start_pos, seed=0):
    """Q/K/V stacks and start rows exactly as smollm.py:147-161 builds them."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, T, D, generator=g)
    k = torch.randn(B, Hq, Tk, D, generator=g)
    v = torch.randn(B, Hq, Tk, D, generator=g)
    n_q = -(-T // BR)
    q = torch.cat([q, q.new_zeros(B, Hq, n_q * BR - T, D)], dim=2)
    N = B * Hq * n_q
    q_stack = q.view(B, Hq, n_q, BR, D).reshape(N, BR, D).contiguous()
    k_stack = k.unsqueeze(2).expand(B, Hq, n_q, Tk, D).reshape(N, Tk, D).contiguous()
    v_stack = v.unsqueeze(2).expand(B, Hq, n_q, Tk, D).reshape(N, Tk, D).contiguous()
    rows = [i * BR + start_pos for _ in range(B * Hq) for i in range(n_q)]
    return q_stack, k_stack, v_stack, rows, n_q


def test_run_batch_recognises_the_reference_block_layout():
    """NpuAttention finds the (batch, head) units of the reference caller's
    stacks (n_q blocks per unit, identical K/V within a unit) and refuses
    anything else, which then runs block by block."""
    from npu_b200 import NpuAttention

    attn = NpuAttention(BR=32, BC=32, D=64, n_cores=4)  # smollm.py:318
    q, k, v, rows, n_q = _reference_stacks(2, 3, 100, 128, 32, 64, start_pos=0)
    assert n_q == 4 and attn._units_of_blocks(k, v, rows) == 4
    q, k, v, rows, n_q = _reference_stacks(1, 2, 64, 96, 32, 64, start_pos=32, seed=1)  # chunked prefill
    assert attn._units_of_blocks(k, v, rows) == 2
    # one K element changed inside a unit
    k2 = k.clone()
    k2[1, 5, 3] += 1.0
    assert attn._units_of_blocks(k2, v, rows) == 1
    # a V difference too
    v2 = v.clone()
    v2[3, 0, 0] -= 1.0
    assert attn._units_of_blocks(k, v2, rows) == 1
    # start rows that do not follow i * BR + s0, or a dummy block
    assert attn._units_of_blocks(k, v, [0, 32, 0, 33]) == 1
    assert attn._units_of_blocks(k, v, [0, 32, 0, -1_000_000]) == 1
    # single blocks (decode through run_batch) stay on the per-block path
    assert attn._units_of_blocks(k[:1], v[:1], [7]) == 1
    assert attn._units_of_blocks(k, v, [5, 5, 5, 5]) == 1


def test_profiler_interface_and_disabled_noop():
    """npu_b200.profiler keeps the reference profiler's interface
    (npu/profiler.py): a shared no-op when disabled, per-name totals and call
    counts when enabled, a report, and reset."""
    from npu_b200.profiler import PROF, profile

    PROF.reset()
    PROF.disable()
    assert profile("x") is profile("y")  # the shared no-op context manager
    with profile("x"):
        pass
    assert PROF.stats() == {}
    PROF.enable()
    try:
        for _ in range(3):
            with profile("rms1"):
                torch.ones(64).sum()
        with profile("total"):
            pass
        st = PROF.stats()
        assert st["rms1"]["calls"] == 3 and st["rms1"]["host_ms"] >= 0
        assert st["total"]["calls"] == 1
        if not torch.cuda.is_available():
            assert st["rms1"]["device_ms"] is None
        PROF.report()
    finally:
        PROF.disable()
        PROF.reset()
    assert PROF.stats() == {}
