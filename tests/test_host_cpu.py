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
