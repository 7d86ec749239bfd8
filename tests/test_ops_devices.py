"""The torch front end refuses tensors that are not on the call's GPU.

The library receives raw addresses: a host tensor, or another GPU's tensor,
handed to a kernel would be a memory fault on the device instead of an error
the caller sees.  Every op therefore checks, before it calls the library,
that all of its tensors are CUDA tensors on one device.  The first test needs
no GPU (host tensors are refused before anything is loaded or launched); the
second mixes one host tensor into otherwise valid GPU calls and checks that
the call raises and the output is left untouched."""

import numpy as np
import pytest
import torch

from hcp_vllm_plugin_b200 import _capi as C
from hcp_vllm_plugin_b200 import ops

H, HKV, D, BS = 28, 4, 128, 16


def test_every_op_refuses_host_tensors():
    q = torch.zeros(4, H, D, dtype=torch.bfloat16)
    k = torch.zeros(8, HKV, D, dtype=torch.bfloat16)
    lse = torch.zeros(H, 4)
    cache = torch.zeros(2, HKV, BS, 2 * D, dtype=torch.bfloat16)
    sm = torch.zeros(4, dtype=torch.int64)
    work = ops.make_work([(0, 4, 0, 0, (C.HCP_SRC_A, 0, 8, -1), None)])
    calls = [
        lambda: ops.ring_attn_fwd(q, work, scale=1.0, num_kv_heads=HKV, out=q, k_a=k, v_a=k),
        lambda: ops.ring_attn_with_lse(q, k, k, 1.0, None),
        lambda: ops.decode_splitkv(q, np.zeros((0, 6), np.int32), scale=1.0, num_kv_heads=HKV, out=q),
        lambda: ops.merge_attn_states(q, q, lse, q, lse),
        lambda: ops.merge_attn_states_n(q, torch.zeros(2, 4, H, D), torch.zeros(2, H, 4)),
        lambda: ops.kv_cache_update(k[:4], k[:4], cache, sm),
        lambda: ops.kv_cache_gather(cache, sm),
    ]
    for fn in calls:
        with pytest.raises(ValueError, match="CPU path|must be on"):
            fn()


@pytest.mark.gpu
def test_a_host_tensor_in_a_gpu_call_is_refused():
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(64, H, D, generator=g, device=dev, dtype=torch.bfloat16)
    k = torch.randn(128, HKV, D, generator=g, device=dev, dtype=torch.bfloat16)
    out = torch.zeros_like(q)
    lse = torch.zeros(H, 64, device=dev)
    work = ops.make_work([(0, 64, 0, 0, (C.HCP_SRC_A, 0, 128, -1), None)])
    with pytest.raises(ValueError, match="k_a must be on"):
        ops.ring_attn_fwd(q, work, scale=D ** -0.5, num_kv_heads=HKV, out=out, k_a=k.cpu(), v_a=k)
    with pytest.raises(ValueError, match="out must be on"):
        ops.ring_attn_fwd(q, work, scale=D ** -0.5, num_kv_heads=HKV, out=out.cpu(), k_a=k, v_a=k)
    with pytest.raises(ValueError, match="lse must be on"):
        ops.ring_attn_fwd(q, work, scale=D ** -0.5, num_kv_heads=HKV, out=out, lse=lse.cpu(), k_a=k, v_a=k)
    with pytest.raises(ValueError, match="ext"):
        ops.ring_attn_fwd(q, ops.make_work([(0, 64, 0, 0, (C.HCP_SRC_EXT0, 0, 128, -1), None)]), scale=D ** -0.5,
                          num_kv_heads=HKV, out=out, ext=[(k.cpu(), k.cpu())])
    cache = torch.zeros(16, HKV, BS, 2 * D, device=dev, dtype=torch.bfloat16)
    sm = torch.arange(64, dtype=torch.int64)
    with pytest.raises(ValueError, match="slot_mapping must be on"):
        ops.kv_cache_update(q[:64, :HKV], q[:64, :HKV], cache, sm)
    with pytest.raises(ValueError, match="slot_mapping must be on"):
        ops.kv_cache_gather(cache, sm)
    with pytest.raises(ValueError, match="prefix_lse must be on"):
        ops.merge_attn_states(out, q, lse.cpu(), q, lse)
    seqs = np.array([(0, 0, 128, 0, 0, 0)], np.int32)
    with pytest.raises(ValueError, match="peer_v must be on"):
        ops.decode_splitkv(q[:1], seqs, scale=D ** -0.5, num_kv_heads=HKV, out=out[:1], peer_k=k, peer_v=k.cpu())
    torch.cuda.synchronize()
    assert bool((out == 0).all()) and bool((cache == 0).all())  # nothing was launched
    assert C.device_status() == 0
    # the same calls with every tensor on the GPU go through
    ops.ring_attn_fwd(q, work, scale=D ** -0.5, num_kv_heads=HKV, out=out, lse=lse, k_a=k, v_a=k)
    ops.kv_cache_update(q[:64, :HKV], q[:64, :HKV], cache, sm.to(dev))
    torch.cuda.synchronize()
    assert bool(out.abs().sum() > 0) and bool(cache.abs().sum() > 0)
