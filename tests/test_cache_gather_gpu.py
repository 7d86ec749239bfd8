"""``hcp_kv_cache_gather`` (pool -> chunk extraction) against the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ring_oracle as orc


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hkv,d,bs", [(torch.bfloat16, 4, 128, 16), (torch.float16, 2, 64, 32),
                                            (torch.bfloat16, 8, 128, 64)])
def test_gather_matches_oracle(dtype, hkv, d, bs):
    from hcp_vllm_plugin_b200 import ops

    g = torch.Generator().manual_seed(hkv * 1000 + d + bs)
    nb = 37
    cache = torch.randn(nb, hkv, bs, 2 * d, generator=g).to(dtype).cuda()
    slots = torch.randint(0, nb * bs, (300,), generator=g)
    slots[[0, 7, 299]] = torch.tensor([-1, nb * bs, -5])   # padding and out-of-range rows -> zeros
    k, v = ops.kv_cache_gather(cache, slots.cuda())
    torch.cuda.synchronize()
    ek, ev = orc.kv_cache_gather(_bits(cache), slots.numpy())
    np.testing.assert_array_equal(_bits(k), ek)
    np.testing.assert_array_equal(_bits(v), ev)


@pytest.mark.gpu
def test_update_then_gather_round_trip():
    """Scatter rows to distinct slots, gather them back: identical rows."""
    from hcp_vllm_plugin_b200 import ops

    g = torch.Generator().manual_seed(5)
    nb, hkv, d, bs, n = 64, 4, 128, 16, 700
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device="cuda")
    slots = torch.randperm(nb * bs, generator=g)[:n].cuda()
    key = torch.randn(n, hkv, d, generator=g).to(torch.bfloat16).cuda()
    value = torch.randn(n, hkv, d, generator=g).to(torch.bfloat16).cuda()
    ops.kv_cache_update(key, value, cache, slots)
    k, v = ops.kv_cache_gather(cache, slots)
    # into strided destinations (rows of a wider buffer)
    wide = torch.zeros(n, 2, hkv, d, dtype=torch.bfloat16, device="cuda")
    ops.kv_cache_gather(cache, slots, key=wide[:, 0], value=wide[:, 1])
    torch.cuda.synchronize()
    assert torch.equal(k, key) and torch.equal(v, value)
    assert torch.equal(wide[:, 0], key) and torch.equal(wide[:, 1], value)
