"""The allocation-free split-KV decode entry point, called through the C ABI.

``hcp_ring_decode_splitkv_noalloc`` is for callers that cannot allocate
device memory at decode time (a plain C/FFI host without an allocator, or an
engine whose HBM is already reserved for its KV cache): it keeps the split-KV
partials in a fixed 16 MiB array inside the library.  This test checks that
two calls in a row - on different inputs, so the second finds the first's
leftovers in the shared array - give the same results as the workspace entry
point (and, for the first, the CPU oracle), that neither allocates device
memory, and that a call needing more scratch than the array holds is refused
without launching anything.  The file name sorts last so a run that stops at
the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, HKV, D, BS = 28, 4, 128, 16


def _problem(seed, dev, peer_lens, local_lens):
    g = torch.Generator(device="cpu").manual_seed(seed)
    n = len(peer_lens)
    q = torch.randn(n, H, D, generator=g).bfloat16().to(dev)
    pk = torch.randn(max(1, sum(peer_lens)), HKV, D, generator=g).bfloat16().to(dev)
    pv = torch.randn(max(1, sum(peer_lens)), HKV, D, generator=g).bfloat16().to(dev)
    nbs = [(L + BS - 1) // BS for L in local_lens]
    nblocks = sum(nbs) + 3
    perm = np.random.default_rng(seed).permutation(nblocks)
    bt = np.zeros((n, max(nbs)), np.int32)
    o = 0
    for r, nb in enumerate(nbs):
        bt[r, :nb] = perm[o:o + nb]
        o += nb
    cache = torch.randn(nblocks, HKV, BS, 2 * D, generator=g).bfloat16().to(dev)
    seqs, off = [], 0
    for r in range(n):
        seqs.append((r, off, peer_lens[r], r, 0, local_lens[r]))
        off += peer_lens[r]
    return q, pk, pv, cache, torch.from_numpy(bt).to(dev), np.array(seqs, np.int32)


def test_noalloc_decode_matches_workspace_decode_on_two_calls():
    """Two calls in a row (different inputs, so the second finds the first's
    partials in the shared array) equal the workspace entry point bit for bit
    (same kernels, same split), the first also the CPU oracle; the calls
    allocate no device memory: the free bytes the driver reports and the
    torch caching allocator's count are unchanged across each call."""
    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops
    from oracle import ring_oracle as ro
    dev = torch.device("cuda:0")
    lib = C.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for seed, peer_lens, local_lens in ((0, [4096, 700, 64], [6000, 1500, 300]),
                                        (1, [2048, 0, 5000, 33], [1000, 4096, 16, 2500])):
        q, pk, pv, cache, bt, seqs = _problem(seed, dev, peer_lens, local_lens)
        kw = dict(scale=D ** -0.5, num_kv_heads=HKV, peer_k=pk, peer_v=pv, kv_cache=cache,
                  block_table=bt)
        out_ws = torch.empty_like(q)
        lse_ws = torch.empty(H, q.shape[0], dtype=torch.float32, device=dev)
        ops.decode_splitkv(q, seqs, out=out_ws, lse=lse_ws, **kw)
        out_na = torch.full_like(q, float("nan"))
        lse_na = torch.full_like(lse_ws, float("nan"))
        args, keep = ops.decode_args(q, seqs, out=out_na, lse=lse_na, **kw)
        assert lib.hcp_decode_workspace_bytes(ctypes.byref(args)) <= 16 * 1024 * 1024
        torch.cuda.synchronize()
        free0, alloc0 = torch.cuda.mem_get_info(dev)[0], torch.cuda.memory_allocated(dev)
        rc = lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(args), stream)
        assert rc == C.HCP_OK, C.STATUS_NAMES.get(rc, rc)
        torch.cuda.synchronize()
        free1, alloc1 = torch.cuda.mem_get_info(dev)[0], torch.cuda.memory_allocated(dev)
        assert (free1, alloc1) == (free0, alloc0), "the allocation-free entry point allocated device memory"
        assert torch.equal(out_na, out_ws) and torch.equal(lse_na, lse_ws)
        if seed == 0:
            cf = cache.float().cpu().numpy()
            btn = bt.cpu().numpy()
            for (qr, ps, pl, preq, ls, ll) in seqs:
                kl, vl = ro.paged_gather(cf, btn[preq], ls + ll)
                k = np.concatenate([pk[ps:ps + pl].float().cpu().numpy(), kl[ls:]], 0)
                v = np.concatenate([pv[ps:ps + pl].float().cpu().numpy(), vl[ls:]], 0)
                want, want_lse = ro.attn_with_lse(q[qr:qr + 1].float().cpu().numpy(), k, v, D ** -0.5, None)
                assert np.abs(out_na[qr].float().cpu().numpy() - want[0]).max() <= 2e-3
                assert np.abs(lse_na[:, qr].cpu().numpy() - want_lse[:, 0]).max() <= 1e-3
        del keep
    assert C.device_status() == 0


def test_noalloc_decode_refuses_calls_beyond_its_scratch():
    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops
    dev = torch.device("cuda:0")
    lib = C.load()
    # 2 x 65536 keys in 64-key chunks: 2048 partials x 28 heads x 129 floats > 16 MiB
    n, plen = 2, 65536
    q = torch.zeros(n, H, D, dtype=torch.bfloat16, device=dev)
    pk = torch.zeros(n * plen, HKV, D, dtype=torch.bfloat16, device=dev)
    seqs = np.array([(r, r * plen, plen, 0, 0, 0) for r in range(n)], np.int32)
    out = torch.zeros_like(q)
    args, keep = ops.decode_args(q, seqs, scale=D ** -0.5, num_kv_heads=HKV, out=out, peer_k=pk,
                                 peer_v=pk, chunk_keys=64)
    assert lib.hcp_decode_workspace_bytes(ctypes.byref(args)) > 16 * 1024 * 1024
    rc = lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 5, C.STATUS_NAMES.get(rc, rc)  # HCP_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert bool((out == 0).all())  # nothing was launched
    del keep
