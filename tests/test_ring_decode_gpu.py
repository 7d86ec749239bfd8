"""Decode ring on the GPU: the N-way merge kernel, the sharded partials +
merge composition on one GPU, and RingDecode over NCCL on 2+ GPUs."""

from __future__ import annotations

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

import parity as P
from oracle import ring_oracle as ro

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("n,d,out_dtype", [(1, 128, torch.float32), (2, 128, torch.float32),
                                           (5, 64, torch.float32), (8, 128, torch.bfloat16)])
def test_merge_n_matches_oracle_chain(n, d, out_dtype):
    from hcp_vllm_plugin_b200 import ops

    g = torch.Generator().manual_seed(n * 7 + d)
    t, h = 37, 28
    so = torch.randn(n, t, h, d, generator=g)
    sl = torch.randn(n, h, t, generator=g) * 4
    if n > 1:
        sl[0, :, 3] = float("-inf")       # an empty partial
        sl[1, :5, 4] = float("inf")       # vLLM's marker of an empty partial
        sl[:, 2, 6] = float("-inf")       # a row with no keys in any shard
    out = torch.empty(t, h, d, dtype=out_dtype, device="cuda")
    out_lse = torch.empty(h, t, device="cuda")
    ops.merge_attn_states_n(out, so.cuda(), sl.cuda(), out_lse)
    torch.cuda.synchronize()
    want, want_lse = ro.merge_chain(so.numpy(), sl.numpy())
    got = out.float().cpu().numpy()
    tol = 1e-5 if out_dtype == torch.float32 else 2.0 ** -8
    np.testing.assert_allclose(got, want, atol=tol, rtol=tol)
    gl = out_lse.cpu().numpy()
    assert np.array_equal(np.isneginf(gl), np.isneginf(want_lse))
    fin = np.isfinite(want_lse)
    np.testing.assert_allclose(gl[fin], want_lse[fin], atol=1e-5, rtol=1e-6)


def test_sharded_decode_equals_single_pass():
    """Eight shards' partials (split-KV decode per shard) merged with one N-way
    launch equal one decode over all keys (fp32 outputs, 65k keys, GQA 28/4)."""
    from hcp_vllm_plugin_b200 import ops

    g = torch.Generator().manual_seed(3)
    B, H, HKV, D, W = 4, 28, 4, 128, 8
    lens = [8192, 5000, 1, 3000]                     # keys per shard, per request
    q = torch.randn(B, H, D, generator=g).bfloat16().cuda()
    shards_k, shards_v = [], []
    for _ in range(W):
        shards_k.append([torch.randn(n, HKV, D, generator=g).bfloat16() for n in lens])
        shards_v.append([torch.randn(n, HKV, D, generator=g).bfloat16() for n in lens])
    states_o = torch.empty(W, B, H, D, device="cuda")
    states_lse = torch.empty(W, H, B, device="cuda")
    for w in range(W):
        k = torch.cat(shards_k[w]).cuda()
        v = torch.cat(shards_v[w]).cuda()
        starts = np.cumsum([0] + lens[:-1])
        seqs = np.array([(b, starts[b], lens[b], -1, 0, 0) for b in range(B)], np.int32)
        ops.decode_splitkv(q, seqs, scale=D ** -0.5, num_kv_heads=HKV, out=states_o[w], lse=states_lse[w],
                           peer_k=k, peer_v=v)
    out = torch.empty(B, H, D, device="cuda")
    out_lse = torch.empty(H, B, device="cuda")
    ops.merge_attn_states_n(out, states_o, states_lse, out_lse)
    # one pass over every request's keys (shards concatenated in order)
    allk = torch.cat([torch.cat([shards_k[w][b] for w in range(W)]) for b in range(B)]).cuda()
    allv = torch.cat([torch.cat([shards_v[w][b] for w in range(W)]) for b in range(B)]).cuda()
    tot = [W * n for n in lens]
    starts = np.cumsum([0] + tot[:-1])
    seqs = np.array([(b, starts[b], tot[b], -1, 0, 0) for b in range(B)], np.int32)
    ref = torch.empty(B, H, D, device="cuda")
    ref_lse = torch.empty(H, B, device="cuda")
    ops.decode_splitkv(q, seqs, scale=D ** -0.5, num_kv_heads=HKV, out=ref, lse=ref_lse, peer_k=allk, peer_v=allv)
    torch.cuda.synchronize()
    # Both paths are held to the parity bar of tests/parity.py against the oracle.
    for b in range(B):
        kk = torch.cat([shards_k[w][b] for w in range(W)]).float().numpy()
        vv = torch.cat([shards_v[w][b] for w in range(W)]).float().numpy()
        want, want_lse = ro.attn_with_lse(q[b:b + 1].float().cpu().numpy(), kk, vv, D ** -0.5, None)
        for name, got, got_lse in (("ring", out, out_lse), ("one launch", ref, ref_lse)):
            P.check_out(got[b].float().cpu().numpy(), want[0], f"{name} request {b}")
            P.check_lse(got_lse[:, b].cpu().numpy(), want_lse[:, 0], f"{name} request {b}")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ring_decode_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), os.path.join(HERE, "ring_decode_gpu_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
