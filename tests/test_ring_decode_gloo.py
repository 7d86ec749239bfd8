"""Decode ring host logic on CPU: gloo ranks run RingDecode (query broadcast,
round-robin growth placement, per-rank partials, gather and N-way merge)
with the device ops replaced by the CPU oracle.  Every step's output must
equal attention of the query over all keys so far (prefix chunks of every
rank plus every decode token), and rank r must hold exactly the decode
tokens at positions p with p mod N == r (``ring_decode.py:30-43``)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ring_oracle as ro

H, HKV, D, LAYERS, STEPS = 4, 2, 16, 2, 7
CHUNKS = (8, 12, 5)  # per-rank prefix rows of each request


def _cpu_partial(q, kv_k, kv_v, segs, *, scale, num_kv_heads, out, lse):
    for i, start, n in segs:
        if n == 0:
            out[i] = 0
            lse[:, i] = float("-inf")
            continue
        rows = slice(start, start + n)
        o, l = ro.attn_with_lse(q[i:i + 1].float().numpy(), kv_k[rows].float().numpy(),
                                kv_v[rows].float().numpy(), scale, None)
        out[i] = torch.from_numpy(o[0])
        lse[:, i] = torch.from_numpy(l[:, 0])


def _cpu_merge(out, states_o, states_lse, out_lse):
    o, l = ro.merge_chain(states_o.numpy(), states_lse.numpy())
    out.copy_(torch.from_numpy(o).to(out.dtype))
    if out_lse is not None:
        out_lse.copy_(torch.from_numpy(l))


def _data(world):
    g = torch.Generator().manual_seed(world)
    B = len(CHUNKS)
    total = [c * world + STEPS for c in CHUNKS]
    ks = [[torch.randn(t, HKV, D, generator=g) for t in total] for _ in range(LAYERS)]
    vs = [[torch.randn(t, HKV, D, generator=g) for t in total] for _ in range(LAYERS)]
    qs = [[torch.randn(B, H, D, generator=g) for _ in range(STEPS)] for _ in range(LAYERS)]
    return ks, vs, qs


def cpu_ring_decode():
    """RingDecode with the CPU checkers as its device ops (a subclass, so the
    product class is left as it is for other tests in the same process)."""
    from hcp_vllm_plugin_b200.ring_decode import RingDecode

    class CpuRingDecode(RingDecode):
        partial_fn = staticmethod(_cpu_partial)
        merge_fn = staticmethod(_cpu_merge)

    return CpuRingDecode


def _run(rank, world, result_q=None):
    RingDecode = cpu_ring_decode()
    ks, vs, qs = _data(world)
    B = len(CHUNKS)
    cap = max(CHUNKS) + STEPS
    rd = RingDecode(LAYERS, B, cap, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32)
    for layer in range(LAYERS):
        for b, c in enumerate(CHUNKS):
            sl = slice(rank * c, (rank + 1) * c)
            rd.set_chunk(layer, b, ks[layer][b][sl], vs[layer][b][sl])
    worst = 0.0
    for t in range(STEPS):
        pos = [c * world + t for c in CHUNKS]
        for layer in range(LAYERS):
            if rank == rd.owner:
                k_new = torch.stack([ks[layer][b][pos[b]] for b in range(B)])
                v_new = torch.stack([vs[layer][b][pos[b]] for b in range(B)])
                out = torch.empty(B, H, D)
                out_lse = torch.empty(H, B)
                rd.step(layer, pos, qs[layer][t], k_new, v_new, out, out_lse)
                for b in range(B):
                    want, want_lse = ro.attn_with_lse(qs[layer][t][b:b + 1].numpy(),
                                                      ks[layer][b][:pos[b] + 1].numpy(),
                                                      vs[layer][b][:pos[b] + 1].numpy(), D ** -0.5, None)
                    worst = max(worst, float(np.abs(out[b].numpy() - want[0]).max()),
                                float(np.abs(out_lse[:, b].numpy() - want_lse[:, 0]).max()))
            else:
                assert rd.step(layer, pos) is None
    growth_ok = all(rd.growth_positions[layer][b] == [c * world + t for t in range(STEPS)
                                                       if (c * world + t) % world == rank]
                    for layer in range(LAYERS) for b, c in enumerate(CHUNKS))
    if result_q is not None:
        result_q.put((rank, worst if rank == rd.owner else None, growth_ok))
    return worst, growth_ok


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run(rank, world, result_q)
    finally:
        dist.destroy_process_group()


def test_ring_decode_single_rank():
    worst, growth_ok = _run(0, 1)
    assert worst < 1e-5 and growth_ok


@pytest.mark.parametrize("world", [2, 3, 8])
def test_ring_decode_gloo(world):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = [q.get(timeout=10) for _ in range(world)]
    assert all(ok for _, _, ok in res), res
    worst = [w for _, w, _ in res if w is not None][0]
    assert worst < 1e-5, worst
