"""The backend drives the decode ring: decode rows of requests registered in
``DECODE_RING_MAP`` (``ring_backend.py:153-211, 630-730``) leave the local
plan and run as one ring step per layer.

CPU, two gloo ranks on a standalone ring (as two vLLM instances would form
it): rank 0 is a peer serving its prefix chunk, rank 1 the owner calling
``HcpRingAttentionImpl.forward`` for two registered requests over three
decode steps.  The device ops are the CPU checkers (the paged gather, the
partial and the merge); the owner's paged cache holds its own chunk after
the prefix positions, and NaN where the prefix (held by the peer) would be,
so reading the prefix from the pool would show.  Each output row must equal
attention over the peer chunk, the request's own chunk and its decode tokens
so far."""

from __future__ import annotations

import socket
import types

import numpy as np
import torch
import torch.multiprocessing as mp

from oracle import ring_oracle as ro

H, HKV, D, LAYERS, BS = 4, 2, 64, 2, 4
PREFIX = 8                      # tokens held by the peer (block aligned)
OWN = (6, 9)                    # each request's own prompt tokens
STEPS = 3
NAMES = [f"model.layers.{i}.self_attn.attn" for i in range(LAYERS)]


def _data():
    g = torch.Generator().manual_seed(3)
    peer = [(torch.randn(PREFIX, HKV, D, generator=g), torch.randn(PREFIX, HKV, D, generator=g))
            for _ in range(LAYERS)]
    own = [[(torch.randn(n, HKV, D, generator=g), torch.randn(n, HKV, D, generator=g)) for _ in range(LAYERS)]
           for n in OWN]
    # per step, request, layer: (q [1,H,D], k [1,Hkv,D], v)
    tok = [[[(torch.randn(1, H, D, generator=g), torch.randn(1, HKV, D, generator=g),
              torch.randn(1, HKV, D, generator=g)) for _ in range(LAYERS)] for _ in OWN] for _ in range(STEPS)]
    return peer, own, tok


def _cpu_gather(cache, slots, key, value):
    blk, off = slots // BS, slots % BS
    rows = cache[blk, :, off]
    key.copy_(rows[..., :D])
    value.copy_(rows[..., D:])


def _rank(rank, port, q):
    try:
        q.put((rank, _body(rank, port)))
    except BaseException as e:  # noqa: BLE001 - reported to the test
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def _body(rank, port):
    from hcp_vllm_plugin_b200 import ops
    from hcp_vllm_plugin_b200 import ring_backend as rb
    from hcp_vllm_plugin_b200.ring_decode import RingComm
    from tests.test_ring_decode_gloo import cpu_ring_decode

    ops.kv_cache_gather = _cpu_gather          # this process only
    RingDecode = cpu_ring_decode()
    comm = RingComm.standalone("127.0.0.1", port, rank, 2, backend="gloo", timeout_s=60, connect_timeout_s=60)
    ring = RingDecode(LAYERS, 2, max(PREFIX, *OWN) + STEPS, H, HKV, D, D ** -0.5, torch.device("cpu"),
                      dtype=torch.float32, comm=comm)
    peer, own, tok = _data()
    if rank == 0:
        ring.serve(lambda layer: peer[layer], poll_s=0.2)
        return {"steps": ring.steps_served}

    # owner: paged caches, two requests with their own blocks
    impl = rb.HcpRingAttentionImpl(H, D, D ** -0.5, HKV)
    nblk = [(PREFIX + n + STEPS + BS - 1) // BS for n in OWN]
    bt = torch.zeros(2, max(nblk), dtype=torch.int32)
    bt[0, :nblk[0]] = torch.arange(nblk[0])
    bt[1, :nblk[1]] = torch.arange(nblk[0], nblk[0] + nblk[1])
    caches = []
    for layer in range(LAYERS):
        c = torch.full((sum(nblk), HKV, BS, 2 * D), float("nan"))
        for r, n in enumerate(OWN):
            for j in range(n):
                p = PREFIX + j
                b, o = int(bt[r, p // BS]), p % BS
                c[b, :, o, :D] = own[r][layer][0][j]
                c[b, :, o, D:] = own[r][layer][1][j]
        caches.append(c)
    for r in range(2):
        rb.register_decode_ring(int(bt[r, 0]), ring, slot=r, prefix_len=PREFIX)
    worst = 0.0
    for t in range(STEPS):
        seq = [PREFIX + n + t + 1 for n in OWN]
        meta = types.SimpleNamespace(query_start_loc=torch.tensor([0, 1, 2], dtype=torch.int32),
                                     seq_lens=torch.tensor(seq, dtype=torch.int32), block_table=bt,
                                     num_actual_tokens=2)
        for layer in range(LAYERS):
            qq = torch.cat([tok[t][r][layer][0] for r in range(2)])
            kk = torch.cat([tok[t][r][layer][1] for r in range(2)])
            vv = torch.cat([tok[t][r][layer][2] for r in range(2)])
            out = torch.zeros(2, H, D)
            impl.forward(types.SimpleNamespace(layer_name=NAMES[layer]), qq, kk, vv, caches[layer], meta, out)
            for r in range(2):
                keys = torch.cat([peer[layer][0], own[r][layer][0]] + [tok[j][r][layer][1] for j in range(t + 1)])
                vals = torch.cat([peer[layer][1], own[r][layer][1]] + [tok[j][r][layer][2] for j in range(t + 1)])
                want, _ = ro.attn_with_lse(qq[r:r + 1].numpy(), keys.numpy(), vals.numpy(), D ** -0.5, None)
                err = float(np.abs(out[r].numpy() - want[0]).max())
                worst = max(worst, err if np.isfinite(err) else float("inf"))  # NaN must fail
    ring.stop()
    for r in range(2):
        rb.clear_decode_ring(int(bt[r, 0]))
    return {"worst": worst, "ring_steps": rb.IMPL_STATS["decode_ring"],
            "growth": [ring.growth_positions[0][r] for r in range(2)]}


def test_backend_routes_decode_rows_to_the_ring():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert all(isinstance(v, dict) for v in res.values()), res
    assert all(p.exitcode == 0 for p in procs)
    assert res[0]["steps"] == STEPS
    owner = res[1]
    assert owner["worst"] < 1e-5, owner
    assert owner["ring_steps"] == STEPS * LAYERS
    # the owner (rank 1 of 2) keeps the decode tokens at odd positions
    for r, n in enumerate(OWN):
        pos = [PREFIX + n + t for t in range(STEPS)]
        assert owner["growth"][r] == [p for p in pos if p % 2 == 1]
