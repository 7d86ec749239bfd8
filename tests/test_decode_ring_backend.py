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
import pytest
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
        comm.close()
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
    released = []
    rb.set_staging_release_fn(released.append)
    for r in range(2):
        rb.register_decode_ring(int(bt[r, 0]), ring, slot=r, prefix_len=PREFIX)
        rb.map_request_peer(int(bt[r, 0]), ["c0"])      # its prefix was staged for the prefill
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
    comm.close()
    for r in range(2):
        rb.clear_decode_ring(int(bt[r, 0]))
    return {"worst": worst, "ring_steps": rb.IMPL_STATS["decode_ring"], "released": released,
            "first_blocks": [int(bt[r, 0]) for r in range(2)],
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
    # each request's staged prefix is released once, at its first decode step
    assert owner["released"] == owner["first_blocks"]
    # the owner (rank 1 of 2) keeps the decode tokens at odd positions
    for r, n in enumerate(OWN):
        pos = [PREFIX + n + t for t in range(STEPS)]
        assert owner["growth"][r] == [p for p in pos if p % 2 == 1]


# ---------------------------------------------------------------------------
# GPU: the same routing on the B200 kernels
# ---------------------------------------------------------------------------
def _tol_ok(got, want):
    import parity as P
    try:
        return True, P.check_out(np.asarray(got, np.float32), np.asarray(want, np.float32), "decode ring").err
    except AssertionError as ex:
        return False, str(ex)


@pytest.mark.gpu
def test_backend_decode_ring_mixed_batch_one_gpu():
    """One GPU, a one-rank ring (the owner alone, no peer chunk): a batch of
    a decode-ring request, a plain decode request and a prefill over cached
    tokens.  The ring request's own chunk moves from the paged cache into its
    ring slot (``hcp_kv_cache_gather``) at its first decode step, its tokens
    go to its growth rows, and the other rows run the local plan; every row
    equals the oracle (2e-3 + 2^-7 |ref|, bf16 output)."""
    from vllm.forward_context import override_forward_context

    from hcp_vllm_plugin_b200 import ring_backend as rb
    from hcp_vllm_plugin_b200.ring_decode import RingDecode

    dev = torch.device("cuda:0")
    h, hkv, d, bs, layers, steps = 28, 4, 128, 16, 2, 3
    own0, ctx1, cached2, new2 = 200, 300, 96, 64
    total = [own0 + steps, ctx1 + steps, cached2 + new2]
    g = torch.Generator().manual_seed(5)
    K = [[torch.randn(n, hkv, d, generator=g).bfloat16() for n in total] for _ in range(layers)]
    V = [[torch.randn(n, hkv, d, generator=g).bfloat16() for n in total] for _ in range(layers)]
    nblk = [(n + bs - 1) // bs for n in total]
    perm = torch.randperm(sum(nblk), generator=g).to(torch.int32)
    bt = torch.zeros(3, max(nblk), dtype=torch.int32)
    o = 0
    for r, n in enumerate(nblk):
        bt[r, :n] = perm[o:o + n]
        o += n
    caches = []
    for layer in range(layers):
        c = torch.zeros(sum(nblk), hkv, bs, 2 * d, dtype=torch.bfloat16)
        for r, n in enumerate(total):
            n = own0 if r == 0 else n          # the ring request's decode tokens never reach this pool
            pos = torch.arange(n)
            blk = bt[r, pos // bs].long()
            c[blk, :, pos % bs, :d] = K[layer][r][:n]
            c[blk, :, pos % bs, d:] = V[layer][r][:n]
        caches.append(c.to(dev))
    ring = RingDecode(layers, 2, own0 + steps + 1, h, hkv, d, d ** -0.5, dev)
    rb.DECODE_RING_MAP.clear()
    rb.reset_impl_stats()
    rb.reset_write_tracking()
    rb.register_decode_ring(int(bt[0, 0]), ring, slot=1, prefix_len=0)
    impl = rb.HcpRingAttentionImpl(h, d, d ** -0.5, hkv)
    worst = 0.0
    try:
        for t in range(steps):
            reqs = [0, 1, 2] if t == 0 else [0, 1]
            qlen = {0: 1, 1: 1, 2: new2}
            seq = {0: own0 + t + 1, 1: ctx1 + t + 1, 2: cached2 + new2}
            qsl = np.concatenate([[0], np.cumsum([qlen[r] for r in reqs])])
            meta = types.SimpleNamespace(
                num_actual_tokens=int(qsl[-1]),
                query_start_loc=torch.tensor(qsl, dtype=torch.int32, device=dev),
                seq_lens=torch.tensor([seq[r] for r in reqs], dtype=torch.int32, device=dev),
                block_table=bt[reqs].to(dev))
            pos = [torch.arange(seq[r] - qlen[r], seq[r]) for r in reqs]
            slots = torch.cat([bt[r, p // bs].long() * bs + p % bs for r, p in zip(reqs, pos)]).to(dev)
            for layer in range(layers):
                name = f"model.layers.{layer}.self_attn.attn"
                lay = types.SimpleNamespace(layer_name=name)
                q = torch.randn(int(qsl[-1]), h, d, generator=g).bfloat16()
                kn = torch.cat([K[layer][r][seq[r] - qlen[r]:seq[r]] for r in reqs]).to(dev)
                vn = torch.cat([V[layer][r][seq[r] - qlen[r]:seq[r]] for r in reqs]).to(dev)
                with override_forward_context(types.SimpleNamespace(attn_metadata={name: meta})):
                    impl.do_kv_cache_update(lay, kn, vn, caches[layer], slots)
                out = torch.zeros(int(qsl[-1]) + 4, h, d, dtype=torch.bfloat16, device=dev)
                impl.forward(lay, q.to(dev), kn, vn, caches[layer], meta, out)
                torch.cuda.synchronize()
                got = out.float().cpu().numpy()
                for i, r in enumerate(reqs):
                    rows = slice(int(qsl[i]), int(qsl[i + 1]))
                    want, _ = ro.attn_with_lse(q[rows].float().numpy(), K[layer][r][:seq[r]].float().numpy(),
                                               V[layer][r][:seq[r]].float().numpy(), d ** -0.5,
                                               seq[r] - qlen[r])
                    ok, err = _tol_ok(got[rows], want)
                    assert ok, (t, layer, r, err)
                    worst = max(worst, err)
        assert rb.IMPL_STATS["decode_ring"] == steps * layers
        assert ring.lens[0][1] == own0 + steps          # own chunk + every decode token (one rank)
        assert rb.WRITE_TRACK["skipped"] == steps * layers
        p0 = torch.arange(own0, own0 + steps)
        for layer in range(layers):                      # the ring's tokens are not in this pool
            assert torch.all(caches[layer][bt[0, p0 // bs].long().to(dev), :, (p0 % bs).to(dev)] == 0)
    finally:
        rb.DECODE_RING_MAP.clear()
        rb.WRITE_TRACK["enabled"] = False


@pytest.mark.gpu
def test_backend_decode_ring_nccl_two_gpus():
    """Two GPUs: a peer process serves its chunk on GPU 0 while the owner on
    GPU 1 runs the backend's forward for two decode-ring requests; the ring
    is a standalone NCCL group (``decode_ring_backend_worker.py``)."""
    import os
    import subprocess
    import sys

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.path.dirname(here))
    procs = [subprocess.Popen([sys.executable, os.path.join(here, "decode_ring_backend_worker.py"), str(r),
                               str(port)], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for r in range(2)]
    outs = []
    for p in procs:
        try:
            outs.append(p.communicate(timeout=400)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            outs.append(p.communicate()[0])
    assert all(p.returncode == 0 for p in procs), "\n".join(o[-3000:] for o in outs)
    assert '"ok": true' in outs[1], outs[1][-3000:]


def test_pool_write_skips_decode_ring_tokens(monkeypatch):
    """``do_kv_cache_update`` does not write a decode-ring request's new
    token into this pool (its assignee keeps it, ``ring_backend.py:519-531``);
    every other row is written, and ``WRITE_TRACK`` records both."""
    from vllm.forward_context import override_forward_context

    from hcp_vllm_plugin_b200 import ops
    from hcp_vllm_plugin_b200 import ring_backend as rb

    def cpu_scatter(key, value, cache, slots):
        for i, s in enumerate(slots.tolist()):
            if s >= 0:
                cache[s // BS, :, s % BS, :D] = key[i]
                cache[s // BS, :, s % BS, D:] = value[i]

    monkeypatch.setattr(ops, "kv_cache_update", cpu_scatter)
    rb.DECODE_RING_MAP.clear()
    rb.register_decode_ring(7, ring=None, slot=0, prefix_len=0)
    name = "model.layers.0.self_attn.attn"
    # rows: ring decode (block 7), plain decode (block 3), a 3-token prefill (block 9)
    meta = types.SimpleNamespace(query_start_loc=torch.tensor([0, 1, 2, 5]), seq_lens=torch.tensor([10, 6, 3]),
                                 block_table=torch.tensor([[7, 8, 0], [2, 3, 0], [9, 0, 0]], dtype=torch.int32))
    slots = torch.tensor([7 * BS + 1, 3 * BS + 1, 9 * BS, 9 * BS + 1, 9 * BS + 2])
    cache = torch.zeros(10, HKV, BS, 2 * D)
    key, value = torch.ones(5, HKV, D), torch.full((5, HKV, D), 2.0)
    impl = rb.HcpRingAttentionImpl(H, D, D ** -0.5, HKV)
    rb.reset_write_tracking()
    try:
        with override_forward_context(types.SimpleNamespace(attn_metadata={name: meta})):
            impl.do_kv_cache_update(types.SimpleNamespace(layer_name=name), key, value, cache, slots)
        assert torch.all(cache[7] == 0)                       # the ring token went nowhere here
        for s in slots.tolist()[1:]:
            assert torch.all(cache[s // BS, :, s % BS, :D] == 1) and torch.all(cache[s // BS, :, s % BS, D:] == 2)
        assert rb.WRITE_TRACK["skipped"] == 1 and rb.WRITE_TRACK["slots"] == set(slots.tolist()[1:])
        # without a forward context nothing can be attributed: every row is written
        impl.do_kv_cache_update(types.SimpleNamespace(layer_name=name), key, value, cache, slots)
        assert torch.all(cache[7, :, 1, :D] == 1)
    finally:
        rb.DECODE_RING_MAP.clear()
        rb.WRITE_TRACK["enabled"] = False
