"""Decode-ring serving protocol on CPU: a standalone gloo ring (TCPStore
rendezvous, as separately launched vLLM instances would form it), peers in
``RingDecode.serve`` and the owner posting one header per engine step.

Requests join and leave the decode batch between steps and reuse slots; the
peers serve one chunk for every request (the reference's node serves its own
chunk snapshot, ``ring_decode.py:246-249``), the owner installs each
request's own chunk.  Every layer's output must equal attention of the query
over all keys the request has so far (every peer chunk, its own chunk and its
decode tokens), and the decode tokens must land round-robin by position
(``ring_decode.py:30-43``), isolated per request."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import ring_oracle as ro

H, HKV, D, LAYERS, WORLD, SLOTS = 4, 2, 16, 2, 3, 2
PEER_CHUNK = (6, 9)           # rows of rank 0's and rank 1's chunk
OWN = {"A": 7, "B": 4, "C": 5}
# engine steps: (request, slot, fresh) per row
SCHEDULE = [
    [("A", 0, True)],
    [("A", 0, False), ("B", 1, True)],
    [("B", 1, False), ("A", 0, False)],
    [("B", 1, False)],                       # A finished
    [("C", 0, True), ("B", 1, False)],       # C reuses A's slot
    [("C", 0, False)],
    [("C", 0, False), ("B", 1, False)],
]


def _data():
    g = torch.Generator().manual_seed(7)
    peer = [[(torch.randn(n, HKV, D, generator=g), torch.randn(n, HKV, D, generator=g))
             for n in PEER_CHUNK] for _ in range(LAYERS)]
    own = {r: [(torch.randn(n, HKV, D, generator=g), torch.randn(n, HKV, D, generator=g))
               for _ in range(LAYERS)] for r, n in OWN.items()}
    steps = len(SCHEDULE)
    tok = {r: [[(torch.randn(1, HKV, D, generator=g), torch.randn(1, HKV, D, generator=g),
                 torch.randn(1, H, D, generator=g)) for _ in range(LAYERS)] for _ in range(steps)] for r in OWN}
    return peer, own, tok


def _cpu_ops():
    from tests.test_ring_decode_gloo import cpu_ring_decode
    return cpu_ring_decode()


def _rank(rank, port, q):
    try:
        q.put((rank, _rank_body(rank, port)))
    except BaseException as e:  # noqa: BLE001 - reported to the test
        q.put((rank, repr(e)))


def _rank_body(rank, port):
    from hcp_vllm_plugin_b200.ring_decode import RingComm
    RingDecode = _cpu_ops()
    comm = RingComm.standalone("127.0.0.1", port, rank, WORLD, backend="gloo", timeout_s=60,
                               connect_timeout_s=60)
    cap = max(max(PEER_CHUNK), max(OWN.values())) + len(SCHEDULE)
    ring = RingDecode(LAYERS, SLOTS, cap, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32,
                      comm=comm)
    peer, own, tok = _data()
    if rank != ring.owner:
        ring.serve(lambda layer: peer[layer][rank], poll_s=0.2)
        return {"steps": ring.steps_served}
    worst = 0.0
    seen = {r: 0 for r in OWN}                 # decode tokens so far per request
    for t, rows in enumerate(SCHEDULE):
        base = sum(PEER_CHUNK)
        positions = [base + OWN[r] + seen[r] for r, _, _ in rows]
        slots = [s for _, s, _ in rows]
        ring.begin_step(slots, positions, [s for _, s, f in rows if f])
        for layer in range(LAYERS):
            for r, s, f in rows:
                if f:
                    ring.set_chunk(layer, s, *own[r][layer])
            q = torch.cat([tok[r][seen[r]][layer][2] for r, _, _ in rows])
            kn = torch.cat([tok[r][seen[r]][layer][0] for r, _, _ in rows])
            vn = torch.cat([tok[r][seen[r]][layer][1] for r, _, _ in rows])
            out = torch.empty(len(rows), H, D)
            ring.step(layer, positions, q, kn, vn, out, slots=slots)
            for i, (r, _, _) in enumerate(rows):
                keys = [peer[layer][0][0], peer[layer][1][0], own[r][layer][0]] + \
                       [tok[r][j][layer][0] for j in range(seen[r] + 1)]
                vals = [peer[layer][0][1], peer[layer][1][1], own[r][layer][1]] + \
                       [tok[r][j][layer][1] for j in range(seen[r] + 1)]
                want, _ = ro.attn_with_lse(q[i:i + 1].numpy(), torch.cat(keys).numpy(),
                                           torch.cat(vals).numpy(), D ** -0.5, None)
                err = float(np.abs(out[i].numpy() - want[0]).max())
                worst = max(worst, err if np.isfinite(err) else float("inf"))  # NaN must fail
        for r, _, _ in rows:
            seen[r] += 1
    ring.stop()
    # owner's growth: positions p with p mod N == owner, per slot, C's only in slot 0
    own_growth = ring.growth_positions[0]
    return {"worst": worst, "growth_slot0": own_growth[0], "growth_slot1": own_growth[1]}


def test_decode_ring_serving_protocol():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), res
    assert all(isinstance(v, dict) for v in res.values()), res
    assert res[0]["steps"] == res[1]["steps"] == len(SCHEDULE)
    owner = res[WORLD - 1]
    assert owner["worst"] < 1e-5, owner
    # slot 0 holds only C's growth (C restarted it after A), slot 1 B's
    base = sum(PEER_CHUNK)
    steps = {r: sum(1 for rows in SCHEDULE for x in rows if x[0] == r) for r in OWN}
    assert steps == {"A": 3, "B": 5, "C": 3}
    for slot, r in ((0, "C"), (1, "B")):
        pos = [base + OWN[r] + j for j in range(steps[r])]
        assert owner[f"growth_slot{slot}"] == [p for p in pos if p % WORLD == WORLD - 1]


@pytest.mark.parametrize("world", [1])
def test_decode_ring_owner_alone(world):
    """A one-rank ring needs no store: begin_step is a no-op and the owner's
    step is its own partial."""
    RingDecode = _cpu_ops()
    peer, own, tok = _data()
    ring = RingDecode(LAYERS, SLOTS, 16, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32)
    ring.begin_step([0], [OWN["A"]], [0])
    ring.set_chunk(0, 0, *own["A"][0])
    kn, vn, qq = tok["A"][0][0]
    out = torch.empty(1, H, D)
    ring.step(0, [OWN["A"]], qq, kn, vn, out, slots=[0])
    want, _ = ro.attn_with_lse(qq.numpy(), torch.cat([own["A"][0][0], kn]).numpy(),
                               torch.cat([own["A"][0][1], vn]).numpy(), D ** -0.5, None)
    assert np.abs(out.numpy() - want).max() < 1e-5


# ---------------------------------------------------------------------------
# failure paths on the host: a dead peer, a silent owner
# ---------------------------------------------------------------------------
def _dead_peer_rank(rank, port, q):
    """Rank 0 joins the ring and exits without serving; rank 1 (the owner)
    must get an error from its step within the group's timeout."""
    import time

    from hcp_vllm_plugin_b200.ring_decode import RingComm
    RingDecode = _cpu_ops()
    comm = RingComm.standalone("127.0.0.1", port, rank, 2, backend="gloo", timeout_s=5, connect_timeout_s=60)
    ring = RingDecode(1, 1, 8, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32, comm=comm)
    if rank == 0:
        q.put((rank, "left"))
        return
    time.sleep(1.0)
    t0 = time.time()
    ring.begin_step([0], [5], [0])
    try:
        ring.step(0, [5], torch.randn(1, H, D), torch.randn(1, HKV, D), torch.randn(1, HKV, D),
                  torch.empty(1, H, D), slots=[0])
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - the expected failure
        q.put((rank, ("error", time.time() - t0, type(e).__name__)))


def test_owner_step_fails_when_a_peer_is_gone():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dead_peer_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "left"
    assert isinstance(res[1], tuple) and res[1][0] == "error", res[1]
    assert res[1][1] < 60, res[1]                 # bounded by the group's timeout, no hang


def _silent_owner_rank(rank, port, q):
    """The owner joins and never posts a step; the peer's serve loop keeps
    polling the store and returns once its stop event is set."""
    import threading
    import time

    from hcp_vllm_plugin_b200.ring_decode import RingComm
    RingDecode = _cpu_ops()
    comm = RingComm.standalone("127.0.0.1", port, rank, 2, backend="gloo", timeout_s=30, connect_timeout_s=60)
    ring = RingDecode(1, 1, 8, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32, comm=comm)
    if rank == 1:
        time.sleep(3.0)                            # stay in the group while the peer polls
        q.put((rank, "done"))
        return
    stop = threading.Event()
    threading.Timer(1.0, stop.set).start()
    t0 = time.time()
    ring.serve(lambda layer: (torch.zeros(1, HKV, D), torch.zeros(1, HKV, D)), stop=stop, poll_s=0.2)
    q.put((rank, (ring.steps_served, time.time() - t0)))


def test_peer_serve_loop_stops_without_an_owner_step():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_silent_owner_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    steps, waited = res[0]
    assert steps == 0 and 0.9 < waited < 10, res[0]
