"""Host logic of the balanced ring plan (no GPU)."""

import pytest

from hcp_vllm_plugin_b200.ring_schedule import ideal_speedup, plan_balanced


@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 8])
def test_plan_conserves_work_and_balances(world):
    chunk = 131072 // world if 131072 % world == 0 else 16384
    plan = plan_balanced(world, chunk)
    total = sum(plan.work_units(x) for x in range(world))
    assert abs(total - world * world / 2.0) < 1e-9  # work is moved, never lost
    for owner, (helper, rows) in plan.give.items():
        assert rows % 128 == 0 and 0 < rows <= chunk // 2
        assert helper == world - 1 - owner and helper < owner
    if world in (1, 2, 4, 8):
        assert ideal_speedup(plan) > 0.97 * world


def test_plain_ring_bound():
    # without balancing the last rank limits 8 GPUs to 32/7.5 = 4.27x
    plan = plan_balanced(8, 16384, balance=False)
    assert abs(ideal_speedup(plan) - 32 / 7.5) < 1e-9
    assert ideal_speedup(plan_balanced(8, 16384)) > 7.8


@pytest.mark.parametrize("world", [2, 3, 4, 5, 6, 7, 8, 16])
@pytest.mark.parametrize("balance", [True, False])
def test_hop_schedule_pairs_and_coverage(world, balance):
    """Every send meets its receive at the same hop, each hop is a permutation
    (a rank sends and receives at most one chunk), every chunk a rank reads
    arrives exactly once, slots alternate, and the first received chunk
    covers every row group a later one is merged into."""
    from hcp_vllm_plugin_b200.ring_schedule import hop_schedule, needs_chunk
    plan = plan_balanced(world, 1024, balance=balance)
    sched = {x: {h.hop: h for h in hop_schedule(plan, x)} for x in range(world)}
    for x in range(world):
        got = []
        for h in sched[x].values():
            if h.send_to is not None:
                peer = sched[h.send_to].get(h.hop)
                assert peer is not None and peer.recv_chunk == x
            if h.recv_chunk is not None:
                peer = sched[h.recv_chunk].get(h.hop)
                assert peer is not None and peer.send_to == x
                got.append(h.recv_chunk)
                assert h.own_rows or h.helper_rows
        assert sorted(got) == [j for j in range(world) if needs_chunk(plan, x, j)]
        recv = [h for h in sorted(sched[x].values(), key=lambda h: h.hop) if h.recv_chunk is not None]
        assert [h.slot for h in recv] == [i % 2 for i in range(len(recv))]
        if recv:
            assert recv[0].own_rows or not any(h.own_rows for h in recv)
            assert recv[0].helper_rows or not any(h.helper_rows for h in recv)
    # moved bytes: only what is read, never more than an all-gather
    moved = sum(len([h for h in sched[x].values() if h.recv_chunk is not None]) for x in range(world))
    assert moved <= world * (world - 1)


def test_outbox_pulls_stay_inside_the_owners_outbox():
    """Every copy-engine pull of the ce transport (K, V of a received chunk;
    the partner's Q rows) reads inside the source rank's outbox, for both
    parity halves, and the halves do not overlap."""
    from types import SimpleNamespace

    from hcp_vllm_plugin_b200.ring_runner import RingPrefill
    from hcp_vllm_plugin_b200.ring_schedule import hop_schedule

    H, HKV, D = 28, 4, 128
    for world in (2, 3, 4, 5, 6, 8):
        chunk = 2048
        plan = plan_balanced(world, chunk)
        kv = chunk * HKV * D
        size = {r: 2 * (2 * kv + plan.rows_given(r) * H * D) for r in range(world)}
        for x in range(world):
            me = SimpleNamespace(chunk=chunk, Hkv=HKV, H=H, D=D, plan=plan)
            pulls = [(hp.recv_chunk, "k") for hp in hop_schedule(plan, x) if hp.recv_chunk is not None]
            pulls += [(hp.recv_chunk, "v") for hp in hop_schedule(plan, x) if hp.recv_chunk is not None]
            owner = plan.helped_owner(x)
            if owner is not None and plan.rows_given(owner):
                pulls.append((owner, "q"))
            for r, what in pulls:
                for par in (0, 1):
                    k_off, v_off, q_off = RingPrefill._box_offsets(me, r, par)
                    off, n = {"k": (k_off, kv), "v": (v_off, kv),
                              "q": (q_off, plan.rows_given(r) * H * D)}[what]
                    assert 0 <= off and off + n <= size[r], (world, x, r, what, par)
                    assert n > 0
                    # parity halves are disjoint
                    half = size[r] // 2
                    assert (off >= half) == (par == 1) and (off + n <= half) == (par == 0)


def _model_layer_time(world: int, chunk: int, slots: int = 2, xfer: float = 0.01) -> float:
    """Per-layer time of the hop schedule in units of one C x C block of
    attention work, when a chunk lands ``xfer`` after both its owner and its
    receiver are ready and a receive slot frees when the launch that read it
    ends (the copy-engine transport: waiting holds no SMs).  The own causal
    launch (0.5 units) fills the gaps of the hop stream."""
    from hcp_vllm_plugin_b200.ring_schedule import hop_schedule

    plan = plan_balanced(world, chunk)
    end = {}
    for x in range(world):
        give = plan.rows_given(x)
        owner = plan.helped_owner(x)
        g = plan.rows_given(owner) if owner is not None else 0
        t, busy, first, free = 0.0, 0.0, True, {}
        for hp in hop_schedule(plan, x, slots):
            if hp.recv_chunk is None:
                continue
            rows = (chunk - give if hp.own_rows else 0) + (g * (2 if first else 1) if hp.helper_rows else 0)
            start = max(t, free.get(hp.slot, 0.0) + xfer)
            t = start + rows / chunk
            busy += rows / chunk
            free[hp.slot] = t
            first = False
        # the causal launch runs in the gaps; whatever is left runs after
        gaps = t - busy
        end[x] = t + max(0.0, 0.5 - gaps)
    return max(end.values())


@pytest.mark.parametrize("world", [2, 3, 4, 5, 6, 8])
def test_hop_schedule_model_is_balanced(world):
    """With waits that hold no SMs, the balanced plan's hop schedule comes
    within 3% of the ideal per-layer time (world / 2 blocks of C x C work)."""
    t = _model_layer_time(world, 16384)
    ideal = world / 2.0
    assert t <= ideal * 1.03 + 0.02, (world, t, ideal)
