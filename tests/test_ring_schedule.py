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
