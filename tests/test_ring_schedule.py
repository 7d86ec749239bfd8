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
