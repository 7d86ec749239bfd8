"""Balanced work plan for ring context-parallel prefill of one long sequence.

The sequence is split into ``world`` contiguous chunks; rank ``x`` durably
owns chunk ``x`` (its queries and its keys/values), exactly the memory-split
ownership of the reference (``ring_connector.py:21-32``: each node holds only
its own chunk's KV).  Causal attention makes the work per rank grow with the
rank: rank ``x`` attends its own chunk causally (half a unit) and every earlier
chunk in full (``x`` units), so a plain ring is limited by the last rank:
``world^2/2`` units over ``world - 0.5`` → at most 4.27x on 8 GPUs.

The plan pairs rank ``r < world/2`` (light) with rank ``s = world-1-r``
(heavy).  The heavy rank hands the first ``give`` rows of its query chunk to
its light partner, which computes their attention over the peer chunks
``0..s-1`` (non-causal) and returns the partial (O, LSE); the heavy rank keeps
the causal diagonal part of those rows and merges.  With
``f = (world-2r-1) / (2(world-1-r))`` both partners end with ``world/2`` units.
Rows are moved in multiples of the 128-row query tile.
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class RingPlan:
    world: int
    chunk: int
    tile: int = 128
    # owner rank -> (helper rank, rows [0, give) handed over)
    give: dict = field(default_factory=dict)

    def helper_of(self, owner: int) -> int | None:
        g = self.give.get(owner)
        return None if g is None else g[0]

    def rows_given(self, owner: int) -> int:
        g = self.give.get(owner)
        return 0 if g is None else g[1]

    def helped_owner(self, helper: int) -> int | None:
        for owner, (h, rows) in self.give.items():
            if h == helper and rows > 0:
                return owner
        return None

    def work_units(self, rank: int) -> float:
        """Attention work of ``rank`` in chunk-pair units (a full chunk x chunk
        block is 1; the causal diagonal block is 0.5)."""
        units = rank + 0.5
        rows = self.rows_given(rank)
        units -= rank * rows / self.chunk
        owner = self.helped_owner(rank)
        if owner is not None:
            units += owner * self.rows_given(owner) / self.chunk
        return units


def plan_balanced(world: int, chunk: int, tile: int = 128, balance: bool = True) -> RingPlan:
    if world < 1 or chunk < 1:
        raise ValueError("world and chunk must be positive")
    give: dict[int, tuple[int, int]] = {}
    if balance and world > 1:
        for r in range(world // 2):
            s = world - 1 - r
            if s == r:
                continue
            f = (world - 2 * r - 1) / (2.0 * (world - 1 - r))
            rows = int(round(f * chunk / tile)) * tile
            rows = max(0, min(chunk, rows))
            if rows > 0:
                give[s] = (r, rows)
    return RingPlan(world=world, chunk=chunk, tile=tile, give=give)


def needs_chunk(plan: RingPlan, x: int, j: int) -> bool:
    """Does rank ``x`` read chunk ``j``'s K/V (``j != x``)?  Its own rows past
    the hand-off see every earlier chunk; the rows it computes for its partner
    ``s`` see chunks ``0..s-1``."""
    if j == x:
        return False
    if j < x and plan.rows_given(x) < plan.chunk:
        return True
    owner = plan.helped_owner(x)
    return owner is not None and j < owner


@dataclass(frozen=True)
class Hop:
    """One step of the chunk rotation on one rank.  At hop ``h`` rank ``x``
    sends its chunk to ``x + h`` and receives chunk ``x - h`` (mod world), each
    only if the receiving rank reads that chunk: every hop is a permutation of
    the ranks, so no link carries two chunks at once."""
    hop: int
    send_to: int | None      # rank that receives this rank's chunk now
    recv_chunk: int | None   # chunk (= its owner's rank) received now
    slot: int                # receive buffer slot, -1 when nothing is received
    own_rows: bool           # this rank's rows past the hand-off attend the chunk
    helper_rows: bool        # the rows computed for the partner attend it


def hop_schedule(plan: RingPlan, x: int, slots: int = 2) -> list[Hop]:
    """The hops of rank ``x`` that move a chunk (in or out), in hop order;
    received chunks cycle through ``slots`` receive buffers."""
    world = plan.world
    owner = plan.helped_owner(x)
    hops, n = [], 0
    for h in range(1, world):
        j, y = (x - h) % world, (x + h) % world
        recv = j if needs_chunk(plan, x, j) else None
        send = y if needs_chunk(plan, y, x) else None
        if recv is None and send is None:
            continue
        slot, own, helper = -1, False, False
        if recv is not None:
            slot, n = n % slots, n + 1
            own = j < x and plan.rows_given(x) < plan.chunk
            helper = owner is not None and j < owner
        hops.append(Hop(h, send, recv, slot, own, helper))
    return hops


def ideal_speedup(plan: RingPlan) -> float:
    """Total work over the slowest rank's work (the scaling bound of the plan)."""
    total = plan.world * plan.world / 2.0
    return total / max(plan.work_units(x) for x in range(plan.world))
