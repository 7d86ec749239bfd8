"""Synchronisation protocol of the forward kernel's named-barrier issuer
(``ring_fwd_kernel<D, F16, NB=true>``, ``csrc/ring_fwd.cuh``), checked on the
CPU before and beside any GPU run.

A named barrier cannot time out, so the protocol itself must guarantee that
every ``bar.sync`` is met.  This model runs the four roles of one CTA - TMA
producer, MMA issuer, softmax warpgroups A and B - as the kernel orders
their steps (mbarrier waits with parity semantics, commits, named-barrier
arrive / sync counted to 160 threads) and asserts, for many work items, that

* every role finishes (no deadlock) and no named-barrier instance ever
  collects more arrivals than its 160 (pairing holds);
* the same holds on the abort path, where every mbarrier wait gives up at
  once and the producer stops early: the events still pair up.

The tile bookkeeping (keys per segment, tiles, ``active``) restates the
kernel's ``segment_keys`` / ``tiles0`` / ``active``.
"""

from __future__ import annotations

import random

import pytest

BLOCK_M, BLOCK_N, STAGES, NB = 128, 128, 2, 160
SRC_NONE = 0


def segment_keys(seg, q0, rows):
    src, _start, length, causal = seg
    if rows <= 0 or src == SRC_NONE or length <= 0:
        return 0
    if causal < 0:
        return length
    return max(0, min(length, causal + q0 + rows))


def tiles_of(work, q0):
    """n_tiles and active(x, t) of the CTA whose first row is q0."""
    q_len, seg0, seg1 = work
    rows = [max(0, min(BLOCK_M, q_len - q0 - x * BLOCK_M)) for x in (0, 1)]
    k0 = [segment_keys(seg0, q0 + x * BLOCK_M, rows[x]) for x in (0, 1)]
    k1 = [segment_keys(seg1, q0 + x * BLOCK_M, rows[x]) for x in (0, 1)]
    tiles0 = (max(k0) + BLOCK_N - 1) // BLOCK_N
    n = tiles0 + (max(k1) + BLOCK_N - 1) // BLOCK_N

    def active(x, t):
        seg_first = t < tiles0
        key0 = (t if seg_first else t - tiles0) * BLOCK_N
        return key0 < (k0[x] if seg_first else k1[x])

    return n, active


def programs(n, active):
    """Step lists of the four roles (the kernel's order, NB = true)."""
    ph = lambda t: (t // STAGES) & 1  # noqa: E731
    prod = [("arrive", "q")]
    for t in range(n):
        s = t % STAGES
        prod += [("wait", f"kempty{s}", ph(t) ^ 1), ("arrive", f"kfull{s}"),
                 ("wait", f"vempty{s}", ph(t) ^ 1), ("arrive", f"vfull{s}")]
    iss = []
    for t in range(n + 1):
        for x in (0, 1):
            pv = t >= 1 and active(x, t - 1)
            if pv:
                iss += [("nsync", f"ev{x}", 32), ("narrive", f"ack{x}", 32), ("arrive", f"odone{x}")]
            if t < n and active(x, t):
                if not pv:
                    iss += [("nsync", f"ev{x}", 32), ("narrive", f"ack{x}", 32)]
                iss += [("arrive", f"sfull{x}")]
        if t >= 1:
            iss.append(("arrive", f"vempty{(t - 1) % STAGES}"))
        if t < n:
            iss.append(("arrive", f"kempty{t % STAGES}"))
    soft = []
    for x in (0, 1):
        acts = [t for t in range(n) if active(x, t)]
        prog = []
        if acts:
            prog += [("wait", "q", 0), ("wait", f"kfull{acts[0] % STAGES}", ph(acts[0])),
                     ("narrive", f"ev{x}", 128)]
        for j, t in enumerate(acts):
            nt = acts[j + 1] if j + 1 < len(acts) else n
            merged = nt == t + 1 and nt < n
            prog.append(("wait", f"sfull{x}", j & 1))
            if j >= 1:
                prog.append(("wait", f"odone{x}", (j - 1) & 1))
            prog.append(("wait", f"vfull{t % STAGES}", ph(t)))
            if merged:
                prog.append(("wait", f"kfull{nt % STAGES}", ph(nt)))
            prog += [("nsync", f"ack{x}", 128), ("narrive", f"ev{x}", 128)]
            if nt < n and not merged:
                prog += [("wait", f"kfull{nt % STAGES}", ph(nt)), ("nsync", f"ack{x}", 128),
                         ("narrive", f"ev{x}", 128)]
        if acts:
            prog += [("wait", f"odone{x}", (len(acts) - 1) & 1), ("nsync", f"ack{x}", 128)]
        soft.append(prog)
    return {"producer": prod, "issuer": iss, "softA": soft[0], "softB": soft[1]}


def run(progs, abort=False, producer_stop=None, rng=None):
    """Interleave the roles until all finish; raise on deadlock or overflow."""
    phases: dict[str, int] = {}          # mbarrier -> completed phases (count-1 barriers)
    named: dict[str, int] = {}           # named barrier -> arrivals in the open instance
    released: dict[str, int] = {}        # named barrier -> completed instances
    waiting: dict[str, tuple[str, int]] = {}   # role -> (barrier, instance it waits for)
    pc = {r: 0 for r in progs}
    if producer_stop is not None:
        progs = dict(progs, producer=progs["producer"][:producer_stop])

    def can_run(role):
        step = progs[role][pc[role]]
        if role in waiting:
            bar, inst = waiting[role]
            return released.get(bar, 0) > inst
        if step[0] == "wait":
            if abort:
                return True
            _, bar, parity = step
            return (phases.get(bar, 0) & 1) != parity
        return True

    def add(bar, k):
        named[bar] = named.get(bar, 0) + k
        if named[bar] > NB:
            raise AssertionError(f"named barrier {bar} overflow ({named[bar]} > {NB})")
        if named[bar] == NB:
            named[bar] = 0
            released[bar] = released.get(bar, 0) + 1

    steps = 0
    while True:
        live = [r for r in progs if pc[r] < len(progs[r])]
        if not live:
            return steps
        ready = [r for r in live if can_run(r)]
        if not ready:
            raise AssertionError(f"deadlock: {[(r, progs[r][pc[r]]) for r in live]}")
        role = rng.choice(ready) if rng else ready[0]
        step = progs[role][pc[role]]
        if role in waiting:                   # a bar.sync that completed
            del waiting[role]
            pc[role] += 1
        elif step[0] == "wait":
            pc[role] += 1
        elif step[0] == "arrive":
            phases[step[1]] = phases.get(step[1], 0) + 1
            pc[role] += 1
        elif step[0] == "narrive":
            add(step[1], step[2])
            pc[role] += 1
        elif step[0] == "nsync":
            inst = released.get(step[1], 0)
            add(step[1], step[2])
            if released.get(step[1], 0) > inst:
                pc[role] += 1                 # this sync completed the instance
            else:
                waiting[role] = (step[1], inst)
        steps += 1


def _work_items(rng, n):
    """Work items like the ring plan's and harsher: peer (non-causal) +
    causal local, causal only, non-causal only, and causal first segments
    with a second segment (tile gaps for the shorter query tile)."""
    items = []
    for _ in range(n):
        q_len = rng.choice([1, 37, 128, 129, 256, 300, 700])
        kind = rng.randrange(4)
        peer = (1, 0, rng.choice([0, 64, 128, 500, 1024]), -1)
        local = (2, 0, q_len + rng.choice([0, 0, 128, 333]), rng.choice([0, 128, 333]))
        if kind == 0:
            items.append((q_len, peer, local))
        elif kind == 1:
            items.append((q_len, local, (SRC_NONE, 0, 0, 0)))
        elif kind == 2:
            items.append((q_len, peer, (SRC_NONE, 0, 0, 0)))
        else:
            items.append((q_len, local, peer))   # causal first, then a second segment
    return items


@pytest.mark.parametrize("seed", range(4))
def test_named_barrier_protocol_pairs_and_completes(seed):
    rng = random.Random(seed)
    gaps = 0
    for work in _work_items(rng, 60):
        q_len = work[0]
        for q0 in range(0, q_len, 2 * BLOCK_M):
            n, active = tiles_of(work, q0)
            acts = [[t for t in range(n) if active(x, t)] for x in (0, 1)]
            gaps += sum(1 for a in acts for i in range(1, len(a)) if a[i] != a[i - 1] + 1)
            progs = programs(n, active)
            run(progs, rng=random.Random(rng.random()))                   # normal path
            run(progs, abort=True, rng=random.Random(rng.random()))       # every wait gives up
            cut = rng.randrange(len(progs["producer"]) + 1)
            run(progs, abort=True, producer_stop=cut, rng=random.Random(rng.random()))
    assert gaps > 0          # the gap events were exercised


def test_model_catches_a_missing_ack():
    """The model is strict: without the ack barrier an aborting warpgroup
    runs ahead and overflows the event barrier (the reason for the ack)."""
    n, active = tiles_of((256, (1, 0, 1024, -1), (2, 0, 256, 0)), 0)
    progs = programs(n, active)
    no_ack = {r: [s for s in p if not (s[0] in ("nsync", "narrive") and s[1].startswith("ack"))]
              for r, p in progs.items()}
    with pytest.raises(AssertionError, match="overflow|deadlock"):
        run(no_ack, abort=True)
