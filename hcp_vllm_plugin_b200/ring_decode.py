"""Memory-split decode across the GPUs of one box (the decode ring).

The reference (``hcp_vllm_plugin/ring_decode.py``, driven from
``ring_backend.py:630-730``) keeps the context KV split over the ring for
decode too: node r holds its prefill chunk plus its share of the decode
growth (token at global position p goes to node ``p mod N``,
``growth_assignee``, ``ring_decode.py:30-43``), and every decode step of
every layer sends the owner's query with an (O, LSE) accumulator through all
nodes over TCP; each node adds its partial (its chunk + its growth,
non-causal) with ``_merge_pair`` and forwards the packet.  That is N-1
serial network hops per layer per token, one packet per request.

Here the same math runs as one collective step per layer for the whole
decode batch, rank r = node r, the owner = rank N-1 (the last chunk):

1. the owner broadcasts the step's queries and the new tokens' K/V (one
   NCCL broadcast over NVLink);
2. the assignee of each new token appends it to its growth rows (so the
   token is in this step's partials; the reference ships it one step late
   and counts it in the owner's local partial meanwhile - same keys);
3. every rank computes its partial over its own chunk + growth in its own
   HBM with the split-KV decode kernel, in parallel;
4. the partials (O fp32 [n, H, D], LSE [H, n]) are gathered to the owner
   and merged in one ``hcp_merge_attn_states_n`` launch.

A rank keeps, per layer, one row range per request slot: ``[chunk rows |
growth rows]``, so a partial is one contiguous segment per request and
nothing is concatenated per step.  Every rank calls ``step`` for every layer
in the same order.

Serving (one vLLM instance per GPU, each with its own default process
group): ``RingComm.standalone`` builds the ring's own c10d group from a
TCPStore.  The owner posts one header per engine step in that store (which
slots decode, their positions, which slots start this step); the peers'
``serve`` loop waits for it on the host, then runs the step's layers in
lockstep with the owner.  Collectives therefore only run while the owner is
decoding; between steps nothing waits on a GPU.
"""

from __future__ import annotations

import datetime
import json
import threading

import numpy as np
import torch
import torch.distributed as dist

from . import _capi, ops

OP_STOP, OP_STEP = 0, 1
_HDR = "hcp_decode_ring/hdr/"
_HDR_KEEP = 64          # step headers kept in the store


def growth_assignee(pos: int, ring_size: int, policy: str = "rr") -> int:
    """Rank that keeps the KV of the decode token at global position ``pos``:
    round-robin ``pos mod N`` (``"rr"``) or always the owner (``"owner"``)."""
    if policy == "owner":
        return ring_size - 1
    if policy != "rr":
        raise ValueError(f"unknown growth policy {policy!r}")
    return pos % ring_size


def _cuda_partial(q, kv_k, kv_v, segs, *, scale, num_kv_heads, out, lse):
    """Partial attention of q[i] over arena rows [start, start + n) for each
    (i, start, n) of ``segs``, written normalised with its natural-log LSE;
    an empty segment gives (0, -inf)."""
    seqs = [(i, s, int(n), -1, 0, 0) for i, s, n in segs if n > 0]
    empty = [i for i, _, n in segs if n <= 0]
    if empty:
        idx = torch.tensor(empty, device=out.device)
        out.index_fill_(0, idx, 0.0)
        lse.index_fill_(1, idx, float("-inf"))
    if seqs:
        ops.decode_splitkv(q, np.array(seqs, np.int32), scale=scale, num_kv_heads=num_kv_heads,
                           out=out, lse=lse, peer_k=kv_k, peer_v=kv_v)


def _cuda_merge(out, states_o, states_lse, out_lse):
    ops.merge_attn_states_n(out, states_o, states_lse, out_lse)


class RingComm:
    """The decode ring's collectives and control plane.

    Either a group of the default world (``group``; the ranks were launched
    together, e.g. by torchrun) or a standalone c10d process group over a
    TCPStore (``standalone``): the form for separately launched processes
    that each already own their default world, as vLLM instances do.  The
    control plane (step headers) needs the store, so ``serve`` /
    ``begin_step`` need the standalone form."""

    def __init__(self, group=None, pg=None, store=None):
        self.group, self.pg, self.store = group, pg, store
        if pg is not None:
            self.rank, self.world = pg.rank(), pg.size()
        elif dist.is_available() and dist.is_initialized():
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1

    @classmethod
    def standalone(cls, host: str, port: int, rank: int, world: int, backend: str = "nccl",
                   timeout_s: float = 300.0, connect_timeout_s: float = 3600.0) -> "RingComm":
        """Join the ring's own group: rank 0 hosts the store at host:port; the
        call returns once all ``world`` ranks have joined.  ``timeout_s``
        bounds every collective (they run only inside a step)."""
        store = dist.TCPStore(host, port, world, rank == 0,
                              timeout=datetime.timedelta(seconds=connect_timeout_s))
        pg_store = dist.PrefixStore("hcp_decode_ring/pg", store)
        td = datetime.timedelta(seconds=timeout_s)
        if backend == "nccl":
            pg = dist.ProcessGroupNCCL(pg_store, rank, world, td)
        elif backend == "gloo":
            pg = dist.ProcessGroupGloo(pg_store, rank, world, td)
        else:
            raise ValueError(f"unknown backend {backend!r}")
        return cls(pg=pg, store=store)

    def close(self) -> None:
        """Shut the standalone group down (its communicators and watchdog);
        a group of the default world belongs to its owner."""
        if self.pg is not None:
            self.pg.shutdown()
            self.pg = None

    def _global(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        if self.world == 1:
            return
        if self.pg is not None:
            o = dist.BroadcastOptions()
            o.rootRank, o.rootTensor = src, 0
            self.pg.broadcast([t], o).wait()
        else:
            dist.broadcast(t, src=self._global(src), group=self.group)

    def gather(self, t: torch.Tensor, dst: int, out: list | None) -> None:
        """``out`` (one tensor per rank) on ``dst``; None elsewhere."""
        if self.world == 1:
            out[0].copy_(t)
            return
        if self.pg is not None:
            o = dist.GatherOptions()
            o.rootRank = dst
            self.pg.gather([out] if self.rank == dst else [], [t], o).wait()
        else:
            dist.gather(t, out if self.rank == dst else None, dst=self._global(dst), group=self.group)

    # -- control plane -------------------------------------------------------
    def post_header(self, seq: int, header: dict) -> None:
        if self.store is None:
            raise RuntimeError("the decode ring's control plane needs RingComm.standalone")
        self.store.set(f"{_HDR}{seq}", json.dumps(header))
        if seq >= _HDR_KEEP:
            # A peer reads header k before it joins step k's collectives, and
            # the owner's host waits for its GPU at least once per engine step
            # (vLLM samples every step), which needs step k's collectives
            # done; so headers this old have been read by every peer.
            self.store.delete_key(f"{_HDR}{seq - _HDR_KEEP}")

    def wait_header(self, seq: int, timeout_s: float) -> dict | None:
        """The owner's header ``seq``, or None if it has not come within
        ``timeout_s`` (the caller polls, so a stop request is seen)."""
        if self.store is None:
            raise RuntimeError("the decode ring's control plane needs RingComm.standalone")
        key = f"{_HDR}{seq}"
        try:
            self.store.wait([key], datetime.timedelta(seconds=timeout_s))
        except Exception:  # noqa: BLE001 - the store reports a timeout as an error
            return None
        return json.loads(self.store.get(key))


class RingDecode:
    # The device ops.  Tests of the host-side schedule and communication
    # substitute CPU checkers here; the product always runs the CUDA ops.
    partial_fn = staticmethod(_cuda_partial)
    merge_fn = staticmethod(_cuda_merge)

    def __init__(self, num_layers: int, batch: int, capacity: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, scale: float, device: torch.device, dtype: torch.dtype = torch.bfloat16,
                 group=None, growth_policy: str = "rr", comm: RingComm | None = None):
        """``batch``: request slots (and the largest decode batch of a step);
        ``capacity``: rows per slot per layer on this rank (its chunk rows
        plus the largest growth share it will receive)."""
        self.comm = comm if comm is not None else RingComm(group=group)
        self.world, self.rank = self.comm.world, self.comm.rank
        self.owner = self.world - 1
        self.L, self.B, self.cap = num_layers, batch, capacity
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim
        self.scale = scale
        self.device = device
        self.dtype = dtype
        self.policy = growth_policy
        self.k = torch.zeros(num_layers, batch * capacity, num_kv_heads, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        # Run the growth append's index kernels once now (row 0 onto itself):
        # a rank that launches them for the first time inside a step loads
        # their module there, and every rank's next collective waits for it.
        idx = torch.zeros(1, dtype=torch.long, device=device)
        self.k[0].index_copy_(0, idx, self.k[0].index_select(0, idx))
        self.lens = [[0] * batch for _ in range(num_layers)]
        self.growth_positions = [[[] for _ in range(batch)] for _ in range(num_layers)]
        h, d, hkv = num_heads, head_dim, num_kv_heads
        # broadcast payload: q [n, H, D] + k_new, v_new [n, Hkv, D]
        self._payload = torch.empty(batch * (h * d + 2 * hkv * d), dtype=dtype, device=device)
        # gathered partials: o [n, H, D] + lse [H, n], fp32, one slot per rank
        self._part = torch.empty(batch * h * d + h * batch, dtype=torch.float32, device=device)
        self._parts = [torch.empty_like(self._part) for _ in range(self.world)] \
            if self.rank == self.owner else None
        self._seq = 0                      # control-plane header sequence
        self.steps_served = 0
        self.launches = 0  # kernels of this library launched (for counting in benchmarks)
        # device-side failures of earlier steps surface as HcpError at the next step
        self._watch = _capi.DeviceStatusWatch() if device.type == "cuda" else None

    # ------------------------------------------------------------------ setup
    def install_rows(self, layer: int, slot: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Start ``slot`` afresh for ``layer`` with an ``n``-row chunk and
        return the K, V row views [n, Hkv, D] to fill with it."""
        if n > self.cap:
            raise ValueError(f"chunk of {n} rows exceeds the capacity {self.cap}")
        base = slot * self.cap
        self.lens[layer][slot] = n
        self.growth_positions[layer][slot] = []
        return self.k[layer, base:base + n], self.v[layer, base:base + n]

    def set_chunk(self, layer: int, slot: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """This rank's prefill chunk of the request in ``slot`` for ``layer``
        ([C, Hkv, D])."""
        kk, vv = self.install_rows(layer, slot, k.shape[0])
        kk.copy_(k)
        vv.copy_(v)

    # ------------------------------------------------------------------ step
    def step(self, layer: int, positions, q: torch.Tensor | None = None, k_new: torch.Tensor | None = None,
             v_new: torch.Tensor | None = None, out: torch.Tensor | None = None,
             out_lse: torch.Tensor | None = None, slots=None) -> torch.Tensor | None:
        """One decode step of one layer for ``n = len(positions)`` requests.

        ``positions``: host list of the new tokens' global positions and
        ``slots`` the requests' slots (default 0..n-1), the same on every
        rank.  On the owner: ``q`` [n, H, D], ``k_new`` / ``v_new``
        [n, Hkv, D] and ``out`` [n, H, D] (written); other ranks pass
        nothing.  Returns ``out`` on the owner, None elsewhere.
        """
        n = len(positions)
        slots = list(range(n)) if slots is None else [int(s) for s in slots]
        if n == 0:
            return out
        if self._watch is not None:
            self._watch.check("decode ring")
        if n > self.B or len(slots) != n:
            raise ValueError(f"a step of {n} requests (slots {slots}) for {self.B} slots")
        H, D, Hkv = self.H, self.D, self.Hkv
        nq, nk = n * H * D, n * Hkv * D
        pay = self._payload[:nq + 2 * nk]
        if self.rank == self.owner:
            pay[:nq].view(n, H, D).copy_(q)
            pay[nq:nq + nk].view(n, Hkv, D).copy_(k_new)
            pay[nq + nk:].view(n, Hkv, D).copy_(v_new)
        self.comm.broadcast(pay, self.owner)
        qb = pay[:nq].view(n, H, D)
        kb = pay[nq:nq + nk].view(n, Hkv, D)
        vb = pay[nq + nk:].view(n, Hkv, D)
        lens = self.lens[layer]
        mine = [i for i, pos in enumerate(positions)
                if growth_assignee(int(pos), self.world, self.policy) == self.rank]
        # every token this rank keeps must fit before any state changes
        extra: dict[int, int] = {}
        for i in mine:
            extra[slots[i]] = extra.get(slots[i], 0) + 1
        for s, e in extra.items():
            if lens[s] + e > self.cap:
                raise RuntimeError(f"slot {s}: growth exceeds the capacity {self.cap} on rank {self.rank}")
        rows = []
        for i in mine:
            s = slots[i]
            rows.append(s * self.cap + lens[s])
            lens[s] += 1
            self.growth_positions[layer][s].append(int(positions[i]))
        if mine:
            # every token this rank keeps, in one copy for K and one for V
            src = torch.tensor(mine, dtype=torch.long).to(self.device, non_blocking=True)
            dst = torch.tensor(rows, dtype=torch.long).to(self.device, non_blocking=True)
            self.k[layer].index_copy_(0, dst, kb.index_select(0, src))
            self.v[layer].index_copy_(0, dst, vb.index_select(0, src))
        part = self._part[:nq + H * n]
        o = part[:nq].view(n, H, D)
        lse = part[nq:].view(H, n)
        segs = [(i, s * self.cap, lens[s]) for i, s in enumerate(slots)]
        self.partial_fn(qb, self.k[layer], self.v[layer], segs, scale=self.scale, num_kv_heads=Hkv,
                        out=o, lse=lse)
        self.launches += 1
        parts = [p[:nq + H * n] for p in self._parts] if self.rank == self.owner else None
        self.comm.gather(part, self.owner, parts)
        if self._watch is not None:
            self._watch.record(torch.cuda.current_stream(self.device))
        if self.rank != self.owner:
            return None
        states_o = torch.stack([p[:nq].view(n, H, D) for p in parts])
        states_lse = torch.stack([p[nq:].view(H, n) for p in parts])
        self.merge_fn(out, states_o, states_lse, out_lse)
        self.launches += 1
        return out

    # ------------------------------------------------------------------ serving
    def begin_step(self, slots, positions, fresh) -> None:
        """Owner, once per engine step before its first layer: tell the peers
        which slots decode (``positions`` of their new tokens) and which of
        them start this step (``fresh``: the peers install their chunk into
        those slots at every layer)."""
        if self.rank != self.owner:
            raise RuntimeError("begin_step is the owner's call")
        if self.world > 1:
            self.comm.post_header(self._seq, {"op": OP_STEP, "slots": [int(s) for s in slots],
                                              "positions": [int(p) for p in positions],
                                              "fresh": [int(s) for s in fresh]})
        self._seq += 1

    def stop(self) -> None:
        """Owner: end the peers' ``serve`` loops."""
        if self.rank == self.owner and self.world > 1:
            self.comm.post_header(self._seq, {"op": OP_STOP})
            self._seq += 1

    def serve(self, chunk_fn, stop: threading.Event | None = None, poll_s: float = 1.0) -> None:
        """Peer loop: for each of the owner's step headers, install this
        rank's chunk (``chunk_fn(layer) -> (k, v)``, [C, Hkv, D]) into the
        step's fresh slots and run every layer's step in order.  Returns on
        the owner's stop header or when ``stop`` is set."""
        if self.rank == self.owner:
            raise RuntimeError("serve is the peers' loop")
        while stop is None or not stop.is_set():
            hdr = self.comm.wait_header(self._seq, poll_s)
            if hdr is None:
                continue
            self._seq += 1
            if hdr["op"] == OP_STOP:
                return
            slots, positions, fresh = hdr["slots"], hdr["positions"], hdr["fresh"]
            for layer in range(self.L):
                if fresh:
                    k, v = chunk_fn(layer)
                    for s in fresh:
                        self.set_chunk(layer, s, k, v)
                self.step(layer, positions, slots=slots)
            self.steps_served += 1
