"""In-box ring context-parallel prefill over NVLink (one process per GPU).

Replaces the reference's HTTP peer-KV pull and neighbour accumulate-forward
(``ring_connector.py:21-32, 777-859``) inside one 8xB200 box.  Rank ``x``
durably owns contiguous chunk ``x`` (its q/k/v); every layer, the earlier
chunks it reads arrive hop by hop over NVLink while it computes, and only
the chunks a rank reads are moved.  The work plan
(``ring_schedule.plan_balanced``) moves query rows from heavy to light ranks
so 8 ranks stay balanced.

Per layer on rank x (chunk C, ``give`` rows handed to a helper, P ranks):

* caller's stream (lowest priority), at once:
    own rows [0, C) vs the own chunk, causal  ->  acc_own (fp32 O, LSE)
* communication stream, hop by hop h = 1..P-1: chunk x-h is brought into
  one of two receive slots if this rank reads it; a slot is refilled only
  after the launch that read it has finished.
* hop stream (high priority), one launch per received chunk, each merging
  into the previous one's (O, LSE) in its epilogue (acc_peer):
    own rows [give, C) vs the chunk when it precedes x, and the rows computed
    for the partner vs the chunk when it precedes the partner (the first such
    launch also attends the helper's own chunk for those rows).
  The high priority lets each hop launch take the SMs first; the causal
  launch's short CTAs fill the tail of each hop launch.
* end: the helper returns its partner's partial (O, LSE); the caller's
  stream merges acc_own with acc_peer for rows [give, C) and acc_own with the
  returned partial for rows [0, give), writing the output dtype directly.

Transports (``transport=``):

* ``"ce"`` (default on CUDA): every rank copies its K/V (and the Q rows its
  helper computes) into an outbox buffer exported once by CUDA IPC; after one
  4-byte all-reduce per layer (every outbox filled) each receiver pulls the
  chunks it reads from the owners' outboxes with the copy engine, when its
  slot is free.  No SM waits on a peer: a NCCL kernel posted before its peer
  is ready holds SMs until the peer arrives, which on 8 ranks cost more than
  the transfers.  Outboxes alternate between two buffers by layer parity; a
  rank refills one only after the next layer's all-reduce, which every rank
  reaches after its pulls of the layer before.
* ``"p2p"``: NCCL send/recv per hop (the only transport of a CPU / gloo
  group, where the tests of the schedule run).

The partials go back by NCCL send/recv; the owner posts its receive once its
own hop launches end.  TMA reads only this GPU's HBM: received chunks sit in
local slots.  Every rank issues its collectives in the same order.
"""

from __future__ import annotations

import contextlib
import ctypes

import torch
import torch.distributed as dist

from . import _capi as C
from . import ops
from .ring_schedule import Hop, RingPlan, hop_schedule, plan_balanced


def _cuda_attn(q, work, *, scale, num_kv_heads, out, lse, **src):
    ops.ring_attn_fwd(q, work, scale=scale, num_kv_heads=num_kv_heads, out=out, lse=lse, **src)


def _cuda_merge(out, prefix_o, prefix_lse, suffix_o, suffix_lse, out_lse):
    ops.merge_attn_states(out, prefix_o, prefix_lse, suffix_o, suffix_lse, out_lse)


class RingPrefill:
    # The device ops.  Tests of the host-side schedule and communication
    # substitute CPU checkers here; the product always runs the CUDA ops.
    attn_fn = staticmethod(_cuda_attn)
    merge_fn = staticmethod(_cuda_merge)

    def __init__(self, seq_len: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 scale: float, device: torch.device, dtype: torch.dtype = torch.bfloat16,
                 group=None, balance: bool = True, slots: int = 2, transport: str | None = None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if seq_len % self.world:
            raise ValueError("seq_len must split evenly over the ranks")
        if slots < 1:
            raise ValueError("slots must be >= 1")
        self.chunk = seq_len // self.world
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim
        self.scale = scale
        self.device = device
        self.dtype = dtype
        self.plan: RingPlan = plan_balanced(self.world, self.chunk, balance=balance)
        x, c = self.rank, self.chunk
        self.give = self.plan.rows_given(x)
        self.helper = self.plan.helper_of(x) if self.give else None
        self.owner = self.plan.helped_owner(x)
        self.owner_give = self.plan.rows_given(self.owner) if self.owner is not None else 0
        self.hops: list[Hop] = hop_schedule(self.plan, x, slots) if self.world > 1 else []
        recv_hops = [h for h in self.hops if h.recv_chunk is not None]
        self.own_peer = any(h.own_rows for h in recv_hops)
        help_hops = [h for h in recv_hops if h.helper_rows]
        # the first hop launch writes acc_peer without merging, so it must
        # cover every row group a later hop launch merges into
        if recv_hops and ((self.own_peer and not recv_hops[0].own_rows)
                          or (help_hops and not recv_hops[0].helper_rows)):
            raise RuntimeError(f"ring plan: rank {x}'s first received chunk does not cover all its rows")
        f32 = torch.float32
        g = self.owner_give
        self.slot_k: list[torch.Tensor] = []
        self.slot_v: list[torch.Tensor] = []
        if self.world > 1:
            ns = min(slots, len(recv_hops))
            self.slot_k = [torch.empty(c, num_kv_heads, head_dim, dtype=dtype, device=device) for _ in range(ns)]
            self.slot_v = [torch.empty_like(t) for t in self.slot_k]
            self.acc_own = torch.empty(c, num_heads, head_dim, dtype=f32, device=device)
            self.lse_own = torch.empty(num_heads, c, dtype=f32, device=device)
            # acc_peer rows: own rows [0, C), then the partner's rows
            rows = c + g
            self.acc_peer = torch.empty(rows, num_heads, head_dim, dtype=f32, device=device)
            self.lse_peer = torch.empty(num_heads, rows, dtype=f32, device=device)
            self.q_comb = torch.empty(rows, num_heads, head_dim, dtype=dtype, device=device) if g else None
        if g:
            self.lse_help = torch.empty(num_heads, g, dtype=f32, device=device)
        if self.give:
            self.o_part = torch.empty(self.give, num_heads, head_dim, dtype=f32, device=device)
            self.lse_part = torch.empty(num_heads, self.give, dtype=f32, device=device)
        self._cuda = device.type == "cuda"
        if transport is None:
            transport = "ce" if self._cuda else "p2p"
        if transport not in ("ce", "p2p") or (transport == "ce" and not self._cuda):
            raise ValueError(f"ring prefill: transport {transport!r} (ce needs CUDA tensors; p2p works on both)")
        self.transport = transport if self.world > 1 else "none"
        if self._cuda and self.world > 1:
            self.s_hop = torch.cuda.Stream(device, priority=-100)   # clamped to the highest
            self.s_comm = torch.cuda.Stream(device, priority=-100)
            self.slot_free = [torch.cuda.Event() for _ in self.slot_k]
        # device-side failures of earlier layers surface as HcpError at the next
        self._watch = C.DeviceStatusWatch() if self._cuda else None
        self._peer_bases: list[int] = []
        if self.world > 1:
            # NCCL wants every rank of a group in its first collective; the
            # per-hop send/recv calls involve only pairs
            dist.barrier(group=group)
        if self.transport == "ce":
            self._open_outboxes()
        self.launches = 0  # kernels of this library launched (for the bench's count)

    # ------------------------------------------------------------------ ce transport
    def _box_offsets(self, rank: int, parity: int) -> tuple[int, int, int]:
        """Element offsets of K, V and the handed-off Q rows in parity half
        ``parity`` of ``rank``'s outbox (its halves hold its own ``give``)."""
        kv = self.chunk * self.Hkv * self.D
        base = parity * (2 * kv + self.plan.rows_given(rank) * self.H * self.D)
        return base, base + kv, base + 2 * kv

    def _open_outboxes(self) -> None:
        """Allocate this rank's outbox (two parity halves of [K | V | Q rows
        [0, give)]), export it, and map the outboxes of the ranks whose chunk
        or Q rows this rank reads.  Collective.  If any rank cannot export
        or map (memory that CUDA IPC cannot share, e.g. an allocator with
        expandable segments), every rank falls back to the p2p transport
        together, so all take the same collective steps."""
        c, hkv, h, d = self.chunk, self.Hkv, self.H, self.D
        self.outbox = torch.empty(2, 2 * c * hkv * d + self.give * h * d, dtype=self.dtype, device=self.device)
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_int64()
        lib = C.load()
        rc = lib.hcp_ipc_export(self.outbox.data_ptr(), handle, ctypes.byref(offset))
        mine = (bytes(handle).hex(), int(offset.value)) if rc == C.HCP_OK else None
        allx: list = [None] * self.world
        dist.all_gather_object(allx, mine, group=self.group)
        need = {hp.recv_chunk for hp in self.hops if hp.recv_chunk is not None}
        if self.owner_give:
            need.add(self.owner)
        self._elt = self.outbox.element_size()
        self._peer_box: dict[int, int] = {}
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        ok = all(x is not None for x in allx)
        if ok:
            for r in sorted(need):
                hx, off = allx[r]
                base = ctypes.c_void_p()
                if lib.hcp_ipc_open(bytes.fromhex(hx), dev, ctypes.byref(base)) != C.HCP_OK:
                    ok = False
                    break
                self._peer_bases.append(base.value)
                self._peer_box[r] = base.value + off
        oks: list = [None] * self.world
        dist.all_gather_object(oks, ok, group=self.group)
        if not all(oks):
            self.close()
            self.outbox = None
            self.transport = "p2p"
            return
        self._sig = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._parity = 0

    def _pull(self, dst: torch.Tensor, rank: int, elem_off: int, stream) -> None:
        """Copy engine: ``dst.numel()`` elements of ``rank``'s outbox from
        element ``elem_off`` into ``dst`` (stream-ordered)."""
        src = self._peer_box[rank] + elem_off * self._elt
        C.check(C.load().hcp_peer_copy(dst.data_ptr(), src, dst.numel() * self._elt, stream.cuda_stream),
                "hcp_peer_copy")

    def close(self) -> None:
        """Unmap the peers' outboxes (the buffers stay with their owners)."""
        lib = C.load() if self._peer_bases else None
        for b in self._peer_bases:
            lib.hcp_ipc_close(b)
        self._peer_bases = []

    # ------------------------------------------------------------------ helpers
    def _attn(self, q, items, out, lse, **src):
        self.attn_fn(q, ops.make_work(items), scale=self.scale, num_kv_heads=self.Hkv,
                     out=out, lse=lse, **src)
        self.launches += 1

    def _merge(self, out, a, la, b, lb, out_lse):
        self.merge_fn(out, a, la, b, lb, out_lse)
        self.launches += 1

    @staticmethod
    def _on(stream):
        return torch.cuda.stream(stream) if stream is not None else contextlib.nullcontext()

    @staticmethod
    def _record(stream):
        if stream is None:
            return None
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev

    @staticmethod
    def _p2p(ops_):
        return dist.batch_isend_irecv(ops_) if ops_ else []

    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    # ------------------------------------------------------------------ forward
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                lse: torch.Tensor | None = None) -> torch.Tensor:
        """One attention layer.  q [C, H, D], k/v [C, Hkv, D] (contiguous) of
        this rank's chunk (global positions [x*C, (x+1)*C)); writes out
        [C, H, D] (and lse [H, C]) in stream order on the caller's current
        stream."""
        x, c = self.rank, self.chunk
        A, B = C.HCP_SRC_A, C.HCP_SRC_B
        if self._watch is not None:
            self._watch.check("ring prefill")
        if self.world == 1:
            self._attn(q, [(0, c, 0, 0, (A, 0, c, 0), None)], out, lse, k_a=k, v_a=v)
            if self._watch is not None:
                self._watch.record(torch.cuda.current_stream(self.device))
            return out
        if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
            raise ValueError("ring prefill: q, k and v must be contiguous (they are sent as they are)")
        grp = self.group
        give, g = self.give, self.owner_give
        ce = self.transport == "ce"
        s0 = torch.cuda.current_stream(self.device) if self._cuda else None
        s_hop = self.s_hop if self._cuda else None
        s_comm = self.s_comm if self._cuda else None
        if g:
            self.q_comb[:c].copy_(q)
        ev_in = self._record(s0)
        # 1. own rows vs the own chunk, causal: no communication needed
        self._attn(q, [(0, c, 0, 0, (A, 0, c, 0), None)], self.acc_own, self.lse_own, k_a=k, v_a=v)
        # 2. communication: Q rows to the helper, then the hops
        if self._cuda:
            s_comm.wait_event(ev_in)
            s_hop.wait_event(ev_in)
        send_works: list = []
        par = 0
        if ce:
            par = self._parity
            self._parity ^= 1
            k_off, v_off, q_off = self._box_offsets(x, par)
            with self._on(s_comm):
                box = self.outbox.view(-1)
                kv = c * self.Hkv * self.D
                box[k_off:k_off + kv].view_as(k).copy_(k)
                box[v_off:v_off + kv].view_as(v).copy_(v)
                if give:
                    box[q_off:q_off + give * self.H * self.D].view(give, self.H, self.D).copy_(q[:give])
                # every outbox of this layer is filled (and, in each rank's
                # stream order, its pulls of the layer before are done)
                dist.all_reduce(self._sig, op=dist.ReduceOp.MAX, group=grp, async_op=True).wait()
                if g:
                    self._pull(self.q_comb[c:], self.owner, self._box_offsets(self.owner, par)[2], s_comm)
            ev_q = self._record(s_comm) if g else None
        else:
            with self._on(s_comm):
                q_ops = []
                if give:
                    q_ops.append(dist.P2POp(dist.isend, q[:give], self._peer(self.helper), group=grp))
                if g:
                    q_ops.append(dist.P2POp(dist.irecv, self.q_comb[c:], self._peer(self.owner), group=grp))
                q_works = self._p2p(q_ops)
            if g:
                with self._on(s_hop):
                    for w in q_works:
                        w.wait()
            send_works = list(q_works) if give else []
        qsrc = self.q_comb if g else q
        first = True
        used = [False] * len(self.slot_k)
        for hop in self.hops:
            s = hop.slot
            if ce and hop.recv_chunk is None:
                continue          # the receivers pull: nothing to do for a send
            with self._on(s_comm):
                if s >= 0 and used[s] and self._cuda:
                    s_comm.wait_event(self.slot_free[s])
                works = []
                if ce:
                    pk, pv, _ = self._box_offsets(hop.recv_chunk, par)
                    self._pull(self.slot_k[s], hop.recv_chunk, pk, s_comm)
                    self._pull(self.slot_v[s], hop.recv_chunk, pv, s_comm)
                    ev_chunk = self._record(s_comm)
                else:
                    hop_ops = []
                    if hop.send_to is not None:
                        dst = self._peer(hop.send_to)
                        hop_ops += [dist.P2POp(dist.isend, k, dst, group=grp),
                                    dist.P2POp(dist.isend, v, dst, group=grp)]
                    if hop.recv_chunk is not None:
                        src = self._peer(hop.recv_chunk)
                        hop_ops += [dist.P2POp(dist.irecv, self.slot_k[s], src, group=grp),
                                    dist.P2POp(dist.irecv, self.slot_v[s], src, group=grp)]
                    works = self._p2p(hop_ops)
            if hop.recv_chunk is None:
                # only sends: waited for at the end.  A hop that also receives
                # is waited for on the hop stream below, which the caller's
                # stream waits for (a work is waited for once: gloo blocks on
                # a second wait)
                send_works += works
                continue
            with self._on(s_hop):
                if ce:
                    s_hop.wait_event(ev_chunk)     # after the Q rows' pull too (stream order)
                for w in works:
                    w.wait()
                items = []
                if hop.own_rows:
                    items.append((give, c - give, 0, give, (A, 0, c, -1), None))
                if hop.helper_rows:
                    # the first launch over the partner's rows also attends this rank's own chunk
                    items.append((c, g, 0, c, (A, 0, c, -1), (B, 0, c, -1) if first else None))
                merge = {} if first else {"merge_o": self.acc_peer, "merge_lse": self.lse_peer}
                self._attn(qsrc, items, self.acc_peer, self.lse_peer, k_a=self.slot_k[s], v_a=self.slot_v[s],
                           k_b=k, v_b=v, **merge)
                if self._cuda:
                    self.slot_free[s].record(s_hop)
            used[s] = True
            first = False
        if g and first:
            # a helper that receives nothing: the partner's rows see only this chunk
            with self._on(s_hop):
                if ce:
                    s_hop.wait_event(ev_q)
                self._attn(qsrc, [(c, g, 0, c, (A, 0, c, -1), None)], self.acc_peer, self.lse_peer,
                           k_a=k, v_a=v)
        # 3. partials back to the owners (NCCL; a posted NCCL kernel holds SMs
        # until its peer arrives, so each side posts once its own launches end)
        ret_works = []
        if g:
            with self._on(s_hop):
                self.lse_help.copy_(self.lse_peer[:, c:])
            ev_help = self._record(s_hop)
            with self._on(s_comm):
                if self._cuda:
                    s_comm.wait_event(ev_help)
                dst = self._peer(self.owner)
                send_works += self._p2p([dist.P2POp(dist.isend, self.acc_peer[c:], dst, group=grp),
                                         dist.P2POp(dist.isend, self.lse_help, dst, group=grp)])
        if give:
            with self._on(s_comm):
                if self._cuda:
                    s_comm.wait_stream(s_hop)
                src = self._peer(self.helper)
                ret_works = self._p2p([dist.P2POp(dist.irecv, self.o_part, src, group=grp),
                                       dist.P2POp(dist.irecv, self.lse_part, src, group=grp)])
        # 4. the caller's stream: wait for the hops, merge, write the output dtype
        if self._cuda:
            s0.wait_stream(s_hop)
        if give < c:
            o_lse = None if lse is None else lse[:, give:]
            if self.own_peer:
                self._merge(out[give:], self.acc_own[give:], self.lse_own[:, give:], self.acc_peer[give:c],
                            self.lse_peer[:, give:c], o_lse)
            else:
                out[give:].copy_(self.acc_own[give:])
                if o_lse is not None:
                    o_lse.copy_(self.lse_own[:, give:])
        if give:
            for w in ret_works:
                w.wait()
            o_lse = None if lse is None else lse[:, :give]
            self._merge(out[:give], self.acc_own[:give], self.lse_own[:, :give], self.o_part, self.lse_part,
                        o_lse)
        # the caller may overwrite q/k/v once this returns: wait for the sends
        # (and, with ce, for the outbox copies on the communication stream)
        for w in send_works:
            w.wait()
        if self._cuda:
            s0.wait_stream(s_comm)
        if self._watch is not None:
            self._watch.record(s0)
        return out
