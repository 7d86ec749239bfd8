"""In-box ring context-parallel prefill over NVLink (one process per GPU).

Replaces the reference's HTTP peer-KV pull and neighbour accumulate-forward
(``ring_connector.py:21-32, 777-859``) inside one 8xB200 box: every layer, the
K/V chunks rotate around the ring over NVLink (NCCL ring all-gather), then
the peer chunks, now in local HBM, and the resident chunk are attended in
one launch.  The work plan (``ring_schedule.plan_balanced``) moves query
rows from heavy to light ranks so 8 ranks stay balanced.

Per layer on rank x (chunk C tokens, ``give`` rows handed to a helper):
  1. all-gather K and V of this layer; owner -> helper: Q[0:give]
  2. ONE launch over every row this rank computes, fp32 out + LSE:
       rows [give, C): peer chunks [0, x) (non-causal) and the own chunk
                       (causal) in one online softmax - final values;
       rows [0, give): the own chunk only (causal) - a partial;
       helper rows:    the partner's Q rows vs its peer chunks [0, s).
     The host orders CTAs heaviest first, so the long peer CTAs start first
     and the short causal ones fill the end of the launch (separate launches
     per part each ended in a partial wave of equally long CTAs).
  3. helper: send its partial back; owner: merge rows [0, give) with it;
     rows [give, C) are cast to the output dtype.
Every rank issues the same collectives in the same order.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _capi as C
from . import ops
from .ring_schedule import RingPlan, plan_balanced


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
                 group=None, balance: bool = True):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if seq_len % self.world:
            raise ValueError("seq_len must split evenly over the ranks")
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
        f32 = torch.float32
        if self.world > 1:
            self.k_all = torch.empty(self.world * c, num_kv_heads, head_dim, dtype=dtype, device=device)
            self.v_all = torch.empty_like(self.k_all)
            # combined rows of the one launch: own chunk rows, then helper rows
            rows = c + self.owner_give
            self.q_comb = torch.empty(rows, num_heads, head_dim, dtype=dtype, device=device)
            self.acc = torch.empty(rows, num_heads, head_dim, dtype=f32, device=device)
            self.acc_lse = torch.empty(num_heads, rows, dtype=f32, device=device)
        if self.owner is not None:
            g = self.owner_give
            self.q_help = self.q_comb[c:]
            self.o_help = self.acc[c:]
            self.lse_help = torch.empty(num_heads, g, dtype=f32, device=device)
        if self.give:
            self.o_part = torch.empty(self.give, num_heads, head_dim, dtype=f32, device=device)
            self.lse_part = torch.empty(num_heads, self.give, dtype=f32, device=device)
        self.launches = 0  # kernels of this library launched (for the bench's count)

    # ------------------------------------------------------------------ helpers
    def _attn(self, q, items, out, lse, **src):
        self.attn_fn(q, ops.make_work(items), scale=self.scale, num_kv_heads=self.Hkv,
                     out=out, lse=lse, **src)
        self.launches += 1

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
                lse: torch.Tensor | None = None) -> torch.Tensor:
        """One attention layer.  q [C, H, D], k/v [C, Hkv, D] of this rank's
        chunk (global positions [x*C, (x+1)*C)); writes out [C, H, D]."""
        x, c = self.rank, self.chunk
        A = C.HCP_SRC_A
        if self.world == 1:
            self._attn(q, [(0, c, 0, 0, (A, 0, c, 0), None)], out, lse, k_a=k, v_a=v)
            return out
        g = self.group
        give = self.give
        # 1. this layer's K/V to every rank (NCCL, NVLink); Q rows to the helper
        hk = dist.all_gather_into_tensor(self.k_all, k, group=g, async_op=True)
        hv = dist.all_gather_into_tensor(self.v_all, v, group=g, async_op=True)
        p2p = []
        if give:
            p2p.append(dist.P2POp(dist.isend, q[:give], self._peer(self.helper), group=g))
        if self.owner is not None:
            p2p.append(dist.P2POp(dist.irecv, self.q_help, self._peer(self.owner), group=g))
        hq = dist.batch_isend_irecv(p2p) if p2p else []
        self.q_comb[:c].copy_(q)
        for h in (hk, hv, *hq):
            h.wait()
        # 2. one launch over all rows of this rank
        own = (A, x * c, c, 0)                      # own chunk, causal
        items = []
        if give:
            items.append((0, give, 0, 0, own, None))
        if give < c:
            if x > 0:
                items.append((give, c - give, 0, give, (A, 0, x * c, -1), (A, x * c, c, give)))
            else:
                items.append((give, c - give, 0, give, (A, x * c, c, give), None))
        if self.owner is not None:
            items.append((c, self.owner_give, 0, c, (A, 0, self.owner * c, -1), None))
        self._attn(self.q_comb, items, self.acc, self.acc_lse, k_a=self.k_all, v_a=self.v_all)
        # 3. helper partial back to its owner; merges and the output cast
        send = []
        if self.owner is not None:
            self.lse_help.copy_(self.acc_lse[:, c:])
            dst = self._peer(self.owner)
            send = [dist.P2POp(dist.isend, self.o_help, dst, group=g),
                    dist.P2POp(dist.isend, self.lse_help, dst, group=g)]
        recv = []
        if give:
            src = self._peer(self.helper)
            recv = [dist.P2POp(dist.irecv, self.o_part, src, group=g),
                    dist.P2POp(dist.irecv, self.lse_part, src, group=g)]
        hs = dist.batch_isend_irecv(send + recv) if (send or recv) else []
        if give < c:
            out[give:].copy_(self.acc[give:c])
            if lse is not None:
                lse[:, give:].copy_(self.acc_lse[:, give:c])
        for h in hs:
            h.wait()
        if give:
            o_lse = None if lse is None else lse[:, :give]
            self.merge_fn(out[:give], self.acc[:give], self.acc_lse[:, :give], self.o_part,
                          self.lse_part, o_lse)
            self.launches += 1
        return out

    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r
