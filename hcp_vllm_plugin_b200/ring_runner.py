"""In-box ring context-parallel prefill over NVLink (one process per GPU).

Replaces the reference's HTTP peer-KV pull and neighbour accumulate-forward
(``ring_connector.py:21-32, 777-859``) inside one 8xB200 box: every layer, the
K/V chunks rotate around the ring over NVLink (NCCL ring all-gather on the
process group's stream) while each rank attends its resident chunk causally;
then the peer chunks, now in local HBM, are attended non-causally and merged
in the kernel epilogue.  The work plan (``ring_schedule.plan_balanced``)
moves query rows from heavy to light ranks so 8 ranks stay balanced.

Per layer on rank x (chunk C tokens, ``give`` rows handed to a helper):
  1. async: all-gather K and V of this layer; owner -> helper: Q[0:give]
  2. own chunk, causal (resident, overlaps step 1) -> fp32 partial (O, LSE)
  3. helper: its partner's Q rows vs chunks [0, s) -> fp32 partial, sent back
  4. rows [give, C) vs chunks [0, x), merged with step 2 in the epilogue
  5. owner: rows [0, give): merge step 2 with the helper's partial
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
            self.acc = torch.empty(c, num_heads, head_dim, dtype=f32, device=device)
            self.acc_lse = torch.empty(num_heads, c, dtype=f32, device=device)
        if self.owner is not None:
            g = self.owner_give
            self.q_help = torch.empty(g, num_heads, head_dim, dtype=dtype, device=device)
            self.o_help = torch.empty(g, num_heads, head_dim, dtype=f32, device=device)
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
        # 1. ring rotation of this layer's K/V (NCCL on its own stream, NVLink)
        hk = dist.all_gather_into_tensor(self.k_all, k, group=g, async_op=True)
        hv = dist.all_gather_into_tensor(self.v_all, v, group=g, async_op=True)
        p2p = []
        if self.give:
            p2p.append(dist.P2POp(dist.isend, q[: self.give], self._peer(self.helper), group=g))
        if self.owner is not None:
            p2p.append(dist.P2POp(dist.irecv, self.q_help, self._peer(self.owner), group=g))
        hq = dist.batch_isend_irecv(p2p) if p2p else []
        # 2. resident chunk, causal: overlaps the rotation
        if x == 0:
            self._attn(q, [(0, c, 0, 0, (A, 0, c, 0), None)], out, lse, k_a=k, v_a=v)
        else:
            self._attn(q, [(0, c, 0, 0, (A, 0, c, 0), None)], self.acc, self.acc_lse, k_a=k, v_a=v)
        hk.wait()
        hv.wait()
        for h in hq:
            h.wait()
        # 3. helper: the partner's rows against its peer chunks [0, s)
        send = []
        if self.owner is not None:
            s, gq = self.owner, self.owner_give
            self._attn(self.q_help, [(0, gq, 0, 0, (A, 0, s * c, -1), None)], self.o_help,
                       self.lse_help, k_a=self.k_all, v_a=self.v_all)
            dst = self._peer(s)
            send = [dist.P2POp(dist.isend, self.o_help, dst, group=g),
                    dist.P2POp(dist.isend, self.lse_help, dst, group=g)]
        # The partial's return is issued before step 4 is launched: a NCCL
        # call waits for the work already queued on the compute stream, so
        # issued here it overlaps step 4 instead of following it.
        recv = []
        if self.give:
            src = self._peer(self.helper)
            recv = [dist.P2POp(dist.irecv, self.o_part, src, group=g),
                    dist.P2POp(dist.irecv, self.lse_part, src, group=g)]
        hs = dist.batch_isend_irecv(send + recv) if (send or recv) else []
        # 4. own rows [give, C) against peer chunks [0, x), merged with step 2
        if x > 0 and self.give < c:
            rows = c - self.give
            self._attn(q, [(self.give, rows, 0, self.give, (A, 0, x * c, -1), None)], out, lse,
                       k_a=self.k_all, v_a=self.v_all, merge_o=self.acc, merge_lse=self.acc_lse)
        for h in hs:
            h.wait()
        # 5. owner: merge the helper's partial for rows [0, give)
        if self.give:
            gv = self.give
            o_lse = None if lse is None else lse[:, :gv]
            self.merge_fn(out[:gv], self.acc[:gv], self.acc_lse[:, :gv], self.o_part,
                          self.lse_part, o_lse)
            self.launches += 1
        return out

    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r
