"""Memory-split decode across the GPUs of one box (the decode ring).

The reference (``hcp_vllm_plugin/ring_decode.py``, driven from
``ring_backend.py:630-730``) keeps the context KV split over the ring for
decode too: node r holds its prefill chunk plus its share of the decode
growth (token at global position p goes to node ``p mod N``,
``growth_assignee``, ``ring_decode.py:30-43``), and every decode step of
every layer sends the owner's query with an (O, LSE) accumulator through all
nodes over TCP; each node adds its partial (its chunk + its growth,
non-causal) with ``_merge_pair`` and forwards the packet.  That is N-1
serial network hops per layer per token.

Here the same math runs as one collective step per layer, rank r = node r,
the owner = rank N-1 (the last chunk):

1. the owner broadcasts the step's queries and the new tokens' K/V (one
   NCCL broadcast over NVLink);
2. the assignee of each new token appends it to its growth arena (so the
   token is in this step's partials; the reference ships it one step late
   and counts it in the owner's local partial meanwhile - same keys);
3. every rank computes its partial over its own chunk + growth in its own
   HBM with the split-KV decode kernel, in parallel;
4. the partials (O fp32 [B, H, D], LSE [H, B]) are gathered to the owner
   and merged in one ``hcp_merge_attn_states_n`` launch.

The arena of a rank holds, per layer, one row range per request:
``[chunk rows | growth rows]``, so the partial is one contiguous segment per
request and nothing is concatenated per step.  Every rank calls ``step``
for every layer in the same order.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import ops


def growth_assignee(pos: int, ring_size: int, policy: str = "rr") -> int:
    """Rank that keeps the KV of the decode token at global position ``pos``:
    round-robin ``pos mod N`` (``"rr"``) or always the owner (``"owner"``)."""
    if policy == "owner":
        return ring_size - 1
    if policy != "rr":
        raise ValueError(f"unknown growth policy {policy!r}")
    return pos % ring_size


def _cuda_partial(q, kv_k, kv_v, lens, cap, *, scale, num_kv_heads, out, lse):
    """Partial attention of q[b] over rows [b*cap, b*cap + lens[b]) of the
    arena, written normalised with its natural-log LSE; empty -> (0, -inf)."""
    seqs = [(b, b * cap, int(n), -1, 0, 0) for b, n in enumerate(lens) if n > 0]
    empty = [b for b, n in enumerate(lens) if n <= 0]
    if empty:
        idx = torch.tensor(empty, device=out.device)
        out.index_fill_(0, idx, 0.0)
        lse.index_fill_(1, idx, float("-inf"))
    if seqs:
        ops.decode_splitkv(q, np.array(seqs, np.int32), scale=scale, num_kv_heads=num_kv_heads,
                           out=out, lse=lse, peer_k=kv_k, peer_v=kv_v)


def _cuda_merge(out, states_o, states_lse, out_lse):
    ops.merge_attn_states_n(out, states_o, states_lse, out_lse)


class RingDecode:
    # The device ops.  Tests of the host-side schedule and communication
    # substitute CPU checkers here; the product always runs the CUDA ops.
    partial_fn = staticmethod(_cuda_partial)
    merge_fn = staticmethod(_cuda_merge)

    def __init__(self, num_layers: int, batch: int, capacity: int, num_heads: int, num_kv_heads: int,
                 head_dim: int, scale: float, device: torch.device, dtype: torch.dtype = torch.bfloat16,
                 group=None, growth_policy: str = "rr"):
        """``capacity``: rows per request per layer on this rank (its chunk
        rows plus the largest growth share it will receive)."""
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
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
        # broadcast payload: q [B, H, D] + k_new, v_new [B, Hkv, D]
        self._payload = torch.empty(batch * (h * d + 2 * hkv * d), dtype=dtype, device=device)
        # gathered partials: o [B, H, D] + lse [H, B], fp32, one slot per rank
        self._part = torch.empty(batch * h * d + h * batch, dtype=torch.float32, device=device)
        self._parts = [torch.empty_like(self._part) for _ in range(self.world)] \
            if self.rank == self.owner else None
        self.launches = 0  # kernels of this library launched (for counting in benchmarks)

    # ------------------------------------------------------------------ setup
    def set_chunk(self, layer: int, b: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """This rank's prefill chunk of request ``b`` for ``layer`` ([C, Hkv, D])."""
        c = k.shape[0]
        if c > self.cap:
            raise ValueError(f"chunk of {c} rows exceeds the capacity {self.cap}")
        base = b * self.cap
        self.k[layer, base:base + c].copy_(k)
        self.v[layer, base:base + c].copy_(v)
        self.lens[layer][b] = c
        self.growth_positions[layer][b] = []

    # ------------------------------------------------------------------ step
    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def step(self, layer: int, positions, q: torch.Tensor | None = None, k_new: torch.Tensor | None = None,
             v_new: torch.Tensor | None = None, out: torch.Tensor | None = None,
             out_lse: torch.Tensor | None = None) -> torch.Tensor | None:
        """One decode step of one layer for the whole batch.

        ``positions``: host list of the new tokens' global positions (the
        same on every rank).  On the owner: ``q`` [B, H, D], ``k_new`` /
        ``v_new`` [B, Hkv, D] and ``out`` [B, H, D] (written); other ranks
        pass nothing.  Returns ``out`` on the owner, None elsewhere.
        """
        B, H, D, Hkv = self.B, self.H, self.D, self.Hkv
        nq, nk = B * H * D, B * Hkv * D
        pay = self._payload
        if self.rank == self.owner:
            pay[:nq].view(B, H, D).copy_(q)
            pay[nq:nq + nk].view(B, Hkv, D).copy_(k_new)
            pay[nq + nk:].view(B, Hkv, D).copy_(v_new)
        if self.world > 1:
            dist.broadcast(pay, src=self._peer(self.owner), group=self.group)
        qb = pay[:nq].view(B, H, D)
        kb = pay[nq:nq + nk].view(B, Hkv, D)
        vb = pay[nq + nk:].view(B, Hkv, D)
        lens = self.lens[layer]
        mine, rows = [], []
        for b, pos in enumerate(positions):
            if growth_assignee(int(pos), self.world, self.policy) != self.rank:
                continue
            if lens[b] >= self.cap:
                raise RuntimeError(f"request {b}: growth exceeds the capacity {self.cap} on rank {self.rank}")
            mine.append(b)
            rows.append(b * self.cap + lens[b])
            lens[b] += 1
            self.growth_positions[layer][b].append(int(pos))
        if mine:
            # every token this rank keeps, in one copy for K and one for V
            src = torch.tensor(mine, dtype=torch.long).to(self.device, non_blocking=True)
            dst = torch.tensor(rows, dtype=torch.long).to(self.device, non_blocking=True)
            self.k[layer].index_copy_(0, dst, kb.index_select(0, src))
            self.v[layer].index_copy_(0, dst, vb.index_select(0, src))
        o = self._part[:nq].view(B, H, D)
        lse = self._part[nq:].view(H, B)
        self.partial_fn(qb, self.k[layer], self.v[layer], lens, self.cap, scale=self.scale,
                        num_kv_heads=Hkv, out=o, lse=lse)
        self.launches += 1
        if self.world > 1:
            dist.gather(self._part, self._parts if self.rank == self.owner else None,
                        dst=self._peer(self.owner), group=self.group)
        if self.rank != self.owner:
            return None
        parts = self._parts if self.world > 1 else [self._part]
        states_o = torch.stack([p[:nq].view(B, H, D) for p in parts])
        states_lse = torch.stack([p[nq:].view(H, B) for p in parts])
        self.merge_fn(out, states_o, states_lse, out_lse)
        self.launches += 1
        return out
