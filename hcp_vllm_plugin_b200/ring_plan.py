"""Host-side plan of one attention-layer call: which rows go to the fused
prefill kernel (as work items) and which to the split-KV decode kernel.

Mirrors the per-request bookkeeping of the reference's
``HcpRingAttentionImpl.forward`` (``hcp_vllm_plugin/ring_backend.py:611-832``)
without its per-request launches:

* ``qpos0 = seq_len - q_len`` is the global position of the request's first
  query (``:627``);
* staged peer KV takes precedence over ``HCP_RING_SPLIT_TOKENS``
  (``:738-781``); ``peer_end = min(len(peer), seq_len)``;
* the ``n_a`` queries still inside the peer region attend every key
  causally (``:811-818``); the rest attend the peer keys (non-causal) and the
  local keys ``[peer_end, seq_len)`` causally at offset
  ``qpos0 + n_a - peer_end``, merged by LSE (``:819-832``) - here in one pass;
* a request with a single query token goes to the split-KV decode kernel;
* ``HCP_RING_SPLIT_TOKENS`` (single-instance validation, ``:776-778``): with
  no staged peer the first ``split`` keys of the request's own paged cache
  play the peer chunk - a non-causal paged segment merged with the causal
  remainder in the same launch (``split`` must be block aligned).

No vLLM import: the plan is plain integers and is tested on CPU.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ._capi import HCP_SRC_A, HCP_SRC_PAGED


@dataclass
class LayerPlan:
    work: np.ndarray                 # [n, 12] int32 fused-prefill work items
    decode: np.ndarray               # [m, 6] int32 decode sequences
    peer_parts: list = field(default_factory=list)   # (k, v) tensors, in arena order
    peer_rows: int = 0
    stats: dict = field(default_factory=dict)
    part_requests: list = field(default_factory=list)  # requests whose chunks fill the arena, in order


def plan_layer(query_start_loc, seq_lens, block_size: int, peers: dict, split_tokens: int = 0,
               decode_kernel: bool = True, exclude=frozenset()) -> LayerPlan:
    """Build the plan.

    ``peers`` maps a request index to its ordered list of staged ``(k, v)``
    chunk tensors for this layer (``[T, Hkv, D]`` each), or is missing the
    request when it has none.  ``split_tokens`` > 0 splits the paged cache
    itself when no peer KV is staged (the single-process validation mode).
    Requests in ``exclude`` are computed elsewhere (the decode ring) and get
    no work here.
    """
    qsl = [int(x) for x in query_start_loc]
    lens = [int(x) for x in seq_lens]
    work: list[list[int]] = []
    dec: list[list[int]] = []
    parts: list = []
    part_reqs: list[int] = []
    arena = 0
    stats = {"requests": len(lens), "prefill_rows": 0, "decode_rows": 0, "peer_requests": 0}
    for r, tk in enumerate(lens):
        qs, qe = qsl[r], qsl[r + 1]
        tq = qe - qs
        if tq <= 0 or r in exclude:
            continue
        qpos0 = tk - tq
        chunks = peers.get(r)
        peer_end = 0
        peer_off = 0
        split_mode = False
        if chunks:
            peer_len = sum(int(k.shape[0]) for k, _ in chunks)
            peer_end = min(peer_len, tk)
            peer_off = arena
            parts.extend(chunks)
            part_reqs.append(r)
            arena += peer_len
            stats["peer_requests"] += 1
        elif split_tokens > 0:
            peer_end = min(split_tokens, tk)
            split_mode = True
        if tq == 1 and decode_kernel:
            stats["decode_rows"] += 1
            if peer_end > 0 and not split_mode:
                # query at position tk-1: every key is visible
                dec.append([qs, peer_off, peer_end, r, peer_end, tk - peer_end])
            else:
                dec.append([qs, 0, 0, r, 0, tk])
            continue
        stats["prefill_rows"] += tq
        if peer_end == 0:
            work.append([qs, tq, r, qs, HCP_SRC_PAGED, 0, tk, qpos0, 0, 0, 0, 0])
            continue
        n_a = max(0, min(tq, peer_end - qpos0))
        if n_a > 0:
            work.append([qs, n_a, r, qs, HCP_SRC_PAGED, 0, tk, qpos0, 0, 0, 0, 0])
        if n_a < tq:
            local = tk - peer_end
            seg_local = [HCP_SRC_PAGED, peer_end, local, qpos0 + n_a - peer_end] if local > 0 else [0, 0, 0, 0]
            seg_peer = [HCP_SRC_PAGED, 0, peer_end, -1] if split_mode else [HCP_SRC_A, peer_off, peer_end, -1]
            work.append([qs + n_a, tq - n_a, r, qs + n_a, *seg_peer, *seg_local])
    return LayerPlan(
        work=np.array(work, dtype=np.int32).reshape(-1, 12),
        decode=np.array(dec, dtype=np.int32).reshape(-1, 6),
        peer_parts=parts,
        peer_rows=arena,
        stats=stats,
        part_requests=part_reqs,
    )


def misaligned_paged_starts(plan: LayerPlan, block_size: int) -> bool:
    """True if any paged segment starts off a block boundary (the kernels
    need block-aligned paged starts)."""
    w = plan.work
    for j in (0, 1):
        src = w[:, 4 + 4 * j]
        start = w[:, 5 + 4 * j]
        if np.any((src == HCP_SRC_PAGED) & (start % block_size != 0)):
            return True
    d = plan.decode
    return bool(np.any((d[:, 5] > 0) & (d[:, 4] % block_size != 0)))
