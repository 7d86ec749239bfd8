"""Host-side plan of one attention-layer call: which rows go to the fused
prefill kernel (as work items) and which to the split-KV decode kernel.

Mirrors the per-request bookkeeping of the reference's
``HcpRingAttentionImpl.forward`` (``hcp_vllm_plugin/ring_backend.py:611-832``)
without its per-request launches:

* ``qpos0 = seq_len - q_len`` is the global position of the request's first
  query (``:627``);
* staged peer KV takes precedence over ``HCP_RING_SPLIT_TOKENS``
  (``:738-781``); ``peer_end = min(len(peer), seq_len)``; the reference
  concatenates a request's ordered chunks into one peer segment
  (``:751-772``) - here each chunk stays where it is staged and is one
  segment of the request's work item;
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

from ._capi import HCP_MAX_EXT_SOURCES, HCP_MAX_ITEM_SEGMENTS, HCP_SRC_EXT0, HCP_SRC_LIST, HCP_SRC_PAGED

CONCAT = -1  # chunk index of a source that is a request's chunks concatenated


@dataclass
class LaunchGroup:
    """The kernels of one group of requests: every staged chunk they read is
    one extra contiguous source (at most HCP_MAX_EXT_SOURCES per group)."""
    work: np.ndarray                 # [n, 12] int32 fused-prefill work items
    seg_list: np.ndarray             # [m, 4] int32 segments of HCP_SRC_LIST items
    decode: np.ndarray               # [d, 6] int32 decode sequences
    peer_src: np.ndarray             # [d] int32 extra source of each decode sequence's peer keys
    sources: list = field(default_factory=list)  # (request, chunk index or CONCAT) per extra source


@dataclass
class LayerPlan:
    groups: list
    stats: dict = field(default_factory=dict)
    concat_requests: list = field(default_factory=list)  # requests with more chunks than one item holds

    @property
    def work(self) -> np.ndarray:
        return np.concatenate([g.work for g in self.groups]) if self.groups else np.zeros((0, 12), np.int32)

    @property
    def decode(self) -> np.ndarray:
        return np.concatenate([g.decode for g in self.groups]) if self.groups else np.zeros((0, 6), np.int32)


class _Group:
    def __init__(self):
        self.work, self.seg_list, self.decode, self.peer_src, self.sources = [], [], [], [], []

    def freeze(self) -> LaunchGroup:
        return LaunchGroup(work=np.array(self.work, dtype=np.int32).reshape(-1, 12),
                           seg_list=np.array(self.seg_list, dtype=np.int32).reshape(-1, 4),
                           decode=np.array(self.decode, dtype=np.int32).reshape(-1, 6),
                           peer_src=np.array(self.peer_src, dtype=np.int32).reshape(-1),
                           sources=self.sources)

    def item(self, qs, tq, r, segs):
        """A work item over ``segs``: inline when two or fewer, else a list."""
        if len(segs) <= 2:
            segs = list(segs) + [[0, 0, 0, 0]] * (2 - len(segs))
            self.work.append([qs, tq, r, qs, *segs[0], *segs[1]])
        else:
            first = len(self.seg_list)
            self.seg_list.extend(segs)
            self.work.append([qs, tq, r, qs, HCP_SRC_LIST, first, len(segs), 0, 0, 0, 0, 0])


def plan_layer(query_start_loc, seq_lens, block_size: int, peers: dict, split_tokens: int = 0,
               decode_kernel: bool = True, exclude=frozenset()) -> LayerPlan:
    """Build the plan.

    ``peers`` maps a request index to its ordered list of staged ``(k, v)``
    chunk tensors for this layer (``[T, Hkv, D]`` each), or is missing the
    request when it has none.  Each chunk is read where it lies (an extra
    source of the kernels), so nothing is concatenated, except for a request
    with more chunks than one work item has segments for.
    ``split_tokens`` > 0 splits the paged cache itself when no peer KV is
    staged (the single-process validation mode).  Requests in ``exclude`` are
    computed elsewhere (the decode ring) and get no work here.
    """
    qsl = [int(x) for x in query_start_loc]
    lens = [int(x) for x in seq_lens]
    groups: list[_Group] = []
    cur = _Group()
    concat: list[int] = []
    stats = {"requests": len(lens), "prefill_rows": 0, "decode_rows": 0, "peer_requests": 0}
    for r, tk in enumerate(lens):
        qs, qe = qsl[r], qsl[r + 1]
        tq = qe - qs
        if tq <= 0 or r in exclude:
            continue
        qpos0 = tk - tq
        chunks = peers.get(r)
        peer_end = 0
        peer_segs: list[list[int]] = []
        split_mode = False
        if chunks:
            lens_c = [int(k.shape[0]) for k, _ in chunks]
            peer_end = min(sum(lens_c), tk)
            stats["peer_requests"] += 1
            if len(chunks) > HCP_MAX_ITEM_SEGMENTS - 1:
                concat.append(r)
                refs, lens_c = [(r, CONCAT)], [sum(lens_c)]
            else:
                refs = [(r, c) for c in range(len(chunks))]
            if len(cur.sources) + len(refs) > HCP_MAX_EXT_SOURCES:
                groups.append(cur)
                cur = _Group()
            left = peer_end
            for ref, n in zip(refs, lens_c):
                take = min(n, left)
                if take > 0:
                    peer_segs.append([HCP_SRC_EXT0 + len(cur.sources), 0, take, -1])
                cur.sources.append(ref)
                left -= take
        elif split_tokens > 0:
            peer_end = min(split_tokens, tk)
            split_mode = True
            peer_segs = [[HCP_SRC_PAGED, 0, peer_end, -1]]
        if tq == 1 and decode_kernel and len(peer_segs) <= 1:
            stats["decode_rows"] += 1
            if peer_end > 0 and not split_mode:
                # query at position tk-1: every key is visible
                cur.decode.append([qs, 0, peer_end, r, peer_end, tk - peer_end])
                cur.peer_src.append(peer_segs[0][0] - HCP_SRC_EXT0)
            else:
                cur.decode.append([qs, 0, 0, r, 0, tk])
                cur.peer_src.append(-1)
            continue
        stats["prefill_rows"] += tq
        if peer_end == 0:
            cur.item(qs, tq, r, [[HCP_SRC_PAGED, 0, tk, qpos0]])
            continue
        n_a = max(0, min(tq, peer_end - qpos0))
        if n_a > 0:
            cur.item(qs, n_a, r, [[HCP_SRC_PAGED, 0, tk, qpos0]])
        if n_a < tq:
            local = tk - peer_end
            segs = list(peer_segs)
            if local > 0:
                segs.append([HCP_SRC_PAGED, peer_end, local, qpos0 + n_a - peer_end])
            cur.item(qs + n_a, tq - n_a, r, segs)
    if cur.work or cur.decode or not groups:
        groups.append(cur)
    return LayerPlan(groups=[g.freeze() for g in groups], stats=stats, concat_requests=concat)


def misaligned_paged_starts(plan: LayerPlan, block_size: int) -> bool:
    """True if any paged segment starts off a block boundary (the kernels
    need block-aligned paged starts)."""
    for g in plan.groups:
        segs = [g.work[:, 4:8], g.work[:, 8:12], g.seg_list]
        for sg in segs:
            if np.any((sg[:, 0] == HCP_SRC_PAGED) & (sg[:, 1] % block_size != 0)):
                return True
        if np.any((g.decode[:, 5] > 0) & (g.decode[:, 4] % block_size != 0)):
            return True
    return False
