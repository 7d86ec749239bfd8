"""HCP ring-attention backend for vLLM, B200 (sm_100a) kernels.

Drop-in for the reference's ``hcp_vllm_plugin.ring_backend``: same backend
name (``CUSTOM``), same impl constructor and ``forward`` contract, same
peer-KV staging registry that the KV connector fills.  What changes is the
body of ``forward``:

* reference (``ring_backend.py:576-834``): a Python loop over requests; per
  request a gather of all paged keys into a contiguous copy, a local causal
  pass, a peer non-causal pass and an LSE merge - three kernel launches plus
  copies per request per layer;
* here: one host sync per engine step (query_start_loc, seq_lens and the
  first block ids, cached on the metadata object), a host plan
  (``ring_plan.plan_layer``), then ONE fused prefill launch for every
  multi-token request (local keys read straight from the paged cache, peer
  keys from the staged segment, both in one online softmax) and ONE
  batch-merged split-KV decode launch for every single-token request.

KV cache layout: ``[num_blocks, Hkv, block_size, 2 * head_size]`` with K in
the first ``head_size`` lanes of the last dimension and V in the second (the
layout of ``hcp_vllm_plugin/file_connector.py:14-16``).  There is no CPU
path: every op runs in ``libhcp_ring.so`` and raises if it is missing.
"""

from __future__ import annotations

import os
import re

import torch

from vllm.logger import init_logger
from vllm.v1.attention.backend import AttentionImpl, AttentionType
from vllm.v1.attention.backends.flash_attn import (
    FlashAttentionBackend,
    FlashAttentionMetadataBuilder,
)

from . import _capi, ops
from .ring_plan import CONCAT, misaligned_paged_starts, plan_layer

logger = init_logger(__name__)
_LAYER_RE = re.compile(r"layers\.(\d+)\.")

# ---------------------------------------------------------------------------
# Peer KV staging (module level), same contract as the reference
# (ring_backend.py:92-136): the connector writes, forward() reads.
# Keyed by (chunk_key, layer_name); a request is bound to its ORDERED prefix
# chunk keys by its first block-table block id.  Connector threads insert
# while the worker thread reads and deletes, so every scan below iterates a
# snapshot (``list(dict)`` copies the keys without running Python code, so no
# other thread can change the dict in between).
# ---------------------------------------------------------------------------
PEER_KV_STAGING: dict[tuple[str, str], tuple[torch.Tensor, torch.Tensor]] = {}
PEER_REQ_MAP: dict[int, list[str]] = {}

STAGING_STATS: dict = {"max_concurrent_chunks": 0, "max_staged_layers": 0, "last_chunk_len": 0}
# Pool-write evidence (validation only, same keys as the reference's
# ring_backend.py:255-267): slots written by do_kv_cache_update while
# enabled, and the decode-ring tokens it skipped.
WRITE_TRACK: dict = {"enabled": False, "slots": set(), "overlap": 0, "skipped": 0}
BATCH_STATS: dict = {"max_reqs": 0}
# Which device paths ran (validation evidence, as the reference's IMPL_STATS).
IMPL_STATS: dict = {"attn_cuda": 0, "decode_cuda": 0, "cache_update_cuda": 0, "peer_concat": 0,
                    "decode_ring": 0}


_STATUS_WATCH: dict = {}  # device index -> _capi.DeviceStatusWatch


def _status_watch(device: torch.device):
    w = _STATUS_WATCH.get(device.index)
    if w is None:
        w = _STATUS_WATCH[device.index] = _capi.DeviceStatusWatch()
    return w


def stage_peer_kv(chunk_key: str, layer_name: str, k: torch.Tensor, v: torch.Tensor) -> None:
    """Stage one peer chunk's K/V ([T, Hkv, D], K post-RoPE) for one layer."""
    PEER_KV_STAGING[(chunk_key, layer_name)] = (k, v)
    STAGING_STATS["max_staged_layers"] = max(STAGING_STATS["max_staged_layers"], len(PEER_KV_STAGING))
    chunks = {key[0] for key in list(PEER_KV_STAGING)}
    STAGING_STATS["max_concurrent_chunks"] = max(STAGING_STATS["max_concurrent_chunks"], len(chunks))
    STAGING_STATS["last_chunk_len"] = int(k.shape[0])


def drop_chunk_kv(chunk_key: str) -> int:
    keys = [key for key in list(PEER_KV_STAGING) if key[0] == chunk_key]
    return sum(PEER_KV_STAGING.pop(key, None) is not None for key in keys)


def map_request_peer(first_block_id: int, chunk_keys) -> None:
    if isinstance(chunk_keys, str):
        chunk_keys = [chunk_keys]
    PEER_REQ_MAP[first_block_id] = list(chunk_keys)


def unmap_request_peer(first_block_id: int) -> None:
    PEER_REQ_MAP.pop(first_block_id, None)


def request_peer_chunk(first_block_id: int) -> list[str] | None:
    return PEER_REQ_MAP.get(first_block_id)


def clear_peer_kv() -> None:
    PEER_KV_STAGING.clear()
    PEER_REQ_MAP.clear()


def reset_staging_stats() -> None:
    STAGING_STATS.update(max_concurrent_chunks=0, max_staged_layers=0, last_chunk_len=0)


def reset_batch_stats() -> None:
    BATCH_STATS["max_reqs"] = 0


def reset_write_tracking() -> None:
    WRITE_TRACK.update(enabled=True, slots=set(), overlap=0, skipped=0)


def reset_impl_stats() -> None:
    for key in IMPL_STATS:
        IMPL_STATS[key] = 0


# ---------------------------------------------------------------------------
# Memory-split decode (the decode ring), same registry as the reference
# (ring_backend.py:153-211): the connector registers a request by its first
# block id; its single-token decode rows then run on the ring
# (``ring_decode.RingDecode``) instead of the local plan.  Entry: ``ring``
# (the owner's RingDecode), ``slot`` (the request's arena slot),
# ``prefix_len`` (tokens held by the peers), ``own_len`` (this instance's
# chunk: set at the first decode step, as the reference does at :648-650),
# ``installed`` (layers whose own chunk is in the slot already).
# ---------------------------------------------------------------------------
DECODE_RING_MAP: dict[int, dict] = {}
# The connector's refcount-aware release of a request's staged prefix, called
# at the request's first decode step (ring_backend.py:156-157, 213-225).
_STAGING_RELEASE_FN = None


def _decode_ring_enabled() -> bool:
    return os.environ.get("HCP_RING_DECODE_RING", "1") == "1"


def set_staging_release_fn(fn) -> None:
    global _STAGING_RELEASE_FN
    _STAGING_RELEASE_FN = fn


def _release_staged_for_request(first_block_id: int) -> None:
    """Decode-ring transition: the staged prefix of this request is not read
    again (the peers hold it), so it is freed now, through the connector when
    it registered a release function."""
    if first_block_id not in PEER_REQ_MAP:
        return
    if _STAGING_RELEASE_FN is not None:
        _STAGING_RELEASE_FN(first_block_id)
    else:
        for ck in PEER_REQ_MAP.pop(first_block_id, None) or []:
            drop_chunk_kv(ck)


def register_decode_ring(first_block_id: int, ring, slot: int, prefix_len: int) -> None:
    DECODE_RING_MAP[first_block_id] = {"ring": ring, "slot": int(slot), "prefix_len": int(prefix_len),
                                       "first_block_id": int(first_block_id), "own_len": None,
                                       "installed": set()}


def clear_decode_ring(first_block_id: int) -> None:
    DECODE_RING_MAP.pop(first_block_id, None)


def layer_index(layer_name: str) -> int:
    m = _LAYER_RE.search(layer_name)
    return int(m.group(1)) if m else 0


def _ring_enabled() -> bool:
    return os.environ.get("HCP_RING_ENABLED", "1") == "1"


def _split_tokens() -> int:
    return int(os.environ.get("HCP_RING_SPLIT_TOKENS", "0"))


class HcpRingAttentionBackend(FlashAttentionBackend):
    """Ring-attention backend.  ``get_name()`` stays ``"CUSTOM"``: vLLM's
    Attention layer looks the backend up by that enum member."""

    forward_includes_kv_cache_update: bool = False

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["HcpRingAttentionImpl"]:
        return HcpRingAttentionImpl

    @staticmethod
    def get_builder_cls() -> type[FlashAttentionMetadataBuilder]:
        return FlashAttentionMetadataBuilder

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = "auto") -> tuple[int, ...]:
        if block_size % 16 != 0:
            raise ValueError("Block size must be a multiple of 16.")
        return (num_blocks, num_kv_heads, block_size, 2 * head_size)

    @staticmethod
    def get_kv_cache_stride_order(include_num_layers_dimension: bool = False) -> tuple[int, ...]:
        return (0, 1, 2, 3, 4) if include_num_layers_dimension else (0, 1, 2, 3)


class HcpRingAttentionImpl(AttentionImpl):
    """Local (causal, paged) + transient peer (non-causal) attention with the
    LSE merge fused, on the B200 kernels.  Same constructor contract as the
    reference (``ring_backend.py:464-498``)."""

    def __init__(self, num_heads: int, head_size: int, scale: float, num_kv_heads: int | None = None,
                 alibi_slopes: list[float] | None = None, sliding_window: int | None = None,
                 kv_cache_dtype: str = "auto", logits_soft_cap: float | None = None,
                 attn_type: str = AttentionType.DECODER,
                 kv_sharing_target_layer_name: str | None = None, **kwargs) -> None:
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        self.kv_cache_dtype = kv_cache_dtype
        self.attn_type = attn_type
        self.kv_sharing_target_layer_name = kv_sharing_target_layer_name
        self.supports_quant_query_input = False
        if alibi_slopes is not None:
            raise NotImplementedError("HCP ring backend: ALiBi not supported")
        if logits_soft_cap:
            raise NotImplementedError("HCP ring backend: soft cap not supported")
        if sliding_window is not None and int(sliding_window) <= 0:
            raise ValueError("HCP ring backend: sliding window must be positive")
        if kv_cache_dtype not in ("auto", "bfloat16", "float16"):
            raise NotImplementedError(f"HCP ring backend: kv cache dtype {kv_cache_dtype}")
        if head_size not in (64, 128):
            raise NotImplementedError("HCP ring backend: head_size must be 64 or 128")
        # As the reference's torch path (ring_backend.py:490-492, 786-826): the
        # window applies to the causal (local) passes; staged peer chunks stay
        # fully visible.  Decode rows then go through the prefill kernel,
        # whose causal segments carry the window.
        self.sliding_window = int(sliding_window) if sliding_window is not None else None
        self.num_queries_per_kv = self.num_heads // self.num_kv_heads

    # -- KV cache update -----------------------------------------------------
    def do_kv_cache_update(self, layer: torch.nn.Module, key: torch.Tensor, value: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
        """Scatter this step's K/V into the paged cache (``hcp_kv_cache_update``;
        the reference's torch index_put, ``ring_backend.py:501-539``)."""
        if self.attn_type in (AttentionType.ENCODER_ONLY, AttentionType.ENCODER):
            return
        n = slot_mapping.shape[0]
        if n == 0:
            return
        sm = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
        skip = self._decode_ring_skip_rows(layer) if (DECODE_RING_MAP and _decode_ring_enabled()) else []
        if skip:
            # Decode-ring tokens are kept by their assignee (memory-split
            # decode growth): they are not written to this pool
            # (ring_backend.py:519-531); -1 makes the scatter skip the row.
            sm = sm.clone()
            idx = torch.tensor(skip, dtype=torch.long)
            sm[idx.pin_memory().to(sm.device, non_blocking=True) if sm.is_cuda else idx] = -1
            WRITE_TRACK["skipped"] += len(skip)
        ops.kv_cache_update(key[:n], value[:n], kv_cache, sm.contiguous())
        IMPL_STATS["cache_update_cuda"] += 1
        if WRITE_TRACK["enabled"]:
            WRITE_TRACK["slots"].update(s for s in sm.tolist() if s >= 0)

    def _decode_ring_skip_rows(self, layer) -> list[int]:
        """Rows of this step's slot mapping that are decode-ring tokens (the
        single-token step of a registered request), from the step's
        attention metadata; none when it cannot be attributed."""
        try:
            from vllm.forward_context import get_forward_context

            raw = get_forward_context().attn_metadata
        except Exception:  # noqa: BLE001 - no forward context: skip nothing
            return []
        if isinstance(raw, list):
            raw = raw[0] if raw else None
        meta = raw.get(getattr(layer, "layer_name", ""), None) if isinstance(raw, dict) else raw
        if meta is None:
            return []
        qsl, _, bt0 = self._host_meta(meta)
        return [qsl[r] for r, _ in self._decode_ring_rows(qsl, bt0)]

    # -- forward -------------------------------------------------------------
    @staticmethod
    def _host_meta(attn_metadata):
        """query_start_loc, seq_lens and first block ids on the host: one
        device-to-host sync per engine step (all layers share the metadata)."""
        cached = getattr(attn_metadata, "_hcp_host_meta", None)
        if cached is not None:
            return cached
        qsl = attn_metadata.query_start_loc.tolist()
        seq_lens = attn_metadata.seq_lens.tolist()
        bt0 = attn_metadata.block_table[: len(seq_lens), 0].tolist()
        if attn_metadata.query_start_loc.is_cuda:
            # the step's one synchronisation has just passed: a device-side
            # failure of an earlier step surfaces here as an HcpError
            _status_watch(attn_metadata.query_start_loc.device).check("HCP ring backend")
        cached = (qsl, seq_lens, bt0)
        try:
            attn_metadata._hcp_host_meta = cached
        except (AttributeError, TypeError):
            pass
        return cached

    def _peers_for_layer(self, layer_name: str, seq_lens, bt0, skip=frozenset()) -> dict:
        peers: dict[int, list] = {}
        if not _ring_enabled():
            return peers
        for r in range(len(seq_lens)):
            if r in skip:
                continue
            ck_list = PEER_REQ_MAP.get(int(bt0[r]))
            if ck_list is None and len(seq_lens) == 1:
                # single-request fallback, as the reference (ring_backend.py:746-755)
                chunks = {key[0] for key in list(PEER_KV_STAGING)}
                if len(chunks) == 1:
                    ck_list = [next(iter(chunks))]
            if not ck_list:
                continue
            parts = []
            for ck in ck_list:
                kv = PEER_KV_STAGING.get((ck, layer_name))
                if kv is None:
                    parts = None
                    break
                parts.append(kv)
            if parts is None:
                logger.warning("HCP ring: request mapped to chunks %s but staging incomplete at layer %s; "
                               "using the local path", ck_list, layer_name)
                continue
            peers[r] = parts
        return peers

    def forward(self, layer: torch.nn.Module, query: torch.Tensor, key: torch.Tensor,
                value: torch.Tensor, kv_cache: torch.Tensor, attn_metadata, output: torch.Tensor,
                output_scale: torch.Tensor | None = None,
                output_block_scale: torch.Tensor | None = None) -> torch.Tensor:
        if output_scale is not None or output_block_scale is not None:
            raise NotImplementedError("fused output quant not supported")
        if attn_metadata is None:
            return output.fill_(0)  # profiling run
        assert self.attn_type == AttentionType.DECODER, "HCP ring backend supports decoder attention only"
        num_actual = attn_metadata.num_actual_tokens
        q = query[:num_actual]
        out = output[:num_actual]
        qsl, seq_lens, bt0 = self._host_meta(attn_metadata)
        BATCH_STATS["max_reqs"] = max(BATCH_STATS["max_reqs"], len(seq_lens))
        layer_name = getattr(layer, "layer_name", "")
        ring_rows = self._decode_ring_rows(qsl, bt0) if (DECODE_RING_MAP and _decode_ring_enabled()) else []
        excluded = frozenset(r for r, _ in ring_rows)
        peers = self._peers_for_layer(layer_name, seq_lens, bt0, excluded) \
            if (PEER_REQ_MAP or PEER_KV_STAGING) else {}
        block_size = kv_cache.shape[2]
        split = _split_tokens() if _ring_enabled() else 0
        # The plan depends on lengths only (requests, staged chunks), which
        # every layer of a step shares: build it once per step and rebuild
        # just this layer's list of staged tensors.
        window = self.sliding_window
        if window is not None and ring_rows:
            raise NotImplementedError("HCP ring backend: the decode ring has no sliding window")
        sig = (block_size, split, excluded, window is None,
               tuple((r, tuple(int(k.shape[0]) for k, _ in ch)) for r, ch in sorted(peers.items())))
        plans = getattr(attn_metadata, "_hcp_plans", None)
        if plans is None:
            plans = {}
            try:
                attn_metadata._hcp_plans = plans
            except (AttributeError, TypeError):
                pass
        plan = plans.get(sig)
        if plan is None:
            plan = plan_layer(qsl, seq_lens, block_size, peers, split, decode_kernel=window is None,
                              exclude=excluded)
            if misaligned_paged_starts(plan, block_size):
                raise ValueError("HCP ring backend: peer prefix length must be a multiple of the block size")
            plans[sig] = plan
        block_table = attn_metadata.block_table
        if block_table.dtype != torch.int32:
            block_table = block_table.to(torch.int32)
        for grp in plan.groups:
            # each staged chunk is read where it lies (an extra source of the
            # kernels); only a request with more chunks than a work item has
            # segments for is concatenated
            ext = []
            for r, c in grp.sources:
                if c == CONCAT:
                    ext.append((torch.cat([k for k, _ in peers[r]], dim=0),
                                torch.cat([v for _, v in peers[r]], dim=0)))
                    IMPL_STATS["peer_concat"] += 1
                else:
                    ext.append(peers[r][c])
            if grp.work.shape[0]:
                ops.ring_attn_fwd(q, grp.work, scale=self.scale, num_kv_heads=self.num_kv_heads, out=out,
                                  kv_cache=kv_cache, block_table=block_table, ext=ext, seg_list=grp.seg_list,
                                  window=window)
                IMPL_STATS["attn_cuda"] += 1
            if grp.decode.shape[0]:
                ops.decode_splitkv(q, grp.decode, scale=self.scale, num_kv_heads=self.num_kv_heads, out=out,
                                   kv_cache=kv_cache, block_table=block_table, ext=ext, peer_src=grp.peer_src)
                IMPL_STATS["decode_cuda"] += 1
        if ring_rows:
            self._decode_ring_forward(layer_index(layer_name), ring_rows, qsl, seq_lens, q, key, value,
                                      kv_cache, block_table, out)
        if q.is_cuda:
            _status_watch(q.device).record(torch.cuda.current_stream(q.device))
        return output

    # -- memory-split decode -------------------------------------------------
    @staticmethod
    def _decode_ring_rows(qsl, bt0) -> list:
        """(request index, registry entry) of this step's decode-ring rows:
        single-token steps of registered requests (``ring_backend.py:639-640``)."""
        rows = []
        for r in range(len(qsl) - 1):
            if qsl[r + 1] - qsl[r] != 1:
                continue
            e = DECODE_RING_MAP.get(int(bt0[r]))
            if e is not None:
                rows.append((r, e))
        return rows

    def _decode_ring_forward(self, li: int, ring_rows, qsl, seq_lens, q, key, value, kv_cache,
                             block_table, out) -> None:
        """The owner's side of one layer of the decode ring for this step's
        ring rows (the reference's per-request local partial + packet,
        ``ring_backend.py:641-729``, here one collective step per ring).

        At a request's first decode step every layer first moves the
        request's own chunk (positions ``[prefix_len, prefix_len + own_len)``
        of its paged cache) into its ring slot, once; the reference rebuilds
        that segment by concatenation at every step."""
        by_ring: dict[int, tuple] = {}
        for r, e in ring_rows:
            by_ring.setdefault(id(e["ring"]), (e["ring"], []))[1].append((r, e))
        for ring, rows in by_ring.values():
            if abs(ring.scale - self.scale) > 1e-6 * self.scale:
                raise ValueError(f"HCP decode ring: ring scale {ring.scale} != layer scale {self.scale}")
            slots, positions, fresh = [], [], []
            for r, e in rows:
                tk = int(seq_lens[r])
                if e["own_len"] is None:
                    e["own_len"] = tk - 1 - e["prefix_len"]  # tk counts the current token
                if not e["installed"]:
                    fresh.append(e["slot"])
                slots.append(e["slot"])
                positions.append(tk - 1)
            if li == 0:
                ring.begin_step(slots, positions, fresh)
                for _, e in rows:
                    if not e["installed"]:
                        _release_staged_for_request(e["first_block_id"])
            for r, e in rows:
                if li not in e["installed"]:
                    self._install_own_chunk(ring, li, r, e, kv_cache, block_table)
                    e["installed"].add(li)
            idx = torch.tensor([qsl[r] for r, _ in rows], dtype=torch.long)
            if q.is_cuda:
                idx = idx.pin_memory().to(q.device, non_blocking=True)
            res = torch.empty(len(rows), q.shape[1], q.shape[2], dtype=out.dtype, device=out.device)
            ring.step(li, positions, q.index_select(0, idx), key.index_select(0, idx),
                      value.index_select(0, idx), res, slots=slots)
            out.index_copy_(0, idx, res)
            IMPL_STATS["decode_ring"] += 1

    @staticmethod
    def _install_own_chunk(ring, li, r, e, kv_cache, block_table) -> None:
        n, start = e["own_len"], e["prefix_len"]
        kk, vv = ring.install_rows(li, e["slot"], n)
        if n <= 0:
            return
        bs = kv_cache.shape[2]
        blocks = block_table[r, start // bs:(start + n + bs - 1) // bs].to(torch.int64)
        offs = torch.arange(bs, dtype=torch.int64, device=blocks.device)
        lead = start % bs
        slots = (blocks[:, None] * bs + offs[None, :]).flatten()[lead:lead + n].contiguous()
        ops.kv_cache_gather(kv_cache, slots, key=kk, value=vv)
