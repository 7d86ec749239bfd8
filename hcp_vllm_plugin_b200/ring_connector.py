"""``HcpRingKvConnector`` inside one box: ring context-parallel prefix KV moved
over NVLink instead of HTTP.

Semantics kept from the reference (``hcp_vllm_plugin/ring_connector.py``):

* roles ``ring`` / ``relay`` (consumer and producer side), ``producer``,
  ``consumer`` (``:255-275``); config keys ``ring_shared_path``,
  ``ring_run_id``, ``ring_chunk_id``, ``ring_prefix_chunk_ids``,
  ``ring_prefix_len``, ``ring_order`` / ``ring_my_chunk``,
  ``ring_ready_poll_interval_s``; per-request overrides in
  ``kv_transfer_params["hcp_ring"]`` (``chunk_ids`` / ``chunk_id``,
  ``peer_urls`` / ``peer_url``, ``prefix_len``) (``:172-220``);
* scheduler side: the prefix is reported as externally computed once every
  prefix chunk is ready, aligned down to the block size, and nothing is
  loaded into the paged pool (``:553-659``); the producer side's own chunk
  is saved from the request's blocks past the prefix (``:636-677``);
* worker side: prefix chunk K/V is staged TRANSIENTLY in
  ``ring_backend.PEER_KV_STAGING`` keyed by ``(chunk, layer)``, the request
  bound to its ordered chunk list by its first block id; a per-request
  stream stages layers in model order at most ``HCP_RING_STREAM_WINDOW``
  layers ahead of ``wait_for_layer_load`` and frees the staging of layers
  already consumed (``:144-170, 794-888``); chunks are refcounted across
  requests and freed when the last user finishes, before the step that may
  recycle its blocks (``:240-250, 939-997``).  That bookkeeping lives in
  ``staging_ledger`` (chunk holds, the per-request layer feed, ready-marker
  lookups, decode-ring slots).

What changes is the transport.  The reference producer writes one
safetensors file per layer and serves its store over HTTP; a consumer
downloads the files and loads them onto its GPU.  Here every producer keeps
its chunk in ONE HBM buffer ``[num_layers, 2, T, Hkv, D]``, filled from the
paged pool by ``hcp_kv_cache_gather`` in ``save_kv_layer``, and exports it
with CUDA IPC; ``wait_for_save`` writes the ``_READY`` marker (same path as
the reference's local store, ``<shared>/<run>/<chunk>/_READY``) with the
handle.  A consumer on any GPU of the box maps that buffer once and copies
each layer it stages with the copy engine over NVLink/NVSwitch
(``hcp_peer_copy``) on a side stream; ``wait_for_layer_load`` orders the
compute stream after that layer's copies.  Every GPU reaches every other at
full bandwidth through NVSwitch, so a consumer pulls each prefix chunk from
its owner directly and the reference's neighbour re-serving is not needed;
``ring_peer_url`` / ``ring_serve_port`` are accepted and unused.  The
producer must outlive the consumers' copies (a serving instance does).
"""

from __future__ import annotations

import ctypes
import json
import os
import re
import threading
import time
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any

import torch

from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
)
from vllm.logger import init_logger

from . import _capi as C
from . import ops
from .ring_backend import (
    PEER_KV_STAGING,
    clear_decode_ring,
    register_decode_ring,
    set_staging_release_fn,
    stage_peer_kv,
)
from .staging_ledger import ChunkLedger, DecodeSlotPool, LayerFeed, ReadinessCache

if TYPE_CHECKING:
    from vllm.config import VllmConfig
    from vllm.forward_context import ForwardContext
    from vllm.v1.core.kv_cache_manager import KVCacheBlocks
    from vllm.v1.core.sched.output import SchedulerOutput
    from vllm.v1.kv_cache_interface import KVCacheConfig
    from vllm.v1.request import Request

logger = init_logger(__name__)
_LAYER_RE = re.compile(r"layers\.(\d+)\.")
_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16}


def decode_ring_on() -> bool:
    """``HCP_RING_DECODE_RING`` (default on, as the reference's
    ``ring_connector.py:129-134``); the ring also needs ``ring_decode_addr``."""
    return os.environ.get("HCP_RING_DECODE_RING", "1") == "1"


def stream_window() -> int:
    """Layers a request's staging may run ahead of the consumed layer
    (``HCP_RING_STREAM_WINDOW``, default 2).  At least 1: with 0, layer i
    could only be staged after layer i was consumed, which waits for it."""
    return max(1, int(os.environ.get("HCP_RING_STREAM_WINDOW", "2")))


def align_down(n: int, block_size: int) -> int:
    return n // block_size * block_size


def layer_index(layer_name: str) -> int:
    m = _LAYER_RE.search(layer_name)
    return int(m.group(1)) if m else 0


def ring_params_from_sampling(sampling_params: Any) -> dict:
    """``extra_args["kv_transfer_params"]["hcp_ring"]`` of a request, or {}."""
    extra = getattr(sampling_params, "extra_args", None) or {}
    return dict((extra.get("kv_transfer_params") or {}).get("hcp_ring") or {})


def as_str_list(value: Any) -> list[str]:
    if value is None:
        return []
    if isinstance(value, str):
        return [s for s in value.split(",") if s]
    return [str(s) for s in value]


def chunks_and_urls(rp: dict, global_ids: list[str],
                    global_urls: list[str] | None = None) -> tuple[list[str], list[str]]:
    """Ordered prefix chunk keys and one peer url per chunk ("" = default).

    Plural keys win over singular ones, per-request values over the global
    ones; a url list shorter than the chunk list is padded with its last
    entry (one predecessor serves the whole accumulated prefix), else with "".
    """
    ids = as_str_list(rp.get("chunk_ids")) or ([str(rp["chunk_id"])] if rp.get("chunk_id") else [])
    if not ids:
        ids = list(global_ids)
    urls = as_str_list(rp.get("peer_urls")) or ([str(rp["peer_url"])] if rp.get("peer_url") else [])
    if not urls and global_urls:
        urls = list(global_urls)
    urls = [u.rstrip("/") for u in urls]
    fill = urls[-1] if urls and len(urls) < len(ids) else ""
    urls = urls + [fill] * (len(ids) - len(urls))
    return ids, urls


def _prefix_len(rp: dict, default: int) -> int:
    # presence, not truthiness: prefix_len=0 opts a request out
    return int(rp["prefix_len"]) if "prefix_len" in rp else default


@dataclass
class RingReqMeta:
    is_store: bool
    chunk_key: str                                  # store side: own chunk
    slot_mapping: torch.Tensor | None = None        # store side: pool slots of the own chunk
    req_id: str = ""                                # load side
    first_block_id: int = -1
    chunk_keys: list[str] = field(default_factory=list)
    peer_urls: list[str] = field(default_factory=list)
    prefix_len: int = 0


@dataclass
class HcpRingConnectorMetadata(KVConnectorMetadata):
    requests: list[RingReqMeta] = field(default_factory=list)
    # finished between the previous and this step: cleaned before this step's
    # forward, because their blocks may already serve requests of this step
    finished_req_ids: list[str] = field(default_factory=list)


# ---------------------------------------------------------------------------
# Transport: HBM chunk store (producer) and mapped sources (consumer)
# ---------------------------------------------------------------------------
# Buffers exported by this process, so a consumer in the same process reads
# them without IPC (a process cannot map its own IPC handle).
_LOCAL_EXPORTS: dict[tuple[str, str], torch.Tensor] = {}


class ChunkSource:
    """A producer's chunk store mapped into this process."""

    def __init__(self, marker: dict, device: torch.device):
        self.tokens = int(marker["tokens"])
        self.shape = [int(x) for x in marker["shape"]]      # [L, 2, T, Hkv, D]
        self.dtype = _DTYPES[marker["dtype"]]
        self.device = device
        self._local = _LOCAL_EXPORTS.get((marker["run"], marker["chunk"])) \
            if int(marker["pid"]) == os.getpid() else None
        self._base = None
        if self._local is None:
            handle = bytes.fromhex(marker["handle"])
            base = ctypes.c_void_p()
            C.check(C.load().hcp_ipc_open(handle, device.index if device.index is not None else 0,
                                          ctypes.byref(base)), "hcp_ipc_open")
            self._base = base.value
            self._addr = base.value + int(marker["offset"])
        else:
            self._addr = self._local.data_ptr()
        self._elt = torch.empty(0, dtype=self.dtype).element_size()

    def layer_bytes(self) -> int:
        _, _, t, hkv, d = self.shape
        return t * hkv * d * self._elt

    def copy_layer(self, idx: int, k: torch.Tensor, v: torch.Tensor, stream) -> None:
        """K and V of layer ``idx`` into ``k``/``v`` [T, Hkv, D] (stream-ordered)."""
        if not 0 <= idx < self.shape[0]:
            raise IndexError(f"layer {idx} not in the chunk store ({self.shape[0]} layers)")
        nbytes = self.layer_bytes()
        src = self._addr + idx * 2 * nbytes
        s = stream.cuda_stream
        C.check(C.load().hcp_peer_copy(k.data_ptr(), src, nbytes, s), "hcp_peer_copy")
        C.check(C.load().hcp_peer_copy(v.data_ptr(), src + nbytes, nbytes, s), "hcp_peer_copy")

    def close(self) -> None:
        if self._base is not None:
            C.load().hcp_ipc_close(self._base)
            self._base = None


class HcpRingKvConnector(KVConnectorBase_V1):
    """Ring-KV connector: external-prefix scheduling + transient NVLink staging."""

    # How a consumer reaches a producer's chunk store (tests of the host-side
    # logic substitute a CPU source; the product maps the store over IPC).
    source_cls = ChunkSource

    def __init__(self, vllm_config: "VllmConfig", role: KVConnectorRole,
                 kv_cache_config: "KVCacheConfig" = None):
        super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
        cfg = self._kv_transfer_config
        self._block_size = vllm_config.cache_config.block_size
        self._num_layers = int(vllm_config.model_config.hf_config.num_hidden_layers)
        self._ring_role = cfg.get_from_extra_config("ring_role", "producer")
        if self._ring_role not in ("ring", "producer", "consumer", "relay"):
            raise ValueError(f"HcpRingKvConnector: unknown ring_role {self._ring_role!r} "
                             "(expected ring|producer|consumer|relay)")
        self._consumer_side = self._ring_role in ("consumer", "relay", "ring")
        self._producer_side = self._ring_role in ("producer", "relay", "ring")
        self._shared_path = cfg.get_from_extra_config("ring_shared_path", "/tmp/hcp_ring_kv")
        self._run_id = cfg.get_from_extra_config("ring_run_id", "run")
        self._chunk_id = cfg.get_from_extra_config("ring_chunk_id", "chunk0")
        self._prefix_chunk_ids = as_str_list(cfg.get_from_extra_config("ring_prefix_chunk_ids", ""))
        self._prefix_len = int(cfg.get_from_extra_config("ring_prefix_len", 0))
        self._prefix_peer_urls: list[str] = []
        order = cfg.get_from_extra_config("ring_order", "")
        my_chunk = cfg.get_from_extra_config("ring_my_chunk", self._chunk_id)
        if order:
            specs = as_str_list(order)
            ids = [s.split("@")[0] for s in specs]
            urls = [s.split("@", 1)[1].rstrip("/") if "@" in s else "" for s in specs]
            if my_chunk in ids:
                i = ids.index(my_chunk)
                self._chunk_id = my_chunk
                self._prefix_chunk_ids = ids[:i]
                self._prefix_peer_urls = [urls[i - 1] if i > 0 else ""] * i
        self._poll_interval = float(cfg.get_from_extra_config("ring_ready_poll_interval_s", 0.5))
        # Memory-split decode (the decode ring): the nodes of ring_order form
        # their own process group, rendezvous at ring_decode_addr
        # ("host:port", hosted by rank 0); a node's rank is its chunk's index
        # in ring_order, so the owner (the last chunk) is rank N-1 and the
        # peers are 0..N-2 in prefix order, as the reference's growth indexing
        # (ring_decode.py:30-43).  Peers serve their chunk store; the owner
        # sends its decode rows through the ring (ring_backend).
        order_ids = [x.split("@")[0] for x in as_str_list(order)]
        self._decode_addr = str(cfg.get_from_extra_config("ring_decode_addr", "") or "")
        self._decode_rank = int(cfg.get_from_extra_config(
            "ring_decode_index", order_ids.index(self._chunk_id) if self._chunk_id in order_ids else -1))
        self._decode_world = int(cfg.get_from_extra_config("ring_decode_world", len(order_ids)))
        self._decode_slots = int(cfg.get_from_extra_config("ring_decode_slots", 4))
        self._decode_capacity = int(cfg.get_from_extra_config("ring_decode_capacity", 17408))
        self._decode_backend = str(cfg.get_from_extra_config("ring_decode_backend", "nccl"))
        # the chunk a peer serves (the reference's ring_partial_chunks, first entry)
        self._decode_chunk_key = (as_str_list(cfg.get_from_extra_config("ring_partial_chunks", ""))
                                  or [self._chunk_id])[0]
        self._decode_on = bool(self._decode_addr) and decode_ring_on() and \
            0 <= self._decode_rank < self._decode_world
        self._decode_owner = self._decode_on and self._decode_rank == self._decode_world - 1
        # With the decode ring, staged prefix KV of a consumed layer is freed
        # at once (memory-split); without it, decode steps read the staged
        # prefix again, so it stays until the request finishes (the
        # reference's bulk staging when the decode ring is off).
        self._drop_consumed = self._decode_on
        self._decode_ring = None
        self._slots = DecodeSlotPool(self._decode_slots)
        self._decode_stop = threading.Event()
        self._decode_thread: threading.Thread | None = None
        self._decode_error: BaseException | None = None
        self._readiness = ReadinessCache(self._poll_interval)
        self._requests_need_load: dict[str, Any] = {}
        # worker-side bookkeeping
        self._ledger = ChunkLedger()
        self._feeds: dict[str, LayerFeed] = {}
        self._sources: dict[str, Any] = {}
        self._stage_lock = threading.Lock()
        self._side_stream = None
        self._stores: dict[str, torch.Tensor] = {}       # producer: chunk -> [L, 2, T, Hkv, D]
        self._store_slots: dict[str, tuple] = {}         # producer: chunk -> (host, device) slots
        self._saved_layers: dict[str, set[int]] = {}
        os.makedirs(self._run_dir(), exist_ok=True)
        if self._role == KVConnectorRole.WORKER:
            # the backend frees a request's staging at its first decode step
            set_staging_release_fn(self._release_request_staging)
        if self._decode_on and not self._decode_owner and self._role == KVConnectorRole.WORKER:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
                else torch.device("cpu")
            self._decode_thread = threading.Thread(target=self._serve_decode_ring, args=(device,), daemon=True)
            self._decode_thread.start()

    # ------------------------------------------------------------------ decode ring
    def _make_decode_ring(self, device: torch.device):
        """Join the decode ring's group (returns once all N nodes joined) and
        build this node's ring state."""
        from .ring_decode import RingComm, RingDecode

        host, port = self._decode_addr.rsplit(":", 1)
        comm = RingComm.standalone(host, int(port), self._decode_rank, self._decode_world,
                                   backend=self._decode_backend)
        hf = self._vllm_config.model_config.hf_config
        h, hkv = hf.num_attention_heads, hf.num_key_value_heads
        d = getattr(hf, "head_dim", None) or hf.hidden_size // h
        return RingDecode(self._num_layers, self._decode_slots, self._decode_capacity, h, hkv, d, d ** -0.5,
                          device, dtype=self._vllm_config.model_config.dtype, comm=comm,
                          growth_policy=os.environ.get("HCP_RING_DECODE_GROWTH", "rr"))

    def _decode_chunk(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """This node's chunk for ``layer``, out of its chunk store (the
        reference's node serves its own chunk snapshot,
        ``ring_decode.py:246-249``)."""
        store = self._stores.get(self._decode_chunk_key)
        if store is None:
            raise RuntimeError(f"HcpRingKvConnector: decode ring peer has no saved chunk {self._decode_chunk_key}")
        return store[layer, 0], store[layer, 1]

    def _serve_decode_ring(self, device: torch.device) -> None:
        """Peer nodes: the ring's serve loop in a thread of the worker, on
        its own stream (the reference's relay thread, ``ring_decode.py:284-318``)."""
        try:
            if device.type == "cuda":
                torch.cuda.set_device(device)
            ring = self._make_decode_ring(device)
            self._decode_ring = ring
            if device.type == "cuda":
                with torch.cuda.stream(torch.cuda.Stream(device=device)):
                    ring.serve(self._decode_chunk, stop=self._decode_stop)
            else:
                ring.serve(self._decode_chunk, stop=self._decode_stop)
        except BaseException as e:  # noqa: BLE001 - a dead peer must not take the worker down
            self._decode_error = e
            logger.error("HcpRingKvConnector: decode ring peer %d stopped: %r", self._decode_rank, e)

    def _register_decode(self, req: "RingReqMeta", expected: int, device: torch.device) -> None:
        if self._decode_ring is None:
            self._decode_ring = self._make_decode_ring(device)
        slot = self._slots.take(req.req_id, req.first_block_id)
        register_decode_ring(req.first_block_id, self._decode_ring, slot, expected)

    # ------------------------------------------------------------------ paths
    def _run_dir(self) -> str:
        return os.path.join(self._shared_path, self._run_id)

    def _chunk_dir(self, chunk_key: str) -> str:
        return os.path.join(self._run_dir(), chunk_key)

    def _ready_marker(self, chunk_key: str) -> str:
        return os.path.join(self._chunk_dir(chunk_key), "_READY")

    # ------------------------------------------------------------------ scheduler side
    def _prefix_ready(self, chunk_key: str) -> bool:
        return self._readiness.is_ready(chunk_key, self._ready_marker(chunk_key))

    def get_num_new_matched_tokens(self, request: "Request",
                                   num_computed_tokens: int) -> tuple[int | None, bool]:
        if not self._consumer_side:
            return 0, False
        rp = (getattr(request, "kv_transfer_params", None) or {}).get("hcp_ring") or {}
        prefix_len = _prefix_len(rp, self._prefix_len)
        if prefix_len == 0:
            return 0, False
        chunk_ids, _ = chunks_and_urls(rp, self._prefix_chunk_ids, self._prefix_peer_urls)
        if not chunk_ids:
            return 0, False
        for ck in chunk_ids:
            if not self._prefix_ready(ck):
                return None, True  # ask again later
        return max(align_down(prefix_len, self._block_size) - num_computed_tokens, 0), False

    def update_state_after_alloc(self, request: "Request", blocks: "KVCacheBlocks",
                                 num_external_tokens: int) -> None:
        if num_external_tokens > 0:
            self._requests_need_load[request.request_id] = request

    def _store_slots_for(self, n_tokens: int, block_ids, skip: int) -> torch.Tensor:
        n = align_down(n_tokens, self._block_size)
        blocks = torch.as_tensor(list(block_ids)[skip // self._block_size: n // self._block_size],
                                 dtype=torch.int64)
        if blocks.numel() == 0:
            return torch.empty(0, dtype=torch.int64)
        offs = torch.arange(self._block_size, dtype=torch.int64)
        return (blocks[:, None] * self._block_size + offs[None, :]).flatten()[: n - skip].contiguous()

    def build_connector_meta(self, scheduler_output: "SchedulerOutput") -> HcpRingConnectorMetadata:
        meta = HcpRingConnectorMetadata()
        meta.finished_req_ids = sorted(scheduler_output.finished_req_ids)
        for new_req in scheduler_output.scheduled_new_reqs:
            rp = ring_params_from_sampling(new_req.sampling_params)
            if new_req.req_id in self._requests_need_load:
                ids, urls = chunks_and_urls(rp, self._prefix_chunk_ids, self._prefix_peer_urls)
                meta.requests.append(RingReqMeta(
                    is_store=False, chunk_key="", req_id=new_req.req_id,
                    first_block_id=int(new_req.block_ids[0][0]), chunk_keys=ids, peer_urls=urls,
                    prefix_len=_prefix_len(rp, self._prefix_len)))
            if self._producer_side:
                skip = align_down(_prefix_len(rp, self._prefix_len), self._block_size) \
                    if self._consumer_side else 0
                sm = self._store_slots_for(len(new_req.prompt_token_ids or []), new_req.block_ids[0], skip)
                if sm.shape[0] > 0:
                    meta.requests.append(RingReqMeta(is_store=True, chunk_key=rp.get("chunk_id") or self._chunk_id,
                                                     slot_mapping=sm))
        self._requests_need_load.clear()
        return meta

    # ------------------------------------------------------------------ worker side: load
    def _source(self, chunk_key: str, device: torch.device):
        src = self._sources.get(chunk_key)
        if src is None:
            path = self._ready_marker(chunk_key)
            try:
                with open(path) as f:
                    marker = json.load(f)
            except OSError as e:
                raise RuntimeError(f"HcpRingKvConnector: chunk {chunk_key} is not ready ({path})") from e
            src = self.source_cls(marker, device)
            self._sources[chunk_key] = src
        return src

    def _stage_layer(self, chunks: list[str], layer_name: str, device: torch.device):
        """Stage every chunk of ``chunks`` for ``layer_name`` (once per chunk
        and layer, whichever request asks first); returns the chunks' token
        counts and an event on the side stream after the copies."""
        lens: dict[str, int] = {}
        for ck in chunks:
            with self._stage_lock:
                staged = PEER_KV_STAGING.get((ck, layer_name))
                if staged is not None:
                    lens[ck] = int(staged[0].shape[0])
                    continue
                src = self._source(ck, device)
                _, _, t, hkv, d = src.shape
                if device.type == "cuda":
                    with torch.cuda.stream(self._side_stream):
                        k = torch.empty(t, hkv, d, dtype=src.dtype, device=device)
                        v = torch.empty_like(k)
                        src.copy_layer(layer_index(layer_name), k, v, self._side_stream)
                else:
                    k = torch.empty(t, hkv, d, dtype=src.dtype, device=device)
                    v = torch.empty_like(k)
                    src.copy_layer(layer_index(layer_name), k, v, None)
                stage_peer_kv(ck, layer_name, k, v)
                lens[ck] = t
        done = None
        if device.type == "cuda":
            done = torch.cuda.Event()
            done.record(self._side_stream)
        return lens, done

    def start_load_kv(self, forward_context: "ForwardContext", **kwargs: Any) -> None:
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, HcpRingConnectorMetadata):
            return
        self._cleanup_finished(metadata.finished_req_ids)
        need = [r for r in metadata.requests if not r.is_store]
        if not need:
            return
        layer_order = list(forward_context.no_compile_layers.keys())
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() \
            else torch.device("cpu")
        for layer in forward_context.no_compile_layers.values():
            cache = getattr(layer, "kv_cache", None)
            if isinstance(cache, (list, tuple)):
                cache = cache[0] if cache else None
            if torch.is_tensor(cache) and cache.numel() > 0:
                device = cache.device
                break
        if device.type == "cuda" and self._side_stream is None:
            self._side_stream = torch.cuda.Stream(device=device)
        for req in need:
            if req.req_id in self._feeds or req.req_id in self._ledger.requests() or \
                    req.req_id in self._slots.holders():
                # loaded again (a request resumed after preemption is
                # rescheduled from its prefill): the new registration replaces
                # the old one, whose chunk holds and ring slot are returned
                self._end_request(req.req_id)
            expected = align_down(req.prefix_len or self._prefix_len, self._block_size)
            if self._decode_owner:
                self._register_decode(req, expected, device)   # may fail: before any other state
            self._ledger.hold(req.req_id, req.first_block_id, req.chunk_keys)
            feed = LayerFeed(req.req_id, layer_order, list(req.chunk_keys), expected, stream_window())
            self._feeds[req.req_id] = feed
            chunks = list(req.chunk_keys)
            feed.start(lambda ln, chunks=chunks: self._stage_layer(chunks, ln, device),
                       init=(lambda: torch.cuda.set_device(device)) if device.type == "cuda" else None)

    def wait_for_layer_load(self, layer_name: str) -> None:
        if not self._feeds:
            return
        idx = layer_index(layer_name)
        cur = torch.cuda.current_stream() if torch.cuda.is_available() else None
        for feed in list(self._feeds.values()):
            if not feed.covers(layer_name):
                continue
            cev = feed.wait(layer_name)
            if cev is not None and cur is not None:
                cur.wait_event(cev)
                for ck in feed.chunks:
                    kv = PEER_KV_STAGING.get((ck, layer_name))
                    if kv is not None:
                        # read on the compute stream: keep the allocator from
                        # recycling these blocks before that work completes
                        kv[0].record_stream(cur)
                        kv[1].record_stream(cur)
            feed.consumed(idx)
        if not self._drop_consumed:
            return
        # transient staging of layers already consumed goes away
        with self._stage_lock:
            for key in [key for key in list(PEER_KV_STAGING) if layer_index(key[1]) < idx]:
                PEER_KV_STAGING.pop(key, None)

    # ------------------------------------------------------------------ worker side: save
    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata: Any,
                      **kwargs: Any) -> None:
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, HcpRingConnectorMetadata):
            return
        idx = layer_index(layer_name)
        for req in metadata.requests:
            if not req.is_store or req.slot_mapping is None or req.slot_mapping.numel() == 0:
                continue
            store = self._stores.get(req.chunk_key)
            n = int(req.slot_mapping.shape[0])
            _, hkv, _, d2 = kv_layer.shape
            if store is None or store.shape[2] != n or store.device != kv_layer.device:
                store = torch.empty(self._num_layers, 2, n, hkv, d2 // 2, dtype=kv_layer.dtype,
                                    device=kv_layer.device)
                self._stores[req.chunk_key] = store
                _LOCAL_EXPORTS[(self._run_id, req.chunk_key)] = store
                self._saved_layers[req.chunk_key] = set()
            # one device copy of this request's slots for all its layers (keyed
            # by the host tensor itself: another request saving the same chunk
            # key from other blocks must not reuse it)
            cached = self._store_slots.get(req.chunk_key)
            if cached is None or cached[0] is not req.slot_mapping:
                cached = (req.slot_mapping, req.slot_mapping.to(kv_layer.device))
                self._store_slots[req.chunk_key] = cached
            ops.kv_cache_gather(kv_layer, cached[1], key=store[idx, 0], value=store[idx, 1])
            self._saved_layers[req.chunk_key].add(idx)

    def wait_for_save(self) -> None:
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, HcpRingConnectorMetadata):
            return
        for req in metadata.requests:
            if not req.is_store or req.chunk_key not in self._stores:
                continue
            store = self._stores[req.chunk_key]
            torch.cuda.current_stream(store.device).synchronize()
            handle = (ctypes.c_uint8 * 64)()
            offset = ctypes.c_int64()
            C.check(C.load().hcp_ipc_export(store.data_ptr(), handle, ctypes.byref(offset)), "hcp_ipc_export")
            marker = dict(tokens=int(store.shape[2]), layers=len(self._saved_layers[req.chunk_key]),
                          ts=time.time(), transport="cuda_ipc", run=self._run_id, chunk=req.chunk_key,
                          pid=os.getpid(), device=store.device.index, handle=bytes(handle).hex(),
                          offset=int(offset.value), shape=list(store.shape),
                          dtype=str(store.dtype).replace("torch.", ""))
            os.makedirs(self._chunk_dir(req.chunk_key), exist_ok=True)
            tmp = self._ready_marker(req.chunk_key) + f".{os.getpid()}.tmp"
            with open(tmp, "w") as f:
                json.dump(marker, f)
            os.replace(tmp, self._ready_marker(req.chunk_key))  # readers never see a partial marker

    # ------------------------------------------------------------------ cleanup
    def get_finished(self, finished_req_ids: set[str]) -> tuple[set[str] | None, set[str] | None]:
        self._cleanup_finished(finished_req_ids)
        return None, None

    def _release_request_staging(self, first_block_id: int) -> None:
        """Backend callback at a decode-ring request's first decode step:
        free its staged prefix (refcounted) and keep its ring registration
        for the decode phase (``ring_connector.py:978-987``)."""
        req_id = self._ledger.request_of_block(first_block_id)
        if req_id is not None:
            self._end_request(req_id, keep_ring_slot=True)

    def _end_request(self, req_id: str, keep_ring_slot: bool = False) -> None:
        """Stop the request's staging thread, release its chunk holds and,
        unless kept for its decode phase, its decode-ring slot."""
        feed = self._feeds.pop(req_id, None)
        if feed is not None:
            feed.stop()
        if not keep_ring_slot:
            fb = self._slots.give_back(req_id)
            if fb is not None:
                clear_decode_ring(fb)
        self._ledger.release(req_id)

    def _cleanup_finished(self, finished_req_ids) -> None:
        for req_id in finished_req_ids:
            self._end_request(req_id)

    @classmethod
    def get_required_kvcache_layout(cls, vllm_config: "VllmConfig") -> str | None:
        return None

    def shutdown(self) -> None:
        for req_id in self._ledger.requests() + self._slots.holders():
            self._end_request(req_id)
        from . import ring_backend
        if ring_backend._STAGING_RELEASE_FN == self._release_request_staging:
            set_staging_release_fn(None)
        if self._decode_owner and self._decode_ring is not None:
            self._decode_ring.stop()          # ends the peers' serve loops
        self._decode_stop.set()
        if self._decode_thread is not None:
            self._decode_thread.join(timeout=30)
        self._ledger.release_all()
        for src in self._sources.values():
            close = getattr(src, "close", None)
            if close is not None:
                close()
        self._sources.clear()
        for ck in list(self._stores):
            _LOCAL_EXPORTS.pop((self._run_id, ck), None)
        self._stores.clear()
