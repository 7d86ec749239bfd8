"""``HcpFileConnector``: import an ``hcp-kv-v1`` prefill export into the
paged KV cache (the PD route), B200 side.

Contract (the reference's ``hcp_vllm_plugin/file_connector.py:3-25``):

* ``<kv_dir>/meta.json`` holds ``format`` (``"hcp-kv-v1"``),
  ``prompt_token_ids``, ``seq_len``, ``num_layers``, ``num_kv_heads``,
  ``head_dim`` and ``dtype``;
* ``<kv_dir>/layer_<i>.safetensors`` holds ``{"kv": [S, 2, Hkv, D]}``
  (``[:, 0]`` = K, ``[:, 1]`` = V, post-RoPE, model dtype);
* registered as ``KVTransferConfig(kv_connector="HcpFileConnector",
  kv_connector_module_path="hcp_vllm_plugin_b200.file_connector",
  kv_role="kv_consumer", kv_connector_extra_config={"hcp_kv_dir": ...})``.

Scheduler side - the reference's decisions (``file_connector.py:114-150``):
a request hits only when its prompt token ids equal the export's; the hit
covers ``len(prompt) - 1`` tokens aligned down to the block size (the tail,
including the last prompt token, is recomputed so there are logits to
sample); the slot mapping is ``block_id * block_size + offset`` over the
request's blocks.  A mismatch of ``num_layers`` / ``num_kv_heads`` /
``head_dim`` / ``dtype`` with the model raises at construction
(``:90-105``).

Worker side - the reference loads every layer file and scatters it with a
torch ``index_put`` inside ``start_load_kv`` before the forward starts
(``:154-179``).  Here ``start_load_kv`` only starts a loader thread: per
layer, in model order, it reads the file into pinned host memory, copies it
to HBM on a side stream (copy engine) and scatters it into the
``[num_blocks, Hkv, block_size, 2*D]`` cache with one
``hcp_kv_cache_update`` launch on that stream, then records a CUDA event.
``wait_for_layer_load(layer)`` makes the compute stream wait on that layer's
event only, so layer i's attention overlaps the import of layers > i.
"""

from __future__ import annotations

import json
import os
import re
import threading
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any

import torch

from vllm.distributed.kv_transfer.kv_connector.v1.base import (
    KVConnectorBase_V1,
    KVConnectorMetadata,
    KVConnectorRole,
)

from . import ops

if TYPE_CHECKING:
    from vllm.config import VllmConfig
    from vllm.forward_context import ForwardContext
    from vllm.v1.core.kv_cache_manager import KVCacheBlocks
    from vllm.v1.core.sched.output import SchedulerOutput
    from vllm.v1.kv_cache_interface import KVCacheConfig
    from vllm.v1.request import Request

FORMAT = "hcp-kv-v1"
_LAYER_RE = re.compile(r"layers\.(\d+)\.")


def align_down(n: int, block_size: int) -> int:
    return n // block_size * block_size


def slot_mapping_for(block_ids, block_size: int, n_tokens: int) -> torch.Tensor:
    """Slots of the first ``n_tokens`` positions of a request whose blocks are
    ``block_ids`` (``file_connector.py:141-147``): int64 [n_tokens]."""
    blocks = torch.as_tensor(list(block_ids), dtype=torch.int64)
    offs = torch.arange(block_size, dtype=torch.int64)
    return (blocks[:, None] * block_size + offs[None, :]).flatten()[:n_tokens].contiguous()


def layer_index(layer_name: str) -> int:
    m = _LAYER_RE.search(layer_name)
    if m is None:
        raise ValueError(f"cannot parse a layer index from {layer_name!r}")
    return int(m.group(1))


@dataclass
class ReqMeta:
    slot_mapping: torch.Tensor  # int64 [n_tokens]
    n_tokens: int


@dataclass
class HcpConnectorMetadata(KVConnectorMetadata):
    requests: list[ReqMeta] = field(default_factory=list)


class _LayerImport:
    """One step's import: a loader thread plus per-layer completion state."""

    def __init__(self, layers: list[str]):
        self.ready = {ln: threading.Event() for ln in layers}
        self.cuda_events: dict[str, torch.cuda.Event] = {}
        self.error: BaseException | None = None
        self.thread: threading.Thread | None = None


class HcpFileConnector(KVConnectorBase_V1):
    """Consumer of an ``hcp-kv-v1`` export (TP=1 contract, no hybrid KV manager)."""

    def __init__(self, vllm_config: "VllmConfig", role: KVConnectorRole,
                 kv_cache_config: "KVCacheConfig" = None):
        super().__init__(vllm_config=vllm_config, role=role, kv_cache_config=kv_cache_config)
        self._block_size = vllm_config.cache_config.block_size
        kv_dir = self._kv_transfer_config.get_from_extra_config("hcp_kv_dir", None)
        if not kv_dir:
            raise ValueError("hcp_kv_dir missing in kv_connector_extra_config")
        self._kv_dir = kv_dir
        with open(os.path.join(kv_dir, "meta.json")) as f:
            self._meta = json.load(f)
        if self._meta.get("format") != FORMAT:
            raise ValueError(f"{kv_dir}: format {self._meta.get('format')!r} is not {FORMAT!r}")
        hf = vllm_config.model_config.hf_config
        head_dim = hf.hidden_size // hf.num_attention_heads
        for name, mine, model in (("num_layers", self._meta["num_layers"], hf.num_hidden_layers),
                                  ("num_kv_heads", self._meta["num_kv_heads"], hf.num_key_value_heads),
                                  ("head_dim", self._meta["head_dim"], head_dim)):
            if mine != model:
                raise ValueError(f"HCP KV meta mismatch: {name} {mine} != vllm {model}")
        model_dtype = str(vllm_config.model_config.dtype).replace("torch.", "")
        if model_dtype != self._meta["dtype"]:
            raise ValueError(f"HCP KV dtype mismatch: {self._meta['dtype']} != vllm {model_dtype}")
        self._prompt = list(self._meta["prompt_token_ids"])
        self._requests_need_load: dict[str, Any] = {}
        self._import: _LayerImport | None = None
        self._stream: torch.cuda.Stream | None = None

    # ------------------------------------------------------------------ scheduler side
    def _hit_tokens(self, token_ids) -> int:
        return align_down(len(token_ids) - 1, self._block_size)

    def get_num_new_matched_tokens(self, request: "Request",
                                   num_computed_tokens: int) -> tuple[int | None, bool]:
        token_ids = list(request.prompt_token_ids or [])
        if token_ids != self._prompt:
            return 0, False
        n = self._hit_tokens(token_ids)
        if n <= num_computed_tokens:
            return 0, False
        return n - num_computed_tokens, False

    def update_state_after_alloc(self, request: "Request", blocks: "KVCacheBlocks",
                                 num_external_tokens: int) -> None:
        if num_external_tokens > 0:
            self._requests_need_load[request.request_id] = request

    def build_connector_meta(self, scheduler_output: "SchedulerOutput") -> HcpConnectorMetadata:
        meta = HcpConnectorMetadata()
        for new_req in scheduler_output.scheduled_new_reqs:
            if new_req.req_id not in self._requests_need_load:
                continue
            n_load = self._hit_tokens(list(new_req.prompt_token_ids or []))
            meta.requests.append(ReqMeta(
                slot_mapping=slot_mapping_for(new_req.block_ids[0], self._block_size, n_load),
                n_tokens=n_load))
        self._requests_need_load.clear()
        return meta

    # ------------------------------------------------------------------ worker side
    def _layer_file(self, idx: int) -> str:
        return os.path.join(self._kv_dir, f"layer_{idx}.safetensors")

    def _run_import(self, job: _LayerImport, layers: list[tuple[str, torch.Tensor]],
                    requests: list[ReqMeta]) -> None:
        from safetensors.torch import load_file

        try:
            device = layers[0][1].device
            torch.cuda.set_device(device)
            stream = self._stream
            slots = [r.slot_mapping.to(device, non_blocking=False) for r in requests]
            n_max = max(r.n_tokens for r in requests)
            in_flight: list[tuple[torch.cuda.Event, torch.Tensor]] = []
            for layer_name, cache in layers:
                kv = load_file(self._layer_file(layer_index(layer_name)))["kv"]
                if kv.dim() != 4 or kv.shape[1] != 2 or kv.dtype != cache.dtype:
                    raise ValueError(f"{layer_name}: kv {tuple(kv.shape)} {kv.dtype} does not match "
                                     f"the cache ({cache.dtype})")
                if kv.shape[0] < n_max:
                    raise ValueError(f"{layer_name}: export holds {kv.shape[0]} tokens, "
                                     f"{n_max} requested")
                host = kv[:n_max].pin_memory()
                with torch.cuda.stream(stream):
                    dev = host.to(device, non_blocking=True)
                    for req, sm in zip(requests, slots):
                        part = dev[:req.n_tokens]
                        ops.kv_cache_update(part[:, 0], part[:, 1], cache, sm)
                    ev = torch.cuda.Event()
                    ev.record(stream)
                job.cuda_events[layer_name] = ev
                job.ready[layer_name].set()
                # A pinned buffer must outlive the copy that reads it; keep two
                # layers in flight so reading the next file overlaps the copy.
                in_flight.append((ev, host))
                if len(in_flight) > 2:
                    in_flight.pop(0)[0].synchronize()
            for ev, _ in in_flight:
                ev.synchronize()
        except BaseException as e:  # noqa: BLE001 - re-raised on the worker thread
            job.error = e
            for ev in job.ready.values():
                ev.set()

    def start_load_kv(self, forward_context: "ForwardContext", **kwargs: Any) -> None:
        metadata = self._get_connector_metadata()
        if not isinstance(metadata, HcpConnectorMetadata) or not metadata.requests:
            return
        self._finish_import()
        layers = []
        for layer_name, layer in forward_context.no_compile_layers.items():
            cache = getattr(layer, "kv_cache", None)
            if isinstance(cache, (list, tuple)):
                cache = cache[0] if cache else None
            if torch.is_tensor(cache) and cache.numel() > 0:
                layers.append((layer_name, cache))
        if not layers:
            return
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=layers[0][1].device)
        job = _LayerImport([ln for ln, _ in layers])
        job.thread = threading.Thread(target=self._run_import,
                                      args=(job, layers, list(metadata.requests)), daemon=True)
        self._import = job
        job.thread.start()

    def wait_for_layer_load(self, layer_name: str) -> None:
        job = self._import
        if job is None or layer_name not in job.ready:
            return
        job.ready[layer_name].wait()
        if job.error is not None:
            raise RuntimeError(f"HcpFileConnector: import of {layer_name} failed") from job.error
        torch.cuda.current_stream().wait_event(job.cuda_events[layer_name])

    def _finish_import(self) -> None:
        """Order every imported layer before the compute stream's later work
        and retire the loader thread (also covers layers the model never
        waited for)."""
        job, self._import = self._import, None
        if job is None:
            return
        if job.thread is not None:
            job.thread.join()
        if job.error is not None:
            raise RuntimeError("HcpFileConnector: KV import failed") from job.error
        for ev in job.cuda_events.values():
            torch.cuda.current_stream().wait_event(ev)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata: Any,
                      **kwargs: Any) -> None:
        return

    def wait_for_save(self) -> None:
        self._finish_import()
