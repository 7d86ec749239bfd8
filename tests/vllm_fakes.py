"""Minimal stand-ins for the vLLM objects a KV connector reads (config,
requests, scheduler output, forward context), for tests without an engine."""

from __future__ import annotations

import types

import torch


def vllm_config(extra: dict, *, block_size: int, num_layers: int, num_kv_heads: int, head_dim: int,
                num_heads: int, dtype=torch.bfloat16):
    kvt = types.SimpleNamespace(get_from_extra_config=lambda k, d=None: extra.get(k, d),
                                kv_connector_extra_config=extra)
    hf = types.SimpleNamespace(hidden_size=num_heads * head_dim, num_attention_heads=num_heads,
                               num_hidden_layers=num_layers, num_key_value_heads=num_kv_heads)
    return types.SimpleNamespace(kv_transfer_config=kvt,
                                 cache_config=types.SimpleNamespace(block_size=block_size),
                                 model_config=types.SimpleNamespace(hf_config=hf, dtype=dtype))


def request(req_id: str, prompt, kv_transfer_params: dict | None = None):
    return types.SimpleNamespace(request_id=req_id, prompt_token_ids=list(prompt),
                                 kv_transfer_params=kv_transfer_params)


def new_request(req_id: str, prompt, block_ids, extra_args: dict | None = None):
    sp = types.SimpleNamespace(extra_args=extra_args or {})
    return types.SimpleNamespace(req_id=req_id, prompt_token_ids=list(prompt), block_ids=[list(block_ids)],
                                 sampling_params=sp)


def scheduler_output(new_reqs, finished=()):
    return types.SimpleNamespace(scheduled_new_reqs=list(new_reqs), finished_req_ids=set(finished))


def forward_context(caches: dict):
    return types.SimpleNamespace(
        no_compile_layers={name: types.SimpleNamespace(kv_cache=c) for name, c in caches.items()})
