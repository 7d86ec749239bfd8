"""Golden fixture for the hcp-kv-v1 file import, made by the reference itself.

Runs the reference ``HcpFileConnector`` (``hcp_vllm_plugin/file_connector.py``)
on CPU: scheduler side (``get_num_new_matched_tokens``,
``update_state_after_alloc``, ``build_connector_meta``) and worker side
(``start_load_kv`` into ``[num_blocks, Hkv, block_size, 2*D]`` caches), on a
seeded two-layer export, and stores inputs and results in
``file_connector_case.npz`` next to this script.

Usage (in a container holding the reference sources and vLLM)::

    HCP_REFERENCE_ROOT=/path/to/hcp-vllm-plugin python tests/golden/make_file_connector_golden.py
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
import types

import numpy as np
import torch

REF_ROOT = os.environ.get("HCP_REFERENCE_ROOT", "")  # the reference checkout (generation only)
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "file_connector_case.npz")

LAYERS, HKV, D, BS, NUM_BLOCKS, HEADS = 2, 2, 64, 16, 12, 4
PROMPT = list(range(1000, 1045))  # 45 tokens: hit = align_down(44, 16) = 32


def fake_config(kv_dir: str):
    extra = {"hcp_kv_dir": kv_dir}
    kvt = types.SimpleNamespace(get_from_extra_config=lambda k, d=None: extra.get(k, d),
                                kv_connector_extra_config=extra)
    hf = types.SimpleNamespace(hidden_size=HEADS * D, num_attention_heads=HEADS,
                               num_hidden_layers=LAYERS, num_key_value_heads=HKV)
    return types.SimpleNamespace(kv_transfer_config=kvt,
                                 cache_config=types.SimpleNamespace(block_size=BS),
                                 model_config=types.SimpleNamespace(hf_config=hf, dtype=torch.bfloat16))


def write_export(kv_dir: str, kvs: list[torch.Tensor]) -> None:
    from safetensors.torch import save_file

    meta = dict(format="hcp-kv-v1", prompt_token_ids=PROMPT, seq_len=len(PROMPT), num_layers=LAYERS,
                num_kv_heads=HKV, head_dim=D, dtype="bfloat16")
    with open(os.path.join(kv_dir, "meta.json"), "w") as f:
        json.dump(meta, f)
    for i, kv in enumerate(kvs):
        save_file({"kv": kv}, os.path.join(kv_dir, f"layer_{i}.safetensors"))


def main() -> None:
    if not REF_ROOT:
        raise SystemExit("set HCP_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, REF_ROOT)
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin.file_connector import HcpFileConnector  # reference code

    torch.manual_seed(3)
    kvs = [torch.randn(len(PROMPT), 2, HKV, D).to(torch.bfloat16) for _ in range(LAYERS)]
    block_ids = [7, 2, 9, 4]
    out: dict[str, np.ndarray] = {}
    with tempfile.TemporaryDirectory() as kv_dir:
        write_export(kv_dir, kvs)
        cfg = fake_config(kv_dir)
        sched = HcpFileConnector(cfg, KVConnectorRole.SCHEDULER, None)
        req = types.SimpleNamespace(request_id="r0", prompt_token_ids=PROMPT)
        other = types.SimpleNamespace(request_id="r1", prompt_token_ids=PROMPT[:-1] + [1])
        matched = [sched.get_num_new_matched_tokens(req, c)[0] for c in (0, 16, 32)]
        matched_other = sched.get_num_new_matched_tokens(other, 0)[0]
        sched.update_state_after_alloc(req, None, matched[0])
        new_req = types.SimpleNamespace(req_id="r0", prompt_token_ids=PROMPT, block_ids=[block_ids])
        meta = sched.build_connector_meta(types.SimpleNamespace(scheduled_new_reqs=[new_req]))
        worker = HcpFileConnector(cfg, KVConnectorRole.WORKER, None)
        worker.bind_connector_metadata(meta)
        caches = [torch.zeros(NUM_BLOCKS, HKV, BS, 2 * D, dtype=torch.bfloat16) for _ in range(LAYERS)]
        layers = {f"model.layers.{i}.self_attn.attn": types.SimpleNamespace(kv_cache=caches[i])
                  for i in range(LAYERS)}
        worker.start_load_kv(types.SimpleNamespace(no_compile_layers=layers))
        out["slot_mapping"] = meta.requests[0].slot_mapping.numpy().astype(np.int64)
        out["n_tokens"] = np.array([meta.requests[0].n_tokens], np.int64)
    out["matched"] = np.array(matched, np.int64)
    out["matched_other"] = np.array([matched_other], np.int64)
    out["block_ids"] = np.array(block_ids, np.int64)
    out["prompt"] = np.array(PROMPT, np.int64)
    out["geometry"] = np.array([LAYERS, HKV, D, BS, NUM_BLOCKS, HEADS], np.int64)
    for i in range(LAYERS):
        out[f"kv{i}"] = kvs[i].view(torch.int16).numpy().view(np.uint16)
        out[f"cache{i}"] = caches[i].view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
