"""hcp-kv-v1 file import: the reference's decisions and cache contents.

The fixture ``golden/file_connector_case.npz`` is the reference
``HcpFileConnector`` itself run on CPU (``make_file_connector_golden.py``):
its matched-token answers, its slot mapping and the caches its
``start_load_kv`` produced.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import ring_oracle as orc
from tests import vllm_fakes as fk

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "file_connector_case.npz")


@pytest.fixture(scope="module")
def case():
    return dict(np.load(GOLDEN))


def _bf16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(u16.view(np.int16).copy()).view(torch.bfloat16)


def _export(tmp_path, case, **meta_over):
    from safetensors.torch import save_file

    layers, hkv, d, bs, nb, heads = (int(x) for x in case["geometry"])
    meta = dict(format="hcp-kv-v1", prompt_token_ids=case["prompt"].tolist(), seq_len=len(case["prompt"]),
                num_layers=layers, num_kv_heads=hkv, head_dim=d, dtype="bfloat16")
    meta.update(meta_over)
    with open(tmp_path / "meta.json", "w") as f:
        json.dump(meta, f)
    for i in range(layers):
        save_file({"kv": _bf16(case[f"kv{i}"])}, str(tmp_path / f"layer_{i}.safetensors"))
    cfg = fk.vllm_config({"hcp_kv_dir": str(tmp_path)}, block_size=bs, num_layers=layers, num_kv_heads=hkv,
                         head_dim=d, num_heads=heads)
    return cfg


def test_oracle_matches_reference_import(case):
    """The oracle's paged scatter reproduces the reference's start_load_kv."""
    layers, hkv, d, bs, nb, _ = (int(x) for x in case["geometry"])
    n = int(case["n_tokens"][0])
    for i in range(layers):
        kv = orc.bf16_bits_to_f32(case[f"kv{i}"])[:n]
        cache = np.zeros((nb, hkv, bs, 2 * d), np.float32)
        orc.kv_cache_update(cache, kv[:, 0], kv[:, 1], case["slot_mapping"])
        np.testing.assert_array_equal(cache, orc.bf16_bits_to_f32(case[f"cache{i}"]))


def test_scheduler_side_matches_reference(tmp_path, case):
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.file_connector import HcpFileConnector

    cfg = _export(tmp_path, case)
    conn = HcpFileConnector(cfg, KVConnectorRole.SCHEDULER, None)
    prompt = case["prompt"].tolist()
    req = fk.request("r0", prompt)
    got = [conn.get_num_new_matched_tokens(req, c)[0] for c in (0, 16, 32)]
    assert got == case["matched"].tolist()
    other = fk.request("r1", prompt[:-1] + [1])
    assert conn.get_num_new_matched_tokens(other, 0)[0] == int(case["matched_other"][0])
    conn.update_state_after_alloc(req, None, got[0])
    meta = conn.build_connector_meta(fk.scheduler_output([fk.new_request("r0", prompt, case["block_ids"])]))
    assert len(meta.requests) == 1
    assert meta.requests[0].n_tokens == int(case["n_tokens"][0])
    np.testing.assert_array_equal(meta.requests[0].slot_mapping.numpy(), case["slot_mapping"])
    # the pending set is consumed by one build
    assert conn.build_connector_meta(fk.scheduler_output([])).requests == []


@pytest.mark.parametrize("over", [{"num_kv_heads": 3}, {"head_dim": 128}, {"num_layers": 5},
                                  {"dtype": "float16"}, {"format": "other"}])
def test_handshake_mismatch_raises(tmp_path, case, over):
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.file_connector import HcpFileConnector

    cfg = _export(tmp_path, case, **over)
    with pytest.raises(ValueError):
        HcpFileConnector(cfg, KVConnectorRole.WORKER, None)


@pytest.mark.gpu
def test_worker_import_bit_exact(tmp_path, case):
    """Layer-pipelined import (side stream, pinned copies, CUDA scatter) gives
    the reference's caches bit for bit."""
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.file_connector import HcpConnectorMetadata, HcpFileConnector, ReqMeta

    layers, hkv, d, bs, nb, _ = (int(x) for x in case["geometry"])
    cfg = _export(tmp_path, case)
    conn = HcpFileConnector(cfg, KVConnectorRole.WORKER, None)
    sm = torch.from_numpy(case["slot_mapping"])
    conn.bind_connector_metadata(HcpConnectorMetadata(requests=[ReqMeta(sm, int(case["n_tokens"][0]))]))
    caches = {f"model.layers.{i}.self_attn.attn": torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16,
                                                             device="cuda") for i in range(layers)}
    conn.start_load_kv(fk.forward_context(caches))
    for name in caches:
        conn.wait_for_layer_load(name)
    conn.wait_for_save()
    torch.cuda.synchronize()
    for i, (name, c) in enumerate(caches.items()):
        got = c.cpu().view(torch.int16).numpy().view(np.uint16)
        np.testing.assert_array_equal(got, case[f"cache{i}"], err_msg=name)
