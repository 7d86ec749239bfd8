"""HcpRingKvConnector: the reference's scheduler decisions, the streaming /
refcount host logic, and the NVLink (CUDA IPC) chunk transport.

* ``golden/ring_connector_case.json`` holds the reference connector's own
  answers (``make_ring_connector_golden.py``); the same scenarios replayed
  here must agree.  One deliberate difference: with peer urls configured the
  reference polls the peer over HTTP, while inside the box readiness is the
  marker in the shared directory, so the ``ring_order`` scenario (which has
  urls) is compared on its metadata only.
* Worker-side host logic runs on CPU with a fake chunk source (the same
  substitution ``RingPrefill`` uses for its device ops).
* GPU tests move real chunks: same process, across processes on one GPU
  (CUDA IPC), and across two GPUs when the box has them.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time

import numpy as np
import pytest
import torch

from oracle import ring_oracle as orc
from tests import vllm_fakes as fk
from tests.golden import make_ring_connector_golden as gold

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "ring_connector_case.json")

L, HKV, D, BS, NB = 4, 4, 128, 16, 40
CHUNK_BLOCKS = [5, 17, 2, 30, 11, 8]          # producer's own chunk: 6 blocks = 96 tokens


def _config(extra, layers=L):
    return fk.vllm_config(extra, block_size=BS, num_layers=layers, num_kv_heads=HKV, head_dim=D, num_heads=28)


@pytest.fixture(autouse=True)
def _clean_staging():
    from hcp_vllm_plugin_b200 import ring_backend as rb
    rb.clear_peer_kv()
    rb.reset_staging_stats()
    yield
    rb.clear_peer_kv()


# ---------------------------------------------------------------------------
# scheduler side vs the reference
# ---------------------------------------------------------------------------
def test_scheduler_decisions_match_reference():
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200 import ring_connector as rc

    with open(GOLDEN) as f:
        ref = json.load(f)

    def fake_config(extra):
        return fk.vllm_config(extra, block_size=gold.BS, num_layers=2, num_kv_heads=4, head_dim=128, num_heads=28)

    mine = gold.run(rc.HcpRingKvConnector, KVConnectorRole.SCHEDULER, rc.chunks_and_urls, fake_config)
    assert mine["urls"] == ref["urls"]
    for name, r in ref["scenarios"].items():
        m = mine["scenarios"][name]
        assert m["meta"] == r["meta"], name
        assert m["finished"] == r["finished"], name
        assert m["before"] == r["before"], name
        if name == "ring_order":
            # in-box readiness is the local marker: ready once written
            assert m["after"] == [[4096, False], [4096, False]]
        else:
            assert m["after"] == r["after"], name


def test_poll_backoff():
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.ring_connector import HcpRingKvConnector

    import tempfile
    with tempfile.TemporaryDirectory() as shared:
        conn = HcpRingKvConnector(_config(dict(ring_role="consumer", ring_shared_path=shared, ring_run_id="run",
                                               ring_prefix_chunk_ids="c0", ring_prefix_len=64,
                                               ring_ready_poll_interval_s=30)), KVConnectorRole.SCHEDULER)
        req = fk.request("r", range(100))
        assert conn.get_num_new_matched_tokens(req, 0) == (None, True)
        os.makedirs(os.path.join(shared, "run", "c0"))
        open(os.path.join(shared, "run", "c0", "_READY"), "w").close()
        # inside the back-off window the marker is not looked at again
        assert conn.get_num_new_matched_tokens(req, 0) == (None, True)
        conn._readiness.look_again_now()
        assert conn.get_num_new_matched_tokens(req, 0) == (64, False)


# ---------------------------------------------------------------------------
# worker-side host logic on CPU
# ---------------------------------------------------------------------------
STORES: dict[str, torch.Tensor] = {}


class FakeSource:
    """CPU stand-in for a mapped chunk store."""

    def __init__(self, marker, device):
        self.store = STORES[marker["chunk"]]
        self.shape = list(self.store.shape)
        self.dtype = self.store.dtype
        self.copies = 0

    def copy_layer(self, idx, k, v, stream):
        k.copy_(self.store[idx, 0])
        v.copy_(self.store[idx, 1])

    def close(self):
        pass


def _write_marker(shared, chunk, store):
    d = os.path.join(shared, "run", chunk)
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "_READY"), "w") as f:
        json.dump({"chunk": chunk, "tokens": store.shape[2]}, f)


def _layers(n):
    return [f"model.layers.{i}.self_attn.attn" for i in range(n)]


class FakeRing:
    """Stand-in for the decode ring's state (no process group): records the
    chunks a peer's serve loop reads."""

    def __init__(self):
        self.served = None
        self.stopped = False

    def serve(self, chunk_fn, stop):
        while not stop.is_set():
            try:
                self.served = [chunk_fn(i) for i in range(2)]
                break
            except RuntimeError:          # chunk not saved yet
                stop.wait(0.01)
        stop.wait(30)

    def stop(self):
        self.stopped = True


# the owner of a 3-node decode ring (config only: the ring itself is faked)
OWNER = dict(ring_decode_addr="127.0.0.1:1", ring_decode_index=2, ring_decode_world=3)


def _consumer(shared, layers, extra=None, role="consumer"):
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.ring_connector import HcpRingKvConnector

    cfg = dict(ring_role=role, ring_shared_path=shared, ring_run_id="run")
    cfg.update(extra or {})

    class CpuConnector(HcpRingKvConnector):
        source_cls = FakeSource

        def _make_decode_ring(self, device):
            return FakeRing()

    return CpuConnector(_config(cfg, layers=layers), KVConnectorRole.WORKER)


def _load_meta(reqs, finished=()):
    from hcp_vllm_plugin_b200.ring_connector import HcpRingConnectorMetadata, RingReqMeta
    return HcpRingConnectorMetadata(
        requests=[RingReqMeta(is_store=False, chunk_key="", req_id=rid, first_block_id=fb, chunk_keys=cks,
                              peer_urls=[""] * len(cks), prefix_len=plen) for rid, fb, cks, plen in reqs],
        finished_req_ids=list(finished))


@pytest.mark.parametrize("window", [1, 2, 3])
def test_streaming_window_and_refcounts(tmp_path, monkeypatch, window):
    """Decode-ring owner: memory-split staging (consumed layers freed at once,
    ``ring_connector.py:861-879``), each request registered for the ring
    with its own slot, released when it finishes."""
    from hcp_vllm_plugin_b200 import ring_backend as rb

    monkeypatch.setenv("HCP_RING_STREAM_WINDOW", str(window))
    nl = 6
    g = torch.Generator().manual_seed(window)
    STORES.clear()
    STORES["c0"] = torch.randn(nl, 2, 32, 2, 8, generator=g)
    STORES["c1"] = torch.randn(nl, 2, 48, 2, 8, generator=g)
    for ck, st in STORES.items():
        _write_marker(str(tmp_path), ck, st)
    conn = _consumer(str(tmp_path), nl, OWNER)
    conn.bind_connector_metadata(_load_meta([("r0", 3, ["c0", "c1"], 80), ("r1", 9, ["c0"], 32)]))
    names = _layers(nl)
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    assert rb.PEER_REQ_MAP == {3: ["c0", "c1"], 9: ["c0"]}
    assert {fb: (e["slot"], e["prefix_len"]) for fb, e in rb.DECODE_RING_MAP.items()} == {3: (0, 80), 9: (1, 32)}
    for i, name in enumerate(names):
        conn.wait_for_layer_load(name)
        for ck in ("c0", "c1"):
            k, v = rb.PEER_KV_STAGING[(ck, name)]
            torch.testing.assert_close(k, STORES[ck][i, 0], rtol=0, atol=0)
            torch.testing.assert_close(v, STORES[ck][i, 1], rtol=0, atol=0)
        # consumed layers are gone, and nothing is staged past the window
        layers_staged = {int(key[1].split(".")[2]) for key in rb.PEER_KV_STAGING}
        assert min(layers_staged) >= i
        assert max(layers_staged) <= i + window + 1
    assert rb.STAGING_STATS["max_staged_layers"] <= (window + 2) * 2
    # r0 starts decoding: the backend frees its staging (c1 is r0's only, c0
    # is shared with r1) and its ring registration stays (ring_connector.py:978-987)
    rb._release_staged_for_request(3)
    assert 3 not in rb.PEER_REQ_MAP and 9 in rb.PEER_REQ_MAP and 3 in rb.DECODE_RING_MAP
    assert not any(key[0] == "c1" for key in rb.PEER_KV_STAGING) and conn._ledger.holder_counts() == {"c0": 1}
    # r0 finishes: its ring slot is released, c0 (shared with r1) stays
    conn.bind_connector_metadata(_load_meta([], finished=["r0"]))
    conn.start_load_kv(fk.forward_context({}))
    assert 3 not in rb.PEER_REQ_MAP and 9 in rb.PEER_REQ_MAP
    assert not any(key[0] == "c1" for key in rb.PEER_KV_STAGING)
    assert any(key[0] == "c0" for key in rb.PEER_KV_STAGING)
    assert list(rb.DECODE_RING_MAP) == [9] and list(conn._slots.free) == [2, 3, 0]
    conn.get_finished({"r1"})
    assert rb.PEER_REQ_MAP == {} and rb.PEER_KV_STAGING == {} and rb.DECODE_RING_MAP == {}
    conn.shutdown()
    assert conn._decode_ring.stopped            # the owner ends the peers' loops


def test_staging_kept_without_decode_ring(tmp_path):
    """No decode ring: decode steps read the staged prefix again, so it stays
    until the request finishes (the reference's bulk staging)."""
    from hcp_vllm_plugin_b200 import ring_backend as rb

    nl = 3
    STORES.clear()
    STORES["c0"] = torch.randn(nl, 2, 16, 2, 8)
    _write_marker(str(tmp_path), "c0", STORES["c0"])
    conn = _consumer(str(tmp_path), nl)
    conn.bind_connector_metadata(_load_meta([("r0", 5, ["c0"], 16)]))
    names = _layers(nl)
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    for step in range(2):                       # the prefill step, then a decode step
        if step:
            conn.bind_connector_metadata(_load_meta([]))
            conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
        for i, name in enumerate(names):
            conn.wait_for_layer_load(name)
            torch.testing.assert_close(rb.PEER_KV_STAGING[("c0", name)][0], STORES["c0"][i, 0], rtol=0, atol=0)
    assert len(rb.PEER_KV_STAGING) == nl and rb.DECODE_RING_MAP == {}
    conn.get_finished({"r0"})
    assert rb.PEER_KV_STAGING == {} and rb.PEER_REQ_MAP == {}
    conn.shutdown()


def test_decode_ring_peer_serves_its_chunk_store(tmp_path):
    """A peer node (rank 0 of 2) runs the ring's serve loop in a worker
    thread over its own chunk store; shutdown ends it."""
    conn = _consumer(str(tmp_path), 2, dict(ring_decode_addr="127.0.0.1:1", ring_decode_index=0,
                                             ring_decode_world=2, ring_chunk_id="c0"), role="producer")
    assert conn._decode_thread is not None and not conn._decode_owner
    store = torch.randn(2, 2, 16, 2, 8)
    conn._stores["c0"] = store                   # what save_kv_layer builds
    t0 = time.time()
    while conn._decode_ring is None or conn._decode_ring.served is None:
        assert time.time() - t0 < 30
        time.sleep(0.01)
    for layer, (k, v) in enumerate(conn._decode_ring.served):
        assert k.data_ptr() == store[layer, 0].data_ptr() and v.data_ptr() == store[layer, 1].data_ptr()
    conn.shutdown()
    assert not conn._decode_thread.is_alive() and conn._decode_error is None


def test_producer_resave_reads_the_new_requests_blocks(tmp_path, monkeypatch):
    """Two requests save the same chunk key, equal length, different blocks:
    the second save must gather from the second request's blocks (the device
    gather is replaced by a CPU restatement of the pool -> chunk copy)."""
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200 import ring_connector as rc

    def cpu_gather(cache, slots, key, value):
        blk, off = slots // BS, slots % BS
        rows = cache[blk, :, off]                       # [n, Hkv, 2D]
        key.copy_(rows[..., :D])
        value.copy_(rows[..., D:])

    monkeypatch.setattr(rc.ops, "kv_cache_gather", cpu_gather)
    caches = _cache(21, "cpu")
    prod = rc.HcpRingKvConnector(_config(dict(ring_role="producer", ring_shared_path=str(tmp_path),
                                              ring_run_id="run", ring_chunk_id="c0")), KVConnectorRole.WORKER)
    for blocks in (CHUNK_BLOCKS, [b + 1 for b in CHUNK_BLOCKS]):
        sm = (torch.tensor(blocks)[:, None] * BS + torch.arange(BS)[None, :]).flatten()
        prod.bind_connector_metadata(rc.HcpRingConnectorMetadata(
            requests=[rc.RingReqMeta(is_store=True, chunk_key="c0", slot_mapping=sm)]))
        for i, c in enumerate(caches):
            prod.save_kv_layer(f"model.layers.{i}.self_attn.attn", c, None)
        store = prod._stores["c0"]
        np_sm = sm.numpy()
        for i, c in enumerate(caches):
            want_k, want_v = orc.kv_cache_gather(c.view(torch.int16).numpy().view(np.uint16), np_sm)
            np.testing.assert_array_equal(store[i, 0].view(torch.int16).numpy().view(np.uint16), want_k)
            np.testing.assert_array_equal(store[i, 1].view(torch.int16).numpy().view(np.uint16), want_v)
    prod.shutdown()


def test_missing_chunk_raises(tmp_path):
    STORES.clear()
    conn = _consumer(str(tmp_path), 2)
    conn.bind_connector_metadata(_load_meta([("r0", 1, ["nope"], 16)]))
    names = _layers(2)
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    with pytest.raises(RuntimeError):
        conn.wait_for_layer_load(names[0])
    conn.shutdown()


def test_prefix_length_mismatch_raises(tmp_path):
    STORES.clear()
    STORES["c0"] = torch.zeros(2, 2, 32, 2, 8)
    _write_marker(str(tmp_path), "c0", STORES["c0"])
    conn = _consumer(str(tmp_path), 2)
    conn.bind_connector_metadata(_load_meta([("r0", 1, ["c0"], 48)]))   # 48 expected, 32 staged
    names = _layers(2)
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    conn._feeds["r0"].join()
    with pytest.raises(RuntimeError):
        conn.wait_for_layer_load(names[1])
    conn.shutdown()


# ---------------------------------------------------------------------------
# GPU: real chunk stores over CUDA IPC / NVLink
# ---------------------------------------------------------------------------
def _cache(seed: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(NB, HKV, BS, 2 * D, generator=g).to(torch.bfloat16).to(device) for _ in range(L)]


def produce(shared: str, device, seed: int):
    """Save the seeded chunk through a producer connector (used in-process and
    by ``ring_connector_worker.py``)."""
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200.ring_connector import HcpRingConnectorMetadata, HcpRingKvConnector, RingReqMeta

    caches = _cache(seed, device)
    prod = HcpRingKvConnector(_config(dict(ring_role="producer", ring_shared_path=shared, ring_run_id="run",
                                           ring_chunk_id="c0")), KVConnectorRole.WORKER)
    sm = (torch.tensor(CHUNK_BLOCKS)[:, None] * BS + torch.arange(BS)[None, :]).flatten()
    prod.bind_connector_metadata(HcpRingConnectorMetadata(
        requests=[RingReqMeta(is_store=True, chunk_key="c0", slot_mapping=sm)]))
    for i, c in enumerate(caches):
        prod.save_kv_layer(f"model.layers.{i}.self_attn.attn", c, None)
    prod.wait_for_save()
    return prod


def _expected(seed: int):
    caches = _cache(seed, "cpu")
    sm = (np.array(CHUNK_BLOCKS)[:, None] * BS + np.arange(BS)[None, :]).reshape(-1)
    out = []
    for c in caches:
        bits = c.view(torch.int16).numpy().view(np.uint16)
        out.append(orc.kv_cache_gather(bits, sm))
    return out


def _consume_and_check(shared: str, device, seed: int):
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin_b200 import ring_backend as rb
    from hcp_vllm_plugin_b200.ring_connector import HcpRingKvConnector

    cons = HcpRingKvConnector(_config(dict(ring_role="consumer", ring_shared_path=shared, ring_run_id="run",
                                           ring_prefix_chunk_ids="c0", ring_prefix_len=96)), KVConnectorRole.WORKER)
    cons.bind_connector_metadata(_load_meta([("r0", 77, ["c0"], 96)]))
    names = _layers(L)
    local = {n: torch.zeros(NB, HKV, BS, 2 * D, dtype=torch.bfloat16, device=device) for n in names}
    cons.start_load_kv(fk.forward_context(local))
    exp = _expected(seed)
    for i, name in enumerate(names):
        cons.wait_for_layer_load(name)
        k, v = rb.PEER_KV_STAGING[("c0", name)]
        assert k.device == torch.device(device) and k.shape == (96, HKV, D)
        torch.cuda.current_stream().synchronize()
        np.testing.assert_array_equal(k.cpu().view(torch.int16).numpy().view(np.uint16), exp[i][0], err_msg=name)
        np.testing.assert_array_equal(v.cpu().view(torch.int16).numpy().view(np.uint16), exp[i][1], err_msg=name)
    cons.get_finished({"r0"})
    assert rb.PEER_KV_STAGING == {}
    cons.shutdown()


@pytest.mark.gpu
def test_chunk_transport_same_process(tmp_path):
    prod = produce(str(tmp_path), torch.device("cuda", 0), seed=11)
    with open(tmp_path / "run" / "c0" / "_READY") as f:
        marker = json.load(f)
    assert marker["tokens"] == 96 and marker["layers"] == L and marker["transport"] == "cuda_ipc"
    _consume_and_check(str(tmp_path), "cuda:0", seed=11)
    prod.shutdown()


def _cross_process(tmp_path, prod_dev: int, cons_dev: int):
    shared = str(tmp_path)
    env = dict(os.environ, PYTHONPATH=ROOT)
    proc = subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "ring_connector_worker.py"), shared,
                             str(prod_dev), "12"], env=env)
    try:
        marker = os.path.join(shared, "run", "c0", "_READY")
        t0 = time.time()
        while not os.path.exists(marker):
            assert proc.poll() is None, "producer exited early"
            assert time.time() - t0 < 300, "producer did not publish its chunk"
            time.sleep(0.05)
        with torch.cuda.device(cons_dev):   # restores the current device afterwards
            _consume_and_check(shared, f"cuda:{cons_dev}", seed=12)
    finally:
        open(os.path.join(shared, "done"), "w").close()
        assert proc.wait(timeout=240) == 0


@pytest.mark.gpu
def test_chunk_transport_cuda_ipc_one_gpu(tmp_path):
    _cross_process(tmp_path, 0, 0)


@pytest.mark.gpu
def test_chunk_transport_nvlink_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _cross_process(tmp_path, 0, 1)


@pytest.mark.gpu
def test_connector_staging_feeds_backend_forward(tmp_path):
    """The reference's data flow on this package: two producers save chunks
    c0, c1 from their paged caches; a consumer connector stages them for a
    request (prefix [c0, c1]); the CUSTOM backend's forward, layer by layer
    after wait_for_layer_load, reads the staged chunks as the non-causal
    peer prefix and the request's own keys from its cache.  Compared with
    the oracle's restatement of the reference forward with the same staged
    prefix (tolerance 2e-3 + 2^-7 |ref|)."""
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    import types
    from hcp_vllm_plugin_b200 import ring_backend as rb
    from hcp_vllm_plugin_b200.ring_connector import HcpRingConnectorMetadata, HcpRingKvConnector, RingReqMeta

    dev = torch.device("cuda:0")
    shared = str(tmp_path)
    layers, h = 2, 28
    names = [f"model.layers.{i}.self_attn.attn" for i in range(layers)]
    g = torch.Generator().manual_seed(21)

    def rnd(*shape):
        return torch.randn(*shape, generator=g).to(torch.bfloat16)

    # producers: chunk c0 (64 tokens), c1 (48 tokens) out of their own pools
    chunk_blocks = {"c0": [3, 7, 1, 9], "c1": [2, 5, 8]}
    prod_caches = {ck: [rnd(12, HKV, BS, 2 * D) for _ in range(layers)] for ck in chunk_blocks}
    producers = []
    for ck, blocks in chunk_blocks.items():
        prod = HcpRingKvConnector(_config(dict(ring_role="producer", ring_shared_path=shared, ring_run_id="run",
                                               ring_chunk_id=ck), layers=layers), KVConnectorRole.WORKER)
        sm = (torch.tensor(blocks)[:, None] * BS + torch.arange(BS)[None, :]).flatten()
        prod.bind_connector_metadata(HcpRingConnectorMetadata(
            requests=[RingReqMeta(is_store=True, chunk_key=ck, slot_mapping=sm)]))
        for i, n in enumerate(names):
            prod.save_kv_layer(n, prod_caches[ck][i].to(dev), None)
        prod.wait_for_save()
        producers.append(prod)
    prefix = sum(len(b) * BS for b in chunk_blocks.values())          # 112 tokens
    # consumer: one request with 40 new tokens after the prefix
    tq = 40
    tk = prefix + tq
    nbl = (tk + BS - 1) // BS
    bt = torch.tensor([[30 + i for i in range(nbl)]], dtype=torch.int32)
    cons_caches = [rnd(30 + nbl, HKV, BS, 2 * D) for _ in range(layers)]
    queries = [rnd(tq, h, D) for _ in range(layers)]
    cons = HcpRingKvConnector(_config(dict(ring_role="consumer", ring_shared_path=shared, ring_run_id="run",
                                           ring_prefix_chunk_ids="c0,c1", ring_prefix_len=prefix), layers=layers),
                              KVConnectorRole.WORKER)
    cons.bind_connector_metadata(_load_meta([("r0", int(bt[0, 0]), ["c0", "c1"], prefix)]))
    dev_caches = {n: c.to(dev) for n, c in zip(names, cons_caches)}
    cons.start_load_kv(fk.forward_context(dev_caches))
    impl = rb.HcpRingAttentionImpl(h, D, D ** -0.5, HKV)
    meta = types.SimpleNamespace(num_actual_tokens=tq, query_start_loc=torch.tensor([0, tq], dtype=torch.int32, device=dev),
                                 seq_lens=torch.tensor([tk], dtype=torch.int32, device=dev), block_table=bt.to(dev))
    for i, n in enumerate(names):
        cons.wait_for_layer_load(n)
        out = torch.zeros(tq, h, D, dtype=torch.bfloat16, device=dev)
        impl.forward(types.SimpleNamespace(layer_name=n), queries[i].to(dev), None, None, dev_caches[n], meta, out)
        torch.cuda.synchronize()
        # oracle: the same staged prefix (chunks gathered from the producers' pools)
        kp, vp = [], []
        for ck, blocks in chunk_blocks.items():
            sm = (np.array(blocks)[:, None] * BS + np.arange(BS)[None, :]).reshape(-1)
            k, v = orc.kv_cache_gather(prod_caches[ck][i].float().numpy(), sm)
            kp.append(k)
            vp.append(v)
        batch = orc.RingBatch(query=queries[i].float().numpy(), cache=cons_caches[i].float().numpy(),
                              block_table=bt.numpy(), query_start_loc=np.array([0, tq]), seq_lens=np.array([tk]),
                              scale=D ** -0.5, staged={0: (np.concatenate(kp), np.concatenate(vp))})
        want = orc.ring_forward(batch, round_to_bf16=False)
        import parity as P
        P.check_out(out.float().cpu().numpy(), want, f"connector-staged forward {n}")
    cons.get_finished({"r0"})
    assert rb.PEER_KV_STAGING == {} and rb.PEER_REQ_MAP == {}
    cons.shutdown()
    for prod in producers:
        prod.shutdown()


def test_decode_ring_slots_exhausted(tmp_path):
    """More decode-ring requests than ``ring_decode_slots`` at once is an
    error, not a shared slot."""
    from hcp_vllm_plugin_b200 import ring_backend as rb

    STORES.clear()
    STORES["c0"] = torch.zeros(2, 2, 16, 2, 8)
    _write_marker(str(tmp_path), "c0", STORES["c0"])
    conn = _consumer(str(tmp_path), 2, dict(OWNER, ring_decode_slots=1))
    conn.bind_connector_metadata(_load_meta([("r0", 1, ["c0"], 16), ("r1", 2, ["c0"], 16)]))
    with pytest.raises(RuntimeError, match="slots"):
        conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in _layers(2)}))
    assert conn._ledger.requests() == ["r0"] and 2 not in rb.PEER_REQ_MAP   # r1 left no state behind
    conn.shutdown()


def test_a_request_loaded_again_replaces_its_registration(tmp_path):
    """A request the scheduler hands the worker again while it is still
    registered (resumed after preemption, it is rescheduled from its
    prefill, with new blocks): its old chunk holds, backend mapping and
    decode-ring slot are returned before the new ones are taken, so nothing
    leaks and the step does not fail."""
    from hcp_vllm_plugin_b200 import ring_backend as rb

    STORES.clear()
    STORES["c0"] = torch.randn(2, 2, 16, 2, 8)
    _write_marker(str(tmp_path), "c0", STORES["c0"])
    conn = _consumer(str(tmp_path), 2, dict(OWNER, ring_decode_slots=2))
    names = _layers(2)
    conn.bind_connector_metadata(_load_meta([("r0", 4, ["c0"], 16)]))
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    for name in names:
        conn.wait_for_layer_load(name)
    conn.bind_connector_metadata(_load_meta([("r0", 8, ["c0"], 16)]))   # the same request, new blocks
    conn.start_load_kv(fk.forward_context({n: torch.empty(0) for n in names}))
    for name in names:
        conn.wait_for_layer_load(name)
    assert rb.PEER_REQ_MAP == {8: ["c0"]} and list(rb.DECODE_RING_MAP) == [8]
    assert conn._ledger.holder_counts() == {"c0": 1} and conn._slots.holders() == ["r0"]
    assert len(conn._slots.free) == 1                    # one slot in use, none leaked
    conn.get_finished({"r0"})
    assert rb.PEER_REQ_MAP == {} and rb.DECODE_RING_MAP == {} and len(conn._slots.free) == 2
    conn.shutdown()
