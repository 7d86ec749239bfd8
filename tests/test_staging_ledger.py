"""The ring connector's worker-side bookkeeping (``staging_ledger``), on CPU.

Contract (reference ``hcp_vllm_plugin/ring_connector.py:144-170, 594-604,
939-997``): a chunk stays staged while any request holds it; staging runs at
most a window of layers ahead of consumption; absent ready markers are looked
for again only after the poll interval; decode-ring slots are reused."""

import threading
import time

import pytest
import torch

from hcp_vllm_plugin_b200 import ring_backend as rb
from hcp_vllm_plugin_b200.staging_ledger import ChunkLedger, DecodeSlotPool, LayerFeed, ReadinessCache


@pytest.fixture(autouse=True)
def _clean_registry():
    rb.clear_peer_kv()
    yield
    rb.clear_peer_kv()


def _stage(ck, layer):
    rb.stage_peer_kv(ck, layer, torch.zeros(4, 1, 8), torch.zeros(4, 1, 8))


def test_chunk_ledger_drops_a_chunk_with_its_last_holder():
    led = ChunkLedger()
    for ck in ("a", "b"):
        _stage(ck, "model.layers.0.attn")
    led.hold("r1", 10, ["a", "b"])
    led.hold("r2", 20, ["a"])
    assert rb.PEER_REQ_MAP[10] == ["a", "b"] and rb.PEER_REQ_MAP[20] == ["a"]
    assert led.holder_counts() == {"a": 2, "b": 1}
    assert led.request_of_block(20) == "r2"
    with pytest.raises(RuntimeError):
        led.hold("r1", 11, ["a"])
    assert led.release("r1")
    assert 10 not in rb.PEER_REQ_MAP
    assert ("a", "model.layers.0.attn") in rb.PEER_KV_STAGING      # r2 still holds it
    assert ("b", "model.layers.0.attn") not in rb.PEER_KV_STAGING
    assert not led.release("r1")
    led.release_all()
    assert not rb.PEER_KV_STAGING and not rb.PEER_REQ_MAP and led.requests() == []


def test_readiness_cache_rate_limits_lookups():
    now = [0.0]
    looks = []
    present = set()

    def exists(path):
        looks.append(path)
        return path in present

    rc = ReadinessCache(0.5, exists=exists, clock=lambda: now[0])
    assert not rc.is_ready("c", "/m/c")
    assert not rc.is_ready("c", "/m/c") and len(looks) == 1          # inside the interval: no look
    present.add("/m/c")
    now[0] = 0.49
    assert not rc.is_ready("c", "/m/c") and len(looks) == 1
    now[0] = 0.5
    assert rc.is_ready("c", "/m/c") and len(looks) == 2
    present.clear()
    assert rc.is_ready("c", "/m/c") and len(looks) == 2              # once ready, stays ready
    assert not rc.is_ready("d", "/m/d")
    rc.look_again_now()
    assert not rc.is_ready("d", "/m/d") and len(looks) == 4


def test_decode_slot_pool_reuses_slots():
    pool = DecodeSlotPool(2)
    assert pool.take("r1", 5) == 0 and pool.take("r2", 6) == 1
    with pytest.raises(RuntimeError, match="decode ring slots"):
        pool.take("r3", 7)
    assert pool.give_back("r1") == 5 and pool.give_back("r1") is None
    assert pool.take("r3", 7) == 0 and pool.holders() == ["r2", "r3"]


def test_layer_feed_stays_within_the_window_and_checks_the_length():
    layers = [f"model.layers.{i}.attn" for i in range(6)]
    staged = []
    lock = threading.Lock()

    def stage(ln):
        with lock:
            staged.append(ln)
        return {"a": 3, "b": 5}, None

    feed = LayerFeed("r", layers, ["a", "b"], expected_total=8, window=2)
    feed.start(stage)
    for i, ln in enumerate(layers):
        assert feed.wait(ln) is None
        time.sleep(0.01)
        with lock:
            assert len(staged) <= i + 1 + 2                 # never more than the window ahead
        feed.consumed(i)
    feed.join()
    assert staged == layers and feed.error is None

    bad = LayerFeed("r2", layers[:2], ["a", "b"], expected_total=16, window=2)  # both without consumption
    bad.start(stage)
    bad.join()
    with pytest.raises(RuntimeError, match="prefill stream for req r2"):
        bad.wait(layers[0])


def test_layer_feed_stop_ends_a_waiting_thread():
    feed = LayerFeed("r", [f"l.layers.{i}.x" for i in range(8)], ["a"], expected_total=1, window=1)
    feed.start(lambda ln: ({"a": 1}, None))
    feed.wait("l.layers.0.x")
    feed.stop()                         # blocked on the window: returns without staging the rest
    assert feed.error is None


def test_chunk_ledger_random_holds_and_releases_follow_a_count_model():
    """500 random holds and releases over 12 requests sharing 6 chunks: a
    chunk stays staged exactly while some request that holds it is in flight,
    the backend's request map holds exactly the live requests, and
    ``release_all`` leaves nothing staged."""
    import random

    rnd = random.Random(5)
    led = ChunkLedger()
    chunks = [f"c{i}" for i in range(6)]
    layer = "model.layers.0.attn"
    live: dict = {}  # request -> (first block id, chunks)
    for step in range(500):
        rid = f"r{rnd.randrange(12)}"
        if rid in live and rnd.random() < 0.6:
            assert led.release(rid)
            del live[rid]
        elif rid not in live:
            held = rnd.sample(chunks, rnd.randint(1, 4))
            for ck in held:  # the connector stages a chunk before a request holds it
                if (ck, layer) not in rb.PEER_KV_STAGING:
                    _stage(ck, layer)
            fb = 1000 + step
            led.hold(rid, fb, held)
            live[rid] = (fb, held)
        want = {}
        for _, held in live.values():
            for ck in held:
                want[ck] = want.get(ck, 0) + 1
        assert led.holder_counts() == want
        staged = {ck for ck, _ in rb.PEER_KV_STAGING}
        # every chunk here is held as soon as it is staged, so staged == held
        assert set(want) <= staged, "a chunk was dropped while a request still held it"
        assert staged <= set(want), "a chunk stayed staged after its last holder left"
        assert sorted(led.requests()) == sorted(live)
        assert {fb: list(h) for fb, h in live.values()} == dict(rb.PEER_REQ_MAP)
    led.release_all()
    assert not rb.PEER_KV_STAGING and not rb.PEER_REQ_MAP and led.holder_counts() == {}


def test_decode_slot_pool_refuses_a_second_slot_for_one_request():
    pool = DecodeSlotPool(3)
    assert pool.take("r1", 5) == 0
    with pytest.raises(RuntimeError, match="already holds decode ring slot 0"):
        pool.take("r1", 6)
    assert pool.holders() == ["r1"] and list(pool.free) == [1, 2]
