"""Golden decisions of the reference ring connector's scheduler side.

Runs the reference ``HcpRingKvConnector`` (``hcp_vllm_plugin/ring_connector.py``)
in the SCHEDULER role with a local store path (no peer url, readiness =
``_READY`` marker files) over a fixed list of scenarios - readiness gating,
global and per-request prefix chunks, singular/plural/short url lists,
``prefix_len`` opt-out, ``ring_order`` derivation, load and store metadata -
and writes every answer to ``ring_connector_case.json`` next to this script.
The same scenarios replayed on this package's connector must give the same
answers (``tests/test_ring_connector.py``).

Usage (in a container holding the reference sources and vLLM)::

    HCP_REFERENCE_ROOT=/path/to/hcp-vllm-plugin python tests/golden/make_ring_connector_golden.py
"""

from __future__ import annotations

import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
REF_ROOT = os.environ.get("HCP_REFERENCE_ROOT", "")  # the reference checkout (generation only)
OUT = os.path.join(HERE, "ring_connector_case.json")

BS = 16

# (name, extra config, list of matched-token queries, meta build)
SCENARIOS = [
    dict(name="global_prefix", extra=dict(ring_role="ring", ring_chunk_id="c2", ring_prefix_chunk_ids="c0,c1",
                                          ring_prefix_len=2050),
         markers_before=[], markers_after=["c0", "c1"],
         queries=[("r0", {}, 0), ("r0", {}, 1024), ("r1", {"prefix_len": 0}, 0),
                  ("r2", {"chunk_ids": "c1", "prefix_len": 100}, 0), ("r3", {"chunk_id": "c0", "prefix_len": 40}, 16)]),
    dict(name="ring_order", extra=dict(ring_role="ring", ring_order="c0@http://a:1/,c1@http://b:2,c2@http://c:3",
                                       ring_my_chunk="c2", ring_prefix_len=4096),
         markers_before=["c0"], markers_after=["c0", "c1"],
         queries=[("r0", {}, 0), ("r1", {"peer_urls": ["http://x"], "chunk_ids": ["c0", "c1"]}, 0)]),
    dict(name="producer_only", extra=dict(ring_role="producer", ring_chunk_id="c0"),
         markers_before=[], markers_after=[], queries=[("r0", {}, 0)]),
    dict(name="consumer", extra=dict(ring_role="consumer", ring_prefix_chunk_ids="c0", ring_prefix_len=512),
         markers_before=[], markers_after=["c0"], queries=[("r0", {}, 0), ("r0", {}, 512)]),
]

# new requests for build_connector_meta: (req_id, prompt_len, block_ids, hcp_ring params, needs_load)
META_REQS = [
    ("r0", 2050 + 300, list(range(40, 40 + 150)), {}, True),
    ("r2", 130, [7, 3, 9, 11, 2, 5, 6, 8, 12], {"chunk_ids": "c1", "prefix_len": 100, "chunk_id": "own7"}, True),
    ("r9", 70, [21, 22, 23, 24, 25], {"prefix_len": 0}, False),
]

URL_CASES = [
    ({"chunk_ids": "a,b,c", "peer_urls": "u1"}, [], []),
    ({"chunk_ids": ["a", "b"], "peer_urls": ["u1/", "u2"]}, [], []),
    ({"chunk_id": "a", "peer_url": "u/"}, ["g"], ["gu"]),
    ({}, ["g1", "g2"], ["gu1"]),
    ({}, ["g1", "g2"], []),
    ({"peer_urls": "p"}, ["g1", "g2", "g3"], ["gu"]),
]


def fake_request(req_id, prompt_len, hcp):
    import types
    return types.SimpleNamespace(request_id=req_id, prompt_token_ids=list(range(prompt_len)),
                                 kv_transfer_params={"hcp_ring": hcp} if hcp else None)


def run(connector_cls, role_scheduler, chunks_and_urls, fake_config) -> dict:
    import types
    out = {"scenarios": {}, "urls": []}
    for sc in SCENARIOS:
        with tempfile.TemporaryDirectory() as shared:
            extra = dict(sc["extra"], ring_shared_path=shared, ring_run_id="run",
                         ring_ready_poll_interval_s=0)
            conn = connector_cls(fake_config(extra), role_scheduler, None)

            def mark(chunks):
                for ck in chunks:
                    os.makedirs(os.path.join(shared, "run", ck), exist_ok=True)
                    with open(os.path.join(shared, "run", ck, "_READY"), "w") as f:
                        f.write("{}")

            res = {"before": [], "after": []}
            mark(sc["markers_before"])
            for rid, hcp, computed in sc["queries"]:
                res["before"].append(list(conn.get_num_new_matched_tokens(fake_request(rid, 3000, hcp), computed)))
            mark(sc["markers_after"])
            for rid, hcp, computed in sc["queries"]:
                res["after"].append(list(conn.get_num_new_matched_tokens(fake_request(rid, 3000, hcp), computed)))
            new_reqs = []
            for rid, plen, blocks, hcp, need in META_REQS:
                if need:
                    conn.update_state_after_alloc(fake_request(rid, plen, hcp), None, 1)
                sp = types.SimpleNamespace(extra_args={"kv_transfer_params": {"hcp_ring": hcp}} if hcp else {})
                new_reqs.append(types.SimpleNamespace(req_id=rid, prompt_token_ids=list(range(plen)),
                                                      block_ids=[blocks], sampling_params=sp))
            meta = conn.build_connector_meta(types.SimpleNamespace(scheduled_new_reqs=new_reqs,
                                                                   finished_req_ids={"z1", "a0"}))
            res["finished"] = list(meta.finished_req_ids)
            res["meta"] = [dict(is_store=m.is_store, chunk_key=m.chunk_key, req_id=m.req_id,
                                first_block_id=int(m.first_block_id), chunk_keys=list(m.chunk_keys),
                                peer_urls=list(m.peer_urls), prefix_len=int(m.prefix_len),
                                slot_mapping=None if m.slot_mapping is None else [int(x) for x in m.slot_mapping])
                           for m in meta.requests]
            out["scenarios"][sc["name"]] = res
    for rp, gids, gurls in URL_CASES:
        out["urls"].append([list(x) for x in chunks_and_urls(rp, gids, gurls)])
    return out


def main() -> None:
    if not REF_ROOT:
        raise SystemExit("set HCP_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, REF_ROOT)
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole
    from hcp_vllm_plugin import ring_connector as rc  # reference code
    from tests import vllm_fakes as fk

    def fake_config(extra):
        return fk.vllm_config(extra, block_size=BS, num_layers=2, num_kv_heads=4, head_dim=128, num_heads=28)

    out = run(rc.HcpRingKvConnector, KVConnectorRole.SCHEDULER, rc._chunks_and_urls, fake_config)
    with open(OUT, "w") as f:
        json.dump(out, f)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
