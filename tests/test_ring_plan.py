"""Host plan of a layer call (no GPU, no vLLM): the rows, segments and
offsets the backend hands to the kernels follow the reference forward()."""

import os

import numpy as np
import torch

from hcp_vllm_plugin_b200 import _capi as C
from hcp_vllm_plugin_b200.ring_plan import misaligned_paged_starts, plan_layer

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _peers_from_fixture(z):
    peers = {}
    for r in range(len(z["seq_lens"])):
        n = int(z["peer_counts"][r])
        if n:
            peers[r] = [(torch.from_numpy(z[f"peer{r}_{c}_k"].view(np.int16)),
                         torch.from_numpy(z[f"peer{r}_{c}_v"].view(np.int16))) for c in range(n)]
    return peers


def test_plan_matches_reference_split():
    z = np.load(os.path.join(GOLD, "forward_case.npz"))
    peers = _peers_from_fixture(z)
    plan = plan_layer(z["query_start_loc"], z["seq_lens"], 16, peers)
    assert len(plan.groups) == 1 and not plan.concat_requests
    g = plan.groups[0]
    # every staged chunk is its own extra source, in request order
    assert g.sources == [(0, 0), (1, 0), (2, 0), (4, 0), (4, 1), (4, 2)]
    E = C.HCP_SRC_EXT0
    # request 2 has a single query token -> decode kernel, peer keys in source 2
    assert plan.decode.shape[0] == 1
    qr, pstart, plen, preq, lstart, llen = plan.decode[0]
    assert (qr, pstart, plen, preq, lstart, llen) == (104, 0, 48, 2, 48, 97 - 48)
    assert list(g.peer_src) == [2]
    w = {tuple(x[:2]): x for x in plan.work}
    # request 0: tq=40, tk=72, staged 32 -> peer non-causal + local [32,72) causal offset 0
    x = w[(0, 40)]
    assert list(x[4:8]) == [E + 0, 0, 32, -1]
    assert list(x[8:12]) == [C.HCP_SRC_PAGED, 32, 40, 0]
    # request 1: tq=64, tk=64, staged 32 -> n_a = 32 rows fully causal over all keys
    x = w[(40, 32)]
    assert list(x[4:8]) == [C.HCP_SRC_PAGED, 0, 64, 0]
    x = w[(72, 32)]
    assert list(x[4:8]) == [E + 1, 0, 32, -1]
    assert list(x[8:12]) == [C.HCP_SRC_PAGED, 32, 32, 0]
    # request 3: no peer -> causal over its own keys at offset qpos0 = 0
    x = w[(105, 24)]
    assert list(x[4:8]) == [C.HCP_SRC_PAGED, 0, 24, 0]
    # request 4: three ordered chunks, each read where it is staged, then the
    # local keys: a segment list of four
    x = w[(129, 30)]
    assert list(x[4:8]) == [C.HCP_SRC_LIST, 0, 4, 0]
    assert [list(r) for r in g.seg_list] == [[E + 3, 0, 32, -1], [E + 4, 0, 16, -1], [E + 5, 0, 16, -1],
                                             [C.HCP_SRC_PAGED, 64, 30, 0]]
    assert not misaligned_paged_starts(plan, 16)
    assert plan.stats["decode_rows"] == 1 and plan.stats["peer_requests"] == 4


def test_plan_groups_sources_and_long_chunk_lists():
    """More than 8 staged chunks in a layer: requests are split into launch
    groups of at most 8 sources; a decode row with several chunks goes to
    the forward kernel; a request with more chunks than a work item holds is
    concatenated (the only copy left)."""
    k = torch.zeros(32, 2, 64)
    peers = {r: [(k, k), (k, k)] for r in range(6)}        # 12 chunks
    peers[6] = [(k, k)] * 9                                  # 9 chunks: concatenated
    qsl = [0, 40, 80, 81, 121, 161, 201, 241]
    lens = [104, 104, 65, 104, 104, 104, 104]
    plan = plan_layer(qsl, lens, 16, peers)
    assert all(len(g.sources) <= C.HCP_MAX_EXT_SOURCES for g in plan.groups)
    assert len(plan.groups) == 2 and plan.concat_requests == [6]
    assert sum(len(g.sources) for g in plan.groups) == 13
    # request 2 (one query, two chunks) is a one-row forward item, not a decode sequence
    assert plan.decode.shape[0] == 0
    assert any(int(x[0]) == 80 and int(x[1]) == 1 for x in plan.work)
    for g in plan.groups:
        for x in g.work:
            if x[4] == C.HCP_SRC_LIST:
                assert x[6] <= C.HCP_MAX_ITEM_SEGMENTS
                for sg in g.seg_list[x[5]:x[5] + x[6]]:
                    if sg[0] >= C.HCP_SRC_EXT0:
                        assert sg[0] - C.HCP_SRC_EXT0 < len(g.sources)


def test_plan_split_tokens_and_misalignment():
    # HCP_RING_SPLIT_TOKENS mode: the first `split` keys of the request's own
    # cache are the peer segment (non-causal), the rest causal at
    # qpos0 + n_a - peer_end (ring_backend.py:776-832)
    plan = plan_layer([0, 10], [50], 16, {}, split_tokens=32)
    assert plan.work.shape[0] == 1
    assert list(plan.work[0][:4]) == [0, 10, 0, 0]
    assert list(plan.work[0][4:8]) == [C.HCP_SRC_PAGED, 0, 32, -1]
    assert list(plan.work[0][8:12]) == [C.HCP_SRC_PAGED, 32, 18, 40 - 32]
    # queries inside the split region (n_a = 32 - 20 = 12) stay fully causal
    plan = plan_layer([0, 30], [50], 16, {}, split_tokens=32)
    w = {tuple(x[:2]): x for x in plan.work}
    assert list(w[(0, 12)][4:8]) == [C.HCP_SRC_PAGED, 0, 50, 20]
    assert list(w[(12, 18)][4:8]) == [C.HCP_SRC_PAGED, 0, 32, -1]
    assert list(w[(12, 18)][8:12]) == [C.HCP_SRC_PAGED, 32, 18, 20 + 12 - 32]
    # a decode row keeps the single paged segment (same keys)
    plan = plan_layer([0, 1], [50], 16, {}, split_tokens=32)
    assert plan.work.shape[0] == 0 and list(plan.decode[0]) == [0, 0, 0, 0, 0, 50]
    # a split that is not block aligned cannot start a paged segment
    assert misaligned_paged_starts(plan_layer([0, 10], [50], 16, {}, split_tokens=20), 16)
    # a staged prefix that is not block aligned cannot be read from the cache
    k = torch.zeros(20, 2, 64)
    plan = plan_layer([0, 10], [50], 16, {0: [(k, k)]})
    assert misaligned_paged_starts(plan, 16)


def test_plan_without_decode_kernel_puts_decode_rows_in_prefill_items():
    """With a sliding window the backend plans without the split-KV decode
    kernel: the single-token request becomes a prefill item whose local
    segment is causal at offset qpos0 - peer_end (the window applies to it in
    the kernel), its staged chunk stays non-causal."""
    z = np.load(os.path.join(GOLD, "forward_case.npz"))
    peers = _peers_from_fixture(z)
    plan = plan_layer(z["query_start_loc"], z["seq_lens"], 16, peers, decode_kernel=False)
    assert plan.decode.shape[0] == 0 and plan.stats["decode_rows"] == 0
    w = {tuple(x[:2]): x for x in plan.work}
    x = w[(104, 1)]
    E = C.HCP_SRC_EXT0
    assert list(x[4:8]) == [E + 2, 0, 48, -1]
    assert list(x[8:12]) == [C.HCP_SRC_PAGED, 48, 97 - 48, 96 - 48]
