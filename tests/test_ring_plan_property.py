"""The host plan of a layer call, executed, equals the reference forward().

Random continuous batches (ragged query and key lengths, single-token rows,
0-3 staged peer chunks per request, sometimes 9 so the request is
concatenated, enough chunks in a step to need several launch groups, and the
single-instance split mode) are planned by ``ring_plan.plan_layer``.  The
plan is then executed by a numpy model of what the kernels compute from it:
each work item's rows attend the union of its segments' visible keys (paged
segments through the block table, extra sources by index, a causal segment
showing keys ``< causal_off + row + 1``, a non-causal one all of its keys),
and each decode sequence its extra-source peer keys plus its paged local
keys.  The result must equal the oracle's restatement of the reference
``HcpRingAttentionImpl.forward`` (``ring_backend.py:597-834``), which splits
and merges per request instead.  No GPU: the kernels' own parity with the
oracle is the GPU suite's job; this pins the planner on arbitrary batches."""

import numpy as np
import pytest
import torch

from hcp_vllm_plugin_b200 import _capi as C
from hcp_vllm_plugin_b200.ring_plan import CONCAT, misaligned_paged_starts, plan_layer
from oracle import ring_oracle as ro

H, HKV, D, BS = 4, 2, 8, 16


def _batch(rng, split_tokens=0):
    n_req = int(rng.integers(1, 7))
    qsl, lens, peers = [0], [], {}
    for r in range(n_req):
        kind = rng.random()
        n_chunks = 0 if split_tokens else int(rng.choice([0, 0, 1, 2, 3, 9], p=[.3, .1, .25, .15, .15, .05]))
        chunk_lens = [BS * int(rng.integers(1, 4)) for _ in range(n_chunks)]
        peer = sum(chunk_lens)
        local = int(rng.integers(1, 70))
        tk = peer + local
        tq = 1 if kind < 0.3 else int(rng.integers(1, min(tk, 60) + 1))
        qsl.append(qsl[-1] + tq)
        lens.append(tk)
        if n_chunks:
            peers[r] = [(torch.from_numpy(rng.standard_normal((c, HKV, D)).astype(np.float32)),
                         torch.from_numpy(rng.standard_normal((c, HKV, D)).astype(np.float32)))
                        for c in chunk_lens]
    blocks = [(tk + BS - 1) // BS for tk in lens]
    nb = sum(blocks) + 3
    perm = rng.permutation(nb)
    bt = np.zeros((n_req, max(blocks)), np.int64)
    o = 0
    for r, b in enumerate(blocks):
        bt[r, :b] = perm[o:o + b]
        o += b
    batch = ro.RingBatch(
        query=rng.standard_normal((qsl[-1], H, D)).astype(np.float32),
        cache=rng.standard_normal((nb, HKV, BS, 2 * D)).astype(np.float32),
        block_table=bt, query_start_loc=np.array(qsl), seq_lens=np.array(lens), scale=D ** -0.5,
        staged={r: (np.concatenate([k.numpy() for k, _ in ch]), np.concatenate([v.numpy() for _, v in ch]))
                for r, ch in peers.items()},
        split_tokens=split_tokens)
    return batch, peers


def _execute(plan, batch, peers):
    """What the kernels compute from the plan (float32, one softmax per row)."""
    out = np.zeros_like(batch.query)
    covered = np.zeros(batch.query.shape[0], bool)

    def paged(req, start, n):
        k, v = ro.paged_gather(batch.cache, batch.block_table[req], start + n)
        return k[start:start + n], v[start:start + n]

    def attend(row, parts):
        k = np.concatenate([p[0] for p in parts])
        v = np.concatenate([p[1] for p in parts])
        o, _ = ro.attn_with_lse(batch.query[row:row + 1], k, v, batch.scale, None)
        assert not covered[row], f"row {row} computed twice"
        covered[row] = True
        out[row] = o[0]

    for g in plan.groups:
        srcs = []
        for r, c in g.sources:
            ch = peers[r] if c == CONCAT else [peers[r][c]]
            srcs.append((np.concatenate([k.numpy() for k, _ in ch]), np.concatenate([v.numpy() for _, v in ch])))
        for x in g.work:
            qs, ql, preq = int(x[0]), int(x[1]), int(x[2])
            segs = [tuple(int(t) for t in s) for s in g.seg_list[x[5]:x[5] + x[6]]] if x[4] == C.HCP_SRC_LIST \
                else [tuple(int(t) for t in x[4:8]), tuple(int(t) for t in x[8:12])]
            keys = []
            for src, start, n, coff in segs:
                if src == C.HCP_SRC_NONE or n <= 0:
                    continue
                if src == C.HCP_SRC_PAGED:
                    k, v = paged(preq, start, n)
                else:
                    assert src >= C.HCP_SRC_EXT0, f"source {src} is not served by the backend's launch"
                    k, v = srcs[src - C.HCP_SRC_EXT0]
                    assert start + n <= k.shape[0]
                    k, v = k[start:start + n], v[start:start + n]
                keys.append((k, v, coff))
            for i in range(ql):
                parts = [(k[:n], v[:n]) for k, v, coff in keys
                         for n in [k.shape[0] if coff < 0 else min(k.shape[0], coff + i + 1)] if n > 0]
                attend(qs + i, parts)
        for j, d in enumerate(g.decode):
            qr, ps, pl, preq, ls, ll = (int(t) for t in d)
            parts = []
            if pl > 0:
                k, v = srcs[int(g.peer_src[j])]
                parts.append((k[ps:ps + pl], v[ps:ps + pl]))
            if ll > 0:
                parts.append(paged(preq, ls, ll))
            attend(qr, parts)
    return out, covered


@pytest.mark.parametrize("split_tokens", [0, 32])
def test_executed_plan_equals_the_reference_forward(split_tokens):
    rng = np.random.default_rng(1234 + split_tokens)
    launches = 0
    for _ in range(60):
        batch, peers = _batch(rng, split_tokens)
        plan = plan_layer(batch.query_start_loc, batch.seq_lens, BS, peers, split_tokens=split_tokens)
        assert not misaligned_paged_starts(plan, BS)
        assert all(len(g.sources) <= C.HCP_MAX_EXT_SOURCES for g in plan.groups)
        got, covered = _execute(plan, batch, peers)
        assert covered.all(), "rows the plan leaves out"
        want = ro.ring_forward(batch, round_to_bf16=False)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=2e-5)
        launches += len(plan.groups)
    if not split_tokens:
        assert launches > 60  # some steps staged more chunks than one launch takes
