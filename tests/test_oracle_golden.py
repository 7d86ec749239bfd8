"""Pin the CPU oracle to golden vectors produced by the reference's own code.

The fixtures under ``tests/golden/`` were written by ``make_golden.py``, which
ran the reference plugin's ``_attn_with_lse``, ``_lse_merge`` and
``HcpRingAttentionImpl.forward`` (torch fp32 path) on CPU.
"""

import os

import numpy as np
import pytest

from oracle import ring_oracle as ro

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _f32(u16, is_bf16):
    if is_bf16:
        return ro.bf16_bits_to_f32(u16)
    return np.asarray(u16, dtype=np.uint16).view(np.float16).astype(np.float32)


def _kernel_cases():
    z = np.load(os.path.join(GOLD, "kernel_cases.npz"))
    return z, int(z["count"][0])


@pytest.mark.parametrize("idx", range(11))
@pytest.mark.parametrize("causal", [True, False])
def test_attn_with_lse_matches_reference(idx, causal):
    z, count = _kernel_cases()
    assert count == 11
    key = f"c{idx:02d}"
    h, hkv, d, tq, tk, off, is_bf16 = (int(x) for x in z[f"{key}_meta"])
    scale = float(z[f"{key}_scale"][0])
    rows = z[f"{key}_rows"]
    q = _f32(z[f"{key}_q"], is_bf16)
    k = _f32(z[f"{key}_k"], is_bf16)
    v = _f32(z[f"{key}_v"], is_bf16)
    tag = "causal" if causal else "noncausal"
    want_o = z[f"{key}_{tag}_out"]
    want_lse = z[f"{key}_{tag}_lse"]
    # Each stored row is computed on its own, at its own causal position.
    for i, r in enumerate(rows):
        o, lse = ro.attn_with_lse(q[i:i + 1], k, v, scale, (off + int(r)) if causal else None)
        np.testing.assert_allclose(o[0], want_o[i], atol=2e-6, rtol=1e-5)
        np.testing.assert_allclose(lse[:, 0], want_lse[:, i], atol=2e-6, rtol=1e-6)


def test_lse_merge_and_two_chunk_identity():
    z = np.load(os.path.join(GOLD, "merge_cases.npz"))
    m = ro.lse_merge(z["o_b"], z["lse_b"], z["o_a"], z["lse_a"])
    np.testing.assert_allclose(m, z["merged"], atol=1e-6, rtol=1e-6)
    # vLLM merge_attn_states(prefix=peer, suffix=local) equals the plain merge
    m2, _ = ro.merge_attn_states(z["o_a"], z["lse_a"], z["o_b"], z["lse_b"])
    np.testing.assert_allclose(m2, z["merged"], atol=1e-6, rtol=1e-6)

    scale = float(z["scale"][0])
    split = int(z["split"][0])
    q3 = _f32(z["q3"], False)
    k3 = _f32(z["k3"], False)
    v3 = _f32(z["v3"], False)
    tk, tq = k3.shape[0], q3.shape[0]
    o_full, lse_full = ro.attn_with_lse(q3, k3, v3, scale, tk - tq)
    np.testing.assert_allclose(o_full, z["o_full"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(lse_full, z["lse_full"], atol=2e-6, rtol=1e-6)
    o_loc, lse_loc = ro.attn_with_lse(q3, k3[split:], v3[split:], scale, tk - tq - split)
    o_peer, lse_peer = ro.attn_with_lse(q3, k3[:split], v3[:split], scale, None)
    merged, lse_m = ro.merge_pair(o_loc, lse_loc, o_peer, lse_peer)
    np.testing.assert_allclose(merged, z["merged3"], atol=2e-6, rtol=1e-5)
    # the merged LSE of the two chunks is the full LSE (ring_decode.py:59-60)
    np.testing.assert_allclose(lse_m, lse_full, atol=1e-5)
    # validate_ring_triton_kernel.py:80-94 tolerance
    assert np.abs(merged - o_full).max() <= 3e-3


def _forward_batch():
    z = np.load(os.path.join(GOLD, "forward_case.npz"))
    h, hkv, d, bs, nreq, ntok = (int(x) for x in z["meta"])
    staged = {}
    for r in range(nreq):
        n = int(z["peer_counts"][r])
        if n:
            ks = [ro.bf16_bits_to_f32(z[f"peer{r}_{c}_k"]) for c in range(n)]
            vs = [ro.bf16_bits_to_f32(z[f"peer{r}_{c}_v"]) for c in range(n)]
            staged[r] = (np.concatenate(ks, 0), np.concatenate(vs, 0))
    batch = ro.RingBatch(
        query=ro.bf16_bits_to_f32(z["query"]),
        cache=ro.bf16_bits_to_f32(z["cache"]),
        block_table=z["block_table"],
        query_start_loc=z["query_start_loc"],
        seq_lens=z["seq_lens"],
        scale=float(z["scale"][0]),
        staged=staged,
    )
    return z, batch


def test_ring_forward_matches_reference_forward():
    z, batch = _forward_batch()
    want = ro.bf16_bits_to_f32(z["output"])
    got = ro.ring_forward(batch, round_to_bf16=True)
    diff = np.abs(got - want)
    # Both sides round an fp32 result to bf16; a value that lands within a
    # few fp32 ulps of a bf16 rounding boundary may round the other way,
    # which moves it by one bf16 ulp (2^-8 relative at most).
    ulp = np.abs(want) * 2.0 ** -7 + 1e-30
    assert (diff <= np.maximum(1e-6, ulp)).all()
    assert (diff > 1e-6).mean() < 1e-3
    # the split shapes the reference's forward produced
    plans = [ro.plan_request(int(z["query_start_loc"][r]),
                             int(z["query_start_loc"][r + 1] - z["query_start_loc"][r]),
                             int(z["seq_lens"][r]),
                             None if r not in batch.staged else batch.staged[r][0].shape[0], 0)
             for r in range(len(z["seq_lens"]))]
    assert [p.n_a for p in plans] == [0, 32, 0, 0, 0]
    assert [p.peer_source for p in plans] == ["staged", "staged", "staged", "none", "staged"]


def test_kv_cache_update_roundtrip():
    rng = np.random.default_rng(0)
    cache = np.zeros((8, 2, 16, 2 * 32), np.float32)
    key = rng.standard_normal((20, 2, 32)).astype(np.float32)
    val = rng.standard_normal((20, 2, 32)).astype(np.float32)
    slots = rng.permutation(8 * 16)[:20]
    slots[3] = -1  # padding token
    ro.kv_cache_update(cache, key, val, slots)
    for i, s in enumerate(slots):
        if s < 0:
            continue
        b, o = divmod(int(s), 16)
        np.testing.assert_array_equal(cache[b, :, o, :32], key[i])
        np.testing.assert_array_equal(cache[b, :, o, 32:], val[i])


def test_visible_pairs_and_flops():
    for tq, tk, off in [(1, 1, 0), (37, 512, 475), (128, 128, 0), (64, 300, 10), (5, 3, 0)]:
        brute = sum(min(tk, off + i + 1) for i in range(tq))
        assert ro.visible_pairs(tq, tk, off) == brute
    assert ro.visible_pairs(7, 9, None) == 63
    # cfg0 work: 524 800 causal + 1 048 576 peer pairs -> 2.256e10 FLOP
    pairs = ro.visible_pairs(1024, 1024, 0) + ro.visible_pairs(1024, 1024, None)
    assert pairs == 1573376
    assert abs(ro.attention_flops(pairs, 28, 128) - 2.2556e10) / 2.2556e10 < 1e-3


def test_growth_assignee():
    assert [ro.growth_assignee(p, 3) for p in range(6)] == [0, 1, 2, 0, 1, 2]
    assert ro.growth_assignee(17, 4, "owner") == 3


def test_bf16_rounding():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.4e38, 1e-40], np.float32)
    r = ro.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == np.float32(1.015625)
    assert r[3] == -2.5


def test_window_attention_matches_reference():
    """``_attn_with_lse`` with a sliding window (``ring_backend.py:391-398``)."""
    z = np.load(os.path.join(GOLD, "window_case.npz"))
    for i in range(3):
        tq, tk, off, w = (int(x) for x in z[f"w{i}_meta"])
        q, k, v = (ro.bf16_bits_to_f32(z[f"w{i}_{n}"]) for n in "qkv")
        rows = z[f"w{i}_rows"]
        o, lse = ro.attn_with_lse(q, k, v, 128 ** -0.5, off, w)
        np.testing.assert_allclose(o[rows], z[f"w{i}_o"], atol=2e-6, rtol=1e-5)
        np.testing.assert_allclose(lse[:, rows], z[f"w{i}_lse"], atol=2e-6, rtol=1e-6)
        assert w < tk  # the window cuts keys in every case


def test_ring_forward_with_window_matches_reference_forward():
    """The reference forward built with ``sliding_window=20``: the window on
    the causal passes only, the staged peer chunks fully visible."""
    z, batch = _forward_batch()
    zw = np.load(os.path.join(GOLD, "window_case.npz"))
    batch.window = int(zw["window"][0])
    want = ro.bf16_bits_to_f32(zw["output"])
    got = ro.ring_forward(batch, round_to_bf16=True)
    diff = np.abs(got - want)
    ulp = np.abs(want) * 2.0 ** -7 + 1e-30
    assert (diff <= np.maximum(1e-6, ulp)).all()
    assert (diff > 1e-6).mean() < 1e-3
    # the window changed the result (it is not a no-op on this batch)
    assert np.abs(want - ro.bf16_bits_to_f32(z["output"])).max() > 0.05
