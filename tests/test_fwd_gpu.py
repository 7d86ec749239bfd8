"""GPU parity of the fused ring-attention forward against the CPU oracle.

All calls go through the C ABI (``libhcp_ring.so``).  The bar is
``tests/parity.py``: LSE within 1e-3; every output element equal to, or one
output-dtype step from, the reference's own output (its fp32 path rounded to
the output dtype), and within 2e-3 of the fp32 oracle or - where the
reference's own output misses 2e-3 - no further off than that output.
Includes BASELINE configs[0] exactly and configs[3] at N=1 (one 131072-token
causal launch, sampled rows).
"""

import os

import numpy as np
import pytest
import torch

import parity as P
from oracle import ring_oracle as ro

pytestmark = pytest.mark.gpu

H28, HKV4, D128 = P.H28, P.HKV4, P.D128
_f = P.f32


@pytest.fixture(scope="module")
def dev():
    from hcp_vllm_plugin_b200 import _capi
    assert torch.cuda.is_available()
    _capi.load()
    _capi.reset_device_status()
    yield torch.device("cuda:0")
    assert _capi.device_status() == 0


@pytest.mark.parametrize("geom", P.PROBE_GEOMS)
@pytest.mark.parametrize("case", P.PROBE)
@pytest.mark.parametrize("causal", [True, False])
def test_ring_attn_with_lse_probe(dev, geom, case, causal):
    from hcp_vllm_plugin_b200.ops import ring_attn_with_lse
    dt = geom[3]
    q, k, v = P.probe_inputs(geom, case)
    scale = geom[2] ** -0.5
    off = case[2] if causal else None
    o, lse = ring_attn_with_lse(q.to(dev), k.to(dev), v.to(dev), scale, off)
    torch.cuda.synchronize()
    want_o, want_lse = ro.attn_with_lse(_f(q), _f(k), _f(v), scale, off)
    name = P.probe_name(geom, case, causal)
    st = P.check_out(_f(o), want_o, name, dt, case=name)
    P.check_lse(_f(lse), want_lse, name)
    print(st.line())


def test_golden_kernel_cases_through_cuda(dev):
    """The reference's own outputs (tests/golden) reproduced by the CUDA path."""
    from hcp_vllm_plugin_b200.ops import ring_attn_with_lse
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "kernel_cases.npz"))
    for idx in range(int(z["count"][0])):
        key = f"c{idx:02d}"
        h, hkv, d, tq, tk, off, is_bf16 = (int(x) for x in z[f"{key}_meta"])
        dt = torch.bfloat16 if is_bf16 else torch.float16

        def t16(a):
            a = torch.from_numpy(np.asarray(a).view(np.int16).copy())
            return a.view(dt)
        rows = z[f"{key}_rows"]
        q = t16(z[f"{key}_q"]).to(dev)
        k = t16(z[f"{key}_k"]).to(dev)
        v = t16(z[f"{key}_v"]).to(dev)
        scale = float(z[f"{key}_scale"][0])
        for causal in (True, False):
            tag = "causal" if causal else "noncausal"
            # stored rows are a subset: run each row at its own causal offset
            for i, r in enumerate(rows):
                o, lse = ring_attn_with_lse(q[i:i + 1], k, v, scale, (off + int(r)) if causal else None)
                P.check_out(_f(o)[0], z[f"{key}_{tag}_out"][i], f"golden {key} row {r} {tag}", dt)
                P.check_lse(_f(lse)[:, 0], z[f"{key}_{tag}_lse"][:, i], f"golden {key}")
    torch.cuda.synchronize()


def _fused_run(dev, q, kp, vp, kl, vl, tpeer, tloc, off):
    from hcp_vllm_plugin_b200 import _capi as C, ops
    tq = q.shape[0]
    out = torch.empty(tq, H28, D128, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(H28, tq, dtype=torch.float32, device=dev)
    segs = []
    if tpeer:
        segs.append((C.HCP_SRC_A, 0, tpeer, -1))
    if tloc:
        segs.append((C.HCP_SRC_B, 0, tloc, off))
    segs += [None] * (2 - len(segs))
    work = ops.make_work([(0, tq, 0, 0, segs[0], segs[1])])
    ops.ring_attn_fwd(q.to(dev), work, scale=D128 ** -0.5, num_kv_heads=HKV4, out=out, lse=lse,
                      k_a=kp.to(dev), v_a=vp.to(dev), k_b=kl.to(dev), v_b=vl.to(dev))
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("c", P.FUSED)
def test_fused_peer_plus_local_equals_merge(dev, c):
    """One launch over [peer (non-causal), local (causal)] equals the reference's
    local pass + peer pass + _lse_merge (ring_backend.py:819-832)."""
    tq, tpeer, tloc, off = c
    q, kp, vp, kl, vl = P.fused_inputs(c)
    out, lse = _fused_run(dev, q, kp, vp, kl, vl, tpeer, tloc, off)
    want, want_lse = P.fused_oracle(c, q, kp, vp, kl, vl)
    st = P.check_out(_f(out), want, P.fused_name(c), case=P.fused_name(c))
    if tpeer >= 512:
        P.check_flat(_f(out), want, "fused peer+local (deployment shape)")
    P.check_lse(_f(lse), want_lse, "fused peer+local")
    print(st.line())


def test_cfg0_exact(dev):
    """BASELINE configs[0] exactly: 1024 queries, 1024 local keys causal
    (global positions 1024-2047), 1024 peer keys non-causal, LSE merge; the
    flat 2e-3 / 1e-3 bar."""
    q, kp, vp, kl, vl = P.cfg0_inputs()
    out, lse = _fused_run(dev, q, kp, vp, kl, vl, 1024, 1024, 0)
    want, want_lse = P.fused_oracle((1024, 1024, 1024, 0), q, kp, vp, kl, vl)
    st = P.check_out(_f(out), want, "cfg0", case="cfg0")
    P.check_flat(_f(out), want, "cfg0")
    P.check_lse(_f(lse), want_lse, "cfg0")
    print(st.line())


def test_cfg3_n1_full_launch_sampled_rows(dev):
    """BASELINE configs[3] at N=1: one 131072-token causal launch (the bench's
    layer), checked against the oracle on the first and last 256-row blocks
    and 64 rows between them, plus LSE; the flat bar holds on every sampled
    row past the first block."""
    from hcp_vllm_plugin_b200.ops import ring_attn_with_lse
    q, k, v = P.cfg3_inputs(dev)
    o, lse = ring_attn_with_lse(q, k, v, D128 ** -0.5, 0)
    torch.cuda.synchronize()
    rows = P.cfg3_rows()
    want, want_lse = P.cfg3_oracle(q, k, v, rows)
    ri = torch.from_numpy(rows).to(dev)
    got, got_lse = _f(o[ri]), _f(lse[:, ri])
    st = P.check_out(got, want, "cfg3 N=1 sampled rows", case="cfg3_n1")
    P.check_lse(got_lse, want_lse, "cfg3 N=1")
    late = rows >= 256
    P.check_flat(got[late], want[late], "cfg3 N=1 rows >= 256")
    print(st.line())


def test_epilogue_merge_chains_hops(dev):
    """Hop 1 writes (O fp32, LSE); hop 2 merges into it in its epilogue; the
    result equals attention over both chunks (ring_decode.py:46-61 algebra)."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    g = torch.Generator(device="cpu").manual_seed(5)
    tq, t1, t2 = 384, 640, 384
    q = torch.randn(tq, H28, D128, generator=g).bfloat16().to(dev)
    k1 = torch.randn(t1, HKV4, D128, generator=g).bfloat16().to(dev)
    v1 = torch.randn(t1, HKV4, D128, generator=g).bfloat16().to(dev)
    k2 = torch.randn(t2, HKV4, D128, generator=g).bfloat16().to(dev)
    v2 = torch.randn(t2, HKV4, D128, generator=g).bfloat16().to(dev)
    scale = D128 ** -0.5
    acc = torch.empty(tq, H28, D128, dtype=torch.float32, device=dev)
    lse = torch.empty(H28, tq, dtype=torch.float32, device=dev)
    w1 = ops.make_work([(0, tq, 0, 0, (C.HCP_SRC_A, 0, t1, -1), None)])
    ops.ring_attn_fwd(q, w1, scale=scale, num_kv_heads=HKV4, out=acc, lse=lse, k_a=k1, v_a=v1)
    out = torch.empty(tq, H28, D128, dtype=torch.bfloat16, device=dev)
    lse2 = torch.empty_like(lse)
    w2 = ops.make_work([(0, tq, 0, 0, (C.HCP_SRC_A, 0, t2, 0), None)])
    ops.ring_attn_fwd(q, w2, scale=scale, num_kv_heads=HKV4, out=out, lse=lse2, k_a=k2, v_a=v2,
                      merge_o=acc, merge_lse=lse)
    torch.cuda.synchronize()
    o1, l1 = ro.attn_with_lse(_f(q), _f(k1), _f(v1), scale, None)
    o2, l2 = ro.attn_with_lse(_f(q), _f(k2), _f(v2), scale, 0)
    want, want_lse = ro.merge_pair(o1, l1, o2, l2)
    P.check_out(_f(out), want, "chained merge")
    P.check_lse(_f(lse2), want_lse, "chained merge")


@pytest.mark.parametrize("odt", [torch.bfloat16, torch.float32])
def test_merge_attn_states_kernel(dev, odt):
    from hcp_vllm_plugin_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(9)
    T = 97
    po = torch.randn(T, H28, D128, generator=g).to(odt)
    so = torch.randn(T, H28, D128, generator=g).to(odt)
    pl = torch.randn(H28, T, generator=g) * 3
    sl = torch.randn(H28, T, generator=g) * 3
    pl[0, 0] = float("inf")   # empty prefix partial
    sl[1, 1] = float("-inf")  # empty suffix partial
    out = torch.empty(T, H28, D128, dtype=odt, device=dev)
    olse = torch.empty(H28, T, dtype=torch.float32, device=dev)
    ops.merge_attn_states(out, po.to(dev), pl.to(dev), so.to(dev), sl.to(dev), olse)
    torch.cuda.synchronize()
    want, want_lse = ro.merge_attn_states(_f(po), pl.numpy(), _f(so), sl.numpy())
    if odt == torch.float32:
        P.check_flat(_f(out), want, "merge kernel fp32", tol=1e-5)
    else:
        P.check_out(_f(out), want, "merge kernel")
    np.testing.assert_allclose(_f(olse), want_lse, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("lens,peer", P.PAGED)
def test_paged_local_plus_peer_batch(dev, lens, peer):
    """cfg1-shaped continuous batch: local keys read straight from the paged
    cache (no gather), peer prefix contiguous; vs the oracle's forward driver."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    b = P.paged_batch(lens, peer)
    items = []
    for r, L in enumerate(lens):
        seg_peer = (C.HCP_SRC_A, r * peer, peer, -1) if peer else None
        # local keys are positions [peer, peer+L) of the request's paged sequence;
        # query 0 sits at local position 0 (qpos0 = peer, n_a = 0)
        seg_loc = (C.HCP_SRC_PAGED, peer, L, 0)
        items.append((int(b["qsl"][r]), L, r, int(b["qsl"][r]), seg_peer, seg_loc))
    work = ops.make_work(items)
    q = b["q"].to(dev)
    out = torch.empty_like(q)
    lse = torch.empty(H28, q.shape[0], dtype=torch.float32, device=dev)
    bt = torch.from_numpy(b["bt"]).to(dev)
    ops.ring_attn_fwd(q, work, scale=D128 ** -0.5, num_kv_heads=HKV4, out=out, lse=lse,
                      k_a=b["kp"].to(dev) if peer else None, v_a=b["vp"].to(dev) if peer else None,
                      kv_cache=b["cache"].to(dev),
                      block_table=bt)
    torch.cuda.synchronize()
    want = P.paged_oracle(b)
    name = P.paged_name(lens, peer)
    st = P.check_out(_f(out), want, name, case=name)
    if peer >= 512:
        P.check_flat(_f(out), want, f"paged batch {lens} (cfg1 shape)")
    print(st.line())


def test_segment_lists_over_separate_chunks(dev):
    """Work items whose peer keys sit in several separately allocated chunks
    (extra sources, as staged) plus paged local keys, as segment lists of up
    to 8 segments, equal the oracle over the concatenated keys; an inline
    item reading an extra source rides in the same launch."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    g = torch.Generator(device="cpu").manual_seed(77)
    E = C.HCP_SRC_EXT0
    b = P.paged_batch([300, 129, 1], 0, seed=7)  # paged local keys only; peers come from chunks
    chunk_lens = [[256, 128, 512], [64] * 7, [1000]]
    chunks = [[(torch.randn(n, HKV4, D128, generator=g).bfloat16(), torch.randn(n, HKV4, D128, generator=g).bfloat16())
               for n in lens] for lens in chunk_lens]
    ext, seg_list, items = [], [], []
    for r, L in enumerate(b["lens"]):
        segs = []
        for k, v in chunks[r]:
            segs.append((E + len(ext), 0, k.shape[0], -1))
            ext.append((k.to(dev), v.to(dev)))
        segs.append((C.HCP_SRC_PAGED, 0, L, 0))
        qs = int(b["qsl"][r])
        if len(segs) <= 2:
            items.append((qs, L, r, qs, segs[0], segs[1]))
        else:
            items.append((qs, L, r, qs, (C.HCP_SRC_LIST, len(seg_list), len(segs), 0), None))
            seg_list.extend(segs)
    assert len(ext) == 11
    # more than 8 sources: two calls, split by request
    q = b["q"].to(dev)
    out = torch.empty_like(q)
    lse = torch.empty(H28, q.shape[0], dtype=torch.float32, device=dev)
    cache, bt = b["cache"].to(dev), torch.from_numpy(b["bt"]).to(dev)
    kw = dict(scale=D128 ** -0.5, num_kv_heads=HKV4, out=out, lse=lse, kv_cache=cache, block_table=bt)
    ops.ring_attn_fwd(q, ops.make_work(items[:1]), ext=ext[:3], seg_list=np.array(seg_list[:4]), **kw)
    sl2 = [(s[0] - 3 if s[0] >= E else s[0], *s[1:]) for s in seg_list[4:]]
    it2 = [items[1][:4] + ((C.HCP_SRC_LIST, 0, 8, 0), None), items[2][:4] + ((E + 7, 0, 1000, -1),) + items[2][5:]]
    ops.ring_attn_fwd(q, ops.make_work(it2), ext=ext[3:], seg_list=np.array(sl2), **kw)
    torch.cuda.synchronize()
    for r, L in enumerate(b["lens"]):
        qs = int(b["qsl"][r])
        kl, vl = ro.paged_gather(_f(b["cache"]), b["bt"][r], L)
        k = np.concatenate([_f(c[0]) for c in chunks[r]] + [kl], 0)
        v = np.concatenate([_f(c[1]) for c in chunks[r]] + [vl], 0)
        want, want_lse = ro.attn_with_lse(_f(b["q"][qs:qs + L]), k, v, D128 ** -0.5, sum(chunk_lens[r]))
        P.check_out(_f(out[qs:qs + L]), want, f"segment list request {r}")
        P.check_lse(_f(lse[:, qs:qs + L]), want_lse, f"segment list request {r}")


def test_many_items_span_several_launches(dev):
    """More work items (200) and segments (~430) than one launch takes (160
    and 320): the host splits the call into several launches of one
    heaviest-first order, and a launch that holds a segment-list item runs
    the list kernel.  Every request equals the oracle."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    rng = np.random.default_rng(21)
    g = torch.Generator(device="cpu").manual_seed(21)
    n = 200
    tq = rng.integers(1, 41, n)
    pl = rng.integers(0, 300, n)          # peer keys, contiguous source A, non-causal
    ll = tq + rng.integers(0, 200, n)     # local keys, contiguous source B, causal
    qs, ps, ls = (np.concatenate([[0], np.cumsum(x)]).astype(int) for x in (tq, pl, ll))
    q = torch.randn(int(qs[-1]), H28, D128, generator=g).bfloat16()
    ka, va = (torch.randn(int(ps[-1]), HKV4, D128, generator=g).bfloat16() for _ in range(2))
    kb, vb = (torch.randn(int(ls[-1]), HKV4, D128, generator=g).bfloat16() for _ in range(2))
    items, seg_list = [], []
    for r in range(n):
        loc = (C.HCP_SRC_B, int(ls[r]), int(ll[r]), int(ll[r] - tq[r]))  # last query sees every local key
        if r % 7 == 3 and pl[r] >= 2:    # the peer keys as two segments of a list
            h = int(pl[r]) // 2
            seg_list += [(C.HCP_SRC_A, int(ps[r]), h, -1), (C.HCP_SRC_A, int(ps[r]) + h, int(pl[r]) - h, -1), loc]
            items.append((int(qs[r]), int(tq[r]), 0, int(qs[r]), (C.HCP_SRC_LIST, len(seg_list) - 3, 3, 0), None))
        else:
            peer = (C.HCP_SRC_A, int(ps[r]), int(pl[r]), -1) if pl[r] else None
            items.append((int(qs[r]), int(tq[r]), 0, int(qs[r]), peer, loc))
    assert len(items) > 160 and sum(3 if it[4] and it[4][0] == C.HCP_SRC_LIST else 2 for it in items) > 320
    qd = q.to(dev)
    out = torch.zeros_like(qd)
    lse = torch.zeros(H28, qd.shape[0], dtype=torch.float32, device=dev)
    ops.ring_attn_fwd(qd, ops.make_work(items), scale=D128 ** -0.5, num_kv_heads=HKV4, out=out, lse=lse,
                      k_a=ka.to(dev), v_a=va.to(dev), k_b=kb.to(dev), v_b=vb.to(dev), seg_list=np.array(seg_list))
    torch.cuda.synchronize()
    got, got_lse = _f(out), _f(lse)
    for r in range(n):
        qr = _f(q[qs[r]:qs[r + 1]])
        want, want_lse = ro.attn_with_lse(qr, _f(kb[ls[r]:ls[r + 1]]), _f(vb[ls[r]:ls[r + 1]]), D128 ** -0.5,
                                          int(ll[r] - tq[r]))
        if pl[r]:
            o_p, l_p = ro.attn_with_lse(qr, _f(ka[ps[r]:ps[r + 1]]), _f(va[ps[r]:ps[r + 1]]), D128 ** -0.5, None)
            want, want_lse = ro.merge_pair(want, want_lse, o_p, l_p)
        P.check_out(got[qs[r]:qs[r + 1]], want, f"request {r} of 200")
        P.check_lse(got_lse[:, qs[r]:qs[r + 1]], want_lse, f"request {r} of 200")


@pytest.mark.parametrize("tq,tk,off,window", [
    (1000, 1000, 0, 1), (1000, 1000, 0, 100), (1000, 1000, 0, 200), (1000, 1000, 0, 700),
    (300, 2000, 1700, 333), (1, 4096, 4095, 129), (513, 513, 0, 128)])
def test_sliding_window_contiguous(dev, tq, tk, off, window):
    """A causal segment with a sliding window (keys j with qpos - window < j <=
    qpos) vs the oracle's ``_attn_with_lse(window=...)`` restatement; whole KV
    tiles below a CTA's window are skipped, the edge tile is masked per row."""
    from hcp_vllm_plugin_b200.ops import ring_attn_with_lse
    g = torch.Generator(device="cpu").manual_seed(tq + tk + window)
    q = torch.randn(tq, H28, D128, generator=g).bfloat16()
    k = torch.randn(tk, HKV4, D128, generator=g).bfloat16()
    v = torch.randn(tk, HKV4, D128, generator=g).bfloat16()
    o, lse = ring_attn_with_lse(q.to(dev), k.to(dev), v.to(dev), D128 ** -0.5, off, window=window)
    torch.cuda.synchronize()
    rows = np.unique(np.r_[np.linspace(0, tq - 1, min(tq, 96)).astype(int), [tq - 1]])
    want_o, want_lse = ro.attn_with_lse(_f(q)[rows[0]:rows[-1] + 1], _f(k), _f(v), D128 ** -0.5,
                                        off + int(rows[0]), window)
    sel = rows - rows[0]
    name = f"window/{tq}x{tk}@{off}/w{window}"
    st = P.check_out(_f(o)[rows], want_o[sel], name)
    P.check_lse(_f(lse)[:, rows], want_lse[:, sel], name)
    print(st.line())


@pytest.mark.parametrize("window", [48, 300, 1500])
def test_sliding_window_paged_with_peers_and_lists(dev, window):
    """A cfg1-shaped batch with a window: the paged local segment is windowed,
    the contiguous peer prefix stays fully visible (the reference's forward,
    ring_backend.py:819-832); one request's keys come as a segment list (the
    list kernel) over two extra sources plus the paged local keys."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    lens, peer = [700, 129, 1, 2048], 512
    b = P.paged_batch(lens, peer, seed=11)
    E = C.HCP_SRC_EXT0
    kp, vp = b["kp"], b["vp"]
    items, seg_list, ext = [], [], []
    for r, L in enumerate(lens):
        qs = int(b["qsl"][r])
        loc = (C.HCP_SRC_PAGED, peer, L, 0)
        if r == 0:
            # the peer prefix as two separately allocated chunks: a list item
            half = peer // 2
            for c in range(2):
                sl = slice(r * peer + c * half, r * peer + (c + 1) * half)
                ext.append((kp[sl].contiguous().to(dev), vp[sl].contiguous().to(dev)))
            seg_list += [(E + 0, 0, half, -1), (E + 1, 0, half, -1), loc]
            items.append((qs, L, r, qs, (C.HCP_SRC_LIST, 0, 3, 0), None))
        else:
            items.append((qs, L, r, qs, (C.HCP_SRC_A, r * peer, peer, -1), loc))
    q = b["q"].to(dev)
    out = torch.empty_like(q)
    lse = torch.empty(H28, q.shape[0], dtype=torch.float32, device=dev)
    ops.ring_attn_fwd(q, ops.make_work(items), scale=D128 ** -0.5, num_kv_heads=HKV4, out=out, lse=lse,
                      k_a=kp.to(dev), v_a=vp.to(dev), kv_cache=b["cache"].to(dev),
                      block_table=torch.from_numpy(b["bt"]).to(dev), ext=ext, seg_list=np.array(seg_list),
                      window=window)
    torch.cuda.synchronize()
    for r, L in enumerate(lens):
        qs = int(b["qsl"][r])
        kl, vl = P.paged_local_kv(b, r)
        qr = _f(b["q"][qs:qs + L])
        o_loc, l_loc = ro.attn_with_lse(qr, _f(kl), _f(vl), D128 ** -0.5, 0, window)
        o_peer, l_peer = ro.attn_with_lse(qr, _f(kp[r * peer:(r + 1) * peer]), _f(vp[r * peer:(r + 1) * peer]),
                                          D128 ** -0.5, None)
        want = ro.lse_merge(o_loc, l_loc, o_peer, l_peer)
        m = np.maximum(l_loc, l_peer)
        want_lse = m + np.log(np.exp(l_loc - m) + np.exp(l_peer - m))
        name = f"window {window} paged request {r} ({'list' if r == 0 else 'inline'})"
        P.check_out(_f(out[qs:qs + L]), want, name)
        P.check_lse(_f(lse[:, qs:qs + L]), want_lse, name)
