"""GPU parity of the fused ring-attention forward against the CPU oracle.

All calls go through the C ABI (``libhcp_ring.so``).  Tolerances:
  * LSE: 1e-3 absolute.
  * Output, fp16: 2e-3 absolute (the reference probe's bar,
    ``validate_ring_triton_kernel.py:55-61``).
  * Output, bf16: 2e-3 absolute plus 2^-7 relative (one bf16 step).  The
    output tensor is bf16 and the reference's own path rounds its fp32
    result to bf16 (``o.to(output.dtype)``, ``ring_backend.py:832``), and
    its kernel feeds P to the PV product in the value dtype
    (``p.to(v.dtype)``, ``ring_triton_attn.py:132``).  Each of these is up to
    2^-9 relative, so rows that see only a handful of keys (|o| ~ 1) cannot
    meet a flat 2e-3 in bf16 - not even the reference's kernel.
  * Output at the deployment shapes (every row sees >= 512 keys, as in the
    BASELINE configs): the flat 2e-3 north-star bar, checked separately.
"""

import numpy as np
import pytest
import torch

from oracle import ring_oracle as ro

pytestmark = pytest.mark.gpu

H28, HKV4, D128 = 28, 4, 128


def _f(t):
    return t.float().cpu().numpy()


def _check_out(got, want, dtype, what):
    got = np.asarray(got, np.float32)
    err = np.abs(got - want)
    if dtype == torch.float16:
        tol = np.full_like(want, 2e-3)
    else:
        tol = 2e-3 + 2.0 ** -7 * np.abs(want)
    bad = err > tol
    assert not bad.any(), (f"{what}: {bad.sum()} / {bad.size} outside tolerance, "
                           f"max err {err.max():.3e}")


def _check_flat(got, want, what, tol=2e-3):
    err = np.abs(np.asarray(got, np.float32) - want)
    assert err.max() <= tol, f"{what}: flat max err {err.max():.3e} > {tol}"


def _check_lse(got, want, what):
    err = np.abs(np.asarray(got) - want)
    assert err.max() <= 1e-3, f"{what}: lse max err {err.max():.3e}"


@pytest.fixture(scope="module")
def dev():
    from hcp_vllm_plugin_b200 import _capi
    assert torch.cuda.is_available()
    _capi.load()
    _capi.reset_device_status()
    yield torch.device("cuda:0")
    assert _capi.device_status() == 0


# Reference probe cases (validate_ring_triton_kernel.py:41-48)
PROBE = [(1, 1, 0), (1, 512, 511), (37, 37, 0), (37, 512, 475), (512, 512, 0), (512, 2048, 1536)]


@pytest.mark.parametrize("geom", [(14, 2, 64, torch.float16), (28, 4, 128, torch.bfloat16),
                                  (28, 4, 128, torch.float16), (14, 2, 64, torch.bfloat16)])
@pytest.mark.parametrize("case", PROBE)
@pytest.mark.parametrize("causal", [True, False])
def test_ring_attn_with_lse_probe(dev, geom, case, causal):
    from hcp_vllm_plugin_b200.ops import ring_attn_with_lse
    h, hkv, d, dt = geom
    tq, tk, off = case
    g = torch.Generator(device="cpu").manual_seed(tq * 7919 + tk)
    q = torch.randn(tq, h, d, generator=g).to(dt)
    k = torch.randn(tk, hkv, d, generator=g).to(dt)
    v = torch.randn(tk, hkv, d, generator=g).to(dt)
    scale = d ** -0.5
    o, lse = ring_attn_with_lse(q.to(dev), k.to(dev), v.to(dev), scale, off if causal else None)
    torch.cuda.synchronize()
    want_o, want_lse = ro.attn_with_lse(_f(q), _f(k), _f(v), scale, off if causal else None)
    _check_out(_f(o), want_o, dt, f"probe {geom[:3]} {case} causal={causal}")
    _check_lse(_f(lse), want_lse, "probe")


def test_golden_kernel_cases_through_cuda(dev):
    """The reference's own outputs (tests/golden) reproduced by the CUDA path."""
    import os
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
                _check_out(_f(o)[0], z[f"{key}_{tag}_out"][i], dt, f"golden {key} row {r} {tag}")
                _check_lse(_f(lse)[:, 0], z[f"{key}_{tag}_lse"][:, i], f"golden {key}")
    torch.cuda.synchronize()


@pytest.mark.parametrize("tq,tpeer,tloc,off", [(1024, 1024, 1024, 0), (300, 517, 300, 0),
                                               (77, 0, 333, 256), (129, 128, 0, 0), (1, 4096, 1, 0)])
def test_fused_peer_plus_local_equals_merge(dev, tq, tpeer, tloc, off):
    """One launch over [peer (non-causal), local (causal)] equals the reference's
    local pass + peer pass + _lse_merge (ring_backend.py:819-832)."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    g = torch.Generator(device="cpu").manual_seed(tq + tpeer + tloc)
    q = torch.randn(tq, H28, D128, generator=g).bfloat16()
    kp = torch.randn(max(tpeer, 1), HKV4, D128, generator=g).bfloat16()
    vp = torch.randn(max(tpeer, 1), HKV4, D128, generator=g).bfloat16()
    kl = torch.randn(max(tloc, 1), HKV4, D128, generator=g).bfloat16()
    vl = torch.randn(max(tloc, 1), HKV4, D128, generator=g).bfloat16()
    scale = D128 ** -0.5
    out = torch.empty(tq, H28, D128, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(H28, tq, dtype=torch.float32, device=dev)
    segs = []
    if tpeer:
        segs.append((C.HCP_SRC_A, 0, tpeer, -1))
    if tloc:
        segs.append((C.HCP_SRC_B, 0, tloc, off))
    segs += [None] * (2 - len(segs))
    work = ops.make_work([(0, tq, 0, 0, segs[0], segs[1])])
    ops.ring_attn_fwd(q.to(dev), work, scale=scale, num_kv_heads=HKV4, out=out, lse=lse,
                      k_a=kp.to(dev), v_a=vp.to(dev), k_b=kl.to(dev), v_b=vl.to(dev))
    torch.cuda.synchronize()
    parts = []
    if tloc:
        parts.append(ro.attn_with_lse(_f(q), _f(kl), _f(vl), scale, off))
    if tpeer:
        parts.append(ro.attn_with_lse(_f(q), _f(kp), _f(vp), scale, None))
    want, want_lse = parts[0]
    if len(parts) == 2:
        want, want_lse = ro.merge_pair(parts[0][0], parts[0][1], parts[1][0], parts[1][1])
    _check_out(_f(out), want, torch.bfloat16, "fused peer+local")
    if tpeer >= 512:
        _check_flat(_f(out), want, "fused peer+local (deployment shape)")
    _check_lse(_f(lse), want_lse, "fused peer+local")


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
    _check_out(_f(out), want, torch.bfloat16, "chained merge")
    _check_lse(_f(lse2), want_lse, "chained merge")


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
    _check_out(_f(out), want, torch.bfloat16, "merge kernel")
    np.testing.assert_allclose(_f(olse), want_lse, atol=1e-5, rtol=1e-5)


def _paged_batch(lens, peer, bs=16, seed=3, h=H28, hkv=HKV4, d=D128):
    """A cfg1-style batch: local K/V in a paged cache behind a random block
    permutation, a contiguous staged peer prefix per request."""
    rng = np.random.default_rng(seed)
    nreq = len(lens)
    blocks_per = [(peer + L + bs - 1) // bs for L in lens]
    num_blocks = sum(blocks_per) + 7
    perm = rng.permutation(num_blocks)
    max_blocks = max(blocks_per)
    bt = np.zeros((nreq, max_blocks), np.int32)
    nxt = 0
    for r, nb in enumerate(blocks_per):
        bt[r, :nb] = perm[nxt:nxt + nb]
        nxt += nb
    g = torch.Generator(device="cpu").manual_seed(seed)
    cache = torch.randn(num_blocks, hkv, bs, 2 * d, generator=g).bfloat16()
    qsl = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    q = torch.randn(int(qsl[-1]), h, d, generator=g).bfloat16()
    kp = torch.randn(nreq * peer, hkv, d, generator=g).bfloat16()
    vp = torch.randn(nreq * peer, hkv, d, generator=g).bfloat16()
    return dict(cache=cache, bt=bt, qsl=qsl, q=q, kp=kp, vp=vp, lens=lens, peer=peer, bs=bs)


@pytest.mark.parametrize("lens,peer", [([512, 1024, 2048, 3072], 1024), ([5, 1, 130, 17], 32),
                                       ([1], 0)])
def test_paged_local_plus_peer_batch(dev, lens, peer):
    """cfg1-shaped continuous batch: local keys read straight from the paged
    cache (no gather), peer prefix contiguous; vs the oracle's forward driver."""
    from hcp_vllm_plugin_b200 import _capi as C, ops
    b = _paged_batch(lens, peer)
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
    staged = {r: (_f(b["kp"][r * peer:(r + 1) * peer]), _f(b["vp"][r * peer:(r + 1) * peer]))
              for r in range(len(lens))} if peer else {}
    batch = ro.RingBatch(query=_f(b["q"]), cache=_f(b["cache"]), block_table=b["bt"],
                         query_start_loc=b["qsl"], seq_lens=np.array([peer + L for L in lens]),
                         scale=D128 ** -0.5, staged=staged)
    want = ro.ring_forward(batch, round_to_bf16=False)
    _check_out(_f(out), want, torch.bfloat16, f"paged batch {lens}")
    if peer >= 512:
        _check_flat(_f(out), want, f"paged batch {lens} (cfg1 shape)")
