"""GPU parity of split-KV decode and the paged-cache scatter against the oracle.

Decode outputs use the bar of ``tests/parity.py`` (LSE 1e-3; every output
element equal to, or one bf16 step from, the reference's own output; within
2e-3 of the fp32 oracle or no further off than the reference's own output)
and the flat 2e-3 wherever every sequence attends >= 1024 keys.  BASELINE
configs[2] is checked at its full size: 64 sequences x (32768 paged + 32768
peer) keys.
"""

import numpy as np
import pytest
import torch

import parity as P
from oracle import ring_oracle as ro

pytestmark = pytest.mark.gpu

_f = P.f32


@pytest.fixture(scope="module")
def dev():
    from hcp_vllm_plugin_b200 import _capi
    _capi.load()
    _capi.reset_device_status()
    yield torch.device("cuda:0")
    assert _capi.device_status() == 0


_decode_case = P.decode_case
_oracle_decode = P.decode_oracle


@pytest.mark.parametrize("peer_lens,local_lens,chunk", P.DECODE)
def test_decode_splitkv_matches_oracle(dev, peer_lens, local_lens, chunk):
    from hcp_vllm_plugin_b200 import ops
    q, pk, pv, cache, bt, seqs = _decode_case(peer_lens, local_lens)
    scale = 128 ** -0.5
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
    ops.decode_splitkv(q.to(dev), seqs, scale=scale, num_kv_heads=4, out=out, lse=lse,
                       peer_k=pk.to(dev), peer_v=pv.to(dev), kv_cache=cache.to(dev),
                       block_table=torch.from_numpy(bt).to(dev), chunk_keys=chunk)
    torch.cuda.synchronize()
    want, want_lse = _oracle_decode(q, pk, pv, cache, bt, seqs, scale)
    name = P.decode_name(peer_lens, local_lens, chunk)
    st = P.check_out(_f(out), want, name, case=name)
    if min(p + l for p, l in zip(peer_lens, local_lens)) >= 1024:
        P.check_flat(_f(out), want, name)
    P.check_lse(_f(lse), want_lse, name)
    print(st.line())


def test_cfg2_full_size(dev):
    """BASELINE configs[2] in full: 64 single-token queries, each over 32768
    paged local keys + 32768 peer keys, one batch-merged launch; flat 2e-3 on
    the output and 1e-3 on the LSE against the fp32 oracle."""
    from hcp_vllm_plugin_b200 import ops
    q, pk, pv, cache, bt, seqs = P.cfg2_inputs(dev)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
    ops.decode_splitkv(q, seqs, scale=P.D128 ** -0.5, num_kv_heads=4, out=out, lse=lse,
                       peer_k=pk, peer_v=pv, kv_cache=cache, block_table=bt.to(dev))
    torch.cuda.synchronize()
    want, want_lse = P.cfg2_oracle(q, pk, pv, cache, bt, seqs)
    st = P.check_out(_f(out), want, "cfg2", case="cfg2")
    P.check_flat(_f(out), want, "cfg2")
    P.check_lse(_f(lse), want_lse, "cfg2")
    print(st.line())


def test_decode_peer_keys_in_separate_sources(dev):
    """Each sequence's peer keys in its own staged tensor (an extra source,
    peer_src), or the common peer arena, or none: equal to the oracle."""
    from hcp_vllm_plugin_b200 import ops
    q, pk, pv, cache, bt, seqs = _decode_case([700, 0, 300, 1000], [500, 129, 0, 2048], seed=5)
    g = torch.Generator(device="cpu").manual_seed(6)
    own = {0: 700, 3: 1000}  # sequences 0 and 3 read their own tensors
    ext, src = [], []
    for r in range(4):
        if r in own:
            k = torch.randn(own[r] + 16, 4, 128, generator=g).bfloat16()
            v = torch.randn(own[r] + 16, 4, 128, generator=g).bfloat16()
            ext.append((k, v))
            seqs[r][1] = 16          # start inside the source
            src.append(len(ext) - 1)
        else:
            src.append(-1)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
    ops.decode_splitkv(q.to(dev), seqs, scale=128 ** -0.5, num_kv_heads=4, out=out, lse=lse,
                       peer_k=pk.to(dev), peer_v=pv.to(dev), kv_cache=cache.to(dev),
                       block_table=torch.from_numpy(bt).to(dev), chunk_keys=256,
                       ext=[(k.to(dev), v.to(dev)) for k, v in ext], peer_src=np.array(src, np.int32))
    torch.cuda.synchronize()
    for r, (qr, ps, pl, preq, ls, ll) in enumerate(seqs):
        kp_, vp_ = (ext[src[r]] if src[r] >= 0 else (pk, pv))
        kloc, vloc = ro.paged_gather(_f(cache), bt[preq], ls + ll)
        k = np.concatenate([_f(kp_[ps:ps + pl]), kloc[ls:]], 0)
        v = np.concatenate([_f(vp_[ps:ps + pl]), vloc[ls:]], 0)
        want, want_lse = ro.attn_with_lse(_f(q[qr:qr + 1]), k, v, 128 ** -0.5, None)
        P.check_out(_f(out[qr]), want[0], f"decode source {src[r]} seq {r}")
        P.check_lse(_f(lse[:, qr]), want_lse[:, 0], f"decode source {src[r]} seq {r}")


def test_decode_fp16_d64(dev):
    from hcp_vllm_plugin_b200 import ops
    q, pk, pv, cache, bt, seqs = _decode_case([512, 100], [700, 33], h=14, hkv=2, d=64,
                                              dt=torch.float16, seed=4)
    scale = 64 ** -0.5
    out = torch.empty(q.shape, dtype=torch.float16, device=dev)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=dev)
    ops.decode_splitkv(q.to(dev), seqs, scale=scale, num_kv_heads=2, out=out, lse=lse,
                       peer_k=pk.to(dev), peer_v=pv.to(dev), kv_cache=cache.to(dev),
                       block_table=torch.from_numpy(bt).to(dev), chunk_keys=256)
    torch.cuda.synchronize()
    want, want_lse = _oracle_decode(q, pk, pv, cache, bt, seqs, scale)
    P.check_out(_f(out), want, "decode fp16 d64", torch.float16)
    P.check_flat(_f(out), want, "decode fp16 d64")
    P.check_lse(_f(lse), want_lse, "decode fp16 d64")


def test_kv_cache_update_matches_oracle(dev):
    from hcp_vllm_plugin_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(11)
    nb, hkv, bs, d, n = 40, 4, 16, 128, 300
    cache = torch.randn(nb, hkv, bs, 2 * d, generator=g).bfloat16()
    key = torch.randn(n, hkv, d, generator=g).bfloat16()
    val = torch.randn(n, hkv, d, generator=g).bfloat16()
    slots = torch.from_numpy(np.random.default_rng(1).permutation(nb * bs)[:n].astype(np.int64))
    slots[7] = -1
    slots[9] = -1
    dc = cache.to(dev)
    ops.kv_cache_update(key.to(dev), val.to(dev), dc, slots.to(dev))
    torch.cuda.synchronize()
    want = _f(cache)
    ro.kv_cache_update(want, _f(key), _f(val), slots.numpy())
    np.testing.assert_array_equal(_f(dc), want)


def test_decode_on_two_streams_keeps_each_streams_partials(dev):
    """The decode ring's serve thread and the backend run split-KV decode on
    different streams of one device at the same time: each stream's calls
    use their own cached workspace, so results launched back to back on two
    streams equal the same calls run one after the other, bit for bit."""
    from hcp_vllm_plugin_b200 import ops
    g = torch.Generator(device=dev).manual_seed(3)
    H, HKV, D, n, keys = 28, 4, 128, 8, 8192

    def problem():
        q = torch.randn(n, H, D, generator=g, device=dev, dtype=torch.bfloat16)
        pk = torch.randn(n * keys, HKV, D, generator=g, device=dev, dtype=torch.bfloat16)
        pv = torch.randn(n * keys, HKV, D, generator=g, device=dev, dtype=torch.bfloat16)
        return q, pk, pv, np.array([(i, i * keys, keys, -1, 0, 0) for i in range(n)], np.int32)

    def run(q, pk, pv, seqs):
        out = torch.empty_like(q)
        lse = torch.empty(H, n, dtype=torch.float32, device=dev)
        ops.decode_splitkv(q, seqs, scale=D ** -0.5, num_kv_heads=HKV, out=out, lse=lse, peer_k=pk, peer_v=pv)
        return out, lse

    probs = [problem(), problem()]
    serial = [run(*p) for p in probs]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    for _ in range(5):
        res = []
        for s, p in zip(streams, probs):
            with torch.cuda.stream(s):
                res.append(run(*p))
        torch.cuda.synchronize()
        for (o, l), (so, sl) in zip(res, serial):
            assert torch.equal(o, so) and torch.equal(l, sl)
