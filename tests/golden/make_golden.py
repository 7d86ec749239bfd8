"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference plugin's own code on CPU (torch fp32 path) and stores its
inputs and outputs as compressed ``.npz`` files next to this script:

* ``kernel_cases.npz`` - ``_attn_with_lse`` on the shape/offset cases of the
  reference's kernel probe ``validate_ring_triton_kernel.py:41-61`` (H=14,
  Hkv=2, D=64, fp16, seed 0), causal and non-causal, plus the same probe at
  the deployment geometry (H=28, Hkv=4, D=128, bf16).  For the larger cases
  only a strided subset of query rows is kept (rows are independent).
* ``merge_cases.npz`` - ``_lse_merge`` (``ring_backend.py:409-421``) and the
  two-chunk-vs-full identity of ``validate_ring_triton_kernel.py:80-94``.
* ``forward_case.npz`` - ``HcpRingAttentionImpl.forward``
  (``ring_backend.py:576-834``) on a small continuous batch: staged peer
  chunks, a request with queries inside the peer region (``n_a > 0``), a
  decode-like single-token request, a request without peer KV, and a
  multi-chunk peer prefix.  The reference cache layout
  ``[num_blocks, 2, block_size, Hkv, D]`` is converted to
  ``[num_blocks, Hkv, block_size, 2*D]`` for storage.
* ``window_case.npz`` (``--window``) - the same batch through a
  ``HcpRingAttentionImpl`` built with ``sliding_window=20`` (the reference
  applies the window to the causal passes, ``ring_backend.py:786-826``), and
  ``_attn_with_lse`` with windows 1, 7 and 64 on causal cases.

Usage (in a container holding the reference sources and vLLM)::

    HCP_REFERENCE_ROOT=/path/to/hcp-vllm-plugin python tests/golden/make_golden.py [--window]
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

REF_ROOT = os.environ.get("HCP_REFERENCE_ROOT", "")  # the reference checkout (generation only)
OUT_DIR = os.path.dirname(os.path.abspath(__file__))


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _rows(tq: int) -> np.ndarray:
    """Query rows kept for a case: all of them when small, else a strided set
    that always includes the first and last rows."""
    if tq <= 8:
        return np.arange(tq)
    r = np.unique(np.concatenate([np.arange(0, tq, max(1, tq // 12)), [tq - 1], np.arange(4)]))
    return r.astype(np.int64)


def kernel_cases(attn_with_lse) -> dict:
    out: dict[str, np.ndarray] = {}
    specs = [
        # (name, H, Hkv, D, dtype, cases) ; cases from validate_ring_triton_kernel.py:41-48
        ("a", 14, 2, 64, torch.float16,
         [(1, 1, 0), (1, 512, 511), (37, 37, 0), (37, 512, 475), (512, 512, 0), (512, 2048, 1536)]),
        ("b", 28, 4, 128, torch.bfloat16,
         [(1, 1, 0), (1, 512, 511), (37, 37, 0), (37, 512, 475), (160, 640, 480)]),
    ]
    idx = 0
    for tag, h, hkv, d, dt, cases in specs:
        torch.manual_seed(0)
        scale = 1.0 / (d ** 0.5)
        for tq, tk, off in cases:
            q = torch.randn(tq, h, d, dtype=dt)
            k = torch.randn(tk, hkv, d, dtype=dt)
            v = torch.randn(tk, hkv, d, dtype=dt)
            rows = _rows(tq)
            key = f"c{idx:02d}"
            out[f"{key}_meta"] = np.array([h, hkv, d, tq, tk, off, 1 if dt == torch.bfloat16 else 0],
                                          np.int64)
            out[f"{key}_scale"] = np.array([scale], np.float64)
            out[f"{key}_rows"] = rows
            out[f"{key}_q"] = _u16(q[rows])
            out[f"{key}_k"] = _u16(k)
            out[f"{key}_v"] = _u16(v)
            for causal in (True, False):
                o, lse = attn_with_lse(q, k, v, scale, off if causal else None, None)
                tag2 = "causal" if causal else "noncausal"
                out[f"{key}_{tag2}_out"] = o[rows].float().numpy()
                out[f"{key}_{tag2}_lse"] = lse[:, rows].float().numpy()
            idx += 1
    out["count"] = np.array([idx], np.int64)
    return out


def merge_cases(attn_with_lse, lse_merge) -> dict:
    out: dict[str, np.ndarray] = {}
    torch.manual_seed(1)
    h, hkv, d = 14, 2, 64
    scale = 1.0 / (d ** 0.5)
    # validate_ring_triton_kernel.py:63-78, reduced to 64 query rows.
    tq, tk_a, tk_b = 32, 512, 512
    q = torch.randn(tq, h, d, dtype=torch.float16)
    ka, va = torch.randn(tk_a, hkv, d, dtype=torch.float16), torch.randn(tk_a, hkv, d, dtype=torch.float16)
    kb, vb = torch.randn(tk_b, hkv, d, dtype=torch.float16), torch.randn(tk_b, hkv, d, dtype=torch.float16)
    o_a, lse_a = attn_with_lse(q, ka, va, scale, None, None)
    o_b, lse_b = attn_with_lse(q, kb, vb, scale, 0, None)
    m = lse_merge(o_b, lse_b, o_a, lse_a)
    out.update(o_a=o_a.numpy(), lse_a=lse_a.numpy(), o_b=o_b.numpy(), lse_b=lse_b.numpy(), merged=m.numpy())
    # validate_ring_triton_kernel.py:80-94: two-chunk merged vs full attention.
    tk_full, split, tq3 = 1024, 512, 32
    q3 = torch.randn(tq3, h, d, dtype=torch.float16)
    k3 = torch.randn(tk_full, hkv, d, dtype=torch.float16)
    v3 = torch.randn(tk_full, hkv, d, dtype=torch.float16)
    o_full, lse_full = attn_with_lse(q3, k3, v3, scale, tk_full - tq3, None)
    o_loc, lse_loc = attn_with_lse(q3, k3[split:], v3[split:], scale, tk_full - tq3 - split, None)
    o_peer, lse_peer = attn_with_lse(q3, k3[:split], v3[:split], scale, None, None)
    merged = lse_merge(o_loc, lse_loc, o_peer, lse_peer)
    out.update(q3=_u16(q3), k3=_u16(k3), v3=_u16(v3), o_full=o_full.numpy(), lse_full=lse_full.numpy(),
               merged3=merged.numpy(), scale=np.array([scale]), split=np.array([split]))
    return out


def forward_case(rb, window: int | None = None) -> dict:
    """Run the reference HcpRingAttentionImpl.forward on CPU over a small batch."""
    torch.manual_seed(2)
    h, hkv, d, bs = 28, 4, 128, 16
    scale = 1.0 / (d ** 0.5)
    # (tq, tk, staged peer lengths) per request.  Request 1 has its queries
    # starting at position 0 with a staged 32-token peer: n_a = 32 > 0.
    reqs = [
        (40, 72, [32]),        # staged single chunk, local 40 keys, qpos0 = 32
        (64, 64, [32]),        # n_a = 32: queries inside the peer region
        (1, 97, [48]),         # decode-like single query
        (24, 24, None),        # no peer: vanilla causal
        (30, 94, [32, 16, 16]),  # multi-chunk ordered prefix (64 tokens)
    ]
    num_blocks = 64
    max_blocks = 8
    cache_ref = torch.zeros(num_blocks, 2, bs, hkv, d, dtype=torch.bfloat16)
    perm = torch.randperm(num_blocks)
    block_table = torch.zeros(len(reqs), max_blocks, dtype=torch.int32)
    nxt = 0
    for r, (tq, tk, peers) in enumerate(reqs):
        nb = (tk + bs - 1) // bs
        block_table[r, :nb] = perm[nxt:nxt + nb].to(torch.int32)
        nxt += nb
        # fill every slot of the request's blocks (peer region included: the
        # reference never reads it on the staged path)
        for b in range(nb):
            blk = int(block_table[r, b])
            cache_ref[blk] = torch.randn(2, bs, hkv, d, dtype=torch.bfloat16)
    qsl = [0]
    for tq, _, _ in reqs:
        qsl.append(qsl[-1] + tq)
    num_tokens = qsl[-1]
    query = torch.randn(num_tokens, h, d, dtype=torch.bfloat16)

    rb.clear_peer_kv()
    staged_np: dict[str, np.ndarray] = {}
    layer_name = "model.layers.0.self_attn.attn"
    for r, (tq, tk, peers) in enumerate(reqs):
        if peers is None:
            continue
        keys = []
        for c, plen in enumerate(peers):
            ck = f"req{r}_chunk{c}"
            kp = torch.randn(plen, hkv, d, dtype=torch.bfloat16)
            vp = torch.randn(plen, hkv, d, dtype=torch.bfloat16)
            rb.stage_peer_kv(ck, layer_name, kp, vp)
            staged_np[f"peer{r}_{c}_k"] = _u16(kp)
            staged_np[f"peer{r}_{c}_v"] = _u16(vp)
            keys.append(ck)
        rb.map_request_peer(int(block_table[r, 0]), keys)

    impl = rb.HcpRingAttentionImpl(h, d, scale, hkv, sliding_window=window)
    meta = types.SimpleNamespace(
        num_actual_tokens=num_tokens,
        query_start_loc=torch.tensor(qsl, dtype=torch.int32),
        seq_lens=torch.tensor([tk for _, tk, _ in reqs], dtype=torch.int32),
        block_table=block_table,
    )
    layer = types.SimpleNamespace(layer_name=layer_name)
    output = torch.zeros(num_tokens, h, d, dtype=torch.bfloat16)
    rb.reset_impl_stats()
    impl.forward(layer, query, None, None, cache_ref, meta, output)
    assert rb.IMPL_STATS["attn_torch"] > 0 and rb.IMPL_STATS["merge_torch"] > 0
    rb.clear_peer_kv()

    # [nb, 2, bs, Hkv, D] -> [nb, Hkv, bs, 2D]
    cache_new = cache_ref.permute(0, 3, 2, 1, 4).reshape(num_blocks, hkv, bs, 2 * d).contiguous()
    out = dict(
        meta=np.array([h, hkv, d, bs, len(reqs), num_tokens], np.int64),
        scale=np.array([scale]),
        query=_u16(query),
        cache=_u16(cache_new),
        block_table=block_table.numpy(),
        query_start_loc=np.array(qsl, np.int64),
        seq_lens=np.array([tk for _, tk, _ in reqs], np.int64),
        peer_counts=np.array([0 if p is None else len(p) for _, _, p in reqs], np.int64),
        output=_u16(output),
        window=np.array([0 if window is None else window], np.int64),
    )
    out.update(staged_np)
    return out


def window_kernel_cases(attn_with_lse) -> dict:
    """``_attn_with_lse`` with a sliding window (H=28, Hkv=4, D=128, bf16)."""
    torch.manual_seed(3)
    out: dict[str, np.ndarray] = {}
    for i, (tq, tk, off, w) in enumerate([(37, 37, 0, 1), (37, 512, 475, 7), (96, 300, 204, 64)]):
        q = torch.randn(tq, 28, 128, dtype=torch.bfloat16)
        k = torch.randn(tk, 4, 128, dtype=torch.bfloat16)
        v = torch.randn(tk, 4, 128, dtype=torch.bfloat16)
        o, lse = attn_with_lse(q, k, v, 128 ** -0.5, off, w)
        rows = _rows(tq)
        out[f"w{i}_q"], out[f"w{i}_k"], out[f"w{i}_v"] = _u16(q), _u16(k), _u16(v)
        out[f"w{i}_rows"] = rows
        out[f"w{i}_o"], out[f"w{i}_lse"] = o.numpy()[rows], lse.numpy()[:, rows]
        out[f"w{i}_meta"] = np.array([tq, tk, off, w], np.int64)
    return out


def main() -> None:
    if not REF_ROOT:
        raise SystemExit("set HCP_REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, REF_ROOT)
    os.environ["HCP_RING_IMPL"] = "torch"
    os.environ["HCP_RING_MERGE"] = "torch"
    os.environ.setdefault("HCP_RING_SPLIT_TOKENS", "0")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from hcp_vllm_plugin import ring_backend as rb  # noqa: E402  (reference code)

    if "--window" in sys.argv:
        # the batch's inputs are those of forward_case.npz (same seed): keep
        # only the windowed output
        full = forward_case(rb, window=20)
        case = {"output": full["output"], "window": full["window"]}
        case.update(window_kernel_cases(rb._attn_with_lse))
        np.savez_compressed(os.path.join(OUT_DIR, "window_case.npz"), **case)
        print("window fixture written to", OUT_DIR)
        return
    np.savez_compressed(os.path.join(OUT_DIR, "kernel_cases.npz"), **kernel_cases(rb._attn_with_lse))
    np.savez_compressed(os.path.join(OUT_DIR, "merge_cases.npz"),
                        **merge_cases(rb._attn_with_lse, rb._lse_merge))
    np.savez_compressed(os.path.join(OUT_DIR, "forward_case.npz"), **forward_case(rb))
    print("golden fixtures written to", OUT_DIR)


if __name__ == "__main__":
    main()
