"""Record how far the reference's own B200 path is from its fp32 torch path.

For every parity case of ``tests/parity.py`` (identical seeded inputs), runs
the reference plugin's GPU path exactly as ``HcpRingAttentionImpl.forward``
does (``hcp_vllm_plugin/ring_backend.py:773-832``): its Triton
``ring_attn_with_lse`` (``ring_triton_attn.py:155-207``) for the local
(causal) and peer (non-causal) passes, vLLM ``merge_attn_states`` for the
merge, the result in the 16-bit output dtype.  Each output is compared with
the oracle (the reference's fp32 torch path restated); the max-abs errors and
the number of elements beyond the flat 2e-3 bar go to ``ref_gpu_errors.json``,
which ``tests/parity.py`` reports beside this library's errors.

Needs a CUDA GPU, vLLM and the reference package::

    HCP_REFERENCE_ROOT=/path/to/reference python tests/golden/make_ref_gpu_errors.py [--out FILE]
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))                   # tests/
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root (oracle)

import parity as P  # noqa: E402
from oracle import ring_oracle as ro  # noqa: E402

REF_ROOT = os.environ.get("HCP_REFERENCE_ROOT", "")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "ref_gpu_errors.json"))
    ap.add_argument("--no-full", action="store_true", help="skip the BASELINE-size cases")
    args = ap.parse_args()
    if not REF_ROOT:
        raise SystemExit("set HCP_REFERENCE_ROOT to the reference package root")
    sys.path.insert(0, REF_ROOT)
    from hcp_vllm_plugin.ring_triton_attn import ring_attn_with_lse  # reference code, unchanged
    from vllm.v1.attention.ops.merge_attn_states import merge_attn_states

    dev = torch.device("cuda:0")
    res: dict[str, dict] = {}

    def attn(q, k, v, scale, off):
        return ring_attn_with_lse(q.to(dev).contiguous(), k.to(dev).contiguous(), v.to(dev).contiguous(),
                                  scale, None if off is None else int(off))

    def ring(q, kp, vp, kl, vl, scale, off):
        """local causal + peer non-causal + merge (ring_backend.py:819-832)."""
        if kp is None:
            return attn(q, kl, vl, scale, off)
        if kl is None:
            return attn(q, kp, vp, scale, None)
        o_loc, lse_loc = attn(q, kl, vl, scale, off)
        o_peer, lse_peer = attn(q, kp, vp, scale, None)
        out = torch.empty_like(o_loc)
        merged_lse = torch.empty_like(lse_loc)
        merge_attn_states(out, o_peer, lse_peer, o_loc, lse_loc, merged_lse)
        return out, merged_lse

    def record(name, got, got_lse, want, want_lse, dtype):
        got = P.f32(got)
        err = np.abs(got - want)
        r = np.abs(P.round_to(want, dtype) - want)
        res[name] = {"out_max_abs": float(err.max()),
                     "out_over_2e-3": int((err > P.FLAT_OUT).sum()),
                     "out_ref_torch_max_abs": float(r.max()),
                     "out_ref_torch_over_2e-3": int((r > P.FLAT_OUT).sum()),
                     "elements": int(err.size)}
        if got_lse is not None:
            res[name]["lse_max_abs"] = float(np.abs(P.f32(got_lse) - want_lse).max())
        print(name, res[name], flush=True)

    for geom in P.PROBE_GEOMS:
        for case in P.PROBE:
            q, k, v = P.probe_inputs(geom, case)
            scale = geom[2] ** -0.5
            for causal in (True, False):
                off = case[2] if causal else None
                o, lse = attn(q, k, v, scale, off)
                want, want_lse = ro.attn_with_lse(P.f32(q), P.f32(k), P.f32(v), scale, off)
                record(P.probe_name(geom, case, causal), o, lse, want, want_lse, geom[3])

    scale = P.D128 ** -0.5
    for c in P.FUSED:
        q, kp, vp, kl, vl = P.fused_inputs(c)
        tq, tpeer, tloc, off = c
        o, lse = ring(q, kp[:tpeer] if tpeer else None, vp[:tpeer] if tpeer else None,
                      kl[:tloc] if tloc else None, vl[:tloc] if tloc else None, scale, off)
        want, want_lse = P.fused_oracle(c, q, kp, vp, kl, vl)
        record(P.fused_name(c), o, lse, want, want_lse, torch.bfloat16)

    q, kp, vp, kl, vl = P.cfg0_inputs()
    o, lse = ring(q, kp, vp, kl, vl, scale, 0)
    want, want_lse = P.fused_oracle((1024, 1024, 1024, 0), q, kp, vp, kl, vl)
    record("cfg0", o, lse, want, want_lse, torch.bfloat16)

    for lens, peer in P.PAGED:
        b = P.paged_batch(lens, peer)
        outs = []
        for r, L in enumerate(lens):
            qs = int(b["qsl"][r])
            kl_r, vl_r = P.paged_local_kv(b, r)
            kp_r = b["kp"][r * peer:(r + 1) * peer] if peer else None
            vp_r = b["vp"][r * peer:(r + 1) * peer] if peer else None
            o, _ = ring(b["q"][qs:qs + L], kp_r, vp_r, kl_r, vl_r, scale, 0)
            outs.append(o)
        record(P.paged_name(lens, peer), torch.cat(outs), None, P.paged_oracle(b), None, torch.bfloat16)

    def decode_ref(q, pk, pv, cache, bt, seqs):
        outs, lses = [], []
        bs = cache.shape[2]
        d = cache.shape[3] // 2
        for row in seqs:
            qr, ps, pl, preq, ls, ll = (int(x) for x in row)
            kl = vl = None
            if ll:
                blocks = torch.as_tensor(bt[preq][: (ls + ll + bs - 1) // bs]).to(torch.int64).to(cache.device)
                kv = cache[blocks].permute(0, 2, 1, 3).reshape(-1, cache.shape[1], cache.shape[3])[ls:ls + ll]
                kl, vl = kv[..., :d], kv[..., d:]
            kp = pk[ps:ps + pl] if pl else None
            vp = pv[ps:ps + pl] if pl else None
            # a single decode query sees every local key: causal offset ll - 1
            o, lse = ring(q[qr:qr + 1], kp, vp, kl, vl, q.shape[2] ** -0.5, ll - 1)
            outs.append(o)
            lses.append(lse)
        return torch.cat(outs), torch.cat(lses, 1)

    for pl_, ll_, chunk in P.DECODE:
        q, pk, pv, cache, bt, seqs = P.decode_case(pl_, ll_)
        o, lse = decode_ref(q, pk, pv, cache, bt, seqs)
        want, want_lse = P.decode_oracle(q, pk, pv, cache, bt, seqs, scale)
        record(P.decode_name(pl_, ll_, chunk), o, lse, want, want_lse, torch.bfloat16)

    if not args.no_full:
        q, pk, pv, cache, bt, seqs = P.cfg2_inputs(dev)
        o, lse = decode_ref(q, pk, pv, cache, bt, seqs)
        want, want_lse = P.cfg2_oracle(q, pk, pv, cache, bt, seqs)
        record("cfg2", o, lse, want, want_lse, torch.bfloat16)
        del q, pk, pv, cache
        q, k, v = P.cfg3_inputs(dev)
        o, lse = ring_attn_with_lse(q, k, v, scale, 0)
        rows = P.cfg3_rows()
        want, want_lse = P.cfg3_oracle(q, k, v, rows)
        ri = torch.from_numpy(rows).to(dev)
        record("cfg3_n1", o[ri], lse[:, ri], want, want_lse, torch.bfloat16)

    meta = {"how": "reference Triton ring_attn_with_lse + vLLM merge_attn_states on these inputs, "
                   "max-abs vs the fp32 oracle",
            "device": torch.cuda.get_device_name(dev), "torch": torch.__version__}
    try:
        import triton
        meta["triton"] = triton.__version__
    except Exception:  # noqa: BLE001
        pass
    with open(args.out, "w") as f:
        json.dump({"meta": meta, "cases": res}, f, indent=1, sort_keys=True)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
