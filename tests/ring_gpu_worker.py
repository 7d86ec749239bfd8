"""Worker for test_ring_multi_gpu.py (run under torchrun, one rank per GPU).

Each rank runs RingPrefill.forward on its contiguous chunk of a seeded
sequence, once per transport (copy-engine pulls from exported outboxes, and
NCCL send/recv); rank 0 gathers the chunks and compares them with the
single-GPU fused kernel over the whole sequence and with the CPU oracle on
sampled rows (the bar of tests/parity.py).  Three layers run back to back
with V scaled by 3, 2 and 1, so a chunk pulled from an outbox a layer too
early or too late (the outboxes alternate by layer parity) shows up in the
last layer's output.  Prints one JSON line per transport on rank 0 and exits
non-zero on mismatch.
"""

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from hcp_vllm_plugin_b200 import _capi, ops  # noqa: E402
from hcp_vllm_plugin_b200.ring_runner import RingPrefill  # noqa: E402
import parity as P  # noqa: E402  (this script's directory is on sys.path)
from oracle import ring_oracle as ro  # noqa: E402

H, HKV, D = 28, 4, 128


def main():
    seq = int(sys.argv[1]) if len(sys.argv) > 1 else 16384
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(seq, H, D, generator=g).bfloat16()
    k = torch.randn(seq, HKV, D, generator=g).bfloat16()
    v = torch.randn(seq, HKV, D, generator=g).bfloat16()
    ok = True
    full = None
    for transport in ("ce", "p2p"):
        runner = RingPrefill(seq, H, HKV, D, D ** -0.5, dev, transport=transport)
        c = runner.chunk
        sl = slice(rank * c, (rank + 1) * c)
        out = torch.empty(c, H, D, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(H, c, dtype=torch.float32, device=dev)
        qd, kd, vd = q[sl].to(dev), k[sl].to(dev), v[sl].to(dev)
        layers = [(qd, kd, (vd.float() * sc).bfloat16()) for sc in (3.0, 2.0)] + [(qd, kd, vd)]
        for ql, kl, vl in layers:  # buffers and outboxes are reused across layers
            runner.forward(ql, kl, vl, out, lse)
        torch.cuda.synchronize()
        runner.close()
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        lses = [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(lses, lse)
        if rank == 0:
            if full is None:
                full = ops.ring_attn_with_lse(q.to(dev), k.to(dev), v.to(dev), D ** -0.5, 0)
            full_o, full_lse = full
            got = torch.cat(outs).float().cpu().numpy()
            got_lse = torch.cat(lses, 1).cpu().numpy()
            single = full_o.float().cpu().numpy()
            # against the one-GPU launch over the whole sequence: equal or one bf16 step apart
            step = P.step_of(single, torch.bfloat16)
            d = np.abs(got - single)
            steps_ok = bool((d <= np.maximum(2e-3, step * 1.0001)).all())
            # against the oracle, on sampled rows (chunk edges included): the parity bar
            rows = np.unique(np.r_[np.linspace(0, seq - 1, 24).astype(int), [c - 1, c, seq - 1]])
            qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
            want = np.empty((len(rows), H, D), np.float32)
            want_lse = np.empty((H, len(rows)), np.float32)
            for i, r in enumerate(rows):
                o, l = ro.attn_with_lse(qf[r:r + 1], kf[: r + 1], vf[: r + 1], D ** -0.5, int(r))
                want[i], want_lse[:, i] = o[0], l[:, 0]
            try:
                st = P.check_out(got[rows], want, f"ring N={world} {transport} sampled rows")
                P.check_lse(got_lse[:, rows], want_lse, f"ring N={world} {transport}")
                oracle_ok, line = True, st.line()
            except AssertionError as e:
                oracle_ok, line = False, str(e)
            res = {"world": world, "seq": seq, "transport": transport, "give": runner.plan.give,
                   "max_vs_single_gpu": float(d.max()), "within_one_step_of_single_gpu": steps_ok,
                   "lse_max_vs_single_gpu": float(np.abs(got_lse - full_lse.cpu().numpy()).max()),
                   "oracle": line, "device_status": _capi.device_status()}
            ok = ok and steps_ok and oracle_ok and res["lse_max_vs_single_gpu"] <= 1e-3 \
                and res["device_status"] == 0
            print(json.dumps(res), flush=True)
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier(device_ids=[local])
    dist.destroy_process_group()
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
