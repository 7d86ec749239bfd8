"""Worker for test_ring_decode_gpu.py (run under torchrun, one rank per GPU).

Each rank holds its contiguous prefix chunk of every request (seeded, the
same data on every rank) and runs RingDecode.step over NCCL for a few decode
steps of two layers; the owner compares every output with the CPU oracle's
attention over all keys so far, and every rank checks that it holds exactly
its round-robin share of the decode tokens.  Prints one JSON line on the
owner and exits non-zero on mismatch.
"""

import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from hcp_vllm_plugin_b200.ring_decode import RingDecode  # noqa: E402
from oracle import ring_oracle as ro  # noqa: E402

H, HKV, D, LAYERS, STEPS = 28, 4, 128, 2, 5
CHUNKS = (1024, 640, 2048)  # per-rank prefix rows of each request


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    g = torch.Generator().manual_seed(0)
    B = len(CHUNKS)
    total = [c * world + STEPS for c in CHUNKS]
    ks = [[torch.randn(t, HKV, D, generator=g).bfloat16() for t in total] for _ in range(LAYERS)]
    vs = [[torch.randn(t, HKV, D, generator=g).bfloat16() for t in total] for _ in range(LAYERS)]
    qs = [[torch.randn(B, H, D, generator=g).bfloat16() for _ in range(STEPS)] for _ in range(LAYERS)]
    rd = RingDecode(LAYERS, B, max(CHUNKS) + STEPS, H, HKV, D, D ** -0.5, dev)
    for layer in range(LAYERS):
        for b, c in enumerate(CHUNKS):
            sl = slice(rank * c, (rank + 1) * c)
            rd.set_chunk(layer, b, ks[layer][b][sl].to(dev), vs[layer][b][sl].to(dev))
    worst = worst_lse = 0.0
    out = torch.empty(B, H, D, dtype=torch.float32, device=dev)
    out_lse = torch.empty(H, B, dtype=torch.float32, device=dev)
    for t in range(STEPS):
        pos = [c * world + t for c in CHUNKS]
        for layer in range(LAYERS):
            if rank == rd.owner:
                k_new = torch.stack([ks[layer][b][pos[b]] for b in range(B)]).to(dev)
                v_new = torch.stack([vs[layer][b][pos[b]] for b in range(B)]).to(dev)
                rd.step(layer, pos, qs[layer][t].to(dev), k_new, v_new, out, out_lse)
                got, got_lse = out.cpu().numpy(), out_lse.cpu().numpy()
                for b in range(B):
                    want, want_lse = ro.attn_with_lse(qs[layer][t][b:b + 1].float().numpy(),
                                                      ks[layer][b][:pos[b] + 1].float().numpy(),
                                                      vs[layer][b][:pos[b] + 1].float().numpy(), D ** -0.5, None)
                    worst = max(worst, float(np.abs(got[b] - want[0]).max()))
                    worst_lse = max(worst_lse, float(np.abs(got_lse[:, b] - want_lse[:, 0]).max()))
            else:
                rd.step(layer, pos)
    torch.cuda.synchronize()
    growth_ok = all(rd.growth_positions[layer][b] == [c * world + t for t in range(STEPS)
                                                       if (c * world + t) % world == rank]
                    for layer in range(LAYERS) for b, c in enumerate(CHUNKS))
    flags = torch.tensor([int(growth_ok)], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    ok = bool(flags.item())
    if rank == rd.owner:
        ok = ok and worst < 2e-3 and worst_lse < 1e-3
        print(json.dumps({"world": world, "max_abs_out": worst, "max_abs_lse": worst_lse,
                          "growth_round_robin": bool(flags.item()), "ok": ok}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
