"""Worker for test_decode_ring_backend.py's two-GPU case: ``<rank> <port>``.

Rank 0 (GPU 0) is a decode-ring peer serving its prefix chunk; rank 1
(GPU 1) is the owner, calling ``HcpRingAttentionImpl.forward`` for two
registered decode-ring requests over three decode steps on the B200
kernels.  The ring is a standalone NCCL group over a TCPStore, as two vLLM
instances form it.  The owner prints one JSON line and exits non-zero on a
mismatch with the oracle (2e-3 + 2^-7 |ref|, bf16 output)."""

import json
import os
import sys
import types

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import parity as P  # noqa: E402  (this script's directory is on sys.path)
from oracle import ring_oracle as ro  # noqa: E402

H, HKV, D, LAYERS, BS = 28, 4, 128, 2, 16
PREFIX = 512                    # tokens held by the peer
OWN = (300, 457)                # each request's own prompt tokens
STEPS = 3


def data():
    g = torch.Generator().manual_seed(11)
    peer = [(torch.randn(PREFIX, HKV, D, generator=g).bfloat16(), torch.randn(PREFIX, HKV, D, generator=g).bfloat16())
            for _ in range(LAYERS)]
    own = [[(torch.randn(n, HKV, D, generator=g).bfloat16(), torch.randn(n, HKV, D, generator=g).bfloat16())
            for _ in range(LAYERS)] for n in OWN]
    tok = [[[(torch.randn(1, H, D, generator=g).bfloat16(), torch.randn(1, HKV, D, generator=g).bfloat16(),
              torch.randn(1, HKV, D, generator=g).bfloat16()) for _ in range(LAYERS)] for _ in OWN]
           for _ in range(STEPS)]
    return peer, own, tok


def main():
    rank, port = int(sys.argv[1]), int(sys.argv[2])
    from hcp_vllm_plugin_b200 import ring_backend as rb
    from hcp_vllm_plugin_b200.ring_decode import RingComm, RingDecode

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    comm = RingComm.standalone("127.0.0.1", port, rank, 2, backend="nccl", timeout_s=120, connect_timeout_s=120)
    ring = RingDecode(LAYERS, 2, max(PREFIX, *OWN) + STEPS, H, HKV, D, D ** -0.5, dev, comm=comm)
    peer, own, tok = data()
    if rank == 0:
        chunks = [(k.to(dev), v.to(dev)) for k, v in peer]
        ring.serve(lambda layer: chunks[layer], poll_s=0.5)
        torch.cuda.synchronize()
        comm.close()
        return 0 if ring.steps_served == STEPS else 1

    impl = rb.HcpRingAttentionImpl(H, D, D ** -0.5, HKV)
    nblk = [(PREFIX + n + STEPS + BS - 1) // BS for n in OWN]
    bt = torch.zeros(2, max(nblk), dtype=torch.int32)
    bt[0, :nblk[0]] = torch.arange(nblk[0])
    bt[1, :nblk[1]] = torch.arange(nblk[0], nblk[0] + nblk[1])
    caches = []
    for layer in range(LAYERS):
        c = torch.full((sum(nblk), HKV, BS, 2 * D), float("nan"), dtype=torch.bfloat16)
        for r, n in enumerate(OWN):
            pos = PREFIX + torch.arange(n)
            blk = bt[r, pos // BS].long()
            c[blk, :, pos % BS, :D] = own[r][layer][0]
            c[blk, :, pos % BS, D:] = own[r][layer][1]
        caches.append(c.to(dev))
    btd = bt.to(dev)
    for r in range(2):
        rb.register_decode_ring(int(bt[r, 0]), ring, slot=r, prefix_len=PREFIX)
    worst, ok = 0.0, True
    for t in range(STEPS):
        seq = [PREFIX + n + t + 1 for n in OWN]
        meta = types.SimpleNamespace(query_start_loc=torch.tensor([0, 1, 2], dtype=torch.int32, device=dev),
                                     seq_lens=torch.tensor(seq, dtype=torch.int32, device=dev), block_table=btd,
                                     num_actual_tokens=2)
        for layer in range(LAYERS):
            qq = torch.cat([tok[t][r][layer][0] for r in range(2)])
            kk = torch.cat([tok[t][r][layer][1] for r in range(2)])
            vv = torch.cat([tok[t][r][layer][2] for r in range(2)])
            out = torch.zeros(2, H, D, dtype=torch.bfloat16, device=dev)
            impl.forward(types.SimpleNamespace(layer_name=f"model.layers.{layer}.self_attn.attn"),
                         qq.to(dev), kk.to(dev), vv.to(dev), caches[layer], meta, out)
            got = out.float().cpu().numpy()
            for r in range(2):
                keys = torch.cat([peer[layer][0], own[r][layer][0]] + [tok[j][r][layer][1] for j in range(t + 1)])
                vals = torch.cat([peer[layer][1], own[r][layer][1]] + [tok[j][r][layer][2] for j in range(t + 1)])
                want, _ = ro.attn_with_lse(qq[r:r + 1].float().numpy(), keys.float().numpy(),
                                           vals.float().numpy(), D ** -0.5, None)
                try:
                    e = P.check_out(got[r], want[0], f"layer {layer} request {r}").err
                except AssertionError as ex:
                    print(ex, flush=True)
                    ok, e = False, float("inf")
                worst = max(worst, e)
    ring.stop()
    torch.cuda.synchronize()
    comm.close()
    growth = [ring.growth_positions[0][r] for r in range(2)]
    ok = ok and all(growth[r] == [PREFIX + n + t for t in range(STEPS) if (PREFIX + n + t) % 2 == 1]
                    for r, n in enumerate(OWN))
    print(json.dumps({"max_abs_out": worst, "growth": growth, "ok": ok}), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
