"""Forward-kernel outputs of the variant this process runs (``HCP_FWD_VARIANT``
is read once per process by the library), saved with ``torch.save`` to the
path given as the only argument, for ``test_fwd_variants_gpu.py`` to compare
between variants.

The cases launch many more 256-row blocks x heads than a B200 has SMs, so a
persistent kernel (variant 7) runs many blocks per CTA: a 16384-token and a
131072-token causal layer (1792 and 14336 blocks x heads), the configs[1]
paged batch with 1024-token peer prefixes (728), a two-hop chain whose second
hop merges into the first hop's fp32 (O, LSE) in its epilogue (448 each), and
a sliding-window causal layer (896)."""

from __future__ import annotations

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

H, HKV, D = 28, 4, 128


def main(path: str) -> None:
    import parity as P
    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops

    dev = torch.device("cuda:0")
    scale = D ** -0.5
    res = {}

    def rnd(g, *shape):  # seeded on the device: the same inputs in every process
        return torch.randn(*shape, generator=g, device=dev, dtype=torch.bfloat16)

    for seq in (16384, 131072):
        g = torch.Generator(device=dev).manual_seed(seq)
        q, k, v = rnd(g, seq, H, D), rnd(g, seq, HKV, D), rnd(g, seq, HKV, D)
        out = torch.empty_like(q)
        lse = torch.empty(H, seq, dtype=torch.float32, device=dev)
        work = ops.make_work([(0, seq, 0, 0, (C.HCP_SRC_A, 0, seq, 0), None)])
        ops.ring_attn_fwd(q, work, scale=scale, num_kv_heads=HKV, out=out, lse=lse, k_a=k, v_a=v)
        # the 131072-token output as every 8th 256-row block (blocks of
        # every round of a persistent CTA), plus the whole LSE
        res[f"causal{seq}"] = (out.view(-1, 256, H, D)[::8].cpu() if seq > 16384 else out.cpu(), lse.cpu())
        del q, k, v, out, lse

    lens, peer = (512, 1024, 2048, 3072), 1024
    b = P.paged_batch(lens, peer)
    items = []
    for r, L in enumerate(lens):
        items.append((int(b["qsl"][r]), L, r, int(b["qsl"][r]), (C.HCP_SRC_A, r * peer, peer, -1),
                      (C.HCP_SRC_PAGED, peer, L, 0)))
    q = b["q"].to(dev)
    out = torch.empty_like(q)
    lse = torch.empty(H, q.shape[0], dtype=torch.float32, device=dev)
    ops.ring_attn_fwd(q, ops.make_work(items), scale=scale, num_kv_heads=HKV, out=out, lse=lse,
                      k_a=b["kp"].to(dev), v_a=b["vp"].to(dev), kv_cache=b["cache"].to(dev),
                      block_table=torch.from_numpy(b["bt"]).to(dev))
    res["paged_cfg1"] = (out.cpu(), lse.cpu())

    g = torch.Generator(device=dev).manual_seed(7)
    tq, t1 = 4096, 3000
    q, k1, v1 = rnd(g, tq, H, D), rnd(g, t1, HKV, D), rnd(g, t1, HKV, D)
    k2, v2 = rnd(g, tq, HKV, D), rnd(g, tq, HKV, D)
    acc = torch.empty(tq, H, D, dtype=torch.float32, device=dev)
    lse1 = torch.empty(H, tq, dtype=torch.float32, device=dev)
    ops.ring_attn_fwd(q, ops.make_work([(0, tq, 0, 0, (C.HCP_SRC_A, 0, t1, -1), None)]), scale=scale,
                      num_kv_heads=HKV, out=acc, lse=lse1, k_a=k1, v_a=v1)
    out = torch.empty(tq, H, D, dtype=torch.bfloat16, device=dev)
    lse2 = torch.empty_like(lse1)
    ops.ring_attn_fwd(q, ops.make_work([(0, tq, 0, 0, (C.HCP_SRC_A, 0, tq, 0), None)]), scale=scale,
                      num_kv_heads=HKV, out=out, lse=lse2, k_a=k2, v_a=v2, merge_o=acc, merge_lse=lse1)
    res["merge_hop1"] = (acc.cpu(), lse1.cpu())
    res["merge_hop2"] = (out.cpu(), lse2.cpu())

    g = torch.Generator(device=dev).manual_seed(9)
    seq = 8192
    q, k, v = rnd(g, seq, H, D), rnd(g, seq, HKV, D), rnd(g, seq, HKV, D)
    out, lse = ops.ring_attn_with_lse(q, k, v, scale, 0, window=3000)
    res["window8192"] = (out.cpu(), lse.cpu())

    torch.cuda.synchronize()
    assert C.device_status() == 0, f"device status {C.device_status():#x}"
    torch.save(res, path)
    print("saved", len(res), "cases")


if __name__ == "__main__":
    main(sys.argv[1])
