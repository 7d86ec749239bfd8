"""Ring context-parallel prefill benchmark.

One step = the attention of all 28 layers of a 131072-token sequence split
into N contiguous chunks, one per GPU (Qwen2.5-7B attention geometry: 28
query heads, 4 KV heads, head_dim 128, bf16, seeded N(0,1) synthetic q/k/v,
one set per layer).  Each rank durably holds only its own chunk; peer K/V
rotate over NVLink every layer (``hcp_vllm_plugin_b200.ring_runner``).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --rows            # the connector / decode-ring rows (opt-in)

Prints one JSON line on rank 0.  ``value`` is whole-job tokens/s measured on
the device (CUDA events, barrier + synchronize around the timed steps, max
over ranks).  ``e2e`` repeats the measurement through the public API with
every layer's q/k/v copied from pinned host memory and the output copied
back.  ``--impl reference`` times the reference's own fp32 torch attention
(``_attn_with_lse`` from the installed reference package, else the oracle's
numpy restatement of it) on the host cores over a bounded sample of the same
step and extrapolates by FLOPs (``"extrapolated": true``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ring-attn TFLOP/s (% bf16 peak); 128k ring-prefill tok/s at 1/2/4/8 B200"
H, HKV, D = 28, 4, 128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def causal_pairs(n: int) -> int:
    return n * (n + 1) // 2


def step_flops(seq: int, layers: int) -> float:
    return 4.0 * D * H * causal_pairs(seq) * layers


def profile_traffic():
    """DRAM bytes per launch of the ring-attention kernel from the committed
    ncu summary (profiles/ring_fwd_traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "ring_fwd_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"hcp_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _reference_attn():
    """The reference plugin's own fp32 torch ``_attn_with_lse``
    (``hcp_vllm_plugin/ring_backend.py:366-406``) from ``baseline/_ref``, or
    None when the package is not installed there."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "hcp_vllm_plugin")):
        return None
    if ref not in sys.path:
        sys.path.append(ref)
    try:
        from hcp_vllm_plugin.ring_backend import _attn_with_lse
    except Exception:  # noqa: BLE001 - fall back to the port
        return None
    return _attn_with_lse


REF_BLOCK = 128


def cpu_rows(args) -> int:
    """Query rows of one CPU sample: the reference's torch path reaches its
    steady rate only in blocks of 128 rows, the port in 32-row blocks."""
    if args.cpu_rows:
        return args.cpu_rows
    return 2 * REF_BLOCK if _reference_attn() is not None else 448


def cpu_sample(seq: int, rows: int, seed: int = 0):
    """Time the reference's CPU path on the last ``rows`` query rows of one
    layer (each sees ~``seq`` keys): its own ``_attn_with_lse`` on the host
    cores when installed (kind "reference"), else the oracle's numpy
    restatement of it (kind "port").  Rows go 128 (32 for the port) at a
    time, since the reference materialises the [H, rows, keys] fp32 scores
    (1.9 GB at 128 rows x 128k keys).  Returns (seconds, flops of the sample,
    threads, kind)."""
    import numpy as np

    rng = np.random.default_rng(seed)
    q = rng.standard_normal((rows, H, D), dtype=np.float32)
    k = rng.standard_normal((seq, HKV, D), dtype=np.float32)
    v = rng.standard_normal((seq, HKV, D), dtype=np.float32)
    flops = 4.0 * D * H * sum(seq - rows + i + 1 for i in range(rows))
    attn = _reference_attn()
    if attn is not None:
        import torch

        qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
        t0 = time.perf_counter()
        for r0 in range(0, rows, REF_BLOCK):
            attn(qt[r0:r0 + REF_BLOCK], kt, vt, D ** -0.5, seq - rows + r0)
        return time.perf_counter() - t0, flops, torch.get_num_threads(), "reference"
    from oracle import ring_oracle as ro

    q, k, v = ro.round_bf16(q), ro.round_bf16(k), ro.round_bf16(v)
    t0 = time.perf_counter()
    ro.attn_with_lse(q, k, v, D ** -0.5, seq - rows, q_block=min(rows, 32))  # ~0.5 GB of scores at a time
    dt = time.perf_counter() - t0
    try:
        from threadpoolctl import threadpool_info
        threads = max([x.get("num_threads", 1) for x in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        threads = os.cpu_count() or 1
    return dt, flops, threads, "port"


def _sample_text(kind: str, rows: int, seq: int, layers: int, secs: float) -> str:
    what = ("the reference's own fp32 torch _attn_with_lse (ring_backend.py:366-406)" if kind == "reference"
            else "fp32 numpy oracle port of ring_backend.py:366-406")
    return (f"one layer, last {rows} query rows x {seq} keys causal, 28 heads, {what}: {secs:.2f} s, "
            f"extrapolated by FLOPs to the whole {seq}-token x {layers}-layer step")


def run_reference(args, rank):
    if rank != 0:
        return
    seq, layers = args.seq, args.layers
    rows = cpu_rows(args)
    total = step_flops(seq, layers)
    for _ in range(args.warmup):  # untimed: first-touch of the ~8 GB of fp32 buffers, BLAS threads
        cpu_sample(seq, min(rows, REF_BLOCK))
    rates, secs = [], []
    threads, kind = 1, "port"
    for _ in range(args.steps):
        dt, fl, threads, kind = cpu_sample(seq, rows)
        rates.append(fl / dt)
        secs.append(dt)
    rate = statistics.median(rates)
    tok_s = seq / (total / rate)
    line = {
        "impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / rate, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(args), "tflops": rate / 1e12,
        "extrapolated": True, "sample_seconds": secs,
        "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": _sample_text(kind, rows, seq, layers, statistics.median(secs))},
        "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config(args):
    return {"workload": "cfg3 ring CP prefill, attention only", "seq_len": args.seq,
            "layers": args.layers, "heads": H, "kv_heads": HKV, "head_dim": D,
            "chunk_per_gpu": args.seq // max(1, args.gpus), "parallelism": f"cp{args.gpus}",
            "global_batch": 1, "l2": "inputs larger than L2 (q 0.94 GB/layer at N=1)",
            "schedule": "balanced pairs" if not args.no_balance else "plain ring",
            "transport": args.ring_transport if args.gpus > 1 else "none"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--cpu-rows", type=int, default=0)  # 0: 256 (reference) / 448 (port), ~10 s each
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-balance", action="store_true")
    ap.add_argument("--no-side", action="store_true")
    ap.add_argument("--ring-transport", choices=["ce", "p2p"], default="ce",
                    help="how chunks move between ranks: copy-engine pulls (default) or NCCL send/recv")
    ap.add_argument("--kernel", choices=["fwd", "decode"], default=None,
                    help="profiling mode: time one kernel on a small case and exit")
    ap.add_argument("--decode-seqs", type=int, default=16)
    ap.add_argument("--iters", type=int, default=1, help="timed launches in --kernel mode")
    ap.add_argument("--rows", action="store_true",
                    help="measure the connector / decode-ring rows instead of the headline")
    ap.add_argument("--ref-gpu", action="store_true",
                    help="time the reference plugin's own B200 path beside this library and exit")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.kernel is not None:
        run_kernel(args)
        return
    if args.rows:
        run_rows(args, world, rank, local_rank)
        return
    if args.ref_gpu:
        import torch
        dev = torch.device("cuda", local_rank)
        torch.cuda.set_device(dev)
        print(json.dumps({"reference_b200": reference_gpu_side(dev, peaks()[0])}), flush=True)
        return

    import datetime

    import torch
    import torch.distributed as dist

    from hcp_vllm_plugin_b200 import _capi
    from hcp_vllm_plugin_b200.ring_runner import RingPrefill

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        # NCCL on high-priority streams: a chunk's send/recv kernels take the
        # first free SM instead of queueing behind attention CTAs
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev, pg_options=opts)
    _capi.load()
    seq, L = args.seq, args.layers
    chunk = seq // world
    scale = D ** -0.5
    runner = RingPrefill(seq, H, HKV, D, scale, dev, balance=not args.no_balance,
                         transport=args.ring_transport if world > 1 else None)

    # resident per-layer inputs of this rank's chunk (seeded)
    qs, ks, vs = [], [], []
    for layer in range(L):
        g = torch.Generator(device=dev).manual_seed(1000 * layer + 17)
        # generate the full layer's rows deterministically, keep this rank's chunk
        q = torch.empty(chunk, H, D, dtype=torch.bfloat16, device=dev)
        k = torch.empty(chunk, HKV, D, dtype=torch.bfloat16, device=dev)
        v = torch.empty(chunk, HKV, D, dtype=torch.bfloat16, device=dev)
        g.manual_seed(1000 * layer + 17 + 7919 * rank)
        q.normal_(generator=g)
        k.normal_(generator=g)
        v.normal_(generator=g)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    out = torch.empty(chunk, H, D, dtype=torch.bfloat16, device=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        for layer in range(L):
            runner.forward(qs[layer], ks[layer], vs[layer], out)
    _capi.check(0, "warmup")
    barrier()

    clocks = ClockSampler(local_rank)
    clocks.start()
    stream = torch.cuda.current_stream(dev)
    ev_layer = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps * L)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    launches0 = runner.launches
    barrier()
    t_start.record(stream)
    i = 0
    for _ in range(args.steps):
        for layer in range(L):
            ev_layer[i][0].record(stream)
            runner.forward(qs[layer], ks[layer], vs[layer], out)
            ev_layer[i][1].record(stream)
            i += 1
    t_end.record(stream)
    barrier()
    clk = clocks.stop()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))
    launches = runner.launches - launches0
    layer_ms = [a.elapsed_time(b) for a, b in ev_layer]
    status = _capi.device_status()
    if status != 0:
        raise SystemExit(f"device reported failure {status:#x}")

    value = seq * args.steps / (elapsed_ms / 1e3)
    total_flops = step_flops(seq, L) * args.steps
    tflops = total_flops / (elapsed_ms / 1e3) / 1e12
    pk, pk_kind = peaks()
    peak_tf = pk["bf16_tflops_sustained"]
    # roofline of the dominant kernel: at N=1 each layer is exactly one launch
    # of the ring-attention kernel; its algorithmic FLOPs are the causal pairs.
    mean_layer_ms = statistics.mean(layer_ms)
    my_flops_layer = step_flops(seq, 1) if world == 1 else (
        4.0 * D * H * runner.chunk * runner.chunk * runner.plan.work_units(rank))
    achieved = my_flops_layer / (mean_layer_ms / 1e3) / 1e12
    traffic = profile_traffic()
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
            "frac": achieved / peak_tf,
            "peak_source": f"bf16_tflops_sustained ({pk_kind})",
            "traffic": None if traffic is None else traffic.get("bytes_per_launch_cfg3_n1"),
            "kernel": "ring_fwd_kernel<128,bf16>",
            "per_launch_ms": mean_layer_ms if world == 1 else None}

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, runner, dev, chunk, L, barrier, max_over_ranks, world)

    side = side_configs(dev, pk) if (world == 1 and not args.no_side) else None
    if not args.no_side:
        # the decode ring's step on the same ranks (collective: every rank);
        # reported beside the headline, so a failure is recorded, not raised
        try:
            ring_dec = decode_ring_step(world, rank, dev, pk, torch.Generator(device=dev).manual_seed(5),
                                        barrier)
        except Exception as e:  # noqa: BLE001 - reported in the line
            ring_dec = {"error": repr(e)[-300:]}
        side = dict(side or {}, decode_ring_step=ring_dec)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu_sample(seq, min(cpu_rows(args), REF_BLOCK))  # untimed first touch
        dt, fl, threads, kind = cpu_sample(seq, cpu_rows(args))
        rate = fl / dt
        cpu = {"value": seq / (step_flops(seq, L) / rate), "unit": "tok/s", "cores": threads,
               "kind": kind, "extrapolated": True,
               "sample": _sample_text(kind, cpu_rows(args), seq, L, dt)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v per layer)", "config": config(args),
            "tflops": tflops, "pct_bf16_peak": 100.0 * tflops / (peak_tf * world),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk,
            "other_configs": side,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def side_configs(dev, pk):
    """Device-timed BASELINE configs[1] (paged continuous-batch prefill) and
    configs[2] (split-KV decode), reported beside the headline at N=1."""
    import numpy as np
    import torch

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops

    res = {}
    g = torch.Generator(device=dev).manual_seed(3)
    scale = D ** -0.5

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    # ---- 4 requests, local {512,1024,2048,3072} + 1024 peer each
    lens, peer, bs = [512, 1024, 2048, 3072], 1024, 16
    nbl = [(peer + L) // bs for L in lens]
    num_blocks = sum(nbl)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(1)).to(torch.int32)
    bt = torch.zeros(len(lens), max(nbl), dtype=torch.int32)
    o = 0
    for r, n in enumerate(nbl):
        bt[r, :n] = perm[o:o + n]
        o += n
    bt = bt.to(dev)
    cache = torch.empty(num_blocks, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    qsl = np.concatenate([[0], np.cumsum(lens)])
    q1 = torch.empty(int(qsl[-1]), H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    kp = torch.empty(len(lens) * peer, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vp = torch.empty_like(kp).normal_(generator=g)
    out1 = torch.empty_like(q1)
    work = ops.make_work([(int(qsl[r]), L, r, int(qsl[r]), (C.HCP_SRC_A, r * peer, peer, -1),
                           (C.HCP_SRC_PAGED, peer, L, 0)) for r, L in enumerate(lens)])
    ms1 = timed(lambda: ops.ring_attn_fwd(q1, work, scale=scale, num_kv_heads=HKV, out=out1, k_a=kp,
                                          v_a=vp, kv_cache=cache, block_table=bt))
    fl1 = 4.0 * D * H * sum(L * (L + 1) // 2 + peer * L for L in lens)
    res["cfg1_batch_prefill"] = {"ms": ms1, "tflops": fl1 / ms1 / 1e9,
                                 "frac_of_bf16_burst": fl1 / ms1 / 1e9 / pk["bf16_tflops"]}
    del cache, q1, kp, vp, out1

    # ---- 64 x (32768 paged local + 32768 peer) single-token decode
    B, LOC, PEER = 64, 32768, 32768
    nb = LOC // bs
    cache = torch.empty(B * nb, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    pk2 = torch.empty(B * PEER, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    pv2 = torch.empty_like(pk2).normal_(generator=g)
    bt2 = torch.randperm(B * nb, generator=torch.Generator().manual_seed(2)).to(torch.int32).view(B, nb).to(dev)
    q2 = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    out2 = torch.empty_like(q2)
    seqs = np.array([(b, b * PEER, PEER, b, 0, LOC) for b in range(B)], np.int32)
    ms2 = timed(lambda: ops.decode_splitkv(q2, seqs, scale=scale, num_kv_heads=HKV, out=out2, peer_k=pk2,
                                           peer_v=pv2, kv_cache=cache, block_table=bt2))
    byts = B * (LOC + PEER) * HKV * D * 2 * 2
    res["cfg2_splitkv_decode"] = {"ms": ms2, "gbs": byts / ms2 / 1e6, "algorithmic_bytes": byts,
                                  "frac_of_hbm": byts / ms2 / 1e6 / pk["hbm_gbs"]}
    try:
        res["fwd_issuer_variants_16k_causal"] = fwd_issuer_variants(16384)
    except Exception as e:  # noqa: BLE001 - reported in the line
        res["fwd_issuer_variants_16k_causal"] = {"error": repr(e)[-300:]}
    try:
        res["reference_b200"] = reference_gpu_side(dev, pk)
    except Exception as e:  # noqa: BLE001 - reported in the line
        res["reference_b200"] = {"error": repr(e)[-300:]}
    return res


REF_PKG = os.path.join(ROOT, "baseline", "_ref")  # the reference plugin, installed unmodified


def reference_gpu_side(dev, pk) -> dict:
    """The reference plugin's own B200 path, timed beside this library on the
    same inputs (CUDA events, 3 warm-up calls, so Triton's JIT compile is
    outside the timed region):

    * ``fwd_16k_causal``: its Triton ``ring_attn_with_lse``
      (``ring_triton_attn.py:155-207``) on one 16384-token causal launch, vs
      ``hcp_ring_attn_fwd`` on the same q/k/v;
    * ``cfg0``: BASELINE configs[0] - its local pass + peer pass + vLLM
      ``merge_attn_states`` (``ring_backend.py:819-832``), vs one fused launch;
    * ``cfg1_plugin_forward_28_layers``: BASELINE configs[1] through each
      plugin's ``HcpRingAttentionImpl.forward`` for a 28-layer engine step (one
      metadata object per step, 28 layers with their own paged caches and
      staged 1024-token peer chunks per request): the reference's per-request
      loop (gather, two Triton passes, merge) vs this backend (one host sync
      per step, one launch per layer).

    The reference is imported unmodified from ``baseline/_ref``."""
    import types

    import torch

    if not os.path.isdir(os.path.join(REF_PKG, "hcp_vllm_plugin")):
        return {"unavailable": "reference package not installed under baseline/_ref"}
    if REF_PKG not in sys.path:
        sys.path.append(REF_PKG)
    from hcp_vllm_plugin import ring_backend as ref_rb  # the reference's own code
    from hcp_vllm_plugin.ring_triton_attn import ring_attn_with_lse as ref_attn
    from vllm.v1.attention.ops.merge_attn_states import merge_attn_states

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops
    from hcp_vllm_plugin_b200 import ring_backend as our_rb

    res: dict = {}
    scale = D ** -0.5
    g = torch.Generator(device=dev).manual_seed(41)

    def timed(fn, n=5):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    def pair(name, fl, ref_fn, our_fn, n=5):
        try:
            ms_ref = timed(ref_fn, n)
            ms_our = timed(our_fn, n)
            res[name] = {"ref_ms": ms_ref, "ours_ms": ms_our, "speedup": ms_ref / ms_our,
                         "ref_tflops": fl / ms_ref / 1e9, "ours_tflops": fl / ms_our / 1e9}
        except Exception as e:  # noqa: BLE001 - reported in the line
            res[name] = {"error": repr(e)[-300:]}

    # ---- one 16384-token causal launch
    s = 16384
    q = torch.empty(s, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    k = torch.empty(s, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    v = torch.empty_like(k).normal_(generator=g)
    out = torch.empty_like(q)
    work = ops.make_work([(0, s, 0, 0, (C.HCP_SRC_A, 0, s, 0), None)])
    pair("fwd_16k_causal", 4.0 * D * H * causal_pairs(s),
         lambda: ref_attn(q, k, v, scale, 0),
         lambda: ops.ring_attn_fwd(q, work, scale=scale, num_kv_heads=HKV, out=out, k_a=k, v_a=v))
    del q, k, v, out

    # ---- local 1024 causal + peer 1024 non-causal + merge
    t = 1024
    q = torch.empty(t, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    kl, vl, kp, vp = (torch.empty(t, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
                      for _ in range(4))
    out = torch.empty_like(q)

    def ref_cfg0():
        o_loc, lse_loc = ref_attn(q, kl, vl, scale, 0)
        o_peer, lse_peer = ref_attn(q, kp, vp, scale, None)
        merged = torch.empty_like(o_loc)
        merge_attn_states(merged, o_peer, lse_peer, o_loc, lse_loc)
        return merged
    w0 = ops.make_work([(0, t, 0, 0, (C.HCP_SRC_A, 0, t, -1), (C.HCP_SRC_B, 0, t, 0))])
    pair("cfg0", 4.0 * D * H * (t * (t + 1) // 2 + t * t), ref_cfg0,
         lambda: ops.ring_attn_fwd(q, w0, scale=scale, num_kv_heads=HKV, out=out, k_a=kp, v_a=vp,
                                   k_b=kl, v_b=vl), n=20)
    del q, kl, vl, kp, vp, out

    # ---- configs[1] through both plugins' forward, a 28-layer step
    try:
        lens, peer, bs, layers = [512, 1024, 2048, 3072], 1024, 16, 28
        nbl = [(peer + L) // bs for L in lens]
        nb = sum(nbl)
        perm = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).to(torch.int32)
        bt = torch.zeros(len(lens), max(nbl), dtype=torch.int32)
        o = 0
        for r, n in enumerate(nbl):
            bt[r, :n] = perm[o:o + n]
            o += n
        bt = bt.to(dev)
        ntok = sum(lens)
        qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=dev)
        seq_lens = torch.tensor([peer + L for L in lens], dtype=torch.int32, device=dev)
        names = [f"model.layers.{i}.self_attn.attn" for i in range(layers)]
        caches = [torch.empty(nb, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
                  for _ in names]
        # the reference's own layout [nb, 2, bs, Hkv, D], same values
        ref_caches = [c.view(nb, HKV, bs, 2, D).permute(0, 3, 2, 1, 4).contiguous() for c in caches]
        qs = [torch.empty(ntok, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in names]
        out = torch.empty(ntok, H, D, dtype=torch.bfloat16, device=dev)
        for mod in (ref_rb, our_rb):
            mod.clear_peer_kv()
        for r in range(len(lens)):
            ck = f"bench_req{r}"
            for nm in names:
                kpr = torch.empty(peer, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
                vpr = torch.empty_like(kpr).normal_(generator=g)
                ref_rb.stage_peer_kv(ck, nm, kpr, vpr)
                our_rb.stage_peer_kv(ck, nm, kpr, vpr)
            fb = int(bt[r, 0])
            ref_rb.map_request_peer(fb, [ck])
            our_rb.map_request_peer(fb, [ck])
        layer_objs = [types.SimpleNamespace(layer_name=nm) for nm in names]

        def meta():  # a fresh metadata object per engine step
            return types.SimpleNamespace(num_actual_tokens=ntok, query_start_loc=qsl, seq_lens=seq_lens,
                                         block_table=bt)
        ref_impl = ref_rb.HcpRingAttentionImpl(H, D, scale, HKV)
        our_impl = our_rb.HcpRingAttentionImpl(H, D, scale, HKV)

        def ref_step():
            m = meta()
            for i in range(layers):
                ref_impl.forward(layer_objs[i], qs[i], None, None, ref_caches[i], m, out)

        def our_step():
            m = meta()
            for i in range(layers):
                our_impl.forward(layer_objs[i], qs[i], None, None, caches[i], m, out)
        our_rb.reset_impl_stats()
        fl = layers * 4.0 * D * H * sum(L * (L + 1) // 2 + peer * L for L in lens)
        pair("cfg1_plugin_forward_28_layers", fl, ref_step, our_step, n=3)
        res["cfg1_plugin_forward_28_layers"]["ours_peer_concat"] = our_rb.IMPL_STATS["peer_concat"]
        res["cfg1_plugin_forward_28_layers"]["ref_impl_stats"] = dict(ref_rb.IMPL_STATS)
    except Exception as e:  # noqa: BLE001 - reported in the line
        res["cfg1_plugin_forward_28_layers"] = {"error": repr(e)[-300:]}
    finally:
        for mod in (ref_rb, our_rb):
            mod.clear_peer_kv()
    return res


def fwd_issuer_variants(seq: int) -> dict:
    """The forward kernel on one ``seq``-token causal launch in each variant
    (``HCP_FWD_VARIANT``): 0 the mbarrier MMA issuer on 320 threads, 1 the
    named-barrier issuer, 2 variant 1 with a quarter of the exponentials on
    the FMA pipe, 3-5 the mbarrier issuer on 384 threads with setmaxnreg
    register split and packed f32x2 softmax math, with 1/4, 3/8 and none of
    the exponentials on the FMA pipe (5 is the default), 6 the named-barrier
    issuer on 384 threads with the setmaxnreg split, 7 variant 5 as a
    persistent kernel (one CTA per SM over a static list of 256-row blocks).
    Each runs in a fresh process, since the library reads the switch once
    per process.  Reported beside the headline only."""
    out = {}
    names = ("mbarrier_issuer", "named_barrier_issuer", "named_barrier_poly_exp2",
             "wide_poly_quarter", "wide_poly_three_eighths", "wide_no_poly", "named_barrier_wide",
             "wide_persistent")
    for variant, name in enumerate(names):
        env = dict(os.environ, HCP_FWD_VARIANT=str(variant))
        cmd = [sys.executable, os.path.abspath(__file__), "--kernel", "fwd", "--seq", str(seq), "--iters", "5"]
        try:
            r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=180)
        except subprocess.TimeoutExpired:
            out[name] = {"error": "timeout"}
            continue
        line = [x for x in r.stdout.splitlines() if x.startswith("kernel=")]
        if r.returncode != 0 or not line:
            out[name] = {"error": (r.stdout + r.stderr)[-300:]}
            continue
        kv = dict(f.split("=", 1) for f in line[-1].split()[1:])
        out[name] = {"ms": float(kv["ms"]), "tflops": float(kv["TFLOP/s"]),
                     "device_status": int(kv["device_status"])}
    return out


def run_kernel(args):
    """Profiling mode (`--kernel fwd|decode`): a few launches of one kernel on
    a small case, timed with CUDA events; prints one line, no JSON.

    fwd:    one causal `--seq` x `--seq` layer on contiguous q/k/v (configs[3]
            at a single-launch size);
    decode: `--decode-seqs` sequences of 32768 paged + 32768 peer keys
            (configs[2] has 64)."""
    import numpy as np
    import torch

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops

    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    if args.kernel == "fwd":
        seq = args.seq
        q = torch.empty(seq, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        k = torch.empty(seq, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        v = torch.empty(seq, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        out = torch.empty_like(q)
        work = ops.make_work([(0, seq, 0, 0, (C.HCP_SRC_A, 0, seq, 0), None)])
        fn = lambda: ops.ring_attn_fwd(q, work, scale=D ** -0.5, num_kv_heads=HKV, out=out, k_a=k, v_a=v)
        work_units, unit = 4.0 * D * H * causal_pairs(seq), "TFLOP/s"
    else:
        B, LOC, PEER, bs = args.decode_seqs, 32768, 32768, 16
        nb = LOC // bs
        cache = torch.empty(B * nb, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        pk = torch.empty(B * PEER, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        pv = torch.empty_like(pk).normal_(generator=g)
        bt = torch.randperm(B * nb, generator=torch.Generator().manual_seed(0)).to(torch.int32).view(B, nb).to(dev)
        q = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
        out = torch.empty_like(q)
        seqs = np.array([(b, b * PEER, PEER, b, 0, LOC) for b in range(B)], np.int32)
        fn = lambda: ops.decode_splitkv(q, seqs, scale=D ** -0.5, num_kv_heads=HKV, out=out, peer_k=pk,
                                        peer_v=pv, kv_cache=cache, block_table=bt)
        work_units, unit = float(B * (LOC + PEER) * HKV * D * 4), "GB/s"
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(max(1, args.iters)):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / max(1, args.iters)
    rate = work_units / ms / (1e9 if unit == "TFLOP/s" else 1e6)
    print(f"kernel={args.kernel} ms={ms:.3f} {unit}={rate:.1f} device_status={C.device_status()}", flush=True)


def decode_ring_step(world, rank, dev, pk, g, barrier) -> dict:
    """One ``RingDecode.step`` over all ranks (collective: every rank calls
    it): 64 requests x 65536 context keys split over the ranks, one layer,
    CUDA events, max over ranks.  Warm-up covers max(3, N) steps so every
    rank has kept a decode token (the growth append's kernels are loaded)
    before timing."""
    import torch
    import torch.distributed as dist

    from hcp_vllm_plugin_b200.ring_decode import RingDecode

    B, total, warm, steps = 64, 65536, max(3, world), 10
    chunk = total // world
    rd = RingDecode(1, B, chunk + warm + steps + 1, H, HKV, D, D ** -0.5, dev)
    for b in range(B):
        base = b * rd.cap
        rd.k[0, base:base + chunk].normal_(generator=g)
        rd.v[0, base:base + chunk].normal_(generator=g)
        rd.lens[0][b] = chunk
    q = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    kn = torch.empty(B, HKV, D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vn = torch.empty_like(kn).normal_(generator=g)
    out = torch.empty(B, H, D, device=dev)
    owner = rank == rd.owner
    args = (q, kn, vn, out) if owner else (None, None, None, None)
    for s in range(warm):
        rd.step(0, [total + s] * B, *args)
    barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(warm, warm + steps):
        rd.step(0, [total + s] * B, *args)
    b_.record()
    barrier()
    ms = a.elapsed_time(b_) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kv_bytes = B * (total + warm + steps // 2) * HKV * D * 2 * 2
    del rd
    return {"ms_per_step": ms, "requests": B, "context_keys": total, "ranks": world,
            "kv_gbs_all_ranks": kv_bytes / ms / 1e6,
            "frac_of_hbm_all_ranks": kv_bytes / ms / 1e6 / (pk["hbm_gbs"] * world)}


def run_rows(args, world, rank, local_rank):
    """``--rows``: one JSON line with device-timed measurements of the rows
    beside the forward kernel (CUDA events, max over ranks where collective):

    f2_gather       pool -> chunk extraction (``hcp_kv_cache_gather``): a
                    16384-token chunk out of each of 28 layers' paged caches
                    (940 MB, more than L2), bytes read + written vs HBM peak;
    f3_merge_n      N-way LSE merge of 8 fp32 partials, 4096 rows x 28 heads;
    f3_ring_decode  RingDecode.step over all ranks: 64 requests x 65536
                    context keys split over the ranks, one layer; per-step
                    time and the K/V bytes scanned per second, all ranks;
    f1_ipc_copy     (N >= 2) a 2 GiB chunk store exported by rank 0 with CUDA
                    IPC, copied by rank 1 with the copy engine over NVLink;
    f4_file_import  (N = 1) hcp-kv-v1 import of 4 layers x 16384 tokens
                    through HcpFileConnector (files just written, so the read
                    comes from the page cache)."""
    import ctypes
    import datetime
    import shutil
    import tempfile
    import types

    import numpy as np
    import torch
    import torch.distributed as dist

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pk, pk_src = peaks()
    res: dict = {}
    g = torch.Generator(device=dev).manual_seed(5)

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    if rank == 0:
        try:  # f2: gather
            L, T, bs = 28, 16384, 16
            nb = T // bs
            caches = [torch.empty(nb, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev).normal_(generator=g)
                      for _ in range(L)]
            slots = [(torch.randperm(nb, generator=torch.Generator().manual_seed(i))[:, None] * bs
                      + torch.arange(bs)[None, :]).flatten().to(dev) for i in range(L)]
            kk = torch.empty(T, HKV, D, dtype=torch.bfloat16, device=dev)
            vv = torch.empty_like(kk)
            ms = timed(lambda: [ops.kv_cache_gather(caches[i], slots[i], key=kk, value=vv) for i in range(L)], 5)
            byts = L * 2 * (T * HKV * 2 * D * 2)
            res["f2_gather"] = {"ms_28_layers": ms, "gbs": byts / ms / 1e6, "bytes": byts,
                                "frac_of_hbm": byts / ms / 1e6 / pk["hbm_gbs"]}
            del caches, slots, kk, vv
        except Exception as e:  # noqa: BLE001 - reported in the line
            res["f2_gather"] = {"error": repr(e)}
        try:  # f3: N-way merge
            n, t = 8, 4096
            so = torch.empty(n, t, H, D, device=dev).normal_(generator=g)
            sl = torch.empty(n, H, t, device=dev).normal_(generator=g)
            o = torch.empty(t, H, D, dtype=torch.bfloat16, device=dev)
            ol = torch.empty(H, t, device=dev)
            ms = timed(lambda: ops.merge_attn_states_n(o, so, sl, ol))
            byts = so.numel() * 4 + sl.numel() * 4 + o.numel() * 2 + ol.numel() * 4
            res["f3_merge_n"] = {"ms": ms, "gbs": byts / ms / 1e6, "frac_of_hbm": byts / ms / 1e6 / pk["hbm_gbs"]}
            del so, sl, o, ol
        except Exception as e:  # noqa: BLE001
            res["f3_merge_n"] = {"error": repr(e)}

    # f3: ring decode over all ranks
    res["f3_ring_decode"] = decode_ring_step(world, rank, dev, pk, g, barrier)

    if world > 1:  # f1: CUDA IPC copy from rank 0's store to rank 1
        nbytes = 2 << 30
        info = [None]
        store = None
        if rank == 0:
            store = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            h = (ctypes.c_uint8 * 64)()
            off = ctypes.c_int64()
            C.check(C.load().hcp_ipc_export(store.data_ptr(), h, ctypes.byref(off)), "hcp_ipc_export")
            info = [(bytes(h).hex(), int(off.value))]
        dist.broadcast_object_list(info, src=0)
        res_ipc = None
        if rank == 1:
            base = ctypes.c_void_p()
            C.check(C.load().hcp_ipc_open(bytes.fromhex(info[0][0]), local_rank, ctypes.byref(base)),
                    "hcp_ipc_open")
            dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            src = base.value + info[0][1]
            st = torch.cuda.current_stream().cuda_stream
            ms = timed(lambda: C.check(C.load().hcp_peer_copy(dst.data_ptr(), src, nbytes, st), "copy"), 5)
            C.load().hcp_ipc_close(base.value)
            res_ipc = {"ms_2GiB": ms, "gbs": nbytes / ms / 1e6}
            del dst
        obj = [res_ipc]
        if world > 1:
            dist.broadcast_object_list(obj, src=1)
        res["f1_ipc_copy"] = obj[0]
        barrier()
        del store

    if world == 1:  # f4: file import
        tmp = tempfile.mkdtemp(prefix="hcp_kv_")
        try:
            from safetensors.torch import save_file
            from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorRole

            from hcp_vllm_plugin_b200.file_connector import HcpConnectorMetadata, HcpFileConnector, ReqMeta
            L4, T, bs = 4, 16384, 16
            with open(os.path.join(tmp, "meta.json"), "w") as f:
                json.dump(dict(format="hcp-kv-v1", prompt_token_ids=list(range(T + 1)), seq_len=T + 1,
                               num_layers=L4, num_kv_heads=HKV, head_dim=D, dtype="bfloat16"), f)
            for i in range(L4):
                save_file({"kv": torch.randn(T, 2, HKV, D).bfloat16()}, os.path.join(tmp, f"layer_{i}.safetensors"))
            extra = {"hcp_kv_dir": tmp}
            kvt = types.SimpleNamespace(get_from_extra_config=lambda k, d=None: extra.get(k, d))
            hf = types.SimpleNamespace(hidden_size=H * D, num_attention_heads=H, num_hidden_layers=L4,
                                       num_key_value_heads=HKV)
            cfg = types.SimpleNamespace(kv_transfer_config=kvt, cache_config=types.SimpleNamespace(block_size=bs),
                                        model_config=types.SimpleNamespace(hf_config=hf, dtype=torch.bfloat16))
            conn = HcpFileConnector(cfg, KVConnectorRole.WORKER, None)
            sm = torch.arange(T, dtype=torch.int64)
            names = [f"model.layers.{i}.self_attn.attn" for i in range(L4)]
            caches = {n: torch.zeros(T // bs + 8, HKV, bs, 2 * D, dtype=torch.bfloat16, device=dev) for n in names}
            fc = types.SimpleNamespace(no_compile_layers={n: types.SimpleNamespace(kv_cache=c) for n, c in caches.items()})
            walls = []
            for _ in range(3):
                conn.bind_connector_metadata(HcpConnectorMetadata(requests=[ReqMeta(sm, T)]))
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                conn.start_load_kv(fc)
                for n in names:
                    conn.wait_for_layer_load(n)
                conn.wait_for_save()
                torch.cuda.synchronize()
                walls.append(time.perf_counter() - t0)
            byts = L4 * T * 2 * HKV * D * 2
            w = min(walls)
            res["f4_file_import"] = {"s_4_layers": w, "gbs": byts / w / 1e9, "bytes": byts,
                                     "timing": "host wall clock, files in the page cache"}
        except Exception as e:  # noqa: BLE001
            res["f4_file_import"] = {"error": repr(e)}
        finally:
            shutil.rmtree(tmp, ignore_errors=True)

    if rank == 0:
        print(json.dumps({"rows": res, "n_gpus": world, "peaks": pk_src, "device_status": C.device_status()}),
              flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, runner, dev, chunk, L, barrier, max_over_ranks, world):
    """Same metric through RingPrefill.forward with inputs copied from pinned
    host memory every layer and the output copied back; copies overlap compute
    on separate streams (double-buffered device inputs)."""
    import torch

    nbuf = 2  # distinct host layers (alternating)
    hq = [torch.randn(chunk, H, D).bfloat16().pin_memory() for _ in range(nbuf)]
    hk = [torch.randn(chunk, HKV, D).bfloat16().pin_memory() for _ in range(nbuf)]
    hv = [torch.randn(chunk, HKV, D).bfloat16().pin_memory() for _ in range(nbuf)]
    hout = [torch.empty(chunk, H, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dq = [torch.empty(chunk, H, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    dk = [torch.empty(chunk, HKV, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    dv = [torch.empty(chunk, HKV, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    dout = [torch.empty(chunk, H, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    for e in in_free + out_free:
        e.record(comp)

    def one_step():
        for layer in range(L):
            b = layer % 2
            hb = layer % nbuf
            with torch.cuda.stream(h2d):
                h2d.wait_event(in_free[b])
                dq[b].copy_(hq[hb], non_blocking=True)
                dk[b].copy_(hk[hb], non_blocking=True)
                dv[b].copy_(hv[hb], non_blocking=True)
                in_ready[b].record(h2d)
            comp.wait_event(in_ready[b])
            comp.wait_event(out_free[b])
            runner.forward(dq[b], dk[b], dv[b], dout[b])
            in_free[b].record(comp)
            out_ready[b].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(out_ready[b])
                hout[b].copy_(dout[b], non_blocking=True)
                out_free[b].record(d2h)

    one_step()
    barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(comp)
    for _ in range(args.steps):
        one_step()
    comp.wait_stream(d2h)
    t1.record(comp)
    barrier()
    ms = max_over_ranks(t0.elapsed_time(t1))
    bi = L * (hq[0].numel() + hk[0].numel() + hv[0].numel()) * 2 * world
    bo = L * hout[0].numel() * 2 * world
    return {"value": args.seq * args.steps / (ms / 1e3), "unit": "tok/s",
            "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "note": "RingPrefill.forward per layer, q/k/v H2D from pinned host and output D2H "
                    "every layer inside the timed region (2 distinct host layers alternate)"}


if __name__ == "__main__":
    main()
