"""N > 1 ring prefill host logic on CPU: two and three gloo ranks run the
RingPrefill schedule (K/V rotation, Q-row hand-off to the light partner,
partial (O, LSE) return and merge) with the device ops replaced by the CPU
oracle; the gathered output must equal causal attention over the whole
sequence."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ring_oracle as ro

H, HKV, D = 4, 2, 16


def _cpu_attn(q, work, *, scale, num_kv_heads, out, lse, k_a=None, v_a=None, k_b=None, v_b=None,
              kv_cache=None, block_table=None, merge_o=None, merge_lse=None):
    """Oracle-backed stand-in for hcp_ring_attn_fwd on contiguous sources."""
    srcs = {1: (k_a, v_a), 2: (k_b, v_b)}
    for row in np.asarray(work):
        qs, ql, _, lcol = (int(x) for x in row[:4])
        qq = q[qs:qs + ql].float().numpy()
        parts = []
        for j in range(2):
            src, start, ln, coff = (int(x) for x in row[4 + 4 * j: 8 + 4 * j])
            if src == 0 or ln == 0:
                continue
            k, v = srcs[src]
            kk = k[start:start + ln].float().numpy()
            vv = v[start:start + ln].float().numpy()
            parts.append(ro.attn_with_lse(qq, kk, vv, scale, None if coff < 0 else coff))
        o, l = parts[0]
        for o2, l2 in parts[1:]:
            o, l = ro.merge_pair(o, l, o2, l2)
        if merge_o is not None:
            o, l = ro.merge_pair(merge_o[qs:qs + ql].float().numpy(),
                                 merge_lse[:, lcol:lcol + ql].numpy(), o, l)
        out[qs:qs + ql] = torch.from_numpy(o).to(out.dtype)
        if lse is not None:
            lse[:, lcol:lcol + ql] = torch.from_numpy(l)


def _cpu_merge(out, prefix_o, prefix_lse, suffix_o, suffix_lse, out_lse):
    o, l = ro.merge_pair(prefix_o.float().numpy(), prefix_lse.numpy(), suffix_o.float().numpy(),
                         suffix_lse.numpy())
    out.copy_(torch.from_numpy(o).to(out.dtype))
    if out_lse is not None:
        out_lse.copy_(torch.from_numpy(l))


def _worker(rank, world, port, seq, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hcp_vllm_plugin_b200.ring_runner import RingPrefill
        RingPrefill.attn_fn = staticmethod(_cpu_attn)
        RingPrefill.merge_fn = staticmethod(_cpu_merge)
        g = torch.Generator().manual_seed(0)
        q = torch.randn(seq, H, D, generator=g)
        k = torch.randn(seq, HKV, D, generator=g)
        v = torch.randn(seq, HKV, D, generator=g)
        runner = RingPrefill(seq, H, HKV, D, D ** -0.5, torch.device("cpu"), dtype=torch.float32)
        c = runner.chunk
        sl = slice(rank * c, (rank + 1) * c)
        out = torch.empty(c, H, D)
        lse = torch.empty(H, c)
        runner.forward(q[sl].contiguous(), k[sl].contiguous(), v[sl].contiguous(), out, lse)
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        lses = [torch.empty_like(lse) for _ in range(world)]
        dist.all_gather(lses, lse)
        if rank == 0:
            want, want_lse = ro.attn_with_lse(q.numpy(), k.numpy(), v.numpy(), D ** -0.5, 0)
            got = torch.cat(outs).numpy()
            got_lse = torch.cat(lses, 1).numpy()
            result_q.put((float(np.abs(got - want).max()), float(np.abs(got_lse - want_lse).max()),
                          runner.plan.give))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,seq", [(2, 512), (3, 768), (4, 1024), (5, 1280), (8, 2048)])
def test_ring_prefill_schedule_gloo(world, seq):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, lerr, give = q.get(timeout=10)
    assert err < 1e-4 and lerr < 1e-4, (err, lerr)
    if world in (2, 4):
        assert give, "balanced plan must hand rows to a light partner"


class _FakeIpcLib:
    """Stand-in for the library's CUDA IPC calls: ``fail_export`` /
    ``fail_open`` make this rank's export or mapping fail."""

    def __init__(self, fail_export=False, fail_open=False):
        self.fail_export, self.fail_open, self.closed = fail_export, fail_open, []

    def hcp_ipc_export(self, ptr, handle, offset):
        return 1 if self.fail_export else 0

    def hcp_ipc_open(self, handle, dev, base):
        if self.fail_open:
            return 1
        base._obj.value = 4096 if hasattr(base, "_obj") else 4096
        return 0

    def hcp_ipc_close(self, b):
        self.closed.append(b)
        return 0


def _transport_worker(rank, world, port, fail_rank, mode, result_q):
    import types

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200.ring_runner import RingPrefill
    from hcp_vllm_plugin_b200.ring_schedule import hop_schedule, plan_balanced

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _FakeIpcLib(fail_export=(mode == "export" and rank == fail_rank),
                          fail_open=(mode == "open" and rank == fail_rank))
        C.load = lambda: lib
        plan = plan_balanced(world, 256)
        me = types.SimpleNamespace(
            chunk=256, Hkv=HKV, H=H, D=D, dtype=torch.float32, device=torch.device("cpu", 0), world=world,
            group=None, plan=plan, give=plan.rows_given(rank), owner=plan.helped_owner(rank),
            owner_give=plan.rows_given(plan.helped_owner(rank)) if plan.helped_owner(rank) is not None else 0,
            hops=hop_schedule(plan, rank), transport="ce", _peer_bases=[])
        me.close = types.MethodType(RingPrefill.close, me)
        RingPrefill._open_outboxes(me)
        result_q.put((rank, me.transport))
    except BaseException as e:  # noqa: BLE001 - reported to the test
        result_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["none", "export", "open"])
def test_ce_transport_falls_back_together(mode):
    """When one rank cannot export or map an outbox (memory CUDA IPC cannot
    share), every rank switches to the p2p transport, so all keep taking the
    same collective steps; otherwise all stay on ce."""
    world = 4
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_transport_worker, args=(r, world, port, 3, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=60) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = "ce" if mode == "none" else "p2p"
    assert got == {r: want for r in range(world)}
