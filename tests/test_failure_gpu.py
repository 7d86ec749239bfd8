"""Failure detection without a GPU fault.

Every wait of the library's kernels is bounded: when it runs out, the kernel
records a code in the device status word, gives up and returns, and kernels
launched while a code is recorded do no work until the host resets it.  The
self-test entry point waits on an mbarrier that nothing arrives on, through
the kernels' own bounded wait, with a short limit; nothing faults, traps or
hangs, and the context stays usable afterwards.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import parity as P
from oracle import ring_oracle as ro

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports():
    from hcp_vllm_plugin_b200 import _capi as C, ops

    lib = C.load()
    C.reset_device_status()
    try:
        _run(C, ops, lib)
    finally:
        C.reset_device_status()  # later tests must not inherit a recorded failure


def _run(C, ops, lib):
    waited = ctypes.c_int32(-1)
    C.check(lib.hcp_selftest_bounded_wait(50_000_000, ctypes.byref(waited)), "hcp_selftest_bounded_wait")
    assert waited.value == 0                      # the wait gave up
    assert C.device_status() == 0x1FF             # and said so

    # While a failure is recorded, launches do no work (fail fast) ...
    g = torch.Generator().manual_seed(0)
    tq, tk, h, hkv, d = 256, 512, 28, 4, 128
    q = torch.randn(tq, h, d, generator=g).bfloat16().cuda()
    k = torch.randn(tk, hkv, d, generator=g).bfloat16().cuda()
    v = torch.randn(tk, hkv, d, generator=g).bfloat16().cuda()
    out = torch.full((tq, h, d), 7.0, dtype=torch.bfloat16, device="cuda")
    lse = torch.full((h, tq), 7.0, device="cuda")
    work = ops.make_work([(0, tq, 0, 0, (C.HCP_SRC_A, 0, tk, tk - tq), None)])
    ops.ring_attn_fwd(q, work, scale=d ** -0.5, num_kv_heads=hkv, out=out, lse=lse, k_a=k, v_a=v)
    torch.cuda.synchronize()
    assert torch.all(out == 7.0) and torch.all(lse == 7.0)
    assert C.device_status() == 0x1FF

    # ... and after the host resets the status the same launch is correct.
    C.reset_device_status()
    ops.ring_attn_fwd(q, work, scale=d ** -0.5, num_kv_heads=hkv, out=out, lse=lse, k_a=k, v_a=v)
    torch.cuda.synchronize()
    assert C.device_status() == 0
    want, want_lse = ro.attn_with_lse(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                      v.float().cpu().numpy(), d ** -0.5, tk - tq)
    P.check_out(out.float().cpu().numpy(), want, "forward after a status reset")
    P.check_lse(lse.cpu().numpy(), want_lse, "forward after a status reset")


def test_backend_surfaces_a_device_failure_at_the_next_step():
    """A bounded wait that ran out makes every later kernel skip its work; the
    vLLM-facing backend must not hand that untouched output on.  Its steps
    queue a copy of the status word behind their launches and read it at the
    next step's host synchronisation: the step after the failure raises
    HcpError; after a reset the backend computes again."""
    import types

    from hcp_vllm_plugin_b200 import _capi as C
    from hcp_vllm_plugin_b200 import ring_backend as rb

    lib = C.load()
    dev = torch.device("cuda:0")
    b = P.paged_batch([40, 1], 0, seed=2)
    impl = rb.HcpRingAttentionImpl(28, 128, 128 ** -0.5, 4)
    cache, bt = b["cache"].to(dev), torch.from_numpy(b["bt"]).to(dev)
    q = b["q"].to(dev)
    layer = types.SimpleNamespace(layer_name="model.layers.0.self_attn.attn")

    def step():
        meta = types.SimpleNamespace(
            num_actual_tokens=q.shape[0],
            query_start_loc=torch.tensor(b["qsl"], dtype=torch.int32, device=dev),
            seq_lens=torch.tensor(b["lens"], dtype=torch.int32, device=dev), block_table=bt)
        out = torch.full_like(q, 7.0)
        impl.forward(layer, q, None, None, cache, meta, out)
        return out

    rb.clear_peer_kv()
    C.reset_device_status()
    try:
        step()
        torch.cuda.synchronize()
        waited = ctypes.c_int32(-1)
        C.check(lib.hcp_selftest_bounded_wait(50_000_000, ctypes.byref(waited)), "hcp_selftest_bounded_wait")
        assert waited.value == 0
        out = step()                      # runs, but its kernels skip their work ...
        torch.cuda.synchronize()
        assert bool((out == 7.0).all())
        with pytest.raises(C.HcpError, match="device-side failure 0x1ff"):
            step()                        # ... and the next step says so
    finally:
        C.reset_device_status()
    out = step()
    torch.cuda.synchronize()
    want = P.paged_oracle(b)
    P.check_out(P.f32(out), want, "backend after a status reset")
