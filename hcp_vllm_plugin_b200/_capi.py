"""ctypes binding of ``libhcp_ring.so`` (the C ABI in ``include/hcp_ring.h``).

The shared library is built in-tree by ``hcp_vllm_plugin_b200/build.py``.
There is no fallback: if the library is missing, every op raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhcp_ring.so")

HCP_OK = 0
STATUS_NAMES = {
    0: "HCP_OK",
    1: "HCP_ERR_INVALID",
    2: "HCP_ERR_UNSUPPORTED",
    3: "HCP_ERR_CUDA",
    4: "HCP_ERR_DEVICE",
    5: "HCP_ERR_SCRATCH_LIMIT",
}

HCP_BF16, HCP_F16, HCP_F32 = 0, 1, 2
HCP_SRC_NONE, HCP_SRC_A, HCP_SRC_B, HCP_SRC_PAGED, HCP_SRC_LIST = 0, 1, 2, 3, 4
HCP_SRC_EXT0 = 16          # HCP_SRC_EXT0 + i: extra contiguous source i
HCP_MAX_ITEM_SEGMENTS = 8  # segments in one work item's list
HCP_MAX_EXT_SOURCES = 8    # extra contiguous sources per call


class HcpKvSource(ctypes.Structure):
    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("row_stride", ctypes.c_int64),
    ]


class HcpKvSegment(ctypes.Structure):
    _fields_ = [
        ("src", ctypes.c_int32),
        ("start", ctypes.c_int32),
        ("len", ctypes.c_int32),
        ("causal_off", ctypes.c_int32),
    ]


class HcpAttnWork(ctypes.Structure):
    _fields_ = [
        ("q_start", ctypes.c_int32),
        ("q_len", ctypes.c_int32),
        ("paged_req", ctypes.c_int32),
        ("lse_col", ctypes.c_int32),
        ("seg", HcpKvSegment * 2),
    ]


class HcpFwdArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("_pad0", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_rows", ctypes.c_int64), ("q_row_stride", ctypes.c_int64),
        ("k_a", ctypes.c_void_p), ("v_a", ctypes.c_void_p), ("rows_a", ctypes.c_int64),
        ("a_row_stride", ctypes.c_int64),
        ("k_b", ctypes.c_void_p), ("v_b", ctypes.c_void_p), ("rows_b", ctypes.c_int64),
        ("b_row_stride", ctypes.c_int64),
        ("kv_cache", ctypes.c_void_p), ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32), ("_pad1", ctypes.c_int32),
        ("block_table", ctypes.c_void_p), ("block_table_stride", ctypes.c_int64),
        ("block_table_rows", ctypes.c_int64),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32), ("_pad2", ctypes.c_int32),
        ("out_row_stride", ctypes.c_int64),
        ("lse", ctypes.c_void_p), ("lse_stride", ctypes.c_int64),
        ("merge_o", ctypes.c_void_p), ("merge_o_dtype", ctypes.c_int32), ("_pad3", ctypes.c_int32),
        ("merge_o_row_stride", ctypes.c_int64),
        ("merge_lse", ctypes.c_void_p), ("merge_lse_stride", ctypes.c_int64),
        ("work", ctypes.POINTER(HcpAttnWork)), ("num_work", ctypes.c_int32),
        ("_pad4", ctypes.c_int32),
        ("ext", ctypes.POINTER(HcpKvSource)), ("num_ext", ctypes.c_int32), ("_pad5", ctypes.c_int32),
        ("seg_list", ctypes.POINTER(HcpKvSegment)), ("num_seg_list", ctypes.c_int32),
        ("_pad6", ctypes.c_int32),
        ("window", ctypes.c_int32), ("_pad7", ctypes.c_int32),
    ]


class HcpDecodeSeq(ctypes.Structure):
    _fields_ = [
        ("q_row", ctypes.c_int32),
        ("peer_start", ctypes.c_int32),
        ("peer_len", ctypes.c_int32),
        ("paged_req", ctypes.c_int32),
        ("local_start", ctypes.c_int32),
        ("local_len", ctypes.c_int32),
    ]


class HcpDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("chunk_keys", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("q_rows", ctypes.c_int64), ("q_row_stride", ctypes.c_int64),
        ("peer_k", ctypes.c_void_p), ("peer_v", ctypes.c_void_p), ("peer_rows", ctypes.c_int64),
        ("peer_row_stride", ctypes.c_int64),
        ("kv_cache", ctypes.c_void_p), ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32), ("_pad0", ctypes.c_int32),
        ("block_table", ctypes.c_void_p), ("block_table_stride", ctypes.c_int64),
        ("block_table_rows", ctypes.c_int64),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32), ("_pad1", ctypes.c_int32),
        ("out_row_stride", ctypes.c_int64),
        ("lse", ctypes.c_void_p), ("lse_stride", ctypes.c_int64),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64),
        ("seqs", ctypes.POINTER(HcpDecodeSeq)), ("num_seqs", ctypes.c_int32),
        ("_pad2", ctypes.c_int32),
        ("ext", ctypes.POINTER(HcpKvSource)), ("num_ext", ctypes.c_int32), ("_pad3", ctypes.c_int32),
        ("peer_src", ctypes.POINTER(ctypes.c_int32)),
    ]


# Every C entry point with its ctypes signature.  ``tests`` check that the
# built library exports exactly the names ``include/hcp_ring.h`` declares.
SIGNATURES = {
    "hcp_ring_attn_fwd": (ctypes.c_int, [ctypes.POINTER(HcpFwdArgs), ctypes.c_void_p]),
    "hcp_merge_attn_states": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    "hcp_ring_decode_splitkv": (ctypes.c_int, [ctypes.POINTER(HcpDecodeArgs), ctypes.c_void_p]),
    "hcp_decode_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(HcpDecodeArgs)]),
    "hcp_ring_decode_splitkv_noalloc": (ctypes.c_int, [ctypes.POINTER(HcpDecodeArgs), ctypes.c_void_p]),
    "hcp_kv_cache_update": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    "hcp_kv_cache_gather": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p]),
    "hcp_ipc_export": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]),
    "hcp_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p)]),
    "hcp_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "hcp_peer_copy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "hcp_merge_attn_states_n": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]),
    "hcp_get_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32)]),
    "hcp_reset_device_status": (ctypes.c_int, []),
    "hcp_device_status_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "hcp_selftest_bounded_wait": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)]),
    "hcp_version": (ctypes.c_char_p, []),
}

_lib = None


class HcpError(RuntimeError):
    """A C-ABI call returned a non-OK status."""


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the shared library; raise if it was not built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise HcpError(
            f"{p} is missing: build it with `python -m hcp_vllm_plugin_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != HCP_OK:
        raise HcpError(f"{what} failed: {STATUS_NAMES.get(rc, rc)}")


def device_status() -> int:
    v = ctypes.c_int32(0)
    check(load().hcp_get_device_status(ctypes.byref(v)), "hcp_get_device_status")
    return int(v.value)


def reset_device_status() -> None:
    check(load().hcp_reset_device_status(), "hcp_reset_device_status")


class DeviceStatusWatch:
    """The library's device status word, watched without synchronising:
    :meth:`record` queues a copy of it into a pinned host word behind the
    work already on a stream; :meth:`check` raises :class:`HcpError` when a
    copy that has completed saw a failure (a bounded wait that ran out, after
    which every later kernel of the library skips its work)."""

    def __init__(self):
        import torch

        self._torch = torch
        self.host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.event = None

    def record(self, stream) -> None:
        torch = self._torch
        check(load().hcp_device_status_async(self.host.data_ptr(), stream.cuda_stream),
              "hcp_device_status_async")
        self.event = torch.cuda.Event()
        self.event.record(stream)

    def check(self, what: str = "device") -> None:
        if self.event is None or not self.event.query():
            return
        v = int(self.host[0])
        if v != 0:
            self.event = None
            raise HcpError(f"{what}: a kernel of this library reported a device-side failure {v:#x} "
                           f"(a bounded wait ran out); later kernels skip their work until "
                           f"hcp_reset_device_status")
