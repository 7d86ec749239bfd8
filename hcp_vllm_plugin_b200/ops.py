"""Torch-tensor front end of the C ABI.

Each function checks its tensors, builds the C argument struct and calls
``libhcp_ring.so`` on the current CUDA stream.  Nothing here computes
attention: there is no CPU path.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _capi as C

_DT = {torch.bfloat16: C.HCP_BF16, torch.float16: C.HCP_F16, torch.float32: C.HCP_F32}

# Work-item row layout shared with ``hcp_attn_work`` (12 int32 per item):
#   q_start, q_len, paged_req, lse_col, then per segment (src, start, len, causal_off) x 2
WORK_FIELDS = 12


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _rows_heads(t: torch.Tensor, name: str) -> int:
    """Row stride (elements) of a [rows, heads, D] tensor whose last two dims are packed."""
    if t.dim() != 3:
        raise ValueError(f"{name} must be [rows, heads, head_dim], got {tuple(t.shape)}")
    if t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError(f"{name} must be contiguous in its last two dims")
    return t.stride(0) if t.shape[0] > 1 else t.shape[1] * t.shape[2]


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _same_device(ref: torch.Tensor, **tensors) -> None:
    """Every given tensor must live on ``ref``'s GPU: the library receives
    raw addresses, and a host tensor or another GPU's tensor handed to a
    kernel is a memory fault on the device, not an error the caller sees."""
    if not ref.is_cuda:
        raise ValueError("tensors must be CUDA tensors (no CPU path)")
    idx = ref.get_device()
    for name, t in tensors.items():
        if t is not None and (not t.is_cuda or t.get_device() != idx):
            raise ValueError(f"{name} must be on {ref.device} (got {t.device})")


def _dev(t: torch.Tensor):
    """Make the tensor's GPU the current device for the library call: the
    library launches on the current device, into a stream of that device."""
    return torch.cuda.device(t.device)


def _ext_sources(ext, dtype, ref: torch.Tensor):
    """ctypes array of ``hcp_kv_source`` for a list of (k, v) tensors, each
    [rows, Hkv, D] with its last two dims packed (k and v of one source share
    a row stride), or None."""
    if not ext:
        return None
    if len(ext) > C.HCP_MAX_EXT_SOURCES:
        raise ValueError(f"at most {C.HCP_MAX_EXT_SOURCES} extra sources per call")
    arr = (C.HcpKvSource * len(ext))()
    for i, (k, v) in enumerate(ext):
        if k.shape != v.shape or k.dtype != dtype or v.dtype != dtype:
            raise ValueError(f"extra source {i}: k and v must be of one shape and q's dtype")
        _same_device(ref, **{f"ext[{i}].k": k, f"ext[{i}].v": v})
        ks, vs = _rows_heads(k, f"ext[{i}].k"), _rows_heads(v, f"ext[{i}].v")
        if ks != vs:
            raise ValueError(f"extra source {i}: k and v must share a row stride")
        arr[i].k, arr[i].v, arr[i].rows, arr[i].row_stride = _ptr(k), _ptr(v), k.shape[0], ks
    return arr


def make_work(items) -> np.ndarray:
    """Pack work items into an int32 [n, 12] array.

    Each item is ``(q_start, q_len, paged_req, lse_col, seg0, seg1)`` with a
    segment ``(src, start, len, causal_off)`` or ``None``.
    """
    arr = np.zeros((len(items), WORK_FIELDS), dtype=np.int32)
    for i, (qs, ql, preq, lcol, s0, s1) in enumerate(items):
        arr[i, :4] = (qs, ql, preq, lcol)
        for j, sg in enumerate((s0, s1)):
            if sg is not None:
                arr[i, 4 + 4 * j: 8 + 4 * j] = sg
    return arr


def ring_attn_fwd(
    q: torch.Tensor,
    work: np.ndarray,
    *,
    scale: float,
    num_kv_heads: int,
    out: torch.Tensor,
    lse: torch.Tensor | None = None,
    k_a: torch.Tensor | None = None,
    v_a: torch.Tensor | None = None,
    k_b: torch.Tensor | None = None,
    v_b: torch.Tensor | None = None,
    kv_cache: torch.Tensor | None = None,
    block_table: torch.Tensor | None = None,
    merge_o: torch.Tensor | None = None,
    merge_lse: torch.Tensor | None = None,
    ext=None,
    seg_list: np.ndarray | None = None,
    window: int | None = None,
) -> None:
    """Fused ring-attention forward over a list of work items (``hcp_ring_attn_fwd``).

    q/out [rows, H, D]; k_*/v_* [rows, Hkv, D]; kv_cache [num_blocks, Hkv,
    block_size, 2*D]; block_table [num_reqs, max_blocks] int32; lse, merge_lse
    [H, cols] float32.  ``work`` comes from :func:`make_work`.  ``ext``: up to
    8 extra contiguous (k, v) sources, named by segments as
    ``HCP_SRC_EXT0 + i``; ``seg_list``: int32 [n, 4] segments that
    ``HCP_SRC_LIST`` items point into (``(HCP_SRC_LIST, first, count, 0)``).
    ``window``: sliding window of the causal segments (keys j with
    ``qpos - window < j <= qpos``), None = none.
    """
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor (no CPU path)")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"unsupported dtype {q.dtype}")
    _same_device(q, k_a=k_a, v_a=v_a, k_b=k_b, v_b=v_b, kv_cache=kv_cache, block_table=block_table, out=out,
                 lse=lse, merge_o=merge_o, merge_lse=merge_lse)
    num_heads, head_dim = q.shape[1], q.shape[2]
    a = C.HcpFwdArgs()
    a.dtype = _DT[q.dtype]
    a.num_heads = num_heads
    a.num_kv_heads = num_kv_heads
    a.head_dim = head_dim
    a.scale = float(scale)
    a.q = _ptr(q)
    a.q_rows = q.shape[0]
    a.q_row_stride = _rows_heads(q, "q")
    for name, kt, vt in (("a", k_a, v_a), ("b", k_b, v_b)):
        if kt is None:
            continue
        if vt is None or kt.shape != vt.shape or kt.dtype != q.dtype or vt.dtype != q.dtype:
            raise ValueError(f"k_{name}/v_{name} must match in shape and dtype")
        ks, vs = _rows_heads(kt, f"k_{name}"), _rows_heads(vt, f"v_{name}")
        if ks != vs:
            raise ValueError(f"k_{name} and v_{name} must share a row stride")
        setattr(a, f"k_{name}", _ptr(kt))
        setattr(a, f"v_{name}", _ptr(vt))
        setattr(a, f"rows_{name}", kt.shape[0])
        setattr(a, f"{name}_row_stride", ks)
    if kv_cache is not None:
        if kv_cache.dim() != 4 or not kv_cache.is_contiguous() or kv_cache.dtype != q.dtype:
            raise ValueError("kv_cache must be a contiguous [num_blocks, Hkv, block_size, 2*D] tensor")
        if block_table is None or block_table.dtype != torch.int32 or block_table.dim() != 2:
            raise ValueError("block_table must be an int32 [num_reqs, max_blocks] tensor")
        if block_table.stride(1) != 1:
            raise ValueError("block_table rows must be contiguous")
        a.kv_cache = _ptr(kv_cache)
        a.num_blocks = kv_cache.shape[0]
        a.block_size = kv_cache.shape[2]
        a.block_table = _ptr(block_table)
        a.block_table_stride = block_table.stride(0)
        a.block_table_rows = block_table.shape[0]
    if out.shape[0] < q.shape[0] or out.shape[1:] != q.shape[1:] or out.device != q.device:
        raise ValueError("out must be [>= q rows, H, D] on q's device")
    a.out = _ptr(out)
    a.out_dtype = _DT[out.dtype]
    a.out_row_stride = _rows_heads(out, "out")
    if lse is not None:
        if lse.dtype != torch.float32 or lse.dim() != 2 or lse.stride(1) != 1:
            raise ValueError("lse must be a float32 [H, cols] tensor with unit column stride")
        if lse.shape[0] != num_heads:
            raise ValueError("lse must have H rows")
        a.lse = _ptr(lse)
        a.lse_stride = lse.stride(0)
    if merge_lse is not None:
        if merge_o is None or merge_lse.dtype != torch.float32 or merge_lse.stride(1) != 1:
            raise ValueError("merge needs merge_o and a float32 merge_lse")
        if merge_lse.shape[0] != num_heads or merge_o.shape[0] < q.shape[0] or merge_o.shape[1:] != q.shape[1:]:
            raise ValueError("merge_o must be [>= q rows, H, D] and merge_lse [H, cols]")
        a.merge_o = _ptr(merge_o)
        a.merge_o_dtype = _DT[merge_o.dtype]
        a.merge_o_row_stride = _rows_heads(merge_o, "merge_o")
        a.merge_lse = _ptr(merge_lse)
        a.merge_lse_stride = merge_lse.stride(0)
    ext_arr = _ext_sources(ext, q.dtype, q)
    if ext_arr is not None:
        a.ext, a.num_ext = ctypes.cast(ext_arr, ctypes.POINTER(C.HcpKvSource)), len(ext_arr)
    if seg_list is not None:
        seg_list = np.ascontiguousarray(seg_list, dtype=np.int32).reshape(-1, 4)
        a.seg_list = seg_list.ctypes.data_as(ctypes.POINTER(C.HcpKvSegment))
        a.num_seg_list = seg_list.shape[0]
    if window is not None:
        if int(window) <= 0:
            raise ValueError("window must be a positive number of keys (or None)")
        a.window = int(window)
    work = np.ascontiguousarray(work, dtype=np.int32)
    a.work = work.ctypes.data_as(ctypes.POINTER(C.HcpAttnWork))
    a.num_work = work.shape[0]
    with _dev(q):
        C.check(C.load().hcp_ring_attn_fwd(ctypes.byref(a), _stream(q)), "hcp_ring_attn_fwd")


def ring_attn_with_lse(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float,
    causal_offset: int | None,
    window: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Flash attention with LSE output; drop-in for the reference's
    ``ring_attn_with_lse`` (``hcp_vllm_plugin/ring_triton_attn.py:155-207``),
    and with ``window`` for its torch path's sliding window
    (``_attn_with_lse``, ``ring_backend.py:366-406``: applied with a causal
    offset only, as there).

    q [Tq, H, D], k/v [Tk, Hkv, D]; ``causal_offset`` = position of query 0 in
    the KV frame, ``None`` = non-causal.  Returns (out [Tq, H, D] in q's dtype,
    lse [H, Tq] float32, natural log).
    """
    tq, num_heads, _ = q.shape
    tk, num_kv_heads, _ = k.shape
    out = torch.empty_like(q)
    lse = torch.empty((num_heads, tq), dtype=torch.float32, device=q.device)
    if tq == 0:
        return out, lse
    seg = (C.HCP_SRC_A, 0, tk, -1 if causal_offset is None else int(causal_offset))
    if causal_offset is not None and causal_offset < 0:
        raise ValueError("causal_offset must be >= 0 or None")
    work = make_work([(0, tq, 0, 0, seg, None)])
    ring_attn_fwd(q, work, scale=scale, num_kv_heads=num_kv_heads, out=out, lse=lse, k_a=k, v_a=v,
                  window=window)
    return out, lse


def merge_attn_states(
    output: torch.Tensor,
    prefix_output: torch.Tensor,
    prefix_lse: torch.Tensor,
    suffix_output: torch.Tensor,
    suffix_lse: torch.Tensor,
    output_lse: torch.Tensor | None = None,
) -> None:
    """vLLM ``merge_attn_states`` contract (``hcp_merge_attn_states``): o tensors
    [T, H, D], lse [H, T] float32; writes ``output`` (and ``output_lse``)."""
    _same_device(output, prefix_output=prefix_output, prefix_lse=prefix_lse, suffix_output=suffix_output,
                 suffix_lse=suffix_lse, output_lse=output_lse)
    num_tokens, num_heads, head_dim = output.shape
    for t in (prefix_lse, suffix_lse) + ((output_lse,) if output_lse is not None else ()):
        if t.dtype != torch.float32 or t.stride(1) != 1:
            raise ValueError("lse tensors must be float32 with unit column stride")
    lib = C.load()
    with _dev(output):
        rc = lib.hcp_merge_attn_states(
            _ptr(output), _DT[output.dtype], _rows_heads(output, "output"),
            _ptr(output_lse), 0 if output_lse is None else output_lse.stride(0),
            _ptr(prefix_output), _DT[prefix_output.dtype], _rows_heads(prefix_output, "prefix_output"),
            _ptr(prefix_lse), prefix_lse.stride(0),
            _ptr(suffix_output), _DT[suffix_output.dtype], _rows_heads(suffix_output, "suffix_output"),
            _ptr(suffix_lse), suffix_lse.stride(0),
            num_tokens, num_heads, head_dim, _stream(output))
    C.check(rc, "hcp_merge_attn_states")


def merge_attn_states_n(output: torch.Tensor, states_o: torch.Tensor, states_lse: torch.Tensor,
                        output_lse: torch.Tensor | None = None) -> None:
    """N-way LSE merge (``hcp_merge_attn_states_n``): states_o [N, T, H, D] and
    states_lse [N, H, T] float32 contiguous -> output [T, H, D] (and output_lse
    [H, T])."""
    _same_device(output, states_o=states_o, states_lse=states_lse, output_lse=output_lse)
    n, t, h, d = states_o.shape
    if states_o.dtype != torch.float32 or states_lse.dtype != torch.float32:
        raise ValueError("states must be float32")
    if not states_o.is_contiguous() or not states_lse.is_contiguous() or tuple(states_lse.shape) != (n, h, t):
        raise ValueError("states_o [N, T, H, D] and states_lse [N, H, T] must be contiguous")
    if tuple(output.shape) != (t, h, d):
        raise ValueError("output must be [T, H, D]")
    if output_lse is not None and (output_lse.dtype != torch.float32 or output_lse.stride(1) != 1):
        raise ValueError("output_lse must be float32 with unit column stride")
    with _dev(output):
        rc = C.load().hcp_merge_attn_states_n(
            _ptr(output), _DT[output.dtype], _rows_heads(output, "output"), _ptr(output_lse),
            0 if output_lse is None else output_lse.stride(0), _ptr(states_o), _ptr(states_lse), n, t, h, d,
            _stream(output))
    C.check(rc, "hcp_merge_attn_states_n")


DECODE_FIELDS = 6  # q_row, peer_start, peer_len, paged_req, local_start, local_len

_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Cached device scratch (grown on demand) for the split-KV partials, one
    per stream: calls on one stream run in order, while the decode ring's
    serve thread and the backend decode on different streams of one device
    at the same time and must not share partials."""
    key = (device.type, device.index, torch.cuda.current_stream(device).cuda_stream)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def decode_args(q, seqs, *, scale, num_kv_heads, out, lse=None, peer_k=None, peer_v=None,
                kv_cache=None, block_table=None, chunk_keys=0, ext=None, peer_src=None):
    """Build ``hcp_decode_args`` (without workspace) plus the host arrays it
    points to (keep them alive until the call).  ``ext``: extra contiguous
    (k, v) peer sources; ``peer_src``: per sequence, -1 for peer_k / peer_v or
    the index of its extra source."""
    if not q.is_cuda or q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("q must be a bf16/fp16 CUDA tensor (no CPU path)")
    _same_device(q, peer_k=peer_k, peer_v=peer_v, kv_cache=kv_cache, block_table=block_table, out=out, lse=lse)
    seqs = np.ascontiguousarray(seqs, dtype=np.int32).reshape(-1, DECODE_FIELDS)
    a = C.HcpDecodeArgs()
    a.dtype = _DT[q.dtype]
    a.num_heads, a.head_dim = q.shape[1], q.shape[2]
    a.num_kv_heads = num_kv_heads
    a.scale = float(scale)
    a.chunk_keys = int(chunk_keys)
    a.q, a.q_rows, a.q_row_stride = _ptr(q), q.shape[0], _rows_heads(q, "q")
    if peer_k is not None:
        if peer_v is None or peer_k.shape != peer_v.shape or peer_k.dtype != q.dtype:
            raise ValueError("peer_k/peer_v must match")
        a.peer_k, a.peer_v = _ptr(peer_k), _ptr(peer_v)
        a.peer_rows, a.peer_row_stride = peer_k.shape[0], _rows_heads(peer_k, "peer_k")
    if kv_cache is not None:
        if kv_cache.dim() != 4 or not kv_cache.is_contiguous() or kv_cache.dtype != q.dtype:
            raise ValueError("kv_cache must be a contiguous [num_blocks, Hkv, block_size, 2*D] tensor")
        if block_table is None or block_table.dtype != torch.int32 or block_table.stride(1) != 1:
            raise ValueError("block_table must be int32 with contiguous rows")
        a.kv_cache, a.num_blocks, a.block_size = _ptr(kv_cache), kv_cache.shape[0], kv_cache.shape[2]
        a.block_table = _ptr(block_table)
        a.block_table_stride, a.block_table_rows = block_table.stride(0), block_table.shape[0]
    if out.shape[0] < q.shape[0] or out.shape[1:] != q.shape[1:]:
        raise ValueError("out must be [>= q rows, H, D]")
    a.out, a.out_dtype, a.out_row_stride = _ptr(out), _DT[out.dtype], _rows_heads(out, "out")
    if lse is not None:
        if lse.dtype != torch.float32 or lse.stride(1) != 1 or lse.shape[0] != q.shape[1]:
            raise ValueError("lse must be float32 [H, cols]")
        a.lse, a.lse_stride = _ptr(lse), lse.stride(0)
    a.seqs = seqs.ctypes.data_as(ctypes.POINTER(C.HcpDecodeSeq))
    a.num_seqs = seqs.shape[0]
    ext_arr = _ext_sources(ext, q.dtype, q)
    if ext_arr is not None:
        a.ext, a.num_ext = ctypes.cast(ext_arr, ctypes.POINTER(C.HcpKvSource)), len(ext_arr)
    if peer_src is not None:
        peer_src = np.ascontiguousarray(peer_src, dtype=np.int32).reshape(-1)
        if peer_src.shape[0] != seqs.shape[0]:
            raise ValueError("peer_src needs one entry per sequence")
        a.peer_src = peer_src.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    return a, (seqs, ext_arr, peer_src)


def decode_splitkv(q, seqs, *, scale, num_kv_heads, out, lse=None, peer_k=None, peer_v=None,
                   kv_cache=None, block_table=None, chunk_keys=0, workspace=None, ext=None,
                   peer_src=None):
    """Batch-merged split-KV decode (``hcp_ring_decode_splitkv``).

    ``seqs`` rows: (q_row, peer_start, peer_len, paged_req, local_start,
    local_len).  Every listed key is visible to the sequence's single query.
    """
    a, keep = decode_args(q, seqs, scale=scale, num_kv_heads=num_kv_heads, out=out, lse=lse,
                          peer_k=peer_k, peer_v=peer_v, kv_cache=kv_cache,
                          block_table=block_table, chunk_keys=chunk_keys, ext=ext, peer_src=peer_src)
    lib = C.load()
    need = lib.hcp_decode_workspace_bytes(ctypes.byref(a))
    if need < 0:
        raise C.HcpError("hcp_decode_workspace_bytes: invalid arguments")
    ws = workspace if workspace is not None else _workspace(q.device, need)
    _same_device(q, workspace=ws)
    a.workspace, a.workspace_bytes = _ptr(ws), ws.numel() * ws.element_size()
    with _dev(q):
        C.check(lib.hcp_ring_decode_splitkv(ctypes.byref(a), _stream(q)), "hcp_ring_decode_splitkv")
    del keep


def kv_cache_gather(kv_cache: torch.Tensor, slot_mapping: torch.Tensor,
                    key: torch.Tensor | None = None,
                    value: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """K/V rows of ``slot_mapping`` out of the paged cache (``hcp_kv_cache_gather``).

    kv_cache [num_blocks, Hkv, block_size, 2*D]; slot_mapping [n] int64 on the
    cache's device.  Returns key, value [n, Hkv, D] (allocated unless given);
    rows of negative or out-of-range slots are zeros.
    """
    _same_device(kv_cache, slot_mapping=slot_mapping, key=key, value=value)
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 tensor")
    if kv_cache.dim() != 4 or not kv_cache.is_contiguous():
        raise ValueError("kv_cache must be a contiguous [num_blocks, Hkv, block_size, 2*D] tensor")
    nb, hkv, bs, d2 = kv_cache.shape
    n = slot_mapping.shape[0]
    if key is None:
        key = torch.empty(n, hkv, d2 // 2, dtype=kv_cache.dtype, device=kv_cache.device)
    if value is None:
        value = torch.empty(n, hkv, d2 // 2, dtype=kv_cache.dtype, device=kv_cache.device)
    if key.shape[0] < n or value.shape[0] < n or key.dtype != kv_cache.dtype or value.dtype != kv_cache.dtype:
        raise ValueError("key/value must hold n rows of the cache's dtype")
    with _dev(kv_cache):
        rc = C.load().hcp_kv_cache_gather(
            _ptr(kv_cache), nb, bs, hkv, d2 // 2, _ptr(slot_mapping), n, _ptr(key), _ptr(value),
            _rows_heads(key, "key"), _rows_heads(value, "value"), _DT[kv_cache.dtype], _stream(kv_cache))
    C.check(rc, "hcp_kv_cache_gather")
    return key, value


def kv_cache_update(key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                    slot_mapping: torch.Tensor) -> None:
    """Paged scatter of new K/V rows (``hcp_kv_cache_update``).

    key/value [n, Hkv, D]; kv_cache [num_blocks, Hkv, block_size, 2*D];
    slot_mapping [n] int64 (negative = padding).
    """
    _same_device(key, value=value, kv_cache=kv_cache, slot_mapping=slot_mapping)
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise ValueError("slot_mapping must be a contiguous int64 tensor")
    if kv_cache.dim() != 4 or not kv_cache.is_contiguous() or kv_cache.dtype != key.dtype:
        raise ValueError("kv_cache must be a contiguous [num_blocks, Hkv, block_size, 2*D] tensor")
    n = min(slot_mapping.shape[0], key.shape[0])
    with _dev(key):
        rc = C.load().hcp_kv_cache_update(
            _ptr(key), _ptr(value), n, _rows_heads(key, "key"), _rows_heads(value, "value"),
            _ptr(slot_mapping), _ptr(kv_cache), kv_cache.shape[0], kv_cache.shape[2], key.shape[1],
            key.shape[2], _DT[key.dtype], _stream(key))
    C.check(rc, "hcp_kv_cache_update")
