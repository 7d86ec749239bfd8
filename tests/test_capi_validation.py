"""The C ABI's argument checks, on the CPU.

Every entry point validates its arguments on the host before it touches the
GPU and returns a status code (``HCP_ERR_INVALID`` for arguments that cannot
be right, ``HCP_ERR_UNSUPPORTED`` for shapes or types this build does not
serve), which the Python wrappers raise as ``HcpError`` - the reference's
convention of raising on a failed attention call (``ring_backend.py:333-336``)
with the status kept for C callers.  Device pointers below are placeholder
addresses: the checks compare them (non-null, 16-byte aligned) but never
read through them, and every case here is refused before the first CUDA
call, so no GPU is needed.  Host arrays (work items, segment lists, extra
sources, decode sequences) are real.
"""

import ctypes
import math

import pytest

from hcp_vllm_plugin_b200 import _capi as C

H, HKV, D = 28, 4, 128
INVALID, UNSUPPORTED, SCRATCH_LIMIT = 1, 2, 5
BASE = 0x7F0000000000  # placeholder device addresses, 16-byte aligned


def _addr(i: int) -> int:
    return BASE + i * 0x10000000


@pytest.fixture(scope="module")
def lib():
    return C.load()


def _work(items):
    arr = (C.HcpAttnWork * max(1, len(items)))()
    for i, (qs, ql, preq, lcol, s0, s1) in enumerate(items):
        arr[i].q_start, arr[i].q_len, arr[i].paged_req, arr[i].lse_col = qs, ql, preq, lcol
        for j, sg in enumerate((s0, s1)):
            if sg is not None:
                arr[i].seg[j].src, arr[i].seg[j].start, arr[i].seg[j].len, arr[i].seg[j].causal_off = sg
    return arr


def _fwd(rows=1024, items=None, **over):
    """Arguments of a valid call: rows x H x D queries, contiguous source A of
    ``rows`` keys, a paged cache of 64 blocks, LSE [H, rows]."""
    a = C.HcpFwdArgs()
    a.dtype, a.num_heads, a.num_kv_heads, a.head_dim, a.scale = C.HCP_BF16, H, HKV, D, D ** -0.5
    a.q, a.q_rows, a.q_row_stride = _addr(1), rows, H * D
    a.k_a, a.v_a, a.rows_a, a.a_row_stride = _addr(2), _addr(3), rows, HKV * D
    a.kv_cache, a.num_blocks, a.block_size = _addr(4), 64, 16
    a.block_table, a.block_table_stride, a.block_table_rows = _addr(5), 64, 1
    a.out, a.out_dtype, a.out_row_stride = _addr(6), C.HCP_BF16, H * D
    a.lse, a.lse_stride = _addr(7), rows
    if items is None:
        items = [(0, 0, 0, 0, (C.HCP_SRC_A, 0, rows, 0), None)]  # one empty item: nothing to launch
    work = _work(items)
    a.work, a.num_work = ctypes.cast(work, ctypes.POINTER(C.HcpAttnWork)), len(items)
    keep = [work]
    for k, v in over.items():
        setattr(a, k, v)
        if isinstance(v, ctypes.Array):
            keep.append(v)
    return a, keep


def _call_fwd(lib, a):
    return lib.hcp_ring_attn_fwd(ctypes.byref(a), None)


def test_forward_valid_call_without_rows_launches_nothing(lib):
    a, keep = _fwd()
    assert _call_fwd(lib, a) == C.HCP_OK
    a, keep = _fwd(num_work=0)
    assert _call_fwd(lib, a) == C.HCP_OK
    assert lib.hcp_ring_attn_fwd(None, None) == INVALID


@pytest.mark.parametrize("field,value,code", [
    ("dtype", 7, UNSUPPORTED),
    ("num_kv_heads", 5, INVALID),          # 28 heads do not split into 5 groups
    ("num_heads", 0, INVALID),
    ("head_dim", 96, UNSUPPORTED),
    ("scale", 0.0, INVALID),
    ("scale", -1.0, INVALID),
    ("scale", math.nan, INVALID),
    ("scale", math.inf, INVALID),
    ("window", -1, INVALID),
    ("q", None, INVALID),
    ("q", BASE + 8, INVALID),              # not 16-byte aligned (TMA)
    ("q_row_stride", H * D - 8, INVALID),
    ("q_row_stride", H * D + 4, INVALID),  # not a multiple of 8 elements
    ("out", None, INVALID),
    ("out_dtype", C.HCP_F16, UNSUPPORTED),  # neither the input type nor fp32
    ("out_row_stride", H * D - 1, INVALID),
    ("merge_lse", _addr(8), INVALID),      # a merge LSE without a merge O
    ("v_a", None, INVALID),
    ("rows_a", 0, INVALID),
    ("a_row_stride", HKV * D - 8, INVALID),
    ("k_a", BASE + 8, INVALID),
    ("block_size", 48, UNSUPPORTED),
    ("num_blocks", 0, INVALID),
    ("block_table", None, INVALID),
    ("kv_cache", BASE + 8, INVALID),
    ("num_ext", 9, INVALID),               # more extra sources than HCP_MAX_EXT_SOURCES
    ("num_ext", 1, INVALID),               # extra sources announced, none given
    ("num_seg_list", 2, INVALID),          # a segment list announced, none given
])
def test_forward_refuses_bad_arguments(lib, field, value, code):
    a, keep = _fwd(**{field: value})
    assert _call_fwd(lib, a) == code


@pytest.mark.parametrize("item,code", [
    ((0, 1025, 0, 0, (C.HCP_SRC_A, 0, 1024, 0), None), INVALID),     # rows past q_rows
    ((-1, 8, 0, 0, (C.HCP_SRC_A, 0, 1024, 0), None), INVALID),
    ((0, 8, 0, 1020, (C.HCP_SRC_A, 0, 1024, 0), None), INVALID),     # LSE columns past lse_stride
    ((0, 8, 0, 0, (C.HCP_SRC_A, 1000, 100, 0), None), INVALID),      # keys past rows_a
    ((0, 8, 0, 0, (C.HCP_SRC_B, 0, 8, 0), None), INVALID),           # source B not given
    ((0, 8, 0, 0, (C.HCP_SRC_PAGED, 8, 16, 0), None), UNSUPPORTED),  # paged start off a block boundary
    ((0, 8, 0, 0, (C.HCP_SRC_PAGED, 0, 64 * 16 + 16, 0), None), INVALID),  # past the block table
    ((0, 8, 1, 0, (C.HCP_SRC_PAGED, 0, 16, 0), None), INVALID),      # block-table row out of range
    ((0, 8, 0, 0, (C.HCP_SRC_LIST, 0, 2, 0), None), INVALID),        # list past num_seg_list
    ((0, 8, 0, 0, (C.HCP_SRC_EXT0, 0, 8, 0), None), INVALID),        # extra source 0 not given
])
def test_forward_refuses_bad_work_items(lib, item, code):
    a, keep = _fwd(items=[item])
    assert _call_fwd(lib, a) == code


def test_forward_refuses_bad_segment_lists_and_sources(lib):
    # a list of 9 segments (more than HCP_MAX_ITEM_SEGMENTS)
    segs = (C.HcpKvSegment * 9)(*[C.HcpKvSegment(C.HCP_SRC_A, 0, 8, -1) for _ in range(9)])
    a, keep = _fwd(items=[(0, 8, 0, 0, (C.HCP_SRC_LIST, 0, 9, 0), None)],
                   seg_list=ctypes.cast(segs, ctypes.POINTER(C.HcpKvSegment)), num_seg_list=9)
    assert _call_fwd(lib, a) == INVALID
    # a list that nests a list
    segs2 = (C.HcpKvSegment * 2)(C.HcpKvSegment(C.HCP_SRC_A, 0, 8, -1), C.HcpKvSegment(C.HCP_SRC_LIST, 0, 1, 0))
    a, keep = _fwd(items=[(0, 8, 0, 0, (C.HCP_SRC_LIST, 0, 2, 0), None)],
                   seg_list=ctypes.cast(segs2, ctypes.POINTER(C.HcpKvSegment)), num_seg_list=2)
    assert _call_fwd(lib, a) == INVALID
    # an extra source with a misaligned V, and one with too few rows for its segment
    ext = (C.HcpKvSource * 1)(C.HcpKvSource(_addr(9), BASE + 24, 64, HKV * D))
    a, keep = _fwd(ext=ctypes.cast(ext, ctypes.POINTER(C.HcpKvSource)), num_ext=1)
    assert _call_fwd(lib, a) == INVALID
    ext = (C.HcpKvSource * 1)(C.HcpKvSource(_addr(9), _addr(10), 64, HKV * D))
    a, keep = _fwd(items=[(0, 8, 0, 0, (C.HCP_SRC_EXT0, 0, 65, -1), None)],
                   ext=ctypes.cast(ext, ctypes.POINTER(C.HcpKvSource)), num_ext=1)
    assert _call_fwd(lib, a) == INVALID


def _dec(seqs, peer_rows=65536, q_rows=None, **over):
    """Arguments of a decode call: one query row per sequence, a contiguous
    peer source of ``peer_rows`` keys, a paged cache of 4096 blocks of 16
    keys with a 2048-entry block-table row per sequence."""
    n = len(seqs)
    a = C.HcpDecodeArgs()
    a.dtype, a.num_heads, a.num_kv_heads, a.head_dim, a.scale = C.HCP_BF16, H, HKV, D, D ** -0.5
    a.q, a.q_rows, a.q_row_stride = _addr(1), n if q_rows is None else q_rows, H * D
    a.peer_k, a.peer_v, a.peer_rows, a.peer_row_stride = _addr(2), _addr(3), peer_rows, HKV * D
    a.kv_cache, a.num_blocks, a.block_size = _addr(4), 4096, 16
    a.block_table, a.block_table_stride, a.block_table_rows = _addr(5), 2048, max(1, n)
    a.out, a.out_dtype, a.out_row_stride = _addr(6), C.HCP_BF16, H * D
    a.lse, a.lse_stride = _addr(7), max(1, n)
    arr = (C.HcpDecodeSeq * max(1, n))()
    for i, s in enumerate(seqs):
        arr[i] = C.HcpDecodeSeq(*s)
    a.seqs, a.num_seqs = ctypes.cast(arr, ctypes.POINTER(C.HcpDecodeSeq)), n
    keep = [arr]
    for k, v in over.items():
        setattr(a, k, v)
        if isinstance(v, ctypes.Array):
            keep.append(v)
    return a, keep


def _cfg2_seqs(n, keys=32768):
    # (q_row, peer_start, peer_len, paged_req, local_start, local_len)
    return [(i, 0, keys, i, 0, keys) for i in range(n)]


@pytest.mark.parametrize("seq,code", [
    ((1, 0, 16, 0, 0, 16), INVALID),          # query row past q_rows
    ((0, 65530, 16, 0, 0, 16), INVALID),      # peer keys past peer_rows
    ((0, 0, 16, 0, 8, 16), UNSUPPORTED),      # local start off a block boundary
    ((0, 0, 16, 0, 0, 2048 * 16 + 1), INVALID),  # local keys past the block table
    ((0, 0, 16, 1, 0, 16), INVALID),          # block-table row out of range
    ((0, -1, 16, 0, 0, 16), INVALID),
])
def test_decode_refuses_bad_sequences(lib, seq, code):
    a, keep = _dec([seq])
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == code
    assert lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(a), None) == code
    assert lib.hcp_decode_workspace_bytes(ctypes.byref(a)) == -1


@pytest.mark.parametrize("field,value,code", [
    ("num_kv_heads", 1, UNSUPPORTED),   # 28 query heads per KV head: more than a decode CTA groups
    ("head_dim", 256, UNSUPPORTED),
    ("scale", math.nan, INVALID),
    ("out_dtype", C.HCP_F16, UNSUPPORTED),
    ("peer_v", None, INVALID),
    ("block_size", 128, UNSUPPORTED),
    ("q", BASE + 4, INVALID),
    ("num_ext", 1, INVALID),
])
def test_decode_refuses_bad_arguments(lib, field, value, code):
    a, keep = _dec(_cfg2_seqs(2), **{field: value})
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == code
    assert lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(a), None) == code


def test_decode_peer_source_index_is_checked(lib):
    ext = (C.HcpKvSource * 1)(C.HcpKvSource(_addr(9), _addr(10), 128, HKV * D))
    for src, code in ((1, INVALID), (-2, INVALID)):
        ps = (ctypes.c_int32 * 1)(src)
        a, keep = _dec([(0, 0, 16, 0, 0, 16)], ext=ctypes.cast(ext, ctypes.POINTER(C.HcpKvSource)), num_ext=1,
                       peer_src=ctypes.cast(ps, ctypes.POINTER(ctypes.c_int32)))
        assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == code
    # extra source 0 has 128 rows: 129 peer keys from it are refused
    ps = (ctypes.c_int32 * 1)(0)
    a, keep = _dec([(0, 0, 129, 0, 0, 16)], ext=ctypes.cast(ext, ctypes.POINTER(C.HcpKvSource)), num_ext=1,
                   peer_src=ctypes.cast(ps, ctypes.POINTER(ctypes.c_int32)))
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == INVALID


def test_decode_workspace_and_the_allocation_free_limit(lib):
    """The workspace a call needs grows with its keys; the workspace entry
    point refuses a call whose workspace is missing or short, and the
    allocation-free one refuses a call beyond its fixed scratch array with
    HCP_ERR_SCRATCH_LIMIT, all before touching the GPU."""
    sizes = []
    for keys in (4096, 32768):
        a, keep = _dec(_cfg2_seqs(64, keys))
        sizes.append(lib.hcp_decode_workspace_bytes(ctypes.byref(a)))
    assert 0 < sizes[0] < sizes[1]
    a, keep = _dec(_cfg2_seqs(64))  # configs[2]: 64 x (32768 paged + 32768 peer)
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == INVALID  # no workspace given
    need = lib.hcp_decode_workspace_bytes(ctypes.byref(a))
    a.workspace, a.workspace_bytes = _addr(11), need - 16
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(a), None) == INVALID
    big, keep2 = _dec(_cfg2_seqs(2, 65536), peer_rows=65536, chunk_keys=64)
    big.block_table_stride = 4096
    assert lib.hcp_decode_workspace_bytes(ctypes.byref(big)) > 16 * 1024 * 1024
    assert lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(big), None) == SCRATCH_LIMIT
    empty, keep3 = _dec([])
    assert lib.hcp_ring_decode_splitkv_noalloc(ctypes.byref(empty), None) == C.HCP_OK
    assert lib.hcp_ring_decode_splitkv(ctypes.byref(empty), None) == C.HCP_OK


def test_merge_and_cache_entry_points_refuse_bad_arguments(lib):
    o, lse = _addr(1), _addr(2)
    merge = lambda **kw: lib.hcp_merge_attn_states(
        kw.get("out", o), kw.get("odt", C.HCP_BF16), kw.get("ostride", H * D), None, 0,
        o, C.HCP_BF16, H * D, lse, kw.get("plse_stride", 16), o, C.HCP_BF16, H * D, lse, 16,
        kw.get("n", 16), H, D, None)
    assert merge(out=None) == INVALID
    assert merge(odt=9) == UNSUPPORTED
    assert merge(ostride=H * D - 1) == INVALID
    assert merge(plse_stride=15) == INVALID       # LSE rows shorter than the token count
    assert merge(n=0) == C.HCP_OK                 # nothing to merge
    upd = lambda **kw: lib.hcp_kv_cache_update(
        kw.get("key", o), o, kw.get("n", 8), kw.get("kstride", HKV * D), HKV * D, lse, _addr(3), 64, 16,
        HKV, kw.get("d", D), kw.get("dt", C.HCP_BF16), None)
    assert upd(dt=C.HCP_F32) == UNSUPPORTED
    assert upd(d=60) == INVALID                   # rows of 16-byte vectors
    assert upd(key=BASE + 8) == INVALID
    assert upd(kstride=HKV * D - 8) == INVALID
    assert upd(n=0) == C.HCP_OK
