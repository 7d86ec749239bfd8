/*
 * hcp_ring.h - C ABI of the B200 (sm_100a) ring context-parallel attention
 * library (libhcp_ring.so).
 *
 * Plain pointers, sizes and a CUDA stream handle (cudaStream_t passed as
 * void*).  No torch types.  Every tensor pointer is a DEVICE pointer unless a
 * comment says "host".  Every entry point returns an hcp_status; launches are
 * asynchronous on the given stream.
 *
 * Layout conventions (all row-major, innermost dimension last):
 *   q / out        [rows, H, D]     row stride given in elements (>= H*D)
 *   k / v          [rows, Hkv, D]   row stride given in elements (>= Hkv*D)
 *   paged kv cache [num_blocks, Hkv, block_size, 2*D]; K = [..., :D], V = [..., D:]
 *   lse            [H, lse_stride]  float32, natural log
 *
 * Interfaces of the reference plugin (stark-sim/hcp-vllm-plugin) that each
 * entry point replaces are cited per declaration.
 */
#ifndef HCP_RING_H_
#define HCP_RING_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum hcp_status {
  HCP_OK = 0,
  HCP_ERR_INVALID = 1,      /* bad argument (null pointer, inconsistent sizes) */
  HCP_ERR_UNSUPPORTED = 2,  /* shape / dtype / device the kernels do not handle */
  HCP_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed */
  HCP_ERR_DEVICE = 4,       /* a kernel reported a device-side failure (timeout) */
  HCP_ERR_SCRATCH_LIMIT = 5 /* the call needs more fixed scratch than the library holds */
} hcp_status;

typedef enum hcp_dtype { HCP_BF16 = 0, HCP_F16 = 1, HCP_F32 = 2 } hcp_dtype;

/* Limits of the segment lists and extra sources below. */
#define HCP_MAX_ITEM_SEGMENTS 8
#define HCP_MAX_EXT_SOURCES 8

/* Where the keys of one KV segment come from. */
typedef enum hcp_kv_src {
  HCP_SRC_NONE = 0,   /* segment unused */
  HCP_SRC_A = 1,      /* contiguous k_a / v_a rows [start, start+len) */
  HCP_SRC_B = 2,      /* contiguous k_b / v_b rows [start, start+len) */
  HCP_SRC_PAGED = 3,  /* paged cache: key positions [start, start+len) of the
                         sequence in block_table row `paged_req`; start must be
                         a multiple of block_size */
  HCP_SRC_LIST = 4,   /* only in a work item's seg[0] (seg[1] unused): the
                         item's segments are seg_list[start, start+len),
                         at most HCP_MAX_ITEM_SEGMENTS of them */
  HCP_SRC_EXT0 = 16   /* HCP_SRC_EXT0 + i: contiguous rows [start, start+len)
                         of extra source ext[i], i < HCP_MAX_EXT_SOURCES */
} hcp_kv_src;

/* A contiguous K/V source: k and v [rows, Hkv, D], row stride in elements
 * (the same for k and v).  Staged peer chunks are passed as they lie, so
 * several chunks or requests need no concatenation. */
typedef struct hcp_kv_source {
  const void* k;
  const void* v;
  int64_t rows;
  int64_t row_stride;
} hcp_kv_source;

/* One KV segment of a work item.  causal_off < 0: non-causal (every key
 * visible).  causal_off >= 0: key j (segment-relative) is visible to query row
 * i (work-item-relative) iff j <= causal_off + i. */
typedef struct hcp_kv_segment {
  int32_t src;
  int32_t start;
  int32_t len;
  int32_t causal_off;
} hcp_kv_segment;

/* One work item: query rows [q_start, q_start+q_len) attend, with ONE online
 * softmax, over the union of up to two KV segments (typically the transient
 * peer prefix, non-causal, then the local chunk, causal).  Row i writes out row
 * q_start+i and lse column lse_col+i. */
typedef struct hcp_attn_work {
  int32_t q_start;
  int32_t q_len;
  int32_t paged_req;
  int32_t lse_col;
  hcp_kv_segment seg[2];
} hcp_attn_work;

/* Arguments of hcp_ring_attn_fwd.  Unused sources may be NULL. */
typedef struct hcp_fwd_args {
  int32_t dtype;          /* HCP_BF16 or HCP_F16 (q, k, v, cache) */
  int32_t num_heads;      /* H */
  int32_t num_kv_heads;   /* Hkv, H % Hkv == 0 */
  int32_t head_dim;       /* D: 64 or 128 */
  float scale;            /* softmax scale */
  int32_t _pad0;
  const void* q;          int64_t q_rows;  int64_t q_row_stride;
  const void* k_a;        const void* v_a; int64_t rows_a; int64_t a_row_stride;
  const void* k_b;        const void* v_b; int64_t rows_b; int64_t b_row_stride;
  const void* kv_cache;   int64_t num_blocks; int32_t block_size; int32_t _pad1;
  const int32_t* block_table; int64_t block_table_stride; int64_t block_table_rows;
  void* out;              int32_t out_dtype; int32_t _pad2; int64_t out_row_stride;
  float* lse;             int64_t lse_stride;            /* may be NULL */
  /* Optional earlier partial result (O, LSE) over other keys, merged into this
   * result in the epilogue (vLLM merge_attn_states semantics).  merge_o may
   * alias out (same dtype and stride) and merge_lse may alias lse. */
  const void* merge_o;    int32_t merge_o_dtype; int32_t _pad3; int64_t merge_o_row_stride;
  const float* merge_lse; int64_t merge_lse_stride;
  const hcp_attn_work* work;  /* HOST array of num_work items */
  int32_t num_work;
  int32_t _pad4;
  /* Optional: extra contiguous sources (HOST array, <= HCP_MAX_EXT_SOURCES)
   * and the segment lists of HCP_SRC_LIST items (HOST array).  NULL / 0
   * when unused. */
  const hcp_kv_source* ext;   int32_t num_ext;     int32_t _pad5;
  const hcp_kv_segment* seg_list; int32_t num_seg_list; int32_t _pad6;
  /* Sliding window, 0 = none: in every causal segment (causal_off >= 0) a
   * query row at position qpos (causal_off + its row in the item) sees the
   * keys j with qpos - window < j <= qpos; non-causal segments stay fully
   * visible (the reference's _attn_with_lse window, applied to the local
   * passes only: ring_backend.py:786-826). */
  int32_t window;         int32_t _pad7;
} hcp_fwd_args;

/*
 * Fused ring-attention forward: flash attention with per-row LSE over the
 * KV segments of each work item - two inline, or a list of up to
 * HCP_MAX_ITEM_SEGMENTS (GQA, global-offset causal mask, paged or contiguous
 * keys, several contiguous sources) - in one online softmax per row, optional
 * merge into an earlier partial (O, LSE).
 * tcgen05 MMA with TMEM accumulators, TMA-staged tiles.
 *
 * Replaces, in the reference:
 *   ring_attn_with_lse           hcp_vllm_plugin/ring_triton_attn.py:155-207
 *   _ring_fwd_kernel             hcp_vllm_plugin/ring_triton_attn.py:35-152
 *   the per-request loop of HcpRingAttentionImpl.forward (gather, local pass,
 *   peer pass, merge)            hcp_vllm_plugin/ring_backend.py:611-832
 *   _merge / merge_attn_states on the prefill path
 *                                hcp_vllm_plugin/ring_backend.py:339-360
 *   the concatenation of ordered staged prefix chunks (and of several
 *   requests' peers) into one peer segment
 *                                hcp_vllm_plugin/ring_backend.py:751-772
 */
int hcp_ring_attn_fwd(const hcp_fwd_args* args, void* stream);

/*
 * Standalone LSE merge of two partial attentions (vLLM merge_attn_states):
 *   out = (prefix_o * e^{prefix_lse - m} + suffix_o * e^{suffix_lse - m}) / sum
 * with +inf LSE treated as -inf.  o: [T, H, D] (row stride in elements), lse:
 * [H, lse_stride].  out_lse may be NULL.  dtypes: HCP_BF16/HCP_F16/HCP_F32 for
 * o tensors (prefix, suffix and out may differ).
 *
 * Replaces: vLLM merge_attn_states as called by _merge
 * (hcp_vllm_plugin/ring_backend.py:339-360) and _merge_pair
 * (hcp_vllm_plugin/ring_decode.py:46-61).
 */
int hcp_merge_attn_states(void* out, int32_t out_dtype, int64_t out_row_stride,
                          float* out_lse, int64_t out_lse_stride,
                          const void* prefix_o, int32_t prefix_dtype, int64_t prefix_row_stride,
                          const float* prefix_lse, int64_t prefix_lse_stride,
                          const void* suffix_o, int32_t suffix_dtype, int64_t suffix_row_stride,
                          const float* suffix_lse, int64_t suffix_lse_stride,
                          int64_t num_tokens, int32_t num_heads, int32_t head_dim, void* stream);

/* One decode sequence: a single query token (row q_row of q/out) attends the
 * peer keys [peer_start, peer_start+peer_len) of peer_k/peer_v (contiguous)
 * and the local keys [local_start, local_start+local_len) of its paged
 * sequence (block_table row paged_req; local_start a multiple of block_size),
 * all visible (a single query: truncate local_len to causal_offset+1). */
typedef struct hcp_decode_seq {
  int32_t q_row;
  int32_t peer_start;
  int32_t peer_len;
  int32_t paged_req;
  int32_t local_start;
  int32_t local_len;
} hcp_decode_seq;

typedef struct hcp_decode_args {
  int32_t dtype;          /* HCP_BF16 or HCP_F16 */
  int32_t num_heads;      /* H */
  int32_t num_kv_heads;   /* Hkv; H / Hkv <= 16 */
  int32_t head_dim;       /* 64 or 128 */
  float scale;
  int32_t chunk_keys;     /* keys per split-KV chunk; 0 = chosen by the library */
  const void* q;          int64_t q_rows; int64_t q_row_stride;
  const void* peer_k;     const void* peer_v; int64_t peer_rows; int64_t peer_row_stride;
  const void* kv_cache;   int64_t num_blocks; int32_t block_size; int32_t _pad0;
  const int32_t* block_table; int64_t block_table_stride; int64_t block_table_rows;
  void* out;              int32_t out_dtype; int32_t _pad1; int64_t out_row_stride;
  float* lse;             int64_t lse_stride;        /* [H, lse_stride], may be NULL */
  void* workspace;        int64_t workspace_bytes;   /* device scratch, 16-byte aligned */
  const hcp_decode_seq* seqs;  /* HOST array */
  int32_t num_seqs;
  int32_t _pad2;
  /* Optional: extra contiguous peer sources (HOST array, <= HCP_MAX_EXT_SOURCES)
   * and, per sequence, where its peer keys are (HOST array of num_seqs:
   * -1 = peer_k / peer_v, i = ext[i]); NULL / 0 = every sequence uses
   * peer_k / peer_v.  Each request's staged chunk is read as it lies. */
  const hcp_kv_source* ext;   int32_t num_ext;   int32_t _pad3;
  const int32_t* peer_src;
} hcp_decode_args;

/*
 * N-way LSE merge of per-shard partials: states_o [num_states, T, H, D] fp32
 * and states_lse [num_states, H, T] fp32 (natural log; -inf or +inf = empty
 * partial), both contiguous -> out [T, H, D] (row stride out_row_stride,
 * dtype out_dtype) and, if out_lse != NULL, the merged lse [H, T] (row
 * stride out_lse_stride).  head_dim <= 256.
 *
 * Replaces: the decode ring's accumulator chain - _merge_pair
 * (hcp_vllm_plugin/ring_decode.py:46-61) applied once per hop in
 * RingDecodeNode.handle_packet (ring_decode.py:187-259) - with one launch
 * over all shards' partials.
 */
int hcp_merge_attn_states_n(void* out, int32_t out_dtype, int64_t out_row_stride, float* out_lse,
                            int64_t out_lse_stride, const float* states_o, const float* states_lse,
                            int32_t num_states, int64_t num_tokens, int32_t num_heads,
                            int32_t head_dim, void* stream);

/*
 * Split-KV decode over a paged local segment plus a contiguous peer segment,
 * batch-merged (all sequences in one launch), LSE-merged across chunks.
 * Needs hcp_decode_workspace_bytes(args) bytes of device workspace.
 *
 * Replaces, in the reference: the decode-time use of ring_attn_with_lse over
 * the local segment and the peer chunks plus the LSE merge of the partials
 * (hcp_vllm_plugin/ring_backend.py:638-727 local partial,
 * hcp_vllm_plugin/ring_decode.py:187-259 peer partials and _merge_pair
 * :46-61), and the per-request decode passes of HcpRingAttentionImpl.forward
 * (ring_backend.py:611-832 with tq == 1).
 */
int hcp_ring_decode_splitkv(const hcp_decode_args* args, void* stream);

/* Workspace bytes hcp_ring_decode_splitkv needs for these arguments
 * (-1 when the arguments are invalid).  No counterpart in the reference. */
int64_t hcp_decode_workspace_bytes(const hcp_decode_args* args);

/*
 * Scatter new K/V rows into the paged cache [num_blocks, Hkv, block_size, 2*D]
 * at slot_mapping (int64, device; slot < 0 = padding, skipped).
 * key/value: [num_tokens, Hkv, D] with the given row strides (elements).
 *
 * Replaces: HcpRingAttentionImpl.do_kv_cache_update
 * (hcp_vllm_plugin/ring_backend.py:501-539, torch advanced-index scatter
 * :532-537) in the [num_blocks, Hkv, block_size, 2*D] layout of
 * hcp_vllm_plugin/file_connector.py:175-179.
 */
int hcp_kv_cache_update(const void* key, const void* value, int64_t num_tokens,
                        int64_t key_row_stride, int64_t value_row_stride,
                        const int64_t* slot_mapping, void* kv_cache, int64_t num_blocks,
                        int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                        int32_t dtype, void* stream);

/*
 * Gather the K/V rows of slot_mapping (int64, device) out of the paged cache
 * [num_blocks, Hkv, block_size, 2*D] into key/value [num_tokens, Hkv, D]
 * (given row strides, elements).  Rows of slots < 0 or beyond the cache are
 * written as zeros.
 *
 * Replaces: HcpRingKvConnector.save_kv_layer's pool -> chunk extraction
 * (hcp_vllm_plugin/ring_connector.py:890-919, torch advanced index
 * kv_layer[block_idxs, :, offsets] :909-910) in the
 * [num_blocks, Hkv, block_size, 2*D] layout.
 */
int hcp_kv_cache_gather(const void* kv_cache, int64_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, const int64_t* slot_mapping,
                        int64_t num_tokens, void* key, void* value, int64_t key_row_stride,
                        int64_t value_row_stride, int32_t dtype, void* stream);

/* Bytes of the fixed device array behind hcp_ring_decode_splitkv_noalloc. */
#define HCP_DECODE_NOALLOC_SCRATCH_BYTES (16LL * 1024 * 1024)

/*
 * Split-KV decode that allocates nothing.  Same arguments, kernels and
 * results as hcp_ring_decode_splitkv, except that args->workspace and
 * args->workspace_bytes are ignored: the per-chunk partials go to a fixed
 * 16 MiB array that is part of this library's device image.
 *
 * For callers that cannot allocate device memory when they decode: a host
 * that talks to the library only through this C ABI and owns no device
 * allocator, or a serving engine that has already handed (almost) all free
 * HBM to its paged KV cache, where an extra allocation at decode time can
 * fail or break the memory budget it planned.
 *
 * Limits and rules:
 *  - every GPU that loads the library holds the 16 MiB array until the
 *    process exits;
 *  - a call whose partials need more than HCP_DECODE_NOALLOC_SCRATCH_BYTES
 *    (hcp_decode_workspace_bytes(args)) returns HCP_ERR_SCRATCH_LIMIT and
 *    launches nothing; a larger args->chunk_keys needs fewer partials;
 *  - the first call in a CUDA context looks up the array's device address
 *    in that context (once per context, with it current); make that first
 *    call before any stream capture begins;
 *  - all calls share the one array and it keeps the last call's contents;
 *    nothing in it has to start at zero (each call writes every partial it
 *    reads), but calls that overlap on the GPU (other streams, other host
 *    threads) race on it: serialise them.
 * No counterpart in the reference.
 */
int hcp_ring_decode_splitkv_noalloc(const hcp_decode_args* args, void* stream);

/*
 * In-box chunk transport (CUDA IPC + copy engine over NVLink).
 *
 * hcp_ipc_export: IPC handle (HCP_IPC_HANDLE_BYTES bytes) of the device
 *   allocation containing ptr, and ptr's byte offset inside it.
 * hcp_ipc_open: map a handle exported by another process into this process
 *   for `device` (peer access enabled lazily); *base_out = allocation base.
 * hcp_ipc_close: unmap a base returned by hcp_ipc_open.
 * hcp_peer_copy: stream-ordered copy of `bytes` between any two device
 *   pointers of the box (local or mapped from a peer GPU).
 *
 * Replace: the HTTP prefill-KV store of HcpRingKvConnector
 * (hcp_vllm_plugin/ring_connector.py:386-548: _start_http_server, _fetch,
 * _remote_exists) for producers and consumers inside one box; the _READY
 * marker (ring_connector.py:547-549, 777-792, 921-937) carries the handle.
 */
#define HCP_IPC_HANDLE_BYTES 64
int hcp_ipc_export(const void* ptr, uint8_t* handle_out, int64_t* offset_out);
int hcp_ipc_open(const uint8_t* handle, int32_t device, void** base_out);
int hcp_ipc_close(void* base);
int hcp_peer_copy(void* dst, const void* src, int64_t bytes, void* stream);

/*
 * Device-side status word shared by all kernels of the library on the
 * current device: 0 when no kernel reported a failure, else the first
 * failure code (bounded waits that ran out).  Synchronises the device.
 * hcp_reset_device_status clears it.  No counterpart in the reference (its
 * Triton launch raises in Python).
 */
int hcp_get_device_status(int32_t* status_out);
int hcp_reset_device_status(void);

/*
 * Stream-ordered copy of the device status word into host memory (use pinned
 * memory for a copy that does not block): the value is valid once the work
 * queued on `stream` before this call has finished.  Lets a serving loop
 * notice a device-side failure at its next synchronisation without adding
 * one.  No counterpart in the reference (its launch errors raise in Python,
 * hcp_vllm_plugin/ring_backend.py:333-336).
 */
int hcp_device_status_async(int32_t* host_out, void* stream);

/*
 * Failure-path self-test: launches one thread that waits, through the
 * kernels' own bounded mbarrier wait, on a barrier nothing arrives on, for
 * timeout_ns (at most 2 s).  The wait runs out, the device status becomes
 * 0x1ff and the kernel returns normally; *waited_out = 0 confirms that the
 * wait gave up.  Synchronises the device.  No counterpart in the reference.
 */
int hcp_selftest_bounded_wait(int64_t timeout_ns, int32_t* waited_out);

/* Library version string (static storage). */
const char* hcp_version(void);

#ifdef __cplusplus
}
#endif

#endif /* HCP_RING_H_ */
