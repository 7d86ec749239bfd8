// libhcp_ring.so: the C ABI declared in include/hcp_ring.h.
//
// Host side of the library: argument validation, TMA tensor-map encoding,
// work scheduling (heaviest query tiles first, GQA heads of one KV head on
// neighbouring CTAs) and kernel launches.  All kernels live in this single
// translation unit so they share one device status word.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "hcp_ring.h"
#include "ring_fwd.cuh"
#include "ring_fwd_persistent.cuh"
#include "decode.cuh"
#include "cache.cuh"
#include "merge.cuh"

namespace hcp {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernels launch on the current device.  A stream that belongs to another
// device is refused (HCP_ERR_INVALID) instead of receiving kernels whose
// addresses and tensor maps were made for that other device.  0, 1 and 2 are
// the runtime's default / legacy / per-thread streams of the current device.
bool stream_on_current_device(void* stream) {
  if (reinterpret_cast<uintptr_t>(stream) <= 2) return true;
  int cur = -1, sdev = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return false;
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return cur == sdev;
}

// log2(n) when n is a power of two, else -1
int pow2_shift(int n) {
  if (n <= 0 || (n & (n - 1)) != 0) return -1;
  int s = 0;
  while ((1 << s) != n) ++s;
  return s;
}

// 128-byte-swizzled tiled map over a 16-bit tensor.  dims/box innermost first;
// strides (bytes) for dims 1..rank-1.
bool encode_map(CUtensorMap* m, bool f16, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5] = {1, 1, 1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides[i];
  const CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// [rows, heads, D] view with the given row stride (elements).
bool encode_rows_heads(CUtensorMap* m, bool f16, const void* base, int64_t rows, int heads, int D,
                       int64_t row_stride) {
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(heads),
                            static_cast<uint64_t>(std::max<int64_t>(rows, 1))};
  const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(row_stride) * 2};
  const uint32_t box[3] = {64, 1, 128};
  return encode_map(m, f16, 3, base, dims, strides, box);
}

std::mutex g_attr_mu;
bool g_attr_done[2][2][8][64];  // variants 0-6, and 7 for the LIST kernel
bool g_dec_attr_done[2][2][64];

// Forward kernel variant (read once per process): HCP_FWD_VARIANT=0..7, or
// HCP_FWD_NAMED_BARRIERS=1 (1) / HCP_FWD_POLY_EXP2=1 (2); default 5, the
// fastest measured (16k / 32k causal launches: +2.2% / +2.3% over 0).  0 -
// the mbarrier MMA issuer on 320 threads; 1 - the named-barrier issuer; 2 -
// 1 with a quarter of the exponentials on the FMA pipe; 3, 4, 5 - the
// mbarrier issuer on 384 threads with the registers split by setmaxnreg and
// packed f32x2 softmax math, with a quarter, three eighths or none of the
// exponentials on the FMA pipe; 6 - the named-barrier issuer on 384 threads
// with the setmaxnreg split; 7 - variant 5 as a persistent kernel, one CTA
// per SM running a static list of 256-row blocks (ring_fwd_persistent.cuh).
int fwd_variant() {
  static const int v = [] {
    auto on = [](const char* name) {
      const char* e = std::getenv(name);
      return e != nullptr && e[0] == '1';
    };
    const char* e = std::getenv("HCP_FWD_VARIANT");
    if (e != nullptr && e[0] >= '0' && e[0] <= '7' && e[1] == 0) return e[0] - '0';
    return on("HCP_FWD_POLY_EXP2") ? 2 : on("HCP_FWD_NAMED_BARRIERS") ? 1 : 5;
  }();
  return v;
}

template <int D, bool F16, int V, bool LIST = false>
int launch_fwd(const FwdParams& p, int grid, cudaStream_t st) {
  constexpr int smem = fwd_smem_bytes<D>();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HCP_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    bool& done = g_attr_done[D == 128][F16][LIST ? 7 : V][dev];
    if (!done) {
      if (cudaFuncSetAttribute(ring_fwd_kernel<D, F16, V, LIST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return HCP_ERR_CUDA;
      if (V >= 3) {
        // setmaxnreg.inc waits until the other warpgroups have released what
        // it asks for: the split must fit the registers the launch holds
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, ring_fwd_kernel<D, F16, V, LIST>) != cudaSuccess) return HCP_ERR_CUDA;
        if (2 * 128 * kRegsSoftmaxWide + 128 * kRegsProducerWide > kThreadsWide * fa.numRegs)
          return HCP_ERR_UNSUPPORTED;
      }
      done = true;
    }
  }
  ring_fwd_kernel<D, F16, V, LIST><<<grid, V >= 3 ? kThreadsWide : kThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

bool g_persist_attr_done[2][2][64];
int g_sm_count[64];

// Variant 7: one CTA per SM (at most one per block x head), each running its
// share of the blocks in the persistent kernel's static order.
template <int D, bool F16>
int launch_fwd_persistent(const FwdParams& p, int jobs, cudaStream_t st) {
  constexpr int smem = fwd_persistent_smem_bytes<D>();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HCP_ERR_CUDA;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    if (!g_persist_attr_done[D == 128][F16][dev]) {
      if (cudaFuncSetAttribute(ring_fwd_persistent_kernel<D, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return HCP_ERR_CUDA;
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, ring_fwd_persistent_kernel<D, F16>) != cudaSuccess) return HCP_ERR_CUDA;
      if (2 * 128 * kRegsSoftmaxWide + 128 * kRegsProducerWide > kThreadsWide * fa.numRegs)
        return HCP_ERR_UNSUPPORTED;
      int n = 0;
      if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return HCP_ERR_CUDA;
      g_sm_count[dev] = n;
      g_persist_attr_done[D == 128][F16][dev] = true;
    }
    sms = g_sm_count[dev];
  }
  const int grid = std::min(jobs, sms);
  ring_fwd_persistent_kernel<D, F16><<<grid, kThreadsWide, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

template <int D, bool F16>
int launch_fwd(const FwdParams& p, int grid, cudaStream_t st, bool list) {
  // items of more than two segments: the segment-table kernel (mbarrier issuer)
  if (list) return launch_fwd<D, F16, 0, true>(p, grid, st);
  switch (fwd_variant()) {
    case 7: return launch_fwd_persistent<D, F16>(p, grid, st);
    case 1: return launch_fwd<D, F16, 1>(p, grid, st);
    case 2: return launch_fwd<D, F16, 2>(p, grid, st);
    case 3: return launch_fwd<D, F16, 3>(p, grid, st);
    case 4: return launch_fwd<D, F16, 4>(p, grid, st);
    case 6: return launch_fwd<D, F16, 6>(p, grid, st);
    case 0: return launch_fwd<D, F16, 0>(p, grid, st);
    default: return launch_fwd<D, F16, 5>(p, grid, st);
  }
}

int64_t segment_cost(const hcp_kv_segment& s, int q_len) {
  if (s.src == HCP_SRC_NONE || s.len <= 0) return 0;
  if (s.causal_off < 0) return static_cast<int64_t>(s.len) * q_len;
  // average visible keys over the rows
  const int64_t first = std::min<int64_t>(s.len, s.causal_off + 1);
  const int64_t last = std::min<int64_t>(s.len, static_cast<int64_t>(s.causal_off) + q_len);
  return (first + last) * q_len / 2;
}

int validate_segment(const hcp_fwd_args* a, const hcp_attn_work& w, const hcp_kv_segment& s) {
  if (s.src == HCP_SRC_NONE || s.len == 0) return HCP_OK;
  if (s.len < 0 || s.start < 0) return HCP_ERR_INVALID;
  switch (s.src) {
    case HCP_SRC_A:
      if (a->k_a == nullptr || a->v_a == nullptr) return HCP_ERR_INVALID;
      if (static_cast<int64_t>(s.start) + s.len > a->rows_a) return HCP_ERR_INVALID;
      return HCP_OK;
    case HCP_SRC_B:
      if (a->k_b == nullptr || a->v_b == nullptr) return HCP_ERR_INVALID;
      if (static_cast<int64_t>(s.start) + s.len > a->rows_b) return HCP_ERR_INVALID;
      return HCP_OK;
    case HCP_SRC_PAGED:
      if (a->kv_cache == nullptr || a->block_table == nullptr) return HCP_ERR_INVALID;
      if (w.paged_req < 0 || w.paged_req >= a->block_table_rows) return HCP_ERR_INVALID;
      if (s.start % a->block_size != 0) return HCP_ERR_UNSUPPORTED;
      if (static_cast<int64_t>(s.start) + s.len > a->block_table_stride * a->block_size)
        return HCP_ERR_INVALID;
      return HCP_OK;
    default:
      if (s.src >= HCP_SRC_EXT0 && s.src < HCP_SRC_EXT0 + a->num_ext) {
        const hcp_kv_source& e = a->ext[s.src - HCP_SRC_EXT0];
        if (static_cast<int64_t>(s.start) + s.len > e.rows) return HCP_ERR_INVALID;
        return HCP_OK;
      }
      return HCP_ERR_INVALID;
  }
}

template <int D, bool F16>
int launch_decode(const DecodeParams& p, int units, int hkv, cudaStream_t st) {
  constexpr int smem = DecSmem<D>::kBytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HCP_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    bool& done = g_dec_attr_done[D == 128][F16][dev];
    if (!done) {
      if (cudaFuncSetAttribute(decode_splitkv_kernel<D, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return HCP_ERR_CUDA;
      done = true;
    }
  }
  decode_splitkv_kernel<D, F16><<<dim3(units, hkv), kDecThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

// Keys per split-KV chunk: enough chunks for ~4 waves of 2 CTAs per SM.
int decode_chunk_keys(const hcp_decode_args* a) {
  if (a->chunk_keys > 0) return ((a->chunk_keys + kDecTileKeys - 1) / kDecTileKeys) * kDecTileKeys;
  int64_t total = 0;
  for (int i = 0; i < a->num_seqs; ++i) total += a->seqs[i].peer_len + a->seqs[i].local_len;
  const int64_t want_units = std::max<int64_t>(1, (8 * 148) / std::max(1, a->num_kv_heads));
  int64_t c = (total + want_units - 1) / want_units;
  c = ((c + kDecTileKeys - 1) / kDecTileKeys) * kDecTileKeys;
  return static_cast<int>(std::min<int64_t>(8192, std::max<int64_t>(256, c)));
}

int64_t decode_units(const hcp_decode_args* a, int chunk) {
  int64_t u = 0;
  for (int i = 0; i < a->num_seqs; ++i) {
    const int64_t pu = (a->seqs[i].peer_len + chunk - 1) / chunk;
    const int64_t lu = (a->seqs[i].local_len + chunk - 1) / chunk;
    u += std::max<int64_t>(1, pu + lu);
  }
  return u;
}

int64_t workspace_need(const hcp_decode_args* a, int chunk) {
  const int64_t units = decode_units(a, chunk);
  return units * a->num_heads * (static_cast<int64_t>(a->head_dim) + 1) * 4;
}

}  // namespace
}  // namespace hcp

using namespace hcp;

extern "C" int hcp_ring_attn_fwd(const hcp_fwd_args* a, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  if (a == nullptr) return HCP_ERR_INVALID;
  if (a->dtype != HCP_BF16 && a->dtype != HCP_F16) return HCP_ERR_UNSUPPORTED;
  const bool f16 = a->dtype == HCP_F16;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim;
  if (H <= 0 || Hkv <= 0 || H % Hkv != 0) return HCP_ERR_INVALID;
  if (D != 64 && D != 128) return HCP_ERR_UNSUPPORTED;
  if (!(a->scale > 0.f) || !std::isfinite(a->scale)) return HCP_ERR_INVALID;
  if (a->num_work < 0 || (a->num_work > 0 && a->work == nullptr)) return HCP_ERR_INVALID;
  if (a->window < 0) return HCP_ERR_INVALID;
  if (a->q == nullptr || a->out == nullptr || a->q_rows < 0) return HCP_ERR_INVALID;
  if (a->q_row_stride < static_cast<int64_t>(H) * D || a->out_row_stride < static_cast<int64_t>(H) * D)
    return HCP_ERR_INVALID;
  if (a->out_dtype != a->dtype && a->out_dtype != HCP_F32) return HCP_ERR_UNSUPPORTED;
  if (!aligned16(a->q) || !aligned16(a->out) || (a->q_row_stride % 8) != 0 ||
      (a->out_row_stride % 8) != 0)
    return HCP_ERR_INVALID;
  if (a->merge_lse != nullptr) {
    if (a->merge_o == nullptr || !aligned16(a->merge_o)) return HCP_ERR_INVALID;
    if (a->merge_o_dtype != a->dtype && a->merge_o_dtype != HCP_F32) return HCP_ERR_UNSUPPORTED;
    if (a->merge_o_row_stride < static_cast<int64_t>(H) * D || (a->merge_o_row_stride % 8) != 0)
      return HCP_ERR_INVALID;
  }
  const bool want_a = a->k_a != nullptr, want_b = a->k_b != nullptr, want_paged = a->kv_cache != nullptr;
  const int64_t kv_row = static_cast<int64_t>(Hkv) * D;
  if (want_a && (a->v_a == nullptr || a->rows_a <= 0 || a->a_row_stride < kv_row ||
                 (a->a_row_stride % 8) != 0 || !aligned16(a->k_a) || !aligned16(a->v_a)))
    return HCP_ERR_INVALID;
  if (want_b && (a->v_b == nullptr || a->rows_b <= 0 || a->b_row_stride < kv_row ||
                 (a->b_row_stride % 8) != 0 || !aligned16(a->k_b) || !aligned16(a->v_b)))
    return HCP_ERR_INVALID;
  if (want_paged) {
    const int bs = a->block_size;
    if (bs != 16 && bs != 32 && bs != 64 && bs != 128) return HCP_ERR_UNSUPPORTED;
    if (a->num_blocks <= 0 || a->num_blocks >= (1ll << 31) || a->block_table == nullptr ||
        a->block_table_stride <= 0 || a->block_table_rows <= 0 || !aligned16(a->kv_cache))
      return HCP_ERR_INVALID;
  }

  if (a->num_ext < 0 || a->num_ext > HCP_MAX_EXT_SOURCES || (a->num_ext > 0 && a->ext == nullptr) ||
      a->num_seg_list < 0 || (a->num_seg_list > 0 && a->seg_list == nullptr))
    return HCP_ERR_INVALID;
  for (int i = 0; i < a->num_ext; ++i) {
    const hcp_kv_source& e = a->ext[i];
    if (e.k == nullptr || e.v == nullptr || e.rows <= 0 || e.row_stride < kv_row || (e.row_stride % 8) != 0 ||
        !aligned16(e.k) || !aligned16(e.v))
      return HCP_ERR_INVALID;
  }

  // Validate and order the work: most expensive items first.  Each item is
  // kept with its segments (the two inline ones, or its list).
  std::vector<hcp_attn_work> items;
  std::vector<std::vector<hcp_kv_segment>> item_segs;
  items.reserve(a->num_work);
  std::vector<int64_t> cost;
  for (int i = 0; i < a->num_work; ++i) {
    const hcp_attn_work& w = a->work[i];
    std::vector<hcp_kv_segment> sg;
    if (w.seg[0].src == HCP_SRC_LIST) {
      if (w.seg[1].src != HCP_SRC_NONE || w.seg[0].start < 0 || w.seg[0].len < 0 ||
          w.seg[0].len > HCP_MAX_ITEM_SEGMENTS || static_cast<int64_t>(w.seg[0].start) + w.seg[0].len > a->num_seg_list)
        return HCP_ERR_INVALID;
      sg.assign(a->seg_list + w.seg[0].start, a->seg_list + w.seg[0].start + w.seg[0].len);
      while (sg.size() < 2) sg.push_back(hcp_kv_segment{HCP_SRC_NONE, 0, 0, 0});
    } else {
      sg.assign(w.seg, w.seg + 2);
    }
    if (w.q_len < 0 || w.q_start < 0 || static_cast<int64_t>(w.q_start) + w.q_len > a->q_rows)
      return HCP_ERR_INVALID;
    if (a->lse != nullptr && (w.lse_col < 0 || static_cast<int64_t>(w.lse_col) + w.q_len > a->lse_stride))
      return HCP_ERR_INVALID;
    if (a->merge_lse != nullptr &&
        (w.lse_col < 0 || static_cast<int64_t>(w.lse_col) + w.q_len > a->merge_lse_stride))
      return HCP_ERR_INVALID;
    for (const hcp_kv_segment& sgi : sg) {
      if (sgi.src == HCP_SRC_LIST) return HCP_ERR_INVALID;
      const int rc = validate_segment(a, w, sgi);
      if (rc != HCP_OK) return rc;
    }
    if (w.q_len == 0) continue;
    items.push_back(w);
    item_segs.push_back(std::move(sg));
  }
  if (items.empty()) return HCP_OK;
  // When every 256-row block of every item fits one launch as an item of its
  // own, split them: the launch then runs the blocks in one heaviest-first
  // order across requests (with whole items, a request's light blocks ran
  // before the next request's heavy ones and lengthened the last wave).  A
  // block starting at row r0 of its item sees its causal segments at offset
  // causal_off + r0; the results are those of the whole item.
  {
    int64_t blocks = 0, segs = 0;
    bool fits = true;
    for (size_t i = 0; i < items.size(); ++i) {
      const int64_t nb = (items[i].q_len + kCtaRows - 1) / kCtaRows;
      blocks += nb;
      segs += nb * static_cast<int64_t>(item_segs[i].size());
      for (const hcp_kv_segment& s : item_segs[i])
        if (s.causal_off >= 0 && static_cast<int64_t>(s.causal_off) + items[i].q_len > INT32_MAX) fits = false;
    }
    if (fits && items.size() > 1 && blocks > static_cast<int64_t>(items.size()) && blocks <= kMaxWork &&
        segs <= kMaxSegs) {
      std::vector<hcp_attn_work> split;
      std::vector<std::vector<hcp_kv_segment>> split_segs;
      for (size_t i = 0; i < items.size(); ++i) {
        for (int r0 = 0; r0 < items[i].q_len; r0 += kCtaRows) {
          hcp_attn_work w = items[i];
          w.q_start += r0;
          w.lse_col += r0;
          w.q_len = std::min(kCtaRows, items[i].q_len - r0);
          std::vector<hcp_kv_segment> sg = item_segs[i];
          for (hcp_kv_segment& s : sg)
            if (s.src != HCP_SRC_NONE && s.causal_off >= 0) s.causal_off += r0;
          split.push_back(w);
          split_segs.push_back(std::move(sg));
        }
      }
      items.swap(split);
      item_segs.swap(split_segs);
    }
  }
  std::vector<int> order(items.size());
  for (size_t i = 0; i < items.size(); ++i) {
    order[i] = static_cast<int>(i);
    int64_t c = 0;
    for (const hcp_kv_segment& sgi : item_segs[i]) c += segment_cost(sgi, items[i].q_len);
    cost.push_back(c);
  }
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return cost[x] > cost[y]; });

  FwdParams p;
  std::memset(&p, 0, sizeof(p));
  if (!encode_rows_heads(&p.tm_q, f16, a->q, a->q_rows, H, D, a->q_row_stride)) return HCP_ERR_CUDA;
  p.tm_ka = p.tm_va = p.tm_kb = p.tm_vb = p.tm_cache = p.tm_q;  // placeholders for absent sources
  if (want_a && (!encode_rows_heads(&p.tm_ka, f16, a->k_a, a->rows_a, Hkv, D, a->a_row_stride) ||
                 !encode_rows_heads(&p.tm_va, f16, a->v_a, a->rows_a, Hkv, D, a->a_row_stride)))
    return HCP_ERR_CUDA;
  if (want_b && (!encode_rows_heads(&p.tm_kb, f16, a->k_b, a->rows_b, Hkv, D, a->b_row_stride) ||
                 !encode_rows_heads(&p.tm_vb, f16, a->v_b, a->rows_b, Hkv, D, a->b_row_stride)))
    return HCP_ERR_CUDA;
  for (int i = 0; i < kMaxExt; ++i) p.tm_ek[i] = p.tm_ev[i] = p.tm_q;
  for (int i = 0; i < a->num_ext; ++i) {
    const hcp_kv_source& e = a->ext[i];
    if (!encode_rows_heads(&p.tm_ek[i], f16, e.k, e.rows, Hkv, D, e.row_stride) ||
        !encode_rows_heads(&p.tm_ev[i], f16, e.v, e.rows, Hkv, D, e.row_stride))
      return HCP_ERR_CUDA;
  }
  if (want_paged) {
    const uint64_t bs = static_cast<uint64_t>(a->block_size);
    const uint64_t dims[4] = {static_cast<uint64_t>(2 * D), bs, static_cast<uint64_t>(Hkv),
                              static_cast<uint64_t>(a->num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(2 * D) * 2, bs * 2 * D * 2,
                                 static_cast<uint64_t>(Hkv) * bs * 2 * D * 2};
    const uint32_t box[4] = {64, static_cast<uint32_t>(bs), 1, 1};
    if (!encode_map(&p.tm_cache, f16, 4, a->kv_cache, dims, strides, box)) return HCP_ERR_CUDA;
  }
  p.block_table = a->block_table;
  p.bt_stride = a->block_table_stride;
  p.bt_rows = a->block_table_rows;
  p.num_blocks = a->num_blocks;
  p.out = a->out;
  p.out_row_stride = a->out_row_stride;
  p.out_f32 = a->out_dtype == HCP_F32;
  p.lse = a->lse;
  p.lse_stride = a->lse_stride;
  p.merge_o = a->merge_o;
  p.merge_o_row_stride = a->merge_o_row_stride;
  p.merge_o_f32 = a->merge_o_dtype == HCP_F32;
  p.merge_lse = a->merge_lse;
  p.merge_lse_stride = a->merge_lse_stride;
  p.num_heads = H;
  p.group = H / Hkv;
  p.block_size = want_paged ? a->block_size : 16;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.window = a->window;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (size_t base = 0; base < order.size();) {
    // one launch: up to kMaxWork items whose segments fit kMaxSegs
    int n = 0, nseg = 0, tiles = 0;
    bool list = false;
    while (base + n < order.size() && n < kMaxWork) {
      const int idx = order[base + n];
      const auto& sg = item_segs[idx];
      if (nseg + static_cast<int>(sg.size()) > kMaxSegs) break;
      const hcp_attn_work& w = items[idx];
      list = list || sg.size() > 2;
      FwdItem& it = p.work[n];
      it.q_start = w.q_start;
      it.q_len = w.q_len;
      it.paged_req = w.paged_req;
      it.lse_col = w.lse_col;
      it.seg_first = nseg;
      it.seg_count = static_cast<int>(sg.size());
      for (const hcp_kv_segment& sgi : sg) p.segs[nseg++] = sgi;
      p.tile_off[n] = tiles;
      tiles += (w.q_len + kCtaRows - 1) / kCtaRows;
      ++n;
    }
    base += n;
    p.tile_off[n] = tiles;
    p.num_work = n;
    p.total_tiles = tiles;
    const int64_t grid = static_cast<int64_t>(tiles) * H;
    if (grid <= 0) continue;
    if (grid > 0x7fffffff) return HCP_ERR_UNSUPPORTED;
    int rc;
    if (D == 128) rc = f16 ? launch_fwd<128, true>(p, static_cast<int>(grid), st, list)
                           : launch_fwd<128, false>(p, static_cast<int>(grid), st, list);
    else rc = f16 ? launch_fwd<64, true>(p, static_cast<int>(grid), st, list)
                  : launch_fwd<64, false>(p, static_cast<int>(grid), st, list);
    if (rc != HCP_OK) return rc;
  }
  return HCP_OK;
}

extern "C" int hcp_merge_attn_states(void* out, int32_t out_dtype, int64_t out_row_stride,
                                     float* out_lse, int64_t out_lse_stride, const void* prefix_o,
                                     int32_t prefix_dtype, int64_t prefix_row_stride,
                                     const float* prefix_lse, int64_t prefix_lse_stride,
                                     const void* suffix_o, int32_t suffix_dtype,
                                     int64_t suffix_row_stride, const float* suffix_lse,
                                     int64_t suffix_lse_stride, int64_t num_tokens,
                                     int32_t num_heads, int32_t head_dim, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  auto ok_dt = [](int dt) { return dt == HCP_BF16 || dt == HCP_F16 || dt == HCP_F32; };
  if (out == nullptr || prefix_o == nullptr || suffix_o == nullptr || prefix_lse == nullptr ||
      suffix_lse == nullptr)
    return HCP_ERR_INVALID;
  if (!ok_dt(out_dtype) || !ok_dt(prefix_dtype) || !ok_dt(suffix_dtype)) return HCP_ERR_UNSUPPORTED;
  if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0) return HCP_ERR_INVALID;
  const int64_t row = static_cast<int64_t>(num_heads) * head_dim;
  if (out_row_stride < row || prefix_row_stride < row || suffix_row_stride < row)
    return HCP_ERR_INVALID;
  if (prefix_lse_stride < num_tokens || suffix_lse_stride < num_tokens ||
      (out_lse != nullptr && out_lse_stride < num_tokens))
    return HCP_ERR_INVALID;
  if (num_tokens == 0) return HCP_OK;
  MergeParams p;
  p.out = out;
  p.pre = prefix_o;
  p.suf = suffix_o;
  p.out_lse = out_lse;
  p.pre_lse = prefix_lse;
  p.suf_lse = suffix_lse;
  p.out_stride = out_row_stride;
  p.pre_stride = prefix_row_stride;
  p.suf_stride = suffix_row_stride;
  p.out_lse_stride = out_lse_stride;
  p.pre_lse_stride = prefix_lse_stride;
  p.suf_lse_stride = suffix_lse_stride;
  p.num_tokens = num_tokens;
  p.num_heads = num_heads;
  p.head_dim = head_dim;
  p.out_dt = out_dtype;
  p.pre_dt = prefix_dtype;
  p.suf_dt = suffix_dtype;
  const int64_t warps = num_tokens * num_heads;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return HCP_ERR_UNSUPPORTED;
  merge_states_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

extern "C" int hcp_merge_attn_states_n(void* out, int32_t out_dtype, int64_t out_row_stride,
                                       float* out_lse, int64_t out_lse_stride, const float* states_o,
                                       const float* states_lse, int32_t num_states, int64_t num_tokens,
                                       int32_t num_heads, int32_t head_dim, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  if (out == nullptr || states_o == nullptr || states_lse == nullptr) return HCP_ERR_INVALID;
  if (out_dtype != HCP_BF16 && out_dtype != HCP_F16 && out_dtype != HCP_F32) return HCP_ERR_UNSUPPORTED;
  if (num_states <= 0 || num_tokens < 0 || num_heads <= 0 || head_dim <= 0) return HCP_ERR_INVALID;
  if (head_dim > 256) return HCP_ERR_UNSUPPORTED;
  if (out_row_stride < static_cast<int64_t>(num_heads) * head_dim ||
      (out_lse != nullptr && out_lse_stride < num_tokens))
    return HCP_ERR_INVALID;
  if (num_tokens == 0) return HCP_OK;
  MergeNParams p;
  p.out = out;
  p.out_lse = out_lse;
  p.states_o = states_o;
  p.states_lse = states_lse;
  p.out_stride = out_row_stride;
  p.out_lse_stride = out_lse_stride;
  p.num_tokens = num_tokens;
  p.num_heads = num_heads;
  p.head_dim = head_dim;
  p.num_states = num_states;
  p.out_dt = out_dtype;
  p.vec_ok = aligned16(states_o) &&
             (out_dtype != HCP_F32 || (aligned16(out) && (out_row_stride % 4) == 0)) ? 1 : 0;
  const int64_t warps = num_tokens * num_heads;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffff) return HCP_ERR_UNSUPPORTED;
  merge_states_n_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

extern "C" int hcp_get_device_status(int32_t* status_out) {
  if (status_out == nullptr) return HCP_ERR_INVALID;
  if (cudaDeviceSynchronize() != cudaSuccess) return HCP_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return HCP_ERR_CUDA;
  *status_out = v;
  return HCP_OK;
}

extern "C" int hcp_device_status_async(int32_t* host_out, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  if (host_out == nullptr) return HCP_ERR_INVALID;
  return cudaMemcpyFromSymbolAsync(host_out, g_device_status, sizeof(int), 0, cudaMemcpyDeviceToHost,
                                   static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? HCP_OK
             : HCP_ERR_CUDA;
}

extern "C" int hcp_reset_device_status(void) {
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess) return HCP_ERR_CUDA;
  return cudaDeviceSynchronize() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

extern "C" int hcp_selftest_bounded_wait(int64_t timeout_ns, int32_t* waited_out) {
  if (timeout_ns <= 0 || timeout_ns > 2000000000ll || waited_out == nullptr) return HCP_ERR_INVALID;
  int* d = nullptr;
  if (cudaMalloc(&d, sizeof(int)) != cudaSuccess) return HCP_ERR_CUDA;
  bounded_wait_selftest_kernel<<<1, 32>>>(static_cast<uint64_t>(timeout_ns), d);
  int r = -1;
  const bool ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess &&
                  cudaMemcpy(&r, d, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess;
  cudaFree(d);
  if (!ok) return HCP_ERR_CUDA;
  *waited_out = r;  // 0: the wait ran out as intended
  return HCP_OK;
}

extern "C" const char* hcp_version(void) { return "hcp_ring 0.1.0 (sm_100a)"; }

namespace {
int validate_decode(const hcp_decode_args* a) {
  if (a == nullptr) return HCP_ERR_INVALID;
  if (a->dtype != HCP_BF16 && a->dtype != HCP_F16) return HCP_ERR_UNSUPPORTED;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim;
  if (H <= 0 || Hkv <= 0 || H % Hkv != 0 || H / Hkv > kDecMaxGroup) return HCP_ERR_UNSUPPORTED;
  if (D != 64 && D != 128) return HCP_ERR_UNSUPPORTED;
  if (!(a->scale > 0.f) || !std::isfinite(a->scale)) return HCP_ERR_INVALID;
  if (a->num_seqs < 0 || (a->num_seqs > 0 && a->seqs == nullptr)) return HCP_ERR_INVALID;
  if (a->q == nullptr || a->out == nullptr || a->q_row_stride < static_cast<int64_t>(H) * D ||
      a->out_row_stride < static_cast<int64_t>(H) * D || (a->q_row_stride % 8) != 0 || !aligned16(a->q))
    return HCP_ERR_INVALID;
  if (a->out_dtype != a->dtype && a->out_dtype != HCP_F32) return HCP_ERR_UNSUPPORTED;
  const bool peer = a->peer_k != nullptr, paged = a->kv_cache != nullptr;
  const int64_t kv_row = static_cast<int64_t>(Hkv) * D;
  if (peer && (a->peer_v == nullptr || a->peer_rows <= 0 || a->peer_row_stride < kv_row ||
               (a->peer_row_stride % 8) != 0 || !aligned16(a->peer_k) || !aligned16(a->peer_v)))
    return HCP_ERR_INVALID;
  if (paged) {
    const int bs = a->block_size;
    if (bs != 16 && bs != 32 && bs != 64) return HCP_ERR_UNSUPPORTED;
    if (a->num_blocks <= 0 || a->num_blocks >= (1ll << 31) || a->block_table == nullptr ||
        a->block_table_stride <= 0 || a->block_table_rows <= 0 || !aligned16(a->kv_cache))
      return HCP_ERR_INVALID;
  }
  if (a->num_ext < 0 || a->num_ext > HCP_MAX_EXT_SOURCES || (a->num_ext > 0 && a->ext == nullptr))
    return HCP_ERR_INVALID;
  for (int i = 0; i < a->num_ext; ++i) {
    const hcp_kv_source& e = a->ext[i];
    if (e.k == nullptr || e.v == nullptr || e.rows <= 0 || e.row_stride < kv_row || (e.row_stride % 8) != 0 ||
        !aligned16(e.k) || !aligned16(e.v))
      return HCP_ERR_INVALID;
  }
  for (int i = 0; i < a->num_seqs; ++i) {
    const hcp_decode_seq& q = a->seqs[i];
    if (q.q_row < 0 || q.q_row >= a->q_rows || q.peer_len < 0 || q.local_len < 0 || q.peer_start < 0)
      return HCP_ERR_INVALID;
    const int src = a->peer_src != nullptr ? a->peer_src[i] : -1;
    if (src < -1 || src >= a->num_ext) return HCP_ERR_INVALID;
    const int64_t src_rows = src < 0 ? (peer ? a->peer_rows : 0) : a->ext[src].rows;
    if (q.peer_len > 0 && static_cast<int64_t>(q.peer_start) + q.peer_len > src_rows)
      return HCP_ERR_INVALID;
    if (q.local_len > 0) {
      if (!paged || q.paged_req < 0 || q.paged_req >= a->block_table_rows || q.local_start < 0)
        return HCP_ERR_INVALID;
      if (q.local_start % a->block_size != 0) return HCP_ERR_UNSUPPORTED;
      if (static_cast<int64_t>(q.local_start) + q.local_len > a->block_table_stride * a->block_size)
        return HCP_ERR_INVALID;
    }
    if (a->lse != nullptr && q.q_row >= a->lse_stride) return HCP_ERR_INVALID;
  }
  return HCP_OK;
}
}  // namespace

extern "C" int64_t hcp_decode_workspace_bytes(const hcp_decode_args* a) {
  if (validate_decode(a) != HCP_OK) return -1;
  return workspace_need(a, decode_chunk_keys(a));
}

extern "C" int hcp_ring_decode_splitkv(const hcp_decode_args* a, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  const int rc0 = validate_decode(a);
  if (rc0 != HCP_OK) return rc0;
  if (a->num_seqs == 0) return HCP_OK;
  const bool f16 = a->dtype == HCP_F16;
  const int H = a->num_heads, Hkv = a->num_kv_heads, D = a->head_dim;
  const int chunk = decode_chunk_keys(a);
  const int64_t need = workspace_need(a, chunk);
  if (a->workspace == nullptr || a->workspace_bytes < need || !aligned16(a->workspace))
    return HCP_ERR_INVALID;
  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  // placeholder maps: a tiny valid map over q stands in for an absent source
  if (!encode_rows_heads(&p.tm_pk, f16, a->q, a->q_rows, H, D, a->q_row_stride)) return HCP_ERR_CUDA;
  p.tm_pv = p.tm_cache = p.tm_pk;
  if (a->peer_k != nullptr) {
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(a->peer_rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(a->peer_row_stride) * 2};
    const uint32_t box[3] = {64, 1, kDecTileKeys};
    if (!encode_map(&p.tm_pk, f16, 3, a->peer_k, dims, strides, box) ||
        !encode_map(&p.tm_pv, f16, 3, a->peer_v, dims, strides, box))
      return HCP_ERR_CUDA;
  }
  if (a->kv_cache != nullptr) {
    const uint64_t bs = static_cast<uint64_t>(a->block_size);
    const uint64_t dims[4] = {static_cast<uint64_t>(2 * D), bs, static_cast<uint64_t>(Hkv),
                              static_cast<uint64_t>(a->num_blocks)};
    const uint64_t strides[3] = {static_cast<uint64_t>(2 * D) * 2, bs * 2 * D * 2,
                                 static_cast<uint64_t>(Hkv) * bs * 2 * D * 2};
    const uint32_t box[4] = {64, static_cast<uint32_t>(bs), 1, 1};
    if (!encode_map(&p.tm_cache, f16, 4, a->kv_cache, dims, strides, box)) return HCP_ERR_CUDA;
  }
  for (int i = 0; i < HCP_MAX_EXT_SOURCES; ++i) p.tm_epk[i] = p.tm_epv[i] = p.tm_pk;
  for (int i = 0; i < a->num_ext; ++i) {
    const hcp_kv_source& e = a->ext[i];
    const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(Hkv), static_cast<uint64_t>(e.rows)};
    const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2, static_cast<uint64_t>(e.row_stride) * 2};
    const uint32_t box[3] = {64, 1, kDecTileKeys};
    if (!encode_map(&p.tm_epk[i], f16, 3, e.k, dims, strides, box) ||
        !encode_map(&p.tm_epv[i], f16, 3, e.v, dims, strides, box))
      return HCP_ERR_CUDA;
  }
  p.q = a->q;
  p.q_row_stride = a->q_row_stride;
  p.block_table = a->block_table;
  p.bt_stride = a->block_table_stride;
  p.bt_rows = a->block_table_rows;
  p.num_blocks = a->num_blocks;
  p.num_heads = H;
  p.num_kv_heads = Hkv;
  p.group = H / Hkv;
  p.block_size = a->kv_cache != nullptr ? a->block_size : 16;
  p.chunk_keys = chunk;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  float* part_o = static_cast<float*>(a->workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int64_t unit_base = 0;
  for (int base = 0; base < a->num_seqs; base += kDecMaxSeqs) {
    const int n = std::min(kDecMaxSeqs, a->num_seqs - base);
    int units = 0;
    CombineParams c;
    std::memset(&c, 0, sizeof(c));
    for (int i = 0; i < n; ++i) {
      const hcp_decode_seq& q = a->seqs[base + i];
      p.seq[i] = DecodeSeq{q.q_row, q.peer_start, q.peer_len, q.paged_req, q.local_start, q.local_len,
                           a->peer_src != nullptr ? a->peer_src[base + i] : -1};
      p.unit_off[i] = units;
      c.unit_off[i] = units;
      c.q_row[i] = q.q_row;
      const int pu = (q.peer_len + chunk - 1) / chunk, lu = (q.local_len + chunk - 1) / chunk;
      units += std::max(1, pu + lu);  // an empty sequence still gets one (empty) unit
    }
    p.unit_off[n] = c.unit_off[n] = units;
    p.num_seqs = n;
    p.total_units = units;
    p.part_o = part_o + unit_base * H * D;
    const int64_t total_units = decode_units(a, chunk);
    p.part_lse = part_o + total_units * H * D + unit_base * H;
    int rc = D == 128 ? (f16 ? launch_decode<128, true>(p, units, Hkv, st) : launch_decode<128, false>(p, units, Hkv, st))
                      : (f16 ? launch_decode<64, true>(p, units, Hkv, st) : launch_decode<64, false>(p, units, Hkv, st));
    if (rc != HCP_OK) return rc;
    c.part_o = p.part_o;
    c.part_lse = p.part_lse;
    c.out = a->out;
    c.out_row_stride = a->out_row_stride;
    c.lse = a->lse;
    c.lse_stride = a->lse_stride;
    c.out_dt = a->out_dtype;
    c.num_heads = H;
    c.head_dim = D;
    c.num_seqs = n;
    decode_combine_kernel<<<dim3(n, H), 128, 0, st>>>(c);
    if (cudaGetLastError() != cudaSuccess) return HCP_ERR_CUDA;
    unit_base += units;
  }
  return HCP_OK;
}

extern "C" int hcp_kv_cache_update(const void* key, const void* value, int64_t num_tokens,
                                   int64_t key_row_stride, int64_t value_row_stride,
                                   const int64_t* slot_mapping, void* kv_cache, int64_t num_blocks,
                                   int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                                   int32_t dtype, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  if (dtype != HCP_BF16 && dtype != HCP_F16) return HCP_ERR_UNSUPPORTED;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || (head_dim % 8) != 0 || block_size <= 0 ||
      num_blocks <= 0)
    return HCP_ERR_INVALID;
  if (num_tokens == 0) return HCP_OK;
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (key == nullptr || value == nullptr || slot_mapping == nullptr || kv_cache == nullptr ||
      key_row_stride < row || value_row_stride < row || (key_row_stride % 8) != 0 ||
      (value_row_stride % 8) != 0 || !aligned16(key) || !aligned16(value) || !aligned16(kv_cache))
    return HCP_ERR_INVALID;
  CacheUpdateParams p;
  p.key = static_cast<const uint16_t*>(key);
  p.value = static_cast<const uint16_t*>(value);
  p.key_row_stride = key_row_stride;
  p.value_row_stride = value_row_stride;
  p.slot_mapping = slot_mapping;
  p.cache = static_cast<uint16_t*>(kv_cache);
  p.num_blocks = num_blocks;
  p.num_tokens = num_tokens;
  p.block_size = block_size;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.bs_shift = pow2_shift(block_size);
  const int64_t blocks = (num_tokens + kCacheTokPerBlock - 1) / kCacheTokPerBlock;
  if (blocks > 0x7fffffff || num_kv_heads > 65535) return HCP_ERR_UNSUPPORTED;
  kv_cache_update_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(num_kv_heads)), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

extern "C" int hcp_kv_cache_gather(const void* kv_cache, int64_t num_blocks, int32_t block_size,
                                   int32_t num_kv_heads, int32_t head_dim, const int64_t* slot_mapping,
                                   int64_t num_tokens, void* key, void* value, int64_t key_row_stride,
                                   int64_t value_row_stride, int32_t dtype, void* stream) {
  if (!stream_on_current_device(stream)) return HCP_ERR_INVALID;
  if (dtype != HCP_BF16 && dtype != HCP_F16) return HCP_ERR_UNSUPPORTED;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || (head_dim % 8) != 0 || block_size <= 0 ||
      num_blocks <= 0)
    return HCP_ERR_INVALID;
  if (num_tokens == 0) return HCP_OK;
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (key == nullptr || value == nullptr || slot_mapping == nullptr || kv_cache == nullptr ||
      key_row_stride < row || value_row_stride < row || (key_row_stride % 8) != 0 ||
      (value_row_stride % 8) != 0 || !aligned16(key) || !aligned16(value) || !aligned16(kv_cache))
    return HCP_ERR_INVALID;
  CacheGatherParams p;
  p.cache = static_cast<const uint16_t*>(kv_cache);
  p.slot_mapping = slot_mapping;
  p.key = static_cast<uint16_t*>(key);
  p.value = static_cast<uint16_t*>(value);
  p.key_row_stride = key_row_stride;
  p.value_row_stride = value_row_stride;
  p.num_blocks = num_blocks;
  p.num_tokens = num_tokens;
  p.block_size = block_size;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.bs_shift = pow2_shift(block_size);
  const int64_t blocks = (num_tokens + kCacheTokPerBlock - 1) / kCacheTokPerBlock;
  if (blocks > 0x7fffffff || num_kv_heads > 65535) return HCP_ERR_UNSUPPORTED;
  kv_cache_gather_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(num_kv_heads)), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Split-KV decode without allocation (hcp_ring_decode_splitkv_noalloc).
//
// Callers that own no device allocator, or whose HBM is already promised to a
// paged KV cache, cannot hand in a workspace.  Their partials live in this
// fixed array instead: it belongs to the library's device image, so every GPU
// that loads the library keeps HCP_DECODE_NOALLOC_SCRATCH_BYTES of it until
// the process exits, and no call allocates or frees device memory.  All
// calls share it; overlapping calls race.
// ---------------------------------------------------------------------------
namespace {

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[HCP_DECODE_NOALLOC_SCRATCH_BYTES];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

CUcontext current_ctx() {
  CtxGetCurrentFn fn = ctx_get_current_fn();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

std::mutex g_noalloc_mu;
// Device address of the array in each CUDA context that asked for it.  A
// device address belongs to one context: a host that makes its own driver
// context current, or re-creates the primary context, gets a fresh lookup.
std::vector<std::pair<CUcontext, void*>> g_noalloc_addr;

// The host-side name of the array is not a device address: ask the runtime
// for it once per CUDA context, with that context current.
int noalloc_scratch_address(void** out) {
  void* p = nullptr;
  CUcontext ctx = current_ctx();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (ctx != nullptr) {
    for (const auto& e : g_noalloc_addr)
      if (e.first == ctx) {
        *out = e.second;
        return HCP_OK;
      }
  }
  if (cudaGetSymbolAddress(&p, g_decode_noalloc_scratch) != cudaSuccess || p == nullptr) return HCP_ERR_CUDA;
  // the lookup may have made the primary context current just now
  if (ctx == nullptr) ctx = current_ctx();
  if (ctx != nullptr) g_noalloc_addr.emplace_back(ctx, p);
  *out = p;
  return HCP_OK;
}

}  // namespace

extern "C" int hcp_ring_decode_splitkv_noalloc(const hcp_decode_args* a, void* stream) {
  const int rc = validate_decode(a);
  if (rc != HCP_OK) return rc;
  if (a->num_seqs == 0) return HCP_OK;
  // Every partial the merge step reads is written earlier in the same call,
  // so the array needs no clearing between calls.
  if (workspace_need(a, decode_chunk_keys(a)) > HCP_DECODE_NOALLOC_SCRATCH_BYTES)
    return HCP_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc2 = noalloc_scratch_address(&scratch);
  if (rc2 != HCP_OK) return rc2;
  hcp_decode_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = HCP_DECODE_NOALLOC_SCRATCH_BYTES;
  return hcp_ring_decode_splitkv(&b, stream);
}

// ---------------------------------------------------------------------------
// In-box chunk transport: CUDA IPC export / open of a device buffer and a
// copy-engine copy between GPUs (NVLink through NVSwitch).  A producer
// exports the buffer holding its chunk's per-layer K/V; a consumer process on
// any GPU of the box maps it and copies the layers it needs into its own HBM.
// ---------------------------------------------------------------------------

namespace {

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  return fn;
}

}  // namespace

extern "C" int hcp_ipc_export(const void* ptr, uint8_t* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return HCP_ERR_INVALID;
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return HCP_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return HCP_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return HCP_ERR_CUDA;
  static_assert(sizeof(h) == HCP_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return HCP_OK;
}

extern "C" int hcp_ipc_open(const uint8_t* handle, int32_t device, void** base_out) {
  if (handle == nullptr || base_out == nullptr || device < 0) return HCP_ERR_INVALID;
  int prev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) return HCP_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return HCP_ERR_CUDA;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return HCP_ERR_CUDA;
  }
  *base_out = p;
  return HCP_OK;
}

extern "C" int hcp_ipc_close(void* base) {
  if (base == nullptr) return HCP_ERR_INVALID;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? HCP_OK : HCP_ERR_CUDA;
}

extern "C" int hcp_peer_copy(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes < 0 || ((dst == nullptr || src == nullptr) && bytes > 0)) return HCP_ERR_INVALID;
  if (bytes == 0) return HCP_OK;
  return cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault,
                         static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? HCP_OK
             : HCP_ERR_CUDA;
}
