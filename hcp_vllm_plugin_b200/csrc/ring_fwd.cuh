// Fused ring-attention forward for B200 (sm_100a).
//
// One CTA computes 256 query rows (two 128-row tiles, "A" and "B") of one
// query head over the union of up to two KV segments (the transient peer
// prefix, non-causal, and the local chunk, causal at a global offset), with an
// online softmax per row, and writes the normalised output plus the per-row
// natural-log LSE.  An earlier partial (O, LSE) can be merged in the epilogue,
// so ring hops chain without a separate merge kernel.
//
// Every K/V tile staged in shared memory feeds both query tiles: the kernel is
// bound by operand traffic (L2 -> shared memory -> tensor core), and sharing
// halves it per FLOP.
//
// Warp roles (320 threads; 384 in variants 3-6, warps 10-11 without a role,
// so setmaxnreg can split the registers per warpgroup):
//   warps 0-3  softmax / O correction / epilogue of query tile A
//   warps 4-7  the same for query tile B.  Thread (w, lane) owns row
//              32*(w%4)+lane of its tile, which is that TMEM lane.
//   warp 8     TMA producer: Q_A, Q_B once, then K and V tiles through a
//              2-stage ring (contiguous 3-D tensor maps, or 4-D maps over the
//              paged cache indexed through the block table)
//   warp 9     tcgen05 MMA issuer (one lane) and TMEM owner.  Per KV tile it
//              issues  O_A += P_A V (previous tile), S_A = Q_A K,
//                      O_B += P_B V (previous tile), S_B = Q_B K,
//              so the tensor core works for one warpgroup while the other
//              computes its softmax.
//
// TMEM (512 columns x 128 lanes, fp32):
//   [  0,128)      S_A,  [128,256) S_B.  P (16-bit, two keys per column) is
//                  written back over columns 0-63 of its S buffer and feeds
//                  O += P V as the A operand; for rows that see few keys the
//                  low part P - bf16(P) goes to columns 64-127 and is
//                  accumulated by a second PV product.
//   [256,256+D)    O_A,  [256+D, 256+2D) O_B
//
// Shared memory (1024-byte aligned, 128-byte swizzle, 64-element boxes):
//   Q_A, Q_B, then per stage a K tile and a V tile, then the mbarriers.
//
// Numerics: scores are scaled into the base-2 domain (scale * log2 e), the
// running max is only raised when a tile's max exceeds it by more than 8
// (P stays <= 2^8) and O is rescaled in TMEM only then.
// LSE = (m + log2 l) * ln 2.
//
// Variants (template parameter V, chosen per process by the host): 0 - the
// MMA issuer waits on mbarriers; 1 - it meets the softmax warpgroups at
// named barriers only and they wait on the mbarriers instead; 2 - as 1, with
// a quarter of the exponentials computed on the FMA pipe (exp2_poly); 3-5 -
// as 0 on 384 threads with the registers split by setmaxnreg and packed
// softmax math (a quarter, three eighths, none of the exponentials on the
// FMA pipe); 6 - as 1 on 384 threads with the setmaxnreg split.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "hcp_ring.h"
#include "sm100_ptx.cuh"

namespace hcp {

__device__ int g_device_status = 0;

constexpr int kBlockM = 128;          // rows per query tile (one TMEM lane each)
constexpr int kCtaRows = 2 * kBlockM;  // query rows per CTA
constexpr int kBlockN = 128;          // keys per KV tile
constexpr int kStages = 2;
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr int kThreads = 320;
// Variants 3-6: a third warpgroup (warps 8-11: TMA, MMA, two idle) so the
// registers can be split by setmaxnreg - 224 for each softmax thread, 56 for
// the producer warpgroup (2*128*224 + 128*56 = 384*168, the launch's total).
constexpr int kThreadsWide = 384;
constexpr int kRegsSoftmaxWide = 224;
constexpr int kRegsProducerWide = 56;
constexpr int kMaxWork = 160;
constexpr int kMaxSegs = 2 * kMaxWork;   // segments of one launch's work items
constexpr int kMaxItemSegs = HCP_MAX_ITEM_SEGMENTS;
constexpr int kMaxExt = HCP_MAX_EXT_SOURCES;
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s
constexpr float kRescaleThreshold = 8.0f;            // log2 units
constexpr int kPreciseKeys = 1024;  // rows seeing fewer keys get the hi+lo P product
// Named barriers of the NB issuer protocol: event barrier of query tile x
// (softmax warpgroup x arrives, the MMA warp syncs) and its acknowledgement
// (the MMA warp arrives, the warpgroup syncs); 128 + 32 threads each.
constexpr int kNbEvent0 = 1;
constexpr int kNbAck0 = 3;
constexpr int kNbThreads = 160;

// Failure codes written to g_device_status.
enum : int {
  kErrWaitProducer = 0x101,
  kErrWaitMma = 0x102,
  kErrWaitSoftmax = 0x103,
  kErrWaitDrain = 0x104,
  kErrWaitSelftest = 0x1ff,
};

// One work item as the kernel sees it: its segments are segs[seg_first ..
// seg_first + seg_count).
struct FwdItem {
  int q_start;
  int q_len;
  int paged_req;
  int lse_col;
  int seg_first;
  int seg_count;
};

struct FwdParams {
  CUtensorMap tm_q;      // {D, H, q_rows}     box {64, 1, 128}
  CUtensorMap tm_ka;     // {D, Hkv, rows_a}   box {64, 1, 128}
  CUtensorMap tm_va;
  CUtensorMap tm_kb;
  CUtensorMap tm_vb;
  CUtensorMap tm_cache;  // {2D, bs, Hkv, nb}  box {64, bs, 1, 1}
  CUtensorMap tm_ek[kMaxExt];  // extra contiguous sources (HCP_SRC_EXT0 + i)
  CUtensorMap tm_ev[kMaxExt];
  const int32_t* block_table;
  long long bt_stride;
  long long bt_rows;
  long long num_blocks;
  void* out;
  long long out_row_stride;
  float* lse;
  long long lse_stride;
  const void* merge_o;
  long long merge_o_row_stride;
  const float* merge_lse;
  long long merge_lse_stride;
  int out_f32;
  int merge_o_f32;
  int num_heads;
  int group;
  int block_size;
  int num_work;
  float scale_log2;
  int total_tiles;
  int window;  // sliding window of causal segments, 0 = none
  int tile_off[kMaxWork + 1];
  FwdItem work[kMaxWork];
  hcp_kv_segment segs[kMaxSegs];
};
// Kernel arguments may take up to 32764 bytes (CUDA 12.1+, compute 7.0+).
static_assert(sizeof(FwdParams) <= 32764, "forward kernel parameters too large");

// Bounded mbarrier wait.  Returns false when this CTA aborted (this wait ran
// out of time, another role of the CTA gave up, or another CTA failed).
__device__ __forceinline__ bool wait_bar_for(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             int code, uint64_t timeout_ns) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (*reinterpret_cast<volatile int*>(&g_device_status) != 0) {
        *abort_flag = 1;
        return false;
      }
      if (ptx::global_timer_ns() - t0 > timeout_ns) {
        *abort_flag = 1;
        atomicCAS(&g_device_status, 0, code);
        return false;
      }
    }
  }
}
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int code) {
  return wait_bar_for(bar, parity, abort_flag, code, kWaitTimeoutNs);
}

// Self-test of the failure path: one thread waits, through the same bounded
// wait as the kernels, on an mbarrier that nothing arrives on.  The wait runs
// out after timeout_ns, records kErrWaitSelftest in g_device_status and the
// kernel returns normally: no fault, the context stays usable.
__global__ void bounded_wait_selftest_kernel(uint64_t timeout_ns, int* result) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  ptx::mbar_init(ptx::smem_u32(&bar), 1);
  ptx::fence_mbar_init();
  const bool ok = wait_bar_for(ptx::smem_u32(&bar), 0, &abort_flag, kErrWaitSelftest, timeout_ns);
  *result = ok ? 1 : 0;
}

// Bounded wait that ignores the abort flag: used at teardown for work that
// completes on its own (TMA copies and MMAs already issued).
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t it = 0;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return;
    if ((it & 63u) == 63u && ptx::global_timer_ns() - t0 > kWaitTimeoutNs) {
      atomicCAS(&g_device_status, 0, kErrWaitDrain);
      return;
    }
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for x <= 0 on the FMA pipe, so part of a tile's exponentials leave the
// MUFU unit (which two softmax warps per SM sub-partition keep busy for as
// long as the tensor work of a tile takes).  Cody-Waite reduction
// x = j + f with j = rint(x) by the 1.5 * 2^23 rounding trick (f in
// [-1/2, 1/2]); 2^f by a degree-3 polynomial, minimax in relative error on
// that interval (Remez exchange; coefficients and their 7.5e-5 error from
// tests/gen_exp2_poly.py); 2^j by adding j to the exponent bits: the low bits of
// the rounded float hold j, and shifting them by 23 drops the rest.  At or
// below -126 the result is 0, as ex2.approx.ftz gives for masked keys.
__device__ __forceinline__ float exp2_poly(float x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0.99992806f, kC1 = 0.69326097f, kC2 = 0.24261113f, kC3 = 0.05517167f;
  const float xc = fmaxf(x, -126.0f);
  const float t = __fadd_rn(xc, kMagic);
  const float f = __fsub_rn(xc, __fsub_rn(t, kMagic));
  const float p = fmaf(fmaf(fmaf(kC3, f, kC2), f, kC1), f, kC0);
  const int bits = __float_as_int(p) + (__float_as_int(t) << 23);
  return x > -126.0f ? __int_as_float(bits) : 0.0f;
}
// Pairs of a 16-pair group whose exponentials take the FMA-pipe path
// (kernel variant 2): one in four.
__device__ __forceinline__ constexpr bool poly_pair(int i) { return (i & 3) == 3; }
// The same choice for variants 3-5: one in four, three in eight, none.
template <int V>
__device__ __forceinline__ constexpr bool poly_pair_v(int i) {
  return V == 3 ? (i & 3) == 3 : V == 4 ? ((i & 7) == 2 || (i & 7) == 5 || (i & 7) == 7) : false;
}

// 2^x of a pair on the FMA pipe with packed f32x2 arithmetic (the steps of
// exp2_poly).  Inputs at or below -126 give 2^-126, not 0: such keys are
// masked ones, whose weight next to a row's largest (>= 1) is immaterial.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float2 xc = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
  const float2 t = __fadd2_rn(xc, make_float2(kMagic, kMagic));
  const float2 j = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), xc);
  float2 q = __ffma2_rn(make_float2(0.05517167f, 0.05517167f), f, make_float2(0.24261113f, 0.24261113f));
  q = __ffma2_rn(q, f, make_float2(0.69326097f, 0.69326097f));
  q = __ffma2_rn(q, f, make_float2(0.99992806f, 0.99992806f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool F16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (F16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <bool F16>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (F16) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  } else {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
}

// In-kernel marker of a non-causal segment (see cta_segment).
constexpr int kNonCausal = -2147483647 - 1;

// Keys of segment `sg` visible to the valid rows [q0, q0+rows) of a query tile.
__device__ __forceinline__ int segment_keys(const hcp_kv_segment& sg, int q0, int rows) {
  if (rows <= 0 || sg.src == HCP_SRC_NONE || sg.len <= 0) return 0;
  if (sg.causal_off == kNonCausal) return sg.len;
  const long long last_visible = static_cast<long long>(sg.causal_off) + q0 + rows;  // exclusive
  return static_cast<int>(max(0ll, min(static_cast<long long>(sg.len), last_visible)));
}

// A segment as the CTA whose rows start at q0 uses it.  Non-causal segments
// (causal_off < 0 at the ABI) get the in-kernel marker kNonCausal, since a
// trimmed causal segment may have a negative offset.  With a sliding window
// (keys j with qpos - window < j <= qpos visible) a causal segment starts at
// the first whole KV tile row q0 sees (a multiple of kBlockN, so of the block
// size too); the keys below the window inside that tile are masked per row.
__device__ __forceinline__ hcp_kv_segment cta_segment(hcp_kv_segment sg, int q0, int window) {
  if (sg.causal_off < 0) {
    sg.causal_off = kNonCausal;
    return sg;
  }
  if (window <= 0 || sg.src == HCP_SRC_NONE || sg.len <= 0) return sg;
  const long long lo = static_cast<long long>(sg.causal_off) + q0 - window + 1;  // first key row q0 sees
  if (lo < kBlockN) return sg;
  const int skip = static_cast<int>(min(static_cast<long long>(sg.len), lo / kBlockN * kBlockN));
  sg.start += skip;
  sg.len -= skip;
  sg.causal_off -= skip;
  return sg;
}

template <int D>
struct FwdSmem {
  static constexpr int kBoxBytes = 128 * 128;  // 128 rows x 64 elems x 2 B
  static constexpr int kTileBytes = (D / 64) * kBoxBytes;
  static constexpr int kNumBars = 8 + 4 * kStages;
  static constexpr int kKvOff = 2 * kTileBytes;                    // after Q_A, Q_B
  static constexpr int kBarOff = kKvOff + 2 * kStages * kTileBytes;
  // after the barriers: TMEM slot + abort flag (16 B), then the CTA's
  // segment table: tile prefix [kMaxItemSegs + 1], keys needed by query tile
  // A and by B [kMaxItemSegs] each, segment count, precise flags A and B
  static constexpr int kSegOff = kBarOff + 8 * kNumBars + 16;
  static constexpr int kSegInts = (kMaxItemSegs + 1) + 2 * kMaxItemSegs + 3 + 4 * kMaxItemSegs;
  static constexpr int kEnd = kSegOff + 4 * kSegInts;
  static constexpr int kBytes = kEnd + 1024;  // + alignment slack
};

// V selects how the MMA issuer synchronises with the softmax warpgroups and
// how exponentials are computed:
// 0 - the issuer waits on mbarriers (P ready, K / V tiles landed);
// 1 - it meets the softmax warpgroups only at named barriers, and they do the
//     mbarrier waits for the tiles their P feeds (see below);
// 2 - as 1, with one in four exponentials of a tile on the FMA pipe
//     (exp2_poly) instead of the MUFU unit.
// LIST: items may have more than two segments (a per-CTA segment table in
// shared memory).  Without it every item has exactly two segments, which each
// thread keeps in registers: the per-tile lookups sit on the MMA issuer's and
// the softmax warps' paths, and a table read there was measured 25% slower.
template <int D, bool F16, int V = 0, bool LIST = false>
__global__ void __launch_bounds__(V >= 3 ? kThreadsWide : kThreads, 1)
    ring_fwd_kernel(const __grid_constant__ FwdParams p) {
  constexpr bool NB = V == 1 || V == 2 || V == 6;
  constexpr bool kPoly = V == 2;
  constexpr bool kWide = V >= 3;
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  using L = FwdSmem<D>;
  constexpr int kHalves = D / 64;
  constexpr int kBoxBytes = L::kBoxBytes;
  constexpr int kTileBytes = L::kTileBytes;
  constexpr uint32_t kIdescQK = ptx::idesc_f16(128, 128, false, false, F16);
  constexpr uint32_t kIdescPV = ptx::idesc_f16(128, D, false, true, F16);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_q = ptx::smem_u32(smem);           // Q_A at s_q, Q_B at s_q + kTileBytes
  const uint32_t s_kv0 = s_q + L::kKvOff;             // stage s: K at +2s tiles, V at +2s+1
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar0 = ptx::smem_u32(bars);
  const uint32_t b_q = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + kStages + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + 2 * kStages + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 3 * kStages + s); };
  auto b_sfull = [&](int x) { return bar0 + 8u * (1 + 4 * kStages + x); };
  auto b_pfull = [&](int x) { return bar0 + 8u * (3 + 4 * kStages + x); };
  auto b_odone = [&](int x) { return bar0 + 8u * (5 + 4 * kStages + x); };
  const uint32_t b_final = bar0 + 8u * (7 + 4 * kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- which (work item, 256-row block, head) this CTA owns
  const int H = p.num_heads;
  const int tile_global = blockIdx.x / H;
  const int head = blockIdx.x - tile_global * H;
  const int kvh = head / p.group;
  int lo = 0, hi = p.num_work - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_off[mid] <= tile_global) lo = mid; else hi = mid - 1;
  }
  const FwdItem& wk = p.work[lo];
  const hcp_kv_segment* segs = p.segs + wk.seg_first;
  const int n_blocks = (wk.q_len + kCtaRows - 1) / kCtaRows;
  const int m_blk = n_blocks - 1 - (tile_global - p.tile_off[lo]);  // heaviest (last) first
  const int q0 = m_blk * kCtaRows;
  const int rows_a = max(0, min(kBlockM, wk.q_len - q0));
  const int rows_b = max(0, min(kBlockM, wk.q_len - q0 - kBlockM));
  // Two-segment items: every thread's own copy of the table, in registers.
  hcp_kv_segment sg0{}, sg1{};
  int ka0 = 0, kb0 = 0, ka1 = 0, kb1 = 0, tiles0 = 0, tiles2 = 0;
  bool pre_a = false, pre_b = false;
  if constexpr (!LIST) {
    sg0 = cta_segment(segs[0], q0, p.window);
    sg1 = cta_segment(segs[1], q0, p.window);
    ka0 = segment_keys(sg0, q0, rows_a);
    kb0 = segment_keys(sg0, q0 + kBlockM, rows_b);
    ka1 = segment_keys(sg1, q0, rows_a);
    kb1 = segment_keys(sg1, q0 + kBlockM, rows_b);
    tiles0 = (max(ka0, kb0) + kBlockN - 1) / kBlockN;
    tiles2 = tiles0 + (max(ka1, kb1) + kBlockN - 1) / kBlockN;
    // Rows that see few keys in total get P as hi + lo 16-bit parts.
    pre_a = segment_keys(sg0, q0, 1) + segment_keys(sg1, q0, 1) < kPreciseKeys;
    pre_b = segment_keys(sg0, q0 + kBlockM, 1) + segment_keys(sg1, q0 + kBlockM, 1) < kPreciseKeys;
  }
  // LIST: the CTA's segment table (shared memory, filled by thread 0 at
  // setup): the KV tiles of segment s are [sg_base[s], sg_base[s+1]); query
  // tile A needs its first sg_need_a[s] keys, B its first sg_need_b[s].
  int* sg_base = reinterpret_cast<int*>(smem + L::kSegOff);
  int* sg_need_a = sg_base + kMaxItemSegs + 1;
  int* sg_need_b = sg_need_a + kMaxItemSegs;
  int* sg_misc = sg_need_b + kMaxItemSegs;  // [0] segments, [1] precise A, [2] precise B
  hcp_kv_segment* sg_trim = reinterpret_cast<hcp_kv_segment*>(sg_misc + 3);  // the segments, windowed

  // ---- setup
  if (LIST && threadIdx.x == 0) {
    // keys each query tile needs from each segment; the KV tile list covers all
    int tiles = 0, keys_a = 0, keys_b = 0;
    const int n_seg = min(wk.seg_count, kMaxItemSegs);
    for (int s = 0; s < n_seg; ++s) {
      const hcp_kv_segment sg = cta_segment(segs[s], q0, p.window);
      sg_trim[s] = sg;
      const int ka = segment_keys(sg, q0, rows_a), kb = segment_keys(sg, q0 + kBlockM, rows_b);
      sg_base[s] = tiles;
      sg_need_a[s] = ka;
      sg_need_b[s] = kb;
      tiles += (max(ka, kb) + kBlockN - 1) / kBlockN;
      keys_a += segment_keys(sg, q0, 1);
      keys_b += segment_keys(sg, q0 + kBlockM, 1);
    }
    sg_base[n_seg] = tiles;
    sg_misc[0] = n_seg;
    // Rows that see few keys in total get P as hi + lo 16-bit parts.
    sg_misc[1] = keys_a < kPreciseKeys;
    sg_misc[2] = keys_b < kPreciseKeys;
  }
  if (threadIdx.x == 0) {
    ptx::mbar_init(b_q, 1);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(b_kfull(s), 1);
      ptx::mbar_init(b_kempty(s), 1);
      ptx::mbar_init(b_vfull(s), 1);
      ptx::mbar_init(b_vempty(s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      ptx::mbar_init(b_sfull(x), 1);
      ptx::mbar_init(b_pfull(x), 128);
      ptx::mbar_init(b_odone(x), 1);
    }
    ptx::mbar_init(b_final, 1);
    // A CTA starting after another one failed does no work.
    *abort_flag = *reinterpret_cast<volatile int*>(&g_device_status) != 0 ? 1 : 0;
    ptx::fence_mbar_init();
  }
  if (warp == kWarpMma) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), kTmemCols);
    ptx::tmem_relinquish();
  }
  if (warp == kWarpTma && lane == 0) {
    ptx::prefetch_tmap(&p.tm_q);
    ptx::prefetch_tmap(&p.tm_ka);
    ptx::prefetch_tmap(&p.tm_va);
    ptx::prefetch_tmap(&p.tm_cache);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_seg = LIST ? sg_misc[0] : 2;
  const int n_tiles = LIST ? sg_base[n_seg] : tiles2;
  const bool precise_a = LIST ? sg_misc[1] != 0 : pre_a;
  const bool precise_b = LIST ? sg_misc[2] != 0 : pre_b;
  auto tile_seg = [&](int t) {
    if constexpr (!LIST) {
      return t < tiles0 ? 0 : 1;
    } else {
      int s = 0;
      while (s + 1 < n_seg && t >= sg_base[s + 1]) ++s;
      return s;
    }
  };
  auto seg_base = [&](int s) {
    if constexpr (!LIST) return s == 0 ? 0 : tiles0;
    else return sg_base[s];
  };
  auto seg_at = [&](int s) -> hcp_kv_segment {
    if constexpr (!LIST) return s == 0 ? sg0 : sg1;
    else return sg_trim[s];
  };
  auto tile_key0 = [&](int t) { return (t - seg_base(tile_seg(t))) * kBlockN; };
  // is KV tile t needed by query tile x (0 = A, 1 = B)?
  auto active = [&](int x, int t) {
    const int s = tile_seg(t);
    int need;
    if constexpr (!LIST) need = s == 0 ? (x == 0 ? ka0 : kb0) : (x == 0 ? ka1 : kb1);
    else need = x == 0 ? sg_need_a[s] : sg_need_b[s];
    return (t - seg_base(s)) * kBlockN < need;
  };
  const bool skip_all = *abort_flag != 0;
  // Each warpgroup's setmaxnreg opens its own branch (every thread of the
  // warpgroup runs it, whatever its role or the abort state), so the code of
  // each role is register-allocated under that warpgroup's limit.
  if (warp >= 8) {
  // ============================================== producer warpgroup: TMA, MMA
  // (and, in variants 3-5, the spare warps 10-11 with no role)
  if constexpr (kWide) ptx::setmaxnreg_dec<kRegsProducerWide>();
  if (skip_all) {
    // nothing issued, nothing to drain
  } else if (warp == kWarpTma) {
    // ================================================================ producer
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(b_q, 2 * kTileBytes);
      for (int x = 0; x < 2; ++x)
        for (int hf = 0; hf < kHalves; ++hf)
          ptx::tma_load_3d(s_q + x * kTileBytes + hf * kBoxBytes, &p.tm_q, b_q, hf * 64, head,
                           wk.q_start + q0 + x * kBlockM);
    }
    int k_issued = 0, v_issued = 0;
    const int bs = p.block_size;
    const int nblk = kBlockN / bs;
    // Block id of this lane's block of paged KV tile t (lanes < nblk), or an
    // out-of-range id (TMA fills zeros) when the tile is not paged or the
    // block lies outside the table.  Looked up one tile ahead, so the load's
    // latency hides behind the waits and copies of the tile before.
    auto lookup = [&](int t) {
      int blk = static_cast<int>(p.num_blocks);
      if (t < n_tiles && lane < nblk) {
        const hcp_kv_segment sg = seg_at(tile_seg(t));
        if (sg.src == HCP_SRC_PAGED) {
          const int rel = tile_key0(t) + lane * bs;
          const long long bidx = (static_cast<long long>(sg.start) + rel) / bs;
          if (rel < sg.len && bidx < p.bt_stride && wk.paged_req >= 0 && wk.paged_req < p.bt_rows) {
            const int v = __ldg(p.block_table + wk.paged_req * p.bt_stride + bidx);
            if (v >= 0 && v < p.num_blocks) blk = v;
          }
        }
      }
      return blk;
    };
    int blk_next = lookup(0);
    for (int t = 0; t < n_tiles; ++t) {
      const int s = t % kStages;
      const uint32_t ph = (t / kStages) & 1;
      const int key0 = tile_key0(t);
      const hcp_kv_segment seg = seg_at(tile_seg(t));
      const uint32_t s_k = s_kv0 + (2 * s) * kTileBytes;
      const uint32_t s_v = s_k + kTileBytes;
      int blk_ids[8];
      const bool paged = seg.src == HCP_SRC_PAGED;
      const int blk_cur = blk_next;
      blk_next = lookup(t + 1);
      if (paged) {
#pragma unroll
        for (int i = 0; i < 8; ++i) blk_ids[i] = __shfl_sync(0xffffffffu, blk_cur, i);
      }
      if (!__all_sync(0xffffffffu, wait_bar(b_kempty(s), ph ^ 1, abort_flag, kErrWaitProducer)))
        break;
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(b_kfull(s), kTileBytes);
        if (paged) {
          for (int i = 0; i < nblk; ++i)
            for (int hf = 0; hf < kHalves; ++hf)
              ptx::tma_load_4d(s_k + hf * kBoxBytes + i * bs * 128, &p.tm_cache, b_kfull(s), hf * 64,
                               0, kvh, blk_ids[i]);
        } else {
          const CUtensorMap* tk = seg.src == HCP_SRC_A   ? &p.tm_ka
                                  : seg.src == HCP_SRC_B ? &p.tm_kb
                                                         : &p.tm_ek[seg.src - HCP_SRC_EXT0];
          for (int hf = 0; hf < kHalves; ++hf)
            ptx::tma_load_3d(s_k + hf * kBoxBytes, tk, b_kfull(s), hf * 64, kvh, seg.start + key0);
        }
      }
      k_issued = t + 1;
      if (!__all_sync(0xffffffffu, wait_bar(b_vempty(s), ph ^ 1, abort_flag, kErrWaitProducer)))
        break;
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(b_vfull(s), kTileBytes);
        if (paged) {
          for (int i = 0; i < nblk; ++i)
            for (int hf = 0; hf < kHalves; ++hf)
              ptx::tma_load_4d(s_v + hf * kBoxBytes + i * bs * 128, &p.tm_cache, b_vfull(s),
                               D + hf * 64, 0, kvh, blk_ids[i]);
        } else {
          const CUtensorMap* tv = seg.src == HCP_SRC_A   ? &p.tm_va
                                  : seg.src == HCP_SRC_B ? &p.tm_vb
                                                         : &p.tm_ev[seg.src - HCP_SRC_EXT0];
          for (int hf = 0; hf < kHalves; ++hf)
            ptx::tma_load_3d(s_v + hf * kBoxBytes, tv, b_vfull(s), hf * 64, kvh, seg.start + key0);
        }
      }
      v_issued = t + 1;
    }
    __syncwarp();
    // Teardown: every TMA copy this warp issued must land before the CTA exits.
    drain_bar(b_q, 0);
    for (int t = max(0, k_issued - kStages); t < k_issued; ++t) {
      const int s = t % kStages;
      const uint32_t ph = (t / kStages) & 1;
      drain_bar(b_kfull(s), ph);
      if (t < v_issued) drain_bar(b_vfull(s), ph);
    }
  } else if (warp == kWarpMma) {
    // ================================================================ MMA issuer
    if constexpr (NB) {
    // Events of query tile x, in order: K(a0) before its first QK; after it
    // each P(t) (P_x of tile t stored, V(t) landed, and K(t+1) landed when
    // tile t+1 is x's next) before PV_x(t); and a K(t') event before QK_x(t')
    // when x's next tile t' is not t+1.  Each event: bar.sync on the event
    // barrier, bar.arrive on its ack, so warpgroup and issuer stay in
    // lockstep.  No mbarrier wait here: those would stall the pipe.
    int pv_count[2] = {0, 0};
    for (int t = 0; t <= n_tiles; ++t) {
      const bool have_prev = t >= 1;
      const bool have_cur = t < n_tiles;
      const int sp = (t - 1) % kStages;
      const int sc = t % kStages;
      for (int x = 0; x < 2; ++x) {
        const bool pv = have_prev && active(x, t - 1);
        if (pv) {
          ptx::named_bar_sync(kNbEvent0 + x, kNbThreads);
          ptx::named_bar_arrive(kNbAck0 + x, kNbThreads);
          ptx::tc_fence_after();
          if (lane == 0) {
            const uint32_t s_v = s_kv0 + (2 * sp + 1) * kTileBytes;
            const uint32_t o_acc = tmem + 256 + x * D;
            const uint32_t p_col = tmem + x * 128;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk) {
              const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
              ptx::umma_ts(o_acc, p_col + kk * 8, bdesc, kIdescPV, (pv_count[x] > 0 || kk > 0) ? 1u : 0u);
            }
            if (x == 0 ? precise_a : precise_b) {
#pragma unroll
              for (int kk = 0; kk < kBlockN / 16; ++kk) {
                const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
                ptx::umma_ts(o_acc, p_col + 64 + kk * 8, bdesc, kIdescPV, 1u);
              }
            }
            ptx::umma_commit(b_odone(x));
          }
          __syncwarp();
          ++pv_count[x];
        }
        if (have_cur && active(x, t)) {
          if (!pv) {  // K(t) event: x's first tile, or its next tile after a gap
            ptx::named_bar_sync(kNbEvent0 + x, kNbThreads);
            ptx::named_bar_arrive(kNbAck0 + x, kNbThreads);
            ptx::tc_fence_after();
          }
          if (lane == 0) {
            const uint32_t s_k = s_kv0 + (2 * sc) * kTileBytes;
            const uint32_t s_qx = s_q + x * kTileBytes;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
              const uint64_t adesc = ptx::sdesc_sw128(s_qx + off, 16, 1024);
              const uint64_t bdesc = ptx::sdesc_sw128(s_k + off, 16, 1024);
              ptx::umma_ss(tmem + x * 128, adesc, bdesc, kIdescQK, kk > 0 ? 1u : 0u);
            }
            ptx::umma_commit(b_sfull(x));
          }
          __syncwarp();
        }
      }
      if (lane == 0) {
        if (have_prev) ptx::umma_commit(b_vempty(sp));
        if (have_cur) ptx::umma_commit(b_kempty(sc));
      }
      __syncwarp();
    }
    if (lane == 0) ptx::umma_commit(b_final);
    __syncwarp();
    drain_bar(b_final, 0);
    } else {
    bool ok = __all_sync(0xffffffffu, wait_bar(b_q, 0, abort_flag, kErrWaitMma));
    int pv_count[2] = {0, 0};  // PV products issued per query tile
    for (int t = 0; t <= n_tiles && ok; ++t) {
      const bool have_prev = t >= 1;
      const bool have_cur = t < n_tiles;
      const int sp = (t - 1) % kStages;   // stage of tile t-1
      const int sc = t % kStages;         // stage of tile t
      bool v_ready = false, k_ready = false;
      for (int x = 0; x < 2 && ok; ++x) {
        if (have_prev && active(x, t - 1)) {
          // O_x += P_x V_{t-1}; P_x is ready once the warpgroup arrived
          ok = __all_sync(0xffffffffu, wait_bar(b_pfull(x), pv_count[x] & 1, abort_flag, kErrWaitMma));
          if (ok && !v_ready) {
            ok = __all_sync(0xffffffffu,
                            wait_bar(b_vfull(sp), ((t - 1) / kStages) & 1, abort_flag, kErrWaitMma));
            v_ready = true;
          }
          if (!ok) break;
          ptx::tc_fence_after();
          if (lane == 0) {
            const uint32_t s_v = s_kv0 + (2 * sp + 1) * kTileBytes;
            const uint32_t o_acc = tmem + 256 + x * D;
            const uint32_t p_col = tmem + x * 128;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk) {
              const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
              ptx::umma_ts(o_acc, p_col + kk * 8, bdesc, kIdescPV,
                           (pv_count[x] > 0 || kk > 0) ? 1u : 0u);
            }
            if (x == 0 ? precise_a : precise_b) {
#pragma unroll
              for (int kk = 0; kk < kBlockN / 16; ++kk) {
                const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
                ptx::umma_ts(o_acc, p_col + 64 + kk * 8, bdesc, kIdescPV, 1u);
              }
            }
            ptx::umma_commit(b_odone(x));
          }
          __syncwarp();
          ++pv_count[x];
        }
        if (have_cur && active(x, t)) {
          // S_x = Q_x K_t
          if (!k_ready) {
            ok = __all_sync(0xffffffffu,
                            wait_bar(b_kfull(sc), (t / kStages) & 1, abort_flag, kErrWaitMma));
            if (!ok) break;
            k_ready = true;
          }
          ptx::tc_fence_after();
          if (lane == 0) {
            const uint32_t s_k = s_kv0 + (2 * sc) * kTileBytes;
            const uint32_t s_qx = s_q + x * kTileBytes;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
              const uint64_t adesc = ptx::sdesc_sw128(s_qx + off, 16, 1024);
              const uint64_t bdesc = ptx::sdesc_sw128(s_k + off, 16, 1024);
              ptx::umma_ss(tmem + x * 128, adesc, bdesc, kIdescQK, kk > 0 ? 1u : 0u);
            }
            ptx::umma_commit(b_sfull(x));
          }
          __syncwarp();
        }
      }
      if (!ok) break;
      // release the stages (tcgen05.commit tracks every MMA issued so far)
      if (lane == 0) {
        if (have_prev) ptx::umma_commit(b_vempty(sp));
        if (have_cur) ptx::umma_commit(b_kempty(sc));
      }
      __syncwarp();
    }
    // Teardown: no MMA may be in flight when TMEM is released.
    if (lane == 0) ptx::umma_commit(b_final);
    __syncwarp();
    drain_bar(b_final, 0);
    }
  }
  } else {
  if constexpr (kWide) ptx::setmaxnreg_inc<kRegsSoftmaxWide>();
  if (!skip_all) {
    // ================================================================ softmax + epilogue
    const int x = warp >> 2;                 // query tile of this warpgroup (0 = A, 1 = B)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;     // == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int qrow = q0 + x * kBlockM + row;  // work-item-relative query row
    const bool precise = x == 0 ? precise_a : precise_b;
    const float scale_log2 = p.scale_log2;
    const uint32_t s_addr = tmem + lane_base + x * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + x * D;
    float m_used = -INFINITY;  // running max of the row, base-2 scaled domain
    float l = 0.f;             // row sum
    bool ok = true;
    int done = 0;              // KV tiles processed by this warpgroup
    if constexpr (NB) {
    // Events for the issuer, in its order (see the MMA issuer): K(a0), then
    // per tile P(t) - with K(t+1) folded in when t+1 is this tile's next -
    // and a separate K event before a next tile after a gap.  Every event is
    // executed even after a failed wait (the work is skipped, never a
    // barrier), so the named barriers always pair up.
    auto next_active = [&](int t) {
      int u = t + 1;
      while (u < n_tiles && !active(x, u)) ++u;
      return u;
    };
    auto kv_phase = [&](int t) { return static_cast<uint32_t>((t / kStages) & 1); };
    const int first = next_active(-1);
    if (first < n_tiles) {
      ok = __all_sync(0xffffffffu, wait_bar(b_q, 0, abort_flag, kErrWaitSoftmax));
      if (ok)
        ok = __all_sync(0xffffffffu,
                        wait_bar(b_kfull(first % kStages), kv_phase(first), abort_flag, kErrWaitSoftmax));
      ptx::tc_fence_before();
      ptx::named_bar_arrive(kNbEvent0 + x, kNbThreads);            // K(a0)
    }
    for (int t = first; t < n_tiles; t = next_active(t)) {
      if (ok) ok = __all_sync(0xffffffffu, wait_bar(b_sfull(x), done & 1, abort_flag, kErrWaitSoftmax));
      if (ok) {
        ptx::tc_fence_after();
        const int key0 = tile_key0(t);
        const hcp_kv_segment seg = seg_at(tile_seg(t));
        int vis = seg.len - key0;
        if (seg.causal_off != kNonCausal) vis = min(vis, seg.causal_off + qrow - key0 + 1);
        vis = max(0, min(vis, kBlockN));
        // keys [0, lo) of the tile are below the row's sliding window
        const int lo = (p.window > 0 && seg.causal_off != kNonCausal) ? seg.causal_off + qrow - p.window + 1 - key0 : 0;

        uint32_t sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          ptx::tmem_ld_32x32b_x32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        ptx::tmem_wait_ld();
        if (vis < kBlockN || lo > 0) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= vis || i < lo) sr[i] = __float_as_uint(-INFINITY);
        }
        float mx8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = __uint_as_float(sr[j]);
#pragma unroll
        for (int i = 8; i < 128; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[i]));
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float mx2 = mx * scale_log2;  // -inf stays -inf
        const bool raise = mx2 > m_used + kRescaleThreshold;
        const float m_new = raise ? mx2 : m_used;
        const float alpha = raise ? ex2_approx(m_used - m_new) : 1.f;  // 0 when m_used = -inf
        const float m_base = (m_new == -INFINITY) ? 0.f : m_new;
        float sums[4] = {0.f, 0.f, 0.f, 0.f};
        if (!precise) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float x0 = fmaf(__uint_as_float(sr[c * 32 + 2 * i]), scale_log2, -m_base);
              const float x1 = fmaf(__uint_as_float(sr[c * 32 + 2 * i + 1]), scale_log2, -m_base);
              const bool fma_pipe = kPoly && poly_pair(i);
              const float p0 = fma_pipe ? exp2_poly(x0) : ex2_approx(x0);
              const float p1 = fma_pipe ? exp2_poly(x1) : ex2_approx(x1);
              sums[i & 3] += p0 + p1;
              pk[i] = pack2<F16>(p0, p1);
            }
            ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16], pl[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float x0 = fmaf(__uint_as_float(sr[c * 32 + 2 * i]), scale_log2, -m_base);
              const float x1 = fmaf(__uint_as_float(sr[c * 32 + 2 * i + 1]), scale_log2, -m_base);
              const bool fma_pipe = kPoly && poly_pair(i);
              const float p0 = fma_pipe ? exp2_poly(x0) : ex2_approx(x0);
              const float p1 = fma_pipe ? exp2_poly(x1) : ex2_approx(x1);
              sums[i & 3] += p0 + p1;
              pk[i] = pack2<F16>(p0, p1);
              const float2 h2 = unpack2<F16>(pk[i]);
              pl[i] = pack2<F16>(p0 - h2.x, p1 - h2.y);
            }
            ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
            ptx::tmem_st_32x32b_x16(s_addr + 64 + c * 16, pl);
          }
        }
        l = l * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
        m_used = m_new;
        if (done >= 1) {
          ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done - 1) & 1, abort_flag, kErrWaitSoftmax));
          if (ok) {
            ptx::tc_fence_after();
            if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
              for (int c = 0; c < D / 32; ++c) {
                uint32_t o[32];
                ptx::tmem_ld_32x32b_x32(o_addr + c * 32, o);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                ptx::tmem_st_32x32b_x32(o_addr + c * 32, o);
              }
            }
          }
        }
      }
      const int nt = next_active(t);
      const bool merged = nt == t + 1 && nt < n_tiles;
      // the tiles the issuer reads after this event: V(t), and K(t+1) if merged
      if (ok) ok = __all_sync(0xffffffffu, wait_bar(b_vfull(t % kStages), kv_phase(t), abort_flag, kErrWaitSoftmax));
      if (ok && merged)
        ok = __all_sync(0xffffffffu, wait_bar(b_kfull(nt % kStages), kv_phase(nt), abort_flag, kErrWaitSoftmax));
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::named_bar_sync(kNbAck0 + x, kNbThreads);
      ptx::named_bar_arrive(kNbEvent0 + x, kNbThreads);            // P(t)
      ++done;
      if (nt < n_tiles && !merged) {
        if (ok)
          ok = __all_sync(0xffffffffu, wait_bar(b_kfull(nt % kStages), kv_phase(nt), abort_flag, kErrWaitSoftmax));
        ptx::tc_fence_before();
        ptx::named_bar_sync(kNbAck0 + x, kNbThreads);
        ptx::named_bar_arrive(kNbEvent0 + x, kNbThreads);          // K(nt)
      }
    }
    if (first < n_tiles) {
      if (ok && done > 0) {
        ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done - 1) & 1, abort_flag, kErrWaitSoftmax));
        ptx::tc_fence_after();
      }
      ptx::named_bar_sync(kNbAck0 + x, kNbThreads);                // ack of the last event
    }
    } else {
    for (int t = 0; t < n_tiles; ++t) {
      if (!active(x, t)) continue;
      ok = __all_sync(0xffffffffu, wait_bar(b_sfull(x), done & 1, abort_flag, kErrWaitSoftmax));
      if (!ok) break;
      ptx::tc_fence_after();
      const int key0 = tile_key0(t);
      const hcp_kv_segment seg = seg_at(tile_seg(t));
      int vis = seg.len - key0;
      if (seg.causal_off != kNonCausal) vis = min(vis, seg.causal_off + qrow - key0 + 1);
      vis = max(0, min(vis, kBlockN));
      // keys [0, lo) of the tile are below the row's sliding window
      const int lo = (p.window > 0 && seg.causal_off != kNonCausal) ? seg.causal_off + qrow - p.window + 1 - key0 : 0;

      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        ptx::tmem_ld_32x32b_x32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      ptx::tmem_wait_ld();
      if (vis < kBlockN || lo > 0) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= vis || i < lo) sr[i] = __float_as_uint(-INFINITY);
      }
      float mx;
      if constexpr (kWide) {
        float mx8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mx8[j] = max3(__uint_as_float(sr[j]), __uint_as_float(sr[j + 8]), __uint_as_float(sr[j + 16]));
#pragma unroll
        for (int i = 24; i < 120; i += 16)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            mx8[j] = max3(mx8[j], __uint_as_float(sr[i + j]), __uint_as_float(sr[i + 8 + j]));
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = fmaxf(mx8[j], __uint_as_float(sr[120 + j]));
        mx = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
      } else {
        float mx8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = __uint_as_float(sr[j]);
#pragma unroll
        for (int i = 8; i < 128; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(sr[i]));
        mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      }
      const float mx2 = mx * scale_log2;  // -inf stays -inf
      const bool raise = mx2 > m_used + kRescaleThreshold;
      const float m_new = raise ? mx2 : m_used;
      const float alpha = raise ? ex2_approx(m_used - m_new) : 1.f;  // 0 when m_used = -inf
      const float m_base = (m_new == -INFINITY) ? 0.f : m_new;
      float sums[4] = {0.f, 0.f, 0.f, 0.f};
      if (kWide && !precise) {
        // packed f32x2: x = s * scale - m two keys at a time, sums likewise;
        // a share of the exponentials on the FMA pipe (poly_pair_v)
        const float2 sc2 = make_float2(scale_log2, scale_log2);
        const float2 mb2 = make_float2(-m_base, -m_base);
        float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 sv = make_float2(__uint_as_float(sr[c * 32 + 2 * i]), __uint_as_float(sr[c * 32 + 2 * i + 1]));
            const float2 xx = __ffma2_rn(sv, sc2, mb2);
            float2 pp;
            if (poly_pair_v<V>(i)) pp = exp2_poly2(xx);
            else pp = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
            acc2[i & 1] = __fadd2_rn(acc2[i & 1], pp);
            pk[i] = pack2<F16>(pp.x, pp.y);
          }
          ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
        }
        sums[0] = acc2[0].x;
        sums[1] = acc2[0].y;
        sums[2] = acc2[1].x;
        sums[3] = acc2[1].y;
      } else if (!precise) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i]), scale_log2, -m_base));
            const float p1 =
                ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i + 1]), scale_log2, -m_base));
            sums[i & 3] += p0 + p1;
            pk[i] = pack2<F16>(p0, p1);
          }
          ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16], pl[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i]), scale_log2, -m_base));
            const float p1 =
                ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i + 1]), scale_log2, -m_base));
            sums[i & 3] += p0 + p1;
            pk[i] = pack2<F16>(p0, p1);
            const float2 h2 = unpack2<F16>(pk[i]);
            pl[i] = pack2<F16>(p0 - h2.x, p1 - h2.y);
          }
          ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
          ptx::tmem_st_32x32b_x16(s_addr + 64 + c * 16, pl);
        }
      }
      l = l * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
      m_used = m_new;

      if (done >= 1) {
        // O_x += P V of the previous tile must have landed before O_x is
        // rescaled and before this P is released to the MMA warp.
        ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done - 1) & 1, abort_flag, kErrWaitSoftmax));
        if (!ok) break;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld_32x32b_x32(o_addr + c * 32, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            ptx::tmem_st_32x32b_x32(o_addr + c * 32, o);
          }
        }
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(b_pfull(x));
      ++done;
    }
    if (ok && done > 0) {
      ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done - 1) & 1, abort_flag, kErrWaitSoftmax));
      ptx::tc_fence_after();
    }
    }
    if (ok) {
      // ---------------------------------------------------------- epilogue
      const bool valid = qrow < wk.q_len;
      const float LN2 = 0.69314718055994530942f;
      float lse_v = (l > 0.f) ? (m_used + lg2_approx(l)) * LN2 : -INFINITY;
      float f_new = (l > 0.f) ? 1.f / l : 0.f;
      float f_old = 0.f;
      const long long out_row = static_cast<long long>(wk.q_start) + qrow;
      const long long lse_idx_col = static_cast<long long>(wk.lse_col) + qrow;
      const bool merging = p.merge_lse != nullptr;
      if (merging && valid) {
        float lp = p.merge_lse[head * p.merge_lse_stride + lse_idx_col];
        if (lp == INFINITY) lp = -INFINITY;
        const float mm = fmaxf(lp, lse_v);
        if (mm == -INFINITY) {
          f_new = 0.f;
          lse_v = -INFINITY;
        } else {
          const float wp = __expf(lp - mm);
          const float wn = __expf(lse_v - mm);
          const float r = 1.f / (wp + wn);
          f_old = wp * r;
          f_new *= wn * r;
          lse_v = mm + __logf(wp + wn);
        }
      }
      const long long col0 = static_cast<long long>(head) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (done > 0) {
          ptx::tmem_ld_32x32b_x32(o_addr + c * 32, r);
          ptx::tmem_wait_ld();
        }
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = done > 0 ? __uint_as_float(r[i]) * f_new : 0.f;
        if (!valid) continue;
        if (merging) {
          const long long base = out_row * p.merge_o_row_stride + col0 + c * 32;
          if (p.merge_o_f32) {
            const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.merge_o) + base);
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4) {
              const float4 v = src[q4];
              o[4 * q4 + 0] += v.x * f_old;
              o[4 * q4 + 1] += v.y * f_old;
              o[4 * q4 + 2] += v.z * f_old;
              o[4 * q4 + 3] += v.w * f_old;
            }
          } else {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.merge_o) + base);
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
              const uint4 v = src[q8];
              const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<F16>(w[e]);
                o[8 * q8 + 2 * e] += f.x * f_old;
                o[8 * q8 + 2 * e + 1] += f.y * f_old;
              }
            }
          }
        }
        const long long obase = out_row * p.out_row_stride + col0 + c * 32;
        if (p.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4)
            dst[q4] = make_float4(o[4 * q4], o[4 * q4 + 1], o[4 * q4 + 2], o[4 * q4 + 3]);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + obase);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            dst[q8] = make_uint4(pack2<F16>(o[8 * q8], o[8 * q8 + 1]), pack2<F16>(o[8 * q8 + 2], o[8 * q8 + 3]),
                                 pack2<F16>(o[8 * q8 + 4], o[8 * q8 + 5]),
                                 pack2<F16>(o[8 * q8 + 6], o[8 * q8 + 7]));
        }
      }
      if (valid && p.lse != nullptr) p.lse[head * p.lse_stride + lse_idx_col] = lse_v;
    }
  }
  }

  // ---- teardown: release TMEM once every role is done with it
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D>
constexpr int fwd_smem_bytes() {
  return FwdSmem<D>::kBytes;
}

}  // namespace hcp
