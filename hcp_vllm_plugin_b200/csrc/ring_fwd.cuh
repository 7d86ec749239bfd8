// Fused ring-attention forward for B200 (sm_100a).
//
// One CTA computes one 128-row query tile of one query head over the union
// of up to two KV segments (the transient peer prefix, non-causal, and the
// local chunk, causal at a global offset), with a single online softmax, and
// writes the normalised output plus the per-row natural-log LSE.  An earlier
// partial (O, LSE) can be merged in the epilogue, so ring hops chain without a
// separate merge kernel.
//
// Warp roles (320 threads):
//   warps 0-7  softmax / O correction / epilogue.  Query row r of the tile is
//              TMEM lane r; warp w handles lanes 32*(w%4).. and key/column half
//              w/4 of every S tile (two threads per row, which keeps two
//              softmax warps per SM sub-partition in flight).  The two halves
//              of a row exchange their partial row max through shared memory
//              once per KV tile (bounded mbarrier, never bar.sync).
//   warp 8     TMA producer: Q once, then K and V tiles through a 2-stage ring
//              (contiguous 3-D tensor maps, or 4-D maps over the paged cache
//              indexed through the block table)
//   warp 9     tcgen05 MMA issuer (one lane) and TMEM owner
//
// TMEM (512 columns x 128 lanes, fp32):
//   [  0,128)  S buffer 0      S = Q K^T of even KV tiles.  P (16-bit, two keys
//   [128,256)  S buffer 1      per column) is written back over columns 0-63 and
//                              feeds O += P V as the A operand; for short rows
//                              the low part P - bf16(P) goes to columns 64-127
//                              and is accumulated by a second PV product
//   [256,256+D) O accumulator
//
// Shared memory (1024-byte aligned, 128-byte swizzle, 64-element boxes):
//   Q tile, then per stage a K tile and a V tile, then the row-max exchange
//   buffers and the mbarriers.
//
// Numerics: scores are scaled into the base-2 domain (scale * log2 e), the
// running max is only raised when a tile's max exceeds it by more than 8
// (P stays <= 2^8) and O is rescaled in TMEM only then.
// LSE = (m + log2 l) * ln 2.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "hcp_ring.h"
#include "sm100_ptx.cuh"

namespace hcp {

__device__ int g_device_status = 0;

constexpr int kBlockM = 128;
constexpr int kBlockN = 128;
constexpr int kStages = 2;
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kWarpTma = 8;
constexpr int kWarpMma = 9;
constexpr int kThreads = 320;
constexpr int kMaxWork = 160;
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;  // 4 s
constexpr float kRescaleThreshold = 8.0f;            // log2 units
constexpr int kPreciseKeys = 256;  // rows seeing fewer keys get the hi+lo P product

// Failure codes written to g_device_status.
enum : int {
  kErrWaitProducer = 0x101,
  kErrWaitMma = 0x102,
  kErrWaitSoftmax = 0x103,
  kErrWaitDrain = 0x104,
};

struct FwdParams {
  CUtensorMap tm_q;      // {D, H, q_rows}     box {64, 1, 128}
  CUtensorMap tm_ka;     // {D, Hkv, rows_a}   box {64, 1, 128}
  CUtensorMap tm_va;
  CUtensorMap tm_kb;
  CUtensorMap tm_vb;
  CUtensorMap tm_cache;  // {2D, bs, Hkv, nb}  box {64, bs, 1, 1}
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
  int tile_off[kMaxWork + 1];
  hcp_attn_work work[kMaxWork];
};

// Bounded mbarrier wait.  Returns false when this CTA aborted (this wait ran
// out of time, another role of the CTA gave up, or another CTA failed).
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         int code) {
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
      if (ptx::global_timer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        atomicCAS(&g_device_status, 0, code);
        return false;
      }
    }
  }
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

// Keys of segment `sg` visible to the valid rows [q0, q0+rows) of a query tile.
__device__ __forceinline__ int segment_keys(const hcp_kv_segment& sg, int q0, int rows) {
  if (sg.src == HCP_SRC_NONE || sg.len <= 0) return 0;
  if (sg.causal_off < 0) return sg.len;
  const long long last_visible = static_cast<long long>(sg.causal_off) + q0 + rows;  // exclusive
  return static_cast<int>(max(0ll, min(static_cast<long long>(sg.len), last_visible)));
}

template <int D>
struct FwdSmem {
  static constexpr int kBoxBytes = 128 * 128;  // 128 rows x 64 elems x 2 B
  static constexpr int kTileBytes = (D / 64) * kBoxBytes;
  static constexpr int kNumBars = 9 + 4 * kStages;
  static constexpr int kRedOff = kTileBytes * (1 + 2 * kStages);  // float red[2][2][128]
  static constexpr int kBarOff = kRedOff + 2 * 2 * 128 * 4;
  static constexpr int kEnd = kBarOff + 8 * kNumBars + 16;
  static constexpr int kBytes = kEnd + 1024;  // + alignment slack
};

template <int D, bool F16>
__global__ void __launch_bounds__(kThreads, 1) ring_fwd_kernel(const __grid_constant__ FwdParams p) {
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
  const uint32_t s_q = ptx::smem_u32(smem);
  const uint32_t s_kv0 = s_q + kTileBytes;  // stage s: K at +2s tiles, V at +2s+1 tiles
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t bar0 = ptx::smem_u32(bars);
  const uint32_t b_q = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + kStages + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + 2 * kStages + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 3 * kStages + s); };
  auto b_sfull = [&](int b) { return bar0 + 8u * (1 + 4 * kStages + b); };
  auto b_pfull = [&](int b) { return bar0 + 8u * (3 + 4 * kStages + b); };
  auto b_red = [&](int b) { return bar0 + 8u * (5 + 4 * kStages + b); };
  const uint32_t b_odone = bar0 + 8u * (7 + 4 * kStages);
  const uint32_t b_final = bar0 + 8u * (8 + 4 * kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- which (work item, query tile, head) this CTA owns
  const int H = p.num_heads;
  const int tile_global = blockIdx.x / H;
  const int head = blockIdx.x - tile_global * H;
  const int kvh = head / p.group;
  int lo = 0, hi = p.num_work - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_off[mid] <= tile_global) lo = mid; else hi = mid - 1;
  }
  const hcp_attn_work& wk = p.work[lo];
  const int n_qtiles = (wk.q_len + kBlockM - 1) / kBlockM;
  const int m_tile = n_qtiles - 1 - (tile_global - p.tile_off[lo]);  // heaviest (last) tile first
  const int q0 = m_tile * kBlockM;
  const int rows_valid = min(kBlockM, wk.q_len - q0);
  const int keys0 = segment_keys(wk.seg[0], q0, rows_valid);
  const int keys1 = segment_keys(wk.seg[1], q0, rows_valid);
  const int tiles0 = (keys0 + kBlockN - 1) / kBlockN;
  const int n_tiles = tiles0 + (keys1 + kBlockN - 1) / kBlockN;
  // Rows that see few keys in total get P as hi + lo 16-bit parts.
  const bool precise =
      segment_keys(wk.seg[0], q0, 1) + segment_keys(wk.seg[1], q0, 1) < kPreciseKeys;

  // ---- setup
  if (threadIdx.x == 0) {
    ptx::mbar_init(b_q, 1);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(b_kfull(s), 1);
      ptx::mbar_init(b_kempty(s), 1);
      ptx::mbar_init(b_vfull(s), 1);
      ptx::mbar_init(b_vempty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(b_sfull(b), 1);
      ptx::mbar_init(b_pfull(b), kSoftmaxThreads);
      ptx::mbar_init(b_red(b), kSoftmaxWarps);
    }
    ptx::mbar_init(b_odone, 1);
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
  const bool skip_all = *abort_flag != 0;

  if (skip_all) {
    // nothing issued, nothing to drain
  } else if (warp == kWarpTma) {
    // ================================================================ producer
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(b_q, kTileBytes);
      for (int hf = 0; hf < kHalves; ++hf)
        ptx::tma_load_3d(s_q + hf * kBoxBytes, &p.tm_q, b_q, hf * 64, head, wk.q_start + q0);
    }
    int k_issued = 0, v_issued = 0;
    for (int t = 0; t < n_tiles; ++t) {
      const int s = t % kStages;
      const uint32_t ph = (t / kStages) & 1;
      const int sg = t < tiles0 ? 0 : 1;
      const int key0 = (sg == 0 ? t : t - tiles0) * kBlockN;
      const hcp_kv_segment& seg = wk.seg[sg];
      const uint32_t s_k = s_kv0 + (2 * s) * kTileBytes;
      const uint32_t s_v = s_k + kTileBytes;
      int blk_ids[8];
      const bool paged = seg.src == HCP_SRC_PAGED;
      const int bs = p.block_size;
      const int nblk = kBlockN / bs;
      if (paged) {
        int blk = static_cast<int>(p.num_blocks);  // out of range: TMA fills zeros
        if (lane < nblk) {
          const int rel = key0 + lane * bs;
          const long long bidx = (static_cast<long long>(seg.start) + rel) / bs;
          if (rel < seg.len && bidx < p.bt_stride && wk.paged_req >= 0 && wk.paged_req < p.bt_rows) {
            const int v = __ldg(p.block_table + wk.paged_req * p.bt_stride + bidx);
            if (v >= 0 && v < p.num_blocks) blk = v;
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) blk_ids[i] = __shfl_sync(0xffffffffu, blk, i);
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
          const CUtensorMap* tk = seg.src == HCP_SRC_A ? &p.tm_ka : &p.tm_kb;
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
          const CUtensorMap* tv = seg.src == HCP_SRC_A ? &p.tm_va : &p.tm_vb;
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
    bool ok = __all_sync(0xffffffffu, wait_bar(b_q, 0, abort_flag, kErrWaitMma));
    auto issue_pv = [&](int j) -> bool {
      const int s = j % kStages;
      const uint32_t ph = (j / kStages) & 1;
      const int b = j & 1;
      if (!__all_sync(0xffffffffu, wait_bar(b_pfull(b), (j >> 1) & 1, abort_flag, kErrWaitMma)))
        return false;
      if (!__all_sync(0xffffffffu, wait_bar(b_vfull(s), ph, abort_flag, kErrWaitMma))) return false;
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint32_t s_v = s_kv0 + (2 * s + 1) * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
          ptx::umma_ts(tmem + 256, tmem + b * 128 + kk * 8, bdesc, kIdescPV,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
        if (precise) {
#pragma unroll
          for (int kk = 0; kk < kBlockN / 16; ++kk) {
            const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
            ptx::umma_ts(tmem + 256, tmem + b * 128 + 64 + kk * 8, bdesc, kIdescPV, 1u);
          }
        }
        ptx::umma_commit(b_vempty(s));
        ptx::umma_commit(b_odone);
      }
      __syncwarp();
      return true;
    };
    for (int t = 0; t < n_tiles && ok; ++t) {
      const int s = t % kStages;
      const uint32_t ph = (t / kStages) & 1;
      const int b = t & 1;
      ok = __all_sync(0xffffffffu, wait_bar(b_kfull(s), ph, abort_flag, kErrWaitMma));
      if (!ok) break;
      ptx::tc_fence_after();
      if (lane == 0) {
        const uint32_t s_k = s_kv0 + (2 * s) * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
          const uint64_t adesc = ptx::sdesc_sw128(s_q + off, 16, 1024);
          const uint64_t bdesc = ptx::sdesc_sw128(s_k + off, 16, 1024);
          ptx::umma_ss(tmem + b * 128, adesc, bdesc, kIdescQK, kk > 0 ? 1u : 0u);
        }
        ptx::umma_commit(b_sfull(b));
        ptx::umma_commit(b_kempty(s));
      }
      __syncwarp();
      if (t >= 1) ok = issue_pv(t - 1);
    }
    if (ok && n_tiles > 0) ok = issue_pv(n_tiles - 1);
    // Teardown: no MMA may be in flight when TMEM is released.
    if (lane == 0) ptx::umma_commit(b_final);
    __syncwarp();
    drain_bar(b_final, 0);
  } else {
    // ================================================================ softmax + epilogue
    const int quarter = warp & 3;
    const int half = warp >> 2;                  // which 64 keys of each S tile / D/2 of O
    const int row = quarter * 32 + lane;         // == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int qrow = q0 + row;                   // work-item-relative query row
    const float scale_log2 = p.scale_log2;
    constexpr int kOHalf = D / 2;                // O columns owned by this thread
    float m_used = -INFINITY;  // running max of the row, base-2 scaled domain
    float l = 0.f;             // this thread's share of the row sum
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int b = t & 1;
      ok = __all_sync(0xffffffffu, wait_bar(b_sfull(b), (t >> 1) & 1, abort_flag, kErrWaitSoftmax));
      if (!ok) break;
      ptx::tc_fence_after();
      const int sg = t < tiles0 ? 0 : 1;
      const int key0 = (sg == 0 ? t : t - tiles0) * kBlockN + half * 64;
      const hcp_kv_segment& seg = wk.seg[sg];
      int vis = seg.len - key0;
      if (seg.causal_off >= 0) vis = min(vis, seg.causal_off + qrow - key0 + 1);
      vis = max(0, min(vis, 64));

      uint32_t sr[64];
      const uint32_t s_addr = tmem + lane_base + b * 128 + half * 64;
      ptx::tmem_ld_32x32b_x32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      ptx::tmem_ld_32x32b_x32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      ptx::tmem_wait_ld();

      float mx = -INFINITY;
      if (vis >= 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float x = i < vis ? __uint_as_float(sr[i]) : -INFINITY;
          sr[i] = __float_as_uint(x);
          mx = fmaxf(mx, x);
        }
      }
      // exchange the partial max with the other half of the row
      float* red_t = red + (t & 1) * 256;
      red_t[half * 128 + row] = mx;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(b_red(b));
      ok = __all_sync(0xffffffffu, wait_bar(b_red(b), (t >> 1) & 1, abort_flag, kErrWaitSoftmax));
      if (!ok) break;
      mx = fmaxf(mx, red_t[(half ^ 1) * 128 + row]);

      const float mx2 = mx * scale_log2;  // -inf stays -inf
      const bool raise = mx2 > m_used + kRescaleThreshold;
      const float m_new = raise ? mx2 : m_used;
      const float alpha = raise ? ex2_approx(m_used - m_new) : 1.f;  // 0 when m_used = -inf
      const float m_base = (m_new == -INFINITY) ? 0.f : m_new;
      float sum0 = 0.f, sum1 = 0.f;
      uint32_t pk[32];
      const uint32_t p_addr = tmem + lane_base + b * 128 + half * 32;
      if (!precise) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * i]), scale_log2, -m_base));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * i + 1]), scale_log2, -m_base));
          sum0 += p0;
          sum1 += p1;
          pk[i] = pack2<F16>(p0, p1);
        }
        ptx::tmem_st_32x32b_x32(p_addr, pk);
      } else {
        uint32_t pl[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * i]), scale_log2, -m_base));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * i + 1]), scale_log2, -m_base));
          sum0 += p0;
          sum1 += p1;
          pk[i] = pack2<F16>(p0, p1);
          const float2 hi2 = unpack2<F16>(pk[i]);
          pl[i] = pack2<F16>(p0 - hi2.x, p1 - hi2.y);
        }
        ptx::tmem_st_32x32b_x32(p_addr, pk);
        ptx::tmem_st_32x32b_x32(p_addr + 64, pl);
      }
      l = l * alpha + (sum0 + sum1);
      m_used = m_new;

      if (t >= 1) {
        // O += P_{t-1} V_{t-1} must have landed before O is rescaled and
        // before P_t is released to the MMA warp.
        ok = __all_sync(0xffffffffu, wait_bar(b_odone, (t - 1) & 1, abort_flag, kErrWaitSoftmax));
        if (!ok) break;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
          const uint32_t o_addr = tmem + lane_base + 256 + half * kOHalf;
#pragma unroll
          for (int c = 0; c < kOHalf / 32; ++c) {
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
      ptx::mbar_arrive(b_pfull(b));
    }

    if (ok && n_tiles > 0) {
      ok = __all_sync(0xffffffffu, wait_bar(b_odone, (n_tiles - 1) & 1, abort_flag, kErrWaitSoftmax));
      ptx::tc_fence_after();
      if (ok) {
        // combine the two halves' row sums (same exchange as the row max)
        const int b = n_tiles & 1;
        float* red_t = red + b * 256;
        red_t[half * 128 + row] = l;
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(b_red(b));
        ok = __all_sync(0xffffffffu,
                        wait_bar(b_red(b), (n_tiles >> 1) & 1, abort_flag, kErrWaitSoftmax));
        if (ok) l += red_t[(half ^ 1) * 128 + row];
      }
    }
    if (ok) {
      // ---------------------------------------------------------- epilogue
      float o[kOHalf];
      if (n_tiles > 0) {
        uint32_t ob[kOHalf];
        const uint32_t o_addr = tmem + lane_base + 256 + half * kOHalf;
#pragma unroll
        for (int c = 0; c < kOHalf / 32; ++c)
          ptx::tmem_ld_32x32b_x32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&ob[c * 32]));
        ptx::tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < kOHalf; ++i) o[i] = __uint_as_float(ob[i]);
      } else {
#pragma unroll
        for (int i = 0; i < kOHalf; ++i) o[i] = 0.f;
      }
      const bool valid = qrow < wk.q_len;
      if (valid) {
        const float LN2 = 0.69314718055994530942f;
        float lse_v = (l > 0.f) ? (m_used + lg2_approx(l)) * LN2 : -INFINITY;
        float f_new = (l > 0.f) ? 1.f / l : 0.f;
        float f_old = 0.f;
        const long long out_row = static_cast<long long>(wk.q_start) + qrow;
        const long long lse_idx_col = static_cast<long long>(wk.lse_col) + qrow;
        const long long col0 = static_cast<long long>(head) * D + half * kOHalf;
        if (p.merge_lse != nullptr) {
          float lp = p.merge_lse[head * p.merge_lse_stride + lse_idx_col];
          if (lp == INFINITY) lp = -INFINITY;
          const float mm = fmaxf(lp, lse_v);
          if (mm == -INFINITY) {
            f_new = 0.f;
            f_old = 0.f;
            lse_v = -INFINITY;
          } else {
            const float wp = __expf(lp - mm);
            const float wn = __expf(lse_v - mm);
            const float inv = 1.f / (wp + wn);
            f_old = wp * inv;
            f_new *= wn * inv;
            lse_v = mm + __logf(wp + wn);
          }
          const long long base = out_row * p.merge_o_row_stride + col0;
          if (p.merge_o_f32) {
            const float4* src =
                reinterpret_cast<const float4*>(static_cast<const float*>(p.merge_o) + base);
#pragma unroll
            for (int c = 0; c < kOHalf / 4; ++c) {
              const float4 v = src[c];
              o[4 * c + 0] = o[4 * c + 0] * f_new + v.x * f_old;
              o[4 * c + 1] = o[4 * c + 1] * f_new + v.y * f_old;
              o[4 * c + 2] = o[4 * c + 2] * f_new + v.z * f_old;
              o[4 * c + 3] = o[4 * c + 3] * f_new + v.w * f_old;
            }
          } else {
            const uint4* src =
                reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.merge_o) + base);
#pragma unroll
            for (int c = 0; c < kOHalf / 8; ++c) {
              const uint4 v = src[c];
              const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = unpack2<F16>(w[e]);
                o[8 * c + 2 * e] = o[8 * c + 2 * e] * f_new + f.x * f_old;
                o[8 * c + 2 * e + 1] = o[8 * c + 2 * e + 1] * f_new + f.y * f_old;
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < kOHalf; ++i) o[i] *= f_new;
        }
        const long long obase = out_row * p.out_row_stride + col0;
        if (p.out_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + obase);
#pragma unroll
          for (int c = 0; c < kOHalf / 4; ++c)
            dst[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + obase);
#pragma unroll
          for (int c = 0; c < kOHalf / 8; ++c)
            dst[c] = make_uint4(pack2<F16>(o[8 * c], o[8 * c + 1]), pack2<F16>(o[8 * c + 2], o[8 * c + 3]),
                                pack2<F16>(o[8 * c + 4], o[8 * c + 5]),
                                pack2<F16>(o[8 * c + 6], o[8 * c + 7]));
        }
        if (p.lse != nullptr && half == 0) p.lse[head * p.lse_stride + lse_idx_col] = lse_v;
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
