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
//   warps 0-7  two softmax warpgroups.  Warpgroup g (warps 4g..4g+3) owns
//              the KV tiles t with t % 2 == g: it keeps its own online-softmax
//              state (running max, row sum) and its own O accumulator, so the
//              two warps that share an SM sub-partition work on different
//              tiles, out of phase.  Thread (w, lane) owns query row
//              32*(w%4)+lane, which is TMEM lane 32*(w%4)+lane.  The two
//              partial results are merged once, in the epilogue.
//   warp 8     TMA producer: Q once, then K and V tiles through a 2-stage ring
//              (contiguous 3-D tensor maps, or 4-D maps over the paged cache
//              indexed through the block table)
//   warp 9     tcgen05 MMA issuer (one lane) and TMEM owner
//
// TMEM (512 columns x 128 lanes, fp32):
//   [  0,128)      S_0 = Q K^T of even KV tiles, [128,256) S_1 of odd tiles.
//                  P (16-bit, two keys per column) is written back over
//                  columns 0-63 of its S buffer and feeds O_g += P V as the A
//                  operand; for short rows the low part P - bf16(P) goes to
//                  columns 64-127 and is accumulated by a second PV product.
//   [256,256+D)    O_0 (even tiles), [256+D, 256+2D) O_1 (odd tiles)
//
// Shared memory (1024-byte aligned, 128-byte swizzle, 64-element boxes):
//   Q tile, then per stage a K tile and a V tile, then the epilogue exchange
//   buffer and the mbarriers.
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
  auto b_odone = [&](int b) { return bar0 + 8u * (5 + 4 * kStages + b); };
  const uint32_t b_red = bar0 + 8u * (7 + 4 * kStages);
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
      ptx::mbar_init(b_pfull(b), kSoftmaxThreads / 2);
      ptx::mbar_init(b_odone(b), 1);
    }
    ptx::mbar_init(b_red, kSoftmaxWarps);
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
        const uint32_t o_acc = tmem + 256 + b * D;  // O_b accumulates the tiles of parity b
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
          ptx::umma_ts(o_acc, tmem + b * 128 + kk * 8, bdesc, kIdescPV, (j >= 2 || kk > 0) ? 1u : 0u);
        }
        if (precise) {
#pragma unroll
          for (int kk = 0; kk < kBlockN / 16; ++kk) {
            const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
            ptx::umma_ts(o_acc, tmem + b * 128 + 64 + kk * 8, bdesc, kIdescPV, 1u);
          }
        }
        ptx::umma_commit(b_vempty(s));
        ptx::umma_commit(b_odone(b));
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
    const int g = warp >> 2;                 // warpgroup: KV tiles t with t % 2 == g
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;     // == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int qrow = q0 + row;               // work-item-relative query row
    const float scale_log2 = p.scale_log2;
    const uint32_t s_addr = tmem + lane_base + g * 128;
    const uint32_t o_own = tmem + lane_base + 256 + g * D;
    constexpr int kOHalf = D / 2;            // output columns this thread writes
    float m_used = -INFINITY;  // running max over this warpgroup's tiles, base-2 scaled domain
    float l = 0.f;             // row sum over this warpgroup's tiles
    bool ok = true;
    int my_tiles = 0;
    for (int t = g; t < n_tiles; t += 2) {
      ok = __all_sync(0xffffffffu, wait_bar(b_sfull(g), (t >> 1) & 1, abort_flag, kErrWaitSoftmax));
      if (!ok) break;
      ptx::tc_fence_after();
      const int sg = t < tiles0 ? 0 : 1;
      const int key0 = (sg == 0 ? t : t - tiles0) * kBlockN;
      const hcp_kv_segment& seg = wk.seg[sg];
      int vis = seg.len - key0;
      if (seg.causal_off >= 0) vis = min(vis, seg.causal_off + qrow - key0 + 1);
      vis = max(0, min(vis, kBlockN));

      uint32_t sr[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        ptx::tmem_ld_32x32b_x32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      ptx::tmem_wait_ld();
      if (vis < kBlockN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= vis) sr[i] = __float_as_uint(-INFINITY);
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

      if (my_tiles >= 1) {
        // O_g += P V of this warpgroup's previous tile must have landed before
        // O_g is rescaled and before this P is released to the MMA warp.
        ok = __all_sync(0xffffffffu,
                        wait_bar(b_odone(g), (my_tiles - 1) & 1, abort_flag, kErrWaitSoftmax));
        if (!ok) break;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld_32x32b_x32(o_own + c * 32, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            ptx::tmem_st_32x32b_x32(o_own + c * 32, o);
          }
        }
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(b_pfull(g));
      ++my_tiles;
    }
    if (ok && my_tiles > 0) {
      ok = __all_sync(0xffffffffu,
                      wait_bar(b_odone(g), (my_tiles - 1) & 1, abort_flag, kErrWaitSoftmax));
      ptx::tc_fence_after();
    }
    // exchange (running max, row sum) with the other warpgroup; its O buffer
    // is complete once it has arrived here
    float2* xch = reinterpret_cast<float2*>(red);  // [2][128]
    if (ok) {
      xch[g * 128 + row] = make_float2(m_used, l);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(b_red);
      ok = __all_sync(0xffffffffu, wait_bar(b_red, 0, abort_flag, kErrWaitSoftmax));
      ptx::tc_fence_after();
    }
    if (ok) {
      // ---------------------------------------------------------- epilogue
      const float2 other = xch[(g ^ 1) * 128 + row];
      const float m0 = g == 0 ? m_used : other.x, l0 = g == 0 ? l : other.y;
      const float m1 = g == 0 ? other.x : m_used, l1 = g == 0 ? other.y : l;
      const float mm2 = fmaxf(m0, m1);
      float f0 = 0.f, f1 = 0.f, lsum = 0.f;
      if (mm2 != -INFINITY) {
        f0 = l0 > 0.f ? ex2_approx(m0 - mm2) : 0.f;
        f1 = l1 > 0.f ? ex2_approx(m1 - mm2) : 0.f;
        lsum = l0 * f0 + l1 * f1;
      }
      const bool valid = qrow < wk.q_len;
      const float LN2 = 0.69314718055994530942f;
      float lse_v = (lsum > 0.f) ? (mm2 + lg2_approx(lsum)) * LN2 : -INFINITY;
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      f0 *= inv;
      f1 *= inv;
      float f_old = 0.f;
      const long long out_row = static_cast<long long>(wk.q_start) + qrow;
      const long long lse_idx_col = static_cast<long long>(wk.lse_col) + qrow;
      const bool merging = p.merge_lse != nullptr;
      if (merging && valid) {
        float lp = p.merge_lse[head * p.merge_lse_stride + lse_idx_col];
        if (lp == INFINITY) lp = -INFINITY;
        const float mm = fmaxf(lp, lse_v);
        if (mm == -INFINITY) {
          f0 = f1 = 0.f;
          lse_v = -INFINITY;
        } else {
          const float wp = __expf(lp - mm);
          const float wn = __expf(lse_v - mm);
          const float r = 1.f / (wp + wn);
          f_old = wp * r;
          f0 *= wn * r;
          f1 *= wn * r;
          lse_v = mm + __logf(wp + wn);
        }
      }
      const bool have0 = n_tiles >= 1, have1 = n_tiles >= 2;
      const long long col0 = static_cast<long long>(head) * D + g * kOHalf;
#pragma unroll
      for (int c = 0; c < kOHalf / 32; ++c) {
        uint32_t r0[32], r1[32];
        if (have0) ptx::tmem_ld_32x32b_x32(tmem + lane_base + 256 + g * kOHalf + c * 32, r0);
        if (have1) ptx::tmem_ld_32x32b_x32(tmem + lane_base + 256 + D + g * kOHalf + c * 32, r1);
        ptx::tmem_wait_ld();
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          o[i] = (have0 ? __uint_as_float(r0[i]) * f0 : 0.f) + (have1 ? __uint_as_float(r1[i]) * f1 : 0.f);
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
      if (valid && p.lse != nullptr && g == 0) p.lse[head * p.lse_stride + lse_idx_col] = lse_v;
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
