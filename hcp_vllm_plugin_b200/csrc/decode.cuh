// Split-KV decode for B200 (sm_100a): one query token per sequence attends
// the transient peer segment (contiguous) and the local segment (paged cache).
//
// The work is HBM-bound (every K/V byte is used for 7 FLOP per GQA group), so
// the design streams K/V with TMA as fast as HBM delivers it:
//   * a CTA owns one (sequence, KV head, key chunk): it reads that chunk's K
//     and V exactly once and serves all query heads of the KV head (GQA);
//   * chunks never straddle the peer/local boundary, so each TMA tile comes
//     from one source: 3-D maps over [rows, Hkv, D] (peer) or 4-D maps over
//     [num_blocks, Hkv, block_size, 2D] through the block table (local);
//   * 128-byte swizzled tiles make the tensor-core fragment reads
//     conflict-free; a 3-stage ring keeps ~96 KB in flight per CTA;
//   * 4 consumer warps split each 64-key tile (16 keys each), compute
//     S = q K^T and O += P V with register-resident mma.sync fragments (the
//     query heads are the M dimension, padded to 16) and keep an online
//     softmax per warp; the CTA merges its warps and writes a normalised
//     partial (O, LSE) to the workspace;
//   * a second kernel merges the chunk partials of every (sequence, head).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "hcp_ring.h"
#include "sm100_ptx.cuh"

namespace hcp {

constexpr int kDecTileKeys = 64;
constexpr int kDecStages = 3;
constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kDecMaxSeqs = 256;
constexpr int kDecMaxGroup = 16;

struct DecodeSeq {
  int q_row;
  int peer_start;
  int peer_len;
  int paged_req;
  int local_start;
  int local_len;
  int peer_src;  // -1: the peer arena (tm_pk / tm_pv); i: extra source i
};

struct DecodeParams {
  CUtensorMap tm_pk;     // peer K {D, Hkv, rows}   box {64, 1, 64}
  CUtensorMap tm_pv;     // peer V
  CUtensorMap tm_cache;  // {2D, bs, Hkv, nb}       box {64, bs, 1, 1}
  CUtensorMap tm_epk[HCP_MAX_EXT_SOURCES];  // extra peer sources, as tm_pk / tm_pv
  CUtensorMap tm_epv[HCP_MAX_EXT_SOURCES];
  const void* q;
  long long q_row_stride;
  const int32_t* block_table;
  long long bt_stride;
  long long bt_rows;
  long long num_blocks;
  float* part_o;      // [units, H, D]
  float* part_lse;    // [units, H]
  int num_heads;
  int num_kv_heads;
  int group;
  int block_size;
  int chunk_keys;     // keys per unit (multiple of kDecTileKeys)
  float scale_log2;
  int num_seqs;
  int total_units;
  int unit_off[kDecMaxSeqs + 1];  // prefix sums of units per sequence
  DecodeSeq seq[kDecMaxSeqs];
};

template <int D>
struct DecSmem {
  static constexpr int kHalfBytes = kDecTileKeys * 128;          // 64 keys x 64 dims x 2 B
  static constexpr int kTileBytes = (D / 64) * kHalfBytes;       // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;             // K + V
  // the warps' partials reuse the stage buffers once every tile is consumed
  static constexpr int kRedOff = 0;
  static constexpr int kRedBytes = kDecConsumerWarps * (kDecMaxGroup * D + 2 * kDecMaxGroup) * 4;
  static_assert(kRedBytes <= kDecStages * kStageBytes, "merge buffer must fit in the stages");
  static constexpr int kBarOff = kDecStages * kStageBytes;
  static constexpr int kEnd = kBarOff + 8 * (2 * kDecStages) + 16;
  static constexpr int kBytes = kEnd + 1024;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool F16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled 64-column box.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int D, bool F16>
__global__ void __launch_bounds__(kDecThreads) decode_splitkv_kernel(const __grid_constant__ DecodeParams p) {
  using L = DecSmem<D>;
  constexpr int kHalves = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s0 = ptx::smem_u32(smem);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kDecStages);
  const uint32_t bar0 = ptx::smem_u32(bars);
  auto b_full = [&](int s) { return bar0 + 8u * s; };
  auto b_empty = [&](int s) { return bar0 + 8u * (kDecStages + s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  const int kvh = blockIdx.y;
  // ---- which sequence / segment / key range
  int lo = 0, hi = p.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.unit_off[mid] <= unit) lo = mid; else hi = mid - 1;
  }
  const DecodeSeq& sq = p.seq[lo];
  const int u_in = unit - p.unit_off[lo];
  const int peer_units = (sq.peer_len + p.chunk_keys - 1) / p.chunk_keys;
  const bool is_peer = u_in < peer_units;
  const int key_begin = (is_peer ? u_in : u_in - peer_units) * p.chunk_keys;
  const int seg_len = is_peer ? sq.peer_len : sq.local_len;
  const int n_keys = min(p.chunk_keys, seg_len - key_begin);
  const int n_tiles = (n_keys + kDecTileKeys - 1) / kDecTileKeys;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      ptx::mbar_init(b_full(s), 1);
      ptx::mbar_init(b_empty(s), kDecConsumerWarps);
    }
    *abort_flag = *reinterpret_cast<volatile int*>(&g_device_status) != 0 ? 1 : 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const bool skip_all = *abort_flag != 0;

  if (warp == kDecConsumerWarps) {
    // ============================================================ producer
    if (skip_all) return;
    int issued = 0;
    for (int t = 0; t < n_tiles; ++t) {
      const int s = t % kDecStages;
      const uint32_t ph = (t / kDecStages) & 1;
      const int k0 = key_begin + t * kDecTileKeys;  // segment-relative
      int blk = static_cast<int>(p.num_blocks);
      const int bs = p.block_size;
      const int nblk = kDecTileKeys / bs;
      if (!is_peer && lane < nblk) {
        const int rel = k0 + lane * bs;
        const long long bidx = (static_cast<long long>(sq.local_start) + rel) / bs;
        if (rel < seg_len && bidx < p.bt_stride && sq.paged_req >= 0 && sq.paged_req < p.bt_rows) {
          const int v = __ldg(p.block_table + sq.paged_req * p.bt_stride + bidx);
          if (v >= 0 && v < p.num_blocks) blk = v;
        }
      }
      int ids[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ids[i] = __shfl_sync(0xffffffffu, blk, i);
      if (!__all_sync(0xffffffffu, wait_bar(b_empty(s), ph ^ 1, abort_flag, kErrWaitProducer))) break;
      if (lane == 0) {
        const uint32_t sk = s0 + s * L::kStageBytes;
        const uint32_t sv = sk + L::kTileBytes;
        ptx::mbar_arrive_expect_tx(b_full(s), L::kStageBytes);
        if (is_peer) {
          const CUtensorMap* tpk = sq.peer_src < 0 ? &p.tm_pk : &p.tm_epk[sq.peer_src];
          const CUtensorMap* tpv = sq.peer_src < 0 ? &p.tm_pv : &p.tm_epv[sq.peer_src];
          for (int hf = 0; hf < kHalves; ++hf) {
            ptx::tma_load_3d(sk + hf * L::kHalfBytes, tpk, b_full(s), hf * 64, kvh, sq.peer_start + k0);
            ptx::tma_load_3d(sv + hf * L::kHalfBytes, tpv, b_full(s), hf * 64, kvh, sq.peer_start + k0);
          }
        } else {
          for (int i = 0; i < nblk; ++i)
            for (int hf = 0; hf < kHalves; ++hf) {
              ptx::tma_load_4d(sk + hf * L::kHalfBytes + i * bs * 128, &p.tm_cache, b_full(s), hf * 64, 0,
                               kvh, ids[i]);
              ptx::tma_load_4d(sv + hf * L::kHalfBytes + i * bs * 128, &p.tm_cache, b_full(s),
                               D + hf * 64, 0, kvh, ids[i]);
            }
        }
      }
      issued = t + 1;
    }
    __syncwarp();
    for (int t = max(0, issued - kDecStages); t < issued; ++t)
      drain_bar(b_full(t % kDecStages), (t / kDecStages) & 1);
    return;
  }

  // ============================================================== consumers
  const int g = lane >> 2, tq = lane & 3;
  const int G = p.group;
  const int H = p.num_heads;
  // Q fragments (A operand, rows = query heads of this KV head, padded to 16)
  uint32_t qa[D / 16][4];
  {
    const uint16_t* qrow = static_cast<const uint16_t*>(p.q) + static_cast<long long>(sq.q_row) * p.q_row_stride;
    const bool valid = g < G;
    const uint16_t* qh = qrow + static_cast<long long>(kvh * G + g) * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t lo32 = 0, hi32 = 0;
      if (valid) {
        lo32 = *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 2 * tq);
        hi32 = *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 2 * tq + 8);
      }
      qa[kk][0] = lo32;
      qa[kk][1] = 0;  // rows 8..15: no query head
      qa[kk][2] = hi32;
      qa[kk][3] = 0;
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row g (head g of the group)
  const float sl2 = p.scale_log2;
  bool ok = !skip_all;
  const int kw0 = warp * 16;  // this warp's keys inside each 64-key tile
  for (int t = 0; t < n_tiles && ok; ++t) {
    const int s = t % kDecStages;
    ok = __all_sync(0xffffffffu, wait_bar(b_full(s), (t / kDecStages) & 1, abort_flag, kErrWaitSoftmax));
    if (!ok) break;
    const uint32_t sk = s0 + s * L::kStageBytes;
    const uint32_t sv = sk + L::kTileBytes;
    // ---- S[16 x 16] = Q K^T for keys kw0 .. kw0+15 (two n-tiles of 8 keys)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      // matrices: (keys kw0..+7, dims lo), (kw0..+7, hi), (kw0+8.., lo), (kw0+8.., hi)
      const int mi = lane >> 3;
      const int key = kw0 + ((mi >> 1) << 3) + (lane & 7);
      const int chunk = kk * 2 + (mi & 1);           // 16-byte chunk of the 128-dim row
      const uint32_t addr = sk + (chunk >> 3) * L::kHalfBytes + sw128(key, chunk & 7);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(addr, b0, b1, b2, b3);
      mma16816<F16>(sc[0], qa[kk], b0, b1);
      mma16816<F16>(sc[1], qa[kk], b2, b3);
    }
    // mask keys past the chunk end (rows g < G only matter)
    const int tile_k0 = t * kDecTileKeys + kw0;  // chunk-relative
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kidx = tile_k0 + n * 8 + 2 * tq + e;
        if (kidx >= n_keys) sc[n][e] = -INFINITY;
      }
    float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx * sl2);
    const float m_base = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = ex2_approx(m_run - m_base);
    float pr[2][2];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) pr[n][e] = ex2_approx(fmaf(sc[n][e], sl2, -m_base));
    float rs = pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l_run = l_run * alpha + rs;
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
    }
    // ---- O[16 x D] += P[16 x 16] V[16 x D], P as a 16-bit high part plus the
    // 16-bit rest P - hi: two products, so P reaches the accumulator with ~16
    // significant bits instead of 8 (the extra tensor work is small next to
    // the K/V bytes this kernel streams).
    uint32_t pa[4], pl[4];
    pa[0] = pack2<F16>(pr[0][0], pr[0][1]);
    pa[1] = 0;
    pa[2] = pack2<F16>(pr[1][0], pr[1][1]);
    pa[3] = 0;
    {
      const float2 h0 = unpack2<F16>(pa[0]), h1 = unpack2<F16>(pa[2]);
      pl[0] = pack2<F16>(pr[0][0] - h0.x, pr[0][1] - h0.y);
      pl[1] = 0;
      pl[2] = pack2<F16>(pr[1][0] - h1.x, pr[1][1] - h1.y);
      pl[3] = 0;
    }
#pragma unroll
    for (int jd = 0; jd < D / 16; ++jd) {
      // matrices: (keys kw0..+7, dims 16jd..+7), (kw0+8.., same), (kw0.., 16jd+8..), (kw0+8.., ...)
      const int mi = lane >> 3;
      const int key = kw0 + ((mi & 1) << 3) + (lane & 7);
      const int chunk = jd * 2 + (mi >> 1);
      const uint32_t addr = sv + (chunk >> 3) * L::kHalfBytes + sw128(key, chunk & 7);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(addr, v0, v1, v2, v3);
      mma16816<F16>(o[2 * jd], pa, v0, v1);
      mma16816<F16>(o[2 * jd + 1], pa, v2, v3);
      mma16816<F16>(o[2 * jd], pl, v0, v1);
      mma16816<F16>(o[2 * jd + 1], pl, v2, v3);
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(b_empty(s));
  }

  // ---- merge the 4 warps' partials: red[w][h][D], then m, l.  The buffer
  // aliases the stages: every consumer warp must be done with them first
  // (the producer has drained its copies before leaving).
  asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
  float* ro = red + warp * (kDecMaxGroup * D + 2 * kDecMaxGroup);
  float* rm = ro + kDecMaxGroup * D;
  float* rl = rm + kDecMaxGroup;
  if (ok && g < G) {
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      ro[g * D + j * 8 + 2 * tq] = o[j][0];
      ro[g * D + j * 8 + 2 * tq + 1] = o[j][1];
    }
    if (tq == 0) {
      rm[g] = m_run;
      rl[g] = l_run;
    }
  }
  // consumer warps only: named barrier 1 over 128 threads (the producer has left)
  asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
  if (!ok || skip_all) return;
  const int tid = threadIdx.x;
  for (int e = tid; e < G * D; e += kDecConsumerWarps * 32) {
    const int h = e / D, d = e - h * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecConsumerWarps; ++w)
      M = fmaxf(M, red[w * (kDecMaxGroup * D + 2 * kDecMaxGroup) + kDecMaxGroup * D + h]);
    float acc = 0.f, Ls = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kDecConsumerWarps; ++w) {
        const float* rw = red + w * (kDecMaxGroup * D + 2 * kDecMaxGroup);
        const float f = ex2_approx(rw[kDecMaxGroup * D + h] - M);
        acc += rw[h * D + d] * f;
        Ls += rw[kDecMaxGroup * D + kDecMaxGroup + h] * f;
      }
    }
    const int head = kvh * G + h;
    p.part_o[(static_cast<long long>(unit) * H + head) * D + d] = Ls > 0.f ? acc / Ls : 0.f;
    if (d == 0)
      p.part_lse[static_cast<long long>(unit) * H + head] =
          Ls > 0.f ? (M + lg2_approx(Ls)) * 0.69314718055994530942f : -INFINITY;
  }
}

// Merge the chunk partials of one (sequence, head): grid (num_seqs, H), D threads.
struct CombineParams {
  const float* part_o;
  const float* part_lse;
  void* out;
  long long out_row_stride;
  float* lse;
  long long lse_stride;
  int out_dt;
  int num_heads;
  int head_dim;
  int num_seqs;
  int unit_off[kDecMaxSeqs + 1];
  int q_row[kDecMaxSeqs];
};

__global__ void __launch_bounds__(128) decode_combine_kernel(const __grid_constant__ CombineParams p) {
  // after a recorded failure the partials were not written: leave out alone
  if (*reinterpret_cast<volatile int*>(&g_device_status) != 0) return;
  const int b = blockIdx.x, h = blockIdx.y;
  const int u0 = p.unit_off[b], u1 = p.unit_off[b + 1];
  const int H = p.num_heads, D = p.head_dim;
  float M = -INFINITY;
  for (int u = u0; u < u1; ++u) M = fmaxf(M, p.part_lse[static_cast<long long>(u) * H + h]);
  float W = 0.f;
  if (M != -INFINITY)
    for (int u = u0; u < u1; ++u) W += __expf(p.part_lse[static_cast<long long>(u) * H + h] - M);
  const long long row = p.q_row[b];
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    if (W > 0.f)
      for (int u = u0; u < u1; ++u) {
        const float w = __expf(p.part_lse[static_cast<long long>(u) * H + h] - M);
        acc += w * p.part_o[(static_cast<long long>(u) * H + h) * D + d];
      }
    const float v = W > 0.f ? acc / W : 0.f;
    const long long idx = row * p.out_row_stride + static_cast<long long>(h) * D + d;
    if (p.out_dt == HCP_F32) static_cast<float*>(p.out)[idx] = v;
    else if (p.out_dt == HCP_F16) static_cast<__half*>(p.out)[idx] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(v);
  }
  if (threadIdx.x == 0 && p.lse != nullptr)
    p.lse[static_cast<long long>(h) * p.lse_stride + row] = W > 0.f ? M + __logf(W) : -INFINITY;
}

}  // namespace hcp
