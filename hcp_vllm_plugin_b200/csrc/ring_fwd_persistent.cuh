// Persistent form of the fused ring-attention forward (kernel variant 7).
//
// The per-CTA work is the one of ring_fwd_kernel (ring_fwd.cuh): one job is
// 256 query rows (query tiles A and B) of one head over the item's two KV
// segments, with the same warp roles, TMEM columns, shared-memory tiles and
// numerics as variant 5 (384 threads, registers split by setmaxnreg, packed
// f32x2 softmax math, the mbarrier MMA issuer).  What changes is the grid:
// one CTA per SM, and each CTA runs a fixed list of jobs one after the other,
// so the set-up (mbarrier init, TMEM allocation, tensor-map prefetch) is paid
// once per SM and, between two jobs,
//   - the producer loads the next job's Q tiles as soon as the last QK
//     product of the current job has read Q, and streams its K / V tiles
//     into the same 2-stage ring without a break;
//   - the MMA warp issues the next job's first QK products while the softmax
//     warpgroups still write the current job's output;
// instead of a CTA exit, a CTA launch, a Q load and a first QK product on
// the critical path of every 256-row block.
//
// Job order: jobs are the blocks of the non-persistent grid (heaviest first:
// block index = 256-row block x heads + head, the host orders the items by
// cost and ring_fwd_kernel's mapping takes each item's last block first).
// Round r hands jobs [r*G, (r+1)*G) to the G CTAs, in CTA order on even
// rounds and in reverse order on odd ones, so a CTA that got one of the
// heaviest jobs of a round gets one of the lightest of the next.  The list
// is static: every role of a CTA walks it on its own, with nothing shared.
//
// Every mbarrier keeps counting across jobs: the K / V ring by the CTA's
// running KV tile count, S / P / O events by the running tile count of each
// query tile, Q by the job count (plus a Q-free barrier the MMA warp commits
// after a job's last QK product).  Every wait is bounded as in
// ring_fwd_kernel, after which the CTA gives up on all its remaining jobs.
#pragma once

#include "ring_fwd.cuh"

namespace hcp {

template <int D>
struct FwdPersistSmem {
  static constexpr int kBoxBytes = 128 * 128;
  static constexpr int kTileBytes = (D / 64) * kBoxBytes;
  static constexpr int kNumBars = 9 + 4 * kStages;  // ring_fwd_kernel's + Q-free
  static constexpr int kKvOff = 2 * kTileBytes;
  static constexpr int kBarOff = kKvOff + 2 * kStages * kTileBytes;
  static constexpr int kEnd = kBarOff + 8 * kNumBars + 16;  // + TMEM slot, abort flag
  static constexpr int kBytes = kEnd + 1024;                // + alignment slack
};

// One job as every thread of the CTA derives it from the launch parameters.
struct FwdJob {
  int item;
  int head;
  int kvh;
  int q0;
  int rows_a;
  int rows_b;
  hcp_kv_segment sg0;
  hcp_kv_segment sg1;
  int ka0, kb0, ka1, kb1;  // keys query tile A / B needs from segment 0 / 1
  int tiles0;              // KV tiles of segment 0
  int n_tiles;             // KV tiles of both segments
  bool pre_a, pre_b;       // hi + lo P for rows that see few keys
};

__device__ __forceinline__ FwdJob fwd_job(const FwdParams& p, int job) {
  FwdJob j;
  const int H = p.num_heads;
  const int tile_global = job / H;
  j.head = job - tile_global * H;
  j.kvh = j.head / p.group;
  int lo = 0, hi = p.num_work - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_off[mid] <= tile_global) lo = mid; else hi = mid - 1;
  }
  j.item = lo;
  const FwdItem& wk = p.work[lo];
  const hcp_kv_segment* segs = p.segs + wk.seg_first;
  const int n_blocks = (wk.q_len + kCtaRows - 1) / kCtaRows;
  const int m_blk = n_blocks - 1 - (tile_global - p.tile_off[lo]);  // heaviest (last) first
  j.q0 = m_blk * kCtaRows;
  j.rows_a = max(0, min(kBlockM, wk.q_len - j.q0));
  j.rows_b = max(0, min(kBlockM, wk.q_len - j.q0 - kBlockM));
  j.sg0 = cta_segment(segs[0], j.q0, p.window);
  j.sg1 = cta_segment(segs[1], j.q0, p.window);
  j.ka0 = segment_keys(j.sg0, j.q0, j.rows_a);
  j.kb0 = segment_keys(j.sg0, j.q0 + kBlockM, j.rows_b);
  j.ka1 = segment_keys(j.sg1, j.q0, j.rows_a);
  j.kb1 = segment_keys(j.sg1, j.q0 + kBlockM, j.rows_b);
  j.tiles0 = (max(j.ka0, j.kb0) + kBlockN - 1) / kBlockN;
  j.n_tiles = j.tiles0 + (max(j.ka1, j.kb1) + kBlockN - 1) / kBlockN;
  j.pre_a = segment_keys(j.sg0, j.q0, 1) + segment_keys(j.sg1, j.q0, 1) < kPreciseKeys;
  j.pre_b = segment_keys(j.sg0, j.q0 + kBlockM, 1) + segment_keys(j.sg1, j.q0 + kBlockM, 1) < kPreciseKeys;
  return j;
}

// Job of round r for this CTA, or -1 when the (last, partial) round has none.
__device__ __forceinline__ int fwd_job_index(int r, int total) {
  const long long base = static_cast<long long>(r) * gridDim.x;
  const long long idx = (r & 1) ? base + gridDim.x - 1 - blockIdx.x : base + blockIdx.x;
  return idx < total ? static_cast<int>(idx) : -1;
}

__device__ __forceinline__ int fwd_rounds(int total) {
  return static_cast<int>((static_cast<long long>(total) + gridDim.x - 1) / gridDim.x);
}

template <int D, bool F16>
__global__ void __launch_bounds__(kThreadsWide, 1)
    ring_fwd_persistent_kernel(const __grid_constant__ FwdParams p) {
  static_assert(D == 64 || D == 128, "head_dim must be 64 or 128");
  using L = FwdPersistSmem<D>;
  constexpr int kHalves = D / 64;
  constexpr int kBoxBytes = L::kBoxBytes;
  constexpr int kTileBytes = L::kTileBytes;
  constexpr uint32_t kIdescQK = ptx::idesc_f16(128, 128, false, false, F16);
  constexpr uint32_t kIdescPV = ptx::idesc_f16(128, D, false, true, F16);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t s_q = ptx::smem_u32(smem);  // Q_A at s_q, Q_B at s_q + kTileBytes
  const uint32_t s_kv0 = s_q + L::kKvOff;    // stage s: K at +2s tiles, V at +2s+1
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
  const uint32_t b_qfree = bar0 + 8u * (8 + 4 * kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = p.total_tiles * p.num_heads;
  const int rounds = fwd_rounds(total);

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
    ptx::mbar_init(b_qfree, 1);
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
    ptx::prefetch_tmap(&p.tm_kb);
    ptx::prefetch_tmap(&p.tm_vb);
    ptx::prefetch_tmap(&p.tm_cache);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool skip_all = *abort_flag != 0;

  // is KV tile t of job j needed by query tile x (0 = A, 1 = B)?
  auto active = [](const FwdJob& j, int x, int t) {
    const bool s0 = t < j.tiles0;
    const int need = s0 ? (x == 0 ? j.ka0 : j.kb0) : (x == 0 ? j.ka1 : j.kb1);
    return (s0 ? t : t - j.tiles0) * kBlockN < need;
  };

  if (warp >= 8) {
  // ============================================== producer warpgroup: TMA, MMA
  ptx::setmaxnreg_dec<kRegsProducerWide>();
  if (skip_all) {
    // nothing issued, nothing to drain
  } else if (warp == kWarpTma) {
    // ================================================================ producer
    const int bs = p.block_size;
    const int nblk = kBlockN / bs;
    int kv_base = 0;              // KV tiles of earlier jobs
    int k_issued = 0, v_issued = 0;
    int q_loads = 0;
    bool ok = true;
    for (int r = 0; r < rounds && ok; ++r) {
      const int job = fwd_job_index(r, total);
      if (job < 0) continue;
      const FwdJob j = fwd_job(p, job);
      const FwdItem& wk = p.work[j.item];
      // Q of the previous job is free once its last QK product completed
      if (q_loads > 0) {
        ok = __all_sync(0xffffffffu, wait_bar(b_qfree, (q_loads - 1) & 1, abort_flag, kErrWaitProducer));
        if (!ok) break;
      }
      if (lane == 0) {
        ptx::mbar_arrive_expect_tx(b_q, 2 * kTileBytes);
        for (int x = 0; x < 2; ++x)
          for (int hf = 0; hf < kHalves; ++hf)
            ptx::tma_load_3d(s_q + x * kTileBytes + hf * kBoxBytes, &p.tm_q, b_q, hf * 64, j.head,
                             wk.q_start + j.q0 + x * kBlockM);
      }
      ++q_loads;
      auto lookup = [&](int t) {
        int blk = static_cast<int>(p.num_blocks);
        if (t < j.n_tiles && lane < nblk) {
          const hcp_kv_segment sg = t < j.tiles0 ? j.sg0 : j.sg1;
          if (sg.src == HCP_SRC_PAGED) {
            const int rel = (t < j.tiles0 ? t : t - j.tiles0) * kBlockN + lane * bs;
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
      for (int t = 0; t < j.n_tiles; ++t) {
        const int g = kv_base + t;
        const int s = g % kStages;
        const uint32_t ph = (g / kStages) & 1;
        const bool in0 = t < j.tiles0;
        const int key0 = (in0 ? t : t - j.tiles0) * kBlockN;
        const hcp_kv_segment seg = in0 ? j.sg0 : j.sg1;
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
        ok = __all_sync(0xffffffffu, wait_bar(b_kempty(s), ph ^ 1, abort_flag, kErrWaitProducer));
        if (!ok) break;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(b_kfull(s), kTileBytes);
          if (paged) {
            for (int i = 0; i < nblk; ++i)
              for (int hf = 0; hf < kHalves; ++hf)
                ptx::tma_load_4d(s_k + hf * kBoxBytes + i * bs * 128, &p.tm_cache, b_kfull(s), hf * 64,
                                 0, j.kvh, blk_ids[i]);
          } else {
            const CUtensorMap* tk = seg.src == HCP_SRC_A   ? &p.tm_ka
                                    : seg.src == HCP_SRC_B ? &p.tm_kb
                                                           : &p.tm_ek[seg.src - HCP_SRC_EXT0];
            for (int hf = 0; hf < kHalves; ++hf)
              ptx::tma_load_3d(s_k + hf * kBoxBytes, tk, b_kfull(s), hf * 64, j.kvh, seg.start + key0);
          }
        }
        k_issued = g + 1;
        ok = __all_sync(0xffffffffu, wait_bar(b_vempty(s), ph ^ 1, abort_flag, kErrWaitProducer));
        if (!ok) break;
        if (lane == 0) {
          ptx::mbar_arrive_expect_tx(b_vfull(s), kTileBytes);
          if (paged) {
            for (int i = 0; i < nblk; ++i)
              for (int hf = 0; hf < kHalves; ++hf)
                ptx::tma_load_4d(s_v + hf * kBoxBytes + i * bs * 128, &p.tm_cache, b_vfull(s),
                                 D + hf * 64, 0, j.kvh, blk_ids[i]);
          } else {
            const CUtensorMap* tv = seg.src == HCP_SRC_A   ? &p.tm_va
                                    : seg.src == HCP_SRC_B ? &p.tm_vb
                                                           : &p.tm_ev[seg.src - HCP_SRC_EXT0];
            for (int hf = 0; hf < kHalves; ++hf)
              ptx::tma_load_3d(s_v + hf * kBoxBytes, tv, b_vfull(s), hf * 64, j.kvh, seg.start + key0);
          }
        }
        v_issued = g + 1;
      }
      kv_base += j.n_tiles;
    }
    __syncwarp();
    // Teardown: every TMA copy this warp issued must land before the CTA
    // exits.  Only the last Q load and the last use of each stage can still
    // be in flight (each earlier one was waited for before its buffer was
    // refilled).
    if (q_loads > 0) drain_bar(b_q, (q_loads - 1) & 1);
    for (int g = max(0, k_issued - kStages); g < k_issued; ++g) {
      const int s = g % kStages;
      const uint32_t ph = (g / kStages) & 1;
      drain_bar(b_kfull(s), ph);
      if (g < v_issued) drain_bar(b_vfull(s), ph);
    }
  } else if (warp == kWarpMma) {
    // ================================================================ MMA issuer
    int kv_base = 0;
    int jobs = 0;
    int pv_count[2] = {0, 0};  // PV products issued per query tile, over all jobs
    bool ok = true;
    for (int r = 0; r < rounds && ok; ++r) {
      const int job = fwd_job_index(r, total);
      if (job < 0) continue;
      const FwdJob j = fwd_job(p, job);
      ok = __all_sync(0xffffffffu, wait_bar(b_q, jobs & 1, abort_flag, kErrWaitMma));
      if (!ok) break;
      const int n_tiles = j.n_tiles;
      if (n_tiles == 0) {
        if (lane == 0) ptx::umma_commit(b_qfree);
        __syncwarp();
      }
      uint32_t pv_started = 0;  // bit x: this job has a PV product of query tile x (the first overwrites O)
      for (int t = 0; t <= n_tiles && ok; ++t) {
        const bool have_prev = t >= 1;
        const bool have_cur = t < n_tiles;
        const int gp = kv_base + t - 1;
        const int gc = kv_base + t;
        const int sp = (gp + kStages) % kStages;
        const int sc = gc % kStages;
        bool v_ready = false, k_ready = false;
        for (int x = 0; x < 2 && ok; ++x) {
          if (have_prev && active(j, x, t - 1)) {
            ok = __all_sync(0xffffffffu, wait_bar(b_pfull(x), pv_count[x] & 1, abort_flag, kErrWaitMma));
            if (ok && !v_ready) {
              ok = __all_sync(0xffffffffu, wait_bar(b_vfull(sp), (gp / kStages) & 1, abort_flag, kErrWaitMma));
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
                ptx::umma_ts(o_acc, p_col + kk * 8, bdesc, kIdescPV, kk > 0 ? 1u : (pv_started >> x) & 1u);
              }
              if (x == 0 ? j.pre_a : j.pre_b) {
                // rows that see few keys only: kept rolled, so the common
                // path's registers are not spent on its descriptors
#pragma unroll 1
                for (int kk = 0; kk < kBlockN / 16; ++kk) {
                  const uint64_t bdesc = ptx::sdesc_sw128(s_v + kk * 2048, kBoxBytes, 1024);
                  ptx::umma_ts(o_acc, p_col + 64 + kk * 8, bdesc, kIdescPV, 1u);
                }
              }
              ptx::umma_commit(b_odone(x));
            }
            __syncwarp();
            ++pv_count[x];
            pv_started |= 1u << x;
          }
          if (have_cur && active(j, x, t)) {
            if (!k_ready) {
              ok = __all_sync(0xffffffffu, wait_bar(b_kfull(sc), (gc / kStages) & 1, abort_flag, kErrWaitMma));
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
        // release the stages (tcgen05.commit tracks every MMA issued so far),
        // and after the job's last QK products its Q tiles
        if (lane == 0) {
          if (have_prev) ptx::umma_commit(b_vempty(sp));
          if (have_cur) ptx::umma_commit(b_kempty(sc));
          if (t == n_tiles - 1) ptx::umma_commit(b_qfree);
        }
        __syncwarp();
      }
      kv_base += n_tiles;
      ++jobs;
    }
    // Teardown: no MMA may be in flight when TMEM is released.
    if (lane == 0) ptx::umma_commit(b_final);
    __syncwarp();
    drain_bar(b_final, 0);
  }
  } else {
  ptx::setmaxnreg_inc<kRegsSoftmaxWide>();
  if (!skip_all) {
    // ================================================================ softmax + epilogue
    const int x = warp >> 2;                 // query tile of this warpgroup (0 = A, 1 = B)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;     // == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const float scale_log2 = p.scale_log2;
    const uint32_t s_addr = tmem + lane_base + x * 128;
    const uint32_t o_addr = tmem + lane_base + 256 + x * D;
    int done_all = 0;  // KV tiles processed by this warpgroup, over all jobs
    bool ok = true;
    for (int r = 0; r < rounds && ok; ++r) {
      const int job = fwd_job_index(r, total);
      if (job < 0) continue;
      const FwdJob j = fwd_job(p, job);
      const FwdItem& wk = p.work[j.item];
      const int qrow = j.q0 + x * kBlockM + row;  // work-item-relative query row
      const bool precise = x == 0 ? j.pre_a : j.pre_b;
      float m_used = -INFINITY;  // running max of the row, base-2 scaled domain
      float l = 0.f;             // row sum
      int done = 0;              // KV tiles of this job processed by this warpgroup
      for (int t = 0; t < j.n_tiles; ++t) {
        if (!active(j, x, t)) continue;
        ok = __all_sync(0xffffffffu, wait_bar(b_sfull(x), done_all & 1, abort_flag, kErrWaitSoftmax));
        if (!ok) break;
        ptx::tc_fence_after();
        const bool in0 = t < j.tiles0;
        const int key0 = (in0 ? t : t - j.tiles0) * kBlockN;
        const hcp_kv_segment seg = in0 ? j.sg0 : j.sg1;
        int vis = seg.len - key0;
        if (seg.causal_off != kNonCausal) vis = min(vis, seg.causal_off + qrow - key0 + 1);
        vis = max(0, min(vis, kBlockN));
        // keys [0, lo) of the tile are below the row's sliding window
        const int lo =
            (p.window > 0 && seg.causal_off != kNonCausal) ? seg.causal_off + qrow - p.window + 1 - key0 : 0;

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
        for (int jj = 0; jj < 8; ++jj)
          mx8[jj] = max3(__uint_as_float(sr[jj]), __uint_as_float(sr[jj + 8]), __uint_as_float(sr[jj + 16]));
#pragma unroll
        for (int i = 24; i < 120; i += 16)
#pragma unroll
          for (int jj = 0; jj < 8; ++jj)
            mx8[jj] = max3(mx8[jj], __uint_as_float(sr[i + jj]), __uint_as_float(sr[i + 8 + jj]));
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) mx8[jj] = fmaxf(mx8[jj], __uint_as_float(sr[120 + jj]));
        const float mx = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        const float mx2 = mx * scale_log2;  // -inf stays -inf
        const bool raise = mx2 > m_used + kRescaleThreshold;
        const float m_new = raise ? mx2 : m_used;
        const float alpha = raise ? ex2_approx(m_used - m_new) : 1.f;  // 0 when m_used = -inf
        const float m_base = (m_new == -INFINITY) ? 0.f : m_new;
        float sums[4] = {0.f, 0.f, 0.f, 0.f};
        if (!precise) {
          // packed f32x2: x = s * scale - m two keys at a time, sums likewise
          const float2 sc2 = make_float2(scale_log2, scale_log2);
          const float2 mb2 = make_float2(-m_base, -m_base);
          float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 sv =
                  make_float2(__uint_as_float(sr[c * 32 + 2 * i]), __uint_as_float(sr[c * 32 + 2 * i + 1]));
              const float2 xx = __ffma2_rn(sv, sc2, mb2);
              const float2 pp = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
              acc2[i & 1] = __fadd2_rn(acc2[i & 1], pp);
              pk[i] = pack2<F16>(pp.x, pp.y);
            }
            ptx::tmem_st_32x32b_x16(s_addr + c * 16, pk);
          }
          sums[0] = acc2[0].x;
          sums[1] = acc2[0].y;
          sums[2] = acc2[1].x;
          sums[3] = acc2[1].y;
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16], pl[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i]), scale_log2, -m_base));
              const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c * 32 + 2 * i + 1]), scale_log2, -m_base));
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
          ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done_all - 1) & 1, abort_flag, kErrWaitSoftmax));
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
        ++done_all;
      }
      if (!ok) break;
      if (done > 0) {
        ok = __all_sync(0xffffffffu, wait_bar(b_odone(x), (done_all - 1) & 1, abort_flag, kErrWaitSoftmax));
        if (!ok) break;
        ptx::tc_fence_after();
      }
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
        float lp = p.merge_lse[j.head * p.merge_lse_stride + lse_idx_col];
        if (lp == INFINITY) lp = -INFINITY;
        const float mm = fmaxf(lp, lse_v);
        if (mm == -INFINITY) {
          f_new = 0.f;
          lse_v = -INFINITY;
        } else {
          const float wp = __expf(lp - mm);
          const float wn = __expf(lse_v - mm);
          const float rr = 1.f / (wp + wn);
          f_old = wp * rr;
          f_new *= wn * rr;
          lse_v = mm + __logf(wp + wn);
        }
      }
      const long long col0 = static_cast<long long>(j.head) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t rg[32];
        if (done > 0) {
          ptx::tmem_ld_32x32b_x32(o_addr + c * 32, rg);
          ptx::tmem_wait_ld();
        }
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = done > 0 ? __uint_as_float(rg[i]) * f_new : 0.f;
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
      if (valid && p.lse != nullptr) p.lse[j.head * p.lse_stride + lse_idx_col] = lse_v;
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
constexpr int fwd_persistent_smem_bytes() {
  return FwdPersistSmem<D>::kBytes;
}

}  // namespace hcp
