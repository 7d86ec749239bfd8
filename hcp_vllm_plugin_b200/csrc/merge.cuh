// Standalone LSE merge of two partial attention results (the vLLM
// merge_attn_states contract): an HBM-bound elementwise kernel, one warp per
// (token, head) row, 16-byte vector loads where the dtype allows.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "hcp_ring.h"

namespace hcp {

struct MergeParams {
  void* out;
  const void* pre;
  const void* suf;
  float* out_lse;
  const float* pre_lse;
  const float* suf_lse;
  long long out_stride, pre_stride, suf_stride;      // row strides (elements)
  long long out_lse_stride, pre_lse_stride, suf_lse_stride;
  long long num_tokens;
  int num_heads;
  int head_dim;
  int out_dt, pre_dt, suf_dt;
};

__device__ __forceinline__ float load_elem(const void* base, int dt, long long i) {
  if (dt == HCP_F32) return static_cast<const float*>(base)[i];
  if (dt == HCP_F16) return __half2float(static_cast<const __half*>(base)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
}
__device__ __forceinline__ void store_elem(void* base, int dt, long long i, float v) {
  if (dt == HCP_F32) static_cast<float*>(base)[i] = v;
  else if (dt == HCP_F16) static_cast<__half*>(base)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
}

__global__ void __launch_bounds__(256) merge_states_kernel(const MergeParams p) {
  // after a recorded failure the partials may be unwritten: leave out alone
  if (*reinterpret_cast<volatile int*>(&g_device_status) != 0) return;
  const long long warp_global = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = p.num_tokens * p.num_heads;
  if (warp_global >= rows) return;
  const long long tok = warp_global / p.num_heads;
  const int h = static_cast<int>(warp_global - tok * p.num_heads);
  float lp = p.pre_lse[h * p.pre_lse_stride + tok];
  float ls = p.suf_lse[h * p.suf_lse_stride + tok];
  if (lp == INFINITY) lp = -INFINITY;  // +inf marks an empty partial
  if (ls == INFINITY) ls = -INFINITY;
  const float m = fmaxf(lp, ls);
  float wp = 0.f, ws = 0.f, lse = -INFINITY;
  if (m != -INFINITY) {
    const float ep = expf(lp - m);
    const float es = expf(ls - m);
    const float tot = ep + es;
    wp = ep / tot;
    ws = es / tot;
    lse = m + logf(tot);
  }
  const long long po = tok * p.pre_stride + static_cast<long long>(h) * p.head_dim;
  const long long so = tok * p.suf_stride + static_cast<long long>(h) * p.head_dim;
  const long long oo = tok * p.out_stride + static_cast<long long>(h) * p.head_dim;
  for (int d = lane; d < p.head_dim; d += 32) {
    const float v = load_elem(p.pre, p.pre_dt, po + d) * wp + load_elem(p.suf, p.suf_dt, so + d) * ws;
    store_elem(p.out, p.out_dt, oo + d, v);
  }
  if (lane == 0 && p.out_lse != nullptr) p.out_lse[h * p.out_lse_stride + tok] = lse;
}

// N-way merge of partial results stacked as o [N, T, H, D] fp32 and lse
// [N, H, T] fp32 (one partial per KV shard): out = sum_i w_i o_i with
// w_i = exp(lse_i - m) / sum_j exp(lse_j - m), m = max_i lse_i, and
// lse = m + log(sum_j exp(lse_j - m)).  Empty partials (lse -inf, or +inf as
// vLLM marks them) get weight 0; a row with no keys at all is 0 with lse -inf.
struct MergeNParams {
  void* out;
  float* out_lse;
  const float* states_o;
  const float* states_lse;
  long long out_stride;      // row stride (elements)
  long long out_lse_stride;
  long long num_tokens;
  int num_heads;
  int head_dim;
  int num_states;
  int out_dt;
  int vec_ok;                // 16-byte aligned partials (and fp32 output rows): float4 path allowed
};

__global__ void __launch_bounds__(256) merge_states_n_kernel(const MergeNParams p) {
  if (*reinterpret_cast<volatile int*>(&g_device_status) != 0) return;
  const long long warp_global = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long rows = p.num_tokens * p.num_heads;
  if (warp_global >= rows) return;
  const long long tok = warp_global / p.num_heads;
  const int h = static_cast<int>(warp_global - tok * p.num_heads);
  const long long lse_state = static_cast<long long>(p.num_heads) * p.num_tokens;
  const long long o_state = p.num_tokens * p.num_heads * p.head_dim;
  const long long row = (tok * p.num_heads + h) * p.head_dim;
  const long long oo = tok * p.out_stride + static_cast<long long>(h) * p.head_dim;
  if (p.vec_ok && p.num_states <= 32 && p.head_dim == 128) {
    // lane i holds state i's LSE; weights by warp shuffles; each lane owns 4
    // consecutive dims (float4 loads of every partial row)
    float l = -INFINITY;
    if (lane < p.num_states) {
      l = p.states_lse[lane * lse_state + h * p.num_tokens + tok];
      if (l == INFINITY) l = -INFINITY;
    }
    float m = l;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
    const float w = (m == -INFINITY || lane >= p.num_states) ? 0.f : expf(l - m);
    float tot = w;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, s);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = 0; i < p.num_states; ++i) {
      const float wi = __shfl_sync(0xffffffffu, w, i);
      if (wi == 0.f) continue;
      const float4 o = reinterpret_cast<const float4*>(p.states_o + i * o_state + row)[lane];
      acc.x += wi * o.x;
      acc.y += wi * o.y;
      acc.z += wi * o.z;
      acc.w += wi * o.w;
    }
    const float inv = tot > 0.f ? 1.f / tot : 0.f;
    const long long d0 = oo + 4 * lane;
    if (p.out_dt == HCP_F32) {
      reinterpret_cast<float4*>(static_cast<float*>(p.out) + d0)[0] =
          make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    } else {
      store_elem(p.out, p.out_dt, d0 + 0, acc.x * inv);
      store_elem(p.out, p.out_dt, d0 + 1, acc.y * inv);
      store_elem(p.out, p.out_dt, d0 + 2, acc.z * inv);
      store_elem(p.out, p.out_dt, d0 + 3, acc.w * inv);
    }
    if (lane == 0 && p.out_lse != nullptr)
      p.out_lse[h * p.out_lse_stride + tok] = tot > 0.f ? m + logf(tot) : -INFINITY;
    return;
  }
  // generic path: any state count, head_dim <= 256
  float m = -INFINITY;
  for (int i = 0; i < p.num_states; ++i) {
    float l = p.states_lse[i * lse_state + h * p.num_tokens + tok];
    if (l == INFINITY) l = -INFINITY;
    m = fmaxf(m, l);
  }
  float tot = 0.f;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  if (m != -INFINITY) {
    for (int i = 0; i < p.num_states; ++i) {
      float l = p.states_lse[i * lse_state + h * p.num_tokens + tok];
      if (l == INFINITY) l = -INFINITY;
      const float w = expf(l - m);
      tot += w;
      if (w == 0.f) continue;
      const float* o = p.states_o + i * o_state + row;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = lane + 32 * j;
        if (d < p.head_dim) acc[j] += w * o[d];
      }
    }
  }
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int d = lane + 32 * j;
    if (d < p.head_dim) store_elem(p.out, p.out_dt, oo + d, acc[j] * inv);
  }
  if (lane == 0 && p.out_lse != nullptr)
    p.out_lse[h * p.out_lse_stride + tok] = tot > 0.f ? m + logf(tot) : -INFINITY;
}

}  // namespace hcp
