// Paged KV-cache scatter and gather.
//
// kv_cache_update_kernel: new K/V rows into [num_blocks, Hkv, block_size, 2D]
// at their slots (block = slot / block_size, offset = slot % block_size).
// 16-byte moves, two tokens per warp in flight; negative or out-of-range
// slots (padding) are skipped.
//
// kv_cache_gather_kernel: the inverse, K/V rows of the given slots out of the
// cache into contiguous [n, Hkv, D] K and V (a chunk extracted from the pool);
// rows of negative or out-of-range slots are written as zeros.
#pragma once

#include <cstdint>

namespace hcp {

struct CacheUpdateParams {
  const uint16_t* key;
  const uint16_t* value;
  long long key_row_stride;    // elements
  long long value_row_stride;
  const int64_t* slot_mapping;
  uint16_t* cache;
  long long num_blocks;
  long long num_tokens;
  int block_size;
  int bs_shift;                // log2(block_size) when it is a power of two, else -1
  int num_kv_heads;
  int head_dim;
};

// Grid (ceil(tokens / 16), Hkv); a block of 8 warps moves 16 tokens of one KV
// head, two per warp with both loads in flight.  Lane i moves the i-th 16-byte
// vector of the head's [K | V] row (D = 128: exactly one vector per lane).
constexpr int kCacheTokPerBlock = 16;

__device__ __forceinline__ bool slot_block(long long slot, long long num_blocks, int bs, int shift,
                                           long long& blk, int& off) {
  if (slot < 0 || slot >= num_blocks * bs) return false;
  if (shift >= 0) {
    blk = slot >> shift;
    off = static_cast<int>(slot & (bs - 1));
  } else {
    blk = slot / bs;
    off = static_cast<int>(slot - blk * bs);
  }
  return true;
}

__global__ void __launch_bounds__(256) kv_cache_update_kernel(const CacheUpdateParams p) {
  const int h = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int D = p.head_dim;
  const int vec = D / 8;
  const long long tok0 = static_cast<long long>(blockIdx.x) * kCacheTokPerBlock + warp;
  for (int i0 = 0; i0 < 2 * vec; i0 += 32) {
    const int i = i0 + lane;
    uint4 val[2];
    uint16_t* dst[2] = {nullptr, nullptr};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const long long tok = tok0 + 8 * j;
      long long blk;
      int off;
      if (tok < p.num_tokens && i < 2 * vec &&
          slot_block(p.slot_mapping[tok], p.num_blocks, p.block_size, p.bs_shift, blk, off)) {
        dst[j] = p.cache + ((blk * p.num_kv_heads + h) * p.block_size + off) * 2LL * D;
        val[j] = i < vec
                     ? reinterpret_cast<const uint4*>(p.key + tok * p.key_row_stride + static_cast<long long>(h) * D)[i]
                     : reinterpret_cast<const uint4*>(p.value + tok * p.value_row_stride +
                                                      static_cast<long long>(h) * D)[i - vec];
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (dst[j] != nullptr) reinterpret_cast<uint4*>(dst[j])[i] = val[j];
  }
}

struct CacheGatherParams {
  const uint16_t* cache;
  const int64_t* slot_mapping;
  uint16_t* key;
  uint16_t* value;
  long long key_row_stride;    // elements
  long long value_row_stride;
  long long num_blocks;
  long long num_tokens;
  int block_size;
  int bs_shift;
  int num_kv_heads;
  int head_dim;
};

__global__ void __launch_bounds__(256) kv_cache_gather_kernel(const CacheGatherParams p) {
  const int h = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int D = p.head_dim;
  const int vec = D / 8;
  const long long tok0 = static_cast<long long>(blockIdx.x) * kCacheTokPerBlock + warp;
  for (int i0 = 0; i0 < 2 * vec; i0 += 32) {
    const int i = i0 + lane;
    uint4 val[2];
    bool live[2] = {false, false};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const long long tok = tok0 + 8 * j;
      if (tok >= p.num_tokens || i >= 2 * vec) continue;
      live[j] = true;
      long long blk;
      int off;
      if (slot_block(p.slot_mapping[tok], p.num_blocks, p.block_size, p.bs_shift, blk, off))
        val[j] = reinterpret_cast<const uint4*>(p.cache + ((blk * p.num_kv_heads + h) * p.block_size + off) * 2LL * D)[i];
      else
        val[j] = make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (!live[j]) continue;
      const long long tok = tok0 + 8 * j;
      if (i < vec)
        reinterpret_cast<uint4*>(p.key + tok * p.key_row_stride + static_cast<long long>(h) * D)[i] = val[j];
      else
        reinterpret_cast<uint4*>(p.value + tok * p.value_row_stride + static_cast<long long>(h) * D)[i - vec] = val[j];
    }
  }
}

}  // namespace hcp
