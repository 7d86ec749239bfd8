// Paged KV-cache scatter and gather.
//
// kv_cache_update_kernel: new K/V rows into [num_blocks, Hkv, block_size, 2D]
// at their slots (block = slot / block_size, offset = slot % block_size).
// One warp per (token, KV head) moves the head's K and V rows with 16-byte
// stores; negative or out-of-range slots (padding) are skipped.
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
  int num_kv_heads;
  int head_dim;
};

__global__ void __launch_bounds__(256) kv_cache_update_kernel(const CacheUpdateParams p) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= p.num_tokens * p.num_kv_heads) return;
  const long long tok = w / p.num_kv_heads;
  const int h = static_cast<int>(w - tok * p.num_kv_heads);
  const long long slot = p.slot_mapping[tok];
  if (slot < 0 || slot >= p.num_blocks * p.block_size) return;
  const long long blk = slot / p.block_size;
  const int off = static_cast<int>(slot - blk * p.block_size);
  const int D = p.head_dim;
  uint16_t* dst = p.cache + (((blk * p.num_kv_heads + h) * p.block_size + off) * 2LL * D);
  const uint16_t* ks = p.key + tok * p.key_row_stride + static_cast<long long>(h) * D;
  const uint16_t* vs = p.value + tok * p.value_row_stride + static_cast<long long>(h) * D;
  const int vec = D / 8;  // 16-byte vectors per row
  for (int i = lane; i < 2 * vec; i += 32) {
    const uint4 v = i < vec ? reinterpret_cast<const uint4*>(ks)[i] : reinterpret_cast<const uint4*>(vs)[i - vec];
    reinterpret_cast<uint4*>(dst)[i] = v;
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
  int num_kv_heads;
  int head_dim;
};

__global__ void __launch_bounds__(256) kv_cache_gather_kernel(const CacheGatherParams p) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= p.num_tokens * p.num_kv_heads) return;
  const long long tok = w / p.num_kv_heads;
  const int h = static_cast<int>(w - tok * p.num_kv_heads);
  const long long slot = p.slot_mapping[tok];
  const bool valid = slot >= 0 && slot < p.num_blocks * p.block_size;
  const long long blk = valid ? slot / p.block_size : 0;
  const int off = valid ? static_cast<int>(slot - blk * p.block_size) : 0;
  const int D = p.head_dim;
  const uint16_t* src = p.cache + (((blk * p.num_kv_heads + h) * p.block_size + off) * 2LL * D);
  uint16_t* kd = p.key + tok * p.key_row_stride + static_cast<long long>(h) * D;
  uint16_t* vd = p.value + tok * p.value_row_stride + static_cast<long long>(h) * D;
  const int vec = D / 8;  // 16-byte vectors per row
  for (int i = lane; i < 2 * vec; i += 32) {
    const uint4 v = valid ? reinterpret_cast<const uint4*>(src)[i] : make_uint4(0u, 0u, 0u, 0u);
    if (i < vec) reinterpret_cast<uint4*>(kd)[i] = v;
    else reinterpret_cast<uint4*>(vd)[i - vec] = v;
  }
}

}  // namespace hcp
