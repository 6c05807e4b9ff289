// Value-row gather across the centroid-range shards of one large table, reading each
// winning row directly from the HBM of the rank that owns it (CUDA IPC peer mapping over
// NVLink: plain 16-byte loads, no multicast). Replaces the materialise-zeros + reduce-scatter
// exchange: every remote row crosses NVLink once, straight into the destination row.
#pragma once

#include "alut_common.cuh"

namespace alut {

constexpr int kPeerMaxWorld = 64;
constexpr int kPeerThreads = 256;  // one warp per row

// out[i] = value row idx[i] of modality (is_vision[i] ? 0 : 1) from the shard owning idx[i]
// (shard r holds centroids [shard_start[r], shard_start[r+1]) at shard_values[r], rows
// stride_k bytes apart, modality planes shard_stride_m[r] elements of esz bytes apart);
// zeros for misses.
__global__ void __launch_bounds__(kPeerThreads) k_gather_sharded(
    int n, const uint8_t* hit, const int64_t* idx, const uint8_t* is_vision, int world,
    const unsigned char* const* shard_values, const int64_t* shard_start, const int64_t* shard_stride_m,
    int esz, int64_t stride_k, int row_bytes, unsigned char* out, int64_t out_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kPeerThreads / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  uint4* dst = reinterpret_cast<uint4*>(out + row * out_stride);
  const int units = row_bytes / 16;
  const int64_t k = idx[row];
  int owner = -1;
  if (hit[row])
    for (int r = 0; r < world; ++r)
      if (k >= shard_start[r] && k < shard_start[r + 1]) owner = r;
  if (owner < 0) {
    for (int u = lane; u < units; u += 32) dst[u] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(shard_values[owner] + (is_vision[row] ? 0 : shard_stride_m[owner] * esz) +
                                                    (k - shard_start[owner]) * stride_k);
  // Four 16-byte loads in flight per lane before the stores (remote latency).
  int u = lane;
  for (; u + 96 < units; u += 128) {
    const uint4 a = src[u], b = src[u + 32], c = src[u + 64], d = src[u + 96];
    dst[u] = a;
    dst[u + 32] = b;
    dst[u + 64] = c;
    dst[u + 96] = d;
  }
  for (; u < units; u += 32) dst[u] = src[u];
}

}  // namespace alut
