// a6: the online window lookup of the hybrid decode search (search.py:778-806,
// `_search_decode_online_into`): the batch's hidden states against the recent tokens kept
// in the layer's window (manager.py:89-155), first-index argmax of the scores rounded to
// the window dtype (the reference's matmul output dtype), valid iff > 0, then the first
// cached slot holding each target expert.
#pragma once

#include "alut_common.cuh"
#include "alut_search.cuh"

namespace alut {

constexpr int kOnlineThreads = 256;
constexpr int kOnlineMaxH = 8192;

struct OnlineArgs {
  int b, h, n, t, s;
  const void* x;
  int64_t x_stride;
  const void* keys;
  int64_t key_stride;
  const int64_t* eids;  // [n][t]
  const int64_t* target;
  int64_t target_stride;
  uint8_t* on_hit;
  int64_t* on_idx;
  int64_t* on_slot;
  int64_t out_stride;
};

// One CTA per token: the token's row in shared memory (fp32), each warp scores window rows
// warp, warp + 8, ... (lanes over H, 8 elements per 16-byte load), score rounded to TK.
template <typename TK>
__global__ void __launch_bounds__(kOnlineThreads) k_online_search(OnlineArgs a) {
  extern __shared__ __align__(16) float xs[];  // [h]
  __shared__ float s_best[kOnlineThreads / 32];
  __shared__ int s_arg[kOnlineThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bt = blockIdx.x;
  const TK* xr = static_cast<const TK*>(a.x) + static_cast<int64_t>(bt) * a.x_stride;
  for (int i = tid; i < a.h; i += kOnlineThreads) xs[i] = to_f32<TK>(xr[i]);
  __syncthreads();
  constexpr int kEpu = 16 / sizeof(TK);  // elements per 16-byte unit
  float best = -INFINITY;
  int arg = -1;
  for (int j = warp; j < a.n; j += kOnlineThreads / 32) {
    const TK* kr = static_cast<const TK*>(a.keys) + static_cast<int64_t>(j) * a.key_stride;
    float acc = 0.f;
    for (int c = lane * kEpu; c < a.h; c += 32 * kEpu) {
      float kv[8];
      unit_to_f32<TK>(kr + c, kv);
#pragma unroll
      for (int e = 0; e < kEpu; ++e) acc = fmaf(kv[e], xs[c + e], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    const float v = round_as<TK>(acc);
    if (v > best) {  // rows visited in increasing order: the first maximum stays
      best = v;
      arg = j;
    }
  }
  if (lane == 0) {
    s_best[warp] = best;
    s_arg[warp] = arg;
  }
  __syncthreads();
  if (tid < 32) {
    float b = tid < kOnlineThreads / 32 ? s_best[tid] : -INFINITY;
    int g = tid < kOnlineThreads / 32 ? s_arg[tid] : -1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, b, o);
      const int og = __shfl_xor_sync(0xffffffffu, g, o);
      if (og >= 0 && (g < 0 || ob > b || (ob == b && og < g))) {
        b = ob;
        g = og;
      }
    }
    if (tid == 0) {
      s_best[0] = b;
      s_arg[0] = g;
    }
  }
  __syncthreads();
  const bool valid = s_arg[0] >= 0 && s_best[0] > 0.f;
  const int top = s_arg[0];
  if (tid == 0) a.on_idx[bt] = valid ? top : -1;
  for (int s = tid; s < a.s; s += kOnlineThreads) {
    int slot = -1;
    if (valid) {
      const int64_t want = a.target[static_cast<int64_t>(bt) * a.target_stride + s];
      for (int k = 0; k < a.t && slot < 0; ++k)
        if (a.eids[static_cast<int64_t>(top) * a.t + k] == want) slot = k;
    }
    a.on_hit[static_cast<int64_t>(bt) * a.out_stride + s] = slot >= 0 ? 1 : 0;
    a.on_slot[static_cast<int64_t>(bt) * a.out_stride + s] = slot >= 0 ? slot : 0;
  }
}

}  // namespace alut
