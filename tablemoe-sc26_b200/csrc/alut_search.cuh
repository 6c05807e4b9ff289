// Kernel 2: the centroid scan (search.py:566-602 semantics over all K centroids).
// A persistent grid walks tiles of (table group, 128-centroid chunk). Each CTA stages
// the queries of up to kSearchGroup pairs routed to one (expert, modality) table in
// shared memory, streams its chunk of the key table once (one centroid row per thread,
// 16-byte loads), and folds the per-pair best candidate into the packed global best
// with a 64-bit atomicMax, whose order independence keeps results deterministic.
#pragma once

#include "alut_common.cuh"

namespace alut {

struct SearchArgs {
  const void* keys;
  int64_t key_stride_e, key_stride_m, key_stride_k;
  int k, l, s, nchunks;
  uint32_t idx_offset;
  const float* qlow;
  const int* sorted;
  const int4* groups;
  const int* meta;
  uint64_t* best;
};

inline size_t search_smem_bytes(int l) { return sizeof(float) * kSearchGroup * l; }

template <typename TK, bool kVec>
__global__ void __launch_bounds__(kSearchThreads) k_search(SearchArgs a) {
  extern __shared__ __align__(16) float qs[];  // [kSearchGroup][L]
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = a.l;
  const int ntiles = a.meta[0] * a.nchunks;
  const TK* keys = static_cast<const TK*>(a.keys);

  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const int table = g.x, start = g.y, cnt = g.z;
    __syncthreads();  // previous tile's readers of qs / pid are done
    if (tid < cnt) pid[tid] = a.sorted[start + tid];
    __syncthreads();
    for (int i = tid; i < cnt * L; i += kSearchThreads) {
      const int j = i / L, c = i % L;
      const int p = pid[j];
      qs[i] = a.qlow[static_cast<int64_t>(p / a.s) * L + c];
    }
    __syncthreads();

    const int kk = chunk * kSearchChunkK + tid;
    const bool valid = kk < a.k;
    float acc[kSearchGroup];
#pragma unroll
    for (int j = 0; j < kSearchGroup; ++j) acc[j] = 0.f;
    if (valid) {
      const TK* row = keys + static_cast<int64_t>(table >> 1) * a.key_stride_e +
                      static_cast<int64_t>(table & 1) * a.key_stride_m +
                      static_cast<int64_t>(kk) * a.key_stride_k;
      if (kVec) {
#pragma unroll 2
        for (int c = 0; c < L; c += 8) {
          float kv[8];
          load8<TK>(row + c, kv);
#pragma unroll
          for (int j = 0; j < kSearchGroup; ++j) {
            if (j < cnt) {
              const float4 qa = *reinterpret_cast<const float4*>(qs + j * L + c);
              const float4 qb = *reinterpret_cast<const float4*>(qs + j * L + c + 4);
              float v = acc[j];
              v = fmaf(kv[0], qa.x, v); v = fmaf(kv[1], qa.y, v);
              v = fmaf(kv[2], qa.z, v); v = fmaf(kv[3], qa.w, v);
              v = fmaf(kv[4], qb.x, v); v = fmaf(kv[5], qb.y, v);
              v = fmaf(kv[6], qb.z, v); v = fmaf(kv[7], qb.w, v);
              acc[j] = v;
            }
          }
        }
      } else {
        for (int c = 0; c < L; ++c) {
          const float kv = to_f32<TK>(row[c]);
#pragma unroll
          for (int j = 0; j < kSearchGroup; ++j)
            if (j < cnt) acc[j] = fmaf(kv, qs[j * L + c], acc[j]);
        }
      }
    }
    // Per pair: warp max of the (rounded) score, lowest centroid among the maxima.
#pragma unroll
    for (int j = 0; j < kSearchGroup; ++j) {
      if (j < cnt) {
        const float sc = valid ? round_as<TK>(acc[j]) : -INFINITY;
        float m = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const unsigned bal = __ballot_sync(0xffffffffu, valid && sc == m);
        if (lane == 0) {
          red_s[warp][j] = m;
          red_k[warp][j] = bal ? (chunk * kSearchChunkK + warp * 32 + __ffs(bal) - 1) : -1;
        }
      }
    }
    __syncthreads();
    if (tid < cnt) {
      uint64_t bestp = 0ull;
#pragma unroll
      for (int w = 0; w < kSearchThreads / 32; ++w) {
        const int k = red_k[w][tid];
        if (k >= 0) {
          const uint64_t c = pack_cand(red_s[w][tid], a.idx_offset + static_cast<uint32_t>(k));
          bestp = c > bestp ? c : bestp;
        }
      }
      if (bestp) atomicMax(reinterpret_cast<unsigned long long*>(a.best + pid[tid]),
                           static_cast<unsigned long long>(bestp));
    }
  }
}

// Packed best -> (hit, idx) for the search API (search.py:597-602 / :689-697).
struct FinalizeArgs {
  const uint64_t* best;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* is_vision;
  const uint8_t* reuse;
  int64_t reuse_stride;
  int q, s, num_experts, cmp_ge;
  float thr_vis, thr_txt;
  uint8_t* out_hit;
  int64_t* out_idx;
  int64_t out_stride;
};

__global__ void k_finalize(FinalizeArgs a) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= static_cast<int64_t>(a.q) * a.s) return;
  const int qq = static_cast<int>(p / a.s), ss = static_cast<int>(p % a.s);
  bool hit = false;
  int64_t idx = 0;
  const bool r = a.reuse ? (a.reuse[qq * a.reuse_stride + ss] != 0) : true;
  if (r) {
    const uint64_t b = a.best[p];
    if (b) {
      const float thr = a.is_vision[qq] ? a.thr_vis : a.thr_txt;
      hit = hit_rule(cand_score(b), thr, a.cmp_ge);
      if (hit) idx = cand_index(b);
    }
  }
  a.out_hit[qq * a.out_stride + ss] = hit ? 1 : 0;
  a.out_idx[qq * a.out_stride + ss] = idx;
}

// Max-merge of per-shard packed candidates, then the hit rule.
struct MergeArgs {
  const uint64_t* packed;
  int world;
  int64_t n;
  int s;
  const uint8_t* is_vision;
  int cmp_ge;
  float thr_vis, thr_txt;
  uint8_t* out_hit;
  int64_t* out_idx;
};

__global__ void k_merge(MergeArgs a) {
  const int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (p >= a.n) return;
  uint64_t b = 0ull;
  for (int w = 0; w < a.world; ++w) {
    const uint64_t c = a.packed[static_cast<int64_t>(w) * a.n + p];
    b = c > b ? c : b;
  }
  bool hit = false;
  int64_t idx = 0;
  if (b) {
    const bool vis = a.is_vision ? (a.is_vision[p / a.s] != 0) : false;
    hit = hit_rule(cand_score(b), vis ? a.thr_vis : a.thr_txt, a.cmp_ge);
    if (hit) idx = cand_index(b);
  }
  a.out_hit[p] = hit ? 1 : 0;
  a.out_idx[p] = idx;
}

}  // namespace alut
