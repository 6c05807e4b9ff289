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
  pdl_wait();
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

namespace alut {

// ---- TMA-staged centroid scan ----------------------------------------------------------
// Same contract as k_search, for tables whose rows are contiguous 16-byte multiples: the
// 128-row chunk of a tile is one contiguous block that a single thread moves into shared
// memory with a bulk asynchronous copy (cp.async.bulk, completion counted on an mbarrier),
// double-buffered so the next tile's chunk streams in while this one is scored. Loads from
// HBM are thus fully coalesced 16-byte-aligned bursts issued by the TMA unit, and the
// threads read their rows from shared memory starting at a per-row rotated 16-byte unit so
// that the 8 threads of a shared-memory phase hit 8 different bank groups.

constexpr int kTmaBuffers = 2;
constexpr uint32_t kWaitLimit = 1u << 20;  // bounded mbarrier wait (iterations of try_wait)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Rows land in shared memory with a 16-byte pad after each (pitch = L*esz + 16), so the
// 8 threads of a shared-memory phase, reading the same 16-byte unit of 8 consecutive rows,
// hit 8 different bank groups while every row is still summed in the same order (exact
// duplicate keys score identically and tie to the lowest index, as in the reference).
__host__ __device__ inline int key_pitch(int l, int esz) { return l * esz + 16; }

inline size_t search_tma_smem_bytes(int l, int esz) {
  return 128 + static_cast<size_t>(kTmaBuffers) * kSearchChunkK * key_pitch(l, esz) + sizeof(float) * kSearchGroup * l;
}

template <typename TK>
__device__ __forceinline__ void unit_to_f32(const TK* p, float (&o)[8]);
template <>
__device__ __forceinline__ void unit_to_f32<float>(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
}
template <>
__device__ __forceinline__ void unit_to_f32<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void unit_to_f32<__half>(const __half* p, float (&o)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

template <typename TK>
__global__ void __launch_bounds__(kSearchThreads) k_search_tma(SearchArgs a, int* err) {
  constexpr int kEpu = 16 / sizeof(TK);  // elements per 16-byte unit
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
  const int L = a.l;
  const int units = L / kEpu;
  const int pitch = key_pitch(L, sizeof(TK));
  unsigned char* kbuf = sm + 128;
  float* qs = reinterpret_cast<float*>(sm + 128 + static_cast<size_t>(kTmaBuffers) * kSearchChunkK * pitch);
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntiles = a.meta[0] * a.nchunks;
  const TK* keys = static_cast<const TK*>(a.keys);

  if (tid == 0) {
    for (int b = 0; b < kTmaBuffers; ++b) mbar_init(&bar[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  __syncthreads();

  auto chunk_rows = [&](int tile) {
    const int chunk = tile % a.nchunks;
    return min(kSearchChunkK, a.k - chunk * kSearchChunkK);
  };
  auto issue = [&](int tile, int b) {  // all threads: one bulk copy per row
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const int rows = chunk_rows(tile);
    const uint32_t row_bytes = static_cast<uint32_t>(L) * sizeof(TK);
    if (tid == 0) {
      fence_async_shared();
      mbar_expect_tx(&bar[b], row_bytes * rows);
    }
    __syncthreads();
    if (tid < rows) {
      const TK* src = keys + static_cast<int64_t>(g.x >> 1) * a.key_stride_e +
                      static_cast<int64_t>(g.x & 1) * a.key_stride_m +
                      (static_cast<int64_t>(chunk) * kSearchChunkK + tid) * L;
      bulk_g2s(kbuf + (static_cast<size_t>(b) * kSearchChunkK + tid) * pitch, src, row_bytes, &bar[b]);
    }
  };

  if (static_cast<int>(blockIdx.x) < ntiles) issue(blockIdx.x, 0);
  int it = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
    const int b = it & 1;
    const uint32_t parity = (it >> 1) & 1;
    const int next = tile + gridDim.x;
    if (next < ntiles) issue(next, b ^ 1);
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const int start = g.y, cnt = g.z;
    if (tid < cnt) pid[tid] = a.sorted[start + tid];
    __syncthreads();
    for (int i = tid; i < cnt * L; i += kSearchThreads) {
      const int j = i / L, c = i % L;
      qs[i] = a.qlow[static_cast<int64_t>(pid[j] / a.s) * L + c];
    }
    // Bounded wait for this tile's keys.
    if (tid == 0) {
      uint32_t n = 0;
      while (!mbar_try_wait(&bar[b], parity)) {
        if (++n >= kWaitLimit) {
          s_abort = 1;
          atomicOr(err, 4);
          break;
        }
      }
    }
    __syncthreads();
    if (s_abort) break;
    const bool ok = mbar_try_wait(&bar[b], parity);  // acquire for every thread (already complete)
    const int rows = chunk_rows(tile);
    const bool valid = ok && tid < rows;
    float acc[kSearchGroup];
#pragma unroll
    for (int j = 0; j < kSearchGroup; ++j) acc[j] = 0.f;
    if (valid) {
      const TK* row = reinterpret_cast<const TK*>(kbuf + (static_cast<size_t>(b) * kSearchChunkK + tid) * pitch);
      for (int u = 0; u < units; ++u) {
        float kv[8];
        unit_to_f32<TK>(row + u * kEpu, kv);
        const int c = u * kEpu;
#pragma unroll
        for (int j = 0; j < kSearchGroup; ++j) {
          if (j < cnt) {
            const float4 qa = *reinterpret_cast<const float4*>(qs + j * L + c);
            float v = acc[j];
            v = fmaf(kv[0], qa.x, v); v = fmaf(kv[1], qa.y, v);
            v = fmaf(kv[2], qa.z, v); v = fmaf(kv[3], qa.w, v);
            if (kEpu == 8) {
              const float4 qb = *reinterpret_cast<const float4*>(qs + j * L + c + 4);
              v = fmaf(kv[4], qb.x, v); v = fmaf(kv[5], qb.y, v);
              v = fmaf(kv[6], qb.z, v); v = fmaf(kv[7], qb.w, v);
            }
            acc[j] = v;
          }
        }
      }
    }
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
    __syncthreads();  // buffer b and the reduction arrays are free again
  }
  // After an aborted wait, give this CTA's copies still in flight (the timed-out one in
  // buffer it&1 and the prefetch in the other buffer) a bounded chance to land before exit.
  if (s_abort && tid == 0) {
    const int pend[2] = {it, it + 1};
    for (int i = 0; i < 2; ++i) {
      const int t = static_cast<int>(blockIdx.x) + pend[i] * static_cast<int>(gridDim.x);
      if (t >= ntiles) continue;
      for (uint32_t n = 0; n < kWaitLimit && !mbar_try_wait(&bar[pend[i] & 1], (pend[i] >> 1) & 1); ++n) {
      }
    }
  }
}

}  // namespace alut

namespace alut {

// ---- Decode scan: no planning pass, overlapped with the projection --------------------
// For small batches (decode: Q <= 32 tokens) the (token, slot) pairs are few, so every CTA
// of a (pair, 128-centroid chunk) grid reads the routing of the whole batch into shared
// memory and works out by itself whether its pair is the first searched pair routed to
// its (expert, modality) table; only that leader CTA scans the chunk, for all pairs of
// the table at once, so each table chunk is still read once. Because this needs nothing
// computed by the projection, the kernel is launched as a programmatic dependent of it:
// the key chunk's bulk copy is issued before griddepcontrol.wait, and streams from HBM
// while the projection is still running; only the dot products wait for the queries.

constexpr int kDecodeMaxPairs = 256;
constexpr int kDecodeMaxTokens = 32;


struct DecodeScanArgs {
  SearchArgs s;
  int q, num_experts;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* is_vision;
  const uint8_t* reuse;
  int64_t reuse_stride;
  int* err;
};

template <typename TK>
__global__ void __launch_bounds__(kSearchThreads) k_search_decode(DecodeScanArgs d) {
  constexpr int kEpu = 16 / sizeof(TK);
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
  const SearchArgs& a = d.s;
  const int L = a.l;
  const int units = L / kEpu;
  const int pitch = key_pitch(L, sizeof(TK));
  unsigned char* kbuf = sm + 128;
  float* qs = reinterpret_cast<float*>(sm + 128 + static_cast<size_t>(kSearchChunkK) * pitch);
  __shared__ int s_table[kDecodeMaxPairs];
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  __shared__ int s_cnt, s_lead, s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pairs = d.q * a.s;
  const int p = blockIdx.x;
  const int chunk = blockIdx.y;
  pdl_launch_dependents();

  // Table of every pair (-1: not searched or bad expert id).
  for (int i = tid; i < pairs; i += kSearchThreads) {
    const int qq = i / a.s, ss = i % a.s;
    const bool r = d.reuse ? (d.reuse[qq * d.reuse_stride + ss] != 0) : true;
    const int64_t e = d.sel[qq * d.sel_stride + ss];
    s_table[i] = (r && e >= 0 && e < d.num_experts) ? static_cast<int>(e) * 2 + (d.is_vision[qq] ? 0 : 1) : -1;
  }
  __syncthreads();
  const int table = s_table[p];
  if (table < 0) return;
  if (tid == 0) {
    int lead = 1;
    for (int i = 0; i < p; ++i) lead &= (s_table[i] != table);
    s_lead = lead;
    int n = 0;
    if (lead)
      for (int i = p; i < pairs && n < kSearchGroup; ++i)
        if (s_table[i] == table) pid[n++] = i;
    s_cnt = n;
    s_abort = 0;
  }
  __syncthreads();
  if (!s_lead) return;
  const int cnt = s_cnt;
  const int rows = min(kSearchChunkK, a.k - chunk * kSearchChunkK);
  const uint32_t row_bytes = static_cast<uint32_t>(L) * sizeof(TK);
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(&bar[0], row_bytes * rows);
  }
  __syncthreads();
  if (tid < rows) {
    const TK* src = static_cast<const TK*>(a.keys) + static_cast<int64_t>(table >> 1) * a.key_stride_e +
                    static_cast<int64_t>(table & 1) * a.key_stride_m +
                    (static_cast<int64_t>(chunk) * kSearchChunkK + tid) * L;
    bulk_g2s(kbuf + static_cast<size_t>(tid) * pitch, src, row_bytes, &bar[0]);
  }
  // The queries (and the zeroed best buffer) come from the projection kernel.
  pdl_wait();
  for (int i = tid; i < cnt * L; i += kSearchThreads) {
    const int j = i / L, c = i % L;
    qs[i] = a.qlow[static_cast<int64_t>(pid[j] / a.s) * L + c];
  }
  if (tid == 0) {
    uint32_t n = 0;
    while (!mbar_try_wait(&bar[0], 0)) {
      if (++n >= kWaitLimit) {
        s_abort = 1;
        atomicOr(d.err, 4);
        break;
      }
    }
  }
  __syncthreads();
  if (s_abort) {
    if (tid == 0)
      for (uint32_t n = 0; n < kWaitLimit && !mbar_try_wait(&bar[0], 0); ++n) {
      }
    return;
  }
  const bool ok = mbar_try_wait(&bar[0], 0);
  const bool valid = ok && tid < rows;
  float acc[kSearchGroup];
#pragma unroll
  for (int j = 0; j < kSearchGroup; ++j) acc[j] = 0.f;
  if (valid) {
    const TK* row = reinterpret_cast<const TK*>(kbuf + static_cast<size_t>(tid) * pitch);
    for (int u = 0; u < units; ++u) {
      float kv[8];
      unit_to_f32<TK>(row + u * kEpu, kv);
      const int c = u * kEpu;
#pragma unroll
      for (int j = 0; j < kSearchGroup; ++j) {
        if (j < cnt) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + j * L + c);
          float v = acc[j];
          v = fmaf(kv[0], qa.x, v); v = fmaf(kv[1], qa.y, v);
          v = fmaf(kv[2], qa.z, v); v = fmaf(kv[3], qa.w, v);
          if (kEpu == 8) {
            const float4 qb = *reinterpret_cast<const float4*>(qs + j * L + c + 4);
            v = fmaf(kv[4], qb.x, v); v = fmaf(kv[5], qb.y, v);
            v = fmaf(kv[6], qb.z, v); v = fmaf(kv[7], qb.w, v);
          }
          acc[j] = v;
        }
      }
    }
  }
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

inline size_t search_decode_smem_bytes(int l, int esz) {
  return 128 + static_cast<size_t>(kSearchChunkK) * key_pitch(l, esz) + sizeof(float) * kSearchGroup * l;
}

}  // namespace alut
