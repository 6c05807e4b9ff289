// Kernel 2: the centroid scan (the semantics of search.py:566-602 / :661-697 over all K
// centroids of a table: first maximal inner product, then the hit rule).
//
// Three launch shapes share one scoring routine:
//  * k_search_decode  - small batches (decode): a (slot, 128-centroid chunk) grid whose CTAs
//    elect one leader per (expert, modality) table from the routing itself, so it needs no
//    planning pass and runs as a programmatic dependent of the projection: the key chunk
//    streams in (TMA bulk copies) while the projection is still running.
//  * k_search_tma     - large batches: a persistent grid over the (table group, chunk) tiles
//    made by the planning CTA, double-buffered TMA bulk copies.
//  * k_search         - any layout (unaligned rows, odd L): plain global loads.
// Each CTA folds its per-slot best into a packed 64-bit candidate with atomicMax, whose
// order independence keeps results deterministic.
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

constexpr int kTmaBuffers = 2;
constexpr uint32_t kWaitLimit = 1u << 20;  // bounded mbarrier wait (iterations of try_wait)
constexpr int kBatch = 4;                   // slots scored together per pass over a row
constexpr int kDecodeMaxPairs = 256;
constexpr int kDecodeMaxTokens = kDecodeMaxPairs;  // any batch of <= 256 slots
#ifndef ALUT_DECODE_RUN
#define ALUT_DECODE_RUN 8
#endif
constexpr int kDecodeRun = ALUT_DECODE_RUN;  // slots of one table a decode-scan leader serves
static_assert(kDecodeRun <= kSearchGroup, "runs fit the scoring group");

// ---- TMA / mbarrier primitives ---------------------------------------------------------

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
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait with a deadline of kWaitNs (each try_wait may itself suspend for a while, so the
// bound is on time, not on the number of tries); false if the deadline passed.
constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t n = 0; n < kWaitLimit; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitNs) return false;
  }
  return false;
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

// Rows land in shared memory with a 16-byte pad after each (pitch = L*esz + 16): the 8
// threads of a shared-memory phase, reading the same 16-byte unit of 8 consecutive rows,
// then hit different bank groups, while every row is still summed in the same order
// (exact duplicate keys score identically and tie to the lowest index, as in the reference).
__host__ __device__ inline int key_pitch(int l, int esz) { return l * esz + 16; }

inline size_t search_smem_bytes(int l) { return sizeof(float) * kSearchGroup * l; }
inline size_t search_tma_smem_bytes(int l, int esz) {
  return 128 + static_cast<size_t>(kTmaBuffers) * kSearchChunkK * key_pitch(l, esz) +
         sizeof(float) * kSearchGroup * l;
}
inline size_t search_decode_smem_bytes(int l, int esz) {
  return 128 + static_cast<size_t>(kSearchChunkK) * key_pitch(l, esz) + sizeof(float) * kSearchGroup * l;
}

// ---- scoring -----------------------------------------------------------------------------

// 16 bytes of keys -> fp32 (4 or 8 elements).
template <typename TK> __device__ __forceinline__ void unit_to_f32(const TK* p, float (&o)[8]);
template <> __device__ __forceinline__ void unit_to_f32<float>(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
}
template <> __device__ __forceinline__ void unit_to_f32<__nv_bfloat16>(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void unit_to_f32<__half>(const __half* p, float (&o)[8]) {
  const uint4 r = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

// Score this thread's key row against the queries of `cnt` slots held in shared memory
// (qs[j*L + c]) and leave, per slot, the warp's best (rounded score, lowest centroid) in
// red_s/red_k[warp][j]. Slots go kBatch at a time so that the code stays small (a decode
// launch runs it once). kVec: the row is read as 16-byte units (L*esz % 16 == 0, aligned).
template <typename TK, bool kVec>
__device__ __forceinline__ void score_row(const TK* row, bool valid, const float* qs, int L, int cnt,
                                          int kbase, float (*red_s)[kSearchGroup],
                                          int (*red_k)[kSearchGroup]) {
  constexpr int kEpu = 16 / sizeof(TK);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int jb = 0; jb < cnt; jb += kBatch) {
    const int nb = min(kBatch, cnt - jb);
    const float* q0 = qs + jb * L;
    float acc[kBatch] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
      if (kVec) {
        for (int c = 0; c < L; c += kEpu) {
          float kv[8];
          unit_to_f32<TK>(row + c, kv);
#pragma unroll
          for (int j = 0; j < kBatch; ++j) {
            if (j < nb) {
              const float4 qa = *reinterpret_cast<const float4*>(q0 + j * L + c);
              float v = acc[j];
              v = fmaf(kv[0], qa.x, v); v = fmaf(kv[1], qa.y, v);
              v = fmaf(kv[2], qa.z, v); v = fmaf(kv[3], qa.w, v);
              if (kEpu == 8) {
                const float4 qb = *reinterpret_cast<const float4*>(q0 + j * L + c + 4);
                v = fmaf(kv[4], qb.x, v); v = fmaf(kv[5], qb.y, v);
                v = fmaf(kv[6], qb.z, v); v = fmaf(kv[7], qb.w, v);
              }
              acc[j] = v;
            }
          }
        }
      } else {
        for (int c = 0; c < L; ++c) {
          const float kv = to_f32<TK>(row[c]);
#pragma unroll
          for (int j = 0; j < kBatch; ++j)
            if (j < nb) acc[j] = fmaf(kv, q0[j * L + c], acc[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (j < nb) {
        const float sc = valid ? round_as<TK>(acc[j]) : -INFINITY;
        float m = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const unsigned bal = __ballot_sync(0xffffffffu, valid && sc == m);
        if (lane == 0) {
          red_s[warp][jb + j] = m;
          red_k[warp][jb + j] = bal ? kbase + warp * 32 + __ffs(bal) - 1 : -1;
        }
      }
    }
  }
}

// score_row with L fixed at compile time (the common ranks): the row's 16-byte units are
// all loaded from shared memory first, then every slot's dot product runs on registers.
template <typename TK, int LC>
__device__ __forceinline__ void score_row_fixed(const TK* row, bool valid, const float* qs, int cnt, int kbase,
                                                float (*red_s)[kSearchGroup], int (*red_k)[kSearchGroup]) {
  constexpr int kEpu = 16 / sizeof(TK);
  constexpr int kUnits = LC / kEpu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float kv[LC];
  if (valid) {
#pragma unroll
    for (int u = 0; u < kUnits; ++u) {
      float t[8];
      unit_to_f32<TK>(row + u * kEpu, t);
#pragma unroll
      for (int e = 0; e < kEpu; ++e) kv[u * kEpu + e] = t[e];
    }
  }
  for (int j = 0; j < cnt; ++j) {
    const float4* q4 = reinterpret_cast<const float4*>(qs + j * LC);
    float a0 = 0.f, a1 = 0.f;  // two partial chains; summed as (a0 + a1) in a fixed order
    if (valid) {
#pragma unroll
      for (int c = 0; c < LC / 4; ++c) {
        const float4 q = q4[c];
        float& a = (c < LC / 8) ? a0 : a1;
        a = fmaf(kv[4 * c + 0], q.x, a);
        a = fmaf(kv[4 * c + 1], q.y, a);
        a = fmaf(kv[4 * c + 2], q.z, a);
        a = fmaf(kv[4 * c + 3], q.w, a);
      }
    }
    const float sc = valid ? round_as<TK>(a0 + a1) : -INFINITY;
    float m = sc;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const unsigned bal = __ballot_sync(0xffffffffu, valid && sc == m);
    if (lane == 0) {
      red_s[warp][j] = m;
      red_k[warp][j] = bal ? kbase + warp * 32 + __ffs(bal) - 1 : -1;
    }
  }
}

// After a __syncthreads: thread j < cnt merges the warps' candidates of slot j and folds
// the result into best[pid[j]].
__device__ __forceinline__ void fold_slots(int cnt, const int* pid, uint32_t idx_offset, uint64_t* best,
                                           const float (*red_s)[kSearchGroup], const int (*red_k)[kSearchGroup]) {
  const int j = threadIdx.x;
  if (j >= cnt) return;
  uint64_t b = 0ull;
#pragma unroll
  for (int w = 0; w < kSearchThreads / 32; ++w) {
    const int k = red_k[w][j];
    if (k >= 0) {
      const uint64_t c = pack_cand(red_s[w][j], idx_offset + static_cast<uint32_t>(k));
      b = c > b ? c : b;
    }
  }
  if (b) atomicMax(reinterpret_cast<unsigned long long*>(best + pid[j]), static_cast<unsigned long long>(b));
}

// ---- generic scan (global loads) ------------------------------------------------------------

template <typename TK, bool kVec>
__global__ void __launch_bounds__(kSearchThreads) k_search(SearchArgs a) {
  extern __shared__ __align__(16) float qs[];  // [kSearchGroup][L]
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  const int tid = threadIdx.x;
  const int L = a.l;
  const int ntiles = a.meta[0] * a.nchunks;
  const TK* keys = static_cast<const TK*>(a.keys);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const int table = g.x, start = g.y, cnt = g.z;
    __syncthreads();  // the previous tile's readers of qs / pid / red are done
    if (tid < cnt) pid[tid] = a.sorted[start + tid];
    __syncthreads();
    for (int i = tid; i < cnt * L; i += kSearchThreads) {
      const int j = i / L, c = i % L;
      qs[i] = a.qlow[static_cast<int64_t>(pid[j] / a.s) * L + c];
    }
    __syncthreads();
    const int kk = chunk * kSearchChunkK + tid;
    const bool valid = kk < a.k;
    const TK* row = keys + static_cast<int64_t>(table >> 1) * a.key_stride_e +
                    static_cast<int64_t>(table & 1) * a.key_stride_m +
                    static_cast<int64_t>(valid ? kk : 0) * a.key_stride_k;
    score_row<TK, kVec>(row, valid, qs, L, cnt, chunk * kSearchChunkK, red_s, red_k);
    __syncthreads();
    fold_slots(cnt, pid, a.idx_offset, a.best, red_s, red_k);
  }
}

// ---- persistent TMA scan (large batches) -----------------------------------------------------
// The 128-row chunk of a tile arrives by one bulk copy per row into the padded layout,
// counted on the buffer's mbarrier; the next tile's chunk is issued into the other buffer
// before this one is scored.

template <typename TK>
__global__ void __launch_bounds__(kSearchThreads) k_search_tma(SearchArgs a, int* err) {
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
  const int L = a.l;
  const int pitch = key_pitch(L, sizeof(TK));
  unsigned char* kbuf = sm + 128;
  float* qs = reinterpret_cast<float*>(sm + 128 + static_cast<size_t>(kTmaBuffers) * kSearchChunkK * pitch);
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  __shared__ int s_abort;
  const int tid = threadIdx.x;
  const int ntiles = a.meta[0] * a.nchunks;
  const TK* keys = static_cast<const TK*>(a.keys);
  const uint32_t row_bytes = static_cast<uint32_t>(L) * sizeof(TK);
  if (tid == 0) {
    for (int b = 0; b < kTmaBuffers; ++b) mbar_init(&bar[b], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  __syncthreads();
  auto rows_of = [&](int tile) { return min(kSearchChunkK, a.k - (tile % a.nchunks) * kSearchChunkK); };
  auto issue = [&](int tile, int b) {  // all threads: one bulk copy per row
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const int rows = rows_of(tile);
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
    if (tid == 0 && !mbar_wait_bounded(&bar[b], parity)) {
      s_abort = 1;
      atomicOr(err, kErrCopyTimeout);
    }
    __syncthreads();
    if (s_abort) break;
    const bool ok = mbar_try_wait(&bar[b], parity);  // completed: acquire for this thread
    const int rows = rows_of(tile);
    const TK* row = reinterpret_cast<const TK*>(kbuf + (static_cast<size_t>(b) * kSearchChunkK + tid) * pitch);
    score_row<TK, true>(row, ok && tid < rows, qs, L, cnt, chunk * kSearchChunkK, red_s, red_k);
    __syncthreads();
    fold_slots(cnt, pid, a.idx_offset, a.best, red_s, red_k);
    __syncthreads();  // buffer b, qs and the reduction arrays are free again
  }
  // After an aborted wait, give this CTA's copies still in flight (the timed-out one and the
  // prefetch) a bounded chance to land before the CTA exits.
  if (s_abort && tid == 0) {
    for (int i = it; i <= it + 1; ++i) {
      if (static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x) >= ntiles) continue;
      mbar_wait_bounded(&bar[i & 1], (i >> 1) & 1);
    }
  }
}

// ---- decode scan: no planning pass, overlapped with the projection ---------------------------

struct DecodeScanArgs {
  SearchArgs s;
  int q, num_experts;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* is_vision;
  const uint8_t* reuse;
  int64_t reuse_stride;
  int* err;
  // Optional (lookup + combine): value rows of the tables, in bytes. Every CTA asks L2 to
  // fetch the value row of its chunk's best candidate of each slot, so the combine that
  // follows reads the winners from L2 instead of HBM.
  const unsigned char* values;
  int64_t vs_e, vs_m, vs_k;
  uint32_t row_bytes;
};

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// LC: L fixed at compile time (64, 96, 128: the row is scored from registers), 0 for any
// other L. Each rank is its own kernel so that registers are sized for that rank alone;
// 4 CTAs per SM stay resident (3 at L = 128, whose row alone takes 128 registers).
template <typename TK, int LC>
__global__ void __launch_bounds__(kSearchThreads, LC == 128 ? 3 : 4) k_search_decode(DecodeScanArgs d) {
  extern __shared__ __align__(128) unsigned char sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm);
  const SearchArgs& a = d.s;
  const int L = a.l;
  const int pitch = key_pitch(L, sizeof(TK));
  unsigned char* kbuf = sm + 128;
  float* qs = reinterpret_cast<float*>(sm + 128 + static_cast<size_t>(kSearchChunkK) * pitch);
  __shared__ int s_table[kDecodeMaxPairs];
  __shared__ float red_s[kSearchThreads / 32][kSearchGroup];
  __shared__ int red_k[kSearchThreads / 32][kSearchGroup];
  __shared__ int pid[kSearchGroup];
  __shared__ int s_cnt, s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int pairs = d.q * a.s;
  const int p = blockIdx.x;
  const int chunk = blockIdx.y;
  ALUT_TRACE(10);
  pdl_launch_dependents();

  // Table of every slot of the batch (-1: not searched or bad expert id).
  for (int i = tid; i < pairs; i += kSearchThreads) {
    const int qq = i / a.s, ss = i % a.s;
    const bool r = d.reuse ? (d.reuse[qq * d.reuse_stride + ss] != 0) : true;
    const int64_t e = d.sel[qq * d.sel_stride + ss];
    const bool in_range = e >= 0 && e < d.num_experts;
    s_table[i] = (r && in_range) ? static_cast<int>(e) * 2 + (d.is_vision[qq] ? 0 : 1) : -1;
    // One CTA reports searched slots with an out-of-range expert id (sticky error bit).
    if (r && !in_range && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(d.err, kErrBadExpert);
  }
  __syncthreads();
  const int table = s_table[p];
  if (table < 0) return;
  // Leaders: the searched slots routed to this table, in slot order, are served in runs of
  // kDecodeRun; the first slot of each run scans the chunk for its run.
  int before = 0;
#pragma unroll
  for (int i0 = 0; i0 < kDecodeMaxPairs; i0 += kSearchThreads) {
    const int i = i0 + tid;
    before += __syncthreads_count(i < p && s_table[i] == table);
  }
  if (before % kDecodeRun) return;
  if (warp == 0) {
    int n = 0;
    for (int base = p; base < pairs && n < kDecodeRun; base += 32) {
      const int i = base + lane;
      const bool m = i < pairs && s_table[i] == table;
      const unsigned bal = __ballot_sync(0xffffffffu, m);
      const int pos = n + __popc(bal & ((1u << lane) - 1u));
      if (m && pos < kDecodeRun) pid[pos] = i;
      n += __popc(bal);
    }
    if (lane == 0) {
      s_cnt = min(n, kDecodeRun);
      s_abort = 0;
    }
  }
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
  const int cnt = s_cnt;
  ALUT_TRACE(11);
  // The queries (and the cleared best buffer) come from the projection kernel.
  pdl_wait();
  ALUT_TRACE(12);
  for (int i = tid; i < cnt * L; i += kSearchThreads) {
    const int j = i / L, c = i % L;
    qs[i] = a.qlow[static_cast<int64_t>(pid[j] / a.s) * L + c];
  }
  if (tid == 0 && !mbar_wait_bounded(&bar[0], 0)) {
    s_abort = 1;
    atomicOr(d.err, kErrCopyTimeout);
  }
  __syncthreads();
  if (s_abort) {
    if (tid == 0) mbar_wait_bounded(&bar[0], 0);
    return;
  }
  ALUT_TRACE(13);
  const bool ok = mbar_try_wait(&bar[0], 0);
  const TK* row = reinterpret_cast<const TK*>(kbuf + static_cast<size_t>(tid) * pitch);
  if constexpr (LC > 0)
    score_row_fixed<TK, LC>(row, ok && tid < rows, qs, cnt, chunk * kSearchChunkK, red_s, red_k);
  else
    score_row<TK, true>(row, ok && tid < rows, qs, L, cnt, chunk * kSearchChunkK, red_s, red_k);
  __syncthreads();
  ALUT_TRACE(14);
  if (tid < cnt) {
    uint64_t b = 0ull;
#pragma unroll
    for (int w = 0; w < kSearchThreads / 32; ++w) {
      const int k = red_k[w][tid];
      if (k >= 0) {
        const uint64_t c = pack_cand(red_s[w][tid], a.idx_offset + static_cast<uint32_t>(k));
        b = c > b ? c : b;
      }
    }
    if (b) {
      atomicMax(reinterpret_cast<unsigned long long*>(a.best + pid[tid]), static_cast<unsigned long long>(b));
      if (d.values)  // every chunk's winner: waiting for the atomic's old value would delay the exit
        prefetch_l2_bulk(d.values + static_cast<int64_t>(table >> 1) * d.vs_e + static_cast<int64_t>(table & 1) * d.vs_m +
                             static_cast<int64_t>(cand_index(b) - a.idx_offset) * d.vs_k,
                         d.row_bytes);
    }
  }
  ALUT_TRACE(15);
}

// ---- packed best -> (hit, idx) (search.py:597-602 / :689-697) -------------------------------

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

// ---- max-merge of per-shard packed candidates, then the hit rule ---------------------------

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
