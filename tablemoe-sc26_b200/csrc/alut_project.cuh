// Kernel 1 of the search: PCA projection of the queries (search.py:476-498) fused with
// the planning step that buckets the searched (token, slot) pairs by (expert, modality)
// table, so that the search kernel streams every table once for all pairs routed to it
// (the reference's Triton kernel re-reads the table once per pair, search.py:80-84).
#pragma once

#include "alut_common.cuh"

namespace alut {

struct ProjPlanArgs {
  // projection
  const void* x;
  int64_t x_stride;
  const uint8_t* is_vision;
  const void* proj[2];
  const void* bias[2];
  int64_t proj_stride;
  const void* q_in;  // optional precomputed query [Q,L] in the key dtype
  int q, h, l, nsplit, qtiles, normalize;
  float eps;
  float* qpart;
  float* qlow;
  uint32_t* counters;
  void* q_out;  // optional typed copy of the query (alut_project)
  int64_t q_out_stride;
  // plan
  int do_plan;
  int s;
  int num_experts;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* reuse;
  int64_t reuse_stride;
  uint64_t* best;
  int* sorted;
  int4* groups;
  int* meta;
};

constexpr int kProjOutPerThread = (kProjTileQ * kMaxL) / kProjThreads;  // 16

// Dynamic shared memory of one projection CTA: the two modalities' basis chunks, then the
// token chunk; the chunk area is reused for the output tile.
inline size_t proj_smem_bytes(int l) {
  size_t ps = sizeof(float) * 2 * kProjChunkH * l;
  size_t xs = sizeof(float) * kProjTileQ * kProjChunkH;
  size_t tile = sizeof(float) * kProjTileQ * l;
  size_t a = ps + xs;
  return a > tile ? a : tile;
}
inline size_t plan_smem_bytes(int num_tables) { return sizeof(int) * 3 * num_tables; }

__device__ __forceinline__ int block_exclusive_scan_256(int v, int* scratch, int* total) {
  // Hillis-Steele inclusive scan over 256 threads, returned as exclusive.
  const int tid = threadIdx.x;
  scratch[tid] = v;
  __syncthreads();
  for (int off = 1; off < kProjThreads; off <<= 1) {
    int add = tid >= off ? scratch[tid - off] : 0;
    __syncthreads();
    scratch[tid] += add;
    __syncthreads();
  }
  int incl = scratch[tid];
  if (total) *total = scratch[kProjThreads - 1];
  __syncthreads();
  return incl - v;
}

// Bucket the searched pairs by table. Runs in one CTA of kProjThreads threads.
__device__ void plan_pairs(const ProjPlanArgs& a, int* smem) {
  const int tid = threadIdx.x;
  const int ntab = 2 * a.num_experts;
  const int64_t pairs = static_cast<int64_t>(a.q) * a.s;
  int* counts = smem;
  int* offs = smem + ntab;
  int* gofs = smem + 2 * ntab;
  __shared__ int scan_scratch[kProjThreads];
  __shared__ int s_tot_c, s_tot_g;

  if (tid == 0) a.meta[1] = 0;
  for (int t = tid; t < ntab; t += kProjThreads) counts[t] = 0;
  __syncthreads();
  for (int64_t p = tid; p < pairs; p += kProjThreads) {
    const int qq = static_cast<int>(p / a.s), ss = static_cast<int>(p % a.s);
    a.best[p] = 0ull;
    const bool r = a.reuse ? (a.reuse[qq * a.reuse_stride + ss] != 0) : true;
    if (!r) continue;
    const int64_t e = a.sel[qq * a.sel_stride + ss];
    if (e < 0 || e >= a.num_experts) {
      atomicOr(&a.meta[1], 1);
      continue;
    }
    const int t = static_cast<int>(e) * 2 + (a.is_vision[qq] ? 0 : 1);
    atomicAdd(&counts[t], 1);
  }
  __syncthreads();
  // Exclusive scans of the pair counts and of the group counts per table.
  const int per = (ntab + kProjThreads - 1) / kProjThreads;
  const int t0 = tid * per;
  const int t1 = min(ntab, t0 + per);
  int lc = 0, lg = 0;
  for (int t = t0; t < t1; ++t) {
    lc += counts[t];
    lg += (counts[t] + kSearchGroup - 1) / kSearchGroup;
  }
  int bc = block_exclusive_scan_256(lc, scan_scratch, &s_tot_c);
  int bg = block_exclusive_scan_256(lg, scan_scratch, &s_tot_g);
  for (int t = t0; t < t1; ++t) {
    offs[t] = bc;
    gofs[t] = bg;
    const int c = counts[t];
    for (int g = 0; g * kSearchGroup < c; ++g) {
      a.groups[bg + g] = make_int4(t, bc + g * kSearchGroup, min(kSearchGroup, c - g * kSearchGroup), 0);
    }
    bc += c;
    bg += (c + kSearchGroup - 1) / kSearchGroup;
  }
  if (tid == 0) a.meta[0] = s_tot_g;
  __syncthreads();
  // Scatter pair ids into their table's bucket (the order inside a bucket does not
  // matter: every pair's result is independent of the others).
  for (int64_t p = tid; p < pairs; p += kProjThreads) {
    const int qq = static_cast<int>(p / a.s), ss = static_cast<int>(p % a.s);
    const bool r = a.reuse ? (a.reuse[qq * a.reuse_stride + ss] != 0) : true;
    if (!r) continue;
    const int64_t e = a.sel[qq * a.sel_stride + ss];
    if (e < 0 || e >= a.num_experts) continue;
    const int t = static_cast<int>(e) * 2 + (a.is_vision[qq] ? 0 : 1);
    const int pos = atomicAdd(&offs[t], 1);
    a.sorted[pos] = static_cast<int>(p);
  }
}

// Bias, rounding to the key dtype and optional L2 normalisation of one finished tile
// held in shared memory (search.py:12-21, :484-488). One warp per row.
template <typename TP, typename TK>
__device__ void finish_tile(const ProjPlanArgs& a, float* tile, int q0, int nq,
                            const int* mod, bool add_bias) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = a.l;
  for (int r = warp; r < nq; r += kProjThreads / 32) {
    const int m = mod[r];
    const TP* b = static_cast<const TP*>(a.bias[m]);
    float ss = 0.f;
    for (int c = lane; c < L; c += 32) {
      float v = tile[r * L + c];
      if (add_bias) v = v + to_f32<TP>(b[c]);
      v = round_as<TK>(v);
      tile[r * L + c] = v;
      ss = fmaf(v, v, ss);
    }
    float denom = 1.f;
    bool zero = false;
    if (a.normalize) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float n = round_as<TK>(sqrtf(ss));
      const float eps = round_as<TK>(a.eps);
      denom = fmaxf(n, eps);
      zero = n <= eps;
    }
    const int64_t row = q0 + r;
    for (int c = lane; c < L; c += 32) {
      float v = tile[r * L + c];
      if (a.normalize) v = zero ? 0.f : round_as<TK>(v / denom);
      a.qlow[row * L + c] = v;
      if (a.q_out) static_cast<TK*>(a.q_out)[row * a.q_out_stride + c] = from_f32<TK>(v);
    }
  }
}

template <typename TX, typename TP, typename TK>
__global__ void __launch_bounds__(kProjThreads) k_project_plan(ProjPlanArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int nproj = a.qtiles * a.nsplit;
  if (a.do_plan && static_cast<int>(blockIdx.x) == nproj) {
    plan_pairs(a, reinterpret_cast<int*>(smem));
    return;
  }
  const int tid = threadIdx.x;
  const int L = a.l;
  const int qt = blockIdx.x / a.nsplit;
  const int sp = blockIdx.x % a.nsplit;
  const int q0 = qt * kProjTileQ;
  const int nq = min(kProjTileQ, a.q - q0);
  __shared__ int mod[kProjTileQ];
  __shared__ int need[2];
  __shared__ int s_last;
  if (tid < 2) need[tid] = 0;
  __syncthreads();
  if (tid < kProjTileQ) {
    const int m = tid < nq ? (a.is_vision[q0 + tid] ? 0 : 1) : 1;
    mod[tid] = m;
    if (tid < nq) need[m] = 1;
  }
  __syncthreads();

  float* tile = smem;
  if (a.q_in) {
    // Precomputed query: copy it (already in the key dtype) and skip the projection.
    const TK* qi = static_cast<const TK*>(a.q_in);
    for (int i = tid; i < nq * L; i += kProjThreads) {
      const int r = i / L, c = i % L;
      const float v = to_f32<TK>(qi[static_cast<int64_t>(q0 + r) * L + c]);
      a.qlow[static_cast<int64_t>(q0 + r) * L + c] = v;
      if (a.q_out) static_cast<TK*>(a.q_out)[static_cast<int64_t>(q0 + r) * a.q_out_stride + c] = qi[static_cast<int64_t>(q0 + r) * L + c];
    }
    return;
  }

  float* ps = smem;                                   // [2][kProjChunkH][L]
  float* xs = smem + 2 * kProjChunkH * L;             // [kProjTileQ][kProjChunkH]
  const int nout = (kProjTileQ * L + kProjThreads - 1) / kProjThreads;
  float acc[kProjOutPerThread];
  int oq[kProjOutPerThread], ol[kProjOutPerThread];
#pragma unroll
  for (int i = 0; i < kProjOutPerThread; ++i) {
    acc[i] = 0.f;
    const int o = tid + i * kProjThreads;
    oq[i] = o / L;
    ol[i] = o % L;
  }
  const int nch = (a.h + kProjChunkH - 1) / kProjChunkH;
  const int c_begin = static_cast<int>(static_cast<int64_t>(sp) * nch / a.nsplit);
  const int c_end = static_cast<int>(static_cast<int64_t>(sp + 1) * nch / a.nsplit);
  const TX* x = static_cast<const TX*>(a.x);
  for (int c = c_begin; c < c_end; ++c) {
    const int h0 = c * kProjChunkH;
    const int hn = min(kProjChunkH, a.h - h0);
    __syncthreads();
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (!need[m]) continue;
      const TP* p = static_cast<const TP*>(a.proj[m]);
      for (int i = tid; i < kProjChunkH * L; i += kProjThreads) {
        const int r = i / L, col = i % L;
        ps[m * kProjChunkH * L + i] =
            r < hn ? to_f32<TP>(p[static_cast<int64_t>(h0 + r) * a.proj_stride + col]) : 0.f;
      }
    }
    for (int i = tid; i < kProjTileQ * kProjChunkH; i += kProjThreads) {
      const int r = i / kProjChunkH, col = i % kProjChunkH;
      xs[i] = (r < nq && col < hn) ? to_f32<TX>(x[static_cast<int64_t>(q0 + r) * a.x_stride + h0 + col]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kProjOutPerThread; ++i) {
      if (i < nout && oq[i] < kProjTileQ) {
        const float* prow = ps + mod[oq[i]] * kProjChunkH * L + ol[i];
        const float* xrow = xs + oq[i] * kProjChunkH;
        float v = acc[i];
#pragma unroll
        for (int hh = 0; hh < kProjChunkH; ++hh) v = fmaf(xrow[hh], prow[hh * L], v);
        acc[i] = v;
      }
    }
  }
  __syncthreads();
  if (a.nsplit == 1) {
#pragma unroll
    for (int i = 0; i < kProjOutPerThread; ++i)
      if (i < nout && oq[i] < kProjTileQ) tile[oq[i] * L + ol[i]] = acc[i];
  } else {
    float* part = a.qpart + static_cast<int64_t>(qt * a.nsplit + sp) * kProjTileQ * L;
#pragma unroll
    for (int i = 0; i < kProjOutPerThread; ++i)
      if (i < nout && oq[i] < kProjTileQ) __stcg(part + oq[i] * L + ol[i], acc[i]);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(&a.counters[qt], 1u) == static_cast<unsigned>(a.nsplit - 1));
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) a.counters[qt] = 0u;
    // The last CTA of the tile sums the partials in split order (deterministic).
    const float* base = a.qpart + static_cast<int64_t>(qt * a.nsplit) * kProjTileQ * L;
    for (int i = tid; i < kProjTileQ * L; i += kProjThreads) {
      float v = 0.f;
      for (int k = 0; k < a.nsplit; ++k) v += __ldcg(base + static_cast<int64_t>(k) * kProjTileQ * L + i);
      tile[i] = v;
    }
  }
  __syncthreads();
  finish_tile<TP, TK>(a, tile, q0, nq, mod, true);
}

}  // namespace alut
