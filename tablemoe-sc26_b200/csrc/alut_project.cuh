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
  // decode path: zero best[0, zero_n) (no planning CTA)
  uint64_t* zero_best;
  int zero_n;
};

constexpr int kProjOutPerThread = (kProjTileQ * kMaxL) / kProjThreads;  // 16

// Dynamic shared memory of one projection CTA: two pipeline buffers, each holding both
// modalities' basis chunk [kProjChunkH][L] and the token chunk [kProjTileQ][kProjChunkH] in
// their storage dtypes (<= 4 bytes); the area is reused for the fp32 output tile.
// Basis rows per pipeline chunk: 64, or 32 when L > 128 so two buffers fit in 227 KB.
__host__ __device__ inline int proj_chunk_rows(int l) { return l > 128 ? kProjChunkH / 2 : kProjChunkH; }
__host__ __device__ inline size_t proj_buffer_bytes(int l) {
  const int hc = proj_chunk_rows(l);
  return align256(sizeof(float) * (2 * hc * l + kProjTileQ * hc));
}
inline size_t proj_smem_bytes(int l) {
  size_t a = 2 * proj_buffer_bytes(l);
  size_t tile = sizeof(float) * kProjTileQ * l;
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
  extern __shared__ __align__(256) float smem[];
  pdl_launch_dependents();
  if (a.zero_best && blockIdx.x == 0)
    for (int i = threadIdx.x; i < a.zero_n; i += kProjThreads) a.zero_best[i] = 0ull;
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

  // Basis and token chunks stream through two shared-memory buffers with cp.async
  // (16-byte copies when rows are 16-byte multiples and aligned, else 4-byte ones or plain
  // loads), so the next chunk is in flight while this one is multiplied.
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
  const int HC = proj_chunk_rows(L);
  const int nch = (a.h + HC - 1) / HC;
  const int c_begin = static_cast<int>(static_cast<int64_t>(sp) * nch / a.nsplit);
  const int c_end = static_cast<int>(static_cast<int64_t>(sp + 1) * nch / a.nsplit);
  const TX* x = static_cast<const TX*>(a.x);
  const size_t buf_bytes = proj_buffer_bytes(L);
  const bool p_vec = (L * sizeof(TP)) % 16 == 0 && (a.proj_stride * sizeof(TP)) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(a.proj[0]) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.proj[1]) & 15) == 0;
  const bool x_vec = (HC * sizeof(TX)) % 16 == 0 && (a.x_stride * sizeof(TX)) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.h * sizeof(TX)) % 16 == 0;
  auto stage = [&](int c, int b) {
    unsigned char* base = reinterpret_cast<unsigned char*>(smem) + b * buf_bytes;
    TP* ps = reinterpret_cast<TP*>(base);                                   // [2][HC][L]
    TX* xs = reinterpret_cast<TX*>(base + sizeof(float) * 2 * HC * L);  // [16][HC]
    const int h0 = c * HC;
    const int hn = min(HC, a.h - h0);
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (!need[m]) continue;
      const TP* pg = static_cast<const TP*>(a.proj[m]) + static_cast<int64_t>(h0) * a.proj_stride;
      TP* pd = ps + m * HC * L;
      if (p_vec) {
        constexpr int kE = 16 / sizeof(TP);
        const int per_row = L / kE;
        for (int i = tid; i < hn * per_row; i += kProjThreads) {
          const int r = i / per_row, u = i % per_row;
          cp_async16(pd + r * L + u * kE, pg + static_cast<int64_t>(r) * a.proj_stride + u * kE);
        }
      } else {
        for (int i = tid; i < hn * L; i += kProjThreads) {
          const int r = i / L, col = i % L;
          pd[r * L + col] = pg[static_cast<int64_t>(r) * a.proj_stride + col];
        }
      }
      for (int i = hn * L + tid; i < HC * L; i += kProjThreads) pd[i] = TP(0.f);
    }
    if (x_vec && hn == HC) {
      constexpr int kE = 16 / sizeof(TX);
      const int per_row = HC / kE;
      for (int i = tid; i < kProjTileQ * per_row; i += kProjThreads) {
        const int r = i / per_row, u = i % per_row;
        if (r < nq) cp_async16(xs + r * HC + u * kE, x + static_cast<int64_t>(q0 + r) * a.x_stride + h0 + u * kE);
        else
          for (int e = 0; e < kE; ++e) xs[r * HC + u * kE + e] = TX(0.f);
      }
    } else {
      for (int i = tid; i < kProjTileQ * HC; i += kProjThreads) {
        const int r = i / HC, col = i % HC;
        xs[i] = (r < nq && col < hn) ? x[static_cast<int64_t>(q0 + r) * a.x_stride + h0 + col] : TX(0.f);
      }
    }
    cp_async_commit();
  };
  if (c_begin < c_end) stage(c_begin, 0);
  for (int c = c_begin; c < c_end; ++c) {
    const int b = (c - c_begin) & 1;
    if (c + 1 < c_end) {
      stage(c + 1, b ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const unsigned char* base = reinterpret_cast<const unsigned char*>(smem) + b * buf_bytes;
    const TP* ps = reinterpret_cast<const TP*>(base);
    const TX* xs = reinterpret_cast<const TX*>(base + sizeof(float) * 2 * HC * L);
#pragma unroll
    for (int i = 0; i < kProjOutPerThread; ++i) {
      if (i < nout && oq[i] < kProjTileQ) {
        const TP* prow = ps + mod[oq[i]] * HC * L + ol[i];
        const TX* xrow = xs + oq[i] * HC;
        float v = acc[i];
#pragma unroll 16
        for (int hh = 0; hh < HC; ++hh) v = fmaf(to_f32<TX>(xrow[hh]), to_f32<TP>(prow[hh * L]), v);
        acc[i] = v;
      }
    }
    __syncthreads();  // buffer b may be refilled by the next iteration's stage()
  }
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
    // Loads are issued 8 splits at a time (independent), then added in split order.
    const int64_t stride = static_cast<int64_t>(kProjTileQ) * L;
    for (int i = tid; i < kProjTileQ * L; i += kProjThreads) {
      float v = 0.f;
      int k = 0;
      for (; k + 8 <= a.nsplit; k += 8) {
        float p[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) p[u] = __ldcg(base + (k + u) * stride + i);
#pragma unroll
        for (int u = 0; u < 8; ++u) v += p[u];
      }
      for (; k < a.nsplit; ++k) v += __ldcg(base + k * stride + i);
      tile[i] = v;
    }
  }
  __syncthreads();
  finish_tile<TP, TK>(a, tile, q0, nq, mod, true);
}

}  // namespace alut
