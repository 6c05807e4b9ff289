// Kernel 1 of the search: PCA projection of the queries (search.py:476-498), plus the
// planning kernel that buckets the searched (token, slot) pairs by (expert, modality)
// table for large batches, so that the scan streams every table once for all pairs routed
// to it (the reference's Triton kernel re-reads the table once per pair, search.py:80-84).
//
// Projection: a CTA computes a 16-token x L tile over a range of H. Basis rows and token
// chunks stream through two shared-memory buffers with cp.async; each thread owns one
// column l and NOUT tokens, so one basis element feeds NOUT FMAs. When H is split over
// several CTAs (small batches), those CTAs form a thread-block cluster and add their
// partial tiles through distributed shared memory in split order - no global partials,
// atomics or fences, and the same sum on every run.
#pragma once

#include <cooperative_groups.h>

#include "alut_common.cuh"

namespace alut {

namespace cg = cooperative_groups;

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
  float* qlow;
  void* q_out;  // optional typed copy of the query (alut_project)
  int64_t q_out_stride;
  // decode path: clear best[0, zero_n) for the scan that follows
  uint64_t* zero_best;
  int zero_n;
  // plan
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
  // tensor-core scan: per-slot candidate counters, cleared with `best` (NULL otherwise)
  int* cand_cnt;
  // tensor-core projection: bf16 split basis [2][3][L][H] (see alut_prepare_basis)
  const __nv_bfloat16* proj_split;
  // plan: slots per search group (kSearchGroup for the CUDA-core scans, 128 for the
  // tensor-core scan); 0 means kSearchGroup
  int group;
};

// Tokens per thread (a thread owns one column l of NOUT tokens; 16/NOUT token groups of L
// threads fit in the CTA): 4 for L <= 64, 8 for L <= 128, 16 for L <= 256.
inline int proj_nout(int l) { return l <= 64 ? 4 : (l <= 128 ? 8 : 16); }

// Basis rows per pipeline chunk: 64, or 32 when L > 128 so that everything fits in 227 KB.
__host__ __device__ inline int proj_chunk_rows(int l) { return l > 128 ? 32 : 64; }

// Shared memory: two pipeline buffers (both modalities' basis chunk [HC][L] and the raw
// token chunk [16][HC], each in its storage dtype of <= 4 bytes), the fp32 token chunk
// transposed [HC][16], and two fp32 [16][L] tiles (this CTA's partial, the reduced rows).
struct ProjSmem {
  size_t buf, xt, tile, red, total;
};
__host__ __device__ inline ProjSmem proj_smem_layout(int l) {
  const int hc = proj_chunk_rows(l);
  ProjSmem s;
  s.buf = align256(sizeof(float) * (2 * hc * l + kProjTileQ * hc));
  s.xt = 2 * s.buf;
  s.tile = s.xt + align256(sizeof(float) * hc * kProjTileQ);
  s.red = s.tile + align256(sizeof(float) * kProjTileQ * l);
  s.total = s.red + align256(sizeof(float) * kProjTileQ * l);
  return s;
}
inline size_t proj_smem_bytes(int l) { return proj_smem_layout(l).total; }
inline size_t plan_smem_bytes(int num_tables, int64_t pairs) {
  return sizeof(int) * (3 * static_cast<size_t>(num_tables) + static_cast<size_t>(pairs));
}

// ---- planning (large batches) --------------------------------------------------------------

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

// Table of slot p, or -1 when the slot is not searched (reuse mask off) or its expert id is
// out of range (then *bad is set).
__device__ __forceinline__ int plan_table(const ProjPlanArgs& a, int64_t p, bool* bad) {
  const int qq = static_cast<int>(p / a.s), ss = static_cast<int>(p % a.s);
  const bool r = a.reuse ? (a.reuse[qq * a.reuse_stride + ss] != 0) : true;
  if (!r) return -1;
  const int64_t e = a.sel[qq * a.sel_stride + ss];
  if (e < 0 || e >= a.num_experts) {
    *bad = true;
    return -1;
  }
  return static_cast<int>(e) * 2 + (a.is_vision[qq] ? 0 : 1);
}

// Bucket the searched pairs by table (one CTA of kProjThreads threads): per-table counts,
// block scans, group list (<= kSearchGroup pairs of one table each), scatter of pair ids.
__global__ void __launch_bounds__(kProjThreads) k_plan(ProjPlanArgs a) {
  extern __shared__ __align__(16) int plan_smem[];
  const int tid = threadIdx.x;
  const int G = a.group > 0 ? a.group : kSearchGroup;
  const int ntab = 2 * a.num_experts;
  const int pairs = a.q * a.s;  // <= kPlanWideSlots (the caller picks the wide plan above)
  int* counts = plan_smem;
  int* offs = plan_smem + ntab;
  int* tab_of = plan_smem + 3 * ntab;  // table of each slot, -1 when not searched
  __shared__ int scan_scratch[kProjThreads];
  __shared__ int s_tot_c, s_tot_g;

  for (int t = tid; t < ntab; t += kProjThreads) counts[t] = 0;
  // Every slot's routing is read once, in independent loads (no atomics in this loop, so
  // the loads of successive slots overlap), into shared memory.
  bool bad = false;
#pragma unroll 4
  for (int p = tid; p < pairs; p += kProjThreads) {
    tab_of[p] = plan_table(a, p, &bad);
    a.best[p] = 0ull;
    if (a.cand_cnt) a.cand_cnt[p] = 0;
  }
  if (bad) atomicOr(&a.meta[1], kErrBadExpert);
  __syncthreads();
  for (int p = tid; p < pairs; p += kProjThreads) {
    const int t = tab_of[p];
    if (t >= 0) atomicAdd(&counts[t], 1);
  }
  __syncthreads();
  const int per = (ntab + kProjThreads - 1) / kProjThreads;
  const int t0 = tid * per;
  const int t1 = min(ntab, t0 + per);
  int lc = 0, lg = 0;
  for (int t = t0; t < t1; ++t) {
    lc += counts[t];
    lg += (counts[t] + G - 1) / G;
  }
  int bc = block_exclusive_scan_256(lc, scan_scratch, &s_tot_c);
  int bg = block_exclusive_scan_256(lg, scan_scratch, &s_tot_g);
  for (int t = t0; t < t1; ++t) {
    offs[t] = bc;
    const int c = counts[t];
    for (int g = 0; g * G < c; ++g)
      a.groups[bg + g] = make_int4(t, bc + g * G, min(G, c - g * G), 0);
    bc += c;
    bg += (c + G - 1) / G;
  }
  if (tid == 0) a.meta[0] = s_tot_g;
  __syncthreads();
  // Scatter slot ids into their table's bucket (the order inside a bucket does not matter:
  // every slot's result is independent of the others).
  for (int p = tid; p < pairs; p += kProjThreads) {
    const int t = tab_of[p];
    if (t < 0) continue;
    const int pos = atomicAdd(&offs[t], 1);
    a.sorted[pos] = p;
  }
}

// ---- plan of large batches: three launches over the whole GPU ----------------------------
// k_plan serialises every slot through one CTA; for large batches the same plan is built by
// (1) k_plan_count: clears `best`, counts the searched slots per table (warp-aggregated
//     shared-memory histogram, one global add per table per CTA), flags bad expert ids;
// (2) k_plan_groups (one CTA): scans the counts into bucket offsets and the group list;
// (3) k_plan_scatter: writes each searched slot id into its table's bucket (warp-aggregated
//     atomics on the bucket cursors). The order inside a bucket does not matter.
// `counts` must be zero before (1).

__global__ void __launch_bounds__(256) k_plan_count(ProjPlanArgs a, int* counts) {
  extern __shared__ __align__(16) int hist[];
  const int ntab = 2 * a.num_experts;
  const int64_t pairs = static_cast<int64_t>(a.q) * a.s;
  for (int t = threadIdx.x; t < ntab; t += blockDim.x) hist[t] = 0;
  __syncthreads();
  bool bad = false;
  const int lane = threadIdx.x & 31;
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) - lane; base < pairs;
       base += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = base + lane;
    int t = -1;
    if (p < pairs) {
      a.best[p] = 0ull;
      if (a.cand_cnt) a.cand_cnt[p] = 0;
      t = plan_table(a, p, &bad);
    }
    const unsigned same = __match_any_sync(0xffffffffu, t);
    if (t >= 0 && lane == __ffs(same) - 1) atomicAdd(&hist[t], __popc(same));
  }
  if (bad) atomicOr(&a.meta[1], kErrBadExpert);
  __syncthreads();
  for (int t = threadIdx.x; t < ntab; t += blockDim.x)
    if (hist[t]) atomicAdd(&counts[t], hist[t]);
}

__global__ void __launch_bounds__(kProjThreads) k_plan_groups(ProjPlanArgs a, const int* counts, int* offs) {
  extern __shared__ __align__(16) int pg_smem[];  // [ntab + 1] first group of each table
  const int tid = threadIdx.x;
  const int G = a.group > 0 ? a.group : kSearchGroup;
  const int ntab = 2 * a.num_experts;
  int* gstart = pg_smem;
  __shared__ int scan_scratch[kProjThreads];
  __shared__ int s_tot_c, s_tot_g;
  const int per = (ntab + kProjThreads - 1) / kProjThreads;
  const int t0 = tid * per;
  const int t1 = min(ntab, t0 + per);
  int lc = 0, lg = 0;
  for (int t = t0; t < t1; ++t) {
    lc += counts[t];
    lg += (counts[t] + G - 1) / G;
  }
  int bc = block_exclusive_scan_256(lc, scan_scratch, &s_tot_c);
  int bg = block_exclusive_scan_256(lg, scan_scratch, &s_tot_g);
  for (int t = t0; t < t1; ++t) {
    offs[t] = bc;
    gstart[t] = bg;
    bc += counts[t];
    bg += (counts[t] + G - 1) / G;
  }
  if (tid == 0) {
    gstart[ntab] = s_tot_g;
    a.meta[0] = s_tot_g;
  }
  __syncthreads();
  // Groups in parallel: group gi belongs to the last table whose first group is <= gi (never
  // an empty table: its first group equals the next table's).
  for (int gi = tid; gi < s_tot_g; gi += kProjThreads) {
    int lo = 0, hi = ntab;  // gstart[lo] <= gi < gstart[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (gstart[mid] <= gi) lo = mid; else hi = mid;
    }
    const int k = gi - gstart[lo];
    a.groups[gi] = make_int4(lo, offs[lo] + k * G, min(G, counts[lo] - k * G), 0);
  }
}

__global__ void __launch_bounds__(256) k_plan_scatter(ProjPlanArgs a, int* offs) {
  const int64_t pairs = static_cast<int64_t>(a.q) * a.s;
  const int lane = threadIdx.x & 31;
  bool bad = false;
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) - lane; base < pairs;
       base += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = base + lane;
    const int t = p < pairs ? plan_table(a, p, &bad) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, t);
    const int leader = __ffs(same) - 1;
    int pos = 0;
    if (t >= 0 && lane == leader) pos = atomicAdd(&offs[t], __popc(same));
    pos = __shfl_sync(0xffffffffu, pos, leader);
    if (t >= 0) a.sorted[pos + __popc(same & ((1u << lane) - 1))] = static_cast<int>(p);
  }
}

// ---- projection ---------------------------------------------------------------------------

// Bias, rounding to the key dtype and optional L2 normalisation of rows [r0, r1) of a
// finished tile (search.py:12-21, :484-488). One warp per row.
template <typename TK>
__device__ void finish_rows(const ProjPlanArgs& a, float* tile_base, int q0, int r0, int r1, const int* mod,
                            const float (*bias)[kMaxL], int tile_row0 = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = a.l;
  float* tile = tile_base - static_cast<int64_t>(tile_row0) * L;  // tile[r * L] for r in [r0, r1)
  for (int r = r0 + warp; r < r1; r += kProjThreads / 32) {
    const float* b = bias[mod[r]];
    float ss = 0.f;
    for (int c = lane; c < L; c += 32) {
      const float v = round_as<TK>(tile[r * L + c] + b[c]);
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

template <typename TX, typename TP, typename TK, int NOUT>
__global__ void __launch_bounds__(kProjThreads) k_project(ProjPlanArgs a) {
  extern __shared__ __align__(256) unsigned char psm[];
  ALUT_TRACE(0);
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  const int L = a.l;
  const int qt = blockIdx.x / a.nsplit;
  const int sp = blockIdx.x % a.nsplit;  // == rank in the cluster when nsplit > 1
  const int q0 = qt * kProjTileQ;
  const int nq = min(kProjTileQ, a.q - q0);
  const ProjSmem lay = proj_smem_layout(L);
  float* tile = reinterpret_cast<float*>(psm + lay.tile);
  float* red = reinterpret_cast<float*>(psm + lay.red);
  float* xt = reinterpret_cast<float*>(psm + lay.xt);
  __shared__ int mod[kProjTileQ];
  __shared__ int need[2];
  __shared__ float s_bias[2][kMaxL];
  // Before waiting for the previous kernel: only static tables are read (the first basis
  // chunk of both modalities and the biases), so this overlaps the predecessor's tail when
  // the kernel is launched as a programmatic dependent.
  // proj_chunk_rows(L) as a constant: NOUT 16 <=> L > 128 <=> 32 rows, else 64.
  constexpr int HC = NOUT == 16 ? 32 : 64;
  const int nch = (a.h + HC - 1) / HC;
  const int c_begin = static_cast<int>(static_cast<int64_t>(sp) * nch / a.nsplit);
  const int c_end = static_cast<int>(static_cast<int64_t>(sp + 1) * nch / a.nsplit);
  const bool p_vec = (L * sizeof(TP)) % 16 == 0 && (a.proj_stride * sizeof(TP)) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(a.proj[0]) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(a.proj[1]) & 15) == 0;
  auto stage_p = [&](int c, int b, int mask) {
    TP* ps = reinterpret_cast<TP*>(psm + b * lay.buf);  // [2][HC][L]
    const int h0 = c * HC;
    const int hn = min(HC, a.h - h0);
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (!((mask >> m) & 1)) continue;
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
  };
  if (!a.q_in) {
    if (c_begin < c_end) stage_p(c_begin, 0, 3);
    cp_async_commit();
    for (int i = tid; i < 2 * L; i += kProjThreads)
      s_bias[i / L][i % L] = to_f32<TP>(static_cast<const TP*>(a.bias[i / L])[i % L]);
  }
  pdl_wait();
  if (a.zero_best && blockIdx.x == 0)
    for (int i = tid; i < a.zero_n; i += kProjThreads) a.zero_best[i] = 0ull;
  if (tid < 2) need[tid] = 0;
  __syncthreads();
  if (tid < kProjTileQ) {
    const int m = tid < nq ? (a.is_vision[q0 + tid] ? 0 : 1) : 1;
    mod[tid] = m;
    if (tid < nq) need[m] = 1;
  }
  __syncthreads();
  ALUT_TRACE(1);

  if (a.q_in) {
    // Precomputed query (already in the key dtype): copy it, no projection (nsplit == 1).
    const TK* qi = static_cast<const TK*>(a.q_in);
    for (int i = tid; i < nq * L; i += kProjThreads) {
      const int64_t o = static_cast<int64_t>(q0) * L + i;
      a.qlow[o] = to_f32<TK>(qi[o]);
      if (a.q_out) static_cast<TK*>(a.q_out)[(q0 + i / L) * a.q_out_stride + i % L] = qi[o];
    }
    return;
  }

  // Thread -> (column l, token group g): tokens g*NOUT .. g*NOUT+NOUT-1.
  constexpr int kGroups = kProjTileQ / NOUT;
  const int l = tid % L;
  const int g = tid / L;
  const bool active = g < kGroups;
  float acc[NOUT];
#pragma unroll
  for (int i = 0; i < NOUT; ++i) acc[i] = 0.f;
  int mbits = 0;  // bit i: token g*NOUT+i is a text token
  if (active)
#pragma unroll
    for (int i = 0; i < NOUT; ++i) mbits |= mod[g * NOUT + i] << i;

  const TX* x = static_cast<const TX*>(a.x);
  const bool x_vec = (HC * sizeof(TX)) % 16 == 0 && (a.x_stride * sizeof(TX)) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  // Token chunk (and, after the first chunk, the needed modalities' basis chunk).
  auto stage = [&](int c, int b, bool with_p) {
    unsigned char* base = psm + b * lay.buf;
    TX* xs = reinterpret_cast<TX*>(base + sizeof(float) * 2 * HC * L);    // [16][HC]
    const int h0 = c * HC;
    const int hn = min(HC, a.h - h0);
    if (with_p) stage_p(c, b, need[0] | (need[1] << 1));
    if (x_vec && hn == HC) {
      constexpr int kE = 16 / sizeof(TX);
      const int per_row = HC / kE;
      for (int i = tid; i < kProjTileQ * per_row; i += kProjThreads) {
        const int r = i / per_row, u = i % per_row;
        if (r < nq) {
          cp_async16(xs + r * HC + u * kE, x + static_cast<int64_t>(q0 + r) * a.x_stride + h0 + u * kE);
        } else {
          for (int e = 0; e < kE; ++e) xs[r * HC + u * kE + e] = TX(0.f);
        }
      }
    } else {
      for (int i = tid; i < kProjTileQ * HC; i += kProjThreads) {
        const int r = i / HC, col = i % HC;
        xs[i] = (r < nq && col < hn) ? x[static_cast<int64_t>(q0 + r) * a.x_stride + h0 + col] : TX(0.f);
      }
    }
    cp_async_commit();
  };

  if (c_begin < c_end) stage(c_begin, 0, false);
  ALUT_TRACE(2);
  for (int c = c_begin; c < c_end; ++c) {
    const int b = (c - c_begin) & 1;
    if (c + 1 < c_end) {
      stage(c + 1, b ^ 1, true);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (c == c_begin) ALUT_TRACE(3);
    const unsigned char* base = psm + b * lay.buf;
    const TP* ps = reinterpret_cast<const TP*>(base);
    const TX* xs = reinterpret_cast<const TX*>(base + sizeof(float) * 2 * HC * L);
    // Tokens to fp32, transposed to [HC][16] so a thread reads its NOUT tokens with 16-byte loads.
#ifdef ALUT_PHASE_TRACE
    const long long ck0 = clock64();
#endif
    for (int i = tid; i < kProjTileQ * HC; i += kProjThreads) {
      const int r = i / HC, hh = i % HC;
      xt[hh * kProjTileQ + r] = to_f32<TX>(xs[i]);
    }
#ifdef ALUT_PHASE_TRACE
    const long long ck1 = clock64();
#endif
    __syncthreads();
#ifdef ALUT_PHASE_TRACE
    const long long ck2 = clock64();
#endif
    if (active && !(need[0] && need[1])) {
      // One modality in the tile (the common case): no per-token select.
      const TP* pb = ps + (need[0] ? 0 : HC * L) + l;
#pragma unroll 16
      for (int hh = 0; hh < HC; ++hh) {
        const float bw = to_f32<TP>(pb[hh * L]);
        const float* xr = xt + hh * kProjTileQ + g * NOUT;
#pragma unroll
        for (int i = 0; i < NOUT; i += 4) {
          const float4 xv = *reinterpret_cast<const float4*>(xr + i);
          acc[i + 0] = fmaf(xv.x, bw, acc[i + 0]);
          acc[i + 1] = fmaf(xv.y, bw, acc[i + 1]);
          acc[i + 2] = fmaf(xv.z, bw, acc[i + 2]);
          acc[i + 3] = fmaf(xv.w, bw, acc[i + 3]);
        }
      }
    } else if (active) {
      const TP* pv = ps + l;
      const TP* pt = ps + HC * L + l;
      const bool nv = need[0], nt = need[1];
#pragma unroll 4
      for (int hh = 0; hh < HC; ++hh) {
        const float bv = nv ? to_f32<TP>(pv[hh * L]) : 0.f;
        const float bt = nt ? to_f32<TP>(pt[hh * L]) : 0.f;
        const float* xr = xt + hh * kProjTileQ + g * NOUT;
#pragma unroll
        for (int i = 0; i < NOUT; i += 4) {
          const float4 xv = *reinterpret_cast<const float4*>(xr + i);
          acc[i + 0] = fmaf(xv.x, (mbits >> (i + 0)) & 1 ? bt : bv, acc[i + 0]);
          acc[i + 1] = fmaf(xv.y, (mbits >> (i + 1)) & 1 ? bt : bv, acc[i + 1]);
          acc[i + 2] = fmaf(xv.z, (mbits >> (i + 2)) & 1 ? bt : bv, acc[i + 2]);
          acc[i + 3] = fmaf(xv.w, (mbits >> (i + 3)) & 1 ? bt : bv, acc[i + 3]);
        }
      }
    }
#ifdef ALUT_PHASE_TRACE
    const long long ck3 = clock64();
    if (c == c_begin) {
      ALUT_TRACE_VAL(33, ck1 - ck0);
      ALUT_TRACE_VAL(34, ck2 - ck1);
      ALUT_TRACE_VAL(35, ck3 - ck2);
    }
#endif
    __syncthreads();  // buffer b and xt may be refilled
    if (c == c_begin) ALUT_TRACE(4);
  }
  ALUT_TRACE(5);
  if (active)
#pragma unroll
    for (int i = 0; i < NOUT; ++i) tile[(g * NOUT + i) * L + l] = acc[i];

  if (a.nsplit == 1) {
    __syncthreads();
    finish_rows<TK>(a, tile, q0, 0, nq, mod, s_bias);
    return;
  }
  // Split over a cluster: rank sp reduces rows [r0, r1) over all ranks' partial tiles, in
  // rank order, then finishes them.
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  ALUT_TRACE(6);
  const int rows_per = (kProjTileQ + a.nsplit - 1) / a.nsplit;
  const int r0 = min(nq, sp * rows_per);
  const int r1 = min(nq, r0 + rows_per);
  for (int i = r0 * L + tid; i < r1 * L; i += kProjThreads) {
    float v = 0.f;
    for (int k = 0; k < a.nsplit; ++k) v += cluster.map_shared_rank(tile, k)[i];
    red[i] = v;
  }
  __syncthreads();
  ALUT_TRACE(7);
  finish_rows<TK>(a, red, q0, r0, r1, mod, s_bias);
  ALUT_TRACE(8);
  cluster.sync();
  ALUT_TRACE(9);  // peers may still be reading this CTA's tile
}

// ---- tensor-core projection (small batches, bf16 tokens, fp32 basis) ----------------------
// q = x @ P with x exact in bf16 and P = hi + mid + lo split into three bf16 parts (the
// split is exact to fp32 precision), so mma.sync m16n8k16 (bf16 in, fp32 accumulate) over
// the three parts gives an fp32-accurate product. One m16 tile is the 16-token tile; warp w
// owns the 8-column n-tiles w, w+8, ...; a CTA covers a range of k-steps (16 rows of H) and
// the split CTAs of a token tile reduce through distributed shared memory as in k_project.
// The split basis is static, so the first block of it is requested before griddepcontrol.wait.

__global__ void __launch_bounds__(kProjThreads) k_split_basis(const float* proj0, const float* proj1,
                                                            int64_t stride_h, int h, int l,
                                                            __nv_bfloat16* out) {
  const int64_t n = static_cast<int64_t>(2) * l * h;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / (static_cast<int64_t>(l) * h));
    const int64_t r = i % (static_cast<int64_t>(l) * h);
    const int col = static_cast<int>(r / h), k = static_cast<int>(r % h);
    const float p = (m == 0 ? proj0 : proj1)[static_cast<int64_t>(k) * stride_h + col];
    const __nv_bfloat16 hi = __float2bfloat16_rn(p);
    const float r1 = p - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    const int64_t plane = static_cast<int64_t>(l) * h;
    __nv_bfloat16* o = out + static_cast<int64_t>(m) * 3 * plane + static_cast<int64_t>(col) * h + k;
    o[0] = hi;
    o[plane] = mid;
    o[2 * plane] = lo;
  }
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kMmaKBlock = 8;             // k-steps whose fragments are loaded together
constexpr size_t kMmaStageBudget = 200 * 1024;  // shared memory for a staged basis slice (L=96, H=2560 fits)

// Shared memory of k_project_mma: the CTA's slice of the split basis (both modalities,
// 3 parts, L columns, rows of krange k padded by 16 bytes so fragment loads of 8 columns
// hit different banks) when it fits, then the receive buffer of the cluster reduction
// ([nsplit][rows_per][L] fp32 partial rows pushed by every rank to the row's owner).
struct MmaSmem {
  int krange, pitch;  // elements of k per slice row, bytes per padded slice row
  bool staged;
  size_t recv, total;
};
__host__ __device__ inline MmaSmem mma_smem_layout(int l, int h, int nsplit) {
  MmaSmem m;
  const int ksteps = h / 16;
  m.krange = ((ksteps + nsplit - 1) / nsplit) * 16;
  m.pitch = m.krange * 2 + 16;
  const size_t sb = static_cast<size_t>(6) * l * m.pitch;
  m.staged = sb <= kMmaStageBudget;
  m.recv = m.staged ? align256(sb) : 0;
  const int rows_per = (kProjTileQ + nsplit - 1) / nsplit;
  m.total = m.recv + align256(sizeof(float) * static_cast<size_t>(nsplit) * rows_per * l);
  return m;
}

// NT: n-tiles a warp takes per pass (1 when L <= 64, 2 above): the register footprint of the
// common L = 64 case stays that of one tile, which keeps room on the SMs for the CTAs of the
// kernels around it.
template <typename TK, int NT>
__global__ void __launch_bounds__(kProjThreads) k_project_mma(ProjPlanArgs a) {
  extern __shared__ __align__(256) unsigned char psm[];
  ALUT_TRACE(0);
  pdl_launch_dependents();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;  // mma fragment row group / thread-in-group
  const int L = a.l, H = a.h;
  const int qt = blockIdx.x / a.nsplit;
  const int sp = blockIdx.x % a.nsplit;
  const int q0 = qt * kProjTileQ;
  const int nq = min(kProjTileQ, a.q - q0);
  const MmaSmem lay = mma_smem_layout(L, H, a.nsplit);
  float* recv = reinterpret_cast<float*>(psm + lay.recv);
  __shared__ int mod[kProjTileQ];
  __shared__ float s_bias[2][kMaxL];
  const int ksteps = H / 16;
  const int k_begin = static_cast<int>(static_cast<int64_t>(sp) * ksteps / a.nsplit);
  const int k_end = static_cast<int>(static_cast<int64_t>(sp + 1) * ksteps / a.nsplit);
  const int ntiles = L / 8;
  const int64_t plane = static_cast<int64_t>(L) * H;
  // Static data first (overlaps the predecessor under programmatic launch): biases and the
  // CTA's slice of the split basis, both modalities, into shared memory.
  for (int i = tid; i < 2 * L; i += kProjThreads)
    s_bias[i / L][i % L] = static_cast<const float*>(a.bias[i / L])[i % L];
  const int kn16 = (k_end - k_begin) * 16;  // elements of k in this slice
  // The text basis is staged before the dependency wait (text is every decode token's
  // modality); the vision basis after it, only when the tile holds a vision token.
  const int units = kn16 / 8;  // 16-byte units per slice row
  auto stage_modality = [&](int m) {
    for (int i = tid; i < 3 * L * units; i += kProjThreads) {
      const int row = m * 3 * L + i / units, u = i % units;  // row = (m*3 + part)*L + col
      cp_async16(psm + static_cast<size_t>(row) * lay.pitch + u * 16,
                 a.proj_split + static_cast<int64_t>(row) * H + static_cast<int64_t>(k_begin) * 16 + u * 8);
    }
  };
  if (lay.staged) stage_modality(1);
  cp_async_commit();
  pdl_wait();
  // This call's inputs, requested together: the first k-block of this thread's x fragments
  // and the modality of every row of the tile (each warp derives what it needs from the
  // latter with shuffles and ballots, so no block barrier sits between the two loads).
  const bool row0_ok = gq < nq, row1_ok = gq + 8 < nq;
  const __nv_bfloat16* xr0 = static_cast<const __nv_bfloat16*>(a.x) + static_cast<int64_t>(q0 + (row0_ok ? gq : 0)) * a.x_stride;
  const __nv_bfloat16* xr1 = static_cast<const __nv_bfloat16*>(a.x) + static_cast<int64_t>(q0 + (row1_ok ? gq + 8 : 0)) * a.x_stride;
  uint32_t xa[kMmaKBlock][4];
  auto load_x = [&](int kb) {
    const int kn = min(kMmaKBlock, k_end - kb);
#pragma unroll
    for (int s = 0; s < kMmaKBlock; ++s) {
      if (s < kn) {
        const int k0 = (kb + s) * 16 + 2 * tq;
        xa[s][0] = row0_ok ? *reinterpret_cast<const uint32_t*>(xr0 + k0) : 0u;
        xa[s][1] = row1_ok ? *reinterpret_cast<const uint32_t*>(xr1 + k0) : 0u;
        xa[s][2] = row0_ok ? *reinterpret_cast<const uint32_t*>(xr0 + k0 + 8) : 0u;
        xa[s][3] = row1_ok ? *reinterpret_cast<const uint32_t*>(xr1 + k0 + 8) : 0u;
      }
    }
  };
  int x_block = k_begin;  // the k-block whose fragments xa holds
  if (warp < ntiles && k_begin < k_end) load_x(k_begin);
  const bool lane_vis = lane < nq && a.is_vision[q0 + lane] != 0;
  const unsigned vis_bits = __ballot_sync(0xffffffffu, lane_vis);
  const unsigned rows_bits = nq >= 32 ? 0xffffffffu : ((1u << nq) - 1u);
  const bool need_m[2] = {vis_bits != 0u, (rows_bits & ~vis_bits) != 0u};
  const int m_r0 = (vis_bits >> gq) & 1u ? 0 : 1, m_r1 = (vis_bits >> (gq + 8)) & 1u ? 0 : 1;
  if (warp == 0 && lane < kProjTileQ) mod[lane] = lane_vis ? 0 : 1;  // for finish_rows
  if (lay.staged && need_m[0]) {  // uniform over the CTA: every warp saw the same ballot
    stage_modality(0);
    cp_async_commit();
  }
  if (a.zero_best && blockIdx.x == 0)
    for (int i = tid; i < a.zero_n; i += kProjThreads) a.zero_best[i] = 0ull;
  cp_async_wait<0>();
  __syncthreads();
  ALUT_TRACE(1);
  const int rows_per = (kProjTileQ + a.nsplit - 1) / a.nsplit;
  cg::cluster_group cluster = cg::this_cluster();
  // Every CTA of the cluster must be running before any writes into its shared memory:
  // arrive now, wait just before the first remote store (the MMAs run in between).
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  bool cluster_ready = false;
  // A warp owns n-tiles warp, warp + 8, ...; it takes them NT at a time so that one load of
  // its x fragments serves them all.
  constexpr int kWarps = kProjThreads / 32;
  for (int nt0 = warp; nt0 < ntiles; nt0 += NT * kWarps) {
    const int nts = (NT == 2 && nt0 + kWarps < ntiles) ? 2 : 1;
    // One accumulator per (n-tile, basis part): independent MMA chains, each n-tile's parts
    // added (hi + mid) + lo at the end.
    float cp[NT][3][4] = {};
    for (int kb = k_begin; kb < k_end; kb += kMmaKBlock) {
      const int kn = min(kMmaKBlock, k_end - kb);
      if (kb != x_block) {
        load_x(kb);
        x_block = kb;
      }
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (!need_m[m]) continue;
        // Rows of the other modality are zeroed in A, so the two passes add exactly.
        const uint32_t keep0 = (m_r0 == m) ? 0xffffffffu : 0u, keep1 = (m_r1 == m) ? 0xffffffffu : 0u;
#pragma unroll
        for (int s = 0; s < kMmaKBlock; ++s) {
          if (s < kn) {
            const uint32_t am[4] = {xa[s][0] & keep0, xa[s][1] & keep1, xa[s][2] & keep0, xa[s][3] & keep1};
            const int kl = (kb + s - k_begin) * 16 + 2 * tq;  // k within the slice
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t < nts) {
#pragma unroll
                for (int part = 0; part < 3; ++part) {
                  const int row = (m * 3 + part) * L + (nt0 + t * kWarps) * 8 + gq;
                  uint32_t b0, b1;
                  if (lay.staged) {
                    const unsigned char* br = psm + static_cast<size_t>(row) * lay.pitch;
                    b0 = *reinterpret_cast<const uint32_t*>(br + kl * 2);
                    b1 = *reinterpret_cast<const uint32_t*>(br + kl * 2 + 16);
                  } else {
                    const __nv_bfloat16* bg =
                        a.proj_split + static_cast<int64_t>(row) * H + static_cast<int64_t>(k_begin) * 16 + kl;
                    b0 = *reinterpret_cast<const uint32_t*>(bg);
                    b1 = *reinterpret_cast<const uint32_t*>(bg + 8);
                  }
                  mma_bf16_16816(cp[t][part], am, b0, b1);
                }
              }
            }
          }
        }
      }
    }
    // Push the partial rows to their owners' receive buffers (slot = this rank).
    if (!cluster_ready) {
      asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
      cluster_ready = true;
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      if (t < nts) {
        float c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = (cp[t][0][i] + cp[t][1][i]) + cp[t][2][i];
        const int col = (nt0 + t * kWarps) * 8 + 2 * tq;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int r = gq + 8 * half;
          const int owner = r / rows_per;
          float* dst =
              cluster.map_shared_rank(recv, owner) + (static_cast<size_t>(sp) * rows_per + r % rows_per) * L + col;
          dst[0] = c[2 * half];
          dst[1] = c[2 * half + 1];
        }
      }
    }
  }
  if (!cluster_ready) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // warps without n-tiles
  ALUT_TRACE(5);
  cluster.sync();  // every partial row has arrived at its owner; nothing remote is read after this
  ALUT_TRACE(6);
  // The owner of rows [r0, r1) sums the ranks' partials in rank order and finishes them.
  const int r0 = min(nq, sp * rows_per);
  const int r1 = min(nq, r0 + rows_per);
  // In place: element (rr, c) of slot 0 is read and written by one thread only.
  for (int i = tid; i < (r1 - r0) * L; i += kProjThreads) {
    const int rr = i / L, c2 = i % L;
    float v = 0.f;
    for (int k = 0; k < a.nsplit; ++k) v += recv[(static_cast<size_t>(k) * rows_per + rr) * L + c2];
    recv[static_cast<size_t>(rr) * L + c2] = v;
  }
  __syncthreads();
  ALUT_TRACE(7);
  finish_rows<TK>(a, recv, q0, r0, r1, mod, s_bias, r0);
  ALUT_TRACE(8);
}

}  // namespace alut
