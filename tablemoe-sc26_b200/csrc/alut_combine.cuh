// Kernel 3: gather / scale / accumulate of the looked-up value rows
// (cached_layers.py:455-465 restricted to the lookup slots, with the survivor
// renormalisation of skip/pruning.py:55-73 fused as a per-token prologue).
// One CTA owns a 512-element slice of one token's output row, so the weighted sum over
// slots is an in-register fp32 sum in slot order: no atomics, deterministic.
#pragma once

#include "alut_common.cuh"

namespace alut {

struct CombineArgs {
  const void* values;
  int64_t vs_e, vs_m, vs_k;
  int h, q, s, num_experts, k;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* is_vision;
  const uint8_t* reuse;
  int64_t reuse_stride;
  // Lookup outcome: either the packed best of the fused search ...
  const uint64_t* best;
  int cmp_ge;
  float thr_vis, thr_txt;
  // ... or the caller's hit / idx arrays.
  const uint8_t* hit_in;
  const int64_t* idx_in;
  int64_t hit_stride;
  const float* w;
  int64_t w_stride;
  const uint8_t* compute;
  int64_t compute_stride;
  int renorm, accumulate;
  void* out;
  int64_t out_stride;
  uint8_t* out_hit;
  int64_t* out_idx;
  int64_t out_hit_stride;
};

constexpr int kCombineSpan = kCombineThreads * 8;
static_assert(kMaxSlots <= kCombineThreads, "one slot per thread in the combine prologue");

// Shared memory of one token's combine.
struct CombineSmem {
  float w[kMaxSlots];
  uint8_t surv[kMaxSlots];
  uint8_t look[kMaxSlots];
  int64_t off[kMaxSlots];
  float wl[kMaxSlots];
  int64_t offl[kMaxSlots];
  int n;
};

// One token's combine by the whole CTA: hit rule per slot (from the packed best, read past
// L1 because other CTAs wrote it with atomics), survivor renormalisation, then the weighted
// fp32 sum of the looked-up rows in slot order over columns [h_begin, h_end), 8 per thread
// per pass. Ends with a barrier, so `sm` may be reused for the next token. Not inlined: the
// decode scan calls it only in the CTAs that complete a token.
template <typename TV, typename TO, bool kVec>
__device__ __noinline__ void combine_token(const CombineArgs& a, int t, int64_t h_begin, int64_t h_end,
                                           bool write_hits, CombineSmem& sm) {
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int m = a.is_vision[t] ? 0 : 1;
  for (int s = tid; s < a.s; s += nthr) {
    const bool r = a.reuse ? (a.reuse[t * a.reuse_stride + s] != 0) : true;
    const int64_t e = a.sel[t * a.sel_stride + s];
    const bool ev = e >= 0 && e < a.num_experts;
    bool hit = false;
    int64_t idx = 0;
    if (a.best) {
      if (r && ev) {
        const uint64_t b =
            __ldcg(reinterpret_cast<const unsigned long long*>(a.best) + static_cast<int64_t>(t) * a.s + s);
        if (b) {
          hit = hit_rule(cand_score(b), m == 0 ? a.thr_vis : a.thr_txt, a.cmp_ge);
          if (hit) idx = cand_index(b);
        }
      }
    } else {
      hit = r && a.hit_in[t * a.hit_stride + s] != 0;
      idx = a.idx_in[t * a.hit_stride + s];
    }
    if (a.out_hit && write_hits) {
      a.out_hit[t * a.out_hit_stride + s] = hit ? 1 : 0;
      a.out_idx[t * a.out_hit_stride + s] = hit ? idx : 0;
    }
    const bool comp = a.compute ? (a.compute[t * a.compute_stride + s] != 0) : false;
    const bool look = hit && ev && idx >= 0 && idx < a.k;
    sm.w[s] = a.w[t * a.w_stride + s];
    sm.surv[s] = (comp || hit) ? 1 : 0;
    sm.look[s] = look ? 1 : 0;
    sm.off[s] = look ? (e * a.vs_e + m * a.vs_m + idx * a.vs_k) : 0;
  }
  __syncthreads();
  if (tid == 0) {
    float kept = 0.f, tot = 0.f;
    for (int s = 0; s < a.s; ++s) {
      kept += sm.surv[s] ? sm.w[s] : 0.f;
      tot += sm.w[s];
    }
    int n = 0;
    for (int s = 0; s < a.s; ++s) {
      if (!sm.look[s]) continue;
      float w = sm.w[s];
      if (a.renorm == ALUT_RENORM_TO_ONE) w = kept > 0.f ? w / kept : 0.f;
      else if (a.renorm == ALUT_RENORM_TO_ROWSUM) w = kept > 0.f ? (w / kept) * tot : 0.f;
      sm.wl[n] = w;
      sm.offl[n] = sm.off[s];
      ++n;
    }
    sm.n = n;
  }
  __syncthreads();
  ALUT_TRACE(23);
  if (a.out) {
    const int n = sm.n;
    const TV* vals = static_cast<const TV*>(a.values);
    for (int64_t h0 = h_begin + static_cast<int64_t>(tid) * 8; h0 < h_end; h0 += static_cast<int64_t>(nthr) * 8) {
      TO* out = static_cast<TO*>(a.out) + static_cast<int64_t>(t) * a.out_stride + h0;
      float acc[8];
      if (kVec) {
        if (a.accumulate) load8_rw<TO>(out, acc);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        }
        // Four rows' loads in flight before their FMAs, which still run in slot order.
        int i = 0;
        for (; i + 4 <= n; i += 4) {
          float v[4][8];
#pragma unroll
          for (int u = 0; u < 4; ++u) load8<TV>(vals + sm.offl[i + u] + h0, v[u]);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float w = sm.wl[i + u];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = fmaf(w, v[u][j], acc[j]);
          }
        }
        for (; i < n; ++i) {
          float v[8];
          load8<TV>(vals + sm.offl[i] + h0, v);
          const float w = sm.wl[i];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = fmaf(w, v[j], acc[j]);
        }
        store8<TO>(out, acc);
      } else {
        const int64_t rem = h_end - h0;
        const int cnt = rem < 8 ? static_cast<int>(rem) : 8;
        for (int j = 0; j < cnt; ++j) acc[j] = a.accumulate ? to_f32<TO>(out[j]) : 0.f;
        for (int i = 0; i < n; ++i) {
          const float w = sm.wl[i];
          for (int j = 0; j < cnt; ++j) acc[j] = fmaf(w, to_f32<TV>(vals[sm.offl[i] + h0 + j]), acc[j]);
        }
        for (int j = 0; j < cnt; ++j) out[j] = from_f32<TO>(acc[j]);
      }
    }
  }
  ALUT_TRACE(24);
  __syncthreads();
}

// Stand-alone combine: one CTA per (token, 512-column slice).
template <typename TV, typename TO, bool kVec>
__global__ void __launch_bounds__(kCombineThreads) k_combine(CombineArgs a) {
  __shared__ CombineSmem sm;
  ALUT_TRACE(20);
  pdl_launch_dependents();
  pdl_wait();
  ALUT_TRACE(22);
  const int64_t h0 = static_cast<int64_t>(blockIdx.y) * kCombineSpan;
  const int64_t h1 = h0 + kCombineSpan < a.h ? h0 + kCombineSpan : a.h;
  combine_token<TV, TO, kVec>(a, blockIdx.x, h0, h1, blockIdx.y == 0, sm);
}

// Bit-exact copy of value rows (manager.py:212-228). Rows are moved as 16-byte words
// when sizes and addresses allow, else element by element.
struct GatherArgs {
  const char* values;
  int64_t vs_e, vs_m, vs_k;  // in bytes
  int64_t row_bytes;
  int esz, num_experts, k;
  const int64_t* eids;
  const int64_t* mids;
  const int64_t* cids;
  const int64_t* out_rows;
  char* out;
  int64_t out_stride;  // in bytes
  int vec;
};

__global__ void k_gather_rows(GatherArgs a) {
  const int i = blockIdx.x;
  const int64_t e = a.eids[i], m = a.mids[i], c = a.cids[i];
  const int64_t r = a.out_rows ? a.out_rows[i] : i;
  char* dst = a.out + r * a.out_stride;
  const bool ok = e >= 0 && e < a.num_experts && m >= 0 && m < 2 && c >= 0 && c < a.k;
  const char* src = a.values + e * a.vs_e + m * a.vs_m + c * a.vs_k;
  if (a.vec) {
    const int64_t nw = a.row_bytes / 16;
    for (int64_t w = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x; w < nw;
         w += static_cast<int64_t>(gridDim.y) * blockDim.x) {
      uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(src) + w) : make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(dst)[w] = v;
    }
  } else {
    for (int64_t b = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x; b < a.row_bytes;
         b += static_cast<int64_t>(gridDim.y) * blockDim.x) {
      dst[b] = ok ? src[b] : 0;
    }
  }
}

}  // namespace alut
