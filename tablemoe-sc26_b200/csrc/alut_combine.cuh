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
  // Optional: the computed experts' outputs [Q, S, H] in the value dtype (the wrapper's
  // collected_expert_outputs, cached_layers.py:455-465): computed slots then add
  // w~ * computed[t, s, :] in slot order with the looked-up rows, so the call produces the
  // whole MoE combine (the reference's bmm of the renormalised weights).
  const void* computed;
  int64_t computed_stride_t, computed_stride_s;
};

constexpr int kCombineSpan = kCombineThreads * 8;
static_assert(kMaxSlots <= kCombineThreads, "one slot per thread in the combine prologue");

template <typename TV, typename TO, bool kVec>
__global__ void __launch_bounds__(kCombineThreads) k_combine(CombineArgs a) {
  __shared__ float s_w[kMaxSlots];
  __shared__ uint8_t s_surv[kMaxSlots];
  __shared__ uint8_t s_look[kMaxSlots];
  __shared__ const TV* s_off[kMaxSlots];
  __shared__ float s_wl[kMaxSlots];
  __shared__ const TV* s_offl[kMaxSlots];
  __shared__ int s_n;
  const int tid = threadIdx.x;
  const int t = blockIdx.x;
  ALUT_TRACE(20);
  pdl_launch_dependents();
  // Inputs first (they do not depend on the search), then wait for the search results.
  bool r_ = false, ev_ = false, comp_ = false;
  int64_t e_ = 0;
  float w_ = 0.f;
  const int m = a.is_vision[t] ? 0 : 1;
  if (tid < a.s) {
    r_ = a.reuse ? (a.reuse[t * a.reuse_stride + tid] != 0) : true;
    e_ = a.sel[t * a.sel_stride + tid];
    ev_ = e_ >= 0 && e_ < a.num_experts;
    comp_ = a.compute ? (a.compute[t * a.compute_stride + tid] != 0) : false;
    w_ = a.w[t * a.w_stride + tid];
  }
  ALUT_TRACE(21);
  pdl_wait();
  ALUT_TRACE(22);
  bool my_surv = false, my_look = false;  // this thread's slot (a.s <= kCombineThreads)
  const TV* my_off = nullptr;
  for (int s = tid; s < a.s; s += kCombineThreads) {
    const bool r = r_;
    const int64_t e = e_;
    const bool ev = ev_;
    bool hit = false;
    int64_t idx = 0;
    if (a.best) {
      if (r && ev) {
        const uint64_t b = a.best[static_cast<int64_t>(t) * a.s + s];
        if (b) {
          hit = hit_rule(cand_score(b), m == 0 ? a.thr_vis : a.thr_txt, a.cmp_ge);
          if (hit) idx = cand_index(b);
        }
      }
    } else {
      hit = r && a.hit_in[t * a.hit_stride + s] != 0;
      idx = a.idx_in[t * a.hit_stride + s];
    }
    if (a.out_hit && blockIdx.y == 0) {
      a.out_hit[t * a.out_hit_stride + s] = hit ? 1 : 0;
      a.out_idx[t * a.out_hit_stride + s] = hit ? idx : 0;
    }
    const bool comp = comp_;
    const bool look = hit && ev && idx >= 0 && idx < a.k;
    const bool add_comp = comp && !look && a.computed != nullptr;  // a hit row wins (cached_layers.py:452)
    my_surv = comp || hit;
    my_look = look || add_comp;
    my_off = add_comp ? static_cast<const TV*>(a.computed) + t * a.computed_stride_t + s * a.computed_stride_s
                      : static_cast<const TV*>(a.values) + (look ? (e * a.vs_e + m * a.vs_m + idx * a.vs_k) : 0);
    s_w[s] = w_;
    s_surv[s] = my_surv ? 1 : 0;
    s_look[s] = my_look ? 1 : 0;
    s_off[s] = my_off;
  }
  if (a.s <= 32) {
    // One warp: survivor and row sums by shuffles, the looked-up slots compacted in slot
    // order by a ballot prefix (the accumulation below keeps slot order).
    if (tid < 32) {
      float kept = my_surv ? w_ : 0.f, tot = w_;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        kept += __shfl_xor_sync(0xffffffffu, kept, o);
        tot += __shfl_xor_sync(0xffffffffu, tot, o);
      }
      const unsigned lm = __ballot_sync(0xffffffffu, my_look);
      if (my_look) {
        float w = w_;
        if (a.renorm == ALUT_RENORM_TO_ONE) w = kept > 0.f ? w / kept : 0.f;
        else if (a.renorm == ALUT_RENORM_TO_ROWSUM) w = kept > 0.f ? (w / kept) * tot : 0.f;
        const int pos = __popc(lm & ((1u << tid) - 1u));
        s_wl[pos] = w;
        s_offl[pos] = my_off;
      }
      if (tid == 0) s_n = __popc(lm);
    }
  } else {
    __syncthreads();
    if (tid == 0) {
      float kept = 0.f, tot = 0.f;
      for (int s = 0; s < a.s; ++s) {
        kept += s_surv[s] ? s_w[s] : 0.f;
        tot += s_w[s];
      }
      int n = 0;
      for (int s = 0; s < a.s; ++s) {
        if (!s_look[s]) continue;
        float w = s_w[s];
        if (a.renorm == ALUT_RENORM_TO_ONE) w = kept > 0.f ? w / kept : 0.f;
        else if (a.renorm == ALUT_RENORM_TO_ROWSUM) w = kept > 0.f ? (w / kept) * tot : 0.f;
        s_wl[n] = w;
        s_offl[n] = s_off[s];
        ++n;
      }
      s_n = n;
    }
  }
  __syncthreads();
  ALUT_TRACE(23);
  if (!a.out) return;
  const int n = s_n;
  const int64_t h0 = static_cast<int64_t>(blockIdx.y) * kCombineSpan + tid * 8;
  if (h0 >= a.h) return;
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
      for (int u = 0; u < 4; ++u) load8<TV>(s_offl[i + u] + h0, v[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = s_wl[i + u];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(w, v[u][j], acc[j]);
      }
    }
    for (; i < n; ++i) {
      float v[8];
      load8<TV>(s_offl[i] + h0, v);
      const float w = s_wl[i];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(w, v[j], acc[j]);
    }
    store8<TO>(out, acc);
    ALUT_TRACE(24);
  } else {
    const int64_t rem = a.h - h0;
    const int cnt = rem < 8 ? static_cast<int>(rem) : 8;
    for (int j = 0; j < cnt; ++j) acc[j] = a.accumulate ? to_f32<TO>(out[j]) : 0.f;
    for (int i = 0; i < n; ++i) {
      const float w = s_wl[i];
      for (int j = 0; j < cnt; ++j) acc[j] = fmaf(w, to_f32<TV>(s_offl[i][h0 + j]), acc[j]);
    }
    for (int j = 0; j < cnt; ++j) out[j] = from_f32<TO>(acc[j]);
  }
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

// Load-time key normalisation (manager.py:24-31 _normalize_last_dim, applied at :205-207):
// y = x / max(||x||, eps) in fp32, rows with ||x|| <= eps set to zero, rounded to the table
// dtype. One warp per row.
template <typename T>
__global__ void k_normalize_rows(int64_t rows, int l, const T* src, int64_t src_stride, T* dst, int64_t dst_stride,
                                 float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (r >= rows) return;
  const T* x = src + r * src_stride;
  float ss = 0.f;
  for (int c = lane; c < l; c += 32) {
    const float v = to_f32<T>(x[c]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float n = sqrtf(ss);
  const float denom = fmaxf(n, eps);
  const bool zero = n <= eps;
  T* y = dst + r * dst_stride;
  for (int c = lane; c < l; c += 32) y[c] = from_f32<T>(zero ? 0.f : to_f32<T>(x[c]) / denom);
}

}  // namespace alut
