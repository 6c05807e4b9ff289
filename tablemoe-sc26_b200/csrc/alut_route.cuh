// The router prologue of a TableMoE layer: top-k softmax over the router logits, then the
// keep mask that splits the routed slots into computed ones and looked-up ones.
//
// Semantics (reference project fanyalun/tablemoe-sc26):
//  * table_moe/ops/qwen_topk_softmax.py:122-153: probabilities = softmax(fp32 logits), the
//    top_k largest in descending order (weights, expert ids); with normalize_topk the
//    weights are divided by their sum clamped at 1e-20;
//  * table_moe/skip/pruning.py:4-15 build_fixed_keep_mask / :51 build_decode_keep_mask:
//    the first keep_k slots of every token are computed (keep_k clamped to [0, top_k];
//    "none" keeps every slot);
//  * table_moe/skip/pruning.py:18-48 build_prefill_keep_mask: per expert the sum of
//    (attn_score[t] * w[t,s]) or (w[t,s] / Q) over its slots; the activated experts (those
//    routed at least once) ranked by that sum, the first max(1, int(n_active * keep_rate))
//    kept; a slot is computed iff its expert is kept.
// The looked-up slots are the complement (cached_layers.py:336-337: search_mask =
// ~compute_mask), so the outputs feed alut_lookup_combine directly.
//
// Kernels:
//  * k_route_topk: one warp per token. The token's probabilities live in shared memory;
//    top_k rounds of a warp arg-max (largest value, lowest expert id on equal values) pick
//    the slots in descending order. Importance mode: each slot's score is added to its
//    expert's sum as a fixed-point integer (2^-40 units, 64-bit atomics), so the sums - and
//    with them the ranking - do not depend on the order of the additions.
//  * k_route_keep (importance mode only, one CTA): ranks the activated experts (larger
//    sum first, lower id on equal sums), marks the kept ones, writes the masks of every
//    slot and clears the sums for the next call.
#pragma once

#include "alut_common.cuh"

namespace alut {

constexpr int kRouteWarps = 4;                 // tokens per CTA of k_route_topk
constexpr int kRouteKeepThreads = 1024;
constexpr int kRouteMaxExperts = kMaxTables;   // probabilities of a token in shared memory
constexpr double kRouteFixedScale = 1099511627776.0;  // 2^40

struct RouteArgs {
  int q, e, k;
  const void* logits;
  int logits_dtype;
  int64_t logits_stride;
  int normalize;
  int mode;     // ALUT_KEEP_*
  int keep_k;   // fixed mode: slots [0, keep_k) computed
  double keep_rate;
  const float* attn;  // [Q] or NULL (importance mode)
  float* w;
  int64_t* sel;
  uint8_t* compute;
  uint8_t* reuse;
  int64_t out_stride;
  unsigned long long* sums;  // [E] fixed-point expert sums (importance mode; zero on entry)
  int* counts;               // [E] slots routed to each expert (importance mode; zero on entry)
};

__device__ __forceinline__ float logit_at(const RouteArgs& a, int64_t t, int j) {
  const int64_t o = t * a.logits_stride + j;
  if (a.logits_dtype == ALUT_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(a.logits)[o]);
  if (a.logits_dtype == ALUT_F16) return __half2float(static_cast<const __half*>(a.logits)[o]);
  return static_cast<const float*>(a.logits)[o];
}

__global__ void __launch_bounds__(kRouteWarps * 32) k_route_topk(RouteArgs a) {
  extern __shared__ float probs[];  // [kRouteWarps][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kRouteWarps + warp;
  if (t >= a.q) return;
  float* p = probs + static_cast<size_t>(warp) * a.e;
  float mx = -INFINITY;
  for (int j = lane; j < a.e; j += 32) {
    const float v = logit_at(a, t, j);
    p[j] = v;
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = lane; j < a.e; j += 32) {
    const float ex = expf(p[j] - mx);
    p[j] = ex;
    sum += ex;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  for (int j = lane; j < a.e; j += 32) p[j] = p[j] / sum;
  __syncwarp();
  // top_k rounds of arg-max; the chosen entry is retired with -1 (probabilities are >= 0).
  __shared__ float s_w[kRouteWarps][kMaxSlots];
  __shared__ int s_i[kRouteWarps][kMaxSlots];
  for (int s = 0; s < a.k; ++s) {
    float bv = -2.f;
    int bi = 0x7fffffff;
    for (int j = lane; j < a.e; j += 32) {
      const float v = p[j];
      if (v > bv) {  // ascending j per lane: the lane's first maximum is kept
        bv = v;
        bi = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      p[bi] = -1.f;
      s_w[warp][s] = bv;
      s_i[warp][s] = bi;
    }
    __syncwarp();
  }
  float tot = 0.f;
  if (a.normalize) {
    // Sum of the selected weights in slot order (the reference's weights.sum(dim=-1)),
    // clamped at 1e-20 (qwen_topk_softmax.py:151).
    for (int s = 0; s < a.k; ++s) tot += s_w[warp][s];
    tot = fmaxf(tot, 1e-20f);
  }
  for (int s = lane; s < a.k; s += 32) {
    float wv = s_w[warp][s];
    const int64_t e = s_i[warp][s];
    if (a.normalize) wv = wv / tot;
    a.w[t * a.out_stride + s] = wv;
    a.sel[t * a.out_stride + s] = e;
    if (a.mode == ALUT_KEEP_FIXED) {
      const bool comp = s < a.keep_k;
      a.compute[t * a.out_stride + s] = comp ? 1 : 0;
      a.reuse[t * a.out_stride + s] = comp ? 0 : 1;
    } else {
      // pruning.py:29-35: attn_scores[t] * w, else w / max(Q, 1) (fp32), summed per expert.
      const float score = a.attn ? a.attn[t] * wv : wv / static_cast<float>(max(a.q, 1));
      const long long fx = __double2ll_rn(static_cast<double>(score) * kRouteFixedScale);
      atomicAdd(&a.sums[e], static_cast<unsigned long long>(fx));
      atomicAdd(&a.counts[e], 1);
    }
  }
}

// Importance sums of given routing (alut_keep_mask): one thread per slot.
__global__ void k_route_scores(RouteArgs a) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(a.q) * a.k) return;
  const int64_t t = i / a.k;
  const int s = static_cast<int>(i % a.k);
  const int64_t e = a.sel[t * a.out_stride + s];
  if (e < 0 || e >= a.e) return;  // rejected by the keep kernel's range check below
  const float wv = a.w[t * a.out_stride + s];
  const float score = a.attn ? a.attn[t] * wv : wv / static_cast<float>(max(a.q, 1));
  atomicAdd(&a.sums[e], static_cast<unsigned long long>(__double2ll_rn(static_cast<double>(score) * kRouteFixedScale)));
  atomicAdd(&a.counts[e], 1);
}

__global__ void __launch_bounds__(kRouteKeepThreads) k_route_keep(RouteArgs a) {
  extern __shared__ unsigned char keep_smem[];
  long long* s_sum = reinterpret_cast<long long*>(keep_smem);                  // [E]
  int* s_act = reinterpret_cast<int*>(keep_smem + sizeof(long long) * a.e);    // [E] activated
  uint8_t* s_kept = reinterpret_cast<uint8_t*>(s_act + a.e);                   // [E]
  __shared__ int s_nact;
  const int tid = threadIdx.x;
  if (tid == 0) s_nact = 0;
  __syncthreads();
  int local = 0;
  for (int e = tid; e < a.e; e += kRouteKeepThreads) {
    s_sum[e] = static_cast<long long>(a.sums[e]);
    const int act = a.counts[e] > 0;
    s_act[e] = act;
    local += act;
    a.sums[e] = 0ull;  // ready for the next call
    a.counts[e] = 0;
  }
  atomicAdd(&s_nact, local);
  __syncthreads();
  const int nact = s_nact;
  // pruning.py:45-46, in double as Python computes it.
  int keep = static_cast<int>(static_cast<double>(nact) * a.keep_rate);
  keep = min(max(keep, 1), nact);
  for (int e = tid; e < a.e; e += kRouteKeepThreads) {
    uint8_t kept = 0;
    if (s_act[e]) {
      const long long v = s_sum[e];
      int rank = 0;
      for (int o = 0; o < a.e; ++o)
        rank += s_act[o] && (s_sum[o] > v || (s_sum[o] == v && o < e));
      kept = rank < keep;
    }
    s_kept[e] = kept;
  }
  __syncthreads();
  const int64_t n = static_cast<int64_t>(a.q) * a.k;
  for (int64_t i = tid; i < n; i += kRouteKeepThreads) {
    const int64_t t = i / a.k;
    const int s = static_cast<int>(i % a.k);
    const int64_t e = a.sel[t * a.out_stride + s];
    const bool comp = e >= 0 && e < a.e && s_kept[e] != 0;
    a.compute[t * a.out_stride + s] = comp ? 1 : 0;
    a.reuse[t * a.out_stride + s] = comp ? 0 : 1;
  }
}

}  // namespace alut
