// Shared helpers of the ALUT kernels: dtype conversion, rounding to the table dtype,
// the packed (score, index) candidate encoding and the workspace layout.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "alut.h"

namespace alut {

// Tokens per projection tile, centroids per search tile, query slots per search group.
constexpr int kProjTileQ = 16;
constexpr int kProjChunkH = 64;
constexpr int kProjThreads = 256;
constexpr int kMaxL = 256;               // L <= kMaxL (outputs per projection thread <= 16)
constexpr int kSearchThreads = 128;      // one centroid per thread
constexpr int kSearchChunkK = kSearchThreads;
constexpr int kSearchGroup = 32;         // (token, slot) pairs scored per search tile
// Slots per search group of the CUDA-core scans of large batches: kSearchGroup, or
// kCcSmallGroup when the batch would otherwise give fewer (group, chunk) tiles than SMs.
constexpr int kCcSmallGroup = 8;
// Candidate rows per slot the tensor-core scan hands to its exact rescoring pass.
constexpr int kTcCandGlobal = 16;
constexpr int kMaxTables = 4096;         // 2 * num_experts
constexpr int kMaxSlots = 64;            // top_k
constexpr int kCombineThreads = 64;      // 8 elements per thread -> 512 per CTA
constexpr int kProjSplitTarget = 296;    // 2 CTAs per SM over 148 SMs

// Error bits of the workspace's meta[1] word (ALUT_ERR_* in alut.h). Kernels only set them
// (atomicOr); they stay set until alut_workspace_errors clears them.
constexpr int kErrBadExpert = 1;    // a searched slot's expert id is outside [0, num_experts)
constexpr int kErrCopyTimeout = 4;  // a TMA / bulk copy did not land within the wait limit
constexpr int kErrMmaTimeout = 8;   // a tensor-core pipeline wait ran out

// ---- element conversion ---------------------------------------------------------

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// Round an fp32 value to the precision of T (round to nearest even) and widen it back.
// This is what a torch op whose output dtype is T does to an fp32-accumulated result.
template <typename T> __device__ __forceinline__ float round_as(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// Host-side version of round_as for the threshold (torch casts a Python float operand
// of a comparison to the tensor's dtype).
float host_round_as(float v, int dtype);

// Convert 8 consecutive elements starting at p (16-byte aligned for 16-bit types,
// 32-byte span for fp32) into fp32.
template <typename T> __device__ __forceinline__ void load8(const T* p, float (&o)[8]);
template <> __device__ __forceinline__ void load8<float>(const float* p, float (&o)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p));
  float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
  o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p,
                                                               float (&o)[8]) {
  uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&o)[8]) {
  uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}

template <typename T> __device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <> __device__ __forceinline__ void store8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
template <> __device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p,
                                                                const float (&v)[8]) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}
template <> __device__ __forceinline__ void store8<__half>(__half* p, const float (&v)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}

// Same as load8 but without the read-only path (for buffers the kernel also writes).
template <typename T> __device__ __forceinline__ void load8_rw(const T* p, float (&o)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = to_f32<T>(p[i]);
}

// ---- optional phase trace (development builds with -DALUT_PHASE_TRACE only) -----------
#ifdef ALUT_PHASE_TRACE
// Per slot: the earliest and the latest %globaltimer at which thread 0 of any CTA passed
// the trace point, plus a free value slot (CTA (0,0) only).
__device__ unsigned long long g_alut_trace[64];
__device__ unsigned long long g_alut_trace_lo[64];
__device__ unsigned long long g_alut_trace_hi[64];
#define ALUT_TRACE(slot)                                                              \
  do {                                                                                \
    if (threadIdx.x == 0) {                                                           \
      unsigned long long t_;                                                          \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                          \
      atomicMin(&g_alut_trace_lo[slot], t_);                                          \
      atomicMax(&g_alut_trace_hi[slot], t_);                                          \
    }                                                                                 \
  } while (0)
#define ALUT_TRACE_VAL(slot, v)                                                      \
  do {                                                                               \
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) g_alut_trace[slot] = (v); \
  } while (0)
#else
#define ALUT_TRACE_VAL(slot, v) \
  do {                          \
  } while (0)
#define ALUT_TRACE(slot) \
  do {                   \
  } while (0)
#endif

// ---- cp.async (16-byte global -> shared copies, waited per commit group) -----------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- programmatic dependent launch --------------------------------------------------------
// A kernel launched with the programmatic-stream-serialization attribute may start while
// its predecessor in the stream is still running; griddepcontrol.wait blocks until the
// predecessor has completed and its memory is visible (a no-op without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- packed candidates -------------------------------------------------------------
// A candidate (score, index) is packed into 64 bits so that unsigned max picks the
// larger score and, among equal scores, the smaller index (search.py:89 / torch.max).
// 0 is below every packed finite score and means "no candidate".

__host__ __device__ __forceinline__ uint32_t order_f32(float f) {
  uint32_t u;
#ifdef __CUDA_ARCH__
  u = __float_as_uint(f);
#else
  __builtin_memcpy(&u, &f, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float unorder_f32(uint32_t o) {
  uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  float f;
#ifdef __CUDA_ARCH__
  f = __uint_as_float(u);
#else
  __builtin_memcpy(&f, &u, 4);
#endif
  return f;
}
__host__ __device__ __forceinline__ uint64_t pack_cand(float score, uint32_t idx) {
  return (static_cast<uint64_t>(order_f32(score)) << 32) |
         static_cast<uint64_t>(0xFFFFFFFFu - idx);
}
__host__ __device__ __forceinline__ float cand_score(uint64_t p) {
  return unorder_f32(static_cast<uint32_t>(p >> 32));
}
__host__ __device__ __forceinline__ uint32_t cand_index(uint64_t p) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(p & 0xFFFFFFFFu);
}

// Hit rule applied to the best score of one slot (search.py:597 / :689).
__device__ __forceinline__ bool hit_rule(float score, float thr, int cmp_ge) {
  return cmp_ge ? (score >= thr) : (score > thr);
}

// ---- workspace layout ---------------------------------------------------------------
// All offsets are multiples of 256 bytes from the workspace base.
struct Workspace {
  size_t meta;      // int32  [8]            [0] search groups, [1] error bits
  size_t qlow;      // f32    [Q * L]        projected queries (already rounded to key dtype)
  size_t best;      // uint64 [Q * S]        packed best candidate per slot
  size_t sorted;    // int32  [Q * S]        slot ids sorted by table
  size_t groups;    // int4   [max_groups]   (table, first sorted slot, count, 0)
  size_t tabs;      // int32  [2 * tables]   per-table slot counts, bucket cursors (large plan)
  // Tensor-core scan only (workspace_layout(..., tc = true)): the searched slots' queries
  // staged per group of <= 128 slots as bf16 operand tiles, and their norms.
  size_t qsplit;    // bf16   [tc_groups][128 * L]
  size_t qnorm;     // f32    [tc_groups][128]
  size_t cand_cnt;  // int32  [Q * S]        candidates of each slot left for the rescoring pass
  size_t cand;      // int32  [Q * S][kTcCandGlobal] their centroid rows
  size_t total;
  int64_t max_groups;
  int64_t tc_groups;
};

__host__ __device__ inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Number of H splits of the projection for q tokens: a power of two <= kMaxClusterSplit
// (the split CTAs form one thread-block cluster) when the batch is small, so that a decode
// batch still spreads its projection over several SMs; 1 for large batches.
constexpr int kMaxClusterSplit = 16;  // a non-portable cluster size, allowed on sm_100
inline int proj_splits(int q, int h) {
  const int qtiles = ceil_div(q, kProjTileQ);
  int cap = kProjSplitTarget / (qtiles > 0 ? qtiles : 1);
  const int by_h = ceil_div(h, kProjChunkH);  // >= 1 chunk per split
  if (cap > by_h) cap = by_h;
  if (cap > kMaxClusterSplit) cap = kMaxClusterSplit;
  int s = 1;
  while (s * 2 <= cap) s *= 2;
  return s;
}

inline Workspace workspace_layout(int q, int s, int l, int num_tables, bool tc = false) {
  Workspace w{};
  const int64_t pairs = static_cast<int64_t>(q) * s;
  w.max_groups = (pairs + kCcSmallGroup - 1) / kCcSmallGroup + (pairs < num_tables ? pairs : num_tables) + 1;
  size_t off = 0;
  w.meta = off;     off = align256(off + sizeof(int32_t) * 8);
  w.qlow = off;     off = align256(off + sizeof(float) * (static_cast<int64_t>(q) * l + 8));
  w.best = off;     off = align256(off + sizeof(uint64_t) * (pairs + 1));
  w.sorted = off;   off = align256(off + sizeof(int32_t) * (pairs + 1));
  w.groups = off;   off = align256(off + sizeof(int4) * w.max_groups);
  w.tabs = off;     off = align256(off + sizeof(int32_t) * 2 * num_tables);
  if (tc) {
    // Groups of <= 128 slots of one table (this bound is below max_groups, which the plan's
    // group list uses in both cases).
    w.tc_groups = (pairs + 127) / 128 + (pairs < num_tables ? pairs : num_tables) + 1;
    w.qsplit = off; off = align256(off + static_cast<size_t>(w.tc_groups) * 128 * l * 2);
    w.qnorm = off;  off = align256(off + sizeof(float) * w.tc_groups * 128);
    w.cand_cnt = off; off = align256(off + sizeof(int32_t) * (pairs + 1));
    w.cand = off;   off = align256(off + sizeof(int32_t) * kTcCandGlobal * (pairs + 1));
  }
  w.total = off;
  return w;
}

}  // namespace alut
