// Tensor-core projection for large batches (prefill): q = x . P + b on tcgen05.
//
// x is bf16 (exact in the operand), P is the fp32 basis as three bf16 parts (hi + mid + lo
// == P to fp32 precision), so x.P is computed to fp32 accuracy as the sum of three bf16
// products per element, accumulated in fp32 in tensor memory (search.py:476-498,
// `_project_queries_into`: proj is applied in the key dtype, here fp32).
//
// Tile: 128 tokens (MMA M) x L columns (MMA N = L), K = H streamed in 64-column chunks.
//   A (tokens): one TMA tensor copy per stage (box 64 columns x 128 rows, 128-byte swizzle,
//       K-major: 8-row atoms of 1 KB), rows past Q filled with zeros by the copy.
//   B (basis): prepared once in core-matrix order per (modality, chunk) by
//       k_split_basis_tc; one TMA bulk copy per stage brings the three parts.
//   D: fp32 in tensor memory, [2 buffers][2 modalities][L columns]. A tile runs one MMA
//       pass per modality present among its tokens; the epilogue (warps 0-3, thread r =
//       token r, TMEM lane r) picks its token's modality, adds the bias, optionally
//       L2-normalises (search.py:12-21), and writes qlow (and the typed q_out copy).
//   warp 4 lane 0 issues both copies of a stage, warp 8 lane 0 the MMAs; barriers:
//   full/empty per stage, full/empty per accumulator buffer.
// Few token tiles (fewer than half the SMs): H is split over a thread-block cluster of
// ksplit CTAs per tile. Each runs the pipeline over its share of the 64-column stages and
// leaves its fp32 partial rows in its own shared memory; after a cluster barrier the
// leader sums the partials over distributed shared memory in rank order (deterministic)
// and finishes the rows; a second barrier keeps the peers' memory alive until then.
// Every wait is bounded in time (error bit, stop, bounded drain, TMEM freed).
#pragma once

#include <cuda.h>

#include <type_traits>

#include <cooperative_groups.h>

#include "alut_common.cuh"
#include "alut_project.cuh"
#include "alut_tc.cuh"

namespace alut {

constexpr int kPtKc = 64;          // K (H) columns per pipeline stage
constexpr int kPtThreads = 288;    // warps 0-3 epilogue, 4 copies, 8 MMA (5-7 idle)
constexpr int kPtMaxStages = 6;
#ifndef ALUT_PT_MIN_TOKENS
#define ALUT_PT_MIN_TOKENS 1024
#endif
constexpr int kPtMinTokens = ALUT_PT_MIN_TOKENS;  // below this the decode-shaped projections are used
constexpr size_t kPtSmemBudget = 200 * 1024;

inline bool pt_shape_ok(int l, int h) { return l > 0 && l % 16 == 0 && l <= kTcMaxL && h > 0 && h % kPtKc == 0; }
// One stage of the basis: three parts x L rows x 64 columns bf16.
__host__ __device__ inline size_t pt_b_stage_bytes(int l) { return static_cast<size_t>(3) * l * kPtKc * 2; }
__host__ __device__ inline size_t pt_a_stage_bytes() { return static_cast<size_t>(kTcRows) * kPtKc * 2; }
inline size_t pt_basis_bytes(int l, int h) { return static_cast<size_t>(2) * (h / kPtKc) * pt_b_stage_bytes(l); }
inline int pt_stages(int l) {
  const size_t st = pt_a_stage_bytes() + pt_b_stage_bytes(l);
  const size_t n = (kPtSmemBudget - 1024) / st;
  return static_cast<int>(n < kPtMaxStages ? n : kPtMaxStages);
}
inline size_t pt_smem_bytes(int l) {
  return 1024 + static_cast<size_t>(pt_stages(l)) * (pt_a_stage_bytes() + pt_b_stage_bytes(l));
}
__host__ __device__ inline uint32_t pt_tmem_cols(int l) {
  uint32_t n = 32;
  while (n < static_cast<uint32_t>(4 * l)) n <<= 1;
  return n;
}

// Basis in the operand order: [2 modalities][H/64 chunks][3 parts][L rows x 64 cols], each
// part in the K-major no-swizzle core-matrix order (tc_off with a 64-column extent).
__global__ void k_split_basis_tc(const float* proj0, const float* proj1, int64_t stride_h, int h, int l,
                                 __nv_bfloat16* out) {
  const int nkc = h / kPtKc;
  const int64_t n = static_cast<int64_t>(2) * l * h;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / (static_cast<int64_t>(l) * h));
    const int64_t r = i % (static_cast<int64_t>(l) * h);
    const int col = static_cast<int>(r % l), k = static_cast<int>(r / l);  // consecutive threads: columns
    const float p = (m == 0 ? proj0 : proj1)[static_cast<int64_t>(k) * stride_h + col];
    const __nv_bfloat16 hi = __float2bfloat16_rn(p);
    const float r1 = p - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    const int kc = k / kPtKc, kk = k % kPtKc;
    unsigned char* stage = reinterpret_cast<unsigned char*>(out) +
                           (static_cast<int64_t>(m) * nkc + kc) * pt_b_stage_bytes(l);
    const uint32_t off = tc_off(col, kk, kPtKc);
    const size_t part = static_cast<size_t>(l) * kPtKc * 2;
    *reinterpret_cast<__nv_bfloat16*>(stage + off) = hi;
    *reinterpret_cast<__nv_bfloat16*>(stage + part + off) = mid;
    *reinterpret_cast<__nv_bfloat16*>(stage + 2 * part + off) = lo;
  }
}

struct PtArgs {
  const __nv_bfloat16* x;
  int64_t x_stride;
  const uint8_t* is_vision;
  const unsigned char* basis;  // k_split_basis_tc layout
  const float* bias[2];
  int q, h, l, stages, normalize;
  int ksplit;  // CTAs per token tile (a cluster) splitting H; 1 = persistent CTAs over tiles
  float eps;
  float* qlow;
  float* q_out;  // optional fp32 copy with its own row stride
  int64_t q_out_stride;
  int* err;
};

// TMA map of the tokens x [Q][H] bf16 (row stride x_stride elements, a multiple of 8): box
// 64 columns x 128 rows, 128-byte swizzle, out-of-range rows read as zeros. Returns false if
// the driver cannot encode it.
inline bool pt_encode_x_map(CUtensorMap* map, const void* x, int64_t q, int64_t h, int64_t x_stride) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !fn)
      return false;
    encode = reinterpret_cast<Encode>(fn);
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(h), static_cast<cuuint64_t>(q)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(x_stride) * 2};
  const cuuint32_t box[2] = {kPtKc, kTcRows};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2D TMA tile load (no multicast): box at (x = column, y = row) of the map into smem.
__device__ __forceinline__ void pt_tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// kind::f16 instruction descriptor: fp32 D, bf16 A and B, K-major, M = 128, N = n.
__host__ __device__ __forceinline__ uint32_t pt_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kTcRows >> 4) << 24);
}
__device__ __forceinline__ uint64_t pt_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
// K-major operand with the 128-byte swizzle: 8-row atoms of 1 KB (SBO), rows of 128 B;
// within an atom the K offset is added to the start address.
__device__ __forceinline__ uint64_t pt_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;           // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // SBO: next 8-row atom
  d |= static_cast<uint64_t>(1) << 46;           // descriptor version
  d |= static_cast<uint64_t>(2) << 61;           // layout: 128-byte swizzle
  return d;
}
__device__ __forceinline__ void pt_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
// tcgen05.ld of W = 32 or 16 consecutive columns of this warp's 32 lanes (warp-collective).
template <int W>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[W]) {
  if constexpr (W == 32) {
    tc_ld32(taddr, v);
  } else {
    static_assert(W == 16, "16 or 32 columns");
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
  }
}

// Modalities present among the tokens of a tile: bit 0 vision, bit 1 text.
__device__ __forceinline__ int pt_tile_mods(const PtArgs& a, int tile) {
  const int t0 = tile * kTcRows, t1 = min(a.q, t0 + kTcRows);
  int mods = 0;
  for (int t = t0; t < t1 && mods != 3; ++t) mods |= a.is_vision[t] ? 1 : 2;
  return mods;
}

__global__ void __launch_bounds__(kPtThreads, 1) k_project_tc(const __grid_constant__ CUtensorMap x_map, PtArgs a) {
  extern __shared__ __align__(1024) unsigned char psm_tc[];
  const int L = a.l;
  const int NS = a.stages;
  const int nkc = a.h / kPtKc;
  const uint32_t a_bytes = static_cast<uint32_t>(pt_a_stage_bytes());
  const uint32_t b_bytes = static_cast<uint32_t>(pt_b_stage_bytes(L));
  const uint32_t part_bytes = b_bytes / 3;
  uint64_t* full = reinterpret_cast<uint64_t*>(psm_tc);  // [kPtMaxStages]
  uint64_t* empty = full + kPtMaxStages;                 // [kPtMaxStages]
  uint64_t* t_full = empty + kPtMaxStages;               // [2]
  uint64_t* t_empty = t_full + 2;                        // [2]
  uint64_t* drain = t_empty + 2;                         // [1]
  unsigned char* stages = psm_tc + 1024;                 // [NS][A | B]
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_issued;
  volatile int* abort_flag = &s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = (a.q + kTcRows - 1) / kTcRows;
  const bool split = a.ksplit > 1;
  // Tiles this CTA runs (tile0, tile0 + tstep, ...) and its stages [kc0, kc1) of each.
  const int rank = split ? static_cast<int>(blockIdx.x) % a.ksplit : 0;
  const int tile0 = split ? static_cast<int>(blockIdx.x) / a.ksplit : static_cast<int>(blockIdx.x);
  const int tstep = split ? ntiles : static_cast<int>(gridDim.x);
  const int kc0 = split ? rank * nkc / a.ksplit : 0;
  const int kc1 = split ? (rank + 1) * nkc / a.ksplit : nkc;
  if (!split && tile0 >= ntiles) return;  // (split grids are exactly ntiles x ksplit)
  const uint32_t ncols = pt_tmem_cols(L);
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < kPtMaxStages; ++i) {
      mbar_init(&full[i], 1);  // the producer's expect_tx; both copies complete the bytes
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], 4);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_issued = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 4) {
    // ---- producer: token tile (TMA tensor copy) + basis parts (bulk copy) per stage --------
    if (lane == 0) {
      int it = 0, st = 0, wrapped = 0;  // stage and the parity of its reuse, without divisions
      bool ok = true;
      for (int tile = tile0; tile < ntiles && ok; tile += tstep) {
        const int mods = pt_tile_mods(a, tile);
        for (int m = 0; m < 2 && ok; ++m) {
          if (!(mods & (1 << m))) continue;
          for (int kc = kc0; kc < kc1; ++kc, ++it, (++st == NS ? (st = 0, wrapped ^= 1) : 0)) {
            if (it >= NS && !tc_wait(&empty[st], wrapped ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            unsigned char* sa = stages + static_cast<size_t>(st) * (a_bytes + b_bytes);
            mbar_expect_tx(&full[st], a_bytes + b_bytes);
            pt_tma_load_2d(sa, &x_map, kc * kPtKc, tile * kTcRows, &full[st]);
            bulk_g2s(sa + a_bytes, a.basis + (static_cast<int64_t>(m) * nkc + kc) * b_bytes, b_bytes, &full[st]);
          }
        }
      }
      s_issued = it;
      if (!ok && !*abort_flag) {
        *abort_flag = 1;
        atomicOr(a.err, kErrMmaTimeout);
      }
    }
  } else if (warp == 8) {
    // ---- MMA issuer ------------------------------------------------------------------------
    if (lane == 0) {
      int it = 0, tc = 0, st = 0, sph = 0;
      bool ok = true;
      const uint32_t idesc = pt_idesc(L);
      for (int tile = tile0; tile < ntiles && ok; tile += tstep, ++tc) {
        const int mods = pt_tile_mods(a, tile);
        const int buf = tc & 1;
        if (tc >= 2 && !tc_wait(&t_empty[buf], ((tc >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int m = 0; m < 2 && ok; ++m) {
          if (!(mods & (1 << m))) continue;
          const uint32_t d = tmem + static_cast<uint32_t>((buf * 2 + m) * L);
          for (int kc = kc0; kc < kc1; ++kc, ++it, (++st == NS ? (st = 0, sph ^= 1) : 0)) {
            if (!tc_wait(&full[st], sph, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_addr(stages + static_cast<size_t>(st) * (a_bytes + b_bytes));
            const uint32_t sb = sa + a_bytes;
            for (int k16 = 0; k16 < kPtKc / 16; ++k16) {
              const uint64_t da = pt_desc_sw128(sa + k16 * 32);
#pragma unroll
              for (int part = 0; part < 3; ++part) {
                const uint64_t db = pt_desc(sb + part * part_bytes + k16 * 256, 128, kPtKc * 16);
                pt_mma(d, da, db, idesc, (kc != kc0 || k16 != 0 || part != 0) ? 1u : 0u);
              }
            }
            tc_commit(&empty[st]);
          }
        }
        if (ok) tc_commit(&t_full[buf]);
      }
      if (!ok && !*abort_flag) {
        *abort_flag = 1;
        atomicOr(a.err, kErrMmaTimeout);
      }
    }
  } else if (warp < 4) {
    // ---- epilogue: thread r = token r of the tile --------------------------------------------
    const int r = tid;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    int tc = 0;
    for (int tile = tile0; tile < ntiles; tile += tstep, ++tc) {
      const int mods = pt_tile_mods(a, tile);
      const int buf = tc & 1;
      const bool ok = tc_wait(&t_full[buf], (tc >> 1) & 1, abort_flag);
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0 && !*abort_flag) {
          *abort_flag = 1;
          atomicOr(a.err, kErrMmaTimeout);
        }
        break;
      }
      tc_fence_after();
      const int tok = tile * kTcRows + r;
      const bool valid = tok < a.q;
      const int mr = valid && !a.is_vision[tok] ? 1 : 0;
      // Section of this lane's modality; when both are present every lane loads both.
      const int m_only = mods == 2 ? 1 : 0;
      if (split) {  // this CTA's share of H: park the row's partial sums for the leader
        float* part = reinterpret_cast<float*>(stages) + static_cast<size_t>(r) * (L + 4);
        for (int c0 = 0; c0 < L; c0 += 16) {
          float v[16];
          __syncwarp();
          tc_ld<16>(lane_base + static_cast<uint32_t>((buf * 2 + m_only) * L + c0), v);
          if (mods == 3) {
            float w[16];
            tc_ld<16>(lane_base + static_cast<uint32_t>((buf * 2 + 1) * L + c0), w);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = mr ? w[j] : v[j];
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
            reinterpret_cast<float4*>(part + c0)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&t_empty[buf]);
        continue;
      }
      const float* bias = a.bias[valid ? mr : m_only];
      float denom = 1.f;
      bool zero = false;
      for (int pass = a.normalize ? 0 : 1; pass < 2; ++pass) {
        float ss = 0.f;
        // 32-column chunks, then a 16-column tail (L % 16 == 0).
        auto chunk = [&](auto width_tag, int c0) {
          constexpr int W = decltype(width_tag)::value;
          float v[W];
          __syncwarp();
          tc_ld<W>(lane_base + static_cast<uint32_t>((buf * 2 + m_only) * L + c0), v);
          if (mods == 3) {
            float w[W];
            tc_ld<W>(lane_base + static_cast<uint32_t>((buf * 2 + 1) * L + c0), w);
#pragma unroll
            for (int j = 0; j < W; ++j) v[j] = mr ? w[j] : v[j];
          }
#pragma unroll
          for (int j = 0; j < W; ++j) v[j] += __ldg(bias + c0 + j);
          if (pass == 0) {
#pragma unroll
            for (int j = 0; j < W; ++j) ss = fmaf(v[j], v[j], ss);
          } else if (valid) {
            if (a.normalize) {
#pragma unroll
              for (int j = 0; j < W; ++j) v[j] = zero ? 0.f : v[j] / denom;
            }
            float4* dst = reinterpret_cast<float4*>(a.qlow + static_cast<int64_t>(tok) * L + c0);
#pragma unroll
            for (int j = 0; j < W / 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            if (a.q_out) {
              float* o = a.q_out + static_cast<int64_t>(tok) * a.q_out_stride + c0;
#pragma unroll
              for (int j = 0; j < W; ++j) o[j] = v[j];
            }
          }
        };
        int c0 = 0;
        for (; c0 + 32 <= L; c0 += 32) chunk(std::integral_constant<int, 32>{}, c0);
        if (c0 < L) chunk(std::integral_constant<int, 16>{}, c0);
        if (pass == 0) {
          const float n = sqrtf(ss);
          denom = fmaxf(n, a.eps);
          zero = n <= a.eps;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[buf]);
    }
  }

  __syncthreads();
  if (split) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every rank's partial rows are in its shared memory
    if (rank == 0 && tid < kTcRows) {
      const int r = tid;
      const int tok = tile0 * kTcRows + r;
      if (tok < a.q) {
        const int mr = a.is_vision[tok] ? 0 : 1;
        const float* bias = a.bias[mr];
        float denom = 1.f;
        bool zero = false;
        for (int pass = a.normalize ? 0 : 1; pass < 2; ++pass) {
          float ss = 0.f;
          for (int c0 = 0; c0 < L; c0 += 16) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0.f;
            for (int k = 0; k < a.ksplit; ++k) {  // rank order: the same sum on every run
              const float* pk = cluster.map_shared_rank(reinterpret_cast<float*>(stages), k) +
                                static_cast<size_t>(r) * (L + 4) + c0;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 f = reinterpret_cast<const float4*>(pk)[j];
                v[4 * j] += f.x;
                v[4 * j + 1] += f.y;
                v[4 * j + 2] += f.z;
                v[4 * j + 3] += f.w;
              }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += __ldg(bias + c0 + j);
            if (pass == 0) {
#pragma unroll
              for (int j = 0; j < 16; ++j) ss = fmaf(v[j], v[j], ss);
            } else {
              if (a.normalize) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = zero ? 0.f : v[j] / denom;
              }
              float4* dst = reinterpret_cast<float4*>(a.qlow + static_cast<int64_t>(tok) * L + c0);
#pragma unroll
              for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
              if (a.q_out) {
                float* o = a.q_out + static_cast<int64_t>(tok) * a.q_out_stride + c0;
#pragma unroll
                for (int j = 0; j < 16; ++j) o[j] = v[j];
              }
            }
          }
          if (pass == 0) {
            const float n = sqrtf(ss);
            denom = fmaxf(n, a.eps);
            zero = n <= a.eps;
          }
        }
      }
    }
    cluster.sync();  // the leader has read every rank's partials
  }
  if (*abort_flag && tid == 32 * 8) {
    tc_commit(drain);
    mbar_wait_bounded(drain, 0);
  }
  if (*abort_flag && tid == 128) {
    const int issued = s_issued;  // copies: the latest use of each stage
    for (int st = 0; st < NS && st < issued; ++st) {
      const int last = st + ((issued - 1 - st) / NS) * NS;
      mbar_wait_bounded(&full[st], (last / NS) & 1);
    }
  }
  __syncthreads();
  if (warp == 8)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
}

}  // namespace alut
