// Tensor-core centroid scan for large batches (prefill, large tables): tcgen05.
//
// Scores of a tile of 128 searched slots x 128 centroids come from tcgen05.mma (kind::f16,
// bf16 operands, fp32 accumulator in tensor memory) of the bf16-rounded query and key:
//   |q.k - bf16(q).bf16(k)| <= (2 + 2^-9) 2^-9 |q| |k| + (fp32 accumulation) <= delta,
//   delta = (2^-8 + 2^-11) |q| max|k|       (Cauchy-Schwarz on the two rounding residues).
// The tensor cores therefore only choose candidates. Each epilogue thread (one slot) keeps
// the running maximum `amax` of its approximate scores and a short list of the centroids
// whose approximate score is >= amax - 2 delta; at the end of its slot's range of centroids
// the survivors are rescored exactly in fp32 (sequential fmaf over l, the summation order
// of the CUDA-core scans, so the scores are bit-identical to theirs) and folded into the
// slot's packed best with atomicMax. The true best always survives: its approximate score
// is within delta of its exact score, which is at least every other exact score. So the
// result is the exact fp32 argmax (first index on ties: tied centroids all survive), as on
// the CUDA-core paths. A full list is first pruned, then rescored on the spot.
//
// Layout: keys are prepared once (alut_prepare_keys) as bf16 128-row chunks in the K-major,
// no-swizzle core-matrix order of the tensor-core operand descriptors, followed by each
// table's largest row norm; the searched slots' queries are staged per search group in the
// same order (k_stage_queries). One TMA bulk copy then brings a whole operand tile.
//
// Pipeline (one CTA per SM, persistent over a contiguous range of (group, tile) pairs so
// that a group's query tile is loaded once and its key tiles stream in order; a tile is
// kTcCpt adjacent 128-row chunks, one MMA of N = 128 kTcCpt centroids):
//   warp 8 (producer): query tile -> A[2], a tile's chunks (one bulk copy) -> stage ring
//                 (mbarrier full/empty);
//   warp 9 (MMA): allocates all 512 TMEM columns, issues L/16 MMAs per tile into one of
//                 kTcAcc fp32 128 x N accumulators, commits to the stage's `empty`, the
//                 accumulator's `full` and, at a group's last tile, the query buffer's
//                 `empty` barrier;
//   warps 0-7 (epilogue): warp w reads TMEM lane quarter w % 4 (slots 32 (w % 4)..) over
//                 column half w / 4 of the tile, 64 columns per load, releases the
//                 accumulator after its last load, filters candidates and hands the
//                 survivors to the exact rescoring at the group's end.
// Every wait is bounded in time; on expiry the CTA records an error bit, stops all roles,
// drains what it has in flight (bounded), frees TMEM and returns.
#pragma once

#include "alut_common.cuh"
#include "alut_search.cuh"

namespace alut {

constexpr int kTcRows = 128;        // slots per tile (MMA M) and centroids per chunk (MMA N)
constexpr int kTcMaxL = 128;
// Epilogue warps 0 .. kTcEpiWarps-1: (TMEM lane quarter, column part); then the producer
// warp and the MMA warp.
#ifndef ALUT_TC_EPI_WARPS
#define ALUT_TC_EPI_WARPS 8
#endif
constexpr int kTcEpiWarps = ALUT_TC_EPI_WARPS;
static_assert(kTcEpiWarps == 8 || kTcEpiWarps == 16, "two or four column parts");
constexpr int kTcColParts = kTcEpiWarps / 4;
constexpr int kTcEpiThreads = 32 * kTcEpiWarps;
constexpr int kTcThreads = kTcEpiThreads + 64;
constexpr int kTcProducerWarp = kTcEpiWarps, kTcMmaWarp = kTcEpiWarps + 1;
#ifndef ALUT_TC_MIN_PAIRS
#define ALUT_TC_MIN_PAIRS 512
#endif
constexpr int kTcMinPairs = ALUT_TC_MIN_PAIRS;  // below this the CUDA-core scans are used
// ... and below this many slots per routed table on average (slots / min(tables, slots)):
// a 128 x 128 MMA tile whose group holds a few slots wastes the tensor cores, and the
// CUDA-core scans are faster there (measured on B200: 64 tokens x top-8 over 128 experts).
#ifndef ALUT_TC_MIN_SLOTS_PER_TABLE
#define ALUT_TC_MIN_SLOTS_PER_TABLE 12
#endif
constexpr int kTcMinSlotsPerTable = ALUT_TC_MIN_SLOTS_PER_TABLE;
inline bool tc_scan_wanted(int64_t slots, int num_tables) {
  const int64_t tables = slots < num_tables ? slots : num_tables;
  return slots >= kTcMinPairs && slots >= kTcMinSlotsPerTable * tables;
}
constexpr int kTcCand = 64 / kTcEpiWarps;  // candidate list per (slot, column part)
constexpr int kTcMaxStages = 8;
// 128-row key chunks per tile: one MMA covers N = 128 * kTcCpt centroids, so the query
// operand is read from shared memory once per kTcCpt chunks.
#ifndef ALUT_TC_CPT
#define ALUT_TC_CPT 2
#endif
constexpr int kTcCpt = ALUT_TC_CPT;
static_assert(kTcCpt == 1 || kTcCpt == 2, "MMA N of 128 or 256");
constexpr int kTcN = kTcRows * kTcCpt;              // centroids per tile (MMA N)
constexpr uint32_t kTcTmemCols = 512;               // all of tensor memory: one CTA per SM
constexpr int kTcAcc = kTcTmemCols / kTcN;          // fp32 128 x N accumulators (4 or 2)
constexpr size_t kTcSmemBudget = 212 * 1024;

// Byte offset of element (row, k) in a [rows][L] bf16 operand in the K-major, no-swizzle
// core-matrix order: 8-row x 16-byte core matrices, k-chunks adjacent (128 B apart), 8-row
// groups L*16 bytes apart.
__host__ __device__ __forceinline__ uint32_t tc_off(int r, int k, int L) {
  return static_cast<uint32_t>((r >> 3) * (L * 16) + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// 128-row chunks per table in the prepared key form: ceil(K / 128) rounded up to whole
// tiles. Rows past K are NaN: their scores are NaN, which max.f32 ignores and which no
// >= comparison accepts, so the scan needs no column mask.
__host__ __device__ inline int tc_prep_chunks(int k) {
  const int c = (k + kTcRows - 1) / kTcRows;
  return (c + kTcCpt - 1) / kTcCpt * kTcCpt;
}

// One operand tile: 128 rows x L bf16.
__host__ __device__ inline size_t tc_tile_bytes(int l) { return static_cast<size_t>(kTcRows) * l * 2; }
// Key stages of kTcCpt chunks each, in the shared memory left after the two query tiles
// and the candidate lists.
inline int tc_stages(int l) {
  const size_t t = tc_tile_bytes(l);
  const size_t n = (kTcSmemBudget - 1024 - 2 * t - sizeof(float) * 2 * kTcCand * kTcEpiThreads) / (kTcCpt * t);
  return static_cast<int>(n < kTcMaxStages ? n : kTcMaxStages);
}
inline size_t search_tc_smem_bytes(int l) {
  return 1024 + (2 + static_cast<size_t>(kTcCpt) * tc_stages(l)) * tc_tile_bytes(l) +
         sizeof(float) * 2 * kTcCand * kTcEpiThreads;
}
// Upper bound of the search groups of the tensor-core plan (groups of <= 128 slots of one table).
__host__ __device__ inline int64_t tc_max_groups(int64_t pairs, int ntab) {
  return (pairs + kTcRows - 1) / kTcRows + (pairs < ntab ? pairs : ntab) + 1;
}

// ---- preparation ---------------------------------------------------------------------------

// out: [tables][nchunks = tc_prep_chunks(K)][128 x L bf16 core-matrix order], then float
// norms[tables].
// One thread per (table, chunk, row, 8 columns): eight reads, one 16-byte store.
__global__ void k_prepare_keys(const float* keys, int64_t se, int64_t sm, int64_t sk, int ntab, int K, int L,
                               int nchunks, __nv_bfloat16* out, float* norms) {
  const int units = L / 8;
  const int64_t total = static_cast<int64_t>(ntab) * nchunks * kTcRows * units;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int u = static_cast<int>(i % units);
    const int64_t rowg = i / units;  // (table, chunk, row)
    const int r = static_cast<int>(rowg % kTcRows);
    const int64_t tcn = rowg / kTcRows;
    const int c = static_cast<int>(tcn % nchunks);
    const int t = static_cast<int>(tcn / nchunks);
    const int kr = c * kTcRows + r;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __int_as_float(0x7fc00000);  // NaN rows past K
    if (kr < K) {
      const float* src = keys + static_cast<int64_t>(t >> 1) * se + static_cast<int64_t>(t & 1) * sm +
                         static_cast<int64_t>(kr) * sk + u * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = src[j];
    }
    __align__(16) __nv_bfloat16 h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = __float2bfloat16_rn(v[j]);
    unsigned char* base = reinterpret_cast<unsigned char*>(out) + tcn * tc_tile_bytes(L);
    *reinterpret_cast<uint4*>(base + tc_off(r, u * 8, L)) = *reinterpret_cast<const uint4*>(h);
  }
  // Largest row norm per table: one thread per (table, row) partial, warp max, atomicMax on
  // the float bits (norms are >= 0, so their bit patterns order like the values; the output
  // norms are zeroed by the caller before the launch).
  const int64_t nrows = static_cast<int64_t>(ntab) * K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i - (threadIdx.x & 31) < nrows;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float nrm = 0.f;
    int t = 0;
    if (i < nrows) {
      t = static_cast<int>(i / K);
      const int kr = static_cast<int>(i % K);
      const float* row = keys + static_cast<int64_t>(t >> 1) * se + static_cast<int64_t>(t & 1) * sm +
                         static_cast<int64_t>(kr) * sk;
      float ss = 0.f;
      for (int k = 0; k < L; ++k) ss = fmaf(row[k], row[k], ss);
      nrm = sqrtf(ss);
    }
    // Lanes of a warp may straddle two tables: reduce per table id.
    const int t0 = __shfl_sync(0xffffffffu, t, 0);
    float m0 = t == t0 ? nrm : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    if ((threadIdx.x & 31) == 0 && i < nrows) atomicMax(reinterpret_cast<int*>(norms + t0), __float_as_int(m0));
    if (t != t0 && i < nrows) atomicMax(reinterpret_cast<int*>(norms + t), __float_as_int(nrm));
  }
}

// The searched slots' queries, per search group of the plan: [groups][128 x L bf16] in the
// operand order, plus each row's |q| (0 for the padding rows of a partial group).
// One thread per (group, row, 8 columns).
__global__ void k_stage_queries(const float* qlow, int L, int s, const int* sorted, const int4* groups,
                                const int* meta, int64_t max_groups, __nv_bfloat16* qsplit, float* qnorm) {
  const int units = L / 8;
  const int64_t ngroups = min(static_cast<int64_t>(meta[0]), max_groups);
  const int64_t total = ngroups * kTcRows * units;
  // When L / 8 is a power of two the threads of a row are an aligned group of adjacent lanes
  // and reduce the squared norm with shuffles; otherwise the row's first thread sums it.
  const bool pow2 = (units & (units - 1)) == 0;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x - (threadIdx.x & 31); i0 < total;
       i0 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = i0 + (threadIdx.x & 31);  // whole warps iterate together (shuffles)
    const bool live = i < total;
    const int u = static_cast<int>(i % units);
    const int r = static_cast<int>((i / units) % kTcRows);
    const int64_t g = i / (static_cast<int64_t>(units) * kTcRows);
    const float* qrow = nullptr;
    if (live) {
      const int4 gg = groups[g];
      const int p = r < gg.z ? sorted[gg.y + r] : -1;
      qrow = p >= 0 ? qlow + static_cast<int64_t>(p / s) * L : nullptr;
    }
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (qrow) {
      const float4 a = *reinterpret_cast<const float4*>(qrow + u * 8);
      const float4 b = *reinterpret_cast<const float4*>(qrow + u * 8 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    float ss = 0.f;
    __align__(16) __nv_bfloat16 h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[j] = __float2bfloat16_rn(v[j]);
      ss = fmaf(v[j], v[j], ss);
    }
    if (pow2) {
      for (int o = units >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    } else if (u == 0 && qrow) {
      ss = 0.f;
      for (int k = 0; k < L; ++k) ss = fmaf(qrow[k], qrow[k], ss);
    }
    if (live) {
      unsigned char* base = reinterpret_cast<unsigned char*>(qsplit) + g * tc_tile_bytes(L);
      *reinterpret_cast<uint4*>(base + tc_off(r, u * 8, L)) = *reinterpret_cast<const uint4*>(h);
      if (u == 0) qnorm[g * kTcRows + r] = sqrtf(ss);
    }
  }
}

// ---- tcgen05 primitives --------------------------------------------------------------------

__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, int L) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((128u >> 4) & 0x3FFF) << 16;                              // LBO: next k-chunk
  d |= static_cast<uint64_t>((static_cast<uint32_t>(L * 16) >> 4) & 0x3FFF) << 32;    // SBO: next 8 rows
  d |= static_cast<uint64_t>(1) << 46;                                                  // descriptor version
  return d;                                                                             // no swizzle
}
// kind::f16 instruction descriptor: fp32 D, bf16 A and B, both K-major, M = 128, N = kTcN.
__host__ __device__ __forceinline__ uint32_t tc_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTcN >> 3) << 17) |
         (static_cast<uint32_t>(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem),
      "l"(da), "l"(db), "r"(tc_idesc()), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
// Warp-collective (.aligned): every lane of the warp must execute it at the same call site.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 64 consecutive columns of this warp's 32 lanes in one load, waited for inside the same
// asm statement (the destination registers are defined only once the data has landed).
__device__ __forceinline__ void tc_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// An epilogue warp is done reading an accumulator (all its loads waited for): one arrival,
// after which the MMA warp may overwrite it.
__device__ __forceinline__ void tc_release(uint64_t* t_empty, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(t_empty);
}

// Bounded wait that also gives up when another role of the CTA has aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case: no timer read
  const uint64_t t0 = global_ns();
  for (uint32_t n = 0;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 15) == 15 && (*abort_flag || global_ns() - t0 > kWaitNs)) return false;
  }
}

// Exact fp32 score of one centroid row: sequential fmaf over l (the CUDA-core scans' order).
// L % 16 == 0: rows are read 32 values (8 float4 of each) at a time, all in flight before
// the dependent FMAs. Used by the in-kernel rescoring and by k_tc_rescore alike, so every
// candidate of a slot is scored by one arithmetic (exact duplicate rows tie to the lowest
// index).
__device__ __forceinline__ float tc_exact(const float* q, const float* kp, int L) {
  float e = 0.f;
  for (int l0 = 0; l0 < L; l0 += 32) {
    float4 a[8], b[8];
    const int nv = min(8, (L - l0) / 4);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < nv) {
        a[i] = *reinterpret_cast<const float4*>(q + l0 + 4 * i);
        b[i] = __ldg(reinterpret_cast<const float4*>(kp + l0 + 4 * i));
      }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < nv) {
        e = fmaf(b[i].x, a[i].x, e);
        e = fmaf(b[i].y, a[i].y, e);
        e = fmaf(b[i].z, a[i].z, e);
        e = fmaf(b[i].w, a[i].w, e);
      }
  }
  return e;
}

// L2 prefetch of a row of L fp32 values (whole 128-byte lines), so that a later exact
// rescoring of it finds it on chip.
__device__ __forceinline__ void tc_prefetch_row(const float* p, int L) {
  for (int o = 0; o < L; o += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + o));
}

// Packed exact candidate of centroid row kr (out of line: rare, and register-hungry).
__device__ __noinline__ unsigned long long tc_rescore(const float* q, const float* kt, int64_t sk, int L, int kr,
                                                      uint32_t idx_offset) {
  return pack_cand(tc_exact(q, kt + static_cast<int64_t>(kr) * sk, L), idx_offset + static_cast<uint32_t>(kr));
}

// A full candidate list (kTcCand entries of epilogue thread e in s_cc/s_cv, stride
// kTcEpiThreads): drop the entries that fell below thr; if none did, rescore them all into
// s_mine[e] and empty the list. Returns the new length. Kept out of line: the filter loop
// that calls it is unrolled, and this path is rare.
__device__ __noinline__ int tc_make_room(int e, float thr, const float* q, const float* kt, int64_t sk, int L,
                                         uint32_t idx_offset, int* s_cc, float* s_cv, unsigned long long* s_mine) {
  int m = 0;
  for (int i = 0; i < kTcCand; ++i)
    if (s_cv[i * kTcEpiThreads + e] >= thr) {
      s_cc[m * kTcEpiThreads + e] = s_cc[i * kTcEpiThreads + e];
      s_cv[m * kTcEpiThreads + e] = s_cv[i * kTcEpiThreads + e];
      ++m;
    }
  if (m < kTcCand) return m;
  unsigned long long mine = s_mine[e];
  for (int i = 0; i < kTcCand; ++i) {
    const unsigned long long c = tc_rescore(q, kt, sk, L, s_cc[i * kTcEpiThreads + e], idx_offset);
    mine = c > mine ? c : mine;
  }
  s_mine[e] = mine;
  return 0;
}

// Three-input maximum (sm_100 max.f32 with three operands; NaN handling as fmaxf).
__device__ __forceinline__ float tc_max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum of 32 values as a tree of three-input maxima: 17 operations (32 -> 11 -> 4 -> 2
// -> 1), all independent within a level.
__device__ __forceinline__ float tc_max32(const float (&v)[32]) {
  float m[11];
#pragma unroll
  for (int j = 0; j < 10; ++j) m[j] = tc_max3(v[3 * j], v[3 * j + 1], v[3 * j + 2]);
  m[10] = fmaxf(v[30], v[31]);
  const float n0 = tc_max3(m[0], m[1], m[2]), n1 = tc_max3(m[3], m[4], m[5]), n2 = tc_max3(m[6], m[7], m[8]),
              n3 = fmaxf(m[9], m[10]);
  return fmaxf(tc_max3(n0, n1, n2), n3);
}

// Bit j set where v[j] >= thr, built as a balanced tree of ORs (depth 5, not a chain of 32).
__device__ __forceinline__ uint32_t tc_mask32(const float (&v)[32], float thr) {
  uint32_t b[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) b[j] = (v[j] >= thr ? 1u : 0u) << j;
#pragma unroll
  for (int w = 16; w > 0; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) b[j] |= b[j + w];
  return b[0];
}

// The (group, tile) items a CTA walks over its range [t_begin, t_end) of group-major tile
// indices, in the same order in every role, without divisions; a segment is the CTA's part
// of one group.
struct TcWalk {
  int nt, glast, cend_last;
  int g, c, ce;  // group, tile, end of the segment
  __device__ __forceinline__ void begin(int t_begin, int t_end, int nt_) {
    nt = nt_;
    g = t_begin / nt;
    c = t_begin - g * nt;
    glast = (t_end - 1) / nt;
    cend_last = t_end - glast * nt;
    ce = g == glast ? cend_last : nt;
  }
  __device__ __forceinline__ bool done() const { return g > glast; }
  __device__ __forceinline__ bool segment_end() const { return c == ce - 1; }
  __device__ __forceinline__ void next() {
    if (++c == ce) {
      ++g;
      c = 0;
      ce = g == glast ? cend_last : nt;
    }
  }
};

// ---- scan ------------------------------------------------------------------------------------

struct TcArgs {
  const unsigned char* ksplit;  // prepared chunks
  const float* knorm;           // [tables] largest row norm
  const float* keys;            // fp32 keys for the exact rescoring
  int64_t key_stride_e, key_stride_m, key_stride_k;
  int k, l, s, nchunks, stages;
  uint32_t idx_offset;
  const float* qlow;
  const unsigned char* qsplit;  // [groups][128 x L bf16]
  const float* qnorm;           // [groups][128]
  const int* sorted;
  const int4* groups;
  const int* meta;
  uint64_t* best;
  int* err;
  int* cand_cnt;  // [pairs] candidates handed to k_tc_rescore (cleared by the plan)
  int* cand;      // [pairs][kTcCandGlobal] their rows (within this table)
};

#ifdef ALUT_PHASE_TRACE
// Development builds: per-thread SM-cycle sums kept in registers (slots 40..55), written once
// at the end by block 0's epilogue thread 0 (40 accumulator wait, 41 TMEM load, 42 group-end
// rescoring, 43 filter, 45 slow-path tiles, 46 list overflows, 48 rescored centroids, 53 the
// whole tile loop, 54 kernel entry to exit), MMA thread (50 stage wait, 51 accumulator wait)
// and producer thread (52 stage wait).
#define TC_TRACE_DECL unsigned long long tc_tr_[16] = {}
#define TC_T0() const long long tc_t0_ = clock64()
#define TC_ACC(slot) tc_tr_[(slot) - 40] += static_cast<unsigned long long>(clock64() - tc_t0_)
#define TC_COUNT() tc_tr_[8] += 1
#define TC_MARK(name) const long long name = clock64()
#define TC_SINCE(name, slot) tc_tr_[(slot) - 40] += static_cast<unsigned long long>(clock64() - name)
#define TC_T0_TID(t) TC_T0()
#define TC_ACC_TID(t, slot) TC_ACC(slot)
#define TC_INC_TID(t, slot) tc_tr_[(slot) - 40] += 1
#define TC_TRACE_FLUSH()                                                                       \
  if (blockIdx.x == 0 && (tid == 0 || tid == 32 * kTcProducerWarp || tid == 32 * kTcMmaWarp)) \
    for (int i = 0; i < 16; ++i)                                                               \
      if (tc_tr_[i]) g_alut_trace[40 + i] += tc_tr_[i]
#else
#define TC_TRACE_DECL do {} while (0)
#define TC_T0() do {} while (0)
#define TC_ACC(slot) do {} while (0)
#define TC_COUNT() do {} while (0)
#define TC_MARK(name) do {} while (0)
#define TC_SINCE(name, slot) do {} while (0)
#define TC_T0_TID(t) do {} while (0)
#define TC_ACC_TID(t, slot) do {} while (0)
#define TC_INC_TID(t, slot) do {} while (0)
#define TC_TRACE_FLUSH() do {} while (0)
#endif

__global__ void __launch_bounds__(kTcThreads, 1) k_search_tc(TcArgs a) {
  extern __shared__ __align__(1024) unsigned char tsm[];
  const int L = a.l;
  const int NS = a.stages;
  const uint32_t tb = static_cast<uint32_t>(tc_tile_bytes(L));
  uint64_t* full = reinterpret_cast<uint64_t*>(tsm);  // [kTcMaxStages]
  uint64_t* empty = full + kTcMaxStages;              // [kTcMaxStages]
  uint64_t* a_full = empty + kTcMaxStages;            // [2] query tiles
  uint64_t* a_empty = a_full + 2;                     // [2]
  uint64_t* t_full = a_empty + 2;                     // [kTcAcc] accumulators
  uint64_t* t_empty = t_full + kTcAcc;                // [kTcAcc]
  uint64_t* drain = t_empty + kTcAcc;                 // [1]
  unsigned char* sA = tsm + 1024;                     // [2][tile]
  unsigned char* sK = sA + 2 * tb;                    // [NS][kTcCpt tiles]
  int* s_cc = reinterpret_cast<int*>(sK + static_cast<size_t>(NS) * kTcCpt * tb);  // [kTcCand][kTcEpiThreads]
  float* s_cv = reinterpret_cast<float*>(s_cc + kTcCand * kTcEpiThreads);  // [kTcCand][kTcEpiThreads]
  __shared__ unsigned long long s_mine[kTcEpiThreads];  // best exactly rescored candidate
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_issued, s_groups_issued;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile int* abort_flag = &s_abort;
  TC_TRACE_DECL;
  TC_MARK(tc_entry_);

  const int nt = a.nchunks / kTcCpt;  // tiles per group (a.nchunks = tc_prep_chunks(K))
  const int ntiles = a.meta[0] * nt;
  const int t_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * ntiles / gridDim.x);
  const int t_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * ntiles / gridDim.x);
  if (t_begin >= t_end) return;
  if (warp == kTcMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < kTcMaxStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kTcAcc; ++i) {
      mbar_init(&t_full[i], 1);
      mbar_init(&t_empty[i], kTcEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
    s_issued = 0;
    s_groups_issued = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == kTcProducerWarp) {
    // ---- producer --------------------------------------------------------------------------
    if (lane == 0) {
      int gi = -1, prev = -1, it = 0, table = 0;
      int st = 0, wrapped = 0;  // stage, and its reuse parity
      bool ok = true;
      TcWalk wk;
      for (wk.begin(t_begin, t_end, nt); !wk.done() && ok; wk.next(), ++it) {
        const int g = wk.g, c = wk.c;
        if (g != prev) {
          table = a.groups[g].x;
          const int ab = (gi + 1) & 1;
          if (gi + 1 >= 2 && !tc_wait(&a_empty[ab], (((gi + 1) >> 1) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          prev = g;
          ++gi;
          mbar_expect_tx(&a_full[ab], tb);
          bulk_g2s(sA + ab * tb, a.qsplit + static_cast<int64_t>(g) * tb, tb, &a_full[ab]);
        }
        bool w;
        {
          TC_T0_TID(32 * kTcProducerWarp);
          w = it < NS || tc_wait(&empty[st], wrapped ^ 1, abort_flag);  // use it - NS done
          TC_ACC_TID(32 * kTcProducerWarp, 52);
        }
        if (!w) {
          ok = false;
          break;
        }
        // The tile's chunks are adjacent in the prepared form (whole tiles): one copy.
        const uint32_t kbytes = static_cast<uint32_t>(kTcCpt) * tb;
        mbar_expect_tx(&full[st], kbytes);
        bulk_g2s(sK + st * kTcCpt * tb, a.ksplit + (static_cast<int64_t>(table) * a.nchunks + c * kTcCpt) * tb, kbytes,
                 &full[st]);
        if (++st == NS) {
          st = 0;
          wrapped ^= 1;
        }
      }
      s_issued = it;
      s_groups_issued = gi + 1;
      if (!ok && !*abort_flag) {
        *abort_flag = 1;
        atomicOr(a.err, kErrMmaTimeout);
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ---- MMA issuer ------------------------------------------------------------------------
    if (lane == 0) {
      int gi = -1, prev = -1, it = 0;
      int st = 0, sph = 0;  // stage and the parity of its current use
      bool ok = true;
      TcWalk wk;
      for (wk.begin(t_begin, t_end, nt); !wk.done(); wk.next(), ++it) {
        const int g = wk.g;
        if (g != prev) {
          prev = g;
          ++gi;
          if (!tc_wait(&a_full[gi & 1], (gi >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
        }
        const int acc = it % kTcAcc;
        bool w1, w2;
        {
          TC_T0_TID(32 * kTcMmaWarp);
          w1 = tc_wait(&full[st], sph, abort_flag);
          TC_ACC_TID(32 * kTcMmaWarp, 50);
        }
        {
          TC_T0_TID(32 * kTcMmaWarp);
          w2 = w1 && (it < kTcAcc || tc_wait(&t_empty[acc], ((it / kTcAcc) - 1) & 1, abort_flag));
          TC_ACC_TID(32 * kTcMmaWarp, 51);
        }
        if (!w1 || !w2) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sA + (gi & 1) * tb), b0 = smem_addr(sK + st * kTcCpt * tb);
        const uint32_t d = tmem + static_cast<uint32_t>(acc * kTcN);
        if (L == 128) {
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) tc_mma(d, tc_desc(a0 + ks * 256, 128), tc_desc(b0 + ks * 256, 128), ks > 0);
        } else if (L == 64) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) tc_mma(d, tc_desc(a0 + ks * 256, 64), tc_desc(b0 + ks * 256, 64), ks > 0);
        } else {
          for (int ks = 0; ks < L / 16; ++ks) tc_mma(d, tc_desc(a0 + ks * 256, L), tc_desc(b0 + ks * 256, L), ks > 0);
        }
        tc_commit(&empty[st]);
        tc_commit(&t_full[acc]);
        if (wk.segment_end()) tc_commit(&a_empty[gi & 1]);
        if (++st == NS) {
          st = 0;
          sph ^= 1;
        }
      }
      if (!ok && !*abort_flag) {
        *abort_flag = 1;
        atomicOr(a.err, kErrMmaTimeout);
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. (slots) over the column part
    // w / 4 of the tile (centroids), 64 columns per load; thread e keeps the running maximum
    // and candidates of its (slot, part).
    const int e = tid;
    const int r = (warp & 3) * 32 + lane;
    const int half = warp >> 2;  // column part
    constexpr int kPartCols = kTcN / kTcColParts;
    constexpr int kSubs = kPartCols / 64;  // 64-column loads per tile
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    int prev = -1, p = -1, n = 0, it = 0;
    float amax = -INFINITY, tw = 0.f;
    const float* q = nullptr;
    const float* kt = nullptr;
    TC_MARK(tc_loop_);
    TcWalk wk;
    for (wk.begin(t_begin, t_end, nt); !wk.done(); wk.next(), ++it) {
      const int g = wk.g, c = wk.c;
      if (g != prev) {
        prev = g;
        const int4 gg = a.groups[g];
        const int table = gg.x;
        p = r < gg.z ? a.sorted[gg.y + r] : -1;
        n = 0;
        s_mine[e] = 0ull;
        amax = -INFINITY;
        if (p >= 0) {
          const float delta = (0x1p-8f + 0x1p-11f) * a.qnorm[static_cast<int64_t>(g) * kTcRows + r] * a.knorm[table];
          tw = 2.f * delta;
          q = a.qlow + static_cast<int64_t>(p / a.s) * L;
          kt = a.keys + static_cast<int64_t>(table >> 1) * a.key_stride_e +
               static_cast<int64_t>(table & 1) * a.key_stride_m;
          if (half == 0) tc_prefetch_row(q, L);
        }
      }
      const int acc = it % kTcAcc;
      bool ok;
      {
        TC_T0();
        ok = tc_wait(&t_full[acc], (it / kTcAcc) & 1, abort_flag);
        TC_ACC(40);
      }
      if (__any_sync(0xffffffffu, !ok)) {
        if (lane == 0 && !*abort_flag) {
          *abort_flag = 1;
          atomicOr(a.err, kErrMmaTimeout);
        }
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int sub = 0; sub < kSubs; ++sub) {
        float v[64];
        {
          TC_T0();
          __syncwarp();
          tc_ld64(lane_base + static_cast<uint32_t>(acc * kTcN + half * kPartCols + sub * 64), v);
          TC_ACC(41);
        }
        if (sub == kSubs - 1) tc_release(&t_empty[acc], lane);
        if (p < 0) continue;
        TC_T0();
        const float m0 = tc_max32(*reinterpret_cast<const float(*)[32]>(v)),
                    m1 = tc_max32(*reinterpret_cast<const float(*)[32]>(v + 32));
        // Columns past K (NaN) never qualify: a block of them has NaN maxima, and every
        // comparison with NaN is false, even while amax is still -inf.
        if (fmaxf(m0, m1) >= amax - tw) {  // rare once amax has settled
          TC_INC_TID(0, 45);
          amax = fmaxf(amax, fmaxf(m0, m1));
          const float thr = amax - tw;
          // Qualifying columns as bit masks, then one insertion per set bit - usually one.
          const uint64_t mk =
              (static_cast<uint64_t>(m1 >= thr ? tc_mask32(*reinterpret_cast<const float(*)[32]>(v + 32), thr) : 0u)
               << 32) |
              (m0 >= thr ? tc_mask32(*reinterpret_cast<const float(*)[32]>(v), thr) : 0u);
          // The stored value: with one qualifying column it is the block maximum itself; with
          // several, amax - an upper bound, so pruning never drops a column that could win.
          const float x = __popcll(static_cast<long long>(mk)) == 1 ? fmaxf(m0, m1) : amax;
          const int kb = c * kTcN + half * kPartCols + sub * 64;
          for (uint64_t m = mk; m; m &= m - 1) {
            const int j = __ffsll(static_cast<long long>(m)) - 1;
            if (n == kTcCand) {
              TC_INC_TID(0, 46);
              n = tc_make_room(e, thr, q, kt, a.key_stride_k, L, a.idx_offset, s_cc, s_cv, s_mine);
            }
            s_cc[n * kTcEpiThreads + e] = kb + j;
            s_cv[n * kTcEpiThreads + e] = x;
            ++n;
          }
        }
        TC_ACC(43);
      }
      if (p >= 0) {
        if (wk.segment_end()) {
          // End of this CTA's part of the group: the surviving candidates go to the rescoring
          // pass (k_tc_rescore) instead of being rescored here, where each one would hold
          // the accumulators for a dependent global load; a full list rescored here.
          TC_T0();
          unsigned long long mine = s_mine[e];
          for (int i = 0; i < n; ++i) {
            if (s_cv[i * kTcEpiThreads + e] < amax - tw) continue;
            const int pos = atomicAdd(a.cand_cnt + p, 1);
            if (pos < kTcCandGlobal) {
              a.cand[static_cast<int64_t>(p) * kTcCandGlobal + pos] = s_cc[i * kTcEpiThreads + e];
            } else {
              const unsigned long long cand =
                  tc_rescore(q, kt, a.key_stride_k, L, s_cc[i * kTcEpiThreads + e], a.idx_offset);
              TC_COUNT();
              mine = cand > mine ? cand : mine;
            }
          }
          n = 0;
          if (mine) atomicMax(reinterpret_cast<unsigned long long*>(a.best + p), mine);
          TC_ACC(42);
        }
      }
    }
    if (tid == 0) TC_SINCE(tc_loop_, 53);
  }

  __syncthreads();
  if (*abort_flag && tid == 32 * kTcMmaWarp) {
    // The MMAs this thread issued: a commit after them, waited (bounded).
    tc_commit(drain);
    mbar_wait_bounded(drain, 0);
  }
  if (*abort_flag && tid == 32 * kTcProducerWarp) {
    // Every copy this CTA issued: the latest use of each stage and query buffer (bounded).
    const int issued = s_issued, gissued = s_groups_issued;
    for (int st = 0; st < NS && st < issued; ++st) {
      const int last = st + ((issued - 1 - st) / NS) * NS;
      mbar_wait_bounded(&full[st], (last / NS) & 1);
    }
    for (int ab = 0; ab < 2 && ab < gissued; ++ab) {
      const int last = ab + ((gissued - 1 - ab) / 2) * 2;
      mbar_wait_bounded(&a_full[ab], (last >> 1) & 1);
    }
  }
  if (tid == 0) TC_SINCE(tc_entry_, 54);
  TC_TRACE_FLUSH();
  __syncthreads();
  if (warp == kTcMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

// The exact fp32 rescoring of the tensor-core scan's candidates: one thread per (slot,
// candidate) - 16 lanes per slot - each computing tc_exact, then the slot's maximum over its
// half-warp and one packed atomicMax, as the scan folds its own.
struct TcRescoreArgs {
  const float* keys;
  int64_t key_stride_e, key_stride_m, key_stride_k;
  int l, s, num_experts;
  int64_t pairs;
  uint32_t idx_offset;
  const float* qlow;
  const int64_t* sel;
  int64_t sel_stride;
  const uint8_t* is_vision;
  const int* cand_cnt;
  const int* cand;
  uint64_t* best;
};

static_assert(kTcCandGlobal == 16, "k_tc_rescore gives each slot a half-warp");

__global__ void __launch_bounds__(256) k_tc_rescore(TcRescoreArgs a) {
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t p = gt >> 4;  // slot
  const int i = static_cast<int>(gt & 15);
  unsigned long long c = 0ull;
  if (p < a.pairs) {
    const int n = min(a.cand_cnt[p], kTcCandGlobal);
    if (i < n) {
      const int64_t t = p / a.s;
      const int64_t e = a.sel[t * a.sel_stride + p % a.s];
      if (e >= 0 && e < a.num_experts) {
        const int table = static_cast<int>(e) * 2 + (a.is_vision[t] ? 0 : 1);
        const int kr = a.cand[p * kTcCandGlobal + i];
        const float* kp = a.keys + static_cast<int64_t>(table >> 1) * a.key_stride_e +
                          static_cast<int64_t>(table & 1) * a.key_stride_m + static_cast<int64_t>(kr) * a.key_stride_k;
        c = pack_cand(tc_exact(a.qlow + t * a.l, kp, a.l), a.idx_offset + static_cast<uint32_t>(kr));
      }
    }
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    const unsigned long long oc = __shfl_xor_sync(0xffffffffu, c, o);
    c = oc > c ? oc : c;
  }
  if (i == 0 && c) atomicMax(reinterpret_cast<unsigned long long*>(a.best + p), c);
}

}  // namespace alut
