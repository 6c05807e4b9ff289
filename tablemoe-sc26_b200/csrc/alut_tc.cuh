// Tensor-core centroid scan for large batches (prefill, large tables): tcgen05.
//
// Scores of a tile of 128 queries x 128 centroids come from tcgen05.mma (kind::f16, bf16
// operands, fp32 accumulator in tensor memory) over a two-part bf16 split of both operands:
//   q . k  ~=  q_hi . k_hi + q_hi . k_lo + q_lo . k_hi      (q_lo = bf16(q - q_hi), same for k)
// whose error is below delta = 2^-13 |q| max|k| (the split leaves ~2^-16 relative per
// product; the bound keeps a wide safety factor). The tensor cores therefore only choose
// candidates: every centroid whose approximate score is within 2*delta of the larger of the
// tile's approximate best and the slot's current exact best is rescored exactly in fp32 on
// the CUDA cores and folded into the slot's packed best with atomicMax. The true best always
// survives the filter (its approximate score is within delta of its exact score, which is
// at least every other exact score), so the result is the exact fp32 argmax (first index on
// ties), as on the CUDA-core paths.
//
// Keys are prepared once (alut_prepare_keys): each table's 128-row chunks as the two bf16
// parts in the K-major core-matrix order of the tensor-core operand descriptors, so one TMA
// bulk copy brings a chunk's operand into shared memory; queries are split while being
// staged. One CTA per SM (persistent over a contiguous range of tiles so that a group's
// queries are staged once), 128 threads: thread r owns TMEM lane r = query row r.
#pragma once

#include "alut_common.cuh"
#include "alut_search.cuh"

namespace alut {

constexpr int kTcRows = 128;   // queries per tile (MMA M) and centroids per chunk (MMA N)
constexpr int kTcMaxL = 128;
constexpr int kTcThreads = 128;
constexpr int kTcMinPairs = 512;  // below this the CUDA-core scans are used

// Byte offset of element (row, k) in a [rows][L] bf16 operand in the K-major, no-swizzle
// core-matrix order: 8-row x 16-byte core matrices, k-chunks adjacent (128 B apart), 8-row
// groups L*16 bytes apart.
__host__ __device__ __forceinline__ uint32_t tc_off(int r, int k, int L) {
  return static_cast<uint32_t>((r >> 3) * (L * 16) + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

__host__ __device__ inline size_t tc_chunk_bytes(int l) { return static_cast<size_t>(2) * kTcRows * l * 2; }

// ---- preparation ---------------------------------------------------------------------------

// out: [tables][nchunks][2 parts][128 x L bf16 core-matrix order], then float norms[tables].
__global__ void k_prepare_keys(const float* keys, int64_t se, int64_t sm, int64_t sk, int ntab, int K, int L,
                               int nchunks, __nv_bfloat16* out, float* norms) {
  const int64_t per_chunk = static_cast<int64_t>(2) * kTcRows * L;
  const int64_t total = static_cast<int64_t>(ntab) * nchunks * kTcRows * L;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % L);
    const int64_t rowg = i / L;  // (table, chunk, row)
    const int r = static_cast<int>(rowg % kTcRows);
    const int64_t tc = rowg / kTcRows;
    const int c = static_cast<int>(tc % nchunks);
    const int t = static_cast<int>(tc / nchunks);
    const int kr = c * kTcRows + r;
    float v = 0.f;
    if (kr < K) v = keys[static_cast<int64_t>(t >> 1) * se + static_cast<int64_t>(t & 1) * sm + kr * sk + k];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16* base = out + tc * per_chunk;
    const uint32_t off = tc_off(r, k, L) / 2;
    base[off] = hi;
    base[static_cast<int64_t>(kTcRows) * L + off] = lo;
  }
  // Largest row norm per table (one warp per table, grid-stride).
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int t = gw; t < ntab; t += nw) {
    float mx = 0.f;
    const float* tb = keys + static_cast<int64_t>(t >> 1) * se + static_cast<int64_t>(t & 1) * sm;
    for (int kr = lane; kr < K; kr += 32) {
      float ss = 0.f;
      for (int k = 0; k < L; ++k) ss = fmaf(tb[kr * sk + k], tb[kr * sk + k], ss);
      mx = fmaxf(mx, sqrtf(ss));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) norms[t] = mx;
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
// kind::f16 instruction descriptor: fp32 D, bf16 A and B, both K-major, M = N = 128.
__host__ __device__ __forceinline__ uint32_t tc_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(kTcRows >> 3) << 17) |
         (static_cast<uint32_t>(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t da, uint64_t db, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem),
      "l"(da), "l"(db), "r"(tc_idesc()), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- scan ------------------------------------------------------------------------------------

struct TcArgs {
  const unsigned char* ksplit;  // prepared chunks
  const float* knorm;           // [tables] largest row norm
  const float* keys;            // fp32 keys for the exact rescoring
  int64_t key_stride_e, key_stride_m, key_stride_k;
  int k, l, s, nchunks;
  uint32_t idx_offset;
  const float* qlow;
  const int* sorted;
  const int4* groups;
  const int* meta;
  uint64_t* best;
  int* err;
};

inline size_t search_tc_smem_bytes(int l) { return 1024 + 3 * tc_chunk_bytes(l); }  // A + 2 x B

__global__ void __launch_bounds__(kTcThreads, 1) k_search_tc(TcArgs a) {
  extern __shared__ __align__(1024) unsigned char tsm[];
  const int L = a.l;
  const size_t cb = tc_chunk_bytes(L);
  unsigned char* sA = tsm + 1024;                         // [2 parts][128 x L] queries
  unsigned char* sB = sA + cb;                            // [2 buffers][2 parts][128 x L] keys
  uint64_t* bar = reinterpret_cast<uint64_t*>(tsm);       // [0],[1] key buffers, [2] MMA done
  __shared__ uint32_t s_tmem;
  __shared__ int pid[kTcRows];
  __shared__ float s_qn[kTcRows];
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int ntiles = a.meta[0] * a.nchunks;
  const int t_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * ntiles / gridDim.x);
  const int t_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * ntiles / gridDim.x);
  if (t_begin >= t_end) return;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(kTcRows)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  auto issue_b = [&](int tile, int b) {  // thread 0
    const int4 g = a.groups[tile / a.nchunks];
    const int chunk = tile % a.nchunks;
    const unsigned char* src = a.ksplit + (static_cast<int64_t>(g.x) * a.nchunks + chunk) * cb;
    fence_async_shared();
    mbar_expect_tx(&bar[b], static_cast<uint32_t>(cb));
    bulk_g2s(sB + b * cb, src, static_cast<uint32_t>(cb), &bar[b]);
  };
  if (tid == 0) issue_b(t_begin, 0);
  int cur_group = -1, table = 0, cnt = 0;
  float qn = 0.f;
  int it = 0;
  for (int tile = t_begin; tile < t_end; ++tile, ++it) {
    const int b = it & 1;
    const int g = tile / a.nchunks, chunk = tile % a.nchunks;
    if (tid == 0 && tile + 1 < t_end) issue_b(tile + 1, b ^ 1);  // that buffer's MMAs finished last iteration
    if (g != cur_group) {
      const int4 gg = a.groups[g];
      table = gg.x;
      cnt = gg.z;
      cur_group = g;
      // Stage the group's queries: thread r splits query r into (hi, lo) bf16 parts.
      const int r = tid;
      float ss = 0.f;
      int p = -1;
      if (r < cnt) p = a.sorted[gg.y + r];
      pid[r] = p;
      const float* q = p >= 0 ? a.qlow + static_cast<int64_t>(p / a.s) * L : nullptr;
      for (int k = 0; k < L; ++k) {
        const float v = q ? q[k] : 0.f;
        ss = fmaf(v, v, ss);
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        const uint32_t off = tc_off(r, k, L);
        *reinterpret_cast<__nv_bfloat16*>(sA + off) = hi;
        *reinterpret_cast<__nv_bfloat16*>(sA + cb / 2 + off) = lo;
      }
      s_qn[r] = sqrtf(ss);
      qn = s_qn[r];
      fence_async_shared();  // generic-proxy writes of A, visible to the tensor cores
    }
    if (tid == 0 && !mbar_wait_bounded(&bar[b], (it >> 1) & 1)) {
      s_abort = 1;  // keys of this tile (and the next, if issued) may still be in flight
      atomicOr(a.err, 8);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (s_abort) break;
    if (tid == 0) {
      const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB + b * cb);
      const uint32_t half = static_cast<uint32_t>(cb / 2);
      int n = 0;
      for (int ks = 0; ks < L / 16; ++ks) {
        const uint32_t o = ks * 256;
        tc_mma(tmem, tc_desc(a0 + o, L), tc_desc(b0 + o, L), n++ > 0);                // hi . hi
        tc_mma(tmem, tc_desc(a0 + o, L), tc_desc(b0 + half + o, L), 1);               // hi . lo
        tc_mma(tmem, tc_desc(a0 + half + o, L), tc_desc(b0 + o, L), 1);               // lo . hi
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_addr(&bar[2]))
                   : "memory");
      if (!mbar_wait_bounded(&bar[2], it & 1)) {
        s_abort = 2;  // the MMAs of this tile may still be running
        atomicOr(a.err, 8);
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (s_abort) break;
    // Epilogue: thread r = query r of the group. tcgen05.ld is warp-collective (.aligned):
    // every load is issued from one call site by the whole, re-converged warp.
    const int r = tid;
    const int rows = min(kTcRows, a.k - chunk * kTcRows);
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m = -INFINITY;
    for (int c0 = 0; c0 < kTcRows; c0 += 32) {
      float v[32];
      __syncwarp();
      tc_ld32(taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < rows) m = fmaxf(m, v[j]);
    }
    const int p = pid[r];
    float thr = INFINITY;
    const float* q = nullptr;
    const float* kt = nullptr;
    if (p >= 0) {
      const uint64_t gb = __ldcg(reinterpret_cast<const unsigned long long*>(a.best) + p);
      const float gs = gb ? cand_score(gb) : -INFINITY;
      const float delta = 0x1p-13f * qn * a.knorm[table];
      thr = fmaxf(m, gs) - 2.f * delta;
      q = a.qlow + static_cast<int64_t>(p / a.s) * L;
      kt = a.keys + static_cast<int64_t>(table >> 1) * a.key_stride_e + static_cast<int64_t>(table & 1) * a.key_stride_m;
    }
    uint64_t mine = 0ull;
    for (int c0 = 0; c0 < kTcRows; c0 += 32) {
      float v[32];
      __syncwarp();
      tc_ld32(taddr + c0, v);
      if (p < 0) continue;
#pragma unroll 1
      for (int j = 0; j < 32; ++j) {
        const int col = c0 + j;
        if (col < rows && v[j] >= thr) {
          const int kr = chunk * kTcRows + col;
          const float* kp = kt + static_cast<int64_t>(kr) * a.key_stride_k;
          float e = 0.f;
          for (int l = 0; l < L; ++l) e = fmaf(q[l], kp[l], e);
          const uint64_t c = pack_cand(e, a.idx_offset + static_cast<uint32_t>(kr));
          mine = c > mine ? c : mine;
        }
      }
    }
    if (mine) atomicMax(reinterpret_cast<unsigned long long*>(a.best + p), static_cast<unsigned long long>(mine));
    __syncwarp();
    tc_fence_before();
    __syncthreads();  // TMEM, A and this key buffer are free again
    tc_fence_after();
  }
  // After an abort at iteration `it`, give what this CTA still has in flight (the MMAs, this
  // tile's key copy, the next tile's key copy) a bounded chance to finish before TMEM is freed.
  if (s_abort && tid == 0) {
    const int tile = t_begin + it;
    if (s_abort == 2) mbar_wait_bounded(&bar[2], it & 1);
    if (s_abort == 1) mbar_wait_bounded(&bar[it & 1], (it >> 1) & 1);
    if (tile + 1 < t_end) mbar_wait_bounded(&bar[(it + 1) & 1], ((it + 1) >> 1) & 1);
  }
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcRows) : "memory");
}

}  // namespace alut
