// C ABI of the ALUT path (declared in include/alut.h): argument checks on the host,
// dtype dispatch, and the launch sequence project+plan -> search -> finalize/combine.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include <cuda.h>

#include "alut_combine.cuh"
#include "alut_common.cuh"
#include "alut_project.cuh"
#include "alut_search.cuh"
#include "alut_tc.cuh"
#include "alut_project_tc.cuh"
#include "alut_peer.cuh"
#include "alut_online.cuh"
#include "alut_route.cuh"

namespace alut {

static void* noalloc_scratch_ptr(int* rc);
static thread_local char g_err[512] = "no error";
static thread_local cudaEvent_t g_prof_start = nullptr;
static thread_local cudaEvent_t g_prof_stop = nullptr;

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

// Records a profiling event (alut_set_profile_events) around the scan: as an external event
// node while the stream is being captured into a graph, as a plain record otherwise.
static int record_profile(cudaEvent_t ev, cudaStream_t st) {
  if (!ev) return ALUT_OK;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(st, &cs);
  if (e == cudaSuccess)
    e = cs == cudaStreamCaptureStatusActive ? cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal)
                                            : cudaEventRecord(ev, st);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "profile event: %s", cudaGetErrorString(e));
  return ALUT_OK;
}

static int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return ALUT_OK;
}

float host_round_as(float v, int dtype) {
  if (dtype == ALUT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == ALUT_F16) return __half2float(__float2half_rn(v));
  return v;
}

static int dtype_size(int d) { return d == ALUT_F32 ? 4 : 2; }
static bool dtype_ok(int d) { return d == ALUT_F32 || d == ALUT_BF16 || d == ALUT_F16; }
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < 64 && cache[dev]) return cache[dev];
  int n = 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  if (dev < 64) cache[dev] = n;
  return n;
}

// Raise a kernel's dynamic shared memory limit once per (kernel, device).
static int allow_smem(const void* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return ALUT_OK;
  struct Entry { const void* k; int dev; int bytes; };
  static Entry table[256];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].k == kernel && table[i].dev == dev && table[i].bytes >= static_cast<int>(bytes))
      return ALUT_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  if (used < 256) table[used++] = Entry{kernel, dev, static_cast<int>(bytes)};
  return ALUT_OK;
}

static size_t basis_plain_bytes(int l, int h) { return static_cast<size_t>(2) * 3 * l * h * sizeof(__nv_bfloat16); }

// Tables whose keys the tensor-core scan can take (once their bf16 form is prepared).
static bool tc_tables_ok(const alut_tables_t* t) {
  return t && t->key_dtype == ALUT_F32 && t->l > 0 && t->l % 16 == 0 && t->l <= kTcMaxL;
}

static int check_tables(const alut_tables_t* t, bool need_proj) {
  if (!t) return fail(ALUT_EINVAL, "tables is NULL");
  if (t->num_experts <= 0 || t->k <= 0 || t->l <= 0 || t->h <= 0)
    return fail(ALUT_EINVAL, "tables: num_experts=%d k=%d l=%d h=%d must be positive",
                t->num_experts, t->k, t->l, t->h);
  if (2 * static_cast<int64_t>(t->num_experts) > kMaxTables)
    return fail(ALUT_ERANGE, "tables: num_experts=%d exceeds %d", t->num_experts, kMaxTables / 2);
  if (t->l > kMaxL) return fail(ALUT_ERANGE, "tables: l=%d exceeds %d", t->l, kMaxL);
  if (!dtype_ok(t->key_dtype) || !dtype_ok(t->value_dtype) || !dtype_ok(t->proj_dtype))
    return fail(ALUT_EDTYPE, "tables: unknown dtype");
  if (need_proj) {
    if (t->proj_dtype != t->key_dtype)
      return fail(ALUT_EDTYPE, "tables: proj dtype (%d) must equal key dtype (%d)", t->proj_dtype,
                  t->key_dtype);
    for (int m = 0; m < 2; ++m)
      if (!t->proj[m] || !t->bias[m]) return fail(ALUT_EINVAL, "tables: proj/bias[%d] is NULL", m);
    if (t->proj_stride_h < t->l) return fail(ALUT_ESHAPE, "tables: proj_stride_h < l");
  }
  return ALUT_OK;
}

static int check_batch(const alut_tables_t* t, const alut_batch_t* b, bool need_x) {
  if (!b) return fail(ALUT_EINVAL, "batch is NULL");
  if (b->q < 0 || b->s < 0) return fail(ALUT_EINVAL, "batch: q=%d s=%d", b->q, b->s);
  if (b->s > kMaxSlots) return fail(ALUT_ERANGE, "batch: s=%d exceeds %d", b->s, kMaxSlots);
  if (static_cast<int64_t>(b->q) * b->s >= (1ll << 31))
    return fail(ALUT_ERANGE, "batch: q*s too large");
  if (b->q == 0 || b->s == 0) return ALUT_OK;
  if (!b->sel || !b->is_vision) return fail(ALUT_EINVAL, "batch: sel/is_vision is NULL");
  if (b->sel_stride < b->s) return fail(ALUT_ESHAPE, "batch: sel_stride < s");
  if (b->reuse && b->reuse_stride < b->s) return fail(ALUT_ESHAPE, "batch: reuse_stride < s");
  if (need_x) {
    if (!b->x) return fail(ALUT_EINVAL, "batch: x is NULL");
    if (!dtype_ok(b->x_dtype)) return fail(ALUT_EDTYPE, "batch: unknown x dtype");
    if (b->x_stride < t->h) return fail(ALUT_ESHAPE, "batch: x_stride < h");
  }
  return ALUT_OK;
}

static int check_params(const alut_tables_t* t, const alut_search_params_t* p, const void** keys) {
  if (!p) return fail(ALUT_EINVAL, "params is NULL");
  if (p->keyset == ALUT_KEYS_NORMALISED) *keys = t->keys;
  else if (p->keyset == ALUT_KEYS_RAW) *keys = t->raw_keys;
  else return fail(ALUT_EINVAL, "params: bad keyset %d", p->keyset);
  if (!*keys) return fail(ALUT_EINVAL, "tables: key set %d is NULL", p->keyset);
  if (t->key_stride[2] < t->l)
    return fail(ALUT_ESHAPE, "tables: key_stride_k < l");
  return ALUT_OK;
}

// ---- launches ------------------------------------------------------------------------

// Launch as a programmatic dependent of the previous kernel in the stream (it may start
// early and waits in griddepcontrol.wait for the predecessor's results).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Projection: grid = qtiles x nsplit CTAs; the nsplit CTAs of a token tile form one
// thread-block cluster (they add their partial tiles through distributed shared memory).
static int launch_project_kernel(void (*kern)(ProjPlanArgs), const ProjPlanArgs& args, size_t smem,
                                 cudaStream_t st) {
  ProjPlanArgs a = args;
  int rc = allow_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kProjThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.nsplit > 8) {
    // Clusters above 8 CTAs are non-portable: opt in once per device, and fall back to 8
    // if this device cannot co-schedule that many CTAs of this size.
    struct Known { const void* k; int dev; size_t smem; int ok; };
    static Known known[128];
    static int nknown = 0;
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    int ok = -1;
    {
      std::lock_guard<std::mutex> lock(mu);
      for (int i = 0; i < nknown; ++i)
        if (known[i].k == reinterpret_cast<const void*>(kern) && known[i].dev == dev && known[i].smem == smem)
          ok = known[i].ok;
    }
    if (ok < 0) {
      ok = 0;
      if (cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
          cudaSuccess) {
        cfg.gridDim = dim3(a.nsplit);
        attr[0].val.clusterDim.x = a.nsplit;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, reinterpret_cast<const void*>(kern), &cfg) == cudaSuccess &&
            clusters > 0)
          ok = 1;
      }
      cudaGetLastError();
      std::lock_guard<std::mutex> lock(mu);
      if (nknown < 128) known[nknown++] = Known{reinterpret_cast<const void*>(kern), dev, smem, ok};
    }
    int* sd = nullptr;
    int two = ok ? 1 : 2;
    sd = &two;
    if (sd && *sd == 2) a.nsplit = 8;
  }
  cfg.gridDim = dim3(a.qtiles * a.nsplit);
  attr[0].val.clusterDim.x = a.nsplit;
  // Programmatic dependent of whatever precedes it in the stream: the kernel prefetches
  // its static tables, then waits (griddepcontrol.wait) before reading any input.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "k_project: %s", cudaGetErrorString(e));
  return check_launch("k_project");
}

template <typename TX, typename TK>
static int launch_project_t(const ProjPlanArgs& a, size_t smem, cudaStream_t st) {
  const int nout = proj_nout(a.l);
  auto kern = nout == 4 ? k_project<TX, TK, TK, 4> : (nout == 8 ? k_project<TX, TK, TK, 8> : k_project<TX, TK, TK, 16>);
  return launch_project_kernel(kern, a, smem, st);
}

template <typename TK>
static int launch_project_k(int x_dtype, const ProjPlanArgs& a, size_t smem, cudaStream_t st) {
  switch (x_dtype) {
    case ALUT_F32: return launch_project_t<float, TK>(a, smem, st);
    case ALUT_BF16: return launch_project_t<__nv_bfloat16, TK>(a, smem, st);
    case ALUT_F16: return launch_project_t<__half, TK>(a, smem, st);
  }
  return fail(ALUT_EDTYPE, "x dtype");
}

// Whether the tensor-core projection applies: split basis present, bf16 tokens with 4-byte
// aligned rows, fp32 basis and keys, H % 16 == 0, L % 8 == 0.
static bool mma_projection_ok(int key_dtype, int x_dtype, const ProjPlanArgs& a) {
  return a.proj_split != nullptr && x_dtype == ALUT_BF16 && key_dtype == ALUT_F32 && a.h % 16 == 0 &&
         a.l % 8 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 3) == 0 && a.x_stride % 2 == 0 && a.q_in == nullptr;
}

static int launch_project(int key_dtype, int x_dtype, const ProjPlanArgs& a, cudaStream_t st) {
  const size_t smem = proj_smem_bytes(a.l);
  if (mma_projection_ok(key_dtype, x_dtype, a) && a.q >= kPtMinTokens && pt_shape_ok(a.l, a.h) &&
      a.x_stride % 8 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.zero_best == nullptr && a.meta) {
    // Large batch: tcgen05 projection over 128-token tiles (the basis's operand-order copy
    // follows the plain split, see alut_prepare_basis).
    PtArgs p{};
    p.x = static_cast<const __nv_bfloat16*>(a.x);
    p.x_stride = a.x_stride;
    p.is_vision = a.is_vision;
    p.basis = reinterpret_cast<const unsigned char*>(a.proj_split) + align256(basis_plain_bytes(a.l, a.h));
    p.bias[0] = static_cast<const float*>(a.bias[0]);
    p.bias[1] = static_cast<const float*>(a.bias[1]);
    p.q = a.q;
    p.h = a.h;
    p.l = a.l;
    p.stages = pt_stages(a.l);
    p.normalize = a.normalize;
    p.eps = a.eps;
    p.qlow = a.qlow;
    p.q_out = static_cast<float*>(a.q_out);
    p.q_out_stride = a.q_out_stride;
    p.err = a.meta + 1;
    CUtensorMap x_map;
    if (!pt_encode_x_map(&x_map, a.x, a.q, a.h, a.x_stride)) return fail(ALUT_ECUDA, "project: tensor map of x");
    const size_t sm = pt_smem_bytes(a.l);
    int rc = allow_smem(reinterpret_cast<const void*>(k_project_tc), sm);
    if (rc) return rc;
    const int ntiles = ceil_div(a.q, kTcRows);
    const int sms = num_sms();
    // Few tiles: split H over a cluster of up to 8 CTAs per tile.
    int ksplit = 1;
    while (ksplit < 8 && ntiles * ksplit * 2 <= sms && ksplit * 2 <= a.h / kPtKc) ksplit *= 2;
    p.ksplit = ksplit;
    if (ksplit == 1) {
      k_project_tc<<<std::min(ntiles, sms), kPtThreads, sm, st>>>(x_map, p);
      return check_launch("k_project_tc");
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntiles * ksplit);
    cfg.blockDim = dim3(kPtThreads);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ksplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_project_tc, x_map, p);
    if (e != cudaSuccess) return fail(ALUT_ECUDA, "k_project_tc (cluster of %d): %s", ksplit, cudaGetErrorString(e));
    return check_launch("k_project_tc");
  }
  if (mma_projection_ok(key_dtype, x_dtype, a)) {
    // The cluster size may drop to 8 inside launch_project_kernel; size for the larger layout.
    const size_t sm = std::max(mma_smem_layout(a.l, a.h, a.nsplit).total,
                               mma_smem_layout(a.l, a.h, std::min(a.nsplit, 8)).total);
    return launch_project_kernel(a.l <= 64 ? k_project_mma<float, 1> : k_project_mma<float, 2>, a, sm, st);
  }
  switch (key_dtype) {
    case ALUT_F32: return launch_project_k<float>(x_dtype, a, smem, st);
    case ALUT_BF16: return launch_project_k<__nv_bfloat16>(x_dtype, a, smem, st);
    case ALUT_F16: return launch_project_k<__half>(x_dtype, a, smem, st);
  }
  return fail(ALUT_EDTYPE, "key dtype");
}

// Slots above which the plan runs over the whole GPU (three launches) instead of one CTA.
constexpr int64_t kPlanWideSlots = 4096;

static int launch_plan(const ProjPlanArgs& a, int* tabs, cudaStream_t st) {
  const int ntab = 2 * a.num_experts;
  const int64_t pairs = static_cast<int64_t>(a.q) * a.s;
  if (pairs > kPlanWideSlots) {
    cudaError_t e = cudaMemsetAsync(tabs, 0, sizeof(int) * ntab, st);
    if (e != cudaSuccess) return fail(ALUT_ECUDA, "plan: %s", cudaGetErrorString(e));
    const int grid = static_cast<int>(std::min<int64_t>((pairs + 255) / 256, static_cast<int64_t>(num_sms()) * 4));
    const size_t hs = sizeof(int) * ntab;
    int rc = allow_smem(reinterpret_cast<const void*>(k_plan_count), hs);
    if (rc) return rc;
    k_plan_count<<<grid, 256, hs, st>>>(a, tabs);
    rc = check_launch("k_plan_count");
    if (rc) return rc;
    const size_t gs = sizeof(int) * (ntab + 1);
    rc = allow_smem(reinterpret_cast<const void*>(k_plan_groups), gs);
    if (rc) return rc;
    k_plan_groups<<<1, kProjThreads, gs, st>>>(a, tabs, tabs + ntab);
    rc = check_launch("k_plan_groups");
    if (rc) return rc;
    k_plan_scatter<<<grid, 256, 0, st>>>(a, tabs + ntab);
    return check_launch("k_plan_scatter");
  }
  const size_t smem = plan_smem_bytes(2 * a.num_experts, pairs);
  int rc = allow_smem(reinterpret_cast<const void*>(k_plan), smem);
  if (rc) return rc;
  k_plan<<<1, kProjThreads, smem, st>>>(a);
  return check_launch("k_plan");
}

template <typename TK>
static int launch_search_t(bool vec, const SearchArgs& a, int grid, size_t smem, cudaStream_t st) {
  if (vec) {
    int rc = allow_smem(reinterpret_cast<const void*>(k_search<TK, true>), smem);
    if (rc) return rc;
    k_search<TK, true><<<grid, kSearchThreads, smem, st>>>(a);
  } else {
    int rc = allow_smem(reinterpret_cast<const void*>(k_search<TK, false>), smem);
    if (rc) return rc;
    k_search<TK, false><<<grid, kSearchThreads, smem, st>>>(a);
  }
  return check_launch("k_search");
}

static int launch_search(int key_dtype, bool vec, const SearchArgs& a, int grid, size_t smem,
                         cudaStream_t st) {
  switch (key_dtype) {
    case ALUT_F32: return launch_search_t<float>(vec, a, grid, smem, st);
    case ALUT_BF16: return launch_search_t<__nv_bfloat16>(vec, a, grid, smem, st);
    case ALUT_F16: return launch_search_t<__half>(vec, a, grid, smem, st);
  }
  return fail(ALUT_EDTYPE, "key dtype");
}

template <typename TK>
static int launch_search_tma_t(const SearchArgs& a, int grid, size_t smem, int* err, cudaStream_t st) {
  int rc = allow_smem(reinterpret_cast<const void*>(k_search_tma<TK>), smem);
  if (rc) return rc;
  k_search_tma<TK><<<grid, kSearchThreads, smem, st>>>(a, err);
  return check_launch("k_search_tma");
}

static int launch_search_tma(int key_dtype, const SearchArgs& a, int grid, size_t smem, int* err,
                             cudaStream_t st) {
  switch (key_dtype) {
    case ALUT_F32: return launch_search_tma_t<float>(a, grid, smem, err, st);
    case ALUT_BF16: return launch_search_tma_t<__nv_bfloat16>(a, grid, smem, err, st);
    case ALUT_F16: return launch_search_tma_t<__half>(a, grid, smem, err, st);
  }
  return fail(ALUT_EDTYPE, "key dtype");
}

template <typename TV, typename TO>
static int launch_combine_t(bool vec, const CombineArgs& a, dim3 grid, cudaStream_t st) {
  cudaError_t e = vec ? launch_pdl(k_combine<TV, TO, true>, grid, dim3(kCombineThreads), 0, st, a)
                      : launch_pdl(k_combine<TV, TO, false>, grid, dim3(kCombineThreads), 0, st, a);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "k_combine: %s", cudaGetErrorString(e));
  return check_launch("k_combine");
}

template <typename TK>
static int launch_search_decode_t(const DecodeScanArgs& d, dim3 grid, size_t smem, cudaStream_t st) {
  // Ranks with a compile-time specialisation (the row lives in registers); others generic.
  auto kern = d.s.l == 64 ? k_search_decode<TK, 64>
                          : (d.s.l == 96 ? k_search_decode<TK, 96> : (d.s.l == 128 ? k_search_decode<TK, 128>
                                                                                   : k_search_decode<TK, 0>));
  int rc = allow_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc) return rc;
  cudaError_t e = launch_pdl(kern, grid, dim3(kSearchThreads), smem, st, d);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "k_search_decode: %s", cudaGetErrorString(e));
  return check_launch("k_search_decode");
}

static int launch_search_decode(int key_dtype, const DecodeScanArgs& d, dim3 grid, size_t smem,
                                cudaStream_t st) {
  switch (key_dtype) {
    case ALUT_F32: return launch_search_decode_t<float>(d, grid, smem, st);
    case ALUT_BF16: return launch_search_decode_t<__nv_bfloat16>(d, grid, smem, st);
    case ALUT_F16: return launch_search_decode_t<__half>(d, grid, smem, st);
  }
  return fail(ALUT_EDTYPE, "key dtype");
}

static int launch_combine(int vd, int od, bool vec, const CombineArgs& a, dim3 grid,
                          cudaStream_t st) {
  if (vd == ALUT_BF16 && od == ALUT_BF16) return launch_combine_t<__nv_bfloat16, __nv_bfloat16>(vec, a, grid, st);
  if (vd == ALUT_F16 && od == ALUT_F16) return launch_combine_t<__half, __half>(vec, a, grid, st);
  if (vd == ALUT_F32 && od == ALUT_F32) return launch_combine_t<float, float>(vec, a, grid, st);
  if (vd == ALUT_BF16 && od == ALUT_F32) return launch_combine_t<__nv_bfloat16, float>(vec, a, grid, st);
  if (vd == ALUT_F16 && od == ALUT_F32) return launch_combine_t<__half, float>(vec, a, grid, st);
  return fail(ALUT_EDTYPE, "combine: value dtype %d with out dtype %d not supported", vd, od);
}

// Projection + plan + centroid scan into the packed best buffer `best`.
// prefetch_values: the value table when a combine follows (the decode scan then asks L2
// for the rows of the running best candidates); NULL otherwise.
static int run_search(const alut_tables_t* t, const alut_batch_t* b, const alut_search_params_t* p,
                      const void* keys, const void* q_low_in, uint32_t idx_offset,
                      uint64_t* best, void* workspace, size_t ws_bytes, cudaStream_t st,
                      const void* prefetch_values = nullptr) {
  const Workspace w = workspace_layout(b->q, b->s, t->l, 2 * t->num_experts);
  if (!workspace) return fail(ALUT_EWORKSPACE, "workspace is NULL");
  if (ws_bytes < w.total)
    return fail(ALUT_EWORKSPACE, "workspace has %zu bytes, needs %zu", ws_bytes, w.total);
  if (!aligned16(workspace)) return fail(ALUT_EWORKSPACE, "workspace must be 16-byte aligned");
  char* base = static_cast<char*>(workspace);

  ProjPlanArgs a{};
  a.x = b->x;
  a.x_stride = b->x_stride;
  a.is_vision = b->is_vision;
  for (int m = 0; m < 2; ++m) {
    a.proj[m] = t->proj[m];
    a.bias[m] = t->bias[m];
  }
  a.proj_stride = t->proj_stride_h;
  a.proj_split = static_cast<const __nv_bfloat16*>(t->proj_split);
  a.q_in = q_low_in;
  a.q = b->q;
  a.h = t->h;
  a.l = t->l;
  a.qtiles = ceil_div(b->q, kProjTileQ);
  a.nsplit = q_low_in ? 1 : proj_splits(b->q, t->h);
  a.normalize = p->normalize_q;
  a.eps = p->eps;
  a.qlow = reinterpret_cast<float*>(base + w.qlow);
  a.s = b->s;
  a.num_experts = t->num_experts;
  a.sel = b->sel;
  a.sel_stride = b->sel_stride;
  a.reuse = b->reuse;
  a.reuse_stride = b->reuse_stride;
  a.best = best;
  a.sorted = reinterpret_cast<int*>(base + w.sorted);
  a.groups = reinterpret_cast<int4*>(base + w.groups);
  a.meta = reinterpret_cast<int*>(base + w.meta);
  const int esz = dtype_size(t->key_dtype);
  const bool vec = (t->l % 8 == 0) && aligned16(keys) && (t->key_stride[0] * esz) % 16 == 0 &&
                   (t->key_stride[1] * esz) % 16 == 0 && (t->key_stride[2] * esz) % 16 == 0;
  const bool tma = vec && t->key_stride[2] == t->l && static_cast<int64_t>(t->l) * esz <= 512;
  const int pairs = b->q * b->s;
  if (tma && b->q <= kDecodeMaxTokens && pairs <= kDecodeMaxPairs) {
    // Decode: projection (which also clears `best`), then the scan as its programmatic
    // dependent, whose key copies overlap the projection.
    a.zero_best = best;
    a.zero_n = pairs;
    if (g_prof_start && g_prof_stop && record_profile(g_prof_start, st)) return ALUT_ECUDA;
    int rc = launch_project(t->key_dtype, b->x_dtype, a, st);
    if (rc) return rc;
    DecodeScanArgs d{};
    d.s.keys = keys;
    d.s.key_stride_e = t->key_stride[0];
    d.s.key_stride_m = t->key_stride[1];
    d.s.key_stride_k = t->key_stride[2];
    d.s.k = t->k;
    d.s.l = t->l;
    d.s.s = b->s;
    d.s.nchunks = ceil_div(t->k, kSearchChunkK);
    d.s.idx_offset = idx_offset;
    d.s.qlow = a.qlow;
    d.s.best = best;
    d.q = b->q;
    d.num_experts = t->num_experts;
    d.sel = b->sel;
    d.sel_stride = b->sel_stride;
    d.is_vision = b->is_vision;
    d.reuse = b->reuse;
    d.reuse_stride = b->reuse_stride;
    d.err = a.meta + 1;
    {
      const int vsz = dtype_size(t->value_dtype);
      const int64_t rb = static_cast<int64_t>(t->h) * vsz;
      if (prefetch_values && aligned16(prefetch_values) && rb % 16 == 0 && rb < (1 << 20) &&
          (t->value_stride[0] * vsz) % 16 == 0 && (t->value_stride[1] * vsz) % 16 == 0 &&
          (t->value_stride[2] * vsz) % 16 == 0) {
        d.values = static_cast<const unsigned char*>(prefetch_values);
        d.vs_e = t->value_stride[0] * vsz;
        d.vs_m = t->value_stride[1] * vsz;
        d.vs_k = t->value_stride[2] * vsz;
        d.row_bytes = static_cast<uint32_t>(rb);
      }
    }
    rc = launch_search_decode(t->key_dtype, d, dim3(pairs, d.s.nchunks), search_decode_smem_bytes(t->l, esz), st);
    if (rc) return rc;
    if (g_prof_start && g_prof_stop && record_profile(g_prof_stop, st)) return ALUT_ECUDA;
    return ALUT_OK;
  }
  // Large batches: precomputed fp32 queries are read in place (no copy into the workspace).
  const bool q_direct = q_low_in != nullptr && t->key_dtype == ALUT_F32 && aligned16(q_low_in);
  if (q_direct) a.qlow = const_cast<float*>(static_cast<const float*>(q_low_in));
  // Large batches on fp32 tables prepared for it, with room in the workspace for the staged
  // queries: tensor-core scan (tcgen05).
  const void* ksplit = keys == t->raw_keys ? t->raw_keys_split : t->keys_split;
  const Workspace wt = workspace_layout(b->q, b->s, t->l, 2 * t->num_experts, true);
  if (ksplit && tc_tables_ok(t) && vec && tc_scan_wanted(pairs, 2 * t->num_experts) && ws_bytes >= wt.total) {
    a.group = kTcRows;
    a.cand_cnt = reinterpret_cast<int*>(base + wt.cand_cnt);
    int rc = launch_plan(a, reinterpret_cast<int*>(base + w.tabs), st);
    if (rc) return rc;
    if (!q_direct) rc = launch_project(t->key_dtype, b->x_dtype, a, st);
    if (rc) return rc;
    const int ntab = 2 * t->num_experts;
    const int nchunks = tc_prep_chunks(t->k);
    TcArgs c{};
    c.ksplit = static_cast<const unsigned char*>(ksplit);
    c.knorm = reinterpret_cast<const float*>(static_cast<const char*>(ksplit) +
                                             align256(static_cast<size_t>(ntab) * nchunks * tc_tile_bytes(t->l)));
    c.keys = static_cast<const float*>(keys);
    c.key_stride_e = t->key_stride[0];
    c.key_stride_m = t->key_stride[1];
    c.key_stride_k = t->key_stride[2];
    c.k = t->k;
    c.l = t->l;
    c.s = b->s;
    c.nchunks = nchunks;
    c.stages = tc_stages(t->l);
    c.idx_offset = idx_offset;
    c.qlow = a.qlow;
    c.qsplit = reinterpret_cast<const unsigned char*>(base + wt.qsplit);
    c.qnorm = reinterpret_cast<const float*>(base + wt.qnorm);
    c.sorted = a.sorted;
    c.groups = a.groups;
    c.meta = a.meta;
    c.best = best;
    c.err = a.meta + 1;
    c.cand_cnt = a.cand_cnt;
    c.cand = reinterpret_cast<int*>(base + wt.cand);
    {
      const int64_t units = wt.tc_groups * kTcRows * (t->l / 8);
      const int grid = static_cast<int>(std::min<int64_t>((units + 255) / 256, static_cast<int64_t>(num_sms()) * 8));
      k_stage_queries<<<std::max(grid, 1), 256, 0, st>>>(a.qlow, t->l, b->s, a.sorted, a.groups, a.meta, wt.tc_groups,
                                                       reinterpret_cast<__nv_bfloat16*>(base + wt.qsplit),
                                                       reinterpret_cast<float*>(base + wt.qnorm));
      rc = check_launch("k_stage_queries");
      if (rc) return rc;
    }
    const size_t smem = search_tc_smem_bytes(t->l);
    rc = allow_smem(reinterpret_cast<const void*>(k_search_tc), smem);
    if (rc) return rc;
    if (g_prof_start && g_prof_stop && record_profile(g_prof_start, st)) return ALUT_ECUDA;
    k_search_tc<<<num_sms(), kTcThreads, smem, st>>>(c);
    rc = check_launch("k_search_tc");
    if (rc) return rc;
    {
      TcRescoreArgs r{};
      r.keys = c.keys;
      r.key_stride_e = c.key_stride_e;
      r.key_stride_m = c.key_stride_m;
      r.key_stride_k = c.key_stride_k;
      r.l = t->l;
      r.s = b->s;
      r.num_experts = t->num_experts;
      r.pairs = pairs;
      r.idx_offset = idx_offset;
      r.qlow = a.qlow;
      r.sel = b->sel;
      r.sel_stride = b->sel_stride;
      r.is_vision = b->is_vision;
      r.cand_cnt = c.cand_cnt;
      r.cand = c.cand;
      r.best = best;
      k_tc_rescore<<<static_cast<unsigned>((static_cast<int64_t>(pairs) * 16 + 255) / 256), 256, 0, st>>>(r);
      rc = check_launch("k_tc_rescore");
      if (rc) return rc;
    }
    if (g_prof_start && g_prof_stop && record_profile(g_prof_stop, st)) return ALUT_ECUDA;
    return ALUT_OK;
  }
  {
    // Few tiles with full groups: smaller groups spread the scan over more SMs (each group
    // reads its table chunk again, from L2).
    const int64_t est_tiles = (static_cast<int64_t>(pairs) + kSearchGroup - 1) / kSearchGroup * ceil_div(t->k, kSearchChunkK);
    a.group = est_tiles < num_sms() ? kCcSmallGroup : kSearchGroup;
  }
  int rc = launch_plan(a, reinterpret_cast<int*>(base + w.tabs), st);
  if (rc) return rc;
  if (!q_direct) rc = launch_project(t->key_dtype, b->x_dtype, a, st);
  if (rc) return rc;

  SearchArgs s{};
  s.keys = keys;
  s.key_stride_e = t->key_stride[0];
  s.key_stride_m = t->key_stride[1];
  s.key_stride_k = t->key_stride[2];
  s.k = t->k;
  s.l = t->l;
  s.s = b->s;
  s.nchunks = ceil_div(t->k, kSearchChunkK);
  s.idx_offset = idx_offset;
  s.qlow = a.qlow;
  s.sorted = a.sorted;
  s.groups = a.groups;
  s.meta = a.meta;
  s.best = best;
  const int64_t max_tiles = w.max_groups * s.nchunks;
  const int grid = static_cast<int>(std::min<int64_t>(max_tiles, static_cast<int64_t>(num_sms()) * 8));
  if (g_prof_start && g_prof_stop && record_profile(g_prof_start, st)) return ALUT_ECUDA;
  if (tma) {
    rc = launch_search_tma(t->key_dtype, s, std::max(grid, 1), search_tma_smem_bytes(t->l, esz),
                           reinterpret_cast<int*>(a.meta) + 1, st);
  } else {
    rc = launch_search(t->key_dtype, vec, s, std::max(grid, 1), search_smem_bytes(t->l), st);
  }
  if (rc) return rc;
  if (g_prof_start && g_prof_stop && record_profile(g_prof_stop, st)) return ALUT_ECUDA;
  return ALUT_OK;
}

static void fill_value_strides(const alut_tables_t* t, CombineArgs& c) {
  c.values = t->values;
  c.vs_e = t->value_stride[0];
  c.vs_m = t->value_stride[1];
  c.vs_k = t->value_stride[2];
  c.h = t->h;
  c.num_experts = t->num_experts;
  c.k = t->k;
}

static bool combine_vec(const alut_tables_t* t, const void* out, int64_t out_stride, int od) {
  const int vsz = dtype_size(t->value_dtype), osz = dtype_size(od);
  return t->h % 8 == 0 && aligned16(t->values) && aligned16(out) &&
         (t->value_stride[0] * vsz) % 16 == 0 && (t->value_stride[1] * vsz) % 16 == 0 &&
         (t->value_stride[2] * vsz) % 16 == 0 && (out_stride * osz) % 16 == 0;
}

}  // namespace alut

using namespace alut;

extern "C" {

int alut_version(void) { return 100; }

#ifdef ALUT_PHASE_TRACE
int alut_debug_trace(unsigned long long* host, int n) {
  return cudaMemcpyFromSymbol(host, g_alut_trace, sizeof(unsigned long long) * (n < 64 ? n : 64)) == cudaSuccess ? 0 : -4;
}
int alut_debug_trace_span(unsigned long long* lo, unsigned long long* hi) {
  if (cudaMemcpyFromSymbol(lo, g_alut_trace_lo, sizeof(unsigned long long) * 64) != cudaSuccess) return -4;
  return cudaMemcpyFromSymbol(hi, g_alut_trace_hi, sizeof(unsigned long long) * 64) == cudaSuccess ? 0 : -4;
}
int alut_debug_trace_reset(void) {
  unsigned long long lo[64], hi[64];
  for (int i = 0; i < 64; ++i) {
    lo[i] = ~0ull;
    hi[i] = 0ull;
  }
  if (cudaMemcpyToSymbol(g_alut_trace_lo, lo, sizeof(lo)) != cudaSuccess) return -4;
  if (cudaMemcpyToSymbol(g_alut_trace, hi, sizeof(hi)) != cudaSuccess) return -4;
  return cudaMemcpyToSymbol(g_alut_trace_hi, hi, sizeof(hi)) == cudaSuccess ? 0 : -4;
}
#endif

int alut_online_search(int32_t b, int32_t h, int32_t n_valid, int32_t t, int32_t s, const void* x,
                       int32_t x_dtype, int64_t x_stride, const void* keys, int32_t key_dtype, int64_t key_stride,
                       const int64_t* eids, const int64_t* target, int64_t target_stride, uint8_t* on_hit,
                       int64_t* on_idx, int64_t* on_slot, int64_t out_stride, alut_stream_t stream) {
  if (b < 0 || h <= 0 || n_valid < 0 || t < 0 || s < 0) return fail(ALUT_EINVAL, "online_search: sizes");
  if (b == 0) return ALUT_OK;
  if (!x || !on_hit || !on_idx || !on_slot || (n_valid > 0 && (!keys || !eids)) || (s > 0 && !target))
    return fail(ALUT_EINVAL, "online_search: NULL argument");
  if (!dtype_ok(x_dtype) || x_dtype != key_dtype)
    return fail(ALUT_EDTYPE, "online_search: x and the window must share one dtype");
  const int esz = dtype_size(key_dtype);
  if (h > kOnlineMaxH || (h * esz) % 16 != 0 || x_stride < h || key_stride < h || (key_stride * esz) % 16 != 0 ||
      !aligned16(keys) || out_stride < s || target_stride < s)
    return fail(ALUT_ESHAPE, "online_search: h=%d must fill 16-byte units (<= %d), strides", h, kOnlineMaxH);
  OnlineArgs a{b, h, n_valid, t, s, x, x_stride, keys, key_stride, eids, target, target_stride, on_hit, on_idx,
               on_slot, out_stride};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = sizeof(float) * h;
  switch (key_dtype) {
    case ALUT_F32: {
      int rc = allow_smem(reinterpret_cast<const void*>(k_online_search<float>), smem);
      if (rc) return rc;
      k_online_search<float><<<b, kOnlineThreads, smem, st>>>(a);
      break;
    }
    case ALUT_BF16: {
      int rc = allow_smem(reinterpret_cast<const void*>(k_online_search<__nv_bfloat16>), smem);
      if (rc) return rc;
      k_online_search<__nv_bfloat16><<<b, kOnlineThreads, smem, st>>>(a);
      break;
    }
    case ALUT_F16: {
      int rc = allow_smem(reinterpret_cast<const void*>(k_online_search<__half>), smem);
      if (rc) return rc;
      k_online_search<__half><<<b, kOnlineThreads, smem, st>>>(a);
      break;
    }
  }
  return check_launch("k_online_search");
}

// ---- peer access for the centroid-range shards (CUDA IPC; no multicast objects) -------------

static_assert(sizeof(cudaIpcMemHandle_t) <= ALUT_PEER_HANDLE_BYTES, "IPC handle size");

int alut_peer_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return fail(ALUT_EINVAL, "peer_export: NULL argument");
  // The handle names the whole allocation; the offset locates ptr inside it.
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return fail(ALUT_ECUDA, "peer_export: cuMemGetAddressRange unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(ALUT_ECUDA, "peer_export: pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "peer_export: %s", cudaGetErrorString(e));
  memset(handle, 0, ALUT_PEER_HANDLE_BYTES);
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return ALUT_OK;
}

int alut_peer_open(const void* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return fail(ALUT_EINVAL, "peer_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "peer_open: %s", cudaGetErrorString(e));
  *ptr = static_cast<char*>(base) + offset;
  return ALUT_OK;
}

int alut_peer_close(void* ptr, uint64_t offset) {
  if (!ptr) return ALUT_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "peer_close: %s", cudaGetErrorString(e));
  return ALUT_OK;
}

int alut_gather_rows_sharded(int32_t n, const uint8_t* hit, const int64_t* idx, const uint8_t* is_vision,
                             int32_t world, const void* const* shard_values, const int64_t* shard_start,
                             const int64_t* shard_stride_m, int64_t value_stride_k, int32_t h, int32_t value_dtype,
                             void* out, int64_t out_stride, alut_stream_t stream) {
  if (n < 0 || world < 1 || world > kPeerMaxWorld) return fail(ALUT_EINVAL, "gather_rows_sharded: n=%d world=%d", n, world);
  if (n == 0) return ALUT_OK;
  if (!hit || !idx || !is_vision || !shard_values || !shard_start || !shard_stride_m || !out)
    return fail(ALUT_EINVAL, "gather_rows_sharded: NULL argument");
  if (!dtype_ok(value_dtype)) return fail(ALUT_EDTYPE, "gather_rows_sharded: value dtype");
  const int esz = dtype_size(value_dtype);
  const int64_t row_bytes = static_cast<int64_t>(h) * esz;
  if (h <= 0 || row_bytes % 16 != 0 || value_stride_k < h || out_stride < h ||
      (value_stride_k * esz) % 16 != 0 || (out_stride * esz) % 16 != 0 || !aligned16(out))
    return fail(ALUT_ESHAPE, "gather_rows_sharded: rows must be whole 16-byte units (h=%d)", h);
  const int grid = ceil_div(n, kPeerThreads / 32);
  k_gather_sharded<<<grid, kPeerThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      n, hit, idx, is_vision, world, reinterpret_cast<const unsigned char* const*>(shard_values), shard_start,
      shard_stride_m, esz, value_stride_k * esz, static_cast<int>(row_bytes), static_cast<unsigned char*>(out),
      out_stride * esz);
  return check_launch("k_gather_sharded");
}

size_t alut_route_workspace_size(int32_t num_experts) {
  if (num_experts <= 0 || num_experts > kRouteMaxExperts) return 0;
  return align256(sizeof(unsigned long long) * num_experts) + align256(sizeof(int) * num_experts);
}

int alut_route(int32_t q, int32_t num_experts, int32_t top_k, const void* logits, int32_t logits_dtype,
               int64_t logits_stride, int32_t normalize_topk, int32_t keep_mode, int32_t keep_k,
               double keep_rate, const float* attn, float* weights, int64_t* sel, uint8_t* compute,
               uint8_t* reuse, int64_t out_stride, void* workspace, size_t workspace_bytes,
               alut_stream_t stream) {
  if (q < 0 || num_experts <= 0 || top_k <= 0) return fail(ALUT_EINVAL, "route: q=%d experts=%d top_k=%d", q, num_experts, top_k);
  if (num_experts > kRouteMaxExperts || top_k > kMaxSlots || top_k > num_experts)
    return fail(ALUT_ERANGE, "route: top_k=%d must be <= min(64, experts) and experts=%d <= %d", top_k, num_experts,
                kRouteMaxExperts);
  if (!dtype_ok(logits_dtype)) return fail(ALUT_EDTYPE, "route: logits dtype");
  if (keep_mode != ALUT_KEEP_FIXED && keep_mode != ALUT_KEEP_IMPORTANCE) return fail(ALUT_EINVAL, "route: keep mode");
  if (q == 0) return ALUT_OK;
  if (!logits || !weights || !sel || !compute || !reuse) return fail(ALUT_EINVAL, "route: NULL argument");
  if (logits_stride < num_experts || out_stride < top_k) return fail(ALUT_ESHAPE, "route: strides");
  const size_t need = alut_route_workspace_size(num_experts);
  if (keep_mode == ALUT_KEEP_IMPORTANCE && (!workspace || workspace_bytes < need))
    return fail(ALUT_EWORKSPACE, "route: workspace has %zu bytes, needs %zu", workspace_bytes, need);
  if (keep_mode == ALUT_KEEP_IMPORTANCE && !(keep_rate >= 0.0))
    return fail(ALUT_EINVAL, "route: keep_rate must be >= 0");
  RouteArgs a{};
  a.q = q;
  a.e = num_experts;
  a.k = top_k;
  a.logits = logits;
  a.logits_dtype = logits_dtype;
  a.logits_stride = logits_stride;
  a.normalize = normalize_topk;
  a.mode = keep_mode;
  a.keep_k = keep_k < 0 ? top_k : std::min(keep_k, top_k);
  a.keep_rate = keep_rate;
  a.attn = attn;
  a.w = weights;
  a.sel = sel;
  a.compute = compute;
  a.reuse = reuse;
  a.out_stride = out_stride;
  if (workspace) {
    a.sums = static_cast<unsigned long long*>(workspace);
    a.counts = reinterpret_cast<int*>(static_cast<char*>(workspace) + align256(sizeof(unsigned long long) * num_experts));
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t sm = sizeof(float) * kRouteWarps * num_experts;
  int rc = allow_smem(reinterpret_cast<const void*>(k_route_topk), sm);
  if (rc) return rc;
  k_route_topk<<<ceil_div(q, kRouteWarps), kRouteWarps * 32, sm, st>>>(a);
  rc = check_launch("k_route_topk");
  if (rc || keep_mode != ALUT_KEEP_IMPORTANCE) return rc;
  const size_t ks = (sizeof(long long) + sizeof(int) + 1) * static_cast<size_t>(num_experts);
  rc = allow_smem(reinterpret_cast<const void*>(k_route_keep), ks);
  if (rc) return rc;
  k_route_keep<<<1, kRouteKeepThreads, ks, st>>>(a);
  return check_launch("k_route_keep");
}

int alut_keep_mask(int32_t q, int32_t num_experts, int32_t top_k, const int64_t* sel, const float* weights,
                   int64_t in_stride, const float* attn, double keep_rate, uint8_t* compute, uint8_t* reuse,
                   int64_t out_stride, void* workspace, size_t workspace_bytes, alut_stream_t stream) {
  if (q < 0 || num_experts <= 0 || top_k <= 0) return fail(ALUT_EINVAL, "keep_mask: sizes");
  if (num_experts > kRouteMaxExperts) return fail(ALUT_ERANGE, "keep_mask: experts=%d > %d", num_experts, kRouteMaxExperts);
  if (q == 0) return ALUT_OK;
  if (!sel || !weights || !compute || !reuse) return fail(ALUT_EINVAL, "keep_mask: NULL argument");
  if (in_stride < top_k || out_stride < top_k) return fail(ALUT_ESHAPE, "keep_mask: strides");
  if (!(keep_rate >= 0.0)) return fail(ALUT_EINVAL, "keep_mask: keep_rate must be >= 0");
  const size_t need = alut_route_workspace_size(num_experts);
  if (!workspace || workspace_bytes < need)
    return fail(ALUT_EWORKSPACE, "keep_mask: workspace has %zu bytes, needs %zu", workspace_bytes, need);
  if (in_stride != out_stride) return fail(ALUT_ESHAPE, "keep_mask: in_stride must equal out_stride");
  RouteArgs a{};
  a.q = q;
  a.e = num_experts;
  a.k = top_k;
  a.mode = ALUT_KEEP_IMPORTANCE;
  a.keep_rate = keep_rate;
  a.attn = attn;
  a.w = const_cast<float*>(weights);
  a.sel = const_cast<int64_t*>(sel);
  a.compute = compute;
  a.reuse = reuse;
  a.out_stride = out_stride;
  a.sums = static_cast<unsigned long long*>(workspace);
  a.counts = reinterpret_cast<int*>(static_cast<char*>(workspace) + align256(sizeof(unsigned long long) * num_experts));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(q) * top_k;
  k_route_scores<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(a);
  int rc = check_launch("k_route_scores");
  if (rc) return rc;
  const size_t ks = (sizeof(long long) + sizeof(int) + 1) * static_cast<size_t>(num_experts);
  rc = allow_smem(reinterpret_cast<const void*>(k_route_keep), ks);
  if (rc) return rc;
  k_route_keep<<<1, kRouteKeepThreads, ks, st>>>(a);
  return check_launch("k_route_keep");
}

int alut_normalize_rows(int64_t rows, int32_t l, const void* src, int64_t src_stride, void* dst, int64_t dst_stride,
                        int32_t dtype, float eps, alut_stream_t stream) {
  if (rows < 0 || l <= 0) return fail(ALUT_EINVAL, "normalize_rows: rows=%lld l=%d", static_cast<long long>(rows), l);
  if (rows == 0) return ALUT_OK;
  if (!src || !dst) return fail(ALUT_EINVAL, "normalize_rows: NULL argument");
  if (!dtype_ok(dtype)) return fail(ALUT_EDTYPE, "normalize_rows: dtype");
  if (src_stride < l || dst_stride < l) return fail(ALUT_ESHAPE, "normalize_rows: strides");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
  switch (dtype) {
    case ALUT_F32:
      k_normalize_rows<float><<<grid, 256, 0, st>>>(rows, l, static_cast<const float*>(src), src_stride,
                                                   static_cast<float*>(dst), dst_stride, eps);
      break;
    case ALUT_BF16:
      k_normalize_rows<__nv_bfloat16><<<grid, 256, 0, st>>>(rows, l, static_cast<const __nv_bfloat16*>(src), src_stride,
                                                           static_cast<__nv_bfloat16*>(dst), dst_stride, eps);
      break;
    case ALUT_F16:
      k_normalize_rows<__half><<<grid, 256, 0, st>>>(rows, l, static_cast<const __half*>(src), src_stride,
                                                    static_cast<__half*>(dst), dst_stride, eps);
      break;
  }
  return check_launch("k_normalize_rows");
}

int alut_workspace_errors(void* workspace, size_t workspace_bytes, int32_t clear, uint32_t* bits,
                          alut_stream_t stream) {
  if (!bits) return fail(ALUT_EINVAL, "workspace_errors: bits is NULL");
  if (!workspace) {  // the no-allocation entry point's scratch
    int rc = ALUT_OK;
    workspace = noalloc_scratch_ptr(&rc);
    if (!workspace) return rc;
    workspace_bytes = ALUT_NOALLOC_SCRATCH_BYTES;
  }
  if (workspace_bytes < 256) return fail(ALUT_EWORKSPACE, "workspace_errors: workspace too small");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // meta sits at offset 0 of every workspace layout; meta[1] is the error word.
  int32_t* word = static_cast<int32_t*>(workspace) + 1;
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, word, sizeof(host), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear && host) {
    e = cudaMemsetAsync(word, 0, sizeof(int32_t), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "workspace_errors: %s", cudaGetErrorString(e));
  *bits = host;
  return ALUT_OK;
}

int alut_set_profile_events(void* start_event, void* stop_event) {
  if ((start_event == nullptr) != (stop_event == nullptr))
    return fail(ALUT_EINVAL, "profile events must be both set or both NULL");
  g_prof_start = static_cast<cudaEvent_t>(start_event);
  g_prof_stop = static_cast<cudaEvent_t>(stop_event);
  return ALUT_OK;
}

const char* alut_last_error(void) { return g_err; }

size_t alut_keys_split_bytes(const alut_tables_t* t) {
  if (!t || t->key_dtype != ALUT_F32 || t->l <= 0 || t->l % 16 != 0 || t->l > kTcMaxL || t->k <= 0 ||
      t->num_experts <= 0)
    return 0;
  const int64_t ntab = 2 * static_cast<int64_t>(t->num_experts);
  const int64_t nchunks = tc_prep_chunks(t->k);
  return align256(ntab * nchunks * tc_tile_bytes(t->l)) + align256(sizeof(float) * ntab);
}

int alut_prepare_keys(const alut_tables_t* t, int32_t keyset, void* out, size_t out_bytes, alut_stream_t stream) {
  const size_t need = alut_keys_split_bytes(t);
  if (need == 0) return fail(ALUT_EINVAL, "prepare_keys: tables do not qualify (fp32 keys, l%%16, l<=%d)", kTcMaxL);
  if (!out || out_bytes < need) return fail(ALUT_EINVAL, "prepare_keys: out needs %zu bytes", need);
  const void* keys = keyset == ALUT_KEYS_RAW ? t->raw_keys : (keyset == ALUT_KEYS_NORMALISED ? t->keys : nullptr);
  if (!keys) return fail(ALUT_EINVAL, "prepare_keys: key set %d is NULL", keyset);
  const int ntab = 2 * t->num_experts;
  const int nchunks = tc_prep_chunks(t->k);
  const size_t body = align256(static_cast<size_t>(ntab) * nchunks * tc_tile_bytes(t->l));
  float* norms = reinterpret_cast<float*>(static_cast<char*>(out) + body);
  cudaError_t e = cudaMemsetAsync(norms, 0, sizeof(float) * ntab, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "prepare_keys: %s", cudaGetErrorString(e));
  k_prepare_keys<<<1184, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(keys), t->key_stride[0], t->key_stride[1], t->key_stride[2], ntab, t->k, t->l,
      nchunks, static_cast<__nv_bfloat16*>(out), norms);
  return check_launch("k_prepare_keys");
}

// Plain split [2][3][L][H] (decode-shaped projection), then, when the shape allows the
// large-batch tensor-core projection, the same parts in its operand order.

size_t alut_basis_split_bytes(const alut_tables_t* t) {
  if (!t || t->proj_dtype != ALUT_F32 || t->h <= 0 || t->l <= 0 || t->h % 16 != 0 || t->l % 8 != 0) return 0;
  const size_t plain = basis_plain_bytes(t->l, t->h);
  return pt_shape_ok(t->l, t->h) ? align256(plain) + pt_basis_bytes(t->l, t->h) : plain;
}

int alut_prepare_basis(const alut_tables_t* t, void* out, size_t out_bytes, alut_stream_t stream) {
  const size_t need = alut_basis_split_bytes(t);
  if (need == 0) return fail(ALUT_EINVAL, "prepare_basis: tables do not qualify (fp32 proj, h%%16, l%%8)");
  if (!out || out_bytes < need) return fail(ALUT_EINVAL, "prepare_basis: out needs %zu bytes", need);
  if (!t->proj[0] || !t->proj[1] || t->proj_stride_h < t->l) return fail(ALUT_EINVAL, "prepare_basis: proj");
  k_split_basis<<<592, kProjThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(t->proj[0]), static_cast<const float*>(t->proj[1]), t->proj_stride_h, t->h, t->l,
      static_cast<__nv_bfloat16*>(out));
  int rc = check_launch("k_split_basis");
  if (rc || !pt_shape_ok(t->l, t->h)) return rc;
  k_split_basis_tc<<<592, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(t->proj[0]), static_cast<const float*>(t->proj[1]), t->proj_stride_h, t->h, t->l,
      reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(out) + align256(basis_plain_bytes(t->l, t->h))));
  return check_launch("k_split_basis_tc");
}

int alut_scan_kind(const alut_tables_t* t, int32_t q, int32_t s) {
  if (!t || q < 0 || s < 0 || t->l <= 0 || t->num_experts <= 0) return fail(ALUT_EINVAL, "scan_kind: arguments");
  const int64_t slots = static_cast<int64_t>(q) * s;
  if (tc_tables_ok(t) && tc_scan_wanted(slots, 2 * t->num_experts)) return ALUT_SCAN_TENSOR_CORE;
  const int esz = dtype_size(t->key_dtype);
  if (t->l % 8 == 0 && static_cast<int64_t>(t->l) * esz <= 512 && q <= kDecodeMaxTokens && slots <= kDecodeMaxPairs)
    return ALUT_SCAN_DECODE;
  return ALUT_SCAN_CUDA_CORE;
}

size_t alut_workspace_size(const alut_tables_t* tables, int32_t q, int32_t s) {
  if (!tables || q < 0 || s < 0 || tables->l <= 0 || tables->num_experts <= 0) return 0;
  const bool tc = tc_tables_ok(tables) && tc_scan_wanted(static_cast<int64_t>(q) * s, 2 * tables->num_experts);
  return workspace_layout(q, s, tables->l, 2 * tables->num_experts, tc).total;
}

int alut_project(const alut_tables_t* tables, const alut_batch_t* batch, int32_t normalize_q,
                 float eps, void* q_low, int64_t q_low_stride, void* workspace,
                 size_t workspace_bytes, alut_stream_t stream) {
  int rc = check_tables(tables, true);
  if (rc) return rc;
  if (!batch) return fail(ALUT_EINVAL, "batch is NULL");
  if (batch->q < 0) return fail(ALUT_EINVAL, "batch: q=%d", batch->q);
  if (batch->q == 0) return ALUT_OK;
  if (!batch->x || !batch->is_vision) return fail(ALUT_EINVAL, "batch: x/is_vision is NULL");
  if (!dtype_ok(batch->x_dtype)) return fail(ALUT_EDTYPE, "batch: unknown x dtype");
  if (batch->x_stride < tables->h) return fail(ALUT_ESHAPE, "batch: x_stride < h");
  if (!q_low || q_low_stride < tables->l) return fail(ALUT_EINVAL, "q_low is NULL or stride < l");
  const Workspace w = workspace_layout(batch->q, 0, tables->l, 2 * tables->num_experts);
  if (!workspace || workspace_bytes < w.total)
    return fail(ALUT_EWORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, w.total);
  char* base = static_cast<char*>(workspace);
  ProjPlanArgs a{};
  a.x = batch->x;
  a.x_stride = batch->x_stride;
  a.is_vision = batch->is_vision;
  for (int m = 0; m < 2; ++m) {
    a.proj[m] = tables->proj[m];
    a.bias[m] = tables->bias[m];
  }
  a.proj_stride = tables->proj_stride_h;
  a.proj_split = static_cast<const __nv_bfloat16*>(tables->proj_split);
  a.q = batch->q;
  a.h = tables->h;
  a.l = tables->l;
  a.qtiles = ceil_div(batch->q, kProjTileQ);
  a.nsplit = proj_splits(batch->q, tables->h);
  a.normalize = normalize_q;
  a.eps = eps;
  a.qlow = reinterpret_cast<float*>(base + w.qlow);
  a.q_out = q_low;
  a.q_out_stride = q_low_stride;
  a.meta = reinterpret_cast<int*>(base + w.meta);
  return launch_project(tables->key_dtype, batch->x_dtype, a, reinterpret_cast<cudaStream_t>(stream));
}

int alut_search(const alut_tables_t* tables, const alut_batch_t* batch,
                const alut_search_params_t* params, const void* q_low_in, uint8_t* out_hit,
                int64_t* out_idx, int64_t out_stride, void* workspace, size_t workspace_bytes,
                alut_stream_t stream) {
  int rc = check_tables(tables, q_low_in == nullptr);
  if (rc) return rc;
  rc = check_batch(tables, batch, q_low_in == nullptr);
  if (rc) return rc;
  const void* keys = nullptr;
  rc = check_params(tables, params, &keys);
  if (rc) return rc;
  if (batch->q == 0 || batch->s == 0) return ALUT_OK;
  if (!out_hit || !out_idx) return fail(ALUT_EINVAL, "out_hit/out_idx is NULL");
  if (out_stride < batch->s) return fail(ALUT_ESHAPE, "out_stride < s");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = workspace_layout(batch->q, batch->s, tables->l, 2 * tables->num_experts);
  if (!workspace || workspace_bytes < w.total)
    return fail(ALUT_EWORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, w.total);
  uint64_t* best = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + w.best);
  rc = run_search(tables, batch, params, keys, q_low_in, 0u, best, workspace, workspace_bytes, st);
  if (rc) return rc;
  FinalizeArgs f{};
  f.best = best;
  f.sel = batch->sel;
  f.sel_stride = batch->sel_stride;
  f.is_vision = batch->is_vision;
  f.reuse = batch->reuse;
  f.reuse_stride = batch->reuse_stride;
  f.q = batch->q;
  f.s = batch->s;
  f.num_experts = tables->num_experts;
  f.cmp_ge = params->cmp_ge;
  f.thr_vis = host_round_as(params->thr_vision, tables->key_dtype);
  f.thr_txt = host_round_as(params->thr_text, tables->key_dtype);
  f.out_hit = out_hit;
  f.out_idx = out_idx;
  f.out_stride = out_stride;
  const int64_t n = static_cast<int64_t>(batch->q) * batch->s;
  cudaError_t e = launch_pdl(k_finalize, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, f);
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "k_finalize: %s", cudaGetErrorString(e));
  return check_launch("k_finalize");
}

int alut_gather_rows(const alut_tables_t* tables, int32_t n, const int64_t* eids,
                     const int64_t* mids, const int64_t* cids, const int64_t* out_rows,
                     void* out, int64_t out_stride, alut_stream_t stream) {
  if (!tables) return fail(ALUT_EINVAL, "tables is NULL");
  if (n < 0) return fail(ALUT_EINVAL, "n=%d", n);
  if (n == 0) return ALUT_OK;
  if (!tables->values || !eids || !mids || !cids || !out)
    return fail(ALUT_EINVAL, "values/eids/mids/cids/out is NULL");
  if (!dtype_ok(tables->value_dtype)) return fail(ALUT_EDTYPE, "value dtype");
  if (tables->h <= 0 || tables->k <= 0 || tables->num_experts <= 0)
    return fail(ALUT_EINVAL, "tables: bad sizes");
  if (out_stride < tables->h) return fail(ALUT_ESHAPE, "out_stride < h");
  const int esz = dtype_size(tables->value_dtype);
  GatherArgs g{};
  g.values = static_cast<const char*>(tables->values);
  g.vs_e = tables->value_stride[0] * esz;
  g.vs_m = tables->value_stride[1] * esz;
  g.vs_k = tables->value_stride[2] * esz;
  g.row_bytes = static_cast<int64_t>(tables->h) * esz;
  g.esz = esz;
  g.num_experts = tables->num_experts;
  g.k = tables->k;
  g.eids = eids;
  g.mids = mids;
  g.cids = cids;
  g.out_rows = out_rows;
  g.out = static_cast<char*>(out);
  g.out_stride = out_stride * esz;
  g.vec = aligned16(tables->values) && aligned16(out) && g.vs_e % 16 == 0 && g.vs_m % 16 == 0 &&
          g.vs_k % 16 == 0 && g.row_bytes % 16 == 0 && g.out_stride % 16 == 0;
  const int64_t words = g.vec ? g.row_bytes / 16 : g.row_bytes;
  const int ychunks = static_cast<int>(std::min<int64_t>(std::max<int64_t>((words + 127) / 128, 1), 64));
  k_gather_rows<<<dim3(n, ychunks), 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(g);
  return check_launch("k_gather_rows");
}

int alut_combine(const alut_tables_t* tables, const alut_batch_t* batch, const uint8_t* hit,
                 const int64_t* idx, int64_t hit_stride, const float* weights,
                 int64_t weight_stride, const uint8_t* compute_mask, int64_t compute_stride,
                 int32_t renorm, int32_t accumulate, void* out, int64_t out_stride,
                 int32_t out_dtype, alut_stream_t stream) {
  if (!tables) return fail(ALUT_EINVAL, "tables is NULL");
  if (!tables->values) return fail(ALUT_EINVAL, "tables: values is NULL");
  if (tables->num_experts <= 0 || tables->k <= 0 || tables->h <= 0)
    return fail(ALUT_EINVAL, "tables: bad sizes");
  int rc = check_batch(tables, batch, false);
  if (rc) return rc;
  if (batch->q == 0) return ALUT_OK;
  if (!out || out_stride < tables->h) return fail(ALUT_EINVAL, "out is NULL or stride < h");
  if (batch->s > 0 && (!hit || !idx || !weights)) return fail(ALUT_EINVAL, "hit/idx/weights is NULL");
  if (batch->s > 0 && (hit_stride < batch->s || weight_stride < batch->s))
    return fail(ALUT_ESHAPE, "hit_stride/weight_stride < s");
  if (compute_mask && compute_stride < batch->s) return fail(ALUT_ESHAPE, "compute_stride < s");
  if (renorm < ALUT_RENORM_NONE || renorm > ALUT_RENORM_TO_ROWSUM)
    return fail(ALUT_EINVAL, "bad renorm %d", renorm);
  if (!dtype_ok(out_dtype)) return fail(ALUT_EDTYPE, "out dtype");
  CombineArgs c{};
  fill_value_strides(tables, c);
  c.q = batch->q;
  c.s = batch->s;
  c.sel = batch->sel;
  c.sel_stride = batch->sel_stride;
  c.is_vision = batch->is_vision;
  c.reuse = batch->reuse;
  c.reuse_stride = batch->reuse_stride;
  c.hit_in = hit;
  c.idx_in = idx;
  c.hit_stride = hit_stride;
  c.w = weights;
  c.w_stride = weight_stride;
  c.compute = compute_mask;
  c.compute_stride = compute_stride;
  c.renorm = renorm;
  c.accumulate = accumulate;
  c.out = out;
  c.out_stride = out_stride;
  dim3 grid(batch->q, ceil_div(tables->h, kCombineSpan));
  return launch_combine(tables->value_dtype, out_dtype, combine_vec(tables, out, out_stride, out_dtype),
                        c, grid, reinterpret_cast<cudaStream_t>(stream));
}

static int lookup_combine_impl(const alut_tables_t* tables, const alut_batch_t* batch,
                               const alut_search_params_t* params, const float* weights, int64_t weight_stride,
                               const uint8_t* compute_mask, int64_t compute_stride, const void* computed,
                               int64_t computed_stride_t, int64_t computed_stride_s, int32_t renorm,
                               int32_t accumulate, void* out, int64_t out_stride, int32_t out_dtype,
                               uint8_t* out_hit, int64_t* out_idx, int64_t out_stride_hit, void* workspace,
                               size_t workspace_bytes, alut_stream_t stream) {
  int rc = check_tables(tables, true);
  if (rc) return rc;
  if (!tables->values) return fail(ALUT_EINVAL, "tables: values is NULL");
  rc = check_batch(tables, batch, true);
  if (rc) return rc;
  const void* keys = nullptr;
  rc = check_params(tables, params, &keys);
  if (rc) return rc;
  if (batch->q == 0 || batch->s == 0) return ALUT_OK;
  if (!out || out_stride < tables->h) return fail(ALUT_EINVAL, "out is NULL or stride < h");
  if (!weights || weight_stride < batch->s) return fail(ALUT_EINVAL, "weights NULL or stride < s");
  if (compute_mask && compute_stride < batch->s) return fail(ALUT_ESHAPE, "compute_stride < s");
  if ((out_hit == nullptr) != (out_idx == nullptr)) return fail(ALUT_EINVAL, "out_hit and out_idx go together");
  if (out_hit && out_stride_hit < batch->s) return fail(ALUT_ESHAPE, "out_stride_hit < s");
  if (renorm < ALUT_RENORM_NONE || renorm > ALUT_RENORM_TO_ROWSUM)
    return fail(ALUT_EINVAL, "bad renorm %d", renorm);
  if (!dtype_ok(out_dtype)) return fail(ALUT_EDTYPE, "out dtype");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const Workspace w = workspace_layout(batch->q, batch->s, tables->l, 2 * tables->num_experts);
  if (!workspace || workspace_bytes < w.total)
    return fail(ALUT_EWORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, w.total);
  uint64_t* best = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + w.best);
  rc = run_search(tables, batch, params, keys, nullptr, 0u, best, workspace, workspace_bytes, st, tables->values);
  if (rc) return rc;
  CombineArgs c{};
  fill_value_strides(tables, c);
  c.q = batch->q;
  c.s = batch->s;
  c.sel = batch->sel;
  c.sel_stride = batch->sel_stride;
  c.is_vision = batch->is_vision;
  c.reuse = batch->reuse;
  c.reuse_stride = batch->reuse_stride;
  c.best = best;
  c.cmp_ge = params->cmp_ge;
  c.thr_vis = host_round_as(params->thr_vision, tables->key_dtype);
  c.thr_txt = host_round_as(params->thr_text, tables->key_dtype);
  c.w = weights;
  c.w_stride = weight_stride;
  c.compute = compute_mask;
  c.compute_stride = compute_stride;
  c.renorm = renorm;
  c.accumulate = accumulate;
  c.out = out;
  c.out_stride = out_stride;
  c.out_hit = out_hit;
  c.out_idx = out_idx;
  c.out_hit_stride = out_stride_hit;
  c.computed = computed;
  c.computed_stride_t = computed_stride_t;
  c.computed_stride_s = computed_stride_s;
  const int vsz = dtype_size(tables->value_dtype);
  const bool vec = combine_vec(tables, out, out_stride, out_dtype) &&
                   (!computed || (aligned16(computed) && (computed_stride_t * vsz) % 16 == 0 &&
                                  (computed_stride_s * vsz) % 16 == 0));
  dim3 grid(batch->q, ceil_div(tables->h, kCombineSpan));
  return launch_combine(tables->value_dtype, out_dtype, vec, c, grid, st);
}

int alut_lookup_combine(const alut_tables_t* tables, const alut_batch_t* batch,
                        const alut_search_params_t* params, const float* weights,
                        int64_t weight_stride, const uint8_t* compute_mask,
                        int64_t compute_stride, int32_t renorm, int32_t accumulate, void* out,
                        int64_t out_stride, int32_t out_dtype, uint8_t* out_hit,
                        int64_t* out_idx, int64_t out_stride_hit, void* workspace,
                        size_t workspace_bytes, alut_stream_t stream) {
  return lookup_combine_impl(tables, batch, params, weights, weight_stride, compute_mask, compute_stride, nullptr, 0,
                             0, renorm, accumulate, out, out_stride, out_dtype, out_hit, out_idx, out_stride_hit,
                             workspace, workspace_bytes, stream);
}

int alut_lookup_combine_experts(const alut_tables_t* tables, const alut_batch_t* batch,
                                const alut_search_params_t* params, const float* weights, int64_t weight_stride,
                                const uint8_t* compute_mask, int64_t compute_stride, const void* computed,
                                int64_t computed_stride_t, int64_t computed_stride_s, int32_t renorm,
                                int32_t accumulate, void* out, int64_t out_stride, int32_t out_dtype,
                                uint8_t* out_hit, int64_t* out_idx, int64_t out_stride_hit, void* workspace,
                                size_t workspace_bytes, alut_stream_t stream) {
  if (!computed || !compute_mask) return fail(ALUT_EINVAL, "lookup_combine_experts: computed/compute_mask is NULL");
  if (batch && tables && (computed_stride_s < tables->h || computed_stride_t < computed_stride_s * batch->s))
    return fail(ALUT_ESHAPE, "lookup_combine_experts: computed strides");
  return lookup_combine_impl(tables, batch, params, weights, weight_stride, compute_mask, compute_stride, computed,
                             computed_stride_t, computed_stride_s, renorm, accumulate, out, out_stride, out_dtype,
                             out_hit, out_idx, out_stride_hit, workspace, workspace_bytes, stream);
}

int alut_search_packed(const alut_tables_t* tables, const alut_batch_t* batch,
                       const alut_search_params_t* params, const void* q_low_in,
                       int64_t idx_offset, uint64_t* out_packed, void* workspace,
                       size_t workspace_bytes, alut_stream_t stream) {
  int rc = check_tables(tables, q_low_in == nullptr);
  if (rc) return rc;
  rc = check_batch(tables, batch, q_low_in == nullptr);
  if (rc) return rc;
  const void* keys = nullptr;
  rc = check_params(tables, params, &keys);
  if (rc) return rc;
  if (batch->q == 0 || batch->s == 0) return ALUT_OK;
  if (!out_packed) return fail(ALUT_EINVAL, "out_packed is NULL");
  if (idx_offset < 0 || idx_offset + tables->k > 0xFFFFFFFFll)
    return fail(ALUT_ERANGE, "idx_offset out of range");
  return run_search(tables, batch, params, keys, q_low_in, static_cast<uint32_t>(idx_offset),
                    out_packed, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int alut_merge_packed(int32_t world, int32_t q, int32_t s, const uint64_t* packed_all,
                      const uint8_t* is_vision, const alut_search_params_t* params,
                      uint8_t* out_hit, int64_t* out_idx, alut_stream_t stream) {
  if (world <= 0 || q < 0 || s < 0) return fail(ALUT_EINVAL, "world=%d q=%d s=%d", world, q, s);
  if (!params) return fail(ALUT_EINVAL, "params is NULL");
  const int64_t n = static_cast<int64_t>(q) * s;
  if (n == 0) return ALUT_OK;
  if (!packed_all || !out_hit || !out_idx) return fail(ALUT_EINVAL, "packed_all/out is NULL");
  MergeArgs m{};
  m.packed = packed_all;
  m.world = world;
  m.n = n;
  m.s = s;
  m.is_vision = is_vision;
  m.cmp_ge = params->cmp_ge;
  m.thr_vis = params->thr_vision;
  m.thr_txt = params->thr_text;
  m.out_hit = out_hit;
  m.out_idx = out_idx;
  k_merge<<<static_cast<unsigned>((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(m);
  return check_launch("k_merge");
}

}  // extern "C"

// ---- no-allocation variant of alut_lookup_combine ------------------------------------------
// The scratch of alut_lookup_combine_noalloc: one fixed array per device, shared by all its
// calls. Host code must not pass the symbol itself to a kernel (on the host it only names a
// stand-in); its device address comes from cudaGetSymbolAddress, looked up once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[ALUT_NOALLOC_SCRATCH_BYTES];

namespace alut {
// The array's address is resolved once per (device, CUDA context): a context created after a
// cudaDeviceReset (or a caller's own driver-API context) loads the module again and gets a
// fresh copy of the array, so the cached address is only reused within the same context.
static void* noalloc_scratch_ptr(int* rc) {
  struct Entry { void* ctx; void* ptr; };
  static Entry cache[64] = {};
  static std::mutex mu;
  using GetCtx = CUresult (*)(CUcontext*);
  static GetCtx get_ctx = nullptr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = fail(ALUT_ECUDA, "noalloc: no usable current device (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!get_ctx) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
      get_ctx = reinterpret_cast<GetCtx>(fn);
  }
  // Before the runtime's first call on this thread there may be no current context yet;
  // cudaGetSymbolAddress binds it, and the key is read again after it.
  CUcontext ctx = nullptr;
  if (get_ctx) get_ctx(&ctx);
  if (!cache[dev].ptr || !ctx || cache[dev].ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *rc = fail(ALUT_ECUDA, "noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    if (get_ctx) get_ctx(&ctx);
    cache[dev] = Entry{ctx, p};
  }
  *rc = ALUT_OK;
  return cache[dev].ptr;
}
}  // namespace alut

extern "C" int alut_lookup_combine_noalloc(const alut_tables_t* tables, const alut_batch_t* batch,
                                           const alut_search_params_t* params, const float* weights,
                                           int64_t weight_stride, const uint8_t* compute_mask,
                                           int64_t compute_stride, int32_t renorm, int32_t accumulate,
                                           void* out, int64_t out_stride, int32_t out_dtype,
                                           uint8_t* out_hit, int64_t* out_idx, int64_t out_stride_hit,
                                           alut_stream_t stream) {
  if (!tables || !batch) return fail(ALUT_EINVAL, "tables/batch is NULL");
  if (batch->q < 0 || batch->s < 0 || tables->l <= 0 || tables->num_experts <= 0)
    return fail(ALUT_EINVAL, "noalloc: bad sizes");
  const size_t need = workspace_layout(batch->q, batch->s, tables->l, 2 * tables->num_experts).total;
  if (need > ALUT_NOALLOC_SCRATCH_BYTES)
    return fail(ALUT_ERANGE, "noalloc: batch needs %zu bytes of scratch, the fixed array holds %u", need,
                ALUT_NOALLOC_SCRATCH_BYTES);
  int rc = ALUT_OK;
  void* scratch = noalloc_scratch_ptr(&rc);
  if (!scratch) return rc;
  // The meta words (group count, error bits) start from zero on every call; everything
  // else in the scratch is written before it is read.
  const Workspace w = workspace_layout(batch->q, batch->s, tables->l, 2 * tables->num_experts);
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(scratch) + w.meta, 0, sizeof(int32_t) * 8,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(ALUT_ECUDA, "noalloc: clearing scratch: %s", cudaGetErrorString(e));
  return alut_lookup_combine(tables, batch, params, weights, weight_stride, compute_mask, compute_stride, renorm,
                             accumulate, out, out_stride, out_dtype, out_hit, out_idx, out_stride_hit, scratch,
                             ALUT_NOALLOC_SCRATCH_BYTES, stream);
}
