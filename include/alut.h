/*
 * alut.h - C ABI of the B200 (sm_100a) approximate-lookup-table (ALUT) path of TableMoE.
 *
 * The ALUT path replaces a skipped routed expert's output by a cached one:
 *   1. project the token's hidden state onto the layer's per-modality PCA basis,
 *   2. find the centroid of the (expert, modality) key table with the largest inner
 *      product (first index wins ties), with a hit threshold,
 *   3. gather that centroid's cached expert output (the value row),
 *   4. scale it by the renormalised routing weight and accumulate it into the layer output.
 *
 * Every entry point is asynchronous on the stream it is given, takes plain device
 * pointers and sizes, and returns ALUT_OK (0) or a negative alut_status_t. Argument
 * errors are detected on the host before anything is launched. Nothing here allocates
 * device memory: scratch lives in a caller-owned workspace whose size comes from
 * alut_workspace_size() and which must be zero-filled once before its first use (the
 * kernels leave it reusable). Calls that share one workspace must be ordered on the
 * GPU (same stream, or events between streams).
 *
 * Reference interfaces replaced (paths are inside the reference project
 * fanyalun/tablemoe-sc26):
 *   alut_project          table_moe/cache_engine/search.py:476  _project_queries_into
 *   alut_search           table_moe/cache_engine/search.py:515  _search_prefill_offline_into
 *                         table_moe/cache_engine/search.py:566  _search_decode_offline_from_low_into
 *                         table_moe/cache_engine/search.py:604  _search_decode_offline_into
 *                         table_moe/cache_engine/search.py:661  _search_offline_dot_from_low_into
 *                         table_moe/cache_engine/search.py:715  search_decode_offline_dot
 *   alut_gather_rows      table_moe/cache_engine/manager.py:212 gather_values
 *                         table_moe/cache_engine/manager.py:216 gather_values_decode_bs1
 *   alut_combine          table_moe/models/qwen3_vl_moe/cached_layers.py:455-465 (lookup slots)
 *                         table_moe/models/deepseek_vl2/deepseek_layers.py:707-729
 *                         table_moe/skip/pruning.py:55 renormalize_surviving_weights
 *   alut_lookup_combine   search + combine in one call (no single reference counterpart;
 *                         it chains search.py:808 and cached_layers.py:340-465)
 *   alut_lookup_combine_experts
 *                         cached_layers.py:340-465 whole (lookups + computed experts' outputs)
 *   alut_route            table_moe/ops/qwen_topk_softmax.py:122-153 + cached_layers.py:69-84
 *   alut_keep_mask        table_moe/skip/pruning.py:18-48 build_prefill_keep_mask
 *   alut_normalize_rows   table_moe/cache_engine/manager.py:24-31, :205-207
 *   alut_search_packed /
 *   alut_merge_packed     centroid-range sharding of one large table (new: the reference
 *                         is single-GPU; the merge rule is the tie rule of search.py:89)
 *
 * Input ordering: batches of <= 256 slots (q x s; the decode chain) read sel, reuse and is_vision
 * before waiting for the kernel that precedes the call on the stream, so that key copies
 * start early; these inputs must be complete when the call is issued (true for inputs
 * written by ordinary stream-ordered work). x is read only after that wait.
 */
#ifndef ALUT_H_
#define ALUT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* alut_stream_t; /* == cudaStream_t; NULL is the legacy default stream */

typedef enum alut_dtype {
  ALUT_F32 = 0,
  ALUT_BF16 = 1,
  ALUT_F16 = 2,
} alut_dtype_t;

typedef enum alut_status {
  ALUT_OK = 0,
  ALUT_EINVAL = -1,     /* null pointer, negative size, bad enum */
  ALUT_EDTYPE = -2,     /* dtype combination not supported */
  ALUT_ESHAPE = -3,     /* shape/stride not supported (e.g. non-unit innermost stride) */
  ALUT_ECUDA = -4,      /* a CUDA launch or API call failed; see alut_last_error() */
  ALUT_EWORKSPACE = -5, /* workspace missing or smaller than alut_workspace_size() */
  ALUT_ERANGE = -6,     /* size beyond what the build supports */
} alut_status_t;

/* Which centroid table a search scores against (manager.py:44-53). */
typedef enum alut_keyset {
  ALUT_KEYS_NORMALISED = 0, /* keys_buffer: rows L2-normalised at load (cosine variants) */
  ALUT_KEYS_RAW = 1,        /* raw_keys_buffer (dot variants) */
} alut_keyset_t;

/* How alut_combine rescales the routing weights of surviving slots
 * (skip/pruning.py:55-73). A slot survives when it was computed (compute_mask) or when
 * its lookup hit. */
typedef enum alut_renorm {
  ALUT_RENORM_NONE = 0,      /* weights are final as given */
  ALUT_RENORM_TO_ONE = 1,    /* w*surv / sum(w*surv)               (Qwen3-VL wrapper) */
  ALUT_RENORM_TO_ROWSUM = 2, /* w*surv / sum(w*surv) * sum(w)       (DeepSeek-VL2 wrapper) */
} alut_renorm_t;

/* One layer's tables, all device-resident. Modality 0 = vision, 1 = text
 * (config.py:28). Strides are in elements; the innermost stride of every tensor is 1. */
typedef struct alut_tables {
  int32_t num_experts; /* E */
  int32_t k;           /* K centroids per (expert, modality) */
  int32_t l;           /* L, PCA rank */
  int32_t h;           /* H, hidden size */
  int32_t key_dtype;   /* alut_dtype_t of keys and raw_keys */
  int32_t value_dtype; /* alut_dtype_t of values */
  int32_t proj_dtype;  /* alut_dtype_t of proj and bias */
  int32_t reserved0;
  const void* keys;     /* [E,2,K,L] keys_buffer (may be NULL if only RAW is used) */
  const void* raw_keys; /* [E,2,K,L] raw_keys_buffer (may be NULL if only NORMALISED is used) */
  const void* values;   /* [E,2,K,H] values_buffer (may be NULL for search-only calls) */
  const void* proj[2];  /* [H,L] per modality */
  const void* bias[2];  /* [L] per modality (= -mean @ proj, manager.py:166) */
  int64_t key_stride[3];   /* strides of dims e, m, k (keys and raw_keys share them) */
  int64_t value_stride[3]; /* strides of dims e, m, k */
  int64_t proj_stride_h;   /* row stride of proj */
  /* Optional: the fp32 basis split into three bf16 parts (hi + mid + lo == proj to fp32
   * precision), written by alut_prepare_basis: [2 modalities][3][L][H], followed (when
   * L % 16 == 0, L <= 128 and H % 64 == 0) by the same parts in the large-batch tensor-core
   * projection's operand order. When set and x is bf16, the projection runs on tensor
   * cores; NULL keeps the CUDA-core path. */
  const void* proj_split;
  /* Optional: fp32 key tables prepared for the tensor-core scan by alut_prepare_keys
   * (keys_split for keys, raw_keys_split for raw_keys; NULL keeps the CUDA-core scans). */
  const void* keys_split;
  const void* raw_keys_split;
} alut_tables_t;

/* One batch of routed tokens. */
typedef struct alut_batch {
  int32_t q;       /* tokens */
  int32_t s;       /* routed slots per token (top_k) */
  int32_t x_dtype; /* alut_dtype_t of x */
  int32_t reserved0;
  const void* x;            /* [Q,H] hidden states */
  int64_t x_stride;         /* row stride of x */
  const int64_t* sel;       /* [Q,S] selected expert ids */
  int64_t sel_stride;       /* row stride of sel */
  const uint8_t* is_vision; /* [Q] bool, nonzero = vision modality */
  const uint8_t* reuse;     /* [Q,S] bool search mask; NULL = every slot searched */
  int64_t reuse_stride;     /* row stride of reuse */
} alut_batch_t;

/* Search parameters (config.py:34-37). */
typedef struct alut_search_params {
  int32_t keyset;       /* alut_keyset_t */
  int32_t normalize_q;  /* 1: L2-normalise the projected query (search.py:495, prefill cosine) */
  int32_t cmp_ge;       /* 1: hit = max >= thr (search.py:597); 0: hit = max > thr (search.py:689) */
  int32_t reserved0;
  float thr_vision;     /* threshold for vision tokens */
  float thr_text;       /* threshold for text tokens */
  float eps;            /* OFFLINE_COSINE_EPS (search.py:13-18) */
  float reserved1;
} alut_search_params_t;

/* Bytes of workspace needed for batches of up to q tokens x s slots on these tables.
 * Returns 0 on invalid arguments. */
size_t alut_workspace_size(const alut_tables_t* tables, int32_t q, int32_t s);

/* Which centroid scan a batch of q tokens x s slots takes on these tables (contiguous,
 * 16-byte aligned key rows assumed): the decode chain (<= 256 slots, any q),
 * the tensor-core scan (fp32 keys with L % 16 == 0, L <= 128, >= 512 slots and >= 12
 * slots per routed table on average; it needs the key form of alut_prepare_keys) or the
 * CUDA-core scans. Negative status on invalid arguments. */
#define ALUT_SCAN_DECODE 0
#define ALUT_SCAN_CUDA_CORE 1
#define ALUT_SCAN_TENSOR_CORE 2
int alut_scan_kind(const alut_tables_t* tables, int32_t q, int32_t s);

/* Bytes of the split basis of these tables (0 if the tables do not qualify: fp32 proj,
 * H % 16 == 0, L % 8 == 0); includes the operand-order copy when the shape allows it. */
size_t alut_basis_split_bytes(const alut_tables_t* tables);

/* Write the split basis (see alut_tables_t.proj_split) of tables->proj into out, a device
 * buffer of alut_basis_split_bytes() bytes. Once per table load; the basis is static. */
int alut_prepare_basis(const alut_tables_t* tables, void* out, size_t out_bytes, alut_stream_t stream);

/* Bytes of the tensor-core form of one fp32 key set of these tables (0 if they do not
 * qualify: fp32 keys, L % 16 == 0, L <= 128): every (expert, modality) table cut into
 * 128-row chunks, each chunk as bf16 (round to nearest) in the tensor cores' K-major
 * core-matrix order, followed by the largest row norm of every table. The tensor-core
 * scan uses it only to choose candidates; every candidate is rescored in fp32 from the
 * original keys, so results equal the CUDA-core scans'. Used for batches of >= 512
 * searched slots when the workspace has room (alut_workspace_size includes it). */
size_t alut_keys_split_bytes(const alut_tables_t* tables);

/* Write that form of the key set `keyset` into out (device, alut_keys_split_bytes bytes).
 * Once per table load; the keys are static. */
int alut_prepare_keys(const alut_tables_t* tables, int32_t keyset, void* out, size_t out_bytes,
                      alut_stream_t stream);

/* a1: q_low[Q,L] = x[mask_m] @ proj_m + bias_m per modality, optionally L2-normalised,
 * written in the key dtype (search.py:476-498). */
int alut_project(const alut_tables_t* tables, const alut_batch_t* batch, int32_t normalize_q,
                 float eps, void* q_low, int64_t q_low_stride, void* workspace,
                 size_t workspace_bytes, alut_stream_t stream);

/* a2-a5: for every slot with reuse: idx = argmax_k q_low . key[e,m,k] (first index on
 * ties), hit = threshold rule. Slots without reuse, and misses, get hit=0, idx=0 (the
 * reference's pre-zeroed outputs). out_hit/out_idx are [Q,S] with row stride out_stride.
 * q_low_in may hold a precomputed [Q,L] query in the key dtype (row stride l); when NULL
 * the query is projected from batch->x. */
int alut_search(const alut_tables_t* tables, const alut_batch_t* batch,
                const alut_search_params_t* params, const void* q_low_in, uint8_t* out_hit,
                int64_t* out_idx, int64_t out_stride, void* workspace, size_t workspace_bytes,
                alut_stream_t stream);

/* a7: out[r_i,:] = values[eids[i], mids[i], cids[i], :] for i < n, a bit-exact copy
 * (manager.py:212-213), with r_i = out_rows[i] when out_rows is given (the slot scatter of
 * gather_values_decode_bs1, manager.py:216-228) and r_i = i otherwise. out has the value
 * dtype and row stride out_stride. Out-of-range ids give a zero row. */
int alut_gather_rows(const alut_tables_t* tables, int32_t n, const int64_t* eids,
                     const int64_t* mids, const int64_t* cids, const int64_t* out_rows,
                     void* out, int64_t out_stride, alut_stream_t stream);

/* a8 for the lookup slots: for each token t,
 *   out[t,:] = (accumulate ? out[t,:] : 0) + sum_{s: hit[t,s]} w~[t,s] * values[sel[t,s], m_t, idx[t,s], :]
 * with w~ the renormalised weights of renorm (survivors = compute_mask | hit;
 * compute_mask NULL means no computed slots). Arithmetic is fp32; out has out_dtype. */
int alut_combine(const alut_tables_t* tables, const alut_batch_t* batch, const uint8_t* hit,
                 const int64_t* idx, int64_t hit_stride, const float* weights,
                 int64_t weight_stride, const uint8_t* compute_mask, int64_t compute_stride,
                 int32_t renorm, int32_t accumulate, void* out, int64_t out_stride,
                 int32_t out_dtype, alut_stream_t stream);

/* alut_search followed by alut_combine without the hit/idx round trip through the
 * caller. out_hit/out_idx may be NULL. */
int alut_lookup_combine(const alut_tables_t* tables, const alut_batch_t* batch,
                        const alut_search_params_t* params, const float* weights,
                        int64_t weight_stride, const uint8_t* compute_mask,
                        int64_t compute_stride, int32_t renorm, int32_t accumulate, void* out,
                        int64_t out_stride, int32_t out_dtype, uint8_t* out_hit,
                        int64_t* out_idx, int64_t out_stride_hit, void* workspace,
                        size_t workspace_bytes, alut_stream_t stream);

/* alut_lookup_combine that also adds the computed experts' outputs, i.e. the whole combine
 * of the MoE layer (cached_layers.py:452-465: collected[t, s] = expert output for computed
 * slots, the looked-up value row for hit slots, then bmm with the renormalised weights):
 *   out[t, :] (+)= sum_s w~[t, s] * (hit[t, s] ? value row : compute_mask[t, s] ?
 *                                     computed[t, s, :] : 0)
 * in slot order, fp32 arithmetic. computed: [Q, S, H] in the value dtype with element
 * strides computed_stride_t (token) and computed_stride_s (slot); rows of non-computed
 * slots are not read. compute_mask is required. */
int alut_lookup_combine_experts(const alut_tables_t* tables, const alut_batch_t* batch,
                                const alut_search_params_t* params, const float* weights, int64_t weight_stride,
                                const uint8_t* compute_mask, int64_t compute_stride, const void* computed,
                                int64_t computed_stride_t, int64_t computed_stride_s, int32_t renorm,
                                int32_t accumulate, void* out, int64_t out_stride, int32_t out_dtype,
                                uint8_t* out_hit, int64_t* out_idx, int64_t out_stride_hit, void* workspace,
                                size_t workspace_bytes, alut_stream_t stream);

/* Centroid-range shard: search a table slice whose row 0 is global centroid idx_offset
 * and write, per (token, slot), the packed best candidate
 *   (order-preserving bits of the score << 32) | (0xFFFFFFFF - global index)
 * so that the largest packed value is the best score with the lowest index; 0 means no
 * candidate. out_packed is [Q*S] (row-major). */
int alut_search_packed(const alut_tables_t* tables, const alut_batch_t* batch,
                       const alut_search_params_t* params, const void* q_low_in,
                       int64_t idx_offset, uint64_t* out_packed, void* workspace,
                       size_t workspace_bytes, alut_stream_t stream);

/* Merge `world` packed candidate arrays ([world][n], contiguous) by max and apply the
 * threshold rule of params to give hit/idx for n = Q*S slots (row-major, no gaps).
 * is_vision may be NULL (all text). Slots whose candidates are all 0 miss. */
int alut_merge_packed(int32_t world, int32_t q, int32_t s, const uint64_t* packed_all,
                      const uint8_t* is_vision, const alut_search_params_t* params,
                      uint8_t* out_hit, int64_t* out_idx, alut_stream_t stream);

/* a6: the online window lookup of the hybrid decode search (search.py:778-806). x [b,h]
 * (x_dtype, row stride x_stride) against the window's first n_valid keys [.,h] (key_dtype
 * == x_dtype, row stride key_stride, 16-byte aligned): scores rounded to that dtype (the
 * reference's matmul output dtype), first index of the maximum, valid iff > 0. eids [.,t]
 * int64 (row stride t) are the window's cached expert ids; target [b,s] (row stride
 * target_stride) the experts of the slots searched online. Writes on_idx[b] (-1 if
 * invalid), on_hit [b,s] u8 and on_slot [b,s] int64 (row stride out_stride elements each):
 * on_hit = valid and target among eids[on_idx]; on_slot = its first position, 0 without a
 * hit (the reference leaves those untouched in buffers its callers pre-zero). */
int alut_online_search(int32_t b, int32_t h, int32_t n_valid, int32_t t, int32_t s, const void* x,
                       int32_t x_dtype, int64_t x_stride, const void* keys, int32_t key_dtype, int64_t key_stride,
                       const int64_t* eids, const int64_t* target, int64_t target_stride, uint8_t* on_hit,
                       int64_t* on_idx, int64_t* on_slot, int64_t out_stride, alut_stream_t stream);

/* ---- peer access for the centroid-range shards (new; no reference counterpart) ----------
 * Each rank exports the device allocation holding its value slice as a CUDA IPC handle
 * (ALUT_PEER_HANDLE_BYTES bytes, plus the slice's offset inside the allocation), the
 * ranks exchange them over their process group, and each opens its peers' handles (peer
 * access over NVLink, no multicast). alut_peer_close undoes alut_peer_open. */
#define ALUT_PEER_HANDLE_BYTES 64
int alut_peer_export(const void* ptr, void* handle, uint64_t* offset);
int alut_peer_open(const void* handle, uint64_t offset, void** ptr);
int alut_peer_close(void* ptr, uint64_t offset);

/* out[i] (row stride out_stride elements) = the value row of centroid idx[i] (global index)
 * and modality (is_vision[i] ? 0 : 1), read from the shard that owns it; zeros where
 * hit[i] == 0. shard_values, shard_start and shard_stride_m are DEVICE arrays: world
 * pointers to each shard's [2][Kr][H] value slice (the caller's own and its peers'
 * alut_peer_open mappings), world + 1 centroid boundaries, and each slice's modality
 * stride in elements; every slice has row stride value_stride_k. Rows are h elements of
 * value_dtype, a whole number of 16-byte units. Replaces the gather + reduce-scatter row
 * exchange of the sharded lookup: each remote row crosses NVLink once. */
int alut_gather_rows_sharded(int32_t n, const uint8_t* hit, const int64_t* idx, const uint8_t* is_vision,
                             int32_t world, const void* const* shard_values, const int64_t* shard_start,
                             const int64_t* shard_stride_m, int64_t value_stride_k, int32_t h, int32_t value_dtype,
                             void* out, int64_t out_stride, alut_stream_t stream);

/* alut_lookup_combine for callers that cannot allocate device memory: those handed only
 * their input and output buffers by another runtime (an FFI host without access to the
 * CUDA allocator, a serving loop that forbids cudaMalloc after start-up because it can
 * synchronise the device). It has no counterpart in the reference. Its scratch is a
 * fixed 2 MiB array inside this library (held by every GPU that loads the library until
 * the process exits). A batch is rejected with ALUT_ERANGE when the scratch of the
 * CUDA-core scans (workspace layout without the tensor-core part) exceeds
 * ALUT_NOALLOC_SCRATCH_BYTES; a batch that would take the tensor-core scan uses it only
 * when that larger layout also fits, and otherwise runs the CUDA-core scan (same results).
 * The first call on a device (and on each new CUDA context of it, e.g. after a
 * cudaDeviceReset) looks up the array's device address: make it before any stream
 * capture. All calls on a device share the array: calls that may overlap on the GPU
 * (different streams without ordering between them) race and give wrong results. The
 * error bits of the array are cleared at the start of every call (read them with
 * alut_workspace_errors(NULL, ...)). It calls no cudaMalloc/cudaFree. */
#define ALUT_NOALLOC_SCRATCH_BYTES (2u << 20)
int alut_lookup_combine_noalloc(const alut_tables_t* tables, const alut_batch_t* batch,
                                const alut_search_params_t* params, const float* weights,
                                int64_t weight_stride, const uint8_t* compute_mask,
                                int64_t compute_stride, int32_t renorm, int32_t accumulate,
                                void* out, int64_t out_stride, int32_t out_dtype,
                                uint8_t* out_hit, int64_t* out_idx, int64_t out_stride_hit,
                                alut_stream_t stream);

/* ---- router prologue (table_moe/ops/qwen_topk_softmax.py:122-153, skip/pruning.py:4-52) ----
 * Which slots a layer computes; the others are looked up (cached_layers.py:336-337). */
typedef enum alut_keep_mode {
  ALUT_KEEP_FIXED = 0,      /* slots [0, keep_k) of every token computed: build_fixed_keep_mask /
                               build_decode_keep_mask (pruning.py:4-15, :51); keep_k < 0 = all */
  ALUT_KEEP_IMPORTANCE = 1, /* build_prefill_keep_mask (pruning.py:18-48) */
} alut_keep_mode_t;

/* Bytes of the workspace of alut_route for num_experts experts (zero-filled once; the
 * kernels leave it zeroed). 0 for invalid sizes. */
size_t alut_route_workspace_size(int32_t num_experts);

/* Top-k softmax routing and keep mask of q tokens in one call:
 *   probabilities = softmax(fp32(logits[t, :num_experts])) (logits f32/bf16/f16, row stride
 *   logits_stride); weights[t, s], sel[t, s] = the top_k largest in descending order (lower
 *   expert id first among equal probabilities); with normalize_topk the weights are divided
 *   by max(their sum, 1e-20) (qwen_topk_softmax.py:150-151);
 *   compute[t, s] = 1 for computed slots, reuse[t, s] = 1 - compute[t, s] for looked-up ones:
 *     ALUT_KEEP_FIXED: s < keep_k;
 *     ALUT_KEEP_IMPORTANCE: expert sel[t, s] is among the first max(1, int(n_active *
 *       keep_rate)) activated experts ranked by the sum over their slots of
 *       attn[t] * weights[t, s] (attn != NULL) or weights[t, s] / q (larger sum first, lower
 *       id on equal sums; sums are accumulated exactly in 2^-40 fixed point, |sum| < 2^23).
 * Outputs are [q, top_k] with row stride out_stride (elements). top_k <= 64 and
 * top_k <= num_experts <= 4096. Replaces qwen_topk_softmax followed by _build_compute_mask
 * (qwen3_vl_moe/cached_layers.py:69-84, :282-286, :336). */
int alut_route(int32_t q, int32_t num_experts, int32_t top_k, const void* logits, int32_t logits_dtype,
               int64_t logits_stride, int32_t normalize_topk, int32_t keep_mode, int32_t keep_k,
               double keep_rate, const float* attn, float* weights, int64_t* sel, uint8_t* compute,
               uint8_t* reuse, int64_t out_stride, void* workspace, size_t workspace_bytes,
               alut_stream_t stream);

/* The importance keep mask alone, for routing computed elsewhere (build_prefill_keep_mask,
 * pruning.py:18-48): sel/weights [q, top_k] (row stride in_stride) in, compute/reuse out
 * (row stride out_stride), same rule and workspace as alut_route's ALUT_KEEP_IMPORTANCE.
 * Expert ids outside [0, num_experts) are never kept. */
int alut_keep_mask(int32_t q, int32_t num_experts, int32_t top_k, const int64_t* sel, const float* weights,
                   int64_t in_stride, const float* attn, double keep_rate, uint8_t* compute, uint8_t* reuse,
                   int64_t out_stride, void* workspace, size_t workspace_bytes, alut_stream_t stream);

/* Load-time key normalisation (table_moe/cache_engine/manager.py:24-31, :205-207): for each
 * of `rows` rows of l elements (dtype, row strides in elements; dst may equal src)
 * dst = src / max(||src||, eps) computed in fp32, zero rows (||src|| <= eps) kept at zero,
 * rounded to dtype. Makes keys_buffer from raw_keys_buffer on the device. */
int alut_normalize_rows(int64_t rows, int32_t l, const void* src, int64_t src_stride, void* dst, int64_t dst_stride,
                        int32_t dtype, float eps, alut_stream_t stream);

/* Device-side error bits of a workspace (or, with workspace NULL, of the no-allocation
 * entry point's scratch). Kernels set them and never clear them, so they accumulate over
 * every call that used the workspace until this function clears them (clear != 0). It
 * waits for the stream (cudaStreamSynchronize), so it belongs in debug checks, not on the
 * hot path. A set bit means some slot's result is wrong (a bad id leaves its slot a miss;
 * a timed-out wait leaves its tile unscored); the reference raises IndexError for the
 * first and has no counterpart of the others. */
#define ALUT_ERR_BAD_EXPERT 1u  /* a searched slot's expert id is outside [0, num_experts) */
#define ALUT_ERR_COPY_TIMEOUT 4u /* a key-chunk copy did not land within 1 s */
#define ALUT_ERR_MMA_TIMEOUT 8u  /* a tensor-core pipeline wait ran out (1 s) */
int alut_workspace_errors(void* workspace, size_t workspace_bytes, int32_t clear, uint32_t* bits,
                          alut_stream_t stream);

/* Profiling hook: when both events are set (cudaEvent_t handles), every following
 * centroid-scan launch made by this thread is bracketed by event records on its stream
 * (as external event nodes when the stream is being captured into a CUDA graph), so the
 * caller can time that kernel alone with cudaEventElapsedTime. Pass NULL, NULL to stop.
 * The events are not owned by the library. */
int alut_set_profile_events(void* start_event, void* stop_event);

/* Text of the last error seen by this thread (never NULL). */
const char* alut_last_error(void);

/* Library version, as major*10000 + minor*100 + patch. */
int alut_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ALUT_H_ */
