/*
 * dwa.h - C ABI of libdwa.so, the B200 (sm_100a) implementation of the DWA
 * (dynamic weight assembly) retrieval + assembly hot path of theorionic/matrix.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, a cudaStream_t), enqueues its work on that stream and
 * returns without synchronising.  No entry point allocates device memory:
 * scratch space is the caller's `workspace`, sized by the matching
 * *_workspace_bytes() query.  Buffers are owned by the caller and are not
 * retained after the call returns.
 *
 * Return value: DWA_OK (0) or a negative DWA_ERR_* code; dwa_last_error()
 * gives the message of the last failure on the calling thread.  Errors found
 * on the device (a row index outside the pool, a wait that ran out) are
 * recorded in a status word inside the workspace; dwa_workspace_status() reads
 * it (that call synchronises the stream).
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   dwa_assemble_fwd   src/dwa/assembly_pallas.py:193-222  pallas_assemble (primal)
 *                      src/dwa/assembly_pallas.py:139-181  _pallas_assemble_forward
 *                      src/dwa/assembly_pallas.py:42-75    assemble_jax (same values)
 *                      src/dwa/model.py:184-195            pool gather (row_index form)
 *   dwa_assemble_bwd   src/dwa/assembly_pallas.py:246-329  _pallas_assemble_bwd
 *   dwa_retrieve       src/dwa/retrieval.py:48-159         MultiAspectRetrieval.__call__
 *   dwa_retrieve_local src/dwa/retrieval.py:74-79, 121-138 model-sharded retrieval
 *   dwa_retrieve_merge src/dwa/model.py:16-47              _distributed_gather of the winners
 *   dwa_key_cache      src/dwa/assembly_pallas.py:392-400  compute_key_cache
 *                      src/dwa/pool.py:37-44               VectorPool.compute_keys
 *   dwa_centroid_ema   train.py:318-328                    centroid EMA of the IVF lists
 *   dwa_rmsnorm_fwd/bwd src/dwa/assembly.py:29, model.py:207 nnx.RMSNorm after the assembly
 *   dwa_pool_grad_scatter src/dwa/model.py:193-195        VJP of the pool gather
 */
#ifndef DWA_H_
#define DWA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DWA_ABI_VERSION 1

#if defined(__GNUC__)
#define DWA_API __attribute__((visibility("default")))
#else
#define DWA_API
#endif

/* status codes */
#define DWA_OK                0
#define DWA_ERR_INVALID_ARG  -1   /* a size, dtype or pointer argument is invalid */
#define DWA_ERR_UNSUPPORTED  -2   /* valid but not supported by this build       */
#define DWA_ERR_CUDA         -3   /* a CUDA runtime / driver call failed          */
#define DWA_ERR_WORKSPACE    -4   /* workspace missing, too small or misaligned   */
#define DWA_ERR_DEVICE       -5   /* the device status word reports an error      */

/* element types */
#define DWA_F32   0
#define DWA_BF16  1

/* bits of the device status word */
#define DWA_STATUS_BAD_ROW_INDEX   0x1u  /* a row index outside [0, n_rows)            */
#define DWA_STATUS_WAIT_TIMEOUT    0x2u  /* a bounded device wait gave up              */
#define DWA_STATUS_BAD_LIST        0x4u  /* list offsets not monotone / out of range   */
#define DWA_STATUS_LIST_OVERFLOW   0x8u  /* a probed list longer than max_list         */
#define DWA_STATUS_FEW_CANDIDATES  0x10u /* fewer candidates than k (tail padded, a=0)  */

/* Shape of one assembly call.  h_A is [B,T,d_A], pool rows are [.., D] with the
 * reference layout [U (d_B x r) | V (r x d_A) | b (d_B) | pad]
 * (src/dwa/config.py:159-165).  The reference requires d_A == d_B. */
typedef struct DwaAssembleDims {
    int32_t B, T, k, D, d_A, d_B, r;
    int32_t act_dtype;   /* DWA_F32 or DWA_BF16: h_A, h_mid, g_hmid, g_hA, W_act */
    int32_t rows_dtype;  /* DWA_F32 or DWA_BF16: element type of `rows`          */
    int32_t reserved;
    int64_t n_rows;      /* rows in `rows` when row_index != NULL (bounds check) */
} DwaAssembleDims;

/* Shape of one retrieval call (src/dwa/retrieval.py:48-159). */
typedef struct DwaRetrieveDims {
    int32_t B, S, d_k, d_A;
    int32_t C;           /* number of lists (centroids); ignored when use_ivf == 0 */
    int32_t m;           /* lists probed per query (min(m, C) is used)              */
    int32_t k;           /* k_max: vectors selected per query                       */
    int32_t max_list;    /* rows in the longest list (bounds candidate scratch)     */
    int64_t N;           /* pool rows                                               */
    float   T;           /* temperature                                             */
    int32_t z_dtype;     /* DWA_F32 or DWA_BF16                                     */
} DwaRetrieveDims;

DWA_API const char* dwa_version(void);
DWA_API int         dwa_abi_version(void);
DWA_API const char* dwa_status_string(int status);
/* Copies the last error message of this thread into buf (NUL-terminated);
 * returns the message length. */
DWA_API int         dwa_last_error(char* buf, size_t buf_bytes);

/* Kernels launched by this library since it was loaded (all threads and
 * devices): total, and how many GEMMs ran on the tensor cores (tcgen05) or on
 * the CUDA cores (fp32 path and shapes TMA cannot address).  No reference
 * counterpart; used to count launches inside a timed region. */
DWA_API void dwa_launch_counters(uint64_t* total, uint64_t* tensor_core_gemms, uint64_t* simt_gemms);

/* Kernel timing hook (no reference counterpart).  While registered, the
 * library records `start_event` on the launching stream just before every
 * launch of the kernel named `kernel` and `stop_event` just after it (both are
 * cudaEvent_t passed as void*).  Names: "query", "coarse", "topm", "fine",
 * "full_scores", "select", "softmax_stats", "softmax_apply", "prep_factors",
 * "prep_bias", "gemm_W", "gemm_apply", "gemm_G", "gemm_gh", "gemm_P",
 * "gemm_Q", "colsum", "finalize", "bias_grad", "seq_mean", "merge",
 * "key_cache", "centroid_ema", "rmsnorm_fwd", "rmsnorm_bwd", "scatter_sort",
 * "scatter_add", "grad_send", "gather_rows", "peer_allgather", "key_grad", "sel_grad",
 * "aux_query", "aux_norm", the decode kernels ("factored_hv", "factored_out",
 * "factored_combine", "base_rows", "cast_w_base", "gemm_base") and
 * "probe_lists"; up to 64 entries.  Passing NULL events removes the entry;
 * dwa_profile_clear() removes all. */
DWA_API int  dwa_profile_kernel(const char* kernel, void* start_event, void* stop_event);
DWA_API void dwa_profile_clear(void);

/* Profiling control: with on != 0, launches that follow use no programmatic
 * dependent launch and the calls' concurrent lanes collapse onto the caller's
 * stream, so each kernel runs alone and the event pairs of dwa_profile_kernel
 * add up to the step.  Off by default; affects launches (and graph captures)
 * made while it is set.  Not thread-scoped: set it only around a profiling
 * pass. */
DWA_API void dwa_profile_serialize(int on);

/* z[b,:] = mean over t of h_A[b,t,:] in float32 (the retrieval query of
 * src/dwa/model.py:171).  h_A [B,T,d] in dtype; z [B,d] f32. */
DWA_API int dwa_sequence_mean(void* stream, int B, int T, int d, int dtype, const void* h_A,
                              float* z);

/* Reads and (if clear != 0) clears the device status word stored in a
 * workspace used by any entry point.  Synchronises `stream`. */
DWA_API int dwa_workspace_status(void* stream, void* workspace, uint32_t* status, int clear);

/* ---------------------------------------------------------------------------
 * Assembly forward.  Replaces pallas_assemble's primal
 * (src/dwa/assembly_pallas.py:193-222, kernel :85-132, pre-factoring :139-181):
 *   W[b]     = W_base + sum_k alpha[b,k] * U_k V_k          (fp32, [B,d_B,d_A])
 *   h_mid[b] = h_A[b] + gamma * h_A[b] W[b]^T + b_base + sum_k alpha[b,k] b_k
 * `rows`: either the gathered rows [B,k,D] (row_index == NULL, as the reference
 * receives them) or the whole pool [n_rows, D] with row_index [B,k] int32
 * selecting each (b,k) row (the gather of src/dwa/model.py:184-195 fused in).
 * alphas [B,k] f32; W_base [d_B,d_A] f32; b_base [d_B] f32; gamma: 1 f32 on
 * the device.  Outputs: h_mid [B,T,d_B] (act_dtype); W_out [B,d_B,d_A] f32 or
 * NULL; W_act [B,d_B,d_A] in act_dtype or NULL (the backward's residual; for
 * act_dtype == DWA_F32 it may be the same buffer as W_out).
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_assemble_workspace_bytes(const DwaAssembleDims* dims, int with_backward);

DWA_API int dwa_assemble_fwd(void* stream, const DwaAssembleDims* dims,
                     const void* rows, const int32_t* row_index,
                     const float* alphas, const void* h_A,
                     const float* W_base, const float* b_base, const float* gamma,
                     void* h_mid, float* W_out, void* W_act,
                     void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Assembly apply, h_mid only.  Replaces the Pallas kernel itself
 * (src/dwa/assembly_pallas.py:85-132 with the pre-factoring of :139-181) when
 * the caller does not use W (generation, train.py:615-616, where XLA drops the
 * W recompute of :212-221):
 *   h_mid[b] = h_A[b] + gamma (h_A[b] W_base^T + (h_A[b] V_s^T) U_f) + pb[b]
 * Same arguments and meaning as dwa_assemble_fwd without W_out / W_act.  For
 * T <= 16 rows per sequence it runs the factored form (each gathered row read
 * once, W never formed); longer sequences take dwa_assemble_fwd's path.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_assemble_apply_workspace_bytes(const DwaAssembleDims* dims);

DWA_API int dwa_assemble_apply(void* stream, const DwaAssembleDims* dims,
                     const void* rows, const int32_t* row_index,
                     const float* alphas, const void* h_A,
                     const float* W_base, const float* b_base, const float* gamma,
                     void* h_mid, void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Assembly backward.  Replaces _pallas_assemble_bwd
 * (src/dwa/assembly_pallas.py:246-329) for the residuals
 * (rows/row_index, alphas, h_A, W, gamma) and cotangents (g_hmid, g_W_out).
 * W_act: the assembled W in act_dtype (the forward's W_act output).
 * g_W_out [B,d_B,d_A] f32 may be NULL (zero cotangent of W).
 * Outputs (all written in full):
 *   g_rows [B,k,D] f32   gradient of the gathered rows (pad columns zero)
 *   g_alpha [B,k] f32, g_hA [B,T,d_A] act_dtype, g_W_base [d_B,d_A] f32,
 *   g_b_base [d_B] f32, g_gamma [1] f32.
 * ------------------------------------------------------------------------- */
DWA_API int dwa_assemble_bwd(void* stream, const DwaAssembleDims* dims,
                     const void* rows, const int32_t* row_index,
                     const float* alphas, const void* h_A, const void* W_act,
                     const float* gamma, const void* g_hmid, const float* g_W_out,
                     float* g_rows, float* g_alpha, void* g_hA, float* g_W_base,
                     float* g_b_base, float* g_gamma,
                     void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Retrieval.  Replaces MultiAspectRetrieval.__call__ (src/dwa/retrieval.py:48-159)
 * on one device.  Parameters: W_Q [S,d_k,d_A] f32, aspect_weights [S] f32,
 * tau [1] f32, centroids [S,C,d_k] f32 (IVF only); list_offsets [C+1] int64
 * CSR row ranges of the lists (list c = rows [off[c], off[c+1]); the
 * reference's equal lists are off[c] = c*N/C); pool_keys [S,N,d_k] f32;
 * z [B,d_A] (z_dtype); lambda_val [1] f32 on the device.
 * use_ivf != 0: coarse scoring + top-m lists + fine scoring of the probed
 * lists (retrieval.py:81-119); use_ivf == 0: full search (:121-138).
 * is_warmup != 0: top-k of s_i + softmax (:143-147); else sigmoid-gated
 * selection (:149-156).  Ties between equal scores go to the lower pool row.
 * Outputs: alphas [B,k] f32, indices [B,k] int32 (pool rows, ordered by
 * descending score), soft_full [B,N] f32 = softmax(s_full / T) or NULL.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_retrieve_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf,
                                    int want_soft_full);

DWA_API int dwa_retrieve(void* stream, const DwaRetrieveDims* dims, int use_ivf, int is_warmup,
                 const float* lambda_val, const void* z, const float* W_Q,
                 const float* aspect_weights, const float* tau, const float* centroids,
                 const int64_t* list_offsets, const float* pool_keys,
                 float* alphas, int32_t* indices, float* soft_full,
                 void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Row-sharded retrieval over P ranks.  Replaces the model-sharded branch of
 * MultiAspectRetrieval.__call__ (src/dwa/retrieval.py:74-79, 121-138: IVF off,
 * every rank scores its pool rows, scores all-gathered) and the masked-psum
 * gather of the winners (src/dwa/model.py:16-47), keeping IVF on: rank p
 * holds the keys of pool rows [row_lo, row_lo + N) (whole lists, or any
 * contiguous slice); centroids, W_Q, aspect weights, tau and the global
 * list_offsets are replicated.  Per call:
 *   1. dwa_retrieve_local on every rank: the same coarse top-m lists, the
 *      rank's part of them scored, its top-k written as a summary
 *      [B, 2k+3] f32 (k scores best first, k global rows as int32 bits, the
 *      partial gate sum, the soft_full max and sum of exp(s/T - max)), and
 *      soft_full (if given) [B, N] left as raw scores of the rank's rows.
 *   2. an all-gather of the summaries into [P, B, 2k+3] (NCCL, by the caller).
 *   3. dwa_retrieve_merge on every rank: the global top-k (ties to the lower
 *      pool row), alphas and indices exactly as dwa_retrieve defines them,
 *      and the rank's soft_full slice normalised with the merged statistics.
 * The result equals dwa_retrieve on the whole pool (indices bit-exact; alphas
 * and soft_full up to the order of the partial sums).
 * dims: the local call's N is the rank's row count (workspace from
 * dwa_retrieve_workspace_bytes with those dims); the merge's N is the row
 * count of the soft_full slice it normalises (0 without soft_full).
 * ------------------------------------------------------------------------- */
typedef struct DwaShard {
    int64_t row_lo;    /* global pool row of the rank's first key row */
    int64_t n_global;  /* rows of the whole pool (< 2^31) */
} DwaShard;

DWA_API int dwa_retrieve_local(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard,
                               int use_ivf, int is_warmup, const float* lambda_val, const void* z,
                               const float* W_Q, const float* aspect_weights, const float* tau,
                               const float* centroids, const int64_t* list_offsets,
                               const float* pool_keys, float* summary, float* soft_full,
                               void* workspace, size_t workspace_bytes);

DWA_API size_t dwa_retrieve_merge_workspace_bytes(const DwaRetrieveDims* dims);

DWA_API int dwa_retrieve_merge(void* stream, const DwaRetrieveDims* dims, int world,
                               const float* summaries, int is_warmup, const float* lambda_val,
                               const float* tau, float* alphas, int32_t* indices, float* soft_full,
                               void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Retrieval VJP.  The backward that jax.vjp derives for
 * MultiAspectRetrieval.__call__ (src/dwa/retrieval.py:64-158): the cotangents
 * g_alphas [B,k] and g_soft_full [B,N] (f32; either may be NULL) of the
 * forward's outputs back to
 *   g_z [B,d_A] f32, g_W_Q [S,d_k,d_A], g_aspect_weights [S], g_tau [1]
 * and, when g_pool_keys is non-NULL, the key cache g_pool_keys [S,N,d_k]
 * (B <= 32).  The forward's alphas and indices (with g_alphas) and its
 * normalised soft_full (with g_soft_full) are inputs; the queries, the probed
 * lists and the candidate scores are recomputed from the same arguments as
 * dwa_retrieve's.  indices and the coarse top-m carry no gradient (integer /
 * piecewise constant), so centroids get none.  Every output is overwritten;
 * reductions run in a fixed order.  Needs d_k % 4 == 0 and S*d_k <= 1024.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_retrieve_bwd_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf);
DWA_API int dwa_retrieve_bwd(void* stream, const DwaRetrieveDims* dims, int use_ivf, int is_warmup,
                             const float* lambda_val, const void* z, const float* W_Q,
                             const float* aspect_weights, const float* tau, const float* centroids,
                             const int64_t* list_offsets, const float* pool_keys, const float* alphas,
                             const int32_t* indices, const float* soft_full, const float* g_alphas,
                             const float* g_soft_full, float* g_z, float* g_W_Q,
                             float* g_aspect_weights, float* g_tau, float* g_pool_keys,
                             void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Retrieval VJP over a row-sharded pool (the backward of dwa_retrieve_local +
 * dwa_retrieve_merge): dims->N = the rank's rows, shard->row_lo its first
 * global row; the same workspace (dwa_retrieve_bwd_local_workspace_bytes) goes
 * to the three phases of one call.
 *   phase 1 (dwa_retrieve_bwd_local1): part1 [B, k+3] = the scores of the
 *     winners this rank holds (0 for the others), Σ raw over its candidates,
 *     Σ g_soft·soft over its rows, its candidate count;
 *   the caller sums part1 over the ranks (one all-reduce);
 *   phase 2 (dwa_retrieve_bwd_local2): dL/ds on this rank's rows from the sums,
 *     the key pass over them; part2 [B, S*d_k+1] = this rank's A and g_tau
 *     share; its key gradient when g_pool_keys is non-NULL (B <= 32);
 *   the caller sums part2 over the ranks (one all-reduce);
 *   phase 3 (dwa_retrieve_bwd_finish): g_z, g_W_Q, g_aspect_weights, g_tau
 *     (needs no rows: a rank that holds none passes zero partials to the sums
 *     and runs only this phase, with dims->N = 1 and its own workspace).
 * soft_full / g_soft_full are the rank's [B, N] slices; alphas, indices,
 * g_alphas are the merged [B, k] values every rank holds.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_retrieve_bwd_local_workspace_bytes(const DwaRetrieveDims* dims, int use_ivf);
DWA_API int dwa_retrieve_bwd_local1(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard,
                                    int use_ivf, int is_warmup, const float* lambda_val, const void* z,
                                    const float* W_Q, const float* aspect_weights, const float* tau,
                                    const float* centroids, const int64_t* list_offsets,
                                    const float* local_keys, const int32_t* indices,
                                    const float* soft_full, const float* g_soft_full, float* part1,
                                    void* workspace, size_t workspace_bytes);
DWA_API int dwa_retrieve_bwd_local2(void* stream, const DwaRetrieveDims* dims, const DwaShard* shard,
                                    int use_ivf, int is_warmup, const float* lambda_val, const float* tau,
                                    const float* aspect_weights, const int64_t* list_offsets,
                                    const float* local_keys, const float* alphas, const int32_t* indices,
                                    const float* soft_full, const float* g_alphas,
                                    const float* g_soft_full, const float* part1_sum, float* part2,
                                    float* g_pool_keys, void* workspace, size_t workspace_bytes);
DWA_API int dwa_retrieve_bwd_finish(void* stream, const DwaRetrieveDims* dims, int use_ivf, const void* z,
                                    const float* W_Q, const float* aspect_weights,
                                    const float* part2_sum, float* g_z, float* g_W_Q,
                                    float* g_aspect_weights, float* g_tau, void* workspace,
                                    size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Peer access to a row-sharded pool (one process per GPU, one node).  Replaces
 * _distributed_gather (src/dwa/model.py:16-47), which all-reduces B*k*D values
 * over the model axis, by direct reads of the owning rank's rows.
 *   dwa_ipc_handle: the CUDA IPC handle (dwa_ipc_handle_bytes() bytes) of the
 *     allocation holding ptr, and ptr's byte offset in it;
 *   dwa_ipc_open / dwa_ipc_close: map / unmap a peer's handle (+ offset);
 *   dwa_gather_rows: out[i, :] = pool row indices[i] for i < n, read from the
 *     shard that holds it (plain 16-byte loads, NVLink for peers' rows); rows
 *     outside [row_lo[0], row_lo[world]) set DWA_STATUS_BAD_ROW_INDEX in the
 *     workspace's status word and come out as zeros.  D * element size must be
 *     a multiple of 16 bytes; n <= 65535 per call.
 * ------------------------------------------------------------------------- */
typedef struct DwaPoolShards {
    int32_t world;               /* <= 16 */
    const void* const* bases;    /* host array [world]: device pointer of rank r's first row */
    const int64_t* row_lo;       /* host array [world + 1]: rank r holds global rows [row_lo[r], row_lo[r+1]) */
} DwaPoolShards;
DWA_API size_t dwa_ipc_handle_bytes(void);
DWA_API int dwa_ipc_handle(const void* ptr, void* handle, int64_t* offset);
DWA_API int dwa_ipc_open(const void* handle, int64_t offset, void** ptr);
DWA_API int dwa_ipc_close(void* ptr, int64_t offset);
DWA_API size_t dwa_gather_rows_workspace_bytes(void);
DWA_API int dwa_gather_rows(void* stream, int n, int64_t D, int dtype, const int32_t* indices,
                            const DwaPoolShards* shards, void* out, void* workspace,
                            size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Auxiliary losses.  Replaces aux_losses (src/dwa/losses.py:9-73) and its
 * jax.grad: from the forward's alphas [B,k], indices [B,k], the key cache
 * [S,N,d_k], the assembled W [B,d_B,d_A] f32, W_base [d_B,d_A] and the
 * normalised soft_full [B,N],
 *   losses[5] = {l_util, l_div, l_norm, l_sparse, total_aux}
 * with total_aux = Σ lambda * loss (TrainConfig.lambda_*, config.py:181-184),
 * and the gradients of total_aux (each output may be NULL):
 *   g_alphas [B,k], g_soft_full [B,N], g_W [B,d_B,d_A], g_W_base [d_B,d_A]
 *   (overwritten), g_pool_keys [S,N,d_k] (ADDED into, at the retrieved rows,
 *   so it composes with dwa_retrieve_bwd's key gradient).
 * B*k <= 8192; reductions in a fixed order.
 * ------------------------------------------------------------------------- */
typedef struct DwaAuxDims {
    int32_t B, k, S, d_k, d_B, d_A;
    int64_t N;
} DwaAuxDims;
typedef struct DwaAuxWeights {
    float util, div, norm, sparse;   /* lambda_util, lambda_div, lambda_norm, lambda_sparse */
} DwaAuxWeights;
/* Over a row-sharded pool: this rank holds pool / key / soft_full rows
 * [row_lo, row_lo + dims->N) of n_global and the assembled W of w_batch of the
 * dims->B sequences (its own).  Phase 1 (dwa_aux_losses_local): part [2] =
 * this rank's shares of l_util's and l_norm's sums, rk_part [B, k, d_k] = the
 * aspect-mean keys of the winners it holds (zeros elsewhere), g_soft_full of
 * its rows, g_W of its sequences, its share of g_W_base.  The caller sums
 * part, rk_part and g_W_base over the ranks.  Phase 2 (dwa_aux_losses_finish,
 * the same workspace size): losses[5], g_alphas, and l_div's key gradient
 * added into this rank's rows of g_pool_keys. */
typedef struct DwaAuxShard {
    int64_t row_lo, n_global;
    int32_t w_batch;
} DwaAuxShard;
DWA_API size_t dwa_aux_losses_workspace_bytes(const DwaAuxDims* dims);
DWA_API int dwa_aux_losses(void* stream, const DwaAuxDims* dims, const DwaAuxWeights* lambdas,
                           const float* alphas, const int32_t* indices, const float* pool_keys,
                           const float* W, const float* W_base, const float* soft_full,
                           float* losses, float* g_alphas, float* g_soft_full, float* g_W,
                           float* g_W_base, float* g_pool_keys, void* workspace,
                           size_t workspace_bytes);
DWA_API int dwa_aux_losses_local(void* stream, const DwaAuxDims* dims, const DwaAuxShard* shard,
                                 const DwaAuxWeights* lambdas, const int32_t* indices,
                                 const float* local_keys, const float* W, const float* W_base,
                                 const float* soft_full, float* part, float* rk_part,
                                 float* g_soft_full, float* g_W, float* g_W_base_part,
                                 void* workspace, size_t workspace_bytes);
DWA_API int dwa_aux_losses_finish(void* stream, const DwaAuxDims* dims, const DwaAuxShard* shard,
                                  const DwaAuxWeights* lambdas, const float* alphas,
                                  const int32_t* indices, const float* part_sum, const float* rk_sum,
                                  float* losses, float* g_alphas, float* g_pool_keys, void* workspace,
                                  size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Key cache.  Replaces compute_key_cache (src/dwa/assembly_pallas.py:392-400) and
 * VectorPool.compute_keys (src/dwa/pool.py:37-44): keys [S,N,d_k] f32 =
 * einsum("nd,sda->sna", pool_vectors [N,D], key_proj [S,D,d_k]) in fp32, both
 * inputs of `dtype` (DWA_BF16: tcgen05 GEMM, DWA_F32: CUDA-core GEMM).  Called
 * once per training window (train.py:253-256).
 * ------------------------------------------------------------------------- */
typedef struct DwaKeyCacheDims {
    int64_t N;       /* pool rows */
    int32_t D;       /* pool row width */
    int32_t S;       /* aspects */
    int32_t d_k;     /* key dim per aspect */
    int32_t dtype;   /* DWA_F32 or DWA_BF16: pool_vectors and key_proj */
} DwaKeyCacheDims;

DWA_API size_t dwa_key_cache_workspace_bytes(const DwaKeyCacheDims* dims);

DWA_API int dwa_key_cache(void* stream, const DwaKeyCacheDims* dims, const void* pool_vectors,
                          const void* key_proj, float* keys, void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Centroid EMA.  Replaces train.py:318-328: centroids [S,C,d_k] f32 (in place)
 * = decay * centroids + (1 - decay) * mean of the keys of each list (CSR
 * list_offsets [C+1] into keys [S,N,d_k]); the reference uses decay 0.9 with
 * equal lists.  Empty lists keep their centroid.  workspace: >= 256 bytes,
 * 256-byte aligned, its first word the device status.
 * ------------------------------------------------------------------------- */
DWA_API int dwa_centroid_ema(void* stream, int S, int C, int d_k, int64_t N, const float* keys,
                             const int64_t* list_offsets, float decay, float* centroids,
                             void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * RMSNorm of the assembly output.  Replaces the assembler's layer_norm
 * (flax nnx.RMSNorm(d_B), src/dwa/assembly.py:29, applied at
 * src/dwa/model.py:207-219): over rows of x [rows, d] (x_dtype),
 *   y = x * (rsqrt(mean(x^2) + eps) * scale),  scale [d] f32, eps 1e-6 in flax,
 * statistics in fp32, y [rows, d] in y_dtype (flax promotes bf16 x with its fp32
 * scale to fp32), rstd [rows] f32 saved for the backward.  The backward takes
 * g_y [rows, d] (g_dtype) and writes g_x [rows, d] (x_dtype) and g_scale [d]
 * f32 (overwritten; deterministic).  d % 8 == 0, 16-byte aligned rows.
 * ------------------------------------------------------------------------- */
DWA_API int dwa_rmsnorm_fwd(void* stream, int64_t rows, int d, int x_dtype, int y_dtype, const void* x,
                            const float* scale, float eps, void* y, float* rstd);

DWA_API size_t dwa_rmsnorm_bwd_workspace_bytes(int64_t rows, int d);

DWA_API int dwa_rmsnorm_bwd(void* stream, int64_t rows, int d, int x_dtype, int g_dtype, const void* x,
                            const float* scale, const float* rstd, const void* g_y, void* g_x,
                            float* g_scale, void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Pool-row gradient scatter: the VJP of the gather pool[indices]
 * (src/dwa/model.py:193-195; of _distributed_gather, model.py:16-47, with the
 * pool row-sharded).  For the n contributions g_rows [n, D] f32 of pool rows
 * indices [n] int32 (the backward's g_rows [B,k,D] and the retrieval indices),
 *   g_pool[row - row_lo, :] += sum of the g_rows of that row
 * over the rows inside [row_lo, row_hi) of an n_global-row pool; g_pool is
 * [row_hi - row_lo, D] in g_dtype (DWA_F32 or DWA_BF16, rounded once per row).
 * Rows of other windows are skipped; rows outside [0, n_global) set
 * DWA_STATUS_BAD_ROW_INDEX.  Deterministic (no atomics); n <= 8192 per call.
 * Rows not selected are left as they are: pass a zeroed g_pool for the dense
 * gradient the reference's autodiff forms.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_pool_grad_scatter_workspace_bytes(int n);

/* Index value of an empty slot: skipped by the scatter without a status bit. */
#define DWA_PAD_INDEX (-2147483647 - 1)

DWA_API int dwa_pool_grad_scatter(void* stream, int n, int D, const int32_t* indices, const float* g_rows,
                                  int64_t n_global, int64_t row_lo, int64_t row_hi, int g_dtype,
                                  void* g_pool, void* workspace, size_t workspace_bytes);

/* The same scatter with the contributions in rows_dtype (DWA_F32 or DWA_BF16),
 * e.g. the bf16 rows a receive area of dwa_pool_grad_send holds. */
DWA_API int dwa_pool_grad_scatter_typed(void* stream, int n, int D, const int32_t* indices, int rows_dtype,
                                        const void* g_rows, int64_t n_global, int64_t row_lo, int64_t row_hi,
                                        int g_dtype, void* g_pool, void* workspace, size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * Returning row gradients to the ranks that own the rows (row-sharded pool).
 * Replaces the transpose of _distributed_gather (src/dwa/model.py:16-47), whose
 * autodiff reduces a dense [B,k,D] cotangent over the model axis, and the
 * all-gather of every rank's rows: rank `rank` stores each of its n <= slot
 * contributions (g_rows [n, D] f32, pool rows indices [n]) straight into the
 * receive area of the rank that owns the row, converted to rows_dtype (bf16,
 * the pool's dtype, halves the bytes that cross NVLink).
 *  - recv: bases[q] = rank q's receive area mapped on this GPU (CUDA IPC;
 *    dwa_pool_grad_recv_bytes each, 256-byte aligned), row_lo = the owners' row
 *    bounds; world * slot <= 8192.
 *  - Area layout: idx [world * slot] int32 (padded to 256 bytes), then rows
 *    [world * slot, D].  Slot rank * slot + i holds contribution i of `rank`;
 *    the slots of rows owned elsewhere, and slots i >= n, hold DWA_PAD_INDEX.
 *  - After every rank's send, a collective (any; it orders the stores before
 *    the reads), then each owner calls dwa_pool_grad_scatter_typed on its own
 *    area (n = world * slot, rows_dtype) into its rows [row_lo, row_hi).
 *  - An area is overwritten by the next send into it: alternate two areas
 *    between calls, so that a rank one call ahead never writes into an area
 *    its owner is still reading.
 *  - Indices outside every owner set DWA_STATUS_BAD_ROW_INDEX (workspace).
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_pool_grad_recv_bytes(int world, int slot, int64_t D, int rows_dtype);
DWA_API int dwa_pool_grad_send(void* stream, int rank, int n, int slot, int64_t D, const int32_t* indices,
                               const float* g_rows, int rows_dtype, const DwaPoolShards* recv, void* workspace,
                               size_t workspace_bytes);

/* ---------------------------------------------------------------------------
 * All-gather of a few kilobytes per rank among the ranks of one node (one
 * process per GPU), for the two small exchanges of a row-sharded step: the
 * query means z and the retrieval summaries (gather_summaries, in place of an
 * NCCL all-gather whose fixed cost is tens of microseconds).
 *  - Every rank allocates one exchange buffer of
 *    dwa_peer_allgather_buffer_bytes(world, bytes), zero-filled, 256-byte
 *    aligned, and maps every other rank's (CUDA IPC); peer_buffers[r] is rank
 *    r's buffer on this GPU (this rank's own at r == rank).
 *  - Each call copies `bytes` (a multiple of 16) from src into every rank's
 *    buffer, signals each peer, waits for every peer's data of the same call
 *    and writes out[world * bytes] in rank order.  Every rank makes the same
 *    sequence of calls on the same buffers; a call's buffers alternate
 *    between two halves, so a rank one call ahead never overwrites data its
 *    owner is still reading.  Capturable in a CUDA graph.
 *  - Waits are bounded (about 1 s); a wait that gives up sets
 *    DWA_STATUS_WAIT_TIMEOUT in the buffer's status word, read (and cleared)
 *    with dwa_peer_allgather_status.  Ranks must run on distinct GPUs.
 * ------------------------------------------------------------------------- */
DWA_API size_t dwa_peer_allgather_buffer_bytes(int world, size_t bytes);
DWA_API int dwa_peer_allgather(void* stream, int rank, int world, const void* src, size_t bytes,
                               void* const* peer_buffers, void* out);
DWA_API int dwa_peer_allgather_status(void* stream, const void* buffer, uint32_t* status, int clear);

/* ---------------------------------------------------------------------------
 * Retrieval without a workspace.  No counterpart in the reference: it exists for
 * callers that cannot hand this library scratch memory or let it allocate, such
 * as a legacy XLA custom-call target that receives only its operand and result
 * buffers, or code that runs while a CUDA stream is being captured, where
 * cudaMalloc is not allowed.  Same arguments and results as dwa_retrieve minus
 * the workspace; the scratch is a fixed 8 MiB device array inside libdwa that
 * every GPU loading the library keeps until the process exits.
 *  - Shapes whose scratch need (dwa_retrieve_workspace_bytes) exceeds 8 MiB are
 *    rejected with DWA_ERR_UNSUPPORTED and a message; nothing is launched.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) and caches it; make that first call before any
 *    stream capture.
 *  - Allocates nothing (no cudaMalloc / cudaFree, no allocating library call).
 *  - All calls share the one array: calls that overlap on the GPU (other
 *    streams, other threads) race and must be serialised by the caller.
 *  - The device status word (DWA_STATUS_* bits: a bad row index, bad list
 *    offsets, a bounded wait that ran out) lives in that shared scratch; each
 *    call clears it first.  dwa_retrieve_noalloc_status reads it back.
 *  - The cached array address is per CUDA context, so a call from a context
 *    that has not used the array yet does the look-up again: make the first
 *    call of every context before any stream capture.
 * ------------------------------------------------------------------------- */
DWA_API int dwa_retrieve_noalloc(void* stream, const DwaRetrieveDims* dims, int use_ivf,
                                 int is_warmup, const float* lambda_val, const void* z,
                                 const float* W_Q, const float* aspect_weights, const float* tau,
                                 const float* centroids, const int64_t* list_offsets,
                                 const float* pool_keys, float* alphas, int32_t* indices,
                                 float* soft_full);

/* The status word of the last dwa_retrieve_noalloc call on the current device
 * and context, as dwa_workspace_status reports it for a workspace: copied on
 * `stream` after the call's kernels (the stream is synchronised), cleared when
 * `clear` is non-zero; DWA_ERR_DEVICE when a bit is set.  No counterpart in the
 * reference (companion of dwa_retrieve_noalloc).  Allocates nothing. */
DWA_API int dwa_retrieve_noalloc_status(void* stream, uint32_t* status, int clear);

#ifdef __cplusplus
}
#endif
#endif /* DWA_H_ */
