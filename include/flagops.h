/*
 * flagops.h — C ABI of the B200 (sm_100a) five-operator kernel set.
 *
 * Every entry point takes raw device pointers, int64 sizes, dtype codes and a
 * cudaStream_t passed as void*.  Nothing here allocates device memory (only
 * fo_peer_open maps a buffer that another process allocated): scratch
 * ("workspace") is owned by the caller, sized by the matching *_workspace_bytes
 * query.  Calls are stream-ordered and never synchronise the host.  The return
 * value is a status code (FO_OK == 0); fo_last_error() gives the message of the
 * most recent failure on the calling thread.
 *
 * Each declaration names the reference (iamsuperfly/Flag-Operators) interface
 * it replaces as path:line inside that project.
 */
#ifndef FLAGOPS_H
#define FLAGOPS_H

#include <stdint.h>

#if defined(__GNUC__)
#define FO_API __attribute__((visibility("default")))
#else
#define FO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes shared by every entry point */
enum fo_dtype {
  FO_F32 = 0,
  FO_F16 = 1,
  FO_BF16 = 2,
  FO_F64 = 3,
  FO_I32 = 4,
  FO_I64 = 5
};

/* status codes */
enum fo_status {
  FO_OK = 0,
  FO_EINVAL = -1,       /* bad argument (shape, pointer, alignment)       */
  FO_EDTYPE = -2,       /* dtype not supported by this entry point         */
  FO_ECUDA = -3,        /* CUDA launch / runtime error                     */
  FO_EWORKSPACE = -4,   /* workspace missing or too small                  */
  FO_EUNSUPPORTED = -5  /* configuration not supported (e.g. head dim)     */
};

/* scatter_reduce reduce codes (operators/scatter_reduce.py:306) */
enum fo_reduce {
  FO_SUM = 0,
  FO_PROD = 1,
  FO_MEAN = 2,
  FO_AMAX = 3,
  FO_AMIN = 4
};

/* cross-entropy reduction codes (operators/fused_cross_entropy.py:325) */
enum fo_reduction {
  FO_RED_NONE = 0,
  FO_RED_MEAN = 1,
  FO_RED_SUM = 2
};

/* Message of the last failed call on this thread ("" if none). */
FO_API const char* fo_last_error(void);
/* ABI revision; bumped on any signature change. */
FO_API int fo_abi_version(void);

/* ------------------------------------------------------------------------ */
/* rms_norm                                                                  */
/* ------------------------------------------------------------------------ */
/*
 * y[m, :] = x[m, :] * inv_rms[m] * weight,  inv_rms[m] = 1/sqrt(mean(x[m,:]^2) + eps)
 * x, y: [M, N] contiguous (x_dtype); weight: [N] (w_dtype); inv_rms: [M] fp32.
 * Replaces rms_norm_forward, operators/rms_norm.py:186-228 (and its kernels
 * _rms_norm_small_kernel rms_norm.py:50-90, _rms_norm_loop_kernel rms_norm.py:97-176).
 */
FO_API int fo_rms_norm_fwd(const void* x, const void* weight, void* y, float* inv_rms,
                    int64_t M, int64_t N, float eps, int x_dtype, int w_dtype,
                    void* stream);

/*
 * rms_norm backward from the forward's inv_rms (dy, x, dx: [M, N] x_dtype; weight, dw: [N]
 * w_dtype; inv_rms: [M] fp32):
 *   dx = inv * (dy * w) - x * inv^3 * sum_j(dy_j w_j x_j) / N,   dw = sum_m dy * x * inv
 * Scratch: fo_rms_norm_bwd_workspace_bytes(M, N) bytes (dw partial sums).  The reference
 * returns inv_rms "for backward" (operators/rms_norm.py:10,17,186-228; its API is the
 * FlagGems one) and has no backward kernel of its own; this is the backward of its CPU
 * formula (rms_norm.py:211-216).
 */
FO_API int fo_rms_norm_bwd_workspace_bytes(int64_t M, int64_t N, int64_t* bytes);
FO_API int fo_rms_norm_bwd(const void* dy, const void* x, const void* weight,
                           const float* inv_rms, void* dx, void* dw, int64_t M, int64_t N,
                           int x_dtype, int w_dtype, void* workspace, int64_t ws_bytes,
                           void* stream);

/* ------------------------------------------------------------------------ */
/* median                                                                    */
/* ------------------------------------------------------------------------ */
/*
 * Lower median of each row of x [M, N] (contiguous): values [M] (dtype of x),
 * indices [M] int64, with torch CPU semantics: the index is the k-th entry
 * (k = (N-1)/2) of a stable ascending sort, -0.0 == +0.0, and any NaN in a
 * row gives NaN with the index of the row's first NaN.
 * Replaces _median_dim, operators/median.py:241-305 (kernels median.py:82-192).
 */
FO_API int fo_median_dim(const void* x, void* values, int64_t* indices, int64_t M,
                  int64_t N, int dtype, void* stream);

/*
 * Lower median of all n elements of x (contiguous), written to value[0]
 * (dtype of x).  Replaces _median_global, operators/median.py:308-325.
 * workspace: fo_median_all_workspace_bytes(n) bytes.
 */
FO_API int fo_median_all_workspace_bytes(int64_t n, int64_t* bytes);
FO_API int fo_median_all(const void* x, void* value, int64_t n, int dtype,
                  void* workspace, int64_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* scatter_reduce                                                            */
/* ------------------------------------------------------------------------ */
/*
 * out[..., index[p], ...] = reduce(out[...], src[p]) along `dim` for every
 * position p of index (torch.Tensor.scatter_reduce_ semantics).  `out` holds
 * self's values on entry (the caller copies self into it for the out-of-place
 * and out= variants).  ndim in [1, 4]; index_shape / index_strides /
 * src_strides / out_shape / out_strides are ndim-long arrays, strides in
 * elements.  Indices outside [0, out_shape[dim]) are skipped and counted into
 * *err_count (device int32, nullable).
 * Replaces scatter_reduce_ / scatter_reduce / scatter_reduce_out and their
 * launcher, operators/scatter_reduce.py:327-468 (kernels 69-276).
 */
FO_API int fo_scatter_reduce_workspace_bytes(int64_t out_numel, int reduce,
                                      int include_self, int dtype,
                                      int64_t* bytes);
/*
 * Extra workspace (bytes, appended after fo_scatter_reduce_workspace_bytes')
 * that lets fo_scatter_reduce use its destination-binned pass for n updates
 * into an output spanning out_span elements: 0 when that pass does not apply.
 * The pass runs when ndim == 1, index and src are contiguous and ws_bytes
 * covers both parts; otherwise every update is an atomic.  Replaces the same
 * launcher as fo_scatter_reduce (operators/scatter_reduce.py:327-375).
 */
FO_API int fo_scatter_reduce_binned_bytes(int64_t out_span, int64_t n, int reduce, int dtype,
                                          int64_t* bytes);
FO_API int fo_scatter_reduce(void* out, const void* src, const void* index, int ndim,
                      const int64_t* index_shape, const int64_t* index_strides,
                      const int64_t* src_strides, const int64_t* out_shape,
                      const int64_t* out_strides, int dim, int reduce,
                      int include_self, int dtype, int index_dtype,
                      void* workspace, int64_t ws_bytes, int32_t* err_count,
                      void* stream);

/*
 * Allocation-free scatter_reduce: same arguments and results as
 * fo_scatter_reduce, without the workspace.  No counterpart in the reference.
 * For callers that cannot allocate device memory (a framework that owns the
 * whole device heap, a cgo / JNI / plugin caller without the program's
 * allocator, code that must avoid the device synchronisation of cudaMalloc).
 * The scratch is one static 12 MiB device array per device, reserved when the
 * library is loaded and held until the process exits.  It covers an output
 * whose memory span (1 + sum over dims of (size - 1) * stride, in elements, so
 * a strided view counts the whole range it spans, not its cell count) is at
 * most 2^20; larger calls fail with FO_EWORKSPACE.  Arguments are checked
 * first, with the same status codes and messages as fo_scatter_reduce.  The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and keeps it, so make that first call before any
 * stream capture, and do not use this entry point after a cudaDeviceReset in
 * the same process (the kept address may then be stale).  Every call reuses
 * the same array (it is re-initialised per call): calls that overlap on the
 * GPU, from several streams or threads, race and must not be issued.
 * Allocates nothing.
 */
FO_API int fo_scatter_reduce_noalloc(void* out, const void* src, const void* index, int ndim,
                                     const int64_t* index_shape, const int64_t* index_strides,
                                     const int64_t* src_strides, const int64_t* out_shape,
                                     const int64_t* out_strides, int dim, int reduce,
                                     int include_self, int dtype, int index_dtype,
                                     int32_t* err_count, void* stream);

/* ------------------------------------------------------------------------ */
/* fused cross-entropy                                                       */
/* ------------------------------------------------------------------------ */
/*
 * Forward over logits [B, V] (row stride ld elements, dtype) and target [B]
 * int64.  Writes per-row loss loss_rows [B] fp32 (0 for ignored rows), lse [B]
 * fp32, and out_scalar[0] fp32 = sum (FO_RED_SUM) or sum / n_valid
 * (FO_RED_MEAN; NaN when every row is ignored, as torch); n_valid_out[0] fp32 =
 * number of rows whose target != ignore_index.  label_smoothing in [0, 1) is
 * fused (loss = lse - (1-e) x_t - e mean(x)).  When dlogits (contiguous
 * [B, V], logits' dtype) is non-null the
 * gradient d loss / d logits for grad_output == 1 is written in the same pass
 * (row re-read from L2), so a later fo_ce_scale_grad completes backward.
 * workspace: fo_ce_workspace_bytes(B) bytes.
 * Replaces _FusedCrossEntropy.forward, operators/fused_cross_entropy.py:243-274,
 * and _fused_ce_fwd_kernel (fused_cross_entropy.py:63-148).
 */
FO_API int fo_ce_workspace_bytes(int64_t B, int64_t* bytes);
FO_API int fo_ce_fwd(const void* logits, const int64_t* target, float* loss_rows,
              float* lse, float* out_scalar, float* n_valid_out, void* dlogits,
              int64_t B, int64_t V, int64_t ld, int64_t ignore_index,
              float label_smoothing, int reduction, int dtype, void* workspace,
              int64_t ws_bytes, void* stream);

/*
 * Backward by recomputation: dlogits = dout * (softmax(x) - (1-e) onehot - e/V)
 * / (n_valid for mean), 0 on ignored rows; dlogits is contiguous [B, V].
 * dout is a device scalar
 * (dout_is_vector == 0) or a [B] vector (reduction none).
 * Replaces _FusedCrossEntropy.backward, fused_cross_entropy.py:276-295, and
 * _fused_ce_bwd_kernel (fused_cross_entropy.py:155-234).
 */
FO_API int fo_ce_bwd(const void* logits, const int64_t* target, const float* lse,
              const void* dout, int dout_dtype, int dout_is_vector,
              const float* n_valid, void* dlogits, int64_t B, int64_t V,
              int64_t ld, int64_t ignore_index, float label_smoothing,
              int reduction, int dtype, void* stream);

/*
 * dlogits *= dout (device scalar, dout_dtype) or dlogits[b, :] *= dout[b]
 * (dout_is_vector); a no-op pass-through when the scalar is exactly 1.
 * Completes backward after fo_ce_fwd wrote the gradient.
 */
FO_API int fo_ce_scale_grad(void* dlogits, const void* dout, int dout_dtype,
                     int dout_is_vector, int64_t B, int64_t V, int64_t ld,
                     int dtype, void* stream);

/*
 * Vocabulary-sharded forward, step 1 (no reference counterpart; the reference
 * is single-device): per-row statistics of this rank's column slice
 * [B, V_local] whose first column is global column v_offset.
 * stats [B, 4] fp32 = (row max, sum exp(x - max), target logit or 0,
 * row sum of logits).
 */
FO_API int fo_ce_shard_stats(const void* logits, const int64_t* target, float* stats,
                      int64_t B, int64_t V_local, int64_t ld, int64_t v_offset,
                      int64_t ignore_index, int dtype, void* stream);
/*
 * Step 2, after the stats of all P ranks were gathered into
 * all_stats [P, B, 4]: combine into lse [B], loss_rows [B], out_scalar,
 * n_valid_out, exactly as fo_ce_fwd does for one rank.  V is the full vocab.
 */
FO_API int fo_ce_shard_combine(const float* all_stats, int P, const int64_t* target,
                        float* loss_rows, float* lse, float* out_scalar,
                        float* n_valid_out, int64_t B, int64_t V,
                        int64_t ignore_index, float label_smoothing,
                        int reduction, void* stream);
/*
 * Step 3: this rank's slice of the gradient (as fo_ce_bwd, columns offset by
 * v_offset, softmax normalised by the global lse).
 */
FO_API int fo_ce_shard_bwd(const void* logits, const int64_t* target, const float* lse,
                    const void* dout, int dout_dtype, int dout_is_vector,
                    const float* n_valid, void* dlogits, int64_t B,
                    int64_t V_local, int64_t ld, int64_t v_offset, int64_t V,
                    int64_t ignore_index, float label_smoothing, int reduction,
                    int dtype, void* stream);

/*
 * Vocabulary-sharded forward and gradient in ONE kernel that exchanges the
 * per-row statistics over NVLink peer memory instead of a collective (no
 * reference counterpart; the reference is single-device, and this replaces
 * the three steps above when every rank has its own GPU with peer access).
 * regions[p] (p < P <= 8) is rank p's region of fo_ce_shard_p2p_region_bytes(P,
 * rows_cap) bytes, zeroed once before its first use and mapped into this
 * process (fo_peer_open; regions[rank] is this rank's own); B <= rows_cap.
 * Every rank calls with the same B, P, rows_cap and epoch, and epoch grows by
 * one per call (starting at 1).  Writes loss_rows, lse, out_scalar and
 * n_valid_out as fo_ce_fwd (the full-vocabulary loss, identical on every rank)
 * and, when dlogits ([B, V_local], logits' dtype) is non-null, this rank's
 * gradient slice for grad_output == 1 (complete backward with
 * fo_ce_scale_grad).  One HBM read and one write of the rank's block.  Waits on
 * other ranks are bounded: one that runs out is counted by fo_ce_p2p_timeouts
 * and leaves NaN in the rows it could not complete.
 */
FO_API int fo_ce_shard_p2p_region_bytes(int P, int64_t rows_cap, int64_t* bytes);
FO_API int fo_ce_shard_p2p_fwd(const void* logits, const int64_t* target, float* loss_rows,
                               float* lse, float* out_scalar, float* n_valid_out,
                               void* dlogits, int64_t B, int64_t V_local, int64_t ld,
                               int64_t v_offset, int64_t V, int64_t ignore_index,
                               float label_smoothing, int reduction, int dtype,
                               void* const* regions, int P, int rank, int64_t rows_cap,
                               uint32_t epoch, void* stream);
/* Number of peer waits of fo_ce_shard_p2p_fwd that ran out of polls since the
 * library was loaded (0 in a healthy run).  Synchronous read of a device
 * counter. */
FO_API int fo_ce_p2p_timeouts(unsigned int* count);

/*
 * Peer-memory plumbing (no reference counterpart).  fo_peer_export gives the
 * CUDA IPC handle (fo_peer_handle_bytes() bytes) of the allocation holding the
 * device pointer ptr, and ptr's offset inside it; fo_peer_open maps such a
 * handle from another process into the current device (plain IPC mapping with
 * peer access, no multicast) and returns the pointer at the offset;
 * fo_peer_close unmaps it.  fo_peer_can_access reports whether device can
 * load and store peer_device's memory.
 */
FO_API int fo_peer_handle_bytes(void);
FO_API int fo_peer_export(const void* ptr, void* handle_out, int64_t* offset_out);
FO_API int fo_peer_open(const void* handle, int64_t offset, void** ptr_out);
FO_API int fo_peer_close(void* ptr, int64_t offset);
FO_API int fo_peer_can_access(int device, int peer_device, int* ok);

/*
 * Row-sharded cross-entropy: each rank holds a block of rows [B_local, V] of
 * the batch.  fo_ce_count_valid counts this rank's non-ignored targets; the
 * caller sums the counts over ranks (one all-reduce) and passes the total as
 * n_valid_global.  fo_ce_rows_fwd then writes per-row loss and lse, the
 * gradient for grad_output == 1 (dlogits nullable; scaled by 1/n_valid_global
 * for FO_RED_MEAN) and local_sum_out[0] = sum of this rank's row losses, which
 * the caller sums over ranks (second all-reduce) and divides by n_valid_global
 * for 'mean'.  The backward for other grad_output values is fo_ce_bwd with
 * n_valid = n_valid_global.  Partitions the rows of
 * operators/fused_cross_entropy.py:302-357 (no counterpart in the reference).
 */
FO_API int fo_ce_count_valid(const int64_t* target, int64_t B, int64_t ignore_index,
                             float* n_valid_out, void* stream);
FO_API int fo_ce_rows_fwd(const void* logits, const int64_t* target, float* loss_rows,
                          float* lse, float* local_sum_out, const float* n_valid_global,
                          void* dlogits, int64_t B, int64_t V, int64_t ld,
                          int64_t ignore_index, float label_smoothing, int reduction,
                          int dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* chunk_gated_delta_rule                                                    */
/* ------------------------------------------------------------------------ */
/*
 * h_t = g_t h_{t-1} + beta_t (v_t - h_{t-1} k_t) k_t^T,  o_t = h_t q_t
 * q, k, v, o: [B, H, L, D] contiguous (dtype); beta, g: [B, H, L] (gate_dtype);
 * h0: [B, H, D, D] fp32 initial state or NULL (zeros); hT: [B, H, D, D] fp32
 * final state or NULL (h0 and hT must not alias).  D in {16, 32, 64, 128}.
 * bf16/fp16 inputs run the chunked tcgen05 kernel (D < 128 as D = 128 with
 * zero channels), whose operands are
 * fp16 tiles: a head whose fp16 operands would leave the fp16 range (|x| >=
 * 65504, e.g. bf16 inputs of 1e5) is marked in the workspace (one int per head,
 * fo_gdr_workspace_bytes) and recomputed by the fp32 per-step kernel in the
 * same call, so finite inputs never turn into inf/NaN.  The other cases run
 * the per-step kernel and need no workspace.
 * Replaces chunk_gated_delta_rule, operators/chunk_gated_delta_rule.py:208-268
 * (kernels chunk_gated_delta_rule.py:71-191).
 */
FO_API int fo_gdr_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t D, int dtype,
                                  int64_t* bytes);
FO_API int fo_gdr_fwd(const void* q, const void* k, const void* v, const void* beta,
               const void* g, const float* h0, void* o, float* hT, int64_t B,
               int64_t H, int64_t L, int64_t D, int dtype, int gate_dtype,
               void* workspace, int64_t ws_bytes, void* stream);
/* Same recurrence, always through the per-step CUDA-core kernel (any D in
 * {16,32,64,128}); kept as an independent on-device cross-check. */
FO_API int fo_gdr_fwd_stepwise(const void* q, const void* k, const void* v,
                        const void* beta, const void* g, const float* h0,
                        void* o, float* hT, int64_t B, int64_t H, int64_t L,
                        int64_t D, int dtype, int gate_dtype, void* stream);

/* Number of tensor-core waits of the chunked kernel that ran out of polls since
 * the library was loaded (0 in a healthy run; a timed-out head leaves its
 * outputs incomplete).  Synchronous read of a device counter. */
FO_API int fo_gdr_timeouts(unsigned int* count);

/*
 * Backward of the same recurrence: gradients of a loss L(o, h_T) given
 * d_o = dL/do ([B, H, L, D], dtype) and dhT = dL/dh_T ([B, H, D, D] fp32, or
 * NULL when the final state is not used).  Writes dq, dk, dv ([B, H, L, D],
 * dtype), dbeta, dg ([B, H, L], gate_dtype) and, when dh0 is not NULL, the
 * gradient of the initial state ([B, H, D, D] fp32); h0 is the forward's
 * initial state or NULL.  Computed in fp32 on the CUDA cores from the inputs
 * alone (it does not read the forward's outputs): the states are recomputed
 * from checkpoints every 16 steps kept in the workspace
 * (fo_gdr_bwd_workspace_bytes: B*H*(ceil(L/16) + min(L, 16))*D*D*4 bytes,
 * 16-byte aligned).  Deterministic (fixed-order
 * sums).  D in {16, 32, 64, 128}.
 * The reference has no backward kernel: its CPU path
 * (_ref_forward, operators/chunk_gated_delta_rule.py:286-310) is differentiated
 * by torch autograd, and these are those gradients.
 */
FO_API int fo_gdr_bwd_workspace_bytes(int64_t B, int64_t H, int64_t L, int64_t D,
                                      int64_t* bytes);
FO_API int fo_gdr_bwd(const void* q, const void* k, const void* v, const void* beta,
                      const void* g, const float* h0, const void* d_o, const float* dhT,
                      void* dq, void* dk, void* dv, void* dbeta, void* dg, float* dh0,
                      int64_t B, int64_t H, int64_t L, int64_t D, int dtype, int gate_dtype,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* Number of hand-off waits of the producer/consumer median kernel (rows of
 * 1024 < N <= 2048) that ran out of polls since the library was loaded (0 in a
 * healthy run; a timed-out CTA stops and leaves its remaining rows unwritten).
 * Synchronous read of a device counter.  No reference counterpart. */
FO_API int fo_median_timeouts(unsigned int* count);

/* Operand-layout self-test of the tensor-core path (no reference counterpart):
 * d[128, N] (fp32) = A[128, K] . B[N, K]^T on one CTA with tcgen05.mma, bf16 A/B.
 * a is [128][K] (a_mn = 0, K-major) or [K][128] (a_mn = 1); b is [N][K] (b_mn = 0)
 * or [K][N] (b_mn = 1).  N, K in {64, 128}. */
FO_API int fo_tc05_selftest(const void* a, const void* b, float* d, int64_t N, int64_t K,
                            int a_mn, int b_mn, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLAGOPS_H */
