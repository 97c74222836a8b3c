/*
 * fuselse_b200 — C ABI of the B200 (sm_100a) row log-sum-exp library.
 *
 * Every entry point takes plain device pointers, int64 sizes and a CUDA
 * stream, launches its kernels asynchronously on that stream and returns a
 * status code (FL_OK == 0).  No compute entry point allocates device
 * memory: outputs are caller-owned buffers (the fl_ipc_buffer_* helpers,
 * which create and map buffers shared between processes, are the
 * exception).  On a non-zero status, fl_last_error() returns a message for
 * the calling thread.
 *
 * Pointer rules shared by all entry points:
 *   - all pointers are device (or managed) memory of the device that owns
 *     `stream` (the NULL stream means the device that owns the first input);
 *   - arrays are dense row-major (C-contiguous), element-aligned;
 *   - a NULL pointer is accepted only when the array it stands for is empty.
 *
 * Each function names the reference interface it replaces (file:line in the
 * FuseLSE/IntLSE reference sources).
 */
#ifndef FUSELSE_B200_H
#define FUSELSE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t, declared without pulling in CUDA headers. */
typedef struct CUstream_st* fl_stream_t;

enum fl_status {
    FL_OK = 0,
    FL_ERR_INVALID_ARGUMENT = 1, /* shape, pointer or alignment rejected */
    FL_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed */
    FL_ERR_UNSUPPORTED = 3       /* well-formed request outside the supported range */
};

/* Message of the last failed call on this host thread ("" if none). */
const char* fl_last_error(void);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int fl_version(void);

/* The binary version (major*10 + minor, 100 for sm_100a) of the kernels this
 * library loads on `device`, from cudaFuncGetAttributes (needs a GPU). */
int fl_binary_version(int device, int* version);

/* ------------------------------------------------------------------------
 * FuseLSE fp32 forward: out[b] = log(sum_n exp(x[b, n])), x (B, N) fp32.
 *   robust != 0: IEEE rules — any NaN in the row -> NaN, else any +inf ->
 *   +inf, -inf entries contribute nothing, an all--inf row -> -inf.
 *   robust == 0: finite inputs assumed; an empty row (N == 0) gives -1e30.
 * Replaces onepass_lse_float / onepass_lse_float_robust
 * (fuselse/gpu/fused_fp32_kernel.cu:154-194, binding :255-259).
 * ---------------------------------------------------------------------- */
int fl_lse_f32_fwd(const float* x, float* out, int64_t B, int64_t N,
                   int robust, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * FuseLSE fp32 backward: gx[b, n] = g[b] * exp(x[b, n] - lse[b]).
 * g, lse (B,), x and gx (B, N) fp32.
 * Replaces onepass_lse_float_backward (fuselse/gpu/fused_fp32_kernel.cu:196-252).
 * ---------------------------------------------------------------------- */
int fl_lse_f32_bwd(const float* g, const float* x, const float* lse,
                   float* gx, int64_t B, int64_t N, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Strided rows (no contiguous copy).  Row r of x (N contiguous elements)
 * starts at element
 *     r * row_stride                                   if r < rows_per_group
 *     (r / rows_per_group) * group_stride + (r % rows_per_group) * row_stride
 * — the leading two dims of a sliced tensor such as logits[:, :-1, :]
 * (rows_per_group = T - 1, group_stride = T*V, row_stride = V).
 * rows_per_group < 0 means dense rows (row_stride N).  out, lse, g and gx
 * stay dense (B,) / (B, N).  The reference reduces a contiguous copy made by
 * its autograd wrapper (fuselse/gpu/autograd.py:19,56); no reference
 * counterpart.
 * ---------------------------------------------------------------------- */
int fl_lse_f32_fwd_strided(const float* x, float* out, int64_t B, int64_t N,
                           int64_t rows_per_group, int64_t group_stride,
                           int64_t row_stride, int robust, fl_stream_t stream);
int fl_lse_f32_bwd_strided(const float* g, const float* x, const float* lse,
                           float* gx, int64_t B, int64_t N, int64_t rows_per_group,
                           int64_t group_stride, int64_t row_stride,
                           fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Reduction over a dim that is not the last: x dense, viewed as
 * (outer, N, inner), out[o, i] = LSE_n x[o, n, i] and
 * gx[o, n, i] = g[o, i] * exp(x[o, n, i] - lse[o, i]); out, g, lse are
 * (outer, inner).  inner == 1 is the row case.  The reference delegates
 * dim != -1 to torch.logsumexp (fuselse/gpu/autograd.py:44-49); no
 * reference counterpart.
 * ---------------------------------------------------------------------- */
int fl_lse_f32_fwd_dim(const float* x, float* out, int64_t outer, int64_t N,
                       int64_t inner, int robust, fl_stream_t stream);
int fl_lse_f32_bwd_dim(const float* g, const float* x, const float* lse, float* gx,
                       int64_t outer, int64_t N, int64_t inner, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Selective log-softmax, fused: one pass over each row gives
 *   lse[b]  = LSE over x[b, :]                      (as fl_lse_f32_fwd)
 *   logp[b] = x[b, index[b]] - lse[b]
 * Replaces the caller's two passes — torch.gather of the target logit plus
 * one LSE call per sequence — in trl.trainer.utils.selective_log_softmax
 * (trl 1.0.0) as used by experiment_rlhf_logsumexp/run_rlhf.py:145-157 with
 * torch.logsumexp routed to onepass_lse_float (rlhf_timing.py:23-37).  No
 * reference kernel.  index is int64 (B,); an index outside [0, N) gives
 * logp[b] = NaN and, when err_flag is not NULL, sets *err_flag |= 1 (the
 * caller zeroes it; the kernel never faults on it).  lse is required (the
 * backward needs it).  N must be >= 1 when B > 0.
 * fp16 input: fp32 arithmetic, empty-row value -1e30 as fl_lse_f16_fwd.
 * ---------------------------------------------------------------------- */
int fl_selective_logsoftmax_f32(const float* x, const int64_t* index, float* logp,
                                float* lse, int64_t B, int64_t N, int robust,
                                int* err_flag, fl_stream_t stream);
int fl_selective_logsoftmax_f16(const uint16_t* x, const int64_t* index, float* logp,
                                float* lse, int64_t B, int64_t N, int* err_flag,
                                fl_stream_t stream);
/* Strided rows as fl_lse_f32_fwd_strided; index, logp, lse dense (B,). */
int fl_selective_logsoftmax_f32_strided(const float* x, const int64_t* index, float* logp,
                                        float* lse, int64_t B, int64_t N,
                                        int64_t rows_per_group, int64_t group_stride,
                                        int64_t row_stride, int robust, int* err_flag,
                                        fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Selective log-softmax backward (fp32):
 *   gx[b, j] = g[b] * ([j == index[b]] - exp(x[b, j] - lse[b]))
 * i.e. d logp / d x scaled by the upstream gradient g (B,).  An index
 * outside [0, N) contributes no one-hot term.  No reference counterpart
 * (the reference differentiates only the LSE, onepass_lse_float_backward).
 * ---------------------------------------------------------------------- */
int fl_selective_logsoftmax_bwd(const float* g, const float* x, const float* lse,
                                const int64_t* index, float* gx, int64_t B, int64_t N,
                                fl_stream_t stream);
/* Strided x rows as fl_lse_f32_fwd_strided; gx dense (B, N). */
int fl_selective_logsoftmax_bwd_strided(const float* g, const float* x, const float* lse,
                                        const int64_t* index, float* gx, int64_t B, int64_t N,
                                        int64_t rows_per_group, int64_t group_stride,
                                        int64_t row_stride, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * FuseLSE16 forward: out[b] (fp32) = LSE over x[b, :] given as IEEE fp16
 * (uint16 bit patterns), fp32 arithmetic.  Same rules as robust fp32.
 * Replaces batched_logsumexp_fp16 (fuselse/gpu/fused_fp16_kernel.cu:112-132).
 * ---------------------------------------------------------------------- */
int fl_lse_f16_fwd(const uint16_t* x, float* out, int64_t B, int64_t N,
                   fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Per-row partial state for vocab-sharded rows (no reference counterpart;
 * it splits the reference's one-block-per-row reduction at a shard edge):
 *   ms[2*b]   = m_b = max_n x[b, n]   (NaN if any NaN)
 *   ms[2*b+1] = s_b = sum_n exp(x[b, n] - m'_b),  m'_b = (m_b == -inf ? 0 : m_b)
 * `ms` holds B float pairs.  fp32 and fp16 inputs.
 * ---------------------------------------------------------------------- */
int fl_lse_f32_partial(const float* x, float* ms, int64_t B, int64_t N,
                       fl_stream_t stream);
int fl_lse_f16_partial(const uint16_t* x, float* ms, int64_t B, int64_t N,
                       fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Combine G shard partials per row: ms (G, B, 2) as written by
 * fl_lse_*_partial on each shard (shard-major), out (B,) fp32:
 *   out[b] = M + log(sum_g s_gb * exp(m_gb - M)),  M = max_g m_gb
 * with the robust rules (NaN wins, then +inf, all--inf gives -inf).
 * ---------------------------------------------------------------------- */
int fl_lse_combine(const float* ms, float* out, int64_t G, int64_t B,
                   fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Vocab-sharded log-sum-exp with the exchange done over NVLink peer memory
 * (no reference counterpart; the reference is single-GPU).  G ranks hold
 * the same B rows split by columns; rank `rank` passes its (B, N) shard x
 * (dtype 0: fp32, 1: fp16).  `local_buf` is this rank's exchange buffer of
 * fl_vocab_exchange_bytes(G, B) bytes (256-byte aligned, zero-filled once
 * before first use on every rank, then left to the library), and
 * `peer_bufs` a DEVICE array of the G ranks' buffer addresses as mapped on
 * this device (e.g. buffers of fl_ipc_buffer_alloc mapped with
 * fl_ipc_buffer_open; peer_bufs[rank] == local_buf).
 * Writes out (B,) fp32 on every rank.  Every rank must make the same
 * sequence of calls with the same B.  If a peer's contribution does not
 * arrive within the wait limit (2 s unless changed by
 * fl_vocab_exchange_set_wait_limit) the rows are NaN and the 32-bit word at
 * byte offset 4 of local_buf becomes non-zero (sticky); the call epoch
 * still advances, so the buffer must be zero-filled again on every rank
 * before the group makes another exchange.
 * ---------------------------------------------------------------------- */
int fl_vocab_exchange_bytes(int64_t G, int64_t B, int64_t* bytes);
int fl_lse_vocab_exchange(const void* x, int dtype, int64_t B, int64_t N,
                          void* const* peer_bufs, void* local_buf, int rank, int G,
                          float* out, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Exchange buffers shared between processes by CUDA IPC (no reference
 * counterpart).  These four are the only entry points that allocate or map
 * device memory: a CUDA IPC handle names a whole cudaMalloc allocation, so a
 * buffer meant for other processes cannot come from a caller's pool.
 *   fl_ipc_buffer_alloc: `bytes` zero-filled bytes on `device`, 256-byte
 *     aligned; *buf = its address here, ipc_handle (64 bytes) = its handle
 *     for the other processes;
 *   fl_ipc_buffer_open: maps another process's buffer on `device` (plain
 *     unicast peer mapping, no NVLS group) and returns its address here;
 *   fl_ipc_buffer_close: unmaps a buffer opened by fl_ipc_buffer_open;
 *   fl_ipc_buffer_free: waits for the device and frees a buffer of
 *     fl_ipc_buffer_alloc (every other process must have closed it first).
 * ---------------------------------------------------------------------- */
int fl_ipc_buffer_alloc(int device, int64_t bytes, void** buf, void* ipc_handle);
int fl_ipc_buffer_open(int device, const void* ipc_handle, void** buf);
int fl_ipc_buffer_close(int device, void* buf);
int fl_ipc_buffer_free(int device, void* buf);

/* Sets the limit of the exchange's wait for a peer (per combine CTA and
 * peer), in nanoseconds within [1e6, 6e10], for launches made after the
 * call, process-wide; *previous (if not NULL) receives the old limit.
 * No reference counterpart. */
int fl_vocab_exchange_set_wait_limit(int64_t ns, int64_t* previous);

/* ------------------------------------------------------------------------
 * The single-rank (G = 1) fl_lse_vocab_exchange without any device
 * allocation (no counterpart in the reference).  For callers that cannot
 * allocate device memory: a host whose GPU is driven through a plugin or
 * embedded runtime that owns every allocation, or code whose memory budget
 * is fixed before these calls.  Instead of a caller buffer, the exchange
 * buffer is a file-scope array compiled into this library: 4 MiB per
 * device, held by every GPU that loads the library until the process exits.
 * Limit: B <= 262,112 rows (larger requests are rejected with
 * FL_ERR_INVALID_ARGUMENT and a message giving the maximum).  x (B, N) of
 * dtype 0 (fp32) or 1 (fp16), out (B,) fp32, on the device of `stream`.
 * The first call on a device resolves the array's device address, clears
 * its counters and synchronizes the device: make it before any stream
 * capture.  All calls on a device share the array, which keeps the last
 * call's contents: calls that overlap on a GPU (other streams, other
 * threads) race and must not be issued.
 * ---------------------------------------------------------------------- */
int fl_lse_vocab_exchange_noalloc(const void* x, int dtype, int64_t B, int64_t N,
                                  float* out, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * IntLSE Q16.16 with fp32 base-e input: q = rint_sat(x * log2(e) * 2^16),
 * pairwise base-2 Mitchell reduction with the 64-entry correction table
 * (use_lut != 0) or without it (use_lut == 0), out = acc * ln2 / 2^16.
 * Bit-identical to the reference kernel on the same input buffer.
 * Replaces batched_logsumexp / batched_logsumexp_nolut
 * (intlse/gpu/lse_kernel.cu:164-202, binding :204-209).
 * ---------------------------------------------------------------------- */
int fl_intlse_q16_f32(const float* x, float* out, int64_t B, int64_t N,
                      int use_lut, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * IntLSE Q16.16 with int32 input already in Q16.16 base-2 fixed point.
 * Same reduction order as fl_intlse_q16_f32 minus the float conversion, so
 * feeding q[b, n] = rint_sat(x[b, n] * log2(e) * 2^16) reproduces
 * fl_intlse_q16_f32(x) (and the reference batched_logsumexp) bit for bit.
 * Derived from intlse/gpu/lse_kernel.cu:67-159 (the conversion at :114 removed).
 * ---------------------------------------------------------------------- */
int fl_intlse_q16_i32(const int32_t* q, float* out, int64_t B, int64_t N,
                      int use_lut, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * IntLSE Q10.6: int16 (B, N) base-2 Q10.6 input -> fp32 base-e (B,).
 * Bit-identical to the reference kernel.
 * Replaces batched_logsumexp_q10_6 (intlse/gpu/lse_kernel_q10_6.cu:144-165).
 * ---------------------------------------------------------------------- */
int fl_intlse_q10_6_i16(const int16_t* q, float* out, int64_t B, int64_t N,
                        fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Sparse probabilistic-circuit sum layer (pyjuice layout), in place:
 *   for k in [0, num_nblocks), p in [0, block_size), b in [0, batch):
 *     node_mars[(nids[k] + p) * batch + b] =
 *         LSE_e( log(max(params[pids[k, e] + p], 1e-45)) + element_mars[cids[k, e] * batch + b] )
 * node_mars (num_nodes, batch), element_mars (num_elements, batch), params
 * (num_params,) fp32; nids (num_nblocks,), cids and pids (num_nblocks,
 * num_edges) int64.  Index arrays are bounds-checked on the device: an
 * out-of-range child or parameter index makes that output NaN, an
 * out-of-range node index skips the write, and either sets *err_flag = 1
 * when err_flag is non-NULL (a device int the caller zeroes first).
 * fl_sparse_f32 replaces sparse_forward_float
 * (experiment_pyjuice/sparse_float_kernel.cu:110-167);
 * fl_sparse_q16 replaces sparse_forward_q16
 * (experiment_pyjuice/sparse_q16_kernel.cu:139-202) and is bit-identical to it.
 * ---------------------------------------------------------------------- */
int fl_sparse_f32(float* node_mars, const float* element_mars,
                  const float* params, const int64_t* nids,
                  const int64_t* cids, const int64_t* pids,
                  int64_t num_nodes, int64_t num_elements, int64_t num_params,
                  int64_t num_nblocks, int64_t num_edges, int64_t batch,
                  int64_t block_size, int* err_flag, fl_stream_t stream);
int fl_sparse_q16(float* node_mars, const float* element_mars,
                  const float* params, const int64_t* nids,
                  const int64_t* cids, const int64_t* pids,
                  int64_t num_nodes, int64_t num_elements, int64_t num_params,
                  int64_t num_nblocks, int64_t num_edges, int64_t batch,
                  int64_t block_size, int* err_flag, fl_stream_t stream);

/* ------------------------------------------------------------------------
 * The per-edge log-weight exactly as both sparse kernels form it on the
 * device: logw[i] = __logf(fmaxf(params[i], 1e-45f)), n values.
 * (experiment_pyjuice/sparse_q16_kernel.cu:102 and
 * sparse_float_kernel.cu:76 compute the same expression in shared memory.)  Exposed so a host checker can replay the
 * Q16.16 reduction bit for bit from device-formed log-weights.
 * ---------------------------------------------------------------------- */
int fl_sparse_log_weights(const float* params, float* logw, int64_t n,
                          fl_stream_t stream);

/* ------------------------------------------------------------------------
 * Sparse sum-layer backward (fp32), the gradient of fl_sparse_f32.  With
 * G = node_grads (d loss / d node_mars, (num_nodes, batch)) and node_mars
 * the forward's output, ADDS to the caller's buffers
 *   element_grads[c, b] += sum over edges (k, e, p) with cids[k, e] = c of
 *                          G[n, b] * exp(lw + element_mars[c, b] - node_mars[n, b])
 *   param_grads[q]      += sum over edges with pids[k, e] + p = q and over b of
 *                          G[n, b] * exp(element_mars[c, b] - node_mars[n, b])
 * with n = nids[k] + p and lw = log(max(params[q], 1e-45)); a parameter at or
 * below the clamp gets no gradient, a node whose node_mars is -inf passes
 * none.  Either output may be NULL (not computed).  element_grads needs the
 * child -> parent-unit index of the layer, built once per structure: the
 * parent units (edge, p) of child c are [child_ptr[c], child_ptr[c+1]) of
 * unit_node (their node rows nids[k] + p) and unit_param (pids[k, e] + p);
 * num_units is the length of those two arrays.  Indices out of range are
 * skipped and set *err_flag = 1 when given.  workspace (256-byte aligned, at
 * least fl_sparse_f32_bwd_workspace bytes, contents undefined on entry and
 * exit, one call in flight per workspace) lets the element gradients fold each layer row's G and node_mars
 * into one gathered row first, and, with both outputs requested, takes the
 * parameter gradients from the same child-major pass; NULL gathers both rows
 * per parent and the children's rows per node instead (same results to
 * rounding).  The reference has no backward
 * (experiment_pyjuice/sparse_float_kernel.cu is forward only); no reference
 * counterpart.
 * ---------------------------------------------------------------------- */
int fl_sparse_f32_bwd(const float* node_mars, const float* node_grads,
                      const float* element_mars, const float* params,
                      const int64_t* nids, const int64_t* cids, const int64_t* pids,
                      const int64_t* child_ptr, const int64_t* unit_node,
                      const int64_t* unit_param, int64_t num_units,
                      float* element_grads, float* param_grads, int64_t num_nodes,
                      int64_t num_elements, int64_t num_params, int64_t num_nblocks,
                      int64_t num_edges, int64_t batch, int64_t block_size,
                      void* workspace, int64_t workspace_bytes,
                      int* err_flag, fl_stream_t stream);

/* Bytes of fl_sparse_f32_bwd's workspace for node_mars of (num_nodes, batch)
 * and num_units parent units. */
int fl_sparse_f32_bwd_workspace(int64_t num_nodes, int64_t batch, int64_t num_units,
                                int64_t* bytes);

#ifdef __cplusplus
}
#endif

#endif /* FUSELSE_B200_H */
