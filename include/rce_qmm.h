/*
 * rce_qmm.h -- C ABI of the B200 GGUF quantized-matmul library
 * (librce_qmm.so), the drop-in for the reference crate rce-op-qmm's operator
 * API for the Q8_0, Q4_0, Q4_K, Q5_K and Q6_K weight formats.
 *
 * Reference interfaces replaced (paths relative to openIE-dev/rce,
 * compute/crates/):
 *   QuantWeight          rce-op-qmm/src/lib.rs:77-210
 *   mm_1d                rce-op-qmm/src/lib.rs:216-270
 *   mm_1d_serial         rce-op-qmm/src/lib.rs:281-304
 *   mm_batched           rce-op-qmm/src/lib.rs:967-1023
 *   QuantWeight::dequant_row / dequantize_to_f32
 *                        rce-op-qmm/src/lib.rs:150-166, rce-ingest-gguf/src/dequant.rs:115-134
 *   tensor_byte_size     rce-ingest-gguf/src/dequant.rs:18-58
 *   QmmDispatch::qmm_1d  rce-placement-adapter/src/lib.rs:130-134
 *   QmmLeaf::execute     rce-op-qmm/src/lib.rs:2096-2130
 *   moe_router / moe_combine
 *                        rce-op-moe/src/lib.rs:35-73, 98-110
 *   moe_ffn_forward      rce-qwen36-moe/src/lib.rs:666-705 (routed experts; the
 *                        shared expert, :684-705, rce_qmm_moe_shared_expert_device)
 *
 * Conventions (after the reference's own C ABI, rce-c/src/lib.rs:8-100):
 *   - every function returns RCE_QMM_OK (0) or an error code; the message of
 *     the last failure on the calling thread is rce_qmm_last_error();
 *   - inputs are borrowed for the duration of the call; handles are freed by
 *     the matching *_free / *_destroy function;
 *   - "host" entry points take host pointers and copy in and out themselves
 *     (synchronous); "_device" entry points take device pointers and a
 *     cudaStream_t (passed as void*, NULL = the context's default stream) and
 *     are asynchronous on that stream;
 *   - every entry point is thread-safe: each calling thread gets its own
 *     stream and staging buffers, as the reference's callers run qmm from many
 *     rayon threads at once (rce-qwen36-moe/src/lib.rs:688-698).
 * Where the reference panics (mm_1d on an unsupported dtype, lib.rs:268) or
 * returns InterpretError::Unsupported (QmmLeaf), this ABI returns
 * RCE_QMM_ERR_UNSUPPORTED or RCE_QMM_ERR_INVALID.
 */
#ifndef RCE_QMM_H
#define RCE_QMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RCE_QMM_ABI_VERSION 1

/* Status codes. */
#define RCE_QMM_OK 0
#define RCE_QMM_ERR_INVALID 1     /* bad argument: null pointer, size, shape */
#define RCE_QMM_ERR_UNSUPPORTED 2 /* dtype or shape outside this library */
#define RCE_QMM_ERR_CUDA 3        /* a CUDA runtime call failed */
#define RCE_QMM_ERR_NOMEM 4       /* device or host allocation failed */
#define RCE_QMM_ERR_TIMEOUT 5     /* a bounded wait inside a kernel expired, or a gathered
                                   * output's buffer was overwritten by a later call */

/* GGUF dtype tags (rce-ingest-gguf/src/parser.rs:308-338). */
#define RCE_QMM_GGUF_Q4_0 2
#define RCE_QMM_GGUF_Q8_0 8
#define RCE_QMM_GGUF_Q4_K 12
#define RCE_QMM_GGUF_Q5_K 13
#define RCE_QMM_GGUF_Q6_K 14

typedef struct rce_qmm_ctx rce_qmm_ctx;
typedef struct rce_qmm_weight rce_qmm_weight;

/* ABI version (RCE_QMM_ABI_VERSION). */
int rce_qmm_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char *rce_qmm_last_error(void);

/* Bytes of a GGUF tensor of `numel` values (tensor_byte_size,
 * rce-ingest-gguf/src/dequant.rs:18-58); 0 for dtypes outside this library. */
size_t rce_qmm_tensor_byte_size(int gguf_dtype, uint64_t numel);

/* A context binds one CUDA device. */
int rce_qmm_ctx_create(int device, rce_qmm_ctx **out);
int rce_qmm_ctx_destroy(rce_qmm_ctx *ctx);
/* Number of SMs of the context's device. */
int rce_qmm_ctx_sm_count(const rce_qmm_ctx *ctx, int *out);
/* mm_batched (host and device) runs the tensor-core prefill GEMM for batches
 * of at least `n` tokens (default 16): weights dequantised to fp16 and
 * activations rounded to fp16 with a per-token power-of-two scale, f32
 * accumulation, within the 1e-3 normwise bar but not bit-identical to mm_1d.
 * Smaller batches take the decode path, whose results per token are
 * bit-identical to mm_1d whatever the batch, as the reference's mm_batched
 * guarantees (rce-op-qmm/src/lib.rs:2575-2616).  n = 0 keeps every batch on
 * the decode path. */
int rce_qmm_ctx_set_prefill_min_tokens(rce_qmm_ctx *ctx, int n);
int rce_qmm_ctx_get_prefill_min_tokens(const rce_qmm_ctx *ctx, int *n);

/* Register a GGUF weight [n_rows = N_out][n_cols = K_in] (row-major blocks,
 * the layout QuantWeight keeps, rce-op-qmm/src/lib.rs:15-19).  The bytes are
 * copied to the device once and repacked into the device tile layout (a byte
 * permutation: same byte count, recoverable bit for bit).  n_cols must be a
 * multiple of the block size (32; 256 for Q4_K, Q5_K and Q6_K) and nbytes must equal
 * rce_qmm_tensor_byte_size(dtype, n_rows * n_cols). */
int rce_qmm_weight_register(rce_qmm_ctx *ctx, const void *gguf_bytes, size_t nbytes, int gguf_dtype,
                            int64_t n_rows, int64_t n_cols, rce_qmm_weight **out);
/* As rce_qmm_weight_register, from GGUF bytes already in device memory. */
int rce_qmm_weight_register_device(rce_qmm_ctx *ctx, const void *d_gguf_bytes, size_t nbytes,
                                   int gguf_dtype, int64_t n_rows, int64_t n_cols, void *stream,
                                   rce_qmm_weight **out);
/* Zero-copy sub-view (QuantWeight::sub_view, rce-op-qmm/src/lib.rs:99-118),
 * e.g. one expert of a stacked [n_expert * n_rows, n_cols] tensor.  The view
 * must start on a row that is a multiple of 16 and keep n_cols; byte_offset and
 * byte_len are GGUF byte counts relative to the parent.  The parent must
 * outlive the view. */
int rce_qmm_weight_sub_view(const rce_qmm_weight *parent, size_t byte_offset, size_t byte_len,
                            int64_t n_rows, int64_t n_cols, rce_qmm_weight **out);
int rce_qmm_weight_free(rce_qmm_weight *w);
/* dtype, shape and GGUF byte count of a weight. */
int rce_qmm_weight_info(const rce_qmm_weight *w, int *gguf_dtype, int64_t *n_rows, int64_t *n_cols,
                        size_t *nbytes);
/* Device address and byte count of the tile storage (for tools/tests). */
int rce_qmm_weight_device_storage(const rce_qmm_weight *w, const void **dev_ptr, size_t *dev_bytes);
/* The weight's GGUF bytes (QuantWeight::bytes, rce-op-qmm/src/lib.rs:87-91),
 * rebuilt from the device tiles into host memory (nbytes = the GGUF size). */
int rce_qmm_weight_read_bytes(const rce_qmm_weight *w, void *host_out, size_t nbytes);

/* out[j] = a . W[j,:] for j < n_rows (mm_1d, rce-op-qmm/src/lib.rs:216).
 * a_len must equal n_cols, out_len >= n_rows.  Host buffers, synchronous. */
int rce_qmm_mm_1d(rce_qmm_ctx *ctx, const float *a, size_t a_len, const rce_qmm_weight *w, float *out,
                  size_t out_len);
/* mm_1d_serial (rce-op-qmm/src/lib.rs:281): identical results to mm_1d. */
int rce_qmm_mm_1d_serial(rce_qmm_ctx *ctx, const float *a, size_t a_len, const rce_qmm_weight *w,
                         float *out, size_t out_len);
/* out[T, n_rows] = a[T, n_cols] . W^T (mm_batched, rce-op-qmm/src/lib.rs:967).
 * Host buffers, synchronous.  Below the context's prefill_min_tokens
 * (default 16) every token's row is bit-identical to mm_1d's, the reference's
 * mm_batched guarantee (lib.rs:2575-2616); from there on the tensor-core GEMM
 * (fp16 weights, activations as two fp16 terms up to 64 tokens, one above)
 * holds each output row within 1e-3 of the f32 result but not bit for bit.
 * Callers that need the identity at every batch size set prefill_min_tokens
 * to 0 (rce_qmm_ctx_set_prefill_min_tokens). */
int rce_qmm_mm_batched(rce_qmm_ctx *ctx, const float *a, size_t t_rows, const rce_qmm_weight *w,
                       float *out, size_t out_len);
/* Device variant: d_a is [t_rows][lda] f32, d_out [t_rows][ldo] f32. */
int rce_qmm_mm_batched_device(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                              const rce_qmm_weight *w, float *d_out, size_t ldo, void *stream);

/* n_w (1..4) rce_qmm_mm_batched_device calls that share their activations,
 * in one launch: d_outs[i] ([t_rows][ldos[i]] f32) = d_a . ws[i]^T.  The
 * weights must have the same dtype and n_cols.  No counterpart in the
 * reference (it runs mm_batched per weight, rce-op-qmm/src/lib.rs); serving
 * code uses it for matrices that read the same input (attention q, k, v; FFN
 * gate, up), whose tiles the decode GEMV then splits over the GPU as one
 * matrix.  Batches of prefill_min_tokens or more run the tensor-core GEMM per
 * weight.  Per-weight results equal rce_qmm_mm_batched_device's to the
 * tolerance of the decode path (the summation order follows the group's
 * split); within a group, every token's result is independent of the batch
 * size. */
int rce_qmm_mm_batched_device_multi(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                    const rce_qmm_weight *const *ws, size_t n_w, float *const *d_outs,
                                    const size_t *ldos, void *stream);

/* As rce_qmm_mm_batched_device, for callers that cannot allocate device
 * memory: an engine whose own allocator has reserved the whole device, or a
 * serving loop that forbids cudaMalloc after start-up.  No counterpart in the
 * reference: its CPU path never allocates device memory.  The regular entry
 * point allocates the tensor-core GEMM's workspace (fp16 activations and
 * per-token scales) on first use; this one keeps it in one fixed 16 MiB
 * device array per GPU, held from library load to process exit, and calls no
 * cudaMalloc, cudaFree or allocating library routine.  Outputs equal
 * rce_qmm_mm_batched_device's bit for bit under the same context settings.
 * Limits: a GEMM batch (prefill_min_tokens tokens or more) needing more than
 * 16 MiB of workspace -- t_rows * n_cols * 2 bytes (twice that for batches of
 * up to 64 tokens, whose activations the GEMM carries as two fp16 terms)
 * rounded up to 256, plus 4 bytes per token rounded up to 256; 2047 tokens at
 * n_cols 4096 -- is rejected with RCE_QMM_ERR_INVALID.  (Weights of few rows,
 * such as row shards, may also keep split-K partial sums there, on both
 * entry points alike, only when they fit the 16 MiB.)  Every call on a GPU shares the array, whatever its
 * context or stream, so calls that overlap on the GPU race: order them.  The
 * array keeps the last call's contents; nothing in it needs to start at zero.
 * The first call on each GPU looks up the array's device address, so make it
 * before any stream capture; the address is kept for the life of the
 * process, so, like every handle of this library, the entry point must not
 * be used after cudaDeviceReset.  A weight too large for the decode GEMV's
 * shared-memory plan is rejected with RCE_QMM_ERR_UNSUPPORTED. */
int rce_qmm_mm_batched_device_noalloc(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                      const rce_qmm_weight *w, float *d_out, size_t ldo, void *stream);

/* dequant_row (rce-op-qmm/src/lib.rs:150-166): n_cols f32 values of row
 * `row`, bit-exact with dequantize_to_f32.  Host output, synchronous. */
int rce_qmm_dequant_row(rce_qmm_ctx *ctx, const rce_qmm_weight *w, int64_t row, float *out,
                        size_t out_len);
/* Device variant: rows [row0, row1) into d_out[(row - row0) * ldo + col]. */
int rce_qmm_dequant_device(rce_qmm_ctx *ctx, const rce_qmm_weight *w, int64_t row0, int64_t row1,
                           float *d_out, size_t ldo, void *stream);

/* The context's kernel error word: 0, or the code a kernel recorded when one
 * of its bounded waits expired (its outputs are then invalid).  Host entry
 * points check it themselves and return RCE_QMM_ERR_TIMEOUT; after
 * asynchronous _device calls, synchronise the stream and read it here.
 * clear != 0 re-arms it. */
int rce_qmm_device_error(rce_qmm_ctx *ctx, int *code, int clear);

/* Wait for all work this thread queued on the context's streams. */
int rce_qmm_synchronize(rce_qmm_ctx *ctx);

/* ---- row sharding over GPUs, all-gather fused over peer memory ------------ */

/* The reference splits a matmul's rows over the threads of one host (rayon
 * in mm_1d_q4_0 / mm_1d_q8_0 / mm_1d_q4_k, rce-op-qmm/src/lib.rs:502, 654,
 * 742: rows are independent, so the split changes no result).  Its
 * multi-GPU counterpart here shards rows over the GPUs of one node and
 * gathers the outputs with NVLink stores from the matmul itself.  These
 * entry points have no counterpart in the reference.
 *
 * Device memory that the other processes of the node can map: `bytes`
 * zeroed bytes at *d_ptr, and its 64-byte CUDA IPC handle in ipc_handle. */
int rce_qmm_peer_alloc(rce_qmm_ctx *ctx, size_t bytes, void **d_ptr, void *ipc_handle);
int rce_qmm_peer_free(rce_qmm_ctx *ctx, void *d_ptr);
/* Map another process's rce_qmm_peer_alloc buffer (its 64-byte handle). */
int rce_qmm_peer_open(rce_qmm_ctx *ctx, const void *ipc_handle, void **d_ptr);
int rce_qmm_peer_close(rce_qmm_ctx *ctx, void *d_ptr);

/* mm_batched for rank `rank` of `world` (2..8) holding rows [row_offset,
 * row_offset + w.n_rows) of a row-sharded weight.  The rows' outputs go to
 * this rank's full output d_y ([t_rows][ldy], at row_offset) and, as 8-byte
 * words {value, epoch} written over NVLink, into every other rank's
 * receive buffer d_ll[r] (t_rows x ldy words, as addressable in this
 * context; rce_qmm_peer_alloc memory) at the same place.  No fence, flag or
 * collective: a receiver knows a word has arrived when it carries the
 * epoch it expects (rce_qmm_peer_unpack).  Use a new epoch for every call
 * that writes a given receive buffer (epochs only grow; 0 is never valid). */
int rce_qmm_mm_batched_device_gather(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                     const rce_qmm_weight *w, int world, int rank, int64_t row_offset,
                                     float *d_y, size_t ldy, unsigned long long *const *d_ll, unsigned epoch,
                                     const unsigned *d_epoch_base, void *stream);
/* rce_qmm_mm_batched_device_gather for 1..4 weights that share their
 * activations (one launch, as rce_qmm_mm_batched_device_multi): weight i's
 * rows go to d_ys[i] (+ row_offsets[i], leading dimension ldys[i]) and, as
 * {value, epoch} words, to every other rank's receive buffer
 * d_lls[i * world + r].  One epoch for all the outputs of the call. */
int rce_qmm_mm_batched_device_multi_gather(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                           const rce_qmm_weight *const *ws, size_t n_w, int world, int rank,
                                           const int64_t *row_offsets, float *const *d_ys, const size_t *ldys,
                                           unsigned long long *const *d_lls, unsigned epoch,
                                           const unsigned *d_epoch_base, void *stream);

/* Bulk mode of the gathered matmul, for large outputs (prefill batches; no
 * counterpart in the reference): the matmul per weight (the tensor-core
 * GEMM from prefill_min_tokens tokens), then this rank's rows as plain f32
 * into every other rank's bulk buffer d_bulks[i * world + r] at the same
 * [t][ldys[i]] positions, then one flag per peer (slot `rank` of the u32
 * flags at byte flag_offsets[i] of the peer's buffer, after the values)
 * released at system scope with the call's epoch.  Half the NVLink bytes of
 * the {value, epoch} words.  The receiver calls rce_qmm_peer_unpack_bulk. */
int rce_qmm_mm_batched_device_multi_gather_bulk(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                                const rce_qmm_weight *const *ws, size_t n_w, int world, int rank,
                                                const int64_t *row_offsets, float *const *d_ys, const size_t *ldys,
                                                float *const *d_bulks, const size_t *flag_offsets, unsigned epoch,
                                                const unsigned *d_epoch_base, void *stream);
/* Wait (bounded) until every other rank's flag in this rank's bulk buffer
 * carries the epoch, then copy their rows (columns [0, n) except
 * [own0, own1)) of the [t_rows][ldy] values into d_y.  The values carry no
 * epoch, so a peer must not write the next call's rows into a bulk buffer
 * that is still being unpacked: alternate two bulk buffers per output (a
 * peer may then run one call ahead, not two).  A flag that already carries
 * a later epoch is reported in the device error word (code 2) and nothing
 * is copied. */
int rce_qmm_peer_unpack_bulk(rce_qmm_ctx *ctx, const float *d_bulk, size_t flag_offset, float *d_y, size_t ldy,
                             size_t t_rows, int64_t n, int64_t own0, int64_t own1, int world, int rank, unsigned epoch,
                             const unsigned *d_epoch_base, void *stream);

/* Complete a gathered output on this rank: wait (bounded, 1 s; an expired
 * wait sets the device error word) until every word of d_ll in rows
 * [0, t_rows) and columns [0, n) outside this rank's [own0, own1) carries
 * `epoch` or a later one, and copy those values into d_y.  (A later epoch
 * means a later call already overwrote that word: keep peers from running
 * ahead into a buffer that is still being unpacked when its values matter,
 * e.g. with alternating buffers.) */
int rce_qmm_peer_unpack(rce_qmm_ctx *ctx, const unsigned long long *d_ll, float *d_y, size_t ldy, size_t t_rows,
                        int64_t n, int64_t own0, int64_t own1, unsigned epoch, const unsigned *d_epoch_base,
                        void *stream);
/* d_epoch_base (optional, device memory): when given, the epochs of the two
 * calls above are relative to *d_epoch_base, read on the device, so that
 * calls captured in a CUDA graph use new epochs on every replay; advance it
 * (on the stream, before the replayed calls) with: */
int rce_qmm_peer_epoch_advance(rce_qmm_ctx *ctx, unsigned *d_epoch_base, unsigned delta, void *stream);

/* ---- expert-grouped MoE FFN ---------------------------------------------- */

/* moe_router (rce-op-moe/src/lib.rs:35-73) on given router logits, on the
 * device: for each of t_rows tokens, softmax over n_experts (<= 256) logits
 * at d_logits[t * ld_logits], the top_k largest probabilities (ties to the
 * lower expert index) into d_idx[t * top_k + j] / d_w[...], renormalised to
 * sum 1 when normalize != 0.  Asynchronous on `stream`. */
int rce_qmm_moe_route_device(rce_qmm_ctx *ctx, const float *d_logits, size_t ld_logits, size_t t_rows,
                             int n_experts, int top_k, int normalize, int32_t *d_idx, float *d_w, void *stream);

/* moe_router (rce-op-moe/src/lib.rs:35-73) with the router's quantized gate
 * weight router_w [n_experts x d_model] (n_experts <= 256): per token the
 * logits router_w . x, computed as mm_batched computes them (the decode
 * path, per token as mm_1d, below the context's prefill_min_tokens; set it
 * to 0 for that path at every batch size), into d_logits [t_rows][ld_logits],
 * then softmax / top_k / renormalise as rce_qmm_moe_route_device.
 * Asynchronous on `stream`. */
int rce_qmm_moe_router_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                              const rce_qmm_weight *router_w, int top_k, int normalize, float *d_logits,
                              size_t ld_logits, int32_t *d_idx, float *d_w, void *stream);

/* The expert-grouped SwiGLU FFN of moe_ffn_forward
 * (rce-qwen36-moe/src/lib.rs:666-705) with moe_router / moe_combine
 * (rce-op-moe/src/lib.rs:35-110): route every token as
 * rce_qmm_moe_route_device does (normalised), then for each routed expert e
 * g = W_gate[e] x, u = W_up[e] x, h = silu(g) * u, y = W_down[e] h, and
 * out[t] = sum over route slots j, in order, of w_j * y_j.  Experts outside
 * [expert_begin, expert_end) are skipped (their slots add nothing), so with
 * the experts placed across GPUs the sum of every GPU's output is the full
 * FFN (for top_k <= 2 bit for bit: adding zeros and swapping two terms
 * round alike).  gate/up/down hold n_experts weight handles each (entries
 * outside the local range may be NULL); gate/up are [d_ff x d_model], down
 * [d_model x d_ff].  From prefill_min_tokens tokens (and experts of one
 * format) the experts run as expert-grouped tensor-core launches with the
 * row counts read on the device (no host synchronisation: the call can be
 * captured in a CUDA graph); below, each expert's rows run through
 * mm_batched's dispatch, sized by row counts the call copies to the host
 * (one synchronisation of `stream`).  Device buffers; a per-stream
 * workspace grows on first use.  d_idx / d_w (optional, [t_rows][top_k])
 * receive the routes. */
int rce_qmm_moe_ffn_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                           const float *d_logits, size_t ld_logits, int n_experts, int top_k,
                           int expert_begin, int expert_end, const rce_qmm_weight *const *gate,
                           const rce_qmm_weight *const *up, const rce_qmm_weight *const *down, float *d_out,
                           size_t ldo, int32_t *d_idx, float *d_w, void *stream);

/* The always-on shared expert of moe_ffn_forward
 * (rce-qwen36-moe/src/lib.rs:684-705), added into out:
 * sh = W_down (silu(W_gate x) * (W_up x)) with the shared weights, then
 * out[t] += sigmoid(gate_inp . x[t]) * sh[t], the dot product summed left
 * to right in f32.  Called after rce_qmm_moe_ffn_device on the same out it
 * completes moe_ffn_forward: the routed combine first, then the shared term,
 * the order in which the reference adds them.  gate/up [n_ff x d_model],
 * down [d_model x n_ff]; gate_inp device f32 [d_model].  The matmuls run
 * through mm_batched's dispatch.  Asynchronous on `stream`; uses the
 * stream's MoE workspace. */
int rce_qmm_moe_shared_expert_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                                     const rce_qmm_weight *gate, const rce_qmm_weight *up,
                                     const rce_qmm_weight *down, const float *d_gate_inp, float *d_out,
                                     size_t ldo, void *stream);

/* Host-buffer rce_qmm_moe_ffn_device, synchronous (the MoE FFN call of the
 * reference's runtimes, rce-qwen36-moe/src/lib.rs:666-705, routed by
 * moe_router, rce-op-moe/src/lib.rs:35-73): x [t_rows][d_model] and out
 * [t_rows][d_model] host f32.  The routes come from router_logits
 * ([t_rows][n_experts] host f32) or, when it is NULL, from the gate weight
 * router_w as rce_qmm_moe_router_device computes them.  idx_out / w_out
 * (optional, host, [t_rows][top_k]) receive the routes. */
int rce_qmm_moe_ffn(rce_qmm_ctx *ctx, const float *x, size_t t_rows, const float *router_logits,
                    const rce_qmm_weight *router_w, int n_experts, int top_k, int expert_begin, int expert_end,
                    const rce_qmm_weight *const *gate, const rce_qmm_weight *const *up,
                    const rce_qmm_weight *const *down, float *out, int32_t *idx_out, float *w_out);

#ifdef __cplusplus
}
#endif
#endif /* RCE_QMM_H */
