// qmm_internal.h -- launch wrappers shared between the kernel files and the
// C-ABI layer.  Not part of the public interface (include/rce_qmm.h is).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "qmm_layout.cuh"

namespace rce {

// GGUF bytes (device) -> T16 tiles (device).  Rows [0, n_rows) of the source.
cudaError_t launch_repack(int dt, const uint8_t *gguf, uint8_t *tiles, const Geometry &g,
                          cudaStream_t s);
// T16 tiles -> GGUF bytes for rows [row0, row1) (dst holds those rows only).
cudaError_t launch_unpack(int dt, const uint8_t *tiles, uint8_t *gguf, const Geometry &g,
                          int64_t row0, int64_t row1, cudaStream_t s);
// Bit-exact dequantize_to_f32 of rows [row0, row1) into out[(row-row0)*ldo + col].
cudaError_t launch_dequant(int dt, const uint8_t *tiles, float *out, size_t ldo, const Geometry &g,
                           int64_t row0, int64_t row1, cudaStream_t s);

// Q6_K (qmm_q6k.cu): repack / unpack / dequant as above, and the decode GEMV
// for m <= kQ6MaxTokens tokens.
constexpr int kQ6MaxTokens = 2;
cudaError_t launch_repack_q6k(const uint8_t *gguf, uint8_t *tiles, const Geometry &g, cudaStream_t s);
cudaError_t launch_unpack_q6k(const uint8_t *tiles, uint8_t *gguf, const Geometry &g, int64_t row0, int64_t row1,
                              cudaStream_t s);
cudaError_t launch_dequant_q6k(const uint8_t *tiles, float *out, size_t ldo, const Geometry &g, int64_t row0,
                               int64_t row1, cudaStream_t s);
int q6k_gemv_warps(const Geometry &g, int sm_count);
cudaError_t launch_gemv_q6k(const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx, float *y,
                            size_t ldy, int m, int sm_count, int *err, cudaStream_t s);

// Fused all-gather of a row-sharded output over peer memory (see
// qmm_gather.cuh): rank `rank` of `world` computes rows [row_off, row_off +
// n) of the output, stores them in its own y, and stores each value with
// the call's epoch, as one 8-byte word, into every other rank's receive
// buffer ll[r] (t rows x ldy words, as addressable here) at the same place.
// The epoch is `epoch` (+ *epoch_base when set, read on the device).
constexpr int kMaxPeers = 8;
struct GatherArgs {
    int world = 1, rank = 0;
    int64_t row_off = 0;
    unsigned long long *ll[kMaxPeers] = {};
    unsigned epoch = 0;
    const unsigned *epoch_base = nullptr;
};

// Decode GEMV / small-M matmul: y[t][row] = sum_k x[t][k] W[row][k], for
// t < m <= kGemvMaxTokens, rows [0, n_rows).  `err` (device-visible int)
// receives a non-zero code if a bounded wait inside the kernel expires.
constexpr int kGemvMaxTokens = 4;
struct GemvPlan {
    int clusters = 1;    // clusters of two CTAs, each owning a block of whole tiles
    int panels = 1;      // K halves a cluster's units are ordered by (1 or 2)
    int kmax = 2;        // partial-sum slots per warp
    int nt = 1;          // token slots compiled in (1, 2 or 4); larger batches take several launches
    int stages = 4;      // TMA ring depth per warp
    int window = 16;     // chunks of activations staged per CTA (the largest)
    size_t smem = 0;     // dynamic shared memory
};
GemvPlan plan_gemv(int dt, const Geometry &g, int m, int sm_count);
cudaError_t launch_gemv(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx,
                        float *y, size_t ldy, int m, const GemvPlan &plan, int *err, cudaStream_t s,
                        const GatherArgs *ga = nullptr);
// Up to kGemvMaxGroup weights with the same dtype and K (n_cols) read by one
// launch, each into its own output (y[i]: [m][ldy[i]]).  The grid splits the
// weights' tiles as one matrix, so small matrices sharing an activation
// (attention q, k, v; FFN gate, up) cost one launch.  Plan it with
// plan_gemv(dt, group_geometry(grp), m, sm_count).  Gathered outputs: ga
// holds one GatherArgs per weight (same world, rank and epoch; each its own
// row offset and receive buffers), or is null.
constexpr int kGemvMaxGroup = 4;
struct GemvGroup {
    int n = 0;
    const uint8_t *w[kGemvMaxGroup] = {};
    Geometry g[kGemvMaxGroup] = {};
    float *y[kGemvMaxGroup] = {};
    size_t ldy[kGemvMaxGroup] = {};
};
Geometry group_geometry(const GemvGroup &grp);
cudaError_t launch_gemv_group(int dt, const GemvGroup &grp, const float *x, size_t ldx, int m,
                              const GemvPlan &plan, int *err, cudaStream_t s, const GatherArgs *ga = nullptr);
// Gather helpers.  push: for kernels that write only locally (the prefill
// GEMM), store rows [0, t_rows) x [row_off, row_off + n) of y (leading
// dimension ldy) into the peers' receive buffers.  unpack: wait (bounded)
// until this rank's receive buffer `ll` holds epoch e (+ *epoch_base) in
// every word of the rows other ranks own -- rows [0, t_rows), columns
// [0, n) except [own0, own1) -- and copy those values into y.
cudaError_t launch_gather_push(const GatherArgs &ga, const float *y, int t_rows, int64_t n, size_t ldy,
                               cudaStream_t s);
cudaError_t launch_gather_unpack(const unsigned long long *ll, float *y, int t_rows, int64_t n, size_t ldy,
                                 int64_t own0, int64_t own1, unsigned epoch, const unsigned *epoch_base, int *err,
                                 cudaStream_t s);
cudaError_t launch_epoch_advance(unsigned *epoch_base, unsigned delta, cudaStream_t s);
// Bulk mode (large outputs): push rows [row_off, row_off + n_own) of
// y[t_rows][ldy] as plain f32 into every peer's bulk buffer (same
// positions), then release flag slot `rank` of each peer's flags (at byte
// flag_off of its buffer) with the call's epoch; unpack waits (bounded) for
// every other rank's flag and copies their rows.
cudaError_t launch_gather_push_bulk(int world, int rank, float *const *peer_bufs, size_t flag_off, const float *y,
                                    int t_rows, int64_t row_off, int64_t n_own, size_t ldy, unsigned epoch,
                                    const unsigned *epoch_base, cudaStream_t s);
// Only the flags of a bulk push whose values are already in the peers'
// buffers (stored by the GEMM itself, BulkPush): one system-scope release of
// the epoch into slot `rank` of each peer's flags.
cudaError_t launch_gather_flags_bulk(int world, int rank, float *const *peer_bufs, size_t flag_off, unsigned epoch,
                                     const unsigned *epoch_base, cudaStream_t s);
cudaError_t launch_gather_unpack_bulk(const float *buf, size_t flag_off, float *y, int t_rows, int64_t n, size_t ldy,
                                      int64_t own0, int64_t own1, int world, int rank, unsigned epoch,
                                      const unsigned *epoch_base, int *err, cudaStream_t s);

// Prefill matmul on tcgen05 (fp16 operands, f32 accumulation in tensor
// memory) for t_rows tokens at once.  `workspace` holds
// gemm_workspace_bytes() bytes (the fp16 activations and per-token scales).
// Batches of up to kGemmTwoTermMaxTokens tokens carry each activation as two
// fp16 terms (gemm_terms() == 2: high + low, about 22 significant bits).
constexpr int kGemmTwoTermMaxTokens = 64;
int gemm_terms(int t_rows);
// Weights of few row blocks (row shards) split K over CTAs when their
// workspace -- activations, inverse scales and partial outputs -- stays
// within this many bytes (the allocation-free entry point's fixed array, so
// both entry points run a batch the same way).
constexpr size_t kGemmSplitWorkspace = size_t(16) << 20;
size_t gemm_workspace_bytes(int dt, const Geometry &g, int t_rows);
// Bulk all-gather fused into the GEMM: every output value the GEMM writes at
// y[t * ldy + r] is also stored at peer[p][t * ldy + r] for each peer p (the
// peers' bulk buffers, offset by this rank's row offset; entries of this
// rank and of ranks beyond world are ignored).  Release the flags with
// launch_gather_flags_bulk after the GEMM.
struct BulkPush {
    int world = 0, rank = 0;
    float *peer[kMaxPeers] = {};
};
cudaError_t launch_gemm(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx, float *y,
                        size_t ldy, int t_rows, void *workspace, int *err, cudaStream_t s,
                        const BulkPush *push = nullptr);

// Expert-grouped prefill matmul: one launch for up to kGemmMaxGroup weights
// of one shape.  Entry z multiplies ws[z] by the two-term fp16 activation
// rows [off[set[z]], off[set[z] + 1]) of xh ([2][rows][g.n_cols]: high terms,
// then low terms, scaled per row as the MoE prep kernels write them, 1/scale
// in inv) into the same rows of ys[z] (row stride ldy).  off (n_sets + 1 entries) is read on the device; no set
// may hold more than max_rows rows; rows_hint (the expected rows over all
// sets) sizes the token tile.
constexpr int kGemmMaxGroup = 32;
// The grouped launch's epilogue (GroupEpilogue): kGroupStore stores each
// output row; kGroupSwiGLU takes entry z's gate weight from ws and its up
// weight from ws2 (same shape), 64 rows of each per CTA, and stores
// h = silu(gate) * up (the f32 arithmetic of the separate SwiGLU); kGroupCombine
// adds row_w[r] * y into out[row_token[r]] atomically instead of storing y
// (out cleared beforehand; exact and order-free for at most two route slots
// per token, as a + b = b + a and 0 + a = a).
enum GroupEpilogue { kGroupStore = 0, kGroupSwiGLU = 1, kGroupCombine = 2 };
struct GroupEpi {
    int mode = kGroupStore;
    const uint8_t *const *ws2 = nullptr;  // kGroupSwiGLU: up weights, entry by entry
    const int32_t *row_token = nullptr;   // kGroupCombine
    const float *row_w = nullptr;
    float *out = nullptr;
    size_t ldo = 0;
};
cudaError_t launch_gemm_grouped(int dt, const uint8_t *const *ws, float *const *ys, const int *set, int n,
                                const Geometry &g, const void *xh, const float *inv, int rows, int rows_hint,
                                const int32_t *off, int n_sets, int max_rows, size_t ldy, int *err, cudaStream_t s,
                                const GroupEpi &epi = GroupEpi());

// MoE pieces (qmm_moe.cu).  route: per token softmax / top_k / renormalise
// of router logits [t_rows][ld] into idx, w [t_rows][top_k] (n_experts <=
// 256).  plan: rows for the (token, slot) pairs whose expert lies in
// [e_begin, e_end), grouped by expert: offsets [n_local + 1], pos [pairs]
// (-1: not local), token [rows].  gather: xg[row] = x[token[row]].
// swiglu: h = silu(g) * u.  combine: out[t] = sum_j w[t][j] y[pos[t][j]].
cudaError_t launch_moe_route(const float *logits, size_t ld, int t_rows, int n_experts, int top_k, int normalize,
                             int32_t *idx, float *w, cudaStream_t s);
cudaError_t launch_moe_plan(const int32_t *idx, const float *w, int pairs, int top_k, int e_begin, int e_end,
                            int32_t *offsets, int32_t *pos, int32_t *token, float *row_w, cudaStream_t s);
// route then plan in one single-CTA launch (also row_w[row] = w[pair] when
// row_w is given)
cudaError_t launch_moe_route_plan(const float *logits, size_t ld, int t_rows, int n_experts, int top_k, int normalize,
                                  int32_t *idx, float *w, int e_begin, int e_end, int32_t *offsets, int32_t *pos,
                                  int32_t *token, float *row_w, cudaStream_t s);
cudaError_t launch_moe_gather(const float *x, size_t ldx, const int32_t *token, int rows, int d_model, float *xg,
                              cudaStream_t s);
cudaError_t launch_swiglu(const float *g, const float *u, float *h, size_t n, cudaStream_t s);
// The GEMM inputs of the grouped path, for rows r < *n_rows (a device
// count; max_rows bounds it): gather_prep v = x[token[r]], h_prep v = h[r]
// (rows of ld floats), each as two fp16 terms xh[r] = fp16(v * s_r) and
// xh[max_rows + r] = fp16(v * s_r - xh[r]); s_r a power of two with
// |v * s_r| < 2^14, inv[r] = 1 / s_r.  gather_prep also clears rows
// [0, zero_rows) of zero (d_model floats each) when zero is given.
cudaError_t launch_moe_gather_prep(const float *x, size_t ldx, const int32_t *token, const int32_t *n_rows,
                                   int max_rows, int d_model, void *xh, float *inv, float *zero, size_t ldz,
                                   int zero_rows, cudaStream_t s);
cudaError_t launch_moe_h_prep(const float *h, size_t ld, const int32_t *n_rows, int max_rows, int d_ff, void *xh,
                              float *inv, cudaStream_t s);
// The shared expert's gate and add: out[t] += sigmoid(gate_inp . x[t]) * sh[t].
cudaError_t launch_moe_shared_combine(const float *x, size_t ldx, int t_rows, int d_model, const float *gate_inp,
                                      const float *sh, size_t ldsh, float *out, size_t ldo, cudaStream_t s);
cudaError_t launch_moe_combine(const float *y, int d_model, const int32_t *pos, const float *w, int t_rows, int top_k,
                               float *out, size_t ldo, cudaStream_t s);

// Kernel error codes written to the context's error word.
constexpr int kKernelErrWaitTimeout = 1;
// A bulk receive buffer already held a later call's rows when its unpack
// looked (a peer ran more than one call ahead into the same buffer).
constexpr int kKernelErrOverrun = 2;

}  // namespace rce
