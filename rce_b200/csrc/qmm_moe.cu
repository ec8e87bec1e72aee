// qmm_moe.cu -- the device side of the expert-grouped MoE FFN: routing,
// grouping of (token, route slot) pairs by expert, the gather of their
// activations, the SwiGLU product between the gate/up and down matmuls, and
// the weighted combine.  The matmuls themselves are the library's quantized
// matmul (qmm_gemv.cu / qmm_gemm.cu) over each expert's rows.
//
// Reference: moe_router and moe_combine (rce-op-moe/src/lib.rs:35-110) and
// the SwiGLU expert FFN moe_ffn_forward (rce-qwen36-moe/src/lib.rs:666-705,
// silu :649-656).
#include <cuda_runtime.h>

#include <cstdint>

#include "qmm_internal.h"
#include "qmm_prep.cuh"

namespace rce {
namespace {

// One thread per token: softmax over all experts (max subtracted), the
// top_k largest probabilities (ties to the lower expert index), optionally
// renormalised to sum 1 -- the arithmetic of moe_router
// (rce-op-moe/src/lib.rs:49-72): exp of (l - max), a left-to-right f32 sum,
// one IEEE division per probability, the selected weights summed in rank
// order.  exp is the device expf (the reference uses the platform libm; the
// two may differ in the last bit).
__device__ __forceinline__ void route_token(const float *logits, size_t ld, int t, int n_experts, int top_k,
                                            int normalize, int32_t *idx, float *w) {
    const float *l = logits + (size_t)t * ld;
    float mx = -INFINITY;
    for (int e = 0; e < n_experts; e++) mx = fmaxf(mx, l[e]);
    float sum = 0.f;
    for (int e = 0; e < n_experts; e++) sum = sum + expf(l[e] - mx);
    // top_k by repeated selection of the largest remaining probability;
    // each probability is recomputed exactly as above (same operands, same
    // rounding), so no per-expert array is needed
    uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // bit set of chosen experts (n_experts <= 256)
    float s = 0.f;
    for (int j = 0; j < top_k; j++) {
        int best = -1;
        float bp = 0.f;
        for (int e = 0; e < n_experts; e++) {
            if (taken[e >> 5] & (1u << (e & 31))) continue;
            float p = expf(l[e] - mx);
            if (sum > 0.f) p = p / sum;
            if (best < 0 || p > bp) {  // strictly greater: ties keep the lower index
                best = e;
                bp = p;
            }
        }
        taken[best >> 5] |= 1u << (best & 31);
        idx[(size_t)t * top_k + j] = best;
        w[(size_t)t * top_k + j] = bp;
    }
    if (normalize) {
        for (int j = 0; j < top_k; j++) s = s + w[(size_t)t * top_k + j];
        if (s > 0.f)
            for (int j = 0; j < top_k; j++) w[(size_t)t * top_k + j] = w[(size_t)t * top_k + j] / s;
    }
}

__global__ void route_kernel(const float *logits, size_t ld, int t_rows, int n_experts, int top_k, int normalize,
                             int32_t *idx, float *w) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < t_rows) route_token(logits, ld, t, n_experts, top_k, normalize, idx, w);
}

// One CTA: rows for the (token, slot) pairs routed to experts [e_begin,
// e_end), grouped by expert.  offsets[i] = first row of local expert i
// (offsets[n_local] = rows in all); pos[pair] = its row or -1; token[row] =
// the pair's token.  The order of rows inside an expert is not defined (it
// does not change any result: every row of a matmul is computed on its own).
// With w, also row_w[row] = the pair's route weight (the fused combine's
// factor).
__device__ __forceinline__ void plan_cta(const int32_t *idx, const float *w, int pairs, int top_k, int e_begin,
                                         int e_end, int32_t *offsets, int32_t *pos, int32_t *token, float *row_w) {
    extern __shared__ int32_t cnt[];  // [n_local + 1]
    const int n_local = e_end - e_begin;
    for (int i = threadIdx.x; i <= n_local; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int e = idx[p];
        pos[p] = (e >= e_begin && e < e_end) ? atomicAdd(&cnt[e - e_begin], 1) : -1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int i = 0; i < n_local; i++) {
            const int c = cnt[i];
            cnt[i] = run;
            offsets[i] = run;
            run += c;
        }
        offsets[n_local] = run;
    }
    __syncthreads();
    for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
        const int e = idx[p];
        if (e >= e_begin && e < e_end) {
            const int row = cnt[e - e_begin] + pos[p];
            pos[p] = row;
            token[row] = p / top_k;
            if (row_w) row_w[row] = w[p];
        }
    }
}

__global__ void __launch_bounds__(1024) plan_kernel(const int32_t *idx, const float *w, int pairs, int top_k,
                                                    int e_begin, int e_end, int32_t *offsets, int32_t *pos,
                                                    int32_t *token, float *row_w) {
    plan_cta(idx, w, pairs, top_k, e_begin, e_end, offsets, pos, token, row_w);
}

// route_kernel then plan_kernel in one CTA: every token routed (a thread per
// token, in turn), then the grouping; one launch instead of two.
__global__ void __launch_bounds__(1024) route_plan_kernel(const float *logits, size_t ld, int t_rows, int n_experts,
                                                          int top_k, int normalize, int32_t *idx, float *w,
                                                          int e_begin, int e_end, int32_t *offsets, int32_t *pos,
                                                          int32_t *token, float *row_w) {
    for (int t = threadIdx.x; t < t_rows; t += blockDim.x)
        route_token(logits, ld, t, n_experts, top_k, normalize, idx, w);
    __syncthreads();  // (the routes are this CTA's own global writes)
    plan_cta(idx, w, t_rows * top_k, top_k, e_begin, e_end, offsets, pos, token, row_w);
}

// xg[row] = x[token[row]], d_model floats per row.
__global__ void gather_kernel(const float *x, size_t ldx, const int32_t *token, int rows, int d_model, float *xg) {
    const int r = blockIdx.y;
    if (r >= rows) return;
    const float *src = x + (size_t)token[r] * ldx;
    float *dst = xg + (size_t)r * d_model;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d_model; i += gridDim.x * blockDim.x) dst[i] = src[i];
}

// h = silu(g) * u, element by element (h may be g).
__global__ void swiglu_kernel(const float *g, const float *u, float *h, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        h[i] = __fmul_rn(silu_ref(g[i]), u[i]);
}

// GEMM input of the grouped path, row r = blockIdx.x: x[token[r]] scaled and
// rounded to two fp16 terms (high in xh, low in xl; the gather and the dense
// prep in one pass).  With zero, block r < zero_rows also clears row r of
// zero (the output the fused combine adds into).
__global__ void __launch_bounds__(kPrepThreads) gather_prep_kernel(const float *x, size_t ldx, const int32_t *token,
                                                                    const int32_t *n_rows, int d_model, __half *xh,
                                                                    float *inv, __half *xl, float *zero, size_t ldz,
                                                                    int zero_rows) {
    const int r = blockIdx.x;
    if (zero && r < zero_rows)
        for (int i = threadIdx.x; i < d_model; i += kPrepThreads) zero[(size_t)r * ldz + i] = 0.f;
    if (r >= *n_rows) return;
    const float *src = x + (size_t)token[r] * ldx;
    prep_row([&](int i) { return src[i]; }, d_model, xh + (size_t)r * d_model, inv + r, xl + (size_t)r * d_model);
}

// GEMM input of the down matmul when the gate/up launch wrote h itself (its
// SwiGLU epilogue): row r = blockIdx.x of h, scaled and rounded to two fp16
// terms.
__global__ void __launch_bounds__(kPrepThreads) h_prep_kernel(const float *h, size_t ld, const int32_t *n_rows,
                                                               int d_ff, __half *xh, float *inv, __half *xl) {
    const int r = blockIdx.x;
    if (r >= *n_rows) return;
    const float *hr = h + (size_t)r * ld;
    prep_row([&](int i) { return hr[i]; }, d_ff, xh + (size_t)r * d_ff, inv + r, xl + (size_t)r * d_ff);
}

// out[t] = sum over route slots j (in order, from 0) of w[t][j] * y[pos[t][j]],
// slots whose expert is not local skipped (moe_combine, rce-op-moe/src/lib.rs:98-110).
__global__ void combine_kernel(const float *y, int d_model, const int32_t *pos, const float *w, int top_k,
                               float *out, size_t ldo) {
    const int t = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d_model; i += gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < top_k; j++) {
            const int r = pos[(size_t)t * top_k + j];
            if (r >= 0) acc = __fadd_rn(acc, __fmul_rn(w[(size_t)t * top_k + j], y[(size_t)r * d_model + i]));
        }
        out[(size_t)t * ldo + i] = acc;
    }
}

// sigmoid as moe_ffn_forward's shared-expert gate computes it
// (rce-qwen36-moe/src/lib.rs:465-467), each operation rounded on its own.
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.f) return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x)));
    const float e = expf(x);
    return __fdiv_rn(e, __fadd_rn(1.f, e));
}

// The shared expert's contribution, token t = blockIdx.x: g = sum_i
// gate_inp[i] * x[t][i] left to right (one thread: the reference's order),
// then out[t][i] += sigmoid(g) * sh[t][i] (moe_ffn_forward,
// rce-qwen36-moe/src/lib.rs:697-704).
__global__ void shared_combine_kernel(const float *x, size_t ldx, int d_model, const float *gate_inp,
                                      const float *sh, size_t ldsh, float *out, size_t ldo) {
    __shared__ float alpha;
    const int t = blockIdx.x;
    if (threadIdx.x == 0) {
        const float *xt = x + (size_t)t * ldx;
        float acc = 0.f;
        for (int i = 0; i < d_model; i++) acc = __fadd_rn(acc, __fmul_rn(gate_inp[i], xt[i]));
        alpha = sigmoid_ref(acc);
    }
    __syncthreads();
    const float a = alpha;
    const float *st = sh + (size_t)t * ldsh;
    float *ot = out + (size_t)t * ldo;
    for (int i = threadIdx.x; i < d_model; i += blockDim.x) ot[i] = __fadd_rn(ot[i], __fmul_rn(a, st[i]));
}

}  // namespace

cudaError_t launch_moe_shared_combine(const float *x, size_t ldx, int t_rows, int d_model, const float *gate_inp,
                                      const float *sh, size_t ldsh, float *out, size_t ldo, cudaStream_t s) {
    if (t_rows <= 0) return cudaSuccess;
    shared_combine_kernel<<<t_rows, 256, 0, s>>>(x, ldx, d_model, gate_inp, sh, ldsh, out, ldo);
    return cudaGetLastError();
}

cudaError_t launch_moe_route(const float *logits, size_t ld, int t_rows, int n_experts, int top_k, int normalize,
                             int32_t *idx, float *w, cudaStream_t s) {
    if (t_rows <= 0) return cudaSuccess;
    if (n_experts < 1 || n_experts > 256 || top_k < 1 || top_k > n_experts) return cudaErrorInvalidValue;
    route_kernel<<<(t_rows + 127) / 128, 128, 0, s>>>(logits, ld, t_rows, n_experts, top_k, normalize, idx, w);
    return cudaGetLastError();
}

cudaError_t launch_moe_plan(const int32_t *idx, const float *w, int pairs, int top_k, int e_begin, int e_end,
                            int32_t *offsets, int32_t *pos, int32_t *token, float *row_w, cudaStream_t s) {
    const int n_local = e_end - e_begin;
    if (pairs <= 0 || n_local < 1) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(n_local + 1) * sizeof(int32_t);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    plan_kernel<<<1, 1024, smem, s>>>(idx, w, pairs, top_k, e_begin, e_end, offsets, pos, token, row_w);
    return cudaGetLastError();
}

cudaError_t launch_moe_route_plan(const float *logits, size_t ld, int t_rows, int n_experts, int top_k, int normalize,
                                  int32_t *idx, float *w, int e_begin, int e_end, int32_t *offsets, int32_t *pos,
                                  int32_t *token, float *row_w, cudaStream_t s) {
    const int n_local = e_end - e_begin;
    if (t_rows <= 0 || n_local < 1) return cudaErrorInvalidValue;
    if (n_experts < 1 || n_experts > 256 || top_k < 1 || top_k > n_experts) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(n_local + 1) * sizeof(int32_t);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    route_plan_kernel<<<1, 1024, smem, s>>>(logits, ld, t_rows, n_experts, top_k, normalize, idx, w, e_begin, e_end,
                                            offsets, pos, token, row_w);
    return cudaGetLastError();
}

cudaError_t launch_moe_gather(const float *x, size_t ldx, const int32_t *token, int rows, int d_model, float *xg,
                              cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    dim3 grid((d_model + 255) / 256 < 8 ? (d_model + 255) / 256 : 8, rows);
    gather_kernel<<<grid, 256, 0, s>>>(x, ldx, token, rows, d_model, xg);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const float *g, const float *u, float *h, size_t n, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    size_t blocks = (n + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    swiglu_kernel<<<(unsigned)blocks, 256, 0, s>>>(g, u, h, n);
    return cudaGetLastError();
}

cudaError_t launch_moe_gather_prep(const float *x, size_t ldx, const int32_t *token, const int32_t *n_rows,
                                   int max_rows, int d_model, void *xh, float *inv, float *zero, size_t ldz,
                                   int zero_rows, cudaStream_t s) {
    if (max_rows <= 0) return cudaSuccess;
    if (zero && zero_rows > max_rows) return cudaErrorInvalidValue;
    __half *hi = static_cast<__half *>(xh);
    gather_prep_kernel<<<max_rows, kPrepThreads, 0, s>>>(x, ldx, token, n_rows, d_model, hi, inv,
                                                          hi + (size_t)max_rows * d_model, zero, ldz, zero_rows);
    return cudaGetLastError();
}

cudaError_t launch_moe_h_prep(const float *h, size_t ld, const int32_t *n_rows, int max_rows, int d_ff, void *xh,
                              float *inv, cudaStream_t s) {
    if (max_rows <= 0) return cudaSuccess;
    __half *hi = static_cast<__half *>(xh);
    h_prep_kernel<<<max_rows, kPrepThreads, 0, s>>>(h, ld, n_rows, d_ff, hi, inv, hi + (size_t)max_rows * d_ff);
    return cudaGetLastError();
}

cudaError_t launch_moe_combine(const float *y, int d_model, const int32_t *pos, const float *w, int t_rows, int top_k,
                               float *out, size_t ldo, cudaStream_t s) {
    if (t_rows <= 0) return cudaSuccess;
    dim3 grid((d_model + 255) / 256 < 8 ? (d_model + 255) / 256 : 8, t_rows);
    combine_kernel<<<grid, 256, 0, s>>>(y, d_model, pos, w, top_k, out, ldo);
    return cudaGetLastError();
}

}  // namespace rce
