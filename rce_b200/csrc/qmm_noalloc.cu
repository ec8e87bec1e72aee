// qmm_noalloc.cu -- rce_qmm_mm_batched_device_noalloc, the decode matmul for
// callers that cannot allocate device memory: a custom allocator that owns
// all of the device's memory, a serving loop that forbids cudaMalloc after
// start-up, or a host that only hands us pointers it already owns.
//
// Every batch goes through the decode GEMV, in passes of at most
// kGemvMaxTokens tokens.  The GEMV keeps its partial sums in the shared
// memory of its CTA clusters and needs no device workspace, so this entry
// point calls no cudaMalloc, cudaFree or allocating library routine (the
// regular entry point sends batches of prefill_min_tokens or more through the
// tensor-core GEMM, whose activation workspace it allocates per stream on
// first use).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/rce_qmm.h"
#include "qmm_handles.h"
#include "qmm_internal.h"

namespace {

int err(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return rce_qmm_set_error(code, buf);
}

// Makes ctx's device current for the call and restores the caller's after.
struct CurrentDevice {
    int prev = -1;
    cudaError_t status = cudaSuccess;
    explicit CurrentDevice(int dev) {
        status = cudaGetDevice(&prev);
        if (status == cudaSuccess && prev != dev) status = cudaSetDevice(dev);
    }
    ~CurrentDevice() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" int rce_qmm_mm_batched_device_noalloc(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                                 const rce_qmm_weight *w, float *d_out, size_t ldo, void *stream) {
    if (!ctx || !w || !w->dev) return err(RCE_QMM_ERR_INVALID, "mm_batched_device_noalloc: null ctx or weight");
    if (w->ctx != ctx) return err(RCE_QMM_ERR_INVALID, "mm_batched_device_noalloc: weight belongs to another context");
    if (t_rows == 0) return RCE_QMM_OK;
    if (!d_a || !d_out) return err(RCE_QMM_ERR_INVALID, "mm_batched_device_noalloc: null buffer");
    const rce::Geometry &g = w->g;
    if (lda < (size_t)g.n_cols || ldo < (size_t)g.n_rows)
        return err(RCE_QMM_ERR_INVALID, "mm_batched_device_noalloc: lda %zu < k %lld or ldo %zu < n %lld", lda,
                   (long long)g.n_cols, ldo, (long long)g.n_rows);
    CurrentDevice cd(ctx->device);
    if (cd.status != cudaSuccess)
        return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: set device: %s", cudaGetErrorString(cd.status));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (w->dtype == rce::GGUF_Q6_K) {  // Q6_K's decode GEMV: no workspace either
        for (size_t t0 = 0; t0 < t_rows; t0 += (size_t)rce::kQ6MaxTokens) {
            const size_t left = t_rows - t0;
            const int m = (int)(left < (size_t)rce::kQ6MaxTokens ? left : (size_t)rce::kQ6MaxTokens);
            cudaError_t e = rce::launch_gemv_q6k(w->dev, g, d_a + t0 * lda, lda, d_out + t0 * ldo, ldo, m,
                                                 ctx->sm_count, s);
            if (e != cudaSuccess)
                return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: launch: %s", cudaGetErrorString(e));
        }
        return RCE_QMM_OK;
    }
    for (size_t t0 = 0; t0 < t_rows;) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv(w->dtype, g, m, ctx->sm_count);
        cudaError_t e = rce::launch_gemv(w->dtype, w->dev, g, d_a + t0 * lda, lda, d_out + t0 * ldo, ldo, m, plan,
                                         ctx->err_dev, s);
        if (e == cudaErrorNotSupported)
            return err(RCE_QMM_ERR_UNSUPPORTED, "mm_batched_device_noalloc: a %lld x %lld weight does not fit the GEMV",
                       (long long)g.n_rows, (long long)g.n_cols);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: launch: %s", cudaGetErrorString(e));
        t0 += (size_t)m;
    }
    return RCE_QMM_OK;
}
