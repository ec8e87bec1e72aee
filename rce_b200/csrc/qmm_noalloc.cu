// qmm_noalloc.cu -- rce_qmm_mm_batched_device_noalloc, rce_qmm_mm_batched_device
// for callers that cannot allocate device memory: an engine whose own
// allocator has already reserved the whole device, a serving loop that
// forbids cudaMalloc after start-up (an allocation there can stall every
// stream or fail under memory pressure), or a host that only hands us
// pointers it already owns.
//
// The regular entry point runs batches of prefill_min_tokens or more through
// the tensor-core GEMM, whose workspace (the activations rounded to fp16 and
// one inverse scale per token) it allocates per stream on first use.  Here
// that workspace is a file-scope __device__ array of kNoallocScratchBytes
// (16 MiB) instead, which every GPU that loads the library holds until the
// process exits.  Smaller batches run the decode GEMV exactly as the regular
// entry point does; it keeps its partial sums in shared memory and needs no
// workspace.  Outputs are bit-identical to rce_qmm_mm_batched_device's for
// the same context settings.
//
// Rules that follow from the one shared array:
//  - a batch whose workspace exceeds kNoallocScratchBytes (t_rows * n_cols * 2
//    bytes, twice that for the GEMM's two-term activations at up to 64
//    tokens, rounded up to 256, plus 4 bytes per token rounded up to 256) is
//    rejected with RCE_QMM_ERR_INVALID; the GEMM splits K over its CTAs
//    (weights of few rows) only when the partial sums fit the same bytes, so
//    this entry point and the regular one run every batch the same way;
//  - every call on a device uses the same array, whatever its context or
//    stream, so calls whose GEMM launches overlap on the GPU race and return
//    garbage: order them on one stream or with events;
//  - the array keeps the previous call's contents; the GEMM's prep kernel
//    writes every workspace byte it later reads (rows beyond t_rows come from
//    the tensor map's zero fill), so nothing has to be cleared;
//  - the first call on a device looks the array's device address up
//    (cudaGetSymbolAddress, which may load the module), so make that first
//    call before any stream capture;
//  - the address is cached for the life of the process: after a
//    cudaDeviceReset (which also frees every weight this library holds) the
//    entry point must not be used.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/rce_qmm.h"
#include "qmm_handles.h"
#include "qmm_internal.h"

static constexpr size_t kNoallocScratchBytes = size_t(16) << 20;

// The GEMM workspace of this entry point.  In host code this name is a
// host-side stand-in, not a device address: kernels get the address from
// scratch_address().
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_dev[kMaxDevices];  // device address of g_noalloc_scratch per device, once looked up

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

// Device address of g_noalloc_scratch on `dev` (which must be current):
// looked up on the first call per device, cached after.
cudaError_t scratch_address(int dev, void **out) {
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_dev[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        if (!p) return cudaErrorInvalidSymbol;
        g_scratch_dev[dev] = p;
    }
    *out = g_scratch_dev[dev];
    return cudaSuccess;
}

// Most tokens whose GEMM workspace fits the array at this weight's n_cols.
size_t max_gemm_tokens(int dt, const rce::Geometry &g) {
    size_t t = kNoallocScratchBytes / ((size_t)g.n_cols * 2 + 4);
    while (t > 0 && rce::gemm_workspace_bytes(dt, g, (int)t) > kNoallocScratchBytes) t--;
    while (rce::gemm_workspace_bytes(dt, g, (int)(t + 1)) <= kNoallocScratchBytes) t++;
    return t;
}

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

    // the regular entry point's routing (run_matmul), GEMM workspace aside
    if (ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens && t_rows <= (size_t)INT32_MAX) {
        const size_t need = rce::gemm_workspace_bytes(w->dtype, g, (int)t_rows);
        if (need > kNoallocScratchBytes)
            return err(RCE_QMM_ERR_INVALID,
                       "mm_batched_device_noalloc: %zu tokens x k %lld need %zu bytes of GEMM workspace, above this "
                       "entry point's fixed %zu (at most %zu tokens at this k)",
                       t_rows, (long long)g.n_cols, need, kNoallocScratchBytes, max_gemm_tokens(w->dtype, g));
        void *ws = nullptr;
        cudaError_t e = scratch_address(ctx->device, &ws);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: scratch address: %s", cudaGetErrorString(e));
        e = rce::launch_gemm(w->dtype, w->dev, g, d_a, lda, d_out, ldo, (int)t_rows, ws, ctx->err_dev, s);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: launch: %s", cudaGetErrorString(e));
        return RCE_QMM_OK;
    }
    if (w->dtype == rce::GGUF_Q6_K) {  // Q6_K's decode GEMV, passes of kQ6MaxTokens tokens
        for (size_t t0 = 0; t0 < t_rows; t0 += (size_t)rce::kQ6MaxTokens) {
            const size_t left = t_rows - t0;
            const int m = (int)(left < (size_t)rce::kQ6MaxTokens ? left : (size_t)rce::kQ6MaxTokens);
            cudaError_t e = rce::launch_gemv_q6k(w->dev, g, d_a + t0 * lda, lda, d_out + t0 * ldo, ldo, m,
                                                 ctx->sm_count, ctx->err_dev, s);
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
