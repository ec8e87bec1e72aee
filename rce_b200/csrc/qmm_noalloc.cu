// qmm_noalloc.cu -- rce_qmm_mm_batched_device_noalloc, the decode matmul for
// callers that cannot allocate device memory: a custom allocator that owns
// all of the device's memory, a serving loop that forbids cudaMalloc after
// start-up, or a host that only hands us pointers it already owns.  When it
// splits K across CTAs, this entry point always adds the partial sums through
// a fixed array compiled into the library (the regular entry point uses
// cluster shared memory, or for the widest splits a per-stream scratch it
// allocates on first use); it calls no cudaMalloc, cudaFree or allocating
// library routine.
//
// Limits and sharing:
//  * the array holds kNoAllocPartialFloats split-K partial sums (1 MiB) and
//    kNoAllocCounters arrival counters (4 KiB); every GPU that loads the
//    library keeps them until the process exits.  A split needs
//    k_splits x min(t_rows, 4) x 16 * ceil(n_rows / 16) floats; the planner
//    splits K only while the row blocks alone leave SMs idle, so the decode
//    shapes need well under the limit, and a shape that would need more is
//    rejected with RCE_QMM_ERR_UNSUPPORTED before anything is launched;
//  * all calls on a device share the one array and it keeps the last call's
//    contents: each call clears the counters it uses before its kernels, and
//    calls whose work overlaps on the GPU (different streams, or different
//    host threads without ordering) race on it and give wrong results.
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/rce_qmm.h"
#include "qmm_handles.h"
#include "qmm_internal.h"

namespace {

constexpr size_t kNoAllocPartialFloats = size_t(1) << 18;  // 1 MiB of f32 partial sums
constexpr size_t kNoAllocCounters = 1024;                  // 4 KiB of arrival counters

// In host code these names are host-side stand-ins, not device addresses:
// only the addresses from cudaGetSymbolAddress may be passed to a kernel.
static __device__ __align__(256) float g_noalloc_partials[kNoAllocPartialFloats];
static __device__ __align__(256) unsigned g_noalloc_counters[kNoAllocCounters];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
bool g_ready[kMaxDevices];
float *g_partials[kMaxDevices];
unsigned *g_counters[kMaxDevices];

int err(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return rce_qmm_set_error(code, buf);
}

// Device addresses of the fixed arrays on `device`, which must be current.
int noalloc_addresses(int device, float **partials, unsigned **counters) {
    if (device < 0 || device >= kMaxDevices) return err(RCE_QMM_ERR_UNSUPPORTED, "noalloc: device %d", device);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ready[device]) {
        void *p = nullptr, *c = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "noalloc: cudaGetSymbolAddress(partials): %s", cudaGetErrorString(e));
        e = cudaGetSymbolAddress(&c, g_noalloc_counters);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "noalloc: cudaGetSymbolAddress(counters): %s", cudaGetErrorString(e));
        g_partials[device] = static_cast<float *>(p);
        g_counters[device] = static_cast<unsigned *>(c);
        g_ready[device] = true;
    }
    *partials = g_partials[device];
    *counters = g_counters[device];
    return RCE_QMM_OK;
}

struct CurrentDevice {
    int prev = -1;
    bool changed = false;
    cudaError_t status = cudaSuccess;
    explicit CurrentDevice(int dev) {
        status = cudaGetDevice(&prev);
        if (status == cudaSuccess && prev != dev) {
            status = cudaSetDevice(dev);
            changed = status == cudaSuccess;
        }
    }
    ~CurrentDevice() {
        if (changed) cudaSetDevice(prev);
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
    const int m_max = (int)(t_rows < (size_t)rce::kGemvMaxTokens ? t_rows : (size_t)rce::kGemvMaxTokens);
    const rce::GemvPlan worst = rce::plan_gemv_scratch(w->dtype, g, m_max, ctx->sm_count);
    if (worst.scratch_floats > 0 &&
        (worst.scratch_floats > kNoAllocPartialFloats || (size_t)worst.counters > kNoAllocCounters))
        return err(RCE_QMM_ERR_UNSUPPORTED,
                   "mm_batched_device_noalloc: a %lld x %lld weight with %d tokens per pass needs %zu split-K partial "
                   "sums and %d counters; the fixed scratch holds %zu and %zu",
                   (long long)g.n_rows, (long long)g.n_cols, m_max, worst.scratch_floats, worst.counters,
                   kNoAllocPartialFloats, kNoAllocCounters);
    float *partials = nullptr;
    unsigned *counters = nullptr;
    int rc = noalloc_addresses(ctx->device, &partials, &counters);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (worst.scratch_floats > 0) {
        cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)worst.counters * sizeof(unsigned), s);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: clear counters: %s", cudaGetErrorString(e));
    }
    for (size_t t0 = 0; t0 < t_rows;) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv_scratch(w->dtype, g, m, ctx->sm_count);
        cudaError_t e = rce::launch_gemv(w->dtype, w->dev, g, d_a + t0 * lda, lda, d_out + t0 * ldo, ldo, m, plan,
                                         plan.scratch_floats > 0 ? partials : nullptr,
                                         plan.scratch_floats > 0 ? counters : nullptr, ctx->err_dev, s);
        if (e != cudaSuccess)
            return err(RCE_QMM_ERR_CUDA, "mm_batched_device_noalloc: launch: %s", cudaGetErrorString(e));
        t0 += (size_t)m;
    }
    return RCE_QMM_OK;
}
