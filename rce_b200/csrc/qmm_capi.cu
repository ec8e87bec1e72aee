// qmm_capi.cu -- the extern "C" boundary declared in include/rce_qmm.h:
// contexts, the device weight registry, per-thread streams and staging, the
// split-K scratch pool and argument validation.  All compute is delegated to
// the kernel launchers in qmm_internal.h; there is no CPU fallback: a failed
// launch is an error returned to the caller.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>

#include "../../include/rce_qmm.h"
#include "qmm_handles.h"
#include "qmm_internal.h"

using rce::Geometry;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int ok() { return RCE_QMM_OK; }

#define CUDA_TRY(expr)                                                                         \
    do {                                                                                       \
        cudaError_t e_ = (expr);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(e_ == cudaErrorMemoryAllocation ? RCE_QMM_ERR_NOMEM : RCE_QMM_ERR_CUDA, \
                        "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

}  // namespace

int rce_qmm_set_error(int code, const char *msg) {
    g_last_error = msg;
    return code;
}

namespace {

struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && prev != dev) {
            changed = cudaSetDevice(dev) == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (changed) cudaSetDevice(prev);
    }
};

uint64_t next_serial() {
    static std::atomic<uint64_t> n{0};
    return ++n;
}

int thread_state(rce_qmm_ctx *ctx, RceThreadState **out) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    RceThreadState &ts = ctx->threads[std::this_thread::get_id()];
    if (!ts.stream) CUDA_TRY(cudaStreamCreateWithFlags(&ts.stream, cudaStreamNonBlocking));
    *out = &ts;
    return ok();
}

int grow_device(float **p, size_t *cap, size_t need_floats) {
    if (*cap >= need_floats) return ok();
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    CUDA_TRY(cudaMalloc(p, need_floats * sizeof(float)));
    *cap = need_floats;
    return ok();
}

int grow_pinned(RceThreadState *ts, size_t bytes) {
    if (ts->h_cap >= bytes) return ok();
    if (ts->h_pin) cudaFreeHost(ts->h_pin);
    ts->h_pin = nullptr;
    ts->h_cap = 0;
    CUDA_TRY(cudaMallocHost(&ts->h_pin, bytes));
    ts->h_cap = bytes;
    return ok();
}

// After the caller's stream has been synchronised: turn a kernel-reported
// error (a bounded wait that expired) into a status, and re-arm the word.
int take_kernel_error(rce_qmm_ctx *ctx) {
    const int code = *reinterpret_cast<volatile int *>(ctx->err_host);
    if (code == 0) return ok();
    *reinterpret_cast<volatile int *>(ctx->err_host) = 0;
    if (code == rce::kKernelErrOverrun)
        return fail(RCE_QMM_ERR_TIMEOUT, "a gathered output's bulk buffer held a later call's rows when it was "
                                         "unpacked (a peer ran more than one call ahead); its results are invalid");
    return fail(RCE_QMM_ERR_TIMEOUT, "a kernel's bounded wait expired (device error code %d); its results are invalid",
                code);
}

int check_weight(const rce_qmm_weight *w) {
    if (!w || !w->ctx || !w->dev) return fail(RCE_QMM_ERR_INVALID, "null or freed weight handle");
    return ok();
}

// Prefill GEMM workspace for stream s, one per stream (work on one stream is
// ordered, so its kernels never share it concurrently).  Growing it
// synchronises the stream, so the first call with the largest shape must
// come before any CUDA-graph capture on that stream.
int stream_gemm_ws(rce_qmm_ctx *ctx, cudaStream_t s, size_t bytes, void **out) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    RceScratch &sc = ctx->scratch[s];
    if (sc.gemm_ws_bytes < bytes) {
        CUDA_TRY(cudaStreamSynchronize(s));
        if (sc.gemm_ws) cudaFree(sc.gemm_ws);
        sc.gemm_ws = nullptr;
        sc.gemm_ws_bytes = 0;
        CUDA_TRY(cudaMalloc(&sc.gemm_ws, bytes));
        sc.gemm_ws_bytes = bytes;
    }
    *out = sc.gemm_ws;
    return ok();
}

// y[t_rows][ldo] = x[t_rows][lda] . W^T on stream s (device pointers).
int run_matmul(rce_qmm_ctx *ctx, const rce_qmm_weight *w, const float *d_x, size_t lda, size_t t_rows,
               float *d_y, size_t ldo, cudaStream_t s) {
    const Geometry &g = w->g;
    if (ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens && t_rows <= (size_t)INT32_MAX) {
        void *ws = nullptr;
        int rc = stream_gemm_ws(ctx, s, rce::gemm_workspace_bytes(w->dtype, g, (int)t_rows), &ws);
        if (rc) return rc;
        CUDA_TRY(rce::launch_gemm(w->dtype, w->dev, g, d_x, lda, d_y, ldo, (int)t_rows, ws, ctx->err_dev, s));
        return ok();
    }
    size_t t0 = 0;
    if (w->dtype == rce::GGUF_Q6_K) {  // its own decode GEMV, passes of kQ6MaxTokens tokens
        for (; t0 < t_rows; t0 += (size_t)rce::kQ6MaxTokens) {
            const size_t left = t_rows - t0;
            const int m = (int)(left < (size_t)rce::kQ6MaxTokens ? left : (size_t)rce::kQ6MaxTokens);
            CUDA_TRY(rce::launch_gemv_q6k(w->dev, g, d_x + t0 * lda, lda, d_y + t0 * ldo, ldo, m, ctx->sm_count,
                                          ctx->err_dev, s));
        }
        return ok();
    }
    while (t0 < t_rows) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv(w->dtype, g, m, ctx->sm_count);
        CUDA_TRY(rce::launch_gemv(w->dtype, w->dev, g, d_x + t0 * lda, lda, d_y + t0 * ldo, ldo, m, plan, ctx->err_dev,
                                  s));
        t0 += (size_t)m;
    }
    return ok();
}

// MoE FFN workspace for stream s (grown like the GEMM workspace) and its
// pinned host mirror of the per-expert row offsets.
int stream_moe_ws(rce_qmm_ctx *ctx, cudaStream_t s, size_t bytes, size_t host_n, void **ws, int32_t **host) {
    std::lock_guard<std::mutex> lk(ctx->mu);
    RceScratch &sc = ctx->scratch[s];
    if (sc.moe_ws_bytes < bytes) {
        CUDA_TRY(cudaStreamSynchronize(s));
        if (sc.moe_ws) cudaFree(sc.moe_ws);
        sc.moe_ws = nullptr;
        sc.moe_ws_bytes = 0;
        CUDA_TRY(cudaMalloc(&sc.moe_ws, bytes));
        sc.moe_ws_bytes = bytes;
    }
    if (sc.moe_host_n < host_n) {
        CUDA_TRY(cudaStreamSynchronize(s));
        if (sc.moe_host) cudaFreeHost(sc.moe_host);
        sc.moe_host = nullptr;
        sc.moe_host_n = 0;
        CUDA_TRY(cudaMallocHost(&sc.moe_host, host_n * sizeof(int32_t)));
        sc.moe_host_n = host_n;
    }
    *ws = sc.moe_ws;
    *host = sc.moe_host;
    return ok();
}

int register_common(rce_qmm_ctx *ctx, const void *src, bool src_on_device, size_t nbytes, int dtype,
                    int64_t n_rows, int64_t n_cols, cudaStream_t s, rce_qmm_weight **out) {
    if (!ctx || !src || !out) return fail(RCE_QMM_ERR_INVALID, "weight_register: null argument");
    *out = nullptr;
    if (!rce::dtype_supported(dtype))
        return fail(RCE_QMM_ERR_UNSUPPORTED,
                    "weight_register: GGUF dtype %d is not supported (Q4_0=2, Q8_0=8, Q4_K=12, Q5_K=13, Q6_K=14)",
                    dtype);
    if (n_rows <= 0 || n_cols <= 0)
        return fail(RCE_QMM_ERR_INVALID, "weight_register: shape %lld x %lld", (long long)n_rows,
                    (long long)n_cols);
    if (n_cols % rce::gguf_block(dtype) != 0)
        return fail(RCE_QMM_ERR_INVALID, "weight_register: n_cols %lld is not a multiple of the block size %d",
                    (long long)n_cols, rce::gguf_block(dtype));
    if (n_rows > (int64_t)1 << 31 || n_cols > (int64_t)1 << 31)
        return fail(RCE_QMM_ERR_UNSUPPORTED, "weight_register: dimension too large");
    Geometry g = rce::make_geometry(dtype, n_rows, n_cols);
    if (nbytes != g.gguf_bytes)
        return fail(RCE_QMM_ERR_INVALID, "weight_register: %zu bytes given, %zu expected for %lld x %lld dtype %d",
                    nbytes, g.gguf_bytes, (long long)n_rows, (long long)n_cols, dtype);
    DeviceGuard dg(ctx->device);
    uint8_t *tmp = nullptr, *dev = nullptr;
    const uint8_t *gguf_dev = static_cast<const uint8_t *>(src);
    if (!src_on_device) {
        cudaError_t e = cudaMalloc(&tmp, nbytes);
        if (e != cudaSuccess) return fail(RCE_QMM_ERR_NOMEM, "weight_register: cudaMalloc(%zu): %s", nbytes,
                                          cudaGetErrorString(e));
        e = cudaMemcpyAsync(tmp, src, nbytes, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) {
            cudaFree(tmp);
            return fail(RCE_QMM_ERR_CUDA, "weight_register: copy to device: %s", cudaGetErrorString(e));
        }
        gguf_dev = tmp;
    }
    cudaError_t e = cudaMalloc(&dev, g.dev_bytes);
    if (e != cudaSuccess) {
        if (tmp) cudaFree(tmp);
        return fail(RCE_QMM_ERR_NOMEM, "weight_register: cudaMalloc(%zu): %s", g.dev_bytes, cudaGetErrorString(e));
    }
    e = rce::launch_repack(dtype, gguf_dev, dev, g, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        cudaFree(dev);
        return fail(RCE_QMM_ERR_CUDA, "weight_register: repack: %s", cudaGetErrorString(e));
    }
    rce_qmm_weight *w = new rce_qmm_weight;
    w->ctx = ctx;
    w->serial = next_serial();
    w->dtype = dtype;
    w->g = g;
    w->dev = dev;
    w->owner = true;
    *out = w;
    return ok();
}

}  // namespace

extern "C" {

int rce_qmm_abi_version(void) { return RCE_QMM_ABI_VERSION; }

const char *rce_qmm_last_error(void) { return g_last_error.c_str(); }

size_t rce_qmm_tensor_byte_size(int dt, uint64_t n) {
    switch (dt) {
    case RCE_QMM_GGUF_Q4_0: return (size_t)((n + 31) / 32 * 18);
    case RCE_QMM_GGUF_Q8_0: return (size_t)((n + 31) / 32 * 34);
    case RCE_QMM_GGUF_Q4_K: return (size_t)((n + 255) / 256 * 144);
    case RCE_QMM_GGUF_Q5_K: return (size_t)((n + 255) / 256 * 176);
    case RCE_QMM_GGUF_Q6_K: return (size_t)((n + 255) / 256 * 210);
    default: return 0;
    }
}

int rce_qmm_ctx_create(int device, rce_qmm_ctx **out) {
    if (!out) return fail(RCE_QMM_ERR_INVALID, "ctx_create: null out");
    *out = nullptr;
    int n = 0;
    CUDA_TRY(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(RCE_QMM_ERR_INVALID, "ctx_create: device %d of %d", device, n);
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(RCE_QMM_ERR_UNSUPPORTED, "ctx_create: device %d is sm_%d%d; this library is built for sm_100a",
                    device, prop.major, prop.minor);
    DeviceGuard dg(device);
    int *err_host = nullptr, *err_dev = nullptr;
    CUDA_TRY(cudaHostAlloc(&err_host, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    *err_host = 0;
    cudaError_t e = cudaHostGetDevicePointer(&err_dev, err_host, 0);
    if (e != cudaSuccess) {
        cudaFreeHost(err_host);
        return fail(RCE_QMM_ERR_CUDA, "ctx_create: mapped error word: %s", cudaGetErrorString(e));
    }
    rce_qmm_ctx *c = new rce_qmm_ctx;
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    c->err_host = err_host;
    c->err_dev = err_dev;
    *out = c;
    return ok();
}

int rce_qmm_ctx_destroy(rce_qmm_ctx *ctx) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "ctx_destroy: null");
    DeviceGuard dg(ctx->device);
    for (auto &kv : ctx->threads) {
        RceThreadState &ts = kv.second;
        if (ts.stream) cudaStreamSynchronize(ts.stream);
        for (auto &g : ts.graphs) cudaGraphExecDestroy(g.second);
        ts.graphs.clear();
        if (ts.d_in) cudaFree(ts.d_in);
        if (ts.d_out) cudaFree(ts.d_out);
        if (ts.h_pin) cudaFreeHost(ts.h_pin);
        if (ts.stream) cudaStreamDestroy(ts.stream);
    }
    for (auto &kv : ctx->scratch) {
        if (kv.second.gemm_ws) cudaFree(kv.second.gemm_ws);
        if (kv.second.moe_ws) cudaFree(kv.second.moe_ws);
        if (kv.second.moe_host) cudaFreeHost(kv.second.moe_host);
    }
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    delete ctx;
    return ok();
}

int rce_qmm_ctx_set_prefill_min_tokens(rce_qmm_ctx *ctx, int n) {
    if (!ctx || n < 0) return fail(RCE_QMM_ERR_INVALID, "ctx_set_prefill_min_tokens: null ctx or negative count");
    ctx->prefill_min_tokens = n;
    return ok();
}

int rce_qmm_ctx_get_prefill_min_tokens(const rce_qmm_ctx *ctx, int *n) {
    if (!ctx || !n) return fail(RCE_QMM_ERR_INVALID, "ctx_get_prefill_min_tokens: null argument");
    *n = ctx->prefill_min_tokens;
    return ok();
}

int rce_qmm_ctx_sm_count(const rce_qmm_ctx *ctx, int *out) {
    if (!ctx || !out) return fail(RCE_QMM_ERR_INVALID, "ctx_sm_count: null argument");
    *out = ctx->sm_count;
    return ok();
}

int rce_qmm_weight_register(rce_qmm_ctx *ctx, const void *bytes, size_t nbytes, int dtype, int64_t n_rows,
                            int64_t n_cols, rce_qmm_weight **out) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "weight_register: null ctx");
    DeviceGuard dg(ctx->device);
    RceThreadState *ts = nullptr;
    int rc = thread_state(ctx, &ts);
    if (rc) return rc;
    return register_common(ctx, bytes, false, nbytes, dtype, n_rows, n_cols, ts->stream, out);
}

int rce_qmm_weight_register_device(rce_qmm_ctx *ctx, const void *d_bytes, size_t nbytes, int dtype,
                                   int64_t n_rows, int64_t n_cols, void *stream, rce_qmm_weight **out) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "weight_register_device: null ctx");
    DeviceGuard dg(ctx->device);
    return register_common(ctx, d_bytes, true, nbytes, dtype, n_rows, n_cols, (cudaStream_t)stream, out);
}

int rce_qmm_weight_sub_view(const rce_qmm_weight *parent, size_t byte_offset, size_t byte_len, int64_t n_rows,
                            int64_t n_cols, rce_qmm_weight **out) {
    if (!out) return fail(RCE_QMM_ERR_INVALID, "sub_view: null out");
    *out = nullptr;
    int rc = check_weight(parent);
    if (rc) return rc;
    const Geometry &pg = parent->g;
    if (n_cols != pg.n_cols)
        return fail(RCE_QMM_ERR_UNSUPPORTED, "sub_view: n_cols %lld differs from the parent's %lld",
                    (long long)n_cols, (long long)pg.n_cols);
    if (n_rows <= 0 || byte_offset % pg.gguf_row_bytes != 0)
        return fail(RCE_QMM_ERR_INVALID, "sub_view: byte offset %zu is not on a row boundary", byte_offset);
    const int64_t row0 = (int64_t)(byte_offset / pg.gguf_row_bytes);
    if (row0 % rce::TILE_ROWS != 0)
        return fail(RCE_QMM_ERR_UNSUPPORTED, "sub_view: first row %lld is not a multiple of %d", (long long)row0,
                    rce::TILE_ROWS);
    if (byte_len != (size_t)n_rows * pg.gguf_row_bytes || row0 + n_rows > pg.n_rows)
        return fail(RCE_QMM_ERR_INVALID, "sub_view: %zu+%zu bytes / %lld rows outside the parent", byte_offset,
                    byte_len, (long long)n_rows);
    rce_qmm_weight *w = new rce_qmm_weight;
    w->ctx = parent->ctx;
    w->serial = next_serial();
    w->dtype = parent->dtype;
    w->g = rce::make_geometry(parent->dtype, n_rows, n_cols);
    w->dev = parent->dev + (size_t)(row0 / rce::TILE_ROWS) * pg.n_chunks * rce::chunk_bytes(parent->dtype);
    w->owner = false;
    *out = w;
    return ok();
}

int rce_qmm_weight_free(rce_qmm_weight *w) {
    if (!w) return fail(RCE_QMM_ERR_INVALID, "weight_free: null");
    if (w->owner && w->dev) {
        DeviceGuard dg(w->ctx->device);
        cudaFree(w->dev);
    }
    w->dev = nullptr;
    delete w;
    return ok();
}

int rce_qmm_weight_info(const rce_qmm_weight *w, int *dtype, int64_t *n_rows, int64_t *n_cols, size_t *nbytes) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (dtype) *dtype = w->dtype;
    if (n_rows) *n_rows = w->g.n_rows;
    if (n_cols) *n_cols = w->g.n_cols;
    if (nbytes) *nbytes = w->g.gguf_bytes;
    return ok();
}

int rce_qmm_weight_device_storage(const rce_qmm_weight *w, const void **dev_ptr, size_t *dev_bytes) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (dev_ptr) *dev_ptr = w->dev;
    if (dev_bytes) *dev_bytes = w->g.dev_bytes;
    return ok();
}

int rce_qmm_weight_read_bytes(const rce_qmm_weight *w, void *host_out, size_t nbytes) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (!host_out || nbytes != w->g.gguf_bytes)
        return fail(RCE_QMM_ERR_INVALID, "weight_read_bytes: need a buffer of %zu bytes", w->g.gguf_bytes);
    DeviceGuard dg(w->ctx->device);
    RceThreadState *ts = nullptr;
    rc = thread_state(w->ctx, &ts);
    if (rc) return rc;
    uint8_t *tmp = nullptr;
    CUDA_TRY(cudaMalloc(&tmp, nbytes));
    cudaError_t e = rce::launch_unpack(w->dtype, w->dev, tmp, w->g, 0, w->g.n_rows, ts->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(host_out, tmp, nbytes, cudaMemcpyDeviceToHost, ts->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ts->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail(RCE_QMM_ERR_CUDA, "weight_read_bytes: %s", cudaGetErrorString(e));
    return ok();
}

int rce_qmm_mm_batched_device(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                              const rce_qmm_weight *w, float *d_out, size_t ldo, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device: null ctx");
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device: weight belongs to another context");
    if (t_rows == 0) return ok();
    if (!d_a || !d_out) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device: null buffer");
    if (lda < (size_t)w->g.n_cols || ldo < (size_t)w->g.n_rows)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device: lda %zu < k %lld or ldo %zu < n %lld", lda,
                    (long long)w->g.n_cols, ldo, (long long)w->g.n_rows);
    DeviceGuard dg(ctx->device);
    return run_matmul(ctx, w, d_a, lda, t_rows, d_out, ldo, (cudaStream_t)stream);
}

int rce_qmm_mm_batched_device_multi(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                    const rce_qmm_weight *const *ws, size_t n_w, float *const *d_outs,
                                    const size_t *ldos, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: null ctx");
    if (!ws || !d_outs || !ldos || n_w < 1 || n_w > (size_t)rce::kGemvMaxGroup)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: need 1..%d weights, outputs and strides",
                    rce::kGemvMaxGroup);
    for (size_t i = 0; i < n_w; i++) {
        int rc = check_weight(ws[i]);
        if (rc) return rc;
        if (ws[i]->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: weight %zu belongs to another context", i);
        if (ws[i]->dtype != ws[0]->dtype || ws[i]->g.n_cols != ws[0]->g.n_cols)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: weight %zu differs from weight 0 in dtype or k", i);
        if (!d_outs[i] || ldos[i] < (size_t)ws[i]->g.n_rows)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: output %zu null or ldo %zu < n %lld", i, ldos[i],
                        (long long)ws[i]->g.n_rows);
    }
    if (t_rows == 0) return ok();
    if (!d_a || lda < (size_t)ws[0]->g.n_cols)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi: null activations or lda %zu < k %lld", lda,
                    (long long)ws[0]->g.n_cols);
    DeviceGuard dg(ctx->device);
    cudaStream_t s = (cudaStream_t)stream;
    if ((ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens) ||
        ws[0]->dtype == rce::GGUF_Q6_K) {
        // the tensor-core GEMM (or Q6_K's own GEMV), one weight at a time
        for (size_t i = 0; i < n_w; i++) {
            int rc = run_matmul(ctx, ws[i], d_a, lda, t_rows, d_outs[i], ldos[i], s);
            if (rc) return rc;
        }
        return ok();
    }
    rce::GemvGroup grp;
    grp.n = (int)n_w;
    for (size_t i = 0; i < n_w; i++) {
        grp.w[i] = ws[i]->dev;
        grp.g[i] = ws[i]->g;
        grp.ldy[i] = ldos[i];
    }
    const rce::Geometry gg = rce::group_geometry(grp);
    for (size_t t0 = 0; t0 < t_rows;) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv(ws[0]->dtype, gg, m, ctx->sm_count);
        for (size_t i = 0; i < n_w; i++) grp.y[i] = d_outs[i] + t0 * ldos[i];
        CUDA_TRY(rce::launch_gemv_group(ws[0]->dtype, grp, d_a + t0 * lda, lda, m, plan, ctx->err_dev, s));
        t0 += (size_t)m;
    }
    return ok();
}

constexpr size_t kMaxHostGraphs = 1024;  // per thread; all are dropped when full

void clear_graphs(RceThreadState *ts) {
    for (auto &kv : ts->graphs) cudaGraphExecDestroy(kv.second);
    ts->graphs.clear();
}

// Copies a host call's activations from the pinned staging buffer (mapped
// into the device's address space) to the device buffer.  It releases its
// dependent grid at once, so the matmul launched after it (programmatic
// stream serialisation) starts streaming its weights while the activations
// cross the bus; the matmul reads them only after its grid-dependency wait.
__global__ void __launch_bounds__(256) stage_in_kernel(const float *src, float *dst, size_t n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        const size_t n4 = n / 4;
        for (size_t j = i; j < n4; j += stride)
            reinterpret_cast<float4 *>(dst)[j] = reinterpret_cast<const float4 *>(src)[j];
        for (size_t j = 4 * n4 + i; j < n; j += stride) dst[j] = src[j];
    } else {
        for (; i < n; i += stride) dst[i] = src[i];
    }
}

// Records rce_qmm_mm_batched's device steps for w and t_rows on the thread's
// staging buffers (activations in by stage_in_kernel, matmul into the pinned
// buffer) as an executable graph.
int record_host_call(rce_qmm_ctx *ctx, RceThreadState *ts, const rce_qmm_weight *w, size_t t_rows,
                     cudaGraphExec_t *exec) {
    *exec = nullptr;
    const size_t k = (size_t)w->g.n_cols, n = (size_t)w->g.n_rows;
    cudaGraph_t graph = nullptr;
    CUDA_TRY(cudaStreamBeginCapture(ts->stream, cudaStreamCaptureModeThreadLocal));
    // the activations in by a kernel (not a copy node), so that the matmul's
    // weight stream overlaps their transfer
    const size_t in_f = t_rows * k;
    unsigned blocks = (unsigned)((in_f / 4 + 255) / 256);
    blocks = blocks < 1 ? 1 : (blocks > 8 ? 8 : blocks);
    stage_in_kernel<<<blocks, 256, 0, ts->stream>>>(static_cast<const float *>(ts->h_pin), ts->d_in, in_f);
    cudaError_t e = cudaGetLastError();
    // the matmul writes its (small, decode-sized) output straight into the
    // pinned staging buffer (mapped into the device's address space): no
    // device-to-host copy after it
    int rc = e == cudaSuccess ? run_matmul(ctx, w, ts->d_in, k, t_rows, static_cast<float *>(ts->h_pin), n, ts->stream)
                              : 0;
    const cudaError_t ee = cudaStreamEndCapture(ts->stream, &graph);
    if (e == cudaSuccess) e = ee;
    if (e == cudaSuccess && rc == 0) e = cudaGraphInstantiate(exec, graph, 0);
    if (graph) cudaGraphDestroy(graph);
    if (e != cudaSuccess || rc != 0) {
        *exec = nullptr;
        cudaGetLastError();  // (the direct path runs instead)
        return 1;
    }
    return 0;
}

int rce_qmm_mm_batched(rce_qmm_ctx *ctx, const float *a, size_t t_rows, const rce_qmm_weight *w, float *out,
                       size_t out_len) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched: null ctx");
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched: weight belongs to another context");
    if (t_rows == 0) return ok();
    if (!a || !out) return fail(RCE_QMM_ERR_INVALID, "mm_batched: null buffer");
    const size_t k = (size_t)w->g.n_cols, n = (size_t)w->g.n_rows;
    if (out_len < t_rows * n)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched: output holds %zu values, %zu needed", out_len, t_rows * n);
    DeviceGuard dg(ctx->device);
    RceThreadState *ts = nullptr;
    rc = thread_state(ctx, &ts);
    if (rc) return rc;
    const size_t in_f = t_rows * k, out_f = t_rows * n;
    const void *bufs[3] = {ts->d_in, ts->d_out, ts->h_pin};
    if ((rc = grow_device(&ts->d_in, &ts->d_in_cap, in_f))) return rc;
    if ((rc = grow_device(&ts->d_out, &ts->d_out_cap, out_f))) return rc;
    if ((rc = grow_pinned(ts, (in_f > out_f ? in_f : out_f) * sizeof(float)))) return rc;
    if (bufs[0] != ts->d_in || bufs[1] != ts->d_out || bufs[2] != ts->h_pin) clear_graphs(ts);
    std::memcpy(ts->h_pin, a, in_f * sizeof(float));
    // the decode route (no workspace: the graph stays valid) replays a cached
    // graph of the three steps; the first call of a (weight, batch) records it
    const bool decode = ctx->prefill_min_tokens == 0 || t_rows < (size_t)ctx->prefill_min_tokens;
    cudaGraphExec_t exec = nullptr;
    if (decode && t_rows < 256) {
        const uint64_t key = (w->serial << 8) | (uint64_t)t_rows;
        auto it = ts->graphs.find(key);
        if (it != ts->graphs.end()) {
            exec = it->second;
        } else if (record_host_call(ctx, ts, w, t_rows, &exec) == 0 && exec) {
            if (ts->graphs.size() >= kMaxHostGraphs) clear_graphs(ts);
            ts->graphs[key] = exec;
        }
    }
    if (exec) {
        CUDA_TRY(cudaGraphLaunch(exec, ts->stream));
    } else {
        CUDA_TRY(cudaMemcpyAsync(ts->d_in, ts->h_pin, in_f * sizeof(float), cudaMemcpyHostToDevice, ts->stream));
        rc = run_matmul(ctx, w, ts->d_in, k, t_rows, ts->d_out, n, ts->stream);
        if (rc) return rc;
        CUDA_TRY(cudaMemcpyAsync(ts->h_pin, ts->d_out, out_f * sizeof(float), cudaMemcpyDeviceToHost, ts->stream));
    }
    CUDA_TRY(cudaStreamSynchronize(ts->stream));
    if ((rc = take_kernel_error(ctx))) return rc;
    std::memcpy(out, ts->h_pin, out_f * sizeof(float));
    return ok();
}

int rce_qmm_mm_1d(rce_qmm_ctx *ctx, const float *a, size_t a_len, const rce_qmm_weight *w, float *out,
                  size_t out_len) {
    int rc = check_weight(w);
    if (rc) return rc;
    if (a_len != (size_t)w->g.n_cols)
        return fail(RCE_QMM_ERR_INVALID, "mm_1d: activation len %zu != k %lld", a_len, (long long)w->g.n_cols);
    return rce_qmm_mm_batched(ctx, a, 1, w, out, out_len);
}

int rce_qmm_mm_1d_serial(rce_qmm_ctx *ctx, const float *a, size_t a_len, const rce_qmm_weight *w, float *out,
                         size_t out_len) {
    return rce_qmm_mm_1d(ctx, a, a_len, w, out, out_len);
}

int rce_qmm_dequant_device(rce_qmm_ctx *ctx, const rce_qmm_weight *w, int64_t row0, int64_t row1, float *d_out,
                           size_t ldo, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "dequant_device: null ctx");
    int rc = check_weight(w);
    if (rc) return rc;
    if (row0 < 0 || row1 > w->g.n_rows || row0 > row1)
        return fail(RCE_QMM_ERR_INVALID, "dequant_device: rows [%lld, %lld) outside [0, %lld)", (long long)row0,
                    (long long)row1, (long long)w->g.n_rows);
    if (!d_out || ldo < (size_t)w->g.n_cols) return fail(RCE_QMM_ERR_INVALID, "dequant_device: bad output");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(rce::launch_dequant(w->dtype, w->dev, d_out, ldo, w->g, row0, row1, (cudaStream_t)stream));
    return ok();
}

int rce_qmm_dequant_row(rce_qmm_ctx *ctx, const rce_qmm_weight *w, int64_t row, float *out, size_t out_len) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "dequant_row: null ctx");
    int rc = check_weight(w);
    if (rc) return rc;
    if (row < 0 || row >= w->g.n_rows)
        return fail(RCE_QMM_ERR_INVALID, "dequant_row: row %lld >= n_rows %lld", (long long)row,
                    (long long)w->g.n_rows);
    const size_t k = (size_t)w->g.n_cols;
    if (!out || out_len < k) return fail(RCE_QMM_ERR_INVALID, "dequant_row: output holds %zu < %zu", out_len, k);
    DeviceGuard dg(ctx->device);
    RceThreadState *ts = nullptr;
    rc = thread_state(ctx, &ts);
    if (rc) return rc;
    if ((rc = grow_device(&ts->d_out, &ts->d_out_cap, k))) return rc;
    if ((rc = grow_pinned(ts, k * sizeof(float)))) return rc;
    CUDA_TRY(rce::launch_dequant(w->dtype, w->dev, ts->d_out, k, w->g, row, row + 1, ts->stream));
    CUDA_TRY(cudaMemcpyAsync(ts->h_pin, ts->d_out, k * sizeof(float), cudaMemcpyDeviceToHost, ts->stream));
    CUDA_TRY(cudaStreamSynchronize(ts->stream));
    std::memcpy(out, ts->h_pin, k * sizeof(float));
    return ok();
}

int rce_qmm_device_error(rce_qmm_ctx *ctx, int *code, int clear) {
    if (!ctx || !code) return fail(RCE_QMM_ERR_INVALID, "device_error: null argument");
    *code = *reinterpret_cast<volatile int *>(ctx->err_host);
    if (clear) *reinterpret_cast<volatile int *>(ctx->err_host) = 0;
    return ok();
}

int rce_qmm_synchronize(rce_qmm_ctx *ctx) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "synchronize: null ctx");
    DeviceGuard dg(ctx->device);
    RceThreadState *ts = nullptr;
    int rc = thread_state(ctx, &ts);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(ts->stream));
    return ok();
}

int rce_qmm_peer_alloc(rce_qmm_ctx *ctx, size_t bytes, void **d_ptr, void *ipc_handle) {
    if (!ctx || !d_ptr || !ipc_handle || bytes == 0) return fail(RCE_QMM_ERR_INVALID, "peer_alloc: bad arguments");
    DeviceGuard dg(ctx->device);
    void *p = nullptr;
    CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(RCE_QMM_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *d_ptr = p;
    return ok();
}

int rce_qmm_peer_free(rce_qmm_ctx *ctx, void *d_ptr) {
    if (!ctx || !d_ptr) return fail(RCE_QMM_ERR_INVALID, "peer_free: null");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(cudaFree(d_ptr));
    return ok();
}

int rce_qmm_peer_open(rce_qmm_ctx *ctx, const void *ipc_handle, void **d_ptr) {
    if (!ctx || !ipc_handle || !d_ptr) return fail(RCE_QMM_ERR_INVALID, "peer_open: null");
    DeviceGuard dg(ctx->device);
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return ok();
}

int rce_qmm_peer_close(rce_qmm_ctx *ctx, void *d_ptr) {
    if (!ctx || !d_ptr) return fail(RCE_QMM_ERR_INVALID, "peer_close: null");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(cudaIpcCloseMemHandle(d_ptr));
    return ok();
}

int rce_qmm_mm_batched_device_gather(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                     const rce_qmm_weight *w, int world, int rank, int64_t row_offset,
                                     float *d_y, size_t ldy, unsigned long long *const *d_ll, unsigned epoch,
                                     const unsigned *d_epoch_base, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: null ctx");
    int rc = check_weight(w);
    if (rc) return rc;
    if (w->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: weight of another context");
    if (world < 2 || world > rce::kMaxPeers || rank < 0 || rank >= world)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: world %d (2..%d), rank %d", world,
                    rce::kMaxPeers, rank);
    if (t_rows == 0) return ok();
    if (!d_a || !d_y || !d_ll || row_offset < 0 || lda < (size_t)w->g.n_cols ||
        ldy < (size_t)(row_offset + w->g.n_rows))
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: null buffer, lda < k or ldy < row_offset + n");
    for (int r = 0; r < world; r++)
        if (r != rank && !d_ll[r]) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: null d_ll[%d]", r);
    if (epoch == 0 && !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_gather: epoch 0");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rce::GatherArgs ga;
    ga.world = world;
    ga.rank = rank;
    ga.row_off = row_offset;
    for (int r = 0; r < world; r++) ga.ll[r] = d_ll[r];
    ga.epoch = epoch;
    ga.epoch_base = d_epoch_base;
    const Geometry &g = w->g;
    float *y_own = d_y + row_offset;
    if ((ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens && t_rows <= (size_t)INT32_MAX) ||
        w->dtype == rce::GGUF_Q6_K) {
        rc = run_matmul(ctx, w, d_a, lda, t_rows, y_own, ldy, s);
        if (rc) return rc;
        CUDA_TRY(rce::launch_gather_push(ga, d_y, (int)t_rows, g.n_rows, ldy, s));
        return ok();
    }
    for (size_t t0 = 0; t0 < t_rows;) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv(w->dtype, g, m, ctx->sm_count);
        rce::GatherArgs gp = ga;
        for (int r = 0; r < world; r++) gp.ll[r] = d_ll[r] ? d_ll[r] + t0 * ldy : nullptr;
        CUDA_TRY(rce::launch_gemv(w->dtype, w->dev, g, d_a + t0 * lda, lda, y_own + t0 * ldy, ldy, m, plan, ctx->err_dev,
                                  s, &gp));
        t0 += (size_t)m;
    }
    return ok();
}

int rce_qmm_mm_batched_device_multi_gather(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                           const rce_qmm_weight *const *ws, size_t n_w, int world, int rank,
                                           const int64_t *row_offsets, float *const *d_ys, const size_t *ldys,
                                           unsigned long long *const *d_lls, unsigned epoch,
                                           const unsigned *d_epoch_base, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: null ctx");
    if (!ws || !row_offsets || !d_ys || !ldys || !d_lls || n_w < 1 || n_w > (size_t)rce::kGemvMaxGroup)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: need 1..%d weights with offsets, outputs, "
                    "strides and receive buffers", rce::kGemvMaxGroup);
    if (world < 2 || world > rce::kMaxPeers || rank < 0 || rank >= world)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: world %d (2..%d), rank %d", world,
                    rce::kMaxPeers, rank);
    if (epoch == 0 && !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: epoch 0");
    for (size_t i = 0; i < n_w; i++) {
        int rc = check_weight(ws[i]);
        if (rc) return rc;
        if (ws[i]->ctx != ctx)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: weight %zu of another context", i);
        if (ws[i]->dtype != ws[0]->dtype || ws[i]->g.n_cols != ws[0]->g.n_cols)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: weight %zu differs in dtype or k", i);
        if (!d_ys[i] || row_offsets[i] < 0 || ldys[i] < (size_t)(row_offsets[i] + ws[i]->g.n_rows))
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: output %zu null or ldy < row_offset + n", i);
        for (int r = 0; r < world; r++)
            if (r != rank && !d_lls[i * world + r])
                return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: null receive buffer %zu/%d", i, r);
    }
    if (t_rows == 0) return ok();
    if (!d_a || lda < (size_t)ws[0]->g.n_cols)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather: null activations or lda < k");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rce::GatherArgs ga[rce::kGemvMaxGroup];
    for (size_t i = 0; i < n_w; i++) {
        ga[i].world = world;
        ga[i].rank = rank;
        ga[i].row_off = row_offsets[i];
        for (int r = 0; r < world; r++) ga[i].ll[r] = d_lls[i * world + r];
        ga[i].epoch = epoch;
        ga[i].epoch_base = d_epoch_base;
    }
    if ((ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens && t_rows <= (size_t)INT32_MAX) ||
        ws[0]->dtype == rce::GGUF_Q6_K) {
        // the tensor-core GEMM (or Q6_K's GEMV) per weight, each output pushed
        // to the peers after it
        for (size_t i = 0; i < n_w; i++) {
            int rc = run_matmul(ctx, ws[i], d_a, lda, t_rows, d_ys[i] + row_offsets[i], ldys[i], s);
            if (rc) return rc;
            CUDA_TRY(rce::launch_gather_push(ga[i], d_ys[i], (int)t_rows, ws[i]->g.n_rows, ldys[i], s));
        }
        return ok();
    }
    rce::GemvGroup grp;
    grp.n = (int)n_w;
    for (size_t i = 0; i < n_w; i++) {
        grp.w[i] = ws[i]->dev;
        grp.g[i] = ws[i]->g;
        grp.ldy[i] = ldys[i];
    }
    const rce::Geometry gg = rce::group_geometry(grp);
    for (size_t t0 = 0; t0 < t_rows;) {
        const size_t left = t_rows - t0;
        const int m = (int)(left < (size_t)rce::kGemvMaxTokens ? left : (size_t)rce::kGemvMaxTokens);
        const rce::GemvPlan plan = rce::plan_gemv(ws[0]->dtype, gg, m, ctx->sm_count);
        rce::GatherArgs gp[rce::kGemvMaxGroup];
        for (size_t i = 0; i < n_w; i++) {
            grp.y[i] = d_ys[i] + row_offsets[i] + t0 * ldys[i];
            gp[i] = ga[i];
            for (int r = 0; r < world; r++) gp[i].ll[r] = ga[i].ll[r] ? ga[i].ll[r] + t0 * ldys[i] : nullptr;
        }
        CUDA_TRY(rce::launch_gemv_group(ws[0]->dtype, grp, d_a + t0 * lda, lda, m, plan, ctx->err_dev, s, gp));
        t0 += (size_t)m;
    }
    return ok();
}

int rce_qmm_mm_batched_device_multi_gather_bulk(rce_qmm_ctx *ctx, const float *d_a, size_t lda, size_t t_rows,
                                                const rce_qmm_weight *const *ws, size_t n_w, int world, int rank,
                                                const int64_t *row_offsets, float *const *d_ys, const size_t *ldys,
                                                float *const *d_bulks, const size_t *flag_offsets, unsigned epoch,
                                                const unsigned *d_epoch_base, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: null ctx");
    if (!ws || !row_offsets || !d_ys || !ldys || !d_bulks || !flag_offsets || n_w < 1 ||
        n_w > (size_t)rce::kGemvMaxGroup)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: need 1..%d weights with offsets, "
                    "outputs, strides, bulk buffers and flag offsets", rce::kGemvMaxGroup);
    if (world < 2 || world > rce::kMaxPeers || rank < 0 || rank >= world)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: world %d (2..%d), rank %d", world,
                    rce::kMaxPeers, rank);
    if (epoch == 0 && !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: epoch 0");
    if (t_rows > 65535) return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: t_rows > 65535");
    for (size_t i = 0; i < n_w; i++) {
        int rc = check_weight(ws[i]);
        if (rc) return rc;
        if (ws[i]->ctx != ctx)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: weight %zu of another context", i);
        if (ws[i]->g.n_cols != ws[0]->g.n_cols)
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: weight %zu differs in k", i);
        if (!d_ys[i] || row_offsets[i] < 0 || ldys[i] < (size_t)(row_offsets[i] + ws[i]->g.n_rows) ||
            flag_offsets[i] % 4 || flag_offsets[i] < t_rows * ldys[i] * sizeof(float))
            return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: output %zu null, ldy < row_offset "
                        "+ n, or flags inside the values", i);
        for (int r = 0; r < world; r++)
            if (r != rank && !d_bulks[i * world + r])
                return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: null bulk buffer %zu/%d", i, r);
    }
    if (t_rows == 0) return ok();
    if (!d_a || lda < (size_t)ws[0]->g.n_cols)
        return fail(RCE_QMM_ERR_INVALID, "mm_batched_device_multi_gather_bulk: null activations or lda < k");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (size_t i = 0; i < n_w; i++) {
        const bool gemm = ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens;
        if (gemm) {
            // the GEMM (or its split-K reduce) stores every value into the
            // peers' bulk buffers itself; then the flags
            rce::BulkPush push;
            push.world = world;
            push.rank = rank;
            for (int r = 0; r < world; r++)
                push.peer[r] = r == rank ? nullptr : d_bulks[i * world + r] + row_offsets[i];
            void *wsp = nullptr;
            int rc = stream_gemm_ws(ctx, s, rce::gemm_workspace_bytes(ws[i]->dtype, ws[i]->g, (int)t_rows), &wsp);
            if (rc) return rc;
            CUDA_TRY(rce::launch_gemm(ws[i]->dtype, ws[i]->dev, ws[i]->g, d_a, lda, d_ys[i] + row_offsets[i], ldys[i],
                                      (int)t_rows, wsp, ctx->err_dev, s, &push));
            CUDA_TRY(rce::launch_gather_flags_bulk(world, rank, d_bulks + i * world, flag_offsets[i], epoch,
                                                   d_epoch_base, s));
            continue;
        }
        int rc = run_matmul(ctx, ws[i], d_a, lda, t_rows, d_ys[i] + row_offsets[i], ldys[i], s);
        if (rc) return rc;
        CUDA_TRY(rce::launch_gather_push_bulk(world, rank, d_bulks + i * world, flag_offsets[i], d_ys[i], (int)t_rows,
                                              row_offsets[i], ws[i]->g.n_rows, ldys[i], epoch, d_epoch_base, s));
    }
    return ok();
}

int rce_qmm_peer_unpack_bulk(rce_qmm_ctx *ctx, const float *d_bulk, size_t flag_offset, float *d_y, size_t ldy,
                             size_t t_rows, int64_t n, int64_t own0, int64_t own1, int world, int rank, unsigned epoch,
                             const unsigned *d_epoch_base, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "peer_unpack_bulk: null ctx");
    if (t_rows == 0) return ok();
    if (!d_bulk || !d_y || n <= 0 || (size_t)n > ldy || own0 < 0 || own0 > own1 || own1 > n || t_rows > 65535 ||
        flag_offset % 4 || flag_offset < t_rows * ldy * sizeof(float))
        return fail(RCE_QMM_ERR_INVALID, "peer_unpack_bulk: bad buffers or ranges");
    if (world < 2 || world > rce::kMaxPeers || rank < 0 || rank >= world)
        return fail(RCE_QMM_ERR_INVALID, "peer_unpack_bulk: world %d, rank %d", world, rank);
    if (epoch == 0 && !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "peer_unpack_bulk: epoch 0");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(rce::launch_gather_unpack_bulk(d_bulk, flag_offset, d_y, (int)t_rows, n, ldy, own0, own1, world, rank,
                                            epoch, d_epoch_base, ctx->err_dev, static_cast<cudaStream_t>(stream)));
    return ok();
}

int rce_qmm_peer_unpack(rce_qmm_ctx *ctx, const unsigned long long *d_ll, float *d_y, size_t ldy, size_t t_rows,
                        int64_t n, int64_t own0, int64_t own1, unsigned epoch, const unsigned *d_epoch_base,
                        void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "peer_unpack: null ctx");
    if (t_rows == 0) return ok();
    if (!d_ll || !d_y || n <= 0 || (size_t)n > ldy || own0 < 0 || own0 > own1 || own1 > n || t_rows > (size_t)INT32_MAX)
        return fail(RCE_QMM_ERR_INVALID, "peer_unpack: bad buffers or ranges");
    if (epoch == 0 && !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "peer_unpack: epoch 0");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(rce::launch_gather_unpack(d_ll, d_y, (int)t_rows, n, ldy, own0, own1, epoch, d_epoch_base, ctx->err_dev,
                                       static_cast<cudaStream_t>(stream)));
    return ok();
}

int rce_qmm_peer_epoch_advance(rce_qmm_ctx *ctx, unsigned *d_epoch_base, unsigned delta, void *stream) {
    if (!ctx || !d_epoch_base) return fail(RCE_QMM_ERR_INVALID, "peer_epoch_advance: null");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(rce::launch_epoch_advance(d_epoch_base, delta, static_cast<cudaStream_t>(stream)));
    return ok();
}

int rce_qmm_moe_route_device(rce_qmm_ctx *ctx, const float *d_logits, size_t ld_logits, size_t t_rows,
                             int n_experts, int top_k, int normalize, int32_t *d_idx, float *d_w, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "moe_route_device: null ctx");
    if (n_experts < 1 || n_experts > 256 || top_k < 1 || top_k > n_experts)
        return fail(RCE_QMM_ERR_INVALID, "moe_route_device: n_experts %d (1..256), top_k %d (1..n_experts)",
                    n_experts, top_k);
    if (t_rows == 0) return ok();
    if (!d_logits || !d_idx || !d_w || ld_logits < (size_t)n_experts || t_rows > (size_t)INT32_MAX)
        return fail(RCE_QMM_ERR_INVALID, "moe_route_device: null buffer, ld_logits < n_experts or too many rows");
    DeviceGuard dg(ctx->device);
    CUDA_TRY(rce::launch_moe_route(d_logits, ld_logits, (int)t_rows, n_experts, top_k, normalize, d_idx, d_w,
                                   (cudaStream_t)stream));
    return ok();
}

int rce_qmm_moe_router_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                              const rce_qmm_weight *router_w, int top_k, int normalize, float *d_logits,
                              size_t ld_logits, int32_t *d_idx, float *d_w, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "moe_router_device: null ctx");
    int rc = check_weight(router_w);
    if (rc) return rc;
    if (router_w->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "moe_router_device: weight of another context");
    const int64_t n_experts = router_w->g.n_rows;
    if (n_experts < 1 || n_experts > 256 || top_k < 1 || top_k > n_experts)
        return fail(RCE_QMM_ERR_INVALID, "moe_router_device: n_experts %lld (1..256), top_k %d (1..n_experts)",
                    (long long)n_experts, top_k);
    if (t_rows == 0) return ok();
    if (!d_x || !d_logits || !d_idx || !d_w || ldx < (size_t)router_w->g.n_cols || ld_logits < (size_t)n_experts ||
        t_rows > (size_t)INT32_MAX)
        return fail(RCE_QMM_ERR_INVALID, "moe_router_device: null buffer, ldx < d_model, ld_logits < n_experts or "
                                         "too many rows");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = run_matmul(ctx, router_w, d_x, ldx, t_rows, d_logits, ld_logits, s);
    if (rc) return rc;
    CUDA_TRY(rce::launch_moe_route(d_logits, ld_logits, (int)t_rows, (int)n_experts, top_k, normalize, d_idx, d_w, s));
    return ok();
}

int rce_qmm_moe_ffn_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                           const float *d_logits, size_t ld_logits, int n_experts, int top_k,
                           int expert_begin, int expert_end, const rce_qmm_weight *const *gate,
                           const rce_qmm_weight *const *up, const rce_qmm_weight *const *down, float *d_out,
                           size_t ldo, int32_t *d_idx, float *d_w, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: null ctx");
    if (n_experts < 1 || n_experts > 256 || top_k < 1 || top_k > n_experts)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: n_experts %d (1..256), top_k %d (1..n_experts)",
                    n_experts, top_k);
    if (expert_begin < 0 || expert_end > n_experts || expert_begin >= expert_end)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: expert range [%d, %d) of %d", expert_begin, expert_end,
                    n_experts);
    if (!gate || !up || !down) return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: null weight array");
    // shapes: every local expert's gate/up are [d_ff x d_model], down [d_model x d_ff]
    const rce_qmm_weight *g0 = gate[expert_begin];
    int rc = check_weight(g0);
    if (rc) return rc;
    const int64_t d_model = g0->g.n_cols, d_ff = g0->g.n_rows;
    for (int e = expert_begin; e < expert_end; e++) {
        const rce_qmm_weight *ws[3] = {gate[e], up[e], down[e]};
        for (int q = 0; q < 3; q++) {
            rc = check_weight(ws[q]);
            if (rc) return rc;
            if (ws[q]->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: weight of another context");
        }
        if (gate[e]->g.n_rows != d_ff || gate[e]->g.n_cols != d_model || up[e]->g.n_rows != d_ff ||
            up[e]->g.n_cols != d_model || down[e]->g.n_rows != d_model || down[e]->g.n_cols != d_ff)
            return fail(RCE_QMM_ERR_INVALID,
                        "moe_ffn_device: expert %d: gate/up must be [%lld x %lld] and down [%lld x %lld]", e,
                        (long long)d_ff, (long long)d_model, (long long)d_model, (long long)d_ff);
    }
    if (t_rows == 0) return ok();
    if (!d_x || !d_logits || !d_out) return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: null buffer");
    if (ldx < (size_t)d_model || ldo < (size_t)d_model || ld_logits < (size_t)n_experts)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: ldx %zu / ldo %zu < d_model %lld or ld_logits %zu < %d",
                    ldx, ldo, (long long)d_model, ld_logits, n_experts);
    if (t_rows * (size_t)top_k > (size_t)INT32_MAX / 2)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn_device: too many tokens");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int n_local = expert_end - expert_begin;
    const size_t P = t_rows * (size_t)top_k;
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    size_t o = 0;
    const size_t o_idx = o;
    o += al(P * 4);
    const size_t o_w = o;
    o += al(P * 4);
    const size_t o_pos = o;
    o += al(P * 4);
    const size_t o_tok = o;
    o += al(P * 4);
    const size_t o_off = o;
    o += al((size_t)(n_local + 1) * 4);
    const size_t o_rw = o;  // route weight of each grouped row (the fused combine's factor)
    o += al(P * 4);
    const size_t o_xg = o;
    o += al(P * (size_t)d_model * 4);
    const size_t o_g = o;
    o += al(P * (size_t)d_ff * 4);
    const size_t o_u = o;
    o += al(P * (size_t)d_ff * 4);
    const size_t o_y = o;
    o += al(P * (size_t)d_model * 4);
    // grouped path: the gate/up input's two fp16 terms reuse xg's bytes; the
    // SwiGLU outputs' two fp16 terms; both inputs' row scales
    const size_t o_xh2 = o;
    o += al(2 * P * (size_t)d_ff * 2);
    const size_t o_inv = o;
    o += al(P * 4);
    const size_t o_inv2 = o;
    o += al(P * 4);
    void *wsv = nullptr;
    int32_t *host_off = nullptr;
    rc = stream_moe_ws(ctx, s, o, (size_t)n_local + 1, &wsv, &host_off);
    if (rc) return rc;
    uint8_t *ws = static_cast<uint8_t *>(wsv);
    int32_t *idx = d_idx ? d_idx : reinterpret_cast<int32_t *>(ws + o_idx);
    float *wt = d_w ? d_w : reinterpret_cast<float *>(ws + o_w);
    int32_t *pos = reinterpret_cast<int32_t *>(ws + o_pos);
    int32_t *tok = reinterpret_cast<int32_t *>(ws + o_tok);
    int32_t *off = reinterpret_cast<int32_t *>(ws + o_off);
    float *xg = reinterpret_cast<float *>(ws + o_xg);
    float *gb = reinterpret_cast<float *>(ws + o_g);
    float *ub = reinterpret_cast<float *>(ws + o_u);
    float *yb = reinterpret_cast<float *>(ws + o_y);
    float *rw = reinterpret_cast<float *>(ws + o_rw);

    // routing and the grouping by expert: one single-CTA launch
    CUDA_TRY(rce::launch_moe_route_plan(d_logits, ld_logits, (int)t_rows, n_experts, top_k, 1, idx, wt, expert_begin,
                                        expert_end, off, pos, tok, rw, s));
    // Prefill-sized batches: every local expert's gate and up in one grouped
    // tensor-core launch, the down matmuls in another, the row counts read
    // on the device (no host synchronisation; the call can be captured in a
    // CUDA graph).  Smaller batches, prefill_min_tokens = 0 (the exact
    // path) and experts of mixed formats: each expert's matmuls on their own,
    // sized by the row counts copied to the host.
    bool grouped = ctx->prefill_min_tokens > 0 && t_rows >= (size_t)ctx->prefill_min_tokens;
    for (int e = expert_begin; e < expert_end && grouped; e++)
        grouped = gate[e]->dtype == g0->dtype && up[e]->dtype == g0->dtype &&
                  down[e]->dtype == down[expert_begin]->dtype;
    if (grouped) {
        // Launches: route+plan, gather_prep (also clears the output), the
        // gate/up matmuls of every local expert with h = silu(g) * u from
        // their epilogue, h_prep, the down matmuls adding w * y into the
        // output from their epilogue (at most two route slots per token: a
        // sum of two is the same in either order, so the atomic adds give
        // the combine's bits; more slots keep the ordered combine kernel).
        constexpr int kG = rce::kGemmMaxGroup;
        const int32_t *n_rows = off + n_local;
        const int max_rows = (int)t_rows;  // a token picks an expert at most once
        const int rows_hint = (int)(P * (size_t)n_local / (size_t)n_experts);
        const bool fuse_combine = top_k <= 2;
        void *xh = ws + o_xg, *xh2 = ws + o_xh2;
        float *inv = reinterpret_cast<float *>(ws + o_inv), *inv2 = reinterpret_cast<float *>(ws + o_inv2);
        const uint8_t *wz[kG], *w2z[kG];
        float *yz[kG];
        int sz[kG];
        CUDA_TRY(rce::launch_moe_gather_prep(d_x, ldx, tok, n_rows, (int)P, (int)d_model, xh, inv,
                                             fuse_combine ? d_out : nullptr, ldo, (int)t_rows, s));
        for (int i0 = 0; i0 < n_local; i0 += kG) {  // entry i: gate and up of local expert i, h into gb
            int n = 0;
            for (int i = i0; i < n_local && i < i0 + kG; i++)
                wz[n] = gate[expert_begin + i]->dev, w2z[n] = up[expert_begin + i]->dev, yz[n] = gb, sz[n++] = i;
            rce::GroupEpi ge;
            ge.mode = rce::kGroupSwiGLU;
            ge.ws2 = w2z;
            CUDA_TRY(rce::launch_gemm_grouped(g0->dtype, wz, yz, sz, n, g0->g, xh, inv, (int)P, rows_hint, off,
                                              n_local, max_rows, (size_t)d_ff, ctx->err_dev, s, ge));
        }
        CUDA_TRY(rce::launch_moe_h_prep(gb, (size_t)d_ff, n_rows, (int)P, (int)d_ff, xh2, inv2, s));
        const rce_qmm_weight *d0 = down[expert_begin];
        rce::GroupEpi de;
        if (fuse_combine) {
            de.mode = rce::kGroupCombine;
            de.row_token = tok;
            de.row_w = rw;
            de.out = d_out;
            de.ldo = ldo;
        }
        for (int i0 = 0; i0 < n_local; i0 += kG) {
            int n = 0;
            for (int i = i0; i < n_local && i < i0 + kG; i++) wz[n] = down[expert_begin + i]->dev, yz[n] = yb, sz[n++] = i;
            CUDA_TRY(rce::launch_gemm_grouped(d0->dtype, wz, yz, sz, n, d0->g, xh2, inv2, (int)P, rows_hint, off,
                                              n_local, max_rows, (size_t)d_model, ctx->err_dev, s, de));
        }
        if (!fuse_combine)
            CUDA_TRY(rce::launch_moe_combine(yb, (int)d_model, pos, wt, (int)t_rows, top_k, d_out, ldo, s));
        return ok();
    }
    // the per-expert row counts size the matmuls below
    CUDA_TRY(cudaMemcpyAsync(host_off, off, (size_t)(n_local + 1) * 4, cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaStreamSynchronize(s));
    const int rows = host_off[n_local];
    if (rows > 0) {
        CUDA_TRY(rce::launch_moe_gather(d_x, ldx, tok, rows, (int)d_model, xg, s));
        for (int i = 0; i < n_local; i++) {
            const size_t r0 = (size_t)host_off[i], n = (size_t)(host_off[i + 1] - host_off[i]);
            if (n == 0) continue;
            const int e = expert_begin + i;
            rc = run_matmul(ctx, gate[e], xg + r0 * d_model, (size_t)d_model, n, gb + r0 * d_ff, (size_t)d_ff, s);
            if (rc) return rc;
            rc = run_matmul(ctx, up[e], xg + r0 * d_model, (size_t)d_model, n, ub + r0 * d_ff, (size_t)d_ff, s);
            if (rc) return rc;
        }
        CUDA_TRY(rce::launch_swiglu(gb, ub, gb, (size_t)rows * d_ff, s));
        for (int i = 0; i < n_local; i++) {
            const size_t r0 = (size_t)host_off[i], n = (size_t)(host_off[i + 1] - host_off[i]);
            if (n == 0) continue;
            rc = run_matmul(ctx, down[expert_begin + i], gb + r0 * d_ff, (size_t)d_ff, n, yb + r0 * d_model,
                            (size_t)d_model, s);
            if (rc) return rc;
        }
    }
    CUDA_TRY(rce::launch_moe_combine(yb, (int)d_model, pos, wt, (int)t_rows, top_k, d_out, ldo, s));
    return ok();
}

int rce_qmm_moe_shared_expert_device(rce_qmm_ctx *ctx, const float *d_x, size_t ldx, size_t t_rows,
                                     const rce_qmm_weight *gate, const rce_qmm_weight *up,
                                     const rce_qmm_weight *down, const float *d_gate_inp, float *d_out,
                                     size_t ldo, void *stream) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "moe_shared_expert_device: null ctx");
    for (const rce_qmm_weight *w : {gate, up, down}) {
        const int rc = check_weight(w);
        if (rc) return rc;
        if (w->ctx != ctx) return fail(RCE_QMM_ERR_INVALID, "moe_shared_expert_device: weight of another context");
    }
    const int64_t d_model = gate->g.n_cols, n_ff = gate->g.n_rows;
    if (up->g.n_rows != n_ff || up->g.n_cols != d_model || down->g.n_rows != d_model || down->g.n_cols != n_ff)
        return fail(RCE_QMM_ERR_INVALID,
                    "moe_shared_expert_device: gate/up must be [%lld x %lld] and down [%lld x %lld]",
                    (long long)n_ff, (long long)d_model, (long long)d_model, (long long)n_ff);
    if (t_rows == 0) return ok();
    if (!d_x || !d_gate_inp || !d_out) return fail(RCE_QMM_ERR_INVALID, "moe_shared_expert_device: null buffer");
    if (ldx < (size_t)d_model || ldo < (size_t)d_model)
        return fail(RCE_QMM_ERR_INVALID, "moe_shared_expert_device: ldx %zu / ldo %zu < d_model %lld", ldx, ldo,
                    (long long)d_model);
    if (t_rows > (size_t)INT32_MAX) return fail(RCE_QMM_ERR_INVALID, "moe_shared_expert_device: too many tokens");
    DeviceGuard dg(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // workspace: g and u [t][n_ff] (h = silu(g) * u written over g), sh [t][d_model]
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    const size_t o_u = al(t_rows * (size_t)n_ff * 4), o_sh = o_u + al(t_rows * (size_t)n_ff * 4);
    void *wsv = nullptr;
    int32_t *host_off = nullptr;
    int rc = stream_moe_ws(ctx, s, o_sh + al(t_rows * (size_t)d_model * 4), 1, &wsv, &host_off);
    if (rc) return rc;
    float *gb = static_cast<float *>(wsv);
    float *ub = reinterpret_cast<float *>(static_cast<uint8_t *>(wsv) + o_u);
    float *sh = reinterpret_cast<float *>(static_cast<uint8_t *>(wsv) + o_sh);
    rc = run_matmul(ctx, gate, d_x, ldx, t_rows, gb, (size_t)n_ff, s);
    if (rc) return rc;
    rc = run_matmul(ctx, up, d_x, ldx, t_rows, ub, (size_t)n_ff, s);
    if (rc) return rc;
    CUDA_TRY(rce::launch_swiglu(gb, ub, gb, t_rows * (size_t)n_ff, s));
    rc = run_matmul(ctx, down, gb, (size_t)n_ff, t_rows, sh, (size_t)d_model, s);
    if (rc) return rc;
    CUDA_TRY(rce::launch_moe_shared_combine(d_x, ldx, (int)t_rows, (int)d_model, d_gate_inp, sh, (size_t)d_model,
                                            d_out, ldo, s));
    return ok();
}

int rce_qmm_moe_ffn(rce_qmm_ctx *ctx, const float *x, size_t t_rows, const float *router_logits,
                    const rce_qmm_weight *router_w, int n_experts, int top_k, int expert_begin, int expert_end,
                    const rce_qmm_weight *const *gate, const rce_qmm_weight *const *up,
                    const rce_qmm_weight *const *down, float *out, int32_t *idx_out, float *w_out) {
    if (!ctx) return fail(RCE_QMM_ERR_INVALID, "moe_ffn: null ctx");
    if (!gate || !up || !down || expert_begin < 0 || expert_begin >= n_experts)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn: null weight array or bad expert range");
    int rc = check_weight(gate[expert_begin]);
    if (rc) return rc;
    if (t_rows == 0) return ok();
    if (!x || !out) return fail(RCE_QMM_ERR_INVALID, "moe_ffn: null buffer");
    if (!router_logits) {
        if ((rc = check_weight(router_w))) return rc;
        if (router_w->g.n_rows != n_experts || router_w->g.n_cols != gate[expert_begin]->g.n_cols)
            return fail(RCE_QMM_ERR_INVALID, "moe_ffn: router weight is [%lld x %lld], [n_experts x d_model] needed",
                        (long long)router_w->g.n_rows, (long long)router_w->g.n_cols);
    }
    if (top_k < 1 || top_k > n_experts || n_experts > 256)
        return fail(RCE_QMM_ERR_INVALID, "moe_ffn: n_experts %d (1..256), top_k %d (1..n_experts)", n_experts, top_k);
    const size_t d_model = (size_t)gate[expert_begin]->g.n_cols;
    DeviceGuard dg(ctx->device);
    RceThreadState *ts = nullptr;
    if ((rc = thread_state(ctx, &ts))) return rc;
    // device staging: x and logits in d_in; out, weights and indices in d_out
    const size_t xf = t_rows * d_model, lf = t_rows * (size_t)n_experts, rf = t_rows * (size_t)top_k;
    const size_t in_f = xf + lf, out_f = xf + 2 * rf;
    if ((rc = grow_device(&ts->d_in, &ts->d_in_cap, in_f))) return rc;
    if ((rc = grow_device(&ts->d_out, &ts->d_out_cap, out_f))) return rc;
    if ((rc = grow_pinned(ts, (in_f > out_f ? in_f : out_f) * sizeof(float)))) return rc;
    float *d_x = ts->d_in, *d_lg = ts->d_in + xf, *d_y = ts->d_out, *d_w = ts->d_out + xf;
    int32_t *d_idx = reinterpret_cast<int32_t *>(ts->d_out + xf + rf);
    float *h = static_cast<float *>(ts->h_pin);
    std::memcpy(h, x, xf * sizeof(float));
    if (router_logits) std::memcpy(h + xf, router_logits, lf * sizeof(float));
    CUDA_TRY(cudaMemcpyAsync(d_x, h, (router_logits ? in_f : xf) * sizeof(float), cudaMemcpyHostToDevice, ts->stream));
    if (!router_logits) {
        rc = run_matmul(ctx, router_w, d_x, d_model, t_rows, d_lg, (size_t)n_experts, ts->stream);
        if (rc) return rc;
    }
    rc = rce_qmm_moe_ffn_device(ctx, d_x, d_model, t_rows, d_lg, (size_t)n_experts, n_experts, top_k, expert_begin,
                                expert_end, gate, up, down, d_y, d_model, d_idx, d_w, ts->stream);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(h, d_y, out_f * sizeof(float), cudaMemcpyDeviceToHost, ts->stream));
    CUDA_TRY(cudaStreamSynchronize(ts->stream));
    if ((rc = take_kernel_error(ctx))) return rc;
    std::memcpy(out, h, xf * sizeof(float));
    if (w_out) std::memcpy(w_out, h + xf, rf * sizeof(float));
    if (idx_out) std::memcpy(idx_out, h + xf + rf, rf * sizeof(int32_t));
    return ok();
}

}  // extern "C"
