// qmm_gather.cu -- the fused all-gather's stand-alone kernels: pushing a
// shard that a kernel wrote only locally (the prefill GEMM) to the peers'
// receive buffers, unpacking a receive buffer once its words carry the
// expected epoch, the bulk mode for large outputs (plain values and one
// release flag per peer), and advancing the device epoch base.
#include <cuda_runtime.h>

#include "qmm_gather.cuh"
#include "qmm_internal.h"

namespace rce {
namespace {

constexpr unsigned long long kUnpackWaitNs = 1000000000ull;  // 1 s per launch

__global__ void push_kernel(GatherArgs ga, const float *y, int t_rows, int64_t n, size_t ldy) {
    const unsigned e = gather_epoch(ga);
    const size_t total = (size_t)t_rows * (size_t)n;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / (size_t)n, c = i % (size_t)n;
        const size_t off = t * ldy + (size_t)ga.row_off + c;
        gather_send(ga, off, y[off], e);
    }
}

__global__ void unpack_kernel(const unsigned long long *ll, float *y, int t_rows, int64_t n, size_t ldy,
                              int64_t own0, int64_t own1, unsigned epoch_rel, const unsigned *epoch_base, int *err) {
    const unsigned e = epoch_base ? epoch_rel + *reinterpret_cast<const volatile unsigned *>(epoch_base) : epoch_rel;
    const int64_t others = n - (own1 - own0);
    const size_t total = (size_t)t_rows * (size_t)others;
    unsigned long long t0 = 0;
    bool timed = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t t = i / (size_t)others;
        int64_t c = (int64_t)(i % (size_t)others);
        if (c >= own0) c += own1 - own0;  // skip this rank's own rows
        const size_t off = t * ldy + (size_t)c;
        unsigned long long w = *reinterpret_cast<const volatile unsigned long long *>(ll + off);
        while ((int)((unsigned)(w >> 32) - e) < 0) {  // this epoch or a later one (a later call's value)
            if (!timed) {
                asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
                timed = true;
            }
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (now - t0 > kUnpackWaitNs) {
                *reinterpret_cast<volatile int *>(err) = kKernelErrWaitTimeout;
                return;
            }
            w = *reinterpret_cast<const volatile unsigned long long *>(ll + off);
        }
        y[off] = __uint_as_float((unsigned)w);
    }
}

// Bulk mode, for large outputs (prefill): plain f32 values into each peer's
// bulk buffer at the same [t][ldy] positions, then (push_flags, a kernel
// that runs after this one on the stream) one release flag per peer.  Half
// the NVLink bytes of the {value, epoch} words; the flags cost a
// system-scope release per call, negligible next to a large output.
struct BulkPeers {
    float *buf[kMaxPeers];  // peers' bulk buffers (this rank's entry unused)
};

__global__ void push_bulk_kernel(BulkPeers bp, int world, int rank, const float *y, int64_t row_off, int64_t n_own,
                                 size_t ldy, int vec4) {
    const int t = blockIdx.y;
    const float *src = y + (size_t)t * ldy + row_off;
    if (vec4) {
        const int64_t n4 = n_own / 4;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
            const float4 v = reinterpret_cast<const float4 *>(src)[i];
            for (int r = 0; r < world; r++)
                if (r != rank) reinterpret_cast<float4 *>(bp.buf[r] + (size_t)t * ldy + row_off)[i] = v;
        }
    } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_own; i += (int64_t)gridDim.x * blockDim.x) {
            const float v = src[i];
            for (int r = 0; r < world; r++)
                if (r != rank) bp.buf[r][(size_t)t * ldy + row_off + i] = v;
        }
    }
    __threadfence_system();  // the values reach the peers before the flags that follow this kernel
}

// flags[r] of peer r's buffer, slot `rank`: this call's epoch, released at
// system scope.
__global__ void push_flags_kernel(BulkPeers bp, size_t flag_off, int world, int rank, unsigned epoch_rel,
                                  const unsigned *epoch_base) {
    const unsigned e = epoch_base ? epoch_rel + *reinterpret_cast<const volatile unsigned *>(epoch_base) : epoch_rel;
    const int r = threadIdx.x;
    if (r < world && r != rank) {
        unsigned *f = reinterpret_cast<unsigned *>(reinterpret_cast<uint8_t *>(bp.buf[r]) + flag_off) + rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
    }
}

// Wait (bounded) until every other rank's flag carries this epoch, then copy
// their rows out of the local bulk buffer.  A flag that already carries a
// later epoch means a later call has overwritten the rows: that is reported
// in the error word (kKernelErrOverrun) and nothing is copied, never a mix
// of two calls' rows.
__global__ void unpack_bulk_kernel(const float *buf, size_t flag_off, float *y, int t_rows, int64_t n, size_t ldy,
                                   int64_t own0, int64_t own1, int world, int rank, unsigned epoch_rel,
                                   const unsigned *epoch_base, int *err) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    const unsigned e = epoch_base ? epoch_rel + *reinterpret_cast<const volatile unsigned *>(epoch_base) : epoch_rel;
    const int r = threadIdx.x;
    if (r < world && r != rank) {
        const unsigned *f =
            reinterpret_cast<const unsigned *>(reinterpret_cast<const uint8_t *>(buf) + flag_off) + r;
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        unsigned long long t0 = 0, now = 0;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        while ((int)(v - e) < 0) {
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (now - t0 > kUnpackWaitNs) {
                failed = 1;
                *reinterpret_cast<volatile int *>(err) = kKernelErrWaitTimeout;
                break;
            }
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        }
        if (!failed && v != e) {
            failed = 1;
            *reinterpret_cast<volatile int *>(err) = kKernelErrOverrun;
        }
    }
    __syncthreads();
    if (failed) return;
    const int t = blockIdx.y;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < n; c += (int64_t)gridDim.x * blockDim.x) {
        if (c >= own0 && c < own1) continue;
        y[(size_t)t * ldy + c] = __ldcv(buf + (size_t)t * ldy + c);
    }
}

__global__ void advance_kernel(unsigned *base, unsigned delta) { *base += delta; }

}  // namespace

cudaError_t launch_gather_push(const GatherArgs &ga, const float *y, int t_rows, int64_t n, size_t ldy,
                               cudaStream_t s) {
    if (ga.world < 2 || ga.world > kMaxPeers) return cudaErrorInvalidValue;
    const size_t total = (size_t)t_rows * (size_t)n;
    unsigned blocks = (unsigned)((total + 255) / 256);
    if (blocks > 1024) blocks = 1024;
    if (blocks < 1) blocks = 1;
    push_kernel<<<blocks, 256, 0, s>>>(ga, y, t_rows, n, ldy);
    return cudaGetLastError();
}

cudaError_t launch_gather_unpack(const unsigned long long *ll, float *y, int t_rows, int64_t n, size_t ldy,
                                 int64_t own0, int64_t own1, unsigned epoch, const unsigned *epoch_base, int *err,
                                 cudaStream_t s) {
    const size_t total = (size_t)t_rows * (size_t)(n - (own1 - own0));
    if (total == 0) return cudaSuccess;
    unsigned blocks = (unsigned)((total + 255) / 256);
    if (blocks > 592) blocks = 592;
    unpack_kernel<<<blocks, 256, 0, s>>>(ll, y, t_rows, n, ldy, own0, own1, epoch, epoch_base, err);
    return cudaGetLastError();
}

cudaError_t launch_gather_push_bulk(int world, int rank, float *const *peer_bufs, size_t flag_off, const float *y,
                                    int t_rows, int64_t row_off, int64_t n_own, size_t ldy, unsigned epoch,
                                    const unsigned *epoch_base, cudaStream_t s) {
    if (world < 2 || world > kMaxPeers || t_rows <= 0 || t_rows > 65535) return cudaErrorInvalidValue;
    BulkPeers bp = {};
    for (int r = 0; r < world; r++) bp.buf[r] = peer_bufs[r];
    const int vec4 = (ldy % 4 == 0 && row_off % 4 == 0 && n_own % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(y) & 15) == 0) ? 1 : 0;
    for (int r = 0; r < world; r++)
        if (r != rank && (reinterpret_cast<uintptr_t>(bp.buf[r]) & 15)) return cudaErrorInvalidValue;
    const int64_t items = vec4 ? n_own / 4 : n_own;
    unsigned bx = (unsigned)((items + 255) / 256);
    if (bx > 64) bx = 64;
    if (bx < 1) bx = 1;
    push_bulk_kernel<<<dim3(bx, t_rows), 256, 0, s>>>(bp, world, rank, y, row_off, n_own, ldy, vec4);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    push_flags_kernel<<<1, 32, 0, s>>>(bp, flag_off, world, rank, epoch, epoch_base);
    return cudaGetLastError();
}

cudaError_t launch_gather_flags_bulk(int world, int rank, float *const *peer_bufs, size_t flag_off, unsigned epoch,
                                     const unsigned *epoch_base, cudaStream_t s) {
    if (world < 2 || world > kMaxPeers) return cudaErrorInvalidValue;
    BulkPeers bp = {};
    for (int r = 0; r < world; r++) bp.buf[r] = peer_bufs[r];
    push_flags_kernel<<<1, 32, 0, s>>>(bp, flag_off, world, rank, epoch, epoch_base);
    return cudaGetLastError();
}

cudaError_t launch_gather_unpack_bulk(const float *buf, size_t flag_off, float *y, int t_rows, int64_t n, size_t ldy,
                                      int64_t own0, int64_t own1, int world, int rank, unsigned epoch,
                                      const unsigned *epoch_base, int *err, cudaStream_t s) {
    if (world < 2 || world > kMaxPeers || t_rows <= 0 || t_rows > 65535) return cudaErrorInvalidValue;
    unsigned bx = (unsigned)((n + 255) / 256);
    if (bx > 16) bx = 16;
    if (bx < 1) bx = 1;
    unpack_bulk_kernel<<<dim3(bx, t_rows), 256, 0, s>>>(buf, flag_off, y, t_rows, n, ldy, own0, own1, world, rank,
                                                        epoch, epoch_base, err);
    return cudaGetLastError();
}

cudaError_t launch_epoch_advance(unsigned *epoch_base, unsigned delta, cudaStream_t s) {
    advance_kernel<<<1, 1, 0, s>>>(epoch_base, delta);
    return cudaGetLastError();
}

}  // namespace rce
