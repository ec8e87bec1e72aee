// qmm_gather.cu -- the fused all-gather's stand-alone kernels: pushing a
// shard that a kernel wrote only locally (the prefill GEMM) to the peers'
// receive buffers, unpacking a receive buffer once its words carry the
// expected epoch, and advancing the device epoch base.
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

cudaError_t launch_epoch_advance(unsigned *epoch_base, unsigned delta, cudaStream_t s) {
    advance_kernel<<<1, 1, 0, s>>>(epoch_base, delta);
    return cudaGetLastError();
}

}  // namespace rce
