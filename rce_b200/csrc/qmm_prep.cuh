// qmm_prep.cuh -- the activation side of the tensor-core GEMM: one row of f32
// values scaled by a power of two s (|v * s| < 2^14, so the scaling is exact
// and no value overflows fp16) and rounded to fp16 (the high term), with 1/s
// kept per row; optionally also the low term, the fp16 rounding of the
// remainder v * s - high (exact in f32), so that high + low carries about 22
// significant bits of v.  Shared by the dense prep kernel (qmm_gemm.cu) and
// the MoE gather and SwiGLU preps (qmm_moe.cu), so every GEMM input is
// rounded the same way.
#pragma once

#include <cuda_fp16.h>

namespace rce {

constexpr int kPrepThreads = 256;

// One kPrepThreads-thread block per row: val(i) yields element i (it is
// called twice per element, for the row maximum and for the store); o_lo
// (optional) receives the low terms.  A row
// holding a NaN or an infinity gets s = 0 and 1/s = NaN, so its outputs are
// NaN as the f32 arithmetic would make them.
template <class Val>
__device__ __forceinline__ void prep_row(Val val, int k, __half *o, float *inv, __half *o_lo = nullptr) {
    float mx = 0.f;
    bool fin = true;
    for (int i = threadIdx.x; i < k; i += kPrepThreads) {
        const float v = val(i);
        mx = fmaxf(mx, fabsf(v));
        fin = fin && isfinite(v);
    }
    if (!fin) mx = INFINITY;
    __shared__ float red[kPrepThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    float v = 0.f;
    for (int w = 0; w < kPrepThreads / 32; w++) v = fmaxf(v, red[w]);
    float s = 1.f, is = 1.f;
    if (!isfinite(v)) {
        s = 0.f;
        is = __int_as_float(0x7fc00000);
    } else if (v > 0.f) {
        int e;
        frexpf(v, &e);
        e = max(-100, min(100, e));
        s = ldexpf(1.f, 14 - e);
        is = ldexpf(1.f, e - 14);
    }
    // the GEMM may start its weight copies now; it reads these rows only
    // after griddepcontrol.wait, i.e. after this grid has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (o_lo) {
        for (int i = threadIdx.x; i < k; i += kPrepThreads) {
            const float v = val(i) * s;
            const __half hi = __float2half_rn(v);
            o[i] = hi;
            o_lo[i] = __float2half_rn(v - __half2float(hi));
        }
    } else {
        for (int i = threadIdx.x; i < k; i += kPrepThreads) o[i] = __float2half_rn(val(i) * s);
    }
    if (threadIdx.x == 0) *inv = is;
}

// silu as moe_ffn_forward's expert computes it (rce-qwen36-moe/src/lib.rs:649-656):
// x / (1 + exp(-x)) for x >= 0, x e^x / (1 + e^x) below, each operation
// rounded on its own (exp is the device's expf).
__device__ __forceinline__ float silu_ref(float x) {
    if (x >= 0.f) {
        const float den = __fadd_rn(1.f, expf(-x));
        return __fdiv_rn(x, den);
    }
    const float e = expf(x);
    const float num = __fmul_rn(x, e);
    const float den = __fadd_rn(1.f, e);
    return __fdiv_rn(num, den);
}

// The same silu with the hardware exponential (__expf) and a correctly
// rounded reciprocal in place of the division: within a few units in the
// last place of silu_ref, at a fraction of its instructions (the grouped
// GEMM's SwiGLU epilogue runs it in its tail, with nothing to overlap).
__device__ __forceinline__ float silu_fast(float x) {
    if (x >= 0.f) return __fmul_rn(x, __frcp_rn(__fadd_rn(1.f, __expf(-x))));
    const float e = __expf(x);
    return __fmul_rn(__fmul_rn(x, e), __frcp_rn(__fadd_rn(1.f, e)));
}

}  // namespace rce
