// qmm_gemv.cu -- decode GEMV / small-M matmul over T16 weight tiles.
//
// y[t][row] = sum_k x[t][k] * W[row][k], the arithmetic of the reference's
// mm_1d (rce-op-qmm/src/lib.rs:496-522 Q4_0, :648-670 Q8_0, :730-781 Q4_K)
// up to f32 summation order.
//
// Design (HBM-bound; every weight byte is read once):
//  * Each warp owns one 16-row tile and streams its 256-column chunks with
//    128-bit ld.global.nc.L1::no_allocate loads; the T16 layout makes every
//    warp-wide load one contiguous 512-byte segment.  The next chunk is in
//    flight while the current one is computed.
//  * Dequantisation stays in registers and stays exact: the quant codes are
//    turned into fp16 integers (q, q-8 or the signed byte) with lop3/prmt
//    magic-number tricks, which are exact for |q| <= 2048.  The block scales
//    are applied in f32 after the dot product of each 32-value sub-block, so
//    no weight is ever rounded.
//  * The dot products run on the tensor cores (mma.sync m16n8k16, f32
//    accumulate) as a throughput device: a CUDA-core FFMA loop would need
//    ~3 ALU ops per weight, more than the SM issues at HBM speed for 4-bit
//    formats.  Each lane feeds one column group g (its two sub-blocks), and
//    the activation operand is block-diagonal: column 2g holds the fp16 "hi"
//    part of x and column 2g+1 the "lo" remainder, so D[r][2g] + D[r][2g+1]
//    is the sub-block dot product with ~22 significant bits of x.
//  * x is scaled per token by a power of two (exact) so hi/lo stay inside
//    fp16's range; the scale is undone on the f32 partial sums.
//  * Q4_K's min term uses per-sub-block activation sums (the "asum hoist"),
//    one FFMA per sub-block instead of one per weight.
//  * K is split across CTAs when there are too few rows to fill 148 SMs;
//    partial sums go to scratch and the last CTA to arrive for a row block
//    adds them in split order (deterministic), then re-arms its counter.
#include <cuda_fp16.h>

#include "qmm_internal.h"

namespace rce {
namespace {

struct GemvArgs {
    const uint8_t *w;
    const float *x;
    float *y;
    float *partial;
    unsigned *counters;
    Geometry g;
    size_t ldx, ldy;
    int m, cps, k_splits, n_pad;
};

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint2 ldg_stream2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// (a & mask) | orv
__device__ __forceinline__ uint32_t lop3_ao(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t comp(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

template <int DT>
struct Fmt {
    static constexpr int NQ = DT == GGUF_Q8_0 ? 8 : 4;  // 16-byte quant loads per lane per chunk
};

template <int DT>
struct ChunkRegs {
    uint4 q[Fmt<DT>::NQ];
    uint4 h0, h1;  // Q4_K: headers of rows r and r+8; Q4_0/Q8_0: h0.xy = the lane's 4 scales
};

template <int DT>
__device__ __forceinline__ void load_chunk(ChunkRegs<DT> &c, const uint8_t *chunk, int lane) {
#pragma unroll
    for (int i = 0; i < Fmt<DT>::NQ; i++) c.q[i] = ldg_stream(chunk + (i * 32 + lane) * 16);
    if (DT == GGUF_Q4_K) {
        c.h0 = ldg_stream(chunk + 2048 + (lane >> 2) * 16);
        c.h1 = ldg_stream(chunk + 2048 + ((lane >> 2) + 8) * 16);
    } else {
        const uint2 s = ldg_stream2(chunk + quant_bytes(DT) + lane * 8);
        c.h0.x = s.x;
        c.h0.y = s.y;
        c.h0.z = 0;
        c.h0.w = 0;
        c.h1 = c.h0;
    }
}

// The exact fp16 operand of step j (16 columns) for rows r (a0, a2) and
// r + 8 (a1, a3).  a0/a1 hold columns (e0, e2) and a2/a3 (e1, e3) of the
// lane's four columns 64g + 4(j%8...) -- see qmm_layout.cuh.
template <int DT>
__device__ __forceinline__ void make_a(const ChunkRegs<DT> &c, int j, uint32_t (&a)[4]) {
    const int h = j >> 3, jj = j & 7;
    if (DT == GGUF_Q4_K) {
        const uint32_t wr = comp(c.q[jj >> 2], jj & 3);
        const uint32_t w8 = comp(c.q[2 + (jj >> 2)], jj & 3);
        if (h == 0) {  // low nibbles: fp16(1024 + q) - 1024
            a[0] = hsub2(lop3_ao(wr, 0x000F000Fu, 0x64006400u), 0x64006400u);
            a[2] = hsub2(lop3_ao(wr >> 8, 0x000F000Fu, 0x64006400u), 0x64006400u);
            a[1] = hsub2(lop3_ao(w8, 0x000F000Fu, 0x64006400u), 0x64006400u);
            a[3] = hsub2(lop3_ao(w8 >> 8, 0x000F000Fu, 0x64006400u), 0x64006400u);
        } else {  // high nibbles: fp16(1024 + 16q) / 16 - 64
            a[0] = hfma2(lop3_ao(wr, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD400D400u);
            a[2] = hfma2(lop3_ao(wr >> 8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD400D400u);
            a[1] = hfma2(lop3_ao(w8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD400D400u);
            a[3] = hfma2(lop3_ao(w8 >> 8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD400D400u);
        }
    } else if (DT == GGUF_Q4_0) {
        const uint32_t wr = comp(c.q[h], jj & 3);
        const uint32_t w8 = comp(c.q[2 + h], jj & 3);
        if ((jj >> 2) == 0) {  // low nibbles: fp16(1024 + n) - 1032 = n - 8
            a[0] = hsub2(lop3_ao(wr, 0x000F000Fu, 0x64006400u), 0x64086408u);
            a[2] = hsub2(lop3_ao(wr >> 8, 0x000F000Fu, 0x64006400u), 0x64086408u);
            a[1] = hsub2(lop3_ao(w8, 0x000F000Fu, 0x64006400u), 0x64086408u);
            a[3] = hsub2(lop3_ao(w8 >> 8, 0x000F000Fu, 0x64006400u), 0x64086408u);
        } else {  // high nibbles: fp16(1024 + 16n) / 16 - 72 = n - 8
            a[0] = hfma2(lop3_ao(wr, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
            a[2] = hfma2(lop3_ao(wr >> 8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
            a[1] = hfma2(lop3_ao(w8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
            a[3] = hfma2(lop3_ao(w8 >> 8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, 0xD480D480u);
        }
    } else {  // Q8_0: byte ^ 0x80 = q + 128; fp16(1024 + q + 128) - 1152 = q
        const uint32_t wr = comp(c.q[2 * h + (jj >> 2)], jj & 3) ^ 0x80808080u;
        const uint32_t w8 = comp(c.q[4 + 2 * h + (jj >> 2)], jj & 3) ^ 0x80808080u;
        a[0] = hsub2(prmt(wr, 0x64646464u, 0x4240u), 0x64806480u);
        a[2] = hsub2(prmt(wr, 0x64646464u, 0x4341u), 0x64806480u);
        a[1] = hsub2(prmt(w8, 0x64646464u, 0x4240u), 0x64806480u);
        a[3] = hsub2(prmt(w8, 0x64646464u, 0x4341u), 0x64806480u);
    }
}

// Q4_K header fields for lane group g: d, dmin and the 24-bit scale field.
__device__ __forceinline__ void q4k_header(const uint4 &hd, int g, float &d1, float &m1, float &d2,
                                           float &m2) {
    const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
    const uint32_t lo = g < 2 ? hd.y : (g == 2 ? hd.z : hd.w);
    const uint32_t hi = g < 2 ? hd.z : (g == 2 ? hd.w : 0u);
    const uint32_t sh = g == 0 ? 0u : (g == 1 ? 24u : (g == 2 ? 16u : 8u));
    const uint32_t v = __funnelshift_r(lo, hi, sh) & 0xFFFFFFu;
    d1 = d * (float)(v & 63u);
    m1 = dmin * (float)((v >> 6) & 63u);
    d2 = d * (float)((v >> 12) & 63u);
    m2 = dmin * (float)((v >> 18) & 63u);
}

template <int DT, int NT>
__device__ __forceinline__ void process_chunk(const ChunkRegs<DT> &c, float (&acc)[NT][2],
                                              const uint2 *__restrict__ tbl, int tok_stride,
                                              const float *__restrict__ asum, int asum_stride, int m,
                                              int lane, bool bact, int boff) {
    const int g = lane & 3;
    float ds[2][2], mn[2][2];
    if (DT == GGUF_Q4_K) {
        q4k_header(c.h0, g, ds[0][0], mn[0][0], ds[1][0], mn[1][0]);
        q4k_header(c.h1, g, ds[0][1], mn[0][1], ds[1][1], mn[1][1]);
    } else {
        ds[0][0] = h2f(c.h0.x);
        ds[1][0] = h2f(c.h0.x >> 16);
        ds[0][1] = h2f(c.h0.y);
        ds[1][1] = h2f(c.h0.y >> 16);
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float d[NT][4];
#pragma unroll
        for (int t = 0; t < NT; t++) d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
            const int j = 8 * h + jj;
            uint32_t a[4];
            make_a<DT>(c, j, a);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                if (t < m) {
                    uint2 b = tbl[t * tok_stride + j * 8 + boff];
                    if (!bact) b = make_uint2(0u, 0u);
                    mma16816(d[t], a, b.x, b.y);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            acc[t][0] = fmaf(ds[h][0], d[t][0] + d[t][1], acc[t][0]);
            acc[t][1] = fmaf(ds[h][1], d[t][2] + d[t][3], acc[t][1]);
        }
    }
    if (DT == GGUF_Q4_K) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
            if (t < m) {
                const float2 s = *reinterpret_cast<const float2 *>(asum + t * asum_stride + 2 * g);
                acc[t][0] -= fmaf(mn[0][0], s.x, mn[1][0] * s.y);
                acc[t][1] -= fmaf(mn[0][1], s.x, mn[1][1] * s.y);
            }
        }
    }
}

template <int DT, int NT, int RT>
__global__ void __launch_bounds__(256, (NT <= 4 ? 2 : 1)) gemv_kernel(GemvArgs p) {
    constexpr int KQ = 8 / RT;
    constexpr int CB = chunk_bytes(DT);
    extern __shared__ __align__(16) uint8_t smem[];
    const int cps = p.cps, m = p.m;
    const int c0 = blockIdx.y * cps;
    const int nc = min(cps, p.g.n_chunks - c0);
    uint2 *tbl = reinterpret_cast<uint2 *>(smem);                 // [m][cps][16 steps][8]
    float *asum = reinterpret_cast<float *>(tbl + (size_t)m * cps * 128);  // [m][cps][8]
    float *red = asum + (size_t)m * cps * 8;                       // [8 warps][NT][16]
    float *scl = red + 8 * NT * 16;                                // [NT] scale, [NT] inverse
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // Weight loads do not depend on x: issue the first chunk before the
    // activation table is built so its latency overlaps that work.
    const int rt_local = warp % RT, kq = warp / RT;
    const int tile = blockIdx.x * RT + rt_local;
    const bool tile_ok = tile < p.g.n_tiles;
    const uint8_t *wbase = p.w + ((size_t)tile * p.g.n_chunks + c0) * CB;
    ChunkRegs<DT> cur;
    if (tile_ok && kq < nc) load_chunk<DT>(cur, wbase + (size_t)kq * CB, lane);

    // Per-token power-of-two scale for this CTA's column slice.
    const int64_t k_lo = (int64_t)c0 * CHUNK_K;
    const int64_t k_hi = min((int64_t)(c0 + nc) * CHUNK_K, p.g.n_cols);
    float mx[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) {
        mx[t] = 0.f;
        if (t < m)
            for (int64_t k = k_lo + tid; k < k_hi; k += 256) mx[t] = fmaxf(mx[t], fabsf(p.x[t * p.ldx + k]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx[t] = fmaxf(mx[t], __shfl_xor_sync(0xffffffffu, mx[t], o));
        if (lane == 0) red[warp * NT + t] = mx[t];
    }
    __syncthreads();
    if (tid < NT) {
        float v = 0.f;
        for (int w = 0; w < 8; w++) v = fmaxf(v, red[w * NT + tid]);
        float s = 1.f, inv = 1.f;
        if (v > 0.f && isfinite(v)) {
            int e;
            frexpf(v, &e);  // v < 2^e
            e = max(-100, min(100, e));
            s = ldexpf(1.f, 14 - e);
            inv = ldexpf(1.f, e - 14);
        }
        scl[tid] = s;
        scl[NT + tid] = inv;
    }
    __syncthreads();

    // Activation table: per (token, chunk, step j, group g, part) one uint2 =
    // the B fragment (x[e0], x[e2]), (x[e1], x[e3]) as fp16, part 0 = hi,
    // part 1 = lo remainder.
    for (int idx = tid; idx < m * nc * 64; idx += 256) {
        const int t = idx / (nc * 64), rem = idx % (nc * 64);
        const int c = rem >> 6, q = rem & 63, gg = q >> 4, j = q & 15;
        const int64_t k = (int64_t)(c0 + c) * CHUNK_K + 64 * gg + 4 * j;
        const float s = scl[t];
        __half hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float v = (k + e < p.g.n_cols) ? p.x[t * p.ldx + k + e] * s : 0.f;
            hi[e] = __float2half_rn(v);
            lo[e] = __float2half_rn(v - __half2float(hi[e]));
        }
        uint2 *dst = tbl + ((size_t)(t * cps + c) * 16 + j) * 8 + gg * 2;
        dst[0] = make_uint2(__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[2]) << 16),
                            __half_as_ushort(hi[1]) | ((uint32_t)__half_as_ushort(hi[3]) << 16));
        dst[1] = make_uint2(__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[2]) << 16),
                            __half_as_ushort(lo[1]) | ((uint32_t)__half_as_ushort(lo[3]) << 16));
    }
    if (DT == GGUF_Q4_K) {
        for (int idx = tid; idx < m * nc * 8; idx += 256) {
            const int t = idx / (nc * 8), rem = idx % (nc * 8), c = rem >> 3, u = rem & 7;
            const int64_t k = (int64_t)(c0 + c) * CHUNK_K + 32 * u;
            const float s = scl[t];
            float sum = 0.f;
            for (int l = 0; l < 32; l++) sum += (k + l < p.g.n_cols) ? p.x[t * p.ldx + k + l] * s : 0.f;
            asum[(t * cps + c) * 8 + u] = sum;
        }
    }
    __syncthreads();

    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.f;
    const bool bact = (lane >> 3) == (lane & 3);
    const int boff = (lane & 3) * 2 + ((lane >> 2) & 1);
    if (tile_ok) {
        for (int cl = kq; cl < nc; cl += KQ) {
            ChunkRegs<DT> nxt;
            const bool more = cl + KQ < nc;
            if (more) load_chunk<DT>(nxt, wbase + (size_t)(cl + KQ) * CB, lane);
            process_chunk<DT, NT>(cur, acc, tbl + (size_t)cl * 128, cps * 128, asum + cl * 8, cps * 8, m,
                                  lane, bact, boff);
            if (more) cur = nxt;
        }
    }

    // Sum the four column groups of each row (lanes 4r .. 4r+3).
    __syncthreads();
#pragma unroll
    for (int t = 0; t < NT; t++) {
        float v0 = acc[t][0], v1 = acc[t][1];
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
        v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
        if ((lane & 3) == 0) {
            red[(warp * NT + t) * 16 + (lane >> 2)] = v0;
            red[(warp * NT + t) * 16 + (lane >> 2) + 8] = v1;
        }
    }
    __syncthreads();
    for (int idx = tid; idx < RT * m * 16; idx += 256) {
        const int rtl = idx / (m * 16), rem = idx % (m * 16), t = rem >> 4, r16 = rem & 15;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < KQ; q++) v += red[((rtl + q * RT) * NT + t) * 16 + r16];
        v *= scl[NT + t];
        const int64_t row = (int64_t)(blockIdx.x * RT + rtl) * 16 + r16;
        if (row < p.g.n_rows) {
            if (p.k_splits == 1)
                p.y[t * p.ldy + row] = v;
            else
                p.partial[((size_t)blockIdx.y * m + t) * p.n_pad + row] = v;
        }
    }
    if (p.k_splits > 1) {
        __shared__ int is_last;
        __threadfence();
        __syncthreads();
        if (tid == 0) is_last = atomicAdd(&p.counters[blockIdx.x], 1u) == (unsigned)(p.k_splits - 1);
        __syncthreads();
        if (is_last) {
            __threadfence();
            for (int idx = tid; idx < RT * m * 16; idx += 256) {
                const int rtl = idx / (m * 16), rem = idx % (m * 16), t = rem >> 4, r16 = rem & 15;
                const int64_t row = (int64_t)(blockIdx.x * RT + rtl) * 16 + r16;
                if (row < p.g.n_rows) {
                    float v = 0.f;
                    for (int ks = 0; ks < p.k_splits; ks++)
                        v += __ldcg(&p.partial[((size_t)ks * m + t) * p.n_pad + row]);
                    p.y[t * p.ldy + row] = v;
                }
            }
            if (tid == 0) p.counters[blockIdx.x] = 0u;
        }
    }
}

size_t gemv_smem(int m, int cps, int nt) {
    return (size_t)m * cps * (128 * 8 + 8 * 4) + (size_t)8 * nt * 16 * 4 + (size_t)2 * nt * 4;
}

template <int DT, int NT, int RT>
cudaError_t launch_one(const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
    auto kern = gemv_kernel<DT, NT, RT>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, 256, smem, s>>>(a);
    return cudaGetLastError();
}

template <int DT, int RT>
cudaError_t launch_nt(int nt, const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
    switch (nt) {
    case 1: return launch_one<DT, 1, RT>(a, grid, smem, s);
    case 2: return launch_one<DT, 2, RT>(a, grid, smem, s);
    case 4: return launch_one<DT, 4, RT>(a, grid, smem, s);
    case 8: return launch_one<DT, 8, RT>(a, grid, smem, s);
    case 16: return launch_one<DT, 16, RT>(a, grid, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

GemvPlan plan_gemv(int dt, const Geometry &g, int m, int sm_count) {
    (void)dt;
    GemvPlan p;
    p.nt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : m <= 8 ? 8 : 16;
    p.rt = 8;
    // The split depends on the weight's shape only, never on m, so a row's
    // result is bit-identical whatever the batch (mm_batched == T x mm_1d).
    // At most 4 chunks per split keeps the activation table of 16 tokens
    // (16 x 4 x 1056 B) inside shared memory.
    const int rows_ctas = (g.n_tiles + p.rt - 1) / p.rt;
    const int target = 2 * sm_count;
    const int k_want = (target + rows_ctas - 1) / rows_ctas;
    int cps = (g.n_chunks + k_want - 1) / k_want;
    if (cps > 4) cps = 4;
    if (cps < 1) cps = 1;
    p.cps = cps;
    p.k_splits = (g.n_chunks + cps - 1) / cps;
    p.smem = gemv_smem(m, p.cps, p.nt);
    if (p.k_splits > 1) {
        p.scratch_floats = (size_t)p.k_splits * m * g.n_tiles * 16;
        p.counters = rows_ctas;
    }
    return p;
}

cudaError_t launch_gemv(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx,
                        float *y, size_t ldy, int m, const GemvPlan &plan, float *scratch,
                        unsigned *counters, cudaStream_t s) {
    if (m <= 0 || g.n_rows <= 0) return cudaSuccess;
    GemvArgs a;
    a.w = tiles;
    a.x = x;
    a.y = y;
    a.partial = scratch;
    a.counters = counters;
    a.g = g;
    a.ldx = ldx;
    a.ldy = ldy;
    a.m = m;
    a.cps = plan.cps;
    a.k_splits = plan.k_splits;
    a.n_pad = g.n_tiles * 16;
    dim3 grid((g.n_tiles + plan.rt - 1) / plan.rt, plan.k_splits);
    if (plan.rt != 8) return cudaErrorInvalidValue;
    switch (dt) {
    case GGUF_Q4_K: return launch_nt<GGUF_Q4_K, 8>(plan.nt, a, grid, plan.smem, s);
    case GGUF_Q4_0: return launch_nt<GGUF_Q4_0, 8>(plan.nt, a, grid, plan.smem, s);
    case GGUF_Q8_0: return launch_nt<GGUF_Q8_0, 8>(plan.nt, a, grid, plan.smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace rce
