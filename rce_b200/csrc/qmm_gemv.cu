// qmm_gemv.cu -- decode GEMV / small-M matmul over T16 weight tiles.
//
// y[t][row] = sum_k x[t][k] * W[row][k], the arithmetic of the reference's
// mm_1d (rce-op-qmm/src/lib.rs:496-522 Q4_0, :648-670 Q8_0, :730-781 Q4_K)
// up to f32 summation order.
//
// Design (HBM-bound; every weight byte is read once):
//  * Each warp owns one 16-row tile and a strided subset of its 256-column
//    chunks.  Its lane 0 streams the chunks into a private shared-memory ring
//    with TMA bulk copies (cp.async.bulk + mbarrier complete_tx), S chunks
//    ahead, so ~70 KB per CTA are in flight from the first instruction on
//    and no registers are spent on loads in flight.  Every wait on an
//    mbarrier is bounded (%globaltimer); on expiry the kernel records an
//    error word, waits (bounded) for its own copies and finishes.
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
//  * The activation table (the B fragments) is built per window of chunks
//    with vectorised loads while the first weight copies are in flight.
//  * The grid puts 1-8 tiles in a CTA so that all CTAs are resident in one
//    wave; K is split across CTAs only when the rows alone cannot occupy the
//    SMs.  Split partial sums go to scratch and the last CTA to arrive for a
//    row block adds them in split order (deterministic).
// The plan depends on the weight's shape only, never on the batch, so each
// token's result is bit-identical whatever the batch size.
#include <cuda_fp16.h>

#include <atomic>

#include "qmm_internal.h"

namespace rce {
namespace {

constexpr int kMaxStages = 4;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s per wait

struct GemvArgs {
    const uint8_t *w;
    const float *x;
    float *y;
    float *partial;
    unsigned *counters;
    int *err;
    Geometry g;
    size_t ldx, ldy;
    int m, cps, k_splits, n_pad;
    int stages, window, x_vec4;
};

// ---- PTX helpers ---------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Expect `bytes` of transactions on `bar` and copy `bytes` from global `src`
// into shared `dst`; the copy's completion completes the transactions.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar`, at most kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > kWaitLimitNs) return false;
    }
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
    static constexpr int NQ = DT == GGUF_Q8_0 ? 8 : 4;  // 16-byte quant pieces per lane per chunk
};

template <int DT>
struct ChunkRegs {
    uint4 q[Fmt<DT>::NQ];
    uint4 h0, h1;  // Q4_K: headers of rows r and r+8; Q4_0/Q8_0: h0.xy = the lane's 4 scales
};

// One chunk's lane data from its shared-memory ring slot (conflict-free:
// lanes read consecutive 16-byte pieces).
template <int DT>
__device__ __forceinline__ void load_chunk(ChunkRegs<DT> &c, const uint8_t *slot, int lane) {
#pragma unroll
    for (int i = 0; i < Fmt<DT>::NQ; i++) c.q[i] = *reinterpret_cast<const uint4 *>(slot + (i * 32 + lane) * 16);
    if (DT == GGUF_Q4_K) {
        c.h0 = *reinterpret_cast<const uint4 *>(slot + 2048 + (lane >> 2) * 16);
        c.h1 = *reinterpret_cast<const uint4 *>(slot + 2048 + ((lane >> 2) + 8) * 16);
    } else {
        const uint2 s = *reinterpret_cast<const uint2 *>(slot + quant_bytes(DT) + lane * 8);
        c.h0 = make_uint4(s.x, s.y, 0u, 0u);
        c.h1 = c.h0;
    }
}

// The exact fp16 operand of step j (16 columns) for rows r (a0, a2) and
// r + 8 (a1, a3).  a0/a1 hold columns (e0, e2) and a2/a3 (e1, e3) of the
// lane's four columns 64 g + 4 j + (0..3) -- see qmm_layout.cuh.
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

// Q4_K header fields for lane group g: d*sc and dmin*m of sub-blocks 2g, 2g+1.
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

// Shared-memory carve-up, identical on host and device.
struct SmemLayout {
    size_t mbar, ring, tbl, qsum, asum, red, scl, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int dt, int nt, int m, int stages, int window) {
    SmemLayout L;
    size_t o = 0;
    L.mbar = o;
    o += 8 * kMaxStages * 8;
    o = align_up(o, 128);
    L.ring = o;
    o += (size_t)8 * stages * chunk_bytes(dt);
    o = align_up(o, 16);
    L.tbl = o;
    o += (size_t)m * window * 128 * 8;
    L.qsum = o;
    o += (size_t)m * window * 64 * 4;
    L.asum = o;
    o += (size_t)m * window * 8 * 4;
    L.red = o;
    o += (size_t)8 * nt * 16 * 4;
    L.scl = o;
    o += (size_t)2 * nt * 4;
    L.total = align_up(o, 16);
    return L;
}

template <int DT, int NT, int RT>
__global__ void __launch_bounds__(256, 2) gemv_kernel(GemvArgs p) {
    constexpr int KQ = 8 / RT;
    constexpr int CB = chunk_bytes(DT);
    extern __shared__ __align__(128) uint8_t smem[];
    const int m = p.m, S = p.stages, W = p.window;
    const SmemLayout L = smem_layout(DT, NT, m, S, W);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.mbar);
    uint8_t *ring = smem + L.ring;
    uint2 *tbl = reinterpret_cast<uint2 *>(smem + L.tbl);    // [m][W][16 steps][8]
    float *qsum = reinterpret_cast<float *>(smem + L.qsum);  // [m][W][4 groups][16 steps]
    float *asum = reinterpret_cast<float *>(smem + L.asum);  // [m][W][8 sub-blocks]
    float *red = reinterpret_cast<float *>(smem + L.red);    // [8 warps][NT][16]
    float *scl = reinterpret_cast<float *>(smem + L.scl);    // [NT] scale, [NT] inverse
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const int cps = p.cps;
    const int c0 = blockIdx.y * cps;
    const int nc = min(cps, p.g.n_chunks - c0);
    const int rt_local = warp % RT, kq = warp / RT;
    const int tile = blockIdx.x * RT + rt_local;
    const bool tile_ok = tile < p.g.n_tiles;
    // chunks of this warp: kq, kq + KQ, ... (< nc), the i-th in ring slot i % S
    const int nw = (tile_ok && kq < nc) ? (nc - kq + KQ - 1) / KQ : 0;
    const uint8_t *gsrc = p.w + ((size_t)(tile_ok ? tile : 0) * p.g.n_chunks + c0) * CB;
    const uint32_t mb0 = smem_u32(mbar + warp * kMaxStages);
    const uint32_t ring0 = smem_u32(ring + (size_t)warp * S * CB);

    // Weight copies do not depend on x: start them before anything else.
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(mb0 + 8 * s, 1);
        fence_mbar_init();
        for (int i = 0; i < min(S, nw); i++)
            bulk_load(ring0 + i * CB, gsrc + (size_t)(kq + i * KQ) * CB, CB, mb0 + 8 * i);
    }
    __syncwarp();

    // Per-token power-of-two scale for this CTA's column slice.
    const int64_t k_lo = (int64_t)c0 * CHUNK_K;
    const int64_t k_hi = min((int64_t)(c0 + nc) * CHUNK_K, p.g.n_cols);
#pragma unroll
    for (int t = 0; t < NT; t++) {
        float mx = 0.f;
        if (t < m) {
            const float *xr = p.x + t * p.ldx;
            for (int64_t k = k_lo + 4 * tid; k < k_hi; k += 1024) {
                float4 v;
                if (p.x_vec4) {
                    v = *reinterpret_cast<const float4 *>(xr + k);
                } else {
                    v = make_float4(xr[k], xr[k + 1], xr[k + 2], xr[k + 3]);
                }
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp * NT + t] = mx;
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

    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.f;
    const bool bact = (lane >> 3) == (lane & 3);
    const int boff = (lane & 3) * 2 + ((lane >> 2) & 1);
    int i = 0;          // next chunk of this warp
    bool failed = false;

    for (int win0 = 0; win0 < nc; win0 += W) {
        const int wn = min(W, nc - win0);
        __syncthreads();  // scales ready; the previous window's table is no longer read
        // Activation table for chunks [win0, win0 + wn): per (token, chunk,
        // step j, group g, part) one uint2 = the B fragment (x[e0], x[e2]),
        // (x[e1], x[e3]) as fp16, part 0 = hi, part 1 = lo remainder.
        for (int idx = tid; idx < m * wn * 64; idx += 256) {
            const int t = idx / (wn * 64), rem = idx % (wn * 64);
            const int c = rem >> 6, q = rem & 63, gg = q >> 4, j = q & 15;
            const int64_t k = (int64_t)(c0 + win0 + c) * CHUNK_K + 64 * gg + 4 * j;
            const float s = scl[t];
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (k < p.g.n_cols) {
                const float *xr = p.x + t * p.ldx + k;
                if (p.x_vec4) {
                    const float4 f = *reinterpret_cast<const float4 *>(xr);
                    v[0] = f.x;
                    v[1] = f.y;
                    v[2] = f.z;
                    v[3] = f.w;
                } else {
                    v[0] = xr[0];
                    v[1] = xr[1];
                    v[2] = xr[2];
                    v[3] = xr[3];
                }
            }
            __half hi[4], lo[4];
            float sum = 0.f;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float vs = v[e] * s;
                sum += vs;
                hi[e] = __float2half_rn(vs);
                lo[e] = __float2half_rn(vs - __half2float(hi[e]));
            }
            uint2 *dst = tbl + ((size_t)(t * W + c) * 16 + j) * 8 + gg * 2;
            dst[0] = make_uint2(__half_as_ushort(hi[0]) | ((uint32_t)__half_as_ushort(hi[2]) << 16),
                                __half_as_ushort(hi[1]) | ((uint32_t)__half_as_ushort(hi[3]) << 16));
            dst[1] = make_uint2(__half_as_ushort(lo[0]) | ((uint32_t)__half_as_ushort(lo[2]) << 16),
                                __half_as_ushort(lo[1]) | ((uint32_t)__half_as_ushort(lo[3]) << 16));
            qsum[(t * W + c) * 64 + gg * 16 + j] = sum;
        }
        if (DT == GGUF_Q4_K) {
            __syncthreads();
            // sub-block u of a chunk = group u/2, steps 8 (u%2) .. +7
            for (int idx = tid; idx < m * wn * 8; idx += 256) {
                const int t = idx / (wn * 8), rem = idx % (wn * 8), c = rem >> 3, u = rem & 7;
                const float *qs = qsum + (t * W + c) * 64 + (u >> 1) * 16 + 8 * (u & 1);
                float s = 0.f;
#pragma unroll
                for (int jj = 0; jj < 8; jj++) s += qs[jj];
                asum[(t * W + c) * 8 + u] = s;
            }
        }
        __syncthreads();

        while (!failed && i < nw && kq + i * KQ < win0 + wn) {
            const int cl = kq + i * KQ;
            const int slot = i % S;
            if (!mbar_wait_bounded(mb0 + 8 * slot, (uint32_t)((i / S) & 1))) {
                failed = true;
                break;
            }
            ChunkRegs<DT> cur;
            load_chunk<DT>(cur, ring + ((size_t)warp * S + slot) * CB, lane);
            __syncwarp();
            if (lane == 0 && i + S < nw) {
                fence_proxy_async();  // this slot's reads happen before the copy that refills it
                bulk_load(ring0 + slot * CB, gsrc + (size_t)(kq + (i + S) * KQ) * CB, CB, mb0 + 8 * slot);
            }
            process_chunk<DT, NT>(cur, acc, tbl + (size_t)(cl - win0) * 128, W * 128, asum + (cl - win0) * 8, W * 8,
                                  m, lane, bact, boff);
            i++;
        }
    }
    if (failed) {
        // Report, then let this warp's copies in flight land before exiting.
        if (lane == 0) {
            *reinterpret_cast<volatile int *>(p.err) = kKernelErrWaitTimeout;
            for (int j = i; j < min(nw, i + S); j++) mbar_wait_bounded(mb0 + 8 * (j % S), (uint32_t)((j / S) & 1));
        }
        __syncwarp();
    }

    // Sum the four column groups of each row (lanes 4r .. 4r+3), then the KQ
    // warps of each tile in a fixed order.
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
                    const float *src = p.partial + (size_t)t * p.n_pad + row;
                    const size_t stride = (size_t)m * p.n_pad;
                    float v = 0.f;
                    int ks = 0;
                    for (; ks + 4 <= p.k_splits; ks += 4) {  // four loads in flight, summed in split order
                        const float a0 = __ldcg(src + (size_t)ks * stride);
                        const float a1 = __ldcg(src + (size_t)(ks + 1) * stride);
                        const float a2 = __ldcg(src + (size_t)(ks + 2) * stride);
                        const float a3 = __ldcg(src + (size_t)(ks + 3) * stride);
                        v += a0;
                        v += a1;
                        v += a2;
                        v += a3;
                    }
                    for (; ks < p.k_splits; ks++) v += __ldcg(src + (size_t)ks * stride);
                    p.y[t * p.ldy + row] = v;
                }
            }
            if (tid == 0) p.counters[blockIdx.x] = 0u;
        }
    }
}

// Opt a kernel in to the device's full shared memory once per device (a
// host-side attribute; not a stream operation).  `done` is the caller's
// per-kernel record of the devices already set.
template <typename Kern>
cudaError_t ensure_smem_optin(Kern kern, std::atomic<unsigned long long> &done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load() & bit)) return cudaSuccess;
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    // dynamic + static shared memory may not exceed the opt-in maximum
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit);
    return e;
}

template <int DT, int NT, int RT>
cudaError_t launch_one(const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
    static std::atomic<unsigned long long> done{0};  // one per instantiation
    auto kern = gemv_kernel<DT, NT, RT>;
    cudaError_t e = ensure_smem_optin(kern, done);
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, smem, s>>>(a);
    return cudaGetLastError();
}

template <int DT, int RT>
cudaError_t launch_nt(int nt, const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
    switch (nt) {
    case 1: return launch_one<DT, 1, RT>(a, grid, smem, s);
    case 2: return launch_one<DT, 2, RT>(a, grid, smem, s);
    case 4: return launch_one<DT, 4, RT>(a, grid, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

template <int DT>
cudaError_t launch_rt(int rt, int nt, const GemvArgs &a, dim3 grid, size_t smem, cudaStream_t s) {
    switch (rt) {
    case 1: return launch_nt<DT, 1>(nt, a, grid, smem, s);
    case 2: return launch_nt<DT, 2>(nt, a, grid, smem, s);
    case 4: return launch_nt<DT, 4>(nt, a, grid, smem, s);
    case 8: return launch_nt<DT, 8>(nt, a, grid, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

GemvPlan plan_gemv(int dt, const Geometry &g, int m, int sm_count) {
    GemvPlan p;
    p.nt = m <= 1 ? 1 : m <= 2 ? 2 : 4;
    // Tiles per CTA: the fewest that keep every CTA resident in one wave (two
    // CTAs per SM).  Split K across CTAs only if the rows leave SMs idle.
    const int wave = 2 * sm_count;
    int rt = 1;
    while (rt < 8 && (g.n_tiles + rt - 1) / rt > wave) rt *= 2;
    p.rt = rt;
    const int kq = 8 / rt;
    const int rows_ctas = (g.n_tiles + rt - 1) / rt;
    int ks = 1;
    if (rows_ctas < sm_count) {
        ks = (sm_count + rows_ctas - 1) / rows_ctas;
        if (ks > 8) ks = 8;
        const int max_ks = g.n_chunks / kq;  // at least one chunk per warp
        if (ks > max_ks) ks = max_ks < 1 ? 1 : max_ks;
    }
    p.cps = (g.n_chunks + ks - 1) / ks;
    p.k_splits = (g.n_chunks + p.cps - 1) / p.cps;
    p.stages = dt == GGUF_Q8_0 ? 2 : (p.nt <= 2 ? 4 : 2);
    int w = 16 / p.nt;
    if (w < kq) w = kq;
    w = (w + kq - 1) / kq * kq;
    if (w > p.cps) w = p.cps;
    p.window = w;
    p.smem = smem_layout(dt, p.nt, m, p.stages, p.window).total;
    if (p.k_splits > 1) {
        p.scratch_floats = (size_t)p.k_splits * m * g.n_tiles * 16;
        p.counters = rows_ctas;
    }
    return p;
}

cudaError_t launch_gemv(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx,
                        float *y, size_t ldy, int m, const GemvPlan &plan, float *scratch,
                        unsigned *counters, int *err, cudaStream_t s) {
    if (m <= 0 || g.n_rows <= 0) return cudaSuccess;
    if (m > plan.nt || m > 4) return cudaErrorInvalidValue;
    GemvArgs a;
    a.w = tiles;
    a.x = x;
    a.y = y;
    a.partial = scratch;
    a.counters = counters;
    a.err = err;
    a.g = g;
    a.ldx = ldx;
    a.ldy = ldy;
    a.m = m;
    a.cps = plan.cps;
    a.k_splits = plan.k_splits;
    a.n_pad = g.n_tiles * 16;
    a.stages = plan.stages;
    a.window = plan.window;
    a.x_vec4 = ((ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
    dim3 grid((g.n_tiles + plan.rt - 1) / plan.rt, plan.k_splits);
    switch (dt) {
    case GGUF_Q4_K: return launch_rt<GGUF_Q4_K>(plan.rt, plan.nt, a, grid, plan.smem, s);
    case GGUF_Q4_0: return launch_rt<GGUF_Q4_0>(plan.rt, plan.nt, a, grid, plan.smem, s);
    case GGUF_Q8_0: return launch_rt<GGUF_Q8_0>(plan.rt, plan.nt, a, grid, plan.smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace rce
