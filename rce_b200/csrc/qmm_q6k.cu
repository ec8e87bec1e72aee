// qmm_q6k.cu -- the Q6_K format: repack (GGUF -> T16), unpack, the
// reference's dequantisation, and the decode GEMV.
//
// Q6_K (rce-ingest-gguf/src/dequant.rs:658-698, rce-op-qmm/src/lib.rs:
// 1667-1705): a super-block of 256 values is 210 bytes -- ql[128] (low four
// bits), qh[64] (high two bits), 16 int8 scales (one per 16 values) and an
// f16 d; value v = 128 o + 32 q + l takes its low bits from ql[64 o + 32 (q &
// 1) + l] (low nibble for q < 2, high nibble above) and its high bits from
// bits 2q, 2q + 1 of qh[32 o + l], and equals (d * sc[v / 16]) * (code - 32).
// The T16 chunk (qmm_layout.cuh) keeps the same bits ordered by value, so a
// lane reads the eight values 8L .. 8L + 7 of a row from one 32-bit and one
// 16-bit word.
//
// GEMV: one CTA per 16-row tile, W warps splitting the tile's chunks
// (chunk c to warp c % W), each warp streaming its chunks through a private
// shared-memory ring filled by TMA bulk copies; lane L takes values 8L .. 8L + 7 of every row of a
// chunk, so its activations are loaded once and used for all 16 rows.  Per
// row and chunk the eight products q' x, q' = 0.5 + u / 256 exact, are summed
// in f32 (two f32x2 chains), turned into sum (u - 32) x with the chunk's
// activation sum, scaled by d * sc once, and added to the lane's
// row sum; a warp then reduces its lanes' sums (halving exchanges: 16
// shuffles per token) and the W warps' sums are added in warp order.  Every
// output is therefore a sum in a fixed order, the same for every batch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "qmm_internal.h"

namespace rce {
namespace {

__device__ __forceinline__ float f16_to_f32(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// The six-bit code (0..63) of value v of a GGUF Q6_K block.
__device__ __forceinline__ int gguf_code(const uint8_t *blk, int v) {
    const int o = v >> 7, q = (v >> 5) & 3, l = v & 31;
    const uint8_t b = blk[64 * o + 32 * (q & 1) + l];
    const int lo = q < 2 ? (b & 0x0F) : (b >> 4);
    const int hi = (blk[128 + 32 * o + l] >> (2 * q)) & 3;
    return lo | (hi << 4);
}

// One thread per (tile, chunk, row of the tile): that row's bytes of the
// chunk (zeros for rows and chunks past the weight).
__global__ void repack_q6k_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst, Geometry g) {
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)g.n_tiles * g.n_chunks * 16;
    if (idx >= total) return;
    const int r = (int)(idx % 16);
    const size_t tc = idx / 16;
    const int64_t tile = (int64_t)(tc / g.n_chunks);
    const int c = (int)(tc % g.n_chunks);
    const int64_t row = tile * 16 + r;
    const int64_t bpr = g.n_cols / 256;
    uint8_t *ch = dst + tc * (size_t)chunk_bytes(GGUF_Q6_K);
    uint8_t lo[128], hi[64], sc[16], d[2];
    const bool live = row < g.n_rows && c < bpr;
    const uint8_t *blk = live ? src + row * g.gguf_row_bytes + (int64_t)c * 210 : nullptr;
    for (int i = 0; i < 64; i++) hi[i] = 0;
    for (int v = 0; v < 256; v += 2) {
        const int u0 = live ? gguf_code(blk, v) : 0, u1 = live ? gguf_code(blk, v + 1) : 0;
        lo[v >> 1] = (uint8_t)((u0 & 15) | ((u1 & 15) << 4));
        hi[v >> 2] |= (uint8_t)(((u0 >> 4) << (2 * (v & 3))) | ((u1 >> 4) << (2 * ((v + 1) & 3))));
    }
    for (int i = 0; i < 16; i++) sc[i] = live ? blk[192 + i] : 0;
    d[0] = live ? blk[208] : 0;
    d[1] = live ? blk[209] : 0;
    for (int i = 0; i < 128; i++) ch[r * 128 + i] = lo[i];
    for (int i = 0; i < 64; i++) ch[kQ6Hi + r * 64 + i] = hi[i];
    for (int i = 0; i < 16; i++) ch[kQ6Sc + r * 16 + i] = sc[i];
    ch[kQ6D + 2 * r] = d[0];
    ch[kQ6D + 2 * r + 1] = d[1];
}

// Code of value v of row r16 in a T16 chunk.
__device__ __forceinline__ int t16_code(const uint8_t *ch, int r16, int v) {
    const int lo = (ch[r16 * 128 + (v >> 1)] >> (4 * (v & 1))) & 15;
    const int hi = (ch[kQ6Hi + r16 * 64 + (v >> 2)] >> (2 * (v & 3))) & 3;
    return lo | (hi << 4);
}

// One thread per GGUF block: its 210 bytes rebuilt from the chunk.
__global__ void unpack_q6k_kernel(const uint8_t *__restrict__ tiles, uint8_t *__restrict__ dst, Geometry g,
                                  int64_t row0, int64_t row1) {
    const int64_t bpr = g.n_cols / 256;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (row1 - row0) * bpr) return;
    const int64_t row = row0 + idx / bpr, blk = idx % bpr;
    const uint8_t *ch = tiles + ((size_t)(row / 16) * g.n_chunks + blk) * chunk_bytes(GGUF_Q6_K);
    const int r16 = (int)(row % 16);
    uint8_t *out = dst + (row - row0) * g.gguf_row_bytes + blk * 210;
    for (int i = 0; i < 192; i++) out[i] = 0;
    for (int v = 0; v < 256; v++) {
        const int u = t16_code(ch, r16, v);
        const int o = v >> 7, q = (v >> 5) & 3, l = v & 31;
        out[64 * o + 32 * (q & 1) + l] |= (uint8_t)((u & 15) << (q < 2 ? 0 : 4));
        out[128 + 32 * o + l] |= (uint8_t)((u >> 4) << (2 * q));
    }
    for (int i = 0; i < 16; i++) out[192 + i] = ch[kQ6Sc + r16 * 16 + i];
    out[208] = ch[kQ6D + 2 * r16];
    out[209] = ch[kQ6D + 2 * r16 + 1];
}

// One thread per GGUF block: dequant_q6_k's arithmetic, (d * sc) * (u - 32)
// with each product rounded on its own.
__global__ void dequant_q6k_kernel(const uint8_t *__restrict__ tiles, float *__restrict__ out, size_t ldo,
                                   Geometry g, int64_t row0, int64_t row1) {
    const int64_t bpr = g.n_cols / 256;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (row1 - row0) * bpr) return;
    const int64_t row = row0 + idx / bpr, blk = idx % bpr;
    const uint8_t *ch = tiles + ((size_t)(row / 16) * g.n_chunks + blk) * chunk_bytes(GGUF_Q6_K);
    const int r16 = (int)(row % 16);
    const float d = f16_to_f32(ch[kQ6D + 2 * r16] | (ch[kQ6D + 2 * r16 + 1] << 8));
    float *o = out + (size_t)(row - row0) * ldo + blk * 256;
    for (int v = 0; v < 256; v++) {
        const float ds = __fmul_rn(d, (float)(int8_t)ch[kQ6Sc + r16 * 16 + (v >> 4)]);
        o[v] = __fmul_rn(ds, (float)(t16_code(ch, r16, v) - 32));
    }
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
    return (unsigned long long)__float_as_uint(lo) | ((unsigned long long)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ unsigned long long u2pack(uint32_t lo, uint32_t hi) {
    return (unsigned long long)lo | ((unsigned long long)hi << 32);
}
__device__ __forceinline__ unsigned long long f2add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2mul(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ float f2lo(unsigned long long v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2hi(unsigned long long v) { return __uint_as_float((uint32_t)(v >> 32)); }

constexpr int kQ6MaxWarps = 16;

struct Q6Args {
    const uint8_t *w;
    const float *x;
    float *y;
    size_t ldx, ldy;
    Geometry g;
    int x_vec4;  // x rows 16-byte aligned: float4 loads
    int stages;  // chunk slots per warp in shared memory
    int *err;    // kernel error word (a bounded wait expired)
};

constexpr unsigned long long kQ6WaitNs = 1000000000ull;

__device__ __forceinline__ uint32_t q6_smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long q6_gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool q6_mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false if the phase did not complete within kQ6WaitNs.
__device__ __forceinline__ bool q6_mbar_wait(uint32_t bar, uint32_t parity) {
    if (q6_mbar_try(bar, parity)) return true;
    const unsigned long long t0 = q6_gtimer();
    while (!q6_mbar_try(bar, parity))
        if (q6_gtimer() - t0 > kQ6WaitNs) return false;
    return true;
}
// One chunk from global memory into a shared-memory slot, completing on bar.
__device__ __forceinline__ void q6_bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Shared memory of a launch: stages chunk slots per warp, then one mbarrier
// per slot.
__host__ __device__ inline size_t q6_smem_bytes(int warps, int stages) {
    return (size_t)warps * stages * (chunk_bytes(GGUF_Q6_K) + 8);
}

// Sum over the lane's eight values of one row of q' * x, q' = 0.5 + u / 256
// (exact: the code byte under the exponent byte of 0.5), in f32x2 pairs
// (values 2p, 2p + 1), the two lanes of the pair chain added at the end.
// The caller recovers sum (u - 32) * x = 256 * sum q' x - 160 * sum x.
// lo: the row's lo-plane word (value e in bits 4e .. 4e + 3), hi: its
// hi-plane half word (value e in bits 2e, 2e + 1).
template <int NT>
__device__ __forceinline__ void row_dot(uint32_t lo, uint32_t hi, const unsigned long long (&xp)[NT][4],
                                        float (&dot)[NT]) {
    // bytes b of ua / ub: the codes of values 2b / 2b + 1
    const uint32_t s = prmt(hi & 0x0F0Fu, (hi >> 4) & 0x0F0Fu, 0x5140u);  // byte b = hi bits of values 2b, 2b+1
    const uint32_t ua = (lo & 0x0F0F0F0Fu) | ((s << 4) & 0x30303030u);
    const uint32_t ub = ((lo >> 4) & 0x0F0F0F0Fu) | ((s << 2) & 0x30303030u);
    unsigned long long acc[NT];
#pragma unroll
    for (int p = 0; p < 4; p++) {
        const uint32_t sel = 0x7054u | ((uint32_t)p << 8);  // bytes: 0, 0, code byte p, 0x3F
        const unsigned long long q = u2pack(prmt(ua, 0x3F000000u, sel), prmt(ub, 0x3F000000u, sel));
#pragma unroll
        for (int t = 0; t < NT; t++) acc[t] = p == 0 ? f2mul(q, xp[t][0]) : f2fma(q, xp[t][p], acc[t]);
    }
#pragma unroll
    for (int t = 0; t < NT; t++) dot[t] = f2lo(acc[t]) + f2hi(acc[t]);
}

template <int NT>
__global__ void __launch_bounds__(kQ6MaxWarps * 32) gemv_q6k_kernel(const Q6Args a) {
    constexpr int CB = chunk_bytes(GGUF_Q6_K);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int tile = blockIdx.x;
    const int nc = a.g.n_chunks;
    const uint8_t *tbase = a.w + (size_t)tile * nc * CB;
    float acc[16][NT];
#pragma unroll
    for (int r = 0; r < 16; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.f;
    // this warp's chunks c = warp, warp + nw, ... stream through its ring of
    // S slots by TMA bulk copies (the weights do not depend on the previous
    // kernel, so the first S are requested before waiting for it)
    extern __shared__ __align__(128) uint8_t q6smem[];
    const int S = a.stages;
    uint8_t *ring = q6smem + (size_t)warp * S * CB;
    const uint32_t bar0 = q6_smem_u32(q6smem + (size_t)nw * S * CB) + 8u * (uint32_t)(warp * S);
    const int nmine = warp < nc ? (nc - warp + nw - 1) / nw : 0;
    if (lane == 0) {
        for (int i = 0; i < S; i++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar0 + 8u * i), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < S && i < nmine; i++)
            q6_bulk_load(q6_smem_u32(ring + (size_t)i * CB), tbase + (size_t)(warp + i * nw) * CB, CB, bar0 + 8u * i);
    }
    __syncwarp();
    // the activations may be the previous kernel's output
    asm volatile("griddepcontrol.wait;" ::: "memory");
    int failed_at = nmine;
    for (int j = 0; j < nmine; j++) {
        const int c = warp + j * nw, slot = j % S;
        if (!q6_mbar_wait(bar0 + 8u * slot, (uint32_t)((j / S) & 1))) {
            failed_at = j;
            break;
        }
        const uint8_t *ch = ring + (size_t)slot * CB;
        unsigned long long xp[NT][4];
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float *xr = a.x + (size_t)t * a.ldx + (size_t)c * 256 + 8 * lane;
            if (a.x_vec4) {
                const float4 x0 = reinterpret_cast<const float4 *>(xr)[0], x1 = reinterpret_cast<const float4 *>(xr)[1];
                xp[t][0] = f2pack(x0.x, x0.y);
                xp[t][1] = f2pack(x0.z, x0.w);
                xp[t][2] = f2pack(x1.x, x1.y);
                xp[t][3] = f2pack(x1.z, x1.w);
            } else {
#pragma unroll
                for (int p = 0; p < 4; p++) xp[t][p] = f2pack(xr[2 * p], xr[2 * p + 1]);
            }
        }
        // -160 * (the lane's eight activations), once per chunk for all rows
        float m160[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const unsigned long long s2 = f2add(f2add(xp[t][0], xp[t][1]), f2add(xp[t][2], xp[t][3]));
            m160[t] = -160.f * (f2lo(s2) + f2hi(s2));
        }
        const uint4 d0 = *reinterpret_cast<const uint4 *>(ch + kQ6D), d1 = *reinterpret_cast<const uint4 *>(ch + kQ6D + 16);
        const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int h = 0; h < 2; h++) {  // rows 8h .. 8h + 7: their words first, then the arithmetic
            uint32_t lo[8], hi[8];
            int sc[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = 8 * h + i;
                lo[i] = *reinterpret_cast<const uint32_t *>(ch + r * 128 + 4 * lane);
                hi[i] = *reinterpret_cast<const uint16_t *>(ch + kQ6Hi + r * 64 + 2 * lane);
                sc[i] = *reinterpret_cast<const int8_t *>(ch + kQ6Sc + r * 16 + (lane >> 1));
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int r = 8 * h + i;
                float dot[NT];
                row_dot<NT>(lo[i], hi[i], xp, dot);
                const float ds = f16_to_f32(dw[r >> 1] >> (16 * (r & 1))) * (float)sc[i];
#pragma unroll
                for (int t = 0; t < NT; t++) acc[r][t] = fmaf(ds, fmaf(256.f, dot[t], m160[t]), acc[r][t]);
            }
        }
        // the slot's reads are done: refill it with chunk j + S
        __syncwarp();
        if (lane == 0 && j + S < nmine) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            q6_bulk_load(q6_smem_u32(ring + (size_t)slot * CB), tbase + (size_t)(c + S * nw) * CB, CB,
                         bar0 + 8u * slot);
        }
    }
    if (failed_at < nmine) {
        // report, then let this warp's copies in flight (numbers failed_at ..
        // min(failed_at + S, nmine) - 1) land before the CTA exits
        if (lane == 0) {
            *reinterpret_cast<volatile int *>(a.err) = kKernelErrWaitTimeout;
            for (int j = failed_at; j < nmine && j < failed_at + S; j++)
                q6_mbar_wait(bar0 + 8u * (j % S), (uint32_t)((j / S) & 1));
        }
        __syncwarp();
    }
    // warp reduction by halving exchanges: after step k (offsets 16, 8, 4,
    // 2) a lane keeps 16 >> (k + 1) rows -- those whose index has the lane's
    // bits -- summed over 2^(k + 1) lanes; the last step (offset 1) completes
    // one row per lane pair.
    float red[NT];
    {
        float v8[8][NT], v4[4][NT], v2[2][NT];
        const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4, b2 = lane & 2;
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float keep = b16 ? acc[8 + i][t] : acc[i][t], send = b16 ? acc[i][t] : acc[8 + i][t];
                v8[i][t] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
            }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float keep = b8 ? v8[4 + i][t] : v8[i][t], send = b8 ? v8[i][t] : v8[4 + i][t];
                v4[i][t] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float keep = b4 ? v4[2 + i][t] : v4[i][t], send = b4 ? v4[i][t] : v4[2 + i][t];
                v2[i][t] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float keep = b2 ? v2[1][t] : v2[0][t], send = b2 ? v2[0][t] : v2[1][t];
            red[t] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
            red[t] += __shfl_xor_sync(0xffffffffu, red[t], 1);
        }
    }
    // lane's row: bit 3 from lane bit 4, bit 2 from bit 3, bit 1 from bit 2, bit 0 from bit 1
    const int row16 = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
    __shared__ float part[kQ6MaxWarps][16][2];
    if ((lane & 1) == 0)
#pragma unroll
        for (int t = 0; t < NT; t++) part[warp][row16][t] = red[t];
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x < 16 * NT) {
        const int r = threadIdx.x % 16, t = threadIdx.x / 16;
        float s = 0.f;
        for (int w = 0; w < nw; w++) s += part[w][r][t];
        const int64_t row = (int64_t)tile * 16 + r;
        if (row < a.g.n_rows) a.y[(size_t)t * a.ldy + row] = s;
    }
}

}  // namespace

cudaError_t launch_repack_q6k(const uint8_t *gguf, uint8_t *tiles, const Geometry &g, cudaStream_t s) {
    const size_t total = (size_t)g.n_tiles * g.n_chunks * 16;
    if (total == 0) return cudaSuccess;
    repack_q6k_kernel<<<(unsigned)((total + 127) / 128), 128, 0, s>>>(gguf, tiles, g);
    return cudaGetLastError();
}

cudaError_t launch_unpack_q6k(const uint8_t *tiles, uint8_t *gguf, const Geometry &g, int64_t row0, int64_t row1,
                              cudaStream_t s) {
    const int64_t n = (row1 - row0) * (g.n_cols / 256);
    if (n <= 0) return cudaSuccess;
    unpack_q6k_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(tiles, gguf, g, row0, row1);
    return cudaGetLastError();
}

cudaError_t launch_dequant_q6k(const uint8_t *tiles, float *out, size_t ldo, const Geometry &g, int64_t row0,
                               int64_t row1, cudaStream_t s) {
    const int64_t n = (row1 - row0) * (g.n_cols / 256);
    if (n <= 0) return cudaSuccess;
    dequant_q6k_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(tiles, out, ldo, g, row0, row1);
    return cudaGetLastError();
}

int q6k_gemv_warps(const Geometry &g, int sm_count) {
    // about two waves of 20 resident warps per SM, in warps per tile that
    // divide the work evenly where they can (powers of two), at most one
    // chunk per warp
    const long target = 2L * 20 * sm_count;
    int w = 1;
    while (w < kQ6MaxWarps && (long)w * g.n_tiles < target && w < g.n_chunks) w *= 2;
    return w;
}

cudaError_t launch_gemv_q6k(const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx, float *y,
                            size_t ldy, int m, int sm_count, int *err, cudaStream_t s) {
    if (m <= 0 || g.n_tiles == 0) return cudaSuccess;
    if (m > kQ6MaxTokens) return cudaErrorInvalidValue;
    const int warps = q6k_gemv_warps(g, sm_count);
    // slots per warp: up to four, within ~110 KB per CTA (two CTAs per SM)
    const int per_warp = (int)((g.n_chunks + warps - 1) / warps);
    int stages = (int)((110 * 1024) / ((size_t)warps * (chunk_bytes(GGUF_Q6_K) + 8)));
    if (stages > 4) stages = 4;
    if (stages > per_warp) stages = per_warp;
    if (stages < 1) stages = 1;
    const size_t smem = q6_smem_bytes(warps, stages);
    {
        static std::atomic<unsigned long long> done{0};
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
        if (!bit || !(done.load() & bit)) {
            e = cudaFuncSetAttribute(gemv_q6k_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(gemv_q6k_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            if (e != cudaSuccess) return e;
            if (bit) done.fetch_or(bit);
        }
    }
    Q6Args a;
    a.stages = stages;
    a.err = err;
    a.x_vec4 = !(reinterpret_cast<uintptr_t>(x) & 15) && (m == 1 || !(ldx & 3));
    a.w = tiles;
    a.x = x;
    a.y = y;
    a.ldx = ldx;
    a.ldy = ldy;
    a.g = g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)g.n_tiles, 1, 1);
    cfg.blockDim = dim3((unsigned)(32 * warps), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return m == 1 ? cudaLaunchKernelEx(&cfg, gemv_q6k_kernel<1>, a) : cudaLaunchKernelEx(&cfg, gemv_q6k_kernel<2>, a);
}

}  // namespace rce
