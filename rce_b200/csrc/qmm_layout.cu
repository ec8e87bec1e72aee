// qmm_layout.cu -- repack (GGUF -> T16), unpack (T16 -> GGUF) and the
// bit-exact dequantisation kernels.  The T16 layout is described in
// qmm_layout.cuh.  These run once per weight (repack) or on demand
// (dequant_row, read-back), so they favour simplicity over speed.
#include <cuda_fp16.h>

#include "qmm_internal.h"

namespace rce {
namespace {

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// The (sc, m) pair of sub-block j from GGUF's 12 packed scale bytes:
// q4_k_get_scale_min (rce-op-qmm/src/lib.rs:720-728).
__device__ __forceinline__ void q4k_scale_min(const uint8_t *s, int j, int &sc, int &m) {
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// One thread per 16-byte piece of the T16 output.
template <int DT>
__global__ void repack_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                              Geometry g) {
    constexpr int PPC = chunk_bytes(DT) / 16;
    constexpr int QP = quant_bytes(DT) / 16;
    const size_t total = (size_t)g.n_tiles * g.n_chunks * PPC;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const size_t tc = idx / PPC;
    const int p = (int)(idx % PPC);
    const int64_t tile = (int64_t)(tc / g.n_chunks);
    const int c = (int)(tc % g.n_chunks);
    const int64_t blocks_per_row = g.n_cols / gguf_block(DT);
    uint8_t buf[16];
#pragma unroll
    for (int b = 0; b < 16; b++) buf[b] = 0;
    if (p < QP) {
        const int i = p / 32, lane = p % 32, r = lane >> 2, gq = lane & 3;
        int64_t row;
        int64_t blk;
        int off;
        if (kquant45(DT)) {
            row = tile * 16 + r + 8 * (i >> 1);
            blk = c;
            off = (DT == GGUF_Q5_K ? 48 : 16) + 32 * gq + 16 * (i & 1);
        } else if (DT == GGUF_Q4_0) {
            row = tile * 16 + r + 8 * (i >> 1);
            blk = (int64_t)c * 8 + 2 * gq + (i & 1);
            off = 2;
        } else {
            row = tile * 16 + r + 8 * (i >> 2);
            blk = (int64_t)c * 8 + 2 * gq + ((i >> 1) & 1);
            off = 2 + 16 * (i & 1);
        }
        if (row < g.n_rows && blk < blocks_per_row) {
            const uint8_t *s = src + row * g.gguf_row_bytes + blk * gguf_block_bytes(DT) + off;
#pragma unroll
            for (int b = 0; b < 16; b++) buf[b] = s[b];
        }
    } else if (DT == GGUF_Q5_K && p >= QP + 16) {
        // fifth bits of lane (r, gq): Y0, Y1 of row r, then of row r + 8
        const int lane = p - QP - 16, r = lane >> 2, gq = lane & 3;
#pragma unroll
        for (int rr = 0; rr < 2; rr++) {
            const int64_t row = tile * 16 + r + 8 * rr;
            if (row >= g.n_rows || c >= blocks_per_row) continue;
            const uint8_t *qh = src + row * g.gguf_row_bytes + (int64_t)c * 176 + 16;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                uint32_t y = 0;
                for (int l = 0; l < 32; l++) y |= (uint32_t)((qh[l] >> (2 * gq + h)) & 1) << (8 * (l & 3) + (l >> 2));
                buf[8 * rr + 4 * h] = (uint8_t)y;
                buf[8 * rr + 4 * h + 1] = (uint8_t)(y >> 8);
                buf[8 * rr + 4 * h + 2] = (uint8_t)(y >> 16);
                buf[8 * rr + 4 * h + 3] = (uint8_t)(y >> 24);
            }
        }
    } else {
        const int q = p - QP;  // 0..15
        if (kquant45(DT)) {
            const int64_t row = tile * 16 + q;
            if (row < g.n_rows && c < blocks_per_row) {
                const uint8_t *h = src + row * g.gguf_row_bytes + (int64_t)c * gguf_block_bytes(DT);
                buf[0] = h[0];
                buf[1] = h[1];
                buf[2] = h[2];
                buf[3] = h[3];
#pragma unroll
                for (int gq = 0; gq < 4; gq++) {
                    int sc1, m1, sc2, m2;
                    q4k_scale_min(h + 4, 2 * gq, sc1, m1);
                    q4k_scale_min(h + 4, 2 * gq + 1, sc2, m2);
                    const uint32_t v = (uint32_t)sc1 | ((uint32_t)m1 << 6) | ((uint32_t)sc2 << 12) |
                                       ((uint32_t)m2 << 18);
                    buf[4 + 3 * gq] = (uint8_t)(v & 0xFF);
                    buf[5 + 3 * gq] = (uint8_t)((v >> 8) & 0xFF);
                    buf[6 + 3 * gq] = (uint8_t)((v >> 16) & 0xFF);
                }
            }
        } else {
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int lane = 2 * q + half, r = lane >> 2, gq = lane & 3;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int64_t row = tile * 16 + r + 8 * (e >> 1);
                    const int64_t blk = (int64_t)c * 8 + 2 * gq + (e & 1);
                    if (row < g.n_rows && blk < blocks_per_row) {
                        const uint8_t *s = src + row * g.gguf_row_bytes + blk * gguf_block_bytes(DT);
                        buf[8 * half + 2 * e] = s[0];
                        buf[8 * half + 2 * e + 1] = s[1];
                    }
                }
            }
        }
    }
    uint4 v;
    v.x = buf[0] | (buf[1] << 8) | (buf[2] << 16) | ((uint32_t)buf[3] << 24);
    v.y = buf[4] | (buf[5] << 8) | (buf[6] << 16) | ((uint32_t)buf[7] << 24);
    v.z = buf[8] | (buf[9] << 8) | (buf[10] << 16) | ((uint32_t)buf[11] << 24);
    v.w = buf[12] | (buf[13] << 8) | (buf[14] << 16) | ((uint32_t)buf[15] << 24);
    reinterpret_cast<uint4 *>(dst)[idx] = v;
}

// Location of GGUF block `blk` of row `row` inside the T16 tiles.
struct BlockLoc {
    const uint8_t *chunk;
    int r16, gq, hb, lane;
};

template <int DT>
__device__ __forceinline__ BlockLoc locate(const uint8_t *tiles, const Geometry &g, int64_t row,
                                           int64_t blk) {
    BlockLoc L;
    const int64_t tile = row / 16;
    L.r16 = (int)(row % 16);
    const int64_t c = kquant45(DT) ? blk : blk / 8;
    const int bl = kquant45(DT) ? 0 : (int)(blk % 8);
    L.gq = bl / 2;
    L.hb = bl % 2;
    L.lane = 4 * (L.r16 % 8) + L.gq;
    L.chunk = tiles + ((size_t)tile * g.n_chunks + c) * chunk_bytes(DT);
    return L;
}

// One thread per GGUF block: rebuild its bytes from the tiles.
template <int DT>
__global__ void unpack_kernel(const uint8_t *__restrict__ tiles, uint8_t *__restrict__ dst,
                              Geometry g, int64_t row0, int64_t row1) {
    const int64_t bpr = g.n_cols / gguf_block(DT);
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (row1 - row0) * bpr) return;
    const int64_t row = row0 + idx / bpr, blk = idx % bpr;
    uint8_t *out = dst + (row - row0) * g.gguf_row_bytes + blk * gguf_block_bytes(DT);
    if (kquant45(DT)) {
        BlockLoc L = locate<DT>(tiles, g, row, blk);
        const int qs0 = DT == GGUF_Q5_K ? 48 : 16;
        const uint8_t *h = L.chunk + 2048 + L.r16 * 16;
        out[0] = h[0];
        out[1] = h[1];
        out[2] = h[2];
        out[3] = h[3];
        int sc[8], mn[8];
        for (int gq = 0; gq < 4; gq++) {
            const uint32_t v = h[4 + 3 * gq] | (h[5 + 3 * gq] << 8) | ((uint32_t)h[6 + 3 * gq] << 16);
            sc[2 * gq] = v & 63;
            mn[2 * gq] = (v >> 6) & 63;
            sc[2 * gq + 1] = (v >> 12) & 63;
            mn[2 * gq + 1] = (v >> 18) & 63;
        }
        // GGUF's packing (the inverse of q4_k_get_scale_min; the reference's
        // pack_scales, rce-vm-backend-cpu/src/ml/kquant.rs:284-292).
        for (int j = 0; j < 4; j++) {
            out[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            out[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
            out[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
        }
        const int rh = L.r16 >= 8 ? 1 : 0;
        for (int gq = 0; gq < 4; gq++)
            for (int hh = 0; hh < 2; hh++) {
                const int i = 2 * rh + hh, lane = 4 * (L.r16 % 8) + gq;
                const uint8_t *q = L.chunk + (i * 32 + lane) * 16;
                for (int b = 0; b < 16; b++) out[qs0 + 32 * gq + 16 * hh + b] = q[b];
            }
        if (DT == GGUF_Q5_K) {  // qh[l] bit 2 gq + h from word Y_h of lane (r, gq)
            for (int l = 0; l < 32; l++) out[16 + l] = 0;
            for (int gq = 0; gq < 4; gq++) {
                const uint8_t *yw = L.chunk + kQ5Hi + (4 * (L.r16 % 8) + gq) * 16 + 8 * rh;
                for (int h = 0; h < 2; h++) {
                    const uint32_t y = yw[4 * h] | (yw[4 * h + 1] << 8) | (yw[4 * h + 2] << 16) |
                                       ((uint32_t)yw[4 * h + 3] << 24);
                    for (int l = 0; l < 32; l++)
                        out[16 + l] |= (uint8_t)(((y >> (8 * (l & 3) + (l >> 2))) & 1) << (2 * gq + h));
                }
            }
        }
    } else {
        BlockLoc L = locate<DT>(tiles, g, row, blk);
        const int rh = L.r16 >= 8 ? 1 : 0;
        const uint8_t *sc = L.chunk + quant_bytes(DT) + L.lane * 8 + (2 * rh + L.hb) * 2;
        out[0] = sc[0];
        out[1] = sc[1];
        if (DT == GGUF_Q4_0) {
            const uint8_t *q = L.chunk + ((2 * rh + L.hb) * 32 + L.lane) * 16;
            for (int b = 0; b < 16; b++) out[2 + b] = q[b];
        } else {
            for (int half = 0; half < 2; half++) {
                const int i = 4 * rh + 2 * L.hb + half;
                const uint8_t *q = L.chunk + (i * 32 + L.lane) * 16;
                for (int b = 0; b < 16; b++) out[2 + 16 * half + b] = q[b];
            }
        }
    }
}

// One thread per GGUF block: the reference's dequant arithmetic
// (rce-ingest-gguf/src/dequant.rs:360-383 Q4_0, :438-456 Q8_0, :546-591
// Q4_K).  __fmul_rn/__fsub_rn keep each product and difference a separate
// rounding, as in the reference (no FMA contraction).
template <int DT>
__global__ void dequant_kernel(const uint8_t *__restrict__ tiles, float *__restrict__ out,
                               size_t ldo, Geometry g, int64_t row0, int64_t row1) {
    const int64_t bpr = g.n_cols / gguf_block(DT);
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (row1 - row0) * bpr) return;
    const int64_t row = row0 + idx / bpr, blk = idx % bpr;
    float *o = out + (size_t)(row - row0) * ldo + blk * gguf_block(DT);
    BlockLoc L = locate<DT>(tiles, g, row, blk);
    const int rh = L.r16 >= 8 ? 1 : 0;
    if (kquant45(DT)) {
        const uint8_t *h = L.chunk + 2048 + L.r16 * 16;
        const float d = f16_bits_to_f32((uint16_t)(h[0] | (h[1] << 8)));
        const float dmin = f16_bits_to_f32((uint16_t)(h[2] | (h[3] << 8)));
        for (int gq = 0; gq < 4; gq++) {
            const uint32_t v = h[4 + 3 * gq] | (h[5 + 3 * gq] << 8) | ((uint32_t)h[6 + 3 * gq] << 16);
            const float d1 = __fmul_rn(d, (float)(v & 63));
            const float min1 = __fmul_rn(dmin, (float)((v >> 6) & 63));
            const float d2 = __fmul_rn(d, (float)((v >> 12) & 63));
            const float min2 = __fmul_rn(dmin, (float)((v >> 18) & 63));
            const int lane = 4 * (L.r16 % 8) + gq;
            uint32_t y0 = 0, y1 = 0;  // Q5_K fifth bits of sub-blocks 2 gq, 2 gq + 1
            if (DT == GGUF_Q5_K) {
                const uint8_t *yw = L.chunk + kQ5Hi + lane * 16 + 8 * rh;
                y0 = yw[0] | (yw[1] << 8) | (yw[2] << 16) | ((uint32_t)yw[3] << 24);
                y1 = yw[4] | (yw[5] << 8) | (yw[6] << 16) | ((uint32_t)yw[7] << 24);
            }
            for (int hh = 0; hh < 2; hh++) {
                const uint8_t *q = L.chunk + ((2 * rh + hh) * 32 + lane) * 16;
                for (int b = 0; b < 16; b++) {
                    const int l = 16 * hh + b, bit = 8 * (l & 3) + (l >> 2);
                    const uint32_t c0 = (q[b] & 0x0F) | (((y0 >> bit) & 1) << 4);
                    const uint32_t c1 = (q[b] >> 4) | (((y1 >> bit) & 1) << 4);
                    o[64 * gq + l] = __fsub_rn(__fmul_rn(d1, (float)c0), min1);
                    o[64 * gq + 32 + l] = __fsub_rn(__fmul_rn(d2, (float)c1), min2);
                }
            }
        }
    } else {
        const uint8_t *sc = L.chunk + quant_bytes(DT) + L.lane * 8 + (2 * rh + L.hb) * 2;
        const float d = f16_bits_to_f32((uint16_t)(sc[0] | (sc[1] << 8)));
        if (DT == GGUF_Q4_0) {
            const uint8_t *q = L.chunk + ((2 * rh + L.hb) * 32 + L.lane) * 16;
            for (int b = 0; b < 16; b++) {
                o[b] = __fmul_rn((float)((int)(q[b] & 0x0F) - 8), d);
                o[b + 16] = __fmul_rn((float)((int)(q[b] >> 4) - 8), d);
            }
        } else {
            for (int half = 0; half < 2; half++) {
                const int i = 4 * rh + 2 * L.hb + half;
                const uint8_t *q = L.chunk + (i * 32 + L.lane) * 16;
                for (int b = 0; b < 16; b++) o[16 * half + b] = __fmul_rn((float)(int8_t)q[b], d);
            }
        }
    }
}

}  // namespace

cudaError_t launch_repack(int dt, const uint8_t *gguf, uint8_t *tiles, const Geometry &g,
                          cudaStream_t s) {
    const size_t total = g.dev_bytes / 16;
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    switch (dt) {
    case GGUF_Q6_K: return launch_repack_q6k(gguf, tiles, g, s);
    case GGUF_Q4_K: repack_kernel<GGUF_Q4_K><<<blocks, threads, 0, s>>>(gguf, tiles, g); break;
    case GGUF_Q5_K: repack_kernel<GGUF_Q5_K><<<blocks, threads, 0, s>>>(gguf, tiles, g); break;
    case GGUF_Q4_0: repack_kernel<GGUF_Q4_0><<<blocks, threads, 0, s>>>(gguf, tiles, g); break;
    case GGUF_Q8_0: repack_kernel<GGUF_Q8_0><<<blocks, threads, 0, s>>>(gguf, tiles, g); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_unpack(int dt, const uint8_t *tiles, uint8_t *gguf, const Geometry &g,
                          int64_t row0, int64_t row1, cudaStream_t s) {
    const int64_t n = (row1 - row0) * (g.n_cols / gguf_block(dt));
    if (n <= 0) return cudaSuccess;
    const int threads = 128;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    switch (dt) {
    case GGUF_Q6_K: return launch_unpack_q6k(tiles, gguf, g, row0, row1, s);
    case GGUF_Q4_K: unpack_kernel<GGUF_Q4_K><<<blocks, threads, 0, s>>>(tiles, gguf, g, row0, row1); break;
    case GGUF_Q5_K: unpack_kernel<GGUF_Q5_K><<<blocks, threads, 0, s>>>(tiles, gguf, g, row0, row1); break;
    case GGUF_Q4_0: unpack_kernel<GGUF_Q4_0><<<blocks, threads, 0, s>>>(tiles, gguf, g, row0, row1); break;
    case GGUF_Q8_0: unpack_kernel<GGUF_Q8_0><<<blocks, threads, 0, s>>>(tiles, gguf, g, row0, row1); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant(int dt, const uint8_t *tiles, float *out, size_t ldo, const Geometry &g,
                           int64_t row0, int64_t row1, cudaStream_t s) {
    const int64_t n = (row1 - row0) * (g.n_cols / gguf_block(dt));
    if (n <= 0) return cudaSuccess;
    const int threads = 128;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    switch (dt) {
    case GGUF_Q6_K: return launch_dequant_q6k(tiles, out, ldo, g, row0, row1, s);
    case GGUF_Q4_K: dequant_kernel<GGUF_Q4_K><<<blocks, threads, 0, s>>>(tiles, out, ldo, g, row0, row1); break;
    case GGUF_Q5_K: dequant_kernel<GGUF_Q5_K><<<blocks, threads, 0, s>>>(tiles, out, ldo, g, row0, row1); break;
    case GGUF_Q4_0: dequant_kernel<GGUF_Q4_0><<<blocks, threads, 0, s>>>(tiles, out, ldo, g, row0, row1); break;
    case GGUF_Q8_0: dequant_kernel<GGUF_Q8_0><<<blocks, threads, 0, s>>>(tiles, out, ldo, g, row0, row1); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace rce
