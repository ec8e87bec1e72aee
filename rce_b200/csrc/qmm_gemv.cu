// qmm_gemv.cu -- decode GEMV / small-M matmul over T16 weight tiles.
//
// y[t][row] = sum_k x[t][k] * W[row][k], the arithmetic of the reference's
// mm_1d (rce-op-qmm/src/lib.rs:496-522 Q4_0, :648-670 Q8_0, :730-781 Q4_K)
// up to f32 summation order.
//
// Design (HBM-bound; every weight byte is read once):
//  * Work split: clusters of two CTAs (one CTA of 16 warps per SM).  Cluster
//    c owns a block of whole 16-row tiles, so no sum leaves the cluster; the
//    block's units (tile x 256-column chunk) are cut into 32 equal runs of
//    consecutive units, one per warp, so every warp of the grid streams the
//    same number of chunks (see "Work split" below).
//  * Each warp's lane 0 streams its chunks into a private shared-memory ring
//    with TMA bulk copies (cp.async.bulk + mbarrier complete_tx), S chunks
//    ahead.  Every wait on an mbarrier is bounded (%globaltimer); on expiry
//    the kernel records an error word, waits (bounded) for its own copies
//    and finishes.
//  * The dot products are exact integer arithmetic on the tensor cores
//    (mma.sync m16n8k32, u8/s8 x s8 -> s32).  The weight codes are the A
//    operand as they are stored: Q8_0's int8 bytes need no unpacking at all,
//    Q4_K/Q4_0 nibbles one mask per 4 codes.  Activations become a
//    fixed-point integer per token and chunk, X = x * 2^e rounded to 31 bits
//    with the power of two chosen from the chunk's maximum, whose four
//    balanced base-256 digits are simply the bytes of (X + 0x80808080) ^
//    0x80808080; the B operand is block-diagonal so that lane g's columns
//    hold digits of its own column group.  Sub-block sums are exact in s32;
//    Q4_K keeps them integer through the whole super-block (sc and m are
//    integers) and meets d and dmin once per chunk in f64; sums across
//    chunks run in f64 and are rounded to f32 once per segment, so x keeps
//    2^-30 of its chunk maximum and the weights are never rounded.
//  * Q4_K's min term and Q4_0's -8 offset use per-sub-block sums of the
//    integer activations (one product per sub-block).
//  * The activation table (the B fragments) covers the CTA's window of
//    chunks; its loads are issued before most of the weight prefetch.
//  * Launched with programmatic stream serialization: a kernel's CTAs start
//    while the previous kernel on the stream drains, issue their first
//    weight copies (which depend on nothing), and only then wait for the
//    previous grid (griddepcontrol.wait) before touching the activations or
//    writing outputs.  Each CTA signals its dependents once its main loop is
//    done.
// The plan depends on the weight's shape only, never on the batch, so each
// token's result is bit-identical whatever the batch size.
#include <cuda_fp16.h>

#include <atomic>

#include "qmm_gather.cuh"
#include "qmm_internal.h"

namespace rce {
namespace {

constexpr int kMaxStages = 4;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s per wait

// x / d for 0 <= x < 2^31 as a multiply and a shift (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994,
// Theorem 4.2 with N = 31: m = ceil(2^(31+l) / d), l = ceil(log2 d)).
struct FastDiv {
    uint32_t m = 1u << 31, s = 31;  // d = 1
};
__host__ inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f;
    if (d <= 1) return f;
    uint32_t l = 0;
    while ((1ull << l) < d) l++;
    f.m = (uint32_t)(((1ull << (31 + l)) + d - 1) / d);
    f.s = 31 + l;
    return f;
}
__host__ __device__ __forceinline__ uint32_t udiv(uint32_t x, const FastDiv &f) {
    return (uint32_t)(((uint64_t)x * f.m) >> f.s);
}

// Up to kGemvMaxGroup weights with the same dtype and K, read by one launch:
// their tiles are numbered one after the other (weight i's tiles start at
// tile0[i]) and split over the grid as one matrix.
struct GemvArgs {
    const uint8_t *w[kGemvMaxGroup];
    float *y[kGemvMaxGroup];
    size_t ldy[kGemvMaxGroup];
    int64_t n_rows[kGemvMaxGroup];
    int tile0[kGemvMaxGroup];
    int n_w;
    const float *x;
    int *err;
    Geometry g;  // n_tiles: all weights' tiles; n_chunks, n_cols: shared
    size_t ldx;
    int m, stages, pre, x_vec4;
    int n_clusters;  // clusters of kClusterCtas CTAs; cluster c owns a block of whole tiles
    int panels;      // 1 or 2 (the work split)
    int tiles_base, tiles_extra;   // clusters c < tiles_extra hold tiles_base + 1 tiles
    FastDiv fd_pw0, fd_pw1, fd_u[2];  // division by the run lengths and by the units of a cluster (base, base + 1)
    int win, kmax;   // shared-memory maxima: table chunks, slots per warp
    GatherArgs ga[kGemvMaxGroup];  // fused all-gather over peer memory (ga[0].world > 1), per weight
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

// Expect `bytes` of transactions on `bar` and copy `bytes` from global `src`
// into shared `dst`; the copy's completion completes the transactions.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// bulk_load preceded by fence_proxy_async, by the lanes with `pred` only
// (predicated, not a branch).
__device__ __forceinline__ void bulk_refill(bool pred, uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %4, 0;\n\t"
        "@p fence.proxy.async.shared::cta;\n\t"
        "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%3], %2;\n\t"
        "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n\t}" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "r"((uint32_t)pred)
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

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// D(s32) += A(16x32, u8 or s8) x B(32x8, s8), exact; ZERO: D = A x B.
template <bool A_SIGNED, bool ZERO = false>
__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if (ZERO) {
        if (A_SIGNED)
            asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%10,%10,%10,%10};"
                : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
        else
            asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%10,%10,%10,%10};"
                : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
    } else {
        if (A_SIGNED)
            asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
        else
            asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ uint32_t comp(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// One output value: to y, and with the fused all-gather also to every other
// rank's receive buffer (at this rank's rows of the full output).
// The weight of global tile `tile`.
__device__ __forceinline__ int group_of(const GemvArgs &p, int tile) {
    int wi = 0;
#pragma unroll
    for (int i = 1; i < kGemvMaxGroup; i++) wi += (i < p.n_w && tile >= p.tile0[i]) ? 1 : 0;
    return wi;
}

// Chunk `chunk` of global tile `tile`.
__device__ __forceinline__ const uint8_t *tile_src(const GemvArgs &p, int tile, int chunk, int cb) {
    const int wi = group_of(p, tile);
    return p.w[wi] + ((size_t)(tile - p.tile0[wi]) * p.g.n_chunks + chunk) * cb;
}

// Output row r (0..15) of global tile `tile`, token t (< m): into its
// weight's y, and to the peers when the output is gathered (one weight).
__device__ __forceinline__ void put_y(const GemvArgs &p, int t, int tile, int r, float v, unsigned epoch) {
    const int wi = group_of(p, tile);
    const int64_t row = (int64_t)(tile - p.tile0[wi]) * 16 + r;
    if (row >= p.n_rows[wi]) return;
    p.y[wi][t * p.ldy[wi] + row] = v;
    if (p.ga[0].world > 1)
        gather_send(p.ga[wi], (size_t)t * p.ldy[wi] + (size_t)p.ga[wi].row_off + (size_t)row, v, epoch);
}

template <int DT>
struct Fmt {
    static constexpr int NQ = DT == GGUF_Q8_0 ? 8 : 4;  // 16-byte quant pieces per lane per chunk
};

template <int DT>
struct ChunkRegs {
    uint4 q[Fmt<DT>::NQ];
    uint4 h0, h1;  // Q4_K/Q5_K: headers of rows r and r+8; Q4_0/Q8_0: h0.xy = the lane's 4 scales
    uint4 y;       // Q5_K: fifth bits, words Y0, Y1 of row r, Y0, Y1 of row r + 8
};

// One chunk's lane data from its shared-memory ring slot (conflict-free:
// lanes read consecutive 16-byte pieces).
// Q4_K: h0/h1 = {d | dmin << 16, the two header words holding lane group
// g's 24 bits of (sc, m) fields} of rows r and r + 8; `hw` is the byte
// offset of the first of those words within a row's 16-byte header
// (4 + 4 * (3g / 4)).  For g = 3 the second word lies past the row's header
// (the next row's, or the bytes after the chunk) and is never used.
template <int DT>
__device__ __forceinline__ void load_chunk(ChunkRegs<DT> &c, const uint8_t *slot, int lane, int hw) {
#pragma unroll
    for (int i = 0; i < Fmt<DT>::NQ; i++) c.q[i] = *reinterpret_cast<const uint4 *>(slot + (i * 32 + lane) * 16);
    if (DT == GGUF_Q5_K) c.y = *reinterpret_cast<const uint4 *>(slot + kQ5Hi + lane * 16);
    if (kquant45(DT)) {
        const uint8_t *h0 = slot + 2048 + (lane >> 2) * 16, *h1 = h0 + 8 * 16;
        c.h0 = make_uint4(*reinterpret_cast<const uint32_t *>(h0), *reinterpret_cast<const uint32_t *>(h0 + hw),
                          *reinterpret_cast<const uint32_t *>(h0 + hw + 4), 0u);
        c.h1 = make_uint4(*reinterpret_cast<const uint32_t *>(h1), *reinterpret_cast<const uint32_t *>(h1 + hw),
                          *reinterpret_cast<const uint32_t *>(h1 + hw + 4), 0u);
    } else {
        const uint2 s = *reinterpret_cast<const uint2 *>(slot + quant_bytes(DT) + lane * 8);
        c.h0 = make_uint4(s.x, s.y, 0u, 0u);
        c.h1 = c.h0;
    }
}

// The A operand of step s (0..7) for rows r (a0: columns 64g + 8s + 0..3,
// a2: + 4..7) and r + 8 (a1, a3): the stored codes, one byte per value.
// Sub-block (unit) 2g + (s >> 2); see qmm_layout.cuh for where the bytes sit.
template <int DT>
__device__ __forceinline__ void make_a(const ChunkRegs<DT> &c, int s, uint32_t (&a)[4]) {
    const int h = s >> 2, ss = s & 3;
    if (DT == GGUF_Q5_K) {
        // the low (h = 0) or high (h = 1) nibbles as bytes, plus the fifth
        // bit at bit 4: bit 8b + j of Y_h (j = 2 ss for a[0]/a[1], 2 ss + 1
        // for a[2]/a[3]) moved to bit 8b + 4
        const uint32_t r0 = comp(c.q[ss >> 1], (2 * ss) & 3), r1 = comp(c.q[ss >> 1], (2 * ss + 1) & 3);
        const uint32_t e0 = comp(c.q[2 + (ss >> 1)], (2 * ss) & 3), e1 = comp(c.q[2 + (ss >> 1)], (2 * ss + 1) & 3);
        const uint32_t yr = h ? c.y.y : c.y.x, ye = h ? c.y.w : c.y.z;
        const int j0 = 2 * ss, j1 = 2 * ss + 1;
        auto fifth = [](uint32_t y, int j) { return (j <= 4 ? y << (4 - j) : y >> (j - 4)) & 0x10101010u; };
        const int sh = 4 * h;
        a[0] = ((r0 >> sh) & 0x0F0F0F0Fu) | fifth(yr, j0);
        a[2] = ((r1 >> sh) & 0x0F0F0F0Fu) | fifth(yr, j1);
        a[1] = ((e0 >> sh) & 0x0F0F0F0Fu) | fifth(ye, j0);
        a[3] = ((e1 >> sh) & 0x0F0F0F0Fu) | fifth(ye, j1);
    } else if (DT == GGUF_Q4_K) {
        // group g's 32 qs bytes per row: words 2ss, 2ss+1; low nibbles are
        // sub-block 2g, high nibbles sub-block 2g+1
        const uint32_t r0 = comp(c.q[ss >> 1], (2 * ss) & 3), r1 = comp(c.q[ss >> 1], (2 * ss + 1) & 3);
        const uint32_t e0 = comp(c.q[2 + (ss >> 1)], (2 * ss) & 3), e1 = comp(c.q[2 + (ss >> 1)], (2 * ss + 1) & 3);
        // (sub-block 2g+1 as 16 * code, unshifted: its sums are divided by 16
        // after the chain, exactly)
        const uint32_t mk = h == 0 ? 0x0F0F0F0Fu : 0xF0F0F0F0u;
        a[0] = r0 & mk;
        a[2] = r1 & mk;
        a[1] = e0 & mk;
        a[3] = e1 & mk;
    } else if (DT == GGUF_Q4_0) {
        // block 2g + h: bytes 0..15; low nibbles are values 0..15, high 16..31
        const int wp = (ss & 1) * 2, sh = 4 * (ss >> 1);
        const uint32_t r0 = comp(c.q[h], wp), r1 = comp(c.q[h], wp + 1);
        const uint32_t e0 = comp(c.q[2 + h], wp), e1 = comp(c.q[2 + h], wp + 1);
        a[0] = (r0 >> sh) & 0x0F0F0F0Fu;
        a[2] = (r1 >> sh) & 0x0F0F0F0Fu;
        a[1] = (e0 >> sh) & 0x0F0F0F0Fu;
        a[3] = (e1 >> sh) & 0x0F0F0F0Fu;
    } else {
        // block 2g + h: 32 int8 values, words 2ss, 2ss+1
        a[0] = comp(c.q[2 * h + (ss >> 1)], (2 * ss) & 3);
        a[2] = comp(c.q[2 * h + (ss >> 1)], (2 * ss + 1) & 3);
        a[1] = comp(c.q[4 + 2 * h + (ss >> 1)], (2 * ss) & 3);
        a[3] = comp(c.q[4 + 2 * h + (ss >> 1)], (2 * ss + 1) & 3);
    }
}

// Q4_K header fields of lane group g (sub-blocks 2g, 2g+1) from the words
// load_chunk picked: sc[h], m[h] (6-bit integers); `sh` = 24g mod 32.
__device__ __forceinline__ void q4k_fields(const uint4 &hd, uint32_t sh, int (&sc)[2], int (&mn)[2]) {
    const uint32_t v = __funnelshift_r(hd.y, hd.z, sh);
    sc[0] = (int)(v & 63u);
    mn[0] = (int)((v >> 6) & 63u);
    sc[1] = (int)((v >> 12) & 63u);
    mn[1] = (int)((v >> 18) & 63u);
}

// One chunk: 8 steps, two sub-blocks (units) per lane.  bp[t] points at the
// lane's B fragments of this chunk for token t (or at the zero block);
// sint at the chunk's per-unit integer activation sums (low and high digit
// pairs); isc[t] is the chunk's activation scale for token t; `sh` is the
// lane group's Q4_K field shift.
//
// Q4_K: a chunk is one super-block, so the lane's two sub-blocks share d and
// dmin and the sums stay integers up to the chunk's end: with X the
// fixed-point activations, Iq = sum_h sc_h * sum q X and Im = sum_h m_h *
// sum X, each held as two int32 digit-pair halves (|sc * sum q X| < 2^30 per
// half; two sub-blocks < 2^31), then d * Iq - dmin * Im in f64 (exact up to
// 2^-53).  Q4_0 / Q8_0 scale every 32-value block by its own f16 d, so their
// sub-block sums meet the scale one by one (f64).  Sums across chunks run in
// f64, so cancelling terms keep their bits.
// The digit sums of one chunk: per sub-block h and token t, da (digits 0, 1)
// and db (digits 2, 3) of rows r (entries 0, 1) and r + 8 (entries 2, 3).
template <int NT>
struct ChunkSums {
    int da[2][NT][4], db[2][NT][4];
};

// Phase 1 of a chunk: the MMAs.  Per sub-block h and token, two chains
// (digits 0-1, 2-3) of four steps; with few tokens both sub-blocks' chains
// run together.  bp[t] points at the lane's B fragments of this chunk for
// token t (or at the zero block).
template <int DT, int NT>
__device__ __forceinline__ void chunk_mma(const ChunkRegs<DT> &c, const uint2 *const (&bp)[NT], ChunkSums<NT> &r) {
    constexpr bool SIGNED = DT == GGUF_Q8_0;
    constexpr int HB = NT <= 2 ? 2 : 1;  // sub-blocks whose chains run together
#pragma unroll
    for (int h0 = 0; h0 < 2; h0 += HB)
#pragma unroll
        for (int ss = 0; ss < 4; ss++)
#pragma unroll
            for (int hh = 0; hh < HB; hh++) {
                const int h = h0 + hh, s = 4 * h + ss;
                uint32_t a[4];
                make_a<DT>(c, s, a);
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    // xy: tile A (digit 0 in col 2g, digit 1 in col 2g+1); zw: tile B (digits 2, 3)
                    const uint4 b = *reinterpret_cast<const uint4 *>(bp[t] + s * 16);
                    if (ss == 0) {
                        imma16832<SIGNED, true>(r.da[h][t], a, b.x, b.y);
                        imma16832<SIGNED, true>(r.db[h][t], a, b.z, b.w);
                    } else {
                        imma16832<SIGNED>(r.da[h][t], a, b.x, b.y);
                        imma16832<SIGNED>(r.db[h][t], a, b.z, b.w);
                    }
                }
            }
}

// Phase 2 of a chunk: the sums meet the scales.  sint points at the chunk's
// per-unit integer activation sums (low and high digit pairs); isc[t] is the
// chunk's activation scale for token t; `sh` is the lane group's Q4_K field
// shift.
//
// Q4_K: a chunk is one super-block, so the lane's two sub-blocks share d and
// dmin and the sums stay integers up to the chunk's end: with X the
// fixed-point activations, Iq = sum_h sc_h * sum q X and Im = sum_h m_h *
// sum X, each held as two int32 digit-pair halves (|sc * sum q X| < 2^30 per
// half; two sub-blocks < 2^31), then d * Iq - dmin * Im in f64 (exact up to
// 2^-53).  Q4_0 / Q8_0 scale every 32-value block by its own f16 d, so their
// sub-block sums meet the scale one by one (f64).  Sums across chunks run in
// f64, so cancelling terms keep their bits.
template <int DT, int NT>
__device__ __forceinline__ void chunk_epilogue(const ChunkRegs<DT> &c, const ChunkSums<NT> &r, double (&acc)[NT][2],
                                               const int *__restrict__ sint, int s_stride, const float (&isc)[NT],
                                               uint32_t sh, int lane) {
    const int g = lane & 3;
    int sc[2][2], mn[2][2];  // Q4_K / Q5_K: [row r / r+8][sub-block h]
    float ds[2][2];          // Q4_0 / Q8_0: [sub-block h][row r / r+8]
    if (kquant45(DT)) {
        q4k_fields(c.h0, sh, sc[0], mn[0]);
        q4k_fields(c.h1, sh, sc[1], mn[1]);
    } else {
        ds[0][0] = h2f(c.h0.x);
        ds[1][0] = h2f(c.h0.x >> 16);
        ds[0][1] = h2f(c.h0.y);
        ds[1][1] = h2f(c.h0.y >> 16);
    }
    int iq[NT][2][2], im[NT][2][2];  // Q4_K: [token][row][low / high digit-pair half]
    // Q5_K: per token and row, the sum over both sub-blocks of sc * (hi * 2^16
    // + lo) in 64 bits (a sub-block's sc * sum q X stays below 2^31, two of
    // them need not: codes up to 31 instead of 15)
    long long iq5[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++)
#pragma unroll
        for (int w = 0; w < 2; w++) {
            iq[t][w][0] = iq[t][w][1] = im[t][w][0] = im[t][w][1] = 0;
            iq5[t][w] = 0;
        }
#pragma unroll
    for (int h = 0; h < 2; h++) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
            // digit pairs: lo = d1*2^8 + d0, hi = d3*2^8 + d2 (each exact in s32)
            int lo0 = r.da[h][t][1] * 256 + r.da[h][t][0], hi0 = r.db[h][t][1] * 256 + r.db[h][t][0];  // row r
            int lo1 = r.da[h][t][3] * 256 + r.da[h][t][2], hi1 = r.db[h][t][3] * 256 + r.db[h][t][2];  // row r + 8
            const int2 sx = *reinterpret_cast<const int2 *>(sint + (t * s_stride + 2 * g + h) * 2);
            if (kquant45(DT)) {
                if (DT == GGUF_Q4_K && h == 1) {  // 16 * code (make_a): exact multiples of 16
                    lo0 >>= 4;
                    hi0 >>= 4;
                    lo1 >>= 4;
                    hi1 >>= 4;
                }
                if (DT == GGUF_Q5_K) {
                    iq5[t][0] += (long long)(sc[0][h] * lo0) + (long long)(sc[0][h] * hi0) * 65536;
                    iq5[t][1] += (long long)(sc[1][h] * lo1) + (long long)(sc[1][h] * hi1) * 65536;
                } else {
                    iq[t][0][0] += sc[0][h] * lo0;
                    iq[t][0][1] += sc[0][h] * hi0;
                    iq[t][1][0] += sc[1][h] * lo1;
                    iq[t][1][1] += sc[1][h] * hi1;
                }
                im[t][0][0] += mn[0][h] * sx.x;
                im[t][0][1] += mn[0][h] * sx.y;
                im[t][1][0] += mn[1][h] * sx.x;
                im[t][1][1] += mn[1][h] * sx.y;
            } else {
                if (DT == GGUF_Q4_0) {  // sum (n - 8) X = sum n X - 8 sum X, per digit pair
                    lo0 -= 8 * sx.x;
                    lo1 -= 8 * sx.x;
                    hi0 -= 8 * sx.y;
                    hi1 -= 8 * sx.y;
                }
                // isc[t] (a power of two) turns the chunk's fixed point back into x
                const double v0 = fma((double)hi0, 65536.0, (double)lo0);
                const double v1 = fma((double)hi1, 65536.0, (double)lo1);
                acc[t][0] = fma((double)(ds[h][0] * isc[t]), v0, acc[t][0]);
                acc[t][1] = fma((double)(ds[h][1] * isc[t]), v1, acc[t][1]);
            }
        }
    }
    if (kquant45(DT)) {
        const float d0 = h2f(c.h0.x), m0 = h2f(c.h0.x >> 16), d1 = h2f(c.h1.x), m1 = h2f(c.h1.x >> 16);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const double q0 = DT == GGUF_Q5_K ? (double)iq5[t][0] : (double)((long long)iq[t][0][1] * 65536 + iq[t][0][0]);
            const double q1 = DT == GGUF_Q5_K ? (double)iq5[t][1] : (double)((long long)iq[t][1][1] * 65536 + iq[t][1][0]);
            const double s0 = (double)((long long)im[t][0][1] * 65536 + im[t][0][0]);
            const double s1 = (double)((long long)im[t][1][1] * 65536 + im[t][1][0]);
            acc[t][0] = fma((double)(d0 * isc[t]), q0, fma((double)(-m0 * isc[t]), s0, acc[t][0]));
            acc[t][1] = fma((double)(d1 * isc[t]), q1, fma((double)(-m1 * isc[t]), s1, acc[t][1]));
        }
    }
}

// Balanced base-256 digits of a fixed-point activation |X| < 2^30: with
// Y = X + 0x80808080 (mod 2^32) the bytes of Y are d_i + 128, so the bytes of
// Y ^ 0x80808080 are the int8 digits d_i of X = sum d_i 256^i.
__device__ __forceinline__ uint32_t biased(int X) { return (uint32_t)X + 0x80808080u; }

// 4x4 byte transpose: out[d] = byte d of w0, w1, w2, w3 (low to high).
__device__ __forceinline__ void transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&o)[4]) {
    const uint32_t t0 = prmt(w0, w1, 0x5140u), t1 = prmt(w0, w1, 0x7362u);
    const uint32_t t2 = prmt(w2, w3, 0x5140u), t3 = prmt(w2, w3, 0x7362u);
    o[0] = prmt(t0, t2, 0x5410u);
    o[1] = prmt(t0, t2, 0x7632u);
    o[2] = prmt(t1, t3, 0x5410u);
    o[3] = prmt(t1, t3, 0x7632u);
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of a cluster barrier that orders nothing: arrive early,
// wait where the other CTAs must have started.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// ---- Work split ------------------------------------------------------------------
//
// Clusters of two CTAs (the two SMs of a TPC).  Cluster c owns the whole tiles
// [tile0, tile0 + nt), so no sum leaves the cluster.  Its nt x n_chunks units
// (one 16-row tile x one 256-column chunk) are ordered in runs -- run r < nt
// is tile r's chunks [0, pw0), run nt + r (two panels only) tile r's chunks
// [pw0, n_chunks) -- and cut into 32 equal ranges, one per warp of the
// cluster.  With two panels (pw0 = ceil(n_chunks / 2); clusters of few
// tiles) CTA 0 covers about the first half of K of every tile and CTA 1 the
// second, so each CTA stages the activations of half of K; with one panel
// (many tiles per cluster) each CTA covers half of the tiles.  A warp adds
// the units of one run (a segment) in registers.  A segment that is a whole
// tile goes straight to y; any other goes to slot [warp][k] (k: the
// segment's place among the warp's) of the CTA that finalises the tile
// (local tile i -> CTA i % 2), over DSMEM, and after one cluster barrier that
// CTA adds the tile's segments in chunk order.  The split depends on the
// weight's shape and the SM count only, never on the batch.

constexpr int kWarps = 16;        // warps per CTA (one CTA per SM)
constexpr int kClusterCtas = 2;   // CTAs per cluster
constexpr int kClusterWarps = kWarps * kClusterCtas;
constexpr int kTwoPanelMaxTiles = 15;  // two panels while clusters hold at most this many tiles
constexpr int kTableBatch = 2;         // activation-table items a warp loads before the ring's rest

// The unit order of a cluster of nt tiles (units < 2^25, so every numerator
// below is < 2^31).  The divisions by pw0, pw1 and U are multiplies by the
// plan's precomputed FastDivs.
struct Split {
    int nt, n_chunks, pw0, pw1;  // tiles, chunks, run lengths of panel 0 and panel 1 (0: one panel)
    uint32_t U;                  // units
    FastDiv d0, d1, dU;          // division by pw0, pw1, U
    __host__ __device__ Split(int nt_, int n_chunks_, int panels, const FastDiv &f0, const FastDiv &f1,
                              const FastDiv &fU) {
        nt = nt_;
        n_chunks = n_chunks_;
        pw0 = panel0_width(n_chunks_, panels);
        pw1 = n_chunks_ - pw0;
        U = (uint32_t)nt_ * (uint32_t)n_chunks_;
        d0 = f0;
        d1 = f1;
        dU = fU;
    }
    __host__ __device__ static int panel0_width(int n_chunks, int panels) {
        return panels == 2 ? (n_chunks + 1) / 2 : n_chunks;
    }
    __host__ static Split make(int nt, int n_chunks, int panels) {
        const int p0 = panel0_width(n_chunks, panels);
        return Split(nt, n_chunks, panels, make_fastdiv((uint32_t)p0), make_fastdiv((uint32_t)(n_chunks - p0)),
                     make_fastdiv((uint32_t)nt * (uint32_t)n_chunks));
    }
    __host__ __device__ uint32_t warp_u0(uint32_t g) const { return g * U / kClusterWarps; }
    // the non-empty warp whose range holds unit u
    __host__ __device__ uint32_t warp_of(uint32_t u) const { return udiv((u + 1) * kClusterWarps + U - 1, dU) - 1; }
    __host__ __device__ uint32_t run_of(uint32_t u) const {
        const uint32_t first = (uint32_t)nt * pw0;
        return u < first ? udiv(u, d0) : nt + udiv(u - first, d1);
    }
    __host__ __device__ uint32_t run_start(uint32_t r) const {
        return r < (uint32_t)nt ? r * pw0 : (uint32_t)nt * pw0 + (r - nt) * pw1;
    }
    __host__ __device__ uint32_t run_len(uint32_t r) const { return r < (uint32_t)nt ? pw0 : pw1; }
    __host__ __device__ int run_tile(uint32_t r) const { return r < (uint32_t)nt ? (int)r : (int)(r - nt); }
    __host__ __device__ int run_chunk0(uint32_t r) const { return r < (uint32_t)nt ? 0 : pw0; }
    __host__ __device__ int runs_per_tile() const { return pw1 > 0 ? 2 : 1; }
    // the slot of warp g's segment k (one panel: whole-tile segments have none)
    __host__ __device__ int slot_of(int k) const { return pw1 > 0 ? k : (k == 0 ? 0 : 1); }
    // A contiguous cover [lo, lo + n) of the chunks of units [u0, u1).
    __host__ __device__ void window(uint32_t u0, uint32_t u1, int &lo, int &n) const {
        if (u1 <= u0) {
            lo = 0;
            n = 0;
            return;
        }
        const uint32_t ra = run_of(u0), rb = run_of(u1 - 1);
        const int ca = run_chunk0(ra) + (int)(u0 - run_start(ra)), cb = run_chunk0(rb) + (int)(u1 - 1 - run_start(rb));
        const bool pa = ra >= (uint32_t)nt, pb = rb >= (uint32_t)nt;
        int hi;
        if (ra == rb) {  // one run
            lo = ca;
            hi = cb;
        } else if (pa == pb) {  // several runs of one panel: the whole panel
            lo = pa ? pw0 : 0;
            hi = pa ? n_chunks - 1 : pw0 - 1;
        } else {  // the tail of panel 0 and the head of panel 1
            lo = ra == (uint32_t)nt - 1 ? ca : 0;
            hi = rb == (uint32_t)nt ? cb : n_chunks - 1;
        }
        n = hi - lo + 1;
    }
};

// The tiles of cluster c: [tile0, tile0 + n); clusters c < extra hold base + 1.
__host__ __device__ inline void cluster_tiles(int c, int base, int extra, int &tile0, int &n) {
    tile0 = c * base + (c < extra ? c : extra);
    n = base + (c < extra ? 1 : 0);
}

// Walks consecutive units without division (one division to start).
struct UnitIter {
    uint32_t run, left;  // current run, units left in it
    int tile, chunk;
    __host__ __device__ __forceinline__ void init(uint32_t u, const Split &sp) {
        run = sp.run_of(u);
        const uint32_t off = u - sp.run_start(run);
        left = sp.run_len(run) - off;
        tile = sp.run_tile(run);
        chunk = sp.run_chunk0(run) + (int)off;
    }
    __host__ __device__ __forceinline__ void next_run(const Split &sp) {
        run++;
        left = sp.run_len(run);
        tile = sp.run_tile(run);
        chunk = sp.run_chunk0(run);
    }
    __host__ __device__ __forceinline__ void next(const Split &sp) {
        chunk++;
        if (--left == 0) next_run(sp);
    }
};

// Shared memory of one CTA.  Identical in the two CTAs of a cluster (slots
// are addressed remotely at the local offset), so it is sized from the
// plan's maxima, not from the CTA's own window.
struct SmemLayout {
    size_t mbar, zero, ring, tbl, sint, inv, slot, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int dt, int nt, int stages, int win, int kmax) {
    SmemLayout L;
    size_t o = 0;
    L.mbar = o;
    o += (size_t)kWarps * kMaxStages * 8;
    o = align_up(o, 16);
    L.zero = o;
    o += 1024;
    o = align_up(o, 128);
    L.ring = o;
    o += (size_t)kWarps * stages * chunk_bytes(dt);
    o = align_up(o, 16);
    L.tbl = o;
    o += (size_t)nt * win * 128 * 8;
    L.sint = o;
    o += (size_t)nt * win * 8 * 8;
    L.inv = o;
    o += (size_t)nt * win * 4;
    o = align_up(o, 16);
    L.slot = o;
    o += (size_t)kClusterWarps * kmax * nt * 16 * 4;
    L.total = align_up(o, 16);
    return L;
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_shared(const void *local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    return remote;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Decode GEMV over clusters of two CTAs (the work split above).  Each warp
// streams its units' chunks through a private TMA ring.  A token's result is
// the same sum in the same order whatever the batch.
template <int DT, int NT>
__global__ void __launch_bounds__(kWarps * 32, 1) gemv_kernel(GemvArgs p) {
    constexpr int CB = chunk_bytes(DT);
    constexpr int FIXED_BITS = 30;  // |x * scale| < 2^30: four balanced int8 digits
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The peer CTA's shared memory is written only after the wait below.
    cluster_arrive_relaxed();
    const int m = p.m, S = p.stages, C = p.g.n_chunks;
    const int rank = (int)cluster_rank();
    const int cl = blockIdx.x / kClusterCtas;
    int T0 = 0, NTc = 0;
    cluster_tiles(cl, p.tiles_base, p.tiles_extra, T0, NTc);
    const Split sp(NTc, C, p.panels, p.fd_pw0, p.fd_pw1, p.fd_u[cl < p.tiles_extra ? 1 : 0]);
    int wlo = 0, nwin = 0;
    sp.window(sp.warp_u0(rank * kWarps), sp.warp_u0((rank + 1) * kWarps), wlo, nwin);
    const SmemLayout L = smem_layout(DT, NT, S, p.win, p.kmax);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.mbar);
    const uint2 *zero = reinterpret_cast<const uint2 *>(smem + L.zero);
    uint8_t *ring = smem + L.ring;
    uint2 *tbl = reinterpret_cast<uint2 *>(smem + L.tbl);    // [NT][nwin][8 steps][4 groups][2 parts][2 tiles]
    int *sint = reinterpret_cast<int *>(smem + L.sint);      // [NT][nwin][8 units][2]
    float *inv = reinterpret_cast<float *>(smem + L.inv);    // [NT][nwin]
    float *slot = reinterpret_cast<float *>(smem + L.slot);  // [32 warps][kmax][NT][16]

    // this warp's units
    const uint32_t gw = (uint32_t)(rank * kWarps + warp);
    const uint32_t u0 = sp.warp_u0(gw), u1 = sp.warp_u0(gw + 1);
    const int nu = (int)(u1 - u0);
    const uint32_t mb0 = smem_u32(mbar + warp * kMaxStages);
    const uint32_t ring0 = smem_u32(ring + (size_t)warp * S * CB);
    UnitIter issue;  // the next unit to copy into the ring
    if (nu > 0) issue.init(u0, sp);
    auto src_next = [&]() {
        const uint8_t *src = tile_src(p, T0 + issue.tile, issue.chunk, CB);
        issue.next(sp);
        return src;
    };

    // The weight copies depend on nothing: start p.pre of them before waiting
    // for the previous kernel (more would queue ahead of the activation loads).
    const int first = min(S, nu), pre = min(p.pre, first);
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(mb0 + 8 * s, 1);
        fence_mbar_init();
        for (int i = 0; i < pre; i++) bulk_load(ring0 + i * CB, src_next(), CB, mb0 + 8 * i);
    }
    if (tid < 256) reinterpret_cast<uint32_t *>(smem + L.zero)[tid] = 0u;  // 1 KB
    // The activations may be the previous kernel's output: wait for it.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const unsigned gepoch = p.ga[0].world > 1 ? gather_epoch(p.ga[0]) : 0u;

    // Activation table: warp item (token t, window chunk j); lane = group gg
    // (64 columns) x step s (8 columns).  The chunk's power of two comes from
    // its own maximum, so no other warp is involved.  The first kTableBatch
    // items' activations are loaded before the rest of the ring is requested,
    // so that those loads are not queued behind the weight copies.
    const int gg = lane >> 3, st = lane & 7;
    auto load_item = [&](int t, int j, float (&v)[8]) {
        const int64_t k = (int64_t)(wlo + j) * CHUNK_K + 64 * gg + 8 * st;
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = 0.f;
        if (t < m && k < p.g.n_cols) {
            const float *src = p.x + (size_t)t * p.ldx + k;
            if (p.x_vec4) {
                const float4 f0 = *reinterpret_cast<const float4 *>(src);
                const float4 f1 = *reinterpret_cast<const float4 *>(src + 4);
                v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
                v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = src[e];
            }
        }
    };
    auto build_item = [&](int t, int j, const float (&v)[8]) {
        // the chunk's largest magnitude, as bits (ordered like the values;
        // inf and NaN above every finite value)
        uint32_t mb = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) mb = max(mb, __float_as_uint(v[e]) & 0x7FFFFFFFu);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, o));
        float sc = 1.f, is = 1.f;
        if (mb >= 0x7F800000u) {
            sc = 0.f;  // non-finite activations: the outputs become NaN
            is = __int_as_float(0x7fc00000);
        } else if (mb != 0u) {
            // max < 2^e (e from the exponent field); below 2^-96 the scale
            // stays 2^126 so that it and its inverse are normal floats
            const int e = max((int)(mb >> 23) - 126, -96);
            sc = __uint_as_float((uint32_t)(127 + FIXED_BITS - e) << 23);  // 2^(30 - e)
            is = __uint_as_float((uint32_t)(127 - FIXED_BITS + e) << 23);  // 2^(e - 30)
        }
        uint32_t y[8];
        uint32_t slo = 0, shi = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            y[e] = biased(__float2int_rn(v[e] * sc));
            slo += y[e] & 0xFFFFu;  // d1*256 + d0 + 0x8080
            shi += y[e] >> 16;      // d3*256 + d2 + 0x8080
            y[e] ^= 0x80808080u;    // the digit bytes
        }
        uint32_t a[4], b[4];
        transpose4(y[0], y[1], y[2], y[3], a);
        transpose4(y[4], y[5], y[6], y[7], b);
        uint4 *dst = reinterpret_cast<uint4 *>(tbl + (size_t)(t * nwin + j) * 128 + st * 16 + gg * 4);
        // part 0 (col 2g): tile A digit 0, tile B digit 2; part 1 (col 2g+1): digits 1, 3
        dst[0] = make_uint4(a[0], b[0], a[2], b[2]);
        dst[1] = make_uint4(a[1], b[1], a[3], b[3]);
        // per-unit (32 values = steps 4h .. 4h+3 of group gg) integer sums
        int lo = (int)slo - 8 * 0x8080, hi = (int)shi - 8 * 0x8080;
        lo += __shfl_xor_sync(0xffffffffu, lo, 1);
        hi += __shfl_xor_sync(0xffffffffu, hi, 1);
        lo += __shfl_xor_sync(0xffffffffu, lo, 2);
        hi += __shfl_xor_sync(0xffffffffu, hi, 2);
        if ((st & 3) == 0) {
            const int u = 2 * gg + (st >> 2);
            sint[((t * nwin + j) * 8 + u) * 2] = lo;
            sint[((t * nwin + j) * 8 + u) * 2 + 1] = hi;
        }
        if (lane == 0) inv[t * nwin + j] = is;
    };
    // this warp's items: (t, j) for every token slot t and j = warp, warp + 16, ...
    int it_t = 0, it_j = warp;
    auto item_next = [&]() {
        it_j += kWarps;
        if (it_j >= nwin) {
            it_j = warp;
            it_t++;
        }
    };
    if (it_j >= nwin) it_t = NT;  // no items
    float xv[kTableBatch][8];
    int bt[kTableBatch], bj[kTableBatch];
#pragma unroll
    for (int b = 0; b < kTableBatch; b++) {
        bt[b] = it_t;
        bj[b] = it_j;
        if (it_t < NT) {
            load_item(it_t, it_j, xv[b]);
            item_next();
        }
    }
    // the rest of the ring
    if (lane == 0)
        for (int i = pre; i < first; i++) bulk_load(ring0 + i * CB, src_next(), CB, mb0 + 8 * i);
#pragma unroll
    for (int b = 0; b < kTableBatch; b++)
        if (bt[b] < NT) build_item(bt[b], bj[b], xv[b]);
    while (it_t < NT) {
        float v[8];
        load_item(it_t, it_j, v);
        build_item(it_t, it_j, v);
        item_next();
    }
    // the table visible to the CTA; the peer CTA started
    __syncthreads();
    cluster_wait();

    // B fragments: lane (n = lane / 4, k-group lane % 4) reads column n; the
    // block-diagonal operand is non-zero only where n / 2 == k-group.
    const bool bact = (lane >> 3) == (lane & 3);
    const int hw = 4 + 4 * ((3 * (lane & 3)) >> 2);      // Q4_K header words of this lane's group
    const uint32_t hsh = (uint32_t)(24 * (lane & 3)) & 31u;
    const int boff = (lane & 3) * 4 + ((lane >> 2) & 1) * 2;
    int slt = 0, issued = first, failed_at = nu;
    uint32_t phase = 0;
    double acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.0;
    const uint8_t *myring = ring + (size_t)warp * S * CB;
    // refill state: the source of the next copy and the units left in its run
    // (consecutive chunks of a run are consecutive in memory)
    const uint8_t *rsrc = first < nu ? tile_src(p, T0 + issue.tile, issue.chunk, CB) : nullptr;
    uint32_t rleft = issue.left;
    // After unit i's slot is read: refill it with unit i + S (lane 0; the
    // branch is warp-uniform) and step to the next slot.
    auto refill = [&](int i) {
        if (i + S < nu) {
            // this slot's reads happen before the copy that refills it
            bulk_refill(lane == 0, ring0 + slt * CB, rsrc, CB, mb0 + 8 * slt);
            issued++;
            rsrc += CB;
            if (--rleft == 0 && i + S + 1 < nu) {
                issue.next_run(sp);
                rsrc = tile_src(p, T0 + issue.tile, issue.chunk, CB);
                rleft = issue.left;
            }
        }
        if (++slt == S) {
            slt = 0;
            phase ^= 1u;
        }
    };
    auto table_bp = [&](int j, const uint2 *(&bp)[NT]) {
#pragma unroll
        for (int t = 0; t < NT; t++) bp[t] = bact ? tbl + (size_t)(t * nwin + j) * 128 + boff : zero;
    };
    auto table_isc = [&](int j, float (&isc)[NT]) {
#pragma unroll
        for (int t = 0; t < NT; t++) isc[t] = inv[t * nwin + j];
    };
    // Segments: this warp's units of one run each; the current one starts at
    // chunk seg_c0 of run un.run and has seg_len units, seg_left still to end.
    UnitIter un;
    if (nu > 0) un.init(u0, sp);
    int seg_k = 0, seg_len = nu > 0 ? min(nu, (int)un.left) : 0, seg_left = seg_len, seg_c0 = un.chunk;
    // the segment's row sums: add the four column groups (lanes 4r .. 4r+3)
    // and send them to the tile's slot, or to y when the segment is the tile
    auto end_segment = [&]() {
        const int seg_tile = un.tile;
        const bool whole = sp.pw1 == 0 && seg_len == (int)sp.run_len(un.run) && seg_c0 == sp.run_chunk0(un.run);
        const int owner = seg_tile % kClusterCtas;
        const uint32_t rb = map_shared(slot + ((size_t)gw * p.kmax + sp.slot_of(seg_k)) * NT * 16, (uint32_t)owner);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            double d0 = acc[t][0], d1 = acc[t][1];
            d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
            d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
            d0 += __shfl_xor_sync(0xffffffffu, d0, 2);
            d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
            const float v0 = (float)d0, v1 = (float)d1;
            if ((lane & 3) == 0) {
                const int r = lane >> 2;
                if (whole) {  // the tile's only segment: straight to y
                    if (t < m) {
                        put_y(p, t, T0 + seg_tile, r, v0, gepoch);
                        put_y(p, t, T0 + seg_tile, r + 8, v1, gepoch);
                    }
                } else if (sp.slot_of(seg_k) < p.kmax) {
                    st_cluster_f32(rb + 4 * (t * 16 + r), v0);
                    st_cluster_f32(rb + 4 * (t * 16 + r + 8), v1);
                }
            }
            acc[t][0] = acc[t][1] = 0.0;
        }
    };
    if constexpr (NT == 1) {
        // A one-chunk pipeline: unit i's epilogue runs beside unit i + 1's MMAs.
        int jcur = un.chunk - wlo;  // table index of the unit in `cur`
        ChunkRegs<DT> cur;
        ChunkSums<NT> sums;
        if (nu > 0) {
            if (mbar_wait_bounded(mb0 + 8 * slt, phase)) {
                load_chunk<DT>(cur, myring + slt * CB, lane, hw);
                __syncwarp();
                refill(0);
                const uint2 *bp[NT];
                table_bp(jcur, bp);
                chunk_mma<DT, NT>(cur, bp, sums);
            } else {
                failed_at = 0;
            }
        }
        for (int i = 0; i + 1 < nu && failed_at == nu; i++) {
            const bool seg_end = seg_left == 1;
            const int jn = seg_end ? sp.run_chunk0(un.run + 1) - wlo : jcur + 1;
            if (!mbar_wait_bounded(mb0 + 8 * slt, phase)) {
                failed_at = i + 1;
                break;
            }
            ChunkRegs<DT> nxt;
            load_chunk<DT>(nxt, myring + slt * CB, lane, hw);
            __syncwarp();
            refill(i + 1);
            {
                float isc[NT];
                table_isc(jcur, isc);
                chunk_epilogue<DT, NT>(cur, sums, acc, sint + jcur * 16, nwin * 8, isc, hsh, lane);
            }
            ChunkSums<NT> nsums;
            {
                const uint2 *bp[NT];
                table_bp(jn, bp);
                chunk_mma<DT, NT>(nxt, bp, nsums);
            }
            if (seg_end) {
                end_segment();
                seg_k++;
                un.next_run(sp);
                seg_len = min(nu - (i + 1), (int)un.left);
                seg_left = seg_len;
                seg_c0 = un.chunk;
            } else {
                seg_left--;
            }
            cur = nxt;
            sums = nsums;
            jcur = jn;
        }
        if (failed_at == nu && nu > 0) {
            float isc[NT];
            table_isc(jcur, isc);
            chunk_epilogue<DT, NT>(cur, sums, acc, sint + jcur * 16, nwin * 8, isc, hsh, lane);
            end_segment();
        }
    } else {
        // one chunk at a time (more tokens leave no registers for a pipeline)
        int j = un.chunk - wlo;
        for (int i = 0; i < nu; i++) {
            if (!mbar_wait_bounded(mb0 + 8 * slt, phase)) {
                failed_at = i;
                break;
            }
            ChunkRegs<DT> cur;
            load_chunk<DT>(cur, myring + slt * CB, lane, hw);
            __syncwarp();
            refill(i);
            ChunkSums<NT> sums;
            {
                const uint2 *bp[NT];
                table_bp(j, bp);
                chunk_mma<DT, NT>(cur, bp, sums);
            }
            {
                float isc[NT];
                table_isc(j, isc);
                chunk_epilogue<DT, NT>(cur, sums, acc, sint + j * 16, nwin * 8, isc, hsh, lane);
            }
            if (seg_left == 1) {
                end_segment();
                if (i + 1 < nu) {
                    seg_k++;
                    un.next_run(sp);
                    seg_len = min(nu - (i + 1), (int)un.left);
                    seg_left = seg_len;
                    seg_c0 = un.chunk;
                    j = un.chunk - wlo;
                }
            } else {
                seg_left--;
                j++;
            }
        }
    }
    if (failed_at < nu) {
        // Report, then let this warp's copies in flight (numbers failed_at ..
        // issued - 1; copy n sits in slot n % S, phase n / S) land.
        if (lane == 0) {
            *reinterpret_cast<volatile int *>(p.err) = kKernelErrWaitTimeout;
            for (int n = failed_at; n < issued; n++) mbar_wait_bounded(mb0 + 8 * (n % S), (uint32_t)((n / S) & 1));
        }
        __syncwarp();
    }
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // every partial of the cluster in place (the last cluster-wide access)
    cluster_sync();

    // finalise this CTA's tiles that have more than one segment: the segments
    // run by run, warp by warp, i.e. in chunk order
    const int runs = sp.runs_per_tile();
    for (int tl = rank + kClusterCtas * warp; tl < NTc; tl += kClusterCtas * kWarps) {
        uint32_t ga[2], gb[2];
        int ka[2];  // the segment number, within warp ga[h], of its piece of run h
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (h < runs) {
                const uint32_t run = (uint32_t)tl + (uint32_t)h * NTc;
                const uint32_t a = sp.run_start(run);
                ga[h] = sp.warp_of(a);
                gb[h] = sp.warp_of(a + sp.run_len(run) - 1);
                ka[h] = (int)(run - sp.run_of(sp.warp_u0(ga[h])));
            }
        }
        if (runs == 1 && ga[0] == gb[0]) continue;  // one segment: written directly
        float v[2] = {0.f, 0.f};                  // q = lane, lane + 32 (q = t * 16 + r)
#pragma unroll
        for (int h = 0; h < 2; h++)
            for (uint32_t g = ga[h]; h < runs && g <= gb[h]; g++) {
                if (sp.warp_u0(g + 1) == sp.warp_u0(g)) continue;  // no units
                const int sl = sp.slot_of(g == ga[h] ? ka[h] : 0);
                if (sl >= p.kmax) continue;
                const float *src = slot + ((size_t)g * p.kmax + sl) * NT * 16;
#pragma unroll
                for (int e = 0; e < 2; e++)
                    if (lane + 32 * e < NT * 16) v[e] += src[lane + 32 * e];
            }
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int q = lane + 32 * e, t = q >> 4, r = q & 15;
            if (q < NT * 16 && t < m) put_y(p, t, T0 + tl, r, v[e], gepoch);
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

template <int DT, int NT>
cudaError_t launch_one(const GemvArgs &a, size_t smem, cudaStream_t s) {
    static std::atomic<unsigned long long> done{0};  // one per instantiation
    auto kern = gemv_kernel<DT, NT>;
    cudaError_t e = ensure_smem_optin(kern, done);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_clusters * kClusterCtas, 1, 1);
    cfg.blockDim = dim3(kWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kClusterCtas;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT>
cudaError_t launch_nt(int nt, const GemvArgs &a, size_t smem, cudaStream_t s) {
    switch (nt) {
    case 1: return launch_one<DT, 1>(a, smem, s);
    case 2: return launch_one<DT, 2>(a, smem, s);
    case 4: return launch_one<DT, 4>(a, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

constexpr size_t kSmemBudget = 225 * 1024;

}  // namespace

namespace {

// The plan of one work-split choice (panels = 1 or 2).
GemvPlan plan_split(int dt, const Geometry &g, int m, int nc, int panels) {
    GemvPlan p;
    p.clusters = nc;
    p.panels = panels;
    const int nt_min = g.n_tiles / nc, nt_max = (g.n_tiles + nc - 1) / nc;
    // the largest table window of any CTA and the most segments of any warp
    // (clusters hold nt_min or nt_max tiles)
    int win = 1, kmax = 2;
    for (int nt : {nt_min, nt_max}) {
        const Split sp = Split::make(nt, g.n_chunks, panels);
        for (int r = 0; r < kClusterCtas; r++) {
            int lo = 0, n = 0;
            sp.window(sp.warp_u0(r * kWarps), sp.warp_u0((r + 1) * kWarps), lo, n);
            if (n > win) win = n;
        }
        if (panels == 2)
            for (uint32_t w = 0; w < (uint32_t)kClusterWarps; w++) {
                const uint32_t u0 = sp.warp_u0(w), u1 = sp.warp_u0(w + 1);
                if (u1 > u0) {
                    const int k = (int)(sp.run_of(u1 - 1) - sp.run_of(u0)) + 1;
                    if (k > kmax) kmax = k;
                }
            }
    }
    p.window = win;
    p.kmax = kmax;
    // tokens per launch: the batch's slot count, fewer when the activation
    // table would not fit next to a 2-stage ring
    p.nt = m <= 1 ? 1 : m <= 2 ? 2 : 4;
    while (p.nt > 1 && smem_layout(dt, p.nt, 2, win, kmax).total > kSmemBudget) p.nt /= 2;
    // TMA ring: as deep as the shared memory left over allows (2..4 stages)
    p.stages = kMaxStages;
    while (p.stages > 2 && smem_layout(dt, p.nt, p.stages, win, kmax).total > kSmemBudget) p.stages--;
    p.smem = smem_layout(dt, p.nt, p.stages, win, kmax).total;
    return p;
}

}  // namespace

GemvPlan plan_gemv(int dt, const Geometry &g, int m, int sm_count) {
    // one cluster per TPC, never more clusters than tiles
    int nc = sm_count / kClusterCtas;
    if (nc > g.n_tiles) nc = g.n_tiles;
    if (nc < 1) nc = 1;
    const int nt_max = (g.n_tiles + nc - 1) / nc;
    const bool two = g.n_chunks >= 2;
    GemvPlan p = plan_split(dt, g, m, nc, (nt_max <= kTwoPanelMaxTiles && two) ? 2 : 1);
    // many tiles per cluster and a long K: halve the table with two panels
    if (p.smem > kSmemBudget && p.panels == 1 && two) p = plan_split(dt, g, m, nc, 2);
    return p;
}

cudaError_t launch_gemv_group(int dt, const GemvGroup &grp, const float *x, size_t ldx, int m,
                              const GemvPlan &plan, int *err, cudaStream_t s, const GatherArgs *ga) {
    if (m <= 0) return cudaSuccess;
    if (m > kGemvMaxTokens || plan.nt < 1 || grp.n < 1 || grp.n > kGemvMaxGroup) return cudaErrorInvalidValue;
    if (ga && ga[0].world > kMaxPeers) return cudaErrorInvalidValue;
    const Geometry g = group_geometry(grp);
    // 32-bit unit arithmetic in the kernel (numerators < 2^31)
    if (plan.smem > 227 * 1024 || (uint64_t)g.n_tiles * g.n_chunks >= (1ull << 25)) return cudaErrorNotSupported;
    if (g.n_tiles == 0) return cudaSuccess;
    GemvArgs a;
    a.n_w = grp.n;
    float *ybase[kGemvMaxGroup];
    for (int i = 0; i < kGemvMaxGroup; i++) {
        const int k = i < grp.n ? i : 0;  // unused entries repeat weight 0
        a.w[i] = grp.w[k];
        a.n_rows[i] = grp.g[k].n_rows;
        a.ldy[i] = grp.ldy[k];
        ybase[i] = grp.y[k];
    }
    for (int i = 0, t = 0; i < kGemvMaxGroup; i++) {
        a.tile0[i] = t;
        if (i < grp.n) t += (int)grp.g[i].n_tiles;
    }
    a.err = err;
    a.g = g;
    a.ldx = ldx;
    a.stages = plan.stages;
    a.pre = plan.stages < 2 ? plan.stages : 2;
    a.n_clusters = plan.clusters;
    a.panels = plan.panels;
    a.win = plan.window;
    a.kmax = plan.kmax;
    a.tiles_base = (int)(g.n_tiles / plan.clusters);
    a.tiles_extra = (int)(g.n_tiles % plan.clusters);
    {
        const int p0 = Split::panel0_width((int)g.n_chunks, plan.panels);
        a.fd_pw0 = make_fastdiv((uint32_t)p0);
        a.fd_pw1 = make_fastdiv((uint32_t)(g.n_chunks - p0));
        a.fd_u[0] = make_fastdiv((uint32_t)(a.tiles_base * g.n_chunks));
        a.fd_u[1] = make_fastdiv((uint32_t)((a.tiles_base + 1) * g.n_chunks));
    }
    a.x_vec4 = ((ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
    // token groups of plan.nt (one launch when the table fits the batch)
    for (int t0 = 0; t0 < m; t0 += plan.nt) {
        a.x = x + (size_t)t0 * ldx;
        for (int i = 0; i < kGemvMaxGroup; i++) a.y[i] = ybase[i] + (size_t)t0 * a.ldy[i];
        a.m = m - t0 < plan.nt ? m - t0 : plan.nt;
        if (ga) {
            for (int i = 0; i < grp.n; i++) {
                a.ga[i] = ga[i];
                for (int r = 0; r < ga[i].world; r++)
                    if (a.ga[i].ll[r]) a.ga[i].ll[r] += (size_t)t0 * a.ldy[i];
            }
        }
        cudaError_t e;
        switch (dt) {
        case GGUF_Q4_K: e = launch_nt<GGUF_Q4_K>(plan.nt, a, plan.smem, s); break;
        case GGUF_Q5_K: e = launch_nt<GGUF_Q5_K>(plan.nt, a, plan.smem, s); break;
        case GGUF_Q4_0: e = launch_nt<GGUF_Q4_0>(plan.nt, a, plan.smem, s); break;
        case GGUF_Q8_0: e = launch_nt<GGUF_Q8_0>(plan.nt, a, plan.smem, s); break;
        default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

Geometry group_geometry(const GemvGroup &grp) {
    Geometry g = grp.g[0];
    int64_t tiles = 0;
    for (int i = 0; i < grp.n; i++) tiles += grp.g[i].n_tiles;
    g.n_tiles = tiles;
    g.n_rows = tiles * 16;
    return g;
}

cudaError_t launch_gemv(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx,
                        float *y, size_t ldy, int m, const GemvPlan &plan, int *err, cudaStream_t s,
                        const GatherArgs *ga) {
    if (g.n_rows <= 0) return cudaSuccess;
    GemvGroup grp;
    grp.n = 1;
    grp.w[0] = tiles;
    grp.g[0] = g;
    grp.y[0] = y;
    grp.ldy[0] = ldy;
    return launch_gemv_group(dt, grp, x, ldx, m, plan, err, s, ga);
}

}  // namespace rce
