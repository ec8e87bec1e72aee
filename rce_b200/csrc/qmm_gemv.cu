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
//    ahead, so ~70 KB per CTA are in flight from the first instruction on.
//    Every wait on an mbarrier is bounded (%globaltimer); on expiry the
//    kernel records an error word, waits (bounded) for its own copies and
//    finishes.
//  * The dot products are exact integer arithmetic on the tensor cores
//    (mma.sync m16n8k32, u8/s8 x s8 -> s32).  The weight codes are the A
//    operand as they are stored: Q8_0's int8 bytes need no unpacking at all,
//    Q4_K/Q4_0 nibbles one and/shift per 4 codes.  Activations become a
//    fixed-point integer per token, X = x * 2^e rounded to 31 bits with the
//    power of two chosen from the CTA's slice of x, whose four balanced
//    base-256 digits are simply the bytes of (X + 0x80808080) ^ 0x80808080;
//    the B operand is block-diagonal so that lane g's columns hold digits of
//    its own column group (tile A digits 0-1, tile B digits 2-3).  Each digit
//    pair's 32-value sub-block sum is exact in s32; the two pairs meet in f32
//    and the block scales (d, d*sc, dmin*m) are applied once per sub-block,
//    so no weight is rounded and x keeps 2^-30 of its slice maximum (below
//    f32's own rounding of the reference's sums).
//  * Q4_K's min term and Q4_0's -8 offset use per-sub-block sums of the
//    integer activations (the "asum hoist"): one op per sub-block.
//  * The activation table (the B fragments) is built per window of chunks
//    with vectorised loads while the first weight copies are in flight.
//  * Launched with programmatic stream serialization: a kernel's CTAs start
//    while the previous kernel on the stream drains, issue their weight
//    copies (which depend on nothing), and only then wait for the previous
//    grid (griddepcontrol.wait) before touching the activations or writing
//    outputs.  Each CTA signals its dependents once its main loop is done.
//  * The grid puts 1-8 tiles in a CTA so that all CTAs are resident in one
//    wave; K is split across CTAs only when the rows alone cannot occupy the
//    SMs.  Split partial sums go to scratch and the last CTA to arrive for a
//    row block adds them in split order (deterministic).
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
    int stages, red_mode, x_vec4;
    GatherArgs ga;  // fused all-gather over peer memory (ga.world > 1)
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

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// D(s32) += A(16x32, u8 or s8) x B(32x8, s8), exact.
template <bool A_SIGNED>
__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if (A_SIGNED)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t comp(const uint4 &v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

// One output value: to y, and with the fused all-gather also to every other
// rank's receive buffer (at this rank's rows of the full output).
__device__ __forceinline__ void put_y(const GemvArgs &p, int t, int64_t row, float v, unsigned epoch) {
    p.y[t * p.ldy + row] = v;
    if (p.ga.world > 1) gather_send(p.ga, (size_t)t * p.ldy + (size_t)p.ga.row_off + (size_t)row, v, epoch);
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

// The A operand of step s (0..7) for rows r (a0: columns 64g + 8s + 0..3,
// a2: + 4..7) and r + 8 (a1, a3): the stored codes, one byte per value.
// Sub-block (unit) 2g + (s >> 2); see qmm_layout.cuh for where the bytes sit.
template <int DT>
__device__ __forceinline__ void make_a(const ChunkRegs<DT> &c, int s, uint32_t (&a)[4]) {
    const int h = s >> 2, ss = s & 3;
    if (DT == GGUF_Q4_K) {
        // group g's 32 qs bytes per row: words 2ss, 2ss+1; low nibbles are
        // sub-block 2g, high nibbles sub-block 2g+1
        const uint32_t r0 = comp(c.q[ss >> 1], (2 * ss) & 3), r1 = comp(c.q[ss >> 1], (2 * ss + 1) & 3);
        const uint32_t e0 = comp(c.q[2 + (ss >> 1)], (2 * ss) & 3), e1 = comp(c.q[2 + (ss >> 1)], (2 * ss + 1) & 3);
        const int sh = 4 * h;
        a[0] = (r0 >> sh) & 0x0F0F0F0Fu;
        a[2] = (r1 >> sh) & 0x0F0F0F0Fu;
        a[1] = (e0 >> sh) & 0x0F0F0F0Fu;
        a[3] = (e1 >> sh) & 0x0F0F0F0Fu;
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

// One chunk: 8 steps, two sub-blocks (units) per lane.  bp[t] points at the
// lane's B fragments of this chunk for token t (or at the zero block);
// sint/sflt at the chunk's per-unit integer activation sums.
template <int DT, int NT>
__device__ __forceinline__ void process_chunk(const ChunkRegs<DT> &c, float (&acc)[NT][2], const uint2 *const (&bp)[NT],
                                              const int *__restrict__ sint, const float *__restrict__ sflt,
                                              int s_stride, int lane) {
    constexpr bool SIGNED = DT == GGUF_Q8_0;
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
        int da[NT][4], db[NT][4];
#pragma unroll
        for (int t = 0; t < NT; t++)
#pragma unroll
            for (int i = 0; i < 4; i++) da[t][i] = db[t][i] = 0;
#pragma unroll
        for (int ss = 0; ss < 4; ss++) {
            const int s = 4 * h + ss;
            uint32_t a[4];
            make_a<DT>(c, s, a);
#pragma unroll
            for (int t = 0; t < NT; t++) {
                // xy: tile A (digit 0 in col 2g, digit 1 in col 2g+1); zw: tile B (digits 2, 3)
                const uint4 b = *reinterpret_cast<const uint4 *>(bp[t] + s * 16);
                imma16832<SIGNED>(da[t], a, b.x, b.y);
                imma16832<SIGNED>(db[t], a, b.z, b.w);
            }
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            // digit pairs: lo = d1*2^8 + d0, hi = d3*2^8 + d2 (each exact in s32)
            int lo0 = da[t][1] * 256 + da[t][0], hi0 = db[t][1] * 256 + db[t][0];  // row r
            int lo1 = da[t][3] * 256 + da[t][2], hi1 = db[t][3] * 256 + db[t][2];  // row r + 8
            if (DT == GGUF_Q4_0) {  // sum (n - 8) X = sum n X - 8 sum X, per digit pair
                const int2 sx = *reinterpret_cast<const int2 *>(sint + (t * s_stride + 2 * g + h) * 2);
                lo0 -= 8 * sx.x;
                lo1 -= 8 * sx.x;
                hi0 -= 8 * sx.y;
                hi1 -= 8 * sx.y;
            }
            const float v0 = fmaf((float)hi0, 65536.f, (float)lo0);
            const float v1 = fmaf((float)hi1, 65536.f, (float)lo1);
            acc[t][0] = fmaf(ds[h][0], v0, acc[t][0]);
            acc[t][1] = fmaf(ds[h][1], v1, acc[t][1]);
            if (DT == GGUF_Q4_K) {  // - dmin*m * sum X
                const float sx = sflt[t * s_stride + 2 * g + h];
                acc[t][0] = fmaf(-mn[h][0], sx, acc[t][0]);
                acc[t][1] = fmaf(-mn[h][1], sx, acc[t][1]);
            }
        }
    }
}

// Shared-memory carve-up, identical on host and device.
struct SmemLayout {
    size_t mbar, zero, ring, xs, tbl, ssum, sint, sflt, red, scl, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr int kNumBars = 8 * kMaxStages;  // one weight-ring mbarrier per warp and stage

__host__ __device__ inline SmemLayout smem_layout(int dt, int nt, int stages, int cps) {
    SmemLayout L;
    size_t o = 0;
    L.mbar = o;
    o += kNumBars * 8;
    o = align_up(o, 16);
    L.zero = o;
    o += 1024;
    o = align_up(o, 128);
    L.ring = o;
    o += (size_t)8 * stages * chunk_bytes(dt);
    o = align_up(o, 16);
    L.xs = o;
    o += (size_t)nt * cps * CHUNK_K * 4;
    L.tbl = o;
    o += (size_t)nt * cps * 128 * 8;
    L.ssum = o;
    o += (size_t)nt * cps * 32 * 8;
    L.sint = o;
    o += (size_t)nt * cps * 8 * 8;
    L.sflt = o;
    o += (size_t)nt * cps * 8 * 4;
    L.red = o;
    o += (size_t)8 * nt * 16 * 4;
    L.scl = o;
    o += (size_t)2 * nt * 4;
    L.total = align_up(o, 16);
    return L;
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

// A float in the shared memory of cluster CTA `rank`, at the offset of `local`.
__device__ __forceinline__ float ld_cluster(const float *local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// Cross-CTA reduction of split-K partial sums.
enum : int { kRedNone = 0, kRedCluster = 1, kRedScratch = 2 };

template <int DT, int NT, int RT>
__global__ void __launch_bounds__(256, 2) gemv_kernel(GemvArgs p) {
    constexpr int KQ = 8 / RT;
    constexpr int CB = chunk_bytes(DT);
    constexpr int FIXED_BITS = 30;  // |x * scale| < 2^30: four balanced int8 digits
    extern __shared__ __align__(128) uint8_t smem[];
    const int m = p.m, S = p.stages, cps = p.cps;
    const SmemLayout L = smem_layout(DT, NT, S, cps);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.mbar);
    const uint2 *zero = reinterpret_cast<const uint2 *>(smem + L.zero);
    uint8_t *ring = smem + L.ring;
    float *xs = reinterpret_cast<float *>(smem + L.xs);     // [NT][cps * 256] this CTA's slice of x
    uint2 *tbl = reinterpret_cast<uint2 *>(smem + L.tbl);   // [NT][cps][8 steps][4 groups][2 parts][2 tiles]
    int2 *ssum = reinterpret_cast<int2 *>(smem + L.ssum);   // [NT][cps][4 groups][8 steps] (lo, hi pair sums)
    int *sint = reinterpret_cast<int *>(smem + L.sint);     // [NT][cps][8 units][2]
    float *sflt = reinterpret_cast<float *>(smem + L.sflt); // [NT][cps][8 units]
    float *red = reinterpret_cast<float *>(smem + L.red);   // [8 warps][NT][16]
    float *scl = reinterpret_cast<float *>(smem + L.scl);   // [NT] scale, [NT] inverse
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const int c0 = blockIdx.y * cps;
    const int nc = min(cps, p.g.n_chunks - c0);
    const int rt_local = warp % RT, kq = warp / RT;
    const int tile = blockIdx.x * RT + rt_local;
    const bool tile_ok = tile < p.g.n_tiles;
    // chunks of this warp: kq, kq + KQ, ... (< nc)
    const int nw = (tile_ok && kq < nc) ? (nc - kq + KQ - 1) / KQ : 0;
    const uint8_t *gsrc = p.w + ((size_t)(tile_ok ? tile : 0) * p.g.n_chunks + c0) * CB;
    const uint32_t mb0 = smem_u32(mbar + warp * kMaxStages);
    const uint32_t ring0 = smem_u32(ring + (size_t)warp * S * CB);
    const int64_t k_lo = (int64_t)c0 * CHUNK_K;
    const int64_t k_hi = min((int64_t)(c0 + nc) * CHUNK_K, p.g.n_cols);
    const int xn = (int)(k_hi - k_lo);  // activations of this slice (a multiple of 32)

    // The weight copies depend on nothing: start them before anything else.
    if (lane == 0) {
        for (int s = 0; s < S; s++) mbar_init(mb0 + 8 * s, 1);
        fence_mbar_init();
        for (int i = 0; i < min(S, nw); i++)
            bulk_load(ring0 + i * CB, gsrc + (size_t)(kq + i * KQ) * CB, CB, mb0 + 8 * i);
    }
    // The activations may be the previous kernel's output: wait for it.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const unsigned gepoch = p.ga.world > 1 ? gather_epoch(p.ga) : 0u;
    // The CTA's activation slice comes in through ordinary coalesced loads
    // (the load/store path), not the TMA queue, which is busy with the weight
    // prefetch; each thread tracks the maximum of what it loaded.
    reinterpret_cast<uint32_t *>(smem + L.zero)[tid] = 0u;  // 256 x 4 B
    float xmax[NT];
#pragma unroll
    for (int t = 0; t < NT; t++) {
        float mx = 0.f;
        bool fin = true;
        float *xd = xs + t * cps * CHUNK_K;
        if (t >= m) {  // padding tokens are zero
            for (int k = tid; k < xn; k += 256) xd[k] = 0.f;
        } else if (p.x_vec4) {
            const float4 *src = reinterpret_cast<const float4 *>(p.x + t * p.ldx + k_lo);
            for (int k4 = tid; k4 < xn / 4; k4 += 256) {
                const float4 v = src[k4];
                reinterpret_cast<float4 *>(xd)[k4] = v;
                mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                fin = fin && isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
            }
        } else {  // unaligned activations: scalar loads
            for (int k = tid; k < xn; k += 256) {
                const float v = p.x[t * p.ldx + k_lo + k];
                xd[k] = v;
                mx = fmaxf(mx, fabsf(v));
                fin = fin && isfinite(v);
            }
        }
        xmax[t] = fin ? mx : INFINITY;
    }
    __syncthreads();  // barrier inits visible before anyone waits
    bool failed = false;

    // Per-token power-of-two scale for this CTA's column slice: x * scale
    // lies inside +-2^FIXED_BITS.
#pragma unroll
    for (int t = 0; t < NT; t++) {
        float mx = xmax[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp * NT + t] = mx;
    }
    __syncthreads();
    if (tid < NT) {
        float v = 0.f;
        for (int w = 0; w < 8; w++) v = fmaxf(v, red[w * NT + tid]);
        float s = 1.f, inv = 1.f;
        if (!isfinite(v)) {
            s = 0.f;  // non-finite activations: the outputs become NaN
            inv = __int_as_float(0x7fc00000);
        } else if (v > 0.f) {
            int e;
            frexpf(v, &e);  // v < 2^e
            e = max(-100, min(100, e));
            s = ldexpf(1.f, FIXED_BITS - e);
            inv = ldexpf(1.f, e - FIXED_BITS);
        }
        scl[tid] = s;
        scl[NT + tid] = inv;
    }
    __syncthreads();

    // Activation table: per (token, chunk, group gg, step s) the digits of the
    // 8 values 64 gg + 8 s + 0..7 as B fragments, and their pair sums.
    for (int idx = tid; idx < NT * nc * 32; idx += 256) {
        const int t = idx / (nc * 32), rem = idx % (nc * 32);
        const int c = rem >> 5, q = rem & 31, gg = q >> 3, s = q & 7;
        const int k = c * CHUNK_K + 64 * gg + 8 * s;
        float v[8];
        if (k < xn) {
            const float4 f0 = *reinterpret_cast<const float4 *>(xs + t * cps * CHUNK_K + k);
            const float4 f1 = *reinterpret_cast<const float4 *>(xs + t * cps * CHUNK_K + k + 4);
            v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
            v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.f;
        }
        const float sc = scl[t];
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
        uint4 *dst = reinterpret_cast<uint4 *>(tbl + (size_t)(t * cps + c) * 128 + s * 16 + gg * 4);
        // part 0 (col 2g): tile A digit 0, tile B digit 2; part 1 (col 2g+1): digits 1, 3
        dst[0] = make_uint4(a[0], b[0], a[2], b[2]);
        dst[1] = make_uint4(a[1], b[1], a[3], b[3]);
        ssum[((t * cps + c) * 4 + gg) * 8 + s] = make_int2((int)slo - 8 * 0x8080, (int)shi - 8 * 0x8080);
    }
    if (DT != GGUF_Q8_0) {
        __syncthreads();
        // unit u = group u/2, steps 4 (u%2) .. +3
        for (int idx = tid; idx < NT * nc * 8; idx += 256) {
            const int t = idx / (nc * 8), rem = idx % (nc * 8), c = rem >> 3, u = rem & 7;
            const int2 *src = ssum + ((t * cps + c) * 4 + (u >> 1)) * 8 + 4 * (u & 1);
            const int lo = src[0].x + src[1].x + src[2].x + src[3].x;
            const int hi = src[0].y + src[1].y + src[2].y + src[3].y;
            sint[((t * cps + c) * 8 + u) * 2] = lo;
            sint[((t * cps + c) * 8 + u) * 2 + 1] = hi;
            sflt[(t * cps + c) * 8 + u] = fmaf((float)hi, 65536.f, (float)lo);
        }
    }
    __syncthreads();

    float acc[NT][2];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = 0.f;
    // B fragments: lane (n = lane / 4, k-group lane % 4) reads column n; the
    // block-diagonal operand is non-zero only where n / 2 == k-group.
    const bool bact = (lane >> 3) == (lane & 3);
    const int boff = (lane & 3) * 4 + ((lane >> 2) & 1) * 2;
    int i = 0, slot = 0;
    uint32_t phase = 0;
    while (!failed && i < nw) {
        const int cl = kq + i * KQ;
        if (!mbar_wait_bounded(mb0 + 8 * slot, phase)) {
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
        const uint2 *bp[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) bp[t] = bact ? tbl + (size_t)(t * cps + cl) * 128 + boff : zero;
        process_chunk<DT, NT>(cur, acc, bp, sint + cl * 16, sflt + cl * 8, cps * 8, lane);
        i++;
        if (++slot == S) {
            slot = 0;
            phase ^= 1u;
        }
    }
    if (failed) {
        // Report, then let this warp's copies in flight land before exiting.
        if (lane == 0) {
            *reinterpret_cast<volatile int *>(p.err) = kKernelErrWaitTimeout;
            int sl = slot;
            uint32_t ph = phase;
            for (int j = i; j < min(nw, i + S); j++) {
                mbar_wait_bounded(mb0 + 8 * sl, ph);
                if (++sl == S) {
                    sl = 0;
                    ph ^= 1u;
                }
            }
        }
        __syncwarp();
    }

    // Sum the four column groups of each row (lanes 4r .. 4r+3), then the KQ
    // warps of each tile in a fixed order, and undo the activation scale.
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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
    // part[rtl][t][r16] = this CTA's partial sums; reuses the front of xs
    float *part = xs;
    for (int idx = tid; idx < RT * NT * 16; idx += 256) {
        const int rtl = idx / (NT * 16), rem = idx % (NT * 16), t = rem >> 4, r16 = rem & 15;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < KQ; q++) v += red[((rtl + q * RT) * NT + t) * 16 + r16];
        v *= scl[NT + t];
        const int64_t row = (int64_t)(blockIdx.x * RT + rtl) * 16 + r16;
        if (p.red_mode == kRedCluster) {
            part[idx] = v;
        } else if (t < m && row < p.g.n_rows) {
            if (p.k_splits == 1)
                put_y(p, t, row, v, gepoch);
            else
                p.partial[((size_t)blockIdx.y * m + t) * p.n_pad + row] = v;
        }
    }
    if (p.red_mode == kRedCluster) {
        // The k_splits CTAs of this row block form one cluster (ranks =
        // blockIdx.y); rank 0 adds their partial sums in rank order.
        cluster_sync();
        if (blockIdx.y == 0) {
            for (int idx = tid; idx < RT * NT * 16; idx += 256) {
                const int rtl = idx / (NT * 16), rem = idx % (NT * 16), t = rem >> 4, r16 = rem & 15;
                const int64_t row = (int64_t)(blockIdx.x * RT + rtl) * 16 + r16;
                if (t < m && row < p.g.n_rows) {
                    float v = 0.f;
                    for (int q = 0; q < p.k_splits; q++) v += ld_cluster(part + idx, (uint32_t)q);
                    put_y(p, t, row, v, gepoch);
                }
            }
        }
        cluster_sync();  // keep every CTA's shared memory alive until rank 0 has read it
    } else if (p.red_mode == kRedScratch) {
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
                    put_y(p, t, row, v, gepoch);
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
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    unsigned n = 0;
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
    if (a.red_mode == kRedCluster) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = 1;
        attr[n].val.clusterDim.y = grid.y;
        attr[n].val.clusterDim.z = 1;
        n++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, a);
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
    // The activation slice and its table take nt x cps x 2 KB of shared
    // memory: at most 8 chunks per CTA.  Nothing below depends on m, so a
    // token's result is the same whatever the batch.
    const int cps_cap = 8;
    const int ks_min = (g.n_chunks + cps_cap - 1) / cps_cap;
    // Tiles per CTA and the K split: the largest tile count (one warp per
    // tile: the CTA's activation table serves 8 tiles) whose grid still
    // covers every SM, within one resident wave (two CTAs per SM).
    int best_rt = 1, best_ks = ks_min, best_ctas = -1;
    for (int rt = 8; rt >= 1; rt /= 2) {
        const int kq = 8 / rt;
        const int rows = (g.n_tiles + rt - 1) / rt;
        int ks = (2 * sm_count) / rows;
        if (ks > 8) ks = 8;
        if (ks > g.n_chunks / kq) ks = g.n_chunks / kq;  // at least one chunk per warp
        if (ks < ks_min) ks = ks_min;
        if (ks < 1) ks = 1;
        const int cps = (g.n_chunks + ks - 1) / ks;
        ks = (g.n_chunks + cps - 1) / cps;
        const int ctas = rows * ks;
        if (ctas > best_ctas) {
            best_rt = rt;
            best_ks = ks;
            best_ctas = ctas;
        }
        if (ctas >= sm_count) break;
    }
    p.rt = best_rt;
    p.cps = (g.n_chunks + best_ks - 1) / best_ks;
    p.k_splits = (g.n_chunks + p.cps - 1) / p.cps;
    p.red_mode = p.k_splits == 1 ? kRedNone : (p.k_splits <= 8 ? kRedCluster : kRedScratch);
    // TMA ring depth: as deep as shared memory allows for two CTAs per SM
    p.stages = kMaxStages;
    while (p.stages > 2 && smem_layout(dt, p.nt, p.stages, p.cps).total > 110 * 1024) p.stages--;
    (void)m;
    p.window = p.cps;
    p.smem = smem_layout(dt, p.nt, p.stages, p.cps).total;
    if (p.red_mode == kRedScratch) {
        p.scratch_floats = (size_t)p.k_splits * m * g.n_tiles * 16;
        p.counters = (g.n_tiles + p.rt - 1) / p.rt;
    }
    return p;
}

GemvPlan plan_gemv_scratch(int dt, const Geometry &g, int m, int sm_count) {
    GemvPlan p = plan_gemv(dt, g, m, sm_count);
    if (p.red_mode == kRedCluster) {
        p.red_mode = kRedScratch;
        p.scratch_floats = (size_t)p.k_splits * m * g.n_tiles * 16;
        p.counters = (g.n_tiles + p.rt - 1) / p.rt;
    }
    return p;
}

cudaError_t launch_gemv(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx,
                        float *y, size_t ldy, int m, const GemvPlan &plan, float *scratch,
                        unsigned *counters, int *err, cudaStream_t s, const GatherArgs *ga) {
    if (m <= 0 || g.n_rows <= 0) return cudaSuccess;
    if (ga && ga->world > kMaxPeers) return cudaErrorInvalidValue;
    if (m > plan.nt || m > kGemvMaxTokens) return cudaErrorInvalidValue;
    if (plan.red_mode == kRedScratch && (!scratch || !counters)) return cudaErrorInvalidValue;
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
    a.red_mode = plan.red_mode;
    a.x_vec4 = ((ldx & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) ? 1 : 0;
    if (ga) a.ga = *ga;
    dim3 grid((g.n_tiles + plan.rt - 1) / plan.rt, plan.k_splits);
    switch (dt) {
    case GGUF_Q4_K: return launch_rt<GGUF_Q4_K>(plan.rt, plan.nt, a, grid, plan.smem, s);
    case GGUF_Q4_0: return launch_rt<GGUF_Q4_0>(plan.rt, plan.nt, a, grid, plan.smem, s);
    case GGUF_Q8_0: return launch_rt<GGUF_Q8_0>(plan.rt, plan.nt, a, grid, plan.smem, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace rce
