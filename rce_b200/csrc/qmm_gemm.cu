// qmm_gemm.cu -- prefill matmul on the 5th-generation tensor cores (tcgen05).
//
// Y[t][row] = sum_k X[t][k] * W[row][k] for t_rows tokens, W a registered
// GGUF weight in the T16 layout (qmm_layout.cuh).  Same operator as the
// reference's mm_batched (rce-op-qmm/src/lib.rs:967-1023), which for these
// formats is t_rows independent mm_1d calls.
//
// Numerics: the weights are dequantised exactly in f32 (d*sc*q - dmin*m, as
// dequantize_to_f32 computes them) and rounded once to fp16; activations are
// scaled per token by a power of two (exact) so that |x * s| < 2^14 and
// rounded to fp16; products accumulate in f32 in tensor memory.  fp16 (11
// significant bits) instead of bf16 (8) keeps the output within the 1e-3
// bar for Q4_K, at the same tensor-core rate.  Token tiles of up to
// kTwoTermMaxTile tokens (dense batches of up to kGemmTwoTermMaxTokens
// tokens, and every expert-grouped launch) carry each activation as two fp16
// terms, high + low (about 22 significant bits): the low rows sit after the
// high rows in the activation stage, one MMA of N = high + low rows covers
// both, and the epilogue adds the two accumulator halves.  Up to 64 tokens
// (N <= 128) an MMA instruction costs the same as for the high rows alone,
// and the only rounding left is the weights' (the activations' rounding is what
// gives the one-term path its error tail on outputs that partly cancel,
// e.g. an MoE token's weighted sum of two experts).
//
// Structure (one CTA = 128 weight rows x BN tokens, all of K; BN up to 512,
// i.e. two N = 256 accumulators filling tensor memory, so that a weight
// tile is dequantised once per 512 tokens):
//   prep kernel: X (f32) -> Xh (fp16, [t_rows][K]) and 1/s per token;
//   warp 0     : TMA bulk copies of the packed T16 chunks (8 tiles x 256
//                columns per slot, 2-4 slots as shared memory allows);
//   warps 1-16 : dequantisers in two groups of eight that take alternate
//                k-blocks, half a weight row per thread (32 values), into
//                the A tile (fp16, K-major, 128-byte swizzle); then the
//                epilogue (tcgen05.ld from tensor memory, scale, store);
//   warp 17    : one thread issues tcgen05.mma (kind::f16, M=128, N<=256,
//                K=16 per instruction) into f32 accumulators in tensor
//                memory and frees each stage with tcgen05.commit;
//   warp 18    : TMA tensor loads of the 128B-swizzled Xh tile of each
//                64-column k-block (after the prep kernel, via PDL).
// Every mbarrier wait is bounded (%globaltimer, 1 s); on expiry the CTA
// records the kernel error word and unwinds without further waits that
// could block, releasing its tensor memory.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "qmm_internal.h"
#include "qmm_prep.cuh"

namespace rce {
namespace {

constexpr unsigned long long kWaitNs = 1000000000ull;
constexpr int kBK = 64;                // k-block (one 128-byte swizzle row of fp16)
constexpr int kBM = 128;               // weight rows per CTA (UMMA M)
constexpr int kDqWarps = 16;           // dequantiser warps (four threads per weight row)
constexpr int kWeightWarp = 0;         // TMA bulk copies of the packed weight chunks
constexpr int kMaxMmaWarps = 2;       // tcgen05.mma issuers (K split between them; see mma_warps)
constexpr int kMmaWarp = kDqWarps + 1;  // the first; also tcgen05.alloc / dealloc
constexpr int kActWarp = kDqWarps + 1 + kMaxMmaWarps;  // TMA tensor loads of the activation k-blocks
constexpr int kThreads = 32 * (kActWarp + 1);

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false if the phase did not complete within kWaitNs.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > kWaitNs) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// One chunk (256 columns) of 8 consecutive 16-row tiles of a T16 weight:
// the 4-d tensor map of weight_map, coordinates (0, 0, chunk, first tile).
__device__ __forceinline__ void tma_4d(uint32_t dst, const CUtensorMap *map, int c, int t, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(map), "r"(0), "r"(0), "r"(c), "r"(t), "r"(bar)
        : "memory");
}

// kps k-blocks of the activations, all terms, bn rows from `row`: the 4-d
// tensor map of act_map4, coordinates (0, row, 0, first k-block).
__device__ __forceinline__ void tma_act4(uint32_t dst, const CUtensorMap *map, int row, int kb, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(dst),
        "l"(map), "r"(0), "r"(row), "r"(0), "r"(kb), "r"(bar)
        : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // SBO
    d |= (uint64_t)1 << 46;                 // descriptor version
    d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
    return d;
}

// Instruction descriptor: D f32, A/B fp16, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// The MMA issuers run as whole warps with warp-uniform operands (kept in
// uniform registers) and one elected lane issues: a single thread issuing
// from divergent code spends 60-95 cycles per instruction, an elected lane
// of a converged warp reaches the tensor pipe's own rate (~40 cycles per
// M = 128, N <= 32, K = 16 instruction).  The same lane is elected every
// time (the lowest), so its commits track its MMAs.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
        : "memory");
}
// The same with A in tensor memory (128 lanes = rows, K packed two fp16
// per 32-bit column).
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
// 32 consecutive 32-bit columns of this thread's tensor-memory lane (the
// warp's 32 lanes at once).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFF)));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

struct GemmArgs {
    const uint8_t *w;
    float *y;
    const float *inv_scale;  // per token
    int *err;
    Geometry g;
    size_t ldy;
    int t_rows;
    int bn;
    int box_rows;  // rows of one activation TMA box
    int lo_row;    // two-term activations: row of the tensor map where the low terms start (0: one term)
    int splits;    // split-K: CTA z of the dense launch covers chunks [z C / splits, (z + 1) C / splits)
    float *part;   // split-K partial outputs [splits][t_rows][n_rows] (splits > 1)
    BulkPush push; // fused bulk all-gather (push.world > 1; dense launches without splits)
    int kps_log;   // log2 of the k-blocks per activation stage: 0 (2-d map, a box per k-block and term) or
                   // 1, 2 (4-d map over [k-block][term][row][64], one copy per stage; dense launches)
};

// Packed f32x2 arithmetic (two lanes of f32 per instruction).
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
    return (unsigned long long)__float_as_uint(lo) | ((unsigned long long)__float_as_uint(hi) << 32);
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
// fp16x2 of the two f32 lanes (round to nearest even).
__device__ __forceinline__ uint32_t f2_to_h2(unsigned long long v) {
    return pack_h2(__uint_as_float((uint32_t)v), __uint_as_float((uint32_t)(v >> 32)));
}

// Packed fp16x2 arithmetic, round to nearest even, subnormals kept.
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// Shared-space loads and stores by 32-bit shared address (the dequantiser's
// pointers pass through a struct; generic accesses would go the long way).
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ uint32_t h2dup(uint32_t bits16) { return (bits16 & 0xFFFFu) | (bits16 << 16); }
// Bytes P and P + 1 (P = 0 or 2) of v under the fp16 exponent of 1024: the
// fp16 pair (1024 + b_P, 1024 + b_{P+1}), exact for bytes up to 1023, in one
// byte permute.
template <int P>
__device__ __forceinline__ uint32_t byte_h2(uint32_t v) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(0x64646464u), "r"(P == 0 ? 0x4140u : 0x4342u));
    return r;
}
// The fp16 pair of a small integer 0 .. 1023 in both halves (exact).
__device__ __forceinline__ uint32_t small_h2(uint32_t v) { return h2sub(h2dup(0x6400u | v), 0x64006400u); }

// A thread's half of weight row `row` (32 of the 64 values of each k-block),
// the rows' scales decoded once per chunk.  Values are exact in f32 (as the
// reference's dequantize_to_f32 computes them) and rounded once to fp16; per
// k-block one 16-byte load of the codes and, for Q4_K, no header work.
//
// Q4_K / Q5_K / Q4_0 / Q8_0 values are built in fp16 arithmetic: one byte
// permute gives the pair (1024 + code); for the K-quants an exact fp16 FMA
// gives sc * code (at most 63 * 31 = 1953, so exact in fp16: the product is
// exact inside the FMA and so is the result) and a second FMA gives
// d * (sc * code) - fp16(dmin * m), rounded once to fp16; for Q4_0 / Q8_0 an
// exact subtraction gives code - offset and one multiply d * (code - offset),
// rounded once (the same fp16 value as rounding the exact f32 product).
// Against rounding the exact f32 value d * sc * code - dmin * m once, the
// K-quants add only the rounding of dmin * m to fp16.  Q6_K keeps the f32
// path ((d * sc) * (code - 32), rounded as the reference rounds it).
template <int DT>
struct RowHalf {
    uint32_t ch;  // shared address of this row's 16-row tile in the packed chunk
    int row, hf, r16, r, rh;
    unsigned long long s[4][2];                   // Q6_K: [k-block j][16-value group] scale pairs (f32x2)
    uint32_t hs[4][2], hc[4][2], hm[4][2], hd;     // K-quants: fp16 pairs sc, -1024 sc, -(dmin * m); d

    // k-blocks G and G + 2 of the chunk (the ones dequantiser group G fills)
    template <int G>
    __device__ __forceinline__ void begin(const uint8_t *slot, int row_, int hf_) {
        constexpr int CB = chunk_bytes(DT);
        row = row_;
        hf = hf_;
        const int tile = row >> 4;
        r16 = row & 15;
        r = r16 & 7;
        rh = r16 >> 3;
        ch = smem_u32(slot) + (uint32_t)(tile * CB);
        if (kquant45(DT)) {
            const uint4 h4 = lds128(ch + 2048 + r16 * 16);
            hd = h2dup(h4.x);                                // d
            const uint32_t ndmin = h2dup(h4.x >> 16) ^ 0x80008000u;  // -dmin
            kq_scales<G>(h4, ndmin);
            kq_scales<G + 2>(h4, ndmin);
        } else if (DT == GGUF_Q6_K) {
            const float d = h2f(lds16(ch + kQ6D + 2 * r16));
            const uint4 sv = lds128(ch + kQ6Sc + r16 * 16);
            q6_scales<G>(d, sv);
            q6_scales<G + 2>(d, sv);
        }
    }

    // The same for k-block J alone (a thread that fills one k-block of the
    // chunk, both halves: for K-quants the scales do not depend on hf, so a
    // copy of this object with hf = 1 serves the other half; Q6_K's do).
    template <int J>
    __device__ __forceinline__ void begin1(const uint8_t *slot, int row_, int hf_) {
        constexpr int CB = chunk_bytes(DT);
        row = row_;
        hf = hf_;
        const int tile = row >> 4;
        r16 = row & 15;
        r = r16 & 7;
        rh = r16 >> 3;
        ch = smem_u32(slot) + (uint32_t)(tile * CB);
        if (kquant45(DT)) {
            const uint4 h4 = lds128(ch + 2048 + r16 * 16);
            hd = h2dup(h4.x);
            kq_scales<J>(h4, h2dup(h4.x >> 16) ^ 0x80008000u);
        } else if (DT == GGUF_Q6_K) {
            q6_scales<J>(h2f(lds16(ch + kQ6D + 2 * r16)), lds128(ch + kQ6Sc + r16 * 16));
        }
    }

    // K-quant scales of k-block j (sub-blocks 2 j, 2 j + 1) from the 16-byte
    // row header (d, dmin, then the 12 permuted scale bytes: 24 bits per
    // k-block, sc and m of 6 bits per sub-block)
    template <int j>
    __device__ __forceinline__ void kq_scales(const uint4 &h4, uint32_t ndmin) {
        const uint32_t lo = j < 2 ? h4.y : (j == 2 ? h4.z : h4.w);
        const uint32_t hi = j < 2 ? h4.z : (j == 2 ? h4.w : 0u);
        const uint32_t sh = j == 0 ? 0u : (j == 1 ? 24u : (j == 2 ? 16u : 8u));
        const uint32_t f = __funnelshift_r(lo, hi, sh) & 0xFFFFFFu;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t sc = small_h2((f >> (12 * h)) & 63u), m = small_h2((f >> (12 * h + 6)) & 63u);
            hs[j][h] = sc;
            hc[j][h] = h2mul(sc, 0xE400E400u);  // -1024 * sc, exact
            hm[j][h] = h2mul(ndmin, m);          // -(dmin * m), rounded once to fp16
        }
    }
    // Q6_K, k-block j, 16-value group k2 of this half: scale 4 j + 2 hf + k2,
    // d * sc exact in f32 (11 x 8 bits)
    template <int j>
    __device__ __forceinline__ void q6_scales(float d, const uint4 &sv) {
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int k2 = 0; k2 < 2; k2++) {
            const int i = 4 * j + 2 * hf + k2;  // hf is 0 or 1: the word is sw[j]
            const float ds = d * (float)(int8_t)(sw[i >> 2] >> (8 * (i & 3)));
            s[j][k2] = f2pack(ds, ds);
        }
    }

    // K-quant value pair from the fp16 pair (1024 + code): sc * code exactly,
    // then d * (sc * code) - dmin * m with one rounding (sub-block h of
    // k-block j)
    __device__ __forceinline__ uint32_t kq_pair(uint32_t c1024, int j, int h) const {
        return h2fma(h2fma(c1024, hs[j][h], hc[j][h]), hd, hm[j][h]);
    }

    // k-block J of the chunk: this thread's 32 fp16 values (h) and the four
    // 16-byte chunks of its A-tile row they fill (cc)
    template <int J>
    __device__ __forceinline__ void compute(uint32_t (&h)[16], int (&cc)[4]) const {
        const int lane = 4 * r + J;
        if (DT == GGUF_Q6_K) {
            // columns 32 hf .. 32 hf + 31 of the k-block: 16 lo-plane bytes
            // (two codes each) and 8 hi-plane bytes (four each); value =
            // (d * sc) * (code - 32), one rounding as in dequant_q6_k, then fp16
            const uint4 lq = lds128(ch + r16 * 128 + 32 * J + 16 * hf);
            const uint2 hq = lds64(ch + kQ6Hi + r16 * 64 + 16 * J + 8 * hf);
            const uint32_t lw[4] = {lq.x, lq.y, lq.z, lq.w};
            const unsigned long long bias = f2pack(-8388640.f, -8388640.f);  // 2^23 + 32
#pragma unroll
            for (int k = 0; k < 4; k++) {  // values 8k .. 8k + 7
                const uint32_t hw = ((k < 2 ? hq.x : hq.y) >> (16 * (k & 1))) & 0xFFFFu;
                uint32_t sp;
                asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(sp) : "r"(hw & 0x0F0Fu), "r"((hw >> 4) & 0x0F0Fu));
                const uint32_t ua = (lw[k] & 0x0F0F0F0Fu) | ((sp << 4) & 0x30303030u);         // values 2b
                const uint32_t ub = ((lw[k] >> 4) & 0x0F0F0F0Fu) | ((sp << 2) & 0x30303030u);  // values 2b + 1
#pragma unroll
                for (int p = 0; p < 4; p++) {
                    uint32_t fa, fb;
                    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(fa) : "r"(ua), "r"(0x4B000000u), "r"(0x7540u | p));
                    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(fb) : "r"(ub), "r"(0x4B000000u), "r"(0x7540u | p));
                    const unsigned long long q =
                        f2add((unsigned long long)fa | ((unsigned long long)fb << 32), bias);
                    h[4 * k + p] = f2_to_h2(f2mul(q, s[J][k >> 1]));
                }
                cc[k] = 4 * hf + k;
            }
        } else if (DT == GGUF_Q5_K) {
            // Q4_K's nibbles plus the fifth bit of value l = 16 hf + 8 qq + b
            // at bit 8 (l & 3) + (l >> 2) of Y0 (low nibbles) / Y1 (high)
            const uint4 q = lds128(ch + ((2 * rh + hf) * 32 + lane) * 16);
            const uint2 y = lds64(ch + kQ5Hi + lane * 16 + 8 * rh);
            const uint32_t y0 = y.x >> (4 * hf), y1 = y.y >> (4 * hf);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int qq = 0; qq < 2; qq++)
#pragma unroll
                for (int wi = 0; wi < 2; wi++) {
                    // byte c of word 2 qq + wi: its fifth bits are bits 8 c + 2 qq + wi
                    // of Y0 / Y1, i.e. one shift and one mask put all four at bit 4
                    const int sh = 2 * qq + wi;
                    const uint32_t wd = w[2 * qq + wi];
                    const uint32_t lo = (wd & 0x0F0F0F0Fu) | (((y0 >> sh) & 0x01010101u) << 4);
                    const uint32_t hi = ((wd >> 4) & 0x0F0F0F0Fu) | (((y1 >> sh) & 0x01010101u) << 4);
                    h[8 * qq + 2 * wi] = kq_pair(byte_h2<0>(lo), J, 0);
                    h[8 * qq + 2 * wi + 1] = kq_pair(byte_h2<2>(lo), J, 0);
                    h[8 * qq + 4 + 2 * wi] = kq_pair(byte_h2<0>(hi), J, 1);
                    h[8 * qq + 5 + 2 * wi] = kq_pair(byte_h2<2>(hi), J, 1);
                }
            cc[0] = 2 * hf;
            cc[1] = 4 + 2 * hf;
            cc[2] = 2 * hf + 1;
            cc[3] = 5 + 2 * hf;
        } else if (DT == GGUF_Q4_K) {
            // per word the low and the high nibble planes by two masks, then
            // one byte permute per value
            const uint4 q = lds128(ch + ((2 * rh + hf) * 32 + lane) * 16);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int qq = 0; qq < 2; qq++)  // quarter 2 hf + qq: bytes 8 qq .. 8 qq + 7
#pragma unroll
                for (int wi = 0; wi < 2; wi++) {
                    const uint32_t lo = w[2 * qq + wi] & 0x0F0F0F0Fu, hi = (w[2 * qq + wi] >> 4) & 0x0F0F0F0Fu;
                    h[8 * qq + 2 * wi] = kq_pair(byte_h2<0>(lo), J, 0);
                    h[8 * qq + 2 * wi + 1] = kq_pair(byte_h2<2>(lo), J, 0);
                    h[8 * qq + 4 + 2 * wi] = kq_pair(byte_h2<0>(hi), J, 1);
                    h[8 * qq + 5 + 2 * wi] = kq_pair(byte_h2<2>(hi), J, 1);
                }
            cc[0] = 2 * hf;
            cc[1] = 4 + 2 * hf;
            cc[2] = 2 * hf + 1;
            cc[3] = 5 + 2 * hf;
        } else {
#pragma unroll
            for (int qq = 0; qq < 2; qq++) {
                const int qr = 2 * hf + qq;
                const uint2 sc = lds64(ch + quant_bytes(DT) + lane * 8);
                const uint32_t sw = rh ? sc.y : sc.x;
                const uint32_t d2 = h2dup(sw >> (16 * hf));  // the block's fp16 d in both halves
                if (DT == GGUF_Q4_0) {
                    constexpr uint32_t kOff = 0x64086408u;  // (1032, 1032): 1024 + the offset 8
                    const uint2 q = lds64(ch + ((2 * rh + hf) * 32 + lane) * 16 + 8 * (qr & 1));
                    const uint32_t w[2] = {q.x, q.y};
#pragma unroll
                    for (int wi = 0; wi < 2; wi++) {
                        const uint32_t lo = w[wi] & 0x0F0F0F0Fu, hi = (w[wi] >> 4) & 0x0F0F0F0Fu;
                        h[8 * qq + 2 * wi] = h2mul(h2sub(byte_h2<0>(lo), kOff), d2);
                        h[8 * qq + 2 * wi + 1] = h2mul(h2sub(byte_h2<2>(lo), kOff), d2);
                        h[8 * qq + 4 + 2 * wi] = h2mul(h2sub(byte_h2<0>(hi), kOff), d2);
                        h[8 * qq + 5 + 2 * wi] = h2mul(h2sub(byte_h2<2>(hi), kOff), d2);
                    }
                    cc[2 * qq] = 4 * hf + (qr & 1);
                    cc[2 * qq + 1] = cc[2 * qq] + 2;
                } else {
                    constexpr uint32_t kOff = 0x64806480u;  // (1152, 1152): 1024 + 128
                    const uint4 q = lds128(ch + ((4 * rh + qr) * 32 + lane) * 16);
                    const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                                           q.w ^ 0x80808080u};
#pragma unroll
                    for (int wi = 0; wi < 4; wi++) {  // byte ^ 0x80 = q + 128
                        h[8 * qq + 2 * wi] = h2mul(h2sub(byte_h2<0>(w[wi]), kOff), d2);
                        h[8 * qq + 2 * wi + 1] = h2mul(h2sub(byte_h2<2>(w[wi]), kOff), d2);
                    }
                    cc[2 * qq] = 2 * qr;
                    cc[2 * qq + 1] = 2 * qr + 1;
                }
            }
        }
    }
    // the values into row `row` of the A tile at shared address a (K-major,
    // 128-byte swizzle)
    __device__ __forceinline__ void store(uint32_t a, const uint32_t (&h)[16], const int (&cc)[4]) const {
        const uint32_t dst = a + (uint32_t)((row >> 3) * 1024 + (row & 7) * 128);
#pragma unroll
        for (int i = 0; i < 4; i++)
            sts128(dst + (uint32_t)((cc[i] ^ (row & 7)) * 16), h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
    }
};

// Shared-memory plan of one CTA for token-tile width bn.
struct GemmSmem {
    size_t a, b, packed, bars, tmem_slot, total;
    int a_stages, b_stages, pslots;
};

constexpr int kMaxA = 12, kMaxB = 16, kMaxP = 4;  // ring depth limits (barrier slots)
constexpr int kBars = 2 * kMaxP + 2 * kMaxA + 2 * kMaxB + 1;  // mbarriers of the CTA
constexpr int kMaxASmem = 8;  // A stages in shared memory at most
constexpr uint32_t kTmemCols = 512;  // tensor memory of the CTA (all of the SM's)
constexpr uint32_t kTmemStage = kBK / 2;  // columns of one A k-block in tensor memory

// Activation stages of several k-blocks: one tensor copy (and one mbarrier
// phase) per stage instead of one box per k-block and term.  A copy costs
// the TMA unit a few hundred cycles whatever its size, so per-k-block boxes
// of a small token tile cannot keep up with the MMAs.
constexpr size_t kActStageBudget = 128 * 1024;

// log2 of the k-blocks per activation stage of a dense launch: with A in
// tensor memory, 4 or 2 if two such stages fit kActStageBudget, else 1.
__host__ __device__ inline int act_kps_log(int bn, int terms, bool tmem_a) {
    if (!tmem_a) return 0;
    const size_t kb_bytes = (size_t)terms * bn * kBK * 2;
    if (2 * 4 * kb_bytes <= kActStageBudget) return 2;
    if (2 * 2 * kb_bytes <= kActStageBudget) return 1;
    return 0;
}

// Token tiles up to this width carry two-term activations (N = 2 bn <= 256).
constexpr int kTwoTermMaxTile = 128;

// Activation stages per k-block: the 512-token tile's k-block is two stages
// of 256 rows (one tensor-map box and one N = 256 accumulator half each), so
// that with the same shared memory three of four halves can be in flight
// while the MMAs read the fourth (with whole-k-block stages, one of two).
__host__ __device__ inline int act_halves(int bn, int terms) { return terms * bn > 256 ? 2 : 1; }

__host__ __device__ inline GemmSmem gemm_smem(int dt, int bn, int terms, bool tmem_a, int kps_log) {
    // Rings as deep as 227 KB allow: the dequantiser <-> MMA hand-off takes
    // a few thousand cycles, so the A ring should span several k-blocks;
    // the activation ring shrinks as its stages grow with bn.
    constexpr size_t kLimit = 227 * 1024;  // dynamic shared memory per CTA (opt-in)
    GemmSmem L;
    const int brows = terms * bn;  // activation rows per stage
    // at least 2-4 stages, and up to 8 of them within 32 KB (A tile in
    // shared memory) or kMaxB within 64 KB (A in tensor memory): at small
    // token tiles a stage is consumed faster than an L2 round trip
    L.b_stages = brows > 256 ? 2 : (brows > 128 ? 3 : 4);
    const int halves = act_halves(bn, terms);  // (tmem_a is false there: 512 accumulator columns)
    L.b_stages *= halves;
    const int by_bytes = (int)(((tmem_a ? 64 : 32) * 1024) / (brows * kBK * 2));
    const int max_b = tmem_a ? kMaxB : 8;
    if (by_bytes > L.b_stages) L.b_stages = by_bytes < max_b ? by_bytes : max_b;
    const int kps = 1 << kps_log;
    if (kps > 1) {  // stages of kps k-blocks: as many as kActStageBudget holds (at least 2)
        const int n = (int)(kActStageBudget / ((size_t)kps * brows * kBK * 2));
        L.b_stages = n < 2 ? 2 : (n > kMaxB ? kMaxB : n);
    }
    const size_t a_stage = (size_t)kBM * kBK * 2;
    const size_t b_bytes = (size_t)L.b_stages * kps * (brows / halves) * kBK * 2;
    const size_t slot = (size_t)8 * chunk_bytes(dt);
    const size_t misc = kBars * 8 + 16 + 1024;
    L.pslots = 2;
    size_t avail = kLimit > b_bytes + misc + 2 * slot ? kLimit - b_bytes - misc - 2 * slot : 0;
    if (tmem_a) {  // the A stages live in tensor memory: all the rest buys weight slots
        while (L.pslots < kMaxP && slot <= avail) {
            L.pslots++;
            avail -= slot;
        }
        L.a_stages = 0;
        L.a = 0;
        L.b = 0;
        size_t o = b_bytes;
        L.packed = o;
        o += (size_t)L.pslots * slot;
        o = (o + 15) / 16 * 16;
        L.bars = o;
        o += kBars * 8;
        L.tmem_slot = o;
        o += 16;
        L.total = o + 1024;
        return L;
    }
    // the 512-token tile with the larger chunks of Q8_0 / Q6_K: fewer
    // activation halves (at least one k-block's two) until two A stages fit
    size_t b_now = b_bytes;
    while (halves == 2 && L.b_stages > 2 && avail < 2 * a_stage) {
        L.b_stages--;
        b_now = (size_t)L.b_stages * kps * (brows / halves) * kBK * 2;
        avail = kLimit > b_now + misc + 2 * slot ? kLimit - b_now - misc - 2 * slot : 0;
    }
    int na = (int)(avail / a_stage);
    if (na > kMaxASmem) na = kMaxASmem;
    // leftover room buys a third and fourth weight slot
    while (L.pslots < kMaxP && na >= 3 && (size_t)na * a_stage + slot <= avail) {
        L.pslots++;
        avail -= slot;
    }
    // an even number of A stages: k-block kb uses stage kb % NA, so with NA
    // even each stage only ever holds k-blocks of one dequantiser group, which
    // waits for the stage's previous use before refilling it (a stage shared
    // by the two groups could be refilled two phases ahead of its consumer,
    // which a parity wait cannot tell from one phase behind)
    na &= ~1;
    L.a_stages = na < 2 ? 2 : na;
    size_t o = 0;
    L.a = o;  // 1024-aligned stages
    o += (size_t)L.a_stages * a_stage;
    L.b = o;
    o += b_now;
    L.packed = o;
    o += (size_t)L.pslots * slot;
    o = (o + 15) / 16 * 16;
    L.bars = o;
    o += kBars * 8;
    L.tmem_slot = o;
    o += 16;
    L.total = o + 1024;  // slack to align the base to 1024
    return L;
}

__host__ __device__ inline uint32_t tmem_cols(int bn) {
    return bn <= 32 ? 32u : (bn <= 64 ? 64u : (bn <= 128 ? 128u : (bn <= 256 ? 256u : 512u)));
}

// MMA issuer warps for token-tile width bn: k-blocks are dealt round-robin
// to this many warps, each with its own accumulator (terms * bn columns of
// tensor memory each, 512 in all), and the epilogue adds them.  A thread
// issues a tcgen05.mma about every 60-95 cycles whatever N, while the tensor
// pipe takes one M = 128, K = 16 instruction every ~40 cycles at N <= 32
// (~48 at N = 64) when two threads issue (no faster with four): at small
// token tiles one issuer would bound the k-block rate.
__host__ __device__ inline int mma_warps(int bn, int terms) {
    const int by_tmem = 512 / (int)tmem_cols(terms * bn);
    return by_tmem < kMaxMmaWarps ? by_tmem : kMaxMmaWarps;
}

// One dequantiser group's loop (group G takes k-blocks j = G and G + 2 of
// every chunk): per chunk both k-blocks' values are computed before their A
// stages are awaited, then stored with one proxy fence and arrival; needs at
// least 4 A stages (the two k-blocks in distinct stages).  Returns false if a
// bounded wait expired.
template <int DT, int G>
__device__ __forceinline__ bool dequant_group_pairs(const GemmArgs &p, uint8_t *pk, uint8_t *a_st, uint32_t bar0,
                                                    int row, int hf, int ntiles, int nchunks, int NP, int NA,
                                                    int lane) {
    constexpr int CB = chunk_bytes(DT);
    auto PF = [&](int s) { return bar0 + 8 * (0 + s); };
    auto PE = [&](int s) { return bar0 + 8 * (kMaxP + s); };
    auto AF = [&](int s) { return bar0 + 8 * (2 * kMaxP + s); };
    auto AE = [&](int s) { return bar0 + 8 * (2 * kMaxP + kMaxA + s); };
    int s = 0, st = G;  // packed slot and A stage (of k-block 4 c + G), with their phases
    uint32_t sph = 0, aph = 0;
    const bool live = row < ntiles * 16;
    const uint32_t a0 = smem_u32(a_st);
    for (int c = 0; c < nchunks; c++) {
        if (!mbar_wait(PF(s), sph)) return false;
        uint32_t h0[16], h1[16];
        int c0[4], c1[4];
        RowHalf<DT> rw;
        if (live) {
            rw.template begin<G>(pk + (size_t)s * 8 * CB, row, hf);
            rw.template compute<G>(h0, c0);
            rw.template compute<G + 2>(h1, c1);
        }
        // the stage of k-block 4 c + G + 2, two stages on
        int st1 = st + 2;
        uint32_t aph1 = aph;
        if (st1 >= NA) {
            st1 -= NA;
            aph1 ^= 1;
        }
        const int kb = 4 * c + G;
        if (kb >= NA && !mbar_wait(AE(st), aph ^ 1)) return false;
        if (kb + 2 >= NA && !mbar_wait(AE(st1), aph1 ^ 1)) return false;
        const uint32_t t0 = a0 + (uint32_t)(st * kBM * kBK * 2), t1 = a0 + (uint32_t)(st1 * kBM * kBK * 2);
        if (live) {
            rw.store(t0, h0, c0);
            rw.store(t1, h1, c1);
        } else {  // rows past the weight: zeros
            const uint32_t o = (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + 64 * hf);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                sts128(t0 + o + 16 * q, 0u, 0u, 0u, 0u);
                sts128(t1 + o + 16 * q, 0u, 0u, 0u, 0u);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) {  // one arrival per warp and stage; this group is done with the chunk
            mbar_arrive(AF(st));
            mbar_arrive(AF(st1));
            mbar_arrive(PE(s));
        }
        st = st1 + 2;
        aph = aph1;
        if (st >= NA) {
            st -= NA;
            aph ^= 1;
        }
        if (++s == NP) {
            s = 0;
            sph ^= 1;
        }
    }
    return true;
}

// The same, one k-block at a time (2 A stages: one per group).
template <int DT, int G>
__device__ __forceinline__ bool dequant_group_single(const GemmArgs &p, uint8_t *pk, uint8_t *a_st, uint32_t bar0,
                                                     int row, int hf, int ntiles, int nchunks, int NP, int NA,
                                                     int lane) {
    constexpr int CB = chunk_bytes(DT);
    auto PF = [&](int s) { return bar0 + 8 * (0 + s); };
    auto PE = [&](int s) { return bar0 + 8 * (kMaxP + s); };
    auto AF = [&](int s) { return bar0 + 8 * (2 * kMaxP + s); };
    auto AE = [&](int s) { return bar0 + 8 * (2 * kMaxP + kMaxA + s); };
    int s = 0, st = G;  // packed slot and A stage, with their phases
    uint32_t sph = 0, aph = 0;
    const bool live = row < ntiles * 16;
    const uint32_t a0 = smem_u32(a_st);
    for (int c = 0; c < nchunks; c++) {
        if (!mbar_wait(PF(s), sph)) return false;
        RowHalf<DT> rw;
        if (live) rw.template begin<G>(pk + (size_t)s * 8 * CB, row, hf);
#pragma unroll
        for (int jj = 0; jj < 2; jj++) {
            uint32_t h[16];
            int cc[4];
            if (live) {
                if (jj == 0)
                    rw.template compute<G>(h, cc);
                else
                    rw.template compute<G + 2>(h, cc);
            }
            const int kb = 4 * c + G + 2 * jj;
            if (kb >= NA && !mbar_wait(AE(st), aph ^ 1)) return false;
            const uint32_t t = a0 + (uint32_t)(st * kBM * kBK * 2);
            if (live) {
                rw.store(t, h, cc);
            } else {  // rows past the weight: zeros
                const uint32_t o = (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + 64 * hf);
#pragma unroll
                for (int q = 0; q < 4; q++) sts128(t + o + 16 * q, 0u, 0u, 0u, 0u);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
            __syncwarp();
            if (lane == 0) {  // one arrival per warp
                mbar_arrive(AF(st));
                if (jj == 1) mbar_arrive(PE(s));  // this group is done with the chunk
            }
            st += 2;
            if (st >= NA) {
                st -= NA;
                aph ^= 1;
            }
        }
        if (++s == NP) {
            s = 0;
            sph ^= 1;
        }
    }
    return true;
}

// A in tensor memory: dequantiser warp w (1 .. 16) fills k-block
// J = (w - 1) / 4 of every chunk for the 32 rows of its lane quadrant
// (w % 4, the tensor-memory lanes a warp may write), one weight row per
// thread, all 64 values; stages of kTmemStage columns from ta0, chunk c's
// k-block J in stage 4 (c % NC) + J.  No shared-memory A tile, swizzle or
// proxy fence: the values go from registers to tensor memory
// (tcgen05.st), and the MMA reads A from there.
template <int DT, int J>
__device__ __forceinline__ bool dequant_tmem(uint8_t *pk, uint32_t bar0, uint32_t ta0, int row, int ntiles,
                                             int nchunks, int NP, int NC, int lane) {
    constexpr int CB = chunk_bytes(DT);
    auto PF = [&](int s) { return bar0 + 8 * (0 + s); };
    auto PE = [&](int s) { return bar0 + 8 * (kMaxP + s); };
    auto AF = [&](int s) { return bar0 + 8 * (2 * kMaxP + s); };
    auto AE = [&](int s) { return bar0 + 8 * (2 * kMaxP + kMaxA + s); };
    int s = 0, sc = 0;  // packed slot, stage chunk (chunk c % NC), with their phases
    uint32_t sph = 0, aph = 0;
    const bool live = row < ntiles * 16;
    for (int c = 0; c < nchunks; c++) {
        if (!mbar_wait(PF(s), sph)) return false;
        uint32_t v[32];  // column i of the k-block: values 2 i, 2 i + 1
        if (live) {
            const uint8_t *slot = pk + (size_t)s * 8 * CB;
            RowHalf<DT> r0;
            r0.template begin1<J>(slot, row, 0);
            RowHalf<DT> r1 = r0;
            r1.hf = 1;
            if (DT == GGUF_Q6_K) r1.template begin1<J>(slot, row, 1);
            uint32_t h[16];
            int cc[4];
            r0.template compute<J>(h, cc);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int u = 0; u < 4; u++) v[4 * cc[i] + u] = h[4 * i + u];
            r1.template compute<J>(h, cc);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int u = 0; u < 4; u++) v[4 * cc[i] + u] = h[4 * i + u];
        } else {  // rows past the weight (their outputs are not stored)
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = 0u;
        }
        const int st = 4 * sc + J;
        if (c >= NC && !mbar_wait(AE(st), aph ^ 1)) return false;  // the MMAs of chunk c - NC are done
        tc_fence_after();
        tmem_st32(ta0 + (uint32_t)st * kTmemStage, v);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(AF(st));
            mbar_arrive(PE(s));
        }
        if (++sc == NC) {
            sc = 0;
            aph ^= 1;
        }
        if (++s == NP) {
            s = 0;
            sph ^= 1;
        }
    }
    return true;
}

template <int DT, int G>
__device__ __forceinline__ bool dequant_group(const GemmArgs &p, uint8_t *pk, uint8_t *a_st, uint32_t bar0, int row,
                                              int hf, int ntiles, int nchunks, int NP, int NA, int lane) {
    return NA >= 4 ? dequant_group_pairs<DT, G>(p, pk, a_st, bar0, row, hf, ntiles, nchunks, NP, NA, lane)
                   : dequant_group_single<DT, G>(p, pk, a_st, bar0, row, hf, ntiles, nchunks, NP, NA, lane);
}

// Expert-grouped launch: blockIdx.z selects entry z, which multiplies
// weight w[z] by the activation rows [off[set[z]], off[set[z] + 1]) into the
// same rows of y[z].  The row ranges are read on the device (written by an
// earlier kernel), so the host never waits for them; CTAs whose token tile
// lies past their entry's rows exit at once.
struct GemmGroup {
    const uint8_t *w[kGemmMaxGroup];
    const uint8_t *w2[kGemmMaxGroup];  // kGroupSwiGLU: the up weights (w: the gate weights)
    float *y[kGemmMaxGroup];
    int set[kGemmMaxGroup];
    const int32_t *off;
    int epi;                   // GroupEpilogue
    const int32_t *row_token;  // kGroupCombine: the token of each activation row
    const float *row_w;        //   and its route weight
    float *out;                //   out[token][row] += w * value
    size_t ldo;
};
struct NoGroup {};

template <int DT, class Grp, bool TA>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, const GemmArgs p,
                const __grid_constant__ Grp q) {
    constexpr int CB = chunk_bytes(DT);
    constexpr bool kGrouped = std::is_same<Grp, GemmGroup>::value;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array itself (an
    // integer round trip would turn every access into a generic one)
    uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int bn = p.bn;
    const int terms = p.lo_row ? 2 : 1;
    const int KL = p.kps_log, KPS = 1 << KL;  // k-blocks per activation stage
    const GemmSmem L = gemm_smem(DT, bn, terms, TA, KL);
    const int NB = L.b_stages, NP = L.pslots;
    const int BH = act_halves(bn, terms);  // activation stages per k-block (1, or 2 at 512 tokens)
    const size_t b_sbytes = (size_t)terms * bn / BH * kBK * 2;  // bytes of one activation stage
    uint8_t *a_st = smem + L.a;
    uint8_t *b_st = smem + L.b;
    uint8_t *pk = smem + L.packed;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bars);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem_slot);
    // barriers: packed full / empty [kMaxP each], A full / empty [kMaxA
    // each], B full / empty [kMaxB each], accumulator full
    const uint32_t bar0 = smem_u32(bars);
    auto PF = [&](int s) { return bar0 + 8 * (0 + s); };
    auto PE = [&](int s) { return bar0 + 8 * (kMaxP + s); };
    auto AF = [&](int s) { return bar0 + 8 * (2 * kMaxP + s); };
    auto AE = [&](int s) { return bar0 + 8 * (2 * kMaxP + kMaxA + s); };
    auto BF = [&](int s) { return bar0 + 8 * (2 * kMaxP + 2 * kMaxA + s); };
    auto BE = [&](int s) { return bar0 + 8 * (2 * kMaxP + 2 * kMaxA + kMaxB + s); };
    const uint32_t ACC = bar0 + 8 * (2 * kMaxP + 2 * kMaxA + 2 * kMaxB);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // SwiGLU epilogue (grouped): the CTA's tiles are gate / up tile pairs,
    // gate and up tile hb + t / 2 at tile t = even / odd, so that a lane
    // quadrant holds 16 gate rows (lanes 0-15) and the same 16 up rows
    int gepi = kGroupStore;
    if constexpr (kGrouped) gepi = q.epi;
    const bool swiglu = gepi == kGroupSwiGLU;
    const int hb = blockIdx.x * 4;     // SwiGLU: first gate / up tile of this CTA
    const int tile0 = blockIdx.x * 8;  // first 16-row tile of this CTA
    const int ntiles = swiglu ? 2 * min(4, p.g.n_tiles - hb) : min(8, p.g.n_tiles - tile0);
    // this CTA's weight, output and activation rows t_begin + tok0 ..
    const uint8_t *wt = p.w, *wt2 = nullptr;
    float *yo = p.y;
    int t_begin = 0, t_count = p.t_rows;
    if constexpr (kGrouped) {
        const int z = blockIdx.z;
        wt = q.w[z];
        wt2 = q.w2[z];
        yo = q.y[z];
        t_begin = q.off[q.set[z]];
        t_count = q.off[q.set[z] + 1] - t_begin;
    }
    const int tok0 = blockIdx.y * bn;
    if (tok0 >= t_count) return;  // the whole CTA, before any barrier or tensor memory
    const int live = min(bn, t_count - tok0);  // tokens of this tile
    // activation rows loaded per k-block (whole boxes) and MMA width
    const int b_rows = kGrouped ? (live + p.box_rows - 1) / p.box_rows * p.box_rows : bn;
    const int ncol = kGrouped ? (live + 15) / 16 * 16 : bn;
    // two terms: the low rows follow the b_rows high rows of a stage, so
    // the MMA's N covers b_rows + ncol rows and accumulator column c's low
    // part sits at column b_rows + c
    const int nmma = terms == 2 ? b_rows + ncol : ncol;
    // split-K (dense launches): this CTA's chunks [ch0, ch0 + nchunks) of K
    const int sz = kGrouped ? 0 : (int)blockIdx.z;
    const int ch0 = kGrouped ? 0 : sz * p.g.n_chunks / p.splits;
    const int nchunks = (kGrouped ? p.g.n_chunks : (sz + 1) * p.g.n_chunks / p.splits) - ch0;
    const int nkb = nchunks * 4;
    // MMA issuers (an issuer per stage at most), their accumulators from
    // column 0; with A in tensor memory (TA) the stages follow them, at
    // least 256 columns, in whole chunks (4 k-blocks)
    const uint32_t acc_cols = tmem_cols(terms * bn);
    int MW = min(mma_warps(bn, terms), NB);
    if (TA) MW = min(MW, (int)(256u / acc_cols));
    else MW = min(MW, L.a_stages);
    const uint32_t a_col = TA ? acc_cols * (uint32_t)MW : 0u;
    const int NA = TA ? min((int)((kTmemCols - a_col) / kTmemStage) & ~3, kMaxA) : L.a_stages;
    const uint32_t ncols = TA ? kTmemCols : acc_cols * (uint32_t)MW;

    if (tid == 0) {
        for (int s = 0; s < NP; s++) {
            mbar_init(PF(s), 1);
            mbar_init(PE(s), kDqWarps);
        }
        for (int s = 0; s < NA; s++) {
            mbar_init(AF(s), TA ? 4 : kDqWarps / 2);  // four quadrant warps / one group fill a stage
            mbar_init(AE(s), 1);
        }
        for (int s = 0; s < NB; s++) {
            mbar_init(BF(s), 1);
            mbar_init(BE(s), min(MW, KPS));  // each issuer with k-blocks in the stage commits once
        }
        mbar_init(ACC, MW);  // each MMA warp's final commit
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {  // tensor memory for the bn f32 accumulator columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp == kWeightWarp) {
        // packed T16 chunks (the weights do not depend on the previous kernel)
        if (lane == 0) {
            // stage s and phase ph of chunk c, advanced without division
            int c = 0, s = 0;
            uint32_t ph = 0;
            for (; c < nchunks; c++) {
                if (c >= NP && !mbar_wait(PE(s), ph ^ 1)) {
                    ok = false;
                    break;
                }
                if (kGrouped) {  // one bulk copy per tile (each entry its own weight)
                    mbar_expect_tx(PF(s), (uint32_t)(ntiles * CB));
                    for (int t = 0; t < ntiles; t++) {
                        const uint8_t *src = swiglu ? (t & 1 ? wt2 : wt) : wt;
                        const int tile = swiglu ? hb + (t >> 1) : tile0 + t;
                        bulk_g2s(smem_u32(pk + (size_t)(s * 8 + t) * CB),
                                 src + ((size_t)tile * p.g.n_chunks + ch0 + c) * CB, CB, PF(s));
                    }
                } else {  // the 8 tiles' chunk in one tensor copy (tiles past the weight read as zeros)
                    mbar_expect_tx(PF(s), (uint32_t)(8 * CB));
                    tma_4d(smem_u32(pk + (size_t)s * 8 * CB), &wmap, ch0 + c, tile0, PF(s));
                }
                if (++s == NP) {
                    s = 0;
                    ph ^= 1;
                }
            }
            if (!ok)  // let every copy this thread issued land before the CTA exits
                for (int u = max(0, c - NP); u < c; u++) mbar_wait(PF(u % NP), (u / NP) & 1);
        }
    } else if (warp == kActWarp) {
        // activation k-blocks: the prep kernel just before this one writes Xh
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0 && KPS > 1) {
            // one copy per stage: kps k-blocks x terms x bn rows
            const uint32_t sbytes = (uint32_t)(terms * bn * kBK * 2) << KL;
            const int nst = nkb >> KL;
            int cs = 0, st = 0;
            uint32_t ph = 0;
            for (; cs < nst; cs++) {
                if (cs >= NB && !mbar_wait(BE(st), ph ^ 1)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(BF(st), sbytes);
                tma_act4(smem_u32(b_st + (size_t)st * sbytes), &xmap, tok0, 4 * ch0 + (cs << KL), BF(st));
                if (++st == NB) {
                    st = 0;
                    ph ^= 1;
                }
            }
            if (!ok)
                for (int u = max(0, cs - NB); u < cs; u++) mbar_wait(BF(u % NB), (u / NB) & 1);
        } else if (lane == 0 && BH == 2) {
            // the 512-token tile: stage f holds rows 256 (f % 2) .. + 255 of
            // k-block f / 2 (one term)
            int f = 0, st = 0;
            uint32_t ph = 0;
            for (; f < 2 * nkb; f++) {
                if (f >= NB && !mbar_wait(BE(st), ph ^ 1)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(BF(st), (uint32_t)b_sbytes);
                tma_2d(smem_u32(b_st + (size_t)st * b_sbytes), &xmap, (4 * ch0 + (f >> 1)) * kBK,
                       t_begin + tok0 + 256 * (f & 1), BF(st));
                if (++st == NB) {
                    st = 0;
                    ph ^= 1;
                }
            }
            if (!ok)
                for (int u = max(0, f - NB); u < f; u++) mbar_wait(BF(u % NB), (u / NB) & 1);
        } else if (lane == 0) {
            int kb = 0, st = 0;
            uint32_t ph = 0;
            for (; kb < nkb; kb++) {
                if (kb >= NB && !mbar_wait(BE(st), ph ^ 1)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(BF(st), (uint32_t)(terms * b_rows * kBK * 2));
                uint8_t *dst = b_st + (size_t)st * b_sbytes;
                for (int r0 = 0; r0 < b_rows; r0 += p.box_rows) {  // a tensor-map box is at most 256 rows
                    const int kx = (4 * ch0 + kb) * kBK;
                    tma_2d(smem_u32(dst + (size_t)r0 * kBK * 2), &xmap, kx, t_begin + tok0 + r0, BF(st));
                    if (terms == 2)
                        tma_2d(smem_u32(dst + (size_t)(b_rows + r0) * kBK * 2), &xmap, kx,
                               p.lo_row + t_begin + tok0 + r0, BF(st));
                }
                if (++st == NB) {
                    st = 0;
                    ph ^= 1;
                }
            }
            if (!ok)
                for (int u = max(0, kb - NB); u < kb; u++) mbar_wait(BF(u % NB), (u / NB) & 1);
        }
    } else if (TA && warp >= 1 && warp <= kDqWarps) {
        const int qd = warp & 3, j = (warp - 1) >> 2;
        const int row = 32 * qd + lane;
        const uint32_t ta0 = tmem + ((uint32_t)(32 * qd) << 16) + a_col;
        const int NC = NA / 4;
        switch (j) {
        case 0: ok = dequant_tmem<DT, 0>(pk, bar0, ta0, row, ntiles, nchunks, NP, NC, lane); break;
        case 1: ok = dequant_tmem<DT, 1>(pk, bar0, ta0, row, ntiles, nchunks, NP, NC, lane); break;
        case 2: ok = dequant_tmem<DT, 2>(pk, bar0, ta0, row, ntiles, nchunks, NP, NC, lane); break;
        default: ok = dequant_tmem<DT, 3>(pk, bar0, ta0, row, ntiles, nchunks, NP, NC, lane); break;
        }
    } else if (warp >= 1 && warp <= kDqWarps) {
        // dequantisers: two groups of eight warps take alternate k-blocks
        // (each warp has two k-blocks' time for its chain of waits, loads,
        // arithmetic and stores); two threads per weight row, 32 values each
        const int grp = (warp - 1) / (kDqWarps / 2);
        const int gt = tid - 32 - grp * (kDqWarps / 2) * 32;
        const int row = gt >> 1, hf = gt & 1;
        if (grp == 0)
            ok = dequant_group<DT, 0>(p, pk, a_st, bar0, row, hf, ntiles, nchunks, NP, NA, lane);
        else
            ok = dequant_group<DT, 1>(p, pk, a_st, bar0, row, hf, ntiles, nchunks, NP, NA, lane);
    } else if (warp >= kMmaWarp && warp < kMmaWarp + MW) {
        // MMA issuer w takes k-blocks w, w + MW, ... into its own accumulator
        // (columns w * acc_cols ..); per k-block, bn / 256 (at least one)
        // sub-accumulators of up to 256 columns, 4 instructions of K = 16.
        // The whole warp runs the loop, one elected lane issues; descriptors
        // advance by 32 bytes (2 in the >> 4 address field) per K = 16 step
        // and by a whole stage per stage.
        const int w = warp - kMmaWarp;
        const int nsub = nmma > 256 ? nmma / 256 : 1, nw = nmma > 256 ? 256 : nmma;
        const uint32_t idesc = idesc_f16(nw);
        const uint32_t acc = tmem + (uint32_t)w * acc_cols;
        {
            const uint64_t da0 = sw128_desc(smem_u32(a_st)), db0 = sw128_desc(smem_u32(b_st));
            const uint64_t a_step = (uint64_t)(kBM * kBK * 2) >> 4, b_step = (uint64_t)b_sbytes >> 4;
            const uint64_t h_step = (uint64_t)(256 * kBK * 2) >> 4;
            // A stage of k-block kb = w; activation stage sb of stage index bi (k-blocks bi * KPS ..)
            int sa = w, sb = 0, bi = 0;
            uint32_t aph = 0, bph = 0;
            const uint64_t bs_step = b_step << KL;
            // the 512-token tile (one issuer, A in shared memory): half h of
            // k-block kb is activation stage 2 kb + h, released once its
            // four MMAs are done; each half's N covers only its live tokens
            const int nlive = (live + 15) / 16 * 16;
            const int n0 = min(256, nlive), n1 = min(256, max(0, nlive - 256));
            const uint32_t id0 = idesc_f16(max(n0, 16)), id1 = idesc_f16(max(n1, 16));
            for (int kb = 0; BH == 2 && kb < nkb; kb++) {
                if (!__all_sync(0xffffffffu, mbar_wait(AF(sa), aph))) {
                    ok = false;
                    break;
                }
                const uint64_t da = da0 + (uint64_t)sa * a_step;
                for (int h = 0; h < 2 && ok; h++) {
                    if (!__all_sync(0xffffffffu, mbar_wait(BF(sb), bph))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t db = db0 + (uint64_t)sb * b_step;
                    if ((h ? n1 : n0) > 0)
#pragma unroll
                        for (int k = 0; k < kBK / 16; k++)
                            umma_f16(acc + (uint32_t)(h * 256), da + 2 * k, db + 2 * k, h ? id1 : id0,
                                     (kb || k) ? 1u : 0u);
                    umma_commit(BE(sb));
                    if (++sb == NB) {
                        sb = 0;
                        bph ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(AE(sa));
                if (++sa == NA) {
                    sa = 0;
                    aph ^= 1;
                }
            }
            for (int kb = w; BH == 1 && kb < nkb; kb += MW) {
                for (; bi < (kb >> KL); bi++)
                    if (++sb == NB) {
                        sb = 0;
                        bph ^= 1;
                    }
                const bool got = mbar_wait(AF(sa), aph) && mbar_wait(BF(sb), bph);
                if (!__all_sync(0xffffffffu, got)) {  // (the lanes leave together)
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t da = da0 + (uint64_t)sa * a_step,
                               db = db0 + (uint64_t)sb * bs_step + (uint64_t)(kb & (KPS - 1)) * b_step;
                if (TA) {
                    const uint32_t ta = tmem + a_col + (uint32_t)sa * kTmemStage;
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)  // 16 fp16 = 8 columns of A, 32 bytes of B
                        umma_f16_ta(acc, ta + 8 * k, db + 2 * k, idesc, (kb != w || k) ? 1u : 0u);
                } else {
                    for (int h = 0; h < nsub; h++) {
#pragma unroll
                        for (int k = 0; k < kBK / 16; k++)  // 16 fp16 = 32 bytes per instruction
                            umma_f16(acc + (uint32_t)(h * 256), da + 2 * k, db + (uint64_t)h * h_step + 2 * k,
                                     idesc, (kb != w || k) ? 1u : 0u);
                    }
                }
                umma_commit(AE(sa));
                // this issuer's last k-block of the stage: it may refill once these MMAs are done
                if (((kb + MW) >> KL) != (kb >> KL) || kb + MW >= nkb) umma_commit(BE(sb));
                sa += MW;
                if (sa >= NA) {
                    sa -= NA;
                    aph ^= 1;
                }
            }
            umma_commit(ACC);  // arrives once this warp's MMAs above have completed
        }
        __syncwarp();
    }

    // epilogue: dequantiser warp w owns tensor-memory lanes 32 * (w % 4) ..
    // + 31 (the only lanes a warp may read) and one of four column groups
    if (warp >= 1 && warp <= kDqWarps) {
        if (ok && !mbar_wait(ACC, 0)) ok = false;
        if constexpr (kGrouped) ok = __all_sync(0xffffffffu, ok);  // (the SwiGLU epilogue exchanges values between lanes)
        tc_fence_after();
        const int lane_base = 32 * (warp & 3);
        const int cpg = (ncol / 8 + 3) / 4 * 8;  // columns per group, a multiple of 8
        const int c_begin = ((warp - 1) >> 2) * cpg, c_end = min(ncol, c_begin + cpg);
        const int row = tile0 * 16 + lane_base + lane;
        if (ok) {
            for (int c0 = c_begin; c0 < c_end; c0 += 8) {
                float v[8];
                for (int w = 0; w < MW; w++) {  // the issuers' accumulators, added in order
                    for (int h = 0; h < terms; h++) {  // high part, then low part
                        uint32_t r[8];
                        const uint32_t col = (uint32_t)w * acc_cols + (uint32_t)(c0 + h * b_rows);
                        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                                       "=r"(r[6]), "=r"(r[7])
                                     : "r"(tmem + ((uint32_t)lane_base << 16) + col));
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            v[i] = (w || h) ? v[i] + __uint_as_float(r[i]) : __uint_as_float(r[i]);
                    }
                }
                if (swiglu) {
                    // h = silu(g) * u for h row hrow: lanes l and l + 16 hold its gate
                    // and up values; after one exchange each of the two computes h
                    // for half of the 8 tokens (lane l tokens 0-3, lane l + 16 tokens 4-7)
                    const int hrow = hb * 16 + 16 * (warp & 3) + (lane & 15);
                    const bool up_lane = lane & 16;
                    float g4[4], u4[4];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int t = t_begin + tok0 + c0 + i;
                        const float o = c0 + i < live ? v[i] * p.inv_scale[t] : 0.f;
                        const float other = __shfl_xor_sync(0xffffffffu, o, 16);
                        if ((i < 4) == !up_lane) {
                            g4[i & 3] = up_lane ? other : o;
                            u4[i & 3] = up_lane ? o : other;
                        }
                    }
                    if (hrow < p.g.n_rows)
#pragma unroll
                        for (int i4 = 0; i4 < 4; i4++) {
                            const int i = (up_lane ? 4 : 0) + i4;
                            if (c0 + i < live)
                                yo[(size_t)(t_begin + tok0 + c0 + i) * p.ldy + hrow] = __fmul_rn(silu_fast(g4[i4]), u4[i4]);
                        }
                } else if (gepi == kGroupCombine) {
                    if constexpr (kGrouped) {
                        if (row < p.g.n_rows)
#pragma unroll
                            for (int i = 0; i < 8; i++) {
                                const int t = t_begin + tok0 + c0 + i;
                                if (c0 + i < live)
                                    atomicAdd(q.out + (size_t)q.row_token[t] * q.ldo + row,
                                              __fmul_rn(q.row_w[t], v[i] * p.inv_scale[t]));
                            }
                    }
                } else if (row < p.g.n_rows) {
                    // split-K: this CTA's partial sums, added in order by reduce_splits
                    float *dst = p.splits > 1 ? p.part + (size_t)sz * p.t_rows * p.g.n_rows : yo;
                    const size_t ld = p.splits > 1 ? (size_t)p.g.n_rows : p.ldy;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int t = t_begin + tok0 + c0 + i;
                        if (c0 + i < live) {
                            const float o = v[i] * p.inv_scale[t];
                            dst[(size_t)t * ld + row] = o;
                            // the fused all-gather: the same value into every
                            // peer's bulk buffer, over NVLink
                            if (p.push.world > 1)
                                for (int q = 0; q < p.push.world; q++)
                                    if (q != p.push.rank) p.push.peer[q][(size_t)t * p.ldy + row] = o;
                        }
                    }
                }
            }
        }
    }
    if (!ok && lane == 0) *reinterpret_cast<volatile int *>(p.err) = kKernelErrWaitTimeout;
    tc_fence_before();
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == kMmaWarp) {
        mbar_wait(ACC, 0);  // no MMA may still write the accumulator (returns at once when done)
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// X f32 [t][ldx] -> Xh fp16 [t][k] with x * 2^e, |x * 2^e| < 2^14, and 1/2^e;
// with xl, also the low terms [t][k].
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(const float *x, size_t ldx, int k, __half *xh,
                                                             float *inv, __half *xl) {
    const int t = blockIdx.x;
    const float *xr = x + (size_t)t * ldx;
    prep_row([&](int i) { return xr[i]; }, k, xh + (size_t)t * k, inv + t, xl ? xl + (size_t)t * k : nullptr);
}

// y[t][r] = sum over z, in order, of part[z][t][r] (split-K partials); with
// a fused bulk all-gather also into every peer's bulk buffer.
__global__ void reduce_splits_kernel(const float *part, int splits, int t_rows, int64_t n, float *y, size_t ldy,
                                     BulkPush push) {
    const size_t total = (size_t)t_rows * (size_t)n;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        float v = part[i];
        for (int z = 1; z < splits; z++) v += part[(size_t)z * total + i];
        const size_t o = (i / (size_t)n) * ldy + i % (size_t)n;
        y[o] = v;
        if (push.world > 1)
            for (int q = 0; q < push.world; q++)
                if (q != push.rank) push.peer[q][o] = v;
    }
}

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

template <int DT, class Grp, bool TA>
cudaError_t launch_dt(const CUtensorMap &map, const CUtensorMap &wmap, const GemmArgs &a, const Grp &q, dim3 grid,
                      size_t smem, cudaStream_t s) {
    static std::atomic<unsigned long long> done{0};
    auto kern = gemm_kernel<DT, Grp, TA>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
    if (!bit || !(done.load() & bit)) {
        int optin = 0;
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, kern);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
        if (e != cudaSuccess) return e;
        if (bit) done.fetch_or(bit);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, map, wmap, a, q);
}

template <class Grp, bool TA>
cudaError_t launch_ta(int dt, const CUtensorMap &map, const CUtensorMap &wmap, const GemmArgs &a, const Grp &q,
                      dim3 grid, size_t smem, cudaStream_t s) {
    switch (dt) {
    case GGUF_Q4_K: return launch_dt<GGUF_Q4_K, Grp, TA>(map, wmap, a, q, grid, smem, s);
    case GGUF_Q4_0: return launch_dt<GGUF_Q4_0, Grp, TA>(map, wmap, a, q, grid, smem, s);
    case GGUF_Q8_0: return launch_dt<GGUF_Q8_0, Grp, TA>(map, wmap, a, q, grid, smem, s);
    case GGUF_Q6_K: return launch_dt<GGUF_Q6_K, Grp, TA>(map, wmap, a, q, grid, smem, s);
    case GGUF_Q5_K: return launch_dt<GGUF_Q5_K, Grp, TA>(map, wmap, a, q, grid, smem, s);
    default: return cudaErrorInvalidValue;
    }
}

// A in tensor memory when the accumulators leave it room: 256 columns of
// accumulator at most (token tiles up to 256 one-term / 128 two-term
// columns); the 512-token tile keeps the shared-memory A tile.
inline bool tmem_a(int bn, int terms) { return tmem_cols(terms * bn) <= 256; }

template <class Grp>
cudaError_t launch_any(int dt, const CUtensorMap &map, const CUtensorMap &wmap, const GemmArgs &a, const Grp &q,
                       dim3 grid, int terms, cudaStream_t s) {
    const bool ta = tmem_a(a.bn, terms);
    const GemmSmem lay = gemm_smem(dt, a.bn, terms, ta, a.kps_log);
    if (lay.pslots < 2) return cudaErrorInvalidConfiguration;
    return ta ? launch_ta<Grp, true>(dt, map, wmap, a, q, grid, lay.total, s)
              : launch_ta<Grp, false>(dt, map, wmap, a, q, grid, lay.total, s);
}

// Tensor map of the fp16 activations [rows][k] (128-byte swizzle, boxes of
// 64 columns x box_rows rows).
cudaError_t act_map(CUtensorMap *map, const void *xh, int rows, int64_t k, int box_rows) {
    EncodeTiled enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(xh), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Tensor map of a T16 weight as 4-d uint8: (piece bytes, pieces of a chunk,
// chunks, tiles), so that one copy with box (piece, pieces, 1, 8) brings one
// chunk of 8 consecutive tiles, tile by tile, as the shared-memory slot holds
// them.  A piece is the largest multiple of 16 bytes up to 256 dividing the
// chunk (256 for Q4_K / Q4_0 / Q8_0 / Q5_K, 240 for Q6_K's 3360).
cudaError_t weight_map(CUtensorMap *map, const uint8_t *tiles, const Geometry &g, int dt) {
    EncodeTiled enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const int cb = chunk_bytes(dt);
    int ip = 256;
    while (ip > 16 && cb % ip) ip -= 16;
    const cuuint64_t dims[4] = {(cuuint64_t)ip, (cuuint64_t)(cb / ip), (cuuint64_t)g.n_chunks, (cuuint64_t)g.n_tiles};
    const cuuint64_t strides[3] = {(cuuint64_t)ip, (cuuint64_t)cb, (cuuint64_t)g.n_chunks * (cuuint64_t)cb};
    const cuuint32_t box[4] = {(cuuint32_t)ip, (cuuint32_t)(cb / ip), 1, 8};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(tiles), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Tensor map of the fp16 activations [terms][rows][k] as 4-d (64 columns,
// rows, terms, k-blocks), 128-byte swizzle, box (64, bn, terms, kps): one
// copy fills an activation stage laid out [k-block][term][row][64], each
// k-block's rows of both terms one 1024-byte-aligned swizzled tile.
cudaError_t act_map4(CUtensorMap *map, const void *xh, int rows, int64_t k, int terms, int bn, int kps) {
    EncodeTiled enc = encode_fn();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[4] = {(cuuint64_t)kBK, (cuuint64_t)rows, (cuuint64_t)terms, (cuuint64_t)(k / kBK)};
    const cuuint64_t strides[3] = {(cuuint64_t)k * 2, (cuuint64_t)k * 2 * (cuuint64_t)rows, (cuuint64_t)kBK * 2};
    const cuuint32_t box[4] = {(cuuint32_t)kBK, (cuuint32_t)bn, (cuuint32_t)terms, (cuuint32_t)kps};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void *>(xh), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

int gemm_bn(int dt, int t_rows) {
    // over 256 tokens: 512-token tiles, whose two N = 256 accumulators fill
    // tensor memory, so each weight tile is dequantised once per 512 tokens
    // (a tile's MMAs cover only its live tokens)
    if (t_rows > 256) return 512;
    if (t_rows >= 256) return 256;
    int bn = (t_rows + 15) / 16 * 16;
    return bn < 16 ? 16 : bn;
}

int gemm_terms(int t_rows) { return t_rows <= kGemmTwoTermMaxTokens ? 2 : 1; }

namespace {

int device_sms() {
    static std::atomic<int> sms_cache[64];
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
        sms = sms_cache[dev].load();
        if (sms <= 0) {
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
            sms_cache[dev].store(sms);
        }
    }
    return sms;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// The dense launch's plan: token tile, K splits and workspace bytes.  When
// the row blocks and token tiles alone would leave most SMs idle (weights
// of few rows: row shards), the CTAs split K -- each a contiguous range of
// chunks, partial outputs summed in order by reduce_splits -- into as many
// splits as the SMs take and the workspace (fp16 activations, inverse
// scales, partials) fits kGemmSplitWorkspace, after narrowing the token tile
// to 128 (more CTAs, each weight tile dequantised once per bn tokens); with
// no room for partials the tile narrows on to 64.  The plan
// depends on the shape, t_rows and the SM count only.
struct GemmPlan {
    int bn = 16, splits = 1, terms = 1;
    size_t xh_bytes = 0, inv_bytes = 0, part_bytes = 0;
    size_t total() const { return xh_bytes + inv_bytes + part_bytes; }
};

GemmPlan plan_dense(int dt, const Geometry &g, int t_rows) {
    GemmPlan pl;
    pl.terms = gemm_terms(t_rows);
    pl.bn = gemm_bn(dt, t_rows);
    pl.xh_bytes = align256((size_t)pl.terms * t_rows * g.n_cols * 2);
    pl.inv_bytes = align256((size_t)t_rows * 4);
    const long sms = device_sms();
    const long rbs = (g.n_tiles + 7) / 8;
    auto ctas = [&](int bn) { return rbs * ((t_rows + bn - 1) / bn); };
    auto idle = [&](int bn) { return ctas(bn) * 10 < sms * 6; };
    if (!idle(pl.bn)) return pl;
    // token tiles down to 128 first (a 512-token tile's two N = 256
    // accumulators leave one MMA issuer), then K splits
    while (pl.bn > 128 && idle(pl.bn)) pl.bn = (pl.bn / 2 + 15) / 16 * 16;
    if (!idle(pl.bn)) return pl;
    long sp = sms / ctas(pl.bn);
    if (sp > g.n_chunks) sp = g.n_chunks;
    const size_t part1 = (size_t)t_rows * (size_t)g.n_rows * 4;
    while (sp >= 2 && pl.xh_bytes + pl.inv_bytes + align256((size_t)sp * part1) > kGemmSplitWorkspace) sp--;
    if (sp >= 2) {
        pl.splits = (int)sp;
        pl.part_bytes = align256((size_t)sp * part1);
        return pl;
    }
    // (bn stays a multiple of 16: the MMA's N step at M = 128, and whole
    // 1024-byte swizzle atoms per activation stage)
    while (pl.bn > 64 && idle(pl.bn)) pl.bn = (pl.bn / 2 + 15) / 16 * 16;
    return pl;
}

}  // namespace

size_t gemm_workspace_bytes(int dt, const Geometry &g, int t_rows) { return plan_dense(dt, g, t_rows).total(); }

cudaError_t launch_gemm(int dt, const uint8_t *tiles, const Geometry &g, const float *x, size_t ldx, float *y,
                        size_t ldy, int t_rows, void *workspace, int *err, cudaStream_t s, const BulkPush *push) {
    if (t_rows <= 0 || g.n_rows <= 0) return cudaSuccess;
    if (push && (push->world > kMaxPeers || push->rank < 0 || push->rank >= push->world)) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    const GemmPlan pl = plan_dense(dt, g, t_rows);
    // workspace: [terms][t_rows][n_cols] fp16 activations (high terms, then
    // low), the per-token inverse scales, the split-K partials
    const int terms = pl.terms, bn = pl.bn;
    __half *xh = static_cast<__half *>(workspace);
    float *inv = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + pl.xh_bytes);
    float *part = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + pl.xh_bytes + pl.inv_bytes);
    prep_kernel<<<t_rows, kPrepThreads, 0, s>>>(x, ldx, (int)g.n_cols, xh, inv,
                                                terms == 2 ? xh + (size_t)t_rows * g.n_cols : nullptr);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap map;
    const int box_rows = bn < 256 ? bn : 256;
    int kl = act_kps_log(bn, terms, tmem_a(bn, terms));
    if (kl > 0 && act_map4(&map, xh, t_rows, g.n_cols, terms, bn, 1 << kl) != cudaSuccess) kl = 0;
    if (kl == 0) {
        e = act_map(&map, xh, terms * t_rows, g.n_cols, box_rows);
        if (e != cudaSuccess) return e;
    }
    GemmArgs a;
    a.kps_log = kl;
    a.lo_row = terms == 2 ? t_rows : 0;
    a.splits = pl.splits;
    a.part = part;
    if (push && push->world > 1 && pl.splits == 1) a.push = *push;
    a.w = tiles;
    a.y = y;
    a.inv_scale = inv;
    a.err = err;
    a.g = g;
    a.ldy = ldy;
    a.t_rows = t_rows;
    a.bn = bn;
    a.box_rows = box_rows;
    CUtensorMap wmap;
    e = weight_map(&wmap, tiles, g, dt);
    if (e != cudaSuccess) return e;
    dim3 grid((g.n_tiles + 7) / 8, (t_rows + bn - 1) / bn, pl.splits);
    e = launch_any(dt, map, wmap, a, NoGroup{}, grid, terms, s);
    if (e != cudaSuccess || pl.splits == 1) return e;
    const size_t total = (size_t)t_rows * (size_t)g.n_rows;
    unsigned blocks = (unsigned)((total + 255) / 256);
    if (blocks > 1184) blocks = 1184;
    reduce_splits_kernel<<<blocks, 256, 0, s>>>(part, pl.splits, t_rows, g.n_rows, y, ldy,
                                                push && push->world > 1 ? *push : BulkPush{});
    return cudaGetLastError();
}

// Token tile of a grouped launch.
static int gemm_grouped_bn(int rows, int n_sets, int max_rows) {
    // twice the average rows per set, in whole 64-row boxes, 64 ..
    // kTwoTermMaxTile (two-term activations): sets up to that size are one
    // token tile (each weight tile dequantised once)
    const long avg2 = n_sets > 0 ? (2L * rows + n_sets - 1) / n_sets : rows;
    long bn = (avg2 + 63) / 64 * 64;
    if (bn > (long)(max_rows + 63) / 64 * 64) bn = (long)(max_rows + 63) / 64 * 64;
    return (int)(bn < 64 ? 64 : (bn > kTwoTermMaxTile ? kTwoTermMaxTile : bn));
}

cudaError_t launch_gemm_grouped(int dt, const uint8_t *const *ws, float *const *ys, const int *set, int n,
                                const Geometry &g, const void *xh, const float *inv, int rows, int rows_hint,
                                const int32_t *off, int n_sets, int max_rows, size_t ldy, int *err, cudaStream_t s,
                                const GroupEpi &epi) {
    if (n <= 0 || rows <= 0 || max_rows <= 0 || g.n_rows <= 0) return cudaSuccess;
    if (n > kGemmMaxGroup || n_sets <= 0) return cudaErrorInvalidValue;
    if (!encode_fn()) return cudaErrorNotSupported;
    const int bn = gemm_grouped_bn(rows_hint, n_sets, max_rows);
    constexpr int kBox = 64;
    CUtensorMap map;
    cudaError_t e = act_map(&map, xh, 2 * rows, g.n_cols, kBox);  // high rows, then low rows
    if (e != cudaSuccess) return e;
    GemmArgs a;
    a.lo_row = rows;
    a.splits = 1;
    a.part = nullptr;
    a.w = nullptr;
    a.y = nullptr;
    a.inv_scale = inv;
    a.err = err;
    a.g = g;
    a.ldy = ldy;
    a.t_rows = 0;
    a.bn = bn;
    a.box_rows = kBox;
    a.kps_log = 0;
    if (epi.mode == kGroupSwiGLU && !epi.ws2) return cudaErrorInvalidValue;
    if (epi.mode == kGroupCombine && (!epi.row_token || !epi.row_w || !epi.out)) return cudaErrorInvalidValue;
    GemmGroup q;
    for (int z = 0; z < kGemmMaxGroup; z++) {
        q.w[z] = z < n ? ws[z] : nullptr;
        q.w2[z] = z < n && epi.mode == kGroupSwiGLU ? epi.ws2[z] : nullptr;
        q.y[z] = z < n ? ys[z] : nullptr;
        q.set[z] = z < n ? set[z] : 0;
        if (z < n && (set[z] < 0 || set[z] >= n_sets)) return cudaErrorInvalidValue;
    }
    q.off = off;
    q.epi = epi.mode;
    q.row_token = epi.row_token;
    q.row_w = epi.row_w;
    q.out = epi.out;
    q.ldo = epi.ldo;
    if ((max_rows + bn - 1) / bn > 65535) return cudaErrorInvalidValue;
    // SwiGLU: 4 gate and 4 up tiles per CTA
    dim3 grid(epi.mode == kGroupSwiGLU ? (g.n_tiles + 3) / 4 : (g.n_tiles + 7) / 8, (max_rows + bn - 1) / bn, n);
    return launch_any(dt, map, map, a, q, grid, 2, s);  // (grouped weights: bulk copies, no weight map)
}

}  // namespace rce
