// qmm_layout.cuh -- the device weight layout ("T16") shared by every kernel.
//
// A registered GGUF weight [n_rows][n_cols] is repacked once, on the device,
// into tiles of 16 rows x 256 columns ("chunks").  The repack is a byte
// permutation (plus, for Q4_K, a bit permutation of the 12 packed scale
// bytes), so the device holds exactly the GGUF byte count per real row and
// the GGUF bytes can be recovered bit for bit (unpack kernel).
//
// Chunks are stored tile-major: chunk (tile t, column-chunk c) lives at
//   base + (t * n_chunks + c) * chunk_bytes(dtype).
// Inside a chunk the quant bytes come first, ordered so that load i of
// lane L of a warp reads the 16 bytes at (i * 32 + L) * 16: every warp-wide
// 128-bit load is one contiguous 512-byte segment.  Lane L = 4 r + g works on
// rows r and r + 8 of the tile and on the 64 columns [64 g, 64 g + 64) of the
// chunk; element (g, step j, slot s) is column 64 g + 4 j + s for every
// format, which is what lets one activation table serve all three.
//
//   Q4_K (144 B per 256 values; chunk 2304 B):
//     quants [i 0..3][lane][16 B]: row r + 8 (i >> 1), qs bytes
//       [32 g + 16 (i & 1), +16) of the super-block (group g = sub-blocks
//       2g (low nibbles) and 2g + 1 (high nibbles));
//     header [row 0..15][16 B]: d (f16), dmin (f16), then for g = 0..3 a
//       24-bit little-endian field sc(2g) | m(2g) << 6 | sc(2g+1) << 12 |
//       m(2g+1) << 18 -- the same 96 bits as GGUF's 12 scale bytes, re-ordered
//       so lane g finds its two sub-blocks in one field.
//   Q4_0 (18 B per 32; chunk 2304 B):
//     quants [i 0..3][lane][16 B]: row r + 8 (i >> 1), the 16 nibble bytes of
//       block 2 g + (i & 1) of the chunk's 8 blocks;
//     scales [lane][4 x f16]: d(r, 2g), d(r, 2g+1), d(r+8, 2g), d(r+8, 2g+1).
//   Q8_0 (34 B per 32; chunk 4352 B):
//     quants [i 0..7][lane][16 B]: row r + 8 (i >> 2), bytes
//       [16 (i & 1), +16) of block 2 g + ((i >> 1) & 1);
//     scales [lane][4 x f16] as Q4_0.
//   Q5_K (176 B per 256; chunk 2816 B): Q4_K's quants and headers (the
//     low four bits of every code), then the fifth bits [lane][16 B] at
//     2304: for lane (r, g) the words Y0, Y1 of row r and Y0, Y1 of row
//     r + 8, where bit 8b + j of Y_h is the fifth bit of value 64 g + 32 h +
//     4 j + b (GGUF: bit 2g + h of qh[4 j + b]) -- so (Y_h >> j) &
//     0x01010101 holds the bits of the four values a[] byte b carries.
//   Q6_K (210 B per 256; chunk 3360 B; qmm_q6k.cu): the six-bit codes
//     u = q + 32 of value v (0..255) of row r, split as in GGUF into four low
//     and two high bits but re-ordered by value: lo plane [row][128 B], byte
//     i = values 2i (low nibble) and 2i + 1 (high nibble); hi plane at 2048
//     [row][64 B], byte i = values 4i .. 4i + 3 (bits 2e, 2e + 1); the 16
//     int8 scales per row at 3072 [row][16 B] and d at 3328 [row][f16], as
//     in GGUF.  Lane L of the GEMV reads values 8L .. 8L + 7 of a row: one
//     32-bit word of the lo plane, one 16-bit word of the hi plane, scale
//     L / 2.
// Rows past n_rows and columns past n_cols are zero (zero scale and zero
// quants), so padded elements contribute exactly 0.
#pragma once
#include <cstddef>
#include <cstdint>

namespace rce {

enum : int { GGUF_F32 = 0, GGUF_F16 = 1, GGUF_Q4_0 = 2, GGUF_Q8_0 = 8, GGUF_Q4_K = 12, GGUF_Q5_K = 13, GGUF_Q6_K = 14 };

constexpr int TILE_ROWS = 16;
constexpr int CHUNK_K = 256;

__host__ __device__ constexpr int chunk_bytes(int dt) {
    return dt == GGUF_Q8_0 ? 4352 : (dt == GGUF_Q6_K ? 3360 : (dt == GGUF_Q5_K ? 2816 : 2304));
}
// Q4_K and Q5_K share the super-block header and the nibble layout.
__host__ __device__ constexpr bool kquant45(int dt) { return dt == GGUF_Q4_K || dt == GGUF_Q5_K; }
__host__ __device__ constexpr int quant_bytes(int dt) {
    return dt == GGUF_Q8_0 ? 4096 : (dt == GGUF_Q6_K ? 3072 : 2048);
}
__host__ __device__ constexpr int gguf_block(int dt) {
    return dt == GGUF_Q4_K || dt == GGUF_Q5_K || dt == GGUF_Q6_K ? 256 : 32;
}
__host__ __device__ constexpr int gguf_block_bytes(int dt) {
    return dt == GGUF_Q4_K ? 144 : (dt == GGUF_Q8_0 ? 34 : (dt == GGUF_Q6_K ? 210 : (dt == GGUF_Q5_K ? 176 : 18)));
}
inline bool dtype_supported(int dt) {
    return dt == GGUF_Q4_0 || dt == GGUF_Q8_0 || dt == GGUF_Q4_K || dt == GGUF_Q5_K || dt == GGUF_Q6_K;
}
// Q5_K fifth-bit plane offset.
constexpr int kQ5Hi = 2304;
// Q6_K chunk planes (qmm_q6k.cu).
constexpr int kQ6Hi = 2048, kQ6Sc = 3072, kQ6D = 3328;

struct Geometry {
    int64_t n_rows = 0, n_cols = 0;
    int n_tiles = 0, n_chunks = 0;
    size_t gguf_row_bytes = 0, gguf_bytes = 0, dev_bytes = 0;
};

inline Geometry make_geometry(int dt, int64_t n_rows, int64_t n_cols) {
    Geometry g;
    g.n_rows = n_rows;
    g.n_cols = n_cols;
    g.n_tiles = (int)((n_rows + TILE_ROWS - 1) / TILE_ROWS);
    g.n_chunks = (int)((n_cols + CHUNK_K - 1) / CHUNK_K);
    g.gguf_row_bytes = (size_t)(n_cols / gguf_block(dt)) * gguf_block_bytes(dt);
    g.gguf_bytes = g.gguf_row_bytes * (size_t)n_rows;
    g.dev_bytes = (size_t)g.n_tiles * g.n_chunks * chunk_bytes(dt);
    return g;
}

}  // namespace rce
