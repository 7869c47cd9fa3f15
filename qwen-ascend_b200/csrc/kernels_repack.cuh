// Load-time repack of the int4pack artifact into the tile-major layout the B200 kernels
// stream.  Run once per weight tensor when a layer is loaded; the artifact itself
// (tools/repack_w4a16.py, tools/repack_w4_em.py) is read unchanged.
//
// Input  w  int32 [E, K, Nw/8]  nibble t of word j = W[k, 8j+t], two's complement
//        s  bf16  [E, K/gs, Nw]
// Output t  int32 [E, MT, K/64, TILE_BLOCK_WORDS]: one 4352-byte block per (expert e,
//        feature tile m, k-block kb), contiguous along kb, so a tile's whole K range is one
//        linear stream and consecutive k-blocks can be fetched by one bulk copy:
//          word tile_word(c, r) = c*128 + (r ^ 8*(c%4)) (c < 8, r < 128): the 8 weights
//            W[kb*64 + 8c + i, f(m, r)] of tile row r as offset-binary nibbles (q + 8) in the
//            order i = 0,2,4,6,1,3,5,7, so that ((word >> 4i) & 0x000f000f) yields the pair
//            (k = 8c+2i, 8c+2i+1).  The XOR swizzle keeps both access patterns free of
//            shared-memory bank conflicts: one thread per tile row reading word c (the GEMM's
//            dequant warps), and the mma fragment order of the decode GEMV, where the four
//            threads of a fragment group read words c = 0..3 (and 4..7) of the same row;
//          half-word 2048 + r: the scale of tile row r for the group holding k-block kb
//            (repeated in every k-block of a group when gs > 64).
// Tile rows: PLAIN  f(m, r) = 128m + r                                 (MT = Nw / 128)
//            SWIGLU f(m, r) = (r odd ? Nw/2 : 0) + 64m + r/2  (gate/up of a feature on
//                             adjacent rows, so a SwiGLU epilogue pairs lanes 2i, 2i+1)
//                                                                        (MT = Nw / 128)
#pragma once
#include "fnx_common.cuh"

namespace fnx {

constexpr int TILE_BLOCK_WORDS = 1024 + 64;                 // 4096 B of weights + 256 B of scales
constexpr int TILE_BLOCK_BYTES = TILE_BLOCK_WORDS * 4;      // 4352

// Position of word c (8 consecutive k) of tile row r inside a tile block.
FNX_DEV int tile_word(int c, int r) { return c * 128 + (r ^ ((c & 3) << 3)); }

FNX_DEV int tile_feature(int m, int r, int Nw, bool swiglu) {
    return swiglu ? ((r & 1) ? Nw / 2 : 0) + 64 * m + (r >> 1) : 128 * m + r;
}

__global__ void __launch_bounds__(256) repack_w4_tiles_kernel(const uint32_t* __restrict__ w, const bf16* __restrict__ s,
                                                              uint32_t* __restrict__ t, int E, int K, int Nw, int gs,
                                                              int swiglu) {
    const int MT = Nw / 128, KB = K / 64, G = K / gs;
    const long long total = (long long)E * MT * KB * TILE_BLOCK_WORDS;
    const int nw8 = Nw / 8;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const int wd = (int)(o % TILE_BLOCK_WORDS);
        long long rest = o / TILE_BLOCK_WORDS;
        const int kb = (int)(rest % KB);
        rest /= KB;
        const int m = (int)(rest % MT);
        const int e = (int)(rest / MT);
        uint32_t out = 0;
        if (wd < 1024) {
            const int c = wd >> 7, r = (wd & 127) ^ ((c & 3) << 3);     // tile_word's inverse
            const int f = tile_feature(m, r, Nw, swiglu != 0);
            const int k0 = kb * 64 + 8 * c;
            const uint32_t* src = w + ((long long)e * K + k0) * nw8 + (f >> 3);
            const int sh = 4 * (f & 7);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t nib = ((src[(long long)i * nw8] >> sh) & 15u) ^ 8u;     // offset binary
                const int pos = (i & 1) ? 4 + (i >> 1) : (i >> 1);                    // 0,2,4,6 -> 0..3; 1,3,5,7 -> 4..7
                out |= nib << (4 * pos);
            }
        } else {
            const int r = 2 * (wd - 1024);
            const bf16* srow = s + ((long long)e * G + (kb * 64) / gs) * Nw;
            const uint32_t lo = bf16_bits(srow[tile_feature(m, r, Nw, swiglu != 0)]);
            const uint32_t hi = bf16_bits(srow[tile_feature(m, r + 1, Nw, swiglu != 0)]);
            out = lo | (hi << 16);
        }
        t[o] = out;
    }
}

// The dequantised pair (k = 8c+2i, 8c+2i+1) of a tile word: bf16(q * s) for both, where
// s2 holds the row's scale in both halves.
FNX_DEV uint32_t tile_pair(uint32_t word, int i, uint32_t s2) {
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t) : "r"(word >> (4 * i)), "r"(0x000f000fu), "r"(0x43004300u));
    uint32_t q;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(q) : "r"(t), "r"(0x43084308u));
    return bmul2(q, s2);
}

// LQP v2o -> int4pack (tools/repack_w4a16.py:41-70 without CANN): v2o uint8 [E, N, K/2], byte
// 64s+j of row n = W[n, 128s+j] (low nibble) | W[n, 128s+64+j] (high), each offset by 8.
// Output word j of (k, e): nibble t = W[8j+t, k] in two's complement (the offset nibble with
// its top bit flipped); K-major [K, E, N/8], or expert-major [E, K, N/8].  One thread per word.
__global__ void __launch_bounds__(256) repack_v2o_kernel(const uint8_t* __restrict__ v2o, int E, int N, int K,
                                                         int expert_major, int32_t* __restrict__ out) {
    const int nw = N / 8;
    const long long total = (long long)E * K * nw;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        // consecutive threads take consecutive words j of one (k, e) row of the output
        const int j = (int)(i % nw);
        const long long r = i / nw;
        int k, e;
        if (expert_major) { e = (int)(r / K); k = (int)(r % K); }
        else { k = (int)(r / E); e = (int)(r % E); }
        const long long byte = 64 * (k >> 7) + (k & 63);
        const int sh = ((k >> 6) & 1) * 4;
        uint32_t w = 0;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const uint32_t b = v2o[((long long)e * N + 8 * j + t) * (K / 2) + byte];
            w |= (((b >> sh) & 15u) ^ 8u) << (4 * t);
        }
        out[i] = (int32_t)w;
    }
}

}  // namespace fnx
