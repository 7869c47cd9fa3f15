// Load-time repack of the int4pack artifact into the tile-major layout the B200 kernels
// stream.  Run once per weight tensor when a layer is loaded; the artifact itself
// (tools/repack_w4a16.py, tools/repack_w4_em.py) is read unchanged.
//
// Input  w  int32 [E, K, Nw/8]  nibble t of word j = W[k, 8j+t], two's complement
//        s  bf16  [E, K/gs, Nw]
// Output tw int32 [E, MT, K/64, 8, 128]: for expert e, feature tile m and k-block kb, word
//        (c, r) holds the 8 weights W[kb*64 + 8c + i, f(m, r)] of tile row r, as offset-binary
//        nibbles (q + 8) in the order i = 0,2,4,6,1,3,5,7, so that
//        ((word >> 4i) & 0x000f000f) yields the pair (k = 8c+2i, 8c+2i+1).
//        ts bf16  [E, MT, K/gs, 128]: the scale of row r for every k group.
// Tile rows: PLAIN  f(m, r) = 128m + r                                 (MT = Nw / 128)
//            SWIGLU f(m, r) = (r odd ? Nw/2 : 0) + 64m + r/2  (gate/up of a feature on
//                             adjacent rows, so a SwiGLU epilogue pairs lanes 2i, 2i+1)
//                                                                        (MT = Nw / 128)
#pragma once
#include "fnx_common.cuh"

namespace fnx {

FNX_DEV int tile_feature(int m, int r, int Nw, bool swiglu) {
    return swiglu ? ((r & 1) ? Nw / 2 : 0) + 64 * m + (r >> 1) : 128 * m + r;
}

__global__ void __launch_bounds__(256) repack_w4_tiles_kernel(const uint32_t* __restrict__ w,
                                                              uint32_t* __restrict__ tw, int E, int K, int Nw,
                                                              int swiglu) {
    const int MT = Nw / 128, KB = K / 64;
    const long long total = (long long)E * MT * KB * 8 * 128;
    const int nw8 = Nw / 8;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(o & 127);
        const int c = (int)((o >> 7) & 7);
        long long rest = o >> 10;
        const int kb = (int)(rest % KB);
        rest /= KB;
        const int m = (int)(rest % MT);
        const int e = (int)(rest / MT);
        const int f = tile_feature(m, r, Nw, swiglu != 0);
        const int k0 = kb * 64 + 8 * c;
        const uint32_t* src = w + ((long long)e * K + k0) * nw8 + (f >> 3);
        const int sh = 4 * (f & 7);
        uint32_t out = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t nib = ((src[(long long)i * nw8] >> sh) & 15u) ^ 8u;     // offset binary
            const int pos = (i & 1) ? 4 + (i >> 1) : (i >> 1);                    // 0,2,4,6 -> 0..3; 1,3,5,7 -> 4..7
            out |= nib << (4 * pos);
        }
        tw[o] = out;
    }
}

__global__ void __launch_bounds__(256) repack_scales_tiles_kernel(const bf16* __restrict__ s, bf16* __restrict__ ts,
                                                                  int E, int G, int Nw, int swiglu) {
    const int MT = Nw / 128;
    const long long total = (long long)E * MT * G * 128;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(o & 127);
        long long rest = o >> 7;
        const int g = (int)(rest % G);
        rest /= G;
        const int m = (int)(rest % MT);
        const int e = (int)(rest / MT);
        ts[o] = s[((long long)e * G + g) * Nw + tile_feature(m, r, Nw, swiglu != 0)];
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

}  // namespace fnx
