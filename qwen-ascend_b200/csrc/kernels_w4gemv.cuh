// The legacy W4 GEMV op (fnx/w4gemv_op.py in the reference, FNX_MOE_KERNEL=1):
//
//   y[e, n] = sum_k W[ids[e]][n, k] * s4t[ids[e]][k / 32][n] * x[e, k]     (fp32)
//
// p4 is [E, N, K/2] bytes with k contiguous per output row n:
//   lay 1: byte j low nibble = W[2j], high = W[2j+1] (x passed split: xe = x[:, 0::2],
//          xo = x[:, 1::2]);  lay 2 ("v2"): byte 64s+j low = W[128s+j], high =
//          W[128s+64+j] (x natural, xe == xo).  Nibbles are two's complement.
// s4t is fp16 [E, K/32, N]; weights and scales are indexed by expert id, x and y by
// slot (fnx/w4gemv_op.py:308-319).  One warp per output row; fp32 arithmetic.
#pragma once
#include <cuda_fp16.h>
#include "fnx_common.cuh"

namespace fnx {

struct W4GemvLayer {
    const uint8_t* p4;
    const __half* s4t;
    const float* xe;
    const float* xo;
    float* y;
};

FNX_DEV float nib_s(uint32_t v) { return (float)((int)((v ^ 8u) & 15u) - 8); }

template <int LAY>
FNX_DEV float w4gemv_row(const W4GemvLayer L, const int32_t* ids, int e, int n, int N, int K) {
    const int lane = threadIdx.x & 31;
    const long long ex = ids ? ids[e] : e;
    const uint8_t* row = L.p4 + (ex * N + n) * (long long)(K / 2);
    const __half* s = L.s4t + ex * (long long)(K / 32) * N + n;
    float acc = 0.f;
    for (int j0 = lane * 16; j0 < K / 2; j0 += 32 * 16) {
        const uint4 v = ld_nc_v4(row + j0);
        const uint32_t b[4] = {v.x, v.y, v.z, v.w};
        if (LAY == 1) {
            // bytes j0..j0+15 hold k = 2*j0 .. 2*j0+31: one scale group
            const float sc = __half2float(s[(long long)(2 * j0 / 32) * N]);
            const float* xe = L.xe + (long long)e * (K / 2) + j0;
            const float* xo = L.xo + (long long)e * (K / 2) + j0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t byte = (b[i >> 2] >> (8 * (i & 3))) & 0xffu;
                acc = fmaf(nib_s(byte) * sc, xe[i], acc);
                acc = fmaf(nib_s(byte >> 4) * sc, xo[i], acc);
            }
        } else {
            // bytes 64s + jj .. +15: low nibbles k = 128s + jj.., high nibbles k = 128s + 64 + jj..
            const int sblk = j0 / 64, jj = j0 % 64;
            const int klo = 128 * sblk + jj, khi = klo + 64;
            const float slo = __half2float(s[(long long)(klo / 32) * N]);
            const float shi = __half2float(s[(long long)(khi / 32) * N]);
            const float* x = L.xe + (long long)e * K;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t byte = (b[i >> 2] >> (8 * (i & 3))) & 0xffu;
                acc = fmaf(nib_s(byte) * slo, x[klo + i], acc);
                acc = fmaf(nib_s(byte >> 4) * shi, x[khi + i], acc);
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

template <int LAY>
__global__ void __launch_bounds__(256) w4gemv_kernel(const W4GemvLayer L, const int32_t* __restrict__ ids, int N, int K,
                                                     int nExp) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= nExp * N) return;
    const int e = row / N, n = row % N;
    const float v = w4gemv_row<LAY>(L, ids, e, n, N, K);
    if ((threadIdx.x & 31) == 0) L.y[(long long)e * N + n] = v;
}

constexpr int W4GEMV_MAX_LAYERS = 64;
struct W4GemvLayers {
    W4GemvLayer L[W4GEMV_MAX_LAYERS];
};

template <int LAY>
__global__ void __launch_bounds__(256) w4gemv_layers_kernel(const W4GemvLayers Ls, int N, int K, int nExp) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= nExp * N) return;
    const int e = row / N, n = row % N;
    const W4GemvLayer L = Ls.L[blockIdx.y];
    const float v = w4gemv_row<LAY>(L, nullptr, e, n, N, K);
    if ((threadIdx.x & 31) == 0) L.y[(long long)e * N + n] = v;
}

}  // namespace fnx
