// Small-M W8A16 dense projection (DenseW8.__call__, fnx/engine.py:350-365, for M <= 16):
// y [M, N] = x [M, K] . bf16(w8t [K, N] * sc [k / gs, n]) with fp32 accumulation.
//
// At M <= 16 the projection is a weight stream (K*N bytes of int8), so it is built as a GEMV:
// a CTA owns 128 output columns (4 per lane: one 4-byte load per weight row, a warp reads a
// full 128-byte line) and one eighth of K; its 8 warps split that eighth by rows.  The 8 CTAs
// of a cluster hold the 8 eighths of K for the same columns and reduce them through
// distributed shared memory in a fixed order, so the sum is deterministic and needs no
// global workspace.  Each weight is dequantised once to the exactly rounded bf16(q * s) the
// reference's antiquant produces, then multiplied into every token's fp32 accumulators.
#pragma once
#include "fnx_common.cuh"

namespace fnx {

constexpr int W8V_COLS = 128;      // output columns per CTA
#ifndef FNX_W8V_CL
#define FNX_W8V_CL 8
#endif
constexpr int W8V_CL = FNX_W8V_CL; // CTAs per cluster (K split)
constexpr int W8V_MAXM = 16;

FNX_DEV float ld_shared_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

inline size_t w8a16_gemv_smem(int MT, int K) {
    const int Kc = K / W8V_CL;
    return sizeof(uint16_t) * (size_t)MT * Kc + sizeof(float) * ((size_t)8 * MT * W8V_COLS + (size_t)MT * W8V_COLS);
}

// two signed bytes (bytes b and b+1 of w, already xor 0x80) -> their exact values as bf16x2
FNX_DEV uint32_t i8pair_bf16x2(uint32_t wx, int b) {
    // 0x4B0000uu = 2^23 + u as fp32; minus 2^23 + 128 leaves the signed value exactly
    const float lo = __int_as_float(__byte_perm(wx, 0x4B000000u, 0x7640 + b)) - 8388736.0f;
    const float hi = __int_as_float(__byte_perm(wx, 0x4B000000u, 0x7641 + b)) - 8388736.0f;
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// grid (ceil(N / 128), 8), cluster (1, 8, 1), 256 threads.  MT: tokens padded to 1/2/4/8/16.
// Needs K % 64 == 0, N % 4 == 0, K % gs == 0.
template <int MT>
__global__ void __launch_bounds__(256, 2) w8a16_gemv_kernel(const bf16* __restrict__ x, const int8_t* __restrict__ w,
                                                            const bf16* __restrict__ sc, bf16* __restrict__ y,
                                                            int M, int K, int N, int gs) {
    extern __shared__ float sm[];
    const int Kc = K / W8V_CL;
    uint16_t* xs = reinterpret_cast<uint16_t*>(sm);                 // [MT][Kc] bf16 bits
    float* red = sm + (MT * Kc + 1) / 2;                              // [8 warps][MT][128]
    float* cpart = red + 8 * MT * W8V_COLS;                           // [MT][128]: this CTA's eighth
    const int crank = (int)cluster_rank();
    const int n0 = blockIdx.x * W8V_COLS;
    const int k0 = crank * Kc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned short* xb = reinterpret_cast<const unsigned short*>(x);
    for (int i = threadIdx.x; i < MT * Kc; i += blockDim.x) {
        const int m = i / Kc, kk = i - m * Kc;
        xs[i] = m < M ? xb[(long long)m * K + k0 + kk] : (uint16_t)0;
    }
    __syncthreads();

    const int col = n0 + lane * 4;
    const bool ok = col < N;
    const int rpw = Kc / 8;                           // rows per warp (K % 64 == 0)
    const int r0 = warp * rpw;
    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;
    // the scale group and where it ends (no division per row)
    int g = (k0 + r0) / gs;
    int g_end = (g + 1) * gs - k0;                    // first row (CTA-relative) of the next group
    uint32_t s01 = 0, s23 = 0;
    if (ok) {
        const uint2 sv = __ldg(reinterpret_cast<const uint2*>(sc + (long long)g * N + col));
        s01 = sv.x; s23 = sv.y;
    }
#ifndef FNX_W8V_RB
#define FNX_W8V_RB 8
#endif
    constexpr int RB = FNX_W8V_RB;                    // rows per batch of loads in flight
    for (int rb = 0; rb < rpw; rb += RB) {
        uint32_t q[RB];
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            const long long k = k0 + r0 + rb + i;
            q[i] = (ok && rb + i < rpw) ? __ldg(reinterpret_cast<const unsigned int*>(w + k * N + col)) : 0u;
        }
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            if (rb + i >= rpw) break;                 // warp-uniform: rows past this warp's share
            const int kr = r0 + rb + i;               // row within the CTA's eighth
            if (kr >= g_end) {                        // warp-uniform
                ++g;
                g_end += gs;
                if (ok) {
                    const uint2 sv = __ldg(reinterpret_cast<const uint2*>(sc + (long long)g * N + col));
                    s01 = sv.x; s23 = sv.y;
                }
            }
            const uint32_t qx = q[i] ^ 0x80808080u;
            const uint32_t w01 = bmul2(i8pair_bf16x2(qx, 0), s01);      // bf16(q * s), exact rounding
            const uint32_t w23 = bmul2(i8pair_bf16x2(qx, 2), s23);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const uint32_t xv = (uint32_t)xs[m * Kc + kr];
                const uint32_t x2 = xv | (xv << 16);
                fma_bf_lo(acc[m][0], w01, x2);
                fma_bf_hi(acc[m][1], w01, x2);
                fma_bf_lo(acc[m][2], w23, x2);
                fma_bf_hi(acc[m][3], w23, x2);
            }
        }
    }
    // the 8 warps of the CTA, in order
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[(warp * MT + m) * W8V_COLS + lane * 4 + c] = acc[m][c];
    __syncthreads();
    for (int i = threadIdx.x; i < MT * W8V_COLS; i += blockDim.x) {
        float v = 0.f;
#pragma unroll
        for (int wv = 0; wv < 8; ++wv) v += red[wv * MT * W8V_COLS + i];
        cpart[i] = v;
    }
    cluster_sync_all();
    // the cluster's 8 eighths of K, in order, by CTA 0
    if (crank == 0) {
        for (int i = threadIdx.x; i < MT * W8V_COLS; i += blockDim.x) {
            float v = cpart[i];
#pragma unroll
            for (int r = 1; r < W8V_CL; ++r) v += ld_shared_cluster_f32(mapa_rank(cpart + i, (uint32_t)r));
            const int m = i / W8V_COLS, n = n0 + (i - m * W8V_COLS);
            if (m < M && n < N) y[(long long)m * N + n] = f2bf(v);
        }
    }
    cluster_sync_all();                               // peers keep their shared memory until read
}

}  // namespace fnx
