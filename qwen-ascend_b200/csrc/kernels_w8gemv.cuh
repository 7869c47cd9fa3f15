// Small-M W8A16 dense projection (DenseW8.__call__, fnx/engine.py:350-365, for M <= 16):
// y [M, N] = x [M, K] . bf16(w8t [K, N] * sc [k / gs, n]) with fp32 accumulation.
//
// At M <= 16 the projection is a weight stream (K*N bytes of int8), so it is built as a GEMV:
// a CTA owns 128 output columns (4 per lane: one 4-byte load per weight row, a warp reads a
// full 128-byte line) and one eighth of K; its 8 warps split that eighth by rows.  The 8 CTAs
// of a cluster hold the 8 eighths of K for the same columns and reduce them through
// distributed shared memory in a fixed order, so the sum is deterministic and needs no
// global workspace.  Each weight is dequantised once to the exactly rounded bf16(q * s) the
// reference's antiquant produces, then multiplied into every token's fp32 accumulators.  The
// tokens are staged in shared memory as fp32, token-minor, so one 16-byte load serves four
// tokens and each product is a plain fp32 FMA.  The first two batches of weight rows are
// requested before the tokens are staged, and every batch is requested one batch ahead of its
// use.
#pragma once
#include "fnx_common.cuh"

#ifndef FNX_W8V_DB
#define FNX_W8V_DB 1
#endif

namespace fnx {

constexpr int W8V_COLS = 128;      // output columns per CTA
constexpr int W8V_MAXM = 16;

FNX_DEV float ld_shared_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

inline size_t w8a16_gemv_smem(int MT, int CL, int K) {
    const int Kc = K / CL;
    return sizeof(float) * ((size_t)Kc * MT + (size_t)8 * MT * W8V_COLS + (size_t)MT * W8V_COLS);
}

// two signed bytes (bytes b and b+1 of w, already xor 0x80) -> their exact values as bf16x2
FNX_DEV uint32_t i8pair_bf16x2(uint32_t wx, int b) {
    return ints_bf16x2(i8x_f32(wx, b), i8x_f32(wx, b + 1));
}

// grid (ceil(N / 128), CL), cluster (1, CL, 1), 256 threads.  MT: tokens padded to 1/2/4/8/16.
// Needs K % 64 == 0, N % 4 == 0, K % gs == 0.  Up to 8 tokens a CTA fits in 80 registers, so
// three CTAs share an SM and the N = 5120 grid (320 CTAs) runs in one wave.
template <int MT, int CL>
__global__ void __launch_bounds__(256, (MT <= 8 ? 3 : 2))
    w8a16_gemv_kernel(const bf16* __restrict__ x, const int8_t* __restrict__ w, const bf16* __restrict__ sc,
                      bf16* __restrict__ y, int M, int K, int N, int gs) {
    extern __shared__ float sm[];
    const int Kc = K / CL;
    float* xs = sm;                                                   // [Kc][MT] tokens as fp32
    float* red = sm + Kc * MT;                                        // [8 warps][MT][128]
    float* cpart = red + 8 * MT * W8V_COLS;                           // [MT][128]: this CTA's eighth
    const int crank = (int)cluster_rank();
    const int n0 = blockIdx.x * W8V_COLS;
    const int k0 = crank * Kc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int col = n0 + lane * 4;
    const bool ok = col < N;
    const int rpw = Kc / 8;                           // rows per warp (K % 64 == 0)
    const int r0 = warp * rpw;
#ifndef FNX_W8V_RB
#define FNX_W8V_RB 8
#endif
    constexpr int RB = FNX_W8V_RB;                    // rows per batch of loads
    auto load = [&](uint32_t (&q)[RB], int rb) {
#pragma unroll
        for (int i = 0; i < RB; ++i) {
            const long long k = k0 + r0 + rb + i;
            q[i] = (ok && rb + i < rpw) ? __ldg(reinterpret_cast<const unsigned int*>(w + k * N + col)) : 0u;
        }
    };
    // the scale group and where it ends (no division per row)
    int g = (k0 + r0) / gs;
    int g_end = (g + 1) * gs - k0;                    // first row (CTA-relative) of the next group
    uint32_t s01 = 0, s23 = 0;
    if (ok) {
        const uint2 sv = __ldg(reinterpret_cast<const uint2*>(sc + (long long)g * N + col));
        s01 = sv.x; s23 = sv.y;
    }
    // the first weight rows are requested before the tokens are staged
    uint32_t qa[RB], qb[RB];
    load(qa, 0);
#if FNX_W8V_DB
    load(qb, RB);
#endif

    const unsigned short* xb = reinterpret_cast<const unsigned short*>(x);
    for (int i = threadIdx.x; i < MT * Kc; i += blockDim.x) {
        const int m = i / Kc, kk = i - m * Kc;
        xs[kk * MT + m] = m < M ? __uint_as_float((uint32_t)xb[(long long)m * K + k0 + kk] << 16) : 0.f;
    }
    __syncthreads();

    float acc[MT][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;
    auto consume = [&](const uint32_t (&q)[RB], int rb) {
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
            // bf16 -> fp32 is exact, so an fp32 FMA of the two gives the product exactly and
            // rounds the sum once
            const float wf[4] = {__uint_as_float(w01 << 16), __uint_as_float(w01 & 0xffff0000u),
                                 __uint_as_float(w23 << 16), __uint_as_float(w23 & 0xffff0000u)};
            const float* xr = xs + kr * MT;
            if constexpr (MT >= 4) {
#pragma unroll
                for (int m = 0; m < MT; m += 4) {
                    const float4 xv = *reinterpret_cast<const float4*>(xr + m);
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        acc[m][c] = __fmaf_rn(wf[c], xv.x, acc[m][c]);
                        acc[m + 1][c] = __fmaf_rn(wf[c], xv.y, acc[m + 1][c]);
                        acc[m + 2][c] = __fmaf_rn(wf[c], xv.z, acc[m + 2][c]);
                        acc[m + 3][c] = __fmaf_rn(wf[c], xv.w, acc[m + 3][c]);
                    }
                }
            } else {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    const float xv = xr[m];
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[m][c] = __fmaf_rn(wf[c], xv, acc[m][c]);
                }
            }
        }
    };
#if FNX_W8V_DB
    // two batches in flight: the next one is requested before the current one is used
    for (int rb = 0; rb < rpw; rb += 2 * RB) {
        consume(qa, rb);
        if (rb + 2 * RB < rpw) load(qa, rb + 2 * RB);
        if (rb + RB < rpw) consume(qb, rb + RB);
        if (rb + 3 * RB < rpw) load(qb, rb + 3 * RB);
    }
#else
    for (int rb = 0; rb < rpw; rb += RB) {
        if (rb) load(qa, rb);
        consume(qa, rb);
    }
    (void)qb;
#endif
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
            for (int r = 1; r < CL; ++r) v += ld_shared_cluster_f32(mapa_rank(cpart + i, (uint32_t)r));
            const int m = i / W8V_COLS, n = n0 + (i - m * W8V_COLS);
            if (m < M && n < N) y[(long long)m * N + n] = f2bf(v);
        }
    }
    cluster_sync_all();                               // peers keep their shared memory until read
}

}  // namespace fnx
