// Decode (M <= 16 tokens) W4A16 MoE layer as three HBM-bound GEMV kernels.
//
//   D1  router logits (bf16 GEMV over [E+1, H]: E router rows + the shared-expert gate
//       row) and the shared expert's gate/up (W4); the last block to finish runs top-k
//       and publishes the routing.
//   D2  routed gate/up for every (token, slot) row + fp32 SwiGLU -> act [M*k, I]
//   D3  routed down for every row + shared down; the last block of each column block
//       does the slot-order weighted reduce and the sigmoid-gated shared merge.
//
// This is the reference's decode branch (fnx/engine.py:1786-1889: concatenated shared
// GEMM, softmax/top-k, gather + W4A16 gate/up, fp32 swiglu, Cartesian down,
// kernels/moe_epilogue) computed without the Cartesian product and without copying
// the selected experts: weights are read straight from the expert-major int4pack.
//
// Weights stream with 16-byte non-allocating loads, are dequantised in registers to the
// exactly rounded bf16(q * s) and multiplied with mixed-precision fp32 FMAs.  Every
// K-split writes fp32 partials; the last block of a group (atomic ticket, no waiting)
// sums them in a fixed order, so results are deterministic.
#pragma once
#include "fnx_common.cuh"
#include "kernels_route.cuh"

namespace fnx {

constexpr int DEC_THREADS = 256;
constexpr int DEC_MAX_M = 16;
constexpr int DEC_FB = 128;          // features per half-block (gate 128 + up 128; down: 128 columns)

struct DecodeParams {
    const bf16* x;                   // [M, H]
    const bf16* router;              // [R, H] router rows 0..E-1, shared gate row E
    const int32_t* gu_w4;            // [E, H, 2I/8]
    const bf16* gu_s;                // [E, H/gs, 2I]
    const int32_t* dn_w4;            // [E, I, H/8]
    const bf16* dn_s;                // [E, I/gs, H]
    const int32_t* sh_gu_w4;         // [H, 2I/8]
    const bf16* sh_gu_s;             // [H/gs, 2I]
    const int32_t* sh_dn_w4;         // [I, H/8]
    const bf16* sh_dn_s;             // [I/gs, H]
    bf16* out;                       // [M, H]
    bf16* w_out;                     // [M, k] bf16 routing weights (optional)
    int64_t* idx_out;                // [M, k] expert ids (optional)
    const float* bias;               // [E] router bias (optional, synthetic load skew)
    // workspace
    bf16* logits;                    // [M, R]
    float* wf;                       // [M*k]
    int32_t* idx;                    // [M*k]
    float* part;                     // K-split partials of the shared gate/up (D1)
    float* part2;                    // K-split partials of the routed gate/up (D2)
    bf16* act;                       // [M*k, I]
    bf16* act_sh;                    // [M, I]
    bf16* yd;                        // [M*k, H]
    bf16* sh;                        // [M, H]
    unsigned* counters;              // zero-initialised tickets
    int M, H, I, E, k, gs, R;
    int ks1, ks2;                    // K splits of the shared and routed gate/up GEMVs
};

// counters layout
FNX_DEV float logit_cg(const bf16* p) {
    return __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(p)) << 16);
}

FNX_DEV unsigned* ctr_d1(const DecodeParams& p) { return p.counters; }
FNX_DEV unsigned* ctr_sh(const DecodeParams& p) { return p.counters + 1; }                                   // [M * I/FB]
FNX_DEV unsigned* ctr_gu(const DecodeParams& p) { return p.counters + 1 + p.M * (p.I / DEC_FB); }             // [M*k * I/FB]
FNX_DEV unsigned* ctr_dn(const DecodeParams& p) { return ctr_gu(p) + p.M * p.k * (p.I / DEC_FB); }            // [H/FB]

// Build scale pairs (s[8w+i], s[8w+i+4]) for the four words of a thread from 32 bf16.
FNX_DEV void scale_pairs(const bf16* s, uint32_t (&sp)[4][4]) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(s + 8 * w));
        asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(sp[w][0]) : "r"(v.x), "r"(v.z));
        asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(sp[w][1]) : "r"(v.x), "r"(v.z));
        asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(sp[w][2]) : "r"(v.y), "r"(v.w));
        asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(sp[w][3]) : "r"(v.y), "r"(v.w));
    }
}

// acc[w][i] (feature 8w+i) and acc[w][4+i] (feature 8w+i+4) += bf16(q*s) * x
FNX_DEV void gemv_w4_uint4(const uint4 wv, const uint32_t (&sp)[4][4], uint16_t xk, float (&acc)[4][8]) {
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t q[4];
        int4x8_to_bf16x2(ww[w], q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t d = bmul2(q[i], sp[w][i]);
            fma_bf_lo_x(acc[w][i], d, xk);
            fma_bf_hi_x(acc[w][4 + i], d, xk);
        }
    }
}

// One block computes a K-slice [k0, k0+nk) of a W4 GEMV for one token over `nseg`
// segments of 128 features (16 words): seg_col[s] is the word column of segment s.
// Result: red[f] for f < nseg*128 (fp32, fixed reduction order), in shared memory.
template <int NSEG>
FNX_DEV void w4_gemv_block(const int32_t* w4, const bf16* scales, int ld_words, int Nw, int gs,
                           const int (&seg_col)[NSEG], const bf16* xrow, int k0, int nk, float* red) {
    constexpr int TPR = NSEG * 4;                 // threads per k row (4 words each)
    constexpr int RPP = DEC_THREADS / TPR;        // rows per pass
    const int tid = threadIdx.x;
    const int q = tid % TPR, r = tid / TPR;
    const int seg = q / 4, wq = (q % 4) * 4;      // word offset within the segment
    const int col = seg_col[seg] + wq;
    float acc[4][8];
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[w][i] = 0.f;
    uint32_t sp[4][4];
    int cur_g = -1;
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(xrow);
    for (int kr = r; kr < nk; kr += RPP * 4) {
        uint4 wv[4];
        uint16_t xk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int kk = k0 + kr + u * RPP;
            if (kr + u * RPP < nk) {
                wv[u] = ld_nc_v4(w4 + (long long)kk * ld_words + col);
                xk[u] = xs[kk];
            } else {
                wv[u] = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);   // q = 0
                xk[u] = 0;
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int kk = k0 + kr + u * RPP;
            if (kr + u * RPP < nk) {
                const int g = kk / gs;
                if (g != cur_g) {
                    cur_g = g;
                    scale_pairs(scales + (long long)g * Nw + col * 8, sp);
                }
                gemv_w4_uint4(wv[u], sp, xk[u], acc);
            }
        }
    }
    // reduce over the RPP rows: lanes of a warp with equal q differ in r
    constexpr int LANES_SAME = 32 / TPR;          // rows per warp
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int o = TPR; o < 32; o <<= 1) acc[w][i] = __fadd_rn(acc[w][i], __shfl_xor_sync(0xffffffffu, acc[w][i], o));
    __shared__ float wred[DEC_THREADS / 32][NSEG * DEC_FB];
    const int warp = tid >> 5, lane = tid & 31;
    if (lane < TPR) {
        const int fb = q * 32;                    // feature offset of this thread's 32 features
#pragma unroll
        for (int w = 0; w < 4; ++w)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                wred[warp][fb + 8 * w + i] = acc[w][i];
                wred[warp][fb + 8 * w + i + 4] = acc[w][4 + i];
            }
    }
    (void)LANES_SAME;
    __syncthreads();
    for (int f = tid; f < NSEG * DEC_FB; f += DEC_THREADS) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < DEC_THREADS / 32; ++w) s = __fadd_rn(s, wred[w][f]);
        red[f] = s;
    }
    __syncthreads();
}

// Last-block ticket: returns true in exactly one block of a group of `n` blocks, after
// all of them have published their partials.
FNX_DEV bool last_block(unsigned* ctr, unsigned n) {
    __shared__ unsigned ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(ctr, 1u);
    __syncthreads();
    const bool last = ticket == n - 1;
    if (last) {
        __threadfence();
        if (threadIdx.x == 0) *ctr = 0;       // re-arm for the next launch
    }
    return last;
}

// ------------------------------------------------------------------ D1
__global__ void __launch_bounds__(DEC_THREADS) decode_d1_kernel(const DecodeParams p, int router_blocks) {
    __shared__ float red[2 * DEC_FB];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nfb = p.I / DEC_FB;
    if ((int)blockIdx.x < router_blocks) {
        // ---- router + shared gate row: one warp per row, all tokens
        const int e = blockIdx.x * (DEC_THREADS / 32) + warp;
        if (e < p.R) {
            float acc[DEC_MAX_M];
#pragma unroll
            for (int t = 0; t < DEC_MAX_M; ++t) acc[t] = 0.f;
            const bf16* wr = p.router + (long long)e * p.H;
            for (int c = lane * 8; c < p.H; c += 256) {
                const uint4 wv = ld_nc_v4(wr + c);
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int t = 0; t < DEC_MAX_M; ++t) {
                    if (t < p.M) {
                        const uint4 xv = *reinterpret_cast<const uint4*>(p.x + (long long)t * p.H + c);
                        const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            fma_bf_lo(acc[t], ww[i], xx[i]);
                            fma_bf_hi(acc[t], ww[i], xx[i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < DEC_MAX_M; ++t) {
                if (t < p.M) {
                    float v = acc[t];
#pragma unroll
                    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                    if (lane == 0) p.logits[(long long)t * p.R + e] = f2bf(v);
                }
            }
        }
    } else {
        // ---- shared expert gate/up: block (t, fb, ks)
        const int b = blockIdx.x - router_blocks;
        const int ks = b % p.ks1, fb = (b / p.ks1) % nfb, t = b / (p.ks1 * nfb);
        const int nk = p.H / p.ks1;
        const int cols[2] = {fb * DEC_FB / 8, (p.I + fb * DEC_FB) / 8};
        w4_gemv_block<2>(p.sh_gu_w4, p.sh_gu_s, 2 * p.I / 8, 2 * p.I, p.gs, cols, p.x + (long long)t * p.H,
                         ks * nk, nk, red);
        float* part = p.part + (((long long)t * nfb + fb) * p.ks1 + ks) * (2 * DEC_FB);
        for (int f = tid; f < 2 * DEC_FB; f += DEC_THREADS) part[f] = red[f];
        if (last_block(ctr_sh(p) + t * nfb + fb, p.ks1)) {
            const float* base = p.part + ((long long)t * nfb + fb) * p.ks1 * (2 * DEC_FB);
            for (int f = tid; f < DEC_FB; f += DEC_THREADS) {
                float g = 0.f, u = 0.f;
                for (int s = 0; s < p.ks1; ++s) {
                    g = __fadd_rn(g, ld_cg_f32(base + s * 2 * DEC_FB + f));
                    u = __fadd_rn(u, ld_cg_f32(base + s * 2 * DEC_FB + DEC_FB + f));
                }
                // shared expert: bf16(bf16(silu(bf16 g)) * bf16 u)   (fnx/engine.py:1788)
                const float gb = round_bf(g), ub = round_bf(u);
                p.act_sh[(long long)t * p.I + fb * DEC_FB + f] = f2bf(__fmul_rn(round_bf(silu_f32(gb)), ub));
            }
        }
    }
    // ---- the last block of D1 routes every token
    if (last_block(ctr_d1(p), gridDim.x)) {
        for (int t = warp; t < p.M; t += DEC_THREADS / 32) {
            // the router kernel's top-k rule, logits read through L2 (written by other blocks)
            const bf16* row = p.logits + (long long)t * p.R;
            float my_p, tot;
            int my_i;
            if (p.E <= 256) topk_warp<8, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
            else if (p.E <= 512) topk_warp<16, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
            else if (p.E <= 1024) topk_warp<32, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
            else topk_warp<64, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
            if (lane < p.k) {
                const bf16 wb = f2bf(my_p / tot);
                const int o = t * p.k + lane;
                p.wf[o] = bf2f(wb);
                p.idx[o] = my_i;
                if (p.w_out) p.w_out[o] = wb;
                if (p.idx_out) p.idx_out[o] = my_i;
            }
        }
    }
}

// ------------------------------------------------------------------ D2
// block (row, fb, ks): routed gate/up over H/ks2 rows of K for one (token, slot) row.
__global__ void __launch_bounds__(DEC_THREADS) decode_d2_kernel(const DecodeParams p) {
    __shared__ float red[2 * DEC_FB];
    const int tid = threadIdx.x;
    const int nfb = p.I / DEC_FB;
    const int b = blockIdx.x;
    const int ks = b % p.ks2, fb = (b / p.ks2) % nfb, row = b / (p.ks2 * nfb);
    const int ex = __ldcg(p.idx + row), t = row / p.k;
    const int nk = p.H / p.ks2;
    const int cols[2] = {fb * DEC_FB / 8, (p.I + fb * DEC_FB) / 8};
    const int G = p.H / p.gs;
    w4_gemv_block<2>(p.gu_w4 + (long long)ex * p.H * (2 * p.I / 8), p.gu_s + (long long)ex * G * 2 * p.I,
                     2 * p.I / 8, 2 * p.I, p.gs, cols, p.x + (long long)t * p.H, ks * nk, nk, red);
    float* part = p.part2 + (((long long)row * nfb + fb) * p.ks2 + ks) * (2 * DEC_FB);
    for (int f = tid; f < 2 * DEC_FB; f += DEC_THREADS) part[f] = red[f];
    if (last_block(ctr_gu(p) + row * nfb + fb, p.ks2)) {
        const float* base = p.part2 + ((long long)row * nfb + fb) * p.ks2 * (2 * DEC_FB);
        for (int f = tid; f < DEC_FB; f += DEC_THREADS) {
            float g = 0.f, u = 0.f;
            for (int s = 0; s < p.ks2; ++s) {
                g = __fadd_rn(g, ld_cg_f32(base + s * 2 * DEC_FB + f));
                u = __fadd_rn(u, ld_cg_f32(base + s * 2 * DEC_FB + DEC_FB + f));
            }
            // routed expert: bf16(silu(g) * u) in fp32 on bf16-rounded gate/up
            const float gb = round_bf(g), ub = round_bf(u);
            p.act[(long long)row * p.I + fb * DEC_FB + f] = f2bf(__fmul_rn(silu_f32(gb), ub));
        }
    }
}

// ------------------------------------------------------------------ D3
// block (row, cb): rows 0..M*k-1 are routed (token, slot) rows, rows M*k.. are the
// shared expert of each token; 128 output columns, all I rows of K.
__global__ void __launch_bounds__(DEC_THREADS) decode_d3_kernel(const DecodeParams p) {
    __shared__ float red[DEC_FB];
    const int tid = threadIdx.x;
    const int ncb = p.H / DEC_FB;
    const int cb = blockIdx.x % ncb, row = blockIdx.x / ncb;
    const int nrows = p.M * p.k;
    const int cols[1] = {cb * DEC_FB / 8};
    const int G = p.I / p.gs;
    if (row < nrows) {
        const int ex = __ldcg(p.idx + row);
        w4_gemv_block<1>(p.dn_w4 + (long long)ex * p.I * (p.H / 8), p.dn_s + (long long)ex * G * p.H, p.H / 8, p.H,
                         p.gs, cols, p.act + (long long)row * p.I, 0, p.I, red);
        for (int f = tid; f < DEC_FB; f += DEC_THREADS) p.yd[(long long)row * p.H + cb * DEC_FB + f] = f2bf(red[f]);
    } else {
        const int t = row - nrows;
        w4_gemv_block<1>(p.sh_dn_w4, p.sh_dn_s, p.H / 8, p.H, p.gs, cols, p.act_sh + (long long)t * p.I, 0, p.I, red);
        for (int f = tid; f < DEC_FB; f += DEC_THREADS) p.sh[(long long)t * p.H + cb * DEC_FB + f] = f2bf(red[f]);
    }
    if (last_block(ctr_dn(p) + cb, nrows + p.M)) {
        const unsigned short* yd = reinterpret_cast<const unsigned short*>(p.yd);
        const unsigned short* sh = reinterpret_cast<const unsigned short*>(p.sh);
        for (int i = tid; i < p.M * DEC_FB; i += DEC_THREADS) {
            const int t = i / DEC_FB, c = cb * DEC_FB + i % DEC_FB;
            float acc = 0.f;
            for (int j = 0; j < p.k; ++j) {
                const float y = __uint_as_float((uint32_t)__ldcg(yd + (long long)(t * p.k + j) * p.H + c) << 16);
                acc = __fadd_rn(acc, round_bf(__fmul_rn(y, ld_cg_f32(p.wf + t * p.k + j))));
            }
            const float a = round_bf(acc);
            const float g = bf2f(p.logits[(long long)t * p.R + p.E]);
            const float sg = round_bf(sigmoid_f32(g));
            const float s = __uint_as_float((uint32_t)__ldcg(sh + (long long)t * p.H + c) << 16);
            p.out[(long long)t * p.H + c] = f2bf(__fadd_rn(a, round_bf(__fmul_rn(s, sg))));
        }
    }
}

}  // namespace fnx
