// Decode (M <= 16 tokens) W4A16 MoE layer as three HBM-bound GEMV kernels.
//
//   D1  router logits (bf16 GEMV over [E+1, H]: E router rows + the shared-expert gate
//       row) and the shared expert's gate/up; the last block to finish runs top-k and
//       publishes the routing.
//   D2  routed gate/up for every (token, slot) row + fp32 SwiGLU -> act [M*k, I]
//   D3  routed down for every row + shared down; the last block of each 128-column tile
//       does the slot-order weighted reduce and the sigmoid-gated shared merge.
//
// This is the reference's decode branch (fnx/engine.py:1786-1889: concatenated shared
// GEMM, softmax/top-k, gather + W4A16 gate/up, fp32 swiglu, Cartesian down,
// kernels/moe_epilogue) computed without the Cartesian product and without copying the
// selected experts.  Weights are read in the tile-major layout (kernels_repack.cuh): one
// thread owns one tile row (one output feature), so each k-block of a tile is a
// contiguous 4 KB stream (plus its inline scales) read as consecutive 4-byte words across
// the block, and a dot product never crosses threads.  K-splits write fp32 partials; the
// last block of a group
// (atomic ticket, no waiting) sums them in a fixed order, so results are deterministic.
#pragma once
#include "fnx_common.cuh"
#include "kernels_repack.cuh"
#include "kernels_route.cuh"

namespace fnx {

constexpr int DEC_THREADS = 256;
constexpr int DEC_MAX_M = 16;
constexpr int DEC_MAX_K = 4096;          // largest K (H or I) a block stages in shared memory

struct DecodeParams {
    const bf16* x;                   // [M, H]
    const bf16* router;              // [R, H] router rows 0..E-1, shared gate row E
    const uint32_t* gu_tw;           // routed gate/up tile blocks, SwiGLU order [E, I/64, H/64, TILE_BLOCK_WORDS]
    const uint32_t* dn_tw;           // routed down tile blocks [E, H/128, I/64, TILE_BLOCK_WORDS]
    const uint32_t* sh_gu_tw;        // shared expert, same layouts with E = 1
    const uint32_t* sh_dn_tw;
    bf16* out;                       // [M, H]
    bf16* w_out;                     // [M, k] bf16 routing weights (optional)
    int64_t* idx_out;                // [M, k] expert ids (optional)
    const float* bias;               // [E] router bias (optional, synthetic load skew)
    // workspace
    bf16* logits;                    // [M, R]
    float* wf;                       // [M*k]
    int32_t* idx;                    // [M*k]
    float* part;                     // shared gate/up partials [M][I/64][ks1][128]
    float* part2;                    // routed gate/up partials [M*k][I/64][ks2][128]
    bf16* act;                       // [M*k, I]
    bf16* act_sh;                    // [M, I]
    bf16* yd;                        // [M*k, H]
    bf16* sh;                        // [M, H]
    unsigned* counters;              // zero-initialised tickets
    int M, H, I, E, k, R;
    int ks1, ks2;                    // K splits of the shared and routed gate/up GEMVs
};

FNX_DEV int gu_tiles(const DecodeParams& p) { return p.I / 64; }
FNX_DEV int dn_tiles(const DecodeParams& p) { return p.H / 128; }
FNX_DEV unsigned* ctr_d1(const DecodeParams& p) { return p.counters; }
FNX_DEV unsigned* ctr_sh(const DecodeParams& p) { return p.counters + 1; }                                 // [M * I/64]
FNX_DEV unsigned* ctr_gu(const DecodeParams& p) { return ctr_sh(p) + p.M * gu_tiles(p); }                 // [M*k * I/64]
FNX_DEV unsigned* ctr_dn(const DecodeParams& p) { return ctr_gu(p) + p.M * p.k * gu_tiles(p); }           // [H/128]

// Last-block ticket: true in exactly one block of a group of `n` blocks, after all of them
// have published their results; the ticket is re-armed for the next launch.
FNX_DEV bool last_block(unsigned* ctr, unsigned n) {
    __shared__ unsigned ticket;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(ctr, 1u);
    __syncthreads();
    const bool last = ticket == n - 1;
    if (last) {
        __threadfence();
        if (threadIdx.x == 0) *ctr = 0;
    }
    return last;
}

// Stage x (bf16 [K]) as bf16 pairs in shared memory.
FNX_DEV void stage_x(uint32_t* xs2, const bf16* x, int K) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(x);
    for (int i = threadIdx.x; i < K / 2; i += blockDim.x) xs2[i] = src[i];
    __syncthreads();
}

// Dot products of the 128 rows of one weight tile with x over k-blocks [kb0, kb1):
// thread (half, r) takes the k-blocks kb0 + half, kb0 + half + 2, ...; the two halves are
// added in a fixed order.  Result in red[r] (shared memory, 128 floats).
FNX_DEV void tile_dot(const uint32_t* __restrict__ tw, const uint32_t* xs2, int kb0, int kb1, float* red) {
    const int r = threadIdx.x & 127, half = threadIdx.x >> 7;
    float a0 = 0.f, a1 = 0.f;
    for (int kb = kb0 + half; kb < kb1; kb += 4) {
        uint32_t wv[2][8], s2[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int kbu = kb + 2 * u;
            if (kbu < kb1) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint32_t v;
                    asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v)
                                 : "l"(tw + (long long)kbu * TILE_BLOCK_WORDS + c * 128 + r));
                    wv[u][c] = v;
                }
                const uint32_t s16 = __ldg(reinterpret_cast<const unsigned short*>(tw + (long long)kbu * TILE_BLOCK_WORDS + 1024) + r);
                s2[u] = s16 | (s16 << 16);
            } else {
#pragma unroll
                for (int c = 0; c < 8; ++c) wv[u][c] = 0x88888888u;      // q = 0
                s2[u] = 0;
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int kbu = kb + 2 * u;
            if (kbu < kb1) {
                const uint4* xq = reinterpret_cast<const uint4*>(xs2 + kbu * 32);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 xv = xq[c];
                    const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t w2 = tile_pair(wv[u][c], i, s2[u]);
                        fma_bf_lo(a0, w2, xx[i]);
                        fma_bf_hi(a1, w2, xx[i]);
                    }
                }
            }
        }
    }
    __shared__ float halves[2][128];
    halves[half][r] = __fadd_rn(a0, a1);
    __syncthreads();
    if (threadIdx.x < 128) red[r] = __fadd_rn(halves[0][r], halves[1][r]);
    __syncthreads();
}

// Sum ks partials [ks][128] in order (read through L2: written by other blocks).
FNX_DEV float sum_parts(const float* base, int ks, int r) {
    float a = 0.f;
    for (int s = 0; s < ks; ++s) a = __fadd_rn(a, ld_cg_f32(base + s * 128 + r));
    return a;
}

// ------------------------------------------------------------------ D1
__global__ void __launch_bounds__(DEC_THREADS) decode_d1_kernel(const DecodeParams p, int router_blocks) {
    __shared__ __align__(16) uint32_t xs2[DEC_MAX_K / 2];
    __shared__ float red[128];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int MT = gu_tiles(p), KB = p.H / 64;
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
        // ---- shared expert gate/up: block (t, m, ks)
        const int b = blockIdx.x - router_blocks;
        const int ks = b % p.ks1, m = (b / p.ks1) % MT, t = b / (p.ks1 * MT);
        const int nkb = KB / p.ks1;
        stage_x(xs2, p.x + (long long)t * p.H, p.H);
        tile_dot(p.sh_gu_tw + (long long)m * KB * TILE_BLOCK_WORDS, xs2, ks * nkb,
                 (ks + 1) * nkb, red);
        float* part = p.part + (((long long)t * MT + m) * p.ks1 + ks) * 128;
        if (tid < 128) part[tid] = red[tid];
        if (last_block(ctr_sh(p) + t * MT + m, p.ks1)) {
            const float* base = p.part + ((long long)t * MT + m) * p.ks1 * 128;
            if (tid < 64) {
                // shared expert: bf16(bf16(silu(bf16 g)) * bf16 u)   (fnx/engine.py:1788)
                const float g = round_bf(sum_parts(base, p.ks1, 2 * tid));
                const float u = round_bf(sum_parts(base, p.ks1, 2 * tid + 1));
                p.act_sh[(long long)t * p.I + m * 64 + tid] = f2bf(__fmul_rn(round_bf(silu_f32(g)), u));
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
// block (row, m, ks): routed gate/up tile m over H/ks2 of K for one (token, slot) row.
__global__ void __launch_bounds__(DEC_THREADS) decode_d2_kernel(const DecodeParams p) {
    __shared__ __align__(16) uint32_t xs2[DEC_MAX_K / 2];
    __shared__ float red[128];
    const int tid = threadIdx.x;
    const int MT = gu_tiles(p), KB = p.H / 64;
    const int b = blockIdx.x;
    const int ks = b % p.ks2, m = (b / p.ks2) % MT, row = b / (p.ks2 * MT);
    const int ex = __ldcg(p.idx + row), t = row / p.k;
    const int nkb = KB / p.ks2;
    stage_x(xs2, p.x + (long long)t * p.H, p.H);
    const long long tile = (long long)ex * MT + m;
    tile_dot(p.gu_tw + tile * KB * TILE_BLOCK_WORDS, xs2, ks * nkb, (ks + 1) * nkb, red);
    float* part = p.part2 + (((long long)row * MT + m) * p.ks2 + ks) * 128;
    if (tid < 128) part[tid] = red[tid];
    if (last_block(ctr_gu(p) + row * MT + m, p.ks2)) {
        const float* base = p.part2 + ((long long)row * MT + m) * p.ks2 * 128;
        if (tid < 64) {
            // routed expert: bf16(silu(g) * u) in fp32 on bf16-rounded gate/up
            const float g = round_bf(sum_parts(base, p.ks2, 2 * tid));
            const float u = round_bf(sum_parts(base, p.ks2, 2 * tid + 1));
            p.act[(long long)row * p.I + m * 64 + tid] = f2bf(__fmul_rn(silu_f32(g), u));
        }
    }
}

// ------------------------------------------------------------------ D3
// block (row, m): rows 0..M*k-1 are routed (token, slot) rows, rows M*k.. the shared
// expert of each token; output tile m = columns [128m, 128m+128), all of K = I.
__global__ void __launch_bounds__(DEC_THREADS) decode_d3_kernel(const DecodeParams p) {
    __shared__ __align__(16) uint32_t xs2[DEC_MAX_K / 2];
    __shared__ float red[128];
    const int tid = threadIdx.x;
    const int MT = dn_tiles(p), KB = p.I / 64;
    const int m = blockIdx.x % MT, row = blockIdx.x / MT;
    const int nrows = p.M * p.k;
    if (row < nrows) {
        const int ex = __ldcg(p.idx + row);
        stage_x(xs2, p.act + (long long)row * p.I, p.I);
        const long long tile = (long long)ex * MT + m;
        tile_dot(p.dn_tw + tile * KB * TILE_BLOCK_WORDS, xs2, 0, KB, red);
        if (tid < 128) p.yd[(long long)row * p.H + m * 128 + tid] = f2bf(red[tid]);
    } else {
        const int t = row - nrows;
        stage_x(xs2, p.act_sh + (long long)t * p.I, p.I);
        tile_dot(p.sh_dn_tw + (long long)m * KB * TILE_BLOCK_WORDS, xs2, 0, KB, red);
        if (tid < 128) p.sh[(long long)t * p.H + m * 128 + tid] = f2bf(red[tid]);
    }
    if (last_block(ctr_dn(p) + m, nrows + p.M)) {
        const unsigned short* yd = reinterpret_cast<const unsigned short*>(p.yd);
        const unsigned short* sh = reinterpret_cast<const unsigned short*>(p.sh);
        for (int i = tid; i < p.M * 128; i += DEC_THREADS) {
            const int t = i / 128, c = m * 128 + i % 128;
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
