// Decode (M <= 16 tokens) W4A16 MoE layer as one cooperative, HBM-bound GEMV kernel that
// runs as a dataflow over work items (described above decode_fused_kernel below).
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
constexpr int DEC_MAX_E = 512;           // routed experts
constexpr int DEC_CH = 16;               // k-blocks per bulk copy (69.6 KB of shared memory)
// dynamic shared memory of the decode kernels: one chunk of tile blocks, or D1's eight
// router rows of H <= DEC_MAX_K bf16
constexpr int DEC_SMEM = DEC_CH * TILE_BLOCK_BYTES > 8 * DEC_MAX_K * 2 ? DEC_CH * TILE_BLOCK_BYTES : 8 * DEC_MAX_K * 2;

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
// counters (zero between calls): tickets of the K-split groups, then the dataflow counts
FNX_DEV unsigned* ctr_sh(const DecodeParams& p) { return p.counters; }                                  // [M * I/64]
FNX_DEV unsigned* ctr_gu(const DecodeParams& p) { return ctr_sh(p) + p.M * gu_tiles(p); }              // [M*k * I/64]
FNX_DEV unsigned* ctr_router(const DecodeParams& p) { return ctr_gu(p) + p.M * p.k * gu_tiles(p); }    // router items done
FNX_DEV unsigned* ctr_routed(const DecodeParams& p) { return ctr_router(p) + 1; }                       // routing published
FNX_DEV unsigned* ctr_shgu_done(const DecodeParams& p) { return ctr_routed(p) + 1; }                    // [M] tiles of act_sh
FNX_DEV unsigned* ctr_gu_done(const DecodeParams& p) { return ctr_shgu_done(p) + p.M; }                 // [M*k] tiles of act
FNX_DEV unsigned* ctr_comb(const DecodeParams& p) { return ctr_gu_done(p) + p.M * p.k; }                // [M * H/128]
FNX_DEV unsigned* ctr_exit(const DecodeParams& p) { return ctr_comb(p) + p.M * dn_tiles(p); }
inline size_t decode_counters(int M, int H, int I, int k) {
    return (size_t)M * (I / 64) + (size_t)M * k * (I / 64) + 2 + M + (size_t)M * k + (size_t)M * (H / 128) + 1;
}

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

// Dot products of the 128 rows of one weight tile with x (bf16 [K], staged into xs2 while
// the first copies are in flight; x_cg reads it through L2) over k-blocks [kb0, kb1).  The
// tile blocks of a chunk of <= DEC_CH k-blocks are contiguous in HBM; thread 0 issues them
// as DEC_SUB-block bulk copies, each on its own mbarrier, all in flight at once, and the
// block computes each piece as soon as it lands, so compute overlaps the rest of the copy.
// Thread (half, r) takes k-block half of each piece of tile row r (conflict-free:
// consecutive rows are consecutive words) and the two halves are added in a fixed order.
// Result in red[r] (shared memory, 128 floats).  `phase` holds one parity bit per mbarrier.
#ifndef FNX_DEC_SUB
#define FNX_DEC_SUB 16
#endif
constexpr int DEC_SUB = FNX_DEC_SUB;             // k-blocks per bulk copy
constexpr int DEC_NBAR = DEC_CH / DEC_SUB;
FNX_DEV void tile_dot(const uint32_t* __restrict__ tw, const bf16* x, int K, bool x_cg, uint32_t* xs2, int kb0,
                      int kb1, uint32_t* wbuf, uint64_t* bar, uint32_t& phase, float* red) {
    const int r = threadIdx.x & 127, half = threadIdx.x >> 7;
    float a0 = 0.f, a1 = 0.f;
    for (int c0 = kb0; c0 < kb1; c0 += DEC_CH) {
        const int n = min(DEC_CH, kb1 - c0);
        const int npieces = (n + DEC_SUB - 1) / DEC_SUB;
        if (threadIdx.x == 0) {
            for (int s = 0; s < npieces; ++s) {
                const int nb = min(DEC_SUB, n - s * DEC_SUB);
                mbar_arrive_expect_tx(bar + s, (uint32_t)nb * TILE_BLOCK_BYTES);
                bulk_load(smem_u32(wbuf + s * DEC_SUB * TILE_BLOCK_WORDS),
                          tw + (long long)(c0 + s * DEC_SUB) * TILE_BLOCK_WORDS, (uint32_t)nb * TILE_BLOCK_BYTES,
                          bar + s, l2_evict_first());
            }
        }
        if (c0 == kb0) {                  // the input row, while the weights are in flight
            const uint32_t* src = reinterpret_cast<const uint32_t*>(x);
            for (int i = threadIdx.x; i < K / 2; i += blockDim.x) xs2[i] = x_cg ? __ldcg(src + i) : src[i];
            __syncthreads();
        }
        for (int s = 0; s < npieces; ++s) {
            mbar_wait(bar + s, (phase >> s) & 1u);   // a timeout is flagged; the block finishes with stale data
            phase ^= 1u << s;
            const int jend = min(n, (s + 1) * DEC_SUB);
            for (int j = s * DEC_SUB + half; j < jend; j += 2) {
                const uint32_t* blk = wbuf + j * TILE_BLOCK_WORDS;
                const uint32_t s16 = reinterpret_cast<const unsigned short*>(blk + 1024)[r];
                const uint32_t s2 = s16 | (s16 << 16);
                const uint4* xq = reinterpret_cast<const uint4*>(xs2 + (c0 + j) * 32);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t w = blk[tile_word(c, r)];
                    const uint4 xv = xq[c];
                    const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t w2 = tile_pair(w, i, s2);       // exactly rounded bf16(q * s)
                        fma_bf_lo(a0, w2, xx[i]);
                        fma_bf_hi(a1, w2, xx[i]);
                    }
                }
            }
        }
        __syncthreads();                  // wbuf is refilled by the next chunk
    }
    __shared__ float halves[2][128];
    halves[half][r] = __fadd_rn(a0, a1);
    __syncthreads();
    if (threadIdx.x < 128) red[r] = __fadd_rn(halves[0][r], halves[1][r]);
    __syncthreads();
}

// The block's bulk-copy mbarriers (initialised once per launch).
FNX_DEV void init_block_bar(uint64_t* bar, int n) {
    if (threadIdx.x == 0) {
        for (int i = 0; i < n; ++i) mbar_init(bar + i, 1);
        fence_mbar_init();
    }
    __syncthreads();
}

// Sum ks partials [ks][128] in order (read through L2: written by other blocks).
FNX_DEV float sum_parts(const float* base, int ks, int r) {
    float a = 0.f;
    for (int s = 0; s < ks; ++s) a = __fadd_rn(a, ld_cg_f32(base + s * 128 + r));
    return a;
}

// ------------------------------------------------------------------ the fused decode kernel
// One cooperative launch (every block resident) walking work items in this order, each block
// taking items blockIdx.x, blockIdx.x + gridDim.x, ...:
//   router rows     router + shared-gate logits, DEC_ROWS rows per item; the block finishing
//                   the last of them routes every token (top-k once) and publishes it
//   shared gate/up  (t, m, ks) K-split GEMV items; the last of a (t, m) group applies the
//                   shared expert's SwiGLU into act_sh and counts the tile for token t
//   routed gate/up  (row, m, ks) after the routing is published; the last of a group applies
//                   the fp32 SwiGLU into act and counts the tile for slot row
//   shared down     (t, m) once all act_sh tiles of token t are counted
//   routed down     (row, m) once all act tiles of slot row are counted
// The k routed down rows and the shared down tile of each (token, output tile) meet at a
// ticket; whichever arrives last combines them (slot-order weighted reduce + gated shared).
// Items only wait for items earlier in the order, and every block walks its items in order,
// so the lowest unfinished item can always run: no barrier is needed and none deadlocks.
// Waits are bounded (FNX_DEVERR_TIMEOUT) like every other spin here.

struct DecodeRouting {
    int idx[DEC_MAX_M * ROUTE_MAX_K];
    float wf[DEC_MAX_M * ROUTE_MAX_K];
};

FNX_DEV unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// thread 0 waits (bounded) until *c >= target; then the block synchronises
FNX_DEV void wait_count(const unsigned* c, unsigned target) {
    if (threadIdx.x == 0) {
        const uint64_t t0 = fnx_globaltimer();
        while (ld_acquire_u32(c) < target) {
            __nanosleep(32);
            if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
                fnx_flag_error(FNX_DEVERR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

// this block's results are visible device-wide before *c counts them
FNX_DEV void count_done(unsigned* c) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(c, 1u);
}

// DEC_ROWS consecutive router rows (rows >= E: the shared-expert gate) and, when it fits,
// the M token rows arrive by bulk copies; two warps per router row take half of H each and
// their fp32 partials are added in a fixed order.
constexpr int DEC_ROWS = 4;
FNX_DEV void router_rows(const DecodeParams& p, int item, uint32_t* wbuf, uint64_t* bar, uint32_t& phase) {
    __shared__ float partial[DEC_ROWS][2][DEC_MAX_M];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = item * DEC_ROWS;
    const int nr = min(DEC_ROWS, p.R - e0);
    const uint32_t rbytes = (uint32_t)nr * p.H * 2, xbytes = (uint32_t)p.M * p.H * 2;
    const bool x_in_smem = DEC_ROWS * p.H * 2 + (int)xbytes <= DEC_SMEM;
    const bf16* xs = x_in_smem ? reinterpret_cast<const bf16*>(wbuf) + DEC_ROWS * p.H : p.x;
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(bar, rbytes + (x_in_smem ? xbytes : 0u));
        bulk_load(smem_u32(wbuf), p.router + (long long)e0 * p.H, rbytes, bar, l2_evict_first());
        if (x_in_smem) bulk_load(smem_u32(xs), p.x, xbytes, bar, l2_evict_last());
    }
    mbar_wait(bar, phase & 1u);
    phase ^= 1u;
    const int row = warp >> 1, hh = warp & 1;
    if (row < nr) {
        const bf16* wr = reinterpret_cast<const bf16*>(wbuf) + (long long)row * p.H;
        for (int t0 = 0; t0 < p.M; t0 += 4) {          // tokens four at a time (register pressure)
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int c = hh * (p.H / 2) + lane * 8; c < (hh + 1) * (p.H / 2); c += 256) {
                const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    if (t0 + tt < p.M) {
                        const uint4 xv = *reinterpret_cast<const uint4*>(xs + (long long)(t0 + tt) * p.H + c);
                        const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            fma_bf_lo(acc[tt], ww[i], xx[i]);
                            fma_bf_hi(acc[tt], ww[i], xx[i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
                if (t0 + tt < p.M) {
                    float v = acc[tt];
#pragma unroll
                    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
                    if (lane == 0) partial[row][hh][t0 + tt] = v;
                }
            }
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nr * p.M; i += blockDim.x) {
        const int rr = i / p.M, t = i % p.M;
        p.logits[(long long)t * p.R + e0 + rr] = f2bf(__fadd_rn(partial[rr][0][t], partial[rr][1][t]));
    }
    __syncthreads();                       // wbuf and partial are reused by the next item
}

// Top-k of every token (the router kernel's rule) into shared memory and the workspace /
// outputs; run by one block.
FNX_DEV void route_tokens(const DecodeParams& p, DecodeRouting& R) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < p.M; t += DEC_THREADS / 32) {
        const bf16* row = p.logits + (long long)t * p.R;
        float my_p, tot;
        int my_i;
        // E <= DEC_MAX_E (wider routers would hold 64+ keys per lane and spill the kernel)
        if (p.E <= 256) topk_warp<8, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
        else topk_warp<16, true>(row, p.bias, p.E, p.k, my_p, my_i, tot);
        if (lane < p.k) {
            const bf16 wb = f2bf(my_p / tot);
            const int o = t * p.k + lane;
            R.idx[o] = my_i;
            R.wf[o] = bf2f(wb);
            p.wf[o] = bf2f(wb);
            p.idx[o] = my_i;
            if (p.w_out) p.w_out[o] = wb;
            if (p.idx_out) p.idx_out[o] = my_i;
        }
    }
    __syncthreads();
}

// Top-k of one token by all 8 warps (the decode of a single token): warp w takes a slice of
// E/8 experts, picks its own top-k by (probability desc, id asc), and warp 0 merges the 8 lists
// by the same order.  Probabilities are the router kernel's softmax (max, exp, sum in a fixed
// order, then * 1/sum); NaN counts as 0, so k valid distinct ids are always chosen.
FNX_DEV void route_one_token_block(const DecodeParams& p, DecodeRouting& R) {
    __shared__ float s_red[8];
    __shared__ uint32_t c_key[8][ROUTE_MAX_K];
    __shared__ int c_id[8][ROUTE_MAX_K];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (p.E + 7) / 8;                        // experts per warp (<= 64)
    const unsigned short* row = reinterpret_cast<const unsigned short*>(p.logits);
    int e[2];
    float v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        e[h] = warp * S + h * 32 + lane;
        v[h] = -INFINITY;
        if (h * 32 + lane < S && e[h] < p.E) {
            v[h] = __uint_as_float((uint32_t)__ldcg(row + e[h]) << 16);
            if (p.bias) v[h] = __fadd_rn(v[h], p.bias[e[h]]);
        }
    }
    float mx = fmaxf(v[0], v[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_red[w]);
    float pr[2], sum;
#pragma unroll
    for (int h = 0; h < 2; ++h) pr[h] = v[h] == -INFINITY ? 0.f : expf(__fsub_rn(v[h], mx));
    sum = __fadd_rn(pr[0], pr[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    __syncthreads();                                    // every warp has read s_red (max)
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = s_red[0];
    for (int w = 1; w < 8; ++w) sum = __fadd_rn(sum, s_red[w]);
    const float inv = 1.0f / sum;
    uint32_t key[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float q = __fmul_rn(pr[h], inv);
        key[h] = (h * 32 + lane < S && e[h] < p.E) ? __float_as_uint(q > 0.f ? q : 0.f) + 1u : 0u;
    }
    for (int j = 0; j < p.k; ++j) {                     // this warp's top-k
        const uint32_t gm = __reduce_max_sync(0xffffffffu, max(key[0], key[1]));
        const uint32_t cand = key[0] == gm ? (uint32_t)e[0] : (key[1] == gm ? (uint32_t)e[1] : 0xffffffffu);
        const uint32_t bi = __reduce_min_sync(0xffffffffu, gm ? cand : 0xffffffffu);
        if (gm && (uint32_t)e[0] == bi) key[0] = 0u;
        if (gm && (uint32_t)e[1] == bi) key[1] = 0u;
        if (lane == 0) { c_key[warp][j] = gm; c_id[warp][j] = (int)bi; }
    }
    __syncthreads();
    if (warp == 0) {                                    // merge the 8 lists
        uint32_t ck[8];
        int ci[8];
        const int n = 8 * p.k;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int c = s * 32 + lane;
            ck[s] = c < n ? c_key[c / p.k][c % p.k] : 0u;
            ci[s] = c < n ? c_id[c / p.k][c % p.k] : 0x7fffffff;
        }
        float my_p = 0.f, tot = 0.f;
        int my_i = 0;
        for (int j = 0; j < p.k; ++j) {
            uint32_t lm = 0;
#pragma unroll
            for (int s = 0; s < 8; ++s) lm = max(lm, ck[s]);
            const uint32_t gm = __reduce_max_sync(0xffffffffu, lm);
            uint32_t cand = 0xffffffffu;
#pragma unroll
            for (int s = 0; s < 8; ++s)
                if (ck[s] == gm && gm) cand = min(cand, (uint32_t)ci[s]);
            const uint32_t bi = __reduce_min_sync(0xffffffffu, cand);
#pragma unroll
            for (int s = 0; s < 8; ++s)
                if (ck[s] == gm && (uint32_t)ci[s] == bi) ck[s] = 0u;
            const float bp = gm ? __uint_as_float(gm - 1u) : 0.f;
            if (lane == j) { my_p = bp; my_i = (int)bi; }
            tot = __fadd_rn(tot, bp);
        }
        if (lane < p.k) {
            const bf16 wb = f2bf(my_p / tot);
            R.idx[lane] = my_i;
            R.wf[lane] = bf2f(wb);
            p.wf[lane] = bf2f(wb);
            p.idx[lane] = my_i;
            if (p.w_out) p.w_out[lane] = wb;
            if (p.idx_out) p.idx_out[lane] = my_i;
        }
    }
    __syncthreads();
}

// the published routing into shared memory (after the flag)
FNX_DEV void load_routing(const DecodeParams& p, DecodeRouting& R) {
    wait_count(ctr_routed(p), 1u);
    for (int i = threadIdx.x; i < p.M * p.k; i += blockDim.x) {
        R.idx[i] = __ldcg(p.idx + i);
        R.wf[i] = ld_cg_f32(p.wf + i);
    }
    __syncthreads();
}

// out[t, 128m .. 128m+127]: the slot-order weighted reduce of the k routed rows and the
// sigmoid-gated shared row (kernels/reduce/reduce.cpp + kernels/post_ops/post_ops.cpp rounding)
FNX_DEV void combine_tile(const DecodeParams& p, const DecodeRouting& R, int t, int m) {
    const unsigned short* yd = reinterpret_cast<const unsigned short*>(p.yd);
    const unsigned short* sh = reinterpret_cast<const unsigned short*>(p.sh);
    const unsigned short* lg = reinterpret_cast<const unsigned short*>(p.logits);
    if (threadIdx.x < 128) {
        const int c = m * 128 + threadIdx.x;
        float acc = 0.f;
        for (int j = 0; j < p.k; ++j) {
            const float y = __uint_as_float((uint32_t)__ldcg(yd + (long long)(t * p.k + j) * p.H + c) << 16);
            acc = __fadd_rn(acc, round_bf(__fmul_rn(y, R.wf[t * p.k + j])));
        }
        const float a = round_bf(acc);
        const float g = __uint_as_float((uint32_t)__ldcg(lg + (long long)t * p.R + p.E) << 16);
        const float sg = round_bf(sigmoid_f32(g));
        const float s = __uint_as_float((uint32_t)__ldcg(sh + (long long)t * p.H + c) << 16);
        p.out[(long long)t * p.H + c] = f2bf(__fadd_rn(a, round_bf(__fmul_rn(s, sg))));
    }
}

__global__ void __launch_bounds__(DEC_THREADS, 2) decode_fused_kernel(const DecodeParams p) {
    extern __shared__ __align__(16) uint32_t wbuf[];
    __shared__ __align__(16) uint32_t xs2[DEC_MAX_K / 2];
    __shared__ float red[128];
    __shared__ uint64_t bar[DEC_NBAR];
    __shared__ DecodeRouting R;
    __shared__ unsigned s_last;
    uint32_t phase = 0;
    bool have_routing = false;                          // block-uniform
    const int tid = threadIdx.x;
    const int MT = gu_tiles(p), KB = p.H / 64;          // gate/up: I/64 feature tiles over K = H
    const int MTd = dn_tiles(p), KBd = p.I / 64;        // down: H/128 feature tiles over K = I
    const int RB = (p.R + DEC_ROWS - 1) / DEC_ROWS;
    const int nsh = p.M * MT * p.ks1, ngu = p.M * p.k * MT * p.ks2, nsd = p.M * MTd, ndn = p.M * p.k * MTd;
    const int total = RB + nsh + ngu + nsd + ndn;
    init_block_bar(bar, DEC_NBAR);

    for (int it = blockIdx.x; it < total; it += gridDim.x) {
        int b = it;
        if (b < RB) {                                    // ---- router rows
            router_rows(p, b, wbuf, bar, phase);
            __threadfence();
            __syncthreads();
            if (tid == 0) s_last = atomicAdd(ctr_router(p), 1u) == (unsigned)RB - 1;
            __syncthreads();
            if (s_last) {                                // every logit is out: route once
                __threadfence();
                if (p.M == 1) route_one_token_block(p, R);
                else route_tokens(p, R);
                __threadfence();
                __syncthreads();
                if (tid == 0) atomicExch(ctr_routed(p), 1u);
                have_routing = true;
            }
            continue;
        }
        b -= RB;
        if (b < nsh) {                                   // ---- shared gate/up
            const int ks = b % p.ks1, m = (b / p.ks1) % MT, t = b / (p.ks1 * MT);
            tile_dot(p.sh_gu_tw + (long long)m * KB * TILE_BLOCK_WORDS, p.x + (long long)t * p.H, p.H, false, xs2,
                     ks * KB / p.ks1, (ks + 1) * KB / p.ks1, wbuf, bar, phase, red);
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
                count_done(ctr_shgu_done(p) + t);
            }
            continue;
        }
        b -= nsh;
        if (!have_routing) {                             // every later item needs the routing
            load_routing(p, R);
            have_routing = true;
        }
        if (b < ngu) {                                   // ---- routed gate/up
            const int ks = b % p.ks2, m = (b / p.ks2) % MT, row = b / (p.ks2 * MT);
            const int ex = R.idx[row], t = row / p.k;
            tile_dot(p.gu_tw + ((long long)ex * MT + m) * KB * TILE_BLOCK_WORDS, p.x + (long long)t * p.H, p.H, false,
                     xs2, ks * KB / p.ks2, (ks + 1) * KB / p.ks2, wbuf, bar, phase, red);
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
                count_done(ctr_gu_done(p) + row);
            }
            continue;
        }
        b -= ngu;
        int t, m;
        if (b < nsd) {                                   // ---- shared down
            m = b % MTd;
            t = b / MTd;
            wait_count(ctr_shgu_done(p) + t, (unsigned)MT);
            tile_dot(p.sh_dn_tw + (long long)m * KBd * TILE_BLOCK_WORDS, p.act_sh + (long long)t * p.I, p.I, true, xs2,
                     0, KBd, wbuf, bar, phase, red);
            if (tid < 128) p.sh[(long long)t * p.H + m * 128 + tid] = f2bf(red[tid]);
        } else {                                         // ---- routed down
            b -= nsd;
            m = b % MTd;
            const int row = b / MTd;
            t = row / p.k;
            const int ex = R.idx[row];
            wait_count(ctr_gu_done(p) + row, (unsigned)MT);
            tile_dot(p.dn_tw + ((long long)ex * MTd + m) * KBd * TILE_BLOCK_WORDS, p.act + (long long)row * p.I, p.I,
                     true, xs2, 0, KBd, wbuf, bar, phase, red);
            if (tid < 128) p.yd[(long long)row * p.H + m * 128 + tid] = f2bf(red[tid]);
        }
        if (last_block(ctr_comb(p) + t * MTd + m, (unsigned)p.k + 1)) combine_tile(p, R, t, m);
    }

    // ---- the last block to leave re-arms the dataflow counts for the next call
    if (last_block(ctr_exit(p), gridDim.x)) {
        for (int i = tid; i < 2 + p.M + p.M * p.k; i += blockDim.x) ctr_router(p)[i] = 0;
    }
}

}  // namespace fnx
