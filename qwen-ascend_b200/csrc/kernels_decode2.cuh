// Decode (M <= 16 tokens) W4A16 MoE layer: the whole layer in one cooperative launch, a
// dataflow over work items whose hand-offs between CTAs are single stores and reads.
//
// This is the reference's decode branch (fnx/engine.py:1786-1889: concatenated shared GEMM,
// softmax/top-k, gather + W4A16 gate/up, fp32 swiglu, down, kernels/moe_epilogue) computed
// without the Cartesian product and without copying the selected experts.  Work items, in
// their global order (CTA b takes items b, b + grid, ...):
//   router   router rows (+ the shared-expert gate row) -> logits
//   shgu     shared gate/up, (token, 128-feature tile, K range) -> fp32 partials
//   gu       routed gate/up, (slot, tile, K range) -> fp32 partials
//   shdn     shared down, (token, 128-feature tile): the item sums all of the token's shared
//            partials in K order, applies the shared SwiGLU into shared memory and computes its
//            tile of sh
//   dn       routed down, (slot, tile): the same from the slot's partials with the fp32 SwiGLU,
//            its tile of yd
//   comb     (token, tile): the slot-order weighted reduce of the k routed rows and the
//            sigmoid-gated shared row into out
// Cross-CTA values are tagged: each is a 64-bit word of a 32-bit payload and the launch's
// 32-bit tag, stored and loaded with single-copy atomicity (st/ld.relaxed.gpu.b64).  A consumer
// reads exactly the words it needs and spins (bounded) until each carries this launch's tag, so
// a hand-off costs one store and one read: no counters, fences or tickets.  The tag is the
// workspace's launch counter (a word at offset 0, bumped by the last CTA to leave) plus one, so
// the words of earlier launches never match and nothing is cleared between calls.
// Each CTA has two roles:
//   * eight compute warps walk the items, staging each item's input row in shared memory and
//     running its weight stages through the tensor cores (mma m16n8k16 on the exactly rounded
//     dequantised weights bf16(q * s), fp32 accumulation);
//   * a copy warp issues the bulk copies of every stage of every item in order into a ring of
//     D2_NS stages, running ahead across items (a down item's weights land while the gate/up
//     results it needs are still being produced).
// Routing has no single owner: each CTA computes the top-k of the tokens its own items touch
// from the tagged logits (a pure function of them: every CTA derives the same ids) and hands
// the expert ids to its copy warp.  Waits only point to items earlier in the global order and
// every CTA walks its items in order, so with all CTAs resident the lowest unfinished item can
// always run.  Every wait is bounded (FNX_WAIT_NS): after a CTA's first timeout it stops
// waiting and finishes its items on whatever data is there (the error word records it).
#pragma once
#include "kernels_decode.cuh"
#include "kernels_hc.cuh"

namespace fnx {

constexpr int D2_CWARPS = 8;                          // compute warps: 16 tile rows each
constexpr int D2_CTHREADS = 32 * D2_CWARPS;
constexpr int D2_COPY_WARP = D2_CWARPS;               // warp 8
constexpr int D2_THREADS = 32 * (D2_CWARPS + 1);
// Ring geometry: two stages of eight tile blocks (35 KB copies).  Measured at M = 1 / 4 (us per
// layer): 2 x 8 blocks 22.7 / 46.7, 1 x 16 22.4 / 50.4, 3 x 6 23.7 / 55.2, 5 x 4 23.8 / 55.8,
// 10 x 2 24.4 / 57.7: a bulk copy has a fixed cost, so fewer, larger copies stream faster.
#ifndef FNX_D2_SK
#define FNX_D2_SK 8
#endif
#ifndef FNX_D2_NS
#define FNX_D2_NS 2
#endif
constexpr int D2_SK = FNX_D2_SK;                      // tile blocks per stage
constexpr int D2_NS = FNX_D2_NS;                      // stages in the ring
constexpr int D2_STAGE_BYTES = D2_SK * TILE_BLOCK_BYTES;
constexpr int D2_RING_BYTES = D2_NS * D2_STAGE_BYTES; // 69,632 B at 2 x 8
constexpr int D2_XRES_BYTES = 16384;                  // the M token rows, resident when M*H*2 fits
constexpr int D2_SMEM = D2_RING_BYTES + D2_XRES_BYTES;
constexpr int D2_BAR = 1;                             // named barrier of the compute warps
constexpr int D2_MAX_ROWS = 4;                        // router rows per item

// router rows per item: as many as fit a stage (4, 2 or 1, so that a row splits evenly over warps)
__host__ __device__ inline int d2_router_rows(int H) {
    const int fit = D2_STAGE_BYTES / (2 * H);
    return fit >= 4 ? 4 : (fit >= 2 ? 2 : 1);
}

typedef unsigned long long tword;                     // (payload, tag) in one 64-bit word

struct StreamParams {
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
    unsigned* epoch;                 // launches completed on this workspace
    unsigned* exit;                  // exit ticket (zero between calls)
    tword* tlog;                     // [M][R]            bf16 logit
    tword* tpart;                    // [M][I/64][ks1][128] fp32 shared gate/up partial
    tword* tpart2;                   // [M*k][I/64][ks2][128] fp32 routed gate/up partial
    tword* tyd;                      // [M*k][H/2]         bf16x2 routed down row
    tword* tsh;                      // [M][H/2]           bf16x2 shared down row
    int M, H, I, E, k, R;
    int ks1, ks2;                    // K splits of the shared and routed gate/up GEMVs
    int logits_ready;                // 1: tlog already carries this launch's tagged logits
                                     // (hc_mix_router_kernel ran before), so the router items are
                                     // empty (kept, so every other item runs on the same block)
};

FNX_DEV void st_tag(tword* p, uint32_t payload, uint32_t tag) {
    const tword v = (tword)payload | ((tword)tag << 32);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
FNX_DEV tword ld_tag(const tword* p) {
    tword v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// One thread waits (bounded) until the word at p carries `tag`, backing off exponentially from
// 32 to FNX_D2_BACKOFF_MAX ns between reads, so that many waiting CTAs do not flood the L2 with
// polls.
#ifndef FNX_D2_BACKOFF_MAX
#define FNX_D2_BACKOFF_MAX 64
#endif
FNX_DEV void poll_tag(const tword* p, uint32_t tag, volatile int* dead) {
    if (*dead || (uint32_t)(ld_tag(p) >> 32) == tag) return;
    const uint64_t t0 = fnx_globaltimer();
    unsigned ns = 32;
    while (true) {
        __nanosleep(ns);
        if (ns < FNX_D2_BACKOFF_MAX) ns <<= 1;
        if ((uint32_t)(ld_tag(p) >> 32) == tag || *dead) return;
        if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
            fnx_flag_error(FNX_DEVERR_TIMEOUT);
            *dead = 1;
            return;
        }
    }
}

// v[i] (i < N, the words p0 + i * stride, those with i >= n unused) all carrying `tag`: every
// word is requested at once, then the ones still pending are requested again together (with
// back-off) until none is (bounded).
template <int N>
FNX_DEV void read_tagged(tword (&v)[N], const tword* p0, long long stride, int n, uint32_t tag, volatile int* dead) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = i < n ? ld_tag(p0 + i * stride) : ((tword)tag << 32);
    const uint64_t t0 = fnx_globaltimer();
    unsigned ns = 32;
    while (true) {
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok &= (uint32_t)(v[i] >> 32) == tag;
        if (ok || *dead) return;
        __nanosleep(ns);
        if (ns < FNX_D2_BACKOFF_MAX) ns <<= 1;
#pragma unroll
        for (int i = 0; i < N; ++i)
            if ((uint32_t)(v[i] >> 32) != tag) v[i] = ld_tag(p0 + i * stride);
        if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
            fnx_flag_error(FNX_DEVERR_TIMEOUT);
            *dead = 1;
            return;
        }
    }
}

// read_tagged over N words at computed addresses (addr(i), for the bits of `valid`): every load is
// issued before any tag is checked, so words from many producers cost one L2 round trip together.
template <int N, class F>
FNX_DEV void read_tagged_fn(tword (&v)[N], F addr, uint32_t valid, uint32_t tag, volatile int* dead) {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = ((valid >> i) & 1u) ? ld_tag(addr(i)) : ((tword)tag << 32);
    const uint64_t t0 = fnx_globaltimer();
    unsigned ns = 32;
    while (true) {
        bool ok = true;
#pragma unroll
        for (int i = 0; i < N; ++i) ok &= (uint32_t)(v[i] >> 32) == tag;
        if (ok || *dead) return;
        __nanosleep(ns);
        if (ns < FNX_D2_BACKOFF_MAX) ns <<= 1;
#pragma unroll
        for (int i = 0; i < N; ++i)
            if ((uint32_t)(v[i] >> 32) != tag) v[i] = ld_tag(addr(i));
        if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
            fnx_flag_error(FNX_DEVERR_TIMEOUT);
            *dead = 1;
            return;
        }
    }
}

enum D2Type { D2_ROUTER = 0, D2_SHGU = 1, D2_GU = 2, D2_SHDN = 3, D2_DN = 4, D2_COMB = 5 };

struct D2Item {
    int type;
    int t, row, m, ks;
    int kb0, kb1;             // k-block range of the tile run (router: rows [kb0, kb1))
    const uint32_t* src;      // k-block 0 of the tile run (router: row kb0)
};

struct D2Shape {
    int RB, nrow, nsh, ngu, nsd, ndn, ncb, total, MT, KB, MTd, KBd;
};

FNX_DEV D2Shape d2_shape(const StreamParams& p) {
    D2Shape s;
    s.nrow = d2_router_rows(p.H);
    s.RB = (p.R + s.nrow - 1) / s.nrow;              // with logits_ready: empty items, same placement
    s.MT = p.I / 64;
    s.KB = p.H / 64;
    s.MTd = p.H / 128;
    s.KBd = p.I / 64;
    s.nsh = p.M * s.MT * p.ks1;
    s.ngu = p.M * p.k * s.MT * p.ks2;
    s.nsd = p.M * s.MTd;
    s.ndn = p.M * p.k * s.MTd;
    s.ncb = p.M * s.MTd;
    s.total = s.RB + s.nsh + s.ngu + s.nsd + s.ndn + s.ncb;
    return s;
}

// Position of item `it` in the global order (type, token, slot, tile, K range); no expert id.
FNX_DEV D2Item d2_item_pos(const StreamParams& p, const D2Shape& S, int it) {
    D2Item d{};
    int b = it;
    if (b < S.RB) {
        d.type = D2_ROUTER;
        d.kb0 = b * S.nrow;
        d.kb1 = min(p.R, d.kb0 + S.nrow);
        return d;
    }
    b -= S.RB;
    if (b < S.nsh) {
        d.type = D2_SHGU;
        d.ks = b % p.ks1;
        d.m = (b / p.ks1) % S.MT;
        d.t = b / (p.ks1 * S.MT);
        d.kb0 = d.ks * S.KB / p.ks1;
        d.kb1 = (d.ks + 1) * S.KB / p.ks1;
        return d;
    }
    b -= S.nsh;
    if (b < S.ngu) {
        d.type = D2_GU;
        d.ks = b % p.ks2;
        d.m = (b / p.ks2) % S.MT;
        d.row = b / (p.ks2 * S.MT);
        d.t = d.row / p.k;
        d.kb0 = d.ks * S.KB / p.ks2;
        d.kb1 = (d.ks + 1) * S.KB / p.ks2;
        return d;
    }
    b -= S.ngu;
    if (b < S.nsd) {
        d.type = D2_SHDN;
        d.m = b % S.MTd;
        d.t = b / S.MTd;
        d.kb0 = 0;
        d.kb1 = S.KBd;
        return d;
    }
    b -= S.nsd;
    if (b < S.ndn) {
        d.type = D2_DN;
        d.m = b % S.MTd;
        d.row = b / S.MTd;
        d.t = d.row / p.k;
        d.kb0 = 0;
        d.kb1 = S.KBd;
        return d;
    }
    b -= S.ndn;
    d.type = D2_COMB;
    d.m = b % S.MTd;
    d.t = b / S.MTd;
    return d;
}

FNX_DEV int d2_expert(const StreamParams& p, const DecodeRouting& R, int row) {
    int ex = R.idx[row];
    if (ex < 0 || ex >= p.E) {
        fnx_flag_error(FNX_DEVERR_BADID);
        ex = 0;
    }
    return ex;
}

// The item with its weight source (routed items read the expert id from the routing in R;
// an id outside [0, E) is flagged and read as expert 0).
FNX_DEV D2Item d2_item(const StreamParams& p, const D2Shape& S, const DecodeRouting& R, int it) {
    D2Item d = d2_item_pos(p, S, it);
    switch (d.type) {
    case D2_ROUTER: d.src = reinterpret_cast<const uint32_t*>(p.router + (long long)d.kb0 * p.H); break;
    case D2_SHGU: d.src = p.sh_gu_tw + (long long)d.m * S.KB * TILE_BLOCK_WORDS; break;
    case D2_GU:
        d.src = p.gu_tw + ((long long)d2_expert(p, R, d.row) * S.MT + d.m) * S.KB * TILE_BLOCK_WORDS;
        break;
    case D2_SHDN: d.src = p.sh_dn_tw + (long long)d.m * S.KBd * TILE_BLOCK_WORDS; break;
    case D2_DN:
        d.src = p.dn_tw + ((long long)d2_expert(p, R, d.row) * S.MTd + d.m) * S.KBd * TILE_BLOCK_WORDS;
        break;
    default: d.src = nullptr;
    }
    return d;
}

FNX_DEV int d2_stages(const D2Item& d) {
    if (d.type == D2_COMB) return 0;
    return d.type == D2_ROUTER ? 1 : (d.kb1 - d.kb0 + D2_SK - 1) / D2_SK;
}

// ------------------------------------------------------------------ routing
// Top-k of token t by one warp, with router_topk_kernel's rule and arithmetic (topk_warp: 16
// experts per lane, max, exp, the lane-then-shuffle sum, reciprocal), so decode and prefill route
// identically given the same logits: (probability desc, id asc), k distinct valid ids, weights
// bf16(p / sum of the k selected p in slot order).  The logits are read as they arrive (tagged).
//
// Selection: topk_select (kernels_route.cuh), the binned candidate ranking with the sequential
// rounds as its fallback -- the same selection and order as router_topk_kernel.
constexpr int D2_RPER = 16;                           // experts per lane (E <= 512)
constexpr int D2_RBINS = 64;                          // the selection's bins (d2_route_block)

FNX_DEV void d2_route_warp(const StreamParams& p, DecodeRouting& R, int t, uint32_t tag, volatile int* dead,
                           TopkScratch& W) {
    const int lane = threadIdx.x & 31;
    const tword* row = p.tlog + (long long)t * p.R;
    tword wv[D2_RPER];
    read_tagged<D2_RPER>(wv, row + lane, 32, (p.E - lane + 31) / 32, tag, dead);
    float v[D2_RPER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < D2_RPER; ++i) {
        const int e = i * 32 + lane;
        float x = -INFINITY;
        if (e < p.E) {
            x = __uint_as_float((uint32_t)wv[i] << 16);
            if (p.bias) x = __fadd_rn(x, p.bias[e]);
        }
        v[i] = x;
        mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < D2_RPER; ++i) {
        const int e = i * 32 + lane;
        const float pe = e < p.E ? expf(__fsub_rn(v[i], mx)) : 0.f;
        v[i] = pe;
        sum = __fadd_rn(sum, pe);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float inv = 1.0f / sum;
    uint32_t key[D2_RPER];
#pragma unroll
    for (int i = 0; i < D2_RPER; ++i) {
        const float pr = __fmul_rn(v[i], inv);
        key[i] = (i * 32 + lane) < p.E ? __float_as_uint(pr > 0.f ? pr : 0.f) + 1u : 0u;
    }
    float my_p, tot;
    int my_i;
    topk_select<D2_RPER>(key, p.k, W, my_p, my_i, tot);
    if (lane < p.k) {
        const bf16 wb = f2bf(my_p / tot);
        const int o = t * p.k + lane;
        R.idx[o] = my_i;
        R.wf[o] = bf2f(wb);
        if (p.w_out) p.w_out[o] = wb;
        if (p.idx_out) p.idx_out[o] = my_i;
    }
}

// Top-k of one token by the eight compute warps (the single-token decode: eight experts' worth of
// softmax per lane instead of sixteen, and the selection of d2_route_warp).  The arithmetic is
// route_one_token_block's (slices of E/8 experts per warp, the warp sums added in warp order).
FNX_DEV void d2_route_block(const StreamParams& p, DecodeRouting& R, int t, uint32_t tag, volatile int* dead) {
    __shared__ float s_red[8];
    __shared__ uint32_t s_umax[8];
    __shared__ int s_cnt[D2_RBINS];
    __shared__ uint32_t c_key[8][ROUTE_MAX_K];
    __shared__ int c_id[8][ROUTE_MAX_K];
    __shared__ int s_n, s_bstar;
    __shared__ float s_prob[ROUTE_MAX_K];
    __shared__ int s_sid[ROUTE_MAX_K];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = (p.E + 7) / 8;
    const tword* row = p.tlog + (long long)t * p.R;
    if (threadIdx.x < D2_RBINS) s_cnt[threadIdx.x] = 0;
    if (threadIdx.x == 0) s_n = 0;
    const int e0 = warp * S + lane;
    const bool ok0 = lane < S && e0 < p.E, ok1 = 32 + lane < S && e0 + 32 < p.E;
    tword wv[2];
    read_tagged<2>(wv, row + e0, 32, ok1 ? 2 : (ok0 ? 1 : 0), tag, dead);
    int e[2] = {e0, e0 + 32};
    float v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        v[h] = -INFINITY;
        if (h ? ok1 : ok0) {
            v[h] = __uint_as_float((uint32_t)wv[h] << 16);
            if (p.bias) v[h] = __fadd_rn(v[h], p.bias[e[h]]);
        }
    }
    float mx = fmaxf(v[0], v[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    named_bar_sync(D2_BAR, D2_CTHREADS);
    mx = s_red[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_red[w]);
    float pr[2], sum;
#pragma unroll
    for (int h = 0; h < 2; ++h) pr[h] = v[h] == -INFINITY ? 0.f : expf(__fsub_rn(v[h], mx));
    sum = __fadd_rn(pr[0], pr[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    named_bar_sync(D2_BAR, D2_CTHREADS);
    if (lane == 0) s_red[warp] = sum;
    named_bar_sync(D2_BAR, D2_CTHREADS);
    sum = s_red[0];
    for (int w = 1; w < 8; ++w) sum = __fadd_rn(sum, s_red[w]);
    const float inv = 1.0f / sum;
    uint32_t key[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float q = __fmul_rn(pr[h], inv);
        key[h] = (h ? ok1 : ok0) ? __float_as_uint(q > 0.f ? q : 0.f) + 1u : 0u;
    }
    const uint32_t wmax = __reduce_max_sync(0xffffffffu, max(key[0], key[1]));
    if (lane == 0) s_umax[warp] = wmax;
    named_bar_sync(D2_BAR, D2_CTHREADS);
    uint32_t kmax = s_umax[0];
    for (int w = 1; w < 8; ++w) kmax = max(kmax, s_umax[w]);
    int bin[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t dist = kmax - key[h];
        bin[h] = key[h] && (dist >> 19) < (uint32_t)D2_RBINS ? (int)(dist >> 19) : D2_RBINS;
        if (bin[h] < D2_RBINS) atomicAdd(&s_cnt[bin[h]], 1);
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
    if (warp == 0) {
        const int c0 = s_cnt[2 * lane], c1 = s_cnt[2 * lane + 1];
        int incl = c0 + c1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const int excl = incl - c0 - c1;
        const bool hit0 = excl + c0 >= p.k, hit1 = incl >= p.k;
        const unsigned bal = __ballot_sync(0xffffffffu, hit0 || hit1);
        int bstar = -1, cnt = 0;
        if (bal) {
            const int l = __ffs(bal) - 1;
            bstar = __shfl_sync(0xffffffffu, hit0 ? 2 * lane : 2 * lane + 1, l);
            cnt = __shfl_sync(0xffffffffu, hit0 ? excl + c0 : incl, l);
        }
        if (lane == 0) s_bstar = (bstar >= 0 && cnt <= 32) ? bstar : -1;
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
    const int bstar = s_bstar;
    if (bstar >= 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (bin[h] <= bstar) {
                const int slot = atomicAdd(&s_n, 1);
                c_key[0][slot] = key[h];
                c_id[0][slot] = e[h];
            }
        }
        named_bar_sync(D2_BAR, D2_CTHREADS);
        if (warp == 0) {
            const int n = s_n;
            const uint32_t mk = lane < n ? c_key[0][lane] : 0u;
            const int mi = lane < n ? c_id[0][lane] : 0x7fffffff;
            int rank = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t kj = __shfl_sync(0xffffffffu, mk, j);
                const int ij = __shfl_sync(0xffffffffu, mi, j);
                rank += (kj > mk || (kj == mk && ij < mi)) ? 1 : 0;
            }
            if (lane < n && rank < p.k) {
                s_prob[rank] = __uint_as_float(mk - 1u);
                s_sid[rank] = mi;
            }
            __syncwarp();
            float tot = 0.f;
            for (int j = 0; j < p.k; ++j) tot = __fadd_rn(tot, s_prob[j]);
            if (lane < p.k) {
                const bf16 wb = f2bf(s_prob[lane] / tot);
                const int o = t * p.k + lane;
                R.idx[o] = s_sid[lane];
                R.wf[o] = bf2f(wb);
                if (p.w_out) p.w_out[o] = wb;
                if (p.idx_out) p.idx_out[o] = s_sid[lane];
            }
        }
        named_bar_sync(D2_BAR, D2_CTHREADS);
        return;
    }
    // sequential selection: per-warp top-k over its slice, then warp 0 merges the 8 lists
    for (int j = 0; j < p.k; ++j) {
        const uint32_t gm = __reduce_max_sync(0xffffffffu, max(key[0], key[1]));
        const uint32_t cand = key[0] == gm ? (uint32_t)e[0] : (key[1] == gm ? (uint32_t)e[1] : 0xffffffffu);
        const uint32_t bi = __reduce_min_sync(0xffffffffu, gm ? cand : 0xffffffffu);
        if (gm && (uint32_t)e[0] == bi) key[0] = 0u;
        if (gm && (uint32_t)e[1] == bi) key[1] = 0u;
        if (lane == 0) { c_key[warp][j] = gm; c_id[warp][j] = (int)bi; }
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
    if (warp == 0) {
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
            const int o = t * p.k + lane;
            R.idx[o] = my_i;
            R.wf[o] = bf2f(wb);
            if (p.w_out) p.w_out[o] = wb;
            if (p.idx_out) p.idx_out[o] = my_i;
        }
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
}

// The down GEMV's input row in shared memory: feature j = 64m + i of the SwiGLU from the K-split
// partials [MT][ks][128] of one slot (gate on tile row 2i, up on 2i+1), each summed in K order:
// routed bf16(silu(g) * u) in fp32 on bf16-rounded g and u; shared bf16(bf16(silu(g)) * u).
// One thread per producing item first waits for that item's first word; then every thread reads
// its partials, eight K ranges at a time.
FNX_DEV void d2_build_act(const tword* part, int MT, int ks, int I, bool shared_form, uint32_t tag,
                          volatile int* dead, uint32_t* xs2) {
    for (int i = threadIdx.x; i < MT * ks; i += D2_CTHREADS) poll_tag(part + (long long)i * 128, tag, dead);
    named_bar_sync(D2_BAR, D2_CTHREADS);
    for (int w = threadIdx.x; w < I / 2; w += D2_CTHREADS) {       // word w: features 2w, 2w+1
        const int j = 2 * w, m = j >> 6, i = j & 63;
        const tword* base = part + (long long)m * ks * 128 + 2 * i;  // rows 2i .. 2i+3 of tile m
        float g0 = 0.f, u0 = 0.f, g1 = 0.f, u1 = 0.f;
        for (int s0 = 0; s0 < ks; s0 += 8) {
            const int n = min(8, ks - s0);
            // v[8r + s]: word r of the 4 (g0, u0, g1, u1) in K part s0 + s; all 4n loads in flight
            tword v[32];
            const uint32_t m8 = (1u << n) - 1u;
            const tword* b0 = base + s0 * 128;
            read_tagged_fn<32>(v, [&](int i) { return b0 + (i & 7) * 128 + (i >> 3); },
                               m8 | (m8 << 8) | (m8 << 16) | (m8 << 24), tag, dead);
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                if (s < n) {
                    g0 = __fadd_rn(g0, __uint_as_float((uint32_t)v[s]));
                    u0 = __fadd_rn(u0, __uint_as_float((uint32_t)v[8 + s]));
                    g1 = __fadd_rn(g1, __uint_as_float((uint32_t)v[16 + s]));
                    u1 = __fadd_rn(u1, __uint_as_float((uint32_t)v[24 + s]));
                }
            }
        }
        g0 = round_bf(g0); u0 = round_bf(u0); g1 = round_bf(g1); u1 = round_bf(u1);
        const float a0 = shared_form ? __fmul_rn(round_bf(silu_f32(g0)), u0) : __fmul_rn(silu_f32(g0), u0);
        const float a1 = shared_form ? __fmul_rn(round_bf(silu_f32(g1)), u1) : __fmul_rn(silu_f32(g1), u1);
        xs2[w] = pack_bf2(a0, a1);
    }
}

// All M token rows into shared memory at entry (n16 16-byte words): four loads per thread in
// flight before their stores.
FNX_DEV void d2_stage_rows(const bf16* __restrict__ x, int n16, uint32_t* dst32) {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(dst32);
    for (int i0 = threadIdx.x; i0 < n16; i0 += 4 * D2_CTHREADS) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * D2_CTHREADS < n16) v[u] = __ldg(src + i0 + u * D2_CTHREADS);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * D2_CTHREADS < n16) dst[i0 + u * D2_CTHREADS] = v[u];
    }
}

// A token row (H bf16, H % 256 == 0) into shared memory: 16-byte loads, up to two per thread in
// flight before their stores (the loads may not pass a store through the generic pointer).
FNX_DEV void d2_stage_row(const bf16* __restrict__ x, int H, uint32_t* xs2) {
    const uint4* src = reinterpret_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(xs2);
    const int n = H / 8;
    for (int i = threadIdx.x; i < n; i += 2 * D2_CTHREADS) {
        const uint4 a = __ldg(src + i);
        const bool two = i + D2_CTHREADS < n;
        uint4 b = a;
        if (two) b = __ldg(src + i + D2_CTHREADS);
        dst[i] = a;
        if (two) dst[i + D2_CTHREADS] = b;
    }
}

// Router rows [e0, e0 + nr) from the stage: D2_CWARPS / nrow warps per row, each a slice of H;
// slice sums added in slice order.  x from shared memory (one token) or global memory.
FNX_DEV void d2_router(const StreamParams& p, const bf16* rows, int e0, int nr, int nrow, const bf16* x, uint32_t tag) {
    __shared__ float partial[D2_MAX_ROWS][D2_CWARPS][DEC_MAX_M];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpr = D2_CWARPS / nrow;
    const int row = warp / wpr, part = warp % wpr;
    const int seg = p.H / wpr;
    if (row < nr) {
        const bf16* wr = rows + (long long)row * p.H;
        for (int t0 = 0; t0 < p.M; t0 += 4) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int c = part * seg + lane * 8; c < (part + 1) * seg; c += 256) {
                const uint4 wv = *reinterpret_cast<const uint4*>(wr + c);
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    if (t0 + tt < p.M) {
                        const uint4 xv = *reinterpret_cast<const uint4*>(x + (long long)(t0 + tt) * p.H + c);
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
                    if (lane == 0) partial[row][part][t0 + tt] = v;
                }
            }
        }
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
    for (int i = threadIdx.x; i < nr * p.M; i += D2_CTHREADS) {
        const int rr = i / p.M, t = i % p.M;
        float s = partial[rr][0][t];
        for (int q = 1; q < wpr; ++q) s = __fadd_rn(s, partial[rr][q][t]);
        st_tag(p.tlog + (long long)t * p.R + e0 + rr, bf16_bits(f2bf(s)), tag);
    }
}

// out[t, 128m .. 128m+127]: the slot-order weighted reduce of the k routed rows and the
// sigmoid-gated shared row (kernels/reduce/reduce.cpp + kernels/post_ops/post_ops.cpp rounding).
// Thread w < 64 waits on and reads the column pair 128m + 2w, 2w + 1 of every row at once (its
// words of the k down items, the shared down item and the gate's router row): one L2 round trip
// after the last word lands, no separate poll.  The other warps go on to their next item.
FNX_DEV void d2_combine(const StreamParams& p, const DecodeRouting& R, int t, int m, uint32_t tag,
                        volatile int* dead) {
    const int hw = p.H / 2;
    const tword* yrow = p.tyd + (long long)t * p.k * hw + m * 64;
    const tword* gp = p.tlog + (long long)t * p.R + p.E;
    const tword* sp = p.tsh + (long long)t * hw + m * 64;
    const int w = threadIdx.x;
    if (w < 64) {
        // the gate logit, the shared row's word and the first 16 routed rows' words in one read
        tword v[18];
        const int n0 = min(16, p.k);
        const tword* yw = yrow + w;
        read_tagged_fn<18>(v, [&](int i) { return i == 0 ? gp : (i == 1 ? sp + w : yw + (long long)(i - 2) * hw); },
                           (1u << (2 + n0)) - 1u, tag, dead);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
            if (jj < n0) {
                const uint32_t y = (uint32_t)v[2 + jj];
                const float wf = R.wf[t * p.k + jj];
                a0 = __fadd_rn(a0, round_bf(__fmul_rn(bf_lo(y), wf)));
                a1 = __fadd_rn(a1, round_bf(__fmul_rn(bf_hi(y), wf)));
            }
        }
        for (int j0 = 16; j0 < p.k; j0 += 16) {
            tword yv[16];
            read_tagged<16>(yv, yrow + (long long)j0 * hw + w, hw, min(16, p.k - j0), tag, dead);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
                if (j0 + jj < p.k) {
                    const uint32_t y = (uint32_t)yv[jj];
                    const float wf = R.wf[t * p.k + j0 + jj];
                    a0 = __fadd_rn(a0, round_bf(__fmul_rn(bf_lo(y), wf)));
                    a1 = __fadd_rn(a1, round_bf(__fmul_rn(bf_hi(y), wf)));
                }
            }
        }
        a0 = round_bf(a0);
        a1 = round_bf(a1);
        const float g = __uint_as_float((uint32_t)v[0] << 16);
        const float sg = round_bf(sigmoid_f32(g));
        const uint32_t sh = (uint32_t)v[1];
        const uint32_t o = pack_bf2(__fadd_rn(a0, round_bf(__fmul_rn(bf_lo(sh), sg))),
                                    __fadd_rn(a1, round_bf(__fmul_rn(bf_hi(sh), sg))));
        *reinterpret_cast<uint32_t*>(p.out + (long long)t * p.H + 2 * (m * 64 + w)) = o;
    }
}

// One stage of a tile run on the tensor cores (mma m16n8k16): warp w computes tile rows
// 16w .. 16w+15 against the item's token (B column 0; the other seven columns are zero).  The A
// fragments are the exactly rounded dequantised weights bf16(q * s) (tile_pair: the reference's
// dequantisation, as in the GEMM's producers), so only the fp32 summation order differs from
// the CUDA-core loop.  Fragment k-slots follow the word order: thread t of a fragment group takes
// words t and t+4 of its two rows, pair u in MMA u, and B takes the same slots of x; the tile-block
// swizzle makes the four word loads conflict-free.  d[0] / d[2]: tile rows 16w + g and
// 16w + g + 8 for the token (in the lanes with t == 0).
FNX_DEV void d2_mma_stage(const uint32_t* __restrict__ wbuf, int n, int kb_first, const uint32_t* xs2, float (&d)[4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int r0 = 16 * warp + g, r1 = r0 + 8;
    const int o00 = tile_word(t, r0), o01 = tile_word(t + 4, r0);
    const int o10 = tile_word(t, r1), o11 = tile_word(t + 4, r1);
    const uint4* xs4 = reinterpret_cast<const uint4*>(xs2);
    for (int j = 0; j < n; ++j) {
        const uint32_t* blk = wbuf + j * TILE_BLOCK_WORDS;
        const uint32_t wa0 = blk[o00], wa1 = blk[o01], wb0 = blk[o10], wb1 = blk[o11];
        const unsigned short* sc = reinterpret_cast<const unsigned short*>(blk + 1024);
        const uint32_t sa = sc[r0], sb = sc[r1];
        const uint32_t s2a = sa | (sa << 16), s2b = sb | (sb << 16);
        const int kb = kb_first + j;
        uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
        if (g == 0) {
            xa = xs4[kb * 8 + t];
            xb = xs4[kb * 8 + 4 + t];
        }
        mma_16816_bf16(d, tile_pair(wa0, 0, s2a), tile_pair(wb0, 0, s2b), tile_pair(wa1, 0, s2a),
                       tile_pair(wb1, 0, s2b), xa.x, xb.x);
        mma_16816_bf16(d, tile_pair(wa0, 1, s2a), tile_pair(wb0, 1, s2b), tile_pair(wa1, 1, s2a),
                       tile_pair(wb1, 1, s2b), xa.y, xb.y);
        mma_16816_bf16(d, tile_pair(wa0, 2, s2a), tile_pair(wb0, 2, s2b), tile_pair(wa1, 2, s2a),
                       tile_pair(wb1, 2, s2b), xa.z, xb.z);
        mma_16816_bf16(d, tile_pair(wa0, 3, s2a), tile_pair(wb0, 3, s2b), tile_pair(wa1, 3, s2a),
                       tile_pair(wb1, 3, s2b), xa.w, xb.w);
    }
}

__global__ void __launch_bounds__(D2_THREADS, 2) decode_stream_kernel(const StreamParams p) {
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ __align__(16) uint32_t xs2[DEC_MAX_K / 2];
    __shared__ float red[128];
    __shared__ uint64_t full[D2_NS], empty[D2_NS], routing_bar;
    __shared__ DecodeRouting R;
    __shared__ TopkScratch RS[D2_CWARPS];
    __shared__ int s_dead;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const D2Shape S = d2_shape(p);
    const int first_routed = S.RB + S.nsh;
    if (tid == 0) {
        for (int s = 0; s < D2_NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], D2_CWARPS);
        }
        mbar_init(&routing_bar, 1);
        s_dead = 0;
        fence_mbar_init();
        // a decode launched behind this one (programmatic dependent launch) may start as this
        // grid's blocks leave: its copy warps prefetch weights into L2, then everything waits
        pdl_launch_dependents();
    }
    __syncthreads();
    volatile int* dead = &s_dead;

    if (warp == D2_COPY_WARP) {
        // ------------------------------------------------ copy warp: every stage of every item, in order
        if (lane == 0) {
            // Until the kernel before this one on the stream is complete (programmatic dependent
            // launch), its writes may not be visible: that kernel may have written the weights
            // (a repack, an expert renumbering).  So before the wait only the first stages' weights
            // are prefetched into L2, which is coherent (lines still being written are read again
            // by the copies after the wait).
            int pre = 0;
            for (int it = blockIdx.x; it < first_routed && pre < D2_NS; it += gridDim.x) {
                const D2Item d = d2_item(p, S, R, it);          // router / shared items: no routing read
                const int ns = (d.type == D2_ROUTER && p.logits_ready) ? 0 : d2_stages(d);
                for (int s2 = 0; s2 < ns && pre < D2_NS; ++s2, ++pre) {
                    if (d.type == D2_ROUTER) {
                        l2_prefetch(d.src, (uint32_t)(d.kb1 - d.kb0) * p.H * 2);
                    } else {
                        const int kb = d.kb0 + s2 * D2_SK;
                        l2_prefetch(d.src + (long long)kb * TILE_BLOCK_WORDS,
                                    (uint32_t)min(D2_SK, d.kb1 - kb) * TILE_BLOCK_BYTES);
                    }
                }
            }
            pdl_wait();
            const uint64_t once = l2_evict_first();
            bool routed = false;
            int j = 0, prev_type = D2_ROUTER;
            for (int it = blockIdx.x; it < S.total; it += gridDim.x) {
                if (it >= first_routed && !routed) {
                    mbar_wait(&routing_bar, 0);
                    routed = true;
                }
                const D2Item d = d2_item(p, S, R, it);
                const int ns = (d.type == D2_ROUTER && p.logits_ready) ? 0 : d2_stages(d);
#ifndef FNX_D2_EAGER_DOWN
                // a down item's weights are requested once the earlier gate/up stages of this CTA
                // are consumed: the gate/up bytes, which the critical path waits for, get the HBM
                // first, and the down bytes still land before the activation they multiply
                if (ns && j > 0 && (d.type == D2_DN || d.type == D2_SHDN) && prev_type != D2_DN &&
                    prev_type != D2_SHDN)
                    mbar_wait(&empty[(j - 1) % D2_NS], ((j - 1) / D2_NS) & 1);
#endif
                if (ns) prev_type = d.type;
                for (int s = 0; s < ns; ++s, ++j) {
                    const int slot = j % D2_NS;
                    mbar_wait(&empty[slot], ((j / D2_NS) & 1) ^ 1);
                    uint32_t bytes;
                    const void* src;
                    if (d.type == D2_ROUTER) {
                        bytes = (uint32_t)(d.kb1 - d.kb0) * p.H * 2;
                        src = d.src;
                    } else {
                        const int kb = d.kb0 + s * D2_SK;
                        bytes = (uint32_t)min(D2_SK, d.kb1 - kb) * TILE_BLOCK_BYTES;
                        src = d.src + (long long)kb * TILE_BLOCK_WORDS;
                    }
                    mbar_arrive_expect_tx(&full[slot], bytes);
                    bulk_load(smem_u32(ring + slot * D2_STAGE_BYTES), src, bytes, &full[slot], once);
                }
            }
        }
        return;
    }

    // ---------------------------------------------------- compute warps
    // The input rows, the workspace (launch counter, tags) and the logits of a logits-ready launch
    // may come from the kernel before this one on the stream, which may still be running when this
    // grid starts (programmatic dependent launch): wait for it here.
    pdl_wait();
    const uint32_t tag = *p.epoch + 1u;          // this launch's tag (the counter is bumped at the end)
    if (tid == 0 && p.logits_ready) {
        // the logits were written by the kernel before this one on the stream, so they carry
        // this launch's tag already; a stale tag means no fnx_hc_mix_router ran on this
        // workspace since the last decode: record it and end at once instead of by timeouts
        for (int t = 0; t < p.M; ++t) {
            const tword* row = p.tlog + (long long)t * p.R;
            if ((uint32_t)(ld_tag(row) >> 32) != tag || (uint32_t)(ld_tag(row + p.R - 1) >> 32) != tag) {
                fnx_flag_error(FNX_DEVERR_NOLOGITS);
                s_dead = 1;
                break;
            }
        }
    }
    named_bar_sync(D2_BAR, D2_CTHREADS);
    // the token rows stay in shared memory for the whole launch when they fit (router and gate/up
    // items then stage nothing); loaded while the copy warp's first stages are in flight
    uint32_t* xres = reinterpret_cast<uint32_t*>(ring + D2_RING_BYTES);
    const bool resident = p.M * p.H * 2 <= D2_XRES_BYTES;
    if (resident) {
        d2_stage_rows(p.x, p.M * p.H / 8, xres);
        named_bar_sync(D2_BAR, D2_CTHREADS);
    }
    int j = 0;
    bool have_routing = false;
    for (int it = blockIdx.x; it < S.total; it += gridDim.x) {
        if (it >= first_routed && !have_routing) {
            // route the tokens this CTA's items touch, as their logits arrive
            unsigned mask = 0;
            for (int i2 = it; i2 < S.total; i2 += gridDim.x) mask |= 1u << d2_item_pos(p, S, i2).t;
            if (p.M == 1) {
                d2_route_block(p, R, 0, tag, dead);
            } else {
                int n = 0;
                for (int t = 0; t < p.M; ++t)
                    if ((mask >> t) & 1u) {
                        if (n % D2_CWARPS == warp) d2_route_warp(p, R, t, tag, dead, RS[warp]);
                        ++n;
                    }
                named_bar_sync(D2_BAR, D2_CTHREADS);
            }
            if (tid == 0) mbar_arrive(&routing_bar);
            have_routing = true;
        }
        const D2Item d = d2_item(p, S, R, it);
        if (d.type == D2_ROUTER && p.logits_ready) continue;
        if (d.type == D2_COMB) {
            d2_combine(p, R, d.t, d.m, tag, dead);
            continue;
        }
        // ---- the item's input row into shared memory
        const uint32_t* xrow = xs2;
        if (d.type == D2_ROUTER) {
            if (p.M == 1 && !resident) d2_stage_row(p.x, p.H, xs2);
        } else if (d.type == D2_SHGU || d.type == D2_GU) {
            if (resident) xrow = xres + (long long)d.t * (p.H / 2);
            else d2_stage_row(p.x + (long long)d.t * p.H, p.H, xs2);
        } else if (d.type == D2_SHDN) {
            d2_build_act(p.tpart + (long long)d.t * S.MT * p.ks1 * 128, S.MT, p.ks1, p.I, true, tag, dead, xs2);
        } else {
            d2_build_act(p.tpart2 + (long long)d.row * S.MT * p.ks2 * 128, S.MT, p.ks2, p.I, false, tag, dead, xs2);
        }
        named_bar_sync(D2_BAR, D2_CTHREADS);

        if (d.type == D2_ROUTER) {
            const int slot = j % D2_NS;
            mbar_wait(&full[slot], (j / D2_NS) & 1);
            d2_router(p, reinterpret_cast<const bf16*>(ring + slot * D2_STAGE_BYTES), d.kb0, d.kb1 - d.kb0, S.nrow,
                      resident ? reinterpret_cast<const bf16*>(xres)
                               : (p.M == 1 ? reinterpret_cast<const bf16*>(xs2) : p.x), tag);
            // every warp is past its reads of the stage (d2_router's barrier)
            if (lane == 0) mbar_arrive(&empty[slot]);
            ++j;
            named_bar_sync(D2_BAR, D2_CTHREADS);     // xs2 and the router partials are reused next
            continue;
        }

        // ---- the tile run, stage by stage, on the tensor cores
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int ns = d2_stages(d);
        for (int s = 0; s < ns; ++s, ++j) {
            const int slot = j % D2_NS;
            mbar_wait(&full[slot], (j / D2_NS) & 1);
            const int kb = d.kb0 + s * D2_SK;
            d2_mma_stage(reinterpret_cast<const uint32_t*>(ring + slot * D2_STAGE_BYTES), min(D2_SK, d.kb1 - kb), kb,
                         xrow, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if ((lane & 3) == 0) {
            red[16 * warp + (lane >> 2)] = acc[0];
            red[16 * warp + (lane >> 2) + 8] = acc[2];
        }
        // every warp is past its last read of xs2, and red is complete
        named_bar_sync(D2_BAR, D2_CTHREADS);
        if (d.type == D2_SHGU) {
            if (tid < 128)
                st_tag(p.tpart + (((long long)d.t * S.MT + d.m) * p.ks1 + d.ks) * 128 + tid, __float_as_uint(red[tid]),
                       tag);
        } else if (d.type == D2_GU) {
            if (tid < 128)
                st_tag(p.tpart2 + (((long long)d.row * S.MT + d.m) * p.ks2 + d.ks) * 128 + tid,
                       __float_as_uint(red[tid]), tag);
        } else if (tid < 64) {
            const uint32_t v = pack_bf2(red[2 * tid], red[2 * tid + 1]);
            if (d.type == D2_SHDN) st_tag(p.tsh + (long long)d.t * (p.H / 2) + d.m * 64 + tid, v, tag);
            else st_tag(p.tyd + (long long)d.row * (p.H / 2) + d.m * 64 + tid, v, tag);
        }
        // red is rewritten only after the next item's staging barrier
    }

    // ---- the last CTA to leave bumps the launch counter (every CTA read it at entry)
    named_bar_sync(D2_BAR, D2_CTHREADS);
    if (tid == 0) {
        const unsigned tk = atomicAdd(p.exit, 1u);
        if (tk == gridDim.x - 1) {
            *p.epoch = tag;
            *p.exit = 0;
        }
    }
}

// The hyper-connection branch mix that produces the decode layer's input (fnx/engine.py:838-845;
// hc_mix_one, the arithmetic of hc_sigmoid_reduce_kernel) with the router GEMV fused behind it.
// Blocks run in clusters of HC_MIX_CLUSTER: block r of a cluster mixes slice r of the M*H outputs
// into its shared memory (the first cluster also stores it, y), the slices are exchanged over
// distributed shared memory, and every block then computes the logits of router rows
// [b*nrow, b*nrow + nrow) from the full mixed rows with d2_router's arithmetic, writing them into
// the decode workspace tagged for the next decode launch on it.  That launch (logits_ready) then
// leaves its router items empty, and routes exactly as if they had produced these logits.  The
// block's router rows are bulk-loaded into shared memory at entry, under the mix.
// x (hn), l bf16 [M, HC*H]; router bf16 [R, H]; dynamic shared memory (M + nrow)*H*2 bytes; the
// grid is a multiple of HC_MIX_CLUSTER (blocks past the last router row only mix).
constexpr int HC_MIX_CLUSTER = 8;

FNX_DEV uint4 ld_shared_cluster_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

__global__ void __cluster_dims__(HC_MIX_CLUSTER, 1, 1) __launch_bounds__(D2_CTHREADS)
    hc_mix_router_kernel(const bf16* __restrict__ x, const bf16* __restrict__ l, int HC, bf16* __restrict__ y,
                         const StreamParams p) {
    extern __shared__ __align__(16) uint8_t mix_raw[];
    __shared__ uint64_t rows_full;
    bf16* xs = reinterpret_cast<bf16*>(mix_raw);            // [M][H]
    const int H = p.H;
    const uint32_t tag = *p.epoch + 1u;                       // the next decode launch's tag
    const int n = p.M * H;                                    // a multiple of 256 (H is)
    bf16* rows = xs + n;                                      // [nrow][H] this block's router rows
    const int nrow = d2_router_rows(H);
    const int e0 = blockIdx.x * nrow;
    const int nr = max(0, min(nrow, p.R - e0));
    if (threadIdx.x == 0 && nr > 0) {
        mbar_init(&rows_full, 1);
        fence_mbar_init();
        const uint32_t bytes = (uint32_t)nr * H * 2;
        mbar_arrive_expect_tx(&rows_full, bytes);
        bulk_load(smem_u32(rows), p.router + (long long)e0 * H, bytes, &rows_full, l2_evict_first());
    }
    const int per = n / HC_MIX_CLUSTER;                       // slice length, a multiple of 32
    const int rank = (int)cluster_rank();
    const bool store = blockIdx.x < HC_MIX_CLUSTER;
    for (int i = rank * per + threadIdx.x; i < (rank + 1) * per; i += D2_CTHREADS) {
        const int t = i / H;
        const bf16 v = hc_mix_one(x, l, t, i - t * H, H, HC);
        xs[i] = v;
        if (store) y[i] = v;
    }
    cluster_sync_all();                                       // every slice is in its block's shared memory
    const int per16 = per / 8;                                // 16-byte words per slice
    for (int r = 1; r < HC_MIX_CLUSTER; ++r) {
        const int src = (rank + r) % HC_MIX_CLUSTER;
        uint4* dst = reinterpret_cast<uint4*>(xs) + src * per16;
        const uint32_t rem = mapa_rank(dst, (uint32_t)src);
        for (int j = threadIdx.x; j < per16; j += D2_CTHREADS) dst[j] = ld_shared_cluster_v4(rem + 16u * j);
    }
    cluster_sync_all();                                       // peers keep their shared memory until read
    if (nr > 0) {
        if (!mbar_wait(&rows_full, 0)) mbar_wait(&rows_full, 0);   // (the copy must land before exit)
        d2_router(p, rows, e0, nr, nrow, xs, tag);
    }
}

}  // namespace fnx
