// Expert-major grouped GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   out[row_begin(e) + n, f] = epilogue( sum_k W_e[k, f] * X[src(row_begin(e) + n), k] )
//
// for every expert e with rows [ends[e-1], ends[e]).  This is the restated
// npu_grouped_matmul(group_type=0) of fnx/engine.py:749-753 (prefill gate/up and down)
// and, with one group, npu_weight_quant_batchmatmul (dense W8A16, router, shared expert).
//
// Orientation ("swap-AB"): the weight features are the UMMA M dimension (128 rows of A)
// and the expert's token rows are N (16..128 in steps of 16), so an expert with ~80
// tokens pads to 80, not to 128.  D[f, n] accumulates in TMEM (fp32, lane = feature,
// column = token), double-buffered so the epilogue of one tile overlaps the next.
// W4: the dequantised A stages live in TMEM too (columns 256..511, tcgen05.st from the
// producers, read by the MMA as its A operand), so shared memory carries only the
// token tiles and the raw int4 blocks.
//
// Warp roles (608 threads):
//   warps 0,16-18 B loaders: gather token rows with cp.async into K-major SW128 tiles; a
//                 stage is full when every lane's copies have landed (cp.async.mbarrier.arrive)
//   warp 1        TMEM allocator + MMA issuer.  It touches no shared memory while MMAs are
//                 in flight (a shared-memory access there waits for the queued MMAs and
//                 halves the issue rate): stages are handed to it by warp 3 through named
//                 barriers, tile sizes come from registers filled once per 256 tiles.
//   warp 2        copy producer: W4 -> tile blocks (4 KB of int4 + their scales) in bulk
//                 copies of four k-blocks; BF16 -> the A tiles by TMA (128-byte swizzle)
//   warp 3        waiter: waits on the stage mbarriers and releases the MMA warp
//   warps 4-7     epilogue warpgroup: tcgen05.ld -> bf16 / SwiGLU -> global
//   warps 8-15    A producers (W4/W8), two groups of four warps taking alternate k-blocks:
//                 int4 / int8 -> bf16(q * s) (exactly rounded) -> TMEM (W4) / SW128 smem (W8)
// Every mbarrier wait is bounded (fnx_common.cuh); a timeout sets an abort flag and the
// roles unwind to the final barrier, where the allocating warp frees TMEM.  The waiter and
// the MMA warp always run their full, identical stage count (the waiter stops waiting
// after an abort but keeps handing over), so the named barriers between them never
// strand a warp.
#pragma once
#include "fnx_common.cuh"
#include "kernels_repack.cuh"

namespace fnx {

enum GemmMode { GEMM_W4 = 0, GEMM_W8 = 1, GEMM_BF16 = 2 };
// EPI_SWIGLU_MIXED: the fp32 SwiGLU for the routed experts and the shared expert's bf16 form
// for expert p.shared_e (the shared expert run as one expert of the same grouped launch).
enum GemmEpi { EPI_PLAIN = 0, EPI_SWIGLU_F32 = 1, EPI_SWIGLU_BF16 = 2, EPI_SWIGLU_MIXED = 3 };

constexpr int G_BM = 128;          // weight features per tile (UMMA M)
constexpr int G_BK = 64;           // k per stage (one 128-byte swizzle row of bf16)
constexpr int G_BN = 128;          // max token rows per tile
constexpr int G_MAX_STAGES = 10;
// Raw int4 ring: G_R_OPS slots of G_OPK tile blocks.  One bulk copy fills a slot with up to
// G_OPK consecutive k-blocks of a tile (17 KB): a bulk copy costs the copy engine a few
// hundred cycles however small it is, so 4 KB copies cap the stream near 4.5 TB/s.
constexpr int G_OPK = 4;
constexpr int G_R_OPS = 4;
constexpr int G_MAX_R_OPS = 8;
constexpr int G_THREADS = 608;    // 19 warps
constexpr int G_LOADERS = 4;       // B loader warps: 0, 16, 17, 18
constexpr int G_BAR_FULL = 1;      // named barrier: waiter -> MMA warp, "stage j is full"
constexpr int G_BAR_TAKEN = 2;     // named barrier: MMA warp -> waiter, "stage j was issued"
constexpr int G_A_BYTES = G_BM * G_BK * 2;     // 16 KB
constexpr int G_B_BYTES = G_BN * G_BK * 2;     // 16 KB
constexpr int G_RAW_W = 8 * 128 * 4;           // 4 KB: the words [8 chunks][128 rows] of a tile block
constexpr int G_RAW_BYTES = TILE_BLOCK_BYTES;  // + the rows' scales for the block's k group
constexpr int G_MAX_E = 1024;

template <int MODE>
struct GemmCfg {
    static constexpr bool A_TMEM = MODE == 0;                 // GEMM_W4: A stages in tensor memory
    static constexpr int STAGES = A_TMEM ? 8 : 6;
    static constexpr int R_SLOTS = MODE == 0 ? G_R_OPS * G_OPK : 0;   // raw tile blocks in the ring
    static constexpr uint32_t TMEM_COLS = A_TMEM ? 512 : 256;
    static constexpr uint32_t A_COL0 = 2 * G_BN;              // A stages follow the two accumulators
    static_assert(STAGES <= G_MAX_STAGES && (!A_TMEM || A_COL0 + STAGES * 32 <= TMEM_COLS), "tmem budget");
};

struct GemmParams {
    CUtensorMap tmap_a;         // BF16: bf16 weights [E*Nw, K], box {64, 128}, 128-byte swizzle
    const bf16* act;            // token rows bf16 [act_rows, K], row stride ld_act elements
    long long ld_act;
    long long act_rows;         // gathered row indices outside [0, act_rows) read zeros (and are flagged)
    const int64_t* row_index;   // null: row r of the problem reads act row r; else row_index[r] / index_div
    int index_div;
    const void* w;              // W4: tile blocks int32 [E, MT, K/64, TILE_BLOCK_WORDS] with their
                                // scales inline (kernels_repack.cuh); W8: int8 [E, K, Nw]; BF16: bf16 [E, Nw, K]
    const bf16* scales;         // W8: bf16 [E, K/gs, Nw] (unused otherwise)
    const int64_t* ends;        // [E] cumulative row counts; null: one group of M rows
    bf16* out;                  // bf16 [M, ld_out]
    long long ld_out;
    int E, M, K, Nw, gs;
    int m_tiles;                // tiles along the feature dimension
    int shared_e;               // EPI_SWIGLU_MIXED: the shared expert's index
    bf16* const* out_rows;      // EPI_PLAIN: row r goes to out_rows[r] (e.g. a peer's buffer); null: out
    // split-K (GEMM_W8, EPI_PLAIN): ksplit > 1 cuts K into ksplit equal ranges, each a tile of
    // its own; the epilogue writes fp32 partials [ksplit][M][Nw] to `partial` and a separate
    // pass sums them in split order (deterministic).  0 or 1: no split.
    int ksplit;
    float* partial;
    // W4: group e multiplies the tile blocks of expert expert_ids[e] of the E_w experts in `w`
    // (null: expert e), so a selection of experts is read in place instead of being copied out
    const int64_t* expert_ids;
    int E_w;
    // CTA-pair W4 kernel without a row index: the token rows of a tile are contiguous, so one thread
    // loads them by TMA (act [act_rows, K], boxes of 32 and 8 rows x 64 k, 128-byte swizzle) in
    // place of the gathering loader warps
    int b_tma;
    CUtensorMap tmap_b32, tmap_b8;
    // at most this many CTAs (0: as many as fit), leaving SMs to kernels of another stream
    int max_ctas;
};

// The expert whose tile blocks group e reads (an id outside [0, E_w) is flagged, and read as 0).
FNX_DEV long long weight_expert(const GemmParams& p, int e) {
    if (!p.expert_ids) return e;
    const long long w = p.expert_ids[e];
    if (w < 0 || w >= p.E_w) {
        fnx_flag_error(FNX_DEVERR_BADID);
        return 0;
    }
    return w;
}

FNX_DEV int gemm_ksplit(const GemmParams& p) { return p.ksplit > 1 ? p.ksplit : 1; }

// destination of output row `row` (a 16-byte aligned row of Nw bf16 when out_rows is set)
FNX_DEV bf16* out_row(const GemmParams& p, long long row) {
    return p.out_rows ? p.out_rows[row] : p.out + row * p.ld_out;
}

struct GemmSmem {
    uint64_t a_full[G_MAX_STAGES], b_full[G_MAX_STAGES], empty[G_MAX_STAGES];
    uint64_t raw_full[G_MAX_R_OPS], raw_empty[G_MAX_R_OPS];
    uint64_t peer_full[G_MAX_STAGES];   // CTA-pair kernel: the peer's stage is full (on rank 0)
    uint64_t b_empty[G_MAX_STAGES];     // CTA-pair kernel: token stage free (its own, deeper ring)
    uint64_t acc_full[2], acc_empty[2], final_bar;
    uint32_t tmem_base;
    volatile int abort;
    int total_tiles;
    int tile_start[G_MAX_E + 1];
};

struct TileInfo {
    int e, m, row0, nrows;
    int ks;            // split-K range of the single-CTA kernel (0 without a split)
};

FNX_DEV bool decode_tile(const GemmSmem& S, const GemmParams& p, int tile, TileInfo& ti) {
    if (tile >= S.total_tiles) return false;
    int lo = 0, hi = p.E;              // largest e with tile_start[e] <= tile
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (S.tile_start[mid] <= tile) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int ksplit = gemm_ksplit(p);
    const int local = tile - S.tile_start[e];
    ti.ks = local % ksplit;                        // the K ranges of one output tile are adjacent
    const int l2 = local / ksplit;
    const int chunk = l2 / p.m_tiles;
    ti.e = e;
    ti.m = l2 % p.m_tiles;
    const long long begin = min((long long)p.M, (long long)(p.ends ? (e ? p.ends[e - 1] : 0) : 0));
    const long long end = min((long long)p.M, (long long)(p.ends ? p.ends[e] : p.M));
    ti.row0 = (int)begin + chunk * G_BN;
    ti.nrows = (int)min((long long)G_BN, end - ti.row0);
    return true;
}

// First weight feature of half h (64 features) in feature tile m.
template <int EPI>
FNX_DEV int half_feature(int h, int m, int Nw) {
    return EPI == EPI_PLAIN ? m * G_BM + h * 64 : (h ? Nw / 2 : 0) + m * 64;
}
// A row holding the feature (half h, word j, nibble pf) of the tile, i.e. feature
// half_feature(h) + 8j + pf.  Rows are ordered nibble-major (8pf + j) so that a warp's
// 16-byte stores of one nibble position fall into eight different swizzle chunks
// (conflict-free); SwiGLU keeps a feature's gate and up on adjacent rows.
template <int EPI>
FNX_DEV int a_row(int h, int j, int pf) {
    const int q = 8 * pf + j;
    return EPI == EPI_PLAIN ? h * 64 + q : 2 * q + h;
}
// Inverse of a_row for the epilogue: the feature offset (within the tile for PLAIN,
// within the half for SwiGLU) held by accumulator lane r.
template <int EPI>
FNX_DEV int lane_feature(int r) {
    if (EPI == EPI_PLAIN) {
        const int q = r & 63;
        return (r & 64) + 8 * (q & 7) + (q >> 3);
    }
    const int q = r >> 1;
    return 8 * (q & 7) + (q >> 3);
}

// ------------------------------------------------------------------ A producers
// W4: thread r of a 128-thread group dequantises tile row r of the stage: eight words
// (8 consecutive k each) from the tile-major block the TMA warp copied, scaled by the
// row's group scale, into 32 registers = the row's 64 bf16 as tensor-memory columns
// (column 4c + i holds k = 8c + 2i in its low half, 8c + 2i + 1 in its high half).
// The reads are consecutive words across the warp: conflict-free.
FNX_DEV void produce_a_w4(const uint8_t* raw, int r, uint32_t (&a)[32]) {
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(raw);
    const uint32_t s16 = reinterpret_cast<const uint16_t*>(raw + G_RAW_W)[r];
    const uint32_t s2 = s16 | (s16 << 16);
    uint32_t wv[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) wv[c] = rw[tile_word(c, r)];
#pragma unroll
    for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) a[4 * c + i] = tile_pair(wv[c], i, s2);
}

// produce_a_w4 straight into tensor memory in two halves of 16 columns (words 0-3, then 4-7):
// half the registers live at once, so the 32 independent conversion chains of a row interleave
// instead of queueing behind a 32-register fragment.
FNX_DEV void produce_store_w4(const uint8_t* raw, int r, uint32_t taddr) {
    const uint32_t* rw = reinterpret_cast<const uint32_t*>(raw);
    const uint32_t s16 = reinterpret_cast<const uint16_t*>(raw + G_RAW_W)[r];
    const uint32_t s2 = s16 | (s16 << 16);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t wv[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) wv[c] = rw[tile_word(4 * half + c, r)];
        uint32_t a[16];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) a[4 * c + i] = tile_pair(wv[c], i, s2);
        tmem_st16(taddr + 16 * half, a);
    }
}

// W8: same block shape, int8 weights read directly (L2-resident dense projections).
template <int EPI>
FNX_DEV void produce_a_w8(const GemmParams& p, const TileInfo& ti, int kb, uint8_t* a_tile, int t) {
    const int j = t & 7, kq = (t >> 3) & 7, h = t >> 6;
    const int fbase = half_feature<EPI>(h, ti.m, p.Nw) + j * 8;
    const int k0 = kb * G_BK + kq * 8;
    const int8_t* wp = reinterpret_cast<const int8_t*>(p.w) + ((long long)ti.e * p.K + k0) * p.Nw + fbase;
    uint2 wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wv[i] = __ldg(reinterpret_cast<const uint2*>(wp + (long long)i * p.Nw));
    const int G = p.K / p.gs;
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(p.scales + ((long long)ti.e * G + k0 / p.gs) * p.Nw + fbase));
    const uint32_t sarr[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int pf = 0; pf < 8; ++pf) {
        const float s = (pf & 1) ? bf_hi(sarr[pf >> 1]) : bf_lo(sarr[pf >> 1]);
        uint32_t outv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w0 = pf < 4 ? wv[2 * i].x : wv[2 * i].y;
            const uint32_t w1 = pf < 4 ? wv[2 * i + 1].x : wv[2 * i + 1].y;
            const int sh = (pf & 3) * 8;
            const float q0 = (float)(int8_t)((w0 >> sh) & 0xffu);
            const float q1 = (float)(int8_t)((w1 >> sh) & 0xffu);
            outv[i] = pack_bf2(__fmul_rn(q0, s), __fmul_rn(q1, s));
        }
        const int r = a_row<EPI>(h, j, pf);
        *reinterpret_cast<uint4*>(a_tile + sw128_offset(r, kq)) = make_uint4(outv[0], outv[1], outv[2], outv[3]);
    }
}

// ------------------------------------------------------------------ epilogue
// PERM: A rows follow a_row() (the W8 producers); otherwise rows are in tile order:
// feature 128m + r, or for SwiGLU gate / up of feature 64m + r/2 on even / odd rows.
template <int EPI, bool PERM>
FNX_DEV void epilogue_chunk(const GemmParams& p, const TileInfo& ti, int r, int n0, const uint32_t (&v)[16]) {
    const int lane = threadIdx.x & 31;
    if (EPI == EPI_PLAIN) {
        const int f = ti.m * G_BM + (PERM ? lane_feature<EPI>(r) : r);
        if (f >= p.Nw) return;                    // the last tile of a width that is not a multiple of 128
        const int lim = ti.nrows - n0;
        if (p.out_rows) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < lim) out_row(p, ti.row0 + n0 + i)[f] = f2bf(__uint_as_float(v[i]));
        } else {
            bf16* o = p.out + (long long)(ti.row0 + n0) * p.ld_out + f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < lim) o[(long long)i * p.ld_out] = f2bf(__uint_as_float(v[i]));
        }
    } else {
        // lane pairs (2i, 2i+1) hold gate / up of feature m*64 + r/2 for 16 tokens;
        // the even lane finishes tokens 0..7, the odd lane tokens 8..15.
        const bool odd = lane & 1;
        float g[8], u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a0 = round_bf(__uint_as_float(v[i]));          // my value, token i
            const float a1 = round_bf(__uint_as_float(v[8 + i]));      // my value, token 8+i
            // send the half the partner finishes, receive the half I finish
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? a0 : a1, 1);
            const float mine = odd ? a1 : a0;
            g[i] = odd ? recv : mine;
            u[i] = odd ? mine : recv;
        }
        const int f = ti.m * 64 + (PERM ? lane_feature<EPI>(r) : (r >> 1));
        const int nb = n0 + (odd ? 8 : 0);
        bf16* o = p.out + (long long)(ti.row0 + nb) * p.ld_out + f;
        const int lim = ti.nrows - nb;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float a;
            if (EPI == EPI_SWIGLU_F32 || (EPI == EPI_SWIGLU_MIXED && ti.e != p.shared_e)) a = __fmul_rn(silu_f32(g[i]), u[i]);
            else a = __fmul_rn(round_bf(silu_f32(g[i])), u[i]);
            if (i < lim) o[(long long)i * p.ld_out] = f2bf(a);
        }
    }
}

// Split-K epilogue (EPI_PLAIN): this K range's fp32 sums for 16 tokens of accumulator lane r,
// into partial[ks][row][feature] (summed in split order by splitk_reduce_kernel).
template <bool PERM>
FNX_DEV void epilogue_partial(const GemmParams& p, const TileInfo& ti, int r, int n0, const uint32_t (&v)[16]) {
    const int f = ti.m * G_BM + (PERM ? lane_feature<EPI_PLAIN>(r) : r);
    const int lim = ti.nrows - n0;
    float* o = p.partial + ((long long)ti.ks * p.M + ti.row0 + n0) * p.Nw + f;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        if (i < lim) o[(long long)i * p.Nw] = __uint_as_float(v[i]);
}

// y[row, f] = bf16(sum over s = 0..ksplit-1 of partial[s][row][f]) in that order; 4 features per
// thread (Nw % 4 == 0), ksplit <= KMAX.  Every partial of a thread is requested before the first
// is added, so the loads overlap instead of forming a chain; KMAX (2, 4, 8, 16: the smallest that
// holds ksplit) keeps the registers to what the split needs.
constexpr int SPLITK_MAX = 16;
template <int KMAX>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partial, bf16* __restrict__ out,
                                                            long long ld_out, int M, int Nw, int ksplit) {
    const long long n4 = (long long)M * (Nw / 4);
    const long long plane = (long long)M * Nw;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / (Nw / 4);
        const int c = (int)(i - row * (Nw / 4)) * 4;
        float4 b[KMAX];
#pragma unroll
        for (int s = 0; s < KMAX; ++s)
            if (s < ksplit) b[s] = __ldcs(reinterpret_cast<const float4*>(partial + s * plane + row * Nw + c));
        float4 a = b[0];
#pragma unroll
        for (int s = 1; s < KMAX; ++s) {
            if (s >= ksplit) break;
            a.x = __fadd_rn(a.x, b[s].x); a.y = __fadd_rn(a.y, b[s].y); a.z = __fadd_rn(a.z, b[s].z);
            a.w = __fadd_rn(a.w, b[s].w);
        }
        const uint2 o = make_uint2(pack_bf2(a.x, a.y), pack_bf2(a.z, a.w));
        *reinterpret_cast<uint2*>(out + row * ld_out + c) = o;
    }
}

// Staged form for tile-ordered rows (the W4 kernels): the warp's 32 accumulator lanes x 16
// tokens go through a 1 KB shared buffer so that global stores are 16-byte vectors along
// the feature dimension (one token row segment per 4 or 2 lanes) instead of 2-byte
// stores strided by the output row.  Needs ld_out % 8 == 0 and a 16-byte aligned out.
template <int EPI>
FNX_DEV void epilogue_chunk_staged(const GemmParams& p, const TileInfo& ti, int w4, int n0, const uint32_t (&v)[16],
                                   uint16_t* stage) {
    const int lane = threadIdx.x & 31;
    if (EPI == EPI_PLAIN) {
        // destinations first: with per-row pointers their loads overlap the staging below
        bf16* dst[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int tok = (q * 32 + lane) >> 2;
            dst[q] = n0 + tok < ti.nrows ? out_row(p, ti.row0 + n0 + tok) : nullptr;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) stage[i * 32 + lane] = (uint16_t)bf16_bits(f2bf(__uint_as_float(v[i])));
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int c = q * 32 + lane, tok = c >> 2, part = c & 3;
            if (dst[q]) {
                const uint4 val = *reinterpret_cast<const uint4*>(stage + tok * 32 + part * 8);
                *reinterpret_cast<uint4*>(dst[q] + ti.m * G_BM + w4 * 32 + part * 8) = val;
            }
        }
    } else {
        const bool odd = lane & 1;
        float g[8], u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float a0 = round_bf(__uint_as_float(v[i]));
            const float a1 = round_bf(__uint_as_float(v[8 + i]));
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? a0 : a1, 1);
            const float mine = odd ? a1 : a0;
            g[i] = odd ? recv : mine;
            u[i] = odd ? mine : recv;
        }
        const int nb = odd ? 8 : 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float a;
            if (EPI == EPI_SWIGLU_F32 || (EPI == EPI_SWIGLU_MIXED && ti.e != p.shared_e)) a = __fmul_rn(silu_f32(g[i]), u[i]);
            else a = __fmul_rn(round_bf(silu_f32(g[i])), u[i]);
            stage[(nb + i) * 16 + (lane >> 1)] = (uint16_t)bf16_bits(f2bf(a));
        }
        __syncwarp();
        const int tok = lane >> 1, part = lane & 1;
        if (n0 + tok < ti.nrows) {
            const uint4 val = *reinterpret_cast<const uint4*>(stage + tok * 16 + part * 8);
            *reinterpret_cast<uint4*>(p.out + (long long)(ti.row0 + n0 + tok) * p.ld_out + ti.m * 64 + w4 * 16 +
                                      part * 8) = val;
        }
    }
    __syncwarp();
}

// ------------------------------------------------------------------ the kernel
template <int MODE, int EPI>
__global__ void __launch_bounds__(G_THREADS, 1) grouped_gemm_kernel(const __grid_constant__ GemmParams p) {
    using C = GemmCfg<MODE>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* b_tiles = base;
    uint8_t* a_tiles = b_tiles + C::STAGES * G_B_BYTES;          // shared-memory A (W8, BF16)
    uint8_t* raw_tiles = a_tiles + (C::A_TMEM ? 0 : C::STAGES * G_A_BYTES);
    GemmSmem& S = *reinterpret_cast<GemmSmem*>(raw_tiles + C::R_SLOTS * G_RAW_BYTES);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // ---- prologue: barriers, TMEM, per-expert tile offsets
    if (tid == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&S.a_full[s], MODE == GEMM_BF16 ? 1 : 4);
            mbar_init(&S.b_full[s], 32 * G_LOADERS);   // one cp.async-completion arrival per loader lane
            mbar_init(&S.empty[s], 1);
        }
        if (MODE == GEMM_W4)
            for (int s = 0; s < G_R_OPS; ++s) {
                mbar_init(&S.raw_full[s], 1);
                mbar_init(&S.raw_empty[s], 8);     // every producer warp releases every op
            }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], 4);
        }
        mbar_init(&S.final_bar, 1);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem_base, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (MODE == GEMM_BF16 && warp == 2 && lane == 0) tma_prefetch_desc(&p.tmap_a);
    {
        // tile_start[e] = sum_{e' < e} ceil(count(e') / G_BN) * m_tiles   (block scan)
        __shared__ int warp_sums[G_THREADS / 32];
        __shared__ int carry;
        if (tid == 0) carry = 0;
        __syncthreads();
        for (int e0 = 0; e0 < p.E; e0 += G_THREADS) {
            const int e = e0 + tid;
            int n = 0;
            if (e < p.E) {
                const long long begin = min((long long)p.M, (long long)(p.ends ? (e ? p.ends[e - 1] : 0) : 0));
                const long long end = min((long long)p.M, (long long)(p.ends ? p.ends[e] : p.M));
                const long long cnt = end > begin ? end - begin : 0;   // malformed ends -> no tiles
                n = (int)((cnt + G_BN - 1) / G_BN) * p.m_tiles * gemm_ksplit(p);
            }
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (lane == 31) warp_sums[warp] = incl;
            __syncthreads();
            int before = carry;
            for (int w = 0; w < warp; ++w) before += warp_sums[w];
            if (e < p.E) S.tile_start[e] = before + incl - n;
            __syncthreads();
            if (tid == G_THREADS - 1) carry = before + incl;
            __syncthreads();
        }
        if (tid == 0) {
            S.tile_start[p.E] = carry;
            S.total_tiles = carry;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    const int KB = p.K / G_BK;
    const int KBt = KB / gemm_ksplit(p);        // k-blocks per tile (the host checks KB % ksplit == 0)

    if (warp == 0 || warp >= 16) {
        // ------------------------------------------------ B loaders
        const int lw = warp == 0 ? 0 : warp - 15;
        const uint64_t keep = l2_evict_last();      // token rows are re-read by every feature tile
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && !S.abort; tile += gridDim.x) {
            TileInfo ti;
            if (!decode_tile(S, p, tile, ti)) break;
            // lane L resolves the source rows of tile rows L, L+32, L+64, L+96 (-1: zeros) ...
            int src_row[G_BN / 32];
#pragma unroll
            for (int i = 0; i < G_BN / 32; ++i) {
                const int n = lane + 32 * i;
                long long src = -1;
                if (n < ti.nrows) {
                    const long long r = ti.row0 + n;
                    src = p.row_index ? p.row_index[r] / p.index_div : r;
                    if (src < 0 || src >= p.act_rows) {
                        fnx_flag_error(FNX_DEVERR_BADID);
                        src = -1;                 // gathered as zeros
                    }
                }
                src_row[i] = (int)src;
            }
            // ... and then holds those of the rows it copies: instruction i = lw + 4u copies tile
            // rows 4i .. 4i+3, lane L row 4i + L/8 (once per tile: the per-stage loop below is
            // address arithmetic and copies only)
            int rix[G_BN / 4 / G_LOADERS];
#pragma unroll
            for (int u = 0; u < G_BN / 4 / G_LOADERS; ++u) {
                const int i = lw + G_LOADERS * u;
                rix[u] = __shfl_sync(0xffffffffu, src_row[u / 2], (4 * i + (lane >> 3)) & 31);
            }
            const int npad = (ti.nrows + 15) & ~15;
            const int c = lane & 7;               // 16-byte chunk of the 128-byte row slice
            for (int kb = 0; kb < KBt; ++kb, ++it) {
                const int s = it % C::STAGES;
                if (!mbar_wait(&S.empty[s], ((it / C::STAGES) & 1) ^ 1)) { S.abort = 1; ok = false; break; }
                const uint32_t bt = smem_u32(b_tiles + s * G_B_BYTES);
                const bf16* kbase = p.act + (ti.ks * KBt + kb) * G_BK + c * 8;
                // one instruction copies 4 whole 128-byte row slices (8 lanes per row), so each
                // touches 4 cache lines instead of 32
#pragma unroll
                for (int u = 0; u < G_BN / 4 / G_LOADERS; ++u) {
                    const int i = lw + G_LOADERS * u;
                    if (4 * i < npad) {
                        const int n = 4 * i + (lane >> 3);
                        const int r = rix[u];
                        cp_async_16_hint(bt + sw128_offset(n, c), r >= 0 ? kbase + (long long)r * p.ld_act : p.act,
                                         r >= 0, keep);
                    }
                }
                // every lane arrives once its own copies of this stage have landed
                cp_async_mbar_arrive(&S.b_full[s]);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (whole warp, one elected lane issues)
        const int my_tiles = S.total_tiles > (int)blockIdx.x ? (S.total_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        const int total_stages = my_tiles * KBt;
        int j = 0;
        uint32_t pack = 0;          // lane L: (token rows / 16 - 1) of tiles 8L .. 8L+7 of the epoch
        for (int i = 0; i < my_tiles; ++i) {
            if ((i & 255) == 0) {
                // once per 256 tiles: the only shared-memory reads of this warp in the loop
                pack = 0;
#pragma unroll 1
                for (int q = 0; q < 8; ++q) {
                    const int t = i + 8 * lane + q;
                    TileInfo ti;
                    if (t < my_tiles && decode_tile(S, p, (int)blockIdx.x + t * (int)gridDim.x, ti))
                        pack |= (uint32_t)(((ti.nrows + 15) >> 4) - 1) << (4 * q);
                }
            }
            const int loc = i & 255;
            const uint32_t n16 = ((__shfl_sync(0xffffffffu, pack, loc >> 3) >> (4 * (loc & 7))) & 15u) + 1u;
            const int ab = i & 1;
            const uint32_t idesc = idesc_bf16_f32(G_BM, (int)n16 * 16);
            const uint32_t d = tmem + ab * G_BN;
            for (int kb = 0; kb < KBt; ++kb, ++j) {
                const int s = j % C::STAGES;
                named_bar_sync(G_BAR_FULL, 64);
                tc_fence_after();
                if (elect_one()) {
                    const uint32_t b0 = smem_u32(b_tiles + s * G_B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < G_BK / 16; ++kk) {
                        if (C::A_TMEM)
                            umma_bf16_ts(d, tmem + C::A_COL0 + s * 32 + kk * 8, sdesc_kmajor_sw128(b0 + kk * 32),
                                         idesc, (kb | kk) ? 1u : 0u);
                        else
                            umma_bf16(d, sdesc_kmajor_sw128(smem_u32(a_tiles + s * G_A_BYTES) + kk * 32),
                                      sdesc_kmajor_sw128(b0 + kk * 32), idesc, (kb | kk) ? 1u : 0u);
                    }
                    umma_commit(&S.empty[s]);
                    if (kb == KBt - 1) umma_commit(&S.acc_full[ab]);
                }
                __syncwarp();
                if (j + 1 < total_stages) named_bar_arrive(G_BAR_TAKEN, 64);
            }
        }
        if (elect_one()) umma_commit(&S.final_bar);
        __syncwarp();
        mbar_wait(&S.final_bar, 0);
    } else if (warp == 2) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0, op = 0;
            const uint64_t stream_once = l2_evict_first();   // each weight block is read once
            for (int tile = blockIdx.x; !S.abort; tile += gridDim.x) {
                TileInfo ti;
                if (!decode_tile(S, p, tile, ti)) break;
                bool ok = true;
                if (MODE == GEMM_W4) {
                    const uint8_t* tsrc = reinterpret_cast<const uint8_t*>(p.w) +
                                          (weight_expert(p, ti.e) * p.m_tiles + ti.m) * KB * (long long)G_RAW_BYTES;
                    for (int kb0 = 0; kb0 < KB; kb0 += G_OPK, ++op) {
                        const int os = op % G_R_OPS;
                        if (!mbar_wait(&S.raw_empty[os], ((op / G_R_OPS) & 1) ^ 1)) { ok = false; break; }
                        const uint32_t bytes = (uint32_t)min(G_OPK, KB - kb0) * G_RAW_BYTES;
                        mbar_arrive_expect_tx(&S.raw_full[os], bytes);
                        bulk_load(smem_u32(raw_tiles + os * G_OPK * G_RAW_BYTES), tsrc + (long long)kb0 * G_RAW_BYTES,
                                  bytes, &S.raw_full[os], stream_once);
                    }
                } else if (MODE == GEMM_BF16) {
                    for (int kb = 0; kb < KBt; ++kb, ++it) {
                        const int s = it % C::STAGES;
                        if (!mbar_wait(&S.empty[s], ((it / C::STAGES) & 1) ^ 1)) { ok = false; break; }
                        mbar_arrive_expect_tx(&S.a_full[s], G_A_BYTES);
                        tma_load_2d(smem_u32(a_tiles + s * G_A_BYTES), &p.tmap_a, &S.a_full[s],
                                    (ti.ks * KBt + kb) * G_BK, ti.e * p.Nw + ti.m * G_BM);
                    }
                }
                if (!ok) { S.abort = 1; break; }
            }
        }
        __syncwarp();
    } else if (warp == 3) {
        // ------------------------------------------------ waiter: mbarriers -> named barriers
        // Runs exactly the MMA warp's stage count.  After an abort it stops waiting (the
        // data may never come) but keeps handing stages over, so the MMA warp never blocks
        // on a named barrier for good; the MMAs then read stale tiles of a failed launch.
        bool dead = false;
        int j = 0, i = 0;
        for (int tile = blockIdx.x; tile < S.total_tiles; tile += gridDim.x, ++i) {
            const int ab = i & 1;
            dead = __any_sync(0xffffffffu, dead || S.abort);
            if (!dead) {
                const bool ok = mbar_wait(&S.acc_empty[ab], ((i >> 1) & 1) ^ 1);
                if (!__all_sync(0xffffffffu, ok)) { dead = true; S.abort = 1; }
            }
            for (int kb = 0; kb < KBt; ++kb, ++j) {
                const int s = j % C::STAGES;
                const uint32_t ph = (j / C::STAGES) & 1;
                dead = __any_sync(0xffffffffu, dead || S.abort);
                if (!dead) {
                    const bool ok = mbar_wait(&S.a_full[s], ph) && mbar_wait(&S.b_full[s], ph);
                    if (!__all_sync(0xffffffffu, ok)) { dead = true; S.abort = 1; }
                }
                if (j > 0) named_bar_sync(G_BAR_TAKEN, 64);
                named_bar_arrive(G_BAR_FULL, 64);
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ epilogue warpgroup
        const int e4 = warp - 4;
        int tcount = 0;
        for (int tile = blockIdx.x; !S.abort; tile += gridDim.x, ++tcount) {
            TileInfo ti;
            if (!decode_tile(S, p, tile, ti)) break;
            const int ab = tcount & 1;
            if (!mbar_wait(&S.acc_full[ab], (tcount >> 1) & 1)) { S.abort = 1; break; }
            tc_fence_after();
            const int r = e4 * 32 + lane;
            const int npad = (ti.nrows + 15) & ~15;
            for (int n0 = 0; n0 < npad; n0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(e4 * 32) << 16) + ab * G_BN + n0, v);
                tmem_ld_wait();
                if (EPI == EPI_PLAIN && p.ksplit > 1)
                    epilogue_partial<MODE == GEMM_W8>(p, ti, r, n0, v);
                else
                    epilogue_chunk<EPI, MODE == GEMM_W8>(p, ti, r, n0, v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.acc_empty[ab]);
        }
    } else if (warp >= 8 && MODE != GEMM_BF16) {
        // ------------------------------------------------ A producers
        const int grp = (warp - 8) >> 2;
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int t = q * 32 + lane;            // tile row
        int it = 0, op = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && !S.abort; tile += gridDim.x) {
            TileInfo ti;
            if (!decode_tile(S, p, tile, ti)) break;
            for (int kb = 0; kb < KBt; ++kb, ++it) {
                const int s = it % C::STAGES;
                if (MODE == GEMM_W4) {
                    const int os = op % G_R_OPS;
                    const uint32_t rph = (op / G_R_OPS) & 1;
                    if ((it & 1) == grp) {
                        const bool got = mbar_wait(&S.raw_full[os], rph) &&
                                         mbar_wait(&S.empty[s], ((it / C::STAGES) & 1) ^ 1);
                        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                        produce_store_w4(raw_tiles + (os * G_OPK + kb % G_OPK) * G_RAW_BYTES, t,
                                         tmem + ((uint32_t)(q * 32) << 16) + C::A_COL0 + s * 32);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&S.a_full[s]);
                    }
                    if (kb % G_OPK == G_OPK - 1 || kb == KB - 1) {
                        // end of a copy: release the slot.  A warp that owned no block of it
                        // first waits for it to have landed, so its release always counts
                        // toward this copy's phase.
                        if (!__all_sync(0xffffffffu, mbar_wait(&S.raw_full[os], rph))) { ok = false; break; }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&S.raw_empty[os]);
                        ++op;
                    }
                } else if ((it & 1) == grp) {
                    if (!mbar_wait(&S.empty[s], ((it / C::STAGES) & 1) ^ 1)) { ok = false; break; }
                    produce_a_w8<EPI>(p, ti, ti.ks * KBt + kb, a_tiles + s * G_A_BYTES, t);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.a_full[s]);
                }
            }
        }
        if (!ok) S.abort = 1;
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int MODE>
inline size_t grouped_gemm_smem_bytes_t() {
    using C = GemmCfg<MODE>;
    return 1024 + (size_t)C::STAGES * (G_B_BYTES + (C::A_TMEM ? 0 : G_A_BYTES)) + (size_t)C::R_SLOTS * G_RAW_BYTES +
           sizeof(GemmSmem);
}
inline size_t grouped_gemm_smem_bytes(int mode) {
    return mode == GEMM_W4 ? grouped_gemm_smem_bytes_t<GEMM_W4>()
                           : mode == GEMM_W8 ? grouped_gemm_smem_bytes_t<GEMM_W8>() : grouped_gemm_smem_bytes_t<GEMM_BF16>();
}

}  // namespace fnx
