// CTA-pair form of the W4A16 grouped GEMM (tcgen05 cta_group::2).
//
// Same problem as grouped_gemm_kernel (kernels_gemm.cuh), computed by clusters of two CTAs
// on two SMs.  A pair takes 256 weight features (feature tiles 2mp and 2mp+1) of one
// expert's token chunk: each CTA dequantises its own 128 features into its own tensor
// memory and gathers half of the chunk's token rows into its own shared memory; rank 0
// issues M = 256 MMAs that read both CTAs' A and B and accumulate 128 feature rows into
// each CTA's tensor memory.  Against the single-CTA kernel this halves the token bytes
// every SM gathers per weight byte (the gather from L2 is the single-CTA kernel's limit)
// and frees shared memory for a deeper weight ring.
//
// Roles per CTA as in the single-CTA kernel.  Cross-CTA hand-offs:
//   rank 1 waiter   relays "stage s full" (its A in TMEM and its B half in smem) to the
//                   peer_full[s] mbarrier of rank 0 (remote arrive)
//   rank 0 waiter   waits its own a_full/b_full, peer_full and acc_empty, then releases
//                   the MMA warp through named barriers
//   rank 0 MMA      commits empty[s] and acc_full[b] to both CTAs (multicast commit)
//   epilogues       both arrive on rank 0's acc_empty[b] (count 8)
// Waits on barriers that another SM completes (the multicast commits, remote arrives) poll
// with test_wait.  Every wait is bounded; the cluster barrier at the end keeps both CTAs
// (their shared and tensor memory) alive until rank 0's MMAs have completed.
#pragma once
#include "kernels_gemm.cuh"

namespace fnx {

// A stage carries P_KS k-blocks (128 k): every hand-off between the roles costs a few hundred
// cycles of latency however little work the stage holds, so stages hold two k-blocks.
constexpr int P_KS = 2;
// Token rows per pair tile.  Tensor memory holds the two accumulators (P_BN columns each) and the A
// ring (64 columns per stage) in 512 columns, so narrower token tiles buy a deeper A ring: 128 rows
// leave 4 stages (8 k-blocks in flight), 96 leave 5.
#ifndef FNX_PAIR_BN
#define FNX_PAIR_BN 128
#endif
constexpr int P_BN = FNX_PAIR_BN;
constexpr int P_STAGES = (512 - 2 * P_BN) / 64;      // A stages in tensor memory
// Token tiles have their own, deeper ring: their path (gather issue + L2 latency + hand-offs)
// is the longest of the stage loop, so it runs further ahead than the TMEM-bound A ring.
#ifndef FNX_PAIR_BSTAGES
#define FNX_PAIR_BSTAGES 7
#endif
#ifndef FNX_PAIR_ROPS
#define FNX_PAIR_ROPS 5
#endif
constexpr int P_BSTAGES = FNX_PAIR_BSTAGES;
// Producers: two groups of eight warps take alternate stages; inside a group, warp w converts
// k-block (w / 4) % 2 of the stage for tensor-memory lane quarter w % 4.  One group of four warps
// per stage (each converting both k-blocks) spent ~1400 cycles per stage on the conversion, a
// latency two groups could not hide (clock-stamped: an MMA stage every ~1120 cycles against 339
// of tensor work); splitting the k-blocks over two warps halves that latency.
#ifndef FNX_PAIR_PROD
#define FNX_PAIR_PROD 8
#endif
constexpr int P_PROD = FNX_PAIR_PROD;                // producer warps: 8 .. 8 + P_PROD - 1 (8 or 16)
constexpr int P_KPW = P_KS * 8 / P_PROD;             // k-blocks of a stage each producer warp converts
constexpr int P_LOADER0 = 8 + P_PROD;                // loader warps 0 and P_LOADER0 .. P_LOADER0 + 2
constexpr int P_THREADS = 32 * (P_LOADER0 + G_LOADERS - 1);   // 27 warps
constexpr int P_BN_HALF = P_BN / 2;                  // token rows per CTA per tile
constexpr int P_B_SUB = P_BN_HALF * G_BK * 2;        // 8 KB: one k-block of this CTA's token rows
constexpr int P_B_BYTES = P_KS * P_B_SUB;            // 16 KB per stage
constexpr int P_R_OPS = FNX_PAIR_ROPS;               // raw ring: copies of 4 tile blocks (17 KB each)
constexpr uint32_t P_TMEM_COLS = 512;
constexpr uint32_t P_A_COL0 = 2 * P_BN;
constexpr uint32_t P_A_COLS = 32 * P_KS;             // tensor-memory columns of one A stage
static_assert(G_OPK % P_KS == 0, "a copy holds whole stages");
static_assert(P_BN % 32 == 0 && P_BN <= G_BN && P_BN_HALF % (4 * G_LOADERS) == 0, "token tile: whole loader rounds");
static_assert(P_KS == 2 && (P_PROD == 8 || P_PROD == 16), "producer groups of 4 or 8 warps over 2 k-blocks");
static_assert(P_STAGES <= G_MAX_STAGES && P_BSTAGES <= G_MAX_STAGES && P_R_OPS <= G_MAX_R_OPS &&
                  P_A_COL0 + P_STAGES * P_A_COLS <= P_TMEM_COLS,
              "budget");

// Pair tile t -> expert, chunk and this CTA's feature tile (2 * pair + rank).
FNX_DEV bool decode_pair_tile(const GemmSmem& S, const GemmParams& p, int tile, uint32_t rank, TileInfo& ti) {
    if (tile >= S.total_tiles) return false;
    int lo = 0, hi = p.E;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (S.tile_start[mid] <= tile) lo = mid; else hi = mid;
    }
    const int e = lo;
    const int pairs = p.m_tiles / 2;
    const int local = tile - S.tile_start[e];
    ti.e = e;
    ti.m = 2 * (local % pairs) + (int)rank;
    const long long begin = min((long long)p.M, (long long)(p.ends ? (e ? p.ends[e - 1] : 0) : 0));
    const long long end = min((long long)p.M, (long long)(p.ends ? p.ends[e] : p.M));
    ti.row0 = (int)begin + (local / pairs) * P_BN;
    ti.nrows = (int)min((long long)P_BN, end - ti.row0);
    return true;
}

template <int EPI>
__global__ void __launch_bounds__(P_THREADS, 1) grouped_gemm_pair_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* b_tiles = base;
    uint8_t* raw_tiles = b_tiles + P_BSTAGES * P_B_BYTES;
    GemmSmem& S = *reinterpret_cast<GemmSmem*>(raw_tiles + P_R_OPS * G_OPK * G_RAW_BYTES);
    uint16_t* epi_stage = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(&S) + ((sizeof(GemmSmem) + 15) & ~15));

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank();
    const int cid = (int)cluster_id_x(), ncl = (int)num_clusters_x();

    // ---- prologue: barriers, TMEM in both CTAs, per-expert pair-tile offsets
    // stage j uses A slot j % P_STAGES (a_full / empty) and token slot j % P_BSTAGES
    // (b_full / b_empty / peer_full)
    if (tid == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&S.a_full[s], P_PROD / 2);     // the eight warps of the stage's group
            mbar_init(&S.empty[s], 1);
        }
        for (int s = 0; s < P_BSTAGES; ++s) {
            mbar_init(&S.b_full[s], p.b_tma ? 1 : 32 * G_LOADERS);
            mbar_init(&S.b_empty[s], 1);
            mbar_init(&S.peer_full[s], 1);
        }
        for (int s = 0; s < P_R_OPS; ++s) {
            mbar_init(&S.raw_full[s], 1);
            mbar_init(&S.raw_empty[s], P_PROD);      // every producer warp releases every copy
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], 8);     // four epilogue warps in each CTA
        }
        mbar_init(&S.final_bar, 1);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(&S.tmem_base, P_TMEM_COLS);
        tmem_relinquish_pair();
    }
    {
        __shared__ int warp_sums[P_THREADS / 32];
        __shared__ int carry;
        if (tid == 0) carry = 0;
        __syncthreads();
        for (int e0 = 0; e0 < p.E; e0 += P_THREADS) {
            const int e = e0 + tid;
            int n = 0;
            if (e < p.E) {
                const long long begin = min((long long)p.M, (long long)(p.ends ? (e ? p.ends[e - 1] : 0) : 0));
                const long long end = min((long long)p.M, (long long)(p.ends ? p.ends[e] : p.M));
                const long long cnt = end > begin ? end - begin : 0;
                n = (int)((cnt + P_BN - 1) / P_BN) * (p.m_tiles / 2);
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
            if (tid == P_THREADS - 1) carry = before + incl;
            __syncthreads();
        }
        if (tid == 0) {
            S.tile_start[p.E] = carry;
            S.total_tiles = carry;
        }
    }
    // both CTAs' barriers are initialised and both tensor memories allocated before any
    // remote arrival or pair MMA
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    const int KB = p.K / G_BK;
    const int KS = KB / P_KS;                            // stages per tile (K % 128 == 0)

    if ((warp == 0 || warp >= P_LOADER0) && p.b_tma) {
        // ------------------------------------------------ B by TMA: this CTA's rows of the chunk are
        // act rows row0 + rank * hp .. + hp - 1 (contiguous); boxes of 32, then 8 rows land at
        // 1024-byte aligned offsets of the stage in the layout the gathering loaders write
        if (warp == 0 && lane == 0) {
            tma_prefetch_desc(&p.tmap_b32);
            tma_prefetch_desc(&p.tmap_b8);
            int it = 0;
            for (int tile = cid; !S.abort; tile += ncl) {
                TileInfo ti;
                if (!decode_pair_tile(S, p, tile, rank, ti)) break;
                const int hp = ((ti.nrows + 15) & ~15) / 2;
                const int r0 = ti.row0 + (int)rank * hp;
                bool ok = true;
                for (int ks = 0; ks < KS; ++ks, ++it) {
                    const int s = it % P_BSTAGES;
                    if (!mbar_wait_cluster(&S.b_empty[s], ((it / P_BSTAGES) & 1) ^ 1)) { ok = false; break; }
                    mbar_arrive_expect_tx(&S.b_full[s], (uint32_t)(P_KS * hp * G_BK * 2));
#pragma unroll
                    for (int h = 0; h < P_KS; ++h) {
                        uint8_t* bt = b_tiles + s * P_B_BYTES + h * P_B_SUB;
                        const int x = (ks * P_KS + h) * G_BK;
                        int n = 0;
                        for (; n + 32 <= hp; n += 32)
                            tma_load_2d(smem_u32(bt + n * G_BK * 2), &p.tmap_b32, &S.b_full[s], x, r0 + n);
                        for (; n < hp; n += 8)
                            tma_load_2d(smem_u32(bt + n * G_BK * 2), &p.tmap_b8, &S.b_full[s], x, r0 + n);
                    }
                }
                if (!ok) { S.abort = 1; break; }
            }
        }
        __syncwarp();
    } else if (warp == 0 || warp >= P_LOADER0) {
        // ------------------------------------------------ B loaders: this CTA's half of the chunk rows
        const int lw = warp == 0 ? 0 : warp - P_LOADER0 + 1;
        const uint64_t keep = l2_evict_last();
        int it = 0;
        bool ok = true;
        for (int tile = cid; ok && !S.abort; tile += ncl) {
            TileInfo ti;
            if (!decode_pair_tile(S, p, tile, rank, ti)) break;
            const int npad = (ti.nrows + 15) & ~15;
            const int hp = npad / 2;                       // rows per CTA, a multiple of 8
            const int rbase = (int)rank * hp;
            int src_row[(P_BN_HALF + 31) / 32];            // lane L: local rows L, L+32
#pragma unroll
            for (int i = 0; i < (P_BN_HALF + 31) / 32; ++i) {
                const int n = lane + 32 * i;
                long long src = -1;
                if (n < hp && rbase + n < ti.nrows) {
                    const long long r = ti.row0 + rbase + n;
                    src = p.row_index ? p.row_index[r] / p.index_div : r;
                    if (src < 0 || src >= p.act_rows) {
                        fnx_flag_error(FNX_DEVERR_BADID);
                        src = -1;
                    }
                }
                src_row[i] = (int)src;
            }
            // instruction i = lw + 4u copies local rows 4i .. 4i+3 (8 lanes per row)
            int rix[P_BN_HALF / 4 / G_LOADERS];
#pragma unroll
            for (int u = 0; u < P_BN_HALF / 4 / G_LOADERS; ++u) {
                const int i = lw + G_LOADERS * u;
                rix[u] = __shfl_sync(0xffffffffu, src_row[u / 2], (4 * i + (lane >> 3)) & 31);
            }
            const int c = lane & 7;
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % P_BSTAGES;
                if (!mbar_wait_cluster(&S.b_empty[s], ((it / P_BSTAGES) & 1) ^ 1)) { S.abort = 1; ok = false; break; }
#pragma unroll
                for (int h = 0; h < P_KS; ++h) {
                    const uint32_t bt = smem_u32(b_tiles + s * P_B_BYTES + h * P_B_SUB);
                    const bf16* kbase = p.act + (ks * P_KS + h) * G_BK + c * 8;
#pragma unroll
                    for (int u = 0; u < P_BN_HALF / 4 / G_LOADERS; ++u) {
                        const int i = lw + G_LOADERS * u;
                        if (4 * i < hp) {
                            const int n = 4 * i + (lane >> 3);
                            const int r = rix[u];
                            cp_async_16_hint(bt + sw128_offset(n, c), r >= 0 ? kbase + (long long)r * p.ld_act : p.act,
                                             r >= 0, keep);
                        }
                    }
                }
                cp_async_mbar_arrive(&S.b_full[s]);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (rank 0)
        if (rank == 0) {
            const int my_tiles = S.total_tiles > cid ? (S.total_tiles - 1 - cid) / ncl + 1 : 0;
            const int total_stages = my_tiles * KS;
            int j = 0;
            uint32_t pack = 0;
            for (int i = 0; i < my_tiles; ++i) {
                if ((i & 255) == 0) {
                    pack = 0;
#pragma unroll 1
                    for (int q = 0; q < 8; ++q) {
                        const int t = i + 8 * lane + q;
                        TileInfo ti;
                        if (t < my_tiles && decode_pair_tile(S, p, cid + t * ncl, 0, ti))
                            pack |= (uint32_t)(((ti.nrows + 15) >> 4) - 1) << (4 * q);
                    }
                }
                const int loc = i & 255;
                const uint32_t n16 = ((__shfl_sync(0xffffffffu, pack, loc >> 3) >> (4 * (loc & 7))) & 15u) + 1u;
                const int ab = i & 1;
                const uint32_t idesc = idesc_bf16_f32(2 * G_BM, (int)n16 * 16);
                const uint32_t d = tmem + ab * P_BN;
                for (int ks = 0; ks < KS; ++ks, ++j) {
                    const int s = j % P_STAGES, sb = j % P_BSTAGES;
                    named_bar_sync(G_BAR_FULL, 64);
                    tc_fence_after();
                    if (elect_one()) {
                        const uint32_t b0 = smem_u32(b_tiles + sb * P_B_BYTES);
#pragma unroll
                        for (int h = 0; h < P_KS; ++h)
#pragma unroll
                            for (int kk = 0; kk < G_BK / 16; ++kk)
                                umma_bf16_ts_pair(d, tmem + P_A_COL0 + s * P_A_COLS + h * 32 + kk * 8,
                                                  sdesc_kmajor_sw128(b0 + h * P_B_SUB + kk * 32), idesc,
                                                  (ks | h | kk) ? 1u : 0u);
                        umma_commit_pair(&S.empty[s], 3);
                        umma_commit_pair(&S.b_empty[sb], 3);
                        if (ks == KS - 1) umma_commit_pair(&S.acc_full[ab], 3);
                    }
                    __syncwarp();
                    if (j + 1 < total_stages) named_bar_arrive(G_BAR_TAKEN, 64);
                }
            }
            if (elect_one()) umma_commit_pair(&S.final_bar, 1);
            __syncwarp();
            mbar_wait(&S.final_bar, 0);
        }
    } else if (warp == 2) {
        // ------------------------------------------------ weight copies (this CTA's feature tile)
        if (lane == 0) {
            int op = 0;
            const uint64_t stream_once = l2_evict_first();
            for (int tile = cid; !S.abort; tile += ncl) {
                TileInfo ti;
                if (!decode_pair_tile(S, p, tile, rank, ti)) break;
                bool ok = true;
                const uint8_t* tsrc = reinterpret_cast<const uint8_t*>(p.w) +
                                      (weight_expert(p, ti.e) * p.m_tiles + ti.m) * KB * (long long)G_RAW_BYTES;
                for (int kb0 = 0; kb0 < KB; kb0 += G_OPK, ++op) {
                    const int os = op % P_R_OPS;
                    if (!mbar_wait(&S.raw_empty[os], ((op / P_R_OPS) & 1) ^ 1)) { ok = false; break; }
                    const uint32_t bytes = (uint32_t)min(G_OPK, KB - kb0) * G_RAW_BYTES;
                    mbar_arrive_expect_tx(&S.raw_full[os], bytes);
                    bulk_load(smem_u32(raw_tiles + os * G_OPK * G_RAW_BYTES), tsrc + (long long)kb0 * G_RAW_BYTES, bytes,
                              &S.raw_full[os], stream_once);
                }
                if (!ok) { S.abort = 1; break; }
            }
        }
        __syncwarp();
    } else if (warp == 3) {
        if (rank == 0) {
            // ------------------------------------------------ waiter: own and peer stages -> MMA warp
            bool dead = false;
            int j = 0, i = 0;
            for (int tile = cid; tile < S.total_tiles; tile += ncl, ++i) {
                const int ab = i & 1;
                dead = __any_sync(0xffffffffu, dead || S.abort);
                if (!dead) {
                    const bool ok = mbar_wait_cluster(&S.acc_empty[ab], ((i >> 1) & 1) ^ 1);
                    if (!__all_sync(0xffffffffu, ok)) { dead = true; S.abort = 1; }
                }
                for (int ks = 0; ks < KS; ++ks, ++j) {
                    const int s = j % P_STAGES, sb = j % P_BSTAGES;
                    const uint32_t ph = (j / P_STAGES) & 1, phb = (j / P_BSTAGES) & 1;
                    dead = __any_sync(0xffffffffu, dead || S.abort);
                    if (!dead) {
                        const bool ok = mbar_wait(&S.a_full[s], ph) && mbar_wait(&S.b_full[sb], phb) &&
                                        mbar_wait_cluster(&S.peer_full[sb], phb);
                        if (!__all_sync(0xffffffffu, ok)) { dead = true; S.abort = 1; }
                    }
                    if (j > 0) named_bar_sync(G_BAR_TAKEN, 64);
                    named_bar_arrive(G_BAR_FULL, 64);
                }
            }
        } else {
            // ------------------------------------------------ relay: this CTA's stages -> rank 0
            int j = 0;
            bool ok = true;
            for (int tile = cid; ok && tile < S.total_tiles; tile += ncl) {
                for (int ks = 0; ks < KS; ++ks, ++j) {
                    const int s = j % P_STAGES, sb = j % P_BSTAGES;
                    const uint32_t ph = (j / P_STAGES) & 1, phb = (j / P_BSTAGES) & 1;
                    const bool got = !S.abort && mbar_wait(&S.a_full[s], ph) && mbar_wait(&S.b_full[sb], phb);
                    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }   // rank 0 then times out
                    if (lane == 0) mbar_arrive_remote_relaxed(mapa_rank(&S.peer_full[sb], 0));
                }
            }
            if (!ok) S.abort = 1;
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ epilogue (this CTA's 128 feature rows)
        const int e4 = warp - 4;
        int tcount = 0;
        for (int tile = cid; !S.abort; tile += ncl, ++tcount) {
            TileInfo ti;
            if (!decode_pair_tile(S, p, tile, rank, ti)) break;
            const int ab = tcount & 1;
            if (!mbar_wait_cluster(&S.acc_full[ab], (tcount >> 1) & 1)) { S.abort = 1; break; }
            tc_fence_after();
            const int npad = (ti.nrows + 15) & ~15;
            for (int n0 = 0; n0 < npad; n0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(e4 * 32) << 16) + ab * P_BN + n0, v);
                tmem_ld_wait();
                epilogue_chunk_staged<EPI>(p, ti, e4, n0, v, epi_stage + e4 * 512);
            }
            tc_fence_before();
            __syncwarp();
            // the accumulator reads completed (tcgen05.wait::ld): a relaxed arrival suffices
            if (lane == 0) {
                if (rank == 0) mbar_arrive(&S.acc_empty[ab]);
                else mbar_arrive_remote_relaxed(mapa_rank(&S.acc_empty[ab], 0));
            }
        }
    } else if (warp >= 8 && warp < 8 + P_PROD) {
        // ------------------------------------------------ A producers (this CTA's feature tile)
        const int grp = (warp - 8) / (P_PROD / 2);
        const int q = warp & 3;                          // the tensor-memory lane quarter warp % 4 reaches
        const int h0 = (((warp - 8) >> 2) % (P_PROD / 8)) * P_KPW;   // the first k-block of the stage it converts
        const int t = q * 32 + lane;
        int it = 0, op = 0;
        bool ok = true;
        for (int tile = cid; ok && !S.abort; tile += ncl) {
            TileInfo ti;
            if (!decode_pair_tile(S, p, tile, rank, ti)) break;
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % P_STAGES;
                const int kb0 = ks * P_KS;                 // first k-block of the stage
                const int os = op % P_R_OPS;
                const uint32_t rph = (op / P_R_OPS) & 1;
                if ((it & 1) == grp) {
                    const bool got = mbar_wait(&S.raw_full[os], rph) &&
                                     mbar_wait_cluster(&S.empty[s], ((it / P_STAGES) & 1) ^ 1);
                    if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
#pragma unroll
                    for (int h = h0; h < h0 + P_KPW; ++h)
                        produce_store_w4(raw_tiles + (os * G_OPK + (kb0 + h) % G_OPK) * G_RAW_BYTES, t,
                                         tmem + ((uint32_t)(q * 32) << 16) + P_A_COL0 + s * P_A_COLS + h * 32);
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.a_full[s]);
                }
                if ((kb0 + P_KS) % G_OPK == 0 || kb0 + P_KS == KB) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&S.raw_full[os], rph))) { ok = false; break; }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.raw_empty[os]);
                    ++op;
                }
            }
        }
        if (!ok) S.abort = 1;
    }

    // ---- teardown: rank 0's MMAs (which read both CTAs) are complete before either CTA
    // frees its tensor memory or exits
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, P_TMEM_COLS);
    }
}

inline size_t grouped_gemm_pair_smem_bytes() {
    return 1024 + (size_t)P_BSTAGES * P_B_BYTES + (size_t)P_R_OPS * G_OPK * G_RAW_BYTES +
           ((sizeof(GemmSmem) + 15) & ~(size_t)15) + 4 * 512 * sizeof(uint16_t);
}

}  // namespace fnx
