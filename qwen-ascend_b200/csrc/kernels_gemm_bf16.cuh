// Dense bf16 GEMM on the 5th-generation tensor cores: out[m, n] = bf16( sum_k x[m, k] * w[n, k] )
// with fp32 accumulation and one rounding (x [M, K] and w [N, K] both K-major bf16).  This is the
// router + shared-gate logits GEMM of the layer (fnx/engine.py:1786-1790: one GEMM over the
// concatenated router rows) and the hyper-connection mix's two GEMMs (fnx/engine.py:818-857).
//
// Both operands arrive by TMA (128-byte swizzle) into a ring of T_STAGES k-blocks; one thread
// issues the MMAs (M = 128 tokens, N = BN features, K = 16 each) into a double-buffered tensor-
// memory accumulator and commits each stage back to the copy thread; four epilogue warps drain the
// accumulator of one tile while the next tile accumulates.  Tiles are (128 tokens) x (BN features),
// taken persistently (tile blockIdx.x, + gridDim.x, ...); edges read the tensor maps' zero fill
// and are not stored.  Roles:
//   warp 0, one thread   TMA copies of A (x) and B (w) per k-block, after the stage is released
//   warp 1               tensor-memory allocation; one thread issues the MMAs and the commits
//   warps 2-5            epilogue: tcgen05.ld -> bf16 -> 16-byte row stores (warp w drains lane
//                        quarter w % 4 = tokens 32 (w % 4) .. +31 of the tile)
// Every wait is bounded (fnx_common.cuh): a timeout flags the device error word and the roles run
// out their tile counts (on stale data) to the final barrier, where tensor memory is freed.
#pragma once
#include "fnx_common.cuh"

namespace fnx {

constexpr int T_BM = 128;               // tokens per tile (UMMA M)
constexpr int T_BK = 64;                // k per stage (one 128-byte swizzle row)
constexpr int T_STAGES = 5;
constexpr int T_THREADS = 192;          // 6 warps
constexpr int T_A_BYTES = T_BM * T_BK * 2;

struct TGemmParams {
    CUtensorMap ta;                     // x: bf16 [M, K], box {64, 128}
    CUtensorMap tb;                     // w: bf16 [N, K], box {64, BN}
    bf16* out;                          // [M, ld_out]
    long long ld_out;
    int M, N, K;
};

struct TGemmSmem {
    uint64_t full[T_STAGES], empty[T_STAGES], acc_full[2], acc_empty[2];
    uint32_t tmem_base;
};

template <int BN>
__global__ void __launch_bounds__(T_THREADS, 1) gemm_bf16_tma_kernel(const __grid_constant__ TGemmParams p) {
    constexpr int B_BYTES = BN * T_BK * 2;
    constexpr int STAGE = T_A_BYTES + B_BYTES;             // both multiples of 1024
    constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
    static_assert(BN % 16 == 0 && BN <= 256 && B_BYTES % 1024 == 0, "UMMA N / swizzle atom");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    TGemmSmem& S = *reinterpret_cast<TGemmSmem*>(base + T_STAGES * STAGE);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (p.M + T_BM - 1) / T_BM, nt = (p.N + BN - 1) / BN;
    const int total = mt * nt, KB = p.K / T_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < T_STAGES; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.acc_full[b], 1);
            mbar_init(&S.acc_empty[b], 4);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------ TMA copies
        if (lane == 0) {
            tma_prefetch_desc(&p.ta);
            tma_prefetch_desc(&p.tb);
            int j = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x) {
                const int m = t / nt, n = t % nt;
                for (int kb = 0; kb < KB; ++kb, ++j) {
                    const int s = j % T_STAGES;
                    mbar_wait(&S.empty[s], ((j / T_STAGES) & 1) ^ 1);
                    uint8_t* st = base + s * STAGE;
                    mbar_arrive_expect_tx(&S.full[s], STAGE);
                    tma_load_2d(smem_u32(st), &p.ta, &S.full[s], kb * T_BK, m * T_BM);
                    tma_load_2d(smem_u32(st + T_A_BYTES), &p.tb, &S.full[s], kb * T_BK, n * BN);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issue
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(T_BM, BN);
            int j = 0, i = 0;
            for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
                const int ab = i & 1;
                mbar_wait(&S.acc_empty[ab], ((i >> 1) & 1) ^ 1);
                tc_fence_after();
                const uint32_t d = tmem + ab * BN;
                for (int kb = 0; kb < KB; ++kb, ++j) {
                    const int s = j % T_STAGES;
                    mbar_wait(&S.full[s], (j / T_STAGES) & 1);
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(base + s * STAGE), b0 = a0 + T_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < T_BK / 16; ++kk)
                        umma_bf16(d, sdesc_kmajor_sw128(a0 + kk * 32), sdesc_kmajor_sw128(b0 + kk * 32), idesc,
                                  (kb | kk) ? 1u : 0u);
                    umma_commit(&S.empty[s]);
                }
                umma_commit(&S.acc_full[ab]);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ epilogue (lane quarter warp % 4)
        const int q = warp & 3;
        const bool vec = (p.ld_out & 7) == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0;
        int i = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
            const int ab = i & 1;
            const int m = t / nt, n = t % nt;
            mbar_wait(&S.acc_full[ab], (i >> 1) & 1);
            tc_fence_after();
            const int row = m * T_BM + q * 32 + lane;
            bf16* orow = p.out + (long long)row * p.ld_out;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + ab * BN + c0, v);
                tmem_ld_wait();
                const int col = n * BN + c0;
                if (row < p.M && col < p.N) {
                    uint32_t o[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[e] = pack_bf2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
                    if (vec && col + 16 <= p.N) {
                        *reinterpret_cast<uint4*>(orow + col) = make_uint4(o[0], o[1], o[2], o[3]);
                        *reinterpret_cast<uint4*>(orow + col + 8) = make_uint4(o[4], o[5], o[6], o[7]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (col + e < p.N) orow[col + e] = f2bf(__uint_as_float(v[e]));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.acc_empty[ab]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int BN>
inline size_t gemm_bf16_tma_smem() {
    return 1024 + (size_t)T_STAGES * (T_A_BYTES + BN * T_BK * 2) + sizeof(TGemmSmem);
}

}  // namespace fnx
