// libfnx_b200.so -- the C-ABI of the B200 W4A16 MoE expert path.
//
// One translation unit (so every kernel shares the device error word).  Entry points
// take raw device pointers, sizes and a cudaStream_t (void*); they launch
// asynchronously on that stream, never allocate, never synchronise, and return 0 or a
// negative FNX_E* code when an argument is rejected before launch.  Declarations and
// the reference interface each one replaces are in include/fnx_b200.h.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fnx_common.cuh"
#include "kernels_combine.cuh"
#include "kernels_decode.cuh"
#include "kernels_decode2.cuh"
#include "kernels_ep.cuh"
#include "kernels_gemm.cuh"
#include "kernels_gemm_pair.cuh"
#include "kernels_gemm_bf16.cuh"
#include "kernels_hc.cuh"
#include "kernels_route.cuh"
#include "kernels_w4gemv.cuh"
#include "kernels_w8gemv.cuh"

#define FNX_API extern "C" __attribute__((visibility("default")))

using namespace fnx;

namespace {

// Launch set-up (function attributes, occupancy, SM counts) belongs to a device, and one process
// may drive several GPUs (layers placed on different devices), so it is cached per device.
constexpr int FNX_MAX_DEVICES = 64;
inline int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= FNX_MAX_DEVICES) dev = 0;
    return dev;
}

int num_sms() {
    static int sms[FNX_MAX_DEVICES] = {};
    const int dev = current_device();
    if (!sms[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        sms[dev] = n;
    }
    return sms[dev];
}

inline int launch_rc() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FNX_OK : FNX_ELAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int grid_for(long long work, int threads) {
    long long g = (work + threads - 1) / threads;
    const long long cap = (long long)num_sms() * 8;
    if (g > cap) g = cap;
    return (int)(g < 1 ? 1 : g);
}

int weighted_reduce_launch(const void* in, const void* w, const void* inverse, void* out, int batch, int groups,
                           int width, long long row_stride, int mode, cudaStream_t st) {
    const bool vec = width % 8 == 0 && row_stride % 8 == 0 && aligned16(in) && aligned16(out) &&
                     (mode != 0 || aligned16(w));
    const long long work = (long long)batch * (vec ? width / 8 : width);
    const int grid = grid_for(work, 256);
    const bf16* x = static_cast<const bf16*>(in);
    const int64_t* inv = static_cast<const int64_t*>(inverse);
    bf16* y = static_cast<bf16*>(out);
#define FNX_WR(M, V) weighted_reduce_kernel<M, V><<<grid, 256, 0, st>>>(x, w, inv, y, batch, groups, width, row_stride)
    if (vec) {
        if (mode == 0) FNX_WR(0, true); else if (mode == 1) FNX_WR(1, true); else FNX_WR(2, true);
    } else {
        if (mode == 0) FNX_WR(0, false); else if (mode == 1) FNX_WR(1, false); else FNX_WR(2, false);
    }
#undef FNX_WR
    return launch_rc();
}

int moe_merge_launch(const void* e, const void* s, const void* g, void* y, int batch, int width, cudaStream_t st) {
    const bool vec = width % 8 == 0 && aligned16(e) && aligned16(s) && aligned16(y);
    const long long work = (long long)batch * (vec ? width / 8 : width);
    const int grid = grid_for(work, 256);
    if (vec)
        moe_merge_kernel<true><<<grid, 256, 0, st>>>((const bf16*)e, (const bf16*)s, (const bf16*)g, (bf16*)y, batch, width);
    else
        moe_merge_kernel<false><<<grid, 256, 0, st>>>((const bf16*)e, (const bf16*)s, (const bf16*)g, (bf16*)y, batch, width);
    return launch_rc();
}

// ---- TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry point,
// so the library does not link libcuda and loads on hosts without a GPU driver).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

struct MapKey {
    const void* ptr;
    int dtype, swz;
    unsigned long long d0, d1, stride;
    unsigned b0, b1;
};
struct MapEntry {
    MapKey key;
    CUtensorMap map;
    bool used;
};

// 2-D tiled map: inner dimension d0 (contiguous, elements), outer d1 rows, box {b0, b1}.
// Cached per (pointer, shape) -- weights are long-lived, so repeated calls reuse maps.
int make_map_2d(CUtensorMap* out, const void* ptr, CUtensorMapDataType dt, int esize, unsigned long long d0,
                unsigned long long d1, unsigned b0, unsigned b1, CUtensorMapSwizzle swz,
                unsigned long long stride_bytes = 0) {
    static MapEntry cache[64];
    static int next = 0;
    if (!stride_bytes) stride_bytes = d0 * (unsigned long long)esize;
    const MapKey k{ptr, (int)dt, (int)swz, d0, d1, stride_bytes, b0, b1};
    for (auto& e : cache)
        if (e.used && memcmp(&e.key, &k, sizeof(k)) == 0) {
            *out = e.map;
            return FNX_OK;
        }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return FNX_EDRIVER;
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(out, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return FNX_EALIGN;
    MapEntry& e = cache[next];
    next = (next + 1) % 64;
    e.key = k;
    e.map = *out;
    e.used = true;
    return FNX_OK;
}

template <int MODE, int EPI>
int gemm_launch_t(GemmParams& p, cudaStream_t st) {
    const size_t smem = grouped_gemm_smem_bytes(MODE);
    static bool configured[FNX_MAX_DEVICES] = {};
    const int dev = current_device();
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(grouped_gemm_kernel<MODE, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return FNX_ELAUNCH;
        configured[dev] = true;
    }
    int rc = FNX_OK;
    if (MODE == GEMM_BF16) {
        rc = make_map_2d(&p.tmap_a, p.w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (unsigned long long)p.K,
                         (unsigned long long)p.E * p.Nw, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
    const int grid = p.max_ctas > 0 && p.max_ctas < num_sms() ? p.max_ctas : num_sms();
    grouped_gemm_kernel<MODE, EPI><<<grid, G_THREADS, smem, st>>>(p);
    return launch_rc();
}

// CTA-pair W4 kernel: clusters of two CTAs, as many clusters as fit at once (the tile
// schedule is persistent and static, so every launched cluster must be resident).
template <int EPI>
int gemm_pair_launch_t(GemmParams& p, cudaStream_t st) {
    const size_t smem = grouped_gemm_pair_smem_bytes();
    static int clusters_of[FNX_MAX_DEVICES] = {};
    int& clusters = clusters_of[current_device()];
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!clusters) {
        if (cudaFuncSetAttribute(grouped_gemm_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return FNX_ELAUNCH;
        cfg.gridDim = dim3(2 * (num_sms() / 2));
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_pair_kernel<EPI>, &cfg) != cudaSuccess || n < 1)
            return FNX_ELAUNCH;
        clusters = n < num_sms() / 2 ? n : num_sms() / 2;
    }
    const int use = p.max_ctas >= 2 && p.max_ctas / 2 < clusters ? p.max_ctas / 2 : clusters;
    cfg.gridDim = dim3(2 * use);
    cfg.stream = st;
    if (cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel<EPI>, p) != cudaSuccess) return FNX_ELAUNCH;
    return launch_rc();
}

// FNX_GEMM_B_TMA=0 keeps the gathering loaders for contiguous token rows too (for comparisons).
bool b_tma_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("FNX_GEMM_B_TMA");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// FNX_GEMM_PAIR=0 selects the single-CTA W4 kernel (for comparisons).
bool pair_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("FNX_GEMM_PAIR");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

int gemm_launch(int mode, int epi, GemmParams& p, cudaStream_t st) {
    if (mode == GEMM_W4 && p.m_tiles % 2 == 0 && p.K % (G_BK * P_KS) == 0 && p.ld_out % 8 == 0 && aligned16(p.out) &&
        pair_enabled()) {
        // contiguous token rows (no row index): the pair kernel loads them by TMA
        p.b_tma = 0;
        if (!p.row_index && p.act_rows >= 32 && b_tma_enabled()) {
            const unsigned long long rows = (unsigned long long)p.act_rows;
            int rc = make_map_2d(&p.tmap_b32, p.act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (unsigned long long)p.K, rows,
                                 G_BK, 32, CU_TENSOR_MAP_SWIZZLE_128B, (unsigned long long)p.ld_act * 2);
            if (!rc)
                rc = make_map_2d(&p.tmap_b8, p.act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (unsigned long long)p.K, rows,
                                 G_BK, 8, CU_TENSOR_MAP_SWIZZLE_128B, (unsigned long long)p.ld_act * 2);
            if (rc) return rc;
            p.b_tma = 1;
        }
        if (epi == EPI_PLAIN) return gemm_pair_launch_t<EPI_PLAIN>(p, st);
        if (epi == EPI_SWIGLU_F32) return gemm_pair_launch_t<EPI_SWIGLU_F32>(p, st);
        if (epi == EPI_SWIGLU_MIXED) return gemm_pair_launch_t<EPI_SWIGLU_MIXED>(p, st);
        return gemm_pair_launch_t<EPI_SWIGLU_BF16>(p, st);
    }
    if (mode == GEMM_W4) {
        if (epi == EPI_PLAIN) return gemm_launch_t<GEMM_W4, EPI_PLAIN>(p, st);
        if (epi == EPI_SWIGLU_F32) return gemm_launch_t<GEMM_W4, EPI_SWIGLU_F32>(p, st);
        if (epi == EPI_SWIGLU_MIXED) return gemm_launch_t<GEMM_W4, EPI_SWIGLU_MIXED>(p, st);
        return gemm_launch_t<GEMM_W4, EPI_SWIGLU_BF16>(p, st);
    }
    if (mode == GEMM_W8) return gemm_launch_t<GEMM_W8, EPI_PLAIN>(p, st);
    return gemm_launch_t<GEMM_BF16, EPI_PLAIN>(p, st);
}

// Shape checks shared by the grouped GEMM entry points.
int gemm_check(int mode, int epi, const GemmParams& p) {
    if (p.E < 1 || p.E > G_MAX_E || p.M < 0 || p.K < G_BK || p.K % G_BK || p.Nw < 1) return FNX_EARG;
    if (mode == GEMM_W8 && (p.gs < G_BK || p.gs % G_BK || p.K % p.gs)) return FNX_ESHAPE;
    // bf16 weights: any width (the last tile's rows past Nw read the tensor map's zero fill and
    // are not stored); the quantised layouts come in whole 128-feature tiles
    if (mode != GEMM_BF16 && (epi == EPI_PLAIN ? p.Nw % G_BM : (p.Nw % 128))) return FNX_ESHAPE;
    if (!p.out_rows && p.ld_out < (epi == EPI_PLAIN ? p.Nw : p.Nw / 2)) return FNX_EARG;
    if (p.ld_act % 8 || !aligned16(p.act) || !aligned16(p.w) || (p.scales && !aligned16(p.scales))) return FNX_EALIGN;
    if (p.row_index && p.index_div < 1) return FNX_EARG;
    return FNX_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

// ======================================================================== misc
FNX_API const char* fnx_b200_version(void) { return "fnx_b200 1.0 (sm_100a; tcgen05 grouped GEMM, W4 decode GEMV)"; }

FNX_API unsigned fnx_device_errors(int clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fnx_errors, sizeof(v)) != cudaSuccess) return 0xffffffffu;
    if (clear) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_fnx_errors, &z, sizeof(z));
    }
    return v;
}

// ======================================================================== reference-compatible exports
FNX_API int fnx_weighted_reduce(void* input, void* weights, void* inverse, void* output, int batch, int groups,
                                int width, int row_stride, int mode, int order, void* stream) {
    if (batch < 1 || width < 1 || groups < 1 || groups > 64 || mode < 0 || mode > 2 || order != 0 ||
        row_stride < width)
        return FNX_EARG;
    if (mode == 2 && !inverse) return FNX_EARG;
    return weighted_reduce_launch(input, weights, inverse, output, batch, groups, width, row_stride, mode,
                                  (cudaStream_t)stream);
}

FNX_API int fnx_moe_merge_ex(void* e, void* s, void* g, void* y, int batch, int width, void* stream) {
    if (batch < 1 || width < 1) return FNX_EARG;
    return moe_merge_launch(e, s, g, y, batch, width, (cudaStream_t)stream);
}

FNX_API int fnx_moe_merge(void* e, void* s, void* g, void* y, int batch, void* stream) {
    return fnx_moe_merge_ex(e, s, g, y, batch, 2560, stream);
}

FNX_API int fnx_moe_epilogue_ex(void* y, void* w, void* shared, void* gate, void* out, int k, int width, void* stream) {
    if (k < 1 || k > 64 || width < 1) return FNX_EARG;
    moe_epilogue_kernel<<<(width + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)y, (const bf16*)w, (const bf16*)shared, (const bf16*)gate, (bf16*)out, k, width);
    return launch_rc();
}

FNX_API int fnx_moe_epilogue(void* y, void* w, void* shared, void* gate, void* out, void* stream) {
    return fnx_moe_epilogue_ex(y, w, shared, gate, out, 10, 2560, stream);
}

FNX_API int fnx_gather_pair_ex(void* w, void* s, void* ids, void* ow, void* os, int E, int K, int G, int N,
                               int nslots, void* stream) {
    if (K < 1 || G < 1 || N < 8 || N % 8 || nslots < 1 || nslots > 65535) return FNX_EARG;
    const bool v16 = (N / 2) % 16 == 0 && aligned16(w) && aligned16(s) && aligned16(ow) && aligned16(os);
    if (!v16 && (N / 2) % 2) return FNX_ESHAPE;
    const long long units = ((long long)K * N / 2 + (long long)G * N * 2) / (v16 ? 16 : 2);
    dim3 grid((unsigned)grid_for(units, 256 * 4), (unsigned)nslots);
    gather_pair_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)w, (const uint8_t*)s, (const int64_t*)ids,
                                                                (uint8_t*)ow, (uint8_t*)os, E, K, G, N, nslots);
    return launch_rc();
}

FNX_API int fnx_gather_pair(void* w, void* s, void* ids, void* ow, void* os, int K, int G, int N, void* stream) {
    return fnx_gather_pair_ex(w, s, ids, ow, os, 0, K, G, N, 10, stream);
}

FNX_API int fnx_moe_combine(void* yd, void* wf, void* inverse, void* sh, void* gate, long long gate_ld, void* out, int T,
                            int k, int H, void* stream) {
    if (T < 0 || k < 1 || k > 64 || H < 1 || gate_ld < 1) return FNX_EARG;
    if ((long long)T * k > 0x7fffffffLL) return FNX_ESHAPE;
    if (T == 0) return FNX_OK;
    const bool vec = H % 8 == 0 && aligned16(yd) && aligned16(sh) && aligned16(out);
    const int grid = grid_for((long long)T * (vec ? H / 8 : H), 256);
    cudaStream_t st = (cudaStream_t)stream;
    if (vec)
        moe_combine_kernel<true><<<grid, 256, 0, st>>>((const bf16*)yd, (const float*)wf, (const int64_t*)inverse,
                                                        (const bf16*)sh, (const bf16*)gate, gate_ld, (bf16*)out, T, k, H);
    else
        moe_combine_kernel<false><<<grid, 256, 0, st>>>((const bf16*)yd, (const float*)wf, (const int64_t*)inverse,
                                                         (const bf16*)sh, (const bf16*)gate, gate_ld, (bf16*)out, T, k, H);
    return launch_rc();
}

// inject (kernels/inject/inject.cpp:26): hyper [B, HC*H], y [B, H], gate [B, HC] bf16
FNX_API int fnx_inject_ex(void* h, void* y, void* g, void* out, int batch, int H, int HC, void* stream) {
    if (batch < 1 || H < 8 || H % 8 || HC < 1 || HC > 64 || !h || !y || !g || !out) return FNX_EARG;
    if (!aligned16(h) || !aligned16(y) || !aligned16(out)) return FNX_EALIGN;
    inject_kernel<<<grid_for((long long)batch * (H / 8), 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)h, (const bf16*)y, (const bf16*)g, (bf16*)out, batch, H, HC);
    return launch_rc();
}

FNX_API int fnx_inject(void* h, void* y, void* g, void* out, int batch, void* stream) {
    return fnx_inject_ex(h, y, g, out, batch, 2560, 4, stream);
}

FNX_API int fnx_moe_combine_inject(void* yd, void* wf, void* inverse, void* sh, void* gate, long long gate_ld,
                                   void* hyper, void* inj, void* out_hyper, void* out, int T, int k, int H, int HC,
                                   void* stream) {
    if (T < 0 || k < 1 || k > 16 || H < 8 || H % 8 || gate_ld < 1 || HC < 1 || HC > 64 || !hyper || !inj ||
        !out_hyper)
        return FNX_EARG;
    if (!aligned16(yd) || !aligned16(sh) || !aligned16(hyper) || !aligned16(out_hyper) || (out && !aligned16(out)))
        return FNX_EALIGN;
    if ((long long)T * k > 0x7fffffffLL) return FNX_ESHAPE;
    if (T == 0) return FNX_OK;
    const int grid = grid_for((long long)T * (H / 8), 256);
    moe_combine_kernel<true><<<grid, 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)yd, (const float*)wf, (const int64_t*)inverse, (const bf16*)sh, (const bf16*)gate, gate_ld,
        (bf16*)out, T, k, H, (const bf16*)hyper, (const bf16*)inj, (bf16*)out_hyper, HC);
    return launch_rc();
}

// ------------------------------------------------------------------ hyper-connection mix
FNX_API int fnx_hc_rms_norm(void* x, void* w, void* out, int batch, int H, int HC, float eps, void* stream) {
    if (batch < 0 || H < 1 || HC < 1 || !(eps >= 0.f) || (batch > 0 && (!x || !w || !out))) return FNX_EARG;
    if (batch == 0) return FNX_OK;
    hc_rms_norm_kernel<<<batch * HC, 256, 0, (cudaStream_t)stream>>>((const bf16*)x, (const bf16*)w, (bf16*)out, H,
                                                                      HC, eps);
    return launch_rc();
}

FNX_API int fnx_hc_activation_ex(void* x, void* m, void* g, int batch, int n_mix, int HC, int mode, void* stream) {
    if (batch < 1 || n_mix < 1 || HC < 1 || mode < 0 || mode > 3 || !x || !m || !g) return FNX_EARG;
    hc_activation_kernel<<<grid_for((long long)batch * (n_mix + HC), 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (bf16*)m, (bf16*)g, batch, n_mix, HC, mode);
    return launch_rc();
}

// kernels/post_ops/post_ops.cpp:25: di [batch, 324] -> mixed [batch, 320], gates [batch, 4]
FNX_API int fnx_hc_activation(void* x, void* m, void* g, int batch, int mode, void* stream) {
    return fnx_hc_activation_ex(x, m, g, batch, 320, 4, mode, stream);
}

FNX_API int fnx_hc_sigmoid_reduce_ex(void* x, void* l, void* y, int batch, int H, int HC, void* stream) {
    if (batch < 1 || H < 1 || HC < 1 || !x || !l || !y) return FNX_EARG;
    hc_sigmoid_reduce_kernel<<<grid_for((long long)batch * H, 256), 256, 0, (cudaStream_t)stream>>>(
        (const bf16*)x, (const bf16*)l, (bf16*)y, batch, H, HC);
    return launch_rc();
}

// kernels/post_ops/post_ops.cpp:50: values, logits [batch, 10240] -> mixed [batch, 2560]
FNX_API int fnx_hc_sigmoid_reduce(void* x, void* l, void* y, int batch, void* stream) {
    return fnx_hc_sigmoid_reduce_ex(x, l, y, batch, 2560, 4, stream);
}

// ======================================================================== routing
FNX_API int fnx_router_topk(void* logits, long long ld, void* bias, void* w_out, void* idx_out, void* wf_out, int T,
                            int E, int k, void* stream) {
    if (T < 0 || E < 1 || E > ROUTE_MAX_E || k < 1 || k > ROUTE_MAX_K || k > E || ld < E) return FNX_EARG;
    if (T == 0) return FNX_OK;
    const int blocks = (T + 7) / 8;
    cudaStream_t st = (cudaStream_t)stream;
#define FNX_TOPK(P) router_topk_kernel<P><<<blocks, 256, 0, st>>>((const bf16*)logits, ld, (const float*)bias, \
        (bf16*)w_out, (int64_t*)idx_out, nullptr, (float*)wf_out, T, E, k)
    if (E <= 256) FNX_TOPK(8);
    else if (E <= 512) FNX_TOPK(16);
    else if (E <= 1024) FNX_TOPK(32);
    else FNX_TOPK(64);
#undef FNX_TOPK
    return launch_rc();
}

FNX_API size_t fnx_moe_permute_workspace(int n, int E) {
    const int chunks = (n + PERM_CHUNK - 1) / PERM_CHUNK;
    return (size_t)(chunks < 1 ? 1 : chunks) * E * sizeof(int);
}

namespace {
// stable counting sort of n ids into E buckets of `div` consecutive ids each
// n_dev: optional device-side entry count (<= n); base: added to ends and inverse;
// row_map: order holds row_map[i] in place of the entry index i.
int permute_launch(const void* idx, void* order, void* inverse, void* ends, void* counts, int n, int E, int div,
                   void* workspace, cudaStream_t st, const long long* n_dev = nullptr, long long base = 0,
                   const int64_t* row_map = nullptr) {
    const int chunks = (n + PERM_CHUNK - 1) / PERM_CHUNK;
    int* hist = (int*)workspace;
    if (chunks == 0) {
        if (base == 0) cudaMemsetAsync(ends, 0, sizeof(int64_t) * E, st);
        else fill_i64_kernel<<<1, 256, 0, st>>>((int64_t*)ends, E, base);
        if (counts) cudaMemsetAsync(counts, 0, sizeof(int64_t) * E, st);
        return launch_rc();
    }
    const int dev = current_device();
    const size_t ssm = permute_scatter_smem(E);
    static bool ssm_set[FNX_MAX_DEVICES] = {};
    if (ssm > 48 * 1024 && !ssm_set[dev]) {
        if (cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)permute_scatter_smem(PERM_MAX_E)) != cudaSuccess)
            return FNX_ELAUNCH;
        ssm_set[dev] = true;
    }
    permute_hist_kernel<<<chunks, 256, E * sizeof(int), st>>>((const int64_t*)idx, n, n_dev, E, div, hist);
    static bool scan_set[FNX_MAX_DEVICES] = {};
    if (!scan_set[dev]) {
        if (cudaFuncSetAttribute(permute_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)PERM_SCAN_SMEM) != cudaSuccess)
            return FNX_ELAUNCH;
        scan_set[dev] = true;
    }
    permute_scan_kernel<<<1, 1024, permute_scan_smem(chunks, E), st>>>(hist, chunks, E, (int64_t*)ends,
                                                                       (int64_t*)counts, base);
    permute_scatter_kernel<<<chunks, 32 * PERM_WARPS, ssm, st>>>(
        (const int64_t*)idx, n, n_dev, E, div, hist, (int64_t*)order, (int64_t*)inverse, base, row_map);
    return launch_rc();
}
}  // namespace

FNX_API int fnx_moe_permute(void* idx, void* order, void* inverse, void* ends, void* counts, int n, int E,
                            void* workspace, size_t ws_bytes, void* stream) {
    if (n < 0 || E < 1 || E > PERM_MAX_E) return FNX_EARG;
    if (ws_bytes < fnx_moe_permute_workspace(n, E)) return FNX_EWORKSPACE;
    return permute_launch(idx, order, inverse, ends, counts, n, E, 1, workspace, (cudaStream_t)stream);
}

// ======================================================================== expert parallel
FNX_API size_t fnx_ep_layout_workspace(int n, int G) {
    return (fnx_moe_permute_workspace(n, G) + 15) / 16 * 16 + sizeof(int64_t) * (size_t)(G < 1 ? 1 : G);
}

FNX_API int fnx_ep_dispatch_layout(const void* idx, int n, int E, int G, void* order, void* inverse, void* counts,
                                   void* workspace, size_t ws_bytes, void* stream) {
    if (n < 0 || G < 1 || G > PERM_MAX_E || E < G || E % G != 0 || !counts) return FNX_EARG;
    if (ws_bytes < fnx_ep_layout_workspace(n, G)) return FNX_EWORKSPACE;
    void* ends = (char*)workspace + (fnx_moe_permute_workspace(n, G) + 15) / 16 * 16;
    return permute_launch(idx, order, inverse, ends, counts, n, G, E / G, workspace, (cudaStream_t)stream);
}

FNX_API int fnx_ep_gather_rows(const void* src, long long ld_src, long long src_rows, const void* index, int index_div,
                               const void* ids, int ids_mod, void* dst, long long ld_dst, void* ids_out, long long n,
                               int H, void* stream) {
    if (n < 0 || H < 1 || ld_src < H || ld_dst < H || src_rows < 0 || index_div < 1) return FNX_EARG;
    if (ids_out && (!ids || !index || ids_mod < 1)) return FNX_EARG;
    if (n == 0) return FNX_OK;
    const bool vec = H % 8 == 0 && ld_src % 8 == 0 && ld_dst % 8 == 0 && aligned16(src) && aligned16(dst);
    const long long warps_needed = n;
    long long blocks = (warps_needed + 7) / 8;
    const long long cap = (long long)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    cudaStream_t st = (cudaStream_t)stream;
    if (vec)
        ep_gather_rows_kernel<true><<<(int)blocks, 256, 0, st>>>((const bf16*)src, ld_src, src_rows, (const int64_t*)index,
                                                                 index_div, (const int64_t*)ids, ids_mod, (bf16*)dst,
                                                                 ld_dst, (int64_t*)ids_out, n, H);
    else
        ep_gather_rows_kernel<false><<<(int)blocks, 256, 0, st>>>((const bf16*)src, ld_src, src_rows,
                                                                  (const int64_t*)index, index_div, (const int64_t*)ids,
                                                                  ids_mod, (bf16*)dst, ld_dst, (int64_t*)ids_out, n, H);
    return launch_rc();
}

// ------------------------------------------------------------------ peer-memory exchange
namespace {
struct EPRegion {
    size_t flags, cnt, plan, epoch, tickets, bcount, recv_e, recv_row, recv_x, yb, sink, total;
};
EPRegion ep_region(int H, int k, int T_cap, long long cap, long long cap_tok) {
    EPRegion R{};
    size_t o = 0;
    R.flags = o;    o += align_up(sizeof(unsigned) * EP_PHASES * 2 * EP_MAX_G, 256);
    R.cnt = o;      o += align_up(sizeof(long long) * 2 * EP_MAX_G * EP_MAX_G * 2, 256);
    R.plan = o;     o += align_up(sizeof(long long) * EP_PLAN_LEN, 256);
    R.epoch = o;    R.tickets = o + 16; o += 256;
    R.bcount = o;   o += align_up(sizeof(int) * (size_t)(((long long)T_cap * k + 1023) / 1024 + 1), 256);
    R.recv_e = o;   o += align_up(sizeof(int64_t) * (size_t)cap, 256);
    R.recv_row = o; o += align_up(sizeof(int64_t) * (size_t)cap, 256);
    R.recv_x = o;   o += align_up(sizeof(bf16) * (size_t)(cap_tok + T_cap) * H, 256);
    R.yb = o;       o += align_up(sizeof(bf16) * (size_t)T_cap * k * H, 256);
    R.sink = o;     o += align_up(sizeof(bf16) * (size_t)H, 256);
    R.total = o;
    return R;
}
bool ep_shape_ok(int world, int H, int k, int T_cap) {
    return world >= 1 && world <= EP_MAX_G && H >= 8 && H % 8 == 0 && k >= 1 && k <= 64 && T_cap >= 1 &&
           (long long)world * T_cap * k + T_cap <= 0x7fffffffLL;
}
const EPDesc* ep_desc(const void* d) {
    const EPDesc* e = (const EPDesc*)d;
    return (e && e->world >= 1 && e->world <= EP_MAX_G && e->plan) ? e : nullptr;
}
}  // namespace

FNX_API size_t fnx_ep_p2p_region_bytes(int world, int H, int k, int T_cap) {
    if (!ep_shape_ok(world, H, k, T_cap)) return 0;
    return ep_region(H, k, T_cap, (long long)world * T_cap * k, (long long)world * T_cap).total;
}

FNX_API int fnx_ep_p2p_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return FNX_EARG;
    *ptr = nullptr;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return FNX_ELAUNCH;
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return FNX_ELAUNCH;
    }
    return FNX_OK;
}

FNX_API int fnx_ep_p2p_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? FNX_OK : FNX_ELAUNCH; }

FNX_API int fnx_ep_p2p_export(void* ptr, void* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    if (!ptr || !handle) return FNX_EARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return FNX_ELAUNCH;
    memcpy(handle, &h, sizeof(h));
    return FNX_OK;
}

FNX_API int fnx_ep_p2p_import(const void* handle, void** ptr) {
    if (!ptr || !handle) return FNX_EARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? FNX_OK : FNX_ELAUNCH;
}

FNX_API int fnx_ep_p2p_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? FNX_OK : FNX_ELAUNCH; }

FNX_API size_t fnx_ep_p2p_desc_bytes(void) { return sizeof(EPDesc); }

FNX_API int fnx_ep_p2p_desc(void* desc, int rank, int world, void* const* bases, int H, int k, int T_cap, int Eg) {
    if (!desc || !bases || !ep_shape_ok(world, H, k, T_cap) || rank < 0 || rank >= world || Eg < 1) return FNX_EARG;
    for (int q = 0; q < world; ++q)
        if (!bases[q] || !aligned16(bases[q])) return FNX_EARG;
    EPDesc d{};
    d.rank = rank; d.world = world; d.H = H; d.k = k; d.T_cap = T_cap; d.Eg = Eg;
    d.cap = (long long)world * T_cap * k;
    d.cap_tok = (long long)world * T_cap;
    const EPRegion R = ep_region(H, k, T_cap, d.cap, d.cap_tok);
    char* own = (char*)bases[rank];
    d.plan = (long long*)(own + R.plan);
    d.epoch = (unsigned*)(own + R.epoch);
    d.tickets = (unsigned*)(own + R.tickets);
    d.bcount = (int*)(own + R.bcount);
    d.sink = (bf16*)(own + R.sink);
    for (int q = 0; q < world; ++q) {
        char* b = (char*)bases[q];
        d.flags[q] = (unsigned*)(b + R.flags);
        d.cnt[q] = (long long*)(b + R.cnt);
        d.recv_x[q] = (bf16*)(b + R.recv_x);
        d.recv_e[q] = (int64_t*)(b + R.recv_e);
        d.recv_row[q] = (int64_t*)(b + R.recv_row);
        d.yb[q] = (bf16*)(b + R.yb);
    }
    memcpy(desc, &d, sizeof(d));
    return FNX_OK;
}

FNX_API void* fnx_ep_p2p_local(const void* desc, int which) {
    const EPDesc* d = ep_desc(desc);
    if (!d) return nullptr;
    switch (which) {
        case 0: return d->recv_x[d->rank];
        case 1: return d->recv_e[d->rank];
        case 2: return d->yb[d->rank];
        case 3: return d->plan;
        case 4: return d->recv_row[d->rank];
        default: return nullptr;
    }
}

FNX_API long long fnx_ep_p2p_capacity(const void* desc, int which) {
    const EPDesc* d = ep_desc(desc);
    if (!d) return -1;
    return which == 0 ? d->cap : which == 1 ? d->cap_tok : -1;
}

FNX_API long long fnx_ep_p2p_received(const void* desc) {
    const EPDesc* d = ep_desc(desc);
    long long v = -1;
    if (!d || cudaMemcpy(&v, d->plan + EP_R, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return v;
}

FNX_API int fnx_ep_p2p_dedup(const void* desc, const void* order, const void* counts, int T, void* tok_index,
                             void* tcounts, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || T < 0 || T > d->T_cap || !counts || !tcounts || (T > 0 && (!order || !tok_index))) return FNX_EARG;
    const int n = T * d->k;
    const int blocks = n > 0 ? (n + 1023) / 1024 : 1;
    cudaStream_t st = (cudaStream_t)stream;
    ep_dedup_count_kernel<<<blocks, 1024, 0, st>>>(*d, (const int64_t*)order, (const int64_t*)counts, n);
    ep_dedup_index_kernel<<<blocks, 1024, 0, st>>>(*d, (const int64_t*)order, (const int64_t*)counts, n,
                                                   (int*)tok_index, (int64_t*)tcounts);
    return launch_rc();
}

FNX_API int fnx_ep_p2p_counts(const void* desc, const void* counts, const void* tcounts, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || !counts || !tcounts) return FNX_EARG;
    ep_counts_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(*d, (const int64_t*)counts, (const int64_t*)tcounts);
    return launch_rc();
}

FNX_API int fnx_ep_p2p_push_ex(const void* desc, const void* x, int T, const void* order, const void* idx,
                               const void* tok_index, int flags, int max_blocks, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || T < 0 || T > d->T_cap || (T > 0 && (!x || !order || !idx || !tok_index)) || !aligned16(x) ||
        (flags & ~1) || max_blocks < 0)
        return FNX_EARG;
    const long long rows = (long long)T * d->k + T;
    long long blocks = (rows + 7) / 8;
    if (blocks < 1) blocks = 1;
    if (blocks > (long long)num_sms() * 4) blocks = (long long)num_sms() * 4;
    if (max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
    ep_push_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(*d, (const bf16*)x, T, (const int64_t*)order,
                                                                  (const int64_t*)idx, (const int*)tok_index,
                                                                  (flags & 1) == 0);
    return launch_rc();
}

FNX_API int fnx_ep_p2p_push(const void* desc, const void* x, int T, const void* order, const void* idx,
                            const void* tok_index, void* stream) {
    return fnx_ep_p2p_push_ex(desc, x, T, order, idx, tok_index, 0, 0, stream);
}

FNX_API int fnx_ep_p2p_wait(const void* desc, int phase, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || phase < 0 || phase >= EP_PHASES) return FNX_EARG;
    ep_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*d, phase);
    return launch_rc();
}

FNX_API int fnx_ep_p2p_signal(const void* desc, int phase, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || phase < 0 || phase >= EP_PHASES) return FNX_EARG;
    ep_signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(*d, phase);
    return launch_rc();
}

FNX_API size_t fnx_ep_p2p_recv_workspace(const void* desc) {
    const EPDesc* d = ep_desc(desc);
    return d ? fnx_moe_permute_workspace((int)d->cap, d->Eg) : 0;
}

FNX_API int fnx_ep_p2p_recv_layout(const void* desc, int T, void* order_x, void* ends_x, void* pos, void* rows,
                                   void* sh_out, void* workspace, size_t ws_bytes, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || T < 0 || T > d->T_cap || !order_x || !ends_x || !pos || !rows || !sh_out || !aligned16(sh_out) ||
        d->Eg > PERM_MAX_E)
        return FNX_EARG;
    if (ws_bytes < fnx_ep_p2p_recv_workspace(desc)) return FNX_EWORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    ep_head_kernel<<<num_sms() * 2, 256, 0, st>>>(*d, (int64_t*)order_x, (int64_t*)ends_x, (bf16**)rows,
                                                  (bf16*)sh_out, T);
    const int rc = permute_launch(d->recv_e[d->rank], (int64_t*)order_x + T, pos, (int64_t*)ends_x + 1, nullptr,
                                  (int)d->cap, d->Eg, 1, workspace, st, d->plan + EP_R, T, d->recv_row[d->rank]);
    if (rc) return rc;
    ep_rows_kernel<<<num_sms() * 2, 256, 0, st>>>(*d, (const int64_t*)pos, T, (bf16**)rows);
    return launch_rc();
}

// The received slots alone (the shared expert computed elsewhere, from the rank's own tokens):
// order_r [cap] (token row of each slot in the region, expert-major), ends_r [Eg] (from 0), pos
// [cap] and rows_r [cap] (each slot's down-row destination in its source's return buffer).
FNX_API int fnx_ep_p2p_recv_layout_routed(const void* desc, void* order_r, void* ends_r, void* pos, void* rows_r,
                                          void* workspace, size_t ws_bytes, void* stream) {
    const EPDesc* d = ep_desc(desc);
    if (!d || !order_r || !ends_r || !pos || !rows_r || d->Eg > PERM_MAX_E) return FNX_EARG;
    if (ws_bytes < fnx_ep_p2p_recv_workspace(desc)) return FNX_EWORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    ep_sink_rows_kernel<<<num_sms() * 2, 256, 0, st>>>(*d, (bf16**)rows_r);
    const int rc = permute_launch(d->recv_e[d->rank], order_r, pos, ends_r, nullptr, (int)d->cap, d->Eg, 1, workspace,
                                  st, d->plan + EP_R, 0, d->recv_row[d->rank]);
    if (rc) return rc;
    ep_rows_kernel<<<num_sms() * 2, 256, 0, st>>>(*d, (const int64_t*)pos, 0, (bf16**)rows_r);
    return launch_rc();
}

// ======================================================================== grouped GEMMs
FNX_API int fnx_moe_grouped_w4(const void* act, long long ld_act, long long act_rows, const void* row_index,
                               int index_div, const void* tiles, const void* ends, void* out, long long ld_out, int E,
                               int M, int K, int Nw, int epilogue, void* stream) {
    GemmParams p{};
    p.act = (const bf16*)act; p.ld_act = ld_act; p.row_index = (const int64_t*)row_index; p.index_div = index_div;
    p.act_rows = act_rows;
    if (act_rows < 0 || act_rows > 0x7fffffffLL || (!row_index && act_rows < M)) return FNX_EARG;
    p.w = tiles; p.ends = (const int64_t*)ends; p.out = (bf16*)out; p.ld_out = ld_out;
    p.E = E; p.M = M; p.K = K; p.Nw = Nw; p.gs = 0;
    if (epilogue < 0 || epilogue > 4) return FNX_EARG;
    // 3: shared expert last (expert E-1), 4: shared expert first (expert 0)
    p.shared_e = epilogue == 4 ? 0 : E - 1;
    if (epilogue == 4) epilogue = EPI_SWIGLU_MIXED;
    p.m_tiles = epilogue == EPI_PLAIN ? Nw / G_BM : (Nw / 2) / 64;
    const int rc = gemm_check(GEMM_W4, epilogue, p);
    if (rc) return rc;
    if (M == 0) return FNX_OK;
    return gemm_launch(GEMM_W4, epilogue, p, (cudaStream_t)stream);
}

// fnx_moe_grouped_w4 on at most max_ctas CTAs (0: all that fit), so that kernels of another
// stream (the expert-parallel exchange) keep SMs while it runs.
FNX_API int fnx_moe_grouped_w4_lim(const void* act, long long ld_act, long long act_rows, const void* row_index,
                                   int index_div, const void* tiles, const void* ends, void* out, long long ld_out,
                                   int E, int M, int K, int Nw, int epilogue, int max_ctas, void* stream) {
    if (max_ctas < 0) return FNX_EARG;
    GemmParams p{};
    p.act = (const bf16*)act; p.ld_act = ld_act; p.row_index = (const int64_t*)row_index; p.index_div = index_div;
    p.act_rows = act_rows;
    if (act_rows < 0 || act_rows > 0x7fffffffLL || (!row_index && act_rows < M)) return FNX_EARG;
    p.w = tiles; p.ends = (const int64_t*)ends; p.out = (bf16*)out; p.ld_out = ld_out;
    p.E = E; p.M = M; p.K = K; p.Nw = Nw; p.gs = 0;
    p.max_ctas = max_ctas;
    if (epilogue < 0 || epilogue > 4) return FNX_EARG;
    p.shared_e = epilogue == 4 ? 0 : E - 1;
    if (epilogue == 4) epilogue = EPI_SWIGLU_MIXED;
    p.m_tiles = epilogue == EPI_PLAIN ? Nw / G_BM : (Nw / 2) / 64;
    const int rc = gemm_check(GEMM_W4, epilogue, p);
    if (rc) return rc;
    if (M == 0) return FNX_OK;
    return gemm_launch(GEMM_W4, epilogue, p, (cudaStream_t)stream);
}

// fnx_moe_grouped_w4 over a selection of experts read in place: group e (rows [ends[e-1], ends[e]))
// multiplies the tile blocks of expert expert_ids[e] of the E_w experts in `tiles` (no copy of the
// selected experts, as ExpW4.apply / apply_diag need).
FNX_API int fnx_moe_grouped_w4_sel(const void* act, long long ld_act, long long act_rows, const void* row_index,
                                   int index_div, const void* tiles, int E_w, const void* expert_ids, const void* ends,
                                   void* out, long long ld_out, int E, int M, int K, int Nw, int epilogue,
                                   void* stream) {
    if (!expert_ids || E_w < 1 || epilogue < 0 || epilogue > 2) return FNX_EARG;
    GemmParams p{};
    p.act = (const bf16*)act; p.ld_act = ld_act; p.row_index = (const int64_t*)row_index; p.index_div = index_div;
    p.act_rows = act_rows;
    if (act_rows < 0 || act_rows > 0x7fffffffLL || (!row_index && act_rows < M)) return FNX_EARG;
    p.w = tiles; p.ends = (const int64_t*)ends; p.out = (bf16*)out; p.ld_out = ld_out;
    p.E = E; p.M = M; p.K = K; p.Nw = Nw; p.gs = 0;
    p.expert_ids = (const int64_t*)expert_ids;
    p.E_w = E_w;
    p.shared_e = -1;
    p.m_tiles = epilogue == EPI_PLAIN ? Nw / G_BM : (Nw / 2) / 64;
    const int rc = gemm_check(GEMM_W4, epilogue, p);
    if (rc) return rc;
    if (M == 0) return FNX_OK;
    return gemm_launch(GEMM_W4, epilogue, p, (cudaStream_t)stream);
}

FNX_API int fnx_weighted_sum_f32(const void* y, const void* w, void* out, int nE, int N, void* stream) {
    if (nE < 1 || N < 1 || !y || !w || !out) return FNX_EARG;
    weighted_sum_f32_kernel<<<grid_for(N, 256), 256, 0, (cudaStream_t)stream>>>((const float*)y, (const float*)w,
                                                                             (float*)out, nE, N);
    return launch_rc();
}

FNX_API int fnx_moe_grouped_w4_rows(const void* act, long long ld_act, long long act_rows, const void* row_index,
                                    int index_div, const void* tiles, const void* ends, void* out_rows, int E, int M,
                                    int K, int Nw, void* stream) {
    if (!out_rows) return FNX_EARG;
    GemmParams p{};
    p.act = (const bf16*)act; p.ld_act = ld_act; p.row_index = (const int64_t*)row_index; p.index_div = index_div;
    p.act_rows = act_rows;
    if (act_rows < 0 || act_rows > 0x7fffffffLL || (!row_index && act_rows < M)) return FNX_EARG;
    p.w = tiles; p.ends = (const int64_t*)ends; p.out = nullptr; p.ld_out = Nw;
    p.out_rows = (bf16* const*)out_rows;
    p.E = E; p.M = M; p.K = K; p.Nw = Nw; p.gs = 0;
    p.m_tiles = Nw / G_BM;
    p.shared_e = -1;
    const int rc = gemm_check(GEMM_W4, EPI_PLAIN, p);
    if (rc) return rc;
    if (M == 0) return FNX_OK;
    return gemm_launch(GEMM_W4, EPI_PLAIN, p, (cudaStream_t)stream);
}

namespace {
template <int MT, int CL>
int w8_gemv_launch_t(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int gs,
                     cudaStream_t st) {
    const size_t smem = w8a16_gemv_smem(MT, CL, K);
    static bool configured[FNX_MAX_DEVICES] = {};
    const int dev = current_device();
    if (!configured[dev]) {                           // once per device, for the largest K accepted (8192)
        if (cudaFuncSetAttribute(w8a16_gemv_kernel<MT, CL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)w8a16_gemv_smem(MT, CL, 8192)) != cudaSuccess)
            return FNX_ELAUNCH;
        configured[dev] = true;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = CL;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((N + W8V_COLS - 1) / W8V_COLS), CL, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, w8a16_gemv_kernel<MT, CL>, (const bf16*)x, (const int8_t*)w8t, (const bf16*)sc,
                           (bf16*)y, M, K, N, gs) != cudaSuccess)
        return FNX_ELAUNCH;
    return launch_rc();
}

#ifndef FNX_W8V_CL16
#define FNX_W8V_CL16 4
#endif

bool w8_gemv_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("FNX_W8_GEMV");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}
}  // namespace

namespace {
// Split-K factor of the tcgen05 W8 GEMM: with one token tile the launch has only N / 128 tiles,
// too few for 148 SMs.  Each tile streams its k-blocks one stage after another, so the cost is
// modelled as (rounds of tiles over the SMs) x (k-blocks per tile), the smaller split winning a
// tie; the fp32 partials are kept no larger than the weights (s * M * 4 <= K).
int w8_ksplit(int M, int K, int N) {
    const int KB = K / G_BK;
    const long long tiles = (long long)((M + G_BN - 1) / G_BN) * (N / G_BM);
    const long long nsm = num_sms();
    int best = 1;
    long long best_cost = (tiles + nsm - 1) / nsm * KB;
    for (int s = 2; s <= SPLITK_MAX; ++s) {
        if (KB % s || KB / s < 2 || (long long)s * M * 4 > K) continue;
        const long long cost = (tiles * s + nsm - 1) / nsm * (KB / s);
        if (cost < best_cost) {
            best = s;
            best_cost = cost;
        }
    }
    return best;
}

// Shapes the tcgen05 W8 GEMM takes (gemm_check's rules for one group of W8 weights).
bool w8_gemm_shape(int K, int N, int G) {
    return G >= 1 && K % G == 0 && K >= G_BK && K % G_BK == 0 && (K / G) % G_BK == 0 && N >= G_BM && N % G_BM == 0;
}

// The weight-streaming GEMV takes M <= 16 on the plain entry point.  With a workspace the
// split-K GEMM is faster from 9 tokens on (the GEMV's 16-token form: 31 us at K=2048, N=5120;
// the split GEMM: about 18 us), so there the GEMV keeps M <= 8, and M <= 16 only for shapes the
// GEMM does not take.
bool w8_gemv_route(int M, int K, int N, int G, bool split_path) {
    const bool ok = M >= 1 && M <= W8V_MAXM && G >= 1 && K % G == 0 && K % 64 == 0 && K <= 8192 && N % 4 == 0 &&
                    w8_gemv_enabled();
    if (!ok) return false;
    return !split_path || M <= 8 || !w8_gemm_shape(K, N, G);
}

inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

int w8a16_gemm_impl(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int G, void* ws,
                    size_t ws_bytes, bool split_path, void* stream) {
    // Both routes load x and the weights in 16-byte vectors, the scales as 8-byte pairs and
    // store y as 8-byte quads (the split-K reduce): reject misaligned pointers before either
    // route launches.
    if (M > 0 && (!aligned16(x) || !aligned16(w8t) || !aligned8(sc) || !aligned8(y))) return FNX_EALIGN;
    // small M: the weight-streaming GEMV (cluster K split); larger M: the tcgen05 GEMM
    if (w8_gemv_route(M, K, N, G, split_path)) {
        const int gs = K / G;
        cudaStream_t st = (cudaStream_t)stream;
        if (M == 1) return w8_gemv_launch_t<1, 8>(x, w8t, sc, y, M, K, N, gs, st);
        if (M == 2) return w8_gemv_launch_t<2, 8>(x, w8t, sc, y, M, K, N, gs, st);
        if (M <= 4) return w8_gemv_launch_t<4, 8>(x, w8t, sc, y, M, K, N, gs, st);
        if (M <= 8) return w8_gemv_launch_t<8, 8>(x, w8t, sc, y, M, K, N, gs, st);
        return w8_gemv_launch_t<16, FNX_W8V_CL16>(x, w8t, sc, y, M, K, N, gs, st);
    }
    GemmParams p{};
    p.act = (const bf16*)x; p.ld_act = K; p.w = w8t; p.scales = (const bf16*)sc; p.out = (bf16*)y; p.ld_out = N;
    p.act_rows = M;
    p.E = 1; p.M = M; p.K = K; p.Nw = N; p.gs = G > 0 ? K / G : 0; p.m_tiles = N / G_BM;
    if (G < 1 || K % G) return FNX_EARG;
    const int rc = gemm_check(GEMM_W8, EPI_PLAIN, p);
    if (rc) return rc;
    if (N % 8) return FNX_ESHAPE;
    if (M == 0) return FNX_OK;
    if (ws) {
        const int s = w8_ksplit(M, K, N);
        if (s > 1) {
            if (!aligned16(ws)) return FNX_EALIGN;
            if (ws_bytes < (size_t)s * M * N * sizeof(float)) return FNX_EWORKSPACE;
            p.ksplit = s;
            p.partial = (float*)ws;
            const int r = gemm_launch(GEMM_W8, EPI_PLAIN, p, (cudaStream_t)stream);
            if (r) return r;
            const long long n4 = (long long)M * (N / 4);
            const dim3 grid(grid_for(n4, 256));
            cudaStream_t st = (cudaStream_t)stream;
            if (s <= 2) splitk_reduce_kernel<2><<<grid, 256, 0, st>>>(p.partial, p.out, p.ld_out, M, N, s);
            else if (s <= 4) splitk_reduce_kernel<4><<<grid, 256, 0, st>>>(p.partial, p.out, p.ld_out, M, N, s);
            else if (s <= 8) splitk_reduce_kernel<8><<<grid, 256, 0, st>>>(p.partial, p.out, p.ld_out, M, N, s);
            else splitk_reduce_kernel<SPLITK_MAX><<<grid, 256, 0, st>>>(p.partial, p.out, p.ld_out, M, N, s);
            return launch_rc();
        }
    }
    return gemm_launch(GEMM_W8, EPI_PLAIN, p, (cudaStream_t)stream);
}
}  // namespace

FNX_API int fnx_w8a16_gemm(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int G,
                           void* stream) {
    return w8a16_gemm_impl(x, w8t, sc, y, M, K, N, G, nullptr, 0, false, stream);
}

FNX_API size_t fnx_w8a16_gemm_workspace(int M, int K, int N, int G) {
    if (M < 1 || !w8_gemm_shape(K, N, G) || w8_gemv_route(M, K, N, G, true)) return 0;
    const int s = w8_ksplit(M, K, N);
    return s > 1 ? (size_t)s * M * N * sizeof(float) : 0;
}

FNX_API int fnx_w8a16_gemm_ws(const void* x, const void* w8t, const void* sc, void* y, int M, int K, int N, int G,
                              void* ws, size_t ws_bytes, void* stream) {
    return w8a16_gemm_impl(x, w8t, sc, y, M, K, N, G, ws, ws_bytes, true, stream);
}

namespace {
template <int BN>
int gemm_bf16_tma_launch_t(const void* x, long long ld_x, const void* w, void* y, long long ld_y, int M, int K, int N,
                           cudaStream_t st) {
    const size_t smem = gemm_bf16_tma_smem<BN>();
    static bool configured[FNX_MAX_DEVICES] = {};
    const int dev = current_device();
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(gemm_bf16_tma_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return FNX_ELAUNCH;
        configured[dev] = true;
    }
    TGemmParams p{};
    int rc = make_map_2d(&p.ta, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (unsigned long long)K, (unsigned long long)M,
                         T_BK, T_BM, CU_TENSOR_MAP_SWIZZLE_128B, (unsigned long long)ld_x * 2);
    if (rc) return rc;
    rc = make_map_2d(&p.tb, w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (unsigned long long)K, (unsigned long long)N, T_BK,
                     BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    p.out = (bf16*)y; p.ld_out = ld_y; p.M = M; p.N = N; p.K = K;
    const int tiles = ((M + T_BM - 1) / T_BM) * ((N + BN - 1) / BN);
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gemm_bf16_tma_kernel<BN><<<grid, T_THREADS, smem, st>>>(p);
    return launch_rc();
}
}  // namespace

// y [M, N] (row stride ld_y) = x [M, K] (row stride ld_x) @ w [N, K]^T, bf16 in and out, fp32
// accumulation: the TMA-fed tcgen05 GEMM (kernels_gemm_bf16.cuh); 160-feature tiles when N is a
// multiple of 160 (the router's 640 rows: 128 tiles at T = 4096, one wave), 128 otherwise.
FNX_API int fnx_bf16_gemm_nt(const void* x, long long ld_x, const void* w, void* y, long long ld_y, int M, int K, int N,
                             void* stream) {
    if (M < 0 || K < T_BK || K % T_BK || N < 1 || ld_x < K || ld_y < N) return FNX_EARG;
    if (!aligned16(x) || !aligned16(w) || ld_x % 8) return FNX_EALIGN;
    if (M == 0) return FNX_OK;
    cudaStream_t st = (cudaStream_t)stream;
    if (M < T_BM || N < 128) {
        // fewer rows than one TMA box: the single-CTA kernel (weights by TMA, the few token rows
        // gathered by its loader warps)
        GemmParams p{};
        p.act = (const bf16*)x; p.ld_act = ld_x; p.w = w; p.out = (bf16*)y; p.ld_out = ld_y;
        p.act_rows = M;
        p.E = 1; p.M = M; p.K = K; p.Nw = N; p.gs = K; p.m_tiles = (N + G_BM - 1) / G_BM;
        const int rc = gemm_check(GEMM_BF16, EPI_PLAIN, p);
        if (rc) return rc;
        return gemm_launch(GEMM_BF16, EPI_PLAIN, p, st);
    }
    if (N % 160 == 0) return gemm_bf16_tma_launch_t<160>(x, ld_x, w, y, ld_y, M, K, N, st);
    return gemm_bf16_tma_launch_t<128>(x, ld_x, w, y, ld_y, M, K, N, st);
}

// ======================================================================== load-time repack
FNX_API int fnx_repack_v2o(const void* v2o, int E, int N, int K, int expert_major, void* w4, void* stream) {
    if (!v2o || !w4 || E < 1 || N < 8 || N % 8 || K < 128 || K % 128) return FNX_EARG;
    const long long total = (long long)E * K * (N / 8);
    repack_v2o_kernel<<<grid_for(total, 256), 256, 0, (cudaStream_t)stream>>>((const uint8_t*)v2o, E, N, K,
                                                                             expert_major ? 1 : 0, (int32_t*)w4);
    return launch_rc();
}

FNX_API size_t fnx_w4_tiles_bytes(int E, int K, int Nw) {
    if (E < 1 || K < 64 || K % 64 || Nw < 128 || Nw % 128) return 0;
    return (size_t)E * (Nw / 128) * (K / 64) * TILE_BLOCK_BYTES;
}

FNX_API int fnx_repack_w4_tiles(const void* w4, const void* scales, void* tiles, int E, int K, int Nw, int gs,
                                int swiglu, void* stream) {
    if (E < 1 || K < 64 || K % 64 || Nw < 128 || Nw % 128 || gs < 64 || gs % 64 || K % gs || (swiglu != 0 && swiglu != 1))
        return FNX_EARG;
    if (!aligned16(tiles)) return FNX_EALIGN;
    const long long words = (long long)fnx_w4_tiles_bytes(E, K, Nw) / 4;
    repack_w4_tiles_kernel<<<grid_for(words, 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint32_t*)w4, (const bf16*)scales, (uint32_t*)tiles, E, K, Nw, gs, swiglu);
    return launch_rc();
}

// ======================================================================== decode layer
namespace {
struct DecodeLayout {
    size_t logits, wf, idx, part, part2, act, act_sh, yd, sh, counters, total;
    int ks1, ks2, R;
    // streaming kernel: the launch counter at offset 0, tagged words, the exit ticket last
    // (`counters`: the part that must be zero before the first call)
    size_t tlog, tpart, tpart2, tyd, tsh;
};

// FNX_DECODE_V1=1 selects the first decode kernel (decode_fused_kernel: one bulk-copy chunk per
// item, routing by one CTA) in place of the streaming one, for comparisons.
bool decode_v1() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("FNX_DECODE_V1");
        v = (e && e[0] == '1') ? 1 : 0;
    }
    return v == 1;
}

int env_int(const char* name, int dflt) {
    const char* e = getenv(name);
    return e && *e ? atoi(e) : dflt;
}

DecodeLayout decode_layout(int M, int H, int I, int E, int k) {
    DecodeLayout L{};
    L.R = E + 1;
    const int mt = I / 64, kb = H / 64;
    const int slots = 2 * num_sms();
    // K splits: item i of a group takes k-blocks [i*kb/ks, (i+1)*kb/ks).  The router rows and the
    // shared gate/up (both before the routing is known) together fill about one item per
    // resident CTA.
    const int rows = decode_v1() ? DEC_ROWS : d2_router_rows(H);
    const int rb = (L.R + rows - 1) / rows;
    L.ks1 = 1;
    while (rb + M * mt * (L.ks1 + 1) <= slots && kb / (L.ks1 + 1) >= 2) L.ks1 += 1;
    if (!decode_v1()) {
        // streaming kernel: the routed gate/up is split into at most one item per resident CTA
        // (no CTA holds two items of the critical gate/up phase), never finer than a down item
        const int cap = kb / (I / 64) >= 1 ? kb / (I / 64) : 1;
        const long long groups = (long long)M * k * mt;
        L.ks2 = (int)(slots / groups);                 // about one gate/up item per resident CTA
        if (L.ks2 < 2 && M <= 4) L.ks2 = 2;            // 2 to 4 tokens: halves (measured 46.7 against 50.0 us at M = 4)
        if (L.ks2 > cap) L.ks2 = cap;
        if (L.ks2 < 1) L.ks2 = 1;
        // the shared gate/up does not wait for the routing: a few long items per feature tile
        // leave the CTAs to the routed items once the routing lands (measured, ks1 = 2M:
        // M = 1 21.1 against 22.1 us with the slot rule's 15; M = 4 45.5 against 46.4 with its 4)
        if (M <= 4 && kb / (2 * M) >= 2) L.ks1 = 2 * M;
        const int e1 = env_int("FNX_DEC_KS1", 0), e2 = env_int("FNX_DEC_KS2", 0);
        if (e1 >= 1 && kb / e1 >= 1) L.ks1 = e1;
        if (e2 >= 1 && kb / e2 >= 1) L.ks2 = e2;
        size_t off = 0;
        auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
        take(sizeof(unsigned));                                  // launch counter, offset 0
        L.tlog = take((size_t)M * L.R * 8);
        L.tpart = take((size_t)M * mt * L.ks1 * 128 * 8);
        L.tpart2 = take((size_t)M * k * mt * L.ks2 * 128 * 8);
        L.tyd = take((size_t)M * k * (H / 2) * 8);
        L.tsh = take((size_t)M * (H / 2) * 8);
        L.counters = take(sizeof(unsigned));                     // exit ticket
        L.total = off;
        return L;
    }
    // one copy per item: the routed gate/up split minimises (waves of items) x (k-blocks per
    // item + a fixed per-item cost, measured at about 16 k-blocks' worth: the copy latency, the
    // partial sums and the group ticket)
    L.ks2 = 1;
    double best = 1e30;
    for (int ks = 1; ks <= 32 && kb / ks >= 2; ++ks) {
        const long long items = (long long)M * k * mt * ks;
        const double cost = (double)((items + slots - 1) / slots) * ((double)kb / ks + 16.0);
        if (cost < best - 1e-9) { best = cost; L.ks2 = ks; }
    }
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
    L.logits = take((size_t)M * L.R * 2);
    L.wf = take((size_t)M * k * 4);
    L.idx = take((size_t)M * k * 4);
    L.part = take((size_t)M * mt * L.ks1 * 128 * 4);
    L.part2 = take((size_t)M * k * mt * L.ks2 * 128 * 4);
    L.act = take((size_t)M * k * I * 2);
    L.act_sh = take((size_t)M * I * 2);
    L.yd = take((size_t)M * k * H * 2);
    L.sh = take((size_t)M * H * 2);
    L.counters = take(decode_counters(M, H, I, k) * 4);
    L.total = off;
    return L;
}
}  // namespace

FNX_API size_t fnx_moe_decode_workspace(int M, int H, int I, int E, int k) {
    if (M < 1 || M > DEC_MAX_M || H < 256 || I < 128 || E < 1 || k < 1) return 0;
    return decode_layout(M, H, I, E, k).total;
}

// router: bf16 [E+1, H] (rows 0..E-1 router, row E shared-expert gate); expert weights as
// the tile blocks of fnx_repack_w4_tiles (gate/up in SwiGLU row order, down plain).
// workspace must be zero-filled before its first use; every completed call leaves its
// tickets at zero again.
namespace {
int decode_w4_impl(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                   const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H, int I,
                   int E, int k, void* workspace, size_t ws_bytes, int logits_ready, void* stream);
}

FNX_API int fnx_moe_decode_w4(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                              const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H,
                              int I, int E, int k, void* workspace, size_t ws_bytes, void* stream) {
    return decode_w4_impl(x, router, gu, dn, sh_gu, sh_dn, bias, out, w_out, idx_out, M, H, I, E, k, workspace,
                          ws_bytes, 0, stream);
}

// fnx_moe_decode_w4 whose router logits were already written into the workspace by
// fnx_hc_mix_router (flags bit 0): the launch skips its router items.
FNX_API int fnx_moe_decode_w4_ex(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                                 const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M,
                                 int H, int I, int E, int k, void* workspace, size_t ws_bytes, int flags,
                                 void* stream) {
    if (flags & ~1) return FNX_EARG;
    if ((flags & 1) && decode_v1()) return FNX_EARG;            // the first decode kernel has no such mode
    return decode_w4_impl(x, router, gu, dn, sh_gu, sh_dn, bias, out, w_out, idx_out, M, H, I, E, k, workspace,
                          ws_bytes, flags & 1, stream);
}

// The hyper-connection mix of the decode rows with the router GEMV fused behind it: y bf16 [M, H]
// = the branch mix of x (hn) and l bf16 [M, HC*H], and the router logits of y written, tagged,
// into the decode workspace for the next fnx_moe_decode_w4_ex(..., flags = 1) on it.
FNX_API int fnx_hc_mix_router(const void* x, const void* l, void* y, const void* router, void* workspace,
                              size_t ws_bytes, int M, int H, int I, int E, int k, int HC, void* stream) {
    if (M < 1 || M > DEC_MAX_M || E < 1 || E > ROUTE_MAX_E || k < 1 || k > 32 || k > E || HC < 1 || HC > 64 ||
        !x || !l || !y || !router)
        return FNX_EARG;
    if (H < 256 || I < 128 || H % 256 || I % 128 || H > DEC_MAX_K || I > DEC_MAX_K || E > DEC_MAX_E)
        return FNX_ESHAPE;
    if (decode_v1()) return FNX_EARG;
    const DecodeLayout L = decode_layout(M, H, I, E, k);
    if (!workspace || ws_bytes < L.total) return FNX_EWORKSPACE;
    if (!aligned16(router) || !aligned16(workspace)) return FNX_EALIGN;
    uint8_t* ws = (uint8_t*)workspace;
    StreamParams q{};
    q.router = (const bf16*)router;
    q.epoch = (unsigned*)ws;
    q.tlog = (tword*)(ws + L.tlog);
    q.M = M; q.H = H; q.I = I; q.E = E; q.k = k; q.R = L.R;
    const int rows = d2_router_rows(H);
    const size_t smem = (size_t)(M + rows) * H * 2;
    static bool set[FNX_MAX_DEVICES] = {};
    const int dev = current_device();
    if (!set[dev]) {
        if (cudaFuncSetAttribute(hc_mix_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (DEC_MAX_M + D2_MAX_ROWS) * DEC_MAX_K * 2) != cudaSuccess)
            return FNX_ELAUNCH;
        set[dev] = true;
    }
    const int grid = ((L.R + rows - 1) / rows + HC_MIX_CLUSTER - 1) / HC_MIX_CLUSTER * HC_MIX_CLUSTER;
    hc_mix_router_kernel<<<grid, D2_CTHREADS, smem, (cudaStream_t)stream>>>((const bf16*)x, (const bf16*)l, HC,
                                                                           (bf16*)y, q);
    return launch_rc();
}

namespace {
int decode_w4_impl(const void* x, const void* router, const void* gu, const void* dn, const void* sh_gu,
                   const void* sh_dn, const void* bias, void* out, void* w_out, void* idx_out, int M, int H, int I,
                   int E, int k, void* workspace, size_t ws_bytes, int logits_ready, void* stream) {
    if (M < 1 || M > DEC_MAX_M || E < 1 || E > ROUTE_MAX_E || k < 1 || k > 32 || k > E) return FNX_EARG;
    if (H < 256 || I < 128 || H % 256 || I % 128 || H > DEC_MAX_K || I > DEC_MAX_K || E > DEC_MAX_E)
        return FNX_ESHAPE;
    const DecodeLayout L = decode_layout(M, H, I, E, k);
    if (!workspace || ws_bytes < L.total) return FNX_EWORKSPACE;
    if (!aligned16(x) || !aligned16(router) || !aligned16(gu) || !aligned16(dn) || !aligned16(sh_gu) ||
        !aligned16(sh_dn) || !aligned16(workspace) || (reinterpret_cast<uintptr_t>(out) & 3u))
        return FNX_EALIGN;
    uint8_t* ws = (uint8_t*)workspace;
    if (!decode_v1()) {
        StreamParams q{};
        q.x = (const bf16*)x; q.router = (const bf16*)router;
        q.gu_tw = (const uint32_t*)gu; q.dn_tw = (const uint32_t*)dn;
        q.sh_gu_tw = (const uint32_t*)sh_gu; q.sh_dn_tw = (const uint32_t*)sh_dn;
        q.out = (bf16*)out; q.w_out = (bf16*)w_out; q.idx_out = (int64_t*)idx_out; q.bias = (const float*)bias;
        q.epoch = (unsigned*)ws;
        q.exit = (unsigned*)(ws + L.counters);
        q.tlog = (tword*)(ws + L.tlog); q.tpart = (tword*)(ws + L.tpart); q.tpart2 = (tword*)(ws + L.tpart2);
        q.tyd = (tword*)(ws + L.tyd); q.tsh = (tword*)(ws + L.tsh);
        q.M = M; q.H = H; q.I = I; q.E = E; q.k = k; q.R = L.R; q.ks1 = L.ks1; q.ks2 = L.ks2;
        q.logits_ready = logits_ready;
        // one cooperative launch of every block that fits at once (work items wait for earlier
        // items of other blocks, so all blocks must be resident)
        static int grid2_of[FNX_MAX_DEVICES] = {};
        int& grid2 = grid2_of[current_device()];
        if (!grid2) {
            if (cudaFuncSetAttribute(decode_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, D2_SMEM))
                return FNX_ELAUNCH;
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_stream_kernel, D2_THREADS, D2_SMEM) ||
                per_sm < 1)
                return FNX_ELAUNCH;
            grid2 = per_sm * num_sms();
        }
        // programmatic dependent launch: the blocks may start while the kernel before this one
        // on the stream finishes (their copy warps prefetch the first weights into L2, then all
        // warps wait for it); FNX_DECODE_PDL=0 launches after it as usual
        static const bool pdl = env_int("FNX_DECODE_PDL", 1) != 0;
        cudaLaunchAttribute attr2[2];
        attr2[0].id = cudaLaunchAttributeCooperative;
        attr2[0].val.cooperative = 1;
        attr2[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr2[1].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg2 = {};
        cfg2.gridDim = dim3(grid2);
        cfg2.blockDim = dim3(D2_THREADS);
        cfg2.dynamicSmemBytes = D2_SMEM;
        cfg2.stream = (cudaStream_t)stream;
        cfg2.attrs = attr2;
        cfg2.numAttrs = pdl ? 2 : 1;
        if (cudaLaunchKernelEx(&cfg2, decode_stream_kernel, q) != cudaSuccess) return FNX_ELAUNCH;
        return launch_rc();
    }
    DecodeParams p{};
    p.x = (const bf16*)x; p.router = (const bf16*)router;
    p.gu_tw = (const uint32_t*)gu; p.dn_tw = (const uint32_t*)dn;
    p.sh_gu_tw = (const uint32_t*)sh_gu; p.sh_dn_tw = (const uint32_t*)sh_dn;
    p.out = (bf16*)out; p.w_out = (bf16*)w_out; p.idx_out = (int64_t*)idx_out; p.bias = (const float*)bias;
    p.logits = (bf16*)(ws + L.logits); p.wf = (float*)(ws + L.wf); p.idx = (int32_t*)(ws + L.idx);
    p.part = (float*)(ws + L.part); p.part2 = (float*)(ws + L.part2);
    p.act = (bf16*)(ws + L.act); p.act_sh = (bf16*)(ws + L.act_sh); p.yd = (bf16*)(ws + L.yd); p.sh = (bf16*)(ws + L.sh);
    p.counters = (unsigned*)(ws + L.counters);
    p.M = M; p.H = H; p.I = I; p.E = E; p.k = k; p.R = L.R; p.ks1 = L.ks1; p.ks2 = L.ks2;
    // one cooperative launch of every block that fits at once (work items wait for earlier
    // items of other blocks, so all blocks must be resident)
    static int grid_of[FNX_MAX_DEVICES] = {};
    int& grid = grid_of[current_device()];
    if (!grid) {
        if (cudaFuncSetAttribute(decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM))
            return FNX_ELAUNCH;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_fused_kernel, DEC_THREADS, DEC_SMEM) ||
            per_sm < 1)
            return FNX_ELAUNCH;
        grid = per_sm * num_sms();
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DEC_THREADS);
    cfg.dynamicSmemBytes = DEC_SMEM;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, decode_fused_kernel, p) != cudaSuccess) return FNX_ELAUNCH;
    return launch_rc();
}
}  // namespace

// ======================================================================== legacy W4 GEMV
FNX_API int fnx_w4gemv_launch(void* p4, void* s4t, void* xe, void* xo, void* y, void* dbg, void* ids, int N, int K,
                              int nExp, int nblk, int lay, void* stream) {
    (void)dbg;
    (void)nblk;
    if (N < 1 || K < 128 || K % 128 || nExp < 1 || (lay != 1 && lay != 2)) return FNX_EARG;
    if (!aligned16(p4)) return FNX_EALIGN;
    W4GemvLayer L{(const uint8_t*)p4, (const __half*)s4t, (const float*)xe, (const float*)(xo ? xo : xe), (float*)y};
    const int blocks = (nExp * N + 7) / 8;
    if (lay == 1) w4gemv_kernel<1><<<blocks, 256, 0, (cudaStream_t)stream>>>(L, (const int32_t*)ids, N, K, nExp);
    else w4gemv_kernel<2><<<blocks, 256, 0, (cudaStream_t)stream>>>(L, (const int32_t*)ids, N, K, nExp);
    return launch_rc();
}

FNX_API int fnx_w4gemv_launch_layers(void** p4, void** s4t, void** x, void** y, int nL, int N, int K, int nExp, int nblk,
                                     int lay, void* dbg, void* stream) {
    (void)dbg;
    (void)nblk;
    if (nL < 1 || nL > W4GEMV_MAX_LAYERS || N < 1 || K < 128 || K % 128 || nExp < 1 || (lay != 1 && lay != 2))
        return FNX_EARG;
    W4GemvLayers Ls{};
    for (int i = 0; i < nL; ++i) {
        if (!aligned16(p4[i])) return FNX_EALIGN;
        Ls.L[i] = W4GemvLayer{(const uint8_t*)p4[i], (const __half*)s4t[i], (const float*)x[i],
                              (const float*)x[i], (float*)y[i]};
    }
    dim3 grid((nExp * N + 7) / 8, nL);
    if (lay == 1) w4gemv_layers_kernel<1><<<grid, 256, 0, (cudaStream_t)stream>>>(Ls, N, K, nExp);
    else w4gemv_layers_kernel<2><<<grid, 256, 0, (cudaStream_t)stream>>>(Ls, N, K, nExp);
    return launch_rc();
}

// ======================================================================== decode layer, no allocation
// Some callers cannot allocate device memory: a plugin host or FFI binding that hands the
// library only its input and output buffers (all device memory belongs to the host's own
// pool and no allocator is exposed), or a serving process that forbids device allocation
// once it has started.  For them the decode layer runs on a fixed scratch area compiled
// into the library: FNX_NOALLOC_SCRATCH_BYTES of device memory that every GPU which loads
// the library keeps until the process exits.
#define FNX_NOALLOC_SCRATCH_BYTES (4u << 20)

static __device__ __align__(256) unsigned char g_fnx_noalloc_scratch[FNX_NOALLOC_SCRATCH_BYTES];

namespace {
// Device address of the scratch array for the current device.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per device (with
// that device current) and cached.
// The cache has one slot per device, as the library's other per-device launch caches; host
// threads that make their first calls at the same time store the same address (atomically).
void* noalloc_scratch(int* rc) {
    static void* addr[FNX_MAX_DEVICES] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= FNX_MAX_DEVICES) {
        *rc = FNX_ELAUNCH;
        return nullptr;
    }
    void* cached = __atomic_load_n(&addr[dev], __ATOMIC_ACQUIRE);
    if (!cached) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_fnx_noalloc_scratch) != cudaSuccess || p == nullptr) {
            *rc = FNX_ELAUNCH;
            return nullptr;
        }
        __atomic_store_n(&addr[dev], p, __ATOMIC_RELEASE);
        cached = p;
    }
    return cached;
}
}  // namespace

// fnx_moe_decode_w4 without a caller-provided workspace: the scratch is the library's
// static array.  The first call on each device looks its address up, so make that first
// call before any stream capture.  Shapes whose workspace (fnx_moe_decode_workspace)
// exceeds FNX_NOALLOC_SCRATCH_BYTES are rejected with FNX_EWORKSPACE.  The array is shared
// by every call on a device and keeps the last call's contents; the tickets that must start
// at zero are cleared at the start of each call.  Calls that overlap on the GPU (other
// streams, other threads) race on the array.
FNX_API int fnx_moe_decode_w4_noalloc(const void* x, const void* router, const void* gu, const void* dn,
                                      const void* sh_gu, const void* sh_dn, const void* bias, void* out, void* w_out,
                                      void* idx_out, int M, int H, int I, int E, int k, void* stream) {
    if (M < 1 || M > DEC_MAX_M || E < 1 || E > ROUTE_MAX_E || k < 1 || k > 32 || k > E) return FNX_EARG;
    if (H < 256 || I < 128 || H % 256 || I % 128) return FNX_ESHAPE;
    if (H > DEC_MAX_K || I > DEC_MAX_K) {
        const DecodeLayout L0 = decode_layout(M, H, I, E, k);
        return L0.total > FNX_NOALLOC_SCRATCH_BYTES ? FNX_EWORKSPACE : FNX_ESHAPE;
    }
    const DecodeLayout L = decode_layout(M, H, I, E, k);
    if (L.total > FNX_NOALLOC_SCRATCH_BYTES) return FNX_EWORKSPACE;
    int rc = FNX_OK;
    uint8_t* ws = (uint8_t*)noalloc_scratch(&rc);
    if (!ws) return rc;
    if (cudaMemsetAsync(ws + L.counters, 0, L.total - L.counters, (cudaStream_t)stream) != cudaSuccess)
        return FNX_ELAUNCH;
    return fnx_moe_decode_w4(x, router, gu, dn, sh_gu, sh_dn, bias, out, w_out, idx_out, M, H, I, E, k, ws,
                             FNX_NOALLOC_SCRATCH_BYTES, stream);
}
