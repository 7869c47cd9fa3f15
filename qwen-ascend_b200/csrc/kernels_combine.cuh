// Combine-side kernels: slot-order weighted reduce, sigmoid-gated shared merge, the
// Cartesian-diagonal epilogue and the expert gather copy.  All are HBM-bound
// elementwise / byte work: 16-byte vector accesses, grid sized in SM multiples.
#pragma once
#include "fnx_common.cuh"

namespace fnx {

// ---------------------------------------------------------------- weighted reduce
// mode 1: out[t,c] = bf16( sum_{g<groups} fp32(bf16(in[t*groups+g, c] * w[t*groups+g])) )
// mode 2: same with the row taken from inverse[t*groups+g]
// mode 0: out[t,c] = bf16( 0.25 * sum_g fp32(bf16(in[t*groups+g, c] * wb[(t*groups+g)*width + c])) )
// Sums run sequentially in slot order in fp32, exactly the rounding sequence of
// kernels/reduce/reduce.cpp:39-54 in the reference.
template <int MODE, bool VEC>
__global__ void __launch_bounds__(256) weighted_reduce_kernel(const bf16* __restrict__ in,
                                                              const void* __restrict__ w,
                                                              const int64_t* __restrict__ inverse,
                                                              bf16* __restrict__ out, int batch, int groups,
                                                              int width, long long row_stride) {
    const int per_row = VEC ? width / 8 : width;
    const long long total = (long long)batch * per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        const int c = (int)(i % per_row) * (VEC ? 8 : 1);
        float acc[VEC ? 8 : 1];
#pragma unroll
        for (int j = 0; j < (VEC ? 8 : 1); ++j) acc[j] = 0.f;
        for (int g = 0; g < groups; ++g) {
            const long long slot = (long long)t * groups + g;
            const long long row = MODE == 2 ? inverse[slot] : slot;
            if (MODE == 2 && (row < 0 || row >= (long long)batch * groups)) {   // not a permutation entry
                fnx_flag_error(FNX_DEVERR_BADID);
                continue;
            }
            const bf16* src = in + row * row_stride + c;
            if (VEC) {
                uint4 v = ld_nc_v4(src);
                uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                float wv[8];
                if (MODE == 0) {
                    uint4 wr = ld_nc_v4(reinterpret_cast<const bf16*>(w) + slot * width + c);
                    uint32_t ww[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) { wv[2 * j] = bf_lo(ww[j]); wv[2 * j + 1] = bf_hi(ww[j]); }
                } else {
                    const float s = reinterpret_cast<const float*>(w)[slot];
#pragma unroll
                    for (int j = 0; j < 8; ++j) wv[j] = s;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[2 * j] = __fadd_rn(acc[2 * j], round_bf(__fmul_rn(bf_lo(vv[j]), wv[2 * j])));
                    acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], round_bf(__fmul_rn(bf_hi(vv[j]), wv[2 * j + 1])));
                }
            } else {
                const float x = bf2f(src[0]);
                const float s = MODE == 0 ? bf2f(reinterpret_cast<const bf16*>(w)[slot * width + c])
                                          : reinterpret_cast<const float*>(w)[slot];
                acc[0] = __fadd_rn(acc[0], round_bf(__fmul_rn(x, s)));
            }
        }
        bf16* dst = out + (long long)t * width + c;
        if (VEC) {
            uint4 o;
            const float m = MODE == 0 ? 0.25f : 1.0f;
            o.x = pack_bf2(__fmul_rn(acc[0], m), __fmul_rn(acc[1], m));
            o.y = pack_bf2(__fmul_rn(acc[2], m), __fmul_rn(acc[3], m));
            o.z = pack_bf2(__fmul_rn(acc[4], m), __fmul_rn(acc[5], m));
            o.w = pack_bf2(__fmul_rn(acc[6], m), __fmul_rn(acc[7], m));
            *reinterpret_cast<uint4*>(dst) = o;
        } else {
            dst[0] = f2bf(MODE == 0 ? __fmul_rn(acc[0], 0.25f) : acc[0]);
        }
    }
}

// ---------------------------------------------------------------- shared merge
// out[t,c] = bf16( e + bf16( s * bf16(sigmoid(g[t])) ) )   (kernels/post_ops/post_ops.cpp:72-90)
template <bool VEC>
__global__ void __launch_bounds__(256) moe_merge_kernel(const bf16* __restrict__ e, const bf16* __restrict__ s,
                                                        const bf16* __restrict__ g, bf16* __restrict__ out,
                                                        int batch, int width) {
    const int per_row = VEC ? width / 8 : width;
    const long long total = (long long)batch * per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        const int c = (int)(i % per_row) * (VEC ? 8 : 1);
        const float sg = round_bf(sigmoid_f32(bf2f(g[t])));
        const long long off = (long long)t * width + c;
        if (VEC) {
            uint4 ev = ld_nc_v4(e + off), sv = ld_nc_v4(s + off);
            uint32_t ea[4] = {ev.x, ev.y, ev.z, ev.w}, sa[4] = {sv.x, sv.y, sv.z, sv.w}, oa[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float lo = __fadd_rn(bf_lo(ea[j]), round_bf(__fmul_rn(bf_lo(sa[j]), sg)));
                const float hi = __fadd_rn(bf_hi(ea[j]), round_bf(__fmul_rn(bf_hi(sa[j]), sg)));
                oa[j] = pack_bf2(lo, hi);
            }
            *reinterpret_cast<uint4*>(out + off) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
        } else {
            out[off] = f2bf(__fadd_rn(bf2f(e[off]), round_bf(__fmul_rn(bf2f(s[off]), sg))));
        }
    }
}

// ---------------------------------------------------------------- fused combine
// out[t,c] = bf16( bf16(sum_j fp32(bf16(w[t*k+j] * yd[row(t,j), c]))) + bf16(sh[t,c] * bf16(sigmoid(g[t]))) )
// row(t,j) = inverse[t*k+j] (or t*k+j); g[t] = gate[t * gate_ld].  The reference's
// weighted_reduce mode 2 followed by post_ops.moe_merge (fnx/engine.py:1844-1853),
// with the same roundings, in one pass over yd (the kernel follows the inject helpers).

// inject of 8 columns [c, c+8) of token t for every branch: y (bf16 pairs) * inj[t, b], rounded
// to bf16, added to hyper in fp32 and rounded (kernels/inject/inject.cpp:14-20).
FNX_DEV void inject_vec(const bf16* hyper, const bf16* inj, bf16* out_hyper, long long t, int c, int H, int HC,
                        const uint32_t (&ya)[4]) {
    for (int b = 0; b < HC; ++b) {
        const float gv = bf2f(inj[t * HC + b]);
        const long long o = (t * HC + b) * (long long)H + c;
        const uint4 hv = ld_nc_v4(hyper + o);
        const uint32_t ha[4] = {hv.x, hv.y, hv.z, hv.w};
        uint32_t oa[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float lo = __fadd_rn(bf_lo(ha[q]), round_bf(__fmul_rn(bf_lo(ya[q]), gv)));
            const float hi = __fadd_rn(bf_hi(ha[q]), round_bf(__fmul_rn(bf_hi(ya[q]), gv)));
            oa[q] = pack_bf2(lo, hi);
        }
        *reinterpret_cast<uint4*>(out_hyper + o) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
    }
}

// Standalone inject: out [B, HC*H] from hyper [B, HC*H], y [B, H], inj [B, HC] (H % 8 == 0).
__global__ void __launch_bounds__(256) inject_kernel(const bf16* __restrict__ hyper, const bf16* __restrict__ y,
                                                     const bf16* __restrict__ inj, bf16* __restrict__ out, int B,
                                                     int H, int HC) {
    const int per_row = H / 8;
    const long long total = (long long)B * per_row;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / per_row;
        const int c = (int)(i % per_row) * 8;
        const uint4 yv = ld_nc_v4(y + t * H + c);
        const uint32_t ya[4] = {yv.x, yv.y, yv.z, yv.w};
        inject_vec(hyper, inj, out, t, c, H, HC, ya);
    }
}

// The combine.  With `hyper` (the fused inject of fnx/engine.py:859-877): out_hyper[t, b*H + c] =
// bf16(hyper[t, b*H + c] + bf16(y[t, c] * inj[t, b])) for the HC branches, y the combined
// output (also written to `out` when it is not null).  Needs the vector path (H % 8, k <= 16).
// Vector path: a thread owns 8 columns of one token.  When a token's columns fill whole warps
// (H % 256 == 0) lane q < k of the warp loads slot q's row index and weight once and the warp
// shares them by shuffles as they are used; the k rows are requested FNX_COMBINE_G at a time
// before the in-order sums (T*k < 2^31 rows, checked by the host).
#ifndef FNX_COMBINE_G
#define FNX_COMBINE_G 4
#endif
#ifndef FNX_COMBINE_MINB
#define FNX_COMBINE_MINB 4
#endif
template <bool VEC>
__global__ void __launch_bounds__(256, FNX_COMBINE_MINB) moe_combine_kernel(const bf16* __restrict__ yd, const float* __restrict__ w,
                                                          const int64_t* __restrict__ inverse,
                                                          const bf16* __restrict__ sh, const bf16* __restrict__ gate,
                                                          long long gate_ld, bf16* __restrict__ out, int T, int k,
                                                          int H, const bf16* __restrict__ hyper = nullptr,
                                                          const bf16* __restrict__ inj = nullptr,
                                                          bf16* __restrict__ out_hyper = nullptr, int HC = 0) {
    constexpr int G = FNX_COMBINE_G;
    const int per_row = VEC ? H / 8 : H;
    const long long total = (long long)T * per_row;
    const bool warp_token = VEC && (per_row & 31) == 0;      // a warp's items share one token
    const long long nrows = (long long)T * k;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        const int c = (int)(i % per_row) * (VEC ? 8 : 1);
        float acc[VEC ? 8 : 1];
#pragma unroll
        for (int j = 0; j < (VEC ? 8 : 1); ++j) acc[j] = 0.f;
        if (VEC && k <= 16) {
            // warp_token: lane q < k holds slot q's row and weight; otherwise each thread reads them
            int my_r = -1;
            float my_w = 0.f;
            if (warp_token) {
                const int lane = threadIdx.x & 31;
                if (lane < k) {
                    const long long slot = (long long)t * k + lane;
                    const long long r = inverse ? inverse[slot] : slot;
                    my_r = (r >= 0 && r < nrows) ? (int)r : -1;
                    my_w = w[slot];
                }
            }
            const long long off = (long long)t * H + c;
            const uint4 sv = ld_nc_v4(sh + off);
            const float g = bf2f(gate[(long long)t * gate_ld]);
#pragma unroll
            for (int j0 = 0; j0 < 16; j0 += G) {
                if (j0 >= k) break;
                int r[G];
                float sw[G];
                uint4 v[G];
#pragma unroll
                for (int q = 0; q < G; ++q) {
                    const int j = j0 + q;
                    r[q] = -1;
                    sw[q] = 0.f;
                    if (warp_token) {
                        r[q] = __shfl_sync(0xffffffffu, my_r, j & 31);
                        sw[q] = __shfl_sync(0xffffffffu, my_w, j & 31);
                    } else if (j < k) {
                        const long long slot = (long long)t * k + j;
                        const long long rr = inverse ? inverse[slot] : slot;
                        r[q] = (rr >= 0 && rr < nrows) ? (int)rr : -1;
                        sw[q] = w[slot];
                    }
                }
#pragma unroll
                for (int q = 0; q < G; ++q) {
                    v[q] = make_uint4(0, 0, 0, 0);
                    if (j0 + q < k && r[q] >= 0) v[q] = ld_nc_v4(yd + (long long)r[q] * H + c);
                }
#pragma unroll
                for (int q = 0; q < G; ++q) {
                    if (j0 + q >= k) break;
                    if (r[q] < 0) {                                // an id outside [0, E) left no row
                        fnx_flag_error(FNX_DEVERR_BADID);
                        continue;
                    }
                    const uint32_t vv[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[2 * e] = __fadd_rn(acc[2 * e], round_bf(__fmul_rn(bf_lo(vv[e]), sw[q])));
                        acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], round_bf(__fmul_rn(bf_hi(vv[e]), sw[q])));
                    }
                }
            }
            const float sg = round_bf(sigmoid_f32(g));
            const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
            uint32_t oa[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float lo = __fadd_rn(round_bf(acc[2 * q]), round_bf(__fmul_rn(bf_lo(sa[q]), sg)));
                const float hi = __fadd_rn(round_bf(acc[2 * q + 1]), round_bf(__fmul_rn(bf_hi(sa[q]), sg)));
                oa[q] = pack_bf2(lo, hi);
            }
            if (out) *reinterpret_cast<uint4*>(out + off) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
            if (hyper) inject_vec(hyper, inj, out_hyper, t, c, H, HC, oa);
            continue;
        }
        // slots in groups of four: all four row loads are issued before the in-order sums
        for (int j0 = 0; j0 < k; j0 += 4) {
            uint4 v[4];
            float s[4];
            bool ok[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                ok[q] = false;
                s[q] = 0.f;
                v[q] = make_uint4(0, 0, 0, 0);
                if (j0 + q < k) {
                    const long long slot = (long long)t * k + j0 + q;
                    const long long row = inverse ? inverse[slot] : slot;
                    if (row < 0 || row >= (long long)T * k) {      // an id outside [0, E) left no row
                        fnx_flag_error(FNX_DEVERR_BADID);
                    } else {
                        ok[q] = true;
                        s[q] = w[slot];
                        if (VEC) v[q] = ld_nc_v4(yd + row * H + c);
                        else v[q].x = (uint32_t)bf16_bits(yd[row * H + c]) << 16;
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (!ok[q]) continue;
                if (VEC) {
                    const uint32_t vv[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[2 * e] = __fadd_rn(acc[2 * e], round_bf(__fmul_rn(bf_lo(vv[e]), s[q])));
                        acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], round_bf(__fmul_rn(bf_hi(vv[e]), s[q])));
                    }
                } else {
                    acc[0] = __fadd_rn(acc[0], round_bf(__fmul_rn(bf_hi(v[q].x), s[q])));
                }
            }
        }
        const float sg = round_bf(sigmoid_f32(bf2f(gate[(long long)t * gate_ld])));
        const long long off = (long long)t * H + c;
        if (VEC) {
            const uint4 sv = ld_nc_v4(sh + off);
            const uint32_t sa[4] = {sv.x, sv.y, sv.z, sv.w};
            uint32_t oa[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float lo = __fadd_rn(round_bf(acc[2 * q]), round_bf(__fmul_rn(bf_lo(sa[q]), sg)));
                const float hi = __fadd_rn(round_bf(acc[2 * q + 1]), round_bf(__fmul_rn(bf_hi(sa[q]), sg)));
                oa[q] = pack_bf2(lo, hi);
            }
            *reinterpret_cast<uint4*>(out + off) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
        } else {
            out[off] = f2bf(__fadd_rn(round_bf(acc[0]), round_bf(__fmul_rn(bf2f(sh[off]), sg))));
        }
    }
}

// ---------------------------------------------------------------- Cartesian epilogue
// y: [G, G*W] (row j, column block j is slot j's own expert), w: [1, G] bf16,
// shared [1, W], gate [1]: the diagonal, slot-order weighted reduce and the merge
// (kernels/moe_epilogue/epilogue.cpp:17-39).
__global__ void __launch_bounds__(256) moe_epilogue_kernel(const bf16* __restrict__ y, const bf16* __restrict__ w,
                                                           const bf16* __restrict__ shared,
                                                           const bf16* __restrict__ gate, bf16* __restrict__ out,
                                                           int G, int W) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= W) return;
    float acc = 0.f;
    for (int j = 0; j < G; ++j) {
        const float v = bf2f(y[(long long)j * (G + 1) * W + c]);
        acc = __fadd_rn(acc, round_bf(__fmul_rn(v, bf2f(w[j]))));
    }
    const float a = round_bf(acc);
    const float sg = round_bf(sigmoid_f32(bf2f(gate[0])));
    out[c] = f2bf(__fadd_rn(a, round_bf(__fmul_rn(bf2f(shared[c]), sg))));
}

// ---------------------------------------------------------------- expert gather
// ow[k, j*N/8 + n8] = w[ids[j], k, n8] (int32 words); os[g, j*N + n] = s[ids[j], g, n] (bf16).
// kernels/expert_gather/gather.cpp:4-23.  Copies in 16-byte units when rows allow it.
// With E > 0 an id outside [0, E) writes zeros and flags FNX_DEVERR_BADID.
__global__ void __launch_bounds__(256) gather_pair_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s,
                                                          const int64_t* __restrict__ ids, uint8_t* __restrict__ ow,
                                                          uint8_t* __restrict__ os, int E, int K, int G, int N,
                                                          int nslots) {
    const long long wrow = (long long)N / 2;     // bytes per weight row (N/8 int32)
    const long long srow = (long long)N * 2;     // bytes per scale row (N bf16)
    const int slot = blockIdx.y;
    const long long e = ids[slot];
    const bool ok = E <= 0 || (e >= 0 && e < E);
    if (!ok && threadIdx.x == 0 && blockIdx.x == 0) fnx_flag_error(FNX_DEVERR_BADID);
    const bool v16 = (wrow % 16 == 0) && (srow % 16 == 0);
    const long long unit = v16 ? 16 : 2;
    const long long wunits = (long long)K * wrow / unit, sunits = (long long)G * srow / unit;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < wunits + sunits;
         i += (long long)gridDim.x * blockDim.x) {
        const bool isw = i < wunits;
        const long long u = isw ? i : i - wunits;
        const long long rowb = isw ? wrow : srow;
        const long long r = u * unit / rowb, cb = u * unit % rowb;
        const uint8_t* src = (isw ? w : s) + (e * (isw ? K : G) + r) * rowb + cb;
        uint8_t* dst = (isw ? ow : os) + (r * nslots + slot) * rowb + cb;
        if (v16) {
            uint4 v = ok ? ld_nc_v4(src) : make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(dst) = v;
        } else {
            *reinterpret_cast<uint16_t*>(dst) = ok ? *reinterpret_cast<const uint16_t*>(src) : 0;
        }
    }
}

// out[n] = sum over e in order of fp32(w[e] * y[e, n]) (W4GemvOp.weighted_sum, fnx/w4gemv_op.py:252-264:
// the expert outputs of one token weighted and summed); four columns per thread when aligned.
__global__ void __launch_bounds__(256) weighted_sum_f32_kernel(const float* __restrict__ y, const float* __restrict__ w,
                                                               float* __restrict__ out, int nE, int N) {
    for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
        float acc = 0.f;
        for (int e = 0; e < nE; ++e) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + e), __ldg(y + (long long)e * N + n)));
        out[n] = acc;
    }
}

}  // namespace fnx
