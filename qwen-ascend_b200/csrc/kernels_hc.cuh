// Hyper-connection mix that produces the MoE layer's input (gated_residual,
// fnx/engine.py:818-857, torch path; native forms kernels/post_ops/post_ops.cpp:4-53):
//   hn     = rms_norm per branch of H (fp32, * (1 + w)) -> bf16            hc_rms_norm_kernel
//   di     = hn . W_di^T   (library GEMM: W_di = down rows then HC inject rows)
//   mix    = bf16(silu(bf16(dp / HC))),  inj = bf16(2 * bf16(sigmoid(bf16(ip / HC))))
//                                                                            hc_activation_kernel
//   logits = mix . W_up^T  (library GEMM)
//   mixed  = bf16(sum_b bf16(bf16(sigmoid(logits_b)) * hn_b) / HC)          hc_sigmoid_reduce_kernel
// Every elementwise step rounds where the torch path rounds (each bf16 op computes in fp32 and
// rounds once); the RMS statistic is an fp32 sum whose order is this kernel's own.
#pragma once
#include "fnx_common.cuh"

namespace fnx {

// One block per (token, branch) group of H: x [batch, HC*H] bf16, w [HC*H] bf16 (the weight
// is per element of the flattened row; gamma = 1 + w), out bf16 [batch, HC*H].
__global__ void __launch_bounds__(256) hc_rms_norm_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                          bf16* __restrict__ out, int H, int HC, float eps) {
    __shared__ float red[8];
    const long long g = blockIdx.x;                  // token * HC + branch
    const bf16* xr = x + g * H;
    const bf16* wr = w + (g % HC) * (long long)H;
    float ss = 0.f;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        const float v = bf2f(xr[c]);
        ss = __fadd_rn(ss, __fmul_rn(v, v));        // the torch path squares, then sums
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot = __fadd_rn(tot, red[i]);
    // out = (x * rsqrt(mean + eps)) * (1 + w), each product rounded in fp32
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), eps)));
    bf16* orow = out + g * H;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        const float v = __fmul_rn(bf2f(xr[c]), inv);
        orow[c] = f2bf(__fmul_rn(v, __fadd_rn(1.0f, bf2f(wr[c]))));
    }
}

// mix = bf16(silu(bf16(dp / HC))) for the first n_mix columns of di [batch, n_mix + HC];
// inj = bf16(2 * bf16(sigmoid(bf16(ip / HC)))) for the last HC.  mode (the native kernel's
// options): bit 0 takes sigmoid as a rounded reciprocal, bit 1 takes silu as v * sigmoid
// instead of v / (1 + e^-v); 0 is the torch path.
__global__ void __launch_bounds__(256) hc_activation_kernel(const bf16* __restrict__ di, bf16* __restrict__ mix,
                                                            bf16* __restrict__ inj, int batch, int n_mix, int HC,
                                                            int mode) {
    const int W = n_mix + HC;
    const long long total = (long long)batch * W;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / W;
        const int c = (int)(i - t * W);
        const float v = round_bf(__fdiv_rn(bf2f(di[i]), (float)HC));
        const float d = __fadd_rn(1.0f, expf(-v));
        const float s = (mode & 1) ? __frcp_rn(d) : __fdiv_rn(1.0f, d);
        if (c < n_mix) {
            const float a = (mode & 2) ? __fmul_rn(v, s) : __fdiv_rn(v, d);
            mix[t * n_mix + c] = f2bf(a);
        } else {
            inj[t * HC + (c - n_mix)] = f2bf(__fmul_rn(2.0f, round_bf(s)));
        }
    }
}

// mixed[t, c] = bf16( (sum_b bf16(bf16(sigmoid(l[t, b*H + c])) * x[t, b*H + c])) / HC ), the
// branch sum in order b = 0..HC-1 in fp32.
// One output of the branch mix at (t, c): branches in ascending order, the loads of four
// branches issued before their arithmetic (HC is a runtime value, so the loop is not unrolled).
FNX_DEV bf16 hc_mix_one(const bf16* __restrict__ x, const bf16* __restrict__ l, long long t, int c, int H, int HC) {
    float acc = 0.f;
    for (int b0 = 0; b0 < HC; b0 += 4) {
        bf16 lv[4] = {}, xv[4] = {};
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (b0 + u < HC) {
                const long long o = (t * HC + b0 + u) * (long long)H + c;
                lv[u] = l[o];
                xv[u] = x[o];
            }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (b0 + u < HC) {
                const float sg = round_bf(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-bf2f(lv[u])))));
                acc = __fadd_rn(acc, round_bf(__fmul_rn(sg, bf2f(xv[u]))));
            }
    }
    return f2bf(__fdiv_rn(acc, (float)HC));
}

__global__ void __launch_bounds__(256) hc_sigmoid_reduce_kernel(const bf16* __restrict__ x, const bf16* __restrict__ l,
                                                                bf16* __restrict__ y, int batch, int H, int HC) {
    const long long total = (long long)batch * H;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / H;
        y[i] = hc_mix_one(x, l, t, (int)(i - t * H), H, HC);
    }
}

}  // namespace fnx
