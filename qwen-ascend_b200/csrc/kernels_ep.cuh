// Expert-parallel dispatch and combine: the row moves around the NCCL all-to-all.
//
// Experts are split over G ranks in contiguous blocks of E/G.  A rank sorts its (token, slot)
// entries by owning rank (the permutation kernels with div = E/G), packs one activation row
// per entry in that order together with the entry's expert id local to the owner, and the
// owner, after its grouped GEMMs, returns the down-projection rows in the order it received
// them.  Both moves are row gathers: dst[p] = src[index[p] / div].
#pragma once
#include "fnx_common.cuh"

namespace fnx {

// One warp per destination row, 16-byte loads and stores (H % 8 == 0, 16-byte aligned rows).
// A source row outside [0, src_rows) writes zeros and flags FNX_DEVERR_BADID.  With ids_out,
// lane 0 also writes ids_out[p] = ids[index[p]] % mod (the owner-local expert id; -1 for a
// bad row).
template <bool VEC>
__global__ void __launch_bounds__(256) ep_gather_rows_kernel(const bf16* __restrict__ src, long long ld_src,
                                                             long long src_rows, const int64_t* __restrict__ index,
                                                             int div, const int64_t* __restrict__ ids, int mod,
                                                             bf16* __restrict__ dst, long long ld_dst,
                                                             int64_t* __restrict__ ids_out, long long n, int H) {
    const int lane = threadIdx.x & 31;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n; p += warps) {
        const long long q = index ? __ldg(index + p) : p;
        const long long r = q >= 0 ? q / div : -1;
        const bool ok = r >= 0 && r < src_rows;
        if (lane == 0) {
            if (!ok) fnx_flag_error(FNX_DEVERR_BADID);
            if (ids_out) ids_out[p] = ok ? __ldg(ids + q) % mod : -1;
        }
        bf16* d = dst + p * ld_dst;
        if (VEC) {
            const uint4* s = reinterpret_cast<const uint4*>(src + (ok ? r : 0) * ld_src);
            uint4* o = reinterpret_cast<uint4*>(d);
            const int n16 = H >> 3;
            int c = lane;
            // four 16-byte loads in flight per lane before the stores
            for (; c + 96 < n16; c += 128) {
                uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0, v2 = v0, v3 = v0;
                if (ok) { v0 = __ldg(s + c); v1 = __ldg(s + c + 32); v2 = __ldg(s + c + 64); v3 = __ldg(s + c + 96); }
                o[c] = v0; o[c + 32] = v1; o[c + 64] = v2; o[c + 96] = v3;
            }
            for (; c < n16; c += 32) o[c] = ok ? __ldg(s + c) : make_uint4(0, 0, 0, 0);
        } else {
            const bf16* s = src + (ok ? r : 0) * ld_src;
            for (int c = lane; c < H; c += 32) d[c] = ok ? s[c] : __float2bfloat16_rn(0.f);
        }
    }
}

}  // namespace fnx
