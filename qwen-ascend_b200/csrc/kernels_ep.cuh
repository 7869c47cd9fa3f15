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

// ======================================================================== peer-memory exchange
// The same dispatch and return as the all-to-all, moved by this library's kernels through
// the NVLink peer mappings of the ranks' exchange regions (CUDA IPC; plain loads and stores,
// no multicast).  Nothing waits on the host: the per-owner counts travel by peer stores
// behind release/acquire flags, so the layer needs no host synchronisation.
//
// Every rank's region (one cudaMalloc, zero-filled at setup):
//   flags   u32  [EP_PHASES][2][EP_MAX_G]   flag[ph][parity][q] = last epoch rank q signalled
//   cnt     i64  [2][G][G]                  cnt[parity][q][j] = slots of rank q for owner j
//   recv_x  bf16 [cap + T_cap, H]           received slot rows, then this rank's own tokens
//   recv_e  i64  [cap]                      owner-local expert of each received slot
//   yb      bf16 [T_cap * k, H]             returned down rows, owner-major (this rank's slots)
//   plan    i64  [EP_PLAN_LEN]              local: this step's offsets (below)
//   epoch   u32, tickets u32[4]             local
// Epochs count layer calls (the same on every rank); flags and counts alternate between two
// parities so that a rank one step ahead never overwrites what a peer still reads.
namespace fnx {

constexpr int EP_MAX_G = 8;
enum { EP_PH_CNT = 0, EP_PH_DATA = 1, EP_PH_RET = 2, EP_PHASES = 3 };
// plan entries
constexpr int EP_R = 0, EP_EPOCH = 1;
constexpr int EP_RECV_OFF = 2;                                  // [G+1] prefix of slots received per source
constexpr int EP_SEND_OFF = EP_RECV_OFF + EP_MAX_G + 1;         // [G] my first row in each owner's recv_x
constexpr int EP_SRC_START = EP_SEND_OFF + EP_MAX_G;            // [G+1] owner chunks of my owner-major order
constexpr int EP_RET_OFF = EP_SRC_START + EP_MAX_G + 1;         // [G] first row for me in each source's yb
constexpr int EP_PLAN_LEN = EP_RET_OFF + EP_MAX_G;

struct EPDesc {
    int rank, world, H, k, T_cap, Eg;
    long long cap;
    long long* plan;
    unsigned* epoch;
    unsigned* tickets;
    unsigned* flags[EP_MAX_G];
    long long* cnt[EP_MAX_G];
    bf16* recv_x[EP_MAX_G];
    int64_t* recv_e[EP_MAX_G];
    bf16* yb[EP_MAX_G];
};

FNX_DEV void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FNX_DEV unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
FNX_DEV long long ld_relaxed_sys_i64(const long long* p) {
    long long v;
    asm volatile("ld.relaxed.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
FNX_DEV unsigned* ep_flag(const EPDesc& d, int owner, int phase, unsigned e, int q) {
    return d.flags[owner] + (phase * 2 + (int)(e & 1u)) * EP_MAX_G + q;
}

// threads q < G: tell rank q that this rank reached `phase` of epoch e
FNX_DEV void ep_signal_all(const EPDesc& d, int phase, unsigned e) {
    const int q = threadIdx.x;
    if (q < d.world) st_release_sys(ep_flag(d, q, phase, e, d.rank), e);
}

// threads q < G wait (bounded) until rank q has signalled `phase` of epoch e; then the block
// synchronises.  An expired wait records FNX_DEVERR_TIMEOUT and the kernel goes on.
FNX_DEV void ep_wait_all(const EPDesc& d, int phase, unsigned e) {
    const int q = threadIdx.x;
    if (q < d.world) {
        const unsigned* f = ep_flag(d, d.rank, phase, e, q);
        const uint64_t t0 = fnx_globaltimer();
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            __nanosleep(128);
            if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
                fnx_flag_error(FNX_DEVERR_TIMEOUT);
                break;
            }
        }
    }
    __syncthreads();
}

// One block (64 threads): start epoch e, send this rank's per-owner slot counts to every
// rank, wait for everyone's, and derive this step's offsets.
__global__ void __launch_bounds__(64) ep_counts_kernel(const EPDesc d, const int64_t* __restrict__ counts) {
    __shared__ unsigned se;
    __shared__ long long M[EP_MAX_G][EP_MAX_G];
    const int G = d.world, r = d.rank, t = threadIdx.x;
    if (t == 0) se = atomicAdd(d.epoch, 1u) + 1u;
    __syncthreads();
    const unsigned e = se;
    const int par = (int)(e & 1u);
    if (t < G * G) {
        const int q = t / G, j = t % G;
        d.cnt[q][((long long)par * G + r) * G + j] = counts[j];
    }
    __threadfence_system();
    __syncthreads();
    ep_signal_all(d, EP_PH_CNT, e);
    ep_wait_all(d, EP_PH_CNT, e);
    if (t < G * G) M[t / G][t % G] = ld_relaxed_sys_i64(d.cnt[r] + ((long long)par * G + t / G) * G + t % G);
    __syncthreads();
    if (t == 0) {
        long long* P = d.plan;
        long long acc = 0;
        for (int q = 0; q < G; ++q) { P[EP_RECV_OFF + q] = acc; acc += M[q][r]; }
        P[EP_RECV_OFF + G] = acc;
        if (acc > d.cap) { fnx_flag_error(FNX_DEVERR_OVERFLOW); acc = d.cap; }
        P[EP_R] = acc;
        P[EP_EPOCH] = e;
        for (int j = 0; j < G; ++j) {
            long long s = 0;
            for (int q = 0; q < r; ++q) s += M[q][j];
            P[EP_SEND_OFF + j] = s;
        }
        acc = 0;
        for (int j = 0; j < G; ++j) { P[EP_SRC_START + j] = acc; acc += M[r][j]; }
        P[EP_SRC_START + G] = acc;
        for (int q = 0; q < G; ++q) {
            long long s = 0;
            for (int j = 0; j < r; ++j) s += M[q][j];
            P[EP_RET_OFF + q] = s;
        }
    }
}

// row copy by one warp, 16-byte vectors (H % 8 == 0), four loads in flight per lane
FNX_DEV void ep_copy_row(bf16* dst, const bf16* src, int H, int lane) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* o = reinterpret_cast<uint4*>(dst);
    const int n16 = H >> 3;
    int c = lane;
    for (; c + 96 < n16; c += 128) {
        const uint4 v0 = __ldg(s + c), v1 = __ldg(s + c + 32), v2 = __ldg(s + c + 64), v3 = __ldg(s + c + 96);
        o[c] = v0; o[c + 32] = v1; o[c + 64] = v2; o[c + 96] = v3;
    }
    for (; c < n16; c += 32) o[c] = __ldg(s + c);
}

// the last block of a launch (by ticket) signals `phase` to every rank after all blocks'
// stores are visible system-wide
FNX_DEV void ep_last_block_signal(const EPDesc& d, unsigned* ticket, int phase, unsigned e) {
    __threadfence_system();
    __syncthreads();
    __shared__ unsigned last;
    if (threadIdx.x == 0) {
        const unsigned tk = atomicAdd(ticket, 1u);
        last = tk == gridDim.x - 1;
        if (last) {
            atomicExch(ticket, 0u);
            __threadfence_system();
        }
    }
    __syncthreads();
    if (last) ep_signal_all(d, phase, e);
}

FNX_DEV void ep_load_plan(const EPDesc& d, long long* sp) {
    for (int i = threadIdx.x; i < EP_PLAN_LEN; i += blockDim.x) sp[i] = d.plan[i];
    __syncthreads();
}

// Dispatch: slot p of the owner-major order goes to its owner's recv_x row
// send_off[j] + (p - src_start[j]) (with its owner-local expert in recv_e); this rank's own
// T tokens go to its own rows cap .. cap+T-1 (the shared expert's rows).  Then DATA.
__global__ void __launch_bounds__(256) ep_push_kernel(const EPDesc d, const bf16* __restrict__ x, int T,
                                                      const int64_t* __restrict__ order,
                                                      const int64_t* __restrict__ idx) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    const int G = d.world, H = d.H, k = d.k, lane = threadIdx.x & 31;
    const long long n = (long long)T * k;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n + T; p += warps) {
        if (p < n) {
            int j = 0;
            while (j + 1 < G && p >= sp[EP_SRC_START + j + 1]) ++j;
            const long long row = sp[EP_SEND_OFF + j] + (p - sp[EP_SRC_START + j]);
            const long long q = __ldg(order + p);
            if (row >= d.cap || q < 0 || q >= n) {
                if (lane == 0) fnx_flag_error(row >= d.cap ? FNX_DEVERR_OVERFLOW : FNX_DEVERR_BADID);
                continue;
            }
            if (lane == 0) d.recv_e[j][row] = __ldg(idx + q) % d.Eg;
            ep_copy_row(d.recv_x[j] + row * H, x + (q / k) * H, H, lane);
        } else {
            const long long t = p - n;
            ep_copy_row(d.recv_x[d.rank] + (d.cap + t) * H, x + t * H, H, lane);
        }
    }
    ep_last_block_signal(d, d.tickets + 0, EP_PH_DATA, (unsigned)sp[EP_EPOCH]);
}

// Return: received slot s (from source q, j-th of q's) sends its down row yd[pos[s]] to
// source q's yb row ret_off[q] + j.  Then RET.
__global__ void __launch_bounds__(256) ep_return_kernel(const EPDesc d, const bf16* __restrict__ yd,
                                                        long long yd_rows, const int64_t* __restrict__ pos) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    const int G = d.world, H = d.H, lane = threadIdx.x & 31;
    const long long R = sp[EP_R];
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long s = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); s < R; s += warps) {
        int q = 0;
        while (q + 1 < G && s >= sp[EP_RECV_OFF + q + 1]) ++q;
        const long long row = sp[EP_RET_OFF + q] + (s - sp[EP_RECV_OFF + q]);
        const long long src = __ldg(pos + s);
        if (src < 0 || src >= yd_rows || row >= (long long)d.T_cap * d.k) {
            if (lane == 0) fnx_flag_error(FNX_DEVERR_BADID);
            continue;
        }
        ep_copy_row(d.yb[q] + row * H, yd + src * H, H, lane);
    }
    ep_last_block_signal(d, d.tickets + 1, EP_PH_RET, (unsigned)sp[EP_EPOCH]);
}

// One block: wait until every rank signalled `phase` of this step's epoch.
__global__ void __launch_bounds__(32) ep_wait_kernel(const EPDesc d, int phase) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    ep_wait_all(d, phase, (unsigned)sp[EP_EPOCH]);
}

// The owner's expert-major rows start with the shared expert over its own T tokens (expert 0
// of the grouped launches: order_x[t] = cap + t, ends_x[0] = T).
__global__ void ep_head_kernel(int64_t* __restrict__ order_x, int64_t* __restrict__ ends_x, int T, long long cap) {
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) order_x[t] = cap + t;
    if (blockIdx.x == 0 && threadIdx.x == 0) ends_x[0] = T;
}

}  // namespace fnx
