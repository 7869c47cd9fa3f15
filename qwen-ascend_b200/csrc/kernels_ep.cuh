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
// The dispatch and return of the all-to-all, moved by this library's kernels through the
// NVLink peer mappings of the ranks' exchange regions (CUDA IPC; plain loads and stores, no
// multicast).  Nothing waits on the host: the per-owner counts travel by peer stores behind
// release/acquire flags, so a layer call is one stream of launches.
//
// Dispatch sends each token ONCE per owner that holds any of its k experts (the slots of one
// token for one owner are consecutive in the owner-major order), plus one small entry per
// slot (owner-local expert, token row).  The return is per slot: the owner's down GEMM writes
// each slot's row straight into the source's `yb` through a per-row pointer table, so the
// source reduces the k rows in the reference's slot order.
//
// Every rank's region (one cudaMalloc, zero-filled at setup):
//   flags    u32  [EP_PHASES][2][EP_MAX_G]    flag[ph][parity][q] = last epoch rank q signalled
//   cnt      i64  [2][G][G][2]                cnt[parity][q][j] = (slots, tokens) of rank q for owner j
//   plan     i64  [EP_PLAN_LEN]               local: this call's offsets (below)
//   epoch    u32, tickets u32[4]              local
//   bcount   i32  [ceil(T_cap*k / 1024)]      local: token dedup block counts
//   recv_e   i64  [cap]                       received slots: owner-local expert
//   recv_row i64  [cap]                       received slots: token row in recv_x
//   recv_x   bf16 [cap_tok + T_cap, H]        received token rows, then this rank's own tokens
//   yb       bf16 [T_cap * k, H]              returned down rows, owner-major (this rank's slots)
//   sink     bf16 [H]                         target of rows with no valid destination
// cap = G*T_cap*k slots and cap_tok = G*T_cap token rows always suffice.  Epochs count layer
// calls (the same on every rank); flags and counts alternate between two parities so that a
// rank one call ahead never overwrites what a peer still reads.
namespace fnx {

constexpr int EP_MAX_G = 8;
enum { EP_PH_CNT = 0, EP_PH_DATA = 1, EP_PH_RET = 2, EP_PHASES = 3 };
// plan entries
constexpr int EP_R = 0, EP_EPOCH = 1;
constexpr int EP_RECV_OFF = 2;                                   // [G+1] prefix of slots received per source
constexpr int EP_SEND_OFF = EP_RECV_OFF + EP_MAX_G + 1;          // [G] my first slot row in each owner
constexpr int EP_SRC_START = EP_SEND_OFF + EP_MAX_G;             // [G+1] owner chunks of my owner-major slots
constexpr int EP_RET_OFF = EP_SRC_START + EP_MAX_G + 1;          // [G] first row for me in each source's yb
constexpr int EP_TOK_SEND_OFF = EP_RET_OFF + EP_MAX_G;           // [G] my first token row in each owner
constexpr int EP_TOK_START = EP_TOK_SEND_OFF + EP_MAX_G;         // [G+1] owner chunks of my deduplicated tokens
constexpr int EP_PLAN_LEN = EP_TOK_START + EP_MAX_G + 1;

struct EPDesc {
    int rank, world, H, k, T_cap, Eg;
    long long cap, cap_tok;
    long long* plan;
    unsigned* epoch;
    unsigned* tickets;
    int* bcount;                    // local: dedup block counts [ceil(T_cap*k / 1024)]
    bf16* sink;
    unsigned* flags[EP_MAX_G];
    long long* cnt[EP_MAX_G];
    bf16* recv_x[EP_MAX_G];
    int64_t* recv_e[EP_MAX_G];
    int64_t* recv_row[EP_MAX_G];
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

FNX_DEV void ep_load_plan(const EPDesc& d, long long* sp) {
    for (int i = threadIdx.x; i < EP_PLAN_LEN; i += blockDim.x) sp[i] = d.plan[i];
    __syncthreads();
}

// owner chunk holding entry p of a [G+1] prefix array (G <= 8)
FNX_DEV int ep_chunk(const long long* start, int G, long long p) {
    int j = 0;
    while (j + 1 < G && p >= start[j + 1]) ++j;
    return j;
}

// Token dedup: tok_index[p] = the deduplicated token row of owner-major slot p (counted over
// all owners; a new row starts at each owner chunk and at each change of token), and
// tcounts[j] = the token rows for owner j.  Two launches over blocks of 1024 slots: the first
// counts each block's new rows, the second adds the counts of the blocks before it to a
// block-wide scan; its last block (by ticket) derives tcounts.
FNX_DEV void ep_chunk_starts(const int64_t* counts, int G, long long* start) {
    if (threadIdx.x == 0) {
        long long a = 0;
        for (int j = 0; j < G; ++j) { start[j] = a; a += counts[j]; }
        start[G] = a;
    }
    __syncthreads();
}
FNX_DEV bool ep_first(const int64_t* order, const long long* start, int G, int k, long long p) {
    if (p == 0) return true;
    for (int j = 1; j < G; ++j)
        if (p == start[j]) return true;
    return __ldg(order + p) / k != __ldg(order + p - 1) / k;
}

__global__ void __launch_bounds__(1024) ep_dedup_count_kernel(const EPDesc d, const int64_t* __restrict__ order,
                                                              const int64_t* __restrict__ counts, int n) {
    __shared__ long long start[EP_MAX_G + 1];
    ep_chunk_starts(counts, d.world, start);
    const long long p = (long long)blockIdx.x * 1024 + threadIdx.x;
    const int c = __syncthreads_count(p < n && ep_first(order, start, d.world, d.k, p));
    if (threadIdx.x == 0) d.bcount[blockIdx.x] = c;
}

__global__ void __launch_bounds__(1024) ep_dedup_index_kernel(const EPDesc d, const int64_t* __restrict__ order,
                                                              const int64_t* __restrict__ counts, int n,
                                                              int* __restrict__ tok_index,
                                                              int64_t* __restrict__ tcounts) {
    __shared__ long long start[EP_MAX_G + 1];
    __shared__ int wsum[32];
    __shared__ int base;
    __shared__ unsigned last;
    ep_chunk_starts(counts, d.world, start);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        int b = 0;
        for (int i = 0; i < (int)blockIdx.x; ++i) b += d.bcount[i];
        base = b;
    }
    const long long p = (long long)blockIdx.x * 1024 + threadIdx.x;
    const bool f = p < n && ep_first(order, start, d.world, d.k, p);
    const unsigned m = __ballot_sync(0xffffffffu, f);
    if (lane == 0) wsum[warp] = __popc(m);
    __syncthreads();
    if (warp == 0) {
        const int v = wsum[lane];
        int inc = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += u;
        }
        wsum[lane] = inc - v;
    }
    __syncthreads();
    if (p < n) tok_index[p] = base + wsum[warp] + __popc(m & ((1u << lane) - 1u)) + (f ? 1 : 0) - 1;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(d.tickets + 2, 1u) == gridDim.x - 1;
        if (last) {
            atomicExch(d.tickets + 2, 0u);
            __threadfence();
        }
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        const int G = d.world;
        const int total = n > 0 ? __ldcg(tok_index + n - 1) + 1 : 0;
        long long us[EP_MAX_G + 1];
        us[G] = total;
        for (int j = G - 1; j >= 0; --j) us[j] = start[j] < start[j + 1] ? __ldcg(tok_index + start[j]) : us[j + 1];
        for (int j = 0; j < G; ++j) tcounts[j] = us[j + 1] - us[j];
    }
}

// One block (64 threads): start epoch e, send this rank's per-owner slot and token counts to
// every rank, wait for everyone's, and derive this call's offsets.
__global__ void __launch_bounds__(64) ep_counts_kernel(const EPDesc d, const int64_t* __restrict__ counts,
                                                       const int64_t* __restrict__ tcounts) {
    __shared__ unsigned se;
    __shared__ long long M[EP_MAX_G][EP_MAX_G], U[EP_MAX_G][EP_MAX_G];
    const int G = d.world, r = d.rank, t = threadIdx.x;
    if (t == 0) se = atomicAdd(d.epoch, 1u) + 1u;
    __syncthreads();
    const unsigned e = se;
    const int par = (int)(e & 1u);
    if (t < G * G) {
        const int q = t / G, j = t % G;
        long long* c = d.cnt[q] + (((long long)par * G + r) * G + j) * 2;
        c[0] = counts[j];
        c[1] = tcounts[j];
    }
    __threadfence_system();
    __syncthreads();
    ep_signal_all(d, EP_PH_CNT, e);
    ep_wait_all(d, EP_PH_CNT, e);
    if (t < G * G) {
        const long long* c = d.cnt[r] + (((long long)par * G + t / G) * G + t % G) * 2;
        M[t / G][t % G] = ld_relaxed_sys_i64(c);
        U[t / G][t % G] = ld_relaxed_sys_i64(c + 1);
    }
    __syncthreads();
    if (t == 0) {
        long long* P = d.plan;
        long long acc = 0, tok = 0;
        for (int q = 0; q < G; ++q) { P[EP_RECV_OFF + q] = acc; acc += M[q][r]; tok += U[q][r]; }
        P[EP_RECV_OFF + G] = acc;
        if (acc > d.cap || tok > d.cap_tok) { fnx_flag_error(FNX_DEVERR_OVERFLOW); acc = min(acc, d.cap); }
        P[EP_R] = acc;
        P[EP_EPOCH] = e;
        for (int j = 0; j < G; ++j) {
            long long s = 0, u = 0;
            for (int q = 0; q < r; ++q) { s += M[q][j]; u += U[q][j]; }
            P[EP_SEND_OFF + j] = s;
            P[EP_TOK_SEND_OFF + j] = u;
        }
        acc = tok = 0;
        for (int j = 0; j < G; ++j) {
            P[EP_SRC_START + j] = acc; acc += M[r][j];
            P[EP_TOK_START + j] = tok; tok += U[r][j];
        }
        P[EP_SRC_START + G] = acc;
        P[EP_TOK_START + G] = tok;
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

// Dispatch.  Slot p of the owner-major order (owner j) writes its entry to j's slot row
// send_off[j] + (p - src_start[j]): the owner-local expert and the token row
// tok_send_off[j] + (tok_index[p] - tok_start[j]); the first slot of each token for j also
// copies the token row there.  Each lane takes one slot (32 slots' loads in flight per warp),
// then the warp copies the rows of its first slots one after another.  This rank's own T tokens
// go to its rows cap_tok .. cap_tok+T-1 (the shared expert's rows).  Then DATA.
__global__ void __launch_bounds__(256) ep_push_kernel(const EPDesc d, const bf16* __restrict__ x, int T,
                                                      const int64_t* __restrict__ order,
                                                      const int64_t* __restrict__ idx,
                                                      const int* __restrict__ tok_index, bool copy_own) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    const int G = d.world, H = d.H, k = d.k, lane = threadIdx.x & 31;
    const long long n = (long long)T * k;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (long long b = gw * 32; b < n; b += warps * 32) {
        const long long p = b + lane;
        bool copy = false;
        int j = 0;
        long long trow = 0, src = 0;
        if (p < n) {
            j = ep_chunk(sp + EP_SRC_START, G, p);
            const long long srow = sp[EP_SEND_OFF + j] + (p - sp[EP_SRC_START + j]);
            const int ti = __ldg(tok_index + p);
            trow = sp[EP_TOK_SEND_OFF + j] + (ti - sp[EP_TOK_START + j]);
            const long long q = __ldg(order + p);
            if (srow >= d.cap || trow >= d.cap_tok || trow < 0 || q < 0 || q >= n) {
                fnx_flag_error(q < 0 || q >= n ? FNX_DEVERR_BADID : FNX_DEVERR_OVERFLOW);
            } else {
                d.recv_e[j][srow] = __ldg(idx + q) % d.Eg;
                d.recv_row[j][srow] = trow;
                copy = p == sp[EP_SRC_START + j] || __ldg(tok_index + p - 1) != ti;
                src = q / k;
            }
        }
        unsigned m = __ballot_sync(0xffffffffu, copy);
        while (m) {
            const int l = __ffs(m) - 1;
            m &= m - 1u;
            const int jj = __shfl_sync(0xffffffffu, j, l);
            const long long tr = __shfl_sync(0xffffffffu, trow, l);
            const long long sr = __shfl_sync(0xffffffffu, src, l);
            ep_copy_row(d.recv_x[jj] + tr * H, x + sr * H, H, lane);
        }
    }
    if (copy_own)
        for (long long t = gw; t < T; t += warps)
            ep_copy_row(d.recv_x[d.rank] + (d.cap_tok + t) * H, x + t * H, H, lane);
    ep_last_block_signal(d, d.tickets + 0, EP_PH_DATA, (unsigned)sp[EP_EPOCH]);
}

// One block: wait until every rank signalled `phase` of this call's epoch.
__global__ void __launch_bounds__(32) ep_wait_kernel(const EPDesc d, int phase) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    ep_wait_all(d, phase, (unsigned)sp[EP_EPOCH]);
}

// One block: every prior write of this rank (a finished launch's peer stores included) is made
// visible system-wide, then `phase` of this call's epoch is signalled to every rank.
__global__ void __launch_bounds__(32) ep_signal_kernel(const EPDesc d, int phase) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    __threadfence_system();
    ep_signal_all(d, phase, (unsigned)sp[EP_EPOCH]);
}

// Head of the owner's expert-major rows: the shared expert over its own T tokens is expert 0
// of the grouped launches (order_x[t] = cap_tok + t, ends_x[0] = T, its down rows to
// sh_out); every other down-row destination starts at the sink.
__global__ void __launch_bounds__(256) ep_head_kernel(const EPDesc d, int64_t* __restrict__ order_x,
                                                      int64_t* __restrict__ ends_x, bf16** __restrict__ rows,
                                                      bf16* __restrict__ sh_out, int T) {
    const long long total = (long long)T + d.cap;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        if (i < T) {
            order_x[i] = d.cap_tok + i;
            rows[i] = sh_out + i * d.H;
        } else {
            rows[i] = d.sink;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) ends_x[0] = T;
}

// Every received slot's down-row destination starts at the sink (rows past this call's count).
__global__ void __launch_bounds__(256) ep_sink_rows_kernel(const EPDesc d, bf16** __restrict__ rows) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < d.cap; i += (long long)gridDim.x * blockDim.x)
        rows[i] = d.sink;
}

// Down-row destinations of the received slots: slot s (from source q, the j-th of q's) at
// expert-major position pos[s] (T + its rank when the rank's own T shared-expert rows come
// first, else its rank) returns to source q's yb row ret_off[q] + j.
__global__ void __launch_bounds__(256) ep_rows_kernel(const EPDesc d, const int64_t* __restrict__ pos, int T,
                                                      bf16** __restrict__ rows) {
    __shared__ long long sp[EP_PLAN_LEN];
    ep_load_plan(d, sp);
    const long long R = sp[EP_R];
    const long long lim = (long long)d.T_cap * d.k;
    for (long long s = (long long)blockIdx.x * blockDim.x + threadIdx.x; s < R; s += (long long)gridDim.x * blockDim.x) {
        const int q = ep_chunk(sp + EP_RECV_OFF, d.world, s);
        const long long row = sp[EP_RET_OFF + q] + (s - sp[EP_RECV_OFF + q]);
        const long long ps = pos[s];
        if (ps < T || ps >= T + R || row >= lim) {
            fnx_flag_error(FNX_DEVERR_BADID);
            continue;
        }
        rows[ps] = d.yb[q] + row * d.H;
    }
}

}  // namespace fnx
