// Router top-k and the expert-major permutation.
//
// Routing (fnx/engine.py:1811-1813 in the reference): probs = softmax(fp32(logits));
// (w, idx) = topk(probs, k); w = bf16(w / sum(w)).  Ties are broken by ascending expert
// id (descending probability first), so the selection is a pure function of the bf16
// logits.  Permutation (fnx/engine.py:1817-1840): a stable counting sort of the flattened
// ids -> order (expert-major, (token*k + slot) order inside an expert), its inverse, and
// the cumulative per-expert row counts `ends`.
#pragma once
#include "fnx_common.cuh"

namespace fnx {

constexpr int ROUTE_MAX_E = 2048;     // experts per token row handled by one warp
constexpr int ROUTE_MAX_K = 32;       // top-k slots (one lane each)

// The selection rule on a warp's probability keys (key = bits(p) + 1, 0 for a selected or
// absent expert; expert i*32 + lane in key[i]): k rounds of (highest key, lowest id on ties).
// Lane j < k gets slot j's probability and id; `tot` is the slot-order sum of the k
// probabilities (identical in every lane).
template <int PER>
FNX_DEV void topk_rounds(uint32_t (&key)[PER], int k, float& my_p, int& my_i, float& tot) {
    const int lane = threadIdx.x & 31;
    my_p = 0.f;
    tot = 0.f;
    my_i = 0;
    for (int j = 0; j < k; ++j) {
        // a warp max over the keys, then a warp min over the ids of the lanes holding that key
        // (each lane offers its lowest such id)
        uint32_t lm = 0;
#pragma unroll
        for (int i = 0; i < PER; ++i) lm = max(lm, key[i]);
        const uint32_t gm = __reduce_max_sync(0xffffffffu, lm);
        uint32_t cand = 0xffffffffu;
#pragma unroll
        for (int i = PER - 1; i >= 0; --i)
            if (key[i] == gm) cand = (uint32_t)(i * 32 + lane);
        const int bi = (int)__reduce_min_sync(0xffffffffu, cand);
#pragma unroll
        for (int i = 0; i < PER; ++i)
            if (i * 32 + lane == bi) key[i] = 0u;
        const float bp = __uint_as_float(gm - 1u);
        if (lane == j) { my_p = bp; my_i = bi; }
        tot = __fadd_rn(tot, bp);
    }
}

// The same selection, usually without k rounds: the keys within a factor 16 of the largest fall
// into 64 bins of 2^19 key units (4.4 % in probability); if the smallest set of whole bins holding
// >= k keys holds at most 32, those candidates are ranked at once (a key's rank is the number of
// candidates above it, or equal with a lower id), which gives the rounds' selection and order.
// Otherwise (the k-th key more than a factor 16 below the first, or a crowded last bin) the rounds
// run.  W: this warp's scratch in shared memory.
struct TopkScratch {
    int hist[64];
    uint32_t ck[32];
    int ci[32];
    float prob[ROUTE_MAX_K];
    int sid[ROUTE_MAX_K];
};
template <int PER>
FNX_DEV void topk_select(uint32_t (&key)[PER], int k, TopkScratch& W, float& my_p, int& my_i, float& tot) {
    const int lane = threadIdx.x & 31;
    uint32_t lmax = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) lmax = max(lmax, key[i]);
    const uint32_t kmax = __reduce_max_sync(0xffffffffu, lmax);
    W.hist[lane] = 0;
    W.hist[lane + 32] = 0;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const uint32_t dist = kmax - key[i];
        if (key[i] && (dist >> 19) < 64u) atomicAdd(&W.hist[dist >> 19], 1);
    }
    __syncwarp();
    const int c0 = W.hist[2 * lane], c1 = W.hist[2 * lane + 1];
    int incl = c0 + c1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const int excl = incl - c0 - c1;
    const bool hit0 = excl + c0 >= k, hit1 = incl >= k;
    const unsigned bal = __ballot_sync(0xffffffffu, hit0 || hit1);
    int bstar = -1, cnt = 0;
    if (bal) {
        const int l = __ffs(bal) - 1;
        bstar = __shfl_sync(0xffffffffu, hit0 ? 2 * lane : 2 * lane + 1, l);
        cnt = __shfl_sync(0xffffffffu, hit0 ? excl + c0 : incl, l);
    }
    if (bstar < 0 || cnt > 32) {
        topk_rounds<PER>(key, k, my_p, my_i, tot);
        return;
    }
    // compact the candidates (bin <= bstar) into slots 0..cnt-1, then rank them all at once
    int mine = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) mine += (key[i] && ((kmax - key[i]) >> 19) <= (uint32_t)bstar) ? 1 : 0;
    int off = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, off, o);
        if (lane >= o) off += y;
    }
    off -= mine;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        if (key[i] && ((kmax - key[i]) >> 19) <= (uint32_t)bstar) {
            W.ck[off] = key[i];
            W.ci[off] = i * 32 + lane;
            ++off;
        }
    }
    __syncwarp();
    const uint32_t mk = lane < cnt ? W.ck[lane] : 0u;
    const int mi = lane < cnt ? W.ci[lane] : 0x7fffffff;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const uint32_t kj = __shfl_sync(0xffffffffu, mk, j);
        const int ij = __shfl_sync(0xffffffffu, mi, j);
        rank += (kj > mk || (kj == mk && ij < mi)) ? 1 : 0;
    }
    if (lane < cnt && rank < k) {
        W.prob[rank] = __uint_as_float(mk - 1u);
        W.sid[rank] = mi;
    }
    __syncwarp();
    tot = 0.f;
    for (int j = 0; j < k; ++j) tot = __fadd_rn(tot, W.prob[j]);
    my_p = 0.f;
    my_i = 0;
    if (lane < k) {
        my_p = W.prob[lane];
        my_i = W.sid[lane];
    }
    __syncwarp();
}

// Top-k of one row by one warp; PER = experts per lane (E <= 32*PER).  Returns, in lane
// j < k, slot j's probability (my_p) and expert id (my_i); `tot` is the slot-order sum of
// the k probabilities (identical in every lane).  CG reads the row through L2 (rows
// written by other blocks of the same kernel).  W: scratch for topk_select (null: the rounds).
template <int PER, bool CG>
FNX_DEV void topk_warp(const bf16* row, const float* bias, int E, int k, float& my_p, int& my_i, float& tot,
                       TopkScratch* W = nullptr) {
    const int lane = threadIdx.x & 31;
    float v[PER];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        float x = -INFINITY;
        if (e < E) {
            x = CG ? __uint_as_float((uint32_t)__ldcg(reinterpret_cast<const unsigned short*>(row) + e) << 16)
                   : bf2f(row[e]);
            if (bias) x = __fadd_rn(x, bias[e]);
        }
        v[i] = x;
        mx = fmaxf(mx, x);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = i * 32 + lane;
        const float p = e < E ? expf(__fsub_rn(v[i], mx)) : 0.f;
        v[i] = p;
        sum = __fadd_rn(sum, p);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float inv = 1.0f / sum;
    // probabilities as ordered keys: key = bits(p) + 1 for a non-negative probability (so
    // integer order is probability order), 0 for a selected or absent expert.  A NaN (from
    // NaN logits) counts as probability 0 so that k valid, distinct ids are always selected
    // (garbage logits must never turn into an out-of-range expert id).
    uint32_t key[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float pr = __fmul_rn(v[i], inv);
        key[i] = (i * 32 + lane) < E ? __float_as_uint(pr > 0.f ? pr : 0.f) + 1u : 0u;
    }

    if (W) topk_select<PER>(key, k, *W, my_p, my_i, tot);
    else topk_rounds<PER>(key, k, my_p, my_i, tot);
}

// One warp per token.  logits: bf16 [T, ld] (first E columns); bias: fp32 [E] or null.
template <int PER>
__global__ void __launch_bounds__(256) router_topk_kernel(const bf16* __restrict__ logits, long long ld,
                                                          const float* __restrict__ bias, bf16* __restrict__ w_out,
                                                          int64_t* __restrict__ idx_out, int32_t* __restrict__ idx32_out,
                                                          float* __restrict__ wf_out, int T, int E, int k) {
    __shared__ TopkScratch scratch[8];
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    float my_p, tot;
    int my_i;
    topk_warp<PER, false>(logits + (long long)t * ld, bias, E, k, my_p, my_i, tot, &scratch[threadIdx.x >> 5]);
    if (lane < k) {
        const bf16 wb = f2bf(my_p / tot);
        const long long o = (long long)t * k + lane;
        w_out[o] = wb;
        if (idx_out) idx_out[o] = my_i;
        if (idx32_out) idx32_out[o] = my_i;
        if (wf_out) wf_out[o] = bf2f(wb);
    }
}

// ------------------------------------------------------------------ permutation
__global__ void fill_i64_kernel(int64_t* __restrict__ p, int n, long long v) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

// Stable counting sort of n = T*k expert ids (int64) in chunks of PERM_CHUNK entries.
constexpr int PERM_CHUNK = 1024;
constexpr int PERM_MAX_E = 4096;

// pass 1: per-chunk histograms hist[chunk][E]
// Buckets: id / div for ids in [0, E*div) (div = 1: the expert itself; div = E/G: the rank
// owning a contiguous block of experts, the expert-parallel dispatch).
// n_dev (optional): the entry count lives on the device (at most n, the launch's capacity).
FNX_DEV int perm_count(int n, const long long* n_dev) {
    if (!n_dev) return n;
    const long long v = *n_dev;
    return v < 0 ? 0 : (v < n ? (int)v : n);
}

__global__ void __launch_bounds__(256) permute_hist_kernel(const int64_t* __restrict__ ids, int n,
                                                           const long long* __restrict__ n_dev, int E, int div,
                                                           int* __restrict__ hist) {
    extern __shared__ int sh[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
    __syncthreads();
    n = perm_count(n, n_dev);
    const int c0 = blockIdx.x * PERM_CHUNK;
    const long long lim = (long long)E * div;
    const int lane = threadIdx.x & 31;
    // warp-aggregated: one shared atomic per distinct bucket of the warp's 32 ids (few buckets,
    // e.g. the ranks of the expert-parallel dispatch, would otherwise serialise on one counter)
    for (int i0 = c0 + (threadIdx.x & ~31); i0 < c0 + PERM_CHUNK; i0 += blockDim.x) {
        const int i = i0 + lane;
        int b = -1;
        if (i < n) {
            const long long e = ids[i];
            if (e >= 0 && e < lim) b = (int)(div == 1 ? e : e / div);
            else fnx_flag_error(FNX_DEVERR_BADID);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        if (b >= 0 && lane == __ffs(peers) - 1) atomicAdd(&sh[b], __popc(peers));
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[(long long)blockIdx.x * E + e] = sh[e];
}

// pass 2 (one block): ends[e] = base + inclusive cumsum of counts; hist[c][e] becomes the
// starting output position of chunk c's entries for expert e.  The histogram is staged in
// shared memory when it fits (the per-expert walks over the chunks are dependent chains), and
// the scan over experts is a warp-shuffle scan.
constexpr size_t PERM_SCAN_SMEM = 160 * 1024;
inline size_t permute_scan_smem(int nchunks, int E) {
    const size_t b = sizeof(int) * (size_t)nchunks * E;
    return b <= PERM_SCAN_SMEM ? b : 0;
}

__global__ void __launch_bounds__(1024) permute_scan_kernel(int* __restrict__ hist, int nchunks, int E,
                                                            int64_t* __restrict__ ends, int64_t* __restrict__ counts_out,
                                                            long long base) {
    extern __shared__ int hs[];
    __shared__ int wsum[32];
    __shared__ int carry;
    const bool staged = (size_t)nchunks * E * sizeof(int) <= PERM_SCAN_SMEM;
    int* h = staged ? hs : hist;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tot = nchunks * E;
    if (staged)                                   // eight loads in flight per thread
        for (int i0 = threadIdx.x; i0 < tot; i0 += 8 * blockDim.x) {
            int v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = i0 + u * (int)blockDim.x < tot ? hist[i0 + u * blockDim.x] : 0;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (i0 + u * (int)blockDim.x < tot) hs[i0 + u * blockDim.x] = v[u];
        }
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        int cnt = 0;
        if (e < E)
#pragma unroll 8
            for (int c = 0; c < nchunks; ++c) cnt += h[c * E + e];
        // inclusive scan over the block: within warps, then over the warp totals
        int inc = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += u;
        }
        if (lane == 31) wsum[warp] = inc;
        __syncthreads();
        if (warp == 0) {
            const int v = wsum[lane];
            int wi = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += u;
            }
            wsum[lane] = wi - v;                  // exclusive prefix of the warp totals
        }
        __syncthreads();
        const int incl = carry + wsum[warp] + inc;
        if (e < E) {
            ends[e] = base + incl;
            if (counts_out) counts_out[e] = cnt;
            int pos = incl - cnt;
            for (int c = 0; c < nchunks; ++c) {
                const int v = h[c * E + e];
                h[c * E + e] = pos;
                pos += v;
            }
        }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = incl;
        __syncthreads();
    }
    if (staged)
        for (int i = threadIdx.x; i < tot; i += blockDim.x) hist[i] = hs[i];
}

// pass 3: one block per chunk; its 8 warps take 128 consecutive entries each.  A first walk
// counts each warp's entries per bucket (__match_any_sync groups equal ids of a 32-entry batch),
// the counts are scanned across the warps in order from the chunk's start positions, and a
// second walk places each warp's entries with its own cursors, so positions stay stable
// (chunk order, then warp order, then batch order, then lane order).
// order[pos] = i (or row_map[i]) and inverse[i] = pos_base + pos (the host offsets `order`).
constexpr int PERM_WARPS = 8;
inline size_t permute_scatter_smem(int E) { return sizeof(int) * ((size_t)PERM_WARPS * E + PERM_CHUNK); }

__global__ void __launch_bounds__(32 * PERM_WARPS) permute_scatter_kernel(
        const int64_t* __restrict__ ids, int n, const long long* __restrict__ n_dev, int E, int div,
        const int* __restrict__ start, int64_t* __restrict__ order, int64_t* __restrict__ inverse, long long pos_base,
        const int64_t* __restrict__ row_map) {
    extern __shared__ int psm[];
    int* cur = psm;                              // [PERM_WARPS][E]: counts, then cursors
    int* sid = psm + PERM_WARPS * E;             // [PERM_CHUNK]: bucket of each entry (-1 none)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    n = perm_count(n, n_dev);
    const int c0 = blockIdx.x * PERM_CHUNK;
    if (c0 >= n) return;
    const int c1 = min(n, c0 + PERM_CHUNK);
    for (int i = threadIdx.x; i < PERM_WARPS * E; i += blockDim.x) cur[i] = 0;
    const long long lim = (long long)E * div;
    for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
        const long long e = ids[i];
        sid[i - c0] = (e >= 0 && e < lim) ? (int)(div == 1 ? e : e / div) : -1;
    }
    __syncthreads();
    constexpr int PER_WARP = PERM_CHUNK / PERM_WARPS;
    const int w0 = c0 + warp * PER_WARP, w1 = min(c1, w0 + PER_WARP);
    int* mine = cur + warp * E;
    for (int b = w0; b < w0 + PER_WARP; b += 32) {       // counts (warp-private row)
        const int i = b + lane;
        const int bk = i < w1 ? sid[i - c0] : -1;
        const int key = bk >= 0 ? bk : -1 - lane;        // lanes without a bucket get unique keys
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        if (bk >= 0 && lane == __ffs(peers) - 1) mine[bk] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {  // exclusive scan across the warps
        int run = start[(long long)blockIdx.x * E + e];
        for (int w = 0; w < PERM_WARPS; ++w) {
            const int c = cur[w * E + e];
            cur[w * E + e] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int b = w0; b < w0 + PER_WARP; b += 32) {       // placement
        const int i = b + lane;
        const bool valid = i < w1;
        const int bk = valid ? sid[i - c0] : -1;
        const bool good = bk >= 0;
        const int key = good ? bk : -1 - lane;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int base = 0;
        if (good) base = mine[bk];
        __syncwarp();
        if (good && rank == 0) mine[bk] = base + __popc(peers);
        __syncwarp();
        if (good) {
            const long long pos = base + rank;
            order[pos] = row_map ? row_map[i] : i;
            if (inverse) inverse[i] = pos_base + pos;
        } else if (valid && inverse) {
            inverse[i] = -1;          // an id outside the buckets: no row (flagged by the histogram pass)
        }
    }
}

}  // namespace fnx
