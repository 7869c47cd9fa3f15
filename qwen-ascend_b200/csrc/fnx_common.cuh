// Common device helpers for the B200 (sm_100a) W4A16 MoE expert path.
//
// Everything here is written against the public PTX ISA: mbarriers, TMA
// (cp.async.bulk.tensor), cp.async, tcgen05 (alloc / mma / commit / ld) and the
// bounded-wait convention every spin in this library follows: a wait gives up after
// FNX_WAIT_NS of %globaltimer, records FNX_DEVERR_TIMEOUT in the device error word and
// returns false so the kernel can unwind and the context stays usable.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FNX_DEV __device__ __forceinline__

typedef __nv_bfloat16 bf16;
typedef __nv_bfloat162 bf162;

// Host-visible return codes (0 = launched; negative = rejected before launch).
enum {
    FNX_OK = 0,
    FNX_EARG = -1,        // argument out of the supported range
    FNX_ESHAPE = -2,      // shape the kernel does not support
    FNX_EALIGN = -3,      // pointer / stride alignment
    FNX_ELAUNCH = -4,     // CUDA launch error
    FNX_EWORKSPACE = -5,  // workspace too small
    FNX_EDRIVER = -6,     // driver entry point missing (tensor maps)
};

// Device error word bits (read and cleared by fnx_device_errors()).
enum {
    FNX_DEVERR_TIMEOUT = 1u,   // a bounded wait expired
    FNX_DEVERR_BADID = 2u,     // an expert id outside [0, E)
    FNX_DEVERR_OVERFLOW = 4u,  // a count exceeded its buffer
    FNX_DEVERR_NOLOGITS = 8u,  // a decode with logits_ready found no fresh router logits
};

__device__ unsigned int g_fnx_errors;

#ifndef FNX_WAIT_NS
#define FNX_WAIT_NS 2000000000ull   // 2 s
#endif

FNX_DEV void fnx_flag_error(unsigned bits) { atomicOr(&g_fnx_errors, bits); }

FNX_DEV uint64_t fnx_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

FNX_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ------------------------------------------------------------------ bf16 helpers
FNX_DEV float bf2f(bf16 v) { return __bfloat162float(v); }
FNX_DEV bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
FNX_DEV float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
FNX_DEV float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
FNX_DEV float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
FNX_DEV uint32_t bf16_bits(bf16 v) { return (uint32_t)__bfloat16_as_ushort(v); }
FNX_DEV uint32_t pack_bf2(float lo, float hi) {
    bf162 t = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&t);
}

// sigmoid in fp32 as 1 / (1 + exp(-g)) with IEEE division.
FNX_DEV float sigmoid_f32(float g) { return 1.0f / (1.0f + expf(-g)); }
// silu(x) = x * sigmoid(x), in fp32.
FNX_DEV float silu_f32(float x) { return __fmul_rn(x, 1.0f / (1.0f + expf(-x))); }

FNX_DEV uint4 ld_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
FNX_DEV uint4 ld_cg_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
FNX_DEV float ld_cg_f32(const float* p) {
    float r;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}

// int4 (two's complement, 8 per word, low nibble first) -> four bf16x2 holding the
// integer values of nibble pairs (0,4), (1,5), (2,6), (3,7).  Offset-binary trick:
// (n ^ 8) in the low mantissa bits of 0x4300 (= 128.0) is 128 + (q + 8); subtracting 136
// is exact and leaves q.
FNX_DEV void int4x8_to_bf16x2(uint32_t w, uint32_t (&o)[4]) {
    const uint32_t x = w ^ 0x88888888u;
    const uint32_t mask = 0x000f000fu, magic = 0x43004300u;
    uint32_t t0, t1, t2, t3;
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t0) : "r"(x), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t1) : "r"(x >> 4), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t2) : "r"(x >> 8), "r"(mask), "r"(magic));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t3) : "r"(x >> 12), "r"(mask), "r"(magic));
    const uint32_t k136 = 0x43084308u;   // bf16x2(136, 136)
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(t0), "r"(k136));
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(o[1]) : "r"(t1), "r"(k136));
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(o[2]) : "r"(t2), "r"(k136));
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(o[3]) : "r"(t3), "r"(k136));
}

// bf16x2 multiply, rounded once (the dequantised weight bf16(q * s)).
FNX_DEV uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// int8 weights without integer-to-float conversions: byte b of wx (a word of int8 values with
// their sign bits flipped, w ^ 0x80808080) as its exact fp32 value.  0x4B0000uu is 2^23 + u as
// fp32; taking 2^23 + 128 from it leaves u - 128, the signed byte.
FNX_DEV float i8x_f32(uint32_t wx, int b) {
    return __int_as_float(__byte_perm(wx, 0x4B000000u, 0x7640 + b)) - 8388736.0f;
}
// two exact small integers as bf16x2 (lo in the low half)
FNX_DEV uint32_t ints_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// acc += bf16 a * bf16 b, product and sum in fp32 (mixed-precision FMA, sm_100).
FNX_DEV void fma_bf_lo(float& acc, uint32_t a2, uint32_t b2) {
    asm("{\n .reg .b16 a, b, u;\n mov.b32 {a, u}, %1;\n mov.b32 {b, u}, %2;\n"
        " fma.rn.f32.bf16 %0, a, b, %0;\n}" : "+f"(acc) : "r"(a2), "r"(b2));
}
FNX_DEV void fma_bf_hi(float& acc, uint32_t a2, uint32_t b2) {
    asm("{\n .reg .b16 a, b, u;\n mov.b32 {u, a}, %1;\n mov.b32 {u, b}, %2;\n"
        " fma.rn.f32.bf16 %0, a, b, %0;\n}" : "+f"(acc) : "r"(a2), "r"(b2));
}
// acc += bf16 hi/lo half of a2 times bf16 scalar held in the low half of x
FNX_DEV void fma_bf_lo_x(float& acc, uint32_t a2, uint16_t x) {
    asm("{\n .reg .b16 a, u;\n mov.b32 {a, u}, %1;\n fma.rn.f32.bf16 %0, a, %2, %0;\n}"
        : "+f"(acc) : "r"(a2), "h"(x));
}
FNX_DEV void fma_bf_hi_x(float& acc, uint32_t a2, uint16_t x) {
    asm("{\n .reg .b16 a, u;\n mov.b32 {u, a}, %1;\n fma.rn.f32.bf16 %0, a, %2, %0;\n}"
        : "+f"(acc) : "r"(a2), "h"(x));
}

// D += A * B over one warp: mma m16n8k16, bf16 A (16 x 16, row) and B (16 x 8, col), fp32 D.
// Fragments (PTX ISA, group g = lane / 4, t = lane % 4): a0 = A[g][2t..2t+1], a1 = A[g+8][2t..],
// a2 = A[g][2t+8..], a3 = A[g+8][2t+8..]; b0 = B[2t..2t+1][g], b1 = B[2t+8..][g];
// d0, d1 = D[g][2t], D[g][2t+1]; d2, d3 = D[g+8][2t], D[g+8][2t+1].
FNX_DEV void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                            uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ mbarrier
FNX_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
FNX_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
FNX_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}
FNX_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
FNX_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase.  Returns false (and flags the error) on timeout.
// Failed polls back off for FNX_WAIT_SLEEP_NS: a barrier poll is a shared-memory
// operation, and warps polling without pause queue ahead of the MMA warp's commits.
#ifndef FNX_WAIT_SLEEP_NS
#define FNX_WAIT_SLEEP_NS 64
#endif
FNX_DEV void wait_backoff() {
    if (FNX_WAIT_SLEEP_NS > 0) __nanosleep(FNX_WAIT_SLEEP_NS);
}
FNX_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = fnx_globaltimer();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 32; ++i) {
            wait_backoff();
            if (mbar_try_wait(bar, parity)) return true;
        }
        if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
            fnx_flag_error(FNX_DEVERR_TIMEOUT);
            return false;
        }
    }
}
// cp.async completion -> mbarrier arrival (no expected-count increment)
FNX_DEV void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
FNX_DEV void cp_async_16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
FNX_DEV void cp_async_16_zfill(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
FNX_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ TMA
FNX_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y) : "memory");
}
// L2 cache policies: stream-once data (weights) should not evict data that is re-read
// (gathered activations).
FNX_DEV uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
FNX_DEV uint64_t l2_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Linear bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16),
// completion counted on an mbarrier's transaction bytes.
FNX_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}
// Prefetch a global range (16-byte aligned, size a multiple of 16) into L2.
FNX_DEV void l2_prefetch(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// 16-byte cp.async with zero fill (src_size 0) and an L2 policy.
FNX_DEV void cp_async_16_hint(uint32_t dst, const void* src, bool valid, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;"
                 ::"r"(dst), "l"(src), "r"(valid ? 16 : 0), "l"(policy) : "memory");
}
FNX_DEV void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------ tcgen05
FNX_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
FNX_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
FNX_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// CTA-pair (cta_group::2) forms: one warp in each CTA of the pair allocates the same
// columns in both CTAs' tensor memory; MMAs issued by the pair's rank-0 CTA use both.
FNX_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
FNX_DEV void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
FNX_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
FNX_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FNX_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 x bf16 -> fp32), issued by one thread.
FNX_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
                 ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// Same with A read from tensor memory (M lanes x K/2 columns, two bf16 per column).
FNX_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from 32 registers per thread (warp w reaches
// lanes 32*(w%4) .. +31 only).
FNX_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from 16 registers per thread.
FNX_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
FNX_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (+)= A * B^T over a CTA pair (M = 256: A rows 0..127 from this CTA's tensor memory,
// 128..255 from the peer's at the same address; each CTA holds N/2 rows of B at the same
// shared-memory address; D lands in both CTAs' tensor memory).  Issued by rank 0 only.
FNX_DEV void umma_bf16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                               uint32_t accumulate) {
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on the mbarrier at this shared-memory offset in every CTA of cta_mask once the
// pair MMAs issued so far complete.
FNX_DEV void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_u32(bar)), "h"(cta_mask) : "memory");
}

// ------------------------------------------------------------------ clusters
FNX_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
FNX_DEV uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
FNX_DEV uint32_t num_clusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// All threads of every CTA in the cluster (release / acquire).
FNX_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address of `p` in CTA `rank` of this cluster.
FNX_DEV uint32_t mapa_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
FNX_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Remote arrival without the cluster-scope release.  For announcing data this thread did
// not write and that is already complete in shared / tensor memory (observed through a
// local mbarrier): the release would only wait for this thread's own outstanding memory
// operations, which costs ~860 cycles per call on the relay path.
FNX_DEV void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
FNX_DEV bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
FNX_DEV bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}" : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait on a phase completed by arrivals from another SM (remote arrives, pair
// MMA commits).  Polls with the non-suspending test_wait: a thread suspended in try_wait
// is woken late when the completing arrival comes from another SM.
FNX_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
    if (mbar_test_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = fnx_globaltimer();
    while (true) {
#pragma unroll 1
        for (int i = 0; i < 64; ++i) {
            wait_backoff();
            if (mbar_test_wait_cluster(bar, parity)) return true;
        }
        if (fnx_globaltimer() - t0 > FNX_WAIT_NS) {
            fnx_flag_error(FNX_DEVERR_TIMEOUT);
            return false;
        }
    }
}

// Named CTA barriers (ids 1..15; 0 is __syncthreads).  Executed by whole warps.
FNX_DEV void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
FNX_DEV void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
FNX_DEV bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}" : "=r"(pred));
    return pred != 0;
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
FNX_DEV void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}
FNX_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
FNX_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart
// (start address >> 4 in bits [0,14), LBO 16 B (unused for this layout), SBO 1024 B in
// bits [32,46), descriptor version 1 in bits [46,48), layout SWIZZLE_128B = 2 in [61,64)).
FNX_DEV uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a K-major SW128 tile whose rows
// are 128 bytes (64 bf16) and whose base is 1024-byte aligned.
FNX_DEV uint32_t sw128_offset(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

// Programmatic dependent launch: wait for the preceding grid / let the next one start.
FNX_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FNX_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
