// umma.cuh -- sm_100a tensor-core (tcgen05) building blocks used by the
// chunked delta-rule kernel: shared-memory operand layouts and descriptors,
// instruction descriptors, TMEM allocation, MMA issue/commit, TMEM <-> register
// moves, and bounded mbarrier waits.
//
// Operand layouts (no swizzle).  An MMA operand tile is stored as 8 x 16-byte
// "core matrices" (128 contiguous bytes each):
//   K-major  (rows = M or N, K contiguous): element (r, k) of a tile with KK
//            columns of K sits at  (r/8)*SBO + (k/8)*128 + (r%8)*16 + (k%8)*2
//            [16-bit types; for 32-bit types replace 8 by 4 along k and *2 by *4]
//            LBO = 128 (next 8 k's), SBO = (KK/8)*128 (next 8 rows).
//   MN-major (M or N contiguous): element (k, c) of a tile with CC columns of
//            M/N sits at  (k/8)*LBO + (c/8)*128 + (k%8)*16 + (c%8)*2
//            SBO = 128 (next 8 columns), LBO = (CC/8)*128 (next 8 k's).
// One kind::f16 MMA consumes K = 16 (two 8-k groups); the next K step starts
// 2 groups further on: +256 bytes (K-major) or +2*LBO (MN-major).
//
// Accumulators (fp32, cta_group::1): M = 128 puts row i in TMEM lane i;
// M = 64 puts rows 16q..16q+15 in lanes 32q..32q+15 (q = 0..3).  A warp
// w reads lanes 32*(w%4) .. 32*(w%4)+31 with tcgen05.ld.32x32b.
//
// Waits are bounded: a wait that runs out sets *err (when given) and returns
// false, so a kernel can stop cleanly instead of hanging the GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {
namespace umma {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ descriptors
__host__ __device__ constexpr uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1, no swizzle
}

// The same with the 128-byte swizzle layout (tile base 1024-byte aligned).
//   K-major: 8 rows of 128 bytes (64 16-bit k's) per 1024-byte atom, 16-byte
//            chunk j of row r stored at chunk j ^ (r % 8); SBO = next 8 rows;
//            LBO unused; a K step of 16 advances the start address 32 bytes.
//   MN-major: 8 k-rows of 128 bytes (64 mn's) per atom, same permutation;
//            LBO = next 64 mn's (next atom column), SBO = next 8 k's.
__host__ __device__ constexpr uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return smem_desc(saddr, lbo, sbo) | (2ull << 61);
}

enum Fmt : uint32_t { F16 = 0, BF16 = 1, TF32 = 2 };

// kind::f16 / kind::tf32 instruction descriptor, fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc(int M, int N, uint32_t ab_fmt, bool a_mn_major, bool b_mn_major,
                                             bool a_neg = false) {
    return (1u << 4)                               // D format: F32
           | (ab_fmt << 7) | (ab_fmt << 10)        // A, B formats
           | ((a_neg ? 1u : 0u) << 13)
           | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16)
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ TMEM
// Warp-collective: the calling warp allocates `cols` columns (power of 2,
// >= 32) and the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Make generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void fence_smem_to_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------- MMA
// One lane of a converged warp (elect.sync over the full mask).  MMAs are
// issued by the elected lane with the rest of its warp waiting at the
// following __syncwarp(), which issues faster than a lone divergent thread.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(pred));
    return pred != 0;
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                        bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate ? 1u : 0u));
}
// A operand from TMEM (M = 128 rows in lanes 0..127; a K = 16 step spans 8
// columns, two 16-bit values per column, the lower k in the low half).
__device__ __forceinline__ void mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t id,
                                           bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(id), "r"(accumulate ? 1u : 0u));
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accumulate ? 1u : 0u));
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// -------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
// One poll.  When the phase is still open the thread is suspended in
// hardware until it completes or about `suspend_ns` nanoseconds pass, so
// waiting warps leave the issue slots and the shared-memory pipe to the
// warps that work.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase, uint32_t suspend_ns = 1000) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}
// Wait for the phase with parity `phase` to complete, at most `limit` polls
// (about a second with the suspension honoured, far less if every poll
// returns at once).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t phase, int *err, uint32_t limit = 1u << 20) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, phase)) return true;
    if (err) atomicExch(err, 1);
    return false;
}

// ------------------------------------------- bulk copies (untiled TMA)
// Addresses 16-byte aligned, sizes multiples of 16 bytes.  No multicast.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// global -> shared, completion counted on `bar` (transaction bytes).
__device__ __forceinline__ void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(smem_dst)),
                 "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}
// shared -> global, tracked by bulk groups of the issuing thread.
__device__ __forceinline__ void bulk_store(void *gdst, const void *smem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(smem_src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed groups still read their shared source.
template <int N> __device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed groups are still incomplete.
template <int N> __device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------- TMEM <-> regs
// 32 lanes x 16 consecutive 32-bit columns: thread t gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// The same for 32-bit integer accumulators (kind::i8).
__device__ __forceinline__ void tmem_ld16i(uint32_t taddr, int (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])));
}
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// After tmem_wait_ld: make later uses of registers filled by tcgen05.ld depend
// on a statement that follows the wait, so the compiler cannot hoist them
// above it (the wait itself names no registers).
__device__ __forceinline__ void reg_fence16(float *v) {
    asm volatile(""
                 : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7]),
                   "+f"(v[8]), "+f"(v[9]), "+f"(v[10]), "+f"(v[11]), "+f"(v[12]), "+f"(v[13]), "+f"(v[14]),
                   "+f"(v[15]));
}
__device__ __forceinline__ void reg_fence16i(int *v) {
    asm volatile(""
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                   "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                   "+r"(v[15]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) {
    return base + (lane << 16) + col;
}

// ------------------------------------------------------ layout offsets
// Byte offset of element (r, k) in a K-major 16-bit tile with KK k-columns.
__host__ __device__ constexpr uint32_t kmaj16(uint32_t r, uint32_t k, uint32_t KK) {
    return (r >> 3) * (KK / 8) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
}
// Byte offset of element (k, c) in an MN-major 16-bit tile with CC mn-columns.
__host__ __device__ constexpr uint32_t mnmaj16(uint32_t k, uint32_t c, uint32_t CC) {
    return (k >> 3) * (CC / 8) * 128 + (c >> 3) * 128 + (k & 7) * 16 + (c & 7) * 2;
}
// Descriptor of K-step `ks` (16 k's) of a K-major 16-bit tile with KK columns.
__device__ __forceinline__ uint64_t desc_kmaj16(const void *tile, uint32_t KK, uint32_t ks) {
    return smem_desc(smem_addr(tile) + ks * 256, 128, (KK / 8) * 128);
}
// Descriptor of K-step `ks` of an MN-major 16-bit tile with CC mn-columns.
__device__ __forceinline__ uint64_t desc_mnmaj16(const void *tile, uint32_t CC, uint32_t ks) {
    return smem_desc(smem_addr(tile) + ks * 2 * (CC / 8) * 128, (CC / 8) * 128, 128);
}
// 32-bit (tf32) K-major: 4 k's per 16 bytes; one kind::tf32 MMA consumes K = 8.
__host__ __device__ constexpr uint32_t kmaj32(uint32_t r, uint32_t k, uint32_t KK) {
    return (r >> 3) * (KK / 4) * 128 + (k >> 2) * 128 + (r & 7) * 16 + (k & 3) * 4;
}
__device__ __forceinline__ uint64_t desc_kmaj32(const void *tile, uint32_t KK, uint32_t ks) {
    return smem_desc(smem_addr(tile) + ks * 256, 128, (KK / 4) * 128);
}

}  // namespace umma
}  // namespace gdn
