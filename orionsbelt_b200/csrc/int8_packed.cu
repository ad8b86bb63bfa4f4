// int8_packed.cu -- the int8-weight matmul of the reference's INT8_WEIGHTS
// decode path (matmul_int8 -> gemv_int8_neon / gemm_int8_neon,
// src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:296-358, 608-681) for
// a few activation rows, streamed from HBM through the tcgen05 int8 tensor
// cores over weights packed once into a streaming layout.
//
// C[m][n] = s[n] * sum_k A[m][k] q[k][n].
//
// Activations as fixed point.  A preparation kernel gives each row m one
// scale S_m = max_k |A[m][k]| and writes x = A[m][k] * 127 / S_m as three
// signed bytes, x ~ t0 + t1 / 254 + t2 / 254^2 (t0 = rint(x), t1 = rint((x -
// t0) * 254), t2 = rint(((x - t0) * 254 - t1) * 254), all in [-127, 127]):
// the representation error of an element is at most S_m * 2^-24, the size of
// one fp32 rounding of the row's largest element.  The MMA then computes,
// exactly in int32, D_t[n][m] = sum_k q[k][n] t_k[m][k] for the three terms,
// and
//   C[m][n] = s[n] * S_m / (127 * 254^2) * (D_0 * 254^2 + D_1 * 254 + D_2),
// the bracket an exact integer (|.| < 2^53 for K <= 2^17).  Exact integer
// partial sums make the K split order-free: K parts of a tile are added with
// 64-bit integer atomics and the result does not depend on how the work was
// split or in which order parts arrive (deterministic by construction).
//
// MMA (kind::i8, cta_group::1): D [128 weight columns][48] += W^T . T^T with
//   A operand  the packed weights, K-major, straight from the ring;
//   B operand  the activation terms of 16 rows (t0 rows 0-15, t1 16-31,
//              t2 32-47), K-major;
//   D          int32 in TMEM, 48 columns per 128-column half tile.
// No operand conversion happens on the SM: a stage is two bulk copies and
// four MMAs.
//
// Packed layout (int8_pack_weights): tiles of 256 columns, each tile's K in
// stages of 64 rows, a stage [4 k-groups][256 columns][16 k's] of the signed
// codes (the no-swizzle K-major operand layout: core matrices of 8 columns x
// 16 k's, 128 bytes apart along the columns, 4 KB apart along k), so one
// stage is one contiguous 16 KB bulk copy; rows k >= K and columns n >= N
// hold 0.  Activation terms: [row block of 16][stage][4][48][16] bytes.
//
// Work split (stream-K): the units (tile, stage), tile-major, are divided
// evenly over one wave of CTAs (one per SM), so every SM streams the same
// number of stages whatever the shape.  A CTA's run covers whole tiles in
// the middle and at most a partial tile at each end; a whole tile is written
// straight to C, a partial one is added into a per-tile int64 accumulator
// and the last contributor to arrive converts it, writes C and clears it.
//
// Roles (320 threads): warp 0 fills the ring, warp 1 issues the MMAs, warps
// 2-9 are the epilogue (two per TMEM lane quarter, one per tile half).
// Every wait is bounded: a timeout sets the library's device error word and
// the CTA winds down, still counting itself (marked) in every partial tile
// it owes, so the tile counters and accumulators always return to zero.
//
// Programmatic dependent launch: weights never depend on earlier kernels, so
// the first stages are requested before griddepcontrol.wait; activation
// terms are read and outputs written only after it.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "gdn_internal.cuh"
#include "int8_terms.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int PT = 256;                // columns per tile (two MMA M-tiles)
constexpr int PK = 64;                 // k rows per stage
constexpr int PMT = 16;                // activation rows per pass
constexpr int PNM = 3 * PMT;           // MMA N: t0, t1, t2 rows
constexpr int W_BYTES = PK * PT;       // packed weights per stage
constexpr int T_BYTES = PK * PNM;      // activation terms per stage
constexpr int STAGE = W_BYTES + T_BYTES;
constexpr int NSTG = 11;               // ring depth
constexpr int NEPI = 8;
constexpr int W_PROD = 0, W_MMA = 1, W_EPI0 = 2;
constexpr int PNT = (W_EPI0 + NEPI) * 32;
constexpr int TM_COLS = 256;           // [2 sets][2 halves][PNM] int32
constexpr size_t PSMEM = 1024 + (size_t)NSTG * STAGE;
constexpr long long KMAX = 1ll << 17;  // int32 accumulators stay exact
constexpr float TERM_INV = (float)(1.0 / (127.0 * 254.0 * 254.0));
static_assert(2 * 2 * PNM <= TM_COLS, "TMEM budget");
static_assert(PSMEM <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t id, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(acc ? 1u : 0u));
}
// kind::i8 instruction descriptor: D s32, A and B signed 8-bit, K-major.
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D_0 254^2 + D_1 254 + D_2, exact
__device__ __forceinline__ long long term_sum(int d0, int d1, int d2) {
    return (long long)d0 * 64516 + (long long)d1 * 254 + (long long)d2;
}

struct Split {
    long long U, G, S;  // units, CTAs, stages per tile
    __device__ __forceinline__ long long lo(long long g) const { return g * U / G; }
    // the CTA whose run holds unit u
    __device__ __forceinline__ long long cta_of(long long u) const {
        long long g = u * G / U;
        while (g + 1 < G && lo(g + 1) <= u) ++g;
        while (g > 0 && lo(g) > u) --g;
        return g;
    }
};

// One CTA per activation row: S_m and the three terms of every k (zeros for
// k >= K up to the last stage).  terms [M/RB blocks][S][4][3 RB][16]: per
// stage and k-group, the RB rows of t0, then of t1, then of t2 (RB = 16 for
// the stream kernel, 64 for the row-tiled GEMM).
__global__ void __launch_bounds__(256) act_terms_kernel(const float *__restrict__ A, int8_t *__restrict__ terms,
                                                        float *__restrict__ scale, long long K, long long S, int RB) {
    pdl_trigger();  // the matmul may start streaming its weights meanwhile
    const int m = blockIdx.x, t = threadIdx.x;
    const float *a = A + (long long)m * K;
    __shared__ float red[8];
    float mx = 0.f;
    for (long long k = t; k < K; k += 256) mx = fmaxf(mx, fabsf(a[k]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (t % 32 == 0) red[t / 32] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, red[i]);
    if (K % 16 == 0) {  // 16-byte stores of whole k-groups
        terms::write_row(a, K, S, mx, terms, scale, RB, m);
        return;
    }
    if (t == 0) scale[m] = mx;
    const float inv = mx > 0.f ? 127.0f / mx : 0.f;
    const long long sb = 3ll * RB * PK;  // bytes of one stage of a row block
    int8_t *blk = terms + (long long)(m / RB) * S * sb;
    const int r = m % RB;
    for (long long k = t; k < S * PK; k += 256) {
        float x = k < K ? a[k] * inv : 0.f;
        const float t0 = rintf(x);
        x = (x - t0) * 254.0f;
        const float t1 = rintf(x);
        const float t2 = rintf((x - t1) * 254.0f);
        int8_t *p = blk + (k / PK) * sb + ((k % PK) / 16) * (3 * RB * 16) + (k % 16);
        p[r * 16] = (int8_t)(int)t0;
        p[(RB + r) * 16] = (int8_t)(int)t1;
        p[(2 * RB + r) * 16] = (int8_t)(int)t2;
    }
}

// Grid: G CTAs (G <= SMs), PNT threads.  qp packed weights, terms / scale
// for this pass's 16 rows, s [N], C [M][N]; acc [tiles][PMT][PT] int64 and
// ctr [tiles] zero between calls.
__global__ void __launch_bounds__(PNT, 1)
    int8_packed_kernel(const int8_t *__restrict__ qp, const int8_t *__restrict__ terms,
                       const float *__restrict__ scale, const float *__restrict__ s, float *__restrict__ C, int M,
                       long long N, long long S, long long U, unsigned long long *__restrict__ acc,
                       unsigned int *__restrict__ ctr, int *err) {
    extern __shared__ unsigned char dsm_raw[];
    unsigned char *ring = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);  // [NSTG][STAGE]
    __shared__ uint64_t full[NSTG], empty[NSTG], accf[2], acce[2];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_bad;
    __shared__ unsigned int s_fix;  // bit 0: last arrival of the tile, bit 1: a contributor timed out

    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const Split sp{U, (long long)gridDim.x, S};
    const long long g = blockIdx.x, u0 = sp.lo(g), u1 = sp.lo(g + 1);
    const int n_units = (int)(u1 - u0);

    const int pre = min(n_units, NSTG);
    if (t == 0) {
        for (int i = 0; i < NSTG; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], NEPI);
        }
        s_bad = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // weights never depend on earlier kernels: the first stages go out now
        for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], STAGE);
            bulk_load(ring + i * STAGE, qp + (u0 + i) * W_BYTES, W_BYTES, &full[i]);
        }
    }
    if (warp == W_MMA) tmem_alloc(&tmem_slot, TM_COLS);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_slot;
    pdl_trigger();

    if (warp == W_PROD) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < pre; ++i)
                bulk_load(ring + i * STAGE + W_BYTES, terms + ((u0 + i) % S) * T_BYTES, T_BYTES, &full[i]);
            int issued = pre;
            for (; issued < n_units; ++issued) {
                const int slot = issued % NSTG;
                if (s_bad || !mbar_wait(&empty[slot], (uint32_t)(((issued / NSTG) - 1) & 1), err)) {
                    s_bad = 1;
                    break;
                }
                const long long u = u0 + issued;
                mbar_arrive_expect_tx(&full[slot], STAGE);
                bulk_load(ring + slot * STAGE, qp + u * W_BYTES, W_BYTES, &full[slot]);
                bulk_load(ring + slot * STAGE + W_BYTES, terms + (u % S) * T_BYTES, T_BYTES, &full[slot]);
            }
            // every copy issued lands before the CTA may leave
            for (int i = max(0, issued - NSTG); i < issued; ++i)
                mbar_wait(&full[i % NSTG], (uint32_t)((i / NSTG) & 1), err);
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        // ----------------------------------------------------------- MMA
        constexpr uint32_t id = idesc_s8(128, PNM);
        long long u = u0;
        int i = 0, j = 0;
        bool issued_any = false;
        while (u < u1 && !s_bad) {
            const long long tile = u / S, seg_end = min(u1, (tile + 1) * S);
            const int set = j & 1;
            if (j >= 2 && !mbar_wait(&acce[set], (uint32_t)(((j >> 1) - 1) & 1), err)) {
                s_bad = 1;
                break;
            }
            fence_after_sync();
            for (long long uu = u; uu < seg_end; ++uu, ++i) {
                const int slot = i % NSTG;
                if (s_bad || !mbar_wait(&full[slot], (uint32_t)((i / NSTG) & 1), err)) {
                    s_bad = 1;
                    break;
                }
                fence_after_sync();
                if (elect_one()) {
                    const unsigned char *st = ring + slot * STAGE;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int ks = 0; ks < PK / 32; ++ks)
                            mma_i8(tmem + set * 2 * PNM + h * PNM,
                                   smem_desc(smem_addr(st) + ks * 2 * 4096 + h * 128 * 16, 4096, 128),
                                   smem_desc(smem_addr(st + W_BYTES) + ks * 2 * (PNM * 16), PNM * 16, 128), id,
                                   uu > u || ks > 0);
                    commit(&empty[slot]);
                    if (uu + 1 == seg_end) commit(&accf[set]);
                }
                __syncwarp();
                issued_any = true;
            }
            if (s_bad) break;
            u = seg_end;
            ++j;
        }
        // on a timeout: the MMAs already issued finish before TMEM is freed
        if (s_bad && issued_any) mbar_wait(&empty[(i - 1) % NSTG], (uint32_t)(((i - 1) / NSTG) & 1), err);
    } else {
        // ------------------------------------------------------- epilogue
        const int et = t - W_EPI0 * 32, q4 = warp & 3, hf = (warp - W_EPI0) >> 2;
        const int cc = hf * 128 + q4 * 32 + lane;  // this thread's column of the tile
        pdl_wait();
        float f[PMT];  // S_m / (127 * 254^2)
#pragma unroll
        for (int m = 0; m < PMT; ++m) f[m] = m < M ? scale[m] * TERM_INV : 0.f;
        bool bad = false;
        long long u = u0;
        int j = 0;
        while (u < u1) {
            const long long tile = u / S, seg_end = min(u1, (tile + 1) * S);
            const bool whole = u == tile * S && seg_end == (tile + 1) * S;
            const int set = j & 1;
            if (!bad && (s_bad || !mbar_wait(&accf[set], (uint32_t)((j >> 1) & 1), err))) {
                s_bad = 1;
                bad = true;
            }
            fence_after_sync();
            const long long n = tile * PT + cc;
            if (!bad) {
                int d0[16], d1[16], d2[16];
                const uint32_t c0 = set * 2 * PNM + hf * PNM;
                tmem_ld16i(taddr(tmem, 32 * q4, c0), d0);
                tmem_ld16i(taddr(tmem, 32 * q4, c0 + PMT), d1);
                tmem_ld16i(taddr(tmem, 32 * q4, c0 + 2 * PMT), d2);
                tmem_wait_ld();
                reg_fence16i(d0);
                reg_fence16i(d1);
                reg_fence16i(d2);
                if (whole) {
                    if (n < N) {
                        const float sc = s[n];
#pragma unroll
                        for (int m = 0; m < PMT; ++m)
                            if (m < M) C[(long long)m * N + n] = (float)term_sum(d0[m], d1[m], d2[m]) * (f[m] * sc);
                    }
                } else {
                    unsigned long long *ta = acc + (size_t)tile * PMT * PT + cc;
#pragma unroll
                    for (int m = 0; m < PMT; ++m)
                        if (m < M) atomicAdd(ta + m * PT, (unsigned long long)term_sum(d0[m], d1[m], d2[m]));
                }
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[set]);
            if (!whole) {
                // the last contributor to arrive converts the tile
                __threadfence();
                epi_sync();
                const long long gf = sp.cta_of(tile * S), gl = sp.cta_of((tile + 1) * S - 1);
                if (et == 0) {
                    const unsigned int mine = bad ? 0x10001u : 1u;
                    const unsigned int old = atomicAdd(&ctr[tile], mine);
                    const bool last = (old & 0xFFFFu) == (unsigned)(gl - gf);
                    s_fix = (last ? 1u : 0u) | (((old + mine) >> 16) != 0u ? 2u : 0u);
                }
                epi_sync();
                const unsigned int fx = s_fix;
                if (fx & 1u) {
                    __threadfence();
                    unsigned long long *ta = acc + (size_t)tile * PMT * PT + cc;
                    const float sc = n < N ? s[n] : 0.f;
                    // read every row's sum (all loads in flight at once), clear, convert
                    // (returning atomics here measured 3 us slower: they serialise)
                    long long v[PMT];
#pragma unroll
                    for (int m = 0; m < PMT; ++m) v[m] = m < M ? (long long)__ldcg(ta + m * PT) : 0ll;
#pragma unroll
                    for (int m = 0; m < PMT; ++m)
                        if (m < M) __stcg(ta + m * PT, 0ull);
                    if (!(fx & 2u) && n < N) {
#pragma unroll
                        for (int m = 0; m < PMT; ++m)
                            if (m < M) C[(long long)m * N + n] = (float)v[m] * (f[m] * sc);
                    }
                    if (et == 0) ctr[tile] = 0u;
                }
                epi_sync();
            }
            u = seg_end;
            ++j;
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == W_MMA) {
        fence_after_sync();
        tmem_dealloc(tmem, TM_COLS);
    }
}

// Row-tiled GEMM for many activation rows (a prompt): CTA = (64 rows, 128
// weight columns = half of a packed tile), the whole K, no split.  D^T
// [128 columns][64 rows] per term in TMEM (three int32 accumulators, 192
// columns); per 64-k stage two bulk-copy groups (the weight half's four
// 2 KB k-groups, the 12 KB of activation terms) and six MMAs (3 terms x 2 K
// steps of 32).  Two CTAs per SM, so one CTA's epilogue overlaps the other's
// main loop.  Warp 0 loads, warp 1 issues, warps 2-5 write C (lane = weight
// column, so stores are coalesced).
constexpr int GR = 64, GC = 128;
constexpr int GW_BYTES = PK * GC, GT_BYTES = 3 * GR * PK, GSTAGE = GW_BYTES + GT_BYTES;
constexpr int GNSTG = 5;
constexpr int GNT = 6 * 32;
constexpr size_t GSMEM = 1024 + (size_t)GNSTG * GSTAGE;

__global__ void __launch_bounds__(GNT, 2)
    int8_gemm_kernel(const int8_t *__restrict__ qp, const int8_t *__restrict__ terms, const float *__restrict__ scale,
                     const float *__restrict__ s, float *__restrict__ C, long long M, long long N, long long S,
                     long long ncol_tiles, int *err) {
    extern __shared__ unsigned char dsm_raw[];
    unsigned char *ring = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);  // [GNSTG][GSTAGE]
    __shared__ uint64_t full[GNSTG], empty[GNSTG], accf;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int s_bad;
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const long long ct = (long long)blockIdx.x % ncol_tiles, rt = (long long)blockIdx.x / ncol_tiles;
    const long long ptile = ct / 2, half = ct % 2, n0 = ct * GC, m0 = rt * GR;
    const int pre = (int)min((long long)GNSTG, S);
    auto load_w = [&](int st, int slot) {
        unsigned char *dst = ring + slot * GSTAGE;
#pragma unroll
        for (int kg = 0; kg < 4; ++kg)
            bulk_load(dst + kg * 2048, qp + ((ptile * S + st) * 4 + kg) * 4096 + half * 2048, 2048, &full[slot]);
    };
    if (t == 0) {
        for (int i = 0; i < GNSTG; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(&accf, 1);
        s_bad = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < pre; ++i) {  // weights never depend on earlier kernels
            mbar_arrive_expect_tx(&full[i], GSTAGE);
            load_w(i, i);
        }
    }
    if (warp == W_MMA) tmem_alloc(&tmem_slot, 256);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_slot;
    pdl_trigger();
    if (warp == W_PROD) {
        if (lane == 0) {
            pdl_wait();
            for (int i = 0; i < pre; ++i)
                bulk_load(ring + i * GSTAGE + GW_BYTES, terms + (rt * S + i) * GT_BYTES, GT_BYTES, &full[i]);
            int issued = pre;
            for (; issued < S; ++issued) {
                const int slot = issued % GNSTG;
                if (s_bad || !mbar_wait(&empty[slot], (uint32_t)(((issued / GNSTG) - 1) & 1), err)) {
                    s_bad = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], GSTAGE);
                load_w(issued, slot);
                bulk_load(ring + slot * GSTAGE + GW_BYTES, terms + (rt * S + issued) * GT_BYTES, GT_BYTES,
                          &full[slot]);
            }
            for (int i = max(0, issued - GNSTG); i < issued; ++i)
                mbar_wait(&full[i % GNSTG], (uint32_t)((i / GNSTG) & 1), err);
        }
        __syncwarp();
    } else if (warp == W_MMA) {
        constexpr uint32_t id = idesc_s8(128, GR);
        int done = 0;
        for (int st = 0; st < S; ++st) {
            const int slot = st % GNSTG;
            if (s_bad || !mbar_wait(&full[slot], (uint32_t)((st / GNSTG) & 1), err)) {
                s_bad = 1;
                break;
            }
            fence_after_sync();
            if (elect_one()) {
                const uint32_t a = smem_addr(ring + slot * GSTAGE), b = a + GW_BYTES;
#pragma unroll
                for (int tm = 0; tm < 3; ++tm)
#pragma unroll
                    for (int ks = 0; ks < PK / 32; ++ks)
                        mma_i8(tmem + tm * GR, smem_desc(a + ks * 2 * 2048, 2048, 128),
                               smem_desc(b + tm * GR * 16 + ks * 2 * (3 * GR * 16), 3 * GR * 16, 128), id,
                               st > 0 || ks > 0);
                commit(&empty[slot]);
                if (st + 1 == S) commit(&accf);
            }
            __syncwarp();
            done = st + 1;
        }
        if (s_bad && done > 0) mbar_wait(&empty[(done - 1) % GNSTG], (uint32_t)(((done - 1) / GNSTG) & 1), err);
    } else {
        const int q4 = warp & 3;
        const long long n = n0 + 32 * q4 + lane;
        pdl_wait();
        bool ok = !s_bad && mbar_wait(&accf, 0, err);
        if (!ok) s_bad = 1;
        fence_after_sync();
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            const float sc = n < N ? s[n] : 0.f;
#pragma unroll
            for (int rc = 0; rc < GR; rc += 16) {
                int d0[16], d1[16], d2[16];
                tmem_ld16i(taddr(tmem, 32 * q4, rc), d0);
                tmem_ld16i(taddr(tmem, 32 * q4, GR + rc), d1);
                tmem_ld16i(taddr(tmem, 32 * q4, 2 * GR + rc), d2);
                tmem_wait_ld();
                reg_fence16i(d0);
                reg_fence16i(d1);
                reg_fence16i(d2);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const long long r = m0 + rc + i;
                    if (r < M && n < N)
                        C[r * N + n] = (float)term_sum(d0[i], d1[i], d2[i]) * (scale[r] * TERM_INV * sc);
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == W_MMA) {
        fence_after_sync();
        tmem_dealloc(tmem, 256);
    }
}

__global__ void pack_kernel(const int8_t *__restrict__ q, int8_t *__restrict__ qp, long long K, long long N,
                            long long S, long long chunks) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < chunks;
         e += (long long)gridDim.x * blockDim.x) {
        // e = ((tile * S + stage) * 4 + kg) * PT + c: 16 k's of column c
        const long long c = e % PT, kg = (e / PT) % 4, stage = (e / (4 * PT)) % S, tile = e / (4 * PT * S);
        const long long n = tile * PT + c, k0 = stage * PK + kg * 16;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (n < N) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (k0 + i < K) w[i / 4] |= (uint32_t)(uint8_t)q[(k0 + i) * N + n] << (8 * (i % 4));
        }
        *reinterpret_cast<uint4 *>(qp + e * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Per-stream workspace: activation terms and scales (grown on demand), and
// the per-tile accumulators and counters (zero between calls).
struct PackedWs {
    int device;
    cudaStream_t stream;
    int8_t *terms;
    float *scale;
    unsigned long long *acc;
    unsigned int *ctr;
    size_t nterms, nscale, ntiles;
};
std::mutex g_pws_mu;
std::vector<PackedWs> g_pws;

int packed_workspace(cudaStream_t st, size_t nterms, size_t nscale, size_t ntiles, PackedWs *out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8_packed: cudaGetDevice");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_pws_mu);
    PackedWs *e = nullptr;
    for (auto &x : g_pws)
        if (x.device == dev && x.stream == st) e = &x;
    if (!e) {
        g_pws.push_back({dev, st, nullptr, nullptr, nullptr, nullptr, 0, 0, 0});
        e = &g_pws.back();
    }
    // cudaFree waits for the device, so nothing in flight still uses a buffer
    if (e->nterms < nterms) {
        if ((rc = check_cuda(cudaFree(e->terms), "matmul_int8_packed: cudaFree"))) return rc;
        e->terms = nullptr;
        e->nterms = 0;
        if ((rc = check_cuda(cudaMalloc(&e->terms, nterms), "matmul_int8_packed: cudaMalloc"))) return rc;
        e->nterms = nterms;
    }
    if (e->nscale < nscale) {
        if ((rc = check_cuda(cudaFree(e->scale), "matmul_int8_packed: cudaFree"))) return rc;
        e->scale = nullptr;
        e->nscale = 0;
        const size_t n = std::max<size_t>(nscale, 256);
        if ((rc = check_cuda(cudaMalloc(&e->scale, n * sizeof(float)), "matmul_int8_packed: cudaMalloc"))) return rc;
        e->nscale = n;
    }
    if (e->ntiles < ntiles) {
        if ((rc = check_cuda(cudaFree(e->acc), "matmul_int8_packed: cudaFree"))) return rc;
        if ((rc = check_cuda(cudaFree(e->ctr), "matmul_int8_packed: cudaFree"))) return rc;
        e->acc = nullptr;
        e->ctr = nullptr;
        e->ntiles = 0;
        const size_t n = std::max<size_t>(ntiles, 64);
        const size_t abytes = n * PMT * PT * sizeof(unsigned long long);
        if ((rc = check_cuda(cudaMalloc(&e->acc, abytes), "matmul_int8_packed: cudaMalloc"))) return rc;
        if ((rc = check_cuda(cudaMalloc(&e->ctr, n * sizeof(unsigned int)), "matmul_int8_packed: cudaMalloc")))
            return rc;
        if ((rc = check_cuda(cudaMemsetAsync(e->acc, 0, abytes, st), "matmul_int8_packed: memset"))) return rc;
        if ((rc = check_cuda(cudaMemsetAsync(e->ctr, 0, n * sizeof(unsigned int), st), "matmul_int8_packed: memset")))
            return rc;
        e->ntiles = n;
    }
    *out = *e;
    return KAI_GDN_OK;
}

// Many rows: activation terms in blocks of 64 rows, then the row-tiled GEMM
// (a programmatic dependent of the terms kernel).
int run_gemm(const float *A, const int8_t *qp, const float *s, float *C, size_t M, size_t K, size_t N,
             cudaStream_t st) {
    const long long S = (long long)((K + PK - 1) / PK), ncol = (long long)((N + GC - 1) / GC);
    const long long rows = (long long)((M + GR - 1) / GR), grid = ncol * rows;
    if (grid > 0x7fffffffll || M > 0x7fffffffull) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8_packed: shape");
    PackedWs ws{};
    int rc = packed_workspace(st, (size_t)rows * (size_t)S * GT_BYTES, (size_t)rows * GR, 0, &ws);
    if (rc) return rc;
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    act_terms_kernel<<<(unsigned)M, 256, 0, st>>>(A, ws.terms, ws.scale, (long long)K, S, GR);
    if ((rc = check_launch("act_terms_kernel"))) return rc;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(GNT);
    cfg.dynamicSmemBytes = GSMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, int8_gemm_kernel, qp, (const int8_t *)ws.terms,
                                              (const float *)ws.scale, s, C, (long long)M, (long long)N, S, ncol, err);
    if (le != cudaSuccess) return check_cuda(le, "int8_gemm_kernel launch");
    return check_launch("int8_gemm_kernel");
}

}  // namespace

bool int8_packed_supported(size_t K, size_t N) {
    return K > 0 && N > 0 && N % 16 == 0 && (long long)K <= KMAX && N < (1ull << 31);
}

size_t int8_packed_bytes(size_t K, size_t N) {
    return (N + PT - 1) / PT * ((K + PK - 1) / PK) * (size_t)W_BYTES;
}

int int8_pack_weights(const int8_t *q, int8_t *qp, size_t K, size_t N, cudaStream_t st) {
    if (!q || !qp) return set_error(KAI_GDN_ERR_INVALID, "int8_pack: null pointer");
    if (!int8_packed_supported(K, N) || (uintptr_t)qp % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "int8_pack: N %% 16, K <= 131072 and a 16-byte aligned output");
    const long long S = (long long)((K + PK - 1) / PK), chunks = (long long)(int8_packed_bytes(K, N) / 16);
    pack_kernel<<<(unsigned)std::min<long long>((chunks + 255) / 256, 16ll * sm_count()), 256, 0, st>>>(
        q, qp, (long long)K, (long long)N, S, chunks);
    return check_launch("int8_pack_kernel");
}

namespace {
int packed_attrs() {
    static std::atomic<unsigned long long> attr_set{0};  // per device
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8_packed: cudaGetDevice");
    if (rc) return rc;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        if ((rc = check_cuda(cudaFuncSetAttribute(int8_packed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)PSMEM),
                             "matmul_int8_packed: smem attribute")))
            return rc;
        if ((rc = check_cuda(cudaFuncSetAttribute(int8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  (int)GSMEM),
                             "matmul_int8_packed: smem attribute")))
            return rc;
        attr_set.fetch_or(bit);
    }
    return KAI_GDN_OK;
}
}  // namespace

int launch_matmul_int8_packed(const float *A, const int8_t *qp, const float *s, float *C, size_t M, size_t K,
                              size_t N, cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!A || !qp || !s || !C) return set_error(KAI_GDN_ERR_INVALID, "matmul_int8_packed: null pointer");
    if (!int8_packed_supported(K, N) || (uintptr_t)qp % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED,
                         "matmul_int8_packed: N %% 16, K <= 131072 and 16-byte aligned packed weights");
    if (M > 0x7fffffffull) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8_packed: M too large");
    int rc = packed_attrs();
    if (rc) return rc;
    if (M > (size_t)PMT) return run_gemm(A, qp, s, C, M, K, N, st);
    const long long S = (long long)((K + PK - 1) / PK);
    PackedWs ws{};
    if ((rc = packed_workspace(st, (size_t)S * T_BYTES, PMT, 0, &ws))) return rc;
    act_terms_kernel<<<(unsigned)M, 256, 0, st>>>(A, ws.terms, ws.scale, (long long)K, S, PMT);
    if ((rc = check_launch("act_terms_kernel"))) return rc;
    return launch_matmul_int8_packed_terms(ws.terms, ws.scale, qp, s, C, M, K, N, st);
}

size_t int8_terms_bytes(size_t M, size_t K) {
    return (M + PMT - 1) / PMT * ((K + PK - 1) / PK) * (size_t)T_BYTES;
}

// The weight stream over activation terms already in place (the 16-row
// layout of int8_terms.cuh, scales [M]): one pass over the weights per 16
// rows, each a programmatic dependent of the kernel before it.
int launch_matmul_int8_packed_terms(const int8_t *terms, const float *scale, const int8_t *qp, const float *s,
                                    float *C, size_t M, size_t K, size_t N, cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!terms || !scale || !qp || !s || !C) return set_error(KAI_GDN_ERR_INVALID, "matmul_int8_packed: null pointer");
    if (!int8_packed_supported(K, N) || (uintptr_t)qp % 16 || (uintptr_t)terms % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8_packed: shape or alignment");
    int rc = packed_attrs();
    if (rc) return rc;
    const long long S = (long long)((K + PK - 1) / PK), tiles = (long long)((N + PT - 1) / PT), U = tiles * S;
    const long long G = std::min<long long>(U, sm_count());
    const size_t blocks = (M + PMT - 1) / PMT;
    PackedWs ws{};
    if ((rc = packed_workspace(st, 0, 0, (size_t)tiles, &ws))) return rc;
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    for (size_t b = 0; b < blocks; ++b) {
        const size_t r0 = b * PMT, rows = std::min<size_t>(PMT, M - r0);
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)G);
        cfg.blockDim = dim3(PNT);
        cfg.dynamicSmemBytes = PSMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t le =
            cudaLaunchKernelEx(&cfg, int8_packed_kernel, qp, terms + b * (size_t)S * T_BYTES, scale + r0, s,
                               C + r0 * N, (int)rows, (long long)N, S, U, ws.acc, ws.ctr, err);
        if (le != cudaSuccess) return check_cuda(le, "int8_packed_kernel launch");
        if ((rc = check_launch("int8_packed_kernel"))) return rc;
    }
    return KAI_GDN_OK;
}

}  // namespace gdn
