// chunk_tc32.cu -- the chunkwise gated delta-rule scan for fp32 inputs on the
// tensor cores (sm_100a), fp32-accurate.
//
// Same algorithm and conventions as chunk.cu (the chunked form of
// docs/GDN_ARCHITECTURE_AUDIT.md:142-153).  Per (b, value head) and chunk of
// 64 tokens, G the in-chunk cumulative log decay:
//   A  = beta_r (k_r . k_s) e^{G_r - G_s}          s <  r
//   P  = scale (q_r . k_s) e^{G_r - G_s}           s <= r
//   Tb = (I + A)^-1 diag(beta),   R = P Tb
//   V'' = V - e^G (K S),   O = scale e^G (Q S) + R V''  (= P V', V' = Tb V'')
//   S  <- e^{G_63} S + K^T (e^{G_63 - G} Tb V'') = e^{G_63} S + W^T V'',
//         W = Tb'^T K with Tb' = diag(e^{G_63 - G}) Tb
//
// Precision: every product runs as three bf16 MMAs, hi*hi + hi*lo + lo*hi,
// with each operand split x = hi + lo (hi = bf16(x), lo = bf16(x - hi)), so
// a product carries about 16 significant bits and lo*lo (2^-18 relative) is
// the dropped term; sums accumulate in fp32 in TMEM, the state stays fp32 in
// TMEM for the whole sequence.
//
// Two launches per segment of chunks:
//  * chunk_prep_kernel -- one CTA per (b, key head, chunk), all chunks at
//    once (nothing here depends on the state): K K^T and Q K^T on tcgen05,
//    then for each value head of the group A and P, the blocked inverse on the
//    CUDA cores, Tb, R = P Tb and W = Tb'^T K on tcgen05.  It writes the MMA
//    operand images into a workspace, exactly as the recurrence's shared
//    memory holds them (no-swizzle K-major core-matrix layout, bf16 hi then lo):
//      [K;Q]          128 rows (64 of k, 64 of q) x 128 features      65536 bytes
//      [Tb;R], G, W   128 rows x 64 tokens, G, 64 rows x 128 features 65792 bytes
//  * chunk_rec_kernel -- one CTA per (b, value head, 32 value columns).  The
//    value columns of the state evolve independently, so the 32-column
//    blocks are exact splits; the state block S (128 keys x 32 values, fp32)
//    lives in TMEM.  Per chunk, on one MMA warp (M = 128, N = 32):
//      D_a  = [K;Q] S      K = 128   rows 0-63: K S, rows 64-127: Q S
//      S   += W^T V''      K = 64    A = W's image read MN-major
//      D_b  = [Tb;R] V''   K = 64    rows 64-127: R V'' (for the output only)
//    so the state's chain is two MMA batches and two element-wise passes:
//    V'' and its split (warps 4, 5: rows 0-63), and the state pass (all four
//    warps: the split copy of S for the next D_a, then S *= e^{G_63} of the
//    next chunk, back into TMEM); the output rows (warps 6, 7: Q S and R V'')
//    are written after it.  One warp issues the bulk copies: [K;Q] into a
//    single slot as soon as D_a is done with it, [Tb;R], G, W two chunks deep.
//
// Long sequences run in segments of chunks whose images fit a bounded
// workspace; the state goes through the state buffer between segments.
#include "gdn_internal.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int CH = 64;                       // chunk length
constexpr int DK = 128;                      // key features
constexpr int NV = 32;                       // value columns per recurrence CTA
constexpr int KQ_HALF = 128 * DK * 2;        // one bf16 [K;Q] image
constexpr int KQ_BYTES = 2 * KQ_HALF;        // hi + lo
constexpr int TR_HALF = 128 * CH * 2;        // one bf16 [Tb;R] image
constexpr int WK_OFF = 2 * TR_HALF + CH * 4;   // after [Tb;R] hi, lo and G: the W image
constexpr int WK_HALF = CH * DK * 2;           // one bf16 W image (64 tokens x 128 features)
constexpr int TR_BYTES = WK_OFF + 2 * WK_HALF;  // [Tb;R] hi + lo, G, W hi + lo
constexpr size_t SEG_BUDGET = 256ull << 20;  // workspace bound per launch

// ---------------------------------------------------------------- helpers
__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }

// Eight floats to their bf16 hi and lo parts, packed (lower index in the low half).
__device__ __forceinline__ void split8(const float *x, uint4 &hi, uint4 &lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 hh = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        const float2 hf = __bfloat1622float2(hh);
        h[i] = bf2_bits(hh);
        l[i] = bf2_bits(__floats2bfloat162_rn(x[2 * i] - hf.x, x[2 * i + 1] - hf.y));
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Row `k` (32 values along N) of an MN-major 16-bit operand with NV columns,
// hi image at `hi`, lo image at `lo`.
__device__ __forceinline__ void put_row_mn(unsigned char *hi, unsigned char *lo, int k, const float (&x)[NV]) {
#pragma unroll
    for (int j = 0; j < NV / 8; ++j) {
        uint4 h, l;
        split8(&x[8 * j], h, l);
        const uint32_t off = mnmaj16(k, 8 * j, NV);
        *reinterpret_cast<uint4 *>(hi + off) = h;
        *reinterpret_cast<uint4 *>(lo + off) = l;
    }
}

__device__ __forceinline__ void mbar_arrive1(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// A bounded wait whose outcome is the same for the whole warp (the
// tcgen05.ld / st that follow are warp-collective).
__device__ __forceinline__ bool wait_w(uint64_t *bar, uint32_t phase, int *err) {
    return __all_sync(0xffffffffu, mbar_wait(bar, phase, err));
}

// The same by polling (mbarrier.test_wait never suspends): for the waits on
// the recurrence's critical path, where a suspended thread measured ~200
// cycles to resume after the phase completed.  At most 2^24 polls (well
// under a second), then *err is set.
__device__ __forceinline__ bool test_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool spin_w(uint64_t *bar, uint32_t phase, int *err) {
    bool ok = false;
    for (uint32_t i = 0; i < (1u << 24) && !ok; ++i) ok = test_wait(bar, phase);
    if (!ok && err) atomicExch(err, 1);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[NV]) {
    tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(&v[0]));
    tmem_ld16(taddr + 16, *reinterpret_cast<float(*)[16]>(&v[16]));
    tmem_wait_ld();
    reg_fence16(&v[0]);
    reg_fence16(&v[16]);
}
__device__ __forceinline__ void st32(uint32_t taddr, const float (&v)[NV]) {
    tmem_st16(taddr, *reinterpret_cast<const float(*)[16]>(&v[0]));
    tmem_st16(taddr + 16, *reinterpret_cast<const float(*)[16]>(&v[16]));
    tmem_wait_st();
}

// 32 consecutive values of a row in dtype `dt` (16-byte aligned).
__device__ __forceinline__ void store32(void *base, size_t idx, int dt, const float (&x)[NV]) {
    if (dt == KAI_GDN_F32) {
        float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(base) + idx);
#pragma unroll
        for (int j = 0; j < NV / 4; ++j) p[j] = make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
        return;
    }
    uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(base) + idx);
#pragma unroll
    for (int j = 0; j < NV / 8; ++j) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = x[8 * j + 2 * i], b = x[8 * j + 2 * i + 1];
            if (dt == KAI_GDN_BF16) {
                w[i] = bf2_bits(__floats2bfloat162_rn(a, b));
            } else {
                const __half2 hv = __floats2half2_rn(a, b);
                w[i] = *reinterpret_cast<const uint32_t *>(&hv);
            }
        }
        p[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// ================================================================ prep
constexpr int PT = 256;  // threads
constexpr int LDP = 65;  // 64 x 64 fp32 work matrices
constexpr uint32_t PCOL_KK = 0, PCOL_R = 64, PCOL_W = 128, PTM_COLS = 256;

struct PrepSmem {
    union {
        unsigned char img[KQ_BYTES];  // the [K;Q] image, operands of K K^T and Q K^T, ...
        struct {
            float A[CH * LDP];
            float T[CH * LDP];
            float X[CH * LDP];  // scratch of the blocked inverse
        } w;                     // ... then, with those products in TMEM, the inverse's work
    } u;
    unsigned char pimg[2][CH * CH * 2];   // P (hi, lo): K-major A operand of R = P Tb
    unsigned char tbimg[2][CH * CH * 2];  // Tb (hi, lo): read MN-major as its B operand
    float G[CH];
    float beta[CH];
    uint64_t bar_kk, bar_r, bar_k, bar_w, bar_fin;
    uint32_t tmem;
};

__global__ void __launch_bounds__(PT, 2)
    chunk_prep_kernel(const kai_gdn_chunk_args p, unsigned char *ws_kq, unsigned char *ws_tr, long long c_begin,
                      int nc, int *err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrepSmem &sm = *reinterpret_cast<PrepSmem *>(smem_raw);
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const long long Hk = (long long)p.heads_k, Hv = (long long)p.heads_v, T = (long long)p.seq;
    const int grp = (int)(Hv / Hk);
    const long long cl = blockIdx.x % nc, bh = blockIdx.x / nc;  // bh = b * Hk + hk
    const long long b = bh / Hk, hk = bh % Hk;
    const long long c0 = (c_begin + cl) * CH;
    // the recurrence launch may be scheduled once every CTA of this grid has
    // started; it reads the images only after this grid has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (t == 0) {
        mbar_init(&sm.bar_kk, 1);
        mbar_init(&sm.bar_r, 1);
        mbar_init(&sm.bar_k, 1);
        mbar_init(&sm.bar_w, 1);
        mbar_init(&sm.bar_fin, 1);
    }
    if (warp == 0) tmem_alloc(&sm.tmem, PTM_COLS);

    // ---- k, q rows (zeros past T) into the [K;Q] image, in shared memory for
    // the MMAs below and in the workspace for the recurrence.  Unit u holds 8
    // features of one row; with u = ((row / 8) * 16 + feature group) * 8 +
    // row % 8 its K-major offset is u * 16 (contiguous stores).
    {
        const float *kg = static_cast<const float *>(p.k), *qg = static_cast<const float *>(p.q);
        unsigned char *kq = ws_kq + (size_t)(bh * nc + cl) * KQ_BYTES;
        float4 x[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int u = t + PT * i, row = (u / 128) * 8 + u % 8, g = (u / 8) % (DK / 8);
            const long long tok = c0 + row % CH;
            x[2 * i] = x[2 * i + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (tok < T) {
                const float4 *src = reinterpret_cast<const float4 *>((row < CH ? kg : qg) +
                                                                     ((size_t)(b * T + tok) * Hk + hk) * DK + 8 * g);
                x[2 * i] = __ldg(src);
                x[2 * i + 1] = __ldg(src + 1);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int u = t + PT * i;
            uint4 hv, lv;
            split8(reinterpret_cast<const float *>(&x[2 * i]), hv, lv);
            *reinterpret_cast<uint4 *>(sm.u.img + u * 16) = hv;
            *reinterpret_cast<uint4 *>(sm.u.img + KQ_HALF + u * 16) = lv;
            *reinterpret_cast<uint4 *>(kq + (size_t)u * 16) = hv;
            *reinterpret_cast<uint4 *>(kq + KQ_HALF + (size_t)u * 16) = lv;
        }
        // the K half is copied back in by a bulk copy later (async proxy)
        asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    fence_smem_to_async();
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = sm.tmem;

    // ---- D[128 x 64] = [K;Q] K^T: rows 0-63 K K^T, rows 64-127 Q K^T.  The
    // B operand (64 tokens x 128 features, K-major) is the first 64 rows of
    // the same image, so A and B share descriptors.
    if (warp == 0) {
        if (elect_one()) {
            const uint32_t id = idesc(128, CH, BF16, false, false);
#pragma unroll
            for (int ks = 0; ks < DK / 16; ++ks) {
                const uint64_t hi = desc_kmaj16(sm.u.img, DK, ks), lo = desc_kmaj16(sm.u.img + KQ_HALF, DK, ks);
                mma_f16(tm + PCOL_KK, hi, hi, id, ks > 0);
                mma_f16(tm + PCOL_KK, hi, lo, id, true);
                mma_f16(tm + PCOL_KK, lo, hi, id, true);
            }
            commit(&sm.bar_kk);
        }
        __syncwarp();
    }

    // 16 x 16 block (bi, bj) of a 64 x 64 work matrix
    auto blk = [](float *m, int bi, int bj, int rr, int cc) -> float & { return m[(16 * bi + rr) * LDP + 16 * bj + cc]; };
    float *const A = sm.u.w.A, *const Tm = sm.u.w.T, *const X = sm.u.w.X;
    const int rr = t / 16, cc = t % 16;  // this thread's element of a 16 x 16 block
    const int q4 = warp % 4, hh = warp / 4;  // TMEM lane quarter, half of the 64 columns
    const int L = 32 * q4 + lane;            // this thread's TMEM lane
    const uint32_t lq = (uint32_t)(32 * q4) << 16;
    for (int gi = 0; gi < grp; ++gi) {
        const long long h = hk * grp + gi;
        if (t < 32) {
            // in-chunk inclusive cumsum of g, two rows per lane; beta
            const long long r0 = c0 + 2 * t, r1 = r0 + 1;
            const float g0 = r0 < T ? p.g[(size_t)(b * T + r0) * Hv + h] : 0.f;
            const float g1 = r1 < T ? p.g[(size_t)(b * T + r1) * Hv + h] : 0.f;
            const float b0 = r0 < T ? p.beta[(size_t)(b * T + r0) * Hv + h] : 0.f;
            const float b1 = r1 < T ? p.beta[(size_t)(b * T + r1) * Hv + h] : 0.f;
            const float pair = g0 + g1;
            float incl = pair;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float u = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += u;
            }
            sm.G[2 * t] = incl - pair + g0;
            sm.G[2 * t + 1] = incl;
            sm.beta[2 * t] = b0;
            sm.beta[2 * t + 1] = b1;
        }
        const bool ok_kk = wait_w(&sm.bar_kk, 0, err);
        if (__syncthreads_or(!ok_kk)) break;
        fence_after_sync();
        // ---- A (s < r) into shared memory and T cleared, from the K K^T rows;
        // P (s <= r) into its operand image, from the Q K^T rows
        {
            float v[32];
            ld32(tm + lq + PCOL_KK + 32 * hh, v);
            const int r = L % CH;
            const float gr = sm.G[r];
            if (L < CH) {
                const float br = sm.beta[r];
#pragma unroll
                for (int n = 0; n < 32; ++n) {
                    const int s = 32 * hh + n;
                    A[r * LDP + s] = s < r ? br * v[n] * __expf(gr - sm.G[s]) : 0.f;
                    Tm[r * LDP + s] = 0.f;
                }
            } else {
#pragma unroll
                for (int n = 0; n < 32; ++n) {
                    const int s = 32 * hh + n;
                    v[n] = s <= r ? p.scale * v[n] * __expf(gr - sm.G[s]) : 0.f;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint4 hv, lv;
                    split8(&v[8 * j], hv, lv);
                    const uint32_t off = kmaj16(r, 32 * hh + 8 * j, CH);
                    *reinterpret_cast<uint4 *>(sm.pimg[0] + off) = hv;
                    *reinterpret_cast<uint4 *>(sm.pimg[1] + off) = lv;
                }
            }
        }
        __syncthreads();
        // ---- T = (I + A)^-1, blocked.  Diagonal 16 x 16 blocks by
        // right-looking substitution on the identity: four lanes per column
        // (rows j + 4 m on lane j), x_r reaches the group by a shuffle.
        {
            const int bi = t / 64, col = (t / 4) % 16, j = t % 4;
            float x[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) x[m] = (j + 4 * m == col) ? 1.f : 0.f;
#pragma unroll
            for (int r = 0; r < 15; ++r) {
                float xr = x[r / 4];
                xr = __shfl_sync(0xffffffffu, xr, lane - j + (r % 4));
#pragma unroll
                for (int m = 0; m < 4; ++m)
                    if (j + 4 * m > r) x[m] = fmaf(-blk(A, bi, bi, j + 4 * m, r), xr, x[m]);
            }
#pragma unroll
            for (int m = 0; m < 4; ++m) blk(Tm, bi, bi, j + 4 * m, col) = x[m];
        }
        __syncthreads();
        // Off-diagonal blocks by block forward substitution, one distance
        // d = bi - bj at a time: X = sum_{k=bj}^{bi-1} A_{bi,k} T_{k,bj}, then
        // T_{bi,bj} = -T_{bi,bi} X.
        // (every bound is a constant, so the loops unroll and the loads run
        // ahead of four independent sums; with run-time bounds each step
        // waited for its own load, ~1K cycles per distance)
#pragma unroll
        for (int d = 1; d < 4; ++d) {
#pragma unroll
            for (int bj = 0; bj + d < 4; ++bj) {
                const int bi = bj + d;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int k = 0; k < 16 * d; ++k)
                    acc[k & 3] = fmaf(A[(16 * bi + rr) * LDP + 16 * bj + k], Tm[(16 * bj + k) * LDP + 16 * bj + cc],
                                      acc[k & 3]);
                blk(X, bi, bj, rr, cc) = (acc[0] + acc[1]) + (acc[2] + acc[3]);
            }
            __syncthreads();
#pragma unroll
            for (int bj = 0; bj + d < 4; ++bj) {
                const int bi = bj + d;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int k = 0; k < 16; ++k)
                    acc[k & 3] = fmaf(blk(Tm, bi, bi, rr, k), blk(X, bi, bj, k, cc), acc[k & 3]);
                blk(Tm, bi, bj, rr, cc) = -((acc[0] + acc[1]) + (acc[2] + acc[3]));
            }
            __syncthreads();
        }
        // ---- Tb = T diag(beta): the top half of the [Tb;R] image in the
        // workspace, and in shared memory the B operand of R = P Tb; beside
        // it (in the inverse's scratch, dead now) Tb' = diag(e^{G_63 - G}) Tb,
        // the A operand of W = Tb'^T K
        unsigned char *tr = ws_tr + (size_t)((b * Hv + h) * nc + cl) * TR_BYTES;
        unsigned char *tbp = reinterpret_cast<unsigned char *>(X);
        for (int u = t; u < CH * (CH / 8); u += PT) {
            const int row = (u / 64) * 8 + u % 8, g = (u / 8) % (CH / 8);  // K-major offset u * 16
            const float el = expf(sm.G[CH - 1] - sm.G[row]);
            float x[8], y[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                x[e] = Tm[row * LDP + 8 * g + e] * sm.beta[8 * g + e];
                y[e] = x[e] * el;
            }
            uint4 hv, lv;
            split8(x, hv, lv);
            *reinterpret_cast<uint4 *>(sm.tbimg[0] + u * 16) = hv;
            *reinterpret_cast<uint4 *>(sm.tbimg[1] + u * 16) = lv;
            *reinterpret_cast<uint4 *>(tr + (size_t)u * 16) = hv;
            *reinterpret_cast<uint4 *>(tr + TR_HALF + (size_t)u * 16) = lv;
            split8(y, hv, lv);
            *reinterpret_cast<uint4 *>(tbp + u * 16) = hv;
            *reinterpret_cast<uint4 *>(tbp + CH * CH * 2 + u * 16) = lv;
        }
        if (t < CH) reinterpret_cast<float *>(tr + 2 * TR_HALF)[t] = sm.G[t];
        fence_smem_to_async();
        __syncthreads();
        // ---- R = P Tb (M = 64: rows 16 q .. 16 q + 15 in lanes 32 q .. 32 q + 15);
        // Tb's K-major image read MN-major is Tb as the B operand (K = j, N = s)
        if (warp == 0) {
            if (elect_one()) {
                const uint32_t id = idesc(64, CH, BF16, false, true);
#pragma unroll
                for (int ks = 0; ks < CH / 16; ++ks) {
                    const uint64_t ah = desc_kmaj16(sm.pimg[0], CH, ks), al = desc_kmaj16(sm.pimg[1], CH, ks);
                    const uint64_t bh = desc_mnmaj16(sm.tbimg[0], CH, ks), bl = desc_mnmaj16(sm.tbimg[1], CH, ks);
                    mma_f16(tm + PCOL_R, ah, bh, id, ks > 0);
                    mma_f16(tm + PCOL_R, ah, bl, id, true);
                    mma_f16(tm + PCOL_R, al, bh, id, true);
                }
                commit(&sm.bar_r);
            }
            __syncwarp();
        }
        const bool ok_r = wait_w(&sm.bar_r, (uint32_t)gi & 1, err);
        if (__syncthreads_or(!ok_r)) break;
        fence_after_sync();
        // K's image back into the P / Tb images' space (P Tb is done with
        // them) for W below; the copy overlaps R's readout
        if (t == 0) {
            const unsigned char *kq = ws_kq + (size_t)(bh * nc + cl) * KQ_BYTES;
            mbar_arrive_expect_tx(&sm.bar_k, 2 * CH * DK * 2);
            bulk_load(sm.pimg[0], kq, CH * DK * 2, &sm.bar_k);
            bulk_load(sm.tbimg[0], kq + KQ_HALF, CH * DK * 2, &sm.bar_k);
        }
        // ---- R: the bottom half of the [Tb;R] image
        {
            float v[32];
            ld32(tm + lq + PCOL_R + 32 * hh, v);
            if (lane < 16) {
                const int r = 16 * q4 + lane;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint4 hv, lv;
                    split8(&v[8 * j], hv, lv);
                    const uint32_t off = kmaj16(CH + r, 32 * hh + 8 * j, CH);
                    *reinterpret_cast<uint4 *>(tr + off) = hv;
                    *reinterpret_cast<uint4 *>(tr + TR_HALF + off) = lv;
                }
            }
        }
        fence_before_sync();
        __syncthreads();
        // ---- W = Tb'^T K (M = 64 tokens j, N = 128 features, K = 64 tokens r),
        // so that the recurrence's state update is S += W^T V'' straight from
        // V''.  K's image (hi, lo: the first 16 KB of each half of this chunk's
        // [K;Q] image, written above, copied back before R's readout): read
        // MN-major it is K as the B operand, and Tb''s K-major image read
        // MN-major is Tb'^T as the A operand.
        const bool ok_k = wait_w(&sm.bar_k, (uint32_t)gi & 1, err);
        if (__syncthreads_or(!ok_k)) break;
        if (warp == 0) {
            if (elect_one()) {
                const uint32_t id = idesc(64, DK, BF16, true, true);
#pragma unroll
                for (int ks = 0; ks < CH / 16; ++ks) {
                    const uint64_t ah = desc_mnmaj16(tbp, CH, ks), al = desc_mnmaj16(tbp + CH * CH * 2, CH, ks);
                    const uint64_t bh = desc_mnmaj16(sm.pimg[0], DK, ks), bl = desc_mnmaj16(sm.tbimg[0], DK, ks);
                    mma_f16(tm + PCOL_W, ah, bh, id, ks > 0);
                    mma_f16(tm + PCOL_W, ah, bl, id, true);
                    mma_f16(tm + PCOL_W, al, bh, id, true);
                }
                commit(&sm.bar_w);
            }
            __syncwarp();
        }
        const bool ok_w = wait_w(&sm.bar_w, (uint32_t)gi & 1, err);
        if (__syncthreads_or(!ok_w)) break;
        fence_after_sync();
        // ---- W's image (K-major, rows j, 128 features) after [Tb;R] and G;
        // M = 64: row 16 q + lane in lane 32 q + lane (lane < 16)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            float v[32];
            ld32(tm + lq + PCOL_W + 64 * hh + 32 * half, v);
            if (lane < 16) {
                const int r = 16 * q4 + lane;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint4 hv, lv;
                    split8(&v[8 * j], hv, lv);
                    const uint32_t off = kmaj16(r, 64 * hh + 32 * half + 8 * j, DK);
                    *reinterpret_cast<uint4 *>(tr + WK_OFF + off) = hv;
                    *reinterpret_cast<uint4 *>(tr + WK_OFF + WK_HALF + off) = lv;
                }
            }
        }
        fence_before_sync();
        __syncthreads();  // the next value head rewrites A, T, X, the images and the accumulators
    }
    // every MMA has completed before the TMEM goes
    if (warp == 0) {
        if (elect_one()) commit(&sm.bar_fin);
        __syncwarp();
        wait_w(&sm.bar_fin, 0, err);
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 0) tmem_dealloc(tm, PTM_COLS);
}

// ============================================================ recurrence
constexpr int RT = 256;  // warp 0 copies, warp 1 MMAs, warps 4-7 passes
constexpr uint32_t COL_A = 0, COL_B = 32, COL_S = 64, TM_COLS = 128;

struct RecSmem {
    unsigned char kq[KQ_BYTES];           // [K;Q]: D_a(c) is done with it before chunk c+1's arrives
    unsigned char tr[2][TR_BYTES];        // [Tb;R], G, W: two-deep ring
    unsigned char s_op[2][128 * NV * 2];  // state, MN-major B operand (hi, lo)
    unsigned char vpp[2][CH * NV * 2];    // V'', MN-major B operand of the update and of D_b
    uint64_t kq_full, kq_empty, tr_full[2], tr_empty[2];
    uint64_t bar_a, bar_b, bar_c, bar_s, bar_vpp, bar_o, bar_fin;
    uint32_t tmem;
};
static_assert(sizeof(RecSmem) <= 232448, "recurrence shared memory");

template <int SDT>
__global__ void __launch_bounds__(RT, 1)
    chunk_rec_kernel(const kai_gdn_chunk_args p, const unsigned char *ws_kq, const unsigned char *ws_tr,
                     long long c_begin, int nc, int *err) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    RecSmem &sm = *reinterpret_cast<RecSmem *>(smem_raw);
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const long long Hk = (long long)p.heads_k, Hv = (long long)p.heads_v, T = (long long)p.seq;
    const long long DV = (long long)p.dv;
    const int nvb = (int)(DV / NV);
    const long long unit = blockIdx.x / nvb;  // b * Hv + h
    const int vb = blockIdx.x % nvb;
    const long long b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const long long v0 = (long long)vb * NV;
    const unsigned char *kq_src = ws_kq + (size_t)((b * Hk + hk) * nc) * KQ_BYTES;
    const unsigned char *tr_src = ws_tr + (size_t)(unit * nc) * TR_BYTES;

    if (t == 0) {
        mbar_init(&sm.kq_full, 1);
        mbar_init(&sm.kq_empty, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sm.tr_full[s], 1);
            mbar_init(&sm.tr_empty[s], 1 + 128);  // the D_b commit and the 128 readers of G
        }
        mbar_init(&sm.bar_a, 1);
        mbar_init(&sm.bar_b, 1);
        mbar_init(&sm.bar_c, 1);
        mbar_init(&sm.bar_fin, 1);
        mbar_init(&sm.bar_s, 128);
        mbar_init(&sm.bar_vpp, 64);
        mbar_init(&sm.bar_o, 64);
    }
    if (warp == 1) tmem_alloc(&sm.tmem, TM_COLS);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = sm.tmem;

    if (warp == 0) {
        // ---------------------------------------------------- copy warp
        if (lane == 0) {
            // launched as a programmatic dependent of the prep launch: its
            // images are complete and visible after this wait (only this
            // thread reads them from global memory; everything else here
            // runs ahead of it)
            asm volatile("griddepcontrol.wait;" ::: "memory");
            // [K;Q](c) as soon as D_a(c-1) is done with the single slot;
            // [Tb;R, G, W](c+1) as soon as its slot's chunk c-1 is released
            int kq_n = 0, tr_n = 0;
            bool ok = true;
            mbar_arrive_expect_tx(&sm.tr_full[0], TR_BYTES);
            bulk_load(sm.tr[0], tr_src, TR_BYTES, &sm.tr_full[0]);
            tr_n = 1;
            for (int c = 0; c < nc && ok; ++c) {
                if (c > 0 && !(ok = mbar_wait(&sm.kq_empty, (uint32_t)(c - 1) & 1, err))) break;
                mbar_arrive_expect_tx(&sm.kq_full, KQ_BYTES);
                bulk_load(sm.kq, kq_src + (size_t)c * KQ_BYTES, KQ_BYTES, &sm.kq_full);
                kq_n = c + 1;
                const int cn = c + 1;
                if (cn < nc) {
                    const int sn = cn & 1;
                    if (cn >= 2 && !(ok = mbar_wait(&sm.tr_empty[sn], (uint32_t)((cn >> 1) - 1) & 1, err))) break;
                    mbar_arrive_expect_tx(&sm.tr_full[sn], TR_BYTES);
                    bulk_load(sm.tr[sn], tr_src + (size_t)cn * TR_BYTES, TR_BYTES, &sm.tr_full[sn]);
                    tr_n = cn + 1;
                }
            }
            // no copy may still be landing when the CTA leaves
            if (kq_n > 0) mbar_wait(&sm.kq_full, (uint32_t)(kq_n - 1) & 1, err);
            for (int c = tr_n - 2 < 0 ? 0 : tr_n - 2; c < tr_n; ++c)
                mbar_wait(&sm.tr_full[c & 1], (uint32_t)(c >> 1) & 1, err);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------- MMA warp
        const uint32_t id_n = idesc(128, NV, BF16, false, true);  // A K-major, B MN-major
        const uint32_t id_t = idesc(128, NV, BF16, true, true);   // A = W^T, MN-major
        for (int c = 0; c < nc; ++c) {
            const int s = c & 1;
            const uint32_t ph = (uint32_t)(c >> 1) & 1, pc = (uint32_t)c & 1;
            if (!wait_w(&sm.kq_full, pc, err) || !spin_w(&sm.bar_s, pc, err)) break;
            fence_after_sync();
            // D_a = [K;Q] S
            if (elect_one()) {
#pragma unroll
                for (int ks = 0; ks < DK / 16; ++ks) {
                    const uint64_t ah = desc_kmaj16(sm.kq, DK, ks), al = desc_kmaj16(sm.kq + KQ_HALF, DK, ks);
                    const uint64_t bh = desc_mnmaj16(sm.s_op[0], NV, ks), bl = desc_mnmaj16(sm.s_op[1], NV, ks);
                    mma_f16(tm + COL_A, ah, bh, id_n, ks > 0);
                    mma_f16(tm + COL_A, ah, bl, id_n, true);
                    mma_f16(tm + COL_A, al, bh, id_n, true);
                }
                commit(&sm.bar_a);
                commit(&sm.kq_empty);
            }
            __syncwarp();
            if (!wait_w(&sm.tr_full[s], ph, err) || !spin_w(&sm.bar_vpp, pc, err)) break;
            fence_after_sync();
            // the state update S += W^T V'' (W's K-major image read MN-major
            // is W^T: M = features, K = tokens)
            if (elect_one()) {
                const unsigned char *wk = sm.tr[s] + WK_OFF;
#pragma unroll
                for (int ks = 0; ks < CH / 16; ++ks) {
                    const uint64_t ah = desc_mnmaj16(wk, DK, ks), al = desc_mnmaj16(wk + WK_HALF, DK, ks);
                    const uint64_t bh = desc_mnmaj16(sm.vpp[0], NV, ks), bl = desc_mnmaj16(sm.vpp[1], NV, ks);
                    mma_f16(tm + COL_S, ah, bh, id_t, true);
                    mma_f16(tm + COL_S, ah, bl, id_t, true);
                    mma_f16(tm + COL_S, al, bh, id_t, true);
                }
                commit(&sm.bar_c);
            }
            __syncwarp();
            // D_b = [Tb;R] V'' for the output (off the state's chain), once the
            // output warps have read the previous chunk's
            if (c > 0 && !spin_w(&sm.bar_o, pc ^ 1, err)) break;
            fence_after_sync();
            if (elect_one()) {
#pragma unroll
                for (int ks = 0; ks < CH / 16; ++ks) {
                    const uint64_t ah = desc_kmaj16(sm.tr[s], CH, ks), al = desc_kmaj16(sm.tr[s] + TR_HALF, CH, ks);
                    const uint64_t bh = desc_mnmaj16(sm.vpp[0], NV, ks), bl = desc_mnmaj16(sm.vpp[1], NV, ks);
                    mma_f16(tm + COL_B, ah, bh, id_n, ks > 0);
                    mma_f16(tm + COL_B, ah, bl, id_n, true);
                    mma_f16(tm + COL_B, al, bh, id_n, true);
                }
                commit(&sm.bar_b);
                commit(&sm.tr_empty[s]);
            }
            __syncwarp();
        }
        // every MMA has completed before the TMEM goes (the commit tracks all
        // MMAs this lane issued)
        if (elect_one()) commit(&sm.bar_fin);
        __syncwarp();
        wait_w(&sm.bar_fin, 0, err);
    } else if (warp >= 4) {
        // -------------------------------------------------- pass warps
        using ST = Store<SDT>;
        const int wq = warp - 4, row = 32 * wq + lane, r = row % CH;
        const bool vrow = row < CH;  // warps 4, 5: V''; warps 6, 7: output rows
        const uint32_t loff = (uint32_t)(32 * wq) << 16;
        const uint32_t ta = tm + loff + COL_A, tb = tm + loff + COL_B, ts = tm + loff + COL_S;
        typename ST::T *st = static_cast<typename ST::T *>(p.state) + ((size_t)unit * DK + row) * DV + v0;
        float sv[NV];
        // initial state row `row` (key feature), split for the first D_a and
        // decayed by e^{G_63} of the first chunk into TMEM
#pragma unroll
        for (int n = 0; n < NV; ++n) sv[n] = ST::load(st + n);
        bool ok = wait_w(&sm.tr_full[0], 0, err);
        if (ok) {
            const float e = expf(reinterpret_cast<const float *>(sm.tr[0] + 2 * TR_HALF)[CH - 1]);
            put_row_mn(sm.s_op[0], sm.s_op[1], row, sv);
#pragma unroll
            for (int n = 0; n < NV; ++n) sv[n] *= e;
            st32(ts, sv);
            fence_smem_to_async();
            fence_before_sync();
            mbar_arrive1(&sm.bar_s);
        }
        // V rows (warps 4, 5) are loaded a chunk ahead: with the image copies
        // streaming, a load issued at the chunk's start was still in flight
        // when D_a completed (~1.5K cycles on the chain)
        float vn[NV];
        auto load_v = [&](int cc) {
            const long long tk = (c_begin + cc) * CH + r;
            if (cc < nc && tk < T) {
                const float4 *vs = reinterpret_cast<const float4 *>(static_cast<const float *>(p.v) +
                                                                    ((size_t)(b * T + tk) * Hv + h) * DV + v0);
#pragma unroll
                for (int j = 0; j < NV / 4; ++j) *reinterpret_cast<float4 *>(&vn[4 * j]) = __ldg(vs + j);
            } else {
#pragma unroll
                for (int n = 0; n < NV; ++n) vn[n] = 0.f;
            }
        };
        if (vrow) load_v(0);
        for (int c = 0; ok && c < nc; ++c) {
            const int s = c & 1;
            const uint32_t ph = (uint32_t)(c >> 1) & 1, pc = (uint32_t)c & 1;
            const long long tok = (c_begin + c) * CH + r;
            if (!(ok = wait_w(&sm.tr_full[s], ph, err))) break;
            const float gr = reinterpret_cast<const float *>(sm.tr[s] + 2 * TR_HALF)[r];
            mbar_arrive1(&sm.tr_empty[s]);
            float x[NV];
            if (vrow) {
#pragma unroll
                for (int n = 0; n < NV; ++n) x[n] = vn[n];
                load_v(c + 1);
                if (!(ok = spin_w(&sm.bar_a, pc, err))) break;
                fence_after_sync();
                float ks[NV];
                ld32(ta, ks);
                const float eg = expf(gr);
#pragma unroll
                for (int n = 0; n < NV; ++n) x[n] = fmaf(-eg, ks[n], x[n]);  // V''
                // the previous chunk's D_b has read V'': it was issued before
                // D_a by the same thread, and a commit (bar_a) completes only
                // once every earlier MMA of its thread has
                put_row_mn(sm.vpp[0], sm.vpp[1], r, x);
                fence_smem_to_async();
                fence_before_sync();
                mbar_arrive1(&sm.bar_vpp);
            } else {
                if (!(ok = spin_w(&sm.bar_a, pc, err))) break;
                fence_after_sync();
                ld32(ta, x);  // Q S, kept until the output below
            }
            // ---- the state after this chunk
            const bool fin = c + 1 == nc;
            float gn = 0.f;
            if (!fin) {
                if (!(ok = wait_w(&sm.tr_full[s ^ 1], (uint32_t)((c + 1) >> 1) & 1, err))) break;
                gn = reinterpret_cast<const float *>(sm.tr[s ^ 1] + 2 * TR_HALF)[CH - 1];
            }
            if (!(ok = spin_w(&sm.bar_c, pc, err))) break;
            fence_after_sync();
            ld32(ts, sv);
            if (fin) {
#pragma unroll
                for (int n = 0; n < NV; ++n) ST::store(st + n, sv[n]);
            } else {
                put_row_mn(sm.s_op[0], sm.s_op[1], row, sv);
                const float e = expf(gn);
#pragma unroll
                for (int n = 0; n < NV; ++n) sv[n] *= e;
                st32(ts, sv);
                fence_smem_to_async();
                fence_before_sync();
                mbar_arrive1(&sm.bar_s);
            }
            // ---- the output rows, off the state's chain
            if (!vrow) {
                float y[NV];
                if (!(ok = spin_w(&sm.bar_b, pc, err))) break;
                fence_after_sync();
                ld32(tb, y);  // R V''
                fence_before_sync();
                mbar_arrive1(&sm.bar_o);
                const float f = p.scale * expf(gr);
#pragma unroll
                for (int n = 0; n < NV; ++n) x[n] = fmaf(f, x[n], y[n]);
                if (tok < T) store32(p.o, ((size_t)(b * T + tok) * Hv + h) * DV + v0, p.out_dtype, x);
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    if (warp == 1) tmem_dealloc(tm, TM_COLS);
}

template <int SDT>
int launch_rec(const kai_gdn_chunk_args *a, const unsigned char *kq, const unsigned char *tr, long long c_begin,
               int nc, int *err, cudaStream_t st) {
    static thread_local int done_dev = -1;
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "chunk_tc32: cudaGetDevice");
    if (rc) return rc;
    if (done_dev != dev) {
        rc = check_cuda(cudaFuncSetAttribute(chunk_rec_kernel<SDT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(RecSmem)),
                        "chunk_tc32: smem attribute");
        if (rc) return rc;
        done_dev = dev;
    }
    // a programmatic dependent of the prep launch before it: set-up, the
    // state load and TMEM allocation overlap the prep's last CTAs
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)(a->batch * a->heads_v * (a->dv / NV)));
    cfg.blockDim = dim3(RT);
    cfg.dynamicSmemBytes = sizeof(RecSmem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, chunk_rec_kernel<SDT>, *a, kq, tr, c_begin, nc, err);
    if (le != cudaSuccess) return check_cuda(le, "chunk_tc32_rec launch");
    return check_launch("chunk_tc32_rec");
}

}  // namespace

bool chunk_tc32_supported(const kai_gdn_chunk_args *a) {
    if (a->in_dtype != KAI_GDN_F32 || a->dk != (size_t)DK || a->chunk != (size_t)CH) return false;
    if (a->dv == 0 || a->dv % NV) return false;
    if (((uintptr_t)a->q | (uintptr_t)a->k | (uintptr_t)a->v | (uintptr_t)a->o) % 16) return false;
    if (a->seq > 0x7fffffffull || a->batch * a->heads_v * (a->dv / NV) > 0x7fffffffull) return false;
    return true;
}

int launch_chunk_tc32(const kai_gdn_chunk_args *a, cudaStream_t st) {
    const size_t per_chunk = a->batch * (a->heads_k * (size_t)KQ_BYTES + a->heads_v * (size_t)TR_BYTES);
    const long long nch = (long long)((a->seq + CH - 1) / CH);
    long long seg = (long long)(SEG_BUDGET / per_chunk);
    if (seg < 1) seg = 1;
    if (seg > nch) seg = nch;
    const long long prep_blocks = (long long)(a->batch * a->heads_k) * seg;
    if (prep_blocks > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk_tc32: too many heads");
    void *scr = nullptr;
    int rc = scratch_for_stream(st, (size_t)seg * per_chunk, &scr);
    if (rc) return rc;
    unsigned char *kq = static_cast<unsigned char *>(scr);
    unsigned char *tr = kq + (size_t)seg * a->batch * a->heads_k * KQ_BYTES;
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    static thread_local int prep_dev = -1;
    int dev = 0;
    if ((rc = check_cuda(cudaGetDevice(&dev), "chunk_tc32: cudaGetDevice"))) return rc;
    if (prep_dev != dev) {
        rc = check_cuda(cudaFuncSetAttribute(chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(PrepSmem)),
                        "chunk_tc32: smem attribute");
        if (rc) return rc;
        prep_dev = dev;
    }
    for (long long c_begin = 0; c_begin < nch; c_begin += seg) {
        const int nc = (int)(nch - c_begin < seg ? nch - c_begin : seg);
        chunk_prep_kernel<<<(unsigned)(a->batch * a->heads_k * nc), PT, sizeof(PrepSmem), st>>>(*a, kq, tr, c_begin,
                                                                                                 nc, err);
        if ((rc = check_launch("chunk_tc32_prep"))) return rc;
        switch (a->state_dtype) {
            case KAI_GDN_BF16: rc = launch_rec<KAI_GDN_BF16>(a, kq, tr, c_begin, nc, err, st); break;
            case KAI_GDN_F16: rc = launch_rec<KAI_GDN_F16>(a, kq, tr, c_begin, nc, err, st); break;
            default: rc = launch_rec<KAI_GDN_F32>(a, kq, tr, c_begin, nc, err, st);
        }
        if (rc) return rc;
    }
    return KAI_GDN_OK;
}

}  // namespace gdn
