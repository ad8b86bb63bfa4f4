// chunk_tc.cu -- chunkwise (WY / UT-transform) gated delta-rule scan on the
// sm_100a tensor cores (tcgen05 + TMEM), for bf16 / fp16 q, k, v with fp32
// state and accumulation, dk = dv = 128, chunk C = 64.
//
// Math (docs/GDN_ARCHITECTURE_AUDIT.md:142-153; the chunked form of
// gpu/gdn_gpu_validate.c:100-118).  Per (b, value head h), chunk of 64 tokens,
// G = in-chunk cumulative log decay, gamma = exp(G_63):
//   A  = beta_r (k_r.k_s) exp(G_r - G_s), s <  r        (from  [K;Q] K^T)
//   P  = scale (q_r.k_s) exp(G_r - G_s), s <= r        (same MMA, rows 64..127)
//   T  = (I + A)^-1                                     (CUDA cores, fp32)
//   [W | U] = T [beta K exp(G) | beta V]                (one MMA, N = 256)
//   V' = U - W S                                        (MMA W.S)
//   O  = (scale Q exp(G)) S + P V'                      (MMA Qg.S, then P.V')
//   S <- gamma S + (K exp(G_63 - G))^T V'               (MMA, M = 128)
//
// One CTA (256 threads) owns one (b, h) for the whole sequence; its fp32
// state S [128 x 128] stays in TMEM columns 0..127 and a bf16 copy in shared
// memory feeds the next chunk's MMAs.  Thread 0 issues every MMA; completion
// is signalled with tcgen05.commit on one mbarrier, and every wait is bounded
// (a timeout sets *err and the CTA leaves after freeing its TMEM).
//
// TMEM columns (512, one CTA per SM):
//   [  0,128) S        M=128 (lane = key index d)
//   [128,192) [K;Q]K^T M=128 (lanes 0-63: K K^T rows, 64-127: Q K^T rows)
//   [128,256) W S      M=64  (after [K;Q]K^T has been read)
//   [256,384) W, later O (after W has been copied out), M=64
//   [384,512) U        M=64
// Operand tiles are bf16/fp16 in the no-swizzle core-matrix layouts of
// umma.cuh.  The K-major [K;Q] tile doubles as the MN-major A operand of
// K'^T V' (a K-major tile with 128 columns is the MN-major tile of its
// transpose), so K' is written over K in place.
#include "gdn_internal.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int C = 64, D = 128, NT = 256;
constexpr int LDF = 65;  // padded fp32 row stride (conflict-free column walks)

template <typename IT> struct InTraits;
template <> struct InTraits<__nv_bfloat16> {
    static constexpr uint32_t fmt = BF16;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct InTraits<__half> {
    static constexpr uint32_t fmt = F16;
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

struct __align__(128) TcSmem {
    unsigned char KQ[2 * C * D * 2];   // [K;Q] K-major 128 x 128; later [K';Qg]
    unsigned char R[C * 2 * D * 2];    // [beta K e^G | beta V] MN-major 64 x 256
    unsigned char S[D * D * 2];        // state copy, MN-major (k = d, n = value col)
    unsigned char W[C * D * 2];        // W, K-major 64 x 128
    unsigned char Vp[C * D * 2];       // V', MN-major (k = row, n = value col)
    unsigned char P[C * C * 2];        // P, K-major 64 x 64
    unsigned char T[C * C * 2];        // T, K-major 64 x 64
    float Af[C * LDF];                 // A (strictly lower), fp32
    float Tf[C * LDF];                 // T = (I + A)^-1, fp32
    float Mscr[3 * 16 * 17];           // block products of the inverse
    float G[C], eG[C], eGl[C], beta[C];
    uint64_t bar;
    uint32_t tmem;
    int stop;
};

template <typename IT>
__device__ __forceinline__ void st_vec8(unsigned char *base, uint32_t off, const float (&v)[8]) {
    using TR = InTraits<IT>;
    uint4 u;
    IT *h = reinterpret_cast<IT *>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = TR::from_f(v[i]);
    *reinterpret_cast<uint4 *>(base + off) = u;
}
template <typename IT>
__device__ __forceinline__ void ld_vec8(const unsigned char *base, uint32_t off, float (&v)[8]) {
    using TR = InTraits<IT>;
    uint4 u = *reinterpret_cast<const uint4 *>(base + off);
    const IT *h = reinterpret_cast<const IT *>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = TR::to_f(h[i]);
}

__device__ __forceinline__ float ld_state(const void *p, size_t i, int dt) {
    switch (dt) {
        case KAI_GDN_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
        case KAI_GDN_F16: return __half2float(static_cast<const __half *>(p)[i]);
        default: return static_cast<const float *>(p)[i];
    }
}
__device__ __forceinline__ void st_any(void *p, size_t i, int dt, float v) {
    switch (dt) {
        case KAI_GDN_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
        case KAI_GDN_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
        default: static_cast<float *>(p)[i] = v;
    }
}

// Loads of one chunk held in registers until they are stored to shared
// memory.  Thread t owns row r = 8*(t/32) + t%8 of the chunk and the four
// 8-element column groups cc = 8*(4*i + (t%32)/8), i = 0..3: a warp covers 8
// consecutive rows x 4 column groups, so its 16-byte global loads use whole
// 32-byte sectors and its 16-byte shared stores into the core-matrix layouts
// (8 rows x 16 bytes contiguous) are free of bank conflicts.
struct ChunkRegs {
    uint4 k[4], q[4], v[4];
    float g0, g1, b0, b1;  // gates of rows 2*lane, 2*lane+1 (warp 0 only)
};

template <typename IT>
__device__ __forceinline__ void prefetch_chunk(ChunkRegs &cr, const kai_gdn_chunk_args &p, long long b,
                                               long long h, long long hk, long long c0, int t) {
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k, T = (long long)p.seq;
    const IT *kp = static_cast<const IT *>(p.k), *qp = static_cast<const IT *>(p.q);
    const IT *vp = static_cast<const IT *>(p.v);
    const int r = 8 * (t / 32) + (t % 8), a = (t % 32) / 8;
    const long long tok = c0 + r;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int cc = 8 * (4 * i + a);
        if (tok < T) {
            const size_t ki = ((size_t)(b * T + tok) * Hk + hk) * D + cc;
            const size_t vi = ((size_t)(b * T + tok) * Hv + h) * D + cc;
            cr.k[i] = __ldg(reinterpret_cast<const uint4 *>(kp + ki));
            cr.q[i] = __ldg(reinterpret_cast<const uint4 *>(qp + ki));
            cr.v[i] = __ldg(reinterpret_cast<const uint4 *>(vp + vi));
        } else {
            cr.k[i] = cr.q[i] = cr.v[i] = make_uint4(0, 0, 0, 0);
        }
    }
    if (t < 32) {
        const long long r0 = c0 + 2 * t, r1 = r0 + 1;
        cr.g0 = r0 < T ? __ldg(p.g + (size_t)(b * T + r0) * Hv + h) : 0.f;
        cr.b0 = r0 < T ? __ldg(p.beta + (size_t)(b * T + r0) * Hv + h) : 0.f;
        cr.g1 = r1 < T ? __ldg(p.g + (size_t)(b * T + r1) * Hv + h) : 0.f;
        cr.b1 = r1 < T ? __ldg(p.beta + (size_t)(b * T + r1) * Hv + h) : 0.f;
    }
}

// 16 consecutive output values of one row, as 16-byte vector stores.
__device__ __forceinline__ void st16_out(void *o, size_t idx, int dt, const float (&v)[16]) {
    if (dt == KAI_GDN_F32) {
        float4 *f = reinterpret_cast<float4 *>(static_cast<float *>(o) + idx);
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        return;
    }
    uint4 u[2];
    if (dt == KAI_GDN_BF16) {
        __nv_bfloat16 *hh = reinterpret_cast<__nv_bfloat16 *>(u);
#pragma unroll
        for (int i = 0; i < 16; ++i) hh[i] = __float2bfloat16_rn(v[i]);
    } else {
        __half *hh = reinterpret_cast<__half *>(u);
#pragma unroll
        for (int i = 0; i < 16; ++i) hh[i] = __float2half_rn(v[i]);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(o) + idx);
    dst[0] = u[0];
    dst[1] = u[1];
}

// out(i, j) of the 16x16 block product X[xr.., xc..] . Y[yr.., yc..] (fp32, stride LDF)
__device__ __forceinline__ float bprod(const float *X, int xr, int xc, const float *Y, int yr, int yc, int i,
                                       int j) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = fmaf(X[(xr + i) * LDF + xc + k], Y[(yr + k) * LDF + yc + j], acc);
    return acc;
}

// T = (I + A)^-1 for strictly lower A (64 x 64, fp32), by 16 x 16 blocks:
// diagonal blocks by forward substitution, then T_ij = -T_ii sum_k A_ik T_kj.
__device__ void invert_unit_lower(TcSmem &sm, int t) {
    float *A = sm.Af, *T = sm.Tf, *M = sm.Mscr;
    if (t < 64) {
        const int blk = t / 16, j = t % 16, o = 16 * blk;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float acc = 0.f;
#pragma unroll
            for (int s = 0; s < r; ++s) acc = fmaf(A[(o + r) * LDF + o + s], x[s], acc);
            x[r] = r < j ? 0.f : (r == j ? 1.f : -acc);
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) T[(o + r) * LDF + o + j] = x[r];
    } else {
        // zero the blocks above the diagonal
        for (int e = t - 64; e < 6 * 256; e += NT - 64) {
            // block pairs (0,1) (0,2) (0,3) (1,2) (1,3) (2,3)
            int b = e / 256, w = e % 256, i = w / 16, j = w % 16;
            int bi = b < 3 ? 0 : (b < 5 ? 1 : 2), bj = b < 3 ? b + 1 : (b < 5 ? b - 1 : 3);
            T[(16 * bi + i) * LDF + 16 * bj + j] = 0.f;
        }
    }
    __syncthreads();
    // level 1: (1,0), (2,1), (3,2)
    for (int e = t; e < 3 * 256; e += NT) {
        int b = e / 256, i = (e % 256) / 16, j = e % 16;
        M[b * 272 + i * 17 + j] = bprod(A, 16 * (b + 1), 16 * b, T, 16 * b, 16 * b, i, j);
    }
    __syncthreads();
    for (int e = t; e < 3 * 256; e += NT) {
        int b = e / 256, i = (e % 256) / 16, j = e % 16, r0 = 16 * (b + 1);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = fmaf(T[(r0 + i) * LDF + r0 + k], M[b * 272 + k * 17 + j], acc);
        T[(r0 + i) * LDF + 16 * b + j] = -acc;
    }
    __syncthreads();
    // level 2: (2,0), (3,1)
    for (int e = t; e < 2 * 256; e += NT) {
        int b = e / 256, i = (e % 256) / 16, j = e % 16, ri = 16 * (b + 2), cj = 16 * b;
        M[b * 272 + i * 17 + j] = bprod(A, ri, cj, T, cj, cj, i, j) + bprod(A, ri, cj + 16, T, cj + 16, cj, i, j);
    }
    __syncthreads();
    for (int e = t; e < 2 * 256; e += NT) {
        int b = e / 256, i = (e % 256) / 16, j = e % 16, ri = 16 * (b + 2);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = fmaf(T[(ri + i) * LDF + ri + k], M[b * 272 + k * 17 + j], acc);
        T[(ri + i) * LDF + 16 * b + j] = -acc;
    }
    __syncthreads();
    // level 3: (3,0)
    {
        int i = t / 16, j = t % 16;
        M[i * 17 + j] = bprod(A, 48, 0, T, 0, 0, i, j) + bprod(A, 48, 16, T, 16, 0, i, j) +
                        bprod(A, 48, 32, T, 32, 0, i, j);
    }
    __syncthreads();
    {
        int i = t / 16, j = t % 16;
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = fmaf(T[(48 + i) * LDF + 48 + k], M[k * 17 + j], acc);
        T[(48 + i) * LDF + j] = -acc;
    }
    __syncthreads();
}

// Issue-side helpers (thread 0 only).
__device__ __forceinline__ void issue_sync() {
    fence_smem_to_async();
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
}

template <typename IT>
__global__ void __launch_bounds__(NT, 1) chunk_tc_kernel(kai_gdn_chunk_args p, int *err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(smem_raw);
    using TR = InTraits<IT>;

    const int t = threadIdx.x, warp = t / 32, lane = t % 32, q = warp % 4, hf = warp / 4;
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k, T = (long long)p.seq;
    const long long unit = blockIdx.x, b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const float scale = p.scale;

    if (t == 0) {
        mbar_init(&sm.bar, 1);
        sm.stop = 0;
    }
    if (warp == 0) tmem_alloc(&sm.tmem, 512);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = sm.tmem;
    const uint32_t TS = tm, TD1 = tm + 128, TD3 = tm + 128, TW = tm + 256, TO = tm + 256, TU = tm + 384;
    uint32_t phase = 0;

    // ---- initial state: fp32 into TMEM columns 0..127, bf16 copy into sm.S
    {
        const int d = 32 * q + lane;
        const size_t sb = (size_t)unit * D * D + (size_t)d * D;
        for (int c0 = hf * 64; c0 < hf * 64 + 64; c0 += 16) {
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = ld_state(p.state, sb + c0 + i, p.state_dtype);
            tmem_st16(taddr(TS, 32 * q, c0), v);
            float a[8], c[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                a[i] = v[i];
                c[i] = v[8 + i];
            }
            st_vec8<IT>(sm.S, mnmaj16(d, c0, D), a);
            st_vec8<IT>(sm.S, mnmaj16(d, c0 + 8, D), c);
        }
        tmem_wait_st();
    }

    ChunkRegs cr;
    prefetch_chunk<IT>(cr, p, b, h, hk, 0, t);
    for (long long c0 = 0; c0 < T; c0 += C) {
        // ---------------------------------------------------- L: gates
        if (t < 32) {
            const float g0 = cr.g0, g1 = cr.g1;
            float pair = g0 + g1, incl = pair;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                float u = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += u;
            }
            float excl = incl - pair;
            sm.G[2 * t] = excl + g0;
            sm.G[2 * t + 1] = incl;
            sm.beta[2 * t] = cr.b0;
            sm.beta[2 * t + 1] = cr.b1;
        }
        __syncthreads();
        if (t < C) {
            sm.eG[t] = expf(sm.G[t]);
            sm.eGl[t] = expf(sm.G[C - 1] - sm.G[t]);
        }
        __syncthreads();
        // ------------------------------------------ L: K, Q, V -> tiles
        {
            const int r = 8 * warp + (lane % 8), a = lane / 8;
            const float bk = sm.beta[r] * sm.eG[r], bv = sm.beta[r];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int cc = 8 * (4 * i + a);
                *reinterpret_cast<uint4 *>(sm.KQ + kmaj16(r, cc, D)) = cr.k[i];
                *reinterpret_cast<uint4 *>(sm.KQ + kmaj16(C + r, cc, D)) = cr.q[i];
                const IT *kh = reinterpret_cast<const IT *>(&cr.k[i]), *vh = reinterpret_cast<const IT *>(&cr.v[i]);
                float kv[8], vv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    kv[j] = TR::to_f(kh[j]) * bk;
                    vv[j] = TR::to_f(vh[j]) * bv;
                }
                st_vec8<IT>(sm.R, mnmaj16(r, cc, 2 * D), kv);
                st_vec8<IT>(sm.R, mnmaj16(r, D + cc, 2 * D), vv);
            }
        }
        // ------------------------------------------ M1: [K;Q] K^T
        issue_sync();
        if (t == 0) {
            const uint32_t id = idesc(128, 64, TR::fmt, false, false);
            for (int ks = 0; ks < D / 16; ++ks)
                mma_f16(TD1, desc_kmaj16(sm.KQ, D, ks), desc_kmaj16(sm.KQ, D, ks), id, ks > 0);
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // ------------------------------------------ E1: A, P; K', Qg
        {
            const int i = 32 * q + lane;  // D1 row
            float v[16];
            for (int cb = hf * 32; cb < hf * 32 + 32; cb += 16) {
                tmem_ld16(taddr(TD1, 32 * q, cb), v);
                tmem_wait_ld();
                if (i < C) {
                    const int r = i;
                    const float gr = sm.G[r], br = sm.beta[r];
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int s = cb + jj;
                        sm.Af[r * LDF + s] = s < r ? br * v[jj] * __expf(gr - sm.G[s]) : 0.f;
                    }
                } else {
                    const int r = i - C;
                    const float gr = sm.G[r];
                    float a[8], c[8];
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int s0 = cb + jj, s1 = cb + 8 + jj;
                        a[jj] = s0 <= r ? scale * v[jj] * __expf(gr - sm.G[s0]) : 0.f;
                        c[jj] = s1 <= r ? scale * v[8 + jj] * __expf(gr - sm.G[s1]) : 0.f;
                    }
                    st_vec8<IT>(sm.P, kmaj16(r, cb, C), a);
                    st_vec8<IT>(sm.P, kmaj16(r, cb + 8, C), c);
                }
            }
        }
        // K' = K e^(G_63 - G) over the K rows, Qg = scale Q e^G over the Q rows,
        // from the raw values still in registers; then fetch the next chunk.
        {
            const int r = 8 * warp + (lane % 8), a = lane / 8;
            const float fk = sm.eGl[r], fq = scale * sm.eG[r];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int cc = 8 * (4 * i + a);
                const IT *kh = reinterpret_cast<const IT *>(&cr.k[i]), *qh = reinterpret_cast<const IT *>(&cr.q[i]);
                float kv[8], qv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    kv[j] = TR::to_f(kh[j]) * fk;
                    qv[j] = TR::to_f(qh[j]) * fq;
                }
                st_vec8<IT>(sm.KQ, kmaj16(r, cc, D), kv);
                st_vec8<IT>(sm.KQ, kmaj16(C + r, cc, D), qv);
            }
            if (c0 + C < T) prefetch_chunk<IT>(cr, p, b, h, hk, c0 + C, t);
        }
        __syncthreads();
        // ------------------------------------------ INV: T = (I + A)^-1
        invert_unit_lower(sm, t);
        for (int e = t; e < C * C / 8; e += NT) {
            const int r = e / 8, s0 = (e % 8) * 8;
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = sm.Tf[r * LDF + s0 + i];
            st_vec8<IT>(sm.T, kmaj16(r, s0, C), v);
        }
        // ------------------------------------------ M2: [W | U] = T R
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id = idesc(64, 256, TR::fmt, false, true);
            for (int ks = 0; ks < C / 16; ++ks)
                mma_f16(TW, desc_kmaj16(sm.T, C, ks), desc_mnmaj16(sm.R, 2 * D, ks), id, ks > 0);
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // ------------------------------------------ E2: W -> smem
        {
            const int r = 16 * q + lane;
            for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
                float v[16];
                tmem_ld16(taddr(TW, 32 * q, cb), v);
                tmem_wait_ld();
                if (lane < 16) {
                    float a[8], c[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        a[i] = v[i];
                        c[i] = v[8 + i];
                    }
                    st_vec8<IT>(sm.W, kmaj16(r, cb, D), a);
                    st_vec8<IT>(sm.W, kmaj16(r, cb + 8, D), c);
                }
            }
        }
        // ------------------------------------------ M3: W S, Qg S
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id = idesc(64, 128, TR::fmt, false, true);
            const unsigned char *Qg = sm.KQ + C * D * 2;  // rows 64..127 of the K-major tile
            for (int ks = 0; ks < D / 16; ++ks) {
                const uint64_t bd = desc_mnmaj16(sm.S, D, ks);
                mma_f16(TD3, desc_kmaj16(sm.W, D, ks), bd, id, ks > 0);
                mma_f16(TO, desc_kmaj16(Qg, D, ks), bd, id, ks > 0);
            }
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // ------------------------------------------ E3: V' = U - W S; S *= gamma
        {
            const int r = 16 * q + lane;
            for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
                float ws[16], u[16];
                tmem_ld16(taddr(TD3, 32 * q, cb), ws);
                tmem_ld16(taddr(TU, 32 * q, cb), u);
                tmem_wait_ld();
                if (lane < 16) {
                    float a[8], c[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        a[i] = u[i] - ws[i];
                        c[i] = u[8 + i] - ws[8 + i];
                    }
                    st_vec8<IT>(sm.Vp, mnmaj16(r, cb, D), a);
                    st_vec8<IT>(sm.Vp, mnmaj16(r, cb + 8, D), c);
                }
            }
            const float gamma = sm.eG[C - 1];
            for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
                float s[16];
                tmem_ld16(taddr(TS, 32 * q, cb), s);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; ++i) s[i] *= gamma;
                tmem_st16(taddr(TS, 32 * q, cb), s);
            }
            tmem_wait_st();
        }
        // ------------------------------------------ M4: O += P V'; S += K'^T V'
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id_o = idesc(64, 128, TR::fmt, false, true);
            const uint32_t id_s = idesc(128, 128, TR::fmt, true, true);
            for (int ks = 0; ks < C / 16; ++ks) {
                const uint64_t vd = desc_mnmaj16(sm.Vp, D, ks);
                mma_f16(TO, desc_kmaj16(sm.P, C, ks), vd, id_o, true);
                mma_f16(TS, desc_mnmaj16(sm.KQ, D, ks), vd, id_s, true);
            }
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // ------------------------------------------ E4: O out; S -> smem copy
        {
            const int r = 16 * q + lane;
            const long long tok = c0 + r;
            for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
                float o[16];
                tmem_ld16(taddr(TO, 32 * q, cb), o);
                tmem_wait_ld();
                if (lane < 16 && tok < T) st16_out(p.o, ((size_t)(b * T + tok) * Hv + h) * D + cb, p.out_dtype, o);
            }
            const int d = 32 * q + lane;
            for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
                float s[16];
                tmem_ld16(taddr(TS, 32 * q, cb), s);
                tmem_wait_ld();
                float a[8], c[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    a[i] = s[i];
                    c[i] = s[8 + i];
                }
                st_vec8<IT>(sm.S, mnmaj16(d, cb, D), a);
                st_vec8<IT>(sm.S, mnmaj16(d, cb + 8, D), c);
            }
        }
        fence_before_sync();
        __syncthreads();
        if (sm.stop) break;
    }

    // ---- final state out (fp32 from TMEM)
    fence_after_sync();
    if (!sm.stop) {
        const int d = 32 * q + lane;
        const size_t sb = (size_t)unit * D * D + (size_t)d * D;
        for (int cb = hf * 64; cb < hf * 64 + 64; cb += 16) {
            float s[16];
            tmem_ld16(taddr(TS, 32 * q, cb), s);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) st_any(p.state, sb + cb + i, p.state_dtype, s[i]);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 512);
}

}  // namespace

bool chunk_tc_supported(const kai_gdn_chunk_args *a) {
    if (a->dk != 128 || a->dv != 128 || a->chunk != 64) return false;
    if (a->in_dtype != KAI_GDN_BF16 && a->in_dtype != KAI_GDN_F16) return false;
    if (((uintptr_t)a->q | (uintptr_t)a->k | (uintptr_t)a->v | (uintptr_t)a->o) % 16) return false;
    return true;
}

int launch_chunk_tc(const kai_gdn_chunk_args *a, cudaStream_t st) {
    const long long units = (long long)(a->batch * a->heads_v);
    if (units > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk_tc: too many heads");
    void *flag = nullptr;
    int rc = scratch_for_stream(st, 256, &flag);
    if (rc) return rc;
    if ((rc = check_cuda(cudaMemsetAsync(flag, 0, sizeof(int), st), "chunk_tc: clear flag"))) return rc;
    const size_t smem = sizeof(TcSmem) + 1024;
    if (a->in_dtype == KAI_GDN_BF16) {
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__nv_bfloat16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "chunk_tc: smem attribute");
        if (rc) return rc;
        chunk_tc_kernel<__nv_bfloat16><<<(unsigned)units, NT, smem, st>>>(*a, static_cast<int *>(flag));
    } else {
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "chunk_tc: smem attribute");
        if (rc) return rc;
        chunk_tc_kernel<__half><<<(unsigned)units, NT, smem, st>>>(*a, static_cast<int *>(flag));
    }
    return check_launch("chunk_delta_rule_tc");
}

}  // namespace gdn
