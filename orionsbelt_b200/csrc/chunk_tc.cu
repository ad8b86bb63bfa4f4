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
//   W = T (beta K exp(G)),  U = T (beta V)              (two MMAs)
//   V' = U - W S                                        (MMA W.S)
//   O  = (scale Q exp(G)) S + P V'                      (MMAs Qg.S and P.V')
//   S <- gamma S + (K exp(G_63 - G))^T V'               (MMA, M = 128)
//
// One CTA (256 threads) owns one (b, h) for the whole sequence; its fp32
// state S [128 x 128] stays in TMEM and a 16-bit copy in shared memory feeds
// the next chunk's MMAs.  The kernel is latency-bound (a chain of dependent
// phases per chunk), so it is sized for TWO resident CTAs per SM, whose
// phases interleave: 256 TMEM columns, ~105 KB of shared memory and at most
// 128 registers per thread.  Thread 0 issues every MMA; completion is
// signalled by tcgen05.commit on one mbarrier, and every wait is bounded (a
// timeout sets *err and the CTA leaves after freeing its TMEM).
//
// TMEM (256 columns).  M=64 accumulators put rows 16q..16q+15 in lanes
// 32q..32q+15 ("lower half") or, at lane offset 16, in lanes 32q+16..32q+31
// ("upper half"), so two of them share columns:
//   [  0,128) S             M=128, lane = key index d
//   [128,192) [K;Q] K^T     M=128 (lanes 0-63: K K^T, 64-127: Q K^T)
//   [128,256) W | U         M=64, lower | upper half       (after [K;Q]K^T is read)
//   [128,256) W S | O       M=64, lower | upper half       (after W, U are read)
// A warp's 32x32b TMEM load then returns W S in lanes 0-15 and U (or O) in
// lanes 16-31 of the same columns.
//
// Shared memory, regions reused by lifetime within a chunk:
//   S     16-bit state copy, MN-major                        always
//   A     raw [K;Q] (K-major 128 x 128)       L  .. M1
//         A, T = (I+A)^-1 fp32 (block-packed), then T tile   E1 .. M2
//         K' and Qg (K-major 64 x 128 each)   E2 .. M4
//   B     [beta K e^G | beta V] (MN-major 64 x 256)          L  .. M2
//         W (K-major 64 x 128) | V' (MN-major 64 x 128)      E2 .. M4
//   P     P tile (K-major 64 x 64)                           E1 .. M4
// A K-major tile with 128 columns is also the MN-major tile of its transpose,
// so K' serves directly as the A operand of K'^T V'.
#include "gdn_internal.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int C = 64, D = 128, NT = 256;

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

// Block-packed lower triangle of a 64 x 64 fp32 matrix: the ten 16 x 16
// blocks (bi >= bj) at id = bi(bi+1)/2 + bj, rows padded to 20 floats (16-byte
// aligned rows; eight consecutive rows cover all 32 banks).
constexpr int BLD = 20, BSZ = 16 * BLD;
__host__ __device__ constexpr int blk(int bi, int bj) { return (bi * (bi + 1) / 2 + bj) * BSZ; }

struct __align__(128) TcSmem {
    unsigned char S[D * D * 2];
    union {
        unsigned char KQ[2 * C * D * 2];
        struct {
            union {
                float Af[10 * BSZ];
                unsigned char T[C * C * 2];
            };
            float Tf[10 * BSZ];
            float Mscr[3 * 16 * 17];
        } inv;
        struct {
            unsigned char Kp[C * D * 2];
            unsigned char Qg[C * D * 2];
        } kq;
    } a;
    union {
        unsigned char R[C * 2 * D * 2];
        struct {
            unsigned char W[C * D * 2];
            unsigned char Vp[C * D * 2];
        } wv;
    } b;
    unsigned char P[C * C * 2];
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

// T = (I + A)^-1 for strictly lower A (64 x 64, fp32, block-packed), by
// 16 x 16 blocks: the four diagonal blocks by right-looking substitution (a
// dependency chain of 16 steps per column), then T_ij = -T_ii sum_k A_ik T_kj
// for the block diagonals i - j = 1, 2, 3 with interleaved accumulators.
__device__ void invert_unit_lower(TcSmem &sm, int t) {
    const float *A = sm.a.inv.Af;
    float *T = sm.a.inv.Tf, *M = sm.a.inv.Mscr;
    if (t < 64) {
        const int bb = t / 16, j = t % 16, o = blk(bb, bb);
        float acc[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) acc[r] = 0.f;
#pragma unroll
        for (int s = 0; s < 16; ++s) {
            const float xs = s < j ? 0.f : (s == j ? 1.f : -acc[s]);
            T[o + s * BLD + j] = xs;
#pragma unroll
            for (int r = s + 1; r < 16; ++r) acc[r] = fmaf(A[o + r * BLD + s], xs, acc[r]);
        }
    }
    __syncthreads();
    const int i = t / 16, j = t % 16;
    // level 1: M_b = A_{b+1,b} T_bb, then T_{b+1,b} = -T_{b+1,b+1} M_b  (b = 0, 1, 2)
    {
        float m0 = 0.f, m1 = 0.f, m2 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            m0 = fmaf(A[blk(1, 0) + i * BLD + k], T[blk(0, 0) + k * BLD + j], m0);
            m1 = fmaf(A[blk(2, 1) + i * BLD + k], T[blk(1, 1) + k * BLD + j], m1);
            m2 = fmaf(A[blk(3, 2) + i * BLD + k], T[blk(2, 2) + k * BLD + j], m2);
        }
        M[0 * 272 + i * 17 + j] = m0;
        M[1 * 272 + i * 17 + j] = m1;
        M[2 * 272 + i * 17 + j] = m2;
    }
    __syncthreads();
    {
        float t0 = 0.f, t1 = 0.f, t2 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            t0 = fmaf(T[blk(1, 1) + i * BLD + k], M[0 * 272 + k * 17 + j], t0);
            t1 = fmaf(T[blk(2, 2) + i * BLD + k], M[1 * 272 + k * 17 + j], t1);
            t2 = fmaf(T[blk(3, 3) + i * BLD + k], M[2 * 272 + k * 17 + j], t2);
        }
        T[blk(1, 0) + i * BLD + j] = -t0;
        T[blk(2, 1) + i * BLD + j] = -t1;
        T[blk(3, 2) + i * BLD + j] = -t2;
    }
    __syncthreads();
    // level 2: M_b = A_{b+2,b} T_bb + A_{b+2,b+1} T_{b+1,b}, T_{b+2,b} = -T_{b+2,b+2} M_b  (b = 0, 1)
    {
        float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            a0 = fmaf(A[blk(2, 0) + i * BLD + k], T[blk(0, 0) + k * BLD + j], a0);
            a1 = fmaf(A[blk(2, 1) + i * BLD + k], T[blk(1, 0) + k * BLD + j], a1);
            c0 = fmaf(A[blk(3, 1) + i * BLD + k], T[blk(1, 1) + k * BLD + j], c0);
            c1 = fmaf(A[blk(3, 2) + i * BLD + k], T[blk(2, 1) + k * BLD + j], c1);
        }
        M[0 * 272 + i * 17 + j] = a0 + a1;
        M[1 * 272 + i * 17 + j] = c0 + c1;
    }
    __syncthreads();
    {
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            t0 = fmaf(T[blk(2, 2) + i * BLD + k], M[0 * 272 + k * 17 + j], t0);
            t1 = fmaf(T[blk(3, 3) + i * BLD + k], M[1 * 272 + k * 17 + j], t1);
        }
        T[blk(2, 0) + i * BLD + j] = -t0;
        T[blk(3, 1) + i * BLD + j] = -t1;
    }
    __syncthreads();
    // level 3: M = A_30 T_00 + A_31 T_10 + A_32 T_20, T_30 = -T_33 M
    {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            a0 = fmaf(A[blk(3, 0) + i * BLD + k], T[blk(0, 0) + k * BLD + j], a0);
            a1 = fmaf(A[blk(3, 1) + i * BLD + k], T[blk(1, 0) + k * BLD + j], a1);
            a2 = fmaf(A[blk(3, 2) + i * BLD + k], T[blk(2, 0) + k * BLD + j], a2);
        }
        M[i * 17 + j] = a0 + a1 + a2;
    }
    __syncthreads();
    {
        float t0 = 0.f, t1 = 0.f;
#pragma unroll
        for (int k = 0; k < 16; k += 2) {
            t0 = fmaf(T[blk(3, 3) + i * BLD + k], M[k * 17 + j], t0);
            t1 = fmaf(T[blk(3, 3) + i * BLD + k + 1], M[(k + 1) * 17 + j], t1);
        }
        T[blk(3, 0) + i * BLD + j] = -(t0 + t1);
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

// In-chunk cumulative log decay and its exponentials, from the gate values
// the prefetch left in warp 0's registers.
__device__ __forceinline__ void chunk_gates(TcSmem &sm, const ChunkRegs &cr, int t) {
    if (t < 32) {
        const float g0 = cr.g0, g1 = cr.g1;
        float pair = g0 + g1, incl = pair;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            float u = __shfl_up_sync(0xffffffffu, incl, o);
            if (t >= o) incl += u;
        }
        const float excl = incl - pair, gl = __shfl_sync(0xffffffffu, incl, 31);
        const float G0 = excl + g0, G1 = incl;
        sm.G[2 * t] = G0;
        sm.G[2 * t + 1] = G1;
        sm.beta[2 * t] = cr.b0;
        sm.beta[2 * t + 1] = cr.b1;
        sm.eG[2 * t] = expf(G0);
        sm.eG[2 * t + 1] = expf(G1);
        sm.eGl[2 * t] = expf(gl - G0);
        sm.eGl[2 * t + 1] = expf(gl - G1);
    }
}

template <typename IT>
__global__ void __launch_bounds__(NT, 2) chunk_tc_kernel(kai_gdn_chunk_args p, int *err) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    TcSmem &sm = *reinterpret_cast<TcSmem *>(smem_raw);
    using TR = InTraits<IT>;

    const int t = threadIdx.x, warp = t / 32, lane = t % 32, q = warp % 4, hf = warp / 4;
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k, T = (long long)p.seq;
    const long long unit = blockIdx.x, b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const float scale = p.scale;
    // this thread's row and column groups in the chunk loads (see ChunkRegs)
    const int lr = 8 * warp + (lane % 8), la = lane / 8;

    if (t == 0) {
        mbar_init(&sm.bar, 1);
        sm.stop = 0;
    }
    if (warp == 0) tmem_alloc(&sm.tmem, 256);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = sm.tmem;
    const uint32_t TS = tm, TD1 = tm + 128, TLO = tm + 128, THI = tm + 128 + (16u << 16);
    uint32_t phase = 0;

    // ---- initial state: fp32 into TMEM columns 0..127, a 16-bit copy into sm.S
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
    chunk_gates(sm, cr, t);
    __syncthreads();

    for (long long c0 = 0; c0 < T; c0 += C) {
        // -------------------------------- L: raw K, Q -> [K;Q]; beta K e^G | beta V -> R
        {
            const float bk = sm.beta[lr] * sm.eG[lr], bv = sm.beta[lr];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int cc = 8 * (4 * i + la);
                *reinterpret_cast<uint4 *>(sm.a.KQ + kmaj16(lr, cc, D)) = cr.k[i];
                *reinterpret_cast<uint4 *>(sm.a.KQ + kmaj16(C + lr, cc, D)) = cr.q[i];
                const IT *kh = reinterpret_cast<const IT *>(&cr.k[i]), *vh = reinterpret_cast<const IT *>(&cr.v[i]);
                float kv[8], vv[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    kv[jj] = TR::to_f(kh[jj]) * bk;
                    vv[jj] = TR::to_f(vh[jj]) * bv;
                }
                st_vec8<IT>(sm.b.R, mnmaj16(lr, cc, 2 * D), kv);
                st_vec8<IT>(sm.b.R, mnmaj16(lr, D + cc, 2 * D), vv);
            }
        }
        // -------------------------------- M1: [K;Q] K^T
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id = idesc(128, 64, TR::fmt, false, false);
            for (int ks = 0; ks < D / 16; ++ks)
                mma_f16(TD1, desc_kmaj16(sm.a.KQ, D, ks), desc_kmaj16(sm.a.KQ, D, ks), id, ks > 0);
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // -------------------------------- E1: A (fp32, packed) and P (operand tile)
        {
            const int i = 32 * q + lane;  // row of [K;Q]K^T
            const int cb = hf * 32;
            float v[32];
            tmem_ld16(taddr(TD1, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&v[0]));
            tmem_ld16(taddr(TD1, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
            tmem_wait_ld();
            if (i < C) {
                const int r = i;
                const float gr = sm.G[r], br = sm.beta[r];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int s0 = cb + 16 * half;
                    if (s0 / 16 <= r / 16) {
                        float *dst = sm.a.inv.Af + blk(r / 16, s0 / 16) + (r % 16) * BLD;
#pragma unroll
                        for (int jj = 0; jj < 16; jj += 4) {
                            float4 f;
                            const int s = s0 + jj;
                            f.x = s + 0 < r ? br * v[16 * half + jj + 0] * __expf(gr - sm.G[s + 0]) : 0.f;
                            f.y = s + 1 < r ? br * v[16 * half + jj + 1] * __expf(gr - sm.G[s + 1]) : 0.f;
                            f.z = s + 2 < r ? br * v[16 * half + jj + 2] * __expf(gr - sm.G[s + 2]) : 0.f;
                            f.w = s + 3 < r ? br * v[16 * half + jj + 3] * __expf(gr - sm.G[s + 3]) : 0.f;
                            *reinterpret_cast<float4 *>(dst + jj) = f;
                        }
                    }
                }
            } else {
                const int r = i - C;
                const float gr = sm.G[r];
#pragma unroll
                for (int jj = 0; jj < 32; jj += 8) {
                    float a[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int s = cb + jj + u;
                        a[u] = s <= r ? scale * v[jj + u] * __expf(gr - sm.G[s]) : 0.f;
                    }
                    st_vec8<IT>(sm.P, kmaj16(r, cb + jj, C), a);
                }
            }
        }
        __syncthreads();
        // -------------------------------- INV: T = (I + A)^-1 -> operand tile (over A)
        invert_unit_lower(sm, t);
        for (int e = t; e < C * C / 8; e += NT) {
            const int r = e % C, s0 = (e / C) * 8;
            float v[8];
            if (s0 / 16 <= r / 16) {
                const float *src = sm.a.inv.Tf + blk(r / 16, s0 / 16) + (r % 16) * BLD + (s0 % 16);
                const float4 x0 = *reinterpret_cast<const float4 *>(src);
                const float4 x1 = *reinterpret_cast<const float4 *>(src + 4);
                v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
                v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
            } else {
#pragma unroll
                for (int u = 0; u < 8; ++u) v[u] = 0.f;
            }
            st_vec8<IT>(sm.a.inv.T, kmaj16(r, s0, C), v);
        }
        // -------------------------------- M2: W = T (beta K e^G) -> lower, U = T (beta V) -> upper
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id = idesc(64, 128, TR::fmt, false, true);
            const uint32_t rb = smem_addr(sm.b.R), lbo = (2 * D / 8) * 128;
            for (int ks = 0; ks < C / 16; ++ks) {
                const uint64_t ad = desc_kmaj16(sm.a.inv.T, C, ks);
                mma_f16(TLO, ad, smem_desc(rb + ks * 2 * lbo, lbo, 128), id, ks > 0);
                mma_f16(THI, ad, smem_desc(rb + (D / 8) * 128 + ks * 2 * lbo, lbo, 128), id, ks > 0);
            }
            commit(&sm.bar);
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // -------------------------------- E2: W -> tile; K', Qg -> region A; prefetch next
        {
            const int r = 16 * q + lane;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int cb = hf * 64 + 32 * half;
                float w[32];
                tmem_ld16(taddr(TLO, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&w[0]));
                tmem_ld16(taddr(TLO, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&w[16]));
                tmem_wait_ld();
                if (lane < 16) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        float a[8];
#pragma unroll
                        for (int x = 0; x < 8; ++x) a[x] = w[8 * u + x];
                        st_vec8<IT>(sm.b.wv.W, kmaj16(r, cb + 8 * u, D), a);
                    }
                }
            }
        }
        __syncthreads();  // the T tile (region A) is dead once every thread is past M2's wait
        {
            const float fk = sm.eGl[lr], fq = scale * sm.eG[lr];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int cc = 8 * (4 * i + la);
                const IT *kh = reinterpret_cast<const IT *>(&cr.k[i]), *qh = reinterpret_cast<const IT *>(&cr.q[i]);
                float kv[8], qv[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    kv[jj] = TR::to_f(kh[jj]) * fk;
                    qv[jj] = TR::to_f(qh[jj]) * fq;
                }
                st_vec8<IT>(sm.a.kq.Kp, kmaj16(lr, cc, D), kv);
                st_vec8<IT>(sm.a.kq.Qg, kmaj16(lr, cc, D), qv);
            }
            if (c0 + C < T) prefetch_chunk<IT>(cr, p, b, h, hk, c0 + C, t);
        }
        // -------------------------------- M3: W S -> lower   (overlap: S *= gamma)
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id = idesc(64, 128, TR::fmt, false, true);
            for (int ks = 0; ks < D / 16; ++ks)
                mma_f16(TLO, desc_kmaj16(sm.b.wv.W, D, ks), desc_mnmaj16(sm.S, D, ks), id, ks > 0);
            commit(&sm.bar);
        }
        {
            // TMEM columns 0..127 are not touched by M3 (it reads the copy in sm.S).
            const float gamma = sm.eG[C - 1];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int cb = hf * 64 + 32 * half;
                float s[32];
                tmem_ld16(taddr(TS, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&s[0]));
                tmem_ld16(taddr(TS, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&s[16]));
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < 32; ++x) s[x] *= gamma;
                tmem_st16(taddr(TS, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&s[0]));
                tmem_st16(taddr(TS, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&s[16]));
            }
            tmem_wait_st();
        }
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // -------------------------------- E3: V' = U - W S -> tile (lanes 0-15 W S, 16-31 U)
        {
            const int r = 16 * q + lane;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int cb = hf * 64 + 32 * half;
                float x[32];
                tmem_ld16(taddr(TLO, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&x[0]));
                tmem_ld16(taddr(TLO, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&x[16]));
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float a[8];
#pragma unroll
                    for (int y = 0; y < 8; ++y) {
                        const float uu = __shfl_down_sync(0xffffffffu, x[8 * u + y], 16);
                        a[y] = uu - x[8 * u + y];
                    }
                    if (lane < 16) st_vec8<IT>(sm.b.wv.Vp, mnmaj16(r, cb + 8 * u, D), a);
                }
            }
        }
        // -------------------------------- M4: O = Qg S + P V' -> upper; S += K'^T V'  (overlap: next gates)
        issue_sync();
        if (sm.stop) break;
        if (t == 0) {
            const uint32_t id_o = idesc(64, 128, TR::fmt, false, true);
            const uint32_t id_s = idesc(128, 128, TR::fmt, true, true);
            for (int ks = 0; ks < D / 16; ++ks)
                mma_f16(THI, desc_kmaj16(sm.a.kq.Qg, D, ks), desc_mnmaj16(sm.S, D, ks), id_o, ks > 0);
            for (int ks = 0; ks < C / 16; ++ks) {
                const uint64_t vd = desc_mnmaj16(sm.b.wv.Vp, D, ks);
                mma_f16(THI, desc_kmaj16(sm.P, C, ks), vd, id_o, true);
                mma_f16(TS, desc_mnmaj16(sm.a.kq.Kp, D, ks), vd, id_s, true);
            }
            commit(&sm.bar);
        }
        const bool more = c0 + C < T;
        if (more) chunk_gates(sm, cr, t);  // G, beta, e^G of the next chunk (M4 does not read them)
        if (!mbar_wait(&sm.bar, phase, err)) sm.stop = 1;
        phase ^= 1;
        fence_after_sync();
        // -------------------------------- E4: O out (lanes 16-31); S -> operand copy
        {
            const int r = 16 * q + lane - 16;
            const long long tok = c0 + r;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int cb = hf * 64 + 32 * half;
                float o[32];
                tmem_ld16(taddr(THI - (16u << 16), 32 * q, cb), *reinterpret_cast<float(*)[16]>(&o[0]));
                tmem_ld16(taddr(THI - (16u << 16), 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&o[16]));
                tmem_wait_ld();
                if (lane >= 16 && tok < T) {
                    const size_t oi = ((size_t)(b * T + tok) * Hv + h) * D + cb;
                    st16_out(p.o, oi, p.out_dtype, *reinterpret_cast<float(*)[16]>(&o[0]));
                    st16_out(p.o, oi + 16, p.out_dtype, *reinterpret_cast<float(*)[16]>(&o[16]));
                }
            }
            const int d = 32 * q + lane;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int cb = hf * 64 + 32 * half;
                float s[32];
                tmem_ld16(taddr(TS, 32 * q, cb), *reinterpret_cast<float(*)[16]>(&s[0]));
                tmem_ld16(taddr(TS, 32 * q, cb + 16), *reinterpret_cast<float(*)[16]>(&s[16]));
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float a[8];
#pragma unroll
                    for (int x = 0; x < 8; ++x) a[x] = s[8 * u + x];
                    st_vec8<IT>(sm.S, mnmaj16(d, cb + 8 * u, D), a);
                }
            }
        }
        fence_before_sync();
        __syncthreads();
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
    if (warp == 0) tmem_dealloc(tm, 256);
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
    int *flag = nullptr;
    int rc = device_error_word(&flag);
    if (rc) return rc;
    const size_t smem = sizeof(TcSmem);
    if (a->in_dtype == KAI_GDN_BF16) {
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__nv_bfloat16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "chunk_tc: smem attribute");
        if (rc) return rc;
        // two CTAs per SM need the largest shared-memory carveout
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__nv_bfloat16>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared),
                        "chunk_tc: carveout attribute");
        if (rc) return rc;
        chunk_tc_kernel<__nv_bfloat16><<<(unsigned)units, NT, smem, st>>>(*a, flag);
    } else {
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "chunk_tc: smem attribute");
        if (rc) return rc;
        // two CTAs per SM need the largest shared-memory carveout
        rc = check_cuda(cudaFuncSetAttribute(chunk_tc_kernel<__half>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared),
                        "chunk_tc: carveout attribute");
        if (rc) return rc;
        chunk_tc_kernel<__half><<<(unsigned)units, NT, smem, st>>>(*a, flag);
    }
    return check_launch("chunk_delta_rule_tc");
}

}  // namespace gdn
