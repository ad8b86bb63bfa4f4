// chunk.cu -- chunkwise (WY / UT-transform) gated delta-rule scan, fp32 on
// CUDA cores (sm_100a).
//
// The form named in docs/GDN_ARCHITECTURE_AUDIT.md:142-153 (the reference
// reaches it only through HF transformers' torch_chunk_gated_delta_rule).
// Per (batch b, value head h) and chunk of C = 64 tokens, with G_r the
// in-chunk cumulative log-decay, Q already multiplied by `scale`:
//   A[r][s] = beta_r (k_r . k_s) exp(G_r - G_s)              s <  r
//   P[r][s] = (q_r . k_s) exp(G_r - G_s)                     s <= r
//   W = (I + A)^-1 (beta * K * exp(G)),   U = (I + A)^-1 (beta * V)
//   V' = U - W S
//   O  = (Q * exp(G)) S + P V'
//   S <- exp(G_last) S + (K * exp(G_last - G))^T V'
// (I + A)^-1 is applied by forward substitution, one thread per column.
//
// Work split: one CTA per (b, h, block of DVB value columns).  Every quantity
// above except S, U, V', O depends on the key side only, and the state's value
// columns evolve independently, so value-column blocks are exact splits (the
// key-side work is recomputed per block).  The state block lives in shared
// memory for the whole sequence; the sequence is walked chunk by chunk.
//
// All products use 16x16 thread tiles with fp32 FMA; this is the fp32-exact
// path (1e-4 relative L2 against the token loop) and the reference point for
// the tensor-core kernel.
#include "gdn_internal.cuh"

namespace gdn {
namespace {

constexpr int CH = 64;        // chunk length
constexpr int THREADS = 256;  // 16 x 16

__device__ __forceinline__ void st_any(void *p, size_t i, int dt, float v) {
    switch (dt) {
        case KAI_GDN_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
        case KAI_GDN_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
        default: static_cast<float *>(p)[i] = v;
    }
}

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

// One chunk's k, q (CH x DK) and v (CH x DVB) tiles into
// shared memory.  Every load of the thread is issued before the first store,
// so a chunk waits for one global-memory latency rather than one per element;
// rows past T read as zeros.
template <typename ET, int DK, int DVB, int LDK, int LDV>
__device__ __forceinline__ void load_chunk_tiles(const kai_gdn_chunk_args &p, float *K, float *Q, float *V, long long b,
                                                 long long h, long long hk, long long c0, long long v0, int t) {
    constexpr int NKQ = CH * DK / THREADS, NV = CH * DVB / THREADS;
    const long long T = (long long)p.seq, Hv = (long long)p.heads_v, Hk = (long long)p.heads_k;
    const long long DV = (long long)p.dv;
    const ET *kp = static_cast<const ET *>(p.k), *qp = static_cast<const ET *>(p.q), *vp = static_cast<const ET *>(p.v);
    float kr[NKQ], qr[NKQ], vr[NV];
#pragma unroll
    for (int u = 0; u < NKQ; ++u) {
        const int e = t + u * THREADS, r = e / DK, d = e % DK;
        const long long tok = c0 + r;
        kr[u] = 0.f;
        qr[u] = 0.f;
        if (tok < T) {
            const size_t i = ((size_t)(b * T + tok) * Hk + hk) * DK + d;
            kr[u] = to_f(kp[i]);
            qr[u] = to_f(qp[i]);
        }
    }
#pragma unroll
    for (int u = 0; u < NV; ++u) {
        const int e = t + u * THREADS, r = e / DVB, n = e % DVB;
        const long long tok = c0 + r;
        vr[u] = tok < T ? to_f(vp[((size_t)(b * T + tok) * Hv + h) * DV + v0 + n]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < NKQ; ++u) {
        const int e = t + u * THREADS, r = e / DK, d = e % DK;
        K[r * LDK + d] = kr[u];
        Q[r * LDK + d] = qr[u];
    }
#pragma unroll
    for (int u = 0; u < NV; ++u) {
        const int e = t + u * THREADS, r = e / DVB, n = e % DVB;
        V[r * LDV + n] = vr[u];
    }
}

// fp32 inputs: the same tiles by asynchronous 16-byte copies (cp.async), so
// the next chunk's tiles land while this chunk computes; rows past T are
// zero-filled (source size 0).  Pointers 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
template <int DK, int DVB, int LDK, int LDV>
__device__ __forceinline__ void copy_chunk_tiles(const kai_gdn_chunk_args &p, float *K, float *Q, float *V, long long b,
                                                 long long h, long long hk, long long c0, long long v0, int t) {
    const long long T = (long long)p.seq, Hv = (long long)p.heads_v, Hk = (long long)p.heads_k;
    const long long DV = (long long)p.dv;
    const float *kp = static_cast<const float *>(p.k), *qp = static_cast<const float *>(p.q);
    const float *vp = static_cast<const float *>(p.v);
    constexpr int QK = DK / 4, QV = DVB / 4;  // 16-byte pieces per row
#pragma unroll
    for (int u = 0; u < CH * QK / THREADS; ++u) {
        const int e = t + u * THREADS, r = e / QK, q = e % QK;
        const long long tok = c0 + r;
        const bool ok = tok < T;
        const size_t i = ok ? ((size_t)(b * T + tok) * Hk + hk) * DK + 4 * q : 0;
        cp_async16(K + r * LDK + 4 * q, kp + i, ok);
        cp_async16(Q + r * LDK + 4 * q, qp + i, ok);
    }
#pragma unroll
    for (int u = 0; u < (CH * QV + THREADS - 1) / THREADS; ++u) {
        const int e = t + u * THREADS;
        if (e < CH * QV) {
            const int r = e / QV, q = e % QV;
            const long long tok = c0 + r;
            const bool ok = tok < T;
            const size_t i = ok ? ((size_t)(b * T + tok) * Hv + h) * DV + v0 + 4 * q : 0;
            cp_async16(V + r * LDV + 4 * q, vp + i, ok);
        }
    }
}

// acc[i][j] += sum_k a(ty + 16 i, k) * b(k, tx + 16 j)
//   a(m, k) = TA ? A[k*lda + m] : A[m*lda + k];  b(k, n) = TB ? B[n*ldb + k] : B[k*ldb + n]
template <int MI, int NJ, bool TA, bool TB>
__device__ __forceinline__ void mm(float (&acc)[MI][NJ], const float *A, int lda,
                                   const float *B, int ldb, int kd) {
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll 4
    for (int k = 0; k < kd; ++k) {
        float a[MI], b[NJ];
#pragma unroll
        for (int i = 0; i < MI; ++i) a[i] = TA ? A[k * lda + ty + 16 * i] : A[(ty + 16 * i) * lda + k];
#pragma unroll
        for (int j = 0; j < NJ; ++j) b[j] = TB ? B[(tx + 16 * j) * ldb + k] : B[k * ldb + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
}

// The same with A row-major (not transposed) read four k at a time: rows of
// A 16-byte aligned, lda and kd multiples of 4.  The sums run in k order.
template <int MI, int NJ>
__device__ __forceinline__ void mm_k4(float (&acc)[MI][NJ], const float *A, int lda, const float *B, int ldb, int kd) {
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll 2
    for (int k = 0; k < kd; k += 4) {
        float4 a[MI];
#pragma unroll
        for (int i = 0; i < MI; ++i) a[i] = *reinterpret_cast<const float4 *>(A + (ty + 16 * i) * lda + k);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float b[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j) b[j] = B[(k + u) * ldb + tx + 16 * j];
#pragma unroll
            for (int i = 0; i < MI; ++i) {
                const float av = u == 0 ? a[i].x : u == 1 ? a[i].y : u == 2 ? a[i].z : a[i].w;
#pragma unroll
                for (int j = 0; j < NJ; ++j) acc[i][j] = fmaf(av, b[j], acc[i][j]);
            }
        }
    }
}
// acc[i][j] += sum_k A[k*lda + MI ty + i] * B[k*ldb + tx + 16 j]: A transposed,
// each thread on MI CONSECUTIVE rows (read as float4), MI a multiple of 4.
template <int MI, int NJ>
__device__ __forceinline__ void mm_t4(float (&acc)[MI][NJ], const float *A, int lda, const float *B, int ldb, int kd) {
    static_assert(MI % 4 == 0, "rows in 16-byte groups");
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
#pragma unroll 4
    for (int k = 0; k < kd; ++k) {
        float a[MI], b[NJ];
#pragma unroll
        for (int i = 0; i < MI; i += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(A + k * lda + MI * ty + i);
            a[i] = v.x;
            a[i + 1] = v.y;
            a[i + 2] = v.z;
            a[i + 3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) b[j] = B[k * ldb + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < MI; ++i)
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
}

template <int MI, int NJ>
__device__ __forceinline__ void zero(float (&acc)[MI][NJ]) {
#pragma unroll
    for (int i = 0; i < MI; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
}

// Rows of every tile 16-byte aligned (cp.async and float4 reads); K, Q, V
// double-buffered when two sets fit in shared memory (the next chunk's
// tiles are copied in while this one computes).
template <int DK, int DVB>
struct Geom {
    static constexpr int LDK = DK + 4;   // 4 banks apart: 8 rows fill the 32 banks
    static constexpr int LDV = DVB + 4;
    static constexpr int LDP = CH + 4;
    static constexpr size_t one = sizeof(float) * (2 * CH * LDK + CH * LDV);
    static constexpr size_t rest = sizeof(float) * (2 * CH * LDP + DK * LDV + 4 * CH);
    static constexpr int NB = 2 * one + rest <= 227 * 1024 ? 2 : 1;
};
template <int DK, int DVB>
struct Smem {
    using Gm = Geom<DK, DVB>;
    static constexpr int LDK = Gm::LDK, LDV = Gm::LDV, LDP = Gm::LDP, NB = Gm::NB;
    float K[NB][CH * LDK];
    float Q[NB][CH * LDK];
    float V[NB][CH * LDV];  // V, then beta (V - exp(G) K S), then V', then V' exp(G_last - G)
    float A[CH * LDP];      // strictly lower A
    float P[CH * LDP];      // lower-with-diagonal P (times scale)
    float S[DK * LDV];      // state block [DK][DVB]
    float G[CH], eG[CH], eGl[CH], beta[CH];
};

template <int DK, int DVB, int SDT>
__global__ void __launch_bounds__(THREADS, 1) chunk_scan_fp32_kernel(kai_gdn_chunk_args p) {
    using SM = Smem<DK, DVB>;
    constexpr int LDK = SM::LDK, LDV = SM::LDV, LDP = SM::LDP, NB = SM::NB;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SM &sm = *reinterpret_cast<SM *>(smem_raw);

    const int t = threadIdx.x, tx = t % 16, ty = t / 16;
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k;
    const long long T = (long long)p.seq, DV = (long long)p.dv;
    const int nvb = (int)(DV / DVB);
    const long long unit = blockIdx.x / nvb;  // b * Hv + h
    const int vb = blockIdx.x % nvb;
    const long long b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const long long v0 = (long long)vb * DVB;

    // State block in.
    using S = Store<SDT>;
    const typename S::T *st_in = static_cast<const typename S::T *>(p.state) + (size_t)unit * DK * DV;
    for (int e = t; e < DK * DVB; e += THREADS) {
        int d = e / DVB, n = e % DVB;
        sm.S[d * LDV + n] = S::load(st_in + (size_t)d * DV + v0 + n);
    }

    // fp32 inputs with 16-byte aligned pointers are copied asynchronously,
    // one chunk ahead when the tiles are double-buffered; others go through
    // registers.
    const bool async = p.in_dtype == KAI_GDN_F32 && ((reinterpret_cast<uintptr_t>(p.q) |
                                                      reinterpret_cast<uintptr_t>(p.k) |
                                                      reinterpret_cast<uintptr_t>(p.v)) % 16) == 0;
    auto load_tiles = [&](long long cc0, int bi) {
        if (async) {
            copy_chunk_tiles<DK, DVB, LDK, LDV>(p, sm.K[bi], sm.Q[bi], sm.V[bi], b, h, hk, cc0, v0, t);
            cp_async_commit();
            return;
        }
        switch (p.in_dtype) {
            case KAI_GDN_BF16:
                load_chunk_tiles<__nv_bfloat16, DK, DVB, LDK, LDV>(p, sm.K[bi], sm.Q[bi], sm.V[bi], b, h, hk, cc0, v0, t);
                break;
            case KAI_GDN_F16:
                load_chunk_tiles<__half, DK, DVB, LDK, LDV>(p, sm.K[bi], sm.Q[bi], sm.V[bi], b, h, hk, cc0, v0, t);
                break;
            default: load_chunk_tiles<float, DK, DVB, LDK, LDV>(p, sm.K[bi], sm.Q[bi], sm.V[bi], b, h, hk, cc0, v0, t);
        }
    };
    // gates of the next chunk, held by warp 0 (tokens 2 lane, 2 lane + 1)
    float gn0 = 0.f, gn1 = 0.f, bn0 = 0.f, bn1 = 0.f;
    auto load_gates = [&](long long cc0) {
        const long long r0 = cc0 + 2 * t, r1 = r0 + 1;
        gn0 = r0 < T ? p.g[(size_t)(b * T + r0) * Hv + h] : 0.f;
        bn0 = r0 < T ? p.beta[(size_t)(b * T + r0) * Hv + h] : 0.f;
        gn1 = r1 < T ? p.g[(size_t)(b * T + r1) * Hv + h] : 0.f;
        bn1 = r1 < T ? p.beta[(size_t)(b * T + r1) * Hv + h] : 0.f;
    };
    if (NB == 2) load_tiles(0, 0);
    if (t < 32) load_gates(0);

    for (long long c0 = 0; c0 < T; c0 += CH) {
        const int bi = NB == 2 ? (int)((c0 / CH) & 1) : 0;
        float *const cK = sm.K[bi], *const cQ = sm.Q[bi], *const cV = sm.V[bi];
        // ---- loads (rows past T are zero padding with g = beta = 0)
        if (NB == 2) {
            // this chunk's tiles were requested one chunk ago; request the next
            // chunk's into the other buffer (last read by the previous chunk)
            if (c0 + CH < T) {
                load_tiles(c0 + CH, bi ^ 1);
                if (async) cp_async_wait<1>();
            } else if (async) {
                cp_async_wait<0>();
            }
        } else {
            load_tiles(c0, 0);
            if (async) cp_async_wait<0>();
        }
        if (t < 32) {
            // In-chunk inclusive cumsum of g (2 rows per lane), beta.
            const float g0 = gn0, g1 = gn1, b0 = bn0, b1 = bn1;
            if (c0 + CH < T) load_gates(c0 + CH);
            float pair = g0 + g1, incl = pair;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                float u = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += u;
            }
            float excl = incl - pair;
            sm.G[2 * t] = excl + g0;
            sm.G[2 * t + 1] = incl;
            sm.beta[2 * t] = b0;
            sm.beta[2 * t + 1] = b1;
        }
        __syncthreads();
        if (t < CH) {
            sm.eG[t] = expf(sm.G[t]);
            sm.eGl[t] = expf(sm.G[CH - 1] - sm.G[t]);
        }
        // ---- A = beta K K^T decay (s < r), P = scale Q K^T decay (s <= r)
        {
            float kk[4][4], qk[4][4];
            zero(kk);
            zero(qk);
            // four features per 16-byte load; the sums still run in feature order
#pragma unroll 2
            for (int d = 0; d < DK; d += 4) {
                float4 kr[4], qr[4], ks[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    kr[i] = *reinterpret_cast<const float4 *>(&cK[(ty + 16 * i) * LDK + d]);
                    qr[i] = *reinterpret_cast<const float4 *>(&cQ[(ty + 16 * i) * LDK + d]);
                    ks[i] = *reinterpret_cast<const float4 *>(&cK[(tx + 16 * i) * LDK + d]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        kk[i][j] = fmaf(kr[i].x, ks[j].x, kk[i][j]);
                        kk[i][j] = fmaf(kr[i].y, ks[j].y, kk[i][j]);
                        kk[i][j] = fmaf(kr[i].z, ks[j].z, kk[i][j]);
                        kk[i][j] = fmaf(kr[i].w, ks[j].w, kk[i][j]);
                        qk[i][j] = fmaf(qr[i].x, ks[j].x, qk[i][j]);
                        qk[i][j] = fmaf(qr[i].y, ks[j].y, qk[i][j]);
                        qk[i][j] = fmaf(qr[i].z, ks[j].z, qk[i][j]);
                        qk[i][j] = fmaf(qr[i].w, ks[j].w, qk[i][j]);
                    }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    int r = ty + 16 * i, s = tx + 16 * j;
                    float dec = r >= s ? expf(sm.G[r] - sm.G[s]) : 0.f;
                    sm.A[r * LDP + s] = r > s ? sm.beta[r] * kk[i][j] * dec : 0.f;
                    sm.P[r * LDP + s] = p.scale * qk[i][j] * dec;
                }
        }
        __syncthreads();
        // ---- right-hand side R = beta (V - exp(G) (K S)), in place over V
        {
            float ks[4][DVB / 16];
            zero(ks);
            mm_k4<4, DVB / 16>(ks, cK, LDK, sm.S, LDV, DK);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = ty + 16 * i;
                const float br = sm.beta[r], bg = br * sm.eG[r];
#pragma unroll
                for (int j = 0; j < DVB / 16; ++j) {
                    float &x = cV[r * LDV + tx + 16 * j];
                    x = br * x - bg * ks[i][j];
                }
            }
        }
        __syncthreads();
        // ---- V' = (I + A)^-1 R: right-looking substitution, a group of GT
        // consecutive lanes per column, rows r = j + GT m held by thread j of
        // the group; x_r is final when step r starts and is broadcast to the
        // group by a shuffle.
        {
            constexpr int GT = THREADS / DVB, RPT = CH / GT;
            static_assert(GT <= 32 && 32 % GT == 0, "column groups inside a warp");
            const int n = t / GT, j = t % GT, lane = t % 32;
            float x[RPT];
#pragma unroll
            for (int m = 0; m < RPT; ++m) x[m] = cV[(j + GT * m) * LDV + n];
#pragma unroll 1
            for (int r = 0; r < CH - 1; ++r) {
                const int owner = r % GT, mr = r / GT;
                float xr = 0.f;
#pragma unroll
                for (int m = 0; m < RPT; ++m)
                    if (m == mr) xr = x[m];
                xr = __shfl_sync(0xffffffffu, xr, lane - j + owner);
#pragma unroll
                for (int m = 0; m < RPT; ++m) {
                    const int i = j + GT * m;
                    if (i > r) x[m] = fmaf(-sm.A[i * LDP + r], xr, x[m]);
                }
            }
#pragma unroll
            for (int m = 0; m < RPT; ++m) cV[(j + GT * m) * LDV + n] = x[m];
        }
        __syncthreads();
        // ---- O = scale exp(G) (Q S) + P V'
        {
            float o[4][DVB / 16];
            zero(o);
            mm_k4<4, DVB / 16>(o, cQ, LDK, sm.S, LDV, DK);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float f = p.scale * sm.eG[ty + 16 * i];
#pragma unroll
                for (int j = 0; j < DVB / 16; ++j) o[i][j] *= f;
            }
            mm_k4<4, DVB / 16>(o, sm.P, LDP, cV, LDV, CH);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                long long tok = c0 + ty + 16 * i;
                if (tok < T) {
#pragma unroll
                    for (int j = 0; j < DVB / 16; ++j)
                        st_any(p.o, ((size_t)(b * T + tok) * Hv + h) * DV + v0 + tx + 16 * j, p.out_dtype,
                               o[i][j]);
                }
            }
        }
        __syncthreads();
        // V'' = V' exp(G_last - G) in place (O has read V')
        for (int e = t; e < CH * DVB; e += THREADS) {
            const int r = e / DVB, n = e % DVB;
            cV[r * LDV + n] *= sm.eGl[r];
        }
        __syncthreads();
        // ---- S = exp(G_last) S + K^T V''
        {
            // thread rows MI ty .. MI ty + MI-1 when MI is a multiple of 4, else ty + 16 i
            constexpr int MI = DK / 16, NJ = DVB / 16;
            constexpr bool V4 = MI % 4 == 0;
            auto row = [&](int i) { return V4 ? MI * ty + i : ty + 16 * i; };
            float acc[MI][NJ];
            const float egl = sm.eG[CH - 1];
#pragma unroll
            for (int i = 0; i < MI; ++i)
#pragma unroll
                for (int j = 0; j < NJ; ++j) acc[i][j] = egl * sm.S[row(i) * LDV + tx + 16 * j];
            if constexpr (V4)
                mm_t4<MI, NJ>(acc, cK, LDK, cV, LDV, CH);
            else
                mm<MI, NJ, true, false>(acc, cK, LDK, cV, LDV, CH);
#pragma unroll
            for (int i = 0; i < MI; ++i)
#pragma unroll
                for (int j = 0; j < NJ; ++j) sm.S[row(i) * LDV + tx + 16 * j] = acc[i][j];
        }
        __syncthreads();
    }

    typename S::T *st_out = static_cast<typename S::T *>(p.state) + (size_t)unit * DK * DV;
    for (int e = t; e < DK * DVB; e += THREADS) {
        int d = e / DVB, n = e % DVB;
        S::store(st_out + (size_t)d * DV + v0 + n, sm.S[d * LDV + n]);
    }
}

template <int DK, int DVB>
int run_chunk(const kai_gdn_chunk_args *a, cudaStream_t st) {
    const size_t smem = sizeof(Smem<DK, DVB>);
    const long long blocks = (long long)(a->batch * a->heads_v) * (long long)(a->dv / DVB);
    if (blocks > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk: too many heads");
    int rc = 0;
    switch (a->state_dtype) {
        case KAI_GDN_F32:
            rc = check_cuda(cudaFuncSetAttribute(chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_F32>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "chunk: smem attribute");
            if (!rc) chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_F32><<<(unsigned)blocks, THREADS, smem, st>>>(*a);
            break;
        case KAI_GDN_F16:
            rc = check_cuda(cudaFuncSetAttribute(chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_F16>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "chunk: smem attribute");
            if (!rc) chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_F16><<<(unsigned)blocks, THREADS, smem, st>>>(*a);
            break;
        case KAI_GDN_BF16:
            rc = check_cuda(cudaFuncSetAttribute(chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_BF16>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                            "chunk: smem attribute");
            if (!rc) chunk_scan_fp32_kernel<DK, DVB, KAI_GDN_BF16><<<(unsigned)blocks, THREADS, smem, st>>>(*a);
            break;
    }
    if (rc) return rc;
    return check_launch("chunk_delta_rule_fp32");
}

}  // namespace

int launch_chunk_fp32(const kai_gdn_chunk_args *a, cudaStream_t st) {
    // 64 value columns per CTA halve the recomputed key side; with too few
    // (batch, head) units to fill the SMs, 32 columns double the CTAs.
    const bool few = (long long)(a->batch * a->heads_v) * (long long)(a->dv / 64) < 148;
    if (a->dk == 128 && a->dv % 64 == 0 && !few) return run_chunk<128, 64>(a, st);
    if (a->dk == 64 && a->dv % 64 == 0) return run_chunk<64, 64>(a, st);
    if (a->dk == 32 && a->dv % 32 == 0) return run_chunk<32, 32>(a, st);
    if (a->dk == 64 && a->dv % 32 == 0) return run_chunk<64, 32>(a, st);
    if (a->dk == 128 && a->dv % 32 == 0) return run_chunk<128, 32>(a, st);
    return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk: dk %zu / dv %zu (supported: dk in {32,64,128}, "
                     "dv a multiple of 32)", a->dk, a->dv);
}

int launch_chunk(const kai_gdn_chunk_args *a, cudaStream_t st) {
    if (!a) return set_error(KAI_GDN_ERR_INVALID, "chunk: null args");
    if (a->batch == 0 || a->heads_v == 0 || a->seq == 0) return KAI_GDN_OK;
    if (!a->q || !a->k || !a->v || !a->g || !a->beta || !a->state || !a->o)
        return set_error(KAI_GDN_ERR_INVALID, "chunk: null pointer");
    if (a->heads_k == 0 || a->heads_v % a->heads_k)
        return set_error(KAI_GDN_ERR_INVALID, "chunk: heads_v %zu not a multiple of heads_k %zu",
                         a->heads_v, a->heads_k);
    if (!valid_dtype(a->in_dtype) || !valid_dtype(a->state_dtype) || !valid_dtype(a->out_dtype))
        return set_error(KAI_GDN_ERR_INVALID, "chunk: bad dtype");
    if (a->chunk != (size_t)CH)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk: chunk length %zu (supported: 64)", a->chunk);
    // At the model's head size both input precisions run on the tensor
    // cores (bf16 / fp16 inputs in one warp-specialised kernel, fp32 inputs
    // fp32-accurate in two launches); other head sizes take the fp32
    // CUDA-core kernel.
    if (chunk_ws_supported(a)) return launch_chunk_ws(a, st);
    if (chunk_tc32_supported(a)) return launch_chunk_tc32(a, st);
    return launch_chunk_fp32(a, st);
}

}  // namespace gdn
