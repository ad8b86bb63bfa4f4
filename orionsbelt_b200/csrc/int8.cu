// int8.cu -- int8 weights with one fp32 scale per output column, the weight
// format of the reference's INT8_WEIGHTS decode path:
//   quantize_weight  src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:175-199
//   gemv_int8_neon   gdn_e2e_decode.c:296-358   (M = 1)
//   gemm_int8_neon   gdn_e2e_decode.c:608-678   (M > 1)
//   matmul_int8      gdn_e2e_decode.c:681       (the dispatcher the model calls)
// Layouts as there: B, q [K][N] row-major, s [N], A [M][K], C [M][N].
//
// Quantization is bit-identical to the reference (IEEE division, one rounding
// per product, lroundf = round half away from zero, clamp to [-128, 127]).
// The products sum in fp32 in a different order than the reference's
// k-by-k loop (split over K, fused multiply-add), then take the column scale
// as it does: C = (A q) diag(s).
//
// Weight streaming (M <= 16, the decode shapes): a CTA owns a slab of 64
// columns and a K range, reads 16 columns of a weight row per 16-byte copy and
// keeps up to 12 rows per thread in flight through a cp.async ring; when K is
// split, the parts are added in K order by the slab's last CTA, so the result
// does not depend on timing.  (A thread-block cluster adding the parts through
// distributed shared memory measured ~2 us slower per launch on B200: the
// cluster launch itself.)  The int8 values become fp32 through the exponent
// trick (the byte, biased by 128, is placed in the mantissa of 2^23 and the
// bias subtracted), which is exact.
// Larger M (prefill) takes a tiled CUDA-core GEMM.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <vector>

#include "gdn_internal.cuh"

namespace gdn {
namespace {

// ------------------------------------------------------------ quantization
// A CTA per 32 columns, 8 row lanes: the column max over the lanes' rows
// (order does not matter), then every lane quantizes its rows.
__global__ void __launch_bounds__(256) quantize_int8_kernel(const float *__restrict__ B, int8_t *__restrict__ q,
                                                            float *__restrict__ s, long long K, long long N) {
    __shared__ float part[8][32];
    __shared__ float s_inv[32];
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    const long long n = (long long)blockIdx.x * 32 + tx;
    const bool live = n < N;
    float mx = 0.0f;
    if (live) {
#pragma unroll 4
        for (long long k = ty; k < K; k += 8) {
            const float v = fabsf(B[k * N + n]);
            if (v > mx) mx = v;
        }
    }
    part[ty][tx] = mx;
    __syncthreads();
    if (ty == 0) {
#pragma unroll
        for (int r = 1; r < 8; ++r) mx = fmaxf(mx, part[r][tx]);
        const float sc = mx > 0.0f ? mx / 127.0f : 1.0f;
        s_inv[tx] = 1.0f / sc;
        if (live) s[n] = sc;
    }
    __syncthreads();
    if (!live) return;
    const float inv = s_inv[tx];
#pragma unroll 4
    for (long long k = ty; k < K; k += 8) {
        long v = lroundf(__fmul_rn(B[k * N + n], inv));
        v = v > 127 ? 127 : (v < -128 ? -128 : v);
        q[k * N + n] = (int8_t)v;
    }
}

// ------------------------------------------------------ int8 -> fp32, exact
// Four signed bytes of w as floats: (b ^ 0x80) = b + 128 in [0, 255] goes
// into the low mantissa bits of 2^23, then 2^23 + 128 is subtracted.
__device__ __forceinline__ void deq4(uint32_t w, float &f0, float &f1, float &f2, float &f3) {
    const uint32_t u = w ^ 0x80808080u;
    constexpr float kBias = 8388736.0f;  // 2^23 + 128
    f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - kBias;
    f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - kBias;
    f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - kBias;
    f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - kBias;
}

// ----------------------------------------------- weight-streaming M <= 16
constexpr int SW = 64;   // columns per slab
constexpr int NT = 256;  // 8 warps x (8 row lanes x 4 groups of 16 columns)
constexpr int RL = 64;   // weight rows per CTA step (8 warps x 8 row lanes)
constexpr int ST = 4;    // cp.async ring depth

template <int MB> struct StreamGeo {
    static constexpr int UR = MB == 4 ? 2 : 4;  // rows per thread and ring stage
    static constexpr size_t smem = (size_t)ST * UR * NT * 16 + (size_t)ST * UR * MB * NT * 4;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Grid (slabs, ksplit): CTA (x, y) sums weight rows of K part y for the 64
// columns of slab x.  Each thread copies its own next rows (16 bytes of
// weights and the matching activations) into a four-stage shared-memory ring
// and reads back only what it copied, so the ring needs no barrier.  With
// ksplit > 1 every CTA writes its partial sums to `part`; the last CTA of the
// slab to arrive (counter `ctr[x]`) adds the parts in K order, applies the
// scales and resets the counter for the next call.
template <int MB>
__global__ void __launch_bounds__(NT)
    matmul_int8_stream_kernel(const float *__restrict__ A, const int8_t *__restrict__ q, const float *__restrict__ s,
                              float *__restrict__ C, long long M, long long K, long long N, float *__restrict__ part,
                              unsigned int *__restrict__ ctr) {
    using G = StreamGeo<MB>;
    constexpr int UR = G::UR;
    extern __shared__ __align__(16) unsigned char dsm[];
    uint4 *wbuf = reinterpret_cast<uint4 *>(dsm);                  // [ST][UR][NT]
    float *abuf = reinterpret_cast<float *>(wbuf + ST * UR * NT);  // [ST][UR][MB][NT]
    __shared__ float red[8][MB][SW];
    __shared__ bool s_last;
    const int ksplit = (int)gridDim.y, rank = (int)blockIdx.y;
    const long long slab = blockIdx.x;
    const int t = threadIdx.x, lane = t % 32, w = t / 32;
    const int rl = w * 8 + lane / 4;  // row lane 0..63
    const int cgp = lane % 4;         // columns cgp*16 .. +15 of the slab
    const long long c0 = slab * SW + cgp * 16;
    const bool live = c0 < N;         // N % 16 == 0: a group is whole or absent
    const long long kper = ((K + ksplit - 1) / ksplit + RL - 1) / RL * RL;
    const long long k0 = (long long)rank * kper, k1 = min(K, k0 + kper), kstart = k0 + rl;
    const long long nsteps = (live && kstart < k1) ? (k1 - kstart + RL - 1) / RL : 0;
    const long long ngroups = (nsteps + UR - 1) / UR;

    for (long long m0 = 0; m0 < M; m0 += MB) {
        float acc[MB][16];
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[m][j] = 0.0f;
        auto issue = [&](long long g) {
            if (g < ngroups) {
                const int st = (int)(g % ST);
#pragma unroll
                for (int u = 0; u < UR; ++u) {
                    const long long k = kstart + (g * UR + u) * RL;
                    if (k < k1) {
                        cp_async16(&wbuf[(st * UR + u) * NT + t], q + k * N + c0);
#pragma unroll
                        for (int m = 0; m < MB; ++m)
                            if (m0 + m < M) cp_async4(&abuf[((st * UR + u) * MB + m) * NT + t], A + (m0 + m) * K + k);
                    }
                }
            }
            cp_async_commit();
        };
#pragma unroll
        for (int g = 0; g < ST - 1; ++g) issue(g);
        for (long long g = 0; g < ngroups; ++g) {
            issue(g + ST - 1);
            cp_async_wait<ST - 1>();
            const int st = (int)(g % ST);
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const long long k = kstart + (g * UR + u) * RL;
                if (k >= k1) break;
                const uint4 wv = wbuf[(st * UR + u) * NT + t];
                float a[MB];
#pragma unroll
                for (int m = 0; m < MB; ++m) a[m] = m0 + m < M ? abuf[((st * UR + u) * MB + m) * NT + t] : 0.0f;
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float f[4];
                    deq4(ww[i], f[0], f[1], f[2], f[3]);
#pragma unroll
                    for (int m = 0; m < MB; ++m)
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[m][4 * i + j] = fmaf(a[m], f[j], acc[m][4 * i + j]);
                }
            }
        }
        cp_async_wait<0>();
        // Sum the 8 row lanes of the warp (lane bits 2-4), then the 8 warps.
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float v = acc[m][j];
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                acc[m][j] = v;
            }
        if (lane < 4) {
#pragma unroll
            for (int m = 0; m < MB; ++m)
#pragma unroll
                for (int j = 0; j < 16; ++j) red[w][m][cgp * 16 + j] = acc[m][j];
        }
        __syncthreads();
        for (int i = t; i < MB * SW; i += NT) {
            const int m = i / SW, c = i % SW;
            const long long col = slab * SW + c;
            if (m0 + m >= M || col >= N) continue;
            float v = 0.0f;
#pragma unroll
            for (int ww = 0; ww < 8; ++ww) v += red[ww][m][c];
            if (ksplit == 1)
                C[(m0 + m) * N + col] = v * s[col];
            else
                part[((long long)rank * M + m0 + m) * N + col] = v;
        }
        __syncthreads();  // red is reused by the next row block
    }
    if (ksplit == 1) return;
    // Serial fix-up: the last CTA of the slab adds the parts in K order.
    __threadfence();
    __syncthreads();
    if (t == 0) s_last = atomicAdd(&ctr[slab], 1u) == (unsigned)ksplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (long long i = t; i < M * SW; i += NT) {
        const long long m = i / SW, col = slab * SW + i % SW;
        if (col >= N) continue;
        const float v = sum_parts_ordered(part + (long long)m * N + col, (long long)M * N, ksplit);
        C[m * N + col] = v * s[col];
    }
    if (t == 0) ctr[slab] = 0u;  // ready for the next call on this stream
}

// ------------------------------------------- weight streaming, 4 < M <= 16
// One pass for up to 16 activation rows: a thread owns 8 columns of one
// weight row per step (8 bytes) and keeps all 16 rows' sums as packed fp32
// pairs (fma.rn.f32x2); a warp covers 256 columns of a row, the 8 warps 8
// rows.  The CTA's K range of A is staged transposed in shared memory first
// (At[k][m]), so the 16 activations of a weight row are one broadcast read.
// Weights stream through the per-thread cp.async ring; K parts of a slab meet
// in the serial fix-up as in the kernel above.
constexpr int SW16 = 256;   // columns per slab
constexpr int UR16 = 16;    // weight rows per thread and ring stage (96 KB in flight per CTA)
constexpr int KMAX16 = 768; // largest K range per CTA (At: 768 x 16 floats = 48 KB)

__global__ void __launch_bounds__(NT, 1)
    matmul_int8_m16_kernel(const float *__restrict__ A, const int8_t *__restrict__ q, const float *__restrict__ s,
                           float *__restrict__ C, long long M, long long K, long long N, float *__restrict__ part,
                           unsigned int *__restrict__ ctr) {
    extern __shared__ __align__(16) unsigned char dsm[];
    float *At = reinterpret_cast<float *>(dsm);                  // [KMAX16][16]
    uint2 *wbuf = reinterpret_cast<uint2 *>(At + KMAX16 * 16);   // [ST][UR16][NT]
    float *red = At;                                             // [8][16][SW16] after the loop
    __shared__ bool s_last;
    const int ksplit = (int)gridDim.y, rank = (int)blockIdx.y;
    const long long slab = blockIdx.x;
    const int t = threadIdx.x, lane = t % 32, w = t / 32;
    const long long c0 = slab * SW16 + lane * 8;  // columns c0 .. c0 + 7
    const bool live = c0 < N;                     // N % 16 == 0: eight columns are whole or absent
    const long long kper = ((K + ksplit - 1) / ksplit + 7) / 8 * 8;
    const long long k0 = (long long)rank * kper, k1 = min(K, k0 + kper);
    const int nk = (int)max(0ll, k1 - k0);

    for (int i = t; i < nk * 16; i += NT) {  // At[k][m] = A[m][k0 + k] (0 past M), reads along k
        const int m = i / nk, kk = i % nk;
        At[kk * 16 + m] = m < M ? A[(long long)m * K + k0 + kk] : 0.0f;
    }
    __syncthreads();

    float2 acc[16][4];
#pragma unroll
    for (int m = 0; m < 16; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[m][j] = make_float2(0.0f, 0.0f);
    const int nsteps = (live && w < nk) ? (nk - w + 7) / 8 : 0;  // rows w, w + 8, ... of the range
    const int ngroups = (nsteps + UR16 - 1) / UR16;
    auto issue = [&](int g) {
        if (g < ngroups) {
            const int st = g % ST;
#pragma unroll
            for (int u = 0; u < UR16; ++u) {
                const int kk = w + (g * UR16 + u) * 8;
                if (kk < nk)
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(
                                     (unsigned)__cvta_generic_to_shared(&wbuf[(st * UR16 + u) * NT + t])),
                                 "l"(q + (k0 + kk) * N + c0)
                                 : "memory");
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int g = 0; g < ST - 1; ++g) issue(g);
    for (int g = 0; g < ngroups; ++g) {
        issue(g + ST - 1);
        cp_async_wait<ST - 1>();
        const int st = g % ST;
#pragma unroll
        for (int u = 0; u < UR16; ++u) {
            const int kk = w + (g * UR16 + u) * 8;
            if (kk >= nk) break;
            const uint2 wv = wbuf[(st * UR16 + u) * NT + t];
            float f[8];
            deq4(wv.x, f[0], f[1], f[2], f[3]);
            deq4(wv.y, f[4], f[5], f[6], f[7]);
            const float2 w2[4] = {make_float2(f[0], f[1]), make_float2(f[2], f[3]), make_float2(f[4], f[5]),
                                  make_float2(f[6], f[7])};
            const float4 *a4 = reinterpret_cast<const float4 *>(At + kk * 16);
#pragma unroll
            for (int mq = 0; mq < 4; ++mq) {
                const float4 a = a4[mq];
                const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int mm = 0; mm < 4; ++mm) {
                    const float2 a2 = make_float2(av[mm], av[mm]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[mq * 4 + mm][j] = __ffma2_rn(a2, w2[j], acc[mq * 4 + mm][j]);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();  // At and the ring are done: red reuses them
#pragma unroll
    for (int m = 0; m < 16; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            *reinterpret_cast<float2 *>(&red[(w * 16 + m) * SW16 + lane * 8 + 2 * j]) = acc[m][j];
    __syncthreads();
    const long long col = slab * SW16 + t;  // NT == SW16: one column per thread
    if (col < N) {
        for (int m = 0; m < M; ++m) {
            float v = 0.0f;
#pragma unroll
            for (int ww = 0; ww < 8; ++ww) v += red[(ww * 16 + m) * SW16 + t];
            if (ksplit == 1)
                C[m * N + col] = v * s[col];
            else
                part[((long long)rank * M + m) * N + col] = v;
        }
    }
    if (ksplit == 1) return;
    __threadfence();
    __syncthreads();
    if (t == 0) s_last = atomicAdd(&ctr[slab], 1u) == (unsigned)ksplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (long long i = t; i < M * SW16; i += NT) {
        const long long m = i / SW16, col = slab * SW16 + i % SW16;
        if (col >= N) continue;
        const float v = sum_parts_ordered(part + (long long)m * N + col, (long long)M * N, ksplit);
        C[m * N + col] = v * s[col];
    }
    if (t == 0) ctr[slab] = 0u;
}
static_assert(NT == SW16, "one output column per thread in the epilogue");

// -------------------------------------------------- tiled GEMM, M > 16
// 64 x 64 tile of C per CTA, 256 threads with 4 x 4 each; K in steps of 32,
// A and the dequantized weights staged in shared memory.
constexpr int TM = 64, TN = 64, TK = 32;

__global__ void __launch_bounds__(256) matmul_int8_tiled_kernel(const float *__restrict__ A,
                                                                const int8_t *__restrict__ q,
                                                                const float *__restrict__ s, float *__restrict__ C,
                                                                long long M, long long K, long long N) {
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int t = threadIdx.x, tx = t % 16, ty = t / 16;
    const long long m0 = (long long)blockIdx.y * TM, n0 = (long long)blockIdx.x * TN;
    float acc[4][4] = {};
    for (long long k0 = 0; k0 < K; k0 += TK) {
        // A tile: 64 rows x 32 k, 8 per thread, consecutive threads along k
        for (int i = t; i < TM * TK; i += 256) {
            const int r = i / TK, kk = i % TK;
            const long long m = m0 + r, k = k0 + kk;
            As[kk][r] = (m < M && k < K) ? A[m * K + k] : 0.0f;
        }
        // weight tile: 32 k x 64 columns, consecutive threads along n
        for (int i = t; i < TK * TN; i += 256) {
            const int kk = i / TN, c = i % TN;
            const long long k = k0 + kk, n = n0 + c;
            Bs[kk][c] = (k < K && n < N) ? (float)q[k * N + n] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < TK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const long long m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const long long n = n0 + tx * 4 + j;
            if (n < N) C[m * N + n] = acc[i][j] * s[n];
        }
    }
}

template <int MB>
int launch_stream(const float *A, const int8_t *q, const float *s, float *C, long long M, long long K, long long N,
                  cudaStream_t st) {
    using G = StreamGeo<MB>;
    static std::atomic<unsigned long long> attr_set{0};  // per device: the ring needs > 48 KB
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8: cudaGetDevice");
    if (rc) return rc;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        rc = check_cuda(cudaFuncSetAttribute(matmul_int8_stream_kernel<MB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)G::smem),
                        "matmul_int8: smem attribute");
        if (rc) return rc;
        attr_set.fetch_or(bit);
    }
    const long long slabs = (N + SW - 1) / SW;
    // Split K until the CTAs cover the SMs, keeping two 64-row steps per part.
    int ks = 1;
    while (ks < 16 && slabs * ks < sm_count() && K >= (long long)RL * ks * 4) ks *= 2;
    if (slabs > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8: N too large");
    unsigned int *ctr = nullptr;
    float *part = nullptr;
    if (ks > 1 && (rc = split_workspace(st, (size_t)slabs, (size_t)ks * M * N, &ctr, &part))) return rc;
    matmul_int8_stream_kernel<MB><<<dim3((unsigned)slabs, (unsigned)ks), NT, G::smem, st>>>(A, q, s, C, M, K, N, part,
                                                                                           ctr);
    return check_launch("matmul_int8_stream_kernel");
}

int launch_m16(const float *A, const int8_t *q, const float *s, float *C, long long M, long long K, long long N,
               cudaStream_t st) {
    const size_t smem = std::max((size_t)KMAX16 * 16 * 4 + (size_t)ST * UR16 * NT * 8, (size_t)8 * 16 * SW16 * 4);
    static std::atomic<unsigned long long> attr_set{0};  // per device
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8: cudaGetDevice");
    if (rc) return rc;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        rc = check_cuda(cudaFuncSetAttribute(matmul_int8_m16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "matmul_int8: smem attribute");
        if (rc) return rc;
        attr_set.fetch_or(bit);
    }
    const long long slabs = (N + SW16 - 1) / SW16;
    // One CTA per SM (registers): split K until the CTAs come close to one
    // wave, and until every part fits the staged A.
    int ks = 1;
    while (ks < 64 && (10 * slabs * ks < 9ll * sm_count() || (K + ks - 1) / ks > KMAX16 - 8)) ks *= 2;
    if ((K + ks - 1) / ks > KMAX16 - 8) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8: K too large");
    unsigned int *ctr = nullptr;
    float *part = nullptr;
    if (ks > 1 && (rc = split_workspace(st, (size_t)slabs, (size_t)ks * M * N, &ctr, &part))) return rc;
    matmul_int8_m16_kernel<<<dim3((unsigned)slabs, (unsigned)ks), NT, smem, st>>>(A, q, s, C, M, K, N, part, ctr);
    return check_launch("matmul_int8_m16_kernel");
}

}  // namespace

// Split-K workspace per (device, stream): the slab counters (zeroed once at
// allocation, reset by the kernels) and the partial sums.
struct SplitWs {
    int device;
    cudaStream_t stream;
    unsigned int *ctr;
    float *part;
    size_t nctr, npart;
};
static std::mutex g_ws_mu;
static std::vector<SplitWs> g_ws;

int split_workspace(cudaStream_t st, size_t nctr, size_t npart, unsigned int **ctr, float **part) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8: cudaGetDevice");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_ws_mu);
    SplitWs *e = nullptr;
    for (auto &x : g_ws)
        if (x.device == dev && x.stream == st) e = &x;
    if (!e) {
        g_ws.push_back({dev, st, nullptr, nullptr, 0, 0});
        e = &g_ws.back();
    }
    if (e->nctr < nctr) {
        if ((rc = check_cuda(cudaFree(e->ctr), "matmul_int8: cudaFree"))) return rc;  // waits for the device
        e->ctr = nullptr;
        e->nctr = 0;
        const size_t n = std::max<size_t>(nctr, 4096);
        if ((rc = check_cuda(cudaMalloc(&e->ctr, n * sizeof(unsigned int)), "matmul_int8: cudaMalloc"))) return rc;
        if ((rc = check_cuda(cudaMemsetAsync(e->ctr, 0, n * sizeof(unsigned int), st), "matmul_int8: memset")))
            return rc;
        e->nctr = n;
    }
    if (e->npart < npart) {
        if ((rc = check_cuda(cudaFree(e->part), "matmul_int8: cudaFree"))) return rc;
        e->part = nullptr;
        e->npart = 0;
        const size_t n = std::max<size_t>(npart + npart / 2, 1 << 18);
        if ((rc = check_cuda(cudaMalloc(&e->part, n * sizeof(float)), "matmul_int8: cudaMalloc"))) return rc;
        e->npart = n;
    }
    *ctr = e->ctr;
    *part = e->part;
    return KAI_GDN_OK;
}

int launch_quantize_int8(const float *B, int8_t *q, float *s, size_t K, size_t N, cudaStream_t st) {
    if (K == 0 || N == 0) return KAI_GDN_OK;
    if (!B || !q || !s) return set_error(KAI_GDN_ERR_INVALID, "quantize_int8: null pointer");
    const long long grid = ((long long)N + 31) / 32;
    if (grid > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "quantize_int8: N too large");
    quantize_int8_kernel<<<(unsigned)grid, 256, 0, st>>>(B, q, s, (long long)K, (long long)N);
    return check_launch("quantize_int8_kernel");
}

int launch_matmul_int8(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N,
                       cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!C) return set_error(KAI_GDN_ERR_INVALID, "matmul_int8: null pointer");
    if (K == 0) return check_cuda(cudaMemsetAsync(C, 0, M * N * sizeof(float), st), "matmul_int8: memset");
    if (!A || !q || !s) return set_error(KAI_GDN_ERR_INVALID, "matmul_int8: null pointer");
    const long long m = (long long)M, k = (long long)K, n = (long long)N;
    const bool vec = N % 16 == 0 && (uintptr_t)q % 16 == 0;
    if (gemv_int8_supported(M, K, N, q)) return launch_gemv_int8(A, q, s, C, M, K, N, st);
    if (M <= 16 && vec) {
        if (M == 1) return launch_stream<1>(A, q, s, C, m, k, n, st);
        if (M == 2) return launch_stream<2>(A, q, s, C, m, k, n, st);
        if (M <= 4) return launch_stream<4>(A, q, s, C, m, k, n, st);
        if (M < 16) return launch_m16(A, q, s, C, m, k, n, st);
    }
    if (M >= 16 && vec && K % 4 == 0 && (uintptr_t)A % 16 == 0) return launch_matmul_int8_tc(A, q, s, C, M, K, N, st);
    const long long gy = (m + TM - 1) / TM, gx = (n + TN - 1) / TN;
    if (gy > 65535 || gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8: shape too large");
    matmul_int8_tiled_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, st>>>(A, q, s, C, m, k, n);
    return check_launch("matmul_int8_tiled_kernel");
}

}  // namespace gdn
