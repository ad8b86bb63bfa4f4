// matmul.cu -- the delta-rule matmul C[M][N] = A[M][K] . B[K][N] (fp32) on sm_100a.
//
// src/orionsbelt/engines/cpu/kernels/gdn_delta_matmul.c:164-173 (dispatch) and
// :109-117 (scalar path), and the M=1 GEMV
// kleidiai_submission/kai/ukernels/gdn/kai_gdn_gemv_f32_f32_f32_1x4_neon.c:77-85.
//
// Every output is accumulated over k in increasing order with one rounding per
// multiply and per add (acc = acc + a*b), the reference's scalar order, so the
// result is bit-identical to the reference on x86.  That order is kept on CUDA
// cores on purpose: this standalone operator is fp32 with a 1e-4 elementwise
// relative bar (test_gdn_delta_matmul.c:61-64) and its sizes (K=128, N<=4096,
// M<=64) make it launch- or HBM-bound.  The delta matmuls inside the chunked
// scan are the tensor-core contractions.
//
//  M <= 8 : GEMV form, one CTA per (row of A, 64 columns of B), one thread
//           per column: a 128-row slab of the 64 columns is copied into
//           shared memory by cp.async (every 16-byte piece in flight at
//           once), then each thread sums its column in k order.  B's rows
//           are read coalesced; re-reads of B by other rows of A hit L2.
//  M  > 8 : 64x64 tile per block, 4x4 outputs per thread; for K <= 128 the
//           whole K extent of both tiles is staged by cp.async in one step,
//           otherwise 16 k at a time through registers.
//  Unaligned or ragged shapes take a plain path with the same sums.
#include "gdn_internal.cuh"

namespace gdn {
namespace {

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

constexpr int GC = 64, GK = 128;  // GEMV: columns per CTA, k rows per slab

// A, B, C 16-byte aligned, N % 4 == 0.
__global__ void __launch_bounds__(GC) gemv_slab_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                       float *__restrict__ C, long long K, long long N) {
    __shared__ __align__(16) float Bs[GK][GC];
    __shared__ float As[GK];
    const long long n0 = (long long)blockIdx.x * GC, i = blockIdx.y;
    const int t = threadIdx.x;
    const long long j = n0 + t;
    const int ncol = (int)min((long long)GC, N - n0);  // multiple of 4
    float acc = 0.f;
    for (long long k0 = 0; k0 < K; k0 += GK) {
        const int kr = (int)min((long long)GK, K - k0);
        for (int e = t; e < kr * (ncol / 4); e += GC) {
            const int r = e / (ncol / 4), q = e % (ncol / 4);
            cp_async16(&Bs[r][4 * q], B + (k0 + r) * N + n0 + 4 * q);
        }
        for (int r = t; r < kr; r += GC) As[r] = __ldg(A + i * K + k0 + r);
        cp_async_wait_all();
        __syncthreads();
        if (t < ncol)
            for (int r = 0; r < kr; ++r) acc = __fadd_rn(acc, __fmul_rn(As[r], Bs[r][t]));
        __syncthreads();
    }
    if (t < ncol) C[i * N + j] = acc;
}

// Any alignment: one thread per column, B read directly.
__global__ void __launch_bounds__(256) gemv_cols_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                        float *__restrict__ C, long long K, long long N) {
    const long long j = (long long)blockIdx.x * 256 + threadIdx.x;
    const long long i = blockIdx.y;
    if (j >= N) return;
    float acc = 0.f;
    for (long long k = 0; k < K; ++k) acc = __fadd_rn(acc, __fmul_rn(__ldg(A + i * K + k), __ldg(B + k * N + j)));
    C[i * N + j] = acc;
}

constexpr int TM = 64, TN = 64, TK = 16;

__global__ void __launch_bounds__(256) sgemm_tile_kernel(const float *__restrict__ A,
                                                         const float *__restrict__ B,
                                                         float *__restrict__ C, long long M,
                                                         long long K, long long N) {
    __shared__ float As[TK][TM + 4];
    __shared__ float Bs[TK][TN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const long long m0 = (long long)blockIdx.y * TM, n0 = (long long)blockIdx.x * TN;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
    for (long long k0 = 0; k0 < K; k0 += TK) {
        // 64x16 of A and 16x64 of B, 4 elements per thread each.
        for (int e = threadIdx.x; e < TM * TK; e += 256) {
            int r = e / TK, kk = e % TK;
            long long gm = m0 + r, gk = k0 + kk;
            As[kk][r] = (gm < M && gk < K) ? __ldg(A + gm * K + gk) : 0.f;
        }
        for (int e = threadIdx.x; e < TK * TN; e += 256) {
            int kk = e / TN, cc = e % TN;
            long long gk = k0 + kk, gn = n0 + cc;
            Bs[kk][cc] = (gk < K && gn < N) ? __ldg(B + gk * N + gn) : 0.f;
        }
        __syncthreads();
        int kmax = (int)min((long long)TK, K - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                a[q] = As[kk][ty + 16 * q];
                b[q] = Bs[kk][tx + 16 * q];
            }
#pragma unroll
            for (int p = 0; p < 4; ++p)
#pragma unroll
                for (int q = 0; q < 4; ++q) acc[p][q] = __fadd_rn(acc[p][q], __fmul_rn(a[p], b[q]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            long long gm = m0 + ty + 16 * p, gn = n0 + tx + 16 * q;
            if (gm < M && gn < N) C[gm * N + gn] = acc[p][q];
        }
}

// K <= KF, K % 4 == 0, A and B 16-byte aligned, N % 4 == 0: both tiles' whole
// K extent copied by cp.async in one step (one wait for memory).
constexpr int KF = 128;
__global__ void __launch_bounds__(256) sgemm_fullk_kernel(const float *__restrict__ A, const float *__restrict__ B,
                                                          float *__restrict__ C, long long M, long long K, long long N) {
    extern __shared__ __align__(16) float fs[];
    const int lda = (int)K + 4;                 // As[r][k], rows 16-byte aligned
    float *As = fs;                             // [TM][K + 4]
    float *Bs = fs + (size_t)TM * lda;          // [K][TN + 4]
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const long long m0 = (long long)blockIdx.y * TM, n0 = (long long)blockIdx.x * TN;
    const int mr = (int)min((long long)TM, M - m0), nc = (int)min((long long)TN, N - n0);  // nc % 4 == 0
    const int kq = (int)K / 4;
    for (int e = threadIdx.x; e < TM * kq; e += 256) {
        const int r = e / kq, q = e % kq;
        if (r < mr)
            cp_async16(As + r * lda + 4 * q, A + (m0 + r) * K + 4 * q);
        else
            *reinterpret_cast<float4 *>(As + r * lda + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int e = threadIdx.x; e < (int)K * (TN / 4); e += 256) {
        const int kk = e / (TN / 4), q = e % (TN / 4);
        if (4 * q < nc)
            cp_async16(Bs + kk * (TN + 4) + 4 * q, B + kk * N + n0 + 4 * q);
        else
            *reinterpret_cast<float4 *>(Bs + kk * (TN + 4) + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    cp_async_wait_all();
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < (int)K; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            a[q] = As[(ty + 16 * q) * lda + kk];
            b[q] = Bs[kk * (TN + 4) + tx + 16 * q];
        }
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[p][q] = __fadd_rn(acc[p][q], __fmul_rn(a[p], b[q]));
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const long long gm = m0 + ty + 16 * p, gn = n0 + tx + 16 * q;
            if (gm < M && gn < N) C[gm * N + gn] = acc[p][q];
        }
}

}  // namespace

int launch_matmul(const float *A, const float *B, float *C, size_t M, size_t K, size_t N,
                  cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!C || (K > 0 && (!A || !B))) return set_error(KAI_GDN_ERR_INVALID, "matmul: null pointer");
    if (K == 0) return check_cuda(cudaMemsetAsync(C, 0, M * N * sizeof(float), st), "matmul: k=0 zero fill");
    const bool al16 = (((uintptr_t)A | (uintptr_t)B | (uintptr_t)C) % 16) == 0 && N % 4 == 0;
    if (M <= 8) {
        if (al16) {
            long long gx = ((long long)N + GC - 1) / GC;
            if (gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul: N too large");
            gemv_slab_kernel<<<dim3((unsigned)gx, (unsigned)M), GC, 0, st>>>(A, B, C, (long long)K, (long long)N);
            return check_launch("gemv");
        }
        long long gx = ((long long)N + 255) / 256;
        if (gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul: N too large");
        gemv_cols_kernel<<<dim3((unsigned)gx, (unsigned)M), 256, 0, st>>>(A, B, C, (long long)K, (long long)N);
        return check_launch("gemv");
    }
    long long gx = ((long long)N + TN - 1) / TN, gy = ((long long)M + TM - 1) / TM;
    if (gx > 0x7fffffffll || gy > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul: too large");
    dim3 grid((unsigned)gx, (unsigned)gy);
    if (K <= (size_t)KF && K % 4 == 0 && al16) {
        const size_t smem = sizeof(float) * ((size_t)TM * (K + 4) + K * (TN + 4));
        int rc = check_cuda(cudaFuncSetAttribute(sgemm_fullk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)(sizeof(float) * ((size_t)TM * (KF + 4) + KF * (TN + 4)))),
                            "matmul: smem attribute");
        if (rc) return rc;
        sgemm_fullk_kernel<<<grid, 256, smem, st>>>(A, B, C, (long long)M, (long long)K, (long long)N);
        return check_launch("matmul");
    }
    sgemm_tile_kernel<<<grid, 256, 0, st>>>(A, B, C, (long long)M, (long long)K, (long long)N);
    return check_launch("matmul");
}

}  // namespace gdn
