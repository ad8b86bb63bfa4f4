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
//  M <= 8 : GEMV form, thread per (row, 4 columns); B rows streamed coalesced
//           (HBM-bound: K*N*4 bytes of B per row of A, re-reads hit L2).
//  M  > 8 : 64x64 tile per block, 4x4 outputs per thread, k staged in
//           shared memory 16 at a time.
#include "gdn_internal.cuh"

namespace gdn {
namespace {

__global__ void __launch_bounds__(256) gemv_rows_kernel(const float *__restrict__ A,
                                                        const float *__restrict__ B,
                                                        float *__restrict__ C, long long K,
                                                        long long N, bool vec4) {
    long long j = ((long long)blockIdx.x * 256 + threadIdx.x) * 4;
    long long i = blockIdx.y;
    if (j >= N) return;
    const float *a = A + i * K;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec4) {
        long long k = 0;
        for (; k + 4 <= K; k += 4) {
            float4 b[4];
            float av[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                b[r] = __ldg(reinterpret_cast<const float4 *>(B + (k + r) * N + j));
                av[r] = __ldg(a + k + r);
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                acc[0] = __fadd_rn(acc[0], __fmul_rn(av[r], b[r].x));
                acc[1] = __fadd_rn(acc[1], __fmul_rn(av[r], b[r].y));
                acc[2] = __fadd_rn(acc[2], __fmul_rn(av[r], b[r].z));
                acc[3] = __fadd_rn(acc[3], __fmul_rn(av[r], b[r].w));
            }
        }
        for (; k < K; ++k) {
            float4 b = __ldg(reinterpret_cast<const float4 *>(B + k * N + j));
            float av = __ldg(a + k);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(av, b.x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(av, b.y));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(av, b.z));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(av, b.w));
        }
        *reinterpret_cast<float4 *>(C + i * N + j) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
        int nj = (int)min(4ll, N - j);
        for (long long k = 0; k < K; ++k) {
            float av = __ldg(a + k);
            for (int q = 0; q < nj; ++q)
                acc[q] = __fadd_rn(acc[q], __fmul_rn(av, __ldg(B + k * N + j + q)));
        }
        for (int q = 0; q < nj; ++q) C[i * N + j + q] = acc[q];
    }
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

}  // namespace

int launch_matmul(const float *A, const float *B, float *C, size_t M, size_t K, size_t N,
                  cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!C || (K > 0 && (!A || !B))) return set_error(KAI_GDN_ERR_INVALID, "matmul: null pointer");
    if (K == 0) return check_cuda(cudaMemsetAsync(C, 0, M * N * sizeof(float), st), "matmul: k=0 zero fill");
    if (M <= 8) {
        bool vec4 = (N % 4 == 0) && ((uintptr_t)B % 16 == 0) && ((uintptr_t)C % 16 == 0);
        long long gx = ((long long)N + 1023) / 1024;
        if (gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul: N too large");
        dim3 grid((unsigned)gx, (unsigned)M);
        gemv_rows_kernel<<<grid, 256, 0, st>>>(A, B, C, (long long)K, (long long)N, vec4);
        return check_launch("gemv");
    }
    long long gx = ((long long)N + TN - 1) / TN, gy = ((long long)M + TM - 1) / TM;
    if (gx > 0x7fffffffll || gy > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul: too large");
    dim3 grid((unsigned)gx, (unsigned)gy);
    sgemm_tile_kernel<<<grid, 256, 0, st>>>(A, B, C, (long long)M, (long long)K, (long long)N);
    return check_launch("matmul");
}

}  // namespace gdn
