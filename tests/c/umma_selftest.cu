// umma_selftest.cu -- checks the tcgen05 building blocks of
// orionsbelt_b200/csrc/umma.cuh on the GPU: one CTA computes D = A . B
// (A [M][K], B [K][N], fp32 in global memory) by writing the operands into
// shared memory in the K-major or MN-major no-swizzle layout, issuing
// kind::f16 (bf16) or kind::tf32 MMAs into TMEM, and reading the fp32
// accumulator back with tcgen05.ld using the M=64 / M=128 lane mapping.
// tests/test_gpu_umma.py compares D with numpy.  Test infrastructure, built
// into tests/c/bin/libumma_selftest.so; not part of the product library.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../orionsbelt_b200/csrc/umma.cuh"

using namespace gdn::umma;

namespace {

__global__ void __launch_bounds__(128, 1)
    gemm_kernel(const float *A, const float *B, float *D, int M, int N, int K, int a_mn, int b_mn, int tf32,
                int lane16, int *err) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char *As = smem;                  // up to 128 x 128 x 4 bytes
    unsigned char *Bs = smem + 64 * 1024;      // up to 256 x 128 x 4 bytes (128 KB)
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;

    if (!tf32) {
        for (int e = t; e < M * K; e += 128) {
            int m = e / K, k = e % K;
            uint32_t off = a_mn ? mnmaj16(k, m, M) : kmaj16(m, k, K);
            *reinterpret_cast<__nv_bfloat16 *>(As + off) = __float2bfloat16_rn(A[e]);
        }
        for (int e = t; e < K * N; e += 128) {
            int k = e / N, n = e % N;
            uint32_t off = b_mn ? mnmaj16(k, n, N) : kmaj16(n, k, K);
            *reinterpret_cast<__nv_bfloat16 *>(Bs + off) = __float2bfloat16_rn(B[e]);
        }
    } else {
        for (int e = t; e < M * K; e += 128) {
            int m = e / K, k = e % K;
            *reinterpret_cast<float *>(As + kmaj32(m, k, K)) = A[e];
        }
        for (int e = t; e < K * N; e += 128) {
            int k = e / N, n = e % N;
            *reinterpret_cast<float *>(Bs + kmaj32(n, k, K)) = B[e];
        }
    }
    if (t == 0) mbar_init(&bar, 1);
    if (warp == 0) tmem_alloc(&tmem_slot, 256);
    fence_smem_to_async();
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    // lane16: an M=64 accumulator placed in the upper half of each 32-lane
    // quadrant (TMEM lane offset 16), the second of two interleaved tiles.
    const uint32_t tbase = tmem_slot + (lane16 ? (16u << 16) : 0u);

    if (t == 0) {
        if (!tf32) {
            const uint32_t id = idesc(M, N, BF16, a_mn, b_mn);
            for (int ks = 0; ks < K / 16; ++ks) {
                uint64_t ad = a_mn ? desc_mnmaj16(As, M, ks) : desc_kmaj16(As, K, ks);
                uint64_t bd = b_mn ? desc_mnmaj16(Bs, N, ks) : desc_kmaj16(Bs, K, ks);
                mma_f16(tbase, ad, bd, id, ks > 0);
            }
        } else {
            const uint32_t id = idesc(M, N, TF32, false, false);
            for (int ks = 0; ks < K / 8; ++ks) mma_tf32(tbase, desc_kmaj32(As, K, ks), desc_kmaj32(Bs, K, ks), id, ks > 0);
        }
        commit(&bar);
    }
    __syncwarp();
    bool ok = mbar_wait(&bar, 0, err);
    fence_after_sync();
    if (ok) {
        // M=128: row = 32*warp + lane.  M=64: rows 16*warp + lane for lane < 16.
        const int row = M == 128 ? 32 * warp + lane : 16 * warp + (lane16 ? lane - 16 : lane);
        const bool live = M == 128 || (lane16 ? lane >= 16 : lane < 16);
        for (int c = 0; c < N; c += 16) {
            float v[16];
            tmem_ld16(taddr(tmem_slot, 32 * warp, c), v);
            tmem_wait_ld();
            if (live)
                for (int i = 0; i < 16; ++i) D[row * N + c + i] = v[i];
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem_slot, 256);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int umma_selftest_gemm(const float *A, const float *B, float *D,
                                                                          int M, int N, int K, int a_mn, int b_mn,
                                                                          int tf32, int lane16, int *err) {
    if ((M != 64 && M != 128) || N % 16 || N < 16 || N > 256 || K % 16 || K > 128) return 1;
    if (lane16 && M != 64) return 1;
    const int smem = 64 * 1024 + 128 * 1024;
    cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gemm_kernel<<<1, 128, smem>>>(A, B, D, M, N, K, a_mn, b_mn, tf32, lane16, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return 2;
    e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : 3;
}
