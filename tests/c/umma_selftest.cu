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

#include "../../orionsbelt_b200/csrc/tma.cuh"
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

// ---------------------------------------------------------------------------
// Operand layouts by mode (16-bit):
//   0 K-major, k-groups inner  (kmaj16)         1 MN-major, mn-groups inner (mnmaj16)
//   2 K-major, row-groups inner (TMA order)     3 MN-major, k-groups inner (TMA order)
//   5 K-major, 128-byte swizzle                 6 MN-major, 128-byte swizzle
//   4 A in TMEM (M = 128 only)
// `R` is the operand's M or N extent, `KK` its K extent.
__device__ uint32_t layout_off(int mode, uint32_t r, uint32_t k, uint32_t R, uint32_t KK) {
    switch (mode) {
        case 0: return kmaj16(r, k, KK);
        case 1: return mnmaj16(k, r, R);
        case 2: return (k / 8) * (R / 8) * 128 + (r / 8) * 128 + (r % 8) * 16 + (k % 8) * 2;
        case 3: return (r / 8) * (KK / 8) * 128 + (k / 8) * 128 + (k % 8) * 16 + (r % 8) * 2;
        case 5: {  // 64-k column blocks of R rows x 128 bytes
            const uint32_t row = r, chunk = (k % 64) / 8;
            return (k / 64) * R * 128 + (row / 8) * 1024 + (row % 8) * 128 + ((chunk ^ (row % 8)) * 16) + (k % 8) * 2;
        }
        case 6: {  // 64-mn column blocks of KK k-rows x 128 bytes
            const uint32_t row = k, chunk = (r % 64) / 8;
            return (r / 64) * KK * 128 + (row / 8) * 1024 + (row % 8) * 128 + ((chunk ^ (row % 8)) * 16) + (r % 8) * 2;
        }
    }
    return 0;
}
__device__ uint64_t layout_desc(int mode, const void *tile, uint32_t R, uint32_t KK, uint32_t ks) {
    const uint32_t a = smem_addr(tile);
    switch (mode) {
        case 0: return desc_kmaj16(tile, KK, ks);
        case 1: return desc_mnmaj16(tile, R, ks);
        case 2: return smem_desc(a + ks * 2 * (R / 8) * 128, (R / 8) * 128, 128);
        case 3: return smem_desc(a + ks * 2 * 128, 128, (KK / 8) * 128);
        case 5: return smem_desc_sw128(a + (ks * 16 / 64) * R * 128 + (ks * 16 % 64) * 2, 16, 1024);
        case 6: return smem_desc_sw128(a + ks * 2 * 1024, KK * 128, 1024);
    }
    return 0;
}

__global__ void __launch_bounds__(128, 1)
    gemm2_kernel(const float *A, const float *B, float *D, int M, int N, int K, int a_mode, int b_mode, int *err) {
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char *As = smem;                  // 32 KB
    unsigned char *Bs = smem + 32 * 1024;      // 64 KB
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const bool a_mn = a_mode == 1 || a_mode == 3 || a_mode == 6, b_mn = b_mode == 1 || b_mode == 3 || b_mode == 6;

    if (a_mode != 4)
        for (int e = t; e < M * K; e += 128)
            *reinterpret_cast<__nv_bfloat16 *>(As + layout_off(a_mode, e / K, e % K, M, K)) =
                __float2bfloat16_rn(A[e]);
    for (int e = t; e < K * N; e += 128)
        *reinterpret_cast<__nv_bfloat16 *>(Bs + layout_off(b_mode, e % N, e / N, N, K)) = __float2bfloat16_rn(B[e]);
    if (t == 0) mbar_init(&bar, 1);
    if (warp == 0) tmem_alloc(&tmem_slot, 512);
    fence_smem_to_async();
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = tmem_slot, ta = tm + 256;
    if (a_mode == 4) {  // row m = lane 32*warp + lane, columns 256 + k/2
        const int m = 32 * warp + lane;
        for (int c0 = 0; c0 < K / 2; c0 += 16) {
            uint32_t v[16];
            for (int i = 0; i < 16; ++i) {
                const int k = 2 * (c0 + i);
                const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(A[m * K + k]));
                const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(A[m * K + k + 1]));
                v[i] = lo | (hi << 16);
            }
            tmem_st16u(taddr(ta, 32 * warp, c0), v);
        }
        tmem_wait_st();
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
    }
    if (t == 0) {
        const uint32_t id = idesc(M, N, BF16, a_mn, b_mn);
        for (int ks = 0; ks < K / 16; ++ks) {
            const uint64_t bd = layout_desc(b_mode, Bs, N, K, ks);
            if (a_mode == 4)
                mma_f16_ta(tm, ta + ks * 8, bd, id, ks > 0);
            else
                mma_f16(tm, layout_desc(a_mode, As, M, K, ks), bd, id, ks > 0);
        }
        commit(&bar);
    }
    __syncwarp();
    bool ok = mbar_wait(&bar, 0, err);
    fence_after_sync();
    if (ok) {
        const int row = M == 128 ? 32 * warp + lane : 16 * warp + lane;
        const bool live = M == 128 || lane < 16;
        for (int c = 0; c < N; c += 16) {
            float v[16];
            tmem_ld16(taddr(tm, 32 * warp, c), v);
            tmem_wait_ld();
            if (live)
                for (int i = 0; i < 16; ++i) D[row * N + c + i] = v[i];
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tm, 512);
}

// One TMA chunk load (core-matrix or 128-byte swizzle map), copied out raw.
__global__ void __launch_bounds__(128, 1)
    tma_kernel(const __grid_constant__ CUtensorMap map, uint16_t *out, int t0, int h, int b, int swz, int *err) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ __align__(8) uint64_t bar;
    const int t = threadIdx.x;
    uint16_t *tile = reinterpret_cast<uint16_t *>(smem);
    for (int i = t; i < 8192; i += 128) tile[i] = 0xFFFFu;
    if (t == 0) {
        mbar_init(&bar, 1);
        gdn::tma::prefetch_map(&map);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_smem_to_async();
    __syncthreads();
    if (t == 0) {
        mbar_arrive_expect_tx(&bar, 16384);
        if (swz)
            gdn::tma::load_chunk_sw128(smem, &map, t0, h, b, &bar);
        else
            gdn::tma::load_chunk(smem, &map, t0, h, b, &bar);
    }
    const bool ok = mbar_wait(&bar, 0, err);
    __syncthreads();
    if (ok)
        for (int i = t; i < 8192; i += 128) out[i] = tile[i];
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

extern "C" __attribute__((visibility("default"))) int umma_selftest_gemm2(const float *A, const float *B, float *D,
                                                                           int M, int N, int K, int a_mode,
                                                                           int b_mode, int *err) {
    if ((M != 64 && M != 128) || N % 16 || N < 16 || N > 256 || K % 16 || K > 128) return 1;
    if (a_mode == 4 && M != 128) return 1;
    if (a_mode < 0 || a_mode > 6 || b_mode < 0 || b_mode > 6 || b_mode == 4) return 1;
    if ((a_mode >= 5 && (M % 8 || K % 64)) || (b_mode >= 5 && (N % 64 && b_mode == 6))) return 1;
    if ((a_mode == 6 && M % 64) || (b_mode == 5 && K % 64)) return 1;
    const int smem = 96 * 1024;
    cudaFuncSetAttribute(gemm2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    gemm2_kernel<<<1, 128, smem>>>(A, B, D, M, N, K, a_mode, b_mode, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return 2;
    e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : 3;
}

// Returns 0, 10 + CUresult of the map encoding, or 2/3 on launch errors.
extern "C" __attribute__((visibility("default"))) int umma_selftest_tma(const void *src, uint16_t *out, int bf16,
                                                                         int B, int T, int H, int t0, int h, int b,
                                                                         int swz, int *err) {
    CUtensorMap map;
    int rc = gdn::tma::make_chunk_map(&map, src, bf16 != 0, B, T, H, 128, swz != 0);
    if (rc) return 10 + rc;
    cudaFuncSetAttribute(tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384);
    tma_kernel<<<1, 128, 16384>>>(map, out, t0, h, b, swz, err);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return 2;
    e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : 3;
}

// A bounded mbarrier wait on a barrier nothing arrives on: the wait must run
// out after `limit` polls, set *err and let the kernel finish.
__global__ void timeout_kernel(int *err, int *done, unsigned limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, err, limit);
    if (threadIdx.x == 0) *done = ok ? 2 : 1;
}

extern "C" __attribute__((visibility("default"))) int umma_selftest_timeout(int *err, int *done) {
    timeout_kernel<<<1, 32>>>(err, done, 1u << 12);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return 2;
    e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : 3;
}
