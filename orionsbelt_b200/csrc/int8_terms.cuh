// int8_terms.cuh -- the activation side of the packed int8 matmul: a row of
// fp32 activations as three signed bytes of fixed point per element (see
// int8_packed.cu), written in the layout its kernels read.  Shared by the
// library's own preparation kernel and by kernels that produce a matmul's
// input row and can emit its terms directly.
//
// Layout: [row block of RB][stage of 64 k][4 k-groups][3 RB rows][16 k]:
// per k-group, the RB rows of t0, then of t1, then of t2.  Row scale S (the
// row's largest magnitude) separately, one float per row.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {
namespace terms {

constexpr int KS = 64;  // k per stage

// Bytes of one stage of a row block.
__host__ __device__ constexpr long long stage_bytes(int RB) { return 3ll * RB * KS; }

// Terms of the 16 activations x[0..15] (k = k0 .. k0 + 15, k0 % 16 == 0) of
// row r, inv = 127 / S (0 for an all-zero row), into a row block's buffer.
__device__ __forceinline__ void write16(const float *x, float inv, int8_t *blk, long long k0, int RB, int r) {
    uint32_t w0[4], w1[4], w2[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t a = 0, b = 0, c = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float v = x[4 * q + e] * inv;
            const float t0 = rintf(v);
            v = (v - t0) * 254.0f;
            const float t1 = rintf(v);
            const float t2 = rintf((v - t1) * 254.0f);
            a |= ((uint32_t)(uint8_t)(int8_t)(int)t0) << (8 * e);
            b |= ((uint32_t)(uint8_t)(int8_t)(int)t1) << (8 * e);
            c |= ((uint32_t)(uint8_t)(int8_t)(int)t2) << (8 * e);
        }
        w0[q] = a, w1[q] = b, w2[q] = c;
    }
    int8_t *p = blk + (k0 / KS) * stage_bytes(RB) + ((k0 % KS) / 16) * (3 * RB * 16);
    *reinterpret_cast<uint4 *>(p + r * 16) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    *reinterpret_cast<uint4 *>(p + (RB + r) * 16) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
    *reinterpret_cast<uint4 *>(p + (2 * RB + r) * 16) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
}

// The whole row m (x: K values, in shared or global memory; K % 16 == 0)
// by the calling CTA: the row maximum `mx` is given (the caller has reduced
// it); writes the terms of k < S * 64 (zeros past K) and the row scale.
__device__ __forceinline__ void write_row(const float *x, long long K, long long S, float mx, int8_t *terms,
                                          float *scale, int RB, long long m) {
    if (threadIdx.x == 0) scale[m] = mx;
    const float inv = mx > 0.f ? 127.0f / mx : 0.f;
    int8_t *blk = terms + (m / RB) * S * stage_bytes(RB);
    const int r = (int)(m % RB);
    const float zero[16] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (long long g = threadIdx.x; g < S * (KS / 16); g += blockDim.x) {
        const long long k0 = g * 16;
        write16(k0 < K ? x + k0 : zero, inv, blk, k0, RB, r);
    }
}

}  // namespace terms
}  // namespace gdn
