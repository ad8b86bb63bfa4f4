// int8_tc.cu -- the int8-weight matmul of the reference's INT8_WEIGHTS path
// (gemm_int8_neon, src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:608-678)
// on the tcgen05 tensor cores, for M >= 16 activation rows.
//
// C[m][n] = s[n] * sum_k A[m][k] q[k][n].  The MMA computes D = W^T A^T with
// the 128 weight columns of a CTA tile as its M dimension and the activation
// rows as its N dimension:
//   A operand  the int8 weights of a 64-k chunk, widened to bf16 (exact for
//              |q| <= 128) into an MN-major tile (the weights' own layout:
//              n contiguous);
//   B operand  the fp32 activations split into three bf16 terms, hi + mid +
//              lo (hi = bf16(a), mid = bf16(a - hi), lo = bf16(a - hi - mid):
//              24 mantissa bits between them), K-major, as 3*MT rows;
//   D          fp32 in TMEM, 128 lanes (columns n) x 3*MT columns; the
//              epilogue adds the three terms and applies the column scale.
// A CTA of 256 threads streams its K range: int8 weights and fp32 activations
// of four 64-k chunks in flight through a cp.async ring, each chunk converted
// into one of two operand buffers while the tensor core works on the other,
// four K=16 MMAs per chunk issued by one elected thread and committed to the
// buffer's mbarrier.  K parts of a tile meet in the serial fix-up (last CTA
// adds in K order), so results do not depend on timing.  Every wait is
// bounded: a timeout sets the library's device error word and the CTA skips
// its remaining chunks, frees its TMEM and exits.
#include <algorithm>
#include <atomic>

#include "gdn_internal.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int TN = 128, KC = 64, NST = 4, TCT = 256;

__device__ __forceinline__ void cp16z(void *dst, const void *src, bool full) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(full ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cpc() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cpw() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Four signed bytes as exact floats (byte ^ 0x80 in the mantissa of 2^23).
__device__ __forceinline__ void widen4(uint32_t w, float *f) {
    const uint32_t u = w ^ 0x80808080u;
    constexpr float kBias = 8388736.0f;  // 2^23 + 128
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - kBias;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - kBias;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - kBias;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - kBias;
}
// Two floats that are exact in bf16 (int8 values: at most 8 significant
// bits) as a bf16 pair: their upper halves, no rounding needed.
__device__ __forceinline__ uint32_t pack_bf16_exact(float lo, float hi) {
    return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632);
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

template <int MT> struct TcGeo {
    static constexpr int NM = 3 * MT;                       // MMA N: hi, mid, lo rows
    static constexpr int TMEM_COLS = NM <= 64 ? 64 : NM <= 128 ? 128 : 256;
    static constexpr int RING_W = KC * TN;                  // int8 bytes per stage
    static constexpr int RING_A = MT * KC * 4;              // fp32 bytes per stage
    static constexpr int STAGE = RING_W + RING_A;
    static constexpr int OP_W = KC * TN * 2;                // bf16 weight tile
    static constexpr int OP_B = NM * KC * 2;                // bf16 activation tile
    static constexpr int OP = OP_W + OP_B;
    static constexpr size_t SMEM = (size_t)NST * STAGE + 2 * (size_t)OP + 1024;
};

template <int MT>
__global__ void __launch_bounds__(TCT, 1)
    matmul_int8_tc_kernel(const float *__restrict__ A, const int8_t *__restrict__ q, const float *__restrict__ s,
                          float *__restrict__ C, long long M, long long K, long long N, float *__restrict__ part,
                          unsigned int *__restrict__ ctr, int *err) {
    using G = TcGeo<MT>;
    extern __shared__ unsigned char dsm_raw[];
    // operand tiles want 128-byte alignment at least; round the base up to 1024
    unsigned char *dsm = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);
    unsigned char *op = dsm;                      // [2][OP]: weights (MN-major) then activations (K-major)
    unsigned char *ring = dsm + 2 * G::OP;        // [NST][STAGE]: int8 weights then fp32 activations
    __shared__ uint64_t mma_bar[2];
    __shared__ uint32_t tmem_slot;
    __shared__ bool s_last;

    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const long long n0 = (long long)blockIdx.x * TN, m0 = (long long)blockIdx.y * MT;
    const int ksplit = (int)gridDim.z, rank = (int)blockIdx.z;
    const long long kper = ((K + ksplit - 1) / ksplit + KC - 1) / KC * KC;
    const long long k0 = (long long)rank * kper, k1 = min(K, k0 + kper);
    const int nch = k1 > k0 ? (int)((k1 - k0 + KC - 1) / KC) : 0;

    if (t == 0) {
        mbar_init(&mma_bar[0], 1);
        mbar_init(&mma_bar[1], 1);
    }
    if (warp == 0) tmem_alloc(&tmem_slot, G::TMEM_COLS);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_slot;

    auto issue = [&](int c) {
        if (c < nch) {
            unsigned char *st = ring + (c % NST) * G::STAGE;
            const long long kb = k0 + (long long)c * KC;
            // weights: 64 rows x 8 chunks of 16 bytes
            for (int i = t; i < KC * (TN / 16); i += TCT) {
                const int r = i / (TN / 16), cc = i % (TN / 16);
                const long long k = kb + r, n = n0 + cc * 16;
                const bool ok = k < k1 && n < N;
                cp16z(st + r * TN + cc * 16, q + (ok ? k * N + n : 0), ok);
            }
            // activations: MT rows x 16 chunks of 4 floats
            float *sa = reinterpret_cast<float *>(st + G::RING_W);
            for (int i = t; i < MT * (KC / 4); i += TCT) {
                const int r = i / (KC / 4), cc = i % (KC / 4);
                const long long m = m0 + r, k = kb + cc * 4;
                const bool ok = m < M && k < k1;
                cp16z(sa + r * KC + cc * 4, A + (ok ? m * K + k : 0), ok);
            }
        }
        cpc();
    };

    bool bad = false;
#pragma unroll
    for (int c = 0; c < NST - 1; ++c) issue(c);
    for (int c = 0; c < nch; ++c) {
        cpw<NST - 2>();
        __syncthreads();  // chunk c is in; every thread is done with chunk c - 1's stage
        issue(c + NST - 1);
        const int b = c & 1;
        if (c >= 2 && !mbar_wait(&mma_bar[b], ((c - 2) >> 1) & 1, err)) bad = true;  // MMAs of chunk c - 2 read b
        if (__syncthreads_or(bad)) break;
        fence_after_sync();
        const unsigned char *st = ring + (c % NST) * G::STAGE;
        unsigned char *ow = op + b * G::OP;
        unsigned char *ob = ow + G::OP_W;
        // All of this thread's ring reads first (they would otherwise wait one
        // by one behind the operand stores, which may alias for the compiler).
        constexpr int NW = KC * (TN / 16) / TCT, NA = MT * (KC / 4) / TCT;
        static_assert(NW * TCT == KC * (TN / 16) && NA * TCT == MT * (KC / 4), "copies per thread");
        uint4 wv[NW];
        float4 av4[NA];
        const float *sa = reinterpret_cast<const float *>(st + G::RING_W);
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            const int i = t + j * TCT;
            wv[j] = *reinterpret_cast<const uint4 *>(st + (i / (TN / 16)) * TN + (i % (TN / 16)) * 16);
        }
#pragma unroll
        for (int j = 0; j < NA; ++j) {
            const int i = t + j * TCT;
            av4[j] = *reinterpret_cast<const float4 *>(sa + (i / (KC / 4)) * KC + (i % (KC / 4)) * 4);
        }
        // weights: int8 [k][n] -> bf16 MN-major (n contiguous in groups of 8)
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            const int i = t + j * TCT, r = i / (TN / 16), cc = i % (TN / 16);
            const uint32_t ww[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
            float f[16];
#pragma unroll
            for (int e = 0; e < 4; ++e) widen4(ww[e], f + 4 * e);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 o = make_uint4(pack_bf16_exact(f[8 * h + 0], f[8 * h + 1]),
                                           pack_bf16_exact(f[8 * h + 2], f[8 * h + 3]),
                                           pack_bf16_exact(f[8 * h + 4], f[8 * h + 5]),
                                           pack_bf16_exact(f[8 * h + 6], f[8 * h + 7]));
                *reinterpret_cast<uint4 *>(ow + mnmaj16(r, cc * 16 + 8 * h, TN)) = o;
            }
        }
        // activations: fp32 [m][k] -> hi, mid, lo bf16, K-major rows term * MT + m
#pragma unroll
        for (int j = 0; j < NA; ++j) {
            const int i = t + j * TCT, r = i / (KC / 4), cc = i % (KC / 4);
            const float av[4] = {av4[j].x, av4[j].y, av4[j].z, av4[j].w};
            float hi[4], mid[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hi[e] = __bfloat162float(__float2bfloat16_rn(av[e]));
                const float r1 = av[e] - hi[e];
                mid[e] = __bfloat162float(__float2bfloat16_rn(r1));
                lo[e] = r1 - mid[e];
            }
            *reinterpret_cast<uint2 *>(ob + kmaj16(r, cc * 4, KC)) =
                make_uint2(pack_bf16(hi[0], hi[1]), pack_bf16(hi[2], hi[3]));
            *reinterpret_cast<uint2 *>(ob + kmaj16(MT + r, cc * 4, KC)) =
                make_uint2(pack_bf16(mid[0], mid[1]), pack_bf16(mid[2], mid[3]));
            *reinterpret_cast<uint2 *>(ob + kmaj16(2 * MT + r, cc * 4, KC)) =
                make_uint2(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]));
        }
        fence_smem_to_async();
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
        if (warp == 0) {
            if (elect_one()) {
                const uint32_t id = idesc(TN, G::NM, BF16, true, false);
#pragma unroll
                for (int ks = 0; ks < KC / 16; ++ks)
                    mma_f16(tmem, desc_mnmaj16(ow, TN, ks), desc_kmaj16(ob, KC, ks), id, c > 0 || ks > 0);
                commit(&mma_bar[b]);
            }
            __syncwarp();
        }
    }
    cpw<0>();
    if (!bad && nch > 0 && !mbar_wait(&mma_bar[(nch - 1) & 1], ((nch - 1) >> 1) & 1, err)) bad = true;
    bad = __syncthreads_or(bad);
    fence_after_sync();

    // epilogue (warps 0-3, one TMEM lane quarter each): lane n = 32 warp + lane
    // of the tile; columns m, MT + m, 2 MT + m
    const int wq = warp & 3, wh = warp >> 2;
    const long long n = n0 + 32 * wq + lane;
    if (!bad && wh == 0) {
#pragma unroll
        for (int mc = 0; mc < MT; mc += 16) {
            float h[16], md[16], lw[16];
            if (nch > 0) {
                tmem_ld16(taddr(tmem, 32 * warp, mc), h);
                tmem_ld16(taddr(tmem, 32 * warp, MT + mc), md);
                tmem_ld16(taddr(tmem, 32 * warp, 2 * MT + mc), lw);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) h[i] = md[i] = lw[i] = 0.0f;
            }
            if (n < N) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const long long m = m0 + mc + i;
                    if (m >= M) break;
                    const float v = (h[i] + md[i]) + lw[i];
                    if (ksplit == 1)
                        C[m * N + n] = v * s[n];
                    else
                        part[((long long)rank * M + m) * N + n] = v;
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, G::TMEM_COLS);
    if (ksplit == 1) return;
    // serial fix-up: the last CTA of the tile adds the K parts in order.  A
    // CTA whose wait ran out (bad) wrote no partials but still counts itself
    // (adding a mark in the high half), so the counter always reaches ksplit
    // and the last CTA resets it; when any part of the tile is missing the
    // sum is skipped (the call has already recorded its timeout).
    __shared__ bool s_skip;
    __threadfence();
    __syncthreads();
    const unsigned int tile = blockIdx.y * gridDim.x + blockIdx.x;
    if (t == 0) {
        const unsigned int mine = bad ? 0x10001u : 1u;
        const unsigned int old = atomicAdd(&ctr[tile], mine);
        s_last = (old & 0xFFFFu) == (unsigned)ksplit - 1;
        s_skip = ((old + mine) >> 16) != 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (s_skip) {
        if (t == 0) ctr[tile] = 0u;
        return;
    }
    if (n < N) {
        for (int i = wh; i < MT; i += TCT / 128) {
            const long long m = m0 + i;
            if (m >= M) break;
            const float v = sum_parts_ordered(part + (long long)m * N + n, (long long)M * N, ksplit);
            C[m * N + n] = v * s[n];
        }
    }
    if (t == 0) ctr[tile] = 0u;
}

template <int MT>
int run_tc(const float *A, const int8_t *q, const float *s, float *C, long long M, long long K, long long N,
           cudaStream_t st) {
    using G = TcGeo<MT>;
    static std::atomic<unsigned long long> attr_set{0};  // per device
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "matmul_int8: cudaGetDevice");
    if (rc) return rc;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        rc = check_cuda(cudaFuncSetAttribute(matmul_int8_tc_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)G::SMEM),
                        "matmul_int8: smem attribute");
        if (rc) return rc;
        attr_set.fetch_or(bit);
    }
    const long long nt = (N + TN - 1) / TN, mt = (M + MT - 1) / MT, chunks = (K + KC - 1) / KC;
    if (mt > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "matmul_int8: M too large");
    // split K until the tiles cover the SMs, keeping two chunks per part
    int ks = 1;
    while (ks < 32 && nt * mt * ks < sm_count() && chunks >= 4ll * ks) ks *= 2;
    unsigned int *ctr = nullptr;
    float *part = nullptr;
    if (ks > 1 && (rc = split_workspace(st, (size_t)(nt * mt), (size_t)ks * M * N, &ctr, &part))) return rc;
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    matmul_int8_tc_kernel<MT><<<dim3((unsigned)nt, (unsigned)mt, (unsigned)ks), TCT, G::SMEM, st>>>(
        A, q, s, C, M, K, N, part, ctr, err);
    return check_launch("matmul_int8_tc_kernel");
}

}  // namespace

int launch_matmul_int8_tc(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N,
                          cudaStream_t st) {
    const long long m = (long long)M, k = (long long)K, n = (long long)N;
    if (M <= 16) return run_tc<16>(A, q, s, C, m, k, n, st);
    if (M <= 32) return run_tc<32>(A, q, s, C, m, k, n, st);
    return run_tc<64>(A, q, s, C, m, k, n, st);
}

}  // namespace gdn
