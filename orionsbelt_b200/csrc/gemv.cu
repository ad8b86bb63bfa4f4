// gemv.cu -- int8-weight GEMV for the decode shapes (M <= 8 activation rows),
// C = (A q) diag(s) with q [K][N] int8 and one fp32 scale per column (the
// reference's gemv_int8_neon / gemm_int8_neon, gdn_e2e_decode.c:296-358,
// 608-678), streamed from HBM at the copy rate.
//
// Layout of the work: a warp owns 512 columns (16 per lane, one 16-byte load
// per weight row) and a K range; the 8 warps of a CTA take interleaved rows of
// the CTA's K range and add their sums through shared memory; CTAs split K so
// that the grid covers every SM twice, and the K parts meet in a fix-up by the
// last CTA of a column tile, in K order (deterministic).  Each thread keeps 8
// weight rows (128 bytes) in flight in registers, loaded with non-allocating
// read-only loads, while it converts and accumulates the previous 8: int8 ->
// fp32 exactly (the byte, biased by 128, in the mantissa of 2^23; packed pair
// subtraction) and packed fp32 multiply-adds.
//
// Programmatic dependent launch: the kernel may start while the kernel before
// it on the stream is still running.  Weights never depend on earlier work, so
// every CTA issues its first two weight stages, allows its own dependents to
// launch, and only then waits (griddepcontrol.wait) for the preceding grid
// before it reads the activations and issues the rest of its stages (with all
// six stages issued up front, the activation loads queued behind 28 MB of
// weights: 2.58 -> 2.53 ms per config-4 batch-1 step with two).  The K-part workspace alternates between two halves
// from one launch to the next on a stream, so a dependent that overlaps this
// kernel's fix-up never writes the partial sums being read.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "gdn_internal.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

constexpr int GW = 8;             // consumer warps per CTA
constexpr int KT = 32;            // weight rows per ring stage
constexpr int GNT = GW * 32 + 32;  // + one producer warp
constexpr int KMAX_OCC = 1024;     // longest K part (rows) a CTA takes
constexpr int PRE_STAGES = 2;      // ring stages issued before the dependency wait

// Tile geometry: CPL columns per lane (16: one 16-byte load per row, for up
// to 4 activation rows; 8: an 8-byte load, for 5..8 rows, which keeps the
// accumulators in registers), 32 lanes per tile, NSTG stages of KT rows.  The
// activation tile is [k][m], so a weight row's activations are broadcast
// vector loads.  (At 16 rows this kernel measured 46 us at 16 x 2560 x 9216,
// one CTA per SM by registers, against 39 us on the tensor-core path, which
// keeps M > 8.)
template <int CPL> struct GemvGeo {
    static constexpr int TC = 32 * CPL;         // columns per CTA tile
    static constexpr int STAGE = KT * TC;       // bytes per ring stage
    static constexpr int NSTG = CPL == 16 ? 6 : 8;
};
template <int MB> struct GemvCpl {
    static constexpr int CPL = MB <= 4 ? 16 : 8;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Four signed bytes of w as two float2 pairs, exact.
__device__ __forceinline__ void deq4x2(uint32_t w, float2 &a, float2 &b) {
    const uint32_t u = w ^ 0x80808080u;
    const float2 nbias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128), exact sums
    a = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)),
                               __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651))),
                   nbias);
    b = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)),
                               __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653))),
                   nbias);
}

// acc[m][0 .. CPL/2) (float2 pairs of the lane's columns) += a[m] * row
template <int MB, int CPL>
__device__ __forceinline__ void accumulate(float2 (&acc)[MB][CPL / 2], const uint32_t (&ws)[CPL / 4],
                                           const float *a) {
#pragma unroll
    for (int j = 0; j < CPL / 4; ++j) {
        float2 p0, p1;
        deq4x2(ws[j], p0, p1);
#pragma unroll
        for (int m = 0; m < MB; ++m) {
            const float2 am = make_float2(a[m], a[m]);
            acc[m][2 * j] = __ffma2_rn(am, p0, acc[m][2 * j]);
            acc[m][2 * j + 1] = __ffma2_rn(am, p1, acc[m][2 * j + 1]);
        }
    }
}
template <int CPL> __device__ __forceinline__ void ld_row(const unsigned char *p, uint32_t (&ws)[CPL / 4]);
template <> __device__ __forceinline__ void ld_row<16>(const unsigned char *p, uint32_t (&ws)[4]) {
    const uint4 v = *reinterpret_cast<const uint4 *>(p);
    ws[0] = v.x, ws[1] = v.y, ws[2] = v.z, ws[3] = v.w;
}
template <> __device__ __forceinline__ void ld_row<8>(const unsigned char *p, uint32_t (&ws)[2]) {
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    ws[0] = v.x, ws[1] = v.y;
}

__device__ __forceinline__ void tma_rows(unsigned char *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(umma::smem_addr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
        "r"(umma::smem_addr(bar))
        : "memory");
}

// Grid (ceil(N / TC), ksplit).  A [M][K], s [N], C [M][N]; the weights come
// either through `map` (q [K][N], boxes of 256 columns x KT rows) or, BLK,
// from qb in the blocked layout [ceil(N / TC)][K][TC] (one contiguous bulk
// copy per stage).  part [ksplit][M][N] and ctr [tiles] (zero between calls)
// when ksplit > 1.  Warp 8 (one lane) fills the ring; warps 0-7 take KT / 8
// rows of each stage, each lane CPL columns.
template <int MB, int CPL, bool BLK>
__global__ void __launch_bounds__(GNT) gemv_int8_kernel(const __grid_constant__ CUtensorMap map,
                                                        const int8_t *__restrict__ qb,
                                                        const float *__restrict__ A, const float *__restrict__ s,
                                                        float *__restrict__ C, int M, long long K, long long N,
                                                        long long kper, float *__restrict__ part,
                                                        unsigned int *__restrict__ ctr, int *err, int swiglu) {
    using G = GemvGeo<CPL>;
    constexpr int TC = G::TC, STAGE = G::STAGE, NSTG = G::NSTG;
    extern __shared__ unsigned char dsm_raw[];
    unsigned char *ring = dsm_raw + ((1024u - (umma::smem_addr(dsm_raw) & 1023u)) & 1023u);  // [NSTG][STAGE]
    float *sm_a = reinterpret_cast<float *>(ring + NSTG * STAGE);                          // [kper][MB]
    // after the ring has been drained: one row m at a time, [warp][column % CPL][column / CPL]
    float(*red)[CPL][32] = reinterpret_cast<float(*)[CPL][32]>(ring);
    __shared__ uint64_t full[NSTG], empty[NSTG];
    __shared__ bool s_last;
    const int t = threadIdx.x, w = t / 32, lane = t % 32;
    const int ksplit = (int)gridDim.y, rank = (int)blockIdx.y;
    const long long tile0 = (long long)blockIdx.x * TC;
    const long long k0 = (long long)rank * kper, k1 = min(K, k0 + kper);
    const int nk = k1 > k0 ? (int)((k1 - k0 + KT - 1) / KT) : 0;

    if (t == 0) {
        for (int i = 0; i < NSTG; ++i) {
            umma::mbar_init(&full[i], 1);
            umma::mbar_init(&empty[i], GW);
        }
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    int issued = 0;
    bool bad = false;
    const int8_t *tile_rows = BLK ? qb + (size_t)blockIdx.x * (size_t)K * TC : nullptr;
    auto load_stage = [&](int i, int st) {
        const long long r0 = k0 + (long long)i * KT;
        if (BLK) {
            const uint32_t bytes = (uint32_t)(min((long long)KT, k1 - r0) * TC);
            umma::mbar_arrive_expect_tx(&full[st], bytes);
            umma::bulk_load(ring + st * STAGE, tile_rows + r0 * TC, bytes, &full[st]);
        } else {
            umma::mbar_arrive_expect_tx(&full[st], STAGE);
#pragma unroll
            for (int b = 0; b < TC / 256; ++b)
                tma_rows(ring + st * STAGE + b * (KT * 256), &map, (int)tile0 + 256 * b, (int)r0, &full[st]);
        }
    };
    if (w == GW) {
        // ---- producer: weights never depend on earlier kernels, so the
        // first stages are issued before the dependency wait
        if (lane == 0)
            for (; issued < nk && issued < PRE_STAGES; ++issued) load_stage(issued, issued);
        pdl_trigger();
        pdl_wait();
        if (lane == 0) {
            for (; issued < nk && !bad; ++issued) {
                const int st = issued % NSTG;
                if (issued >= NSTG && !umma::mbar_wait(&empty[st], (uint32_t)(((issued / NSTG) - 1) & 1), err)) {
                    bad = true;
                    break;
                }
                load_stage(issued, st);
            }
            // every issued load lands before the CTA may leave
            for (int i = issued - NSTG > 0 ? issued - NSTG : 0; i < issued; ++i)
                umma::mbar_wait(&full[i % NSTG], (uint32_t)((i / NSTG) & 1), err);
        }
        __syncwarp();
    } else {
        pdl_trigger();
        pdl_wait();
        // this CTA's activations
        const long long kn = k1 > k0 ? k1 - k0 : 0;
        for (long long e = t; e < (long long)MB * kn; e += GW * 32) {
            const int m = (int)(e / kn);
            const long long k = e % kn;
            float a = 0.f;
            if (m < M) {
                if (swiglu) {  // rows [gate (K) | up (K)]: SiLU(gate) * up, the FFN activation
                    const float gv = A[(long long)m * 2 * K + k0 + k];
                    a = gv / (1.0f + expf(-gv)) * A[(long long)m * 2 * K + K + k0 + k];
                } else {
                    a = A[(long long)m * K + k0 + k];
                }
            }
            sm_a[k * MB + m] = a;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(GW * 32) : "memory");
        float2 acc[MB][CPL / 2];
#pragma unroll
        for (int m = 0; m < MB; ++m)
#pragma unroll
            for (int j = 0; j < CPL / 2; ++j) acc[m][j] = make_float2(0.f, 0.f);
        // blocked rows are TC contiguous bytes; TMA stages hold 256-column boxes one after another
        const int lane_off = BLK ? lane * CPL : (lane * CPL / 256) * (KT * 256) + (lane * CPL) % 256;
        const int row_bytes = BLK ? TC : 256;
        for (int i = 0; i < nk; ++i) {
            const int st = i % NSTG;
            if (!umma::mbar_wait(&full[st], (uint32_t)((i / NSTG) & 1), err)) bad = true;
            if (__any_sync(0xffffffffu, bad)) break;
            const unsigned char *sb = ring + st * STAGE + lane_off;
            uint32_t wv[KT / GW][CPL / 4];
#pragma unroll
            for (int j = 0; j < KT / GW; ++j) ld_row<CPL>(sb + (w + GW * j) * row_bytes, wv[j]);
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_addr(&empty[st])) : "memory");
#pragma unroll
            for (int j = 0; j < KT / GW; ++j) {
                const long long rr = k0 + (long long)i * KT + w + GW * j;
                if (rr < k1) {
                    float a[MB];
                    const float *ar = sm_a + (rr - k0) * MB;  // broadcast vector loads
                    if constexpr (MB % 4 == 0) {
#pragma unroll
                        for (int m = 0; m < MB; m += 4) {
                            const float4 v = *reinterpret_cast<const float4 *>(ar + m);
                            a[m] = v.x, a[m + 1] = v.y, a[m + 2] = v.z, a[m + 3] = v.w;
                        }
                    } else {
#pragma unroll
                        for (int m = 0; m < MB; ++m) a[m] = ar[m];
                    }
                    accumulate<MB, CPL>(acc, wv[j], a);
                }
            }
        }
        // add the 8 warps' sums one activation row at a time (in the drained
        // ring); thread e takes column (e % 32) * CPL + e / 32 of the tile
        asm volatile("bar.sync 1, %0;" ::"n"(GW * 32) : "memory");
#pragma unroll
        for (int m = 0; m < MB; ++m) {
#pragma unroll
            for (int j = 0; j < CPL / 2; ++j) {
                red[w][2 * j][lane] = acc[m][j].x;
                red[w][2 * j + 1][lane] = acc[m][j].y;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(GW * 32) : "memory");
            for (int e = t; e < TC; e += GW * 32) {
                const int jj = e / 32, ln = e % 32;
                const long long n = tile0 + ln * CPL + jj;
                float v = 0.f;
#pragma unroll
                for (int ww = 0; ww < GW; ++ww) v += red[ww][jj][ln];
                if (m < M && n < N) {
                    if (ksplit == 1)
                        C[(long long)m * N + n] = v * s[n];
                    else
                        part[((long long)rank * M + m) * N + n] = v;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(GW * 32) : "memory");
        }
    }
    if (ksplit == 1) return;
    // K parts meet in the last CTA of the tile, in K order (a CTA whose wait
    // ran out still counts itself, marked, so the counter always resets)
    __threadfence();
    bad = __syncthreads_or(bad);
    if (t == 0) {
        const unsigned int mine = bad ? 0x10001u : 1u;
        const unsigned int old = atomicAdd(&ctr[blockIdx.x], mine);
        s_last = (old & 0xFFFFu) == (unsigned)ksplit - 1;
        if (s_last && ((old + mine) >> 16) != 0u) {
            ctr[blockIdx.x] = 0u;
            s_last = false;
        }
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int e = t; e < MB * TC; e += GNT) {
        const int m = e / TC, c = e % TC;
        const long long n = tile0 + c;
        if (m >= M || n >= N) continue;
        const float v = sum_parts_ordered(part + (long long)m * N + n, (long long)M * N, ksplit);
        C[(long long)m * N + n] = v * s[n];
    }
    if (t == 0) ctr[blockIdx.x] = 0u;
}

// Per-stream workspace: two halves, alternating per launch.
struct GemvWs {
    int device;
    cudaStream_t stream;
    unsigned int *ctr[2];
    float *part[2];
    size_t nctr, npart;
    unsigned flip;
};
std::mutex g_gemv_mu;
std::vector<GemvWs> g_gemv_ws;

int gemv_workspace(cudaStream_t st, size_t nctr, size_t npart, unsigned int **ctr, float **part) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "gemv: cudaGetDevice");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_gemv_mu);
    GemvWs *e = nullptr;
    for (auto &x : g_gemv_ws)
        if (x.device == dev && x.stream == st) e = &x;
    if (!e) {
        g_gemv_ws.push_back({dev, st, {nullptr, nullptr}, {nullptr, nullptr}, 0, 0, 0});
        e = &g_gemv_ws.back();
    }
    if (e->nctr < nctr || e->npart < npart) {
        for (int h = 0; h < 2; ++h) {  // cudaFree waits for the device
            if (e->ctr[h]) cudaFree(e->ctr[h]);
            if (e->part[h]) cudaFree(e->part[h]);
            e->ctr[h] = nullptr;
            e->part[h] = nullptr;
        }
        const size_t nc = std::max<size_t>(nctr, 4096), np = std::max<size_t>(npart, 1 << 18);
        for (int h = 0; h < 2 && !rc; ++h) {
            rc = check_cuda(cudaMalloc(&e->ctr[h], nc * sizeof(unsigned int)), "gemv: cudaMalloc");
            if (!rc) rc = check_cuda(cudaMemsetAsync(e->ctr[h], 0, nc * sizeof(unsigned int), st), "gemv: memset");
            if (!rc) rc = check_cuda(cudaMalloc(&e->part[h], np * sizeof(float)), "gemv: cudaMalloc");
        }
        if (rc) return rc;
        e->nctr = nc;
        e->npart = np;
    }
    const unsigned h = e->flip++ & 1u;
    *ctr = e->ctr[h];
    *part = e->part[h];
    return KAI_GDN_OK;
}

template <int MB, bool BLK>
int run_gemv(const float *A, const int8_t *q, const float *s, float *Cm, int M, long long K, long long N,
             cudaStream_t st, bool swiglu) {
    constexpr int CPL = GemvCpl<MB>::CPL;
    using G = GemvGeo<CPL>;
    auto kern = gemv_int8_kernel<MB, CPL, BLK>;
    static int occ[64] = {0};  // resident CTAs per SM, per device
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "gemv: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return set_error(KAI_GDN_ERR_UNSUPPORTED, "gemv: device %d", dev);
    const size_t ring = 1024 + (size_t)G::NSTG * G::STAGE;
    if (!occ[dev]) {
        if ((rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024),
                             "gemv: smem attribute")))
            return rc;
        // residency with a K part of up to KMAX_OCC rows of activations
        int n = 0;
        if ((rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, GNT,
                                                                            ring + (size_t)MB * KMAX_OCC * 4),
                             "gemv: occupancy")))
            return rc;
        occ[dev] = std::max(1, n);
    }
    // one wave: tiles x ksplit <= resident CTAs on the device, each K part at
    // most KMAX_OCC rows (the residency assumed above)
    const long long tiles = (N + G::TC - 1) / G::TC;
    const long long slots = (long long)occ[dev] * sm_count();
    long long ksplit = std::max<long long>(1, std::min<long long>(slots / tiles, (K + 2 * KT - 1) / (2 * KT)));
    ksplit = std::max<long long>(ksplit, (K + KMAX_OCC - 1) / KMAX_OCC);
    ksplit = std::min<long long>(ksplit, 0xFFFF);
    long long kper = (K + ksplit - 1) / ksplit;
    kper = (kper + KT - 1) / KT * KT;
    ksplit = (K + kper - 1) / kper;
    const size_t smem = ring + (size_t)MB * (size_t)kper * sizeof(float);
    if (smem > 220 * 1024) return set_error(KAI_GDN_ERR_UNSUPPORTED, "gemv: K part too long");
    unsigned int *ctr = nullptr;
    float *part = nullptr;
    if (ksplit > 1 && (rc = gemv_workspace(st, (size_t)tiles, (size_t)(ksplit * M * N), &ctr, &part))) return rc;
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    CUtensorMap map;
    memset(&map, 0, sizeof(map));
    if (!BLK) {
        tma::EncodeTiled enc = tma::encoder();
        if (!enc) return set_error(KAI_GDN_ERR_CUDA, "gemv: cuTensorMapEncodeTiled unavailable");
        const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)K};
        const cuuint64_t strides[1] = {(cuuint64_t)N};
        const cuuint32_t box[2] = {256, KT};
        const cuuint32_t es[2] = {1, 1};
        const CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(q), dims, strides, box,
                                es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS) return set_error(KAI_GDN_ERR_CUDA, "gemv: tensor map encoding failed (%d)", (int)cr);
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)tiles, (unsigned)ksplit);
    cfg.blockDim = dim3(GNT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, map, q, A, s, Cm, M, K, N, kper, part, ctr, err, swiglu ? 1 : 0);
    if (le != cudaSuccess) return check_cuda(le, "gemv_int8_kernel launch");
    return check_launch("gemv_int8_kernel");
}

template <bool BLK>
int dispatch_gemv(const float *A, const int8_t *q, const float *s, float *Cm, size_t M, size_t K, size_t N,
                  cudaStream_t st, bool swiglu = false) {
    const long long k = (long long)K, n = (long long)N;
    if (M == 1) return run_gemv<1, BLK>(A, q, s, Cm, 1, k, n, st, swiglu);
    if (M == 2) return run_gemv<2, BLK>(A, q, s, Cm, 2, k, n, st, swiglu);
    if (M <= 4) return run_gemv<4, BLK>(A, q, s, Cm, (int)M, k, n, st, swiglu);
    return run_gemv<8, BLK>(A, q, s, Cm, (int)M, k, n, st, swiglu);
}

}  // namespace

bool gemv_int8_supported(size_t M, size_t K, size_t N, const int8_t *q) {
    return M >= 1 && M <= 8 && K > 0 && N % 16 == 0 && (uintptr_t)q % 16 == 0 && K < (1ull << 31) &&
           N < (1ull << 31);
}

int launch_gemv_int8(const float *A, const int8_t *q, const float *s, float *Cm, size_t M, size_t K, size_t N,
                     cudaStream_t st) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!A || !q || !s || !Cm) return set_error(KAI_GDN_ERR_INVALID, "gemv_int8: null pointer");
    if (!gemv_int8_supported(M, K, N, q)) return set_error(KAI_GDN_ERR_UNSUPPORTED, "gemv_int8: shape");
    return dispatch_gemv<false>(A, q, s, Cm, M, K, N, st);
}

// Blocked weight layout for M activation rows: [ceil(N / TC)][K][TC] bytes
// (TC = 512 for M <= 4, 256 for M <= 8; the columns of a tile contiguous row
// after row, the last tile zero-padded), so one tile's rows stream as
// contiguous bulk copies.
size_t gemv_tile_cols(size_t M) { return M <= 4 ? 512 : 256; }

__global__ void block_weights_kernel(const int8_t *__restrict__ q, int8_t *__restrict__ qb, long long K, long long N,
                                     long long TC) {
    const long long tiles = (N + TC - 1) / TC, per = TC / 16, n16 = tiles * K * per;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n16; e += (long long)gridDim.x * blockDim.x) {
        const long long t = e / (K * per), rem = e % (K * per);
        const long long k = rem / per, c16 = rem % per;
        const long long n = t * TC + c16 * 16;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < N) v = *reinterpret_cast<const uint4 *>(q + k * N + n);
        *reinterpret_cast<uint4 *>(qb + (t * K + k) * TC + c16 * 16) = v;
    }
}

size_t gemv_blocked_bytes(size_t M, size_t K, size_t N) {
    const size_t tc = gemv_tile_cols(M);
    return (N + tc - 1) / tc * K * tc;
}

int gemv_block_weights(size_t M, const int8_t *q, int8_t *qb, size_t K, size_t N, cudaStream_t st) {
    if (N % 16 || (uintptr_t)q % 16 || (uintptr_t)qb % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "gemv_block_weights: N % 16 and 16-byte alignment");
    const long long n16 = (long long)gemv_blocked_bytes(M, K, N) / 16;
    block_weights_kernel<<<(unsigned)std::min<long long>((n16 + 255) / 256, 65535), 256, 0, st>>>(
        q, qb, (long long)K, (long long)N, (long long)gemv_tile_cols(M));
    return check_launch("block_weights_kernel");
}

int launch_gemv_int8_blocked(const float *A, const int8_t *qb, const float *s, float *Cm, size_t M, size_t K,
                             size_t N, cudaStream_t st, bool swiglu) {
    if (M == 0 || N == 0) return KAI_GDN_OK;
    if (!A || !qb || !s || !Cm) return set_error(KAI_GDN_ERR_INVALID, "gemv_int8: null pointer");
    if (!gemv_int8_supported(M, K, N, qb)) return set_error(KAI_GDN_ERR_UNSUPPORTED, "gemv_int8: shape");
    return dispatch_gemv<true>(A, qb, s, Cm, M, K, N, st, swiglu);
}

}  // namespace gdn
