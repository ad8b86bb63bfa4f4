// attn_prefill.cu -- causal grouped-query attention over a prompt: every
// query position t of a sequence attends to the cached keys 0 .. pos0 + t of
// its kv head (the reference's full_attn_real_forward,
// src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:1532-1634, applied to
// each prompt token in turn, with the prompt's keys and values already in the
// bf16 cache).  The decode step handles one new token at a time; a prompt of
// T tokens is this one launch.
//
// CTA = (block of QP = 64 / G query positions, kv head, batch): the G query
// heads of the kv head at QP positions are 64 query rows r = p * G + g.  Both
// products run on tcgen05 with the keys as the MMA's M dimension (the decode
// kernel's orientation), per tile of 64 cached tokens:
//   S^T = K Qs^T      M = 64 tokens, N = 128 (two bf16 terms hi + lo of each
//                     fp32 query row: 16 significant bits), K = D.
//   O^T += V^T Ps^T   M = 128 head dims (D / 128 MMAs), N = 128 (two bf16
//                     terms of each softmax weight), K = 64 tokens.
// O^T accumulates in TMEM across the tiles.  The softmax keeps, per query
// row, a reference maximum m: weights are e^(s - m) and only when a score
// exceeds m by more than e^8 (weights stay below 2981, exact enough in two
// bf16 terms) are the tile's maxima reduced, m raised and O^T and the row
// sums rescaled in place -- a handful of times per row, at the first tiles;
// other tiles check their scores against m and need no reduction at all.
//
// Warp 8 issues the loads (TMA, 128-byte swizzle, two stages) and the MMAs;
// warps 0-7 run the softmax (warp w: the tokens of TMEM lanes 32 (w % 4) ..
// +15, query rows 32 (w / 4) .. +31), the rescales and the output (warp w:
// head dims of O^T half w / 4, lanes 32 (w % 4) ..).  Waits are bounded: a
// timeout sets the library's device error word and the CTA stops, frees its
// TMEM and exits.  Heavy CTAs (late query blocks) are scheduled first.
#include <algorithm>
#include <atomic>

#include "gdn_internal.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int PF_TT = 64;    // tokens per tile
constexpr int PF_QR = 64;    // query rows per CTA
constexpr int PF_NQ = 128;   // MMA N: two terms of the query rows
constexpr int PF_AT = 288;   // 8 softmax / output warps + 1 issuing warp
constexpr float PF_RESCALE = 8.0f;  // raise the reference maximum past this margin (natural log)

template <int D> struct PfGeo {
    static constexpr int BOX = PF_TT * 128;        // one 64-feature box of a tile
    static constexpr int KT = PF_TT * D * 2;       // a K (or V) tile
    static constexpr int STAGE = 2 * KT;
    static constexpr int NST = 2;
    static constexpr int QOP = PF_NQ * D * 2;      // Qs, K-major 128 x D
    static constexpr int POP = PF_NQ * PF_TT * 2;  // Ps, K-major 128 x 64
    static constexpr int S_COL = 0;                // TMEM: two S^T buffers
    static constexpr int O_COL = 2 * PF_NQ;        // then O^T, D / 128 halves
    static constexpr int NCOL = O_COL + (D / 128) * PF_NQ;
    static constexpr uint32_t TMEM_COLS = NCOL <= 256 ? 256 : 512;
    static constexpr size_t SMEM = (size_t)NST * STAGE + QOP + 2 * (size_t)POP + 1024;
    static_assert(NCOL <= 512 && SMEM <= 227 * 1024, "fits one SM");
};

struct PfP {
    const float *q;
    float *o;
    long long T, H, Hkv, pos0, nqb;
    float scale;
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Barrier 1 over the 256 threads of warps 0-7, OR-reducing a flag.
__device__ __forceinline__ bool pf_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 256, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ uint32_t pf_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

template <int D, int G>
__global__ void __launch_bounds__(PF_AT, 1)
    attn_prefill_kernel(PfP p, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        int *err) {
    using Gm = PfGeo<D>;
    using T = __nv_bfloat16;
    constexpr int TT = PF_TT, NQ = PF_NQ, QP = PF_QR / G, NH = D / 128, NST = Gm::NST;
    extern __shared__ unsigned char dsm_raw[];
    unsigned char *dsm = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);
    unsigned char *ring = dsm;                    // [NST][K tile | V tile]
    unsigned char *qop = ring + NST * Gm::STAGE;  // Qs
    unsigned char *pop = qop + Gm::QOP;           // [2] Ps
    __shared__ uint64_t full[NST], bar_s[2], bar_o[2], pready[2];
    __shared__ uint32_t tmem_slot;
    __shared__ float s_red[4][PF_QR];   // tile maxima / row sums per lane quarter
    __shared__ float s_m[PF_QR];        // reference maxima of the rows
    __shared__ float s_a[PF_QR];        // rescale factors of the current tile

    const int t = threadIdx.x, lane = t % 32, w = t / 32;
    // heavy blocks first
    const long long qb = p.nqb - 1 - (long long)blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const long long p0 = qb * QP;                              // first query position of the block (prompt index)
    const long long last = min(p.T - 1, p0 + QP - 1) + p.pos0;  // highest cache position any row attends to
    const int ntile = (int)(last / TT) + 1;

    if (w < 8) {
        // Qs: rows (term, r), r = p * G + g; positions past the prompt read as zero
        for (int i = t; i < NQ * (D / 2); i += 256) {
            const int n = i / (D / 2), k = 2 * (i % (D / 2)), term = n / PF_QR, r = n % PF_QR;
            const long long pos = p0 + r / G;
            float v0 = 0.f, v1 = 0.f;
            if (pos < p.T) {
                const float *qr = p.q + ((b * p.T + pos) * p.H + kh * G + r % G) * D + k;
                const float x0 = qr[0], x1 = qr[1];
                const float h0 = __bfloat162float(__float2bfloat16_rn(x0)),
                            h1 = __bfloat162float(__float2bfloat16_rn(x1));
                v0 = term == 0 ? h0 : x0 - h0;
                v1 = term == 0 ? h1 : x1 - h1;
            }
            *reinterpret_cast<uint32_t *>(qop + kmaj16(n, k, D)) = pf_bf16x2(v0, v1);
        }
        if (t < PF_QR) s_m[t] = -INFINITY;
        fence_smem_to_async();
    } else {
        if (lane == 0) {
            for (int s = 0; s < NST; ++s) mbar_init(&full[s], 1);
            for (int s = 0; s < 2; ++s) {
                mbar_init(&bar_s[s], 1);
                mbar_init(&bar_o[s], 1);
                mbar_init(&pready[s], 256);
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            for (int s = 0; s < NST && s < ntile; ++s) {
                mbar_arrive_expect_tx(&full[s], 2 * Gm::KT);
                tma::load_chunk_sw128(ring + s * Gm::STAGE, &kmap, s * TT, (int)kh, (int)b, &full[s], D / 64, Gm::BOX);
                tma::load_chunk_sw128(ring + s * Gm::STAGE + Gm::KT, &vmap, s * TT, (int)kh, (int)b, &full[s], D / 64,
                                      Gm::BOX);
            }
        }
        __syncwarp();
        tmem_alloc(&tmem_slot, Gm::TMEM_COLS);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = tmem_slot;
    bool bad = false;

    if (w == 8) {
        // ------------------------------------------------------ issuing warp
        const uint32_t id_s = idesc(64, NQ, BF16, false, false), id_o = idesc(128, NQ, BF16, true, false);
        int nload = min(NST, ntile), nlanded = 0;
        auto issue_s = [&](int tile) -> bool {
            const int st = tile % NST;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (tile / NST) & 1, err))) return false;
            nlanded = tile + 1;
            if (elect_one()) {
                const uint32_t ka = smem_addr(ring + st * Gm::STAGE);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks)
                    mma_f16(tmem + Gm::S_COL + (tile & 1) * NQ,
                            smem_desc_sw128(ka + (ks / 4) * Gm::BOX + (ks % 4) * 32, 16, 1024),
                            desc_kmaj16(qop, D, ks), id_s, ks > 0);
                commit(&bar_s[tile & 1]);
            }
            __syncwarp();
            return true;
        };
        bad = !issue_s(0);
        for (int j = 0; j < ntile && !bad; ++j) {
            if (j + 1 < ntile && !issue_s(j + 1)) {
                bad = true;
                break;
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&pready[j & 1], (j >> 1) & 1, err))) {
                bad = true;
                break;
            }
            fence_after_sync();
            if (elect_one()) {
                const unsigned char *pb = pop + (j & 1) * Gm::POP;
                const uint32_t va = smem_addr(ring + (j % NST) * Gm::STAGE + Gm::KT);
#pragma unroll
                for (int h2 = 0; h2 < NH; ++h2)
#pragma unroll
                    for (int ks = 0; ks < TT / 16; ++ks)
                        mma_f16(tmem + Gm::O_COL + h2 * NQ,
                                smem_desc_sw128(va + h2 * 2 * Gm::BOX + ks * 2048, Gm::BOX, 1024),
                                desc_kmaj16(pb, TT, ks), id_o, j > 0 || ks > 0);
                commit(&bar_o[j & 1]);
            }
            __syncwarp();
            if (j + NST < ntile) {  // O(j) has released stage j % NST: tile j + NST goes there
                if (!__all_sync(0xffffffffu, mbar_wait(&bar_o[j & 1], (j >> 1) & 1, err))) {
                    bad = true;
                    break;
                }
                if (elect_one()) {
                    const int tile = j + NST, st = tile % NST;
                    unsigned char *kt = ring + st * Gm::STAGE;
                    mbar_arrive_expect_tx(&full[st], 2 * Gm::KT);
                    tma::load_chunk_sw128(kt, &kmap, tile * TT, (int)kh, (int)b, &full[st], D / 64, Gm::BOX);
                    tma::load_chunk_sw128(kt + Gm::KT, &vmap, tile * TT, (int)kh, (int)b, &full[st], D / 64, Gm::BOX);
                }
                __syncwarp();
                nload = j + NST + 1;
            }
        }
        // after a timeout: let the loads in flight land before the CTA exits
        for (int k = nlanded; k < nload; ++k) mbar_wait(&full[k % NST], (k / NST) & 1, nullptr, 1u << 16);
    } else {
        // ------------------------------------------ softmax / output warps
        const int q4 = w % 4, qh = w / 4;           // TMEM lane quarter; query-row half
        const int key_in_tile = 16 * q4 + lane;     // lanes 0-15: rows of the M = 64 S^T tile
        const bool key_lane = lane < 16;
        const float sl2 = p.scale * 1.4426950408889634f;  // scores in log2 units
        const float margin = PF_RESCALE * 1.4426950408889634f;
        float l_part[32], mref[32];  // row sums of this thread's token, reference maxima of its rows
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            l_part[i] = 0.f;
            mref[i] = -INFINITY;
        }
        for (int j = 0; j < ntile; ++j) {
            if (!mbar_wait(&bar_s[j & 1], (j >> 1) & 1, err)) bad = true;
            fence_after_sync();
            bad = __any_sync(0xffffffffu, bad);
            float sc[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) sc[i] = -INFINITY;
            if (!bad) {
                float hv[32], lv[32];
                const uint32_t c0 = Gm::S_COL + (j & 1) * NQ + 32 * qh;
                tmem_ld16(taddr(tmem, 32 * q4, c0), *reinterpret_cast<float(*)[16]>(hv));
                tmem_ld16(taddr(tmem, 32 * q4, c0 + 16), *reinterpret_cast<float(*)[16]>(hv + 16));
                tmem_ld16(taddr(tmem, 32 * q4, c0 + PF_QR), *reinterpret_cast<float(*)[16]>(lv));
                tmem_ld16(taddr(tmem, 32 * q4, c0 + PF_QR + 16), *reinterpret_cast<float(*)[16]>(lv + 16));
                tmem_wait_ld();
                reg_fence16(hv);
                reg_fence16(hv + 16);
                reg_fence16(lv);
                reg_fence16(lv + 16);
                const long long key = (long long)j * TT + key_in_tile;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int r = 32 * qh + i;
                    const long long qpos = p.pos0 + p0 + r / G;
                    const bool valid = key_lane && key <= qpos && p0 + r / G < p.T;
                    sc[i] = valid ? (hv[i] + lv[i]) * sl2 : -INFINITY;
                }
            }
            // Fast path: no score above its row's reference maximum plus the
            // margin (weights stay below e^8) -- nothing to reduce.  Otherwise
            // (and on the first tile) the tile maxima are reduced and the rows
            // that need it raised, with O^T and the row sums rescaled.
            bool over = false;
#pragma unroll
            for (int i = 0; i < 32; ++i) over = over || sc[i] > mref[i] + margin;
            bool resc = false;
            if (pf_sync_or(bad || over)) {
                if (pf_sync_or(bad)) {
                    bad = true;
                    break;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float mx = sc[i];
#pragma unroll
                    for (int mask = 8; mask >= 1; mask >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, mask));
                    if (lane == 0) s_red[q4][32 * qh + i] = mx;
                }
                pf_sync_or(false);
                if (t < PF_QR) {
                    float mt = fmaxf(fmaxf(s_red[0][t], s_red[1][t]), fmaxf(s_red[2][t], s_red[3][t]));
                    if (mt == -INFINITY) mt = 0.f;  // a row past the prompt's end: no token, weights 0
                    const float mo = s_m[t];
                    float a = 1.f;
                    if (mt > mo + margin || mo == -INFINITY) {
                        s_m[t] = mt;
                        a = exp2f(mo - mt);
                        resc = j > 0;
                    }
                    s_a[t] = a;
                }
                resc = pf_sync_or(resc);
#pragma unroll
                for (int i = 0; i < 32; ++i) mref[i] = s_m[32 * qh + i];
            }
            if (resc) {
                // O(j-1) must be complete before O^T is rescaled in TMEM
                if (!mbar_wait(&bar_o[(j - 1) & 1], ((j - 1) >> 1) & 1, err)) bad = true;
                fence_after_sync();
                bad = __any_sync(0xffffffffu, bad);
                if (!bad && qh < NH) {
#pragma unroll
                    for (int c = 0; c < NQ; c += 16) {
                        float ov[16];
                        const uint32_t ad = taddr(tmem, 32 * q4, Gm::O_COL + qh * NQ + c);
                        tmem_ld16(ad, ov);
                        tmem_wait_ld();
                        reg_fence16(ov);
#pragma unroll
                        for (int i = 0; i < 16; ++i) ov[i] *= s_a[(c + i) % PF_QR];
                        tmem_st16(ad, ov);
                    }
                    tmem_wait_st();
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) l_part[i] *= s_a[32 * qh + i];
            }
            // the weights buffer j & 1 was last read by O(j-2)
            if (!resc && j >= 2 && !mbar_wait(&bar_o[j & 1], ((j - 2) >> 1) & 1, err)) bad = true;
            if (!bad && key_lane) {
                unsigned char *pb = pop + (j & 1) * Gm::POP;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int r = 32 * qh + i;
                    const float e = exp2f(sc[i] - mref[i]);  // 0 for masked tokens
                    l_part[i] += e;
                    const __nv_bfloat16 hi = __float2bfloat16_rn(e);
                    *reinterpret_cast<T *>(pb + kmaj16(r, key_in_tile, TT)) = hi;
                    *reinterpret_cast<T *>(pb + kmaj16(PF_QR + r, key_in_tile, TT)) =
                        __float2bfloat16_rn(e - __bfloat162float(hi));
                }
            }
            fence_smem_to_async();
            fence_before_sync();
            mbar_arrive(&pready[j & 1]);
        }
        bad = pf_sync_or(bad);
        // row sums: lanes of a quarter, then the four quarters
        if (!bad) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float l = key_lane ? l_part[i] : 0.f;
#pragma unroll
                for (int mask = 8; mask >= 1; mask >>= 1) l += __shfl_xor_sync(0xffffffffu, l, mask);
                if (lane == 0) s_red[q4][32 * qh + i] = l;
            }
            const int jl = ntile - 1;
            if (!mbar_wait(&bar_o[jl & 1], (jl >> 1) & 1, err)) bad = true;
            fence_after_sync();
        }
        bad = pf_sync_or(bad);
        if (!bad && qh < NH) {
            const int d = 128 * qh + 32 * q4 + lane;
#pragma unroll
            for (int c = 0; c < PF_QR; c += 16) {
                float oh[16], ol[16];
                tmem_ld16(taddr(tmem, 32 * q4, Gm::O_COL + qh * NQ + c), oh);
                tmem_ld16(taddr(tmem, 32 * q4, Gm::O_COL + qh * NQ + PF_QR + c), ol);
                tmem_wait_ld();
                reg_fence16(oh);
                reg_fence16(ol);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int r = c + i;
                    const long long pos = p0 + r / G;
                    if (pos < p.T) {
                        const float L = (s_red[0][r] + s_red[1][r]) + (s_red[2][r] + s_red[3][r]);
                        p.o[((b * p.T + pos) * p.H + kh * G + r % G) * D + d] = (oh[i] + ol[i]) / L;
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (w == 8) tmem_dealloc(tmem, Gm::TMEM_COLS);
}

template <int D, int G>
int run_prefill(const kai_gdn_attn_prefill_args *a, cudaStream_t st) {
    using Gm = PfGeo<D>;
    auto kern = attn_prefill_kernel<D, G>;
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "attention_prefill: cudaGetDevice");
    if (rc) return rc;
    static std::atomic<unsigned long long> attr_set{0};  // per device
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        if ((rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Gm::SMEM),
                             "attention_prefill: smem attribute")))
            return rc;
        attr_set.fetch_or(bit);
    }
    constexpr long long QP = PF_QR / G;
    PfP p{};
    p.q = a->q;
    p.o = a->o;
    p.T = (long long)a->T;
    p.H = (long long)a->heads;
    p.Hkv = (long long)a->kv_heads;
    p.pos0 = (long long)a->pos0;
    p.nqb = (p.T + QP - 1) / QP;
    p.scale = a->scale;
    if (p.nqb > 0x7fffffffll || p.Hkv > 65535 || a->batch > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_prefill: shape too large");
    int *err = nullptr;
    if ((rc = device_error_word(&err))) return rc;
    CUtensorMap kmap, vmap;
    if (tma::make_chunk_map(&kmap, a->k_cache, true, (uint64_t)a->batch, (uint64_t)a->max_ctx, (uint64_t)p.Hkv, D,
                            true, PF_TT) ||
        tma::make_chunk_map(&vmap, a->v_cache, true, (uint64_t)a->batch, (uint64_t)a->max_ctx, (uint64_t)p.Hkv, D,
                            true, PF_TT))
        return set_error(KAI_GDN_ERR_CUDA, "attention_prefill: tensor map encoding failed");
    kern<<<dim3((unsigned)p.nqb, (unsigned)p.Hkv, (unsigned)a->batch), PF_AT, Gm::SMEM, st>>>(p, kmap, vmap, err);
    return check_launch("attn_prefill_kernel");
}

template <int D> int prefill_g(const kai_gdn_attn_prefill_args *a, size_t G, cudaStream_t st) {
    switch (G) {
        case 1: return run_prefill<D, 1>(a, st);
        case 2: return run_prefill<D, 2>(a, st);
        case 4: return run_prefill<D, 4>(a, st);
        default: return run_prefill<D, 8>(a, st);
    }
}

}  // namespace

int launch_attn_prefill(const kai_gdn_attn_prefill_args *a, cudaStream_t st) {
    if (!a) return set_error(KAI_GDN_ERR_INVALID, "attention_prefill: null args");
    if (a->batch == 0 || a->T == 0 || a->heads == 0) return KAI_GDN_OK;
    if (!a->q || !a->k_cache || !a->v_cache || !a->o)
        return set_error(KAI_GDN_ERR_INVALID, "attention_prefill: null pointer");
    if (a->kv_heads == 0 || a->heads % a->kv_heads)
        return set_error(KAI_GDN_ERR_INVALID, "attention_prefill: heads %zu not a multiple of kv_heads %zu", a->heads,
                         a->kv_heads);
    const size_t G = a->heads / a->kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_prefill: %zu query heads per kv head (1, 2, 4, 8)", G);
    if (a->head_dim != 128 && a->head_dim != 256)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_prefill: head_dim %zu (128, 256)", a->head_dim);
    if (a->pos0 + a->T > a->max_ctx)
        return set_error(KAI_GDN_ERR_INVALID, "attention_prefill: positions %zu .. %zu outside the cache (%zu)",
                         a->pos0, a->pos0 + a->T - 1, a->max_ctx);
    if ((uintptr_t)a->k_cache % 16 || (uintptr_t)a->v_cache % 16 || (uintptr_t)a->q % 8 || (uintptr_t)a->o % 4)
        return set_error(KAI_GDN_ERR_INVALID, "attention_prefill: caches must be 16-byte and q 8-byte aligned");
    if (a->head_dim == 128) return prefill_g<128>(a, G, st);
    return prefill_g<256>(a, G, st);
}

}  // namespace gdn
