// attn.cu -- grouped-query attention decode over a growing KV cache: one new
// token per sequence attends to every cached token of its kv head.
//   full_attn_real_forward        src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:1532-1634
//   full_attn_real_forward_int8kv gdn_e2e_decode.c:1652-1830 (int8 cache, one scale per kv head)
// and a bf16 cache (not in the reference), round-to-nearest-even on append.
// Cache layout as the reference's: [batch][max_ctx][kv_heads][head_dim].
//
// Split over the context (flash decoding): CTA (split, kv head, batch) takes a
// run of tokens and the G query heads of its kv head; a second kernel merges
// the splits.  bf16 caches run both products on the tensor cores
// (attn_tc_kernel, described where it is defined).  fp32 and int8 caches use
// attn_split_kernel, streaming K and V tiles through a cp.async ring.  A warp
// takes TB tokens at a time: each lane dots its D/32 elements of each key
// with the G query slices it holds, the G*TB partial sums are reduced
// together by a butterfly (each shuffle round halves the values a lane
// keeps), and the warp keeps its own running softmax and output (lane: its
// D/32 dims of every head).  Products run as packed fp32 pairs
// (fma.rn.f32x2).  The warps merge once per CTA, and the merge kernel
// combines the splits in a fixed order (running max and rescaled sums), so
// the result does not depend on timing.
// The CTA whose split holds `pos` writes the new token into the cache
// (converted to the cache type, int8 as the reference quantizes it) and
// patches the converted value into its own shared-memory tile.
#include <algorithm>
#include <atomic>

#include "gdn_internal.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

constexpr int AT = 256;  // threads per CTA (8 warps)

template <int CDT> struct Cache;
template <> struct Cache<KAI_GDN_F32> {
    using T = float;
    static __device__ __forceinline__ float get(T x) { return x; }
    static __device__ __forceinline__ T put(float x, float) { return x; }
};
template <> struct Cache<KAI_GDN_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float get(T x) { return __bfloat162float(x); }
    static __device__ __forceinline__ T put(float x, float) { return __float2bfloat16_rn(x); }
};
template <> struct Cache<KAI_GDN_I8> {
    using T = int8_t;
    static __device__ __forceinline__ float get(T x) { return (float)x; }
    // lroundf(x * (1 / scale)) clamped, as gdn_e2e_decode.c:1668-1684
    static __device__ __forceinline__ T put(float x, float inv) {
        long v = lroundf(__fmul_rn(x, inv));
        return (T)(v > 127 ? 127 : (v < -128 ? -128 : v));
    }
};

// E consecutive cache elements as E/2 fp32 pairs (bf16: the halves of each
// 32-bit word shifted into place; int8: exact through the exponent trick).
template <int CDT, int E> __device__ __forceinline__ void load_pairs(const typename Cache<CDT>::T *p, float2 *out) {
    using T = typename Cache<CDT>::T;
    constexpr int BYTES = E * (int)sizeof(T);
    static_assert(BYTES % 4 == 0 && BYTES <= 32, "row slice");
    uint32_t w[BYTES / 4];
    if constexpr (BYTES == 32) {
        const uint4 a = reinterpret_cast<const uint4 *>(p)[0], b = reinterpret_cast<const uint4 *>(p)[1];
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else if constexpr (BYTES == 16) {
        const uint4 a = reinterpret_cast<const uint4 *>(p)[0];
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w;
    } else if constexpr (BYTES == 8) {
        const uint2 a = reinterpret_cast<const uint2 *>(p)[0];
        w[0] = a.x, w[1] = a.y;
    } else {
        w[0] = reinterpret_cast<const uint32_t *>(p)[0];
    }
    if constexpr (CDT == KAI_GDN_F32) {
#pragma unroll
        for (int i = 0; i < E / 2; ++i) out[i] = make_float2(__uint_as_float(w[2 * i]), __uint_as_float(w[2 * i + 1]));
    } else if constexpr (CDT == KAI_GDN_BF16) {
#pragma unroll
        for (int i = 0; i < E / 2; ++i) out[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
        constexpr float kBias = 8388736.0f;  // 2^23 + 128: (b ^ 0x80) in the mantissa of 2^23, minus the bias
#pragma unroll
        for (int i = 0; i < E / 4; ++i) {
            const uint32_t u = w[i] ^ 0x80808080u;
            out[2 * i] = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - kBias,
                                     __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - kBias);
            out[2 * i + 1] = make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - kBias,
                                         __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - kBias);
        }
    }
}

// The warp total of NV values (NV a power of two, <= 32): in lane l, the total
// of value index l >> (5 - log2 NV).  NV - 1 + 5 - log2 NV shuffles.
template <int NV> __device__ __forceinline__ float warp_sum_many(float (&v)[NV], int lane) {
    constexpr int LG = NV >= 32 ? 5 : NV >= 16 ? 4 : NV >= 8 ? 3 : NV >= 4 ? 2 : NV >= 2 ? 1 : 0;
    static_assert((1 << LG) == NV, "power of two");
#pragma unroll
    for (int r = 0; r < LG; ++r) {
        const int half = NV >> (r + 1), mask = 16 >> r;
        const bool upper = lane & mask;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
        }
    }
    float x = v[0];
#pragma unroll
    for (int mask = 16 >> LG; mask >= 1; mask >>= 1) x += __shfl_xor_sync(0xffffffffu, x, mask);
    return x;
}

struct AttnP {
    const float *q, *k_new, *v_new;
    void *k_cache, *v_cache;
    const float *k_scale, *v_scale;
    float *o;      // final output (one split) ...
    float *part;   // ... or [B][Hkv][nsplit][G * (D + 2)] partials: m, l, acc
    long long H, Hkv, pos, max_ctx, ctx, split, nch;  // nch = splits per (b, kv head)
    float scale;
};

// The merge kernel is launched as a programmatic dependent of the split
// kernel: every split thread allows its launch at once, so at small batch
// (one wave of split CTAs) the merge's CTAs are placed while the splits run;
// the merge waits (griddepcontrol.wait) for the split grid to complete and
// its writes to be visible before it reads a partial.
__device__ __forceinline__ void allow_merge_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

constexpr int STAGE_BYTES = 32768;  // K and V of one tile
constexpr int NSTAGE = 3;

template <int D, int CDT> struct AttnGeo {
    using T = typename Cache<CDT>::T;
    static constexpr int ROW = D * (int)sizeof(T);           // bytes of one token's head slice
    static constexpr int TT = STAGE_BYTES / (2 * ROW);       // tokens per tile
    static constexpr int CPR = ROW / 16;                     // 16-byte copies per row
    static_assert(TT % 8 == 0, "tile");
};

__device__ __forceinline__ void cp16(void *dst, const void *src, bool full) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(full ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// CTA (split, kv head, batch): tokens [s0, s1) in tiles of TT, streamed
// through an NSTAGE-deep cp.async ring (rows past the end are zero-filled and
// masked).  Each warp takes TB tokens of a tile at a time and keeps its own
// running max, sum and output for the G query heads (lane: dims 8 lane ..
// 8 lane + 7 of every head); the only block barrier per tile hands the ring
// stage over, and the eight warps' states are merged once at the end.
template <int D, int G, int CDT>
__global__ void __launch_bounds__(AT, G == 8 ? 1 : 2) attn_split_kernel(AttnP p) {  // G = 8: 64 query regs
    allow_merge_launch();
    using C = Cache<CDT>;
    using Geo = AttnGeo<D, CDT>;
    using T = typename C::T;
    constexpr int E = D / 32, TT = Geo::TT, ROW = Geo::ROW, CPR = Geo::CPR;
    constexpr int TB = (TT / 8) * G <= 16 ? TT / 8 : 16 / G;  // tokens per warp step (<= 16 sums)
    constexpr int NV = G * TB;
    constexpr int LG = NV >= 32 ? 5 : NV >= 16 ? 4 : NV >= 8 ? 3 : NV >= 4 ? 2 : NV >= 2 ? 1 : 0;
    constexpr int SH = 5 - LG;
    extern __shared__ __align__(16) unsigned char dsm[];
    unsigned char *kt = dsm;                              // [NSTAGE][TT][ROW]
    unsigned char *vt = dsm + NSTAGE * TT * ROW;          // [NSTAGE][TT][ROW]
    float *red = reinterpret_cast<float *>(dsm);          // [8][G][D + 2] after the ring drains
    static_assert(8 * G * (D + 2) * 4 <= 2 * NSTAGE * TT * ROW, "red fits in the ring");
    struct WarpState {
        float m[G], l[G], a[G];
        float p[TB][G];
    };
    __shared__ WarpState ws[8];

    const int t = threadIdx.x, lane = t % 32, w = t / 32;
    const long long c = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const long long s0 = c * p.split, s1 = min(p.ctx, s0 + p.split);
    const int ntile = (int)((s1 - s0 + TT - 1) / TT);
    const long long kvd = p.Hkv * D;
    const size_t head0 = ((size_t)b * p.max_ctx * p.Hkv + kh) * D;  // token 0 of this (b, kv head)
    const T *kc = static_cast<const T *>(p.k_cache) + head0;
    const T *vc = static_cast<const T *>(p.v_cache) + head0;
    const float ks = CDT == KAI_GDN_I8 ? p.k_scale[b * p.Hkv + kh] : 1.0f;
    const float vs = CDT == KAI_GDN_I8 ? p.v_scale[b * p.Hkv + kh] : 1.0f;
    const bool has_new = p.pos >= s0 && p.pos < s1;

    // The new token goes to the cache; this CTA uses its converted value from
    // shared memory (patched into its tile), never reads it back.
    if (has_new) {
        const float ik = CDT == KAI_GDN_I8 ? 1.0f / ks : 1.0f, iv = CDT == KAI_GDN_I8 ? 1.0f / vs : 1.0f;
        T *kw = static_cast<T *>(p.k_cache) + head0 + p.pos * kvd;
        T *vw = static_cast<T *>(p.v_cache) + head0 + p.pos * kvd;
        for (int d = t; d < D; d += AT) {
            kw[d] = C::put(p.k_new[(b * p.Hkv + kh) * D + d], ik);
            vw[d] = C::put(p.v_new[(b * p.Hkv + kh) * D + d], iv);
        }
    }

    auto issue = [&](int tile) {
        if (tile < ntile) {
            const int st = tile % NSTAGE;
            const long long tb = s0 + (long long)tile * TT;
            for (int i = t; i < TT * CPR; i += AT) {
                const int r = i / CPR, cc = i % CPR;
                const long long tok = tb + r;
                const bool ok = tok < s1 && tok != p.pos;
                const long long src = (ok ? tok : 0) * kvd;
                cp16(kt + (st * TT + r) * ROW + cc * 16, reinterpret_cast<const unsigned char *>(kc + src) + cc * 16, ok);
                cp16(vt + (st * TT + r) * ROW + cc * 16, reinterpret_cast<const unsigned char *>(vc + src) + cc * 16, ok);
            }
        }
        cp_commit();
    };

    float2 qr[G][E / 2];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < E / 2; ++i)
            qr[g][i] = *reinterpret_cast<const float2 *>(p.q + ((b * p.H) + kh * G + g) * D + lane * E + 2 * i);
    const float sscale = CDT == KAI_GDN_I8 ? __fmul_rn(ks, p.scale) : p.scale;
    WarpState &my = ws[w];
    if (lane < G) {
        my.m[lane] = -INFINITY;
        my.l[lane] = 0.0f;
    }
    float2 acc[G][E / 2];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E / 2; ++e) acc[g][e] = make_float2(0.0f, 0.0f);

#pragma unroll
    for (int s = 0; s < NSTAGE - 1; ++s) issue(s);
    for (int tile = 0; tile < ntile; ++tile) {
        cp_wait<NSTAGE - 2>();
        const int st = tile % NSTAGE;
        const long long tb = s0 + (long long)tile * TT;
        const int n = (int)min((long long)TT, s1 - tb);
        __syncthreads();           // tile `tile` is in; every warp is done with tile - 1
        issue(tile + NSTAGE - 1);  // into the stage tile - 1 used
        // Patch the new token into its tile, after the barrier: each thread's
        // wait covers only its own copies, and the row's zero-fill may come
        // from another thread.
        if (has_new && p.pos >= tb && p.pos < tb + TT) {
            const int r = (int)(p.pos - tb);
            const float ik = CDT == KAI_GDN_I8 ? 1.0f / ks : 1.0f, iv = CDT == KAI_GDN_I8 ? 1.0f / vs : 1.0f;
            T *kr = reinterpret_cast<T *>(kt + (st * TT + r) * ROW), *vr = reinterpret_cast<T *>(vt + (st * TT + r) * ROW);
            for (int d = t; d < D; d += AT) {
                kr[d] = C::put(p.k_new[(b * p.Hkv + kh) * D + d], ik);
                vr[d] = C::put(p.v_new[(b * p.Hkv + kh) * D + d], iv);
            }
            __syncthreads();
        }

        for (int base = w * TB; base < n; base += 8 * TB) {
            float dots[NV];
            float2 vr[TB][E / 2];
#pragma unroll
            for (int i = 0; i < TB; ++i) {
                float2 kr[E / 2];
                load_pairs<CDT, E>(reinterpret_cast<const T *>(kt + (st * TT + base + i) * ROW) + lane * E, kr);
                load_pairs<CDT, E>(reinterpret_cast<const T *>(vt + (st * TT + base + i) * ROW) + lane * E, vr[i]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int e = 0; e < E / 2; ++e) s2 = __ffma2_rn(qr[g][e], kr[e], s2);
                    dots[g * TB + i] = s2.x + s2.y;
                }
            }
            const float tot = warp_sum_many<NV>(dots, lane);
            if ((lane & ((1 << SH) - 1)) == 0) {
                const int j = lane >> SH, g = j / TB, i = j % TB;
                my.p[i][g] = base + i < n ? tot * sscale : -INFINITY;
            }
            __syncwarp();
            if (lane < G) {  // running softmax of head `lane`
                float mt = -INFINITY;
#pragma unroll
                for (int i = 0; i < TB; ++i) mt = fmaxf(mt, my.p[i][lane]);
                const float m_old = my.m[lane], m_new = fmaxf(m_old, mt);
                float ps = 0.0f;
#pragma unroll
                for (int i = 0; i < TB; ++i) {
                    const float e = expf(my.p[i][lane] - m_new);
                    my.p[i][lane] = e;
                    ps += e;
                }
                const float a = expf(m_old - m_new);  // 0 on the first step
                my.a[lane] = a;
                my.l[lane] = fmaf(my.l[lane], a, ps);
                my.m[lane] = m_new;
            }
            __syncwarp();
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float2 a2 = make_float2(my.a[g], my.a[g]);
#pragma unroll
                for (int e = 0; e < E / 2; ++e) acc[g][e] = __fmul2_rn(acc[g][e], a2);
#pragma unroll
                for (int i = 0; i < TB; ++i) {
                    const float2 p2 = make_float2(my.p[i][g], my.p[i][g]);
#pragma unroll
                    for (int e = 0; e < E / 2; ++e) acc[g][e] = __ffma2_rn(p2, vr[i][e], acc[g][e]);
                }
            }
            __syncwarp();  // my.p is rewritten by the next step
        }
    }
    cp_wait<0>();
    __syncthreads();  // the ring is drained: red reuses it
    {
        float *r = red + w * G * (D + 2);
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int e = 0; e < E / 2; ++e)
                *reinterpret_cast<float2 *>(&r[g * (D + 2) + 2 + lane * E + 2 * e]) = acc[g][e];
            if (lane == 0) {
                r[g * (D + 2)] = my.m[g];
                r[g * (D + 2) + 1] = my.l[g];
            }
        }
    }
    __syncthreads();
    for (int i = t; i < G * D; i += AT) {
        const int g = i / D, d = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < 8; ++k) M = fmaxf(M, red[(k * G + g) * (D + 2)]);
        float L = 0.0f, v = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float* r = red + (k * G + g) * (D + 2);
            const float f = r[0] == -INFINITY ? 0.0f : expf(r[0] - M);  // a warp with no tokens
            L = fmaf(f, r[1], L);
            v = fmaf(f, r[2 + d], v);
        }
        if (p.nch == 1) {
            p.o[((b * p.H) + kh * G + g) * D + d] = v / L * vs;
        } else {
            float *rec = p.part + ((b * p.Hkv + kh) * p.nch + c) * (G * (D + 2)) + g * (D + 2);
            rec[2 + d] = v;
            if (d == 0) {
                rec[0] = M;
                rec[1] = L;
            }
        }
    }
}

// Merge the chunks of one (b, query head): o = sum_c e^(m_c - M) acc_c /
// sum_c e^(m_c - M) l_c (times the int8 value scale).  Warp w folds chunks
// w, w + 8, ... into a running (max, sum, output) of its own, rescaling by
// e^(m_old - m_new) as the maximum grows, with the records of CU chunks in
// flight at once; the eight warps' states are merged in warp order at the
// end.  No step waits on a whole-block quantity before the loads are issued,
// so a merge of many chunks costs about one round of loads.
template <int D, int G>
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnP p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the split kernel has completed
    constexpr int NW = 8, J = D / 64, CU = 4;  // J float2 per lane and chunk
    __shared__ float s_m[NW], s_l[NW], s_acc[NW][D];
    const long long h = blockIdx.x, b = blockIdx.y, kh = h / G;
    const int g = (int)(h % G), lane = threadIdx.x % 32, w = threadIdx.x / 32, nch = (int)p.nch;
    const float *rec = p.part + ((b * p.Hkv + kh) * p.nch) * (G * (D + 2)) + g * (D + 2);
    const long long stride = G * (D + 2);
    float m = -INFINITY, l = 0.0f;
    float2 acc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) acc[j] = make_float2(0.0f, 0.0f);
    for (int c0 = w; c0 < nch; c0 += NW * CU) {
        float mc[CU], lc[CU];
        float2 ac[CU][J];
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            const int c = c0 + u * NW;
            if (c < nch) {
                const float *r = rec + c * stride;
                mc[u] = r[0];
                lc[u] = r[1];
#pragma unroll
                for (int j = 0; j < J; ++j) ac[u][j] = *reinterpret_cast<const float2 *>(r + 2 + 64 * j + 2 * lane);
            }
        }
#pragma unroll
        for (int u = 0; u < CU; ++u) {
            if (c0 + u * NW < nch) {  // every chunk holds a token: mc is finite
                const float mn = fmaxf(m, mc[u]);
                const float a = expf(m - mn), f = expf(mc[u] - mn);  // a = 0 on the first chunk
                l = fmaf(lc[u], f, l * a);
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    acc[j].x = fmaf(ac[u][j].x, f, acc[j].x * a);
                    acc[j].y = fmaf(ac[u][j].y, f, acc[j].y * a);
                }
                m = mn;
            }
        }
    }
    if (lane == 0) {
        s_m[w] = m;
        s_l[w] = l;
    }
#pragma unroll
    for (int j = 0; j < J; ++j) *reinterpret_cast<float2 *>(&s_acc[w][64 * j + 2 * lane]) = acc[j];
    __syncthreads();
    const int d = threadIdx.x;
    if (d >= D) return;
    float M = s_m[0];
#pragma unroll
    for (int ww = 1; ww < NW; ++ww) M = fmaxf(M, s_m[ww]);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int ww = 0; ww < NW; ++ww) {
        if (ww < nch) {  // warps without a chunk hold no state
            const float f = expf(s_m[ww] - M);
            L = fmaf(s_l[ww], f, L);
            o = fmaf(s_acc[ww][d], f, o);
        }
    }
    const float vs = p.v_scale ? p.v_scale[b * p.Hkv + kh] : 1.0f;
    p.o[(b * p.H + h) * D + d] = o / L * vs;
}

// ------------------------------------------ tensor-core split kernel (bf16)
// A bf16 cache takes both products through tcgen05, per tile of TC_TT = 48
// tokens of one (b, kv head):
//   S  = K Qs^T     M = 64 rows (the 48 tokens; rows 48-63 read the next
//                   block's bytes and are masked), N = NQ, K = D.  A: the K
//                   tile; B: the G
//                   query heads split into three bf16 terms (hi + mid + lo =
//                   the fp32 q to 24 bits), rows t*G + h, zero rows after.
//   O^T = V^T Ps^T  M = 128 head dims (D/128 MMAs), N = NQ, K = 48 tokens.
//                   A: the V tile; B: the softmax weights in three terms.
// Every product is exact in fp32 and summed in fp32: scores and outputs keep
// fp32 accuracy.  K and V tiles arrive by TMA in the 128-byte-swizzle layout
// of tma.cuh: features 64j .. 64j+63 in a 6 KB block at 6144j, token row t
// at t*128 with its 16-byte chunks permuted by chunk ^= t % 8.  The S MMA
// reads the K tile as K-major (a K step of 16 features: +32 bytes inside a
// block), the O MMA the V tile as MN-major (next 64 features: the next block,
// LBO 6144; next 8 tokens: SBO 1024).  A 4-stage ring; 128-byte rows per box
// keep the copy engine's requests large (16-byte rows ran at half the rate).
// Measured at B = 16 over 32k tokens: 48-token tiles in 4 stages beat 64 in
// 3 (381 vs 420 us) and 32 in 6 (523 us).
//
// Warp specialised.  Warp 8 issues, per tile j: S(j+1) once its tile has
// landed, the load of tile j+3 into the stage O(j-1) has released, then O(j)
// once the weights of tile j are written.  Warps 0-7, per tile j: wait for
// S(j); warps 0-2 (rows 16w .. 16w+15 of the M = 64 accumulator, lanes
// 0-15) turn it into scores and the tile maximum; after one barrier of the
// eight warps every thread knows the running maximum; every thread folds
// O(j-2) from TMEM into its registers (one head dim, all G heads; issued two
// tiles earlier, so it has long finished); the softmax threads write the
// weights of tile j and all arrive on the weights-ready barrier.  S, O and
// the weights are double-buffered.  Waits are bounded: a timeout sets the
// library's error word and the CTA stops, frees its TMEM and exits.
constexpr int TC_TT = 48;
constexpr int TC_AT = 288;  // 8 softmax / fold warps + 1 issuing warp
template <int D, int G> struct TcAttnGeo {
    static constexpr int NQ = (3 * G + 15) / 16 * 16;  // MMA N: three terms of G heads, padded
    static constexpr int BOX = TC_TT * 128;             // bytes of one 64-feature box
    static constexpr int KT = TC_TT * D * 2;            // bytes of a K (or V) tile
    static constexpr int STAGE = 2 * KT;
    static constexpr int NST = 4;
    static constexpr int QOP = NQ * D * 2;              // Qs, K-major NQ x D
    static constexpr int POP = NQ * TC_TT * 2;          // Ps, K-major NQ x TC_TT
    static constexpr int S_COL = 0, O_COL = 2 * NQ;     // TMEM: S buffers, then O buffers
    static constexpr int OCOLS = (D / 128) * NQ;        // one O buffer
    static constexpr int NCOL = O_COL + 2 * OCOLS;
    static constexpr uint32_t TMEM_COLS = NCOL <= 32 ? 32 : NCOL <= 64 ? 64 : NCOL <= 128 ? 128 : 256;
    static constexpr size_t SMEM = (size_t)NST * STAGE + QOP + 2 * (size_t)POP + 1024;
    static_assert(NCOL <= 256 && SMEM <= 227 * 1024, "fits one SM");
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
// The three bf16 terms of x (hi + mid + lo, 24 significant bits).
__device__ __forceinline__ void split3(float x, float &hi, float &mid, float &lo) {
    hi = __bfloat162float(__float2bfloat16_rn(x));
    const float r = x - hi;
    mid = __bfloat162float(__float2bfloat16_rn(r));
    lo = r - mid;
}
// Barrier 1 over the 256 threads of warps 0-7, OR-reducing a flag.
__device__ __forceinline__ bool compute_sync_or(bool v) {
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
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(umma::smem_addr(bar)) : "memory");
}

template <int D, int G>
__global__ void __launch_bounds__(TC_AT, 1)
    attn_tc_kernel(AttnP p, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   int *err) {
    allow_merge_launch();
    using namespace umma;
    using Gm = TcAttnGeo<D, G>;
    using T = __nv_bfloat16;
    constexpr int TT = TC_TT, NQ = Gm::NQ, NH = D / 128, NST = Gm::NST;
    extern __shared__ unsigned char dsm_raw[];
    unsigned char *dsm = dsm_raw + ((1024u - (smem_addr(dsm_raw) & 1023u)) & 1023u);
    unsigned char *ring = dsm;                            // [NST][K tile | V tile]
    unsigned char *qop = ring + NST * Gm::STAGE;          // Qs
    unsigned char *pop = qop + Gm::QOP;                   // [2] Ps
    __shared__ uint64_t full[NST], bar_s[2], bar_o[2], pready[2];
    __shared__ uint32_t tmem_slot;
    __shared__ float s_red[2][4][G];

    const int t = threadIdx.x, lane = t % 32, w = t / 32;
    const long long c = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
    const long long s0 = c * p.split, s1 = min(p.ctx, s0 + p.split);
    const int ntile = (int)((s1 - s0 + TT - 1) / TT);
    const long long kvd = p.Hkv * D;
    const size_t head0 = ((size_t)b * p.max_ctx * p.Hkv + kh) * D;
    const bool has_new = p.pos >= s0 && p.pos < s1;
    const float *knew = p.k_new + (b * p.Hkv + kh) * D, *vnew = p.v_new + (b * p.Hkv + kh) * D;

    if (w < 8) {
        if (has_new) {  // the new token goes to the cache; the issuing warp patches it into its tile
            T *kw = static_cast<T *>(p.k_cache) + head0 + p.pos * kvd;
            T *vw = static_cast<T *>(p.v_cache) + head0 + p.pos * kvd;
            for (int d = t; d < D; d += 256) {
                kw[d] = __float2bfloat16_rn(knew[d]);
                vw[d] = __float2bfloat16_rn(vnew[d]);
            }
        }
        // Qs (rows t*G + h; rows >= 3G zero) and zeroed Ps buffers
        const float *qg = p.q + (b * p.H + kh * G) * D;
        for (int i = t; i < NQ * (D / 2); i += 256) {
            const int n = i / (D / 2), k = 2 * (i % (D / 2));
            float v0 = 0.0f, v1 = 0.0f;
            if (n < 3 * G) {
                const int term = n / G, h = n % G;
                float hi, mid, lo;
                split3(qg[h * D + k], hi, mid, lo);
                v0 = term == 0 ? hi : term == 1 ? mid : lo;
                split3(qg[h * D + k + 1], hi, mid, lo);
                v1 = term == 0 ? hi : term == 1 ? mid : lo;
            }
            *reinterpret_cast<uint32_t *>(qop + kmaj16(n, k, D)) = pack_bf16x2(v0, v1);
        }
        for (int i = t; i < 2 * Gm::POP / 16; i += 256) reinterpret_cast<uint4 *>(pop)[i] = make_uint4(0, 0, 0, 0);
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
            // the first tiles load while the other warps build the query operand
            for (int s = 0; s < NST && s < ntile; ++s) {
                mbar_arrive_expect_tx(&full[s], 2 * Gm::KT);
                const int t0 = (int)(s0 + (long long)s * TT);
                tma::load_chunk_sw128(ring + s * Gm::STAGE, &kmap, t0, (int)kh, (int)b, &full[s], D / 64, Gm::BOX);
                tma::load_chunk_sw128(ring + s * Gm::STAGE + Gm::KT, &vmap, t0, (int)kh, (int)b, &full[s], D / 64,
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
        int nload = 0, nlanded = 0;  // tiles whose loads were issued / seen landed
        auto load = [&](int tile) {  // elected lane
            const int st = tile % NST;
            unsigned char *kt = ring + st * Gm::STAGE;
            mbar_arrive_expect_tx(&full[st], 2 * Gm::KT);
            const int t0 = (int)(s0 + (long long)tile * TT);
            tma::load_chunk_sw128(kt, &kmap, t0, (int)kh, (int)b, &full[st], D / 64, Gm::BOX);
            tma::load_chunk_sw128(kt + Gm::KT, &vmap, t0, (int)kh, (int)b, &full[st], D / 64, Gm::BOX);
        };
        // Wait for tile `tile`, patch the new token in, issue its S MMAs.
        auto issue_s = [&](int tile) -> bool {
            const int st = tile % NST;
            if (!__all_sync(0xffffffffu, mbar_wait(&full[st], (tile / NST) & 1, err))) return false;
            nlanded = tile + 1;
            unsigned char *kt = ring + st * Gm::STAGE;
            const long long tb = s0 + (long long)tile * TT;
            if (has_new && p.pos >= tb && p.pos < tb + TT) {
                const int r = (int)(p.pos - tb);
                for (int d = lane; d < D; d += 32) {
                    const uint32_t off =
                        (uint32_t)((d >> 6) * Gm::BOX + r * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2);
                    *reinterpret_cast<T *>(kt + off) = __float2bfloat16_rn(knew[d]);
                    *reinterpret_cast<T *>(kt + Gm::KT + off) = __float2bfloat16_rn(vnew[d]);
                }
                fence_smem_to_async();
                __syncwarp();
            }
            if (elect_one()) {
                const uint32_t ka = smem_addr(kt);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks)
                    mma_f16(tmem + Gm::S_COL + (tile & 1) * NQ, smem_desc_sw128(ka + (ks / 4) * Gm::BOX + (ks % 4) * 32, 16, 1024),
                            desc_kmaj16(qop, D, ks), id_s, ks > 0);
                commit(&bar_s[tile & 1]);
            }
            __syncwarp();
            return true;
        };
        nload = min(NST, ntile);  // issued before the set-up barrier
        bad = !issue_s(0);
        for (int j = 0; j < ntile && !bad; ++j) {
            if (j + 1 < ntile && !issue_s(j + 1)) {
                bad = true;
                break;
            }
            if (j >= 1 && j + NST - 1 < ntile) {  // O(j-1) has released its stage: tile j+NST-1 goes there
                if (!__all_sync(0xffffffffu, mbar_wait(&bar_o[(j - 1) & 1], ((j - 1) >> 1) & 1, err))) {
                    bad = true;
                    break;
                }
                if (elect_one()) load(j + NST - 1);
                __syncwarp();
                nload = j + NST;
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
                        mma_f16(tmem + Gm::O_COL + (j & 1) * Gm::OCOLS + h2 * NQ,
                                smem_desc_sw128(va + h2 * 2 * Gm::BOX + ks * 2048, Gm::BOX, 1024), desc_kmaj16(pb, TT, ks),
                                id_o,
                                ks > 0);
                commit(&bar_o[j & 1]);
            }
            __syncwarp();
        }
        // After a timeout: let the loads still in flight land before the CTA exits.
        for (int k = nlanded; k < nload; ++k) mbar_wait(&full[k % NST], (k / NST) & 1, nullptr, 1u << 16);
    } else {
        // ---------------------------------------------- softmax / fold warps
        float m_run[G], a_even[G], a_odd[G], l_part[G], acc[G];  // a_*: rescale factors of even / odd tiles
#pragma unroll
        for (int h = 0; h < G; ++h) {
            m_run[h] = -INFINITY;
            a_even[h] = a_odd[h] = 0.0f;
            l_part[h] = 0.0f;
            acc[h] = 0.0f;
        }
        const int hm = w / 4;  // O half of this thread: head dim 128 hm + 32 (w % 4) + lane
        const bool o_warp = hm < NH;
        const int srow = 16 * w + lane;  // softmax row (token) of warps 0-3, lanes 0-15
        const bool s_thread = w < 4 && lane < 16;
        // fold O(k) (TMEM buffer k & 1) with its factor: acc = acc * a_k + O_k
        auto fold = [&](int k) -> bool {
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar_o[k & 1], (k >> 1) & 1, err));
            fence_after_sync();
            if (!ok) return false;
            if (o_warp) {
                float ov[NQ];
#pragma unroll
                for (int q = 0; q < NQ; q += 16)
                    tmem_ld16(taddr(tmem, 32 * (w % 4), Gm::O_COL + (k & 1) * Gm::OCOLS + hm * NQ + q),
                              *reinterpret_cast<float(*)[16]>(ov + q));
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < NQ; q += 16) reg_fence16(ov + q);
#pragma unroll
                for (int h = 0; h < G; ++h)
                    acc[h] = fmaf(acc[h], (k & 1) ? a_odd[h] : a_even[h], (ov[h] + ov[G + h]) + ov[2 * G + h]);
            }
            return true;
        };
        for (int j = 0; j < ntile; ++j) {
            const long long tb = s0 + (long long)j * TT;
            if (!mbar_wait(&bar_s[j & 1], (j >> 1) & 1, err)) bad = true;
            fence_after_sync();
            bad = __any_sync(0xffffffffu, bad);  // TMEM loads are warp-wide
            const bool valid = s_thread && srow < TT && tb + srow < s1;  // S rows past TT: the next block's bytes
            float sc[G];
            if (w < 4 && !bad) {
                float sv[NQ];
#pragma unroll
                for (int q = 0; q < NQ; q += 16)
                    tmem_ld16(taddr(tmem, 32 * w, Gm::S_COL + (j & 1) * NQ + q),
                              *reinterpret_cast<float(*)[16]>(sv + q));
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < NQ; q += 16) reg_fence16(sv + q);
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    sc[h] = valid ? ((sv[h] + sv[G + h]) + sv[2 * G + h]) * p.scale : -INFINITY;
                    float mx = sc[h];
#pragma unroll
                    for (int mask = 16; mask >= 1; mask >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, mask));
                    if (lane == 0) s_red[j & 1][w][h] = mx;
                }
            }
            if (compute_sync_or(bad)) {
                bad = true;
                break;
            }
            float a[G];
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float mt = fmaxf(fmaxf(s_red[j & 1][0][h], s_red[j & 1][1][h]),
                                       fmaxf(s_red[j & 1][2][h], s_red[j & 1][3][h]));
                const float mn = fmaxf(m_run[h], mt);  // finite: every tile holds a token
                a[h] = expf(m_run[h] - mn);            // 0 on the first tile
                m_run[h] = mn;
            }
            if (j >= 2 && !fold(j - 2)) bad = true;  // also frees the weights buffer j & 1
#pragma unroll
            for (int h = 0; h < G; ++h) {
                if (j & 1)
                    a_odd[h] = a[h];
                else
                    a_even[h] = a[h];
            }
            if (s_thread && srow < TT && !bad) {
                unsigned char *pb = pop + (j & 1) * Gm::POP;
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float e = valid ? expf(sc[h] - m_run[h]) : 0.0f;
                    l_part[h] = fmaf(l_part[h], a[h], e);
                    float hi, mid, lo;
                    split3(e, hi, mid, lo);
                    *reinterpret_cast<T *>(pb + kmaj16(h, srow, TT)) = __float2bfloat16_rn(hi);
                    *reinterpret_cast<T *>(pb + kmaj16(G + h, srow, TT)) = __float2bfloat16_rn(mid);
                    *reinterpret_cast<T *>(pb + kmaj16(2 * G + h, srow, TT)) = __float2bfloat16_rn(lo);
                }
            }
            fence_smem_to_async();
            fence_before_sync();
            mbar_arrive(&pready[j & 1]);
        }
        if (!bad) {
            for (int k = ntile >= 2 ? ntile - 2 : 0; k < ntile; ++k)
                if (!fold(k)) bad = true;
        }
        bad = compute_sync_or(bad);
        if (!bad) {
            if (w < 4) {  // sums of the softmax weights
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    float l = l_part[h];
#pragma unroll
                    for (int mask = 16; mask >= 1; mask >>= 1) l += __shfl_xor_sync(0xffffffffu, l, mask);
                    if (lane == 0) s_red[0][w][h] = l;
                }
            }
            compute_sync_or(false);
            if (o_warp) {
                const int d = 128 * hm + 32 * (w % 4) + lane;
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float L = (s_red[0][0][h] + s_red[0][1][h]) + (s_red[0][2][h] + s_red[0][3][h]);
                    if (p.nch == 1) {
                        p.o[((b * p.H) + kh * G + h) * D + d] = acc[h] / L;
                    } else {
                        float *rec = p.part + ((b * p.Hkv + kh) * p.nch + c) * (G * (D + 2)) + h * (D + 2);
                        rec[2 + d] = acc[h];
                        if (d == 0) {
                            rec[0] = m_run[h];
                            rec[1] = L;
                        }
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (w == 8) tmem_dealloc(tmem, Gm::TMEM_COLS);
}

// Splits per (b, kv head).  The split kernel runs in waves of `slots`
// resident CTAs, and a CTA's time goes with its tiles, so the launch takes
// about waves x (tiles per CTA + RAMP), RAMP standing for a CTA's start-up
// (first loads, final merge) in tiles.  The smallest such cost wins, the
// fewest splits on a tie; a count just above a multiple of the slots (a
// nearly empty last wave of full-length CTAs) is what this avoids.
long long choose_splits(long long pairs, long long tiles, long long slots) {
    constexpr long long RAMP = 2;
    const long long max_n = std::min(tiles, std::max(1ll, 4 * ((slots + pairs - 1) / pairs)));
    long long best = 1, best_cost = -1;
    for (long long n = 1; n <= max_n; ++n) {
        const long long per = (tiles + n - 1) / n;
        const long long nch = (tiles + per - 1) / per;  // splits in whole tiles
        if (nch != n) continue;
        const long long cost = ((pairs * nch + slots - 1) / slots) * (per + RAMP);
        if (best_cost < 0 || cost < best_cost) {
            best = nch;
            best_cost = cost;
        }
    }
    return best;
}

// bf16 caches take the tensor-core split kernel, fp32 and int8 caches the
// CUDA-core one.
template <int D, int G, int CDT>
int run_attn(AttnP p, long long B, cudaStream_t st) {
    constexpr bool TC = CDT == KAI_GDN_BF16;
    using Geo = AttnGeo<D, CDT>;
    constexpr int TT = TC ? TC_TT : Geo::TT;
    const size_t smem = TC ? TcAttnGeo<D, G>::SMEM : 2ull * NSTAGE * Geo::TT * Geo::ROW;
    const void *kern;
    if constexpr (TC)
        kern = reinterpret_cast<const void *>(attn_tc_kernel<D, G>);
    else
        kern = reinterpret_cast<const void *>(attn_split_kernel<D, G, CDT>);
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "attention_decode: cudaGetDevice");
    if (rc) return rc;
    static std::atomic<unsigned long long> attr_set{0};  // per device
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "attention_decode: smem attribute");
        if (rc) return rc;
        attr_set.fetch_or(bit);
    }
    static std::atomic<int> per_sm[64];  // resident split CTAs per SM, per device (0: not asked yet)
    int nb = per_sm[dev & 63].load();
    if (nb == 0) {
        rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, TC ? TC_AT : AT, smem),
                        "attention_decode: occupancy");
        if (rc) return rc;
        nb = std::max(nb, 1);
        per_sm[dev & 63].store(nb);
    }
    const long long pairs = B * p.Hkv, tiles = (p.ctx + TT - 1) / TT;
    const long long nsplit = choose_splits(pairs, tiles, (long long)nb * sm_count());
    const long long per = (tiles + nsplit - 1) / nsplit;
    p.split = per * TT;
    p.nch = (p.ctx + p.split - 1) / p.split;
    if (p.nch > 1) {
        void *scr = nullptr;
        rc = scratch_for_stream(st, (size_t)pairs * p.nch * G * (D + 2) * sizeof(float), &scr);
        if (rc) return rc;
        p.part = static_cast<float *>(scr);
    }
    if (p.nch > 0x7fffffffll || p.Hkv > 65535 || B > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_decode: shape too large");
    const dim3 grid((unsigned)p.nch, (unsigned)p.Hkv, (unsigned)B);
    if constexpr (TC) {
        int *err = nullptr;
        if ((rc = device_error_word(&err))) return rc;
        CUtensorMap kmap, vmap;
        if (tma::make_chunk_map(&kmap, p.k_cache, true, (uint64_t)B, (uint64_t)p.max_ctx, (uint64_t)p.Hkv, D, true,
                                TC_TT) ||
            tma::make_chunk_map(&vmap, p.v_cache, true, (uint64_t)B, (uint64_t)p.max_ctx, (uint64_t)p.Hkv, D, true,
                                TC_TT))
            return set_error(KAI_GDN_ERR_CUDA, "attention_decode: tensor map encoding failed");
        attn_tc_kernel<D, G><<<grid, TC_AT, smem, st>>>(p, kmap, vmap, err);
    } else {
        attn_split_kernel<D, G, CDT><<<grid, AT, smem, st>>>(p);
    }
    rc = check_launch("attention split kernel");
    if (rc || p.nch == 1) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.H, (unsigned)B);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, attn_combine_kernel<D, G>, p);
    if (le != cudaSuccess) return check_cuda(le, "attn_combine_kernel launch");
    return check_launch("attn_combine_kernel");
}

template <int D, int CDT> int dispatch_g(AttnP p, long long B, long long G, cudaStream_t st) {
    switch (G) {
        case 1: return run_attn<D, 1, CDT>(p, B, st);
        case 2: return run_attn<D, 2, CDT>(p, B, st);
        case 4: return run_attn<D, 4, CDT>(p, B, st);
        default: return run_attn<D, 8, CDT>(p, B, st);
    }
}
template <int D> int dispatch_dt(AttnP p, long long B, long long G, int dt, cudaStream_t st) {
    switch (dt) {
        case KAI_GDN_F32: return dispatch_g<D, KAI_GDN_F32>(p, B, G, st);
        case KAI_GDN_BF16: return dispatch_g<D, KAI_GDN_BF16>(p, B, G, st);
        default: return dispatch_g<D, KAI_GDN_I8>(p, B, G, st);
    }
}

}  // namespace

int launch_attn_decode(const kai_gdn_attn_decode_args *a, cudaStream_t st) {
    if (!a) return set_error(KAI_GDN_ERR_INVALID, "attention_decode: null args");
    if (a->batch == 0 || a->heads == 0) return KAI_GDN_OK;
    if (!a->q || !a->k_new || !a->v_new || !a->k_cache || !a->v_cache || !a->o)
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: null pointer");
    if (a->kv_heads == 0 || a->heads % a->kv_heads)
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: heads %zu not a multiple of kv_heads %zu", a->heads,
                         a->kv_heads);
    const size_t G = a->heads / a->kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_decode: %zu query heads per kv head (1, 2, 4, 8)", G);
    if (a->head_dim != 128 && a->head_dim != 256)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_decode: head_dim %zu (128, 256)", a->head_dim);
    if (a->pos >= a->max_ctx)
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: pos %zu outside the cache (%zu)", a->pos, a->max_ctx);
    const int dt = a->cache_dtype;
    if (dt != KAI_GDN_F32 && dt != KAI_GDN_BF16 && dt != KAI_GDN_I8)
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: cache dtype %d", dt);
    if (dt == KAI_GDN_I8 && (!a->k_scale || !a->v_scale))
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: int8 cache needs k_scale and v_scale");
    const size_t esz = dt == KAI_GDN_F32 ? 4 : dt == KAI_GDN_BF16 ? 2 : 1;
    if ((uintptr_t)a->k_cache % 16 || (uintptr_t)a->v_cache % 16 || (uintptr_t)a->q % 16 ||
        (uintptr_t)a->k_new % 4 || (uintptr_t)a->v_new % 4 || (uintptr_t)a->o % 4)
        return set_error(KAI_GDN_ERR_INVALID, "attention_decode: caches and q must be 16-byte aligned");
    (void)esz;

    AttnP p{};
    p.q = a->q;
    p.k_new = a->k_new;
    p.v_new = a->v_new;
    p.k_cache = a->k_cache;
    p.v_cache = a->v_cache;
    p.k_scale = dt == KAI_GDN_I8 ? a->k_scale : nullptr;
    p.v_scale = dt == KAI_GDN_I8 ? a->v_scale : nullptr;
    p.o = a->o;
    p.H = (long long)a->heads;
    p.Hkv = (long long)a->kv_heads;
    p.pos = (long long)a->pos;
    p.max_ctx = (long long)a->max_ctx;
    p.ctx = p.pos + 1;
    p.scale = a->scale;
    const long long B = (long long)a->batch;
    if (a->head_dim == 128) return dispatch_dt<128>(p, B, (long long)G, dt, st);
    return dispatch_dt<256>(p, B, (long long)G, dt, st);
}

}  // namespace gdn
