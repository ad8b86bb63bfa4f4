// attn.cu -- grouped-query attention decode over a growing KV cache: one new
// token per sequence attends to every cached token of its kv head.
//   full_attn_real_forward        src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:1532-1634
//   full_attn_real_forward_int8kv gdn_e2e_decode.c:1652-1830 (int8 cache, one scale per kv head)
// and a bf16 cache (not in the reference), round-to-nearest-even on append.
// Cache layout as the reference's: [batch][max_ctx][kv_heads][head_dim].
//
// Split over the context (flash decoding): CTA (split, kv head, batch) takes a
// run of tokens and the G query heads of its kv head, streaming K and V tiles
// through a cp.async ring.  A warp takes TB tokens at a time: each lane dots
// its D/32 elements of each key with the G query slices it holds, the G*TB
// partial sums are reduced together by a butterfly (each shuffle round halves
// the values a lane keeps), and the warp keeps its own running softmax and
// output (lane: its D/32 dims of every head).  Products run as packed fp32
// pairs (fma.rn.f32x2).  The warps merge once per CTA, and a second kernel
// merges the splits in order (running max and rescaled sums), so the result
// does not depend on timing.
// The chunk that holds `pos` first writes the new token into the cache
// (converted to the cache type, int8 as the reference quantizes it) and reads
// it back after a barrier with ordinary loads.
#include <algorithm>
#include <atomic>

#include "gdn_internal.cuh"

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

template <int D, int G, int CDT>
int run_attn(AttnP p, long long B, cudaStream_t st) {
    using Geo = AttnGeo<D, CDT>;
    const size_t smem = 2ull * NSTAGE * Geo::TT * Geo::ROW;
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "attention_decode: cudaGetDevice");
    if (rc) return rc;
    static std::atomic<unsigned long long> attr_set{0};  // per device
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        rc = check_cuda(cudaFuncSetAttribute(attn_split_kernel<D, G, CDT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem),
                        "attention_decode: smem attribute");
        if (rc) return rc;
        attr_set.fetch_or(bit);
    }
    static std::atomic<int> per_sm[64];  // resident split CTAs per SM, per device (0: not asked yet)
    int nb = per_sm[dev & 63].load();
    if (nb == 0) {
        rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, attn_split_kernel<D, G, CDT>, AT, smem),
                        "attention_decode: occupancy");
        if (rc) return rc;
        nb = std::max(nb, 1);
        per_sm[dev & 63].store(nb);
    }
    const long long pairs = B * p.Hkv, tiles = (p.ctx + Geo::TT - 1) / Geo::TT;
    const long long nsplit = choose_splits(pairs, tiles, (long long)nb * sm_count());
    const long long per = (tiles + nsplit - 1) / nsplit;
    p.split = per * Geo::TT;
    p.nch = (p.ctx + p.split - 1) / p.split;
    if (p.nch > 1) {
        void *scr = nullptr;
        rc = scratch_for_stream(st, (size_t)pairs * p.nch * G * (D + 2) * sizeof(float), &scr);
        if (rc) return rc;
        p.part = static_cast<float *>(scr);
    }
    if (p.nch > 0x7fffffffll || p.Hkv > 65535 || B > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "attention_decode: shape too large");
    attn_split_kernel<D, G, CDT><<<dim3((unsigned)p.nch, (unsigned)p.Hkv, (unsigned)B), AT, smem, st>>>(p);
    rc = check_launch("attn_split_kernel");
    if (rc || p.nch == 1) return rc;
    attn_combine_kernel<D, G><<<dim3((unsigned)p.H, (unsigned)B), 256, 0, st>>>(p);
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
