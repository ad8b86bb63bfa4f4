// chunk_ws.cu -- warp-specialised chunkwise (WY / UT-transform) gated
// delta-rule scan on the sm_100a tensor cores, for bf16 / fp16 q, k, v with
// fp32 state and accumulation, dk = dv = 128, chunk C = 64.
//
// Math (docs/GDN_ARCHITECTURE_AUDIT.md:142-153; the chunked form of
// gpu/gdn_gpu_validate.c:100-118).  Per (b, value head h), chunk of 64 tokens,
// G = in-chunk cumulative log decay, gamma = exp(G_63):
//   A   = beta_r (k_r.k_s) exp(G_r - G_s), s <  r
//   P   = scale (q_r.k_s) exp(G_r - G_s), s <= r
//   T   = (I + A)^-1,  Tb = T diag(beta)
//   V'  = Tb (V - exp(G) (K S))             (= U - W S of the WY form)
//   O   = scale exp(G) (Q S) + P V'
//   S  <- gamma S + (K exp(G_63 - G))^T V'
// Everything except the last three lines is independent of the state, so it
// runs one chunk AHEAD of the recurrence, in three warp groups:
//   key group    (warps 0-7):   TMA loads, [K;Q] K^T, A and P, the inverse,
//                               Tb;
//   state group  (warps 8-11):  the recurrence, with the state held TRANSPOSED
//                               in TMEM (lane = value index i, column = key
//                               index j), so every state-side MMA has M = 128
//                               and reads the 16-bit state copy from TMEM:
//     M3a  [(K S)^T | X^T] = S^T [K; Q]^T    one N = 128 chain, A: S^T
//                                            (TMEM), B: the [K;Q] tile
//     M3b  V'^T      = V^T Tb^T - ((K S)^T exp(G)) Tb^T
//     M4   S^T      += (V' exp(G_63 - G))^T K,   Y^T = V'^T P^T
//   output group (warps 12-15): O = scale exp(G_r) X + Y from TMEM to global
//                               memory, off the recurrence's critical path;
//                               warp 12 also computes every chunk's gate
//                               factors three chunks ahead.
// The groups hand chunks over through mbarriers (key_ready / key_free,
// o_full / o_empty); q, k, v arrive by TMA into a three-deep ring, the
// key-side tiles are double buffered.  Every MMA is issued by one elected
// lane of a converged warp.  One CTA (512 threads, ~225 KB of shared
// memory, all 512 TMEM columns) per (b, h); every wait is bounded (a timeout
// sets *err and all groups leave after their outstanding copies and MMAs have
// completed).
//
// TMEM columns (fp32 unless noted; "16-bit" = two values per column):
//   [  0,128) S^T                 [128,192) S^T 16-bit (A operand)
//   [192,256) (K S)^T, then V'^T, then Y^T     [256,320) X^T (M3a writes
//             (K S)^T and X^T at once)
//   [320,352) -(K S)^T exp(G) 16-bit, then V'^T 16-bit    [352,384) V''^T 16-bit
//   [384,448) [K;Q] K^T  (lanes 0-63: K K^T, 64-127: Q K^T)
// Shared memory: per input stage K and Q interleaved by 64-feature block
// ([K blk0 | Q blk0 | K blk1 | Q blk1], 128-byte swizzle, so [K;Q] is one
// M = 128 operand) and V (128-byte swizzle); per key stage P and Tb (no
// swizzle, K-major) and the gate factors; the fp32 inverse workspace.
#include "gdn_internal.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace gdn {
namespace {

using namespace umma;

constexpr int C = 64, D = 128;
constexpr int KG = 256, SG = 128, OG = 128, NT = KG + SG + OG;
constexpr int NS_IN = 3, NS_K = 2;

constexpr uint32_t COL_ST = 0, COL_SB = 128, COL_VA = 192, COL_OA = 256, COL_KSB = 320, COL_VB = 320,
                   COL_VB2 = 352, COL_KQ = 384;
static_assert(COL_OA == COL_VA + 64, "M3a writes (K S)^T and O^T as one N = 128 accumulator");

// Block-packed lower triangle of a 64 x 64 fp32 matrix: the ten 16 x 16
// blocks (bi >= bj) at id = bi(bi+1)/2 + bj, rows padded to 20 floats.
constexpr int BLD = 20, BSZ = 16 * BLD;
__host__ __device__ constexpr int blk(int bi, int bj) { return (bi * (bi + 1) / 2 + bj) * BSZ; }

struct InStage {
    unsigned char KQ[4 * 8192];  // [K d0-63 | Q d0-63 | K d64-127 | Q d64-127], 64 rows x 128 B each
    unsigned char V[2 * 8192];   // [V d0-63 | V d64-127]
};
struct KeyStage {
    unsigned char P[C * C * 2];
    unsigned char Tb[C * C * 2];
};
// Gate factors of one chunk, in a four-deep ring filled three chunks ahead by
// the output group (fac_full[slot] marks a slot published).
struct Factors {
    float G[C], beta[C], eG[C], eGl[C];
    float u[C];       // exp(G_r - G_{16 floor(r/16)})
    float w[3][C];    // w[b-1][s] = exp(G_{16b} - G_s) for s < 16b
};
constexpr int NS_F = 4;
struct WsSmem {
    InStage in[NS_IN];
    KeyStage ks[NS_K];
    Factors fac[NS_F];
    float Af[10 * BSZ];
    float Tf[10 * BSZ];
    uint64_t full_in[NS_IN], key_ready[NS_K], key_free[NS_K], o_full, o_empty, bar_k, bar_s, fac_full[NS_F];
    uint32_t tmem;
    int stop;
};
constexpr size_t WS_SMEM = sizeof(WsSmem) + 1024;  // + alignment slack
static_assert(WS_SMEM <= 232448, "shared memory");

template <typename IT> struct InT;
template <> struct InT<__nv_bfloat16> {
    static constexpr uint32_t fmt = BF16;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
    static __device__ __forceinline__ uint32_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};
template <> struct InT<__half> {
    static constexpr uint32_t fmt = F16;
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
    static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ uint32_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};
// Two fp32 values rounded to the 16-bit input type, `lo` in the low half (one cvt).
template <typename IT> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

__device__ __forceinline__ void kg_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ void sg_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }
__device__ __forceinline__ void og_sync() { asm volatile("bar.sync 3, 128;" ::: "memory"); }
// Within the key group: warps 0-3 run the inverse (barrier 5); they tell
// warps 4-7 that the blocks of its first two steps are final (barrier 6).
__device__ __forceinline__ void inv_sync() { asm volatile("bar.sync 5, 128;" ::: "memory"); }
__device__ __forceinline__ void inv_signal() { asm volatile("bar.arrive 6, 256;" ::: "memory"); }
__device__ __forceinline__ void inv_await() { asm volatile("bar.sync 6, 256;" ::: "memory"); }
// Group barriers that also OR a per-thread flag: every participant gets the
// same answer, so a group leaves its loop together even while the other group
// writes the shared stop word.
__device__ __forceinline__ bool kg_any(bool f) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\t"
        "bar.red.or.pred b, 1, 256, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)f)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ bool sg_any(bool f) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\t"
        "bar.red.or.pred b, 2, 128, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)f)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ bool og_any(bool f) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.u32 a, %1, 0;\n\t"
        "bar.red.or.pred b, 3, 128, a;\n\tselp.u32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)f)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Descriptors of the swizzled input tiles (K step ks = 16 elements of K).
//   K or Q, K-major (rows = tokens, K = features): features 64b.. in block b
__device__ __forceinline__ uint64_t desc_kq_kmaj(const unsigned char *kq, int which, int ks) {
    return smem_desc_sw128(smem_addr(kq) + which * 8192 + (ks / 4) * 16384 + (ks % 4) * 32, 16, 1024);
}
//   K viewed MN-major (MN = features, K = tokens): ks = 16 tokens
__device__ __forceinline__ uint64_t desc_k_mn(const unsigned char *kq, int ks) {
    return smem_desc_sw128(smem_addr(kq) + ks * 2048, 16384, 1024);
}
//   V viewed MN-major (A = V^T, M = features, K = tokens)
__device__ __forceinline__ uint64_t desc_v_mn(const unsigned char *v, int ks) {
    return smem_desc_sw128(smem_addr(v) + ks * 2048, 8192, 1024);
}

template <typename IT> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <typename IT>
__device__ __forceinline__ void st_vec8(unsigned char *base, uint32_t off, const float (&v)[8]) {
    *reinterpret_cast<uint4 *>(base + off) =
        make_uint4(pack2<IT>(v[0], v[1]), pack2<IT>(v[2], v[3]), pack2<IT>(v[4], v[5]), pack2<IT>(v[6], v[7]));
}

__device__ __forceinline__ float ld_state(const void *p, size_t i, int dt) {
    switch (dt) {
        case KAI_GDN_BF16: return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
        case KAI_GDN_F16: return __half2float(static_cast<const __half *>(p)[i]);
        default: return static_cast<const float *>(p)[i];
    }
}
__device__ __forceinline__ void st_state(void *p, size_t i, int dt, float v) {
    switch (dt) {
        case KAI_GDN_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
        case KAI_GDN_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
        default: static_cast<float *>(p)[i] = v;
    }
}

// T = (I + A)^-1 for strictly lower A (64 x 64, fp32, block-packed), on the
// key group, by doubling the inverted block size:
//   D    T_bb (16 x 16 diagonal blocks) by left-looking substitution, one
//        column per thread (warps 0-1), the column kept in registers;
//   L1   T10 = -T11 (A10 T00),  T32 = -T33 (A32 T22)         (warps 0-1)
//   L2   T_lo = -T_hi (A_lo T_top)  with 32 x 32 blocks: rows 32-63 x cols
//        0-31 of T from its two 32 x 32 diagonal halves         (warps 0-3)
// The 16 x 16 x 16 products of L1 / L2 run on the warp-level tensor-core MMA
// (m16n8k8, tf32) with each operand split into a tf32 head and tail and three
// products per step (hi*hi + hi*lo + lo*hi), which keeps fp32 accuracy.
// Intermediate products live in A's diagonal blocks, dead once D has run.
struct Frag {  // thread's coordinates in the m16n8k8 fragments
    int g, q;  // group (lane / 4), thread in group (lane % 4)
};
// hi = x with the 13 low mantissa bits cleared (a tf32 value), lo = x - hi
// (exact); the MMA reads the top 19 bits of each operand, so hi*hi + hi*lo +
// lo*hi carries about 21 bits of x and y.  Integer and fp32 pipes only.
__device__ __forceinline__ void split_tf32(float x, uint32_t &hi, uint32_t &lo) {
    hi = __float_as_uint(x) & 0xFFFFE000u;
    lo = __float_as_uint(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32_16x8x8(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// acc (16 x 16 as two n-tiles of the m16n8 accumulator) += X Y, X and Y
// 16 x 16 fp32 blocks with row stride BLD.  The three split products keep
// separate accumulators (short dependency chains), added smallest first.
__device__ __forceinline__ void mma16(float (&acc)[2][4], const float *__restrict__ X, const float *__restrict__ Y,
                                      Frag f) {
    float part[3][2][4] = {};
#pragma unroll
    for (int kk = 0; kk < 16; kk += 8) {
        uint32_t ah[4], al[4];
        split_tf32(X[f.g * BLD + kk + f.q], ah[0], al[0]);
        split_tf32(X[(f.g + 8) * BLD + kk + f.q], ah[1], al[1]);
        split_tf32(X[f.g * BLD + kk + f.q + 4], ah[2], al[2]);
        split_tf32(X[(f.g + 8) * BLD + kk + f.q + 4], ah[3], al[3]);
#pragma unroll
        for (int nn = 0; nn < 2; ++nn) {
            uint32_t bh[2], bl[2];
            split_tf32(Y[(kk + f.q) * BLD + 8 * nn + f.g], bh[0], bl[0]);
            split_tf32(Y[(kk + f.q + 4) * BLD + 8 * nn + f.g], bh[1], bl[1]);
            mma_tf32_16x8x8(part[0][nn], al, bh);
            mma_tf32_16x8x8(part[1][nn], ah, bl);
            mma_tf32_16x8x8(part[2][nn], ah, bh);
        }
    }
#pragma unroll
    for (int nn = 0; nn < 2; ++nn)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[nn][e] += (part[0][nn][e] + part[1][nn][e]) + part[2][nn][e];
}
// Store the accumulator (times `sign`) as a 16 x 16 block with row stride BLD.
__device__ __forceinline__ void store16(float *__restrict__ Z, const float (&acc)[2][4], float sign, Frag f) {
#pragma unroll
    for (int nn = 0; nn < 2; ++nn) {
        *reinterpret_cast<float2 *>(Z + f.g * BLD + 8 * nn + 2 * f.q) = make_float2(sign * acc[nn][0], sign * acc[nn][1]);
        *reinterpret_cast<float2 *>(Z + (f.g + 8) * BLD + 8 * nn + 2 * f.q) =
            make_float2(sign * acc[nn][2], sign * acc[nn][3]);
    }
}

// Tb entries of the 16 x 16 block (bi, bj) of T, held as an m16n8
// accumulator pair times `sign`, rounded straight into the operand tile.
template <typename IT>
__device__ __forceinline__ void store_tb16(KeyStage &ks, const Factors &fa, const float (&acc)[2][4], float sign,
                                           int bi, int bj, Frag f) {
#pragma unroll
    for (int nn = 0; nn < 2; ++nn) {
        const int s = 16 * bj + 8 * nn + 2 * f.q;
        const float b0 = fa.beta[s], b1 = fa.beta[s + 1];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int r = 16 * bi + f.g + 8 * hh;
            const float x0 = sign * acc[nn][2 * hh], x1 = sign * acc[nn][2 * hh + 1];
            *reinterpret_cast<uint32_t *>(ks.Tb + kmaj16(r, s, C)) = pack2<IT>(x0 * b0, x1 * b1);
        }
    }
}

// Runs on key-group warps 0-3 (t < 128).  The last step's four blocks go
// straight into Tb; the others stay in T for the helper warps.
template <typename IT>
__device__ __forceinline__ void invert_unit_lower(float *__restrict__ A, float *__restrict__ T, KeyStage &ks,
                                                  const Factors &fa,
                                  int t) {
    const int warp = t / 32;
    const Frag f{(t % 32) / 4, t % 4};
    auto MB = [&](int n) { return A + blk(n, n); };
    if (t < 64) {
        // column j of T_bb by substitution, right-looking in panels of four
        // columns: once s_k (k in the panel) is final it is x_k, and the rows
        // below take the panel's update as one 4-term dot product.  x_k = 0
        // for k < j without special cases (s starts as e_j).
        const int bb = t / 16, j = t % 16, o = blk(bb, bb);
        float sx[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) sx[r] = r == j ? 1.f : 0.f;
#pragma unroll
        for (int pn = 0; pn < 4; ++pn) {
            float4 a[16];
#pragma unroll
            for (int r = 4 * pn + 1; r < 16; ++r) a[r] = *reinterpret_cast<const float4 *>(A + o + r * BLD + 4 * pn);
#pragma unroll
            for (int u = 1; u < 4; ++u) {
                const int r = 4 * pn + u;
                const float av[4] = {a[r].x, a[r].y, a[r].z, a[r].w};
#pragma unroll
                for (int w = 0; w < u; ++w) sx[r] = fmaf(-av[w], sx[4 * pn + w], sx[r]);
            }
#pragma unroll
            for (int r = 4 * pn + 4; r < 16; ++r)
                sx[r] -= fmaf(a[r].x, sx[4 * pn],
                              fmaf(a[r].y, sx[4 * pn + 1], fmaf(a[r].z, sx[4 * pn + 2], a[r].w * sx[4 * pn + 3])));
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) T[o + r * BLD + j] = sx[r];
    }
    inv_sync();
    if (warp < 2) {  // L1 for the pair (b0 + 1, b0), b0 = 2 * warp
        const int b0 = 2 * warp;
        float acc[2][4] = {};
        mma16(acc, A + blk(b0 + 1, b0), T + blk(b0, b0), f);
        store16(MB(warp), acc, 1.f, f);
        __syncwarp();
        float acc2[2][4] = {};
        mma16(acc2, T + blk(b0 + 1, b0 + 1), MB(warp), f);
        store16(T + blk(b0 + 1, b0), acc2, -1.f, f);
    }
    inv_sync();
    inv_signal();  // the diagonal blocks and T10, T32 are final
    {  // L2a: M = A_lo T_top, block (mr, mc)
        //   M00 = A20 T00 + A21 T10   M01 = A21 T11   M10 = A30 T00 + A31 T10   M11 = A31 T11
        const int mr = warp >> 1, mc = warp & 1;
        float acc[2][4] = {};
        mma16(acc, A + blk(2 + mr, 1), T + blk(1, mc), f);
        if (mc == 0) mma16(acc, A + blk(2 + mr, 0), T + blk(0, 0), f);
        store16(MB(warp), acc, 1.f, f);
    }
    inv_sync();
    {  // L2b: T20 = -T22 M00   T21 = -T22 M01   T30 = -(T32 M00 + T33 M10)   T31 = -(T32 M01 + T33 M11)
        const int tr = warp >> 1, tc = warp & 1;
        float acc[2][4] = {};
        mma16(acc, T + blk(2 + tr, 2), MB(tc), f);
        if (tr == 1) mma16(acc, T + blk(3, 3), MB(2 + tc), f);
        store_tb16<IT>(ks, fa, acc, -1.f, 2 + tr, tc, f);
    }
}

// Tb = T diag(beta) for 8 columns s0 .. s0+7 of row r (a lower block),
// rounded into the K-major operand tile.
template <typename IT>
__device__ __forceinline__ void tb_chunk(const float *Tf, KeyStage &ks, const Factors &fa, int r, int s0) {
    const float *src = Tf + blk(r / 16, s0 / 16) + (r % 16) * BLD + (s0 % 16);
    const float4 x0 = *reinterpret_cast<const float4 *>(src);
    const float4 x1 = *reinterpret_cast<const float4 *>(src + 4);
    const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
    float a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] = x[u] * fa.beta[s0 + u];
    st_vec8<IT>(ks.Tb, kmaj16(r, s0, C), a);
}
// Chunk e (< 192) of the Tb blocks the inverse finishes early: the
// diagonal blocks and T10, T32 (the last step writes its own blocks).
template <typename IT>
__device__ __forceinline__ void tb_blocks(const float *Tf, KeyStage &ks, const Factors &fa, int e) {
    const int n = e / 32, row = (e % 32) / 2, half = e % 2;
    const int bi = n < 4 ? n : (n == 4 ? 1 : 3);
    const int bj = n < 4 ? n : (n == 4 ? 0 : 2);
    tb_chunk<IT>(Tf, ks, fa, 16 * bi + row, 16 * bj + 8 * half);
}

// Gate values of one chunk, two tokens per lane of warp 0.
struct Gates {
    float g0, g1, b0, b1;
};
// The loads are volatile so the compiler keeps them where they are written, a
// whole chunk ahead of their use, instead of sinking them to it.
__device__ __forceinline__ float ld_keep(const float *p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void load_gates(Gates &gt, const kai_gdn_chunk_args &p, long long b, long long h,
                                           long long c0, int lane) {
    const long long Hv = (long long)p.heads_v, T = (long long)p.seq;
    const long long r0 = c0 + 2 * lane, r1 = r0 + 1;
    gt.g0 = r0 < T ? ld_keep(p.g + (size_t)(b * T + r0) * Hv + h) : 0.f;
    gt.b0 = r0 < T ? ld_keep(p.beta + (size_t)(b * T + r0) * Hv + h) : 0.f;
    gt.g1 = r1 < T ? ld_keep(p.g + (size_t)(b * T + r1) * Hv + h) : 0.f;
    gt.b1 = r1 < T ? ld_keep(p.beta + (size_t)(b * T + r1) * Hv + h) : 0.f;
}
// In-chunk cumulative log decay G and its exponentials (warp 0, tokens
// 2*lane and 2*lane+1).  Besides exp(G), exp(G_63 - G) it stores the factors
// of exp(G_r - G_s) across 16-token blocks: for s < 16b <= r,
//   exp(G_r - G_s) = u_r * w[b-1][s],  u_r = exp(G_r - G_{16b}),  w = exp(G_{16b} - G_s)
// with b = floor(r/16); both factors are <= 1 because G does not increase.
__device__ __forceinline__ void chunk_gates(Factors &ks, const Gates &gt, int lane) {
    const float pair = gt.g0 + gt.g1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    const float excl = incl - pair, gl = __shfl_sync(0xffffffffu, incl, 31);
    const float G0 = excl + gt.g0, G1 = incl;
    // G_{16b} for b = 0..3 is G0 of lane 8b
    const float R0 = __shfl_sync(0xffffffffu, G0, 0), R1 = __shfl_sync(0xffffffffu, G0, 8);
    const float R2 = __shfl_sync(0xffffffffu, G0, 16), R3 = __shfl_sync(0xffffffffu, G0, 24);
    const int t0 = 2 * lane, blk16 = t0 / 16;
    const float Rb = blk16 == 0 ? R0 : blk16 == 1 ? R1 : blk16 == 2 ? R2 : R3;
    ks.G[t0] = G0;
    ks.G[t0 + 1] = G1;
    ks.beta[t0] = gt.b0;
    ks.beta[t0 + 1] = gt.b1;
    ks.eG[t0] = expf(G0);
    ks.eG[t0 + 1] = expf(G1);
    ks.eGl[t0] = expf(gl - G0);
    ks.eGl[t0 + 1] = expf(gl - G1);
    ks.u[t0] = expf(G0 - Rb);
    ks.u[t0 + 1] = expf(G1 - Rb);
    const float Rs[3] = {R1, R2, R3};
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) {
        const bool live = t0 < 16 * (bb + 1);
        ks.w[bb][t0] = live ? expf(Rs[bb] - G0) : 0.f;
        ks.w[bb][t0 + 1] = live ? expf(Rs[bb] - G1) : 0.f;
    }
}

// 32 consecutive rows r0 .. r0+31 of output column i (one value per row in
// v[]), stored to o[b][t0 + r][h][i] for rows that exist (t0 + r < T).
// 16-bit outputs pair neighbouring columns through a lane exchange so every
// store is 4 bytes: even lanes write row r, odd lanes row r + 1.
template <int ODT>
__device__ __forceinline__ void store_o_rows(void *out, size_t base, size_t rs, int nvalid, int r0, int i, int lane,
                                             const float (&v)[32]) {
    if (ODT == KAI_GDN_F32) {
        float *o = static_cast<float *>(out) + base + (size_t)r0 * rs + i;
#pragma unroll
        for (int rr = 0; rr < 32; ++rr, o += rs)
            if (r0 + rr < nvalid) *o = v[rr];
        return;
    }
    const bool odd = lane & 1;
    uint32_t *o = static_cast<uint32_t *>(out) + (base + (size_t)(r0 + (odd ? 1 : 0)) * rs + (odd ? i - 1 : i)) / 2;
    const size_t step = rs;  // two rows of 16-bit values = rs 4-byte words
#pragma unroll
    for (int rr = 0; rr < 32; rr += 2, o += step) {
        const float send = odd ? v[rr] : v[rr + 1];
        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
        const float lo = odd ? recv : v[rr], hi = odd ? v[rr + 1] : recv;
        const uint32_t w = ODT == KAI_GDN_BF16 ? pack2<__nv_bfloat16>(lo, hi) : pack2<__half>(lo, hi);
        if (r0 + rr + (odd ? 1 : 0) < nvalid) *o = w;
    }
}
__device__ __forceinline__ void store_o(const kai_gdn_chunk_args &p, size_t base, size_t rs, int nvalid, int r0,
                                        int i, int lane, const float (&v)[32]) {
    switch (p.out_dtype) {
        case KAI_GDN_BF16: store_o_rows<KAI_GDN_BF16>(p.o, base, rs, nvalid, r0, i, lane, v); break;
        case KAI_GDN_F16: store_o_rows<KAI_GDN_F16>(p.o, base, rs, nvalid, r0, i, lane, v); break;
        default: store_o_rows<KAI_GDN_F32>(p.o, base, rs, nvalid, r0, i, lane, v);
    }
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float LOG2E = 1.4426950408889634f;

template <typename IT>
__global__ void __launch_bounds__(NT, 1)
    chunk_ws_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, kai_gdn_chunk_args p, int *err) {
    // 1024-byte aligned by pointer arithmetic on the shared array itself, so
    // the compiler keeps every access in the shared address space.
    extern __shared__ unsigned char smem_raw[];
    WsSmem &sm = *reinterpret_cast<WsSmem *>(smem_raw + ((1024u - (umma::smem_addr(smem_raw) & 1023u)) & 1023u));
    using TR = InT<IT>;

    const int t = threadIdx.x, warp = t / 32, lane = t % 32;
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k, T = (long long)p.seq;
    const long long unit = blockIdx.x, b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const float scale = p.scale;
    const int nch = (int)((T + C - 1) / C);
    volatile int *stop = &sm.stop;

    if (t == 0) {
        for (int s = 0; s < NS_IN; ++s) mbar_init(&sm.full_in[s], 1);
        for (int s = 0; s < NS_K; ++s) {
            mbar_init(&sm.key_ready[s], 1);
            mbar_init(&sm.key_free[s], 1);
        }
        mbar_init(&sm.o_full, 1);
        mbar_init(&sm.o_empty, 1);
        for (int s = 0; s < NS_F; ++s) mbar_init(&sm.fac_full[s], 1);
        mbar_init(&sm.bar_k, 1);
        mbar_init(&sm.bar_s, 1);
        sm.stop = 0;
        tma::prefetch_map(&map_q);
        tma::prefetch_map(&map_k);
        tma::prefetch_map(&map_v);
    }
    if (warp == 0) tmem_alloc(&sm.tmem, 512);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tm = sm.tmem;

    auto issue_loads = [&](int c) {  // key-group thread 0
        InStage &s = sm.in[c % NS_IN];
        uint64_t *bar = &sm.full_in[c % NS_IN];
        mbar_arrive_expect_tx(bar, 6 * 8192);
        const int t0 = c * C;
        const uint32_t mb = smem_addr(bar);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            // one 64-feature block of K, Q and V each (128-byte swizzled boxes)
            const uint32_t dk = smem_addr(s.KQ + j * 16384), dq = smem_addr(s.KQ + j * 16384 + 8192);
            const uint32_t dv = smem_addr(s.V + j * 8192);
            asm volatile(
                "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dk),
                "l"(reinterpret_cast<uint64_t>(&map_k)), "r"(64 * j), "r"((int)hk), "r"(t0), "r"((int)b), "r"(mb)
                : "memory");
            asm volatile(
                "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dq),
                "l"(reinterpret_cast<uint64_t>(&map_q)), "r"(64 * j), "r"((int)hk), "r"(t0), "r"((int)b), "r"(mb)
                : "memory");
            asm volatile(
                "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dv),
                "l"(reinterpret_cast<uint64_t>(&map_v)), "r"(64 * j), "r"((int)h), "r"(t0), "r"((int)b), "r"(mb)
                : "memory");
        }
    };

    if (t < KG) {
        // =============================================================== key group
        // Per chunk c:  all 8 warps: E1 (A and P from [K;Q] K^T);
        //   warps 0-3: the inverse, whose last step writes its four blocks
        //     of Tb directly;
        //   warps 4-7 meanwhile: the [K;Q] K^T MMA of chunk c+1 (warp KW)
        //     and Tb of the blocks the inverse finished early;
        //   then hand the chunk over.
        constexpr int KT = 224, KW = KT / 32;  // TMA thread and its warp (MMA)
        int loaded = 0;  // chunks whose loads were issued (thread KT)
        bool fail = false;  // a wait of this thread ran out
        auto issue_m1 = [&](int cc) {  // warp KW (converged), loads of chunk cc complete
            fence_after_sync();
            if (elect_one()) {
                const uint32_t id = idesc(128, 64, TR::fmt, false, false);
                const unsigned char *kq = sm.in[cc % NS_IN].KQ;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks)
                    mma_f16(tm + COL_KQ, desc_kq_kmaj(kq, 0, ks), desc_kq_kmaj(kq, 0, ks), id, ks > 0);
                commit(&sm.bar_k);
            }
            __syncwarp();
        };
        // The upper blocks of Tb stay zero; write them once.
        for (int e = t; e < NS_K * 6 * 32; e += KG) {
            const int st2 = e / (6 * 32), n = (e % (6 * 32)) / 32, x = e % 32;
            // upper blocks (0,1) (0,2) (0,3) (1,2) (1,3) (2,3)
            const int ubi = n < 3 ? 0 : (n < 5 ? 1 : 2), ubj = n < 3 ? n + 1 : (n < 5 ? n - 1 : 3);
            const int r = 16 * ubi + x / 2, s0 = 16 * ubj + 8 * (x % 2);
            *reinterpret_cast<uint4 *>(sm.ks[st2].Tb + kmaj16(r, s0, C)) = make_uint4(0, 0, 0, 0);
        }
        if (t == KT && nch > 0) {
            issue_loads(0);
            loaded = 1;
        }
        if (warp == KW && nch > 0) {
            if (!mbar_wait(&sm.full_in[0], 0, err)) fail = true;
            issue_m1(0);
        }
        const int q4 = warp & 3, hc = warp >> 2;
        int c = 0;
        for (; c < nch; ++c) {
            const int si = c % NS_IN, sk = c % NS_K;
            KeyStage &kst = sm.ks[sk];
            const Factors &fa = sm.fac[c % NS_F];
            if (c >= NS_K && !mbar_wait(&sm.key_free[sk], ((c / NS_K) & 1) ^ 1, err)) fail = true;
            if (t == KT && c + 1 < nch) {  // stage (c+1) % 3 last held chunk c - 2, whose MMAs are done
                issue_loads(c + 1);
                loaded = c + 2;
            }
            if (!mbar_wait(&sm.full_in[si], (c / NS_IN) & 1, err)) fail = true;
            if (!mbar_wait(&sm.bar_k, c & 1, err)) fail = true;  // [K;Q] K^T of this chunk
            if (!mbar_wait(&sm.fac_full[c % NS_F], (c / NS_F) & 1, err)) fail = true;  // its gate factors
            if (kg_any(fail || *stop)) break;
            fence_after_sync();
            // ------------------------------------------ E1: A (fp32, block-packed) and P (tile)
            // exp(G_r - G_s) is computed directly inside the 16 x 16 diagonal
            // blocks and as u_r * w[s] across blocks.
            {
                float v[32];
                tmem_ld16(taddr(tm + COL_KQ, 32 * q4, 32 * hc), *reinterpret_cast<float(*)[16]>(&v[0]));
                tmem_ld16(taddr(tm + COL_KQ, 32 * q4, 32 * hc + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
                tmem_wait_ld();
                reg_fence16(&v[0]);
                reg_fence16(&v[16]);
                const bool arow = q4 < 2;
                const int r = 32 * (q4 & 1) + lane, rb = r / 16;
                const float g2r = fa.G[r] * LOG2E;
                const float rowf = arow ? fa.beta[r] : scale;  // beta_r for A, scale for P
                const float rowu = rowf * fa.u[r];
                const float *wrow = fa.w[rb > 0 ? rb - 1 : 0];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int sb = 2 * hc + half, s0 = 16 * sb;
                    float a[16];
                    if (sb < rb) {
#pragma unroll
                        for (int x = 0; x < 16; x += 4) {
                            const float4 wv = *reinterpret_cast<const float4 *>(wrow + s0 + x);
                            a[x] = v[16 * half + x] * rowu * wv.x;
                            a[x + 1] = v[16 * half + x + 1] * rowu * wv.y;
                            a[x + 2] = v[16 * half + x + 2] * rowu * wv.z;
                            a[x + 3] = v[16 * half + x + 3] * rowu * wv.w;
                        }
                    } else if (sb == rb) {
                        const int lim = arow ? r : r + 1;  // s < r for A, s <= r for P
#pragma unroll
                        for (int x = 0; x < 16; ++x) {
                            const int s = s0 + x;
                            a[x] = s < lim ? rowf * v[16 * half + x] * ex2(g2r - fa.G[s] * LOG2E) : 0.f;
                        }
                    } else {
#pragma unroll
                        for (int x = 0; x < 16; ++x) a[x] = 0.f;
                    }
                    if (arow) {
                        if (sb <= rb) {
                            float *dst = sm.Af + blk(rb, sb) + (r % 16) * BLD;
#pragma unroll
                            for (int x = 0; x < 16; x += 4)
                                *reinterpret_cast<float4 *>(dst + x) = make_float4(a[x], a[x + 1], a[x + 2], a[x + 3]);
                        }
                    } else {
                        st_vec8<IT>(kst.P, kmaj16(r, s0, C), *reinterpret_cast<float(*)[8]>(&a[0]));
                        st_vec8<IT>(kst.P, kmaj16(r, s0 + 8, C), *reinterpret_cast<float(*)[8]>(&a[8]));
                    }
                }
            }
            fence_before_sync();
            kg_sync();
            if (warp < 4) {
                // ------------------------------------------ INV (warps 0-3)
                invert_unit_lower<IT>(sm.Af, sm.Tf, kst, fa, t);
            } else {
                // ------------------------------------------ helpers (warps 4-7)
                if (warp == KW && c + 1 < nch) {  // the TMEM tile was read; start the next chunk's [K;Q] K^T
                    if (!mbar_wait(&sm.full_in[(c + 1) % NS_IN], ((c + 1) / NS_IN) & 1, err)) fail = true;
                    issue_m1(c + 1);
                }
                const int ht = t - 128;
                inv_await();  // diagonal blocks, T10 and T32 are final
                for (int e = ht; e < 6 * 32; e += 128) tb_blocks<IT>(sm.Tf, kst, fa, e);
            }
            fence_smem_to_async();
            kg_sync();
            if (t == 0) mbar_arrive(&sm.key_ready[sk]);
        }
        // leave only once every issued load has landed (every M1 issued was
        // waited for at the top of its chunk, before any exit)
        if (t == KT)
            for (int cc = c; cc < loaded; ++cc) mbar_wait(&sm.full_in[cc % NS_IN], (cc / NS_IN) & 1, err);
        if (c < nch) *stop = 1;
    } else if (t < KG + SG) {
        // =============================================================== state group
        const int st = t - KG, sq = st / 32, i = 32 * sq + lane;  // i = value index = TMEM lane
        const uint32_t lb = 32u * sq;
        // The decay exp(G_63) of a chunk is the last entry of its exp(G) factors.
        bool fail = false;  // a wait of this thread ran out
        if (nch > 0 && !mbar_wait(&sm.fac_full[0], 0, err)) fail = true;
        const float gamma0 = nch > 0 ? sm.fac[0].eG[C - 1] : 1.f;
        // initial state: gamma_0 S^T into TMEM, the unscaled 16-bit copy beside it
        {
            const size_t sb = (size_t)unit * D * D + i;
            for (int j0 = 0; j0 < D; j0 += 32) {
                float v[32];
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = ld_state(p.state, sb + (size_t)(j0 + jj) * D, p.state_dtype);
                uint32_t u[16];
#pragma unroll
                for (int x = 0; x < 16; ++x) u[x] = pack2<IT>(v[2 * x], v[2 * x + 1]);
                tmem_st16u(taddr(tm + COL_SB, lb, j0 / 2), u);
#pragma unroll
                for (int x = 0; x < 32; ++x) v[x] *= gamma0;
                tmem_st16(taddr(tm + COL_ST, lb, j0), *reinterpret_cast<float(*)[16]>(&v[0]));
                tmem_st16(taddr(tm + COL_ST, lb, j0 + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
            }
            tmem_wait_st();
        }
        fence_before_sync();
        uint32_t ph = 0;
        int c = 0;
        for (; c < nch; ++c) {
            const int si = c % NS_IN, sk = c % NS_K;
            InStage &ist = sm.in[si];
            KeyStage &kst = sm.ks[sk];
            if (!mbar_wait(&sm.key_ready[sk], (c / NS_K) & 1, err)) fail = true;
            if (c >= 1 && !mbar_wait(&sm.o_empty, (c - 1) & 1, err)) fail = true;  // O^T of chunk c-1 was read out
            if (sg_any(fail || *stop)) break;
            // ------------------------------------------ M3a: [(K S)^T | X^T] = S^T [K; Q]^T
            // Each 64-feature block of the [K;Q] tile holds the K rows and then
            // the Q rows, so one N = 128 operand covers both products.
            if (sq == 0) {
                fence_after_sync();
                if (elect_one()) {
                    const uint32_t id = idesc(128, 128, TR::fmt, false, false);
#pragma unroll
                    for (int ks = 0; ks < D / 16; ++ks)
                        mma_f16_ta(tm + COL_VA, tm + COL_SB + ks * 8, desc_kq_kmaj(ist.KQ, 0, ks), id, ks > 0);
                    commit(&sm.bar_s);
                }
                __syncwarp();
            }
            const bool more = c + 1 < nch;
            float gamma_next = 1.f;
            if (more) {
                if (!mbar_wait(&sm.fac_full[(c + 1) % NS_F], ((c + 1) / NS_F) & 1, err)) fail = true;
                gamma_next = sm.fac[(c + 1) % NS_F].eG[C - 1];
            }
            if (!mbar_wait(&sm.bar_s, ph, err)) fail = true;
            ph ^= 1;
            fence_after_sync();
            // ------------------------------------------ E3a: -(K S)^T exp(G) -> 16-bit A operand
            {
                const float *eg = sm.fac[c % NS_F].eG;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float v[32];
                    tmem_ld16(taddr(tm + COL_VA, lb, 32 * half), *reinterpret_cast<float(*)[16]>(&v[0]));
                    tmem_ld16(taddr(tm + COL_VA, lb, 32 * half + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
                    tmem_wait_ld();
                    reg_fence16(&v[0]);
                    reg_fence16(&v[16]);
                    uint32_t u[16];
#pragma unroll
                    for (int x = 0; x < 16; x += 2) {
                        const float4 e = *reinterpret_cast<const float4 *>(eg + 32 * half + 2 * x);
                        u[x] = pack2<IT>(-v[2 * x] * e.x, -v[2 * x + 1] * e.y);
                        u[x + 1] = pack2<IT>(-v[2 * x + 2] * e.z, -v[2 * x + 3] * e.w);
                    }
                    tmem_st16u(taddr(tm + COL_KSB, lb, 16 * half), u);
                }
            }
            tmem_wait_st();
            fence_before_sync();
            sg_sync();
            // ------------------------------------------ M3b: V'^T = V^T Tb^T - ((K S)^T exp(G)) Tb^T
            if (sq == 0) {
                fence_after_sync();
                if (elect_one()) {
                    const uint32_t id_v = idesc(128, 64, TR::fmt, true, false);
                    const uint32_t id_t = idesc(128, 64, TR::fmt, false, false);
#pragma unroll
                    for (int ks = 0; ks < C / 16; ++ks)
                        mma_f16(tm + COL_VA, desc_v_mn(ist.V, ks), desc_kmaj16(kst.Tb, C, ks), id_v, ks > 0);
#pragma unroll
                    for (int ks = 0; ks < C / 16; ++ks)
                        mma_f16_ta(tm + COL_VA, tm + COL_KSB + ks * 8, desc_kmaj16(kst.Tb, C, ks), id_t, true);
                    commit(&sm.bar_s);
                }
                __syncwarp();
            }
            if (!mbar_wait(&sm.bar_s, ph, err)) fail = true;
            ph ^= 1;
            fence_after_sync();
            // ------------------------------------------ E3: V' and V'' = V' exp(G_63 - G) -> 16-bit A operands
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float v[32];
                tmem_ld16(taddr(tm + COL_VA, lb, 32 * half), *reinterpret_cast<float(*)[16]>(&v[0]));
                tmem_ld16(taddr(tm + COL_VA, lb, 32 * half + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
                tmem_wait_ld();
                reg_fence16(&v[0]);
                reg_fence16(&v[16]);
                uint32_t u[16], w[16];
#pragma unroll
                for (int x = 0; x < 16; x += 2) {
                    const float4 e = *reinterpret_cast<const float4 *>(&sm.fac[c % NS_F].eGl[32 * half + 2 * x]);
                    u[x] = pack2<IT>(v[2 * x], v[2 * x + 1]);
                    u[x + 1] = pack2<IT>(v[2 * x + 2], v[2 * x + 3]);
                    w[x] = pack2<IT>(v[2 * x] * e.x, v[2 * x + 1] * e.y);
                    w[x + 1] = pack2<IT>(v[2 * x + 2] * e.z, v[2 * x + 3] * e.w);
                }
                tmem_st16u(taddr(tm + COL_VB, lb, 16 * half), u);
                tmem_st16u(taddr(tm + COL_VB2, lb, 16 * half), w);
            }
            tmem_wait_st();
            fence_before_sync();
            sg_sync();
            // ------------------------------------------ M4: S^T update;  Y^T = V'^T P^T (V'^T was read)
            if (sq == 0) {
                fence_after_sync();
                if (elect_one()) {
                    const uint32_t id_o = idesc(128, 64, TR::fmt, false, false);
                    const uint32_t id_s = idesc(128, 128, TR::fmt, false, true);
#pragma unroll
                    for (int ks = 0; ks < C / 16; ++ks)
                        mma_f16_ta(tm + COL_ST, tm + COL_VB2 + ks * 8, desc_k_mn(ist.KQ, ks), id_s, true);
                    commit(&sm.bar_s);
#pragma unroll
                    for (int ks = 0; ks < C / 16; ++ks)
                        mma_f16_ta(tm + COL_VA, tm + COL_VB + ks * 8, desc_kmaj16(kst.P, C, ks), id_o, ks > 0);
                    commit(&sm.key_free[sk]);
                    commit(&sm.o_full);
                }
                __syncwarp();
            }
            if (!mbar_wait(&sm.bar_s, ph, err)) fail = true;
            ph ^= 1;
            fence_after_sync();
            // ------------------------------------------ E4: S^T -> 16-bit copy; gamma_next S^T back
            {
                float v[2][32];
                tmem_ld16(taddr(tm + COL_ST, lb, 0), *reinterpret_cast<float(*)[16]>(&v[0][0]));
                tmem_ld16(taddr(tm + COL_ST, lb, 16), *reinterpret_cast<float(*)[16]>(&v[0][16]));
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    float(&cur)[32] = v[g & 1];
                    tmem_wait_ld();
                    reg_fence16(&cur[0]);
                    reg_fence16(&cur[16]);
                    if (g + 1 < 4) {  // next 32 columns in flight while these are converted
                        tmem_ld16(taddr(tm + COL_ST, lb, 32 * (g + 1)), *reinterpret_cast<float(*)[16]>(&v[(g + 1) & 1][0]));
                        tmem_ld16(taddr(tm + COL_ST, lb, 32 * (g + 1) + 16),
                                  *reinterpret_cast<float(*)[16]>(&v[(g + 1) & 1][16]));
                    }
                    uint32_t u[16];
#pragma unroll
                    for (int x = 0; x < 16; ++x) u[x] = pack2<IT>(cur[2 * x], cur[2 * x + 1]);
                    tmem_st16u(taddr(tm + COL_SB, lb, 16 * g), u);
                    if (more) {
#pragma unroll
                        for (int x = 0; x < 32; ++x) cur[x] *= gamma_next;
                        tmem_st16(taddr(tm + COL_ST, lb, 32 * g), *reinterpret_cast<float(*)[16]>(&cur[0]));
                        tmem_st16(taddr(tm + COL_ST, lb, 32 * g + 16), *reinterpret_cast<float(*)[16]>(&cur[16]));
                    }
                }
                tmem_wait_st();
            }
            fence_before_sync();
        }
        if (c == nch) {
            // final state (fp32 from TMEM, S[j][i] = S^T[i][j]); the last M4 has completed
            const size_t sb = (size_t)unit * D * D + i;
            for (int j0 = 0; j0 < D; j0 += 32) {
                float v[32];
                tmem_ld16(taddr(tm + COL_ST, lb, j0), *reinterpret_cast<float(*)[16]>(&v[0]));
                tmem_ld16(taddr(tm + COL_ST, lb, j0 + 16), *reinterpret_cast<float(*)[16]>(&v[16]));
                tmem_wait_ld();
                reg_fence16(&v[0]);
                reg_fence16(&v[16]);
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) st_state(p.state, sb + (size_t)(j0 + jj) * D, p.state_dtype, v[jj]);
            }
        } else {
            *stop = 1;
        }
        // the O MMAs of the last chunk are covered by the o_full commit the output group waits on
        fence_before_sync();
    } else {
        // =============================================================== output group
        // O = scale exp(G_r) X + Y: X^T (M3a) and Y^T (M4) sit in separate
        // accumulators.  Warp 12 also computes every chunk's gate factors,
        // NS_F - 1 chunks ahead (its gates loaded one chunk before that), and
        // publishes them on fac_full.
        const int ot = t - KG - SG, oq = ot / 32, i = 32 * oq + lane;
        const uint32_t lb = 32u * oq;
        const size_t orow = (size_t)Hv * D;  // output row stride (elements)
        Gates go{};
        auto publish_factors = [&](int cc) {  // warp 12; go holds chunk cc's gates
            const Gates cur = go;
            if (cc + 1 < nch) load_gates(go, p, b, h, (long long)(cc + 1) * C, lane);
            chunk_gates(sm.fac[cc % NS_F], cur, lane);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.fac_full[cc % NS_F]);
        };
        if (oq == 0 && nch > 0) {
            load_gates(go, p, b, h, 0, lane);
            for (int cc = 0; cc < NS_F - 1 && cc < nch; ++cc) publish_factors(cc);
        }
        bool fail = false;
        int c = 0;
        for (; c < nch; ++c) {
            if (oq == 0 && c + NS_F - 1 < nch) publish_factors(c + NS_F - 1);
            const float *eg = sm.fac[c % NS_F].eG;  // published NS_F - 1 chunks ago
            if (!mbar_wait(&sm.o_full, c & 1, err)) fail = true;
            if (og_any(fail || *stop)) break;
            fence_after_sync();
            const long long t0 = (long long)c * C;
            const size_t obase = ((size_t)(b * T + t0) * Hv + h) * D;
            const int nvalid = (int)min((long long)C, T - t0);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float x[32], y[32];
                tmem_ld16(taddr(tm + COL_OA, lb, 32 * half), *reinterpret_cast<float(*)[16]>(&x[0]));
                tmem_ld16(taddr(tm + COL_OA, lb, 32 * half + 16), *reinterpret_cast<float(*)[16]>(&x[16]));
                tmem_ld16(taddr(tm + COL_VA, lb, 32 * half), *reinterpret_cast<float(*)[16]>(&y[0]));
                tmem_ld16(taddr(tm + COL_VA, lb, 32 * half + 16), *reinterpret_cast<float(*)[16]>(&y[16]));
                tmem_wait_ld();
                reg_fence16(&x[0]);
                reg_fence16(&x[16]);
                reg_fence16(&y[0]);
                reg_fence16(&y[16]);
#pragma unroll
                for (int r = 0; r < 32; r += 4) {
                    const float4 f = *reinterpret_cast<const float4 *>(eg + 32 * half + r);
                    x[r] = fmaf(scale * f.x, x[r], y[r]);
                    x[r + 1] = fmaf(scale * f.y, x[r + 1], y[r + 1]);
                    x[r + 2] = fmaf(scale * f.z, x[r + 2], y[r + 2]);
                    x[r + 3] = fmaf(scale * f.w, x[r + 3], y[r + 3]);
                }
                if (half == 1) {
                    fence_before_sync();
                    og_sync();
                    if (ot == 0) mbar_arrive(&sm.o_empty);  // the MMAs may overwrite X^T and Y^T now
                }
                store_o(p, obase, orow, nvalid, 32 * half, i, lane, x);
            }
        }
        if (c < nch) *stop = 1;
        fence_before_sync();
    }
    __syncthreads();
    fence_after_sync();
    if (warp == 0) tmem_dealloc(tm, 512);
}

}  // namespace

bool chunk_ws_supported(const kai_gdn_chunk_args *a) {
    if (a->dk != 128 || a->dv != 128 || a->chunk != 64) return false;
    if (a->in_dtype != KAI_GDN_BF16 && a->in_dtype != KAI_GDN_F16) return false;
    if (((uintptr_t)a->q | (uintptr_t)a->k | (uintptr_t)a->v) % 16) return false;
    if (a->out_dtype != KAI_GDN_F32 && ((uintptr_t)a->o % 4)) return false;
    if (a->seq > 0x7fffffffull || a->batch > 0x7fffffffull || a->heads_v > 0x7fffffffull) return false;
    return true;
}

int launch_chunk_ws(const kai_gdn_chunk_args *a, cudaStream_t st) {
    const long long units = (long long)(a->batch * a->heads_v);
    if (units > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "chunk_ws: too many heads");
    int *flag = nullptr;
    int rc = device_error_word(&flag);
    if (rc) return rc;
    const bool bf16 = a->in_dtype == KAI_GDN_BF16;
    CUtensorMap mq, mk, mv;
    int r1 = tma::make_chunk_map(&mq, a->q, bf16, a->batch, a->seq, a->heads_k, 128, true);
    int r2 = tma::make_chunk_map(&mk, a->k, bf16, a->batch, a->seq, a->heads_k, 128, true);
    int r3 = tma::make_chunk_map(&mv, a->v, bf16, a->batch, a->seq, a->heads_v, 128, true);
    if (r1 || r2 || r3)
        return set_error(KAI_GDN_ERR_CUDA, "chunk_ws: tensor map encoding failed (%d, %d, %d)", r1, r2, r3);
    if (bf16) {
        rc = check_cuda(cudaFuncSetAttribute(chunk_ws_kernel<__nv_bfloat16>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WS_SMEM),
                        "chunk_ws: smem attribute");
        if (rc) return rc;
        chunk_ws_kernel<__nv_bfloat16><<<(unsigned)units, NT, WS_SMEM, st>>>(mq, mk, mv, *a, flag);
    } else {
        rc = check_cuda(cudaFuncSetAttribute(chunk_ws_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)WS_SMEM),
                        "chunk_ws: smem attribute");
        if (rc) return rc;
        chunk_ws_kernel<__half><<<(unsigned)units, NT, WS_SMEM, st>>>(mq, mk, mv, *a, flag);
    }
    return check_launch("chunk_delta_rule_ws");
}

}  // namespace gdn
