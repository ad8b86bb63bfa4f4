// decode.cu -- single-token matrix-state gated delta-rule step on sm_100a.
//
// Per (batch b, value head h), key head hk = h / (Hv/Hk), a = exp(g[b][h]):
//   S *= a;  kv_i = sum_j S[j][i] k_j;  delta_i = (v_i - kv_i) * beta;
//   S[j][i] += k_j delta_i;  o_i = sum_j S[j][i] (scale q_j)
// gpu/gdn_gpu_kernels.cl:158-206 and its C twin gpu/gdn_gpu_validate.c:100-118.
// The OpenCL kernel makes four passes over S (decay, retrieve, write, read);
// here S is read from HBM once and written once: a CTA holds a dk x DVB block
// of value columns of one head's state in registers (32 floats per thread at
// 128 x 64), so the kernel is bound by 2 * dk * dv * sizeof(state) bytes per
// head.
//
// The GDN-2 form (decoupled gating, bench/gdn2_reference.py:58-145) runs in
// the same kernel: per-key-channel decay exp(g_j) instead of one scalar, the
// erase vector b_j k_j in the retrieve, and delta_i = w_i v_i - erase_i (no
// beta).
//
// Thread layout: DVB/4 threads cover one row of the block with 16-byte
// accesses (16 threads, 256 contiguous bytes at DVB = 64), and the 256 threads
// take rows j = rg, rg + RPP, ...  Column sums over j are per-thread partials
// reduced across row groups through shared memory.
#include "gdn_internal.cuh"

namespace gdn {
namespace {

__device__ __forceinline__ void store_any(void *p, size_t i, int dt, float v) {
    switch (dt) {
        case KAI_GDN_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
        case KAI_GDN_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
        default: static_cast<float *>(p)[i] = v;
    }
}

// q, k (one key channel) and v (one value column) of this thread, widened.
template <typename T, int DK, int DVB, typename P>
__device__ __forceinline__ void load_inputs(const P &p, int t, size_t kq, size_t vo, float &kj, float &qj, float &vi) {
    const T *k = static_cast<const T *>(p.k), *q = static_cast<const T *>(p.q), *v = static_cast<const T *>(p.v);
    if (t < DK) {
        kj = static_cast<float>(k[kq + t]);
        qj = static_cast<float>(q[kq + t]);
    }
    if (t < DVB) vi = static_cast<float>(v[vo + t]);
}

// 4 consecutive state elements.
template <int SDT>
__device__ __forceinline__ float4 ld4(const void *base, size_t idx) {
    if (SDT == KAI_GDN_F32) return *reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx);
    uint2 u = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + idx);
    using S = Store<SDT>;
    const typename S::T *h = reinterpret_cast<const typename S::T *>(&u);
    return make_float4(S::load(h), S::load(h + 1), S::load(h + 2), S::load(h + 3));
}
template <int SDT>
__device__ __forceinline__ void st4(void *base, size_t idx, float4 v) {
    if (SDT == KAI_GDN_F32) {
        *reinterpret_cast<float4 *>(static_cast<float *>(base) + idx) = v;
        return;
    }
    using S = Store<SDT>;
    uint2 u;
    typename S::T *h = reinterpret_cast<typename S::T *>(&u);
    S::store(h, v.x);
    S::store(h + 1, v.y);
    S::store(h + 2, v.z);
    S::store(h + 3, v.w);
    *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(base) + idx) = u;
}

// Kernel parameters of both forms: beta (GDN-1) or the erase gate b and the
// write gate w (GDN-2).
struct DecodeP {
    void *state;
    const void *q, *k, *v;
    const float *g;     // GDN-1: [B][Hv];  GDN-2: [B][Hv][dk]
    const float *beta;  // GDN-1: [B][Hv];  GDN-2: erase gate [B][Hv][dk]
    const float *w;     // GDN-2: write gate [B][Hv][dv]
    void *o;
    long long heads_k, heads_v;
    float scale;
    int in_dtype, out_dtype;
};

// One CTA per (b, value head, block of DVB value columns).  The value
// columns of S are independent (kv_i and o_i use only column i), so a head
// splits into D/DVB CTAs with no exchange; each reads the head's whole k and
// q.  Smaller blocks make more, shorter CTAs: the last wave of a launch is
// less empty.
template <int D, int DVB, int NTH, int MINB, int SDT, bool G2>
__global__ void __launch_bounds__(NTH, MINB) decode_step_kernel(DecodeP p) {
    constexpr int DK = D, DV = D;
    constexpr int CPR = DVB / 4;       // threads per row
    constexpr int RPP = NTH / CPR;     // rows per pass
    constexpr int RPT = DK / RPP;      // rows per thread
    constexpr int NB = DV / DVB;       // column blocks per head
    static_assert(RPT >= 1 && DK % RPP == 0, "shape");

    __shared__ float ks[DK], qs[DK], vs[DVB], dl[DVB];
    __shared__ float eg[G2 ? DK : 1], bk[G2 ? DK : 1];  // GDN-2: exp(g_j), b_j k_j
    __shared__ float red[RPP][DVB + 4];

    const long long unit = blockIdx.x / NB;   // b * Hv + h
    const int cb = (int)(blockIdx.x % NB) * DVB;  // first value column of this CTA
    const long long Hv = (long long)p.heads_v, Hk = (long long)p.heads_k;
    const long long b = unit / Hv, h = unit % Hv, hk = h / (Hv / Hk);
    const int t = threadIdx.x, cq = t % CPR, rg = t / CPR;
    const size_t sbase = (size_t)unit * DK * DV + cb;

    // The state loads lead in GDN-1; in GDN-2 the per-channel gate vectors
    // lead, so their latency overlaps the state's instead of trailing it
    // (measured per config-1 layer: GDN-2 53.1 -> 48.3 us, while GDN-1 is 1.6
    // us faster with its state first).
    float4 s[RPT];
    auto load_state = [&]() {
#pragma unroll
        for (int r = 0; r < RPT; ++r) s[r] = ld4<SDT>(p.state, sbase + (size_t)(rg + RPP * r) * DV + 4 * cq);
    };
    if constexpr (!G2) load_state();

    // The vector loads of the prologue are all issued before its first
    // shared-memory store, so they are in flight together (a load through a
    // generic pointer may not move past a shared-memory store): GDN-2 step
    // 55.2 -> 53.0 us per config-1 layer.  GDN-1's two scalar gates are read
    // after the stores, which measured 1.5% faster than reading them first.
    static_assert(DK <= NTH && DVB <= NTH, "one prologue element per thread");
    const size_t kq = (size_t)(b * Hk + hk) * DK, vo = (size_t)unit * DV + cb;
    float kj = 0.f, qj = 0.f, vi = 0.f, gj = 0.f, bj = 0.f, wi = 0.f;
    switch (p.in_dtype) {
        case KAI_GDN_BF16: load_inputs<__nv_bfloat16, DK, DVB>(p, t, kq, vo, kj, qj, vi); break;
        case KAI_GDN_F16: load_inputs<__half, DK, DVB>(p, t, kq, vo, kj, qj, vi); break;
        default: load_inputs<float, DK, DVB>(p, t, kq, vo, kj, qj, vi);
    }
    if (G2) {
        if (t < DK) {
            gj = __ldg(p.g + (size_t)unit * DK + t);
            bj = __ldg(p.beta + (size_t)unit * DK + t);
        }
        if (t < DVB) wi = __ldg(p.w + vo + t);
    }
    if constexpr (G2) load_state();
    if (t < DK) {
        ks[t] = kj;
        qs[t] = __fmul_rn(qj, p.scale);
        if (G2) {
            eg[t] = expf(gj);
            bk[t] = __fmul_rn(bj, kj);
        }
    }
    if (t < DVB) vs[t] = G2 ? __fmul_rn(wi, vi) : vi;
    const float a = G2 ? 1.f : expf(p.g[unit]);
    const float beta = G2 ? 1.f : p.beta[unit];
    __syncthreads();

    // Decay and retrieve: kv partial over this thread's rows.
    float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int j = rg + RPP * r;
        const float kj = G2 ? bk[j] : ks[j], aj = G2 ? eg[j] : a;
        s[r].x = __fmul_rn(s[r].x, aj);
        s[r].y = __fmul_rn(s[r].y, aj);
        s[r].z = __fmul_rn(s[r].z, aj);
        s[r].w = __fmul_rn(s[r].w, aj);
        kv.x = fmaf(s[r].x, kj, kv.x);
        kv.y = fmaf(s[r].y, kj, kv.y);
        kv.z = fmaf(s[r].z, kj, kv.z);
        kv.w = fmaf(s[r].w, kj, kv.w);
    }
    *reinterpret_cast<float4 *>(&red[rg][4 * cq]) = kv;
    __syncthreads();
    for (int i = t; i < DVB; i += NTH) {
        float acc = 0.f;
#pragma unroll
        for (int g2 = 0; g2 < RPP; ++g2) acc += red[g2][i];
        dl[i] = G2 ? vs[i] - acc : (vs[i] - acc) * beta;
    }
    __syncthreads();

    // Rank-1 write, read-out partial, and the store of the new state.
    const float4 d = *reinterpret_cast<const float4 *>(&dl[4 * cq]);
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
        const int j = rg + RPP * r;
        const float kj = ks[j], qj = qs[j];
        s[r].x = fmaf(kj, d.x, s[r].x);
        s[r].y = fmaf(kj, d.y, s[r].y);
        s[r].z = fmaf(kj, d.z, s[r].z);
        s[r].w = fmaf(kj, d.w, s[r].w);
        st4<SDT>(p.state, sbase + (size_t)j * DV + 4 * cq, s[r]);
        o.x = fmaf(s[r].x, qj, o.x);
        o.y = fmaf(s[r].y, qj, o.y);
        o.z = fmaf(s[r].z, qj, o.z);
        o.w = fmaf(s[r].w, qj, o.w);
    }
    *reinterpret_cast<float4 *>(&red[rg][4 * cq]) = o;
    __syncthreads();
    for (int i = t; i < DVB; i += NTH) {
        float acc = 0.f;
#pragma unroll
        for (int g2 = 0; g2 < RPP; ++g2) acc += red[g2][i];
        store_any(p.o, (size_t)unit * DV + cb + i, p.out_dtype, acc);
    }
}

// Geometry per head size: column block, threads, CTAs per SM.  At the
// model's head size (128) two 64-column CTAs per head (32 KB of state each,
// 8 rows per thread) run at 95% of the measured copy peak on B200 against 89%
// for one 128-column CTA per head; 32-column blocks and 128-thread CTAs
// measured no better.
template <int D> struct DecodeGeo;
template <> struct DecodeGeo<32> { static constexpr int DVB = 32, NTH = 256, MINB = 3; };
template <> struct DecodeGeo<64> { static constexpr int DVB = 64, NTH = 256, MINB = 3; };
template <> struct DecodeGeo<128> { static constexpr int DVB = 64, NTH = 256, MINB = 3; };

template <int D, bool G2>
int run_decode(const DecodeP &p, size_t units, int state_dtype, cudaStream_t st) {
    using G = DecodeGeo<D>;
    const long long ctas = (long long)units * (D / G::DVB);
    if (ctas > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "decode: too many heads");
    switch (state_dtype) {
        case KAI_GDN_F32:
            decode_step_kernel<D, G::DVB, G::NTH, G::MINB, KAI_GDN_F32, G2><<<(unsigned)ctas, G::NTH, 0, st>>>(p);
            break;
        case KAI_GDN_F16:
            decode_step_kernel<D, G::DVB, G::NTH, G::MINB, KAI_GDN_F16, G2><<<(unsigned)ctas, G::NTH, 0, st>>>(p);
            break;
        case KAI_GDN_BF16:
            decode_step_kernel<D, G::DVB, G::NTH, G::MINB, KAI_GDN_BF16, G2><<<(unsigned)ctas, G::NTH, 0, st>>>(p);
            break;
    }
    return check_launch(G2 ? "gdn2_delta_rule_decode" : "delta_rule_decode");
}

// Shape, dtype and alignment checks shared by both forms.
int check_decode_shape(const char *name, size_t heads_k, size_t heads_v, int in_dt, int state_dt, int out_dt,
                       const void *state, size_t dk, size_t dv) {
    if (heads_k == 0 || heads_v % heads_k)
        return set_error(KAI_GDN_ERR_INVALID, "%s: heads_v %zu not a multiple of heads_k %zu", name, heads_v,
                         heads_k);
    if (!valid_dtype(in_dt) || !valid_dtype(state_dt) || !valid_dtype(out_dt))
        return set_error(KAI_GDN_ERR_INVALID, "%s: bad dtype", name);
    size_t es = dtype_size(state_dt);
    if ((uintptr_t)state % (4 * es))
        return set_error(KAI_GDN_ERR_INVALID, "%s: state must be %zu-byte aligned", name, 4 * es);
    if (dk != dv) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: dk %zu != dv %zu", name, dk, dv);
    if (dk != 32 && dk != 64 && dk != 128)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: head dim %zu (supported: 32, 64, 128)", name, dk);
    return KAI_GDN_OK;
}

template <bool G2>
int dispatch_decode(const DecodeP &p, size_t units, size_t d, int state_dtype, cudaStream_t st) {
    switch (d) {
        case 32: return run_decode<32, G2>(p, units, state_dtype, st);
        case 64: return run_decode<64, G2>(p, units, state_dtype, st);
        default: return run_decode<128, G2>(p, units, state_dtype, st);
    }
}

}  // namespace

int launch_decode(const kai_gdn_decode_args *a, cudaStream_t st) {
    if (!a) return set_error(KAI_GDN_ERR_INVALID, "decode: null args");
    if (a->batch == 0 || a->heads_v == 0) return KAI_GDN_OK;
    if (!a->state || !a->q || !a->k || !a->v || !a->g || !a->beta || !a->o)
        return set_error(KAI_GDN_ERR_INVALID, "decode: null pointer");
    int rc = check_decode_shape("decode", a->heads_k, a->heads_v, a->in_dtype, a->state_dtype, a->out_dtype,
                                a->state, a->dk, a->dv);
    if (rc) return rc;
    const DecodeP p{a->state, a->q, a->k, a->v, a->g, a->beta, nullptr, a->o, (long long)a->heads_k,
                    (long long)a->heads_v, a->scale, a->in_dtype, a->out_dtype};
    return dispatch_decode<false>(p, a->batch * a->heads_v, a->dk, a->state_dtype, st);
}

int launch_gdn2_decode(const kai_gdn2_decode_args *a, cudaStream_t st) {
    if (!a) return set_error(KAI_GDN_ERR_INVALID, "gdn2_decode: null args");
    if (a->batch == 0 || a->heads_v == 0) return KAI_GDN_OK;
    if (!a->state || !a->q || !a->k || !a->v || !a->g || !a->b_gate || !a->w_gate || !a->o)
        return set_error(KAI_GDN_ERR_INVALID, "gdn2_decode: null pointer");
    int rc = check_decode_shape("gdn2_decode", a->heads_k, a->heads_v, a->in_dtype, a->state_dtype, a->out_dtype,
                                a->state, a->dk, a->dv);
    if (rc) return rc;
    const DecodeP p{a->state, a->q, a->k, a->v, a->g, a->b_gate, a->w_gate, a->o, (long long)a->heads_k,
                    (long long)a->heads_v, a->scale, a->in_dtype, a->out_dtype};
    return dispatch_decode<true>(p, a->batch * a->heads_v, a->dk, a->state_dtype, st);
}

}  // namespace gdn
