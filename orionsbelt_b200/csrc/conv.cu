// conv.cu -- causal depthwise Conv1D, kernel width 4, on sm_100a.
//
//   out[t][c] = w[0][c]*in[t-3][c] + w[1][c]*in[t-2][c] + w[2][c]*in[t-1][c]
//             + w[3][c]*in[t][c],        in[-3..-1][c] = hist[0..2][c]
//
// kleidiai_submission/kai/ukernels/gdn/kai_gdn_causal_dwconv1d_f32_k4_sve.c:149-165.
// Every output is the reference's expression evaluated left to right with one
// rounding per operation, so fp32 results are bit-identical to the reference's
// scalar path on every input, and exact on integer-valued inputs.
//
// HBM-bound (2 bytes moved per element read or written, nothing reused across
// channels).  Each thread owns VEC channels (16 bytes: a float4 or 8 halves)
// and a segment of SEG rows; it keeps a 3-row window in registers, so in[] is
// read once plus a 3-row halo per segment (3/SEG extra, served by L2).
// The thread that owns segment 0 is the only one that reads hist[] and the
// only one that writes it, after its last read, so segments running in other
// blocks never race on the carried history.
#include "gdn_internal.cuh"

namespace gdn {
namespace {

constexpr int SEG = 32;     // rows per thread
constexpr int THREADS = 256;

template <int DT, int VEC>
__device__ __forceinline__ void ld(const void *base, size_t idx, float (&v)[VEC]) {
    using S = Store<DT>;
    const typename S::T *p = static_cast<const typename S::T *>(base) + idx;
    if (DT == KAI_GDN_F32 && VEC == 4) {
        float4 q = __ldg(reinterpret_cast<const float4 *>(p));
        v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    } else if (DT != KAI_GDN_F32 && VEC == 8) {
        uint4 q = __ldg(reinterpret_cast<const uint4 *>(p));
        const typename S::T *h = reinterpret_cast<const typename S::T *>(&q);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = S::load(h + i);
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) v[i] = S::load(p + i);
    }
}

template <int DT, int VEC>
__device__ __forceinline__ void st(void *base, size_t idx, const float (&v)[VEC]) {
    using S = Store<DT>;
    typename S::T *p = static_cast<typename S::T *>(base) + idx;
    if (DT == KAI_GDN_F32 && VEC == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else if (DT != KAI_GDN_F32 && VEC == 8) {
        uint4 q;
        typename S::T *h = reinterpret_cast<typename S::T *>(&q);
#pragma unroll
        for (int i = 0; i < 8; ++i) S::store(h + i, v[i]);
        *reinterpret_cast<uint4 *>(p) = q;
    } else {
#pragma unroll
        for (int i = 0; i < VEC; ++i) S::store(p + i, v[i]);
    }
}

struct ConvParams {
    const void *in;
    const float *w;
    void *out;
    void *hist;
    long long seq, ch;
    int nseg;
};

// One raw 16-byte vector (or one element for the scalar fallback) of a row.
template <int DT, int VEC> struct Raw;
template <int DT> struct Raw<DT, 1> {
    using S = Store<DT>;
    typename S::T v;
    __device__ __forceinline__ void load(const void *base, size_t idx) {
        v = static_cast<const typename S::T *>(base)[idx];
    }
    __device__ __forceinline__ float get(int) const { return S::load(&v); }
};
template <> struct Raw<KAI_GDN_F32, 4> {
    float4 v;
    __device__ __forceinline__ void load(const void *base, size_t idx) {
        v = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(base) + idx));
    }
    __device__ __forceinline__ float get(int i) const { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
};
template <int DT> struct Raw<DT, 8> {
    using S = Store<DT>;
    uint4 v;
    __device__ __forceinline__ void load(const void *base, size_t idx) {
        v = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + idx));
    }
    __device__ __forceinline__ float get(int i) const {
        return S::load(reinterpret_cast<const typename S::T *>(&v) + i);
    }
};

template <int DT, int VEC>
__global__ void __launch_bounds__(THREADS, 2) conv_k4_kernel(ConvParams p) {
    constexpr int R = VEC == 8 ? 4 : 8;  // rows loaded ahead
    const long long c = ((long long)blockIdx.x * THREADS + threadIdx.x) * VEC;
    const int seg = blockIdx.y;
    const long long b = blockIdx.z;
    if (c >= p.ch) return;
    const long long T = p.seq, C = p.ch;
    const size_t xb = (size_t)b * T * C + (size_t)c;   // in/out base
    const size_t hb = (size_t)b * 3 * C + (size_t)c;   // hist base

    float w0[VEC], w1[VEC], w2[VEC], w3[VEC];  // weights: 4*C floats, L2-resident
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        w0[i] = __ldg(p.w + 0 * C + c + i);
        w1[i] = __ldg(p.w + 1 * C + c + i);
        w2[i] = __ldg(p.w + 2 * C + c + i);
        w3[i] = __ldg(p.w + 3 * C + c + i);
    }

    const long long t0 = (long long)seg * SEG;
    const long long t1 = min(t0 + (long long)SEG, T);
    // Window h0 (oldest) .. h2 (newest) = inputs t0-3 .. t0-1.
    float h0[VEC], h1[VEC], h2[VEC];
    {
        Raw<DT, VEC> r0, r1, r2;
        if (seg == 0) {
            r0.load(p.hist, hb + 0 * C);
            r1.load(p.hist, hb + 1 * C);
            r2.load(p.hist, hb + 2 * C);
        } else {
            r0.load(p.in, xb + (size_t)(t0 - 3) * C);
            r1.load(p.in, xb + (size_t)(t0 - 2) * C);
            r2.load(p.in, xb + (size_t)(t0 - 1) * C);
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            h0[i] = r0.get(i);
            h1[i] = r1.get(i);
            h2[i] = r2.get(i);
        }
    }
    auto emit = [&](const Raw<DT, VEC> &cur, long long t) {
        float o[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
            const float x = cur.get(i);
            float acc = __fadd_rn(__fmul_rn(h0[i], w0[i]), __fmul_rn(h1[i], w1[i]));
            acc = __fadd_rn(acc, __fmul_rn(h2[i], w2[i]));
            o[i] = __fadd_rn(acc, __fmul_rn(x, w3[i]));
            h0[i] = h1[i];
            h1[i] = h2[i];
            h2[i] = x;
        }
        st<DT, VEC>(p.out, xb + (size_t)t * C, o);
    };
    long long t = t0;
    for (; t + R <= t1; t += R) {
        Raw<DT, VEC> cur[R];
#pragma unroll
        for (int r = 0; r < R; ++r) cur[r].load(p.in, xb + (size_t)(t + r) * C);
#pragma unroll
        for (int r = 0; r < R; ++r) emit(cur[r], t + r);
    }
    for (; t < t1; ++t) {
        Raw<DT, VEC> cur;
        cur.load(p.in, xb + (size_t)t * C);
        emit(cur, t);
    }
    if (seg == 0) {
        // New history = the last three inputs of the whole call.  With one
        // segment the window already holds them; otherwise read them.
        if (p.nseg > 1) {
            Raw<DT, VEC> r0, r1, r2;
            r0.load(p.in, xb + (size_t)(T - 3) * C);
            r1.load(p.in, xb + (size_t)(T - 2) * C);
            r2.load(p.in, xb + (size_t)(T - 1) * C);
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
                h0[i] = r0.get(i);
                h1[i] = r1.get(i);
                h2[i] = r2.get(i);
            }
        }
        st<DT, VEC>(p.hist, hb + 0 * C, h0);
        st<DT, VEC>(p.hist, hb + 1 * C, h1);
        st<DT, VEC>(p.hist, hb + 2 * C, h2);
    }
}

template <int DT>
int run_conv(ConvParams p, size_t batch, cudaStream_t st) {
    constexpr int VW = DT == KAI_GDN_F32 ? 4 : 8;
    const size_t es = dtype_size(DT);
    bool vec_ok = (p.ch % VW == 0) && ((uintptr_t)p.in % 16 == 0) &&
                  ((uintptr_t)p.out % 16 == 0) && ((uintptr_t)p.hist % 16 == 0) &&
                  ((uintptr_t)p.w % 16 == 0) && ((p.ch * es) % 16 == 0);
    long long nseg = (p.seq + SEG - 1) / SEG;
    if (nseg > 65535 || batch > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "conv: seq/batch too large for the grid");
    p.nseg = (int)nseg;
    int vec = vec_ok ? VW : 1;
    long long gx = (p.ch / vec + THREADS - 1) / THREADS;
    dim3 grid((unsigned)gx, (unsigned)nseg, (unsigned)batch);
    if (vec_ok) conv_k4_kernel<DT, VW><<<grid, THREADS, 0, st>>>(p);
    else conv_k4_kernel<DT, 1><<<grid, THREADS, 0, st>>>(p);
    return check_launch("causal_dwconv1d_k4");
}

}  // namespace

int launch_conv(const void *in, const float *w, void *out, void *hist, int dt,
                size_t batch, size_t seq, size_t ch, cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!in || !w || !out || !hist) return set_error(KAI_GDN_ERR_INVALID, "conv: null pointer");
    ConvParams p{in, w, out, hist, (long long)seq, (long long)ch, 0};
    switch (dt) {
        case KAI_GDN_F32: return run_conv<KAI_GDN_F32>(p, batch, st);
        case KAI_GDN_F16: return run_conv<KAI_GDN_F16>(p, batch, st);
        case KAI_GDN_BF16: return run_conv<KAI_GDN_BF16>(p, batch, st);
    }
    return set_error(KAI_GDN_ERR_INVALID, "conv: bad io dtype %d", dt);
}

}  // namespace gdn
