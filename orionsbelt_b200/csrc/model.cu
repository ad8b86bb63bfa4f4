// model.cu -- decode engine of a Qwen3.5-style GDN hybrid
// on the library's kernels, tensor-parallel over NCCL.
//
// Model (docs/GDN_ARCHITECTURE_AUDIT.md:1-200 for the layer internals; the
// reference's own loop, gdn_e2e_decode.c:2775-2796, has the same block order
// with stand-in layers):
//   h = embed(token)
//   per layer: x = RMSNorm(h)
//     GDN (3 of every 4):  [q|k|v|z|b|a] = x Win;  q, k, v = SiLU(conv_k4([q|k|v]));
//                          q, k L2-normalised per head; beta = sigmoid(b);
//                          g = -exp(A_log) softplus(a + dt_bias);
//                          o = delta-rule decode step (scale 1/sqrt(d));
//                          o = RMSNorm_head(o) w_gn * SiLU(z);  h += o Wout
//     attention (every 4th): [q,gate per head | k | v] = x Wqkv; q, k
//                          RMSNorm per head, RoPE on the first rope_dims dims;
//                          o = GQA decode over the bf16 KV cache (this token
//                          appended); o *= sigmoid(gate);  h += o Wo
//     FFN:                 x = RMSNorm(h);  h += (SiLU(x Wg) * (x Wu)) Wd
//   logits = RMSNorm(h) Wlm;  next token = argmax (greedy)
// Every projection is int8 with one fp32 scale per output column (the
// reference's INT8_WEIGHTS quantize_weight, gdn_e2e_decode.c:175-199) and runs
// on the library's int8 matmul; the embedding table is int8 with one scale per
// token row.  Weights are generated on the device from a seed, N(0, std) by a
// counter hash of (tensor, global row, global column), so every
// tensor-parallel shard holds exactly the codes of the unsharded model.
//
// Tensor parallelism over `tp_size` ranks (one per GPU): GDN key / value heads,
// attention query heads (kv heads split, or replicated when there are fewer
// kv heads than ranks), FFN columns and vocabulary columns are split;
// the output projections (GDN out, attention o, FFN down) are split by rows
// and their partial sums meet in an NCCL all-reduce (sum) of the [B][hidden]
// residual update -- two per layer.  The argmax over the vocabulary shards
// meets in an NCCL all-gather of [B] (value, index) pairs.  NCCL is loaded at
// run time (dlopen of libnccl.so.2, the copy the process already holds if any).
//
// Launches: per token everything but the attention decodes is captured into
// CUDA graphs, one per segment between attention layers (the attention decode
// picks its split count from the context length, so it is launched directly
// with this step's position).  The RoPE kernel reads the position from device
// memory, set by the first launch of each step.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "gdn_internal.cuh"
#include "int8_terms.cuh"

namespace gdn {
namespace {

// ------------------------------------------------------------------ NCCL
struct NcclApi {
    void *h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char *(*errorString)(ncclResult_t) = nullptr;
};
std::mutex g_nccl_mu;
NcclApi g_nccl;

int nccl_api(const NcclApi **out) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (!g_nccl.h) {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return set_error(KAI_GDN_ERR_UNSUPPORTED, "model: libnccl.so.2 not found (%s)", dlerror());
        NcclApi a;
        a.h = h;
        a.getUniqueId = reinterpret_cast<decltype(a.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        a.commInitRank = reinterpret_cast<decltype(a.commInitRank)>(dlsym(h, "ncclCommInitRank"));
        a.allReduce = reinterpret_cast<decltype(a.allReduce)>(dlsym(h, "ncclAllReduce"));
        a.allGather = reinterpret_cast<decltype(a.allGather)>(dlsym(h, "ncclAllGather"));
        a.commDestroy = reinterpret_cast<decltype(a.commDestroy)>(dlsym(h, "ncclCommDestroy"));
        a.errorString = reinterpret_cast<decltype(a.errorString)>(dlsym(h, "ncclGetErrorString"));
        if (!a.getUniqueId || !a.commInitRank || !a.allReduce || !a.allGather || !a.commDestroy || !a.errorString)
            return set_error(KAI_GDN_ERR_UNSUPPORTED, "model: libnccl.so.2 lacks a needed symbol");
        g_nccl = a;
    }
    *out = &g_nccl;
    return KAI_GDN_OK;
}
int check_nccl(const NcclApi *n, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return KAI_GDN_OK;
    return set_error(KAI_GDN_ERR_CUDA, "%s: %s", what, n->errorString(r));
}

// Programmatic dependent launch: every per-token kernel lets its own
// dependents launch at once and waits for the preceding grid before it
// touches memory, so the weight streams of the matmuls that follow start
// early -- even while the matmul before this kernel is still in its tail
// (measured 6.53 -> 6.41 ms per step at batch 16 against waiting first).
// Every dependent waits in turn before reading anything.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
template <typename... KArgs, typename... Args>
int launch_pdl_smem(const char *name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                    Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
    if (e != cudaSuccess) return check_cuda(e, name);
    return check_launch(name);
}
template <typename... KArgs, typename... Args>
int launch_pdl(const char *name, void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    return launch_pdl_smem(name, kernel, grid, block, 0, st, args...);
}

// ------------------------------------------------------------- weights
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// N(0, std) of element (grow0 + r, gcol0 + c) of tensor `tid` (gcols columns
// globally), written to out[r * ld + c]; Box-Muller on two 24-bit uniforms.
__global__ void rng_normal_kernel(float *__restrict__ out, long long rows, long long cols, long long ld,
                                  long long grow0, long long gcol0, long long gcols, unsigned long long seed,
                                  unsigned tid, float stdv) {
    const long long n = rows * cols;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / cols, c = e % cols;
        const unsigned long long idx = (unsigned long long)((grow0 + r) * gcols + gcol0 + c);
        const unsigned long long u = mix64(seed ^ mix64(((unsigned long long)tid << 40) ^ idx));
        const float u1 = ((float)(u >> 40) + 0.5f) * 5.9604644775390625e-8f;
        const float u2 = ((float)(u & 0xFFFFFFull) + 0.5f) * 5.9604644775390625e-8f;
        out[r * ld + c] = stdv * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}
// Uniform(lo, hi) of element idx of tensor `tid` (gate parameters).
__global__ void rng_uniform_kernel(float *__restrict__ out, long long n, long long g0, unsigned long long seed,
                                   unsigned tid, float lo, float hi, int log_of) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const unsigned long long u = mix64(seed ^ mix64(((unsigned long long)tid << 40) ^ (unsigned long long)(g0 + e)));
        const float x = lo + (hi - lo) * (((float)(u >> 40) + 0.5f) * 5.9604644775390625e-8f);
        out[e] = log_of ? logf(x) : x;
    }
}
__global__ void fill_kernel(float *__restrict__ out, long long n, float v) {
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x)
        out[e] = v;
}
// Per-row symmetric int8 quantization (embedding table): s = max|row| / 127.
__global__ void quantize_rows_kernel(const float *__restrict__ x, int8_t *__restrict__ q, float *__restrict__ s,
                                     long long rows, long long cols) {
    const long long r = blockIdx.x;
    if (r >= rows) return;
    __shared__ float red[32];
    float m = 0.f;
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(x[r * cols + c]));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float sc = red[0] / 127.0f;
    if (threadIdx.x == 0) s[r] = sc;
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
        const float v = sc > 0.f ? rintf(x[r * cols + c] / sc) : 0.f;
        q[r * cols + c] = (int8_t)fmaxf(-128.f, fminf(127.f, v));
    }
}

// ------------------------------------------------------------- per token
__device__ __forceinline__ float block_sum(float v, float *red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = threadIdx.x < nw ? red[threadIdx.x] : 0.f;
    if (w == 0)
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void set_pos_kernel(int *pos, int v) { *pos = v; }

// h[b] = E_q[tok[b]] * E_s[tok[b]]
__global__ void embed_kernel(const int *__restrict__ tok, const int8_t *__restrict__ eq, const float *__restrict__ es,
                             float *__restrict__ h, long long H, long long vocab) {
    pdl_enter();
    const long long b = blockIdx.x;
    long long t = tok[b];
    t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const float s = es[t];
    for (long long i = threadIdx.x; i < H; i += blockDim.x) h[b * H + i] = (float)eq[t * H + i] * s;
}
// h += delta (when given); y = h / sqrt(mean(h^2) + eps) * w   (one CTA per row)
__global__ void add_rmsnorm_kernel(float *__restrict__ h, const float *__restrict__ delta, const float *__restrict__ w,
                                   float *__restrict__ y, long long H, float eps) {
    pdl_enter();
    __shared__ float red[32];
    const long long b = blockIdx.x;
    float *hr = h + b * H;
    float ss = 0.f;
    for (long long i = threadIdx.x; i < H; i += blockDim.x) {
        float v = hr[i];
        if (delta) {
            v += delta[b * H + i];
            hr[i] = v;
        }
        ss += v * v;
    }
    const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
    for (long long i = threadIdx.x; i < H; i += blockDim.x) y[b * H + i] = hr[i] * inv * w[i];
}

// GDN input side for one token, one CTA (128 threads) per (b, head) of the
// q, k and v heads of this rank: the Conv1D over [q | k | v] (taps in the
// reference's order, history oldest first), SiLU, L2 normalisation of q and k
// per head; v heads also form beta and g of their head.
//   y     [B][ny]: [q (hk*d) | k (hk*d) | v (hv*d) | z (hv*d) | b (hv) | a (hv) | pad]
//   hist  [B][3][C], C = (2 hk + hv) d;  w [4][C]
__global__ void gdn_prep_kernel(const float *__restrict__ y, long long ny, float *__restrict__ hist,
                                const float *__restrict__ w, const float *__restrict__ A_log,
                                const float *__restrict__ dt_bias, float *__restrict__ q, float *__restrict__ k,
                                float *__restrict__ v, float *__restrict__ beta, float *__restrict__ g, int hk, int hv,
                                int d) {
    pdl_enter();
    __shared__ float red[32];
    const int b = blockIdx.y, head = blockIdx.x, i = threadIdx.x;  // i < d
    const long long C = (long long)(2 * hk + hv) * d;
    const long long ch = (long long)head * d + i;
    float *hb = hist + (long long)b * 3 * C;
    const float x = y[(long long)b * ny + ch];
    const float h0 = hb[ch], h1 = hb[C + ch], h2 = hb[2 * C + ch];
    float c = __fmul_rn(w[ch], h0);
    c = __fadd_rn(c, __fmul_rn(w[C + ch], h1));
    c = __fadd_rn(c, __fmul_rn(w[2 * C + ch], h2));
    c = __fadd_rn(c, __fmul_rn(w[3 * C + ch], x));
    hb[ch] = h1;
    hb[C + ch] = h2;
    hb[2 * C + ch] = x;
    const float s = silu(c);
    if (head < 2 * hk) {
        const float inv = rsqrtf(block_sum(s * s, red) + 1e-6f);
        if (head < hk)
            q[((long long)b * hk + head) * d + i] = s * inv;
        else
            k[((long long)b * hk + head - hk) * d + i] = s * inv;
    } else {
        const int vh = head - 2 * hk;
        v[((long long)b * hv + vh) * d + i] = s;
        if (i == 0) {
            const long long zoff = C + (long long)hv * d;
            const float bb = y[(long long)b * ny + zoff + vh], aa = y[(long long)b * ny + zoff + hv + vh];
            const float xa = aa + dt_bias[vh];
            const float sp = xa > 20.f ? xa : log1pf(expf(xa));
            beta[(long long)b * hv + vh] = sigm(bb);
            g[(long long)b * hv + vh] = -expf(A_log[vh]) * sp;
        }
    }
}
// o_head = o / sqrt(mean(o^2) + eps) * w * SiLU(z)   (one CTA of d threads per (b, head))
__global__ void gated_rmsnorm_kernel(const float *__restrict__ o, const float *__restrict__ y, long long ny,
                                     long long zoff, const float *__restrict__ w, float *__restrict__ out, int hv,
                                     int d, float eps) {
    pdl_enter();
    __shared__ float red[32];
    const int b = blockIdx.y, hh = blockIdx.x, i = threadIdx.x;
    const long long idx = ((long long)b * hv + hh) * d + i;
    const float x = o[idx];
    const float inv = rsqrtf(block_sum(x * x, red) / (float)d + eps);
    const float z = y[(long long)b * ny + zoff + (long long)hh * d + i];
    out[idx] = x * inv * w[i] * silu(z);
}
// Attention input side: per (b, query head) [query | gate] and per (b, kv
// head) k, v from y [B][ny] = [per q head: query (D) | gate (D) ... | k (hkv*D) | v (hkv*D)];
// query and key RMSNormed per head, RoPE (pairs i, i + R/2 of the first R dims)
// at the position in *pos.  One CTA of D threads per head row.
__global__ void attn_prep_kernel(const float *__restrict__ y, long long ny, const float *__restrict__ wq,
                                 const float *__restrict__ wk, const int *__restrict__ pos_p, float *__restrict__ q,
                                 float *__restrict__ gate, float *__restrict__ kn, float *__restrict__ vn, int hq,
                                 int hkv, int D, int R, float theta, float eps) {
    pdl_enter();
    __shared__ float red[32];
    __shared__ float row[512];
    const int b = blockIdx.y, r = blockIdx.x, i = threadIdx.x;  // r < hq + 2 hkv
    const float pos = (float)*pos_p;
    const float *yr = y + (long long)b * ny;
    if (r >= hq + hkv) {  // v
        const int kv = r - hq - hkv;
        vn[((long long)b * hkv + kv) * D + i] = yr[(long long)hq * 2 * D + (long long)(hkv + kv) * D + i];
        return;
    }
    const bool isq = r < hq;
    const float x = isq ? yr[(long long)r * 2 * D + i] : yr[(long long)hq * 2 * D + (long long)(r - hq) * D + i];
    if (isq) gate[((long long)b * hq + r) * D + i] = yr[(long long)r * 2 * D + D + i];
    const float inv = rsqrtf(block_sum(x * x, red) / (float)D + eps);
    const float nx = x * inv * (isq ? wq[i] : wk[i]);
    row[i] = nx;
    __syncthreads();
    float outv = nx;
    if (i < R) {
        const int half = R / 2, j = i < half ? i : i - half;
        const float inv_freq = powf(theta, -2.0f * (float)j / (float)R);
        float sn, cs;
        sincosf(pos * inv_freq, &sn, &cs);
        outv = i < half ? nx * cs - row[i + half] * sn : row[i - half] * sn + nx * cs;
    }
    if (isq)
        q[((long long)b * hq + r) * D + i] = outv;
    else
        kn[((long long)b * hkv + (r - hq)) * D + i] = outv;
}
__global__ void attn_gate_kernel(const float *__restrict__ o, const float *__restrict__ gate, float *__restrict__ out,
                                 long long n) {
    pdl_enter();
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x)
        out[e] = o[e] * sigm(gate[e]);
}
// act = SiLU(gate) * up over rows [gate (I) | up (I)]
__global__ void swiglu_kernel(const float *__restrict__ gu, float *__restrict__ act, long long I, long long n) {
    pdl_enter();
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long b = e / I, c = e % I;
        act[e] = silu(gu[b * 2 * I + c]) * gu[b * 2 * I + I + c];
    }
}
// ------------------------------------------------------------------
// Producers that write a projection's input straight as the packed int8
// matmul's activation terms (int8_terms.cuh), for batches the tensor-core
// stream serves: each is the elementwise kernel above with the row kept in
// shared memory, its largest magnitude reduced and its terms written, so the
// fp32 row never goes through memory and one launch per projection is saved.
// One CTA (1024 threads) per row; dynamic shared memory holds the row.
__device__ __forceinline__ float block_max(float v, float *red) {
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = threadIdx.x < nw ? red[threadIdx.x] : 0.f;
    if (w == 0)
        for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) red[0] = t;
    __syncthreads();
    return red[0];
}
// h += delta (when given); terms of h / sqrt(mean(h^2) + eps) * w   (add_rmsnorm_kernel)
__global__ void addnorm_terms_kernel(float *__restrict__ h, const float *__restrict__ delta,
                                     const float *__restrict__ w, long long H, float eps, long long S,
                                     int8_t *__restrict__ terms, float *__restrict__ scale) {
    pdl_enter();
    extern __shared__ float xs[];
    __shared__ float red[32];
    const long long b = blockIdx.x;
    float *hr = h + b * H;
    float ss = 0.f;
    for (long long i = threadIdx.x; i < H; i += blockDim.x) {
        float v = hr[i];
        if (delta) {
            v += delta[b * H + i];
            hr[i] = v;
        }
        xs[i] = v;
        ss += v * v;
    }
    const float inv = rsqrtf(block_sum(ss, red) / (float)H + eps);
    float mx = 0.f;
    for (long long i = threadIdx.x; i < H; i += blockDim.x) {
        const float x = xs[i] * inv * w[i];
        xs[i] = x;
        mx = fmaxf(mx, fabsf(x));
    }
    mx = block_max(mx, red);
    terms::write_row(xs, H, S, mx, terms, scale, 16, b);
}
// terms of SiLU(gate) * up over rows [gate (I) | up (I)]   (swiglu_kernel)
__global__ void swiglu_terms_kernel(const float *__restrict__ gu, long long I, long long S, int8_t *__restrict__ terms,
                                    float *__restrict__ scale) {
    pdl_enter();
    extern __shared__ float xs[];
    __shared__ float red[32];
    const long long b = blockIdx.x;
    float mx = 0.f;
    for (long long c = threadIdx.x; c < I; c += blockDim.x) {
        const float x = silu(gu[b * 2 * I + c]) * gu[b * 2 * I + I + c];
        xs[c] = x;
        mx = fmaxf(mx, fabsf(x));
    }
    mx = block_max(mx, red);
    terms::write_row(xs, I, S, mx, terms, scale, 16, b);
}
// terms of o_head / sqrt(mean(o_head^2) + eps) * w * SiLU(z)   (gated_rmsnorm_kernel);
// a warp per head
__global__ void gatednorm_terms_kernel(const float *__restrict__ o, const float *__restrict__ y, long long ny,
                                       long long zoff, const float *__restrict__ w, int hv, int d, float eps,
                                       long long S, int8_t *__restrict__ terms, float *__restrict__ scale) {
    pdl_enter();
    extern __shared__ float xs[];
    __shared__ float red[32];
    const long long b = blockIdx.x;
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float mx = 0.f;
    for (int hh = wp; hh < hv; hh += nw) {
        const float *orow = o + ((long long)b * hv + hh) * d;
        float ss = 0.f;
        for (int i = lane; i < d; i += 32) ss += orow[i] * orow[i];
        for (int m = 16; m; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
        const float inv = rsqrtf(ss / (float)d + eps);
        for (int i = lane; i < d; i += 32) {
            const float x = orow[i] * inv * w[i] * silu(y[b * ny + zoff + (long long)hh * d + i]);
            xs[hh * d + i] = x;
            mx = fmaxf(mx, fabsf(x));
        }
    }
    mx = block_max(mx, red);
    terms::write_row(xs, (long long)hv * d, S, mx, terms, scale, 16, b);
}
// terms of o * sigmoid(gate)   (attn_gate_kernel)
__global__ void attngate_terms_kernel(const float *__restrict__ o, const float *__restrict__ gate, long long n,
                                      long long S, int8_t *__restrict__ terms, float *__restrict__ scale) {
    pdl_enter();
    extern __shared__ float xs[];
    __shared__ float red[32];
    const long long b = blockIdx.x;
    float mx = 0.f;
    for (long long i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = o[b * n + i] * sigm(gate[b * n + i]);
        xs[i] = x;
        mx = fmaxf(mx, fabsf(x));
    }
    mx = block_max(mx, red);
    terms::write_row(xs, n, S, mx, terms, scale, 16, b);
}

// Per row: the largest logit and its global index (smallest index on ties).
struct ArgMax {
    float v;
    int i;
};
// Grid (AM_BLOCKS, B): block x of row b scans columns x, x + AM_BLOCKS * 256, ...
// and writes its candidate to out[b * AM_BLOCKS + x].
constexpr int AM_BLOCKS = 64;
__global__ void argmax_kernel(const float *__restrict__ logits, long long V, long long v0, ArgMax *__restrict__ out) {
    pdl_enter();
    __shared__ float sv[32];
    __shared__ int si[32];
    const long long b = blockIdx.y;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < V; c += (long long)gridDim.x * blockDim.x) {
        const float x = logits[b * V + c];
        if (x > best || (x == best && (int)(v0 + c) < bi)) {
            best = x;
            bi = (int)(v0 + c);
        }
    }
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
            if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
                best = sv[w];
                bi = si[w];
            }
        out[b * gridDim.x + blockIdx.x] = {best, bi};
    }
}
// tok[b] = argmax over the candidates all[r][b][0 .. per) of every rank r
__global__ void select_kernel(const ArgMax *__restrict__ all, int world, int B, int per, int *__restrict__ tok) {
    pdl_enter();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    ArgMax best = all[(long long)b * per];
    for (int r = 0; r < world; ++r)
        for (int j = 0; j < per; ++j) {
            const ArgMax c = all[((long long)r * B + b) * per + j];
            if (c.v > best.v || (c.v == best.v && c.i < best.i)) best = c;
        }
    tok[b] = best.i;
}

unsigned grid_for(long long n) { return (unsigned)std::min<long long>((n + 255) / 256, 8ll * sm_count()); }

struct QW {
    int8_t *q = nullptr;   // [K][N]
    int8_t *qb = nullptr;  // the same codes in the GEMV's blocked layout (small batches)
    int8_t *qp = nullptr;  // the same codes packed for the tensor-core stream (larger batches, LM head)
    float *s = nullptr;
    size_t K = 0, N = 0;
};
struct Part {
    unsigned tid;
    size_t gcols, col0, ncols;  // global width of the tensor, first global column, columns taken
};

}  // namespace

struct ModelEngine {
    kai_gdn_model_config cfg{};
    std::vector<unsigned char> is_gdn;
    int device = 0;
    // local widths
    size_t hk = 0, hv = 0, d = 0, C = 0, ny_gdn = 0, hq = 0, hkv = 0, D = 0, ny_att = 0, I = 0, V = 0, v0 = 0;
    size_t kv_first = 0;  // first global kv head of this rank
    struct Layer {
        QW win, wout, wgu, wdown;
        float *w_in = nullptr, *w_post = nullptr, *conv_w = nullptr, *A_log = nullptr, *dt_bias = nullptr,
              *w_gn = nullptr, *w_qn = nullptr, *w_kn = nullptr;
        float *state = nullptr, *hist = nullptr;  // GDN: [B][hv][d][d], [B][3][C]
        void *kc = nullptr, *vc = nullptr;        // attention: [B][max_ctx][hkv][D] bf16
    };
    std::vector<Layer> layers;
    QW lm;
    int8_t *emb_q = nullptr;
    float *emb_s = nullptr, *w_final = nullptr;
    // activations
    float *h = nullptr, *x = nullptr, *y = nullptr, *part = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
          *beta = nullptr, *g = nullptr, *o = nullptr, *o2 = nullptr, *gate = nullptr, *gu = nullptr, *act = nullptr,
          *logits = nullptr;
    int *tok = nullptr, *pos = nullptr;
    ArgMax *cand = nullptr, *cand_all = nullptr;
    std::vector<void *> allocs;
    // batches the tensor-core stream serves: projection inputs go straight
    // to activation terms (fused producers)
    bool fused = false;
    int8_t *terms = nullptr;
    float *tscale = nullptr;
    // prompt workspace (grown on demand by model_prefill): per-token rows
    struct Prompt {
        void *base = nullptr;
        size_t T = 0;
        float *h, *x, *part, *y, *q, *k, *v, *beta, *g, *o, *o2, *gate, *gu, *act;
        int *tok;
    } pf;
    const NcclApi *nccl = nullptr;
    ncclComm_t comm = nullptr;
    // graphs: segment s runs from attention layer s-1 (after its decode) to
    // attention layer s (before its decode); the last one ends with the argmax
    std::vector<size_t> attn_layers;
    std::vector<cudaGraphExec_t> seg;
    cudaStream_t graph_stream = nullptr, last_stream = nullptr;
    int steps = 0;
};

namespace {

int malloc_keep(ModelEngine *e, void **p, size_t bytes, bool zero) {
    int rc = check_cuda(cudaMalloc(p, std::max<size_t>(bytes, 256)), "model: cudaMalloc");
    if (rc) return rc;
    e->allocs.push_back(*p);
    if (zero) rc = check_cuda(cudaMemset(*p, 0, std::max<size_t>(bytes, 256)), "model: cudaMemset");
    return rc;
}

// A [K][N] int8 projection of this rank: the column parts (each a column range
// of a global tensor) side by side, rows [k0, k1) of the global K rows; the
// per-column scales come from all K rows, as in the unsharded model.
// Which kernel streams a projection: the CUDA-core GEMV for batch <= 4 (one
// launch, no activation preparation), the int8 tensor-core stream above that
// and for the LM head at every batch (measured faster there from batch 1).
constexpr size_t GEMV_MAX_BATCH = 4;

int build_qw(ModelEngine *e, QW *w, size_t K, size_t k0, size_t k1, const std::vector<Part> &parts, float stdv,
             bool lm_head = false) {
    size_t N = 0;
    for (const Part &p : parts) N += p.ncols;
    float *tmp = nullptr;
    int8_t *qt = nullptr;
    int rc = check_cuda(cudaMalloc(&tmp, K * N * sizeof(float)), "model: weight workspace");
    if (!rc) rc = check_cuda(cudaMalloc(&qt, K * N), "model: weight workspace");
    size_t col = 0;
    for (const Part &p : parts) {
        if (rc) break;
        rng_normal_kernel<<<grid_for((long long)(K * p.ncols)), 256>>>(tmp + col, (long long)K, (long long)p.ncols,
                                                                      (long long)N, 0, (long long)p.col0,
                                                                      (long long)p.gcols, e->cfg.seed, p.tid, stdv);
        rc = check_launch("rng_normal_kernel");
        col += p.ncols;
    }
    if (!rc) rc = malloc_keep(e, (void **)&w->s, N * sizeof(float), false);
    if (!rc) rc = launch_quantize_int8(tmp, qt, w->s, K, N, 0);
    if (!rc) rc = malloc_keep(e, (void **)&w->q, (k1 - k0) * N, false);
    if (!rc) rc = check_cuda(cudaMemcpy(w->q, qt + k0 * N, (k1 - k0) * N, cudaMemcpyDeviceToDevice), "model: codes");
    const size_t B = e->cfg.batch;
    // packed for the tensor-core stream (decode above batch 4, the LM head,
    // every prompt), and blocked for the GEMV where small batches decode
    if (!rc && int8_packed_supported(k1 - k0, N)) {
        if (!(rc = malloc_keep(e, (void **)&w->qp, int8_packed_bytes(k1 - k0, N), false)))
            rc = int8_pack_weights(w->q, w->qp, k1 - k0, N, 0);
    }
    if (!rc && !lm_head && B <= GEMV_MAX_BATCH && gemv_int8_supported(B, k1 - k0, N, w->q)) {
        if (!(rc = malloc_keep(e, (void **)&w->qb, gemv_blocked_bytes(B, k1 - k0, N), false)))
            rc = gemv_block_weights(B, w->q, w->qb, k1 - k0, N, 0);
    }
    if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "model: weights");
    if (tmp) cudaFree(tmp);
    if (qt) cudaFree(qt);
    w->K = k1 - k0;
    w->N = N;
    return rc;
}
int vec_normal(ModelEngine *e, float **p, size_t n, size_t g0, unsigned tid, float stdv, float mean) {
    int rc = malloc_keep(e, (void **)p, n * sizeof(float), false);
    if (rc) return rc;
    rng_normal_kernel<<<grid_for((long long)n), 256>>>(*p, 1, (long long)n, (long long)n, 0, (long long)g0,
                                                       (long long)n, e->cfg.seed, tid, stdv);
    if ((rc = check_launch("rng_normal_kernel"))) return rc;
    if (mean != 0.f) {
        // mean + N(0, std): used for the norm weights (1 + N(0, std))
        std::vector<float> hbuf(n);
        rc = check_cuda(cudaMemcpy(hbuf.data(), *p, n * sizeof(float), cudaMemcpyDeviceToHost), "model: vec");
        for (float &x : hbuf) x += mean;
        if (!rc) rc = check_cuda(cudaMemcpy(*p, hbuf.data(), n * sizeof(float), cudaMemcpyHostToDevice), "model: vec");
    }
    return rc;
}
int vec_const(ModelEngine *e, float **p, size_t n, float v) {
    int rc = malloc_keep(e, (void **)p, n * sizeof(float), false);
    if (rc) return rc;
    fill_kernel<<<grid_for((long long)n), 256>>>(*p, (long long)n, v);
    return check_launch("fill_kernel");
}

// tensor ids: 64 per layer
enum : unsigned {
    T_Q = 0, T_K, T_V, T_Z, T_B, T_A, T_PAD, T_OUT, T_CONV, T_ALOG, T_DT, T_GN, T_AQ, T_AK, T_AV, T_AO, T_QN, T_KN,
    T_GATE, T_UP, T_DOWN, T_NIN, T_NPOST,
    T_LM = 0xFFFF00, T_EMB, T_FINAL
};
unsigned tidl(size_t layer, unsigned kind) { return (unsigned)(layer * 64 + kind); }

int mm(const float *A, const QW &w, float *Cm, size_t M, cudaStream_t st) {
    if (w.qb && M <= GEMV_MAX_BATCH) return launch_gemv_int8_blocked(A, w.qb, w.s, Cm, M, w.K, w.N, st);
    if (w.qp) return launch_matmul_int8_packed(A, w.qp, w.s, Cm, M, w.K, w.N, st);
    return launch_matmul_int8(A, w.q, w.s, Cm, M, w.K, w.N, st);
}
// A projection of this step's rows together with the producer of its input:
// the fp32 elementwise kernel then mm(), or (fused batches) the producer
// writing the activation terms then the packed weight stream over them.
long long kstages(size_t K) { return (long long)((K + 63) / 64); }
int terms_mm(ModelEngine *e, const QW &w, float *Cm, cudaStream_t st) {
    return launch_matmul_int8_packed_terms(e->terms, e->tscale, w.qp, w.s, Cm, e->cfg.batch, w.K, w.N, st);
}
// h += delta; Cm = RMSNorm(h) w
int norm_mm(ModelEngine *e, const float *delta, const float *wn, const QW &w, float *Cm, cudaStream_t st) {
    const size_t B = e->cfg.batch, H = e->cfg.hidden;
    int rc;
    if (e->fused) {
        rc = launch_pdl_smem("addnorm_terms_kernel", addnorm_terms_kernel, dim3((unsigned)B), dim3(1024),
                             H * sizeof(float), st, e->h, delta, wn, (long long)H, e->cfg.rms_eps, kstages(H), e->terms,
                             e->tscale);
        return rc ? rc : terms_mm(e, w, Cm, st);
    }
    rc = launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel, dim3((unsigned)B), dim3(1024), st, e->h, delta, wn, e->x,
                    (long long)H, e->cfg.rms_eps);
    return rc ? rc : mm(e->x, w, Cm, B, st);
}
// Cm = SwiGLU(gu) w
int swiglu_mm(ModelEngine *e, const QW &w, float *Cm, cudaStream_t st) {
    const size_t B = e->cfg.batch, I = e->I;
    int rc;
    if (e->fused) {
        rc = launch_pdl_smem("swiglu_terms_kernel", swiglu_terms_kernel, dim3((unsigned)B), dim3(1024),
                             I * sizeof(float), st, e->gu, (long long)I, kstages(I), e->terms, e->tscale);
        return rc ? rc : terms_mm(e, w, Cm, st);
    }
    if (w.qb && B <= GEMV_MAX_BATCH)  // the GEMV applies SiLU(gate) * up as it loads its activations
        return launch_gemv_int8_blocked(e->gu, w.qb, w.s, Cm, B, w.K, w.N, st, true);
    rc = launch_pdl("swiglu_kernel", swiglu_kernel, dim3(grid_for((long long)(B * I))), dim3(256), st, e->gu, e->act,
                    (long long)I, (long long)(B * I));
    return rc ? rc : mm(e->act, w, Cm, B, st);
}
// Cm = RMSNormGated(o, z) w   (GDN output side)
int gatednorm_mm(ModelEngine *e, const float *wn, const QW &w, float *Cm, cudaStream_t st) {
    const size_t B = e->cfg.batch, d = e->d;
    int rc;
    if (e->fused) {
        rc = launch_pdl_smem("gatednorm_terms_kernel", gatednorm_terms_kernel, dim3((unsigned)B), dim3(1024),
                             e->hv * d * sizeof(float), st, e->o, e->y, (long long)e->ny_gdn, (long long)e->C, wn,
                             (int)e->hv, (int)d, e->cfg.rms_eps, kstages(e->hv * d), e->terms, e->tscale);
        return rc ? rc : terms_mm(e, w, Cm, st);
    }
    rc = launch_pdl("gated_rmsnorm_kernel", gated_rmsnorm_kernel, dim3((unsigned)e->hv, (unsigned)B), dim3((unsigned)d), st,
                    e->o, e->y, (long long)e->ny_gdn, (long long)e->C, wn, e->o2, (int)e->hv, (int)d, e->cfg.rms_eps);
    return rc ? rc : mm(e->o2, w, Cm, B, st);
}
// Cm = (o * sigmoid(gate)) w   (attention output side)
int attngate_mm(ModelEngine *e, const QW &w, float *Cm, cudaStream_t st) {
    const size_t B = e->cfg.batch, n = e->hq * e->D;
    int rc;
    if (e->fused) {
        rc = launch_pdl_smem("attngate_terms_kernel", attngate_terms_kernel, dim3((unsigned)B), dim3(1024),
                             n * sizeof(float), st, e->o, e->gate, (long long)n, kstages(n), e->terms, e->tscale);
        return rc ? rc : terms_mm(e, w, Cm, st);
    }
    rc = launch_pdl("attn_gate_kernel", attn_gate_kernel, dim3(grid_for((long long)(B * n))), dim3(256), st, e->o,
                    e->gate, e->o2, (long long)(B * n));
    return rc ? rc : mm(e->o2, w, Cm, B, st);
}
int allreduce(ModelEngine *e, float *buf, size_t n, cudaStream_t st) {
    if (e->cfg.tp_size <= 1) return KAI_GDN_OK;
    return check_nccl(e->nccl, e->nccl->allReduce(buf, buf, n, ncclFloat32, ncclSum, e->comm, st), "model: all-reduce");
}

// The greedy token of every sequence from this rank's logits [B][V] (an
// all-gather of the candidates across ranks).
int select_tokens(ModelEngine *e, cudaStream_t st) {
    const kai_gdn_model_config &c = e->cfg;
    const size_t B = c.batch;
    int rc = launch_pdl("argmax_kernel", argmax_kernel, dim3(dim3(AM_BLOCKS, (unsigned)B)), dim3(256), st, e->logits,
                        (long long)e->V, (long long)e->v0, e->cand);
    if (!rc && c.tp_size > 1)
        rc = check_nccl(e->nccl, e->nccl->allGather(e->cand, e->cand_all, B * AM_BLOCKS * 2, ncclFloat32, e->comm, st),
                        "model: all-gather");
    if (!rc)
        rc = launch_pdl("select_kernel", select_kernel, dim3((unsigned)((B + 127) / 128)), dim3(128), st,
                        c.tp_size > 1 ? e->cand_all : e->cand, c.tp_size > 1 ? c.tp_size : 1, (int)B, AM_BLOCKS,
                        e->tok);
    return rc;
}
// LM head over this rank's vocabulary and the greedy tokens, from the
// final-normed rows x [B][H].
int lm_head(ModelEngine *e, cudaStream_t st) {
    int rc = mm(e->x, e->lm, e->logits, e->cfg.batch, st);
    return rc ? rc : select_tokens(e, st);
}

// Segment s of a token (see ModelEngine::seg).
int run_segment(ModelEngine *e, size_t s, cudaStream_t st) {
    const kai_gdn_model_config &c = e->cfg;
    const size_t B = c.batch, H = c.hidden;
    const size_t l_begin = s == 0 ? 0 : e->attn_layers[s - 1];
    const size_t l_end = s < e->attn_layers.size() ? e->attn_layers[s] : c.layers;
    int rc = 0;
#define M_TRY(x)                   \
    do {                           \
        if ((rc = (x))) return rc; \
    } while (0)
    const float *pending = nullptr;  // residual update still to be added to h
    if (s == 0) {
        M_TRY(launch_pdl("embed_kernel", embed_kernel, dim3((unsigned)B), dim3(1024), st, e->tok, e->emb_q, e->emb_s, e->h, (long long)H,
                                                  (long long)c.vocab));
    } else {
        // the rest of attention layer l_begin: gate, o projection, FFN
        const ModelEngine::Layer &L = e->layers[l_begin];
        M_TRY(attngate_mm(e, L.wout, e->part, st));
        M_TRY(allreduce(e, e->part, B * H, st));
        M_TRY(norm_mm(e, e->part, L.w_post, L.wgu, e->gu, st));
        M_TRY(swiglu_mm(e, L.wdown, e->part, st));
        M_TRY(allreduce(e, e->part, B * H, st));
        pending = e->part;
    }
    const size_t first = s == 0 ? 0 : l_begin + 1;
    for (size_t l = first; l < l_end || (l == l_end && l < c.layers); ++l) {
        const ModelEngine::Layer &L = e->layers[l];
        M_TRY(norm_mm(e, pending, L.w_in, L.win, e->y, st));
        pending = nullptr;
        if (l == l_end) {
            // attention layer: projections and the prepared q / k / v; the
            // decode itself follows this segment
            M_TRY(launch_pdl("attn_prep_kernel", attn_prep_kernel, dim3(dim3((unsigned)(e->hq + 2 * e->hkv), (unsigned)B)), dim3((unsigned)e->D), st, e->y, (long long)e->ny_att, L.w_qn, L.w_kn, e->pos, e->q, e->gate, e->k, e->v, (int)e->hq,
                (int)e->hkv, (int)e->D, (int)c.rope_dims, c.rope_theta, c.rms_eps));
            return KAI_GDN_OK;
        }
        // GDN layer
        M_TRY(launch_pdl("gdn_prep_kernel", gdn_prep_kernel, dim3(dim3((unsigned)(2 * e->hk + e->hv), (unsigned)B)), dim3((unsigned)e->d), st, e->y, (long long)e->ny_gdn, L.hist, L.conv_w, L.A_log, L.dt_bias, e->q, e->k, e->v, e->beta, e->g,
            (int)e->hk, (int)e->hv, (int)e->d));
        kai_gdn_decode_args da{};
        da.state = L.state;
        da.q = e->q;
        da.k = e->k;
        da.v = e->v;
        da.g = e->g;
        da.beta = e->beta;
        da.o = e->o;
        da.batch = B;
        da.heads_k = e->hk;
        da.heads_v = e->hv;
        da.dk = e->d;
        da.dv = e->d;
        da.scale = 1.0f / sqrtf((float)e->d);
        da.in_dtype = KAI_GDN_F32;
        da.state_dtype = KAI_GDN_F32;
        da.out_dtype = KAI_GDN_F32;
        M_TRY(launch_decode(&da, st));
        M_TRY(gatednorm_mm(e, L.w_gn, L.wout, e->part, st));
        M_TRY(allreduce(e, e->part, B * H, st));
        M_TRY(norm_mm(e, e->part, L.w_post, L.wgu, e->gu, st));
        M_TRY(swiglu_mm(e, L.wdown, e->part, st));
        M_TRY(allreduce(e, e->part, B * H, st));
        pending = e->part;
    }
    // end of the token: final norm, LM head over this rank's vocabulary, argmax
    M_TRY(norm_mm(e, pending, e->w_final, e->lm, e->logits, st));
    M_TRY(select_tokens(e, st));
#undef M_TRY
    return KAI_GDN_OK;
}

int run_attention(ModelEngine *e, size_t layer, size_t pos, cudaStream_t st) {
    const ModelEngine::Layer &L = e->layers[layer];
    kai_gdn_attn_decode_args a{};
    a.q = e->q;
    a.k_new = e->k;
    a.v_new = e->v;
    a.k_cache = L.kc;
    a.v_cache = L.vc;
    a.o = e->o;
    a.batch = e->cfg.batch;
    a.heads = e->hq;
    a.kv_heads = e->hkv;
    a.head_dim = e->D;
    a.pos = pos;
    a.max_ctx = e->cfg.max_ctx;
    a.scale = 1.0f / sqrtf((float)e->D);
    a.cache_dtype = KAI_GDN_BF16;
    return launch_attn_decode(&a, st);
}

int run_token(ModelEngine *e, size_t pos, cudaStream_t st, bool use_graphs) {
    int rc = 0;
    set_pos_kernel<<<1, 1, 0, st>>>(e->pos, (int)pos);
    if ((rc = check_launch("set_pos_kernel"))) return rc;
    const size_t nseg = e->attn_layers.size() + 1;
    for (size_t s = 0; s < nseg; ++s) {
        if (use_graphs)
            rc = check_cuda(cudaGraphLaunch(e->seg[s], st), "model: graph launch");
        else
            rc = run_segment(e, s, st);
        if (rc) return rc;
        if (s < e->attn_layers.size() && (rc = run_attention(e, e->attn_layers[s], pos, st))) return rc;
    }
    return KAI_GDN_OK;
}


// ---------------------------------------------------------------- prompt
// The prompt of one sequence runs as whole-prompt launches, layer by layer:
// projections with M = T rows, the GDN layers' conv and gates per token and
// the chunked delta-rule scan from the sequence's state, the attention
// layers' keys and values written into the cache and the causal prompt
// attention.  The state a decode step needs afterwards -- conv histories,
// GDN states, KV caches, the last token's hidden state -- is what T decode
// steps would leave.

// GDN input side for every prompt token, one CTA (d threads) per (head,
// token): the Conv1D over the three inputs before the token (the history for
// the first three) in the decode step's order of operations, SiLU, L2
// normalisation of q and k, beta and g of the value heads.
//   y [T][ny] rows as gdn_prep_kernel's; hist [3][C] (read only here)
//   q, k [T][hk][d], v [T][hv][d], beta, g [T][hv]
__global__ void gdn_prompt_prep_kernel(const float *__restrict__ y, long long ny, const float *__restrict__ hist,
                                       const float *__restrict__ w, const float *__restrict__ A_log,
                                       const float *__restrict__ dt_bias, float *__restrict__ q, float *__restrict__ k,
                                       float *__restrict__ v, float *__restrict__ beta, float *__restrict__ g, int hk,
                                       int hv, int d) {
    pdl_enter();
    __shared__ float red[32];
    const long long t = blockIdx.y;
    const int head = blockIdx.x, i = threadIdx.x;
    const long long C = (long long)(2 * hk + hv) * d;
    const long long ch = (long long)head * d + i;
    auto in = [&](long long u) { return u >= 0 ? y[u * ny + ch] : hist[(3 + u) * C + ch]; };
    const float x = y[t * ny + ch], h0 = in(t - 3), h1 = in(t - 2), h2 = in(t - 1);
    float c = __fmul_rn(w[ch], h0);
    c = __fadd_rn(c, __fmul_rn(w[C + ch], h1));
    c = __fadd_rn(c, __fmul_rn(w[2 * C + ch], h2));
    c = __fadd_rn(c, __fmul_rn(w[3 * C + ch], x));
    const float s = silu(c);
    if (head < 2 * hk) {
        const float inv = rsqrtf(block_sum(s * s, red) + 1e-6f);
        if (head < hk)
            q[(t * hk + head) * d + i] = s * inv;
        else
            k[(t * hk + head - hk) * d + i] = s * inv;
    } else {
        const int vh = head - 2 * hk;
        v[(t * hv + vh) * d + i] = s;
        if (i == 0) {
            const long long zoff = C + (long long)hv * d;
            const float bb = y[t * ny + zoff + vh], aa = y[t * ny + zoff + hv + vh];
            const float xa = aa + dt_bias[vh];
            const float sp = xa > 20.f ? xa : log1pf(expf(xa));
            beta[t * hv + vh] = sigm(bb);
            g[t * hv + vh] = -expf(A_log[vh]) * sp;
        }
    }
}
// The conv history after the prompt: its last three inputs (older history
// where the prompt is shorter than three).
__global__ void gdn_prompt_hist_kernel(const float *__restrict__ y, long long ny, float *__restrict__ hist,
                                       long long C, long long T) {
    pdl_enter();
    for (long long ch = blockIdx.x * (long long)blockDim.x + threadIdx.x; ch < C; ch += (long long)gridDim.x * blockDim.x) {
        float nh[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            const long long u = T - 3 + j;
            nh[j] = u >= 0 ? y[u * ny + ch] : hist[(3 + u) * C + ch];
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) hist[j * C + ch] = nh[j];
    }
}
// Attention input side for every prompt token (attn_prep_kernel's
// arithmetic at position pos0 + t): query and gate rows to q / gate
// [T][hq][D], RMSNormed and rotated keys and the values straight into the
// bf16 caches at their positions.  One CTA of D threads per (head row, token).
__global__ void attn_prompt_prep_kernel(const float *__restrict__ y, long long ny, const float *__restrict__ wq,
                                        const float *__restrict__ wk, long long pos0, float *__restrict__ q,
                                        float *__restrict__ gate, __nv_bfloat16 *__restrict__ kc,
                                        __nv_bfloat16 *__restrict__ vc, int hq, int hkv, int D, int R, float theta,
                                        float eps) {
    pdl_enter();
    __shared__ float red[32];
    __shared__ float row[512];
    const long long t = blockIdx.y;
    const int r = blockIdx.x, i = threadIdx.x;
    const long long pos = pos0 + t;
    const float *yr = y + t * ny;
    if (r >= hq + hkv) {  // v
        const int kv = r - hq - hkv;
        vc[(pos * hkv + kv) * D + i] = __float2bfloat16_rn(yr[(long long)hq * 2 * D + (long long)(hkv + kv) * D + i]);
        return;
    }
    const bool isq = r < hq;
    const float x = isq ? yr[(long long)r * 2 * D + i] : yr[(long long)hq * 2 * D + (long long)(r - hq) * D + i];
    if (isq) gate[(t * hq + r) * D + i] = yr[(long long)r * 2 * D + D + i];
    const float inv = rsqrtf(block_sum(x * x, red) / (float)D + eps);
    const float nx = x * inv * (isq ? wq[i] : wk[i]);
    row[i] = nx;
    __syncthreads();
    float outv = nx;
    if (i < R) {
        const int half = R / 2, j = i < half ? i : i - half;
        const float inv_freq = powf(theta, -2.0f * (float)j / (float)R);
        float sn, cs;
        sincosf((float)pos * inv_freq, &sn, &cs);
        outv = i < half ? nx * cs - row[i + half] * sn : row[i - half] * sn + nx * cs;
    }
    if (isq)
        q[(t * hq + r) * D + i] = outv;
    else
        kc[(pos * hkv + (r - hq)) * D + i] = __float2bfloat16_rn(outv);
}

// int8 projection of M prompt rows: the row-tiled int8 GEMM over the packed
// weights (the row-major tensor-core GEMM where they could not be packed).
int mm_rows(const float *A, const QW &w, float *Cm, size_t M, cudaStream_t st) {
    if (w.qp) return launch_matmul_int8_packed(A, w.qp, w.s, Cm, M, w.K, w.N, st);
    return launch_matmul_int8(A, w.q, w.s, Cm, M, w.K, w.N, st);
}

int prompt_workspace(ModelEngine *e, size_t T) {
    ModelEngine::Prompt &P = e->pf;
    if (P.T >= T) return KAI_GDN_OK;
    if (P.base) {
        cudaFree(P.base);  // waits for the device
        P.base = nullptr;
        P.T = 0;
    }
    const size_t H = e->cfg.hidden, d = e->d;
    const size_t widths[] = {H,
                             H,
                             H,
                             std::max(e->ny_gdn, e->ny_att),
                             std::max(e->hk * d, e->hq * e->D),
                             std::max(e->hk * d, (size_t)1),
                             std::max(e->hv * d, (size_t)1),
                             e->hv,
                             e->hv,
                             std::max(e->hv * d, e->hq * e->D),
                             std::max(e->hv * d, e->hq * e->D),
                             e->hq * e->D,
                             2 * e->I,
                             e->I};
    float **ptrs[] = {&P.h, &P.x, &P.part, &P.y, &P.q, &P.k, &P.v, &P.beta, &P.g, &P.o, &P.o2, &P.gate, &P.gu, &P.act};
    size_t total = 0;
    for (size_t wdt : widths) total += (T * wdt * sizeof(float) + 255) / 256 * 256;
    total += (T * sizeof(int) + 255) / 256 * 256;
    int rc = check_cuda(cudaMalloc(&P.base, total), "model_prefill: workspace");
    if (rc) return rc;
    unsigned char *cur = static_cast<unsigned char *>(P.base);
    for (size_t i = 0; i < sizeof(widths) / sizeof(widths[0]); ++i) {
        *ptrs[i] = reinterpret_cast<float *>(cur);
        cur += (T * widths[i] * sizeof(float) + 255) / 256 * 256;
    }
    P.tok = reinterpret_cast<int *>(cur);
    P.T = T;
    return KAI_GDN_OK;
}

// The prompt of sequence b (tokens already in pf.tok) from position pos0:
// leaves the last token's hidden state in h[b] and its final RMSNorm in x[b].
int run_prompt(ModelEngine *e, size_t b, size_t T, size_t pos0, cudaStream_t st) {
    const kai_gdn_model_config &c = e->cfg;
    const size_t H = c.hidden, d = e->d;
    ModelEngine::Prompt &P = e->pf;
    int rc = 0;
#define M_TRY(x)                   \
    do {                           \
        if ((rc = (x))) return rc; \
    } while (0)
    M_TRY(launch_pdl("embed_kernel", embed_kernel, dim3((unsigned)T), dim3(1024), st, P.tok, e->emb_q, e->emb_s, P.h,
                     (long long)H, (long long)c.vocab));
    const float *pending = nullptr;
    for (size_t l = 0; l < c.layers; ++l) {
        ModelEngine::Layer &L = e->layers[l];
        M_TRY(launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel, dim3((unsigned)T), dim3(1024), st, P.h, pending,
                         L.w_in, P.x, (long long)H, c.rms_eps));
        if (e->is_gdn[l]) {
            float *hist = L.hist + b * 3 * e->C;
            M_TRY(mm_rows(P.x, L.win, P.y, T, st));
            M_TRY(launch_pdl("gdn_prompt_prep_kernel", gdn_prompt_prep_kernel,
                             dim3((unsigned)(2 * e->hk + e->hv), (unsigned)T), dim3((unsigned)d), st, P.y,
                             (long long)e->ny_gdn, hist, L.conv_w, L.A_log, L.dt_bias, P.q, P.k, P.v, P.beta, P.g,
                             (int)e->hk, (int)e->hv, (int)d));
            M_TRY(launch_pdl("gdn_prompt_hist_kernel", gdn_prompt_hist_kernel, dim3(grid_for((long long)e->C)),
                             dim3(256), st, P.y, (long long)e->ny_gdn, hist, (long long)e->C, (long long)T));
            kai_gdn_chunk_args ca{};
            ca.q = P.q;
            ca.k = P.k;
            ca.v = P.v;
            ca.g = P.g;
            ca.beta = P.beta;
            ca.state = L.state + b * e->hv * d * d;
            ca.o = P.o;
            ca.batch = 1;
            ca.seq = T;
            ca.heads_k = e->hk;
            ca.heads_v = e->hv;
            ca.dk = d;
            ca.dv = d;
            ca.chunk = 64;
            ca.scale = 1.0f / sqrtf((float)d);
            ca.in_dtype = KAI_GDN_F32;
            ca.state_dtype = KAI_GDN_F32;
            ca.out_dtype = KAI_GDN_F32;
            M_TRY(launch_chunk(&ca, st));
            M_TRY(launch_pdl("gated_rmsnorm_kernel", gated_rmsnorm_kernel, dim3((unsigned)e->hv, (unsigned)T),
                             dim3((unsigned)d), st, P.o, P.y, (long long)e->ny_gdn, (long long)e->C, L.w_gn, P.o2,
                             (int)e->hv, (int)d, c.rms_eps));
        } else {
            const size_t kvrow = e->hkv * e->D;
            __nv_bfloat16 *kc = static_cast<__nv_bfloat16 *>(L.kc) + b * c.max_ctx * kvrow;
            __nv_bfloat16 *vc = static_cast<__nv_bfloat16 *>(L.vc) + b * c.max_ctx * kvrow;
            M_TRY(mm_rows(P.x, L.win, P.y, T, st));
            M_TRY(launch_pdl("attn_prompt_prep_kernel", attn_prompt_prep_kernel,
                             dim3((unsigned)(e->hq + 2 * e->hkv), (unsigned)T), dim3((unsigned)e->D), st, P.y,
                             (long long)e->ny_att, L.w_qn, L.w_kn, (long long)pos0, P.q, P.gate, kc, vc, (int)e->hq,
                             (int)e->hkv, (int)e->D, (int)c.rope_dims, c.rope_theta, c.rms_eps));
            kai_gdn_attn_prefill_args aa{};
            aa.q = P.q;
            aa.k_cache = kc;
            aa.v_cache = vc;
            aa.o = P.o;
            aa.batch = 1;
            aa.T = T;
            aa.heads = e->hq;
            aa.kv_heads = e->hkv;
            aa.head_dim = e->D;
            aa.pos0 = pos0;
            aa.max_ctx = c.max_ctx;
            aa.scale = 1.0f / sqrtf((float)e->D);
            M_TRY(launch_attn_prefill(&aa, st));
            M_TRY(launch_pdl("attn_gate_kernel", attn_gate_kernel, dim3(grid_for((long long)(T * e->hq * e->D))),
                             dim3(256), st, P.o, P.gate, P.o2, (long long)(T * e->hq * e->D)));
        }
        M_TRY(mm_rows(P.o2, L.wout, P.part, T, st));
        M_TRY(allreduce(e, P.part, T * H, st));
        M_TRY(launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel, dim3((unsigned)T), dim3(1024), st, P.h, P.part,
                         L.w_post, P.x, (long long)H, c.rms_eps));
        M_TRY(mm_rows(P.x, L.wgu, P.gu, T, st));
        M_TRY(launch_pdl("swiglu_kernel", swiglu_kernel, dim3(grid_for((long long)(T * e->I))), dim3(256), st, P.gu,
                         P.act, (long long)e->I, (long long)(T * e->I)));
        M_TRY(mm_rows(P.act, L.wdown, P.part, T, st));
        M_TRY(allreduce(e, P.part, T * H, st));
        pending = P.part;
    }
    // the last token: residual, final norm into the decode buffers
    const size_t lr = (T - 1) * H;
    M_TRY(launch_pdl("add_rmsnorm_kernel", add_rmsnorm_kernel, dim3(1), dim3(1024), st, P.h + lr, pending + lr,
                     e->w_final, P.x + lr, (long long)H, c.rms_eps));
    M_TRY(check_cuda(cudaMemcpyAsync(e->h + b * H, P.h + lr, H * sizeof(float), cudaMemcpyDeviceToDevice, st),
                     "model_prefill: copy"));
    M_TRY(check_cuda(cudaMemcpyAsync(e->x + b * H, P.x + lr, H * sizeof(float), cudaMemcpyDeviceToDevice, st),
                     "model_prefill: copy"));
#undef M_TRY
    return KAI_GDN_OK;
}

int capture_segments(ModelEngine *e, cudaStream_t st) {
    for (cudaGraphExec_t x : e->seg)
        if (x) cudaGraphExecDestroy(x);
    e->seg.assign(e->attn_layers.size() + 1, nullptr);
    for (size_t s = 0; s < e->seg.size(); ++s) {
        cudaGraph_t g = nullptr;
        int rc = check_cuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "model: capture");
        if (rc) return rc;
        int rc2 = run_segment(e, s, st);
        rc = check_cuda(cudaStreamEndCapture(st, &g), "model: capture");
        if (rc2 || rc) {
            if (g) cudaGraphDestroy(g);
            return rc2 ? rc2 : rc;
        }
        rc = check_cuda(cudaGraphInstantiate(&e->seg[s], g, 0), "model: instantiate");
        cudaGraphDestroy(g);
        if (rc) return rc;
    }
    e->graph_stream = st;
    return KAI_GDN_OK;
}

}  // namespace

int model_nccl_id(void *out) {
    if (!out) return set_error(KAI_GDN_ERR_INVALID, "model_nccl_id: null");
    const NcclApi *n = nullptr;
    int rc = nccl_api(&n);
    if (rc) return rc;
    ncclUniqueId id;
    if ((rc = check_nccl(n, n->getUniqueId(&id), "model: ncclGetUniqueId"))) return rc;
    static_assert(sizeof(ncclUniqueId) == KAI_GDN_NCCL_ID_BYTES, "id size");
    memcpy(out, &id, sizeof(id));
    return KAI_GDN_OK;
}

int model_destroy(void *engine);

int model_create(const kai_gdn_model_config *cfg, void **out) {
    if (!cfg || !out) return set_error(KAI_GDN_ERR_INVALID, "model_create: null argument");
    *out = nullptr;
    const kai_gdn_model_config &c = *cfg;
    const int W = c.tp_size < 1 ? 1 : c.tp_size, R = c.tp_rank;
    if (!c.is_gdn || !c.layers || !c.batch || !c.hidden || !c.vocab || !c.inter || !c.max_ctx)
        return set_error(KAI_GDN_ERR_INVALID, "model_create: empty dimension");
    if (R < 0 || R >= W) return set_error(KAI_GDN_ERR_INVALID, "model_create: tp_rank %d of %d", R, W);
    if (c.gdn_heads_k % W || c.gdn_heads_v % W || c.attn_heads % W || c.inter % W || c.vocab % W)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "model_create: heads, inter and vocab must divide by tp_size %d", W);
    if (c.gdn_heads_v % c.gdn_heads_k || c.attn_heads % c.attn_kv_heads)
        return set_error(KAI_GDN_ERR_INVALID, "model_create: value / query heads not a multiple of key / kv heads");
    if ((c.gdn_head_dim != 64 && c.gdn_head_dim != 128) || (c.attn_head_dim != 128 && c.attn_head_dim != 256))
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "model_create: head dims (GDN 64/128, attention 128/256)");
    if (c.rope_dims > c.attn_head_dim || c.rope_dims % 2 || c.hidden % 16 || (c.inter / W) % 16 ||
        (c.vocab / W) % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "model_create: widths (hidden, inter/tp, vocab/tp multiples of 16)");
    if (W > 1 && !c.nccl_id) return set_error(KAI_GDN_ERR_INVALID, "model_create: tp_size > 1 needs an NCCL id");

    ModelEngine *e = new ModelEngine();
    e->cfg = c;
    e->cfg.tp_size = W;
    e->is_gdn.assign(c.is_gdn, c.is_gdn + c.layers);
    e->cfg.is_gdn = nullptr;
    e->cfg.nccl_id = nullptr;
    cudaGetDevice(&e->device);
    const size_t B = c.batch, H = c.hidden;
    e->d = c.gdn_head_dim;
    e->hk = c.gdn_heads_k / W;
    e->hv = c.gdn_heads_v / W;
    e->C = (2 * e->hk + e->hv) * e->d;
    const size_t nin = e->C + e->hv * e->d + 2 * e->hv;
    e->ny_gdn = (nin + 15) / 16 * 16;
    e->D = c.attn_head_dim;
    e->hq = c.attn_heads / W;
    const size_t group = c.attn_heads / c.attn_kv_heads;  // query heads per kv head
    if (c.attn_kv_heads >= (size_t)W) {
        if (c.attn_kv_heads % W) {
            delete e;
            return set_error(KAI_GDN_ERR_UNSUPPORTED, "model_create: kv heads must divide by tp_size");
        }
        e->hkv = c.attn_kv_heads / W;
        e->kv_first = R * e->hkv;
    } else {
        if (e->hq == 0 || group % e->hq) {
            delete e;
            return set_error(KAI_GDN_ERR_UNSUPPORTED, "model_create: query heads per rank must tile a kv group");
        }
        e->hkv = 1;
        e->kv_first = (R * e->hq) / group;
    }
    e->ny_att = e->hq * 2 * e->D + 2 * e->hkv * e->D;
    e->I = c.inter / W;
    e->V = c.vocab / W;
    e->v0 = R * e->V;
    for (size_t l = 0; l < c.layers; ++l)
        if (!e->is_gdn[l]) e->attn_layers.push_back(l);

    int rc = 0;
    if (W > 1) {
        rc = nccl_api(&e->nccl);
        ncclUniqueId id;
        memcpy(&id, c.nccl_id, sizeof(id));
        if (!rc) rc = check_nccl(e->nccl, e->nccl->commInitRank(&e->comm, W, id, R), "model: ncclCommInitRank");
    }
    const float sd = c.weight_std > 0.f ? c.weight_std : 0.02f;
    const size_t d = e->d, GK = c.gdn_heads_k * d, GV = c.gdn_heads_v * d, hk0 = R * e->hk, hv0 = R * e->hv;
    const size_t AQ = c.attn_heads * 2 * e->D, AKV = c.attn_kv_heads * e->D, hq0 = R * e->hq;
    e->layers.resize(c.layers);
    for (size_t l = 0; l < c.layers && !rc; ++l) {
        ModelEngine::Layer &L = e->layers[l];
        if (!rc) rc = vec_normal(e, &L.w_in, H, 0, tidl(l, T_NIN), sd, 1.0f);
        if (!rc) rc = vec_normal(e, &L.w_post, H, 0, tidl(l, T_NPOST), sd, 1.0f);
        if (e->is_gdn[l]) {
            std::vector<Part> p = {{tidl(l, T_Q), GK, hk0 * d, e->hk * d},
                                   {tidl(l, T_K), GK, hk0 * d, e->hk * d},
                                   {tidl(l, T_V), GV, hv0 * d, e->hv * d},
                                   {tidl(l, T_Z), GV, hv0 * d, e->hv * d},
                                   {tidl(l, T_B), c.gdn_heads_v, hv0, e->hv},
                                   {tidl(l, T_A), c.gdn_heads_v, hv0, e->hv}};
            if (e->ny_gdn > nin) p.push_back({tidl(l, T_PAD), e->ny_gdn - nin, 0, e->ny_gdn - nin});
            if (!rc) rc = build_qw(e, &L.win, H, 0, H, p, sd);
            if (!rc) rc = build_qw(e, &L.wout, GV, hv0 * d, (hv0 + e->hv) * d, {{tidl(l, T_OUT), H, 0, H}}, sd);
            // conv taps [4][C]: the q, k and v channels of this rank's heads
            if (!rc) rc = malloc_keep(e, (void **)&L.conv_w, 4 * e->C * sizeof(float), false);
            const size_t cw = 2 * GK + GV;  // global conv channels
            const size_t segs[3][2] = {{hk0 * d, e->hk * d}, {GK + hk0 * d, e->hk * d}, {2 * GK + hv0 * d, e->hv * d}};
            size_t col = 0;
            for (int sgi = 0; sgi < 3 && !rc; ++sgi) {
                rng_normal_kernel<<<grid_for((long long)(4 * segs[sgi][1])), 256>>>(
                    L.conv_w + col, 4, (long long)segs[sgi][1], (long long)e->C, 0, (long long)segs[sgi][0],
                    (long long)cw, c.seed, tidl(l, T_CONV), 0.5f);
                rc = check_launch("rng_normal_kernel");
                col += segs[sgi][1];
            }
            if (!rc) rc = malloc_keep(e, (void **)&L.A_log, e->hv * sizeof(float), false);
            if (!rc) {  // A_log = log(U(1, 16)), dt_bias = 1 (docs/GDN_ARCHITECTURE_AUDIT.md:85-90)
                rng_uniform_kernel<<<1, 256>>>(L.A_log, (long long)e->hv, (long long)hv0, c.seed, tidl(l, T_ALOG),
                                               1.0f, 16.0f, 1);
                rc = check_launch("rng_uniform_kernel");
            }
            if (!rc) rc = vec_const(e, &L.dt_bias, e->hv, 1.0f);
            if (!rc) rc = vec_normal(e, &L.w_gn, d, 0, tidl(l, T_GN), sd, 1.0f);
            if (!rc) rc = malloc_keep(e, (void **)&L.state, B * e->hv * d * d * sizeof(float), true);
            if (!rc) rc = malloc_keep(e, (void **)&L.hist, B * 3 * e->C * sizeof(float), true);
        } else {
            std::vector<Part> p;
            for (size_t qh = 0; qh < e->hq; ++qh)
                p.push_back({tidl(l, T_AQ), AQ, (hq0 + qh) * 2 * e->D, 2 * e->D});
            p.push_back({tidl(l, T_AK), AKV, e->kv_first * e->D, e->hkv * e->D});
            p.push_back({tidl(l, T_AV), AKV, e->kv_first * e->D, e->hkv * e->D});
            if (!rc) rc = build_qw(e, &L.win, H, 0, H, p, sd);
            if (!rc)
                rc = build_qw(e, &L.wout, c.attn_heads * e->D, hq0 * e->D, (hq0 + e->hq) * e->D,
                              {{tidl(l, T_AO), H, 0, H}}, sd);
            if (!rc) rc = vec_normal(e, &L.w_qn, e->D, 0, tidl(l, T_QN), sd, 1.0f);
            if (!rc) rc = vec_normal(e, &L.w_kn, e->D, 0, tidl(l, T_KN), sd, 1.0f);
            const size_t cache = B * c.max_ctx * e->hkv * e->D * 2;
            if (!rc) rc = malloc_keep(e, &L.kc, cache, true);
            if (!rc) rc = malloc_keep(e, &L.vc, cache, true);
        }
        const size_t I0 = R * e->I;
        if (!rc)
            rc = build_qw(e, &L.wgu, H, 0, H,
                          {{tidl(l, T_GATE), c.inter, I0, e->I}, {tidl(l, T_UP), c.inter, I0, e->I}}, sd);
        if (!rc) rc = build_qw(e, &L.wdown, c.inter, I0, I0 + e->I, {{tidl(l, T_DOWN), H, 0, H}}, sd);
    }
    if (!rc) rc = build_qw(e, &e->lm, H, 0, H, {{T_LM, c.vocab, e->v0, e->V}}, sd, true);
    if (!rc) rc = vec_normal(e, &e->w_final, H, 0, T_FINAL, sd, 1.0f);
    if (!rc) {  // embedding table [vocab][hidden], int8 per token row (replicated)
        const size_t rows_per = 8192;
        float *tmp = nullptr;
        rc = check_cuda(cudaMalloc(&tmp, rows_per * H * sizeof(float)), "model: embedding workspace");
        if (!rc) rc = malloc_keep(e, (void **)&e->emb_q, c.vocab * H, false);
        if (!rc) rc = malloc_keep(e, (void **)&e->emb_s, c.vocab * sizeof(float), false);
        for (size_t r0 = 0; r0 < c.vocab && !rc; r0 += rows_per) {
            const size_t nr = std::min(rows_per, c.vocab - r0);
            rng_normal_kernel<<<grid_for((long long)(nr * H)), 256>>>(tmp, (long long)nr, (long long)H, (long long)H,
                                                                     (long long)r0, 0, (long long)H, c.seed, T_EMB, sd);
            rc = check_launch("rng_normal_kernel");
            if (!rc) {
                quantize_rows_kernel<<<(unsigned)nr, 256>>>(tmp, e->emb_q + r0 * H, e->emb_s + r0, (long long)nr,
                                                           (long long)H);
                rc = check_launch("quantize_rows_kernel");
            }
        }
        if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "model: embedding");
        if (tmp) cudaFree(tmp);
    }
    struct Buf {
        float **p;
        size_t n;
    } bufs[] = {{&e->h, B * H},
                {&e->x, B * H},
                {&e->y, B * std::max(e->ny_gdn, e->ny_att)},
                {&e->part, B * H},
                {&e->q, B * std::max(e->hk * d, e->hq * e->D)},
                {&e->k, B * std::max(e->hk * d, e->hkv * e->D)},
                {&e->v, B * std::max(e->hv * d, e->hkv * e->D)},
                {&e->beta, B * e->hv},
                {&e->g, B * e->hv},
                {&e->o, B * std::max(e->hv * d, e->hq * e->D)},
                {&e->o2, B * std::max(e->hv * d, e->hq * e->D)},
                {&e->gate, B * e->hq * e->D},
                {&e->gu, B * 2 * e->I},
                {&e->act, B * e->I},
                {&e->logits, B * e->V}};
    for (auto &bf : bufs)
        if (!rc) rc = malloc_keep(e, (void **)bf.p, bf.n * sizeof(float), true);
    if (!rc && B > GEMV_MAX_BATCH) {
        // fused producers need every projection packed and 16-multiple inputs
        bool all = e->lm.qp != nullptr;
        size_t kmax = H;
        for (const ModelEngine::Layer &L : e->layers) {
            for (const QW *w : {&L.win, &L.wout, &L.wgu, &L.wdown}) {
                all = all && w->qp != nullptr && w->K % 16 == 0;
                kmax = std::max(kmax, w->K);
            }
        }
        if (all) {
            rc = malloc_keep(e, (void **)&e->terms, int8_terms_bytes(B, kmax), true);
            if (!rc) rc = malloc_keep(e, (void **)&e->tscale, B * sizeof(float), true);
            e->fused = !rc;
        }
    }
    if (!rc) rc = malloc_keep(e, (void **)&e->tok, B * sizeof(int), true);
    if (!rc) rc = malloc_keep(e, (void **)&e->pos, sizeof(int), true);
    if (!rc) rc = malloc_keep(e, (void **)&e->cand, B * AM_BLOCKS * sizeof(ArgMax), true);
    if (!rc) rc = malloc_keep(e, (void **)&e->cand_all, (size_t)W * B * AM_BLOCKS * sizeof(ArgMax), true);
    if (rc) {
        model_destroy(e);
        return rc;
    }
    *out = e;
    return KAI_GDN_OK;
}

int model_prefill(void *engine, const int *tokens, size_t T, size_t pos0, cudaStream_t st) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e || !tokens) return set_error(KAI_GDN_ERR_INVALID, "model_prefill: null argument");
    if (T == 0) return KAI_GDN_OK;
    if (pos0 + T > e->cfg.max_ctx)
        return set_error(KAI_GDN_ERR_INVALID, "model_prefill: positions %zu .. %zu outside the cache (%zu)", pos0,
                         pos0 + T - 1, e->cfg.max_ctx);
    int rc = prompt_workspace(e, T);
    for (size_t b = 0; b < e->cfg.batch && !rc; ++b) {
        rc = check_cuda(cudaMemcpyAsync(e->pf.tok, tokens + b * T, T * sizeof(int), cudaMemcpyDefault, st),
                        "model_prefill: tokens");
        if (!rc) rc = run_prompt(e, b, T, pos0, st);
    }
    if (!rc) rc = lm_head(e, st);
    if (!rc) rc = check_cuda(cudaStreamSynchronize(st), "model_prefill: sync");
    return rc;
}

int model_step(void *engine, size_t pos, cudaStream_t st) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e) return set_error(KAI_GDN_ERR_INVALID, "model_step: null engine");
    if (pos >= e->cfg.max_ctx)
        return set_error(KAI_GDN_ERR_INVALID, "model_step: position %zu outside the cache (%zu)", pos, e->cfg.max_ctx);
    // The first step on a stream runs eagerly (it creates the library's
    // per-stream workspaces); the next one captures the segment graphs, later
    // ones replay them.
    const bool capturable = st != nullptr && st != cudaStreamLegacy && st != cudaStreamPerThread;
    int rc = 0;
    if (!e->seg.empty() && e->graph_stream == st) {
        rc = run_token(e, pos, st, true);
    } else if (capturable && e->steps >= 1 && e->last_stream == st) {
        rc = capture_segments(e, st);
        if (!rc) rc = run_token(e, pos, st, true);
    } else {
        rc = run_token(e, pos, st, false);
    }
    if (rc) return rc;
    ++e->steps;
    e->last_stream = st;
    return KAI_GDN_OK;
}

int model_tokens(void *engine, int *tokens, int set) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e || !tokens) return set_error(KAI_GDN_ERR_INVALID, "model_tokens: null argument");
    int rc = check_cuda(cudaDeviceSynchronize(), "model_tokens: sync");
    if (rc) return rc;
    const size_t bytes = e->cfg.batch * sizeof(int);
    return check_cuda(set ? cudaMemcpy(e->tok, tokens, bytes, cudaMemcpyDefault)
                          : cudaMemcpy(tokens, e->tok, bytes, cudaMemcpyDefault),
                      "model_tokens: copy");
}

int model_read(void *engine, int what, float *out) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e || !out) return set_error(KAI_GDN_ERR_INVALID, "model_read: null argument");
    int rc = check_cuda(cudaDeviceSynchronize(), "model_read: sync");
    if (rc) return rc;
    const size_t B = e->cfg.batch;
    switch (what) {
        case KAI_GDN_MODEL_HIDDEN:
            return check_cuda(cudaMemcpy(out, e->h, B * e->cfg.hidden * sizeof(float), cudaMemcpyDefault), "read");
        case KAI_GDN_MODEL_LOGITS:
            return check_cuda(cudaMemcpy(out, e->logits, B * e->V * sizeof(float), cudaMemcpyDefault), "read");
    }
    return set_error(KAI_GDN_ERR_INVALID, "model_read: unknown item %d", what);
}

// Copy out one of this rank's weights (for a checker): int8 codes [K][N] and
// scales [N] of projection `which` of `layer`, or an fp32 vector.
int model_weight(void *engine, size_t layer, int which, void *data, float *scales, size_t *rows, size_t *cols) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e || !rows || !cols) return set_error(KAI_GDN_ERR_INVALID, "model_weight: null argument");
    const QW *w = nullptr;
    const float *vec = nullptr;
    size_t n = 0;
    const bool per_layer = which < KAI_GDN_MODEL_W_LM;
    if (per_layer && layer >= e->layers.size()) return set_error(KAI_GDN_ERR_INVALID, "model_weight: layer");
    const ModelEngine::Layer *L = per_layer ? &e->layers[layer] : nullptr;
    switch (which) {
        case KAI_GDN_MODEL_W_IN: w = &L->win; break;
        case KAI_GDN_MODEL_W_OUT: w = &L->wout; break;
        case KAI_GDN_MODEL_W_GATE_UP: w = &L->wgu; break;
        case KAI_GDN_MODEL_W_DOWN: w = &L->wdown; break;
        case KAI_GDN_MODEL_V_NORM_IN: vec = L->w_in, n = e->cfg.hidden; break;
        case KAI_GDN_MODEL_V_NORM_POST: vec = L->w_post, n = e->cfg.hidden; break;
        case KAI_GDN_MODEL_V_CONV: vec = L->conv_w, n = L->conv_w ? 4 * e->C : 0; break;
        case KAI_GDN_MODEL_V_A_LOG: vec = L->A_log, n = L->A_log ? e->hv : 0; break;
        case KAI_GDN_MODEL_V_DT_BIAS: vec = L->dt_bias, n = L->dt_bias ? e->hv : 0; break;
        case KAI_GDN_MODEL_V_NORM_GDN: vec = L->w_gn, n = L->w_gn ? e->d : 0; break;
        case KAI_GDN_MODEL_V_NORM_Q: vec = L->w_qn, n = L->w_qn ? e->D : 0; break;
        case KAI_GDN_MODEL_V_NORM_K: vec = L->w_kn, n = L->w_kn ? e->D : 0; break;
        case KAI_GDN_MODEL_W_LM: w = &e->lm; break;
        case KAI_GDN_MODEL_V_NORM_FINAL: vec = e->w_final, n = e->cfg.hidden; break;
        case KAI_GDN_MODEL_W_EMBED: {
            *rows = e->cfg.vocab;
            *cols = e->cfg.hidden;
            int rc = check_cuda(cudaDeviceSynchronize(), "model_weight: sync");
            if (!rc && data) rc = check_cuda(cudaMemcpy(data, e->emb_q, e->cfg.vocab * e->cfg.hidden, cudaMemcpyDefault), "copy");
            if (!rc && scales)
                rc = check_cuda(cudaMemcpy(scales, e->emb_s, e->cfg.vocab * sizeof(float), cudaMemcpyDefault), "copy");
            return rc;
        }
        default: return set_error(KAI_GDN_ERR_INVALID, "model_weight: unknown item %d", which);
    }
    int rc = check_cuda(cudaDeviceSynchronize(), "model_weight: sync");
    if (rc) return rc;
    if (w) {
        *rows = w->K;
        *cols = w->N;
        if (data) rc = check_cuda(cudaMemcpy(data, w->q, w->K * w->N, cudaMemcpyDefault), "model_weight: copy");
        if (!rc && scales) rc = check_cuda(cudaMemcpy(scales, w->s, w->N * sizeof(float), cudaMemcpyDefault), "copy");
        return rc;
    }
    *rows = 1;
    *cols = n;
    if (!vec) return set_error(KAI_GDN_ERR_INVALID, "model_weight: layer %zu has no item %d", layer, which);
    if (data) rc = check_cuda(cudaMemcpy(data, vec, n * sizeof(float), cudaMemcpyDefault), "model_weight: copy");
    return rc;
}

// Synthetic state of an already-consumed context of `ctx` tokens (a
// stand-in for the prefill), drawn by global index so that every
// tensor-parallel split holds the same state: every attention layer's K/V
// cache rows [0, ctx) N(0, 1) in bf16, every GDN state N(0, 0.02), conv
// histories N(0, 1).
__global__ void fill_cache_kernel(__nv_bfloat16 *__restrict__ c, long long B, long long max_ctx, long long row,
                                  long long grow, long long g0, long long ctx, unsigned long long seed,
                                  unsigned tid) {
    const long long n = B * ctx * row;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const long long bt = e / row, col = e % row, b = bt / ctx, tt = bt % ctx;
        const unsigned long long idx = (unsigned long long)((b * max_ctx + tt) * grow + g0 + col);
        const unsigned long long u = mix64(seed ^ mix64(((unsigned long long)tid << 40) ^ idx));
        const float u1 = ((float)(u >> 40) + 0.5f) * 5.9604644775390625e-8f;
        const float u2 = ((float)(u & 0xFFFFFFull) + 0.5f) * 5.9604644775390625e-8f;
        c[(b * max_ctx + tt) * row + col] = __float2bfloat16_rn(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}
int model_fill(void *engine, size_t ctx, unsigned long long seed) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e) return set_error(KAI_GDN_ERR_INVALID, "model_fill: null engine");
    if (ctx > e->cfg.max_ctx) return set_error(KAI_GDN_ERR_INVALID, "model_fill: ctx %zu > max_ctx", ctx);
    const kai_gdn_model_config &c = e->cfg;
    const size_t B = c.batch, d = e->d, R = (size_t)c.tp_rank;
    const size_t hv0 = R * e->hv, hk0 = R * e->hk, GK = c.gdn_heads_k * d, GV = c.gdn_heads_v * d;
    int rc = 0;
    for (size_t l = 0; l < e->layers.size() && !rc; ++l) {
        ModelEngine::Layer &L = e->layers[l];
        const unsigned t = (unsigned)(l * 64 + 40);
        if (e->is_gdn[l]) {
            // state [B][hv][d][d]: global heads hv0 .. of Hv
            const long long per = (long long)(e->hv * d * d), gper = (long long)(c.gdn_heads_v * d * d);
            rng_normal_kernel<<<grid_for((long long)B * per), 256>>>(L.state, (long long)B, per, per, 0,
                                                                    (long long)(hv0 * d * d), gper, seed, t, 0.02f);
            rc = check_launch("rng_normal_kernel");
            // history [B][3][C]: this rank's q, k and v channels of the global [3][2 GK + GV]
            const size_t gc = 2 * GK + GV;
            const size_t segs[3][2] = {{hk0 * d, e->hk * d}, {GK + hk0 * d, e->hk * d}, {2 * GK + hv0 * d, e->hv * d}};
            size_t col = 0;
            for (int sg = 0; sg < 3 && !rc; ++sg) {
                rng_normal_kernel<<<grid_for((long long)(B * 3 * segs[sg][1])), 256>>>(
                    L.hist + col, (long long)(B * 3), (long long)segs[sg][1], (long long)e->C, 0,
                    (long long)segs[sg][0], (long long)gc, seed, t + 1, 1.0f);
                rc = check_launch("rng_normal_kernel");
                col += segs[sg][1];
            }
        } else if (ctx > 0) {
            const long long row = (long long)(e->hkv * e->D), grow = (long long)(c.attn_kv_heads * e->D);
            const long long g0 = (long long)(e->kv_first * e->D), n = (long long)B * (long long)ctx * row;
            fill_cache_kernel<<<grid_for(n), 256>>>(static_cast<__nv_bfloat16 *>(L.kc), (long long)B,
                                                   (long long)c.max_ctx, row, grow, g0, (long long)ctx, seed, t + 2);
            rc = check_launch("fill_cache_kernel");
            if (!rc)
                fill_cache_kernel<<<grid_for(n), 256>>>(static_cast<__nv_bfloat16 *>(L.vc), (long long)B,
                                                       (long long)c.max_ctx, row, grow, g0, (long long)ctx, seed,
                                                       t + 3);
            if (!rc) rc = check_launch("fill_cache_kernel");
        }
    }
    if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "model_fill: sync");
    return rc;
}

// Every sequence back to position 0: GDN states and conv histories zero (the
// KV cache rows are written before they are read).
int model_reset(void *engine) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e) return set_error(KAI_GDN_ERR_INVALID, "model_reset: null engine");
    const size_t B = e->cfg.batch, d = e->d;
    int rc = check_cuda(cudaDeviceSynchronize(), "model_reset: sync");
    for (size_t l = 0; l < e->layers.size() && !rc; ++l) {
        ModelEngine::Layer &L = e->layers[l];
        if (!e->is_gdn[l]) continue;
        rc = check_cuda(cudaMemset(L.state, 0, B * e->hv * d * d * sizeof(float)), "model_reset: state");
        if (!rc) rc = check_cuda(cudaMemset(L.hist, 0, B * 3 * e->C * sizeof(float)), "model_reset: history");
    }
    return rc;
}

int model_destroy(void *engine) {
    ModelEngine *e = static_cast<ModelEngine *>(engine);
    if (!e) return KAI_GDN_OK;
    cudaDeviceSynchronize();
    for (cudaGraphExec_t x : e->seg)
        if (x) cudaGraphExecDestroy(x);
    if (e->comm && e->nccl) e->nccl->commDestroy(e->comm);
    if (e->pf.base) cudaFree(e->pf.base);
    for (void *p : e->allocs) cudaFree(p);
    delete e;
    return KAI_GDN_OK;
}

}  // namespace gdn
