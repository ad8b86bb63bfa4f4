// scan.cu -- the channel-wise recurrences of the GDN hot path on sm_100a:
//   cumdecay  decay[t] = prod_{i<=t} a[i]      kai_gdn_cumdecay_f32_sve.c:82-89
//   cumsum    gcum[t]  = sum_{i<=t} g[i]       (log-space twin of cumdecay)
//   gated     s[t] = x[t] + s[t-1]*g[t]        kai_gdn_gated_scan_f32_sve.c:86-95
//   gdn2      s[t] = w[t]*x[t] + s[t-1]*(g[t]*b[t])   gdn_sve.c:865-872
//
// All are HBM-bound: one read of each input stream, one write of the output.
// Layout [batch][seq][channels]; a warp covers 32 consecutive channels of one
// row, so every access is a full 128-byte line.
//
// Time parallelism: each thread walks one SEGMENT of SEG_LEN rows of one
// channel sequentially, with the reference's operation order and one rounding
// per operation (__fmul_rn / __fadd_rn, no FMA contraction), so a sequence of
// at most SEG_LEN rows is bit-identical to the reference's scalar path.
// Longer sequences use three launches: (1) each segment's aggregate (the
// product, the sum, or the affine pair (A, B) with s_end = B + s_in*A) goes
// to scratch; (2) one thread per (batch, channel) turns the aggregates into
// each segment's carry-in, in order; (3) every segment re-walks its rows from
// its carry.  Pass 3's re-read of the input is served from L2 for inputs that
// fit in it (126 MB).
#include <mutex>

#include "gdn_internal.cuh"

namespace gdn {
namespace {

constexpr int SEG_LEN = 128;  // rows per thread
constexpr int BATCH_LD = 8;   // loads issued ahead of the dependent chain

enum Op { CUMPROD = 0, CUMSUM = 1, AFFINE = 2, GDN2 = 3 };

struct ScanParams {
    const float *x;  // cumprod: a, cumsum: g, affine/gdn2: x
    const float *g;  // affine/gdn2 gate
    const float *b;  // gdn2 erase gate
    const float *w;  // gdn2 write gate
    void *out;       // [batch][seq][ch]
    void *state;     // affine/gdn2: [batch][ch]
    float *aggA;     // scratch [batch][nseg][ch]
    float *aggB;     // scratch [batch][nseg][ch] (affine/gdn2)
    long long seq, ch;
    int nseg;
    int cw;          // warps per block along channels (block = 32*cw channels)
};

template <int OP> struct Step;
template <> struct Step<CUMPROD> {
    static constexpr int NIN = 1;
    __device__ static float apply(float run, const float *v) { return __fmul_rn(run, v[0]); }
};
template <> struct Step<CUMSUM> {
    static constexpr int NIN = 1;
    __device__ static float apply(float run, const float *v) { return __fadd_rn(run, v[0]); }
};
template <> struct Step<AFFINE> {
    static constexpr int NIN = 2;  // v[0] = x, v[1] = g
    __device__ static float apply(float run, const float *v) {
        return __fadd_rn(v[0], __fmul_rn(run, v[1]));
    }
};
template <> struct Step<GDN2> {
    static constexpr int NIN = 4;  // x, g, b, w
    __device__ static float apply(float run, const float *v) {
        return __fadd_rn(__fmul_rn(v[3], v[0]), __fmul_rn(run, __fmul_rn(v[1], v[2])));
    }
};

template <int OP>
__device__ __forceinline__ void load_row(const ScanParams &p, size_t idx, float *v) {
    v[0] = __ldg(p.x + idx);
    if (OP == AFFINE || OP == GDN2) v[1] = __ldg(p.g + idx);
    if (OP == GDN2) {
        v[2] = __ldg(p.b + idx);
        v[3] = __ldg(p.w + idx);
    }
}

// Thread coordinates: blockDim = (32, 8).  Warps split into cw channel groups
// and 8/cw segment groups.
struct Coord {
    long long c;
    int seg;
    long long b;
    bool live;
};
__device__ __forceinline__ Coord coord(const ScanParams &p) {
    int ty = threadIdx.y;
    int cg = ty % p.cw, sg = ty / p.cw, sw = 8 / p.cw;
    Coord k;
    k.c = (long long)blockIdx.x * (32 * p.cw) + cg * 32 + threadIdx.x;
    k.seg = blockIdx.y * sw + sg;
    k.b = blockIdx.z;
    k.live = k.c < p.ch && k.seg < p.nseg;
    return k;
}

// Pass 1: aggregate of every segment except the last.
template <int OP>
__global__ void __launch_bounds__(256) scan_aggregate_kernel(ScanParams p) {
    Coord k = coord(p);
    if (!k.live || k.seg == p.nseg - 1) return;
    long long t0 = (long long)k.seg * SEG_LEN;
    size_t base = (size_t)k.b * p.seq * p.ch + (size_t)k.c;
    float A = (OP == CUMSUM) ? 0.0f : 1.0f, B = 0.0f;
    for (int r0 = 0; r0 < SEG_LEN; r0 += BATCH_LD) {
        float v[BATCH_LD][4];
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) load_row<OP>(p, base + (size_t)(t0 + r0 + r) * p.ch, v[r]);
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) {
            if (OP == CUMPROD) A = __fmul_rn(A, v[r][0]);
            else if (OP == CUMSUM) A = __fadd_rn(A, v[r][0]);
            else {
                float m = (OP == AFFINE) ? v[r][1] : __fmul_rn(v[r][1], v[r][2]);
                B = Step<OP>::apply(B, v[r]);
                A = __fmul_rn(A, m);
            }
        }
    }
    size_t ai = ((size_t)k.b * p.nseg + k.seg) * p.ch + k.c;
    p.aggA[ai] = A;
    if (OP == AFFINE || OP == GDN2) p.aggB[ai] = B;
}

// Pass 2: carry-in of every segment, in order, one thread per (batch, channel).
// Overwrites aggA[seg] with the carry into seg.
template <int OP, int SDT>
__global__ void scan_carry_kernel(ScanParams p) {
    long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long b = blockIdx.y;
    if (c >= p.ch) return;
    float carry;
    if (OP == CUMPROD) carry = 1.0f;
    else if (OP == CUMSUM) carry = 0.0f;
    else {
        using S = Store<SDT>;
        carry = S::load(reinterpret_cast<const typename S::T *>(p.state) + b * p.ch + c);
    }
    for (int s = 0; s < p.nseg; ++s) {
        size_t ai = ((size_t)b * p.nseg + s) * p.ch + c;
        float A = p.aggA[ai];
        float B = (OP == AFFINE || OP == GDN2) ? p.aggB[ai] : 0.0f;
        p.aggA[ai] = carry;
        if (s == p.nseg - 1) break;
        if (OP == CUMPROD) carry = __fmul_rn(carry, A);
        else if (OP == CUMSUM) carry = __fadd_rn(carry, A);
        else carry = __fadd_rn(B, __fmul_rn(carry, A));
    }
}

// Pass 3 (or the only pass when nseg == 1): walk the segment from its carry.
// ODT: storage type of the output (cumprod only; others write fp32).
// SDT: storage type of the carried state (affine only).
template <int OP, int ODT, int SDT>
__global__ void __launch_bounds__(256) scan_final_kernel(ScanParams p) {
    Coord k = coord(p);
    if (!k.live) return;
    long long t0 = (long long)k.seg * SEG_LEN;
    long long t1 = min(t0 + (long long)SEG_LEN, p.seq);
    size_t base = (size_t)k.b * p.seq * p.ch + (size_t)k.c;
    float run;
    if (p.nseg > 1) {
        run = p.aggA[((size_t)k.b * p.nseg + k.seg) * p.ch + k.c];
    } else if (OP == CUMPROD) {
        run = 1.0f;
    } else if (OP == CUMSUM) {
        run = 0.0f;
    } else {
        using S = Store<SDT>;
        run = S::load(reinterpret_cast<const typename S::T *>(p.state) + k.b * p.ch + k.c);
    }
    using O = Store<ODT>;
    typename O::T *out = reinterpret_cast<typename O::T *>(p.out);
    long long t = t0;
    for (; t + BATCH_LD <= t1; t += BATCH_LD) {
        float v[BATCH_LD][4];
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) load_row<OP>(p, base + (size_t)(t + r) * p.ch, v[r]);
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) {
            run = Step<OP>::apply(run, v[r]);
            O::store(out + base + (size_t)(t + r) * p.ch, run);
        }
    }
    for (; t < t1; ++t) {
        float v[4];
        load_row<OP>(p, base + (size_t)t * p.ch, v);
        run = Step<OP>::apply(run, v);
        O::store(out + base + (size_t)t * p.ch, run);
    }
    if ((OP == AFFINE || OP == GDN2) && k.seg == p.nseg - 1) {
        using S = Store<SDT>;
        S::store(reinterpret_cast<typename S::T *>(p.state) + k.b * p.ch + k.c, run);
    }
}

template <int OP, int ODT, int SDT>
int run_scan(ScanParams p, size_t batch, cudaStream_t st, const char *name) {
    if (batch > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: batch %zu > 65535", name, batch);
    long long nseg = (p.seq + SEG_LEN - 1) / SEG_LEN;
    if (nseg > (1ll << 24)) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: seq too long", name);
    p.nseg = (int)nseg;
    int sw = nseg >= 8 ? 8 : nseg >= 4 ? 4 : nseg >= 2 ? 2 : 1;
    p.cw = 8 / sw;
    dim3 block(32, 8);
    long long gx = (p.ch + 32 * p.cw - 1) / (32 * p.cw);
    long long gy = (nseg + sw - 1) / sw;
    if (gx > 0x7fffffffll || gy > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: shape too large for the grid", name);
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)batch);
    if (nseg > 1) {
        size_t n = batch * (size_t)nseg * (size_t)p.ch;
        int naggs = (OP == AFFINE || OP == GDN2) ? 2 : 1;
        void *scr = nullptr;
        int rc = scratch_for_stream(st, n * naggs * sizeof(float), &scr);
        if (rc) return rc;
        p.aggA = static_cast<float *>(scr);
        p.aggB = p.aggA + n;
        scan_aggregate_kernel<OP><<<grid, block, 0, st>>>(p);
        if ((rc = check_launch(name))) return rc;
        dim3 cgrid((unsigned)((p.ch + 127) / 128), (unsigned)batch);
        scan_carry_kernel<OP, SDT><<<cgrid, 128, 0, st>>>(p);
        if ((rc = check_launch(name))) return rc;
    }
    scan_final_kernel<OP, ODT, SDT><<<grid, block, 0, st>>>(p);
    return check_launch(name);
}

}  // namespace

int launch_cumdecay(const float *a, void *decay, int dt, size_t batch, size_t seq,
                    size_t ch, cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!a || !decay) return set_error(KAI_GDN_ERR_INVALID, "cumdecay: null pointer");
    ScanParams p{};
    p.x = a;
    p.out = decay;
    p.seq = (long long)seq;
    p.ch = (long long)ch;
    switch (dt) {
        case KAI_GDN_F32: return run_scan<CUMPROD, KAI_GDN_F32, KAI_GDN_F32>(p, batch, st, "cumdecay");
        case KAI_GDN_F16: return run_scan<CUMPROD, KAI_GDN_F16, KAI_GDN_F32>(p, batch, st, "cumdecay");
        case KAI_GDN_BF16: return run_scan<CUMPROD, KAI_GDN_BF16, KAI_GDN_F32>(p, batch, st, "cumdecay");
    }
    return set_error(KAI_GDN_ERR_INVALID, "cumdecay: bad decay dtype %d", dt);
}

int launch_cumsum(const float *g, float *gcum, size_t batch, size_t seq, size_t ch,
                  cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!g || !gcum) return set_error(KAI_GDN_ERR_INVALID, "cumsum: null pointer");
    ScanParams p{};
    p.x = g;
    p.out = gcum;
    p.seq = (long long)seq;
    p.ch = (long long)ch;
    return run_scan<CUMSUM, KAI_GDN_F32, KAI_GDN_F32>(p, batch, st, "cumsum");
}

int launch_gated_scan(const float *g, const float *x, float *s, void *state, int sdt,
                      size_t batch, size_t seq, size_t ch, cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!g || !x || !s || !state) return set_error(KAI_GDN_ERR_INVALID, "gated_scan: null pointer");
    ScanParams p{};
    p.x = x;
    p.g = g;
    p.out = s;
    p.state = state;
    p.seq = (long long)seq;
    p.ch = (long long)ch;
    switch (sdt) {
        case KAI_GDN_F32: return run_scan<AFFINE, KAI_GDN_F32, KAI_GDN_F32>(p, batch, st, "gated_scan");
        case KAI_GDN_F16: return run_scan<AFFINE, KAI_GDN_F32, KAI_GDN_F16>(p, batch, st, "gated_scan");
        case KAI_GDN_BF16: return run_scan<AFFINE, KAI_GDN_F32, KAI_GDN_BF16>(p, batch, st, "gated_scan");
    }
    return set_error(KAI_GDN_ERR_INVALID, "gated_scan: bad state dtype %d", sdt);
}

int launch_gdn2_scan(const float *g, const float *bg, const float *wg, const float *x,
                     float *s, float *state, size_t batch, size_t seq, size_t ch,
                     cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!g || !bg || !wg || !x || !s || !state)
        return set_error(KAI_GDN_ERR_INVALID, "gdn2_gated_scan: null pointer");
    ScanParams p{};
    p.x = x;
    p.g = g;
    p.b = bg;
    p.w = wg;
    p.out = s;
    p.state = state;
    p.seq = (long long)seq;
    p.ch = (long long)ch;
    return run_scan<GDN2, KAI_GDN_F32, KAI_GDN_F32>(p, batch, st, "gdn2_gated_scan");
}

// ---------------------------------------------------------------------------
// Allocation-free gated scan.
//
// Some callers cannot allocate device memory when they call us: a serving
// engine that hands all of HBM to its own state / KV pool at start-up and
// budgets nothing for a library, or a host that keeps other streams busy and
// cannot afford cudaMalloc / cudaFree, which may synchronise the whole
// device.  kai_run_gdn_gated_scan_noalloc_sm100a serves them: the segment
// carries of a long scan live in the fixed array below instead of the
// library's cudaMalloc'd per-stream scratch.
//
// The array is part of the library's device image, so every GPU that loads
// the library holds KAI_GDN_NOALLOC_SCRATCH_BYTES of it until the process
// exits.  Host code cannot use the name `g_noalloc_scratch` as a device
// address (on the host it is only a stand-in), so the address is looked up
// once per device with cudaGetSymbolAddress, with that device current, on the
// first call there; that first call should come before any stream capture.
// Every call shares the array and overwrites what it uses (each element a
// call reads was written earlier in the same call, so nothing needs zeroing);
// calls that overlap on the GPU -- two streams, or two host threads -- race
// on it and must be serialised by the caller.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoallocFloats = KAI_GDN_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_noalloc_scratch[kNoallocFloats];

std::mutex g_noalloc_mu;
float *g_noalloc_ptr[64] = {nullptr};

int noalloc_scratch(float **out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "gated_scan_noalloc: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return set_error(KAI_GDN_ERR_UNSUPPORTED, "gated_scan_noalloc: device %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "gated_scan_noalloc: cudaGetSymbolAddress");
        if (rc) return rc;
        g_noalloc_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return KAI_GDN_OK;
}

template <int SDT>
int run_scan_noalloc(ScanParams p, size_t batch, cudaStream_t st) {
    const char *name = "gated_scan_noalloc";
    if (batch > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: batch %zu > 65535", name, batch);
    long long nseg = (p.seq + SEG_LEN - 1) / SEG_LEN;
    if (nseg > (1ll << 24)) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: seq too long", name);
    p.nseg = (int)nseg;
    int sw = nseg >= 8 ? 8 : nseg >= 4 ? 4 : nseg >= 2 ? 2 : 1;
    p.cw = 8 / sw;
    dim3 block(32, 8);
    long long gx = (p.ch + 32 * p.cw - 1) / (32 * p.cw);
    long long gy = (nseg + sw - 1) / sw;
    if (gx > 0x7fffffffll || gy > 65535)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: shape too large for the grid", name);
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)batch);
    int rc;
    if (nseg > 1) {
        size_t n = batch * (size_t)nseg * (size_t)p.ch;
        if (n > kNoallocFloats / 2)
            return set_error(KAI_GDN_ERR_INVALID,
                             "%s: batch*ceil(seq/%d)*channels = %zu needs %zu bytes of scratch; the static "
                             "maximum is %zu bytes (use kai_run_gdn_gated_scan_sm100a for larger calls)",
                             name, SEG_LEN, n, 2 * n * sizeof(float), (size_t)KAI_GDN_NOALLOC_SCRATCH_BYTES);
        float *scr = nullptr;
        if ((rc = noalloc_scratch(&scr))) return rc;
        p.aggA = scr;
        p.aggB = scr + n;
        scan_aggregate_kernel<AFFINE><<<grid, block, 0, st>>>(p);
        if ((rc = check_launch(name))) return rc;
        dim3 cgrid((unsigned)((p.ch + 127) / 128), (unsigned)batch);
        scan_carry_kernel<AFFINE, SDT><<<cgrid, 128, 0, st>>>(p);
        if ((rc = check_launch(name))) return rc;
    }
    scan_final_kernel<AFFINE, KAI_GDN_F32, SDT><<<grid, block, 0, st>>>(p);
    return check_launch(name);
}

}  // namespace

int launch_gated_scan_noalloc(const float *g, const float *x, float *s, void *state, int sdt, size_t batch,
                              size_t seq, size_t ch, cudaStream_t st) {
    if (batch == 0 || seq == 0 || ch == 0) return KAI_GDN_OK;
    if (!g || !x || !s || !state) return set_error(KAI_GDN_ERR_INVALID, "gated_scan_noalloc: null pointer");
    ScanParams p{};
    p.x = x;
    p.g = g;
    p.out = s;
    p.state = state;
    p.seq = (long long)seq;
    p.ch = (long long)ch;
    switch (sdt) {
        case KAI_GDN_F32: return run_scan_noalloc<KAI_GDN_F32>(p, batch, st);
        case KAI_GDN_F16: return run_scan_noalloc<KAI_GDN_F16>(p, batch, st);
        case KAI_GDN_BF16: return run_scan_noalloc<KAI_GDN_BF16>(p, batch, st);
    }
    return set_error(KAI_GDN_ERR_INVALID, "gated_scan_noalloc: bad state dtype %d", sdt);
}

}  // namespace gdn
