// scan.cu -- the channel-wise recurrences of the GDN hot path on sm_100a:
//   cumdecay  decay[t] = prod_{i<=t} a[i]      kai_gdn_cumdecay_f32_sve.c:82-89
//   cumsum    gcum[t]  = sum_{i<=t} g[i]       (log-space twin of cumdecay)
//   gated     s[t] = x[t] + s[t-1]*g[t]        kai_gdn_gated_scan_f32_sve.c:86-95
//   gdn2      s[t] = w[t]*x[t] + s[t-1]*(g[t]*b[t])   gdn_sve.c:865-872
//
// All are HBM-bound: one read of each input stream, one write of the output.
// Layout [batch][seq][channels]; a warp covers 32 consecutive channels of one
// row, so every access is a full 128-byte line.  Every step uses the
// reference's operation order with one rounding per operation
// (__fmul_rn / __fadd_rn, no FMA contraction).
//
// seq <= SEG_LEN (128): one thread walks each channel's whole sequence, so
// the result is bit-identical to the reference's scalar path (the reference's
// own tests require this at T = 64).
//
// Longer sequences: a single pass with decoupled look-back.  A tile is
// 8*RPW rows x 32 channels; each of its 256 threads holds RPW rows of one
// channel in registers.  The tile's aggregate (the product, the sum, or the
// affine map s -> A*s + B) is published per channel; the tile then walks back
// over its predecessors' records, eight at a time (one per warp), composing
// their aggregates until it finds one that already holds its inclusive prefix,
// publishes its own inclusive prefix and writes its outputs from registers.  Tiles are numbered by an
// atomic counter in the order blocks start, so a tile only ever waits for
// tiles that are already running; every wait is bounded and a timeout sets an
// error word instead of hanging.  HBM traffic is the algorithmic one (read
// once, write once) plus a 16-byte record per tile and channel.
#include <mutex>

#include "gdn_internal.cuh"

namespace gdn {
namespace {

constexpr int SEG_LEN = 128;  // rows per thread in the exact single-walk path
constexpr int BATCH_LD = 8;   // loads issued ahead of the dependent chain

enum Op { CUMPROD = 0, CUMSUM = 1, AFFINE = 2, GDN2 = 3 };

struct ScanParams {
    const float *x;  // cumprod: a, cumsum: g, affine/gdn2: x
    const float *g;  // affine/gdn2 gate
    const float *b;  // gdn2 erase gate
    const float *w;  // gdn2 write gate
    void *out;       // [batch][seq][ch]
    void *state;     // affine/gdn2: [batch][ch]
    long long seq, ch;
    int cw;          // single-walk path: warps per block along channels
};

template <int OP> struct Nin { static constexpr int n = OP == GDN2 ? 4 : (OP == AFFINE ? 2 : 1); };

template <int OP>
__device__ __forceinline__ float step(float run, const float *v) {
    if (OP == CUMPROD) return __fmul_rn(run, v[0]);
    if (OP == CUMSUM) return __fadd_rn(run, v[0]);
    if (OP == AFFINE) return __fadd_rn(v[0], __fmul_rn(run, v[1]));
    return __fadd_rn(__fmul_rn(v[3], v[0]), __fmul_rn(run, __fmul_rn(v[1], v[2])));
}

template <int OP>
__device__ __forceinline__ void load_row(const ScanParams &p, size_t idx, float *v) {
    v[0] = __ldg(p.x + idx);
    if (OP == AFFINE || OP == GDN2) v[1] = __ldg(p.g + idx);
    if (OP == GDN2) {
        v[2] = __ldg(p.b + idx);
        v[3] = __ldg(p.w + idx);
    }
}

// Aggregates compose as maps s -> A*s + B (A = product of multipliers, B = the
// scan from 0); for cumprod only A is used, for cumsum only B.
struct Agg {
    float A, B;
};
template <int OP> __device__ __forceinline__ Agg agg_identity() { return {1.0f, 0.0f}; }
// Fold one element into a running aggregate (the element comes after it).
template <int OP>
__device__ __forceinline__ Agg agg_push(Agg a, const float *v) {
    if (OP == CUMPROD) return {__fmul_rn(a.A, v[0]), 0.0f};
    if (OP == CUMSUM) return {1.0f, __fadd_rn(a.B, v[0])};
    const float m = OP == AFFINE ? v[1] : __fmul_rn(v[1], v[2]);
    return {__fmul_rn(a.A, m), step<OP>(a.B, v)};
}
// first, then second
template <int OP>
__device__ __forceinline__ Agg agg_then(Agg first, Agg second) {
    if (OP == CUMPROD) return {__fmul_rn(first.A, second.A), 0.0f};
    if (OP == CUMSUM) return {1.0f, __fadd_rn(first.B, second.B)};
    return {__fmul_rn(first.A, second.A), __fadd_rn(__fmul_rn(first.B, second.A), second.B)};
}
// Apply an aggregate to a carried value.
template <int OP>
__device__ __forceinline__ float agg_apply(Agg a, float s) {
    if (OP == CUMPROD) return __fmul_rn(s, a.A);
    if (OP == CUMSUM) return __fadd_rn(s, a.B);
    return __fadd_rn(a.B, __fmul_rn(s, a.A));
}

template <int OP, int SDT>
__device__ __forceinline__ float initial_carry(const ScanParams &p, long long b, long long c) {
    if (OP == CUMPROD) return 1.0f;
    if (OP == CUMSUM) return 0.0f;
    using S = Store<SDT>;
    return S::load(reinterpret_cast<const typename S::T *>(p.state) + b * p.ch + c);
}

// ------------------------------------------------------ exact single walk
// One thread per channel walks the whole (<= SEG_LEN rows) sequence.
// blockDim = (32, 8): warps are channel groups.
template <int OP, int ODT, int SDT>
__global__ void __launch_bounds__(256) scan_walk_kernel(ScanParams p) {
    const long long c = (long long)blockIdx.x * 256 + threadIdx.y * 32 + threadIdx.x;
    const long long b = blockIdx.z;
    if (c >= p.ch) return;
    const size_t base = (size_t)b * p.seq * p.ch + (size_t)c;
    float run = initial_carry<OP, SDT>(p, b, c);
    using O = Store<ODT>;
    typename O::T *out = reinterpret_cast<typename O::T *>(p.out);
    long long t = 0;
    for (; t + BATCH_LD <= p.seq; t += BATCH_LD) {
        float v[BATCH_LD][4];
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) load_row<OP>(p, base + (size_t)(t + r) * p.ch, v[r]);
#pragma unroll
        for (int r = 0; r < BATCH_LD; ++r) {
            run = step<OP>(run, v[r]);
            O::store(out + base + (size_t)(t + r) * p.ch, run);
        }
    }
    for (; t < p.seq; ++t) {
        float v[4];
        load_row<OP>(p, base + (size_t)t * p.ch, v);
        run = step<OP>(run, v);
        O::store(out + base + (size_t)t * p.ch, run);
    }
    if (OP == AFFINE || OP == GDN2) {
        using S = Store<SDT>;
        S::store(reinterpret_cast<typename S::T *>(p.state) + b * p.ch + c, run);
    }
}

// ------------------------------------------------ single pass, look-back
struct __align__(16) TileRecord {
    unsigned int flag;  // 0 empty, 1 aggregate (A, B) ready, 2 inclusive prefix P ready too
    float A, B;         // the tile's aggregate map (never rewritten once flag is set)
    float P;            // the carried value after the tile
};

struct Lookback {
    unsigned int *counter;  // tile ticket, zeroed before the launch
    int *err;               // set when a wait runs out
    TileRecord *rec;        // [ntiles][32], zeroed before the launch
    long long nct, ntr, batch;
};

constexpr uint32_t SPIN_LIMIT = 1u << 22;

__device__ __forceinline__ unsigned int ld_flag(const TileRecord *r) {
    return *reinterpret_cast<const volatile unsigned int *>(&r->flag);
}

__device__ __forceinline__ void publish_aggregate(TileRecord *r, float A, float B) {
    *reinterpret_cast<volatile float *>(&r->A) = A;
    *reinterpret_cast<volatile float *>(&r->B) = B;
    __threadfence();
    *reinterpret_cast<volatile unsigned int *>(&r->flag) = 1u;
}
__device__ __forceinline__ void publish_prefix(TileRecord *r, float P) {
    *reinterpret_cast<volatile float *>(&r->P) = P;
    __threadfence();
    *reinterpret_cast<volatile unsigned int *>(&r->flag) = 2u;
}

template <int OP, int ODT, int SDT, int RPW>
__global__ void __launch_bounds__(256) scan_lookback_kernel(ScanParams p, Lookback lb) {
    constexpr int NIN = Nin<OP>::n, TROWS = 8 * RPW;
    __shared__ long long s_tile;
    __shared__ float s_A[8][32], s_B[8][32], s_carry[32], s_tile_agg[2][32], s_acc[2][32];
    __shared__ float s_rA[8][32], s_rB[8][32], s_rP[8][32];
    __shared__ unsigned int s_rf[8][32];
    __shared__ int s_done[32];
    const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
    if (threadIdx.x == 0) s_tile = (long long)atomicAdd(lb.counter, 1u);
    __syncthreads();
    const long long id = s_tile;
    const long long chains = lb.batch * lb.nct;
    const long long tr = id / chains, chain = id % chains, b = chain / lb.nct, ct = chain % lb.nct;
    const long long c = ct * 32 + lane;
    const bool live_c = c < p.ch;
    const long long row0 = tr * TROWS + (long long)w * RPW;
    const size_t base = (size_t)b * p.seq * p.ch + (size_t)c;

    // rows of this thread that exist (the last tile of a sequence is ragged)
    const int nrow = live_c ? (int)max(0ll, min((long long)RPW, p.seq - row0)) : 0;
    const size_t first = base + (size_t)row0 * p.ch;
    const size_t stride = (size_t)p.ch;
    float v[RPW][NIN];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        if (r < nrow) {
            float t4[4];
            load_row<OP>(p, first + (size_t)r * stride, t4);
#pragma unroll
            for (int k = 0; k < NIN; ++k) v[r][k] = t4[k];
        }
    }
    Agg a = agg_identity<OP>();
#pragma unroll
    for (int r = 0; r < RPW; ++r)
        if (r < nrow) a = agg_push<OP>(a, v[r]);
    s_A[w][lane] = a.A;
    s_B[w][lane] = a.B;
    __syncthreads();

    // Tile aggregate per channel, published at once so that successors can
    // look past this tile while it looks back itself.
    if (w == 0) {
        Agg tile = agg_identity<OP>();
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) tile = agg_then<OP>(tile, {s_A[ww][lane], s_B[ww][lane]});
        s_tile_agg[0][lane] = tile.A;
        s_tile_agg[1][lane] = tile.B;
        if (tr == 0) s_carry[lane] = live_c ? initial_carry<OP, SDT>(p, b, c) : 0.0f;
        else publish_aggregate(lb.rec + (size_t)id * 32 + lane, tile.A, tile.B);
        s_acc[0][lane] = 1.0f;  // composed maps of the predecessors walked so far
        s_acc[1][lane] = 0.0f;
        s_done[lane] = tr == 0;
    }
    __syncthreads();
    // Look back 8 predecessors per round, one per warp, nearest first.
    for (long long base = tr - 1; base >= 0; base -= 8) {
        if (__syncthreads_and(s_done[lane] != 0) ) break;
        const long long k = base - w;
        unsigned int f = 2u;
        float pA = 1.0f, pB = 0.0f, pP = 0.0f;
        if (k >= 0 && !s_done[lane]) {
            const TileRecord *pr = lb.rec + (size_t)(k * chains + chain) * 32 + lane;
            f = 0;
            for (uint32_t it = 0; it < SPIN_LIMIT; ++it) {
                f = ld_flag(pr);
                if (f) break;
                __nanosleep(32);
            }
            if (!f) {
                atomicExch(lb.err, 1);
                f = 2u;  // give up on this chain: treat as a prefix of 0
            }
            __threadfence();
            pA = *reinterpret_cast<const volatile float *>(&pr->A);
            pB = *reinterpret_cast<const volatile float *>(&pr->B);
            pP = *reinterpret_cast<const volatile float *>(&pr->P);
        }
        s_rf[w][lane] = f;
        s_rA[w][lane] = pA;
        s_rB[w][lane] = pB;
        s_rP[w][lane] = pP;
        __syncthreads();
        if (w == 0 && !s_done[lane]) {
            Agg acc = {s_acc[0][lane], s_acc[1][lane]};
            for (int ww = 0; ww < 8; ++ww) {
                if (base - ww < 0) break;
                if (s_rf[ww][lane] == 2u) {
                    s_carry[lane] = agg_apply<OP>(acc, s_rP[ww][lane]);
                    s_done[lane] = 1;
                    break;
                }
                acc = agg_then<OP>({s_rA[ww][lane], s_rB[ww][lane]}, acc);
            }
            s_acc[0][lane] = acc.A;
            s_acc[1][lane] = acc.B;
        }
    }
    __syncthreads();
    if (w == 0)
        publish_prefix(lb.rec + (size_t)id * 32 + lane,
                       agg_apply<OP>({s_tile_agg[0][lane], s_tile_agg[1][lane]}, s_carry[lane]));
    float run = s_carry[lane];
    for (int ww = 0; ww < w; ++ww) run = agg_apply<OP>({s_A[ww][lane], s_B[ww][lane]}, run);
    using O = Store<ODT>;
    typename O::T *out = reinterpret_cast<typename O::T *>(p.out);
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        if (r < nrow) {
            run = step<OP>(run, v[r]);
            O::store(out + first + (size_t)r * stride, run);
            if ((OP == AFFINE || OP == GDN2) && row0 + r == p.seq - 1) {
                using S = Store<SDT>;
                S::store(reinterpret_cast<typename S::T *>(p.state) + b * p.ch + c, run);
            }
        }
    }
}

template <int OP> constexpr int rows_per_warp() { return OP == GDN2 ? 16 : 32; }

// Scratch bytes of a look-back launch: ticket + error word, then the records.
size_t lookback_bytes(size_t batch, long long seq, long long ch, int rpw) {
    const long long ntr = (seq + 8 * rpw - 1) / (8 * rpw), nct = (ch + 31) / 32;
    return 256 + (size_t)ntr * (size_t)nct * batch * 32 * sizeof(TileRecord);
}

template <int OP, int ODT, int SDT>
int run_scan_with(ScanParams p, size_t batch, cudaStream_t st, const char *name, void *scratch) {
    constexpr int RPW = rows_per_warp<OP>();
    if (p.seq <= SEG_LEN) {
        if (batch > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: batch %zu > 65535", name, batch);
        long long gx = (p.ch + 255) / 256;
        if (gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: too many channels", name);
        scan_walk_kernel<OP, ODT, SDT><<<dim3((unsigned)gx, 1, (unsigned)batch), dim3(32, 8), 0, st>>>(p);
        return check_launch(name);
    }
    Lookback lb;
    lb.ntr = (p.seq + 8 * RPW - 1) / (8 * RPW);
    lb.nct = (p.ch + 31) / 32;
    lb.batch = (long long)batch;
    const long long tiles = lb.ntr * lb.nct * lb.batch;
    if (tiles > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: shape too large", name);
    const size_t bytes = lookback_bytes(batch, p.seq, p.ch, RPW);
    int rc = check_cuda(cudaMemsetAsync(scratch, 0, bytes, st), name);
    if (rc) return rc;
    lb.counter = static_cast<unsigned int *>(scratch);
    lb.err = reinterpret_cast<int *>(static_cast<char *>(scratch) + 16);
    lb.rec = reinterpret_cast<TileRecord *>(static_cast<char *>(scratch) + 256);
    scan_lookback_kernel<OP, ODT, SDT, RPW><<<(unsigned)tiles, 256, 0, st>>>(p, lb);
    return check_launch(name);
}

template <int OP, int ODT, int SDT>
int run_scan(ScanParams p, size_t batch, cudaStream_t st, const char *name) {
    void *scr = nullptr;
    if (p.seq > SEG_LEN) {
        int rc = scratch_for_stream(st, lookback_bytes(batch, p.seq, p.ch, rows_per_warp<OP>()), &scr);
        if (rc) return rc;
    }
    return run_scan_with<OP, ODT, SDT>(p, batch, st, name, scr);
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
// device.  kai_run_gdn_gated_scan_noalloc_sm100a serves them: the look-back
// records of a long scan live in the fixed array below instead of the
// library's cudaMalloc'd per-stream scratch.
//
// The array is part of the library's device image, so every GPU that loads
// the library holds KAI_GDN_NOALLOC_SCRATCH_BYTES of it until the process
// exits.  Host code cannot use the name `g_noalloc_scratch` as a device
// address (on the host it is only a stand-in), so the address is looked up
// once per device with cudaGetSymbolAddress, with that device current, on the
// first call there; that first call should come before any stream capture.
// Every call shares the array; each call clears (cudaMemsetAsync, which
// allocates nothing) the part it uses before its kernel runs.  Calls that
// overlap on the GPU -- two streams, or two host threads -- race on it and
// must be serialised by the caller.
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
    float *scr = nullptr;
    if (p.seq > SEG_LEN) {
        const size_t need = lookback_bytes(batch, p.seq, p.ch, rows_per_warp<AFFINE>());
        if (need > (size_t)KAI_GDN_NOALLOC_SCRATCH_BYTES)
            return set_error(KAI_GDN_ERR_INVALID,
                             "%s: batch %zu x seq %lld x channels %lld needs %zu bytes of scratch; the static "
                             "maximum is %zu bytes (use kai_run_gdn_gated_scan_sm100a for larger calls)",
                             name, batch, p.seq, p.ch, need, (size_t)KAI_GDN_NOALLOC_SCRATCH_BYTES);
        int rc = noalloc_scratch(&scr);
        if (rc) return rc;
    }
    return run_scan_with<AFFINE, KAI_GDN_F32, SDT>(p, batch, st, name, scr);
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
