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
// channel in registers.  A tile issues its loads, and while they are in
// flight walks back over its predecessors' records (eight per round, one per
// warp), composing their aggregates (the product, the sum, or the affine map
// s -> A*s + B) until it finds one that holds its inclusive prefix.  If a
// predecessor has published nothing yet, the tile instead publishes its own
// aggregate as soon as its loads have landed, so that successors can look
// past it, and then looks back again, waiting.  It then publishes its
// inclusive prefix and writes its outputs from registers.  Tiles are numbered
// by an atomic counter in the order blocks start, so a tile only ever waits
// for tiles that are already running; every wait is bounded and a timeout
// sets an error word instead of hanging.  HBM traffic is the algorithmic one
// (read once, write once) plus a 16-byte record per tile and channel.
#include <algorithm>
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
// A lane owns one channel of a tile; its look-back record is one aligned
// 16-byte word, written with one vector store and polled with one vector
// load, so a reader sees a whole record or none of it and no fence is needed
// on either side (nothing else is published through it).  Measured on B200
// against release / acquire accesses of a separate flag: the fences were a
// tenth of the gated scan's time (32768 x 4096: 376 -> 335 us) and a quarter
// of the prefix product's (4096 x 4096: 47 -> 36 us).
struct __align__(16) TileRecord {
    unsigned int flag;  // 0 empty, 1 aggregate (A, B) ready, 2 inclusive prefix P ready too
    float A, B;         // the tile's aggregate map
    float P;            // the carried value after the tile (flag 2)
};
static_assert(sizeof(TileRecord) == 16, "one 16-byte word");

struct Lookback {
    unsigned int *counter;  // tile ticket, zeroed before the launch
    int *err;               // the library's device error word: set when a wait runs out
    void *rec;              // [ntiles][32] TileRecord, zeroed before the launch
    long long nct, ntr, batch;
    unsigned int first_spin;  // polls per record in the overlapped first look-back pass
};

constexpr uint32_t SPIN_LIMIT = 1u << 22;
// Polls of an unpublished record in the first (overlapped) look-back pass
// before a tile falls back to publishing its aggregate.  Worth waiting for
// when many independent chains separate a tile from its predecessor (the
// predecessor has usually finished); with few chains the predecessors run
// concurrently and publishing the aggregate at once lets the chain advance.
__host__ __device__ constexpr uint32_t first_spin(long long chains) { return chains >= 64 ? 16u : 0u; }

// Records go through L2 (volatile: not cached in L1).  A tile writes its
// record at most twice (flag 1, then flag 2), from the same thread.
__device__ __forceinline__ void publish(TileRecord *r, float A, float B, float P, unsigned int flag) {
    asm volatile("st.volatile.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(r), "r"(flag), "r"(__float_as_uint(A)),
                 "r"(__float_as_uint(B)), "r"(__float_as_uint(P))
                 : "memory");
}
__device__ __forceinline__ TileRecord load_record(const TileRecord *r) {
    TileRecord v;
    unsigned int a, b, p;
    asm volatile("ld.volatile.global.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.flag), "=r"(a), "=r"(b), "=r"(p)
                 : "l"(r)
                 : "memory");
    v.A = __uint_as_float(a);
    v.B = __uint_as_float(b);
    v.P = __uint_as_float(p);
    return v;
}

// VEC consecutive fp32 values at p (16-byte aligned when VEC = 4).  The loads
// are volatile so they stay ahead of the look-back, which overlaps them.
template <int VEC> __device__ __forceinline__ void ldv(const float *p, float *v) {
    if (VEC == 4) {
        asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                     : "l"(p));
    } else {
        asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v[0]) : "l"(p));
    }
}
template <int ODT, int VEC> __device__ __forceinline__ void stv(void *base, size_t idx, const float *v) {
    using O = Store<ODT>;
    typename O::T *out = reinterpret_cast<typename O::T *>(base) + idx;
    if (VEC == 4 && ODT == KAI_GDN_F32) {
        *reinterpret_cast<float4 *>(out) = make_float4(v[0], v[1], v[2], v[3]);
    } else if (VEC == 4) {
        uint2 u;
        typename O::T *h = reinterpret_cast<typename O::T *>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) O::store(h + k, v[k]);
        *reinterpret_cast<uint2 *>(out) = u;
    } else {
        O::store(out, v[0]);
    }
}

// Tile: W*RPW rows x 32*VEC channels of one batch; warp w holds rows
// row0 + w*RPW .. + RPW-1, lane l channels l*VEC .. l*VEC + VEC-1.
// Order of work: issue the tile's loads; while they are in flight, try to find
// the carry into the tile from the predecessors' records (composing their
// aggregate maps until one holds its inclusive prefix, giving up at a record
// not yet published); reduce the tile; if the carry is still unknown, publish
// the tile's aggregate and look back again, waiting this time; publish the
// inclusive prefix and write the outputs from registers.
// Zeroes the ticket and records of a look-back launch.  The scan kernel is
// launched as its programmatic dependent: it may be placed at once and waits
// (griddepcontrol.wait) for this kernel to complete before it touches
// memory, which spares the gap between two stream operations.
__global__ void __launch_bounds__(256) zero_records_kernel(uint4 *p, size_t n16) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    for (size_t i = (size_t)blockIdx.x * 256 + threadIdx.x; i < n16; i += (size_t)gridDim.x * 256)
        p[i] = make_uint4(0u, 0u, 0u, 0u);
}

template <int OP, int ODT, int SDT, int VEC, int RPW, int W>
__global__ void __launch_bounds__(32 * W, W < 16 ? 16 / W : 1) scan_lookback_kernel(ScanParams p, Lookback lb) {
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the records are zero
    static_assert(VEC == 1, "one channel per lane: the look-back record is one 16-byte word");
    constexpr int NIN = Nin<OP>::n, TROWS = W * RPW, TC = 32 * VEC;
    using Rec = TileRecord;
    __shared__ long long s_tile;
    __shared__ float s_A[W][TC], s_B[W][TC], s_carry[TC], s_acc[2][TC];
    __shared__ float s_rA[W][TC], s_rB[W][TC], s_rP[W][TC];
    __shared__ unsigned int s_rf[W][32];
    __shared__ int s_done[32];
    const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
    if (threadIdx.x == 0) s_tile = (long long)atomicAdd(lb.counter, 1u);
    __syncthreads();
    const long long id = s_tile;
    const long long chains = lb.batch * lb.nct;
    const long long tr = id / chains, chain = id % chains, b = chain / lb.nct, ct = chain % lb.nct;
    const long long c = ct * TC + (long long)lane * VEC;  // first channel of this lane
    const bool live_c = c < p.ch;
    const long long row0 = tr * TROWS + (long long)w * RPW;
    Rec *rec = static_cast<Rec *>(lb.rec);

    // rows of this thread that exist (the last tile of a sequence is ragged)
    const int nrow = live_c ? (int)max(0ll, min((long long)RPW, p.seq - row0)) : 0;
    const size_t first = (size_t)b * p.seq * p.ch + (size_t)row0 * p.ch + (size_t)c;
    const size_t stride = (size_t)p.ch;
    float v[RPW][NIN][VEC];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        if (r < nrow) {
            const size_t idx = first + (size_t)r * stride;
            ldv<VEC>(p.x + idx, v[r][0]);
            if (OP == AFFINE || OP == GDN2) ldv<VEC>(p.g + idx, v[r][1]);
            if (OP == GDN2) {
                ldv<VEC>(p.b + idx, v[r][2]);
                ldv<VEC>(p.w + idx, v[r][3]);
            }
        }
    }

    // Walk back over the predecessors' records, W per round (one per warp),
    // nearest first, composing aggregate maps until one holds its inclusive
    // prefix.  With `blocking` false a record that is not published yet ends
    // the walk without a result (first pass, while this tile's loads are in
    // flight); with `blocking` true every wait is bounded by SPIN_LIMIT.
    auto look_back = [&](bool blocking) {
        if (w == 0) {
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                const int cc = lane * VEC + k;
                if (tr == 0) s_carry[cc] = live_c ? initial_carry<OP, SDT>(p, b, c + k) : 0.0f;
                s_acc[0][cc] = 1.0f;  // composed maps of the predecessors walked so far
                s_acc[1][cc] = 0.0f;
            }
            s_done[lane] = tr == 0 ? 1 : 0;  // 1 carry known, 2 gave up (blocking == false)
        }
        __syncthreads();
        for (long long base = tr - 1; base >= 0; base -= W) {
            if (__syncthreads_and(s_done[lane] != 0)) break;
            const long long kt = base - w;
            Rec r{2u, 1.0f, 0.0f, 0.0f};
            if (kt >= 0 && !s_done[lane]) {
                const Rec *pr = rec + (size_t)(kt * chains + chain) * 32 + lane;
                r = load_record(pr);
                for (uint32_t it = 0; !r.flag && it < (blocking ? SPIN_LIMIT : lb.first_spin); ++it) {
                    __nanosleep(32);
                    r = load_record(pr);
                }
                if (blocking && !r.flag) {
                    atomicExch(lb.err, 1);
                    r = {2u, 0.0f, 0.0f, 0.0f};  // give up on this chain: treat as a prefix of 0
                }
            }
            s_rf[w][lane] = r.flag;
            s_rA[w][lane] = r.A;
            s_rB[w][lane] = r.B;
            s_rP[w][lane] = r.P;
            __syncthreads();
            if (w == 0 && !s_done[lane]) {
                Agg acc[VEC];
#pragma unroll
                for (int k = 0; k < VEC; ++k) acc[k] = {s_acc[0][lane * VEC + k], s_acc[1][lane * VEC + k]};
                for (int ww = 0; ww < W; ++ww) {
                    if (base - ww < 0) break;
                    const unsigned int fw = s_rf[ww][lane];
                    if (fw == 0u) {  // not published yet (first pass only)
                        s_done[lane] = 2;
                        break;
                    }
                    if (fw == 2u) {
#pragma unroll
                        for (int k = 0; k < VEC; ++k)
                            s_carry[lane * VEC + k] = agg_apply<OP>(acc[k], s_rP[ww][lane * VEC + k]);
                        s_done[lane] = 1;
                        break;
                    }
#pragma unroll
                    for (int k = 0; k < VEC; ++k)
                        acc[k] = agg_then<OP>({s_rA[ww][lane * VEC + k], s_rB[ww][lane * VEC + k]}, acc[k]);
                }
#pragma unroll
                for (int k = 0; k < VEC; ++k) {
                    s_acc[0][lane * VEC + k] = acc[k].A;
                    s_acc[1][lane * VEC + k] = acc[k].B;
                }
            }
        }
        __syncthreads();
    };
    look_back(false);  // overlaps this tile's loads
    // The tile's own aggregate (the loads land here).
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        Agg a = agg_identity<OP>();
#pragma unroll
        for (int r = 0; r < RPW; ++r)
            if (r < nrow) {
                float e[4];
#pragma unroll
                for (int q = 0; q < NIN; ++q) e[q] = v[r][q][k];
                a = agg_push<OP>(a, e);
            }
        s_A[w][lane * VEC + k] = a.A;
        s_B[w][lane * VEC + k] = a.B;
    }
    __syncthreads();
    const bool known = __syncthreads_and(s_done[lane] == 1);
    float tA[VEC], tB[VEC];
    if (w == 0) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            const int cc = lane * VEC + k;
            Agg tile = agg_identity<OP>();
#pragma unroll
            for (int ww = 0; ww < W; ++ww) tile = agg_then<OP>(tile, {s_A[ww][cc], s_B[ww][cc]});
            tA[k] = tile.A;
            tB[k] = tile.B;
        }
        // Successors can look past this tile while it is still looking back.
        if (!known) publish(rec + (size_t)id * 32 + lane, tA[0], tB[0], 0.0f, 1u);
    }
    if (!known) look_back(true);
    if (w == 0) {
        float P[VEC];
#pragma unroll
        for (int k = 0; k < VEC; ++k) P[k] = agg_apply<OP>({tA[k], tB[k]}, s_carry[lane * VEC + k]);
        publish(rec + (size_t)id * 32 + lane, tA[0], tB[0], P[0], 2u);
    }
    float run[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        const int cc = lane * VEC + k;
        run[k] = s_carry[cc];
        for (int ww = 0; ww < w; ++ww) run[k] = agg_apply<OP>({s_A[ww][cc], s_B[ww][cc]}, run[k]);
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        if (r < nrow) {
            const size_t o = first + (size_t)r * stride;
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                float e[4];
#pragma unroll
                for (int q = 0; q < NIN; ++q) e[q] = v[r][q][k];
                run[k] = step<OP>(run[k], e);
            }
            stv<ODT, VEC>(p.out, o, run);
            if ((OP == AFFINE || OP == GDN2) && row0 + r == p.seq - 1) {
                using S = Store<SDT>;
#pragma unroll
                for (int k = 0; k < VEC; ++k)
                    S::store(reinterpret_cast<typename S::T *>(p.state) + b * p.ch + c + k, run[k]);
            }
        }
    }
}

// Geometry of a look-back launch: channels per lane, rows per warp, warps.
struct Geo {
    int vec, rpw, w;
};
// 8 warps of 32 rows (16 for gdn2) x 32 channels: 256-row tiles (128 for gdn2),
// one 128-byte line per warp and row.  Measured on B200 against taller,
// shorter and four-channels-per-lane tiles, this keeps the most tiles of
// independent chains in flight per SM.  The allocation-free entry point uses
// it too, so its scratch bound is fixed.
template <int OP> constexpr Geo narrow_geo() { return {1, OP == GDN2 ? 16 : 32, 8}; }
// With few independent chains (batch x 32-channel groups) the chains' tiles
// mostly wait on one another: each round of a look-back reads one record per
// warp, so a tile far down a chain of 256-row tiles walks many dependent
// rounds (cumsum at 8 x 32768 x 32: 128 tiles per chain).  One-input scans
// then take 1024-row tiles (32 warps x 32 rows): a quarter of the tiles per
// chain, and 32 records per round.  Fewer tiles also means fewer records, so
// the scratch bound of the narrow geometry still holds.
constexpr long long TALL_CHAINS = 32;
template <int OP> constexpr Geo tall_geo() { return {1, 32, 32}; }

// Scratch bytes of a look-back launch: the ticket, then the records.
size_t lookback_bytes(size_t batch, long long seq, long long ch, Geo g) {
    const long long ntr = (seq + g.w * g.rpw - 1) / (g.w * g.rpw), nct = (ch + 32 * g.vec - 1) / (32 * g.vec);
    return 256 + (size_t)ntr * (size_t)nct * batch * 32 * sizeof(TileRecord);
}

template <int OP, int ODT, int SDT, int VEC, int RPW, int W>
int launch_lookback(ScanParams p, size_t batch, cudaStream_t st, const char *name, void *scratch) {
    constexpr Geo g{VEC, RPW, W};
    Lookback lb;
    lb.ntr = (p.seq + W * RPW - 1) / (W * RPW);
    lb.nct = (p.ch + 32 * VEC - 1) / (32 * VEC);
    lb.batch = (long long)batch;
    lb.first_spin = first_spin(lb.nct * lb.batch);
    const long long tiles = lb.ntr * lb.nct * lb.batch;
    if (tiles > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: shape too large", name);
    const size_t n16 = lookback_bytes(batch, p.seq, p.ch, g) / 16;  // 256 + 512 per tile: whole 16-byte words
    lb.counter = static_cast<unsigned int *>(scratch);
    int rc = device_error_word(&lb.err);
    if (rc) return rc;
    lb.rec = static_cast<char *>(scratch) + 256;
    const unsigned zg = (unsigned)std::min<size_t>((n16 + 255) / 256, 4 * (size_t)sm_count());
    zero_records_kernel<<<zg, 256, 0, st>>>(static_cast<uint4 *>(scratch), n16);
    if ((rc = check_launch(name))) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)tiles);
    cfg.blockDim = dim3(32 * W);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, scan_lookback_kernel<OP, ODT, SDT, VEC, RPW, W>, p, lb);
    if (le != cudaSuccess) return check_cuda(le, name);
    return check_launch(name);
}

template <int OP, int ODT, int SDT>
int run_scan_with(ScanParams p, size_t batch, cudaStream_t st, const char *name, void *scratch) {
    if (p.seq <= SEG_LEN) {
        if (batch > 65535) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: batch %zu > 65535", name, batch);
        long long gx = (p.ch + 255) / 256;
        if (gx > 0x7fffffffll) return set_error(KAI_GDN_ERR_UNSUPPORTED, "%s: too many channels", name);
        scan_walk_kernel<OP, ODT, SDT><<<dim3((unsigned)gx, 1, (unsigned)batch), dim3(32, 8), 0, st>>>(p);
        return check_launch(name);
    }
    if constexpr (Nin<OP>::n == 1) {
        if ((long long)batch * ((p.ch + 31) / 32) < TALL_CHAINS) {
            constexpr Geo t = tall_geo<OP>();
            return launch_lookback<OP, ODT, SDT, t.vec, t.rpw, t.w>(p, batch, st, name, scratch);
        }
    }
    constexpr Geo g = narrow_geo<OP>();
    return launch_lookback<OP, ODT, SDT, g.vec, g.rpw, g.w>(p, batch, st, name, scratch);
}

template <int OP, int ODT, int SDT>
int run_scan(ScanParams p, size_t batch, cudaStream_t st, const char *name) {
    void *scr = nullptr;
    if (p.seq > SEG_LEN) {
        int rc = scratch_for_stream(st, lookback_bytes(batch, p.seq, p.ch, narrow_geo<OP>()), &scr);
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
// Every call shares the array; each call clears (with a small zeroing
// kernel, which allocates nothing) the part it uses before its scan kernel
// runs.  Calls that
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
        const size_t need = lookback_bytes(batch, p.seq, p.ch, narrow_geo<AFFINE>());
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
