// e2e.cu -- the reference's end-to-end hybrid decode loop on the GPU: one
// token through every layer, for `batch` independent sequences at once.
//   decode loop          src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:2775-2796
//   GDN layer            gdn_layer_forward      :1426-1490
//   attention layer      full_attn_layer_forward :1492-1522 (the loop's simulated attention)
//   FFN                  ffn_forward            :1834-1855
//   layer pattern        blocks of 3 GDN + 1 attention (:2414-2417)
//   weights              one set shared by all layers, int8 with per-column
//                        scales (the INT8_WEIGHTS build, :2311-2321)
// Per token and layer the engine launches the library's own kernels: the int8
// matmul for the projections (M = batch; the q/k/v projections of a layer and
// the FFN's gate/up pair each as one matmul over their concatenated columns,
// which quantize to the same codes and scales as the separate matrices), the
// causal Conv1D and the gated scan of the GDN stand-in, and two elementwise
// kernels (residual add, SiLU(gate) * up).  The GDN decay is the prefix
// product of one token's constant gate, i.e. the gate itself, so it is formed
// once.  The whole token is captured into a CUDA graph on the caller's stream
// and replayed (~330 launches for a 32-layer token, one graph launch).
//
// The reference's GDN stand-in scans VALUE_DIM channels with a decay vector of
// KEY_DIM entries (:1472-1476); when VALUE_DIM > KEY_DIM (its 4B geometry) it
// reads past that buffer.  This engine repeats the KEY_DIM gate values across
// the value channels there (decay[c] = beta[c mod KEY_DIM]); with KEY_DIM ==
// VALUE_DIM (the 0.8B geometry) it is the reference's computation.
#include <algorithm>
#include <initializer_list>
#include <utility>
#include <vector>

#include "gdn_internal.cuh"

namespace gdn {
namespace {

__global__ void add_kernel(float *__restrict__ out, const float *__restrict__ a, const float *__restrict__ b,
                           long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// act = g / (1 + exp(-g)) * up  (ffn_forward :1844-1847); gu rows are [gate | up]
__global__ void silu_mul_kernel(float *__restrict__ out, const float *__restrict__ gu, long long inter, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const long long b = i / inter, c = i % inter;
        const float x = gu[b * 2 * inter + c];
        out[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, expf(-x))), gu[b * 2 * inter + inter + c]);
    }
}

unsigned ew_grid(long long n) { return (unsigned)std::min<long long>((n + 255) / 256, 4ll * sm_count()); }

struct QWd {
    int8_t *q = nullptr;
    float *s = nullptr;
    size_t K = 0, N = 0;
};

}  // namespace

struct E2EEngine {
    kai_gdn_e2e_config cfg{};
    std::vector<unsigned char> is_gdn;
    int device = 0;
    QWd gqkv, go, fqkv, fo, gu, down;  // [q | k | v] and [gate | up] concatenated by columns
    float *conv_w = nullptr, *beta_b = nullptr;  // [4][conv_dim]; [batch][value_dim]
    std::vector<float *> gdn_state, conv_hist, kv_k, kv_v;
    float *h = nullptr, *h2 = nullptr, *qkv = nullptr, *v = nullptr, *conv_in = nullptr, *conv_out = nullptr,
          *scanned = nullptr, *proj = nullptr, *aqkv = nullptr, *aq = nullptr, *gu_out = nullptr, *act = nullptr;
    std::vector<void *> allocs;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t graph_stream = nullptr, last_stream = nullptr;
    int steps = 0;
};

namespace {

int dalloc(E2EEngine *e, void **p, size_t bytes, bool zero) {
    int rc = check_cuda(cudaMalloc(p, std::max<size_t>(bytes, 16)), "e2e: cudaMalloc");
    if (rc) return rc;
    e->allocs.push_back(*p);
    if (zero) rc = check_cuda(cudaMemset(*p, 0, std::max<size_t>(bytes, 16)), "e2e: cudaMemset");
    return rc;
}

// Quantize the column concatenation of host matrices [K][N_i] into one [K][sum N_i].
int make_qw(E2EEngine *e, QWd *w, std::initializer_list<std::pair<const float *, size_t>> parts, size_t K) {
    size_t N = 0;
    for (auto &pt : parts) {
        if (!pt.first) return set_error(KAI_GDN_ERR_INVALID, "e2e: null weight");
        N += pt.second;
    }
    float *tmp = nullptr;
    int rc = check_cuda(cudaMalloc(&tmp, K * N * sizeof(float)), "e2e: cudaMalloc");
    if (rc) return rc;
    size_t col = 0;
    for (auto &pt : parts) {
        if (!rc)
            rc = check_cuda(cudaMemcpy2D(tmp + col, N * sizeof(float), pt.first, pt.second * sizeof(float),
                                         pt.second * sizeof(float), K, cudaMemcpyHostToDevice),
                            "e2e: weight upload");
        col += pt.second;
    }
    if (!rc) rc = dalloc(e, (void **)&w->q, K * N, false);
    if (!rc) rc = dalloc(e, (void **)&w->s, N * sizeof(float), false);
    if (!rc) rc = launch_quantize_int8(tmp, w->q, w->s, K, N, 0);
    if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "e2e: quantize");
    cudaFree(tmp);
    w->K = K;
    w->N = N;
    return rc;
}

int mm(const float *A, const QWd &w, float *C, size_t M, cudaStream_t st) {
    return launch_matmul_int8(A, w.q, w.s, C, M, w.K, w.N, st);
}

// One token through every layer: h [B][hidden] in, h out.
int run_token(E2EEngine *e, cudaStream_t st) {
    const kai_gdn_e2e_config &c = e->cfg;
    const size_t B = c.batch, H = c.hidden, KD = c.key_dim, VD = c.value_dim, CD = c.conv_dim;
    const size_t qd = c.full_heads * c.full_head_dim, kvd = c.full_kv_heads * c.full_head_dim;
    int rc = 0;
#define E2E_TRY(x)          \
    do {                    \
        if ((rc = (x))) return rc; \
    } while (0)
    const size_t GQ = 2 * KD + VD, AQ = qd + 2 * kvd;  // widths of the concatenated projections
    for (size_t l = 0; l < c.layers; ++l) {
        if (e->is_gdn[l]) {
            // gdn_layer_forward: projections, Conv1D over [q | 0], gated scan of v with the gate
            // as decay, output projection, residual
            E2E_TRY(mm(e->h, e->gqkv, e->qkv, B, st));
            E2E_TRY(check_cuda(cudaMemcpy2DAsync(e->conv_in, CD * sizeof(float), e->qkv, GQ * sizeof(float),
                                                 std::min(KD, CD) * sizeof(float), B, cudaMemcpyDeviceToDevice, st),
                               "e2e: conv input"));
            E2E_TRY(check_cuda(cudaMemcpy2DAsync(e->v, VD * sizeof(float), e->qkv + 2 * KD, GQ * sizeof(float),
                                                 VD * sizeof(float), B, cudaMemcpyDeviceToDevice, st),
                               "e2e: v"));
            E2E_TRY(launch_conv(e->conv_in, e->conv_w, e->conv_out, e->conv_hist[l], KAI_GDN_F32, B, 1, CD, st));
            E2E_TRY(launch_gated_scan(e->beta_b, e->v, e->scanned, e->gdn_state[l], KAI_GDN_F32, B, 1, VD, st));
            E2E_TRY(mm(e->scanned, e->go, e->proj, B, st));
        } else {
            // full_attn_layer_forward: projections, the new K/V into the one-entry cache,
            // output projection of q (the loop's simulated attention), residual
            E2E_TRY(mm(e->h, e->fqkv, e->aqkv, B, st));
            E2E_TRY(check_cuda(cudaMemcpy2DAsync(e->kv_k[l], kvd * sizeof(float), e->aqkv + qd, AQ * sizeof(float),
                                                 kvd * sizeof(float), B, cudaMemcpyDeviceToDevice, st),
                               "e2e: kv"));
            E2E_TRY(check_cuda(cudaMemcpy2DAsync(e->kv_v[l], kvd * sizeof(float), e->aqkv + qd + kvd,
                                                 AQ * sizeof(float), kvd * sizeof(float), B,
                                                 cudaMemcpyDeviceToDevice, st),
                               "e2e: kv"));
            E2E_TRY(check_cuda(cudaMemcpy2DAsync(e->aq, qd * sizeof(float), e->aqkv, AQ * sizeof(float),
                                                 qd * sizeof(float), B, cudaMemcpyDeviceToDevice, st),
                               "e2e: q"));
            E2E_TRY(mm(e->aq, e->fo, e->proj, B, st));
        }
        add_kernel<<<ew_grid((long long)(B * H)), 256, 0, st>>>(e->h2, e->h, e->proj, (long long)(B * H));
        E2E_TRY(check_launch("add_kernel"));
        // ffn_forward: SwiGLU, residual
        E2E_TRY(mm(e->h2, e->gu, e->gu_out, B, st));
        silu_mul_kernel<<<ew_grid((long long)(B * c.inter)), 256, 0, st>>>(e->act, e->gu_out, (long long)c.inter,
                                                                         (long long)(B * c.inter));
        E2E_TRY(check_launch("silu_mul_kernel"));
        E2E_TRY(mm(e->act, e->down, e->proj, B, st));
        add_kernel<<<ew_grid((long long)(B * H)), 256, 0, st>>>(e->h, e->h2, e->proj, (long long)(B * H));
        E2E_TRY(check_launch("add_kernel"));
    }
#undef E2E_TRY
    (void)KD;
    return KAI_GDN_OK;
}

}  // namespace

int e2e_create(const kai_gdn_e2e_config *cfg, const kai_gdn_e2e_weights *w, void **out) {
    if (!cfg || !w || !out) return set_error(KAI_GDN_ERR_INVALID, "e2e_create: null argument");
    *out = nullptr;
    const kai_gdn_e2e_config &c = *cfg;
    if (!c.is_gdn || c.layers == 0 || c.batch == 0 || c.hidden == 0 || c.key_dim == 0 || c.value_dim == 0 ||
        c.conv_dim == 0 || c.inter == 0 || c.full_heads == 0 || c.full_kv_heads == 0 || c.full_head_dim == 0)
        return set_error(KAI_GDN_ERR_INVALID, "e2e_create: empty dimension");
    if (c.hidden % 16 || c.key_dim % 16 || c.value_dim % 16 || c.inter % 16 ||
        (c.full_heads * c.full_head_dim) % 16 || (c.full_kv_heads * c.full_head_dim) % 16)
        return set_error(KAI_GDN_ERR_UNSUPPORTED, "e2e_create: projection widths must be multiples of 16");
    E2EEngine *e = new E2EEngine();
    e->cfg = c;
    e->is_gdn.assign(c.is_gdn, c.is_gdn + c.layers);
    e->cfg.is_gdn = nullptr;
    cudaGetDevice(&e->device);
    const size_t B = c.batch, H = c.hidden, KD = c.key_dim, VD = c.value_dim, CD = c.conv_dim, I = c.inter;
    const size_t qd = c.full_heads * c.full_head_dim, kvd = c.full_kv_heads * c.full_head_dim;
    int rc = 0;
    if (!rc) rc = make_qw(e, &e->gqkv, {{w->g_q_proj, KD}, {w->g_k_proj, KD}, {w->g_v_proj, VD}}, H);
    if (!rc) rc = make_qw(e, &e->go, {{w->g_o_proj, H}}, VD);
    if (!rc) rc = make_qw(e, &e->fqkv, {{w->f_q_proj, qd}, {w->f_k_proj, kvd}, {w->f_v_proj, kvd}}, H);
    if (!rc) rc = make_qw(e, &e->fo, {{w->f_o_proj, H}}, qd);
    if (!rc) rc = make_qw(e, &e->gu, {{w->gate_proj, I}, {w->up_proj, I}}, H);
    if (!rc) rc = make_qw(e, &e->down, {{w->down_proj, H}}, I);
    if (!rc && (!w->g_conv_w || !w->g_beta)) rc = set_error(KAI_GDN_ERR_INVALID, "e2e_create: null weight");
    if (!rc) rc = dalloc(e, (void **)&e->conv_w, 4 * CD * sizeof(float), false);
    if (!rc)
        rc = check_cuda(cudaMemcpy(e->conv_w, w->g_conv_w, 4 * CD * sizeof(float), cudaMemcpyHostToDevice),
                        "e2e: conv weights");
    if (!rc) {  // the per-channel gate = the one-token decay, per sequence (repeated past key_dim)
        std::vector<float> bb(B * VD);
        for (size_t b = 0; b < B; ++b)
            for (size_t ch = 0; ch < VD; ++ch) bb[b * VD + ch] = w->g_beta[ch % KD];
        rc = dalloc(e, (void **)&e->beta_b, bb.size() * sizeof(float), false);
        if (!rc)
            rc = check_cuda(cudaMemcpy(e->beta_b, bb.data(), bb.size() * sizeof(float), cudaMemcpyHostToDevice),
                            "e2e: gates");
    }
    for (size_t l = 0; l < c.layers && !rc; ++l) {
        float *p = nullptr;
        if (e->is_gdn[l]) {
            if (!(rc = dalloc(e, (void **)&p, B * VD * sizeof(float), true))) e->gdn_state.push_back(p);
            if (!rc && !(rc = dalloc(e, (void **)&p, B * 3 * CD * sizeof(float), true))) e->conv_hist.push_back(p);
            e->kv_k.push_back(nullptr);
            e->kv_v.push_back(nullptr);
        } else {
            e->gdn_state.push_back(nullptr);
            e->conv_hist.push_back(nullptr);
            if (!(rc = dalloc(e, (void **)&p, B * kvd * sizeof(float), true))) e->kv_k.push_back(p);
            if (!rc && !(rc = dalloc(e, (void **)&p, B * kvd * sizeof(float), true))) e->kv_v.push_back(p);
        }
    }
    struct Buf {
        float **p;
        size_t n;
    } bufs[] = {{&e->h, B * H},          {&e->h2, B * H},          {&e->qkv, B * (2 * KD + VD)},
                {&e->v, B * VD},          {&e->conv_in, B * CD},    {&e->conv_out, B * CD},
                {&e->scanned, B * VD},    {&e->proj, B * H},        {&e->aqkv, B * (qd + 2 * kvd)},
                {&e->aq, B * qd},         {&e->gu_out, B * 2 * I},  {&e->act, B * I}};
    for (auto &bf : bufs)
        if (!rc) rc = dalloc(e, (void **)bf.p, bf.n * sizeof(float), true);
    if (rc) {
        e2e_destroy(e);
        return rc;
    }
    *out = e;
    return KAI_GDN_OK;
}

int e2e_step(void *engine, const float *hidden_in, float *hidden_out, cudaStream_t st) {
    E2EEngine *e = static_cast<E2EEngine *>(engine);
    if (!e || !hidden_in || !hidden_out) return set_error(KAI_GDN_ERR_INVALID, "e2e_step: null argument");
    const size_t bytes = e->cfg.batch * e->cfg.hidden * sizeof(float);
    int rc = check_cuda(cudaMemcpyAsync(e->h, hidden_in, bytes, cudaMemcpyDefault, st), "e2e_step: input");
    if (rc) return rc;
    // A step on a new stream runs eagerly (it creates the library's
    // workspaces for that stream); the next one on the same stream is
    // captured into a graph, later ones replay it.
    const bool capturable = st != nullptr && st != cudaStreamLegacy && st != cudaStreamPerThread;
    if (e->exec && e->graph_stream == st) {
        rc = check_cuda(cudaGraphLaunch(e->exec, st), "e2e_step: graph launch");
    } else if (capturable && e->steps >= 1 && e->last_stream == st) {
        if (e->exec) {
            cudaGraphExecDestroy(e->exec);
            e->exec = nullptr;
        }
        cudaGraph_t g = nullptr;
        rc = check_cuda(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), "e2e_step: capture");
        if (rc) return rc;
        int rc2 = run_token(e, st);
        rc = check_cuda(cudaStreamEndCapture(st, &g), "e2e_step: capture");
        if (rc2) {
            if (g) cudaGraphDestroy(g);
            return rc2;
        }
        if (rc) return rc;
        rc = check_cuda(cudaGraphInstantiate(&e->exec, g, 0), "e2e_step: instantiate");
        cudaGraphDestroy(g);
        if (rc) return rc;
        e->graph_stream = st;
        rc = check_cuda(cudaGraphLaunch(e->exec, st), "e2e_step: graph launch");
    } else {
        rc = run_token(e, st);
    }
    if (rc) return rc;
    ++e->steps;
    e->last_stream = st;
    return check_cuda(cudaMemcpyAsync(hidden_out, e->h, bytes, cudaMemcpyDefault, st), "e2e_step: output");
}

int e2e_state(void *engine, size_t layer, float *gdn_state, float *conv_hist) {
    E2EEngine *e = static_cast<E2EEngine *>(engine);
    if (!e || layer >= e->cfg.layers) return set_error(KAI_GDN_ERR_INVALID, "e2e_state: bad engine or layer");
    if (!e->is_gdn[layer]) return set_error(KAI_GDN_ERR_INVALID, "e2e_state: layer %zu is not a GDN layer", layer);
    const size_t B = e->cfg.batch;
    int rc = check_cuda(cudaDeviceSynchronize(), "e2e_state: sync");
    if (!rc && gdn_state)
        rc = check_cuda(cudaMemcpy(gdn_state, e->gdn_state[layer], B * e->cfg.value_dim * sizeof(float),
                                   cudaMemcpyDefault),
                        "e2e_state: copy");
    if (!rc && conv_hist)
        rc = check_cuda(cudaMemcpy(conv_hist, e->conv_hist[layer], B * 3 * e->cfg.conv_dim * sizeof(float),
                                   cudaMemcpyDefault),
                        "e2e_state: copy");
    return rc;
}

int e2e_destroy(void *engine) {
    E2EEngine *e = static_cast<E2EEngine *>(engine);
    if (!e) return KAI_GDN_OK;
    cudaDeviceSynchronize();
    if (e->exec) cudaGraphExecDestroy(e->exec);
    for (void *p : e->allocs) cudaFree(p);
    delete e;
    return KAI_GDN_OK;
}

}  // namespace gdn
