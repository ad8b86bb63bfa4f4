// runtime.cu -- host side of libkai_gdn_cuda.so: the extern "C" entry points,
// argument checks, thread-local error state, library-owned scratch, and the
// staging that lets the drop-in symbols take host pointers like the reference.
//
// Drop-in semantics (kleidiai_submission/kai/ukernels/gdn/*.h, gdn_sve.h,
// gdn_delta_matmul.h): caller-owned buffers, synchronous, void return,
// zero-size calls are no-ops that touch nothing.  Each pointer is classified
// with cudaPointerGetAttributes: device or managed memory is used in place;
// host memory (pageable or pinned) is copied into a per-thread device staging
// buffer, the kernel runs, and outputs are copied back before returning.  The
// work is ordered on the legacy default stream, so it also waits for work the
// caller queued on blocking streams.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "gdn_internal.cuh"

namespace gdn {

// ------------------------------------------------------------------ errors
namespace {
thread_local int t_status = KAI_GDN_OK;
thread_local char t_msg[512] = "";
}  // namespace

int set_error(int status, const char *fmt, ...) {
    t_status = status;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return status;
}

int check_cuda(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return KAI_GDN_OK;
    int st = err == cudaErrorMemoryAllocation ? KAI_GDN_ERR_NOMEM : KAI_GDN_ERR_CUDA;
    return set_error(st, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}

int check_launch(const char *kernel) { return check_cuda(cudaGetLastError(), kernel); }

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// -------------------------------------------------------- device error word
// Kernels with bounded waits (the tensor-core chunk scan, the long scans'
// look-back) record a timeout here instead of hanging.  A file-scope device word,
// so launching needs no allocation (and can be captured in a CUDA graph); its
// address is looked up once per device.
namespace {
__device__ int g_wait_timeout;
std::mutex g_errword_mu;
int *g_errword[64] = {nullptr};
}  // namespace

int device_error_word(int **out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "error word: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return set_error(KAI_GDN_ERR_UNSUPPORTED, "error word: device %d", dev);
    std::lock_guard<std::mutex> lock(g_errword_mu);
    if (!g_errword[dev]) {
        void *p = nullptr;
        rc = check_cuda(cudaGetSymbolAddress(&p, g_wait_timeout), "error word: cudaGetSymbolAddress");
        if (rc) return rc;
        g_errword[dev] = static_cast<int *>(p);
    }
    *out = g_errword[dev];
    return KAI_GDN_OK;
}

// Synchronise `st`, read and clear the word; KAI_GDN_ERR_TIMEOUT if it was set.
int check_device_word(cudaStream_t st) {
    int *w = nullptr;
    int rc = device_error_word(&w);
    if (rc) return rc;
    if ((rc = check_cuda(cudaStreamSynchronize(st), "device status: synchronize"))) return rc;
    int v = 0;
    if ((rc = check_cuda(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost), "device status: read"))) return rc;
    if (!v) return KAI_GDN_OK;
    const int zero = 0;
    if ((rc = check_cuda(cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice), "device status: clear")))
        return rc;
    return set_error(KAI_GDN_ERR_TIMEOUT, "a bounded wait inside a kernel ran out; its outputs are not valid");
}

// ----------------------------------------------------------------- scratch
namespace {
struct ScratchEntry {
    int device;
    cudaStream_t stream;
    void *ptr;
    size_t cap;
};
std::mutex g_scratch_mu;
std::vector<ScratchEntry> g_scratch;
}  // namespace

int scratch_for_stream(cudaStream_t stream, size_t bytes, void **out) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "scratch: cudaGetDevice");
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    for (auto &e : g_scratch) {
        if (e.device == dev && e.stream == stream) {
            if (e.cap < bytes) {
                // cudaFree waits for the device, so kernels still reading the
                // old buffer have finished before it goes.
                if ((rc = check_cuda(cudaFree(e.ptr), "scratch: cudaFree"))) return rc;
                e.ptr = nullptr;
                e.cap = 0;
                size_t cap = bytes + bytes / 2;
                if ((rc = check_cuda(cudaMalloc(&e.ptr, cap), "scratch: cudaMalloc"))) return rc;
                e.cap = cap;
            }
            *out = e.ptr;
            return KAI_GDN_OK;
        }
    }
    ScratchEntry e{dev, stream, nullptr, 0};
    size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
    if ((rc = check_cuda(cudaMalloc(&e.ptr, cap), "scratch: cudaMalloc"))) return rc;
    e.cap = cap;
    g_scratch.push_back(e);
    *out = e.ptr;
    return KAI_GDN_OK;
}

// ----------------------------------------------------------------- staging
namespace {

enum Dir { IN = 1, OUT = 2, INOUT = 3 };

struct Arg {
    const void *host;  // caller's pointer
    size_t bytes;
    int dir;
    void *dev;         // pointer handed to the kernel
    bool staged;
};

struct Stage {
    void *buf = nullptr;
    size_t cap = 0;
};
thread_local Stage t_stage[64];

bool is_device_pointer(const void *p) {
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();  // clear: an unknown pointer is host memory
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

// Resolve every argument to a device pointer, copying host inputs in.
int stage_in(Arg *args, int n, cudaStream_t st) {
    int dev = 0;
    int rc = check_cuda(cudaGetDevice(&dev), "stage: cudaGetDevice");
    if (rc) return rc;
    if (dev < 0 || dev >= 64) return set_error(KAI_GDN_ERR_UNSUPPORTED, "stage: device %d", dev);
    size_t need = 0;
    for (int i = 0; i < n; ++i) {
        args[i].staged = args[i].bytes > 0 && !is_device_pointer(args[i].host);
        if (args[i].staged) need += (args[i].bytes + 255) & ~size_t(255);
    }
    Stage &s = t_stage[dev];
    if (need > s.cap) {
        if (s.buf && (rc = check_cuda(cudaFree(s.buf), "stage: cudaFree"))) return rc;
        s.buf = nullptr;
        s.cap = 0;
        if ((rc = check_cuda(cudaMalloc(&s.buf, need), "stage: cudaMalloc"))) return rc;
        s.cap = need;
    }
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        if (!args[i].staged) {
            args[i].dev = const_cast<void *>(args[i].host);
            continue;
        }
        args[i].dev = static_cast<char *>(s.buf) + off;
        off += (args[i].bytes + 255) & ~size_t(255);
        if (args[i].dir & IN) {
            rc = check_cuda(cudaMemcpyAsync(args[i].dev, args[i].host, args[i].bytes,
                                            cudaMemcpyHostToDevice, st),
                            "stage: copy in");
            if (rc) return rc;
        }
    }
    return KAI_GDN_OK;
}

// Copy staged outputs back and wait for everything.
int stage_out(Arg *args, int n, cudaStream_t st) {
    for (int i = 0; i < n; ++i) {
        if (args[i].staged && (args[i].dir & OUT)) {
            int rc = check_cuda(cudaMemcpyAsync(const_cast<void *>(args[i].host), args[i].dev,
                                                args[i].bytes, cudaMemcpyDeviceToHost, st),
                                "stage: copy out");
            if (rc) return rc;
        }
    }
    int rc = check_cuda(cudaStreamSynchronize(st), "stage: synchronize");
    return rc ? rc : check_device_word(st);
}

constexpr cudaStream_t kLegacy = 0;

}  // namespace
}  // namespace gdn

using namespace gdn;

// ======================================================================
// 1. Drop-in symbols
// ======================================================================
extern "C" {

void kai_run_gdn_cumdecay_f32_sve(const float *a, float *decay, size_t seq, size_t channels) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels * sizeof(float);
    Arg args[2] = {{a, n, IN}, {decay, n, OUT}};
    if (stage_in(args, 2, kLegacy)) return;
    if (launch_cumdecay((const float *)args[0].dev, args[1].dev, KAI_GDN_F32, 1, seq, channels, kLegacy)) return;
    stage_out(args, 2, kLegacy);
}

void kai_run_gdn_gated_scan_f32_sve(const float *g, const float *x, float *s, float *state,
                                    size_t seq, size_t channels) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels * sizeof(float);
    Arg args[4] = {{g, n, IN}, {x, n, IN}, {s, n, OUT}, {state, channels * sizeof(float), INOUT}};
    if (stage_in(args, 4, kLegacy)) return;
    if (launch_gated_scan((const float *)args[0].dev, (const float *)args[1].dev, (float *)args[2].dev,
                          args[3].dev, KAI_GDN_F32, 1, seq, channels, kLegacy))
        return;
    stage_out(args, 4, kLegacy);
}

void kai_run_gdn_causal_dwconv1d_f32_k4_sve(const float *in, const float *w, float *out,
                                            float *hist, size_t seq, size_t channels) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels * sizeof(float);
    Arg args[4] = {{in, n, IN},
                   {w, 4 * channels * sizeof(float), IN},
                   {out, n, OUT},
                   {hist, 3 * channels * sizeof(float), INOUT}};
    if (stage_in(args, 4, kLegacy)) return;
    if (launch_conv(args[0].dev, (const float *)args[1].dev, args[2].dev, args[3].dev, KAI_GDN_F32, 1, seq,
                    channels, kLegacy))
        return;
    stage_out(args, 4, kLegacy);
}

void gdn_delta_rule_matmul(const float *A, const float *B, float *C, size_t M, size_t K, size_t N) {
    if (M == 0 || N == 0) return;
    Arg args[3] = {{A, M * K * sizeof(float), IN}, {B, K * N * sizeof(float), IN}, {C, M * N * sizeof(float), OUT}};
    if (stage_in(args, 3, kLegacy)) return;
    if (launch_matmul((const float *)args[0].dev, (const float *)args[1].dev, (float *)args[2].dev, M, K, N,
                      kLegacy))
        return;
    stage_out(args, 3, kLegacy);
}

void kai_run_gdn_gemv_f32_f32_f32_1x4_neon(const float *a, const float *b, float *c, size_t k, size_t n) {
    gdn_delta_rule_matmul(a, b, c, 1, k, n);
}

void gdn_cumdecay_f32(const float *a, float *decay, size_t seq, size_t channels) {
    kai_run_gdn_cumdecay_f32_sve(a, decay, seq, channels);
}

void gdn_gated_scan_f32(const float *g, const float *x, float *s, float *state, size_t seq, size_t channels) {
    kai_run_gdn_gated_scan_f32_sve(g, x, s, state, seq, channels);
}

void gdn_causal_dwconv1d_f32(const float *in, const float *w, float *out, float *hist, size_t seq,
                             size_t channels) {
    kai_run_gdn_causal_dwconv1d_f32_k4_sve(in, w, out, hist, seq, channels);
}

static void cumdecay_narrow(const float *a, uint16_t *decay, size_t seq, size_t channels, int dt) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels;
    Arg args[2] = {{a, n * sizeof(float), IN}, {decay, n * sizeof(uint16_t), OUT}};
    if (stage_in(args, 2, kLegacy)) return;
    if (launch_cumdecay((const float *)args[0].dev, args[1].dev, dt, 1, seq, channels, kLegacy)) return;
    stage_out(args, 2, kLegacy);
}

void gdn_cumdecay_f16(const float *a, uint16_t *decay, size_t seq, size_t channels) {
    cumdecay_narrow(a, decay, seq, channels, KAI_GDN_F16);
}
void gdn_cumdecay_bf16(const float *a, uint16_t *decay, size_t seq, size_t channels) {
    cumdecay_narrow(a, decay, seq, channels, KAI_GDN_BF16);
}

static void scan_narrow(const float *g, const float *x, float *s, uint16_t *state, size_t seq,
                        size_t channels, int dt) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels * sizeof(float);
    Arg args[4] = {{g, n, IN}, {x, n, IN}, {s, n, OUT}, {state, channels * sizeof(uint16_t), INOUT}};
    if (stage_in(args, 4, kLegacy)) return;
    if (launch_gated_scan((const float *)args[0].dev, (const float *)args[1].dev, (float *)args[2].dev,
                          args[3].dev, dt, 1, seq, channels, kLegacy))
        return;
    stage_out(args, 4, kLegacy);
}

void gdn_gated_scan_f16(const float *g, const float *x, float *s, uint16_t *state, size_t seq,
                        size_t channels) {
    scan_narrow(g, x, s, state, seq, channels, KAI_GDN_F16);
}
void gdn_gated_scan_bf16(const float *g, const float *x, float *s, uint16_t *state, size_t seq,
                         size_t channels) {
    scan_narrow(g, x, s, state, seq, channels, KAI_GDN_BF16);
}

void gdn2_gated_scan_f32(const float *g, const float *b_gate, const float *w_gate, const float *x, float *s,
                         float *state, size_t seq, size_t channels) {
    if (seq == 0 || channels == 0) return;
    size_t n = seq * channels * sizeof(float);
    Arg args[6] = {{g, n, IN},  {b_gate, n, IN}, {w_gate, n, IN},
                   {x, n, IN},  {s, n, OUT},     {state, channels * sizeof(float), INOUT}};
    if (stage_in(args, 6, kLegacy)) return;
    if (launch_gdn2_scan((const float *)args[0].dev, (const float *)args[1].dev, (const float *)args[2].dev,
                         (const float *)args[3].dev, (float *)args[4].dev, (float *)args[5].dev, 1, seq,
                         channels, kLegacy))
        return;
    stage_out(args, 6, kLegacy);
}

// ======================================================================
// 2. Stream-ordered device entry points
// ======================================================================
int kai_run_gdn_cumdecay_sm100a(const float *a, void *decay, int decay_dtype, size_t batch, size_t seq,
                                size_t channels, void *stream) {
    return launch_cumdecay(a, decay, decay_dtype, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn_cumsum_f32_sm100a(const float *g, float *gcum, size_t batch, size_t seq, size_t channels,
                                  void *stream) {
    return launch_cumsum(g, gcum, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn_gated_scan_sm100a(const float *g, const float *x, float *s, void *state, int state_dtype,
                                  size_t batch, size_t seq, size_t channels, void *stream) {
    return launch_gated_scan(g, x, s, state, state_dtype, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn_gated_scan_noalloc_sm100a(const float *g, const float *x, float *s, void *state,
                                          int state_dtype, size_t batch, size_t seq, size_t channels,
                                          void *stream) {
    return launch_gated_scan_noalloc(g, x, s, state, state_dtype, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn2_gated_scan_f32_sm100a(const float *g, const float *b_gate, const float *w_gate, const float *x,
                                       float *s, float *state, size_t batch, size_t seq, size_t channels,
                                       void *stream) {
    return launch_gdn2_scan(g, b_gate, w_gate, x, s, state, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn_causal_dwconv1d_k4_sm100a(const void *in, const float *w, void *out, void *hist, int io_dtype,
                                          size_t batch, size_t seq, size_t channels, void *stream) {
    return launch_conv(in, w, out, hist, io_dtype, batch, seq, channels, (cudaStream_t)stream);
}

int kai_run_gdn_matmul_f32_sm100a(const float *A, const float *B, float *C, size_t M, size_t K, size_t N,
                                  void *stream) {
    return launch_matmul(A, B, C, M, K, N, (cudaStream_t)stream);
}

int kai_run_gdn_delta_rule_decode_sm100a(const kai_gdn_decode_args *args, void *stream) {
    return launch_decode(args, (cudaStream_t)stream);
}

int kai_run_gdn2_delta_rule_decode_sm100a(const kai_gdn2_decode_args *args, void *stream) {
    return launch_gdn2_decode(args, (cudaStream_t)stream);
}

int kai_run_gdn_attention_decode_sm100a(const kai_gdn_attn_decode_args *args, void *stream) {
    return launch_attn_decode(args, (cudaStream_t)stream);
}

int kai_run_gdn_attention_prefill_sm100a(const kai_gdn_attn_prefill_args *args, void *stream) {
    return launch_attn_prefill(args, (cudaStream_t)stream);
}

int kai_gdn_e2e_create(const kai_gdn_e2e_config *cfg, const kai_gdn_e2e_weights *weights, void **engine) {
    return e2e_create(cfg, weights, engine);
}

int kai_gdn_e2e_step(void *engine, const float *hidden_in, float *hidden_out, void *stream) {
    return e2e_step(engine, hidden_in, hidden_out, (cudaStream_t)stream);
}

int kai_gdn_e2e_state(void *engine, size_t layer, float *gdn_state, float *conv_hist) {
    return e2e_state(engine, layer, gdn_state, conv_hist);
}

int kai_gdn_e2e_destroy(void *engine) { return e2e_destroy(engine); }

int kai_gdn_model_nccl_id(void *id_out) { return model_nccl_id(id_out); }
int kai_gdn_model_create(const kai_gdn_model_config *cfg, void **engine) { return model_create(cfg, engine); }
int kai_gdn_model_step(void *engine, size_t pos, void *stream) {
    return model_step(engine, pos, (cudaStream_t)stream);
}

int kai_gdn_model_prefill(void *engine, const int32_t *tokens, size_t T, size_t pos0, void *stream) {
    return model_prefill(engine, tokens, T, pos0, (cudaStream_t)stream);
}
int kai_gdn_model_tokens(void *engine, int32_t *tokens, int set) { return model_tokens(engine, tokens, set); }
int kai_gdn_model_read(void *engine, int what, float *out) { return model_read(engine, what, out); }
int kai_gdn_model_weight(void *engine, size_t layer, int which, void *data, float *scales, size_t *rows,
                         size_t *cols) {
    return model_weight(engine, layer, which, data, scales, rows, cols);
}
int kai_gdn_model_fill(void *engine, size_t ctx, unsigned long long seed) { return model_fill(engine, ctx, seed); }

int kai_gdn_model_reset(void *engine) { return model_reset(engine); }
int kai_gdn_model_destroy(void *engine) { return model_destroy(engine); }

int kai_run_gdn_quantize_int8_sm100a(const float *B, int8_t *q, float *s, size_t K, size_t N, void *stream) {
    return launch_quantize_int8(B, q, s, K, N, (cudaStream_t)stream);
}

int kai_run_gdn_matmul_int8_sm100a(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K,
                                   size_t N, void *stream) {
    return launch_matmul_int8(A, q, s, C, M, K, N, (cudaStream_t)stream);
}

size_t kai_gdn_int8_packed_bytes(size_t K, size_t N) { return int8_packed_supported(K, N) ? int8_packed_bytes(K, N) : 0; }

int kai_run_gdn_int8_pack_sm100a(const int8_t *q, int8_t *qp, size_t K, size_t N, void *stream) {
    return int8_pack_weights(q, qp, K, N, (cudaStream_t)stream);
}

int kai_run_gdn_matmul_int8_packed_sm100a(const float *A, const int8_t *qp, const float *s, float *C, size_t M,
                                          size_t K, size_t N, void *stream) {
    return launch_matmul_int8_packed(A, qp, s, C, M, K, N, (cudaStream_t)stream);
}

int kai_run_gdn_chunk_delta_rule_sm100a(const kai_gdn_chunk_args *args, void *stream) {
    return launch_chunk(args, (cudaStream_t)stream);
}

// ======================================================================
// 3. Library control
// ======================================================================
int kai_gdn_cuda_set_device(int device) { return check_cuda(cudaSetDevice(device), "cudaSetDevice"); }

int kai_gdn_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    return n;
}

int kai_gdn_cuda_last_status(void) { return t_status; }
const char *kai_gdn_cuda_last_error(void) { return t_msg; }
void kai_gdn_cuda_clear_error(void) {
    t_status = KAI_GDN_OK;
    t_msg[0] = '\0';
}
const char *kai_gdn_cuda_version(void) { return "kai_gdn_cuda 0.1.0 (sm_100a)"; }
int kai_gdn_cuda_device_status(void *stream) { return gdn::check_device_word((cudaStream_t)stream); }

}  // extern "C"
