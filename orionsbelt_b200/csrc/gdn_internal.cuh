// gdn_internal.cuh -- shared declarations of libkai_gdn_cuda.so (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/kai_gdn_cuda.h"

namespace gdn {

// ------------------------------------------------------------- errors
// Thread-local status + message (runtime.cu).  set_error returns `status`
// so call sites can `return set_error(...)`.
int set_error(int status, const char *fmt, ...);
int check_cuda(cudaError_t err, const char *what);
// Check the launch that was just issued.
int check_launch(const char *kernel);

// Device word where kernels with bounded waits record a timeout (no allocation).
int device_error_word(int **out);
// Synchronise `st`, read and clear the word: KAI_GDN_ERR_TIMEOUT if it was set.
int check_device_word(cudaStream_t st);

// Number of SMs of the current device (cached per device).
int sm_count();

// Scratch memory owned by the library for kernels that need it (the segment
// aggregates of the scan kernels).  One buffer per (device, stream), grown on
// demand with cudaMalloc (which synchronises the device), never shrunk.  The
// returned pointer is valid until the next call for the same stream.
int scratch_for_stream(cudaStream_t stream, size_t bytes, void **out);

// Launchers shared between the drop-in and the device entry points.  All take
// device pointers and return a KAI_GDN_* status.
int launch_cumdecay(const float *a, void *decay, int decay_dtype, size_t batch,
                    size_t seq, size_t ch, cudaStream_t st);
int launch_cumsum(const float *g, float *gcum, size_t batch, size_t seq, size_t ch,
                  cudaStream_t st);
int launch_gated_scan(const float *g, const float *x, float *s, void *state,
                      int state_dtype, size_t batch, size_t seq, size_t ch,
                      cudaStream_t st);
int launch_gated_scan_noalloc(const float *g, const float *x, float *s, void *state,
                              int state_dtype, size_t batch, size_t seq, size_t ch,
                              cudaStream_t st);
int launch_gdn2_scan(const float *g, const float *bg, const float *wg, const float *x,
                     float *s, float *state, size_t batch, size_t seq, size_t ch,
                     cudaStream_t st);
int launch_conv(const void *in, const float *w, void *out, void *hist, int io_dtype,
                size_t batch, size_t seq, size_t ch, cudaStream_t st);
int launch_matmul(const float *A, const float *B, float *C, size_t M, size_t K,
                  size_t N, cudaStream_t st);
int launch_decode(const kai_gdn_decode_args *a, cudaStream_t st);
int launch_gdn2_decode(const kai_gdn2_decode_args *a, cudaStream_t st);
int launch_attn_decode(const kai_gdn_attn_decode_args *a, cudaStream_t st);
int launch_attn_prefill(const kai_gdn_attn_prefill_args *a, cudaStream_t st);
int e2e_create(const kai_gdn_e2e_config *cfg, const kai_gdn_e2e_weights *w, void **out);
int e2e_step(void *engine, const float *hidden_in, float *hidden_out, cudaStream_t st);
int e2e_state(void *engine, size_t layer, float *gdn_state, float *conv_hist);
int e2e_destroy(void *engine);
int model_nccl_id(void *out);
int model_create(const kai_gdn_model_config *cfg, void **out);
int model_step(void *engine, size_t pos, cudaStream_t st);
int model_prefill(void *engine, const int *tokens, size_t T, size_t pos0, cudaStream_t st);
int model_tokens(void *engine, int *tokens, int set);
int model_read(void *engine, int what, float *out);
int model_weight(void *engine, size_t layer, int which, void *data, float *scales, size_t *rows, size_t *cols);
int model_fill(void *engine, size_t ctx, unsigned long long seed);
int model_reset(void *engine);
int model_destroy(void *engine);
int launch_quantize_int8(const float *B, int8_t *q, float *s, size_t K, size_t N, cudaStream_t st);
int launch_matmul_int8(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N,
                       cudaStream_t st);
// Weight-streaming GEMV for M <= 8 (gemv.cu), launched as a programmatic
// dependent of the previous kernel on the stream.
bool gemv_int8_supported(size_t M, size_t K, size_t N, const int8_t *q);
int launch_gemv_int8(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N,
                     cudaStream_t st);
// The same over weights in the blocked layout for M rows (made by
// gemv_block_weights from [K][N]; gemv_blocked_bytes bytes).
size_t gemv_blocked_bytes(size_t M, size_t K, size_t N);
int gemv_block_weights(size_t M, const int8_t *q, int8_t *qb, size_t K, size_t N, cudaStream_t st);
// swiglu: A is [M][2K], rows [gate | up], and the GEMV's activations are
// SiLU(gate) * up (the FFN down projection takes its input straight from the
// gate+up output, one launch fewer).
int launch_gemv_int8_blocked(const float *A, const int8_t *qb, const float *s, float *C, size_t M, size_t K,
                             size_t N, cudaStream_t st, bool swiglu = false);
int launch_matmul_int8_tc(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N,
                          cudaStream_t st);
// Weight-streaming tensor-core matmul over weights packed once into its
// streaming layout (int8_packed.cu): 16 activation rows per launch, launched
// as a programmatic dependent of the previous kernel on the stream.
bool int8_packed_supported(size_t K, size_t N);
size_t int8_packed_bytes(size_t K, size_t N);
int int8_pack_weights(const int8_t *q, int8_t *qp, size_t K, size_t N, cudaStream_t st);
int launch_matmul_int8_packed(const float *A, const int8_t *qp, const float *s, float *C, size_t M, size_t K,
                              size_t N, cudaStream_t st);
// The same over activation terms a producer kernel already wrote
// (int8_terms.cuh, 16-row blocks: int8_terms_bytes(M, K) bytes; scales [M]).
size_t int8_terms_bytes(size_t M, size_t K);
int launch_matmul_int8_packed_terms(const int8_t *terms, const float *scale, const int8_t *qp, const float *s,
                                    float *C, size_t M, size_t K, size_t N, cudaStream_t st);
// Per-stream split-K workspace of the int8 matmuls: slab counters (zero
// between calls: each kernel's last CTA resets its counter) and partial sums.
int split_workspace(cudaStream_t st, size_t nctr, size_t npart, unsigned int **ctr, float **part);
int launch_chunk(const kai_gdn_chunk_args *a, cudaStream_t st);
// Warp-specialised tensor-core chunk scan (chunk_ws.cu): bf16/fp16 q, k, v,
// dk = dv = 128, chunk 64; TMA-fed, tcgen05 MMAs, fp32 state in TMEM.
bool chunk_ws_supported(const kai_gdn_chunk_args *a);
int launch_chunk_ws(const kai_gdn_chunk_args *a, cudaStream_t st);
// Tensor-core chunk scan for fp32 inputs (chunk_tc32.cu): dk = 128, dv a
// multiple of 32, 16-byte aligned q, k, v, o; fp32-accurate (three bf16 MMAs
// per product); a parallel per-chunk launch, then the recurrence.
bool chunk_tc32_supported(const kai_gdn_chunk_args *a);
int launch_chunk_tc32(const kai_gdn_chunk_args *a, cudaStream_t st);

// --------------------------------------------------- storage conversions
// Loads widen to fp32 exactly; stores round to nearest even.
template <int DT> struct Store;
template <> struct Store<KAI_GDN_F32> {
    using T = float;
    static __device__ __forceinline__ float load(const T *p) { return *p; }
    static __device__ __forceinline__ void store(T *p, float v) { *p = v; }
};
template <> struct Store<KAI_GDN_BF16> {
    using T = __nv_bfloat16;
    static __device__ __forceinline__ float load(const T *p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void store(T *p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct Store<KAI_GDN_F16> {
    using T = __half;
    static __device__ __forceinline__ float load(const T *p) { return __half2float(*p); }
    static __device__ __forceinline__ void store(T *p, float v) { *p = __float2half_rn(v); }
};

// sum_{r < n} p[r * stride], added in r order (the same rounding as a plain
// loop), with sixteen loads in flight at a time.  For the K-split fix-ups:
// a dependent L2 load per part cost ~100 ns each, microseconds per launch.
__device__ __forceinline__ float sum_parts_ordered(const float *p, long long stride, int n) {
    float v = 0.f;
    int r = 0;
    for (; r + 16 <= n; r += 16) {
        float x[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = __ldcg(p + (long long)(r + j) * stride);
#pragma unroll
        for (int j = 0; j < 16; ++j) v += x[j];
    }
    float x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = r + j < n ? __ldcg(p + (long long)(r + j) * stride) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (r + j < n) v += x[j];
    return v;
}

static inline bool valid_dtype(int dt) {
    return dt == KAI_GDN_F32 || dt == KAI_GDN_BF16 || dt == KAI_GDN_F16;
}
static inline size_t dtype_size(int dt) { return dt == KAI_GDN_F32 ? 4 : 2; }

}  // namespace gdn
