/*
 * kai_gdn_cuda.h -- C ABI of libkai_gdn_cuda.so, the B200 (sm_100a) Gated
 * DeltaNet hot path that drops in for OrionsBelt's kai GDN operators.
 *
 * Three groups of entry points:
 *
 *  1. Drop-in symbols, with the exact names, signatures and semantics of the
 *     reference's C kernels (caller-owned buffers, [seq][channels] row-major,
 *     `state` / `hist` updated in place, seq == 0 or channels == 0 is a no-op,
 *     the call returns when the result is in place).  They accept host
 *     pointers (staged through device memory) or device / managed pointers
 *     (used in place).  They return void like the originals; a failure is
 *     recorded for kai_gdn_cuda_last_error() and never aborts the process.
 *
 *  2. Stream-ordered device entry points (suffix _sm100a): device pointers
 *     only, launched on `stream` (a cudaStream_t; NULL = the legacy default
 *     stream), asynchronous, returning a KAI_GDN_* status.  They add a batch
 *     dimension, narrow storage types, and the two matrix-state operators the
 *     reference has only in OpenCL / third-party form: the single-token
 *     delta-rule decode step and the chunkwise WY gated delta-rule scan.
 *
 *  3. Library control: device selection, errors, version.
 *
 * Thread safety: every entry point may be called from several host threads;
 * each thread gets its own staging stream and buffers per device.  Calls that
 * share output buffers must be ordered by the caller, as with the reference.
 */
#ifndef KAI_GDN_CUDA_H
#define KAI_GDN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KAI_GDN_API __attribute__((visibility("default")))
#else
#define KAI_GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define KAI_GDN_OK 0
#define KAI_GDN_ERR_INVALID 1     /* bad argument (null pointer, size, shape) */
#define KAI_GDN_ERR_CUDA 2        /* a CUDA runtime call or a launch failed   */
#define KAI_GDN_ERR_UNSUPPORTED 3 /* valid but not implemented (e.g. dk>256)  */
#define KAI_GDN_ERR_NOMEM 4       /* device or pinned allocation failed       */
#define KAI_GDN_ERR_TIMEOUT 5     /* a kernel's bounded wait ran out (see     */
                                  /* kai_gdn_cuda_device_status)              */

/* --------------------------------------------------------- storage types */
#define KAI_GDN_F32 0
#define KAI_GDN_BF16 1 /* bfloat16, round-to-nearest-even on store */
#define KAI_GDN_F16 2  /* IEEE binary16, round-to-nearest-even on store */
#define KAI_GDN_I8 3   /* int8 with one fp32 scale per kv head (attention KV cache only) */

/* ======================================================================
 * 1. Drop-in replacements (host or device pointers, synchronous)
 * ==================================================================== */

/* decay[t][c] = prod_{i<=t} a[i][c].
 * Replaces kleidiai_submission/kai/ukernels/gdn/kai_gdn_cumdecay_f32_sve.h:33 */
KAI_GDN_API void kai_run_gdn_cumdecay_f32_sve(const float *a, float *decay, size_t seq,
                                  size_t channels);

/* s[t][c] = g[t][c] * s[t-1][c] + x[t][c]; state[] is s[-1] on entry and
 * s[seq-1] on exit.
 * Replaces kleidiai_submission/kai/ukernels/gdn/kai_gdn_gated_scan_f32_sve.h:35 */
KAI_GDN_API void kai_run_gdn_gated_scan_f32_sve(const float *g, const float *x, float *s,
                                    float *state, size_t seq, size_t channels);

/* out[t][c] = w[0][c]*in[t-3][c] + w[1][c]*in[t-2][c] + w[2][c]*in[t-1][c]
 *           + w[3][c]*in[t][c], with in[-3..-1] = hist[0..2] (oldest first);
 * hist[] holds the last three inputs on exit.
 * Replaces kleidiai_submission/kai/ukernels/gdn/kai_gdn_causal_dwconv1d_f32_k4_sve.h:39 */
KAI_GDN_API void kai_run_gdn_causal_dwconv1d_f32_k4_sve(const float *in, const float *w,
                                            float *out, float *hist, size_t seq,
                                            size_t channels);

/* c[j] = sum_k a[k] * b[k][j]  (k == 0 writes zeros; n == 0 is a no-op).
 * Replaces kleidiai_submission/kai/ukernels/gdn/kai_gdn_gemv_f32_f32_f32_1x4_neon.h:40 */
KAI_GDN_API void kai_run_gdn_gemv_f32_f32_f32_1x4_neon(const float *a, const float *b, float *c,
                                           size_t k, size_t n);

/* Project-form twins, src/orionsbelt/engines/cpu/kernels/gdn_sve.h:30-86.
 * `__fp16 *` there is ABI-identical to `uint16_t *` here (IEEE binary16 bits);
 * bf16 is the upper half of an fp32, rounded to nearest even. */
KAI_GDN_API void gdn_cumdecay_f32(const float *a, float *decay, size_t seq, size_t channels);
KAI_GDN_API void gdn_gated_scan_f32(const float *g, const float *x, float *s, float *state,
                        size_t seq, size_t channels);
KAI_GDN_API void gdn_causal_dwconv1d_f32(const float *in, const float *w, float *out, float *hist,
                             size_t seq, size_t channels);
KAI_GDN_API void gdn_cumdecay_f16(const float *a, uint16_t *decay, size_t seq, size_t channels);
KAI_GDN_API void gdn_gated_scan_f16(const float *g, const float *x, float *s, uint16_t *state,
                        size_t seq, size_t channels);
KAI_GDN_API void gdn_cumdecay_bf16(const float *a, uint16_t *decay, size_t seq, size_t channels);
KAI_GDN_API void gdn_gated_scan_bf16(const float *g, const float *x, float *s, uint16_t *state,
                         size_t seq, size_t channels);
/* GDN-2 channel scan s[t] = w[t]*x[t] + s[t-1]*(g[t]*b[t]).  gdn_sve.h:79 */
KAI_GDN_API void gdn2_gated_scan_f32(const float *g, const float *b_gate, const float *w_gate,
                         const float *x, float *s, float *state, size_t seq,
                         size_t channels);

/* C[M][N] = A[M][K] . B[K][N], row-major, no bias.
 * Replaces src/orionsbelt/engines/cpu/kernels/gdn_delta_matmul.h:15 */
KAI_GDN_API void gdn_delta_rule_matmul(const float *A, const float *B, float *C, size_t M,
                           size_t K, size_t N);

/* ======================================================================
 * 2. Stream-ordered device entry points (device pointers, asynchronous)
 *    Layouts are row-major; `batch` independent problems lie back to back.
 * ==================================================================== */

/* Prefix product over seq of a[batch][seq][channels]; decay is stored as
 * decay_dtype (F32, F16 or BF16) with an fp32 running product.
 * Batched form of kai_gdn_cumdecay_f32_sve.h:33 / gdn_sve.h:30,57,65. */
KAI_GDN_API int kai_run_gdn_cumdecay_sm100a(const float *a, void *decay, int decay_dtype,
                                size_t batch, size_t seq, size_t channels,
                                void *stream);

/* Log-space decay cumsum gcum[b][t][c] = sum_{i<=t} g[b][i][c] (the form the
 * chunkwise scan consumes; docs/GDN_ARCHITECTURE_AUDIT.md:142-153). */
KAI_GDN_API int kai_run_gdn_cumsum_f32_sm100a(const float *g, float *gcum, size_t batch,
                                  size_t seq, size_t channels, void *stream);

/* Gated scan over [batch][seq][channels]; state[batch][channels] stored as
 * state_dtype (F32, F16 or BF16), widened on entry and narrowed once on exit.
 * Batched form of kai_gdn_gated_scan_f32_sve.h:35 / gdn_sve.h:36,61,69. */
KAI_GDN_API int kai_run_gdn_gated_scan_sm100a(const float *g, const float *x, float *s,
                                  void *state, int state_dtype, size_t batch,
                                  size_t seq, size_t channels, void *stream);

/* The gated scan above with no allocation at call time.  This entry point
 * has no counterpart in the reference.  It is for callers that cannot
 * allocate device memory when they call (an engine that gives all of HBM to
 * its own pools at start-up, or a host whose other streams cannot wait for
 * the device-wide synchronisation cudaMalloc / cudaFree may cause).  A long
 * scan's tile records use a fixed array inside the library image instead
 * of library-allocated scratch: every GPU that loads the library holds
 * KAI_GDN_NOALLOC_SCRATCH_BYTES of device memory until the process exits.
 * Limit: 256 + 512 * batch * ceil(seq / 256) * ceil(channels / 32) bytes
 * <= that size (scans with seq <= 128 need none); larger calls return
 * KAI_GDN_ERR_INVALID with a message.  The first call on a device looks up
 * the array's address (cudaGetSymbolAddress) and should come before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * (several streams or host threads) race and must be serialised.  The
 * looked-up address is kept for the life of the process, so a process that
 * calls cudaDeviceReset must not call this entry point afterwards. */
#define KAI_GDN_NOALLOC_SCRATCH_BYTES (4u << 20)
KAI_GDN_API int kai_run_gdn_gated_scan_noalloc_sm100a(const float *g, const float *x, float *s,
                                                      void *state, int state_dtype, size_t batch,
                                                      size_t seq, size_t channels, void *stream);

/* GDN-2 gated scan (gdn_sve.h:79), fp32 state. */
KAI_GDN_API int kai_run_gdn2_gated_scan_f32_sm100a(const float *g, const float *b_gate,
                                       const float *w_gate, const float *x, float *s,
                                       float *state, size_t batch, size_t seq,
                                       size_t channels, void *stream);

/* Causal depthwise Conv1D k=4 over in[batch][seq][channels]; in, out and
 * hist[batch][3][channels] stored as io_dtype, w[4][channels] fp32, sums in
 * fp32.  Batched form of kai_gdn_causal_dwconv1d_f32_k4_sve.h:39. */
KAI_GDN_API int kai_run_gdn_causal_dwconv1d_k4_sm100a(const void *in, const float *w, void *out,
                                          void *hist, int io_dtype, size_t batch,
                                          size_t seq, size_t channels, void *stream);

/* C = A . B (fp32; M == 1 is the GEMV of kai_gdn_gemv_f32_f32_f32_1x4_neon.h:40,
 * any M is gdn_delta_matmul.h:15). */
KAI_GDN_API int kai_run_gdn_matmul_f32_sm100a(const float *A, const float *B, float *C, size_t M,
                                  size_t K, size_t N, void *stream);

/* Single-token matrix-state delta-rule step for every (batch, value head).
 * Per (b, h), with key head hk = h / (heads_v / heads_k), a = exp(g[b][h]):
 *   S *= a;  kv = S^T k;  delta = (v - kv) * beta;  S += k delta^T;
 *   o = scale * S^T q
 * The math of gpu/gdn_gpu_kernels.cl:158-206 and its C twin
 * gpu/gdn_gpu_validate.c:100-118 (which use one beta and decay for all heads
 * and scale 1), with per-(b,h) gates and grouped value heads. */
typedef struct kai_gdn_decode_args {
    void *state;       /* [batch][heads_v][dk][dv], state_dtype, in/out   */
    const void *q;     /* [batch][heads_k][dk], in_dtype                  */
    const void *k;     /* [batch][heads_k][dk], in_dtype                  */
    const void *v;     /* [batch][heads_v][dv], in_dtype                  */
    const float *g;    /* [batch][heads_v] log-decay (decay = exp(g))     */
    const float *beta; /* [batch][heads_v]                                */
    void *o;           /* [batch][heads_v][dv], out_dtype                 */
    size_t batch, heads_k, heads_v, dk, dv;
    float scale;       /* query scale; 1 = the reference C, 1/sqrt(dk) = HF */
    int in_dtype, state_dtype, out_dtype;
} kai_gdn_decode_args;
KAI_GDN_API int kai_run_gdn_delta_rule_decode_sm100a(const kai_gdn_decode_args *args, void *stream);

/* Single-token matrix-state step of the GDN-2 form (decoupled gating) for
 * every (batch, value head), the recurrence of bench/gdn2_reference.py:58-145
 * (gdn2_recurrent, one token, no q/k normalisation).  Per (b, h), with key
 * head hk = h / (heads_v / heads_k):
 *   S[j][:] *= exp(g[j]);  erase = S^T (b_gate . k);  write = w_gate . v;
 *   S += k (write - erase)^T;  o = scale * S^T q
 * The gates are per channel: g and b_gate per key channel, w_gate per value
 * channel.  Shapes, dtypes and alignment as kai_gdn_decode_args. */
typedef struct kai_gdn2_decode_args {
    void *state;         /* [batch][heads_v][dk][dv], state_dtype, in place */
    const void *q;       /* [batch][heads_k][dk], in_dtype                  */
    const void *k;       /* [batch][heads_k][dk], in_dtype                  */
    const void *v;       /* [batch][heads_v][dv], in_dtype                  */
    const float *g;      /* [batch][heads_v][dk] log-decay per key channel  */
    const float *b_gate; /* [batch][heads_v][dk] erase gate                 */
    const float *w_gate; /* [batch][heads_v][dv] write gate                 */
    void *o;             /* [batch][heads_v][dv], out_dtype                 */
    size_t batch, heads_k, heads_v, dk, dv;
    float scale;
    int in_dtype, state_dtype, out_dtype;
} kai_gdn2_decode_args;
KAI_GDN_API int kai_run_gdn2_delta_rule_decode_sm100a(const kai_gdn2_decode_args *args, void *stream);

/* int8 weights with one fp32 scale per output column (symmetric), the
 * weight format of the reference's INT8_WEIGHTS decode path
 * (src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c).
 *
 * Quantize B [K][N] fp32 (row-major) into q [K][N] int8 and s [N]:
 *   s[n] = max_k |B[k][n]| / 127 (1 for an all-zero column),
 *   q[k][n] = clamp(lroundf(B[k][n] * (1 / s[n])), -128, 127),
 * bit-identical to quantize_weight (gdn_e2e_decode.c:175-199). */
KAI_GDN_API int kai_run_gdn_quantize_int8_sm100a(const float *B, int8_t *q, float *s, size_t K, size_t N,
                                                 void *stream);
/* C [M][N] = (A [M][K] . q) * s[n], fp32: matmul_int8 (gdn_e2e_decode.c:681),
 * i.e. gemv_int8_neon (:296) for M = 1 and gemm_int8_neon (:608) for M > 1.
 * The products are summed in a different order than the reference's (split
 * over K, fused multiply-add); the reference's own accuracy rule
 * (test_gdn_e2e_int8.c: |C - A.B| <= s * sum|a| against the fp32 product)
 * holds.  Deterministic. */
KAI_GDN_API int kai_run_gdn_matmul_int8_sm100a(const float *A, const int8_t *q, const float *s, float *C, size_t M,
                                               size_t K, size_t N, void *stream);
/* The same product over weights packed once for streaming (the analogue of
 * the reference preparing its QW weights once at load, quantize_weight,
 * gdn_e2e_decode.c:175-199).  kai_gdn_int8_packed_bytes gives the size of
 * the packed form of q [K][N] (0 when N % 16 is non-zero or K > 131072);
 * kai_run_gdn_int8_pack_sm100a writes it (qp 16-byte aligned, device
 * memory, not aliasing q); kai_run_gdn_matmul_int8_packed_sm100a computes C
 * from it on the int8 tensor cores: up to 16 activation rows as one stream
 * over the weights, more rows (a prompt) as a GEMM of 64-row x 128-column
 * tiles.  Each activation row is carried as three 8-bit fixed-point terms
 * of its largest magnitude (representation error at most 2^-24 of it, one
 * fp32 rounding) and the products are summed exactly in integers, so the
 * result is deterministic whatever the work split, and agrees with
 * kai_run_gdn_matmul_int8_sm100a to fp32 accuracy.  Activations must be
 * finite. */
KAI_GDN_API size_t kai_gdn_int8_packed_bytes(size_t K, size_t N);
KAI_GDN_API int kai_run_gdn_int8_pack_sm100a(const int8_t *q, int8_t *qp, size_t K, size_t N, void *stream);
KAI_GDN_API int kai_run_gdn_matmul_int8_packed_sm100a(const float *A, const int8_t *qp, const float *s, float *C,
                                                      size_t M, size_t K, size_t N, void *stream);

/* Grouped-query attention decode with a growing KV cache, the full-attention
 * layer of the reference's hybrid decode: full_attn_real_forward
 * (src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:1532-1634, fp32 cache)
 * and full_attn_real_forward_int8kv (:1652-1830, int8 cache with one scale
 * per kv head); bf16 caches store round-to-nearest-even values.  For every
 * sequence b: this token's k_new, v_new are written into the caches at `pos`
 * (int8: clamp(lroundf(x * (1 / scale)), -128, 127)), then query head h
 * (kv head h / (heads / kv_heads)) attends over positions 0..pos:
 *   s_t = (q_h . k_t) * scale   (int8: * (k_scale * scale)),
 *   o_h = sum_t softmax(s)_t v_t   (int8: * v_scale).
 * All sequences are at the same position.  head_dim 128 or 256; 1, 2, 4 or 8
 * query heads per kv head; caches and q 16-byte aligned. */
typedef struct kai_gdn_attn_decode_args {
    const float *q;       /* [batch][heads][head_dim]                        */
    const float *k_new;   /* [batch][kv_heads][head_dim]                     */
    const float *v_new;   /* [batch][kv_heads][head_dim]                     */
    void *k_cache;        /* [batch][max_ctx][kv_heads][head_dim], cache_dtype */
    void *v_cache;        /* same                                            */
    const float *k_scale; /* KAI_GDN_I8: [batch][kv_heads]; otherwise unused */
    const float *v_scale; /* KAI_GDN_I8: [batch][kv_heads]; otherwise unused */
    float *o;             /* [batch][heads][head_dim]                        */
    size_t batch, heads, kv_heads, head_dim, pos, max_ctx;
    float scale;          /* 1 / sqrt(head_dim) in the reference             */
    int cache_dtype;      /* KAI_GDN_F32, KAI_GDN_BF16 or KAI_GDN_I8         */
} kai_gdn_attn_decode_args;
KAI_GDN_API int kai_run_gdn_attention_decode_sm100a(const kai_gdn_attn_decode_args *args, void *stream);

/* The same attention for a whole prompt (not in the reference, which feeds
 * its prompt one token at a time through full_attn_real_forward): the keys
 * and values of positions 0 .. pos0 + T - 1 are already in the bf16 caches,
 * and query t of sequence b (position pos0 + t) attends over positions
 * 0 .. pos0 + t (causal):
 *   o[b][t][h] = sum_{s <= pos0 + t} softmax_s((q[b][t][h] . k_s) * scale) v_s.
 * Equal to T calls of kai_run_gdn_attention_decode_sm100a (positions pos0 ..)
 * to fp32 accuracy (queries and softmax weights carried as two bf16 terms,
 * 16 significant bits; products summed in fp32).  bf16 caches only;
 * head_dim 128 or 256; 1, 2, 4 or 8 query heads per kv head; caches 16-byte
 * aligned. */
typedef struct kai_gdn_attn_prefill_args {
    const float *q;        /* [batch][T][heads][head_dim]                     */
    const void *k_cache;   /* [batch][max_ctx][kv_heads][head_dim] bf16       */
    const void *v_cache;   /* same                                            */
    float *o;              /* [batch][T][heads][head_dim]                     */
    size_t batch, T, heads, kv_heads, head_dim, pos0, max_ctx;
    float scale;
} kai_gdn_attn_prefill_args;
KAI_GDN_API int kai_run_gdn_attention_prefill_sm100a(const kai_gdn_attn_prefill_args *args, void *stream);

/* End-to-end hybrid decode: the reference's decode loop
 * (src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:2775-2796) on the
 * GPU, one token through every layer for `batch` independent sequences:
 * GDN layers as gdn_layer_forward (:1426-1490: q/k/v projections, Conv1D over
 * [q | 0], the per-channel gate as decay, gated scan of v, output projection,
 * residual), attention layers as the loop's full_attn_layer_forward
 * (:1492-1522: projections, the new K/V into a one-entry cache, output
 * projection of q, residual), each followed by ffn_forward (:1834-1855:
 * SwiGLU, residual).  One weight set (the reference's Weights, host fp32,
 * row-major [in][out], conv weights [4][conv_dim]) serves every layer and is
 * quantized to int8 with per-column scales at creation (the INT8_WEIGHTS
 * build).  When value_dim > key_dim the reference's scan reads past its
 * key_dim-long decay vector; the engine repeats the key_dim gates there.
 * The engine captures a token into a CUDA graph on the caller's stream after
 * one eager step on that stream and replays it afterwards. */
typedef struct kai_gdn_e2e_config {
    size_t hidden, key_dim, value_dim, conv_dim, inter;   /* HIDDEN, KEY_DIM, VALUE_DIM, CONV_DIM, INTER */
    size_t full_heads, full_kv_heads, full_head_dim;      /* attention layer geometry            */
    size_t layers;                                        /* NUM_LAYERS                          */
    const unsigned char *is_gdn;                          /* [layers]: 1 GDN, 0 attention        */
    size_t batch;                                         /* sequences decoded together          */
} kai_gdn_e2e_config;
typedef struct kai_gdn_e2e_weights {
    const float *g_q_proj, *g_k_proj, *g_v_proj, *g_o_proj, *g_conv_w, *g_beta;
    const float *f_q_proj, *f_k_proj, *f_v_proj, *f_o_proj;
    const float *gate_proj, *up_proj, *down_proj;
} kai_gdn_e2e_weights;
KAI_GDN_API int kai_gdn_e2e_create(const kai_gdn_e2e_config *cfg, const kai_gdn_e2e_weights *weights,
                                   void **engine);
/* hidden_in, hidden_out: [batch][hidden] fp32, host or device memory. */
KAI_GDN_API int kai_gdn_e2e_step(void *engine, const float *hidden_in, float *hidden_out, void *stream);
/* Copy one GDN layer's recurrent state [batch][value_dim] and Conv1D history
 * [batch][3][conv_dim] out (either may be NULL); synchronises the device. */
KAI_GDN_API int kai_gdn_e2e_state(void *engine, size_t layer, float *gdn_state, float *conv_hist);
KAI_GDN_API int kai_gdn_e2e_destroy(void *engine);

/* Decode engine of a Qwen3.5-style GDN hybrid, tensor
 * parallel over NCCL.  No single reference counterpart: it runs the layer
 * structure of the reference's model notes (docs/GDN_ARCHITECTURE_AUDIT.md
 * sections 2-3) in the block order of its decode loop
 * (gdn_e2e_decode.c:2775-2796), on this library's kernels:
 *   - GDN layers: in-projection, Conv1D + SiLU, L2-normalised q / k, the
 *     decode step, gated RMSNorm, out-projection;
 *   - attention layers: q / gate / k / v, per-head RMSNorm, partial RoPE,
 *     GQA decode over a bf16 KV cache, sigmoid gate, o-projection;
 *   - each layer's SwiGLU FFN after RMSNorm;
 *   - embedding, final RMSNorm, LM head and greedy argmax.
 * All projections are int8 with per-column scales (quantize_weight,
 * gdn_e2e_decode.c:175-199).  The weights are N(0, weight_std) from `seed`,
 * generated on the device; norm weights are 1 + N(0, weight_std).  With
 * tp_size > 1 each rank holds its heads, FFN columns and vocabulary shard,
 * and the output projections meet in NCCL all-reduces (two per layer, over
 * [batch][hidden]).  The engine loads libnccl.so.2 at run time. */
#define KAI_GDN_NCCL_ID_BYTES 128
typedef struct kai_gdn_model_config {
    size_t hidden, layers, vocab, inter;           /* 2560, 32, 151936, 9216 for config 4 */
    const unsigned char *is_gdn;                   /* [layers]: 1 GDN, 0 attention (host)  */
    size_t gdn_heads_k, gdn_heads_v, gdn_head_dim; /* 16, 32, 128                          */
    size_t attn_heads, attn_kv_heads, attn_head_dim, rope_dims; /* 16, 4, 256, 64          */
    float rope_theta, rms_eps;
    size_t batch, max_ctx;                         /* sequences; KV cache capacity (tokens) */
    int tp_rank, tp_size;                          /* tensor-parallel position              */
    const void *nccl_id;                           /* KAI_GDN_NCCL_ID_BYTES, same on every rank (tp_size > 1) */
    unsigned long long seed;
    float weight_std;                              /* 0: 0.02                               */
} kai_gdn_model_config;
/* A fresh NCCL unique id (rank 0 makes it and shares it with the others);
 * an id serves the creation of one engine's communicator. */
KAI_GDN_API int kai_gdn_model_nccl_id(void *id_out);
KAI_GDN_API int kai_gdn_model_create(const kai_gdn_model_config *cfg, void **engine);
/* One greedy decode step of every sequence at position `pos` (0-based): reads
 * the engine's current tokens [batch], leaves the argmax tokens in their
 * place.  Stream-ordered; the first step on a stream runs eagerly, the
 * second captures the per-segment CUDA graphs, later ones replay them. */
KAI_GDN_API int kai_gdn_model_step(void *engine, size_t pos, void *stream);
/* Consume a prompt of T tokens per sequence (tokens [batch][T], int32, host
 * or device memory) at positions pos0 .. pos0 + T - 1, as T decode steps
 * would but in whole-prompt launches: projections over all T rows, the GDN
 * layers' chunked delta-rule scan from their current state, the attention
 * layers' keys and values written into the cache and the causal prompt
 * attention.  Leaves the state for a decode step at position pos0 + T and
 * the greedy next tokens as the current tokens.  Synchronises `stream`. */
KAI_GDN_API int kai_gdn_model_prefill(void *engine, const int32_t *tokens, size_t T, size_t pos0, void *stream);
/* Set (set = 1) or read (set = 0) the current tokens [batch] (int32, host or
 * device memory); synchronises the device. */
KAI_GDN_API int kai_gdn_model_tokens(void *engine, int32_t *tokens, int set);
#define KAI_GDN_MODEL_HIDDEN 0 /* [batch][hidden] residual stream after the last step */
#define KAI_GDN_MODEL_LOGITS 1 /* [batch][vocab / tp_size] this rank's logits         */
KAI_GDN_API int kai_gdn_model_read(void *engine, int what, float *out);
/* Copy out this rank's weight `which` of `layer` (for a checker): int8 codes
 * [rows][cols] and fp32 scales [cols] of a projection (the embedding:
 * [vocab][hidden] codes, one scale per row), or an fp32 vector (rows = 1).
 * data / scales may be NULL to query the shape. */
#define KAI_GDN_MODEL_W_IN 0        /* GDN [q|k|v|z|b|a|pad], attention [q,gate per head|k|v] */
#define KAI_GDN_MODEL_W_OUT 1       /* GDN out / attention o projection (this rank's rows)    */
#define KAI_GDN_MODEL_W_GATE_UP 2   /* FFN [gate | up]                                        */
#define KAI_GDN_MODEL_W_DOWN 3      /* FFN down (this rank's rows)                            */
#define KAI_GDN_MODEL_V_NORM_IN 4
#define KAI_GDN_MODEL_V_NORM_POST 5
#define KAI_GDN_MODEL_V_CONV 6      /* [4][channels]                                          */
#define KAI_GDN_MODEL_V_A_LOG 7
#define KAI_GDN_MODEL_V_DT_BIAS 8
#define KAI_GDN_MODEL_V_NORM_GDN 9
#define KAI_GDN_MODEL_V_NORM_Q 10
#define KAI_GDN_MODEL_V_NORM_K 11
#define KAI_GDN_MODEL_W_LM 12       /* [hidden][vocab / tp_size]                              */
#define KAI_GDN_MODEL_V_NORM_FINAL 13
#define KAI_GDN_MODEL_W_EMBED 14
KAI_GDN_API int kai_gdn_model_weight(void *engine, size_t layer, int which, void *data, float *scales,
                                     size_t *rows, size_t *cols);
/* Synthetic state of `ctx` already-consumed tokens: KV cache rows [0, ctx)
 * N(0, 1) in bf16, GDN states N(0, 0.02), conv histories N(0, 1). */
KAI_GDN_API int kai_gdn_model_fill(void *engine, size_t ctx, unsigned long long seed);
/* Every sequence back to position 0 (a new prompt follows): GDN states and
 * conv histories zero.  Synchronises the device. */
KAI_GDN_API int kai_gdn_model_reset(void *engine);
KAI_GDN_API int kai_gdn_model_destroy(void *engine);

/* Chunkwise (WY / UT-transform) gated delta-rule scan over a whole sequence,
 * for every (batch, value head), chunk length `chunk` (64).  Equal, up to
 * rounding, to applying the decode step above for t = 0 .. seq-1 with
 * g, beta taken per token.  The reference names this form
 * (docs/GDN_ARCHITECTURE_AUDIT.md:142-153) and reaches it only through HF
 * transformers' torch_chunk_gated_delta_rule.
 * fp32 q/k/v at dk = 128 (16-byte aligned q, k, v, o; dv a multiple of 32)
 * run on the tensor cores in two launches whose per-chunk operands go through
 * library scratch of the stream (at most 256 MiB, allocated on the first call
 * that needs it on that stream and kept; a longer sequence runs in segments);
 * bf16 / fp16 inputs and other head sizes use no scratch. */
typedef struct kai_gdn_chunk_args {
    const void *q;     /* [batch][seq][heads_k][dk], in_dtype             */
    const void *k;     /* [batch][seq][heads_k][dk], in_dtype             */
    const void *v;     /* [batch][seq][heads_v][dv], in_dtype             */
    const float *g;    /* [batch][seq][heads_v] log-decay                 */
    const float *beta; /* [batch][seq][heads_v]                           */
    void *state;       /* [batch][heads_v][dk][dv], state_dtype: initial
                          state on entry, final state on exit             */
    void *o;           /* [batch][seq][heads_v][dv], out_dtype            */
    size_t batch, seq, heads_k, heads_v, dk, dv, chunk;
    float scale;
    int in_dtype, state_dtype, out_dtype;
} kai_gdn_chunk_args;
KAI_GDN_API int kai_run_gdn_chunk_delta_rule_sm100a(const kai_gdn_chunk_args *args, void *stream);

/* ======================================================================
 * 3. Library control
 * ==================================================================== */

/* Make `device` current for this host thread (one thread per GPU in the
 * multi-GPU driver).  Returns a status.  The library keeps per-device state
 * for the life of the process (device addresses of its file-scope words,
 * per-stream scratch, tensor-map and attribute caches); a process that calls
 * cudaDeviceReset must not use the library on that device afterwards. */
KAI_GDN_API int kai_gdn_cuda_set_device(int device);
/* Number of visible CUDA devices, or -1 on error. */
KAI_GDN_API int kai_gdn_cuda_device_count(void);
/* Status and message of the last failure on this host thread ("" if none);
 * kai_gdn_cuda_clear_error() resets both. */
KAI_GDN_API int kai_gdn_cuda_last_status(void);
KAI_GDN_API const char *kai_gdn_cuda_last_error(void);
KAI_GDN_API void kai_gdn_cuda_clear_error(void);

/* Kernels that wait on work of other threads of the same kernel (the
 * tensor-core chunk scan's hand-overs, the long scans' look-back) bound every
 * wait; a wait that runs out records it in a word on the current device and
 * the kernel finishes without its result.  The stream-ordered entry points
 * return before their kernels run, so they cannot see it: this call
 * synchronises `stream`, reads and clears the word, and returns
 * KAI_GDN_ERR_TIMEOUT (with a message) if any wait of the kernels before it
 * ran out, else KAI_GDN_OK.  The synchronous drop-in entry points check it
 * themselves.  No reference counterpart (the reference has no such waits). */
KAI_GDN_API int kai_gdn_cuda_device_status(void *stream);
/* Library version string. */
KAI_GDN_API const char *kai_gdn_cuda_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KAI_GDN_CUDA_H */
