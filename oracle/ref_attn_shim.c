/* oracle/ref_attn_shim.c -- test infrastructure only (a parity checker).
 *
 * Runs the reference's own GQA attention decode, full_attn_real_forward
 * (src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:1532-1634) or, built
 * with -DKV_INT8, full_attn_real_forward_int8kv (:1652-1830), on given q, k, v
 * and cache.  Both functions are `static` and wrap the attention in the
 * layer's q/k/v and output projections, so the source is compiled into this
 * translation unit (main() renamed, as test_gdn_e2e_int8.c:24-26 does) and
 * the projections are made exact copies: hidden_in is the unit vector e_R,
 * so q = row R of f_q_proj (likewise k, v), and f_o_proj is a 0/1 selection
 * matrix, so hidden_out[i] = attn_out[sel(i)] exactly (every other product is
 * a zero).  Column R also receives the residual and is skipped; two calls with
 * two selections recover all FULL_HEADS * FULL_HEAD_DIM outputs.  Built by
 * `make -C oracle ref` for the default (4B) geometry. */
#define main gdn_e2e_decode_main_unused
#include "gdn_e2e_decode.c"
#undef main

#define ATT_QD (FULL_HEADS * FULL_HEAD_DIM)
#define ATT_KVD (FULL_KV_HEADS * FULL_HEAD_DIM)
#define ATT_R (HIDDEN - 1)

void ref_attn_geometry(size_t *heads, size_t *kv_heads, size_t *head_dim) {
    *heads = FULL_HEADS;
    *kv_heads = FULL_KV_HEADS;
    *head_dim = FULL_HEAD_DIM;
}

/* q [ATT_QD], k_new, v_new [ATT_KVD]; caches [max_ctx][ATT_KVD] (float, or
 * int8 with k_scale / v_scale [FULL_KV_HEADS] under KV_INT8) are updated in
 * place (the new token at pos); o [ATT_QD]. */
void ref_attn_decode(const float *q, const float *k_new, const float *v_new, void *k_cache, void *v_cache,
                     const float *k_scale, const float *v_scale, size_t pos, size_t max_ctx, float *o) {
    Weights w;
    memset(&w, 0, sizeof(w));
    w.f_q_proj = alloc_aligned((size_t)HIDDEN * ATT_QD);
    w.f_k_proj = alloc_aligned((size_t)HIDDEN * ATT_KVD);
    w.f_v_proj = alloc_aligned((size_t)HIDDEN * ATT_KVD);
    w.f_o_proj = alloc_aligned((size_t)ATT_QD * HIDDEN);
    memcpy(w.f_q_proj + (size_t)ATT_R * ATT_QD, q, ATT_QD * sizeof(float));
    memcpy(w.f_k_proj + (size_t)ATT_R * ATT_KVD, k_new, ATT_KVD * sizeof(float));
    memcpy(w.f_v_proj + (size_t)ATT_R * ATT_KVD, v_new, ATT_KVD * sizeof(float));
    float *hin = alloc_aligned(HIDDEN), *hout = alloc_aligned(HIDDEN);
    hin[ATT_R] = 1.0f;
#ifdef KV_INT8
    const size_t esz = 1;
#else
    const size_t esz = sizeof(float);
#endif
    void *kc = malloc(max_ctx * ATT_KVD * esz), *vc = malloc(max_ctx * ATT_KVD * esz);
    for (int pass = 0; pass < 2; ++pass) {
        const size_t first = pass == 0 ? 0 : (size_t)ATT_QD - ATT_R;  /* attn_out index of column 0 */
        memset(w.f_o_proj, 0, (size_t)ATT_QD * HIDDEN * sizeof(float));
        for (size_t i = 0; i < (size_t)ATT_R; ++i) w.f_o_proj[(first + i) * HIDDEN + i] = 1.0f;
        memcpy(kc, k_cache, max_ctx * ATT_KVD * esz);
        memcpy(vc, v_cache, max_ctx * ATT_KVD * esz);
        LayerState st;
        memset(&st, 0, sizeof(st));
        st.kv_pos = pos;
#ifdef KV_INT8
        st.kv_k_grow_q = (int8_t *)kc;
        st.kv_v_grow_q = (int8_t *)vc;
        st.kv_k_scale = (float *)k_scale;
        st.kv_v_scale = (float *)v_scale;
        full_attn_real_forward_int8kv(&w, &st, hin, hout);
#else
        (void)k_scale;
        (void)v_scale;
        st.kv_k_grow = (float *)kc;
        st.kv_v_grow = (float *)vc;
        full_attn_real_forward(&w, &st, hin, hout);
#endif
        for (size_t i = 0; i < (size_t)ATT_R; ++i) o[first + i] = hout[i];
    }
    memcpy(k_cache, kc, max_ctx * ATT_KVD * esz);
    memcpy(v_cache, vc, max_ctx * ATT_KVD * esz);
    free(kc);
    free(vc);
    free(hin);
    free(hout);
    free(w.f_q_proj);
    free(w.f_k_proj);
    free(w.f_v_proj);
    free(w.f_o_proj);
}
