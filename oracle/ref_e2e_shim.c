/* oracle/ref_e2e_shim.c -- test infrastructure only (a parity checker).
 *
 * Runs the reference's own end-to-end hybrid decode loop
 * (src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c:2775-2796) on given
 * weights and hidden inputs: the layer functions gdn_layer_forward
 * (:1426-1490), full_attn_layer_forward (:1492-1522) and ffn_forward
 * (:1834-1855) are `static`, so the source is compiled into this translation
 * unit with main() renamed (as test_gdn_e2e_int8.c:24-26 does).  Weights are
 * quantized with the reference's quantize_weight as its main() does
 * (:2311-2321) and the per-layer state is set up as there (:2399-2407).
 * Built by `make -C oracle ref` with -DINT8_WEIGHTS -DMODEL_08B: the 0.8B
 * geometry, where KEY_DIM == VALUE_DIM and the GDN stand-in's scan stays
 * inside its decay buffer. */
#define main gdn_e2e_decode_main_unused
#include "gdn_e2e_decode.c"
#undef main

void ref_e2e_geometry(size_t *dims) {
    dims[0] = HIDDEN;
    dims[1] = KEY_DIM;
    dims[2] = VALUE_DIM;
    dims[3] = CONV_DIM;
    dims[4] = INTER;
    dims[5] = FULL_HEADS;
    dims[6] = FULL_KV_HEADS;
    dims[7] = FULL_HEAD_DIM;
    dims[8] = NUM_LAYERS;
}

static float *ref_copy(const float *src, size_t n) {
    float *p = alloc_aligned(n);
    memcpy(p, src, n * sizeof(float));
    return p;
}

/* hidden_in / hidden_out [T][HIDDEN]; gdn_state_out [NUM_LAYERS][VALUE_DIM]
 * (GDN layers' final states; other rows untouched). */
void ref_e2e_decode(const float *g_q, const float *g_k, const float *g_v, const float *g_o, const float *g_conv_w,
                    const float *g_beta, const float *f_q, const float *f_k, const float *f_v, const float *f_o,
                    const float *gate_w, const float *up_w, const float *down_w, const float *hidden_in,
                    float *hidden_out, size_t T, float *gdn_state_out) {
    const size_t qd = FULL_HEADS * FULL_HEAD_DIM, kvd = FULL_KV_HEADS * FULL_HEAD_DIM;
    Weights w;
    memset(&w, 0, sizeof(w));
    w.g_q_proj = ref_copy(g_q, (size_t)HIDDEN * KEY_DIM);
    w.g_k_proj = ref_copy(g_k, (size_t)HIDDEN * KEY_DIM);
    w.g_v_proj = ref_copy(g_v, (size_t)HIDDEN * VALUE_DIM);
    w.g_o_proj = ref_copy(g_o, (size_t)VALUE_DIM * HIDDEN);
    w.g_conv_w = ref_copy(g_conv_w, (size_t)CONV_DIM * CONV_K);
    w.g_beta = ref_copy(g_beta, KEY_DIM);
    w.f_q_proj = ref_copy(f_q, (size_t)HIDDEN * qd);
    w.f_k_proj = ref_copy(f_k, (size_t)HIDDEN * kvd);
    w.f_v_proj = ref_copy(f_v, (size_t)HIDDEN * kvd);
    w.f_o_proj = ref_copy(f_o, qd * HIDDEN);
    w.gate_proj = ref_copy(gate_w, (size_t)HIDDEN * INTER);
    w.up_proj = ref_copy(up_w, (size_t)HIDDEN * INTER);
    w.down_proj = ref_copy(down_w, (size_t)INTER * HIDDEN);
    quantize_weight(w.g_q_proj, &w.g_q_proj_q.q, &w.g_q_proj_q.s, HIDDEN, KEY_DIM);
    quantize_weight(w.g_k_proj, &w.g_k_proj_q.q, &w.g_k_proj_q.s, HIDDEN, KEY_DIM);
    quantize_weight(w.g_v_proj, &w.g_v_proj_q.q, &w.g_v_proj_q.s, HIDDEN, VALUE_DIM);
    quantize_weight(w.g_o_proj, &w.g_o_proj_q.q, &w.g_o_proj_q.s, VALUE_DIM, HIDDEN);
    quantize_weight(w.f_q_proj, &w.f_q_proj_q.q, &w.f_q_proj_q.s, HIDDEN, qd);
    quantize_weight(w.f_k_proj, &w.f_k_proj_q.q, &w.f_k_proj_q.s, HIDDEN, kvd);
    quantize_weight(w.f_v_proj, &w.f_v_proj_q.q, &w.f_v_proj_q.s, HIDDEN, kvd);
    quantize_weight(w.f_o_proj, &w.f_o_proj_q.q, &w.f_o_proj_q.s, qd, HIDDEN);
    quantize_weight(w.gate_proj, &w.gate_proj_q.q, &w.gate_proj_q.s, HIDDEN, INTER);
    quantize_weight(w.up_proj, &w.up_proj_q.q, &w.up_proj_q.s, HIDDEN, INTER);
    quantize_weight(w.down_proj, &w.down_proj_q.q, &w.down_proj_q.s, INTER, HIDDEN);

    LayerState states[NUM_LAYERS];
    memset(states, 0, sizeof(states));
    for (int l = 0; l < NUM_LAYERS; ++l) {
        states[l].gdn_state = alloc_aligned(VALUE_DIM);
        states[l].conv_hist = alloc_aligned((CONV_K - 1) * CONV_DIM);
        states[l].kv_cache_k = alloc_aligned(kvd);
        states[l].kv_cache_v = alloc_aligned(kvd);
    }
    int is_gdn[NUM_LAYERS];
    for (int b = 0; b < NUM_LAYERS / 4; ++b)
        for (int s = 0; s < 4; ++s) is_gdn[b * 4 + s] = (s < 3) ? 1 : 0;

    float *hidden = alloc_aligned(HIDDEN), *hidden_next = alloc_aligned(HIDDEN);
    for (size_t t = 0; t < T; ++t) {
        memcpy(hidden, hidden_in + t * HIDDEN, HIDDEN * sizeof(float));
        for (int l = 0; l < NUM_LAYERS; ++l) {
            if (is_gdn[l])
                gdn_layer_forward(&w, &states[l], hidden, hidden_next, 1);
            else
                full_attn_layer_forward(&w, &states[l], hidden, hidden_next, 1);
            ffn_forward(&w, hidden_next, hidden, 1);
        }
        memcpy(hidden_out + t * HIDDEN, hidden, HIDDEN * sizeof(float));
    }
    for (int l = 0; l < NUM_LAYERS; ++l) {
        if (is_gdn[l] && gdn_state_out) memcpy(gdn_state_out + (size_t)l * VALUE_DIM, states[l].gdn_state, VALUE_DIM * sizeof(float));
        free(states[l].gdn_state);
        free(states[l].conv_hist);
        free(states[l].kv_cache_k);
        free(states[l].kv_cache_v);
    }
    free(hidden);
    free(hidden_next);
    free(w.g_q_proj); free(w.g_k_proj); free(w.g_v_proj); free(w.g_o_proj); free(w.g_conv_w); free(w.g_beta);
    free(w.f_q_proj); free(w.f_k_proj); free(w.f_v_proj); free(w.f_o_proj);
    free(w.gate_proj); free(w.up_proj); free(w.down_proj);
    QW *qws[] = {&w.g_q_proj_q, &w.g_k_proj_q, &w.g_v_proj_q, &w.g_o_proj_q, &w.f_q_proj_q, &w.f_k_proj_q,
                 &w.f_v_proj_q, &w.f_o_proj_q, &w.gate_proj_q, &w.up_proj_q, &w.down_proj_q};
    for (size_t i = 0; i < sizeof(qws) / sizeof(qws[0]); ++i) {
        free(qws[i]->q);
        free(qws[i]->s);
    }
}
