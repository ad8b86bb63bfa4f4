/* oracle/ref_int8_shim.c -- test infrastructure only (a parity checker).
 *
 * The reference keeps its int8 weight functions `static` inside
 * src/orionsbelt/engines/cpu/kernels/gdn_e2e_decode.c (quantize_weight
 * :175-199, gemv_int8_neon :296-358, gemm_int8_neon :608-678).  Its own test
 * reaches them by compiling that file into the test's translation unit with
 * main() renamed (test_gdn_e2e_int8.c:24-26); this file does the same, from
 * the reference tree where it lies (nothing is copied), and exports the three
 * functions under ref_* names for the oracle's pin tests.  Built by
 * `make -C oracle ref` into _ref/libint8ref.so with -DINT8_WEIGHTS. */
#define main gdn_e2e_decode_main_unused
#include "gdn_e2e_decode.c"
#undef main

#include <string.h>

void ref_quantize_int8(const float *B, int8_t *q, float *s, size_t K, size_t N) {
    int8_t *qq = NULL;
    float *ss = NULL;
    quantize_weight(B, &qq, &ss, K, N);
    memcpy(q, qq, K * N);
    memcpy(s, ss, N * sizeof(float));
    free(qq);
    free(ss);
}

void ref_gemv_int8(const float *a, const int8_t *q, const float *s, float *c, size_t K, size_t N) {
    gemv_int8_neon(a, q, s, c, K, N);
}

void ref_gemm_int8(const float *A, const int8_t *q, const float *s, float *C, size_t M, size_t K, size_t N) {
    gemm_int8_neon(A, q, s, C, M, K, N);
}
