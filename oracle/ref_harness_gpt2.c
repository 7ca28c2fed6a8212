/*
 * ref_harness_gpt2.c -- exposes the GPT-2 server's own int8 LM-head code as a
 * shared library (oracle/_ref/liblal_ref_gpt2.so) for parity checks.
 *
 * TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile from the reference
 * sources where they lie; no reference source is copied into this
 * repository.  The server translation unit tools/server/gpt2_server.c is
 * included whole, with its main() renamed, so that its static quantizer
 * lm_head_quantize_x (:1982-1998) and lm_head_int8_parallel (:2125-2214, the
 * int8 logits plus the float re-score of the 512 rows its heap keeps) run
 * exactly as the server compiles them (VOCAB_SIZE 50257, N_EMBD 768);
 * runtime/lal_runtime.c, which the server links for its weight loader, is
 * compiled beside it from the same checkout.  The
 * sampling block (:2862-3013) sits inside the server's forward function and
 * cannot be called alone.
 */
#define main lal_ref_gpt2_server_main
#include "tools/server/gpt2_server.c"
#undef main

#define REF_API __attribute__((visibility("default")))

REF_API int ref_gpt2_vocab(void) { return VOCAB_SIZE; }
REF_API int ref_gpt2_n_embd(void) { return N_EMBD; }

REF_API float ref_gpt2_quantize_x(const float *x, int8_t *xq, int n) {
    return lm_head_quantize_x(x, xq, n);
}

/* lm_head_int8_parallel over the caller's int8 rows and scales (the
 * server's g_wte_q / g_wte_scale), n_threads as the server's --threads */
REF_API void ref_gpt2_lm_head(float *logits, const float *x, int8_t *wte_q, float *scale_w,
                              int n_threads) {
    g_wte_q = wte_q;
    g_wte_scale = scale_w;
    lm_head_int8_parallel(logits, x, n_threads);
    g_wte_q = NULL;
    g_wte_scale = NULL;
}
