/*
 * Drop-in for runtime/lal_q8_kernel.h of samaidev/lal.
 *
 * Put this repository's include/ directory ahead of the LAL checkout on the
 * include path (-I<this repo>/include -I<lal>): a server's
 *     #include "runtime/lal_q8_kernel.h"
 * then resolves here.  The transformer-body kernels of the original header
 * (lal_matmul_q8_signtrick, lal_matmul_q8_0, ...) are still taken from it via
 * #include_next; the decode-tail functions it defines are renamed out of the
 * way and replaced by the GPU versions exported by liblal_tail.so, with the
 * same names and signatures:
 *
 *   lal_quantize_x_int8             runtime/lal_q8_kernel.h:375
 *   lal_compute_abs_xq              runtime/lal_q8_kernel.h:450
 *   lal_lm_head_int8_range          runtime/lal_q8_kernel.h:463
 *   lal_lm_head_int8_range_abs      runtime/lal_q8_kernel.h:506
 *   lal_lm_head_int8_range_abs_8row runtime/lal_q8_kernel.h:551
 *   lal_quantize_q8_per_row         runtime/lal_q8_kernel.h:357
 *
 * Link with -llal_tail.  XQ_MAX must still be defined by the includer, as the
 * original header requires (lal_q8_kernel.h:35-37).
 */
#ifndef LAL_TAIL_DROPIN_Q8_KERNEL_H
#define LAL_TAIL_DROPIN_Q8_KERNEL_H

#include <stdint.h>

#if defined(__has_include_next)
#if __has_include_next("runtime/lal_q8_kernel.h")
#define LAL_TAIL_HAVE_ORIGINAL_Q8 1
#endif
#endif

#ifdef LAL_TAIL_HAVE_ORIGINAL_Q8
#define lal_quantize_x_int8 lal_cpu_quantize_x_int8_replaced
#define lal_compute_abs_xq lal_cpu_compute_abs_xq_replaced
#define lal_lm_head_int8_range lal_cpu_lm_head_int8_range_replaced
#define lal_lm_head_int8_range_abs lal_cpu_lm_head_int8_range_abs_replaced
#define lal_lm_head_int8_range_abs_8row lal_cpu_lm_head_int8_range_abs_8row_replaced
#define lal_quantize_q8_per_row lal_cpu_quantize_q8_per_row_replaced
#include_next "runtime/lal_q8_kernel.h"
#undef lal_quantize_x_int8
#undef lal_compute_abs_xq
#undef lal_lm_head_int8_range
#undef lal_lm_head_int8_range_abs
#undef lal_lm_head_int8_range_abs_8row
#undef lal_quantize_q8_per_row
#endif

#include "../lal_tail.h"

#ifdef __cplusplus
extern "C" {
#endif

/* runtime/lal_q8_kernel.h:375-442: absmax scale floored at 1e-8; round to
 * nearest even for the first n&~7 elements, truncation for the last n%8
 * (the AVX2+FMA build); returns the scale. */
float lal_quantize_x_int8(const float *x, int8_t *xq, int n);

/* runtime/lal_q8_kernel.h:450-460: ax = |xq| as uint8. */
void lal_compute_abs_xq(const int8_t *xq, uint8_t *ax, int n_embd);

/* runtime/lal_q8_kernel.h:463-499: logits[v] = scale_x*scale_w[v]*(float)dot
 * for v in [v_start, v_end).  The host LM head is copied to the GPU on first
 * use and cached by its address (lal_tail_lm_head_forget() drops it).  Safe
 * to call from several host threads on disjoint ranges, as
 * qwen7b_server.c:833-845 does. */
void lal_lm_head_int8_range(float *logits, const int8_t *xq, float scale_x,
                            const int8_t *wte_q, const float *scale_w,
                            int v_start, int v_end, int n_embd);

/* runtime/lal_q8_kernel.h:506-543: same values; ax (= |xq|) is accepted for
 * signature compatibility, the GPU multiplies signed values directly. */
void lal_lm_head_int8_range_abs(float *logits, const int8_t *xq, const uint8_t *ax,
                                float scale_x, const int8_t *wte_q,
                                const float *scale_w, int v_start, int v_end,
                                int n_embd);

/* runtime/lal_q8_kernel.h:551-640: as the original, rows taken in full
 * groups of 8 from v_start sum only the first n_embd & ~31 columns (its
 * 8-row body has no scalar tail); the remaining rows sum all columns. */
void lal_lm_head_int8_range_abs_8row(float *logits, const int8_t *xq,
                                     const uint8_t *ax, float scale_x,
                                     const int8_t *wte_q, const float *scale_w,
                                     int v_start, int v_end, int n_embd);

/* runtime/lal_q8_kernel.h:357-372: per-row absmax int8 quantization with
 * lroundf (half away from zero). */
void lal_quantize_q8_per_row(const float *W, int8_t *q8_T, float *scale,
                             int in_dim, int out_dim);

#ifdef __cplusplus
}
#endif

#endif /* LAL_TAIL_DROPIN_Q8_KERNEL_H */
