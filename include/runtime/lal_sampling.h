/*
 * Drop-in for runtime/lal_sampling.h of samaidev/lal.
 *
 * With this repository's include/ ahead of the LAL checkout on the include
 * path, a server's  #include "runtime/lal_sampling.h"  resolves here.  The
 * sampler and the recent-token ring come from liblal_tail.so with the same
 * names and signatures (lal_sampling.h:46 lal_sample_token, :128
 * LalRecentTokens, :133 lal_recent_push); lal_sample_token runs on the GPU,
 * mutates logits in place like the original and calls rand() once on its
 * non-greedy path, as lal_sampling.h:116 does.  The defaults and the seeding
 * helper are kept as the original declares them (:26-32).
 *
 * Link with -llal_tail.
 */
#ifndef LAL_SAMPLING_H
#define LAL_SAMPLING_H

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../lal_tail.h"

#ifdef __cplusplus
extern "C" {
#endif

/* runtime/lal_sampling.h:46-125: repetition penalty (in place), min-heap
 * top-k threshold, softmax with temperature over {v : logits[v] >= k-th
 * largest}, one rand() draw, ascending-index inverse CDF. */
int lal_sample_token(float *logits, int vocab_size, float temperature, int top_k,
                     float rep_penalty, const int *recent, int n_recent);

/* runtime/lal_sampling.h:127-131 */
typedef struct {
    int tokens[256];
    int n;
} LalRecentTokens;

/* runtime/lal_sampling.h:133-136: FIFO of the last 256 ids. */
void lal_recent_push(LalRecentTokens *rt, int tok);

#ifdef __cplusplus
}
#endif

#ifndef LAL_TAIL_BUILDING
/* lal_sampling.h:26-28, unchanged (including the int-typed temperature). */
static int   lal_g_temperature = 0.8f;
static int   lal_g_top_k = 40;
static float lal_g_rep_penalty = 1.1f;

/* lal_sampling.h:30-32 */
static void lal_sampling_init(void) {
    srand((unsigned)time(NULL));
}
#endif /* LAL_TAIL_BUILDING */

#endif /* LAL_SAMPLING_H */
