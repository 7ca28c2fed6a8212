/*
 * gen_expf_fixups.c -- build-time generator of the expf fix-up table.
 *
 * For every non-positive float x (bit patterns 0x80000000..0xFF800000, i.e.
 * -0 down to -inf), compares the host glibc expf(x) with lal_expf_rounded(x)
 * (lal_expf.h) and writes the inputs where they differ, with glibc's result,
 * as two little-endian uint32 arrays: [n][x_bits ascending...][y_bits...].
 * The device applies these fix-ups, so its weights equal glibc's exactly.
 *
 * Usage: gen_expf_fixups <out.bin> [threads]
 * Build: gcc -O2 -ffp-contract=off -fopenmp gen_expf_fixups.c -lm
 */
#include "lal_expf.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

int main(int argc, char **argv) {
    if (argc < 2) { fprintf(stderr, "usage: %s out.bin [threads]\n", argv[0]); return 2; }
    int nthreads = argc > 2 ? atoi(argv[2]) : omp_get_max_threads();
    const uint64_t lo = 0x80000000ull, hi = 0xFF800000ull;
    const int nchunks = 4096;
    const uint64_t span = (hi - lo + 1 + nchunks - 1) / nchunks;
    uint32_t **cx = calloc(nchunks, sizeof(uint32_t *));
    uint32_t **cy = calloc(nchunks, sizeof(uint32_t *));
    int *cn = calloc(nchunks, sizeof(int));
    #pragma omp parallel for schedule(dynamic, 8) num_threads(nthreads)
    for (int c = 0; c < nchunks; c++) {
        uint64_t a = lo + (uint64_t)c * span, b = a + span;
        if (b > hi + 1) b = hi + 1;
        int cap = 64, n = 0;
        uint32_t *xs = malloc(cap * 4), *ys = malloc(cap * 4);
        for (uint64_t u = a; u < b; u++) {
            float x = lal_u2f((uint32_t)u);
            float g = expf(x);
            float m = lal_expf_rounded(x);
            if (lal_f2u(g) != lal_f2u(m)) {
                if (n == cap) { cap *= 2; xs = realloc(xs, cap * 4); ys = realloc(ys, cap * 4); }
                xs[n] = (uint32_t)u; ys[n] = lal_f2u(g); n++;
            }
        }
        cx[c] = xs; cy[c] = ys; cn[c] = n;
    }
    uint32_t total = 0;
    for (int c = 0; c < nchunks; c++) total += (uint32_t)cn[c];
    FILE *f = fopen(argv[1], "wb");
    if (!f) { perror(argv[1]); return 1; }
    fwrite(&total, 4, 1, f);
    for (int c = 0; c < nchunks; c++) fwrite(cx[c], 4, (size_t)cn[c], f);
    for (int c = 0; c < nchunks; c++) fwrite(cy[c], 4, (size_t)cn[c], f);
    fclose(f);
    fprintf(stderr, "expf fix-ups: %u entries\n", total);
    return 0;
}
