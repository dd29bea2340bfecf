/* oracle_sanitize.c — every function of the CPU oracle (oracle/hx_oracle.c)
 * called on exactly sized heap buffers over edge-case shapes, built with gcc
 * under AddressSanitizer and UndefinedBehaviorSanitizer (tests/cpp/Makefile,
 * target oracle_sanitize; run by tests/test_oracle_sanitize.py).  The parity
 * claims rest on the oracle, so it must not read or write out of bounds or
 * hit undefined behaviour on any shape the tests give it.  Prints "ok" and
 * exits 0 unless a sanitizer stops the process. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "hx_oracle.h"

/* values in [-2, 2] from a 32-bit linear congruential generator */
static float* randv(size_t n, unsigned* seed)
{
    float* v = (float*)malloc((n ? n : 1) * sizeof(float));
    for (size_t i = 0; i < n; ++i) {
        *seed = *seed * 1664525u + 1013904223u;
        v[i] = (float)((int)((*seed >> 8) % 2001u) - 1000) / 500.0f;
    }
    return v;
}

int main(void)
{
    unsigned seed = 20261202u;
    const int hds[] = {2, 64, 128};
    const int heads[][2] = {{1, 1}, {4, 4}, {4, 2}, {28, 4}, {32, 8}};
    const int lens[] = {1, 2, 63, 64, 65, 300};
    for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 5; ++b) {
            const int hd = hds[a], hq = heads[b][0], hkv = heads[b][1];
            const int qd = hq * hd, kd = hkv * hd;
            /* RoPE: scalar step, per-row steps, YaRN, the table */
            for (int rows = 1; rows <= 3; ++rows) {
                float* x = randv((size_t)rows * qd, &seed);
                orc_rope_neox(x, rows, qd, hq, hd, 1023 * rows, 1e6f);
                int* steps = (int*)malloc(rows * sizeof(int));
                for (int r = 0; r < rows; ++r) steps[r] = r * 4095;
                orc_rope_neox_rows(x, rows, qd, hq, hd, steps, 1e4f);
                float* ys = (float*)malloc((hd / 2) * sizeof(float));
                orc_yarn_scale(ys, hd / 2, hd, 4.0f, 1e6f, 32.0f, 1.0f, 32768);
                orc_rope_neox_yarn(x, rows, qd, hq, hd, 40000, 1e6f, ys, orc_yarn_attn_factor(4.0f));
                float* tab = (float*)malloc((size_t)17 * (hd / 2) * 2 * sizeof(float));
                orc_rope_table(tab, 17, hd, 1e4f, NULL, 1.0f);
                orc_rope_table(tab, 17, hd, 1e6f, ys, orc_yarn_attn_factor(4.0f));
                free(tab);
                free(ys);
                free(steps);
                free(x);
            }
            /* attention: one sequence, prefill rows, a batch over threads */
            for (int c = 0; c < 6; ++c) {
                const int L = lens[c];
                float* q = randv(qd, &seed);
                float* k = randv((size_t)L * kd, &seed);
                float* v = randv((size_t)L * kd, &seed);
                float* out = (float*)malloc(qd * sizeof(float));
                orc_decode_attention(q, k, v, L, hq, hkv, hd, out);
                const int start = L / 2, n = L - start;
                float* qs = randv((size_t)n * qd, &seed);
                float* outs = (float*)malloc((size_t)n * qd * sizeof(float));
                orc_prefill_attention(qs, k, v, start, n, hq, hkv, hd, outs);
                const float* ks[2] = {k, k};
                const float* vs[2] = {v, v};
                const int ls[2] = {L, L > 1 ? L - 1 : 1};
                float* q2 = randv((size_t)2 * qd, &seed);
                float* o2 = (float*)malloc((size_t)2 * qd * sizeof(float));
                orc_decode_attention_batch(q2, ks, vs, ls, 2, hq, hkv, hd, o2, 3);
                free(o2);
                free(q2);
                free(outs);
                free(qs);
                free(out);
                free(v);
                free(k);
                free(q);
            }
        }
    for (long n = 1; n <= 1025; n += 256) {
        float* in = randv(n, &seed);
        float* out = (float*)malloc(n * sizeof(float));
        orc_softmax(in, out, n);
        free(out);
        free(in);
    }
    int toks[5] = {0, -1, 152063, 7, 2147483647};
    printf("ok %llu %llu\n", (unsigned long long)orc_fnv1a64(toks, 0),
           (unsigned long long)orc_fnv1a64(toks, 5));
    return 0;
}
