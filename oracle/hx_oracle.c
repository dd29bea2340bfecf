/*
 * hx_oracle.c — CPU oracle for the hxinfer KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker, never the thing measured or shipped.
 * See hx_oracle.h for the contract.  Build: oracle/Makefile (gcc -O2
 * -std=c11 -ffp-contract=off, no -ffast-math, no -march), matching the
 * reference's own host build, which has no FMA contraction on x86-64.
 */
#include "hx_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* rope_cpu.cpp:20-33: per row, per head, per frequency d < head_dim/2. */
static void rope_one_head(float* p, int head_dim, int step, float base)
{
    int half_dim = head_dim / 2;
    for (int d = 0; d < half_dim; d++) {
        float scale   = 1.0f / powf(base, (float)(2 * d) / head_dim);
        float angle   = step * scale;
        float cos_val = cosf(angle);
        float sin_val = sinf(angle);
        float v1 = p[d];
        float v2 = p[d + half_dim];
        p[d]            = v1 * cos_val - v2 * sin_val;
        p[d + half_dim] = v2 * cos_val + v1 * sin_val;
    }
}

void orc_rope_neox(float* x, long rows, int row_dim, int num_heads, int head_dim,
                   int step, float base)
{
    for (long i = 0; i < rows; i++)
        for (int j = 0; j < num_heads; j++)
            rope_one_head(x + i * row_dim + (long)j * head_dim, head_dim, step, base);
}

void orc_rope_neox_rows(float* x, long rows, int row_dim, int num_heads, int head_dim,
                        const int* steps, float base)
{
    for (long i = 0; i < rows; i++)
        for (int j = 0; j < num_heads; j++)
            rope_one_head(x + i * row_dim + (long)j * head_dim, head_dim, steps[i], base);
}

/* rope_cuda.cu:9-11.  M_PI is a double there, so the quotient is formed in
 * double precision and converted to float by logf's parameter. */
static float find_correction_dim(int num_rotations, int dim, float base, int max_pos)
{
    const double pi = 3.14159265358979323846;
    double q = max_pos / ((double)(num_rotations * 2.0f) * pi);
    return (dim * logf((float)q)) / (2.0f * logf(base));
}

/* rope_cuda.cu:13-30 */
void orc_yarn_scale(float* out, int half_dim, int head_dim, float factor, float base,
                    float beta_fast, float beta_slow, int orig_max_pos)
{
    float low  = find_correction_dim((int)beta_fast, head_dim, base, orig_max_pos);
    float high = find_correction_dim((int)beta_slow, head_dim, base, orig_max_pos);
    low  = fmaxf(low, 0.0f);
    high = fminf(high, (float)(half_dim - 1));
    float span = high - low;
    if (span <= 0.0f) span = 1.0f;
    for (int d = 0; d < half_dim; d++) {
        float ramp = (float)d - low;
        ramp = ramp / span;
        ramp = fmaxf(0.0f, fminf(1.0f, ramp));
        out[d] = 1.0f - ramp * (1.0f - 1.0f / factor);
    }
}

/* rope_cuda.cu:32-35 */
float orc_yarn_attn_factor(float factor)
{
    if (factor <= 1.0f) return 1.0f;
    return 0.1f * logf(factor) + 1.0f;
}

/* rope_cuda.cu:56-68 with host libm */
static void rope_one_head_yarn(float* p, int head_dim, int step, float base,
                               const float* yarn_scale, float attn_factor)
{
    int half_dim = head_dim / 2;
    for (int d = 0; d < half_dim; d++) {
        float scale = 1.0f / powf(base, (float)(2 * d) / head_dim);
        if (yarn_scale) scale *= yarn_scale[d];
        float angle   = step * scale;
        float cos_val = cosf(angle) * attn_factor;
        float sin_val = sinf(angle) * attn_factor;
        float v1 = p[d];
        float v2 = p[d + half_dim];
        p[d]            = v1 * cos_val - v2 * sin_val;
        p[d + half_dim] = v2 * cos_val + v1 * sin_val;
    }
}

void orc_rope_neox_yarn(float* x, long rows, int row_dim, int num_heads, int head_dim,
                        int step, float base, const float* yarn_scale, float attn_factor)
{
    for (long i = 0; i < rows; i++)
        for (int j = 0; j < num_heads; j++)
            rope_one_head_yarn(x + i * row_dim + (long)j * head_dim, head_dim, step, base,
                               yarn_scale, attn_factor);
}

void orc_rope_table(float* cos_sin, int max_pos, int head_dim, float base,
                    const float* yarn_scale, float attn_factor)
{
    int half_dim = head_dim / 2;
    for (int pos = 0; pos < max_pos; pos++) {
        for (int d = 0; d < half_dim; d++) {
            float scale = 1.0f / powf(base, (float)(2 * d) / head_dim);
            float c, s;
            if (yarn_scale) {
                scale *= yarn_scale[d];
                float angle = pos * scale;
                c = cosf(angle) * attn_factor;
                s = sinf(angle) * attn_factor;
            } else {
                float angle = pos * scale;
                c = cosf(angle);
                s = sinf(angle);
            }
            cos_sin[((long)pos * half_dim + d) * 2 + 0] = c;
            cos_sin[((long)pos * half_dim + d) * 2 + 1] = s;
        }
    }
}

/* softmax_cpu.cpp:20-37 */
void orc_softmax(const float* in, float* out, long n)
{
    float max_val = -3.402823466e+38f; /* numeric_limits<float>::lowest() */
    for (long i = 0; i < n; i++)
        if (in[i] > max_val) max_val = in[i];
    float sum = 0;
    for (long i = 0; i < n; i++) {
        float e = expf(in[i] - max_val);
        sum = sum + e;
        out[i] = e;
    }
    for (long i = 0; i < n; i++) out[i] = out[i] / sum;
}

/* attention.cpp:52-85 for one q head; kv head from attention_score_cuda.cu:21. */
static void attend_one_head(const float* q, const float* k_cache, const float* v_cache,
                            int L, int kv_dim, int kv_off, int head_dim, float scale,
                            float* scores, float* out)
{
    for (int j = 0; j < L; j++) {
        const float* k = k_cache + (long)j * kv_dim + kv_off;
        float sum = 0;
        for (int sc = 0; sc < head_dim; sc++) sum = sum + q[sc] * k[sc];
        scores[j] = sum * scale;
    }
    float max_score = scores[0];
    for (int d = 1; d < L; d++)
        if (scores[d] > max_score) max_score = scores[d];
    float sum = 0;
    for (int d = 0; d < L; d++) {
        scores[d] = expf(scores[d] - max_score);
        sum = sum + scores[d];
    }
    for (int d = 0; d < L; d++) scores[d] = scores[d] / sum;
    for (int j = 0; j < head_dim; j++) {
        float acc = 0;
        for (int k = 0; k < L; k++) acc = acc + scores[k] * v_cache[(long)k * kv_dim + kv_off + j];
        out[j] = acc;
    }
}

/* attention.cpp:52: float scale = 1.0/std::sqrt(head_dim) (double math, then float). */
static float attn_scale(int head_dim) { return (float)(1.0 / sqrt((double)head_dim)); }

void orc_decode_attention(const float* q, const float* k_cache, const float* v_cache,
                          int L, int Hq, int Hkv, int head_dim, float* out)
{
    int group = Hq / Hkv;
    int kv_dim = Hkv * head_dim;
    float scale = attn_scale(head_dim);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
    for (int i = 0; i < Hq; i++) {
        int kv = i / group;
        attend_one_head(q + (long)i * head_dim, k_cache, v_cache, L, kv_dim, kv * head_dim,
                        head_dim, scale, scores, out + (long)i * head_dim);
    }
    free(scores);
}

void orc_prefill_attention(const float* q, const float* k_cache, const float* v_cache,
                           int start, int n, int Hq, int Hkv, int head_dim, float* out)
{
    long row = (long)Hq * head_dim;
    for (int i = 0; i < n; i++)
        orc_decode_attention(q + i * row, k_cache, v_cache, start + i + 1, Hq, Hkv, head_dim,
                             out + i * row);
}

struct batch_job {
    const float* q;
    const float* const* k_caches;
    const float* const* v_caches;
    const int* lengths;
    int n_seqs, Hq, Hkv, head_dim;
    float* out;
    int tid, nthreads;
};

static void* batch_worker(void* arg)
{
    struct batch_job* j = (struct batch_job*)arg;
    int group = j->Hq / j->Hkv;
    int kv_dim = j->Hkv * j->head_dim;
    float scale = attn_scale(j->head_dim);
    int maxL = 1;
    for (int s = 0; s < j->n_seqs; s++)
        if (j->lengths[s] > maxL) maxL = j->lengths[s];
    float* scores = (float*)malloc(sizeof(float) * (size_t)maxL);
    long units = (long)j->n_seqs * j->Hq;
    for (long u = j->tid; u < units; u += j->nthreads) {
        int s = (int)(u / j->Hq), h = (int)(u % j->Hq);
        long off = ((long)s * j->Hq + h) * j->head_dim;
        attend_one_head(j->q + off, j->k_caches[s], j->v_caches[s], j->lengths[s], kv_dim,
                        (h / group) * j->head_dim, j->head_dim, scale, scores, j->out + off);
    }
    free(scores);
    return NULL;
}

void orc_decode_attention_batch(const float* q, const float* const* k_caches,
                                const float* const* v_caches, const int* lengths, int n_seqs,
                                int Hq, int Hkv, int head_dim, float* out, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    struct batch_job* jobs = (struct batch_job*)malloc(sizeof(struct batch_job) * (size_t)nthreads);
    for (int t = 0; t < nthreads; t++) {
        struct batch_job j = {q, k_caches, v_caches, lengths, n_seqs, Hq, Hkv, head_dim, out, t, nthreads};
        jobs[t] = j;
        pthread_create(&th[t], NULL, batch_worker, &jobs[t]);
    }
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    free(jobs);
    free(th);
}

/* prefix_cache.h:42-49: size_t hash; hash ^= static_cast<size_t>(tok); hash *= prime. */
uint64_t orc_fnv1a64(const int* tokens, long n)
{
    uint64_t hash = 0xcbf29ce484222325ULL;
    for (long i = 0; i < n; i++) {
        hash ^= (uint64_t)(int64_t)tokens[i];
        hash *= 0x100000001b3ULL;
    }
    return hash;
}
