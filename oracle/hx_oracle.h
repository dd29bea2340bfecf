/*
 * hx_oracle.h — CPU oracle for the hxinfer KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * engine's CPU algorithms (RoPE, the CPU attention loop, softmax, the prefix
 * cache hash).  Only the test suite, the smoke check and the CPU-baseline leg
 * of the benchmark load it, and only as the checker.  The product library
 * (hxinfer_b200/csrc) never links or calls it.
 *
 * Parity pin: every function here is compared bit-for-bit against the
 * reference built from its own sources (oracle/ref_driver.cpp +
 * oracle/Makefile -> oracle/_ref/libhxref.so) and against the committed
 * golden vectors in tests/golden/ that the reference produced.
 *
 * All arithmetic is fp32 in the reference's operation order; the library is
 * compiled without FMA contraction (-ffp-contract=off) so each product and
 * sum rounds the way the reference's x86-64 build rounds.
 */
#ifndef HX_ORACLE_H
#define HX_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* NeoX RoPE in place on `rows` rows of `row_dim` floats, `num_heads` heads of
 * `head_dim` each, all at position `step`.
 * Follows hxinfer-engine/src/op/cpu/rope_cpu.cpp:11-35. */
void orc_rope_neox(float* x, long rows, int row_dim, int num_heads, int head_dim,
                   int step, float base);

/* Same as orc_rope_neox but row r is rotated at position steps[r]
 * (a prompt rotated token by token, as the reference prefill loop does). */
void orc_rope_neox_rows(float* x, long rows, int row_dim, int num_heads, int head_dim,
                        const int* steps, float base);

/* YaRN per-frequency multipliers and attention factor.
 * Follows hxinfer-engine/src/op/cuda/rope_cuda.cu:9-35 (host helpers). */
void  orc_yarn_scale(float* out, int half_dim, int head_dim, float factor, float base,
                     float beta_fast, float beta_slow, int orig_max_pos);
float orc_yarn_attn_factor(float factor);

/* YaRN RoPE in place: the angle/cos/sin expressions of
 * hxinfer-engine/src/op/cuda/rope_cuda.cu:46-70 evaluated with host libm. */
void orc_rope_neox_yarn(float* x, long rows, int row_dim, int num_heads, int head_dim,
                        int step, float base, const float* yarn_scale, float attn_factor);

/* cos/sin table [max_pos][head_dim/2][2] holding exactly the cos_val/sin_val
 * that rope_cpu.cpp:22-25 (yarn_scale == NULL) or rope_cuda.cu:56-61
 * (yarn_scale != NULL) compute for every (position, frequency). */
void orc_rope_table(float* cos_sin, int max_pos, int head_dim, float base,
                    const float* yarn_scale, float attn_factor);

/* Safe softmax over n floats.  Follows hxinfer-engine/src/op/cpu/softmax_cpu.cpp:20-37. */
void orc_softmax(const float* in, float* out, long n);

/* One decode step of attention for one sequence.
 * q: [Hq*head_dim] (already rotated); k_cache/v_cache: token-major
 * [L][Hkv*head_dim] fp32; out: [Hq*head_dim].
 * Follows the CPU branch hxinfer-engine/src/layer/attention.cpp:51-85 line
 * for line, with the GQA head mapping kv = h / (Hq/Hkv) of
 * hxinfer-engine/src/op/cuda/attention_score_cuda.cu:20-21,175. */
void orc_decode_attention(const float* q, const float* k_cache, const float* v_cache,
                          int L, int Hq, int Hkv, int head_dim, float* out);

/* Causal attention of n query rows starting at absolute position `start`:
 * row i attends to positions [0, start+i].  Each row is the decode step above
 * (the reference prefills one token per forward call, bench_1024.cpp:62-70). */
void orc_prefill_attention(const float* q, const float* k_cache, const float* v_cache,
                           int start, int n, int Hq, int Hkv, int head_dim, float* out);

/* Many sequences of one layer, spread over `nthreads` POSIX threads by
 * (sequence, q head).  Each unit is computed by the same loop as
 * orc_decode_attention, so the result does not depend on nthreads.
 * k_caches[s]/v_caches[s]: token-major [lengths[s]][Hkv*head_dim];
 * q/out: [n_seqs][Hq*head_dim]. */
void orc_decode_attention_batch(const float* q, const float* const* k_caches,
                                const float* const* v_caches, const int* lengths, int n_seqs,
                                int Hq, int Hkv, int head_dim, float* out, int nthreads);

/* 64-bit FNV-1a over int token ids.
 * Follows hxinfer-engine/include/cache/prefix_cache.h:42-49. */
uint64_t orc_fnv1a64(const int* tokens, long n);

#ifdef __cplusplus
}
#endif
#endif /* HX_ORACLE_H */
