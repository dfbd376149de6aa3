/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle. Never linked into, loaded by, or
 * called from the product library; only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg use it, as the checker.
 *
 * Plain-C restatement of the reference arithmetic on the token loop:
 *   FP16 codec .................. src/reference/kv_reference.cpp:31-134
 *   contiguous attention ........ src/reference/kv_reference.cpp:136-234
 *   paged gather ................ src/cuda/kv/page_kernels.cu:184-242
 *   FP16-rounding decoder ....... tests/cuda/cuda_model_runner_test.cpp:213-420
 *                                 (the reference's own model oracle)
 *   greedy argmax ............... src/cuda/model/kernels.cu:220-293
 * Pinned against the reference itself (oracle/_ref) and its known answers by
 * tests/test_oracle_pinned.py.
 */
#ifndef KK_ORACLE_H
#define KK_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t kko_f2h(float value);
float kko_h2f(uint16_t value);

/* Contiguous [layer][K/V][token][head][dim] FP16 KV, FP32 query/output
 * [layer][head][dim]; one query per KV head. Returns 1 on success. */
int kko_reference_attention(uint32_t layers, uint32_t heads, uint32_t dim, const uint16_t* kv,
    uint32_t tokens, const float* query, float* output);

/* One lane of GQA paged decode attention for one layer: gathers the lane's
 * tokens from the micro / extent pools through its entries (slot, begin,
 * valid, kind), runs the attention above per query head on its KV head, and
 * rounds the output to FP16. q/out: [q_heads][dim]. Returns 1 on success. */
int kko_paged_attention(const uint16_t* micro, const uint16_t* extent, uint32_t layers,
    uint32_t kv_heads, uint32_t dim, uint32_t layer, uint32_t q_heads, const uint32_t* entry_slot,
    const uint32_t* entry_valid, const uint8_t* entry_kind, uint32_t entries, const uint16_t* q,
    uint16_t* out);

/* ---- TinyLlama-shaped FP16 decoder -------------------------------------- */
typedef struct kko_config {
    uint32_t hidden, intermediate, layers, q_heads, kv_heads, head_dim, vocab, max_positions;
    float eps, theta;
} kko_config;

/* weights: FP16 tensors in this order: embed [V][H], lm_head [V][H], final_norm [H],
 * then per layer: input_norm [H], post_norm [H], q [H][H], k [KV][H], v [KV][H],
 * o [H][H], gate [I][H], up [I][H], down [H][I]. Copied (widened) at create. */
void* kko_model_create(const kko_config* config, const uint16_t* const* weights, uint32_t threads);
void kko_model_destroy(void* model);
/* Sequences own their KV (FP16-valued, kept as FP32). */
int kko_seq_create(void* model, uint64_t seq);
int kko_seq_fork(void* model, uint64_t source, uint64_t child);
int kko_seq_release(void* model, uint64_t seq);
uint32_t kko_seq_length(void* model, uint64_t seq);
/* Appends n tokens of given K/V (FP16, [n][layers][kv_heads*dim] each). */
int kko_seq_append_kv(void* model, uint64_t seq, uint32_t n, const uint16_t* k, const uint16_t* v);
/* One position per listed sequence (its current length must equal positions[i]).
 * logits: [n][V] FP32 (may be NULL); final_hidden: [n][H] FP16 (may be NULL);
 * tokens: [n] greedy ids. Returns 1 on success. */
int kko_forward_batch(void* model, uint32_t n, const uint64_t* seqs, const uint32_t* token_ids,
    const uint32_t* positions, float* logits, uint16_t* final_hidden, uint32_t* tokens);

/* 1: projections sum in double precision and round once (a second,
 * equally valid summation order of the same arithmetic), to measure the
 * model's sensitivity to summation order; 0: the reference's order. */
void kko_model_set_wide_sums(void* model, int wide);

/* First maximum (ties -> lowest index). */
uint32_t kko_argmax(const float* values, uint32_t count);

#ifdef __cplusplus
}
#endif

#endif
