/*
 * c2s_oracle.h -- CPU restatement of the c2slm token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a implementation in c2slm_b200/.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs may load it.  The
 * product path never calls into it.
 *
 * Every function restates one scalar function of hazyhaar/c2slm (Go), in the
 * reference's statement order, with the file:line it follows.  The library is
 * compiled with -O2 -ffp-contract=off (no FMA contraction: Go on amd64 never
 * fuses a*b+c, so neither may the oracle).
 *
 * Deliberate deviations from the reference (each forced by the build):
 *   - Q8_K scratch is sized from cols (the reference's pool scratch holds
 *     16384 cols, engine/pool.go:59, and overflows on 18944-col ffn_down).
 *   - Q6_K token embeddings are dequantised (engine/model.go:221-247 has no
 *     Q6_K case); the dequant follows tensor/oracle_q6_k_test.go:62-94.
 *   - The repetition penalty factor and window are parameters
 *     (c2slm.go:157-170 hard-codes 1.15 over 64 positions).
 */
#ifndef C2S_ORACLE_H
#define C2S_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, gguf/reader.go:21-37 */
enum {
    C2O_F32 = 0, C2O_F16 = 1, C2O_Q5_0 = 6, C2O_Q8_0 = 8,
    C2O_Q4_K = 12, C2O_Q6_K = 14
};

/* block byte sizes, tensor/ops.go:11-22 */
enum {
    C2O_QK5_0 = 32, C2O_QK8_0 = 32, C2O_QK_K = 256,
    C2O_BS_Q5_0 = 22, C2O_BS_Q8_0 = 34, C2O_BS_Q4_K = 144,
    C2O_BS_Q6_K = 210, C2O_BS_Q8_K = 292
};

/* ---- scalar kernels ---------------------------------------------------- */
float c2o_fp16_to_f32(uint16_t h);
void  c2o_quantize_row_q8_k(const float *x, uint8_t *y, int cols);
float c2o_dot_q4_k_q8_k(const uint8_t *w, const uint8_t *q8k, int cols);
void  c2o_gemv2_q4_k_q8_k(const uint8_t *w0, const uint8_t *w1, const uint8_t *q8k,
                          int cols, float *out0, float *out1);
void  c2o_gemv2_q6_k_q8_k(const uint8_t *w0, const uint8_t *w1, const uint8_t *q8k,
                          int cols, float *out0, float *out1);
float c2o_dot_q5_0(const uint8_t *w, const float *x, int cols);
float c2o_dot_q8_0(const uint8_t *w, const float *x, int cols);
float c2o_dot_q4_k(const uint8_t *w, const float *x, int cols);
float c2o_dot_q6_k(const uint8_t *w, const float *x, int cols);

/* Integer partials of the K-quant x Q8_K dots, for bit-exact checks.
 * q4k: per row and superblock, 8 int32 sub-block dots (dot_lo, dot_hi for
 *      j = 0..3) -> dots[(r*nsb + sb)*8 + 2j + {0,1}]; and the 4 bsum pairs
 *      of the activation -> bsum_pairs[sb*4 + j] (row independent).
 * q6k: per row and superblock, the int32 isum -> isum[r*nsb + sb].        */
void  c2o_q4k_q8k_partials(const uint8_t *w, const uint8_t *q8k, int rows, int cols,
                           int32_t *dots, int32_t *bsum_pairs);
void  c2o_q6k_q8k_partials(const uint8_t *w, const uint8_t *q8k, int rows, int cols,
                           int32_t *isum);

/* Row matvec with the WorkerPool's dispatch semantics (engine/pool.go:122-154):
 * K-quants quantise x to Q8_K first; Q5_0/Q8_0 use f32 x. q8k_scratch must
 * hold (cols/256)*292 bytes (may be NULL for Q5_0/Q8_0). nthreads <= 1 runs
 * serially; the result does not depend on nthreads.                       */
int   c2o_gemv(int type, const uint8_t *w, const float *x, float *y, int rows, int cols,
               uint8_t *q8k_scratch, int nthreads);
/* f32-x dots over rows (the pool-less DispatchGEMV, engine/model.go:255-269) */
int   c2o_gemv_f32x(int type, const uint8_t *w, const float *x, float *y, int rows, int cols);

int   c2o_dequant_row(int type, const uint8_t *row, float *out, int cols);
void  c2o_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
void  c2o_add_bias(float *x, const float *bias, int n);
void  c2o_rope_table(float *cos_t, float *sin_t, int max_len, int head_dim, float theta);
void  c2o_rope_apply(const float *cos_t, const float *sin_t, int max_len, int head_dim,
                     float *vec, int vec_len, int num_heads, int pos);
void  c2o_rope_neox(float *vec, int num_heads, int head_dim, int pos, float theta);
void  c2o_softmax(float *x, int n);
void  c2o_swiglu(float *out, const float *gate, const float *up, int n);
void  c2o_attn_qk(const float *q, const float *kbase, int pos, int stride, float scale,
                  float *scores, int hd);
void  c2o_attn_av(const float *scores, const float *vbase, int pos, int stride,
                  float *out, int hd);

/* The reference's AVX2 build (GOEXPERIMENT=simd): the kernels whose float
 * order differs from the scalar twins on the Q5_0/Q4_K/Q6_K/Q8_0 path. */
void  c2o_attn_qk_simd(const float *q, const float *kbase, int pos, int stride, float scale,
                       float *scores, int hd);
void  c2o_attn_av_simd(const float *scores, const float *vbase, int pos, int stride,
                       float *out, int hd);
void  c2o_swiglu_simd(float *out, const float *gate, const float *up, int n);

/* ---- model ------------------------------------------------------------- */
typedef struct c2o_model c2o_model;

typedef struct {
    int32_t embd, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float   rope_base, eps;
    int32_t max_tokens;
    int32_t im_end, eos;          /* tokenizer/bpe.go:284-289 (0 when absent) */
    int32_t tied_output;
} c2o_model_info;

/* engine.LoadModel + NewKVCache + NewArena (engine/model.go:58-210,
 * engine/kvcache.go:49, engine/forward.go:28).  Returns NULL on error and
 * writes the reason to err (if non-NULL, errlen bytes).                     */
c2o_model *c2o_model_open(const char *path, int max_tokens, int nthreads,
                          char *err, int errlen);
void  c2o_model_close(c2o_model *m);
void  c2o_model_get_info(const c2o_model *m, c2o_model_info *info);
/* 1: evaluate attention and SwiGLU in the AVX2 build's order (default 0). */
void  c2o_model_set_simd_order(c2o_model *m, int on);

/* engine.Forward (engine/forward.go:54-138); writes NormX (embd floats). */
void  c2o_forward(c2o_model *m, int32_t token, int pos, float *normx_out);
/* engine.ComputeLogits (engine/forward.go:171-191). n_targets == 0 -> full. */
void  c2o_compute_logits(c2o_model *m, const float *normx, float *out,
                         const int32_t *targets, int n_targets);
/* penalty + greedy argmax of c2slm.go:156-180 over logits (modified in place) */
int32_t c2o_select(c2o_model *m, float *logits, int cur_pos, float penalty, int window);

/* KVCache semantics (engine/kvcache.go:101-125) */
int   c2o_kv_seq_len(const c2o_model *m);
void  c2o_kv_set_seq_len(c2o_model *m, int n);
void  c2o_kv_reset(c2o_model *m);
void  c2o_kv_rewind(c2o_model *m, int n);
void  c2o_kv_store_token_id(c2o_model *m, int pos, int32_t tok);
int32_t c2o_kv_token_id(const c2o_model *m, int pos);
/* copies [layer][kv_head][pos][0..hd) of K (is_v=0) or V (is_v=1) */
void  c2o_kv_get(const c2o_model *m, int is_v, int layer, int kv_head, int pos, float *out);

/* c2slm.Engine.IngestFrom (c2slm.go:92-115). Returns number of positions
 * forwarded; last NormX in normx_out if non-NULL and at least one forwarded. */
int   c2o_ingest_from(c2o_model *m, int pos, const int32_t *tokens, int n, float *normx_out);

/* c2slm.Engine.generate (c2slm.go:144-223) on token ids, without the
 * tokenizer: no stop strings, no callback. Starts from the NormX of the last
 * forward. tokens_out receives every selected id (the stop id included);
 * margins_out (optional) receives top1-top2 of the penalised logits and
 * maxabs_out (optional) max |logit|, per step.  Returns the count.        */
int   c2o_generate(c2o_model *m, const float *last_normx, int max_new, float penalty,
                   int window, int stop_on_special, int32_t *tokens_out,
                   float *margins_out, float *maxabs_out);

#ifdef __cplusplus
}
#endif
#endif
