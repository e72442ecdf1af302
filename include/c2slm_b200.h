/*
 * c2slm_b200.h -- C ABI of the B200 (sm_100a) token loop for hazyhaar/c2slm.
 *
 * The reference is pure Go.  Its token loop is engine.Forward ->
 * engine.ComputeLogits -> repetition penalty -> greedy argmax, driven by
 * c2slm.Engine (c2slm.go).  This library replaces that path behind plain C
 * types (no CUDA or torch types in any signature) so the Go packages can bind
 * it through cgo.
 *
 * Conventions
 *   - Every call returns C2S_OK (0) or a negative c2s_status; the reason is
 *     available from c2s_last_error() (thread-local string).
 *   - Buffers passed as `host` pointers are caller-owned host memory.  The
 *     engine copies model tensors to device memory at creation and keeps no
 *     host pointer afterwards.
 *   - One c2s_engine is one sequence on one GPU with one CUDA stream; it is
 *     not thread-safe (like c2slm.Engine, whose Arena.Pool is shared state).
 *     Data parallel serving = one engine per GPU.
 */
#ifndef C2SLM_B200_H
#define C2SLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    C2S_OK = 0,
    C2S_ERR_ARG = -1,         /* invalid argument (rejected on the host before any launch) */
    C2S_ERR_CUDA = -2,        /* a CUDA runtime call failed */
    C2S_ERR_FORMAT = -3,      /* malformed or unsupported GGUF / tensor */
    C2S_ERR_UNSUPPORTED = -4, /* quantisation type or shape this build does not handle */
    C2S_ERR_TIMEOUT = -5,     /* a bounded device-side wait gave up (status read back) */
    C2S_ERR_STATE = -6,       /* call not valid in the engine's current state */
    C2S_ERR_OOM = -7          /* device allocation failed */
} c2s_status;

/* GGML type ids (gguf/reader.go:21-37) accepted by the kernels */
enum { C2S_F32 = 0, C2S_Q5_0 = 6, C2S_Q8_0 = 8, C2S_Q4_K = 12, C2S_Q6_K = 14 };

/* Thread-local description of the last failure in this thread. */
const char *c2s_last_error(void);
/* Library version string, e.g. "c2slm_b200 0.1 sm_100a". */
const char *c2s_version(void);

/* ------------------------------------------------------------------------ */
/* Engine (c2slm.Engine / engine.Model + KVCache + Arena)                    */
/* ------------------------------------------------------------------------ */
typedef struct c2s_engine c2s_engine;

/* Hyper-parameters as engine.LoadModel derives them (engine/model.go:64-148). */
typedef struct {
    int32_t embd, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
    float rope_base, eps;
    int32_t max_tokens;   /* KV capacity (KVCache.MaxTokens) */
    int32_t im_end, eos;  /* special ids (tokenizer/bpe.go:284-289) */
} c2s_model_desc;

/* One GGUF tensor as gguf.TensorInfo exposes it (gguf/reader.go:90-96):
 * dims[0] = ne0 = columns, dims[1] = rows; data = TensorInfo.Data. */
typedef struct {
    const char *name;
    int32_t type;
    int32_t n_dims;
    int64_t dims[4];
    const void *data;     /* host pointer (e.g. the Go mmap slice) */
    uint64_t nbytes;
} c2s_tensor_desc;

/* c2slm.NewEngine minus the tokenizer (c2slm.go:20-41): engine.LoadModel
 * (engine/model.go:58) + NewKVCache (engine/kvcache.go:49) + NewArena
 * (engine/forward.go:28).  Maps the GGUF file, uploads every tensor to HBM in
 * its native block layout and captures the decode-step CUDA graphs.
 * max_tokens <= 0 selects engine.MaxContextLen (16384). */
int c2s_engine_open(const char *gguf_path, int device, int max_tokens, c2s_engine **out);

/* Same, from tensors the caller has already mapped (the cgo path: Go keeps its
 * gguf.File and passes TensorInfo.Data slices).  desc->head_dim, ->vocab,
 * ->im_end, ->eos may be 0 to derive them as LoadModel does. */
int c2s_engine_create(const c2s_model_desc *desc, const c2s_tensor_desc *tensors,
                      int n_tensors, int device, c2s_engine **out);

/* Tensor parallel over `world` GPUs of one node (one process or thread per
 * GPU), the sharding of the 7B-shaped config: rank r holds query heads
 * [h0, h1) (whole 256-column superblocks of attn_output's input: pairs of
 * heads at head_dim 128) with the kv heads they use, FFN rows [f0, f1) in
 * superblocks, and vocabulary rows [v0, v1) of an even split padded to vpad
 * rows.  attn_output and ffn_down run on the rank's columns and are summed
 * by an NCCL allreduce before the residual add; the logits are all-gathered
 * and every rank applies the same penalty and argmax, so all ranks select
 * the same ids.  Every rank must make the same sequence of calls (forward,
 * ingest, generate, decode_step, compute_logits, bench) with the same
 * arguments.  No counterpart in the reference (CPU only). */
#define C2S_NCCL_ID_BYTES 128
/* An NCCL unique id (C2S_NCCL_ID_BYTES bytes) for rank 0 to share with the
 * other ranks. */
int c2s_nccl_unique_id(uint8_t *id_out);
/* The shard of `rank`: plan_out[9] = {h0, h1, g0, g1, f0, f1, v0, v1, vpad}
 * (f in superblocks of 256 rows).  head_dim 0 and vocab are derived as for
 * c2s_engine_create. */
int c2s_tp_plan(const c2s_model_desc *desc, int rank, int world, int32_t *plan_out);
int c2s_engine_create_tp(const c2s_model_desc *desc, const c2s_tensor_desc *tensors, int n_tensors,
                         int device, int rank, int world, const uint8_t *nccl_id, c2s_engine **out);
int c2s_engine_open_tp(const char *gguf_path, int device, int max_tokens, int rank, int world,
                       const uint8_t *nccl_id, c2s_engine **out);

/* Engine.Close (c2slm.go:44-55).  NULL is accepted. */
void c2s_engine_close(c2s_engine *e);

int c2s_engine_desc(const c2s_engine *e, c2s_model_desc *out);

/* engine.Forward(m, cache, a, tokenID, pos) (engine/forward.go:54): one decoder
 * step; K/V for `pos` are written to the device KV cache.  normx_out (host,
 * embd floats) receives the final NormX when non-NULL.  Like the reference,
 * Forward does not touch SeqLen or TokenIDs.  pos must be in [0, max_tokens). */
int c2s_forward(c2s_engine *e, int32_t token, int32_t pos, float *normx_out);

/* engine.ComputeLogits(m, a, normX, out, targets) (engine/forward.go:171).
 * normx_in: host NormX to project, or NULL for the NormX of the last Forward.
 * targets == NULL / n_targets == 0: full vocabulary into logits_out (vocab
 * floats).  Otherwise only logits_out[targets[i]] are written (restricted
 * projection with f32-activation dots, engine/forward.go:174-182,193-212). */
int c2s_compute_logits(c2s_engine *e, const float *normx_in, const int32_t *targets,
                       int n_targets, float *logits_out);

/* KVCache state (engine/kvcache.go:101-125).  SeqLen and TokenIDs live on the
 * device next to K/V; these calls read and write them. */
int c2s_kv_seq_len(const c2s_engine *e);
int c2s_kv_set_seq_len(c2s_engine *e, int seq_len);
int c2s_kv_reset(c2s_engine *e);                      /* KVCache.Reset */
int c2s_kv_rewind(c2s_engine *e, int n);              /* KVCache.Rewind */
int c2s_kv_store_token_id(c2s_engine *e, int pos, int32_t token);  /* StoreTokenID */
int c2s_kv_token_ids(const c2s_engine *e, int32_t *out, int n);    /* TokenIDs[0:n] */
/* KVCache.GetKey / GetValue (engine/kvcache.go:161-169): head_dim floats. */
int c2s_kv_get(const c2s_engine *e, int is_value, int layer, int kv_head, int pos, float *out);

/* Test surface, no counterpart in the reference: buffers of the last layer of
 * the last tensor-core prefill chunk, [tokens][query heads held x head_dim]
 * floats, the first n_floats -- which = 0: the causal attention output
 * (before attn_output), 1: the rotated queries it attended with. */
int c2s_prefill_debug(const c2s_engine *e, int which, float *out, int n_floats);

/* c2slm.Engine.IngestFrom(pos, tokens) (c2slm.go:92-115): clamps pos to
 * [0, SeqLen], rewinds, forwards each token and records it.  Returns the
 * number of tokens forwarded (>= 0) or a negative status; last_normx_out
 * (host, embd floats, optional) receives the NormX of the last one. */
int c2s_ingest_from(c2s_engine *e, int pos, const int32_t *tokens, int n, float *last_normx_out);

/* c2slm.Engine.generate's greedy loop (c2slm.go:144-223) on token ids, run
 * entirely on the device from the state the last Forward left: each step
 * projects the logits, applies the repetition penalty (factor `penalty` over
 * the last `window` positions, skipping im_end/eos), takes the strict-> argmax
 * and forwards the chosen token.  With stop_on_special the loop ends after
 * forwarding im_end/eos, as the reference does.  tokens_out (host) receives
 * the selected ids; *n_out their count.  Stop strings and per-token callbacks
 * stay with the caller: run fewer steps per call and c2s_kv_rewind surplus. */
int c2s_generate(c2s_engine *e, int max_new, float penalty, int window, int stop_on_special,
                 int32_t *tokens_out, int *n_out);

/* One generate step driven from the host, as a GenerateStream caller with an
 * onToken callback sees it: forwards `token` at SeqLen (recording it), then
 * projects, penalises and selects the next id into *next_out (host). */
int c2s_decode_step(c2s_engine *e, int32_t token, float penalty, int window, int32_t *next_out);

/* Timing helpers for benchmarks (not part of the reference surface). */
int c2s_engine_sync(c2s_engine *e);
/* Runs `n_steps` device-resident decode steps (logits+select+forward) without
 * host synchronisation or copies, for throughput measurement. */
int c2s_bench_decode(c2s_engine *e, int n_steps, float penalty, int window);
/* Same, bracketed by CUDA events on the engine's stream; *ms_out = elapsed.
 * period > 0 rewinds SeqLen to its entry value every `period` steps (a
 * KVCache.Rewind, no copy), so a long run keeps decoding the same positions. */
int c2s_bench_decode_timed(c2s_engine *e, int n_steps, float penalty, int window, int period,
                           float *ms_out);
/* Per-stage timing table (the stages of cmd/probe_bench/main.go:70-209):
 * runs n_steps decode steps as eager launches with a CUDA event pair around
 * every kernel.  stage_ms[k] / stage_launches[k] (8 entries each) are indexed
 * 1 = QKV(+embed, norm), 2 = O-proj(+residual), 3 = gate/up(+norm, SwiGLU),
 * 4 = down(+residual), 5 = logits(+final norm, penalty, argmax),
 * 7 = attention(+QK-norm, RoPE, KV append). */
int c2s_profile_step(c2s_engine *e, int n_steps, float penalty, int window, float *stage_ms,
                     int *stage_launches);
/* Phase trace of the persistent decode kernel: runs n_steps decode steps and
 * returns 8 values per [step][phase][cta] in trace_out (n_steps * nphase *
 * n_sms * 8 values): %globaltimer ns at phase start (after the grid barrier),
 * inputs ready, chunks done and end; then SM cycles spent waiting for weight
 * chunks, in the grid barrier before the phase, in the chunk loop, and the
 * cycle counter at phase start.  Values 1, 2, 4 and 6 are 0 for attention
 * phases.  *nphase_out = phases per step (1 logits phase, then 5 per layer:
 * qkv, attention, o-proj, gate/up, down). */
int c2s_trace_decode(c2s_engine *e, int n_steps, float penalty, int window, uint64_t *trace_out,
                     int *nphase_out);
/* Number of kernels one decode step launches on the per-phase (CUDA graph)
 * path (for the bench's launch count). */
int c2s_kernels_per_step(const c2s_engine *e);
/* Kernel launches one c2s_bench_decode / c2s_bench_decode_timed call of
 * n_steps issues: 1 when the persistent decode kernel is in use, else
 * c2s_kernels_per_step(e) * n_steps.  No counterpart in the reference. */
int c2s_decode_launches(const c2s_engine *e, int n_steps);
/* Warp groups of the persistent kernel's weight ring: the log2 of the group
 * count the engine uses for a ring of nslot slots when lng is asked for
 * (clamped so that the group count divides nslot: every slot is consumed by
 * one group only).  Host-only arithmetic, no device call.  No counterpart in
 * the reference (its row split is WorkerPool's, engine/pool.go:98-99). */
int c2s_ring_groups(int nslot, int lng);

/* ------------------------------------------------------------------------ */
/* Kernel-level entry points (tensor.* of the reference), host buffers       */
/* ------------------------------------------------------------------------ */
/* tensor.QuantizeRowQ8_K (tensor/ops.go:170 -> internal/simd/
 * c2_quantize_q8_k_gen.go:11-91): x (cols floats) -> y ((cols/256)*292 bytes,
 * reference byte layout).  cols % 256 == 0. */
int c2s_quantize_row_q8_k(const float *x, uint8_t *y, int cols);

/* DispatchGEMV / WorkerPool.ParallelGEMV (engine/model.go:250,
 * engine/pool.go:122-154): y = W x for a rows x cols tensor of `type`;
 * Q4_K/Q6_K quantise x to Q8_K first, Q5_0/Q8_0 use f32 x. */
int c2s_gemv(int type, const void *weight, const float *x, float *y, int rows, int cols);

/* Device-pointer GEMV on the library's stream for `device` (benchmarks and
 * callers that keep data resident): d_weight must come from cudaMalloc (or
 * be 256-byte aligned) with 64 readable bytes past its end. */
int c2s_gemv_device(int device, int type, const void *d_weight, const float *d_x, float *d_y,
                    int rows, int cols);

/* Single-op benchmark of c2s_gemv_device (config 0 of the bench): `reps`
 * launches back to back on the library's stream for `device`, launch i on
 * weight copy i % n_copies (copy k at d_weight + k * copy_stride bytes; one
 * copy stays L2-resident, many copies stream from HBM), captured in a CUDA
 * graph of up to 1000 launches and timed with CUDA events after one untimed
 * replay.  reps: a multiple of 1000, or at most 4000.  *ms_out = device time
 * of the `reps` launches.  The reference times GEMVQ4_K_Q8_K on the host
 * (tensor/ops_test.go:143-156). */
int c2s_bench_gemv(int device, int type, const void *d_weight, size_t copy_stride, int n_copies,
                   const float *d_x, float *d_y, int rows, int cols, int reps, float *ms_out);

/* c2s_gemv without any device allocation or free, for callers that cannot
 * allocate when they need the matvec (device memory held by another
 * allocator; loops that must not take cudaFree's device-wide
 * synchronisation).  The operands are staged in a 4 MiB statically reserved
 * device array: weights + x + y + 1.5 KB must fit, larger calls return
 * C2S_ERR_ARG.  Runs on the calling thread's default stream and returns when
 * y is written.  The first call on a device does the set-up and should come
 * before any stream capture; calls on one device share the array and must
 * not overlap.  No counterpart in the reference (its GEMV runs on host
 * memory, engine/model.go:250). */
int c2s_gemv_noalloc(int type, const void *weight, const float *x, float *y, int rows, int cols);

/* Integer partials of the K-quant x Q8_K dots, computed by the same device
 * code as c2s_gemv (bit-exact contract):
 *   Q4_K: dots[(r*nsb + sb)*8 + 2j + {0,1}] = sub-block dot (lo, hi nibbles)
 *   Q6_K: dots[r*nsb + sb] = the superblock's int32 isum                   */
int c2s_kquant_partials(int type, const void *weight, const float *x, int32_t *dots,
                        int rows, int cols);

/* f32-activation dots of one row each (tensor.DotQ*_K / DotQ5_0 / DotQ8_0),
 * used by the restricted logits: out[i] = row(rows_idx[i]) . x */
int c2s_dot_rows_f32x(int type, const void *weight, const float *x, const int32_t *rows_idx,
                      int n, float *out, int rows, int cols);

/* tensor.RMSNorm (tensor/ops.go:207-218) */
int c2s_rmsnorm(float *out, const float *x, const float *w, int n, float eps);
/* tensor.SwiGLU (tensor/ops.go:312) */
int c2s_swiglu(float *out, const float *gate, const float *up, int n);
/* Row dequantisation as EmbedToken uses it (engine/model.go:221-247, plus Q6_K). */
int c2s_dequant_row(int type, const void *row, float *out, int cols);

#ifdef __cplusplus
}
#endif
#endif /* C2SLM_B200_H */
