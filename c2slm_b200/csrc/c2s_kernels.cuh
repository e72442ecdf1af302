// c2s_kernels.cuh -- sm_100a kernels of the decode step.
//
// One decode step = per layer {QKV, ATTN, OPROJ, FFN_UP, FFN_DOWN} + LOGITS.
// Every matvec phase runs k_matvec: each CTA owns a contiguous row range of
// every segment (tensor) of the phase, streams those rows' native GGML blocks
// HBM -> shared memory with 1-D TMA bulk copies through a kStages-deep ring,
// and issues the first kStages copies BEFORE griddepcontrol.wait, so weight
// traffic of phase i+1 overlaps the tail of phase i (programmatic dependent
// launch).  Activations are tiny (<= 76 KB) and are re-read from L2 by every
// CTA after the wait.
#pragma once
#include "c2s_device.cuh"

namespace c2s {

struct DevState {
  int fwd_token, fwd_pos, commit;  // written by the host before a forward (12 B)
  int seq_len;                     // KVCache.SeqLen
  int halted, halt_pending, stop_on_special, window;
  float penalty;
  int n_out, out_cap;
  int im_end, eos, vocab;
  unsigned err;
  unsigned logits_counter;
  unsigned attn_counter[64];
};

// K_NORM: final RMSNorm only (NormX of engine.Forward).  K_LOGITS normalises
// X itself unless x_in is given (ComputeLogits on a caller's NormX).
enum Kind { K_RAW = 0, K_QKV = 1, K_OPROJ = 2, K_FFN_UP = 3, K_FFN_DOWN = 4, K_LOGITS = 5, K_NORM = 6 };

struct Seg {
  const uint8_t *w;
  int type, rows, row_bytes, units, rows_per_chunk;
  const float *bias;
  float *out;
};

struct MatParams {
  int kind, nseg;
  Seg seg[kMaxSegs];
  int cols;
  const float *x_in;  // RAW / OPROJ / FFN_DOWN input vector
  float *X;           // residual stream
  const float *norm_w;
  float eps;
  float *h_out;        // FFN_UP output
  float *normx_out;    // LOGITS: NormX written by CTA 0
  const uint8_t *embd_w;
  int embd_type, embd_row_bytes, do_embed;
  DevState *st;
  const int *token_ids;
  int *out_tokens;
  int select;
  float2 *part;
  int commit_here;     // FFN_DOWN of the last layer commits the forwarded token
  int need_f32, need_q8k;
  int32_t *dbg;        // optional int32 partials (K-quants)
  int ybuf_rows;
  int off_bars, off_xn, off_xt, off_q8, off_y, smem_bytes;
  int check_halt;      // engine kernels honour DevState::halted
};

__device__ __forceinline__ void seg_rows(int rows, int c, int G, int &r0, int &r1) {
  r0 = static_cast<int>((static_cast<long long>(c) * rows) / G);
  r1 = static_cast<int>((static_cast<long long>(c + 1) * rows) / G);
}

struct ChunkRef {
  int seg, r0, r1;
};

__device__ __forceinline__ ChunkRef chunk_at(const MatParams &P, const int (&my0)[kMaxSegs],
                                             const int (&my1)[kMaxSegs], int i) {
  ChunkRef c{0, 0, 0};
  for (int s = 0; s < P.nseg; ++s) {
    const int n = my1[s] - my0[s];
    const int cpr = P.seg[s].rows_per_chunk;
    const int nch = (n + cpr - 1) / cpr;
    if (i < nch) {
      c.seg = s;
      c.r0 = my0[s] + i * cpr;
      c.r1 = min(my1[s], c.r0 + cpr);
      return c;
    }
    i -= nch;
  }
  return c;
}

__device__ __forceinline__ void issue_chunk(const MatParams &P, const ChunkRef &c, uint8_t *stage, uint64_t *bar) {
  const Seg &S = P.seg[c.seg];
  const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(c.r0) * S.row_bytes;
  const uintptr_t end = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(c.r1) * S.row_bytes;
  const uintptr_t a0 = src & ~uintptr_t(15);
  const uintptr_t a1 = (end + 15) & ~uintptr_t(15);
  const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s(stage, reinterpret_cast<const void *>(a0), bytes, bar);
}

// Dot products of the rows in one staged chunk; results to y[0..nr).
// Warp/row mapping: wpr warps per row, lanes over units; partials reduced in
// a fixed order (deterministic).
__device__ __forceinline__ void compute_chunk(const MatParams &P, const Seg &S, const uint8_t *rows_smem, int nr,
                                              int grow0, const float *xt, int nbx, const Q8KView &q8,
                                              float *y, float (*red)[kWarps]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = S.units;
  int wpr = 1;  // warps per row: spread few wide rows over several warps
  if (nr < kWarps) {
    const int want = kWarps / nr;
    const int cap = (U + 31) / 32;
    while (wpr * 2 <= want && wpr * 2 <= cap) wpr *= 2;
  }
  const int rows_per_pass = kWarps / wpr;
  const int sub = warp % wpr;
  const int iters = (U + wpr * 32 - 1) / (wpr * 32);
  for (int rb = 0; rb < nr; rb += rows_per_pass) {
    const int r = rb + warp / wpr;
    const bool rowok = r < nr;
    const uint8_t *row = rows_smem + static_cast<size_t>(rowok ? r : 0) * S.row_bytes;
    float acc = 0.f;
    for (int it = 0; it < iters; ++it) {
      const int u = it * wpr * 32 + sub * 32 + lane;
      const bool ok = rowok && u < U;
      if (S.type == T_Q4_K) {
        if (ok) {
          int lo, hi;
          const int sbi = u >> 2, j = u & 3;
          acc += unit_q4k(row + sbi * 144, sbi, j, q8, lo, hi);
          if (P.dbg) {
            const int nsb = U >> 2;
            int32_t *dst = P.dbg + (static_cast<size_t>(grow0 + r) * nsb + sbi) * 8 + 2 * j;
            dst[0] = lo;
            dst[1] = hi;
          }
        }
      } else if (S.type == T_Q6_K) {
        int is = 0;
        const int sbi = u >> 2;
        if (ok) is = unit_q6k_isum(row + sbi * 210, sbi, (u >> 1) & 1, u & 1, q8);
        is += __shfl_xor_sync(0xffffffffu, is, 1);
        is += __shfl_xor_sync(0xffffffffu, is, 2);
        if (ok && (u & 3) == 0) {
          const float d6 = h2f(ld16(row + sbi * 210 + 208));
          acc += __fmul_rn(static_cast<float>(is), __fmul_rn(d6, q8.d[sbi]));
          if (P.dbg) P.dbg[static_cast<size_t>(grow0 + r) * (U >> 2) + sbi] = is;
        }
      } else if (S.type == T_Q5_0) {
        if (ok) acc += unit_q5_0(row + u * 22, xt + u, nbx);
      } else if (S.type == T_Q8_0) {
        if (ok) acc += unit_q8_0(row + u * 34, xt + u, nbx);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0 && rowok) red[r - rb][sub] = acc;
    __syncthreads();
    if (threadIdx.x < rows_per_pass && rb + static_cast<int>(threadIdx.x) < nr) {
      const int rr = rb + threadIdx.x;
      float s = 0.f;
      for (int k = 0; k < wpr; ++k) s += red[rr - rb][k];
      y[rr] = s;
    }
    __syncthreads();
  }
}

// RMSNorm of a shared-memory vector in place (tensor/ops.go:207-218):
// inv = float32(1/sqrt(float64(sumsq/n + eps))); out = (x*inv)*w.
__device__ __forceinline__ void rmsnorm_smem(float *x, const float *w, int n, float eps, float *scratch) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = block_sum(ss, scratch);
  const float mean = __fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps);
  const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(mean)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(__fmul_rn(x[i], inv), __ldg(w + i));
  __syncthreads();
}

// Builds the Q8_K activation in shared memory from a vector `src` (global or
// shared), one warp per superblock.
template <bool kGlobal>
__device__ __forceinline__ void build_q8k(const float *src, int cols, int8_t *qs, float *d, int32_t *bsum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = cols / 256;
  for (int sb = warp; sb < nsb; sb += kWarps) {
    float x[8];
    const float *p = src + sb * 256 + lane * 8;
    if (kGlobal) {
      const float4 a = __ldcg(reinterpret_cast<const float4 *>(p));
      const float4 b = __ldcg(reinterpret_cast<const float4 *>(p + 4));
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = p[i];
    }
    quantize_sb_warp(x, d + sb, bsum + sb * 16, [&](int ln, const int (&q)[8]) {
      const int e0 = sb * 256 + ln * 8;
      int8_t *dst = qs + q8_pad_index(e0);
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w0 |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
        w1 |= (static_cast<uint32_t>(q[4 + i]) & 0xFFu) << (8 * i);
      }
      *reinterpret_cast<uint2 *>(dst) = make_uint2(w0, w1);
    });
  }
}

__global__ void __launch_bounds__(kThreads) k_matvec(const MatParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kWarps][kWarps];
  __shared__ float scratch[kWarps];
  __shared__ int s_flag;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P.off_bars);
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;

  int my0[kMaxSegs], my1[kMaxSegs];
  int nchunks = 0;
  for (int s = 0; s < kMaxSegs; ++s) {
    my0[s] = my1[s] = 0;
    if (s < P.nseg) {
      seg_rows(P.seg[s].rows, c, G, my0[s], my1[s]);
      const int cpr = P.seg[s].rows_per_chunk;
      nchunks += (my1[s] - my0[s] + cpr - 1) / cpr;
    }
  }
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Weights do not depend on earlier kernels: stream them before the wait.
  if (tid == 0) {
    for (int i = 0; i < nchunks && i < kStages; ++i)
      issue_chunk(P, chunk_at(P, my0, my1, i), smem + i * kStageAlloc, &bars[i]);
  }
  pdl_trigger();
  pdl_wait();

  DevState *st = P.st;
  unsigned *err = &st->err;
  bool skip = false;
  if (P.check_halt) skip = (*reinterpret_cast<volatile int *>(&st->halted)) != 0;

  float *xn = reinterpret_cast<float *>(smem + P.off_xn);
  float *xt = reinterpret_cast<float *>(smem + P.off_xt);
  Q8KView q8{};
  int8_t *q8qs = reinterpret_cast<int8_t *>(smem + P.off_q8);
  float *q8d = reinterpret_cast<float *>(smem + P.off_q8 + q8_qs_bytes(P.cols));
  int32_t *q8bs = reinterpret_cast<int32_t *>(smem + P.off_q8 + q8_qs_bytes(P.cols) + 4 * (P.cols / 256));
  q8.qs = q8qs;
  q8.d = q8d;
  q8.bsum = q8bs;
  const int nbx = P.cols / 32;

  if (!skip) {
    // ---- input vector
    const bool normed = P.kind == K_QKV || P.kind == K_FFN_UP || P.kind == K_NORM ||
                        (P.kind == K_LOGITS && P.x_in == nullptr);
    if (normed) {
      if (P.kind == K_QKV && P.do_embed) {
        int tok = st->fwd_token;
        if (tok < 0 || tok >= st->vocab) tok = 0;  // engine/model.go:222-224
        dequant_row_cta(P.embd_type, P.embd_w + static_cast<size_t>(tok) * P.embd_row_bytes, xn, P.cols);
        __syncthreads();
        if (c == 0)
          for (int i = tid; i < P.cols; i += kThreads) P.X[i] = xn[i];
      } else {
        for (int i = tid; i < P.cols; i += kThreads) xn[i] = __ldcg(P.X + i);
        __syncthreads();
      }
      rmsnorm_smem(xn, P.norm_w, P.cols, P.eps, scratch);
      if ((P.kind == K_LOGITS || P.kind == K_NORM) && c == 0 && P.normx_out)
        for (int i = tid; i < P.cols; i += kThreads) P.normx_out[i] = xn[i];
      if (P.need_f32)
        for (int i = tid; i < P.cols; i += kThreads) xt[(i & 31) * nbx + (i >> 5)] = xn[i];
      if (P.need_q8k) build_q8k<false>(xn, P.cols, q8qs, q8d, q8bs);
    } else {
      if (P.need_f32)
        for (int i = tid; i < P.cols; i += kThreads) xt[(i & 31) * nbx + (i >> 5)] = __ldcg(P.x_in + i);
      if (P.need_q8k) build_q8k<true>(P.x_in, P.cols, q8qs, q8d, q8bs);
    }
    __syncthreads();
  }

  // ---- stream the chunks
  float *ybuf = reinterpret_cast<float *>(smem + P.off_y);
  if (skip) {  // halted step: drain the copies already issued, then leave
    if (tid == 0)
      for (int i = 0; i < nchunks && i < kStages; ++i) mbar_wait_bounded(&bars[i], 0, err);
    __syncthreads();
    return;
  }
  bool failed = false;
  int consumed = 0;
  for (int i = 0; i < nchunks; ++i) {
    const int sidx = i % kStages;
    const uint32_t parity = (i / kStages) & 1;
    int ok = mbar_wait_bounded(&bars[sidx], parity, err) ? 1 : 0;
    if (!__syncthreads_and(ok)) {
      failed = true;
      break;
    }
    consumed = i + 1;
    const ChunkRef ch = chunk_at(P, my0, my1, i);
    const Seg &S = P.seg[ch.seg];
    {
      const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(ch.r0) * S.row_bytes;
      const uint8_t *rows = smem + sidx * kStageAlloc + (src & 15);
      compute_chunk(P, S, rows, ch.r1 - ch.r0, ch.r0, xt, nbx, q8,
                    ybuf + ch.seg * P.ybuf_rows + (ch.r0 - my0[ch.seg]), red);
    }
    __syncthreads();
    if (tid == 0 && i + kStages < nchunks)
      issue_chunk(P, chunk_at(P, my0, my1, i + kStages), smem + sidx * kStageAlloc, &bars[sidx]);
  }
  if (failed) {
    // drain copies still in flight (bounded) before the CTA releases its smem
    if (tid == 0) {
      const int issued = min(nchunks, consumed + kStages);
      for (int i = consumed; i < issued; ++i) mbar_wait_bounded(&bars[i % kStages], (i / kStages) & 1, err);
    }
    __syncthreads();
    return;
  }

  // ---- epilogue
  const Seg &S0 = P.seg[0];
  if (P.kind == K_RAW || P.kind == K_QKV || (P.kind == K_LOGITS && !P.select)) {
    for (int s = 0; s < P.nseg; ++s)
      for (int r = my0[s] + tid; r < my1[s]; r += kThreads) {
        float v = ybuf[s * P.ybuf_rows + (r - my0[s])];
        if (P.seg[s].bias) v = __fadd_rn(v, __ldg(P.seg[s].bias + r));
        P.seg[s].out[r] = v;
      }
  } else if (P.kind == K_OPROJ || P.kind == K_FFN_DOWN) {
    for (int r = my0[0] + tid; r < my1[0]; r += kThreads)
      P.X[r] = __fadd_rn(__ldcg(P.X + r), ybuf[r - my0[0]]);
    if (P.kind == K_FFN_DOWN && P.commit_here && c == 0 && tid == 0 && st->commit) {
      const int pos = st->fwd_pos;
      if (pos >= 0 && pos < st->out_cap)  // out_cap == KV capacity
        const_cast<int *>(P.token_ids)[pos] = st->fwd_token;  // KVCache.StoreTokenID
      st->seq_len = pos + 1;
      if (st->halt_pending) {
        st->halted = 1;
        st->halt_pending = 0;
      }
    }
  } else if (P.kind == K_FFN_UP) {
    // SwiGLU (internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19), float64 exp
    for (int r = my0[0] + tid; r < my1[0]; r += kThreads) {
      const double g = static_cast<double>(ybuf[r - my0[0]]);
      const float silu = static_cast<float>(g / (1.0 + exp(-g)));
      P.h_out[r] = __fmul_rn(silu, ybuf[P.ybuf_rows + (r - my0[0])]);
    }
  } else if (P.kind == K_LOGITS) {
    const int n = my1[0] - my0[0];
    for (int r = my0[0] + tid; r < my1[0]; r += kThreads) S0.out[r] = ybuf[r - my0[0]];
    __syncthreads();
    // repetition penalty on this CTA's rows (c2slm.go:156-170), in window order
    if (tid == 0) {
      const int pos = st->seq_len;
      int start = pos - st->window;
      if (start < 0) start = 0;
      const float pen = st->penalty;
      for (int p = start; p < pos; ++p) {
        const int tok = P.token_ids[p];
        if (tok >= 0 && tok < st->vocab && tok != st->im_end && tok != st->eos && tok >= my0[0] && tok < my1[0]) {
          float &v = ybuf[tok - my0[0]];
          v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
        }
      }
    }
    __syncthreads();
    // strict '>' argmax, ties to the lowest id (c2slm.go:173-180)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < n; i += kThreads) {
      const float v = ybuf[i];
      if (v > bv || (v == bv && my0[0] + i < bi)) {
        bv = v;
        bi = my0[0] + i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    __shared__ float s_bv[kWarps];
    __shared__ int s_bi[kWarps];
    if ((tid & 31) == 0) {
      s_bv[tid >> 5] = bv;
      s_bi[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < kWarps; ++w)
        if (s_bv[w] > bv || (s_bv[w] == bv && s_bi[w] < bi)) {
          bv = s_bv[w];
          bi = s_bi[w];
        }
      P.part[c] = make_float2(bv, __int_as_float(bi));
      __threadfence();
      const unsigned t = atomicAdd(&st->logits_counter, 1u);
      s_flag = (t == static_cast<unsigned>(G - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (s_flag && tid == 0) {
      __threadfence();
      float best_v = -INFINITY;
      int best_i = 0x7fffffff;
      for (int k = 0; k < G; ++k) {
        const float2 pv = __ldcg(P.part + k);
        const int pi = __float_as_int(pv.y);
        if (pi == 0x7fffffff) continue;
        if (pv.x > best_v || (pv.x == best_v && pi < best_i) || best_i == 0x7fffffff) {
          best_v = pv.x;
          best_i = pi;
        }
      }
      if (best_i == 0x7fffffff) best_i = 0;
      if (st->n_out < st->out_cap) P.out_tokens[st->n_out] = best_i;
      st->n_out += 1;
      st->fwd_token = best_i;
      st->fwd_pos = st->seq_len;
      st->commit = 1;
      if (st->stop_on_special && (best_i == st->im_end || best_i == st->eos)) st->halt_pending = 1;
      st->logits_counter = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention with fused QK-norm, NeoX RoPE and KV append.
// grid = (n_kv, max_splits).  CTA (g, s) handles query heads g*qpk ..
// (g+1)*qpk-1 over positions [p0, p1) of the current length pos+1.
// (engine/forward.go:79-106,143-155; internal/simd/c2_tensor_attn_nosimd_gen.go;
// tensor/ops.go:262-286,317-339)
// ---------------------------------------------------------------------------
struct AttnParams {
  int layer, n_heads, n_kv, hd, max_tokens, max_splits, rope_len;
  float scale, eps;
  const float *q, *k, *v;
  float *kcache, *vcache;  // K and V planes, each [L][KVH][max_tokens][hd]
  const float *rope_cos, *rope_sin;
  const float *q_norm, *k_norm;
  float *part;  // [n_heads][max_splits][hd + 2]
  float *out;   // [n_heads * hd]
  DevState *st;
  int check_halt;
  int chunk_cap;  // positions per split the shared memory was sized for
};

__device__ __forceinline__ void rope_rotate(float *v, int hd, const float *cs, const float *sn, int tid, int nthr) {
  const int half = hd / 2;
  for (int i = tid; i < half; i += nthr) {
    const float x0 = v[i], x1 = v[i + half];
    const float c = cs[i], s = sn[i];
    v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

__device__ __forceinline__ void head_rmsnorm_warp(float *v, const float *w, int hd, float eps) {
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
  for (int i = lane; i < hd; i += 32) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float inv = static_cast<float>(
      1.0 / sqrt(static_cast<double>(__fadd_rn(__fdiv_rn(ss, static_cast<float>(hd)), eps))));
  __syncwarp();
  for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __ldg(w + i));
  __syncwarp();
}

__host__ __device__ inline int attn_nsplit(int n, int max_splits) {
  int ns = (n + kMinSplitLen - 1) / kMinSplitLen;
  return ns > max_splits ? max_splits : ns;
}

__global__ void __launch_bounds__(kThreads) k_attention(const AttnParams A) {
  extern __shared__ __align__(16) float asmem[];
  __shared__ int s_last;
  __shared__ float s_red[kWarps][8];
  pdl_trigger();
  pdl_wait();
  DevState *st = A.st;
  if (A.check_halt && *reinterpret_cast<volatile int *>(&st->halted)) return;
  const int g = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int hd = A.hd, qpk = A.n_heads / A.n_kv;
  const int pos = st->fwd_pos;
  if (pos < 0 || pos >= A.max_tokens) {
    if (tid == 0 && s == 0 && g == 0) atomicOr(&st->err, kErrPos);
    return;
  }
  const int n = pos + 1;
  const int nsplit = attn_nsplit(n, A.max_splits);
  const int chunk = (n + nsplit - 1) / nsplit;
  if (s >= nsplit) return;
  const int p0 = s * chunk, p1 = min(n, p0 + chunk);
  const int len = p1 - p0;

  float *qs = asmem;            // [qpk][hd]
  float *knew = qs + qpk * hd;  // [hd]
  float *vnew = knew + hd;      // [hd]
  float *sc = vnew + hd;        // [qpk][chunk_cap]
  for (int i = tid; i < qpk * hd; i += kThreads) qs[i] = __ldcg(A.q + g * qpk * hd + i);
  for (int i = tid; i < hd; i += kThreads) {
    knew[i] = __ldcg(A.k + g * hd + i);
    vnew[i] = __ldcg(A.v + g * hd + i);
  }
  __syncthreads();
  if (A.q_norm)  // Qwen3 per-head QK-norm (engine/forward.go:80-91)
    for (int h = warp; h < qpk; h += kWarps) head_rmsnorm_warp(qs + h * hd, A.q_norm, hd, A.eps);
  if (A.k_norm && warp == kWarps - 1) head_rmsnorm_warp(knew, A.k_norm, hd, A.eps);
  __syncthreads();
  if (pos < A.rope_len) {  // RoPETable.Apply rejects pos outside the table (tensor/ops.go:263)
    const float *cs = A.rope_cos + static_cast<size_t>(pos) * (hd / 2);
    const float *sn = A.rope_sin + static_cast<size_t>(pos) * (hd / 2);
    for (int h = 0; h < qpk; ++h) rope_rotate(qs + h * hd, hd, cs, sn, tid, kThreads);
    rope_rotate(knew, hd, cs, sn, tid, kThreads);
  }
  __syncthreads();
  // KV layout [L][KVH][max_tokens][hd] per plane (engine/kvcache.go:127-140)
  const size_t head_stride = static_cast<size_t>(A.max_tokens) * hd;
  const size_t layer_stride = static_cast<size_t>(A.n_kv) * head_stride;
  float *kc = A.kcache + static_cast<size_t>(A.layer) * layer_stride + g * head_stride;
  float *vc = A.vcache + static_cast<size_t>(A.layer) * layer_stride + g * head_stride;
  if (pos >= p0 && pos < p1)  // KVCache.StoreKV (engine/kvcache.go:143-158)
    for (int i = tid; i < hd; i += kThreads) {
      kc[static_cast<size_t>(pos) * hd + i] = knew[i];
      vc[static_cast<size_t>(pos) * hd + i] = vnew[i];
    }

  // scores: s_p = (sum_d q_d k_pd) * scale, d in order, no FMA
  // (internal/simd/c2_tensor_attn_nosimd_gen.go:7-24)
  for (int t = tid; t < len; t += kThreads) {
    const int p = p0 + t;
    const float *kp = (p == pos) ? knew : kc + static_cast<size_t>(p) * hd;
    float acc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = 0.f;
    for (int d = 0; d < hd; d += 4) {
      float4 kv4;
      if (p == pos) kv4 = make_float4(kp[d], kp[d + 1], kp[d + 2], kp[d + 3]);
      else kv4 = __ldcg(reinterpret_cast<const float4 *>(kp + d));
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        if (h < qpk) {
          const float *qh = qs + h * hd + d;
          acc[h] = __fadd_rn(acc[h], __fmul_rn(qh[0], kv4.x));
          acc[h] = __fadd_rn(acc[h], __fmul_rn(qh[1], kv4.y));
          acc[h] = __fadd_rn(acc[h], __fmul_rn(qh[2], kv4.z));
          acc[h] = __fadd_rn(acc[h], __fmul_rn(qh[3], kv4.w));
        }
      }
    }
    for (int h = 0; h < qpk && h < 8; ++h) sc[h * A.chunk_cap + t] = __fmul_rn(acc[h], A.scale);
    for (int h = 8; h < qpk; ++h) {  // GQA groups wider than 8 heads
      const float *qh = qs + h * hd;
      float a = 0.f;
      for (int d = 0; d < hd; ++d) a = __fadd_rn(a, __fmul_rn(qh[d], kp[d]));
      sc[h * A.chunk_cap + t] = __fmul_rn(a, A.scale);
    }
  }
  __syncthreads();
  // per-head max over the split
  for (int h0 = 0; h0 < qpk; h0 += 8) {
    float m[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) m[h] = -INFINITY;
    for (int t = tid; t < len; t += kThreads)
#pragma unroll
      for (int h = 0; h < 8; ++h)
        if (h0 + h < qpk) m[h] = fmaxf(m[h], sc[(h0 + h) * A.chunk_cap + t]);
#pragma unroll
    for (int h = 0; h < 8; ++h) m[h] = warp_max(m[h]);
    if (lane == 0)
#pragma unroll
      for (int h = 0; h < 8; ++h) s_red[warp][h] = m[h];
    __syncthreads();
    if (tid < 8 && h0 + tid < qpk) {
      float mm = -INFINITY;
      for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_red[w][tid]);
      s_red[0][tid] = mm;
    }
    __syncthreads();
    float mh[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) mh[h] = s_red[0][h];
    __syncthreads();
    // e = float32(exp(float64(s - max)))  (tensor/ops.go:329-333)
    for (int t = tid; t < len; t += kThreads)
#pragma unroll
      for (int h = 0; h < 8; ++h)
        if (h0 + h < qpk) {
          float &e = sc[(h0 + h) * A.chunk_cap + t];
          e = static_cast<float>(exp(static_cast<double>(__fsub_rn(e, mh[h]))));
        }
    if (tid < 8 && h0 + tid < qpk) s_red[1][tid] = mh[tid];  // keep the max
    __syncthreads();
    if (tid < 8 && h0 + tid < qpk) {
      float l = 0.f;
      for (int t = 0; t < len; ++t) l = __fadd_rn(l, sc[(h0 + tid) * A.chunk_cap + t]);
      const int h = g * qpk + h0 + tid;
      float *pp = A.part + (static_cast<size_t>(h) * A.max_splits + s) * (hd + 2);
      pp[0] = s_red[1][tid];
      pp[1] = l;
    }
    __syncthreads();
  }
  // acc_d = sum_p e_p v_pd (p in order)
  for (int i = tid; i < qpk * hd; i += kThreads) {
    const int h = i / hd, d = i - h * hd;
    const float *e = sc + h * A.chunk_cap;
    float a = 0.f;
    for (int t = 0; t < len; ++t) {
      const int p = p0 + t;
      const float vv = (p == pos) ? vnew[d] : __ldcg(vc + static_cast<size_t>(p) * hd + d);
      a = __fadd_rn(a, __fmul_rn(e[t], vv));
    }
    float *pp = A.part + (static_cast<size_t>(g * qpk + h) * A.max_splits + s) * (hd + 2);
    pp[2 + d] = a;
  }
  // the last split of this kv head combines (flash-decoding rescale)
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned t = atomicAdd(&st->attn_counter[g], 1u);
    s_last = (t == static_cast<unsigned>(nsplit - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < qpk * hd; i += kThreads) {
    const int h = g * qpk + i / hd, d = i % hd;
    const float *base = A.part + static_cast<size_t>(h) * A.max_splits * (hd + 2);
    float M = -INFINITY;
    for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(base + static_cast<size_t>(k) * (hd + 2)));
    float L = 0.f, O = 0.f;
    for (int k = 0; k < nsplit; ++k) {
      const float *pk = base + static_cast<size_t>(k) * (hd + 2);
      const float w = static_cast<float>(exp(static_cast<double>(__fsub_rn(__ldcg(pk), M))));
      L = __fadd_rn(L, __fmul_rn(w, __ldcg(pk + 1)));
      O = __fadd_rn(O, __fmul_rn(w, __ldcg(pk + 2 + d)));
    }
    A.out[h * hd + d] = __fmul_rn(O, __fdiv_rn(1.f, L));
  }
  if (tid == 0) st->attn_counter[g] = 0;
}

// ---------------------------------------------------------------------------
// Op-level kernels behind the tensor.* entry points of the C ABI
// ---------------------------------------------------------------------------

// tensor.QuantizeRowQ8_K into the reference byte layout (292 B per block).
__global__ void __launch_bounds__(kThreads) k_quantize_q8k(const float *x, uint8_t *y, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sb = blockIdx.x * kWarps + warp;
  if (sb >= cols / 256) return;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = x[sb * 256 + lane * 8 + i];
  uint8_t *blk = y + static_cast<size_t>(sb) * 292;
  float dval = 0.f;
  int32_t bs[16];
  quantize_sb_warp(v, &dval, bs, [&](int ln, const int (&q)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) blk[4 + ln * 8 + i] = static_cast<uint8_t>(static_cast<int8_t>(q[i]));
  });
  // lane 0 holds d; bsum j was written by lane 2j into its private bs[] copy
  dval = __shfl_sync(0xffffffffu, dval, 0);
  if (lane == 0) {
    const uint32_t b = __float_as_uint(dval);
    blk[0] = b & 0xff; blk[1] = (b >> 8) & 0xff; blk[2] = (b >> 16) & 0xff; blk[3] = (b >> 24) & 0xff;
  }
  if ((lane & 1) == 0) {
    const int j = lane >> 1;
    const int val = bs[j];
    blk[260 + 2 * j] = static_cast<uint8_t>(val & 255);
    blk[261 + 2 * j] = static_cast<uint8_t>((val >> 8) & 255);
  }
}

// f32-activation dot of selected rows (tensor.DotQ*: engine/forward.go:193-212),
// one CTA per requested row.
__global__ void __launch_bounds__(kThreads) k_dot_rows_f32x(int type, const uint8_t *w, int row_bytes,
                                                            const float *x, const int *rows_idx, int n,
                                                            float *out, int rows, int cols) {
  __shared__ float scratch[kWarps];
  const int i = blockIdx.x;
  if (i >= n) return;
  const int r = rows_idx[i];
  if (r < 0 || r >= rows) return;  // skipped like the reference's out-of-range targets
  const uint8_t *row = w + static_cast<size_t>(r) * row_bytes;
  float acc = 0.f;
  if (type == T_Q4_K) {
    // per (superblock, j): (sum q*x)*(d*sc) - (sum x)*(dmin*m) for each nibble half
    for (int u = threadIdx.x; u < (cols / 256) * 4; u += blockDim.x) {
      const int sbi = u >> 2, j = u & 3;
      const uint8_t *b = row + sbi * 144;
      const float d = h2f(ld16(b)), dmin = h2f(ld16(b + 2));
      const uint8_t *s = b + 4;
      int sc[2], m[2];
      for (int h = 0; h < 2; ++h) {
        const int idx = 2 * j + h;
        if (idx < 4) { sc[h] = s[idx] & 63; m[h] = s[idx + 4] & 63; }
        else { sc[h] = (s[idx + 4] & 15) | ((s[idx - 4] >> 6) << 4); m[h] = (s[idx + 4] >> 4) | ((s[idx] >> 6) << 4); }
      }
      const float *xl = x + sbi * 256 + 64 * j, *xh = xl + 32;
      float qxl = 0.f, sxl = 0.f, qxh = 0.f, sxh = 0.f;
      for (int l = 0; l < 32; ++l) {
        const uint8_t q = b[16 + 32 * j + l];
        qxl = __fadd_rn(qxl, __fmul_rn(static_cast<float>(q & 15), xl[l]));
        sxl = __fadd_rn(sxl, xl[l]);
        qxh = __fadd_rn(qxh, __fmul_rn(static_cast<float>(q >> 4), xh[l]));
        sxh = __fadd_rn(sxh, xh[l]);
      }
      acc += __fsub_rn(__fmul_rn(qxl, __fmul_rn(d, static_cast<float>(sc[0]))), __fmul_rn(sxl, __fmul_rn(dmin, static_cast<float>(m[0]))));
      acc += __fsub_rn(__fmul_rn(qxh, __fmul_rn(d, static_cast<float>(sc[1]))), __fmul_rn(sxh, __fmul_rn(dmin, static_cast<float>(m[1]))));
    }
  } else if (type == T_Q6_K) {
    for (int e = threadIdx.x; e < cols; e += blockDim.x) {
      const uint8_t *b = row + (e >> 8) * 210;
      const int ee = e & 255, nn = ee >> 7, rr = ee & 127, quarter = rr >> 5, l = rr & 31;
      const uint8_t qlb = b[64 * nn + l + ((quarter & 1) ? 32 : 0)];
      const uint8_t qhb = b[128 + 32 * nn + l];
      const int q = ((quarter < 2) ? (qlb & 15) : (qlb >> 4)) | (((qhb >> (2 * quarter)) & 3) << 4);
      const int8_t sc = static_cast<int8_t>(b[192 + 8 * nn + (l >> 4) + 2 * quarter]);
      const float ds = __fmul_rn(h2f(ld16(b + 208)), static_cast<float>(sc));
      acc += __fmul_rn(__fmul_rn(static_cast<float>(q - 32), ds), x[e]);
    }
  } else if (type == T_Q5_0 || type == T_Q8_0) {
    for (int bi = threadIdx.x; bi < cols / 32; bi += blockDim.x) {
      float v = 0.f;
      for (int e = 0; e < 32; ++e) {
        float q;
        if (type == T_Q8_0) {
          q = static_cast<float>(static_cast<int8_t>(row[bi * 34 + 2 + e]));
        } else {
          const uint8_t *b = row + bi * 22;
          const uint32_t qh = static_cast<uint32_t>(ld16(b + 2)) | (static_cast<uint32_t>(ld16(b + 4)) << 16);
          const int k = e & 15;
          const int nib = e < 16 ? (b[6 + k] & 15) : (b[6 + k] >> 4);
          q = static_cast<float>((nib | (((qh >> (e < 16 ? k : k + 16)) & 1) << 4)) - 16);
        }
        v = __fadd_rn(v, __fmul_rn(q, x[bi * 32 + e]));
      }
      const float d = h2f(ld16(row + bi * (type == T_Q8_0 ? 34 : 22)));
      acc += __fmul_rn(v, d);
    }
  }
  acc = block_sum(acc, scratch);
  if (threadIdx.x == 0) out[i] = acc;
}

__global__ void __launch_bounds__(kThreads) k_rmsnorm_op(float *out, const float *x, const float *w, int n, float eps) {
  extern __shared__ __align__(16) float buf[];
  __shared__ float scratch[kWarps];
  for (int i = threadIdx.x; i < n; i += blockDim.x) buf[i] = x[i];
  __syncthreads();
  rmsnorm_smem(buf, w, n, eps, scratch);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = buf[i];
}

__global__ void k_swiglu_op(float *out, const float *gate, const float *up, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double g = static_cast<double>(gate[i]);
  const float silu = static_cast<float>(g / (1.0 + exp(-g)));
  out[i] = __fmul_rn(silu, up[i]);
}

__global__ void __launch_bounds__(kThreads) k_dequant_op(int type, const uint8_t *row, float *out, int cols) {
  dequant_row_cta(type, row, out, cols);
}

}  // namespace c2s
