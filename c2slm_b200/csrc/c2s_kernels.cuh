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
#include "c2s_rows.cuh"

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
  unsigned attn_counter[64];       // arrivals of a kv head's attention splits
  unsigned xbar;                   // cross-GPU barriers completed (tensor-parallel persistent decode)
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
  int off_bars, off_nw, off_bias, off_xn, off_xt, off_q8, off_y, smem_bytes;
  int check_halt;      // engine kernels honour DevState::halted
};

// rows [r0, r1) of CTA c of G (32-bit: (c + 1) * rows < 2^32 for every
// matrix the engine accepts)
__device__ __forceinline__ void seg_rows(int rows, int c, int G, int &r0, int &r1) {
  r0 = static_cast<int>((static_cast<unsigned>(c) * static_cast<unsigned>(rows)) / static_cast<unsigned>(G));
  r1 = static_cast<int>((static_cast<unsigned>(c + 1) * static_cast<unsigned>(rows)) / static_cast<unsigned>(G));
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

// ---------------------------------------------------------------------------
// Row dot products over one staged chunk.
// ---------------------------------------------------------------------------
// float(b) for a byte b of `w` via the exponent trick: 0x4B0000bb = 2^23 + b.
__device__ __forceinline__ float byte_as_f(uint32_t w, int e) {
  return __int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7440u | static_cast<uint32_t>(e))));
}

// Q8_0 block . f32 x held in registers (lane owns the block).
__device__ __forceinline__ float blockdot_q8_0_reg(const uint8_t *blk, const float (&xr)[32]) {
  const float d = h2f(ld16(blk));
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t w = ld32u(blk + 2 + 4 * t) ^ 0x80808080u;  // int8 -> uint8 + 128
    a0 = fmaf(byte_as_f(w, 0) - 8388736.0f, xr[4 * t + 0], a0);  // 2^23 + 128
    a1 = fmaf(byte_as_f(w, 1) - 8388736.0f, xr[4 * t + 1], a1);
    a2 = fmaf(byte_as_f(w, 2) - 8388736.0f, xr[4 * t + 2], a2);
    a3 = fmaf(byte_as_f(w, 3) - 8388736.0f, xr[4 * t + 3], a3);
  }
  return d * ((a0 + a1) + (a2 + a3));
}

// Q5_0 block . f32 x held in registers: q = (nibble | hbit<<4) - 16.
__device__ __forceinline__ float blockdot_q5_0_reg(const uint8_t *blk, const float (&xr)[32]) {
  const float d = h2f(ld16(blk));
  const uint32_t qh = static_cast<uint32_t>(ld16(blk + 2)) | (static_cast<uint32_t>(ld16(blk + 4)) << 16);
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t w = ld32u(blk + 6 + 4 * t);
    const uint32_t lo = (w & 0x0F0F0F0Fu) | (spread4((qh >> (4 * t)) & 0xFu) << 4);
    const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) | (spread4((qh >> (16 + 4 * t)) & 0xFu) << 4);
    a0 = fmaf(byte_as_f(lo, 0) - 8388624.0f, xr[4 * t + 0], a0);  // 2^23 + 16
    a1 = fmaf(byte_as_f(lo, 1) - 8388624.0f, xr[4 * t + 1], a1);
    a2 = fmaf(byte_as_f(lo, 2) - 8388624.0f, xr[4 * t + 2], a2);
    a3 = fmaf(byte_as_f(lo, 3) - 8388624.0f, xr[4 * t + 3], a3);
    a0 = fmaf(byte_as_f(hi, 0) - 8388624.0f, xr[16 + 4 * t + 0], a0);
    a1 = fmaf(byte_as_f(hi, 1) - 8388624.0f, xr[16 + 4 * t + 1], a1);
    a2 = fmaf(byte_as_f(hi, 2) - 8388624.0f, xr[16 + 4 * t + 2], a2);
    a3 = fmaf(byte_as_f(hi, 3) - 8388624.0f, xr[16 + 4 * t + 3], a3);
  }
  return d * ((a0 + a1) + (a2 + a3));
}

// K-quant rows of one staged chunk with their integer partials recorded in
// P.dbg (c2s_kquant_partials, the bit-exact contract): warp w takes rows w,
// w + kWarps, ...; lanes take the row's 64-value units (unit_q4k /
// unit_q6k_isum, the same integer arithmetic as the warp-row core).
template <int TYPE>
__device__ __forceinline__ void dbg_chunk_t(const MatParams &P, const Seg &S, const uint8_t *rows_smem, int nr,
                                            int grow0, const Q8KView &q8, float *y) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = S.units;
  for (int r = warp; r < nr; r += kWarps) {
    const uint8_t *row = rows_smem + static_cast<size_t>(r) * S.row_bytes;
    const int grow = grow0 + r;
    float acc = 0.f;
    for (int ub = 0; ub < U; ub += 32) {
      const int u = ub + lane;
      const bool ok = u < U;
      if (TYPE == T_Q4_K) {
        if (ok) {
          int lo, hi;
          const int sbi = u >> 2, j = u & 3;
          acc += unit_q4k(row + sbi * 144, sbi, j, q8, lo, hi);
          int32_t *dst = P.dbg + (static_cast<size_t>(grow) * (U >> 2) + sbi) * 8 + 2 * j;
          dst[0] = lo;
          dst[1] = hi;
        }
      } else {
        int is = 0;
        const int sbi = u >> 2;
        if (ok) is = unit_q6k_isum(row + sbi * 210, sbi, (u >> 1) & 1, u & 1, q8);
        is += __shfl_xor_sync(0xffffffffu, is, 1);
        is += __shfl_xor_sync(0xffffffffu, is, 2);
        if (ok && (u & 3) == 0) {
          const float d6 = h2f(ld16(row + sbi * 210 + 208));
          acc += __fmul_rn(static_cast<float>(is), __fmul_rn(d6, q8.d[sbi]));
          P.dbg[static_cast<size_t>(grow) * (U >> 2) + sbi] = is;
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) y[r] = acc;
  }
}

// Loads n floats (n % 4 == 0, 16-B aligned) from global into shared memory,
// every thread's loads in flight before its first store.
__device__ __forceinline__ void load_vec_to_smem(float *dst, const float *src, int n) {
  const int n4 = n >> 2;
  const float4 *s4 = reinterpret_cast<const float4 *>(src);
  float4 *d4 = reinterpret_cast<float4 *>(dst);
  int i = threadIdx.x;
  for (; i + 3 * kThreads < n4; i += 4 * kThreads) {
    const float4 a = __ldcg(s4 + i), b = __ldcg(s4 + i + kThreads), c = __ldcg(s4 + i + 2 * kThreads),
                 d = __ldcg(s4 + i + 3 * kThreads);
    d4[i] = a;
    d4[i + kThreads] = b;
    d4[i + 2 * kThreads] = c;
    d4[i + 3 * kThreads] = d;
  }
  for (; i < n4; i += kThreads) d4[i] = __ldcg(s4 + i);
}

// Same for read-only constants (norm weights): the read-only data path.
__device__ __forceinline__ void load_const_to_smem(float *dst, const float *src, int n) {
  const int n4 = n >> 2;
  const float4 *s4 = reinterpret_cast<const float4 *>(src);
  float4 *d4 = reinterpret_cast<float4 *>(dst);
  for (int i = threadIdx.x; i < n4; i += kThreads) d4[i] = __ldg(s4 + i);
}

// RMSNorm of a shared-memory vector in place (tensor/ops.go:207-218):
// inv = float32(1/sqrt(float64(sumsq/n + eps))); out = (x*inv)*w, w in smem.
// Sum of squares: thread t accumulates float4 t, t + kThreads, ... in order
// (x, y, z, w), then a fixed block tree -- the persistent kernel's prologue
// sums in the same order.
__device__ __forceinline__ void rmsnorm_smem(float *x, const float *w, int n, float eps, float *scratch) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < (n >> 2); i += kThreads) {
    const float4 v = reinterpret_cast<const float4 *>(x)[i];
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = block_sum(ss, scratch);
  const float mean = __fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps);
  const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(mean)));
  for (int k = threadIdx.x; k < n; k += kThreads) x[k] = __fmul_rn(__fmul_rn(x[k], inv), w[k]);
  csync();
}

// Builds the Q8_K activation in shared memory from a shared-memory vector,
// one warp per superblock.
__device__ __forceinline__ void build_q8k(const float *src, int cols, int8_t *qs, float *d, int32_t *bsum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = cols / 256;
  for (int sb = warp; sb < nsb; sb += kWarps) {
    float x[8];
    const float4 a = *reinterpret_cast<const float4 *>(src + sb * 256 + lane * 8);
    const float4 b = *reinterpret_cast<const float4 *>(src + sb * 256 + lane * 8 + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    quantize_sb_warp(x, d + sb, bsum + sb * 16, [&](int ln, const int (&q)[8]) {
      const int e0 = sb * 256 + ln * 8;
      int8_t *dst = qs + q8_pad_index(e0);
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w0 |= (static_cast<uint32_t>(q[k]) & 0xFFu) << (8 * k);
        w1 |= (static_cast<uint32_t>(q[4 + k]) & 0xFFu) << (8 * k);
      }
      *reinterpret_cast<uint2 *>(dst) = make_uint2(w0, w1);
    });
  }
}

__global__ void __launch_bounds__(kThreads) k_matvec(const MatParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
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
  // Weights and constants do not depend on earlier kernels: fetch them
  // before the wait.
  if (tid == 0) {
    for (int i = 0; i < nchunks && i < kStages; ++i)
      issue_chunk(P, chunk_at(P, my0, my1, i), smem + i * kStageAlloc, &bars[i]);
  }
  float *nw = reinterpret_cast<float *>(smem + P.off_nw);
  float *ybias = reinterpret_cast<float *>(smem + P.off_bias);
  const bool normed = P.kind == K_QKV || P.kind == K_FFN_UP || P.kind == K_NORM ||
                      (P.kind == K_LOGITS && P.x_in == nullptr);
  if (normed) load_const_to_smem(nw, P.norm_w, P.cols);
  for (int s = 0; s < P.nseg; ++s)
    if (P.seg[s].bias)
      for (int r = my0[s] + tid; r < my1[s]; r += kThreads) ybias[s * P.ybuf_rows + (r - my0[s])] = __ldg(P.seg[s].bias + r);
  pdl_trigger();
  pdl_wait();

  DevState *st = P.st;
  unsigned *err = &st->err;
  bool skip = false;
  if (P.check_halt) skip = (*reinterpret_cast<volatile int *>(&st->halted)) != 0;
  if (skip) {  // halted step: drain the copies already issued, then leave
    if (tid == 0)
      for (int i = 0; i < nchunks && i < kStages; ++i) mbar_wait_bounded(&bars[i], 0, err);
    __syncthreads();
    return;
  }
  // residual rows of this CTA, fetched early (used by the epilogue)
  float xres = 0.f;
  const bool residual = P.kind == K_OPROJ || P.kind == K_FFN_DOWN;
  if (residual && my0[0] + tid < my1[0]) xres = __ldcg(P.X + my0[0] + tid);

  float *xn = reinterpret_cast<float *>(smem + P.off_xn);
  const int nbx = P.cols / 32;
  int *la = reinterpret_cast<int *>(smem + P.off_xt);
  int *lb = la + 8 * nbx, *lc = lb + 8 * nbx;
  float *ls = reinterpret_cast<float *>(lc + 8 * nbx);
  const LimbsView LV{la, lb, lc, ls, nbx};
  Q8KView q8{};
  int8_t *q8qs = reinterpret_cast<int8_t *>(smem + P.off_q8);
  float *q8d = reinterpret_cast<float *>(smem + P.off_q8 + q8_qs_bytes(P.cols));
  int32_t *q8bs = reinterpret_cast<int32_t *>(smem + P.off_q8 + q8_qs_bytes(P.cols) + ((4 * (P.cols / 256) + 15) & ~15));
  q8.qs = q8qs;
  q8.d = q8d;
  q8.bsum = q8bs;

  // ---- input vector
  if (normed) {
    if (P.kind == K_QKV && P.do_embed) {
      int tok = st->fwd_token;
      if (tok < 0 || tok >= st->vocab) tok = 0;  // engine/model.go:222-224
      dequant_row_cta(P.embd_type, P.embd_w + static_cast<size_t>(tok) * P.embd_row_bytes, xn, P.cols);
      __syncthreads();
      if (c == 0)
        for (int i = tid; i < P.cols; i += kThreads) P.X[i] = xn[i];
    } else {
      load_vec_to_smem(xn, P.X, P.cols);
      __syncthreads();
    }
    rmsnorm_smem(xn, nw, P.cols, P.eps, scratch);
    if ((P.kind == K_LOGITS || P.kind == K_NORM) && c == 0 && P.normx_out)
      for (int i = tid; i < P.cols; i += kThreads) P.normx_out[i] = xn[i];
  } else {
    load_vec_to_smem(xn, P.x_in, P.cols);
    __syncthreads();
  }
  if (P.need_f32) {  // int8 limbs of x, from the float4 each thread reads
    const int n4 = P.cols >> 2;
    for (int i0 = 0; i0 < n4; i0 += kThreads) {
      const int i = i0 + tid;
      const float4 v = i < n4 ? reinterpret_cast<const float4 *>(xn)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      put_limbs(v, i, i < n4, la, lb, lc, ls, nbx);
    }
  }
  if (P.need_q8k) build_q8k(xn, P.cols, q8qs, q8d, q8bs);
  __syncthreads();

  // ---- stream the chunks
  float *ybuf = reinterpret_cast<float *>(smem + P.off_y);
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
      float *y = ybuf + ch.seg * P.ybuf_rows + (ch.r0 - my0[ch.seg]);
      const int nr = ch.r1 - ch.r0, warp = tid >> 5;
      if (P.dbg) {  // integer partials of the K-quant dots (bit-exact contract)
        if (S.type == T_Q4_K)
          dbg_chunk_t<T_Q4_K>(P, S, rows, nr, ch.r0, q8, y);
        else if (S.type == T_Q6_K)
          dbg_chunk_t<T_Q6_K>(P, S, rows, nr, ch.r0, q8, y);
      } else if (warp < nr) {
        const int cnt = (nr - warp + kWarps - 1) / kWarps;
        switch (S.type) {
          case T_Q8_0: warp_rows<T_Q8_0>(rows, S.row_bytes, S.units, warp, cnt, LV, q8, y); break;
          case T_Q5_0: warp_rows<T_Q5_0>(rows, S.row_bytes, S.units, warp, cnt, LV, q8, y); break;
          case T_Q4_K: warp_rows<T_Q4_K>(rows, S.row_bytes, S.units, warp, cnt, LV, q8, y); break;
          case T_Q6_K: warp_rows<T_Q6_K>(rows, S.row_bytes, S.units, warp, cnt, LV, q8, y); break;
          default: break;
        }
      }
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
        if (P.seg[s].bias) v = __fadd_rn(v, ybias[s * P.ybuf_rows + (r - my0[s])]);
        P.seg[s].out[r] = v;
      }
  } else if (residual) {
    if (my0[0] + tid < my1[0]) P.X[my0[0] + tid] = __fadd_rn(xres, ybuf[tid]);
    for (int r = my0[0] + tid + kThreads; r < my1[0]; r += kThreads)
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
  int split_len;  // positions per split: position p is always in split p / split_len
  // tensor parallel: this rank holds query heads [tp_h0, tp_h1) (q and out
  // rows start at tp_h0) and kv heads tp_g0 .. tp_g0 + n_kv - 1; qpk is the
  // model's query heads per kv head.  One GPU: 0, n_heads, 0.
  int qpk, tp_h0, tp_h1, tp_g0;
  int items_cap;  // per-head items while they fit in this many CTAs (the persistent grid)
};

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

// staged rows per K/V sub-chunk (16 KB), and the attention's shared memory
constexpr int kAttnBufs = 4;
__host__ __device__ inline int attn_sub(int hd) { return 4096 / hd; }
__host__ __device__ inline size_t attn_smem_bytes(int hd, int qpk) {
  const size_t sub = static_cast<size_t>(attn_sub(hd));
  return (kAttnBufs * sub * hd + static_cast<size_t>(qpk) * hd + 2 * static_cast<size_t>(hd) +
          static_cast<size_t>(qpk) * kAttnBufs * sub) * 4;
}

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// E consecutive floats of shared memory (16-B aligned for E = 4, 8-B for
// E = 2) in one vector load
template <int E>
__device__ __forceinline__ void lds_vec(const float *p, float (&v)[E]) {
  if constexpr (E == 4) {
    const float4 t = *reinterpret_cast<const float4 *>(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else if constexpr (E == 2) {
    const float2 t = *reinterpret_cast<const float2 *>(p);
    v[0] = t.x, v[1] = t.y;
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = p[j];
  }
}

// Scores of positions a .. a+len-1 (rows of kb) for the qpk (<= QP) heads of
// an item.  The 8 rows of one transposing butterfly are (position p, head h)
// pairs, r = p * QP + h, P = 8 / QP consecutive positions: warp w takes
// positions w*P, w*P + 8P, ..., U butterflies at a time (independent, they
// interleave); lane l holds d = l*E .. l*E+E-1 of q and k.  After the
// butterfly lane 4r holds row r.
template <int E, int QP>
__device__ __forceinline__ void attn_scores(const float *qs, const float *kb, int len, int qpk, float scale,
                                            float *sc, int stride) {
  constexpr int P = 8 / QP, U = P >= 4 ? 1 : 4 / P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hd = 32 * E;
  float qr[QP][E];
#pragma unroll
  for (int h = 0; h < QP; ++h) {
    if (h < qpk) {
      lds_vec<E>(qs + h * hd + lane * E, qr[h]);
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) qr[h][j] = 0.f;
    }
  }
  const int r = lane >> 2, hq = r % QP, pq = r / QP;
  for (int t0 = warp * P; t0 < len; t0 += kWarps * P * U) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float dot[8];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int t = t0 + u * kWarps * P + p;
        float kv[E];
        if (t < len) {
          lds_vec<E>(kb + t * hd + lane * E, kv);
        } else {
#pragma unroll
          for (int j = 0; j < E; ++j) kv[j] = 0.f;
        }
#pragma unroll
        for (int h = 0; h < QP; ++h) {
          float d0 = 0.f;
#pragma unroll
          for (int j = 0; j < E; ++j) d0 = fmaf(qr[h][j], kv[j], d0);
          dot[p * QP + h] = d0;
        }
      }
      v[u] = reduce_rows<8>(dot);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = t0 + u * kWarps * P + pq;
      if ((lane & 3) == 0 && hq < qpk && t < len) sc[hq * stride + t] = __fmul_rn(v[u], scale);
    }
  }
}

// One attention work item: kv head g, split s of the positions [0, pos]
// (decode of one token at pos).  Shared by the per-phase kernel and the
// persistent kernel, so both evaluate the same float operations in the same
// order.
struct AttnJob {
  const float *q, *k, *v;          // projections of this token (bias added)
  const float *q_norm, *k_norm;    // Qwen3 per-head norms, or null
  float *kc, *vc;                  // cache planes of this layer and kv head: row p at [p * hd]
  const float *rope_cs, *rope_sn;  // RoPE row of pos (hd/2 each), or null outside the table
  float *out, *part;               // head h0 + j of this item at out[(h0 + j) * hd]
  unsigned *counter;               // arrivals of the group's splits
  int dist;                        // 1: every split combines a slice of the outputs once all have
                                   // arrived (the group's CTAs are co-resident; the caller clears
                                   // the counter after its next grid barrier); 0: the last one
                                   // combines them all and clears the counter
  int g, s, nsplit, p0, p1, pos, h0;
  int hd, qpk, max_splits;
  int store_kv;                    // this item writes the cache row of pos (one item per kv head)
  float eps, scale;
  // dataflow hand-off of the persistent kernel (tq null: plain q/k/v/out):
  // q/k/v read as tagged words polled until they carry tag_in, outputs
  // stored as tagged words with tag_out; the split arrivals of this phase
  // wait for cnt_base + nsplit (the counter accumulates over the launch)
  const unsigned long long *tq = nullptr, *tk = nullptr, *tv = nullptr;
  unsigned long long *tout = nullptr;
  unsigned tag_in = 0, tag_out = 0, cnt_base = 0;
};

// Work items of the attention of position pos on one rank (nh local query
// heads in n_kv local kv groups): one item per (query head, split) while
// they fit in `cap` CTAs, else one per (kv group, split).  The per-phase and
// persistent kernels choose alike, so both evaluate the same operations.
struct AttnLayout {
  int nsplit, per_head, n_items;
};

__device__ __forceinline__ AttnLayout attn_layout(int pos, int split_len, int n_kv, int nh, int cap) {
  AttnLayout L;
  L.nsplit = (pos + split_len) / split_len;  // positions 0..pos
  L.per_head = (nh <= 64 && nh * L.nsplit <= cap) ? 1 : 0;  // (one counter per head)
  L.n_items = (L.per_head ? nh : n_kv) * L.nsplit;
  return L;
}

// Fill the head range, kv group, store flag and counter of unit x (a local
// query head, or a local kv group) of the layout; false if it has no heads.
// The model has qpk query heads per kv head; this rank holds query heads
// [tp_h0, tp_h1) and kv groups from tp_g0.
__device__ __forceinline__ bool attn_unit(const AttnLayout &L, int x, int qpk, int tp_h0, int tp_h1, int tp_g0,
                                          unsigned *counters, AttnJob &J) {
  int hs, he, gg;
  if (L.per_head) {
    hs = tp_h0 + x;
    he = hs + 1;
    gg = hs / qpk;
    J.store_kv = (hs == max(tp_h0, gg * qpk)) ? 1 : 0;  // the group's first head on this rank
  } else {
    gg = tp_g0 + x;
    hs = max(tp_h0, gg * qpk);
    he = min(tp_h1, (gg + 1) * qpk);
    J.store_kv = 1;
  }
  if (he <= hs) return false;
  J.g = gg - tp_g0;
  J.qpk = he - hs;
  J.h0 = hs - tp_h0;
  J.counter = counters + x;
  return true;
}

// Shared memory: asmem holds [kAttnBufs][SUB][hd] staged K or V rows,
// [qpk][hd] q, [hd] k, [hd] v, [qpk][WIN] scores / weights.  bars[] are the
// staging barriers (one per buffer); uses[] counts their completed phases
// (kept by the caller across items).
//
// The split is taken in windows of WIN = kAttnBufs * SUB positions; each
// window is two passes over the staged rows: the scores of every position
// (K), one softmax over the window per head (warp h owns head h, exp in
// float64), then the weighted sum of V.  Windows after the first rescale the
// running (m, l, acc) as in an online softmax; at the split lengths the
// engine uses (<= WIN) there is one window.  K and V sub-chunks of all
// windows form one load sequence through the buffers, kAttnBufs in flight.
// Returns false if a bounded wait expired.
template <int E, int QP>
__device__ bool attend_t(const AttnJob &J, float *asmem, uint64_t *bars, uint32_t (&uses)[kAttnBufs], unsigned *err) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int hd = 32 * E;
  constexpr int NB = kAttnBufs;
  // softmax and weighted V: WPH warps per head; warp w takes head w / WPH
  // and every WPH-th position of it from w % WPH
  constexpr int WPH = kWarps / QP;
  const int hw = warp / WPH, part = warp % WPH;
  __shared__ float s_red[2][kWarps];
  const int qpk = J.qpk, SUB = attn_sub(hd), WIN = NB * SUB, pos = J.pos, p0 = J.p0, p1 = J.p1;
  float *buf = asmem, *qs = buf + NB * SUB * hd;
  float *knew = qs + qpk * hd, *vnew = knew + hd, *sc = vnew + hd;
  __shared__ int s_last;
  bool ok_in = true;  // a tagged input poll gave up (error flag set)
  const int nwin = (p1 - p0 + WIN - 1) / WIN;
  // load q of the sequence: window w, K (r < nsw) or V, sub-chunk r mod nsw
  struct Ld {
    int a, b, v;  // positions [a, b) of one plane (v: 1 = V)
  };
  auto load_of = [&](int q) {
    int w = q / (2 * NB);
    if (w > nwin - 1) w = nwin - 1;
    const int wa = p0 + w * WIN, wb = min(p1, wa + WIN);
    const int nsw = (wb - wa + SUB - 1) / SUB, r = q - w * 2 * NB;
    const int sub = r >= nsw ? r - nsw : r;
    Ld L;
    L.a = wa + sub * SUB;
    L.b = min(wb, L.a + SUB);
    L.v = r >= nsw ? 1 : 0;
    return L;
  };
  const int last_w = p0 + (nwin - 1) * WIN;
  const int n_loads = (nwin - 1) * 2 * NB + 2 * ((min(p1, last_w + WIN) - last_w + SUB - 1) / SUB);
  // rows below pos come from the cache; row pos is this token's k / v
  auto cached = [&](const Ld &L) { return max(0, min(L.b, pos) - L.a); };
  auto issue = [&](int q) {
    const Ld L = load_of(q);
    const int n = cached(L);
    if (n > 0) {
      const uint32_t bytes = static_cast<uint32_t>(n) * hd * 4;
      uint64_t *bar = &bars[q % NB];
      mbar_arrive_expect_tx(bar, bytes);
      bulk_g2s(buf + (q % NB) * SUB * hd, (L.v ? J.vc : J.kc) + static_cast<size_t>(L.a) * hd, bytes, bar);
    }
  };
  if (tid == 0) {
    // cache rows this CTA stored in earlier calls, and staging rows it wrote,
    // are next accessed by the async proxy
    asm volatile("fence.proxy.async;" ::: "memory");
    for (int q = 0; q < NB && q < n_loads; ++q) issue(q);
  }
  // projections: every load in flight at once
  if (J.tq) {  // tagged words of the QKV phase
    ok_in = poll_to_smem(J.tq, qpk * hd, qs, J.tk, hd, knew, J.tv, hd, vnew, J.tag_in, err);
  } else {
    for (int i = tid; i < qpk * hd; i += kThreads) qs[i] = __ldcg(J.q + i);
    for (int i = tid; i < hd; i += kThreads) {
      knew[i] = __ldcg(J.k + i);
      vnew[i] = __ldcg(J.v + i);
    }
  }
  csync();
  if (J.q_norm || J.k_norm) {  // Qwen3 per-head QK-norm (engine/forward.go:80-91)
    if (J.q_norm)
      for (int h = warp; h < qpk; h += kWarps) head_rmsnorm_warp(qs + h * hd, J.q_norm, hd, J.eps);
    if (J.k_norm && warp == kWarps - 1) head_rmsnorm_warp(knew, J.k_norm, hd, J.eps);
    csync();
  }
  if (J.rope_cs) {  // NeoX RoPE of every q head and k: one thread per (head, pair)
    constexpr int half = hd / 2;
    for (int t = tid; t < (qpk + 1) * half; t += kThreads) {
      const int h = t / half, i = t - h * half;
      float *v = h < qpk ? qs + h * hd : knew;
      const float x0 = v[i], x1 = v[i + half];
      const float c = J.rope_cs[i], sn = J.rope_sn[i];
      v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      v[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    csync();
  }
  if (J.store_kv && pos >= p0 && pos < p1) {  // KVCache.StoreKV (engine/kvcache.go:143-158)
    for (int i = tid; i < hd; i += kThreads) {
      J.kc[static_cast<size_t>(pos) * hd + i] = knew[i];
      J.vc[static_cast<size_t>(pos) * hd + i] = vnew[i];
    }
    // later steps stage this row with bulk copies, possibly from another CTA
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  // running softmax state of head hw (every lane of its warps holds m and l)
  float m = -INFINITY, l = 0.f, acc[E];  // acc: d = lane*E .. lane*E+E-1
#pragma unroll
  for (int j = 0; j < E; ++j) acc[j] = 0.f;
  bool ok = ok_in;
  // wait for load q (if it reads the cache), complete it with row pos, and
  // return its buffer
  auto arrive = [&](int q, const Ld &L) {
    float *b = buf + (q % NB) * SUB * hd;
    if (cached(L) > 0) {  // completions of a buffer's barrier alternate parity
      ok = mbar_wait_bounded(&bars[q % NB], uses[q % NB] & 1u, err) && ok;
      uses[q % NB] += 1;
    }
    if (pos >= L.a && pos < L.b) {
      const float *src = L.v ? vnew : knew;
      for (int i = tid; i < hd; i += kThreads) b[(pos - L.a) * hd + i] = src[i];
      csync();
    }
    return b;
  };
  // after every warp is done with load q's buffer: reuse it for load q + NB
  auto release = [&](int q) {
    csync();
    if (tid == 0 && q + NB < n_loads) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(q + NB);
    }
  };
  int q = 0;
  for (int w = 0; w < nwin; ++w) {
    const int wa = p0 + w * WIN, wb = min(p1, wa + WIN), len = wb - wa;
    const int nsw = (len + SUB - 1) / SUB;
    for (int r = 0; r < nsw; ++r, ++q) {  // pass 1: scores of the window
      const Ld L = load_of(q);
      const float *kb = arrive(q, L);
      attn_scores<E, QP>(qs, kb, L.b - L.a, qpk, J.scale, sc + (L.a - wa), WIN);
      release(q);
    }
    {  // softmax of the window for head hw (fixed-order combination of its warps' shares)
      const float *sh = sc + hw * WIN;
      float mw = -INFINITY;
      if (hw < qpk)
        for (int t = part * 32 + lane; t < len; t += 32 * WPH) mw = fmaxf(mw, sh[t]);
      mw = warp_max(mw);
      if (WPH > 1) {
        if (lane == 0) s_red[0][warp] = mw;
        csync();
        mw = -INFINITY;
#pragma unroll
        for (int k = 0; k < WPH; ++k) mw = fmaxf(mw, s_red[0][hw * WPH + k]);
      }
      const float m_new = fmaxf(m, mw);
      float lw = 0.f;
      if (hw < qpk) {
#pragma unroll 1
        for (int t = part * 32 + lane; t < len; t += 32 * WPH) {
          const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(sh[t], m_new))));
          sc[hw * WIN + t] = e;
          lw += e;
        }
      }
      lw = warp_sum(lw);
      if (WPH > 1) {
        if (lane == 0) s_red[1][warp] = lw;
        csync();  // also: every warp's weights are in sc
        lw = 0.f;
#pragma unroll
        for (int k = 0; k < WPH; ++k) lw += s_red[1][hw * WPH + k];
      }
      const float alpha = static_cast<float>(exp(static_cast<double>(m - m_new)));
      l = l * alpha + lw;
      m = m_new;
#pragma unroll
      for (int j = 0; j < E; ++j) acc[j] *= alpha;
      __syncwarp();
    }
    for (int r = 0; r < nsw; ++r, ++q) {  // pass 2: weighted sum of V
      const Ld L = load_of(q);
      const float *vb = arrive(q, L);
      if (hw < qpk) {  // positions t = part, part + WPH, ... of the sub-chunk
        const float *e = sc + hw * WIN + (L.a - wa) + part;
        const float *vbp = vb + part * hd;
        const int n = (L.b - L.a - part + WPH - 1) / WPH;
        // four interleaved partial sums (positions t mod 4), then combined
        float a[4][E];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int j = 0; j < E; ++j) a[u][j] = 0.f;
        int t = 0;
        for (; t + 3 < n; t += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float eu = e[(t + u) * WPH];
            float vu[E];
            lds_vec<E>(vbp + (t + u) * WPH * hd + lane * E, vu);
#pragma unroll
            for (int j = 0; j < E; ++j) a[u][j] = fmaf(eu, vu[j], a[u][j]);
          }
        }
        for (; t < n; ++t) {
          const float et = e[t * WPH];
          float vt[E];
          lds_vec<E>(vbp + t * WPH * hd + lane * E, vt);
#pragma unroll
          for (int j = 0; j < E; ++j) a[0][j] = fmaf(et, vt[j], a[0][j]);
        }
#pragma unroll
        for (int j = 0; j < E; ++j) acc[j] += (a[0][j] + a[1][j]) + (a[2][j] + a[3][j]);
      }
      release(q);
    }
  }
  if (WPH > 1) {  // the shares of head hw's warps, summed in warp order (the buffers are free)
    float *red = buf;
#pragma unroll
    for (int j = 0; j < E; ++j) red[warp * hd + lane * E + j] = acc[j];
    csync();
    if (part == 0)
#pragma unroll
      for (int j = 0; j < E; ++j) {
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < WPH; ++k) a += red[(hw * WPH + k) * hd + lane * E + j];
        acc[j] = a;
      }
    csync();
  }
  const int h0 = J.h0;
  const bool lead = hw < qpk && part == 0;  // the warp that writes head hw
  if (J.nsplit == 1) {  // single split: normalise and write the heads directly
    if (lead)
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const int o = (h0 + hw) * hd + lane * E + j;
        if (J.tout)
          st_tag(J.tout + o, J.tag_out, acc[j] / l);
        else
          J.out[o] = acc[j] / l;
      }
    return ok;
  }
  // partial (m, l, acc) of this split; the last split of the group combines
  if (lead) {
    float *pp = J.part + (static_cast<size_t>(h0 + hw) * J.max_splits + J.s) * (hd + 2);
    if (lane == 0) {
      pp[0] = m;
      pp[1] = l;
    }
#pragma unroll
    for (int j = 0; j < E; ++j) pp[2 + lane * E + j] = acc[j];
  }
  __threadfence();
  csync();
  const int ns = J.nsplit;
  if (tid == 0) {
    if (J.dist) {  // arrive, then wait (bounded) for every split of the group
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(J.counter) : "memory");
      const long long t0 = clock64();
      for (uint32_t it = 0; ld_acquire_gpu_u32(J.counter) < J.cnt_base + static_cast<unsigned>(ns); ++it)
        if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
          atomicOr(err, kErrCounter);
          ok = false;
          break;
        }
      s_last = 1;
    } else {
      const unsigned t = atomicAdd(J.counter, 1u);
      s_last = (t == static_cast<unsigned>(ns - 1)) ? 1 : 0;
    }
  }
  csync();
  if (!s_last) return ok;
  if (!J.dist) __threadfence();  // (dist: thread 0's acquire load and the CTA barrier order the reads)
  // outputs combined here: all of them, or this split's slice
  int o_lo = 0, o_hi = qpk * hd;
  if (J.dist) seg_rows(qpk * hd, J.s, ns, o_lo, o_hi);
  // combine the splits: per (head, split) weight w = exp(m_k - M) once, then
  // each output sums w_k * acc_k[d] over k in split order.  Shared memory
  // (the K/V buffers are free now): [nh][ns] m then w | [nh][ns] l |
  // [qpk * hd] sums | staged partial sums of a block of outputs
  const int hlo = o_lo / hd, nh = (o_hi - 1) / hd + 1 - hlo;  // heads of the outputs
  float *wm = buf, *wl = wm + nh * ns, *Os = wl + nh * ns, *stage = Os + qpk * hd;
  __shared__ float s_L[8];
  auto part_of = [&](int h, int k) {
    return J.part + (static_cast<size_t>(h0 + h) * J.max_splits + k) * (hd + 2);
  };
  const int cap = kAttnBufs * attn_sub(hd) * hd - static_cast<int>(stage - wm);
  const int nbo = max(1, min(o_hi - o_lo, cap / ns));
  // partial sums of outputs [ob, ob + cnt) of every split -> stage[k * cnt + i]
  auto stage_block = [&](int ob, int cnt) {
    const int tot = cnt * ns;
    // t / cnt = umulhi(t, ceil(2^32 / cnt)) for t * cnt < 2^32 (cnt = 1: t)
    const uint32_t magic = cnt > 1 ? 0xFFFFFFFFu / static_cast<uint32_t>(cnt) + 1u : 0u;
    for (int t0 = 0; t0 < tot; t0 += 4 * kThreads) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = t0 + j * kThreads + tid;
        const int k = cnt > 1 ? static_cast<int>(__umulhi(static_cast<uint32_t>(t), magic)) : t;
        const int i = ob + (t - k * cnt), h = i / hd;
        v[j] = t < tot ? __ldcg(part_of(h, k) + 2 + (i - h * hd)) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (t0 + j * kThreads + tid < tot) stage[t0 + j * kThreads + tid] = v[j];
    }
  };
  // one round of L2 loads: every needed (m, l) and the first block's partials
  for (int t = tid; t < nh * ns; t += kThreads) {
    const int hh = t / ns, k = t - hh * ns;
    wm[t] = __ldcg(part_of(hlo + hh, k));
    wl[t] = __ldcg(part_of(hlo + hh, k) + 1);
  }
  stage_block(o_lo, min(nbo, o_hi - o_lo));
  csync();
  if (warp < nh) {  // warp hh: head hlo + hh
    float *w = wm + warp * ns;
    const float *lk = wl + warp * ns;
    float M = -INFINITY;
    for (int k = lane; k < ns; k += 32) M = fmaxf(M, w[k]);
    M = warp_max(M);
    float L = 0.f;
#pragma unroll 1
    for (int k = lane; k < ns; k += 32) {
      const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(w[k], M))));
      w[k] = e;
      L = fmaf(e, lk[k], L);
    }
    L = warp_sum(L);
    if (lane == 0) s_L[warp] = L;
  }
  csync();
  for (int ob = o_lo; ob < o_hi; ob += nbo) {
    const int cnt = min(nbo, o_hi - ob);
    if (ob != o_lo) {
      stage_block(ob, cnt);
      csync();
    }
    for (int i = tid; i < cnt; i += kThreads) {  // each output sums its splits in order
      const float *w = wm + ((ob + i) / hd - hlo) * ns;
      float O = 0.f;
      for (int k = 0; k < ns; ++k) O = fmaf(w[k], stage[k * cnt + i], O);
      Os[ob + i] = O;
    }
    csync();
  }
  for (int i = o_lo + tid; i < o_hi; i += kThreads) {
    const int h = i / hd, o = (h0 + h) * hd + (i - h * hd);
    if (J.tout)
      st_tag(J.tout + o, J.tag_out, Os[i] / s_L[h - hlo]);
    else
      J.out[o] = Os[i] / s_L[h - hlo];
  }
  if (!J.dist && tid == 0) *J.counter = 0;
  return ok;
}

__device__ __forceinline__ bool attend(const AttnJob &J, float *asmem, uint64_t *bars, uint32_t (&uses)[kAttnBufs],
                                       unsigned *err) {
  if (J.qpk == 1)
    return J.hd == 64 ? attend_t<2, 1>(J, asmem, bars, uses, err) : attend_t<4, 1>(J, asmem, bars, uses, err);
  return J.hd == 64 ? attend_t<2, 8>(J, asmem, bars, uses, err) : attend_t<4, 8>(J, asmem, bars, uses, err);
}

__global__ void __launch_bounds__(kThreads) k_attention(const AttnParams A) {
  extern __shared__ __align__(128) float asmem[];
  __shared__ __align__(8) uint64_t bars[kAttnBufs];
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < kAttnBufs; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();
  DevState *st = A.st;
  if (A.check_halt && *reinterpret_cast<volatile int *>(&st->halted)) return;
  const int x = blockIdx.x, s = blockIdx.y;  // x: local query head or kv group, s: split
  const int pos = st->fwd_pos;
  if (pos < 0 || pos >= A.max_tokens) {
    if (tid == 0 && s == 0 && x == 0) atomicOr(&st->err, kErrPos);
    return;
  }
  const int hd = A.hd;
  const AttnLayout AL = attn_layout(pos, A.split_len, A.n_kv, A.tp_h1 - A.tp_h0, A.items_cap);
  if (s >= AL.nsplit || x >= (AL.per_head ? A.tp_h1 - A.tp_h0 : A.n_kv)) return;
  AttnJob J;
  if (!attn_unit(AL, x, A.qpk, A.tp_h0, A.tp_h1, A.tp_g0, st->attn_counter, J)) return;
  // KV layout [L][KVH][max_tokens][hd] per plane (engine/kvcache.go:127-140)
  const size_t head_stride = static_cast<size_t>(A.max_tokens) * hd;
  const size_t off = static_cast<size_t>(A.layer) * A.n_kv * head_stride + J.g * head_stride;
  J.q = A.q + static_cast<size_t>(J.h0) * hd;
  J.k = A.k + J.g * hd;
  J.v = A.v + J.g * hd;
  J.q_norm = A.q_norm;
  J.k_norm = A.k_norm;
  J.kc = A.kcache + off;
  J.vc = A.vcache + off;
  // RoPETable.Apply rejects pos outside the table (tensor/ops.go:263)
  J.rope_cs = pos < A.rope_len ? A.rope_cos + static_cast<size_t>(pos) * (hd / 2) : nullptr;
  J.rope_sn = pos < A.rope_len ? A.rope_sin + static_cast<size_t>(pos) * (hd / 2) : nullptr;
  J.out = A.out;
  J.part = A.part;
  J.dist = 0;  // the CTAs of a launch are not guaranteed to be co-resident
  J.s = s;
  J.nsplit = AL.nsplit;
  J.p0 = s * A.split_len;
  J.p1 = min(pos + 1, J.p0 + A.split_len);
  J.pos = pos;
  J.hd = hd;
  J.max_splits = A.max_splits;
  J.eps = A.eps;
  J.scale = A.scale;
  uint32_t uses[kAttnBufs] = {};
  attend(J, asmem, bars, uses, &st->err);
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
          const int hb = static_cast<int>((qh >> (e < 16 ? k : k + 16)) & 1u);
          q = static_cast<float>((nib | (hb << 4)) - 16);
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


// ---------------------------------------------------------------------------
// Tensor parallel: the residual add after an allreduced o-proj / down partial
// (commit of the forwarded token after the last layer, as the single-GPU
// down epilogue does), and greedy selection over gathered logits.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) k_residual_add(float *X, const float *delta, int n, DevState *st,
                                                           int *token_ids, int commit_here, int check_halt) {
  pdl_wait();
  if (check_halt && *reinterpret_cast<volatile int *>(&st->halted)) return;
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads) X[i] = __fadd_rn(X[i], delta[i]);
  if (commit_here && blockIdx.x == 0 && threadIdx.x == 0 && st->commit) {
    const int pos = st->fwd_pos;
    if (pos >= 0 && pos < st->out_cap) token_ids[pos] = st->fwd_token;  // KVCache.StoreTokenID
    st->seq_len = pos + 1;
    if (st->halt_pending) {
      st->halted = 1;
      st->halt_pending = 0;
    }
  }
}

// Repetition penalty + strict '>' argmax (ties: lowest id) over `vocab`
// logits (c2slm.go:156-180), then the next forward's state.  Each CTA takes
// a contiguous slice into shared memory; the last CTA to finish reduces the
// per-CTA bests.  Same rules and float operations as the logits epilogue of
// k_matvec.
__global__ void __launch_bounds__(kThreads) k_select(const float *logits, int vocab, DevState *st,
                                                     const int *token_ids, int *out_tokens, float2 *part,
                                                     int check_halt) {
  extern __shared__ __align__(16) float ybuf[];
  __shared__ int s_flag;
  __shared__ float s_bv[kWarps];
  __shared__ int s_bi[kWarps];
  pdl_wait();
  if (check_halt && *reinterpret_cast<volatile int *>(&st->halted)) return;
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  int r0, r1;
  seg_rows(vocab, c, G, r0, r1);
  const int n = r1 - r0;
  for (int i = tid; i < n; i += kThreads) ybuf[i] = __ldcg(logits + r0 + i);
  __syncthreads();
  if (tid == 0) {
    const int pos = st->seq_len;
    int start = pos - st->window;
    if (start < 0) start = 0;
    const float pen = st->penalty;
    for (int p = start; p < pos; ++p) {
      const int tok = token_ids[p];
      if (tok >= 0 && tok < st->vocab && tok != st->im_end && tok != st->eos && tok >= r0 && tok < r1) {
        float &v = ybuf[tok - r0];
        v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
      }
    }
  }
  __syncthreads();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < n; i += kThreads) {
    const float v = ybuf[i];
    if (v > bv || (v == bv && r0 + i < bi)) {
      bv = v;
      bi = r0 + i;
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
    part[c] = make_float2(bv, __int_as_float(bi));
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
      const float2 pv = __ldcg(part + k);
      const int pi = __float_as_int(pv.y);
      if (pi == 0x7fffffff) continue;
      if (pv.x > best_v || (pv.x == best_v && pi < best_i) || best_i == 0x7fffffff) {
        best_v = pv.x;
        best_i = pi;
      }
    }
    if (best_i == 0x7fffffff) best_i = 0;
    if (st->n_out < st->out_cap) out_tokens[st->n_out] = best_i;
    st->n_out += 1;
    st->fwd_token = best_i;
    st->fwd_pos = st->seq_len;
    st->commit = 1;
    if (st->stop_on_special && (best_i == st->im_end || best_i == st->eos)) st->halt_pending = 1;
    st->logits_counter = 0;
  }
}

}  // namespace c2s
