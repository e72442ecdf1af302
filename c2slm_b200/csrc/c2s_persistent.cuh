// c2s_persistent.cuh -- the decode loop as one persistent, cooperative kernel.
//
// One CTA per SM (cooperative launch: all CTAs co-resident).  Each CTA runs
// 8 compute warps and 1 producer warp:
//   * the producer walks the same phase schedule as the compute warps and
//     streams the CTA's share of every matvec phase's weights (native GGML
//     blocks) HBM -> shared memory with 1-D TMA bulk copies into an N-slot
//     ring, limited only by free slots -- so the weight stream of the next
//     phases runs while the compute warps wait at grid barriers;
//   * the compute warps execute the phases of a decode step -- logits +
//     penalty + argmax, then per layer QKV, attention, o-proj, gate/up, down --
//     separated by grid barriers (bounded spins on a global counter).
// Instructions stay resident across phases and steps, and no kernel launch or
// teardown sits between phases.
#pragma once
#include "c2s_kernels.cuh"

namespace c2s {

constexpr int kPThreads = kThreads + 32;  // 8 compute warps + 1 producer warp
constexpr int K_ATTN = 7;

struct PPhase {
  int kind;  // K_QKV, K_ATTN, K_OPROJ, K_FFN_UP, K_FFN_DOWN, K_LOGITS
  int layer, nseg, cols;
  Seg seg[kMaxSegs];
  const float *x_in;    // OPROJ: attention output, DOWN: SwiGLU output
  const float *norm_w;  // QKV / FFN_UP / LOGITS
  const float *q_norm, *k_norm;  // ATTN (Qwen3)
  int do_embed, commit_here, need_f32, need_q8k;
};

constexpr int kMaxLayers = 32;

// One layer's tensors, as the persistent kernel needs them.  The whole table
// travels in the kernel's parameter space (constant bank), so building a
// phase descriptor costs no global-memory round trip.
struct PLayer {
  const uint8_t *q, *k, *v, *o, *gate, *up, *down;
  const float *attn_norm, *ffn_norm, *qb, *kb, *vb, *qn, *kn;
  int8_t tq, tk, tv, to, tg, tu, td, pad;
};

struct PParams {
  PLayer layers[kMaxLayers];
  const uint8_t *out_w;
  const float *out_norm;
  int out_type, n_layers, F, kvd, vocab;
  int nphase, n_steps;
  int nslot;
  int off_full, off_empty, off_abar, off_act;
  int off_xn, off_xt, off_q8, off_y, yrows;  // relative to off_act
  int H, n_heads, n_kv, hd, max_tokens, max_splits, rope_len;
  float eps, scale;
  float *X, *normx, *q, *k, *v, *attn_out, *h, *logits, *part;
  float2 *amax_part;
  float *kcache, *vcache;
  const float *rope_cos, *rope_sin;
  const uint8_t *embd_w;
  int embd_type, embd_row_bytes;
  DevState *st;
  int *token_ids, *out_tokens;
  unsigned *gbar;       // grid barrier arrival counter, zero at launch
  int rewind_period;    // > 0: SeqLen returns to rewind_base every period steps
  int rewind_base;
  unsigned long long *trace;  // optional: [step][phase][cta][kTraceFields], see k_persistent
};

// trace record per (step, phase, CTA): globaltimer ns at phase start (after
// the grid barrier), inputs ready, chunks done and end; then SM cycles thread
// 0 spent waiting for weight chunks, in the grid barrier before the phase, in
// the chunk loop, and the cycle counter at phase start.
constexpr int kTraceFields = 8;

__host__ __device__ inline int qrow_bytes(int type, int cols) {
  return type == T_Q5_0 ? (cols / 32) * 22
         : type == T_Q8_0 ? (cols / 32) * 34
         : type == T_Q4_K ? (cols / 256) * 144
         : type == T_Q6_K ? (cols / 256) * 210 : cols * 4;
}

__device__ __forceinline__ Seg pseg(const uint8_t *w, int type, int rows, int cols, const float *bias, float *out) {
  Seg s;
  s.w = w;
  s.type = type;
  s.rows = rows;
  s.row_bytes = qrow_bytes(type, cols);
  s.units = (type == T_Q4_K || type == T_Q6_K) ? (cols / 256) * 4 : cols / 32;
  s.rows_per_chunk = max(1, kStageBytes / s.row_bytes);
  s.bias = bias;
  s.out = out;
  return s;
}

struct PParams;
__device__ void build_phase(const PParams &P, int pi, PPhase &ph);

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// mutable decode state is read through L2 only (no stale L1 lines across steps)
__device__ __forceinline__ int ldst(const int *p) { return __ldcg(p); }
__device__ __forceinline__ float ldstf(const float *p) { return __ldcg(p); }

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Grid-wide barrier of the compute warps: one monotonically increasing
// arrival counter (zeroed at launch).  Thread 0 of each CTA arrives with a
// release add, then polls with acquire loads until all G CTAs of barrier
// number `seq` have arrived.  Bounded (~2 s): on expiry sets the error flag
// and returns false (the caller stops).
__device__ __forceinline__ bool grid_barrier(unsigned *counter, unsigned seq, unsigned *err, int *s_ok) {
  csync();
  if (threadIdx.x == 0) {
    const unsigned target = seq * gridDim.x;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
    int ok = 1;
    const long long t0 = clock64();
    for (uint32_t it = 0; ld_acquire_u32(counter) < target; ++it) {
      if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
        atomicOr(err, kErrCounter);
        ok = 0;
        break;
      }
    }
    *s_ok = ok;
  }
  csync();
  return *s_ok != 0;
}

// chunk enumeration of one phase for CTA c (same on both sides of the ring)
__device__ __forceinline__ int phase_chunks(const PPhase &ph, int c, int G, int (&my0)[kMaxSegs],
                                            int (&my1)[kMaxSegs]) {
  int n = 0;
  for (int s = 0; s < kMaxSegs; ++s) {
    my0[s] = my1[s] = 0;
    if (s < ph.nseg) {
      seg_rows(ph.seg[s].rows, c, G, my0[s], my1[s]);
      const int cpr = ph.seg[s].rows_per_chunk;
      n += (my1[s] - my0[s] + cpr - 1) / cpr;
    }
  }
  return n;
}

__device__ __forceinline__ ChunkRef phase_chunk_at(const PPhase &ph, const int (&my0)[kMaxSegs],
                                                   const int (&my1)[kMaxSegs], int i) {
  ChunkRef c{0, 0, 0};
  for (int s = 0; s < ph.nseg; ++s) {
    const int cpr = ph.seg[s].rows_per_chunk;
    const int nch = (my1[s] - my0[s] + cpr - 1) / cpr;
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

__device__ __forceinline__ void issue_rows(const Seg &S, const ChunkRef &c, uint8_t *slot, uint64_t *bar) {
  const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(c.r0) * S.row_bytes;
  const uintptr_t end = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(c.r1) * S.row_bytes;
  const uintptr_t a0 = src & ~uintptr_t(15);
  const uintptr_t a1 = (end + 15) & ~uintptr_t(15);
  const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s(slot, reinterpret_cast<const void *>(a0), bytes, bar);
}

// Q8_K of a global vector straight into shared memory: each warp takes 2
// superblocks per round with all their loads in flight.
__device__ __forceinline__ void build_q8k_global(const float *src, int cols, int8_t *qs, float *d, int32_t *bsum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = cols / 256;
  for (int sb0 = warp; sb0 < nsb; sb0 += 2 * kWarps) {
    const int sb1 = sb0 + kWarps;
    float4 a0 = make_float4(0, 0, 0, 0), b0 = a0, a1 = a0, b1 = a0;
    a0 = __ldcg(reinterpret_cast<const float4 *>(src + sb0 * 256 + lane * 8));
    b0 = __ldcg(reinterpret_cast<const float4 *>(src + sb0 * 256 + lane * 8 + 4));
    if (sb1 < nsb) {
      a1 = __ldcg(reinterpret_cast<const float4 *>(src + sb1 * 256 + lane * 8));
      b1 = __ldcg(reinterpret_cast<const float4 *>(src + sb1 * 256 + lane * 8 + 4));
    }
    for (int k = 0; k < 2; ++k) {
      const int sb = k ? sb1 : sb0;
      if (sb >= nsb) break;
      const float4 a = k ? a1 : a0, b = k ? b1 : b0;
      float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      quantize_sb_warp(x, d + sb, bsum + sb * 16, [&](int ln, const int (&q)[8]) {
        int8_t *dst = qs + q8_pad_index(sb * 256 + ln * 8);
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
}

// phase pi of a decode step: 0 = logits, then per layer qkv, attn, o-proj,
// gate/up, down
__device__ void build_phase(const PParams &P, int pi, PPhase &ph) {
  auto needs = [&]() {
    ph.need_f32 = 0;
    ph.need_q8k = 0;
    for (int s = 0; s < ph.nseg; ++s) {
      const int t = ph.seg[s].type;
      if (t == T_Q5_0 || t == T_Q8_0) ph.need_f32 = 1;
      if (t == T_Q4_K || t == T_Q6_K) ph.need_q8k = 1;
    }
  };
  ph.x_in = nullptr;
  ph.norm_w = nullptr;
  ph.q_norm = ph.k_norm = nullptr;
  ph.do_embed = ph.commit_here = 0;
  ph.nseg = 0;
  if (pi == 0) {
    ph.kind = K_LOGITS;
    ph.layer = -1;
    ph.nseg = 1;
    ph.cols = P.H;
    ph.seg[0] = pseg(P.out_w, P.out_type, P.vocab, P.H, nullptr, P.logits);
    ph.norm_w = P.out_norm;
    needs();
    return;
  }
  const int l = (pi - 1) / 5, r = (pi - 1) % 5;
  const PLayer &L = P.layers[l];
  ph.layer = l;
  switch (r) {
    case 0:
      ph.kind = K_QKV;
      ph.nseg = 3;
      ph.cols = P.H;
      ph.seg[0] = pseg(L.q, L.tq, P.H, P.H, L.qb, P.q);
      ph.seg[1] = pseg(L.k, L.tk, P.kvd, P.H, L.kb, P.k);
      ph.seg[2] = pseg(L.v, L.tv, P.kvd, P.H, L.vb, P.v);
      ph.norm_w = L.attn_norm;
      ph.do_embed = (l == 0);
      break;
    case 1:
      ph.kind = K_ATTN;
      ph.cols = 0;
      ph.q_norm = L.qn;
      ph.k_norm = L.kn;
      break;
    case 2:
      ph.kind = K_OPROJ;
      ph.nseg = 1;
      ph.cols = P.H;
      ph.seg[0] = pseg(L.o, L.to, P.H, P.H, nullptr, P.X);
      ph.x_in = P.attn_out;
      break;
    case 3:
      ph.kind = K_FFN_UP;
      ph.nseg = 2;
      ph.cols = P.H;
      ph.seg[0] = pseg(L.gate, L.tg, P.F, P.H, nullptr, nullptr);
      ph.seg[1] = pseg(L.up, L.tu, P.F, P.H, nullptr, nullptr);
      ph.norm_w = L.ffn_norm;
      break;
    default:
      ph.kind = K_FFN_DOWN;
      ph.nseg = 1;
      ph.cols = P.F;
      ph.seg[0] = pseg(L.down, L.td, P.H, P.F, nullptr, P.X);
      ph.x_in = P.h;
      ph.commit_here = (l == P.n_layers - 1);
      break;
  }
  needs();
}

// ---------------------------------------------------------------------------
// attention item (kv head g, split s) of the current position; the last
// split of a group combines.  Shared memory: the activation region.
// ---------------------------------------------------------------------------
__device__ void p_attention(const PParams &P, const PPhase &ph, float *asmem, uint64_t *abar, uint32_t (&uses)[2],
                            int item) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  DevState *st = P.st;
  const int hd = P.hd, qpk = P.n_heads / P.n_kv, SUB = attn_sub(hd);
  const int pos = ldst(&st->fwd_pos);
  if (pos < 0 || pos >= P.max_tokens) {
    if (tid == 0 && item == 0) atomicOr(&st->err, kErrPos);
    return;
  }
  const int n = pos + 1;
  const int nsplit = attn_nsplit(n, P.max_splits);
  if (item >= P.n_kv * nsplit) return;
  const int g = item / nsplit, s = item % nsplit;
  const int chunk = (n + nsplit - 1) / nsplit;
  const int p0 = min(n, s * chunk), p1 = min(n, p0 + chunk);
  const size_t head_stride = static_cast<size_t>(P.max_tokens) * hd;
  const size_t layer_stride = static_cast<size_t>(P.n_kv) * head_stride;
  float *kc = P.kcache + static_cast<size_t>(ph.layer) * layer_stride + g * head_stride;
  float *vc = P.vcache + static_cast<size_t>(ph.layer) * layer_stride + g * head_stride;
  float *kbuf = asmem, *vbuf = kbuf + 2 * SUB * hd, *qs = vbuf + 2 * SUB * hd;
  float *knew = qs + qpk * hd, *vnew = knew + hd, *sc = vnew + hd, *acc = sc + qpk * SUB;
  __shared__ float s_m[8], s_l[8], s_scale[8];
  __shared__ int s_last;
  const int n_sub = (p1 - p0 + SUB - 1) / SUB;
  auto issue = [&](int it) {
    const int a = p0 + it * SUB, b = min(p1, a + SUB);
    const int cached = max(0, min(b, pos) - a);
    if (cached > 0) {
      const uint32_t bytes = static_cast<uint32_t>(cached) * hd * 4;
      uint64_t *bar = &abar[it & 1];
      mbar_arrive_expect_tx(bar, 2 * bytes);
      bulk_g2s(kbuf + (it & 1) * SUB * hd, kc + static_cast<size_t>(a) * hd, bytes, bar);
      bulk_g2s(vbuf + (it & 1) * SUB * hd, vc + static_cast<size_t>(a) * hd, bytes, bar);
    }
  };
  // sub-chunks whose cached part is non-empty use (and advance) their buffer's barrier
  auto uses_bar = [&](int it) {
    const int a = p0 + it * SUB, b = min(p1, a + SUB);
    return min(b, pos) - a > 0;
  };
  if (tid == 0) {
    fence_proxy_async();
    issue(0);
    if (n_sub > 1) issue(1);
  }
  for (int i = tid; i < qpk * hd; i += kThreads) {
    qs[i] = __ldcg(P.q + g * qpk * hd + i);
    acc[i] = 0.f;
  }
  for (int i = tid; i < hd; i += kThreads) {
    knew[i] = __ldcg(P.k + g * hd + i);
    vnew[i] = __ldcg(P.v + g * hd + i);
  }
  if (tid < 8) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
  }
  csync();
  if (ph.q_norm)
    for (int h = warp; h < qpk; h += kWarps) head_rmsnorm_warp(qs + h * hd, ph.q_norm, hd, P.eps);
  if (ph.k_norm && warp == kWarps - 1) head_rmsnorm_warp(knew, ph.k_norm, hd, P.eps);
  csync();
  if (pos < P.rope_len) {
    const float *cs = P.rope_cos + static_cast<size_t>(pos) * (hd / 2);
    const float *sn = P.rope_sin + static_cast<size_t>(pos) * (hd / 2);
    for (int h = 0; h < qpk; ++h) rope_rotate(qs + h * hd, hd, cs, sn, tid, kThreads);
    rope_rotate(knew, hd, cs, sn, tid, kThreads);
  }
  csync();
  if (pos >= p0 && pos < p1) {
    for (int i = tid; i < hd; i += kThreads) {
      kc[static_cast<size_t>(pos) * hd + i] = knew[i];
      vc[static_cast<size_t>(pos) * hd + i] = vnew[i];
    }
    fence_proxy_async();  // later TMA reads of this row see it
  }
  const int E = hd / 32;
  float qr[8][4];
#pragma unroll
  for (int h = 0; h < 8; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) qr[h][j] = (h < qpk && j < E) ? qs[h * hd + lane * E + j] : 0.f;
  for (int it = 0; it < n_sub; ++it) {
    const int a = p0 + it * SUB, b = min(p1, a + SUB), len = b - a;
    if (uses_bar(it)) {  // completions of a buffer's barrier alternate parity
      mbar_wait_bounded(&abar[it & 1], uses[it & 1] & 1u, &st->err);
      uses[it & 1] += 1;
    }
    const float *kb = kbuf + (it & 1) * SUB * hd;
    const float *vb = vbuf + (it & 1) * SUB * hd;
    for (int t = warp; t < len; t += kWarps) {
      const float *kp = (a + t == pos) ? knew : kb + t * hd;
      float kv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = j < E ? kp[lane * E + j] : 0.f;
      float dot[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        float d0 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) d0 = fmaf(qr[h][j], kv[j], d0);
        dot[h] = d0;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int h = 0; h < 8; ++h) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], o);
      if (lane < qpk) {
        float v = dot[0];
#pragma unroll
        for (int h = 1; h < 8; ++h) v = (lane == h) ? dot[h] : v;
        sc[lane * SUB + t] = __fmul_rn(v, P.scale);
      }
    }
    csync();
    for (int h = warp; h < qpk; h += kWarps) {
      float m = -INFINITY;
      for (int t = lane; t < len; t += 32) m = fmaxf(m, sc[h * SUB + t]);
      m = warp_max(m);
      const float m_new = fmaxf(s_m[h], m);
      float l = 0.f;
      for (int t = lane; t < len; t += 32) {
        const float e = static_cast<float>(exp(static_cast<double>(__fsub_rn(sc[h * SUB + t], m_new))));
        sc[h * SUB + t] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float scl = static_cast<float>(exp(static_cast<double>(s_m[h] - m_new)));
        s_scale[h] = scl;
        s_l[h] = s_l[h] * scl + l;
        s_m[h] = m_new;
      }
    }
    csync();
    for (int i = tid; i < qpk * hd; i += kThreads) {
      const int h = i / hd, d = i - h * hd;
      const float *e = sc + h * SUB;
      float a0 = 0.f, a1 = 0.f;
      int t = 0;
      for (; t + 1 < len; t += 2) {
        a0 = fmaf(e[t], (a + t == pos) ? vnew[d] : vb[t * hd + d], a0);
        a1 = fmaf(e[t + 1], (a + t + 1 == pos) ? vnew[d] : vb[(t + 1) * hd + d], a1);
      }
      if (t < len) a0 = fmaf(e[t], (a + t == pos) ? vnew[d] : vb[t * hd + d], a0);
      acc[i] = acc[i] * s_scale[h] + (a0 + a1);
    }
    csync();
    if (tid == 0 && it + 2 < n_sub) issue(it + 2);
  }
  const int h0 = g * qpk;
  if (nsplit == 1) {
    for (int i = tid; i < qpk * hd; i += kThreads) {
      const int h = i / hd;
      P.attn_out[(h0 + h) * hd + (i - h * hd)] = acc[i] / s_l[h];
    }
    return;
  }
  for (int i = tid; i < qpk * (hd + 2); i += kThreads) {
    const int h = i / (hd + 2), kk = i - h * (hd + 2);
    float *pp = P.part + (static_cast<size_t>(h0 + h) * P.max_splits + s) * (hd + 2);
    pp[kk] = kk == 0 ? s_m[h] : (kk == 1 ? s_l[h] : acc[h * hd + kk - 2]);
  }
  __threadfence();
  csync();
  if (tid == 0) {
    const unsigned t = atomicAdd(&st->attn_counter[g], 1u);
    s_last = (t == static_cast<unsigned>(nsplit - 1)) ? 1 : 0;
  }
  csync();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < qpk * hd; i += kThreads) {
    const int h = h0 + i / hd, d = i % hd;
    const float *base = P.part + static_cast<size_t>(h) * P.max_splits * (hd + 2);
    float M = -INFINITY;
    for (int kk = 0; kk < nsplit; ++kk) M = fmaxf(M, __ldcg(base + static_cast<size_t>(kk) * (hd + 2)));
    float L = 0.f, O = 0.f;
    for (int kk = 0; kk < nsplit; ++kk) {
      const float *pk = base + static_cast<size_t>(kk) * (hd + 2);
      const float w = static_cast<float>(exp(static_cast<double>(__fsub_rn(__ldcg(pk), M))));
      L = fmaf(w, __ldcg(pk + 1), L);
      O = fmaf(w, __ldcg(pk + 2 + d), O);
    }
    P.attn_out[h * hd + d] = O / L;
  }
  if (tid == 0) st->attn_counter[g] = 0;
}

// ---------------------------------------------------------------------------
// one matvec phase on the compute warps; weights arrive through the ring
// ---------------------------------------------------------------------------
__device__ bool p_matvec(const PParams &P, const PPhase &ph, uint8_t *smem, uint32_t &k_ring, float (*red)[kWarps],
                         float *scratch, int *s_flag, unsigned long long *tr) {
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  DevState *st = P.st;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.off_full);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + P.off_empty);
  uint8_t *act = smem + P.off_act;
  float *xn = reinterpret_cast<float *>(act + P.off_xn);
  float *xt = reinterpret_cast<float *>(act + P.off_xt);
  int8_t *q8qs = reinterpret_cast<int8_t *>(act + P.off_q8);
  float *q8d = reinterpret_cast<float *>(act + P.off_q8 + q8_qs_bytes(ph.cols));
  int32_t *q8bs = reinterpret_cast<int32_t *>(act + P.off_q8 + q8_qs_bytes(ph.cols) + 4 * (ph.cols / 256));
  float *ybuf = reinterpret_cast<float *>(act + P.off_y);
  Q8KView q8{q8qs, q8d, q8bs};
  int my0[kMaxSegs], my1[kMaxSegs];
  const int nchunks = phase_chunks(ph, c, G, my0, my1);
  const bool residual = ph.kind == K_OPROJ || ph.kind == K_FFN_DOWN;
  const bool normed = ph.kind == K_QKV || ph.kind == K_FFN_UP || ph.kind == K_LOGITS;
  // values the epilogue needs, requested first
  float xres = 0.f, bias[kMaxSegs] = {0.f, 0.f, 0.f};
  if (residual && my0[0] + tid < my1[0]) xres = __ldcg(P.X + my0[0] + tid);
  for (int s = 0; s < ph.nseg; ++s)
    if (ph.seg[s].bias && my0[s] + tid < my1[s]) bias[s] = __ldg(ph.seg[s].bias + my0[s] + tid);
  const int nbx = ph.cols / 32;
  // ---- input vector
  if (normed) {
    // norm weights of this thread's elements, requested with the activation
    float nwr[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int e = tid + k * kThreads;
      nwr[k] = e < ph.cols ? __ldg(ph.norm_w + e) : 0.f;
    }
    if (ph.kind == K_QKV && ph.do_embed) {
      int tok = ldst(&st->fwd_token);
      if (tok < 0 || tok >= st->vocab) tok = 0;  // engine/model.go:222-224
      dequant_row_cta(P.embd_type, P.embd_w + static_cast<size_t>(tok) * P.embd_row_bytes, xn, ph.cols);
      csync();
      if (c == 0)
        for (int i = tid; i < ph.cols; i += kThreads) P.X[i] = xn[i];
    } else {
      load_vec_to_smem(xn, P.X, ph.cols);
      csync();
    }
    // RMSNorm (tensor/ops.go:207-218); norm weights come from L2
    float ss0 = 0.f, ss1 = 0.f;
    int i = tid;
    for (; i + kThreads < ph.cols; i += 2 * kThreads) {
      ss0 = fmaf(xn[i], xn[i], ss0);
      ss1 = fmaf(xn[i + kThreads], xn[i + kThreads], ss1);
    }
    if (i < ph.cols) ss0 = fmaf(xn[i], xn[i], ss0);
    const float ss = block_sum(ss0 + ss1, scratch);
    const float mean = __fadd_rn(__fdiv_rn(ss, static_cast<float>(ph.cols)), P.eps);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(mean)));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int e = tid + k * kThreads;
      if (e < ph.cols) xn[e] = __fmul_rn(__fmul_rn(xn[e], inv), nwr[k]);
    }
    csync();
    if (ph.kind == K_LOGITS && c == 0)
      for (int kk = tid; kk < ph.cols; kk += kThreads) P.normx[kk] = xn[kk];
    if (ph.need_f32)
      for (int kk = tid; kk < ph.cols; kk += kThreads) xt[(kk & 31) * nbx + (kk >> 5)] = xn[kk];
    if (ph.need_q8k) build_q8k(xn, ph.cols, q8qs, q8d, q8bs);
  } else {
    if (ph.need_f32) {
      load_vec_to_smem(xn, ph.x_in, ph.cols);
      csync();
      for (int kk = tid; kk < ph.cols; kk += kThreads) xt[(kk & 31) * nbx + (kk >> 5)] = xn[kk];
    }
    if (ph.need_q8k) build_q8k_global(ph.x_in, ph.cols, q8qs, q8d, q8bs);
  }
  csync();
  XLimbs xl;
  const bool xreg = ph.need_f32 && nbx <= 32;
  if (xreg) lane_limbs(xt, nbx, xl);
  if (tr) tr[1] = globaltimer_ns();
  // ---- chunks from the ring
  long long wait_cyc = 0;
  const long long loop_t0 = tr ? clock64() : 0;
  for (int i = 0; i < nchunks; ++i, ++k_ring) {
    const int slot = static_cast<int>(k_ring % static_cast<uint32_t>(P.nslot));
    const uint32_t parity = (k_ring / static_cast<uint32_t>(P.nslot)) & 1u;
    if (tid == 0) {
      const long long w0 = tr ? clock64() : 0;
      *s_flag = mbar_wait_bounded(&full[slot], parity, &st->err) ? 1 : 0;
      if (tr) wait_cyc += clock64() - w0;
    }
    csync();
    if (!*s_flag) return false;
    const ChunkRef ch = phase_chunk_at(ph, my0, my1, i);
    const Seg &S = ph.seg[ch.seg];
    const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(ch.r0) * S.row_bytes;
    const uint8_t *rows = smem + static_cast<size_t>(slot) * kStageAlloc + (src & 15);
    MatParams dummy{};
    compute_chunk(dummy, S, rows, ch.r1 - ch.r0, ch.r0, xt, nbx, q8,
                  ybuf + ch.seg * P.yrows + (ch.r0 - my0[ch.seg]), red, xl, xreg);
    csync();
    if (tid == 0) mbar_arrive(&empty[slot]);
  }
  if (tr) {
    tr[2] = globaltimer_ns();
    tr[4] = static_cast<unsigned long long>(wait_cyc);
    tr[6] = static_cast<unsigned long long>(clock64() - loop_t0);
  }
  // ---- epilogue
  if (ph.kind == K_QKV) {
    for (int s = 0; s < ph.nseg; ++s)
      if (my0[s] + tid < my1[s])
        ph.seg[s].out[my0[s] + tid] = __fadd_rn(ybuf[s * P.yrows + tid], bias[s]);
  } else if (residual) {
    if (my0[0] + tid < my1[0]) P.X[my0[0] + tid] = __fadd_rn(xres, ybuf[tid]);
    if (ph.kind == K_FFN_DOWN && ph.commit_here && c == 0 && tid == 0 && ldst(&st->commit)) {
      const int pos = ldst(&st->fwd_pos);
      if (pos >= 0 && pos < st->out_cap) P.token_ids[pos] = ldst(&st->fwd_token);  // KVCache.StoreTokenID
      st->seq_len = pos + 1;
      if (ldst(&st->halt_pending)) {
        st->halted = 1;
        st->halt_pending = 0;
      }
    }
  } else if (ph.kind == K_FFN_UP) {
    // SwiGLU (internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19), float64 exp
    if (my0[0] + tid < my1[0]) {
      const double g = static_cast<double>(ybuf[tid]);
      const float silu = static_cast<float>(g / (1.0 + exp(-g)));
      P.h[my0[0] + tid] = __fmul_rn(silu, ybuf[P.yrows + tid]);
    }
  } else if (ph.kind == K_LOGITS) {
    const int n = my1[0] - my0[0];
    for (int r = tid; r < n; r += kThreads) P.logits[my0[0] + r] = ybuf[r];
    // the penalty window's ids, fetched in parallel
    __shared__ int win[kThreads];
    const int wpos = ldst(&st->seq_len);
    const int wlen = max(0, min(st->window, wpos));
    if (tid < wlen) win[tid] = ldst(P.token_ids + wpos - wlen + tid);
    csync();
    if (tid == 0) {  // repetition penalty on this CTA's rows (c2slm.go:156-170)
      const int pos = wpos;
      int start = pos - st->window;
      if (start < 0) start = 0;
      const float pen = st->penalty;
      for (int p = start; p < pos; ++p) {
        const int k = p - (pos - wlen);
        const int tok = k < kThreads ? win[k] : ldst(P.token_ids + p);
        if (tok >= 0 && tok < st->vocab && tok != st->im_end && tok != st->eos && tok >= my0[0] && tok < my1[0]) {
          float &v = ybuf[tok - my0[0]];
          v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
        }
      }
    }
    csync();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = tid; r < n; r += kThreads) {
      const float v = ybuf[r];
      if (v > bv || (v == bv && my0[0] + r < bi)) {
        bv = v;
        bi = my0[0] + r;
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
      red[0][tid >> 5] = bv;
      red[1][tid >> 5] = __int_as_float(bi);
    }
    csync();
    if (tid == 0) {
      for (int w = 1; w < kWarps; ++w) {
        const float v = red[0][w];
        const int ix = __float_as_int(red[1][w]);
        if (v > bv || (v == bv && ix < bi)) {
          bv = v;
          bi = ix;
        }
      }
      P.amax_part[c] = make_float2(bv, __int_as_float(bi));
      __threadfence();
      const unsigned t = atomicAdd(&st->logits_counter, 1u);
      *s_flag = (t == static_cast<unsigned>(G - 1)) ? 1 : 0;
    }
    csync();
    if (*s_flag) {  // the last CTA reduces the G partials (ties: lowest id)
      __threadfence();
      float best_v = -INFINITY;
      int best_i = 0x7fffffff;
      for (int kk = tid; kk < G; kk += kThreads) {
        const float2 pv = __ldcg(P.amax_part + kk);
        const int pi = __float_as_int(pv.y);
        if (pi != 0x7fffffff && (pv.x > best_v || (pv.x == best_v && pi < best_i) || best_i == 0x7fffffff)) {
          best_v = pv.x;
          best_i = pi;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (oi != 0x7fffffff && (best_i == 0x7fffffff || ov > best_v || (ov == best_v && oi < best_i))) {
          best_v = ov;
          best_i = oi;
        }
      }
      csync();
      if ((tid & 31) == 0) {
        red[0][tid >> 5] = best_v;
        red[1][tid >> 5] = __int_as_float(best_i);
      }
      csync();
    }
    if (*s_flag && tid == 0) {
      float best_v = red[0][0];
      int best_i = __float_as_int(red[1][0]);
      for (int w = 1; w < kWarps; ++w) {
        const float v = red[0][w];
        const int ix = __float_as_int(red[1][w]);
        if (ix != 0x7fffffff && (best_i == 0x7fffffff || v > best_v || (v == best_v && ix < best_i))) {
          best_v = v;
          best_i = ix;
        }
      }
      if (best_i == 0x7fffffff) best_i = 0;
      const int n_out = ldst(&st->n_out);
      if (n_out < st->out_cap) P.out_tokens[n_out] = best_i;
      st->n_out = n_out + 1;
      st->fwd_token = best_i;
      st->fwd_pos = ldst(&st->seq_len);
      st->commit = 1;
      if (st->stop_on_special && (best_i == st->im_end || best_i == st->eos)) st->halt_pending = 1;
      st->logits_counter = 0;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kPThreads, 1) k_persistent(const PParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kWarps][kWarps];
  __shared__ float scratch[kWarps];
  __shared__ int s_flag, s_ok;
  __shared__ volatile int s_stop;
  __shared__ PPhase s_ph, s_pph;  // current phase: compute side / producer side
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.off_full);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + P.off_empty);
  uint64_t *abar = reinterpret_cast<uint64_t *>(smem + P.off_abar);
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  DevState *st = P.st;
  if (tid == 0) {
    for (int i = 0; i < P.nslot; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&abar[0], 1);
    mbar_init(&abar[1], 1);
    fence_mbar_init();
    s_stop = 0;
  }
  __syncthreads();

  if (tid >= kThreads) {
    // ------------------------------------------------------------ producer
    if (tid != kThreads) return;
    uint32_t k = 0;
    bool stopped = false;
    for (int step = 0; step < P.n_steps && !stopped; ++step) {
      for (int pi = 0; pi < P.nphase && !stopped; ++pi) {
        build_phase(P, pi, s_pph);
        const PPhase &ph = s_pph;
        if (ph.kind == K_ATTN) continue;
        int my0[kMaxSegs], my1[kMaxSegs];
        const int nch = phase_chunks(ph, c, G, my0, my1);
        for (int i = 0; i < nch; ++i, ++k) {
          const int slot = static_cast<int>(k % static_cast<uint32_t>(P.nslot));
          const uint32_t use = k / static_cast<uint32_t>(P.nslot);
          if (use > 0) {  // wait until the compute warps released the slot
            const uint32_t par = (use - 1) & 1u;
            bool ok = mbar_try_wait(&empty[slot], par);
            const long long t0 = clock64();
            for (uint32_t it = 0; !ok; ++it) {
              if (s_stop) { stopped = true; break; }
              ok = mbar_try_wait(&empty[slot], par);
              if (!ok && (it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
                atomicOr(&st->err, kErrMbarTimeout);
                stopped = true;
                break;
              }
            }
            if (stopped) break;
          }
          issue_rows(ph.seg[phase_chunk_at(ph, my0, my1, i).seg], phase_chunk_at(ph, my0, my1, i),
                     smem + static_cast<size_t>(slot) * kStageAlloc, &full[slot]);
        }
      }
    }
    // drain: wait (bounded) for the compute side to stop, then for every copy
    // issued but not consumed, before the CTA exits
    {
      const long long t0 = clock64();
      for (uint32_t it = 0; !s_stop; ++it)
        if ((it & 255u) == 255u && clock64() - t0 > 2 * kSpinCycles) {
          atomicOr(&st->err, kErrMbarTimeout);
          break;
        }
    }
    const uint32_t consumed_to = s_stop ? static_cast<uint32_t>(s_flag) : 0u;  // set by the compute side at exit
    for (uint32_t j = consumed_to; j < k; ++j)
      mbar_wait_bounded(&full[j % static_cast<uint32_t>(P.nslot)], (j / static_cast<uint32_t>(P.nslot)) & 1u,
                        &st->err);
    return;
  }

  // -------------------------------------------------------------- compute
  uint32_t k_ring = 0;
  uint32_t abar_uses[2] = {0, 0};
  unsigned bar_target = 0;
  bool ok = true;
  for (int step = 0; step < P.n_steps && ok; ++step) {
    for (int pi = 0; pi < P.nphase && ok; ++pi) {
      if (tid == 0) build_phase(P, pi, s_ph);
      csync();
      const PPhase &ph = s_ph;
      const long long b0 = P.trace ? clock64() : 0;
      if (step > 0 || pi > 0) {
        bar_target += 1;
        if (!grid_barrier(P.gbar, bar_target, &st->err, &s_ok)) { ok = false; break; }
      }
      if (pi == 0 && ldst(&st->halted)) { ok = false; break; }
      unsigned long long *tr =
          (P.trace && tid == 0)
              ? P.trace + ((static_cast<size_t>(step) * P.nphase + pi) * G + c) * kTraceFields
              : nullptr;
      if (tr) {
        const long long b1 = clock64();
        tr[0] = globaltimer_ns();
        tr[5] = static_cast<unsigned long long>(b1 - b0);
        tr[7] = static_cast<unsigned long long>(b1);
      }
      if (ph.kind == K_ATTN) {
        p_attention(P, ph, reinterpret_cast<float *>(smem + P.off_act), abar, abar_uses, c);
      } else {
        if (!p_matvec(P, ph, smem, k_ring, red, scratch, &s_flag, tr)) { ok = false; break; }
      }
      csync();
      if (tr) tr[3] = globaltimer_ns();
      // bench rewind: the down phase of the last layer set SeqLen = pos + 1
      if (ph.kind == K_FFN_DOWN && ph.commit_here && P.rewind_period > 0 && c == 0 && tid == 0 &&
          (step + 1) % P.rewind_period == 0)
        st->seq_len = P.rewind_base;
    }
  }
  // tell the producer where consumption stopped, then let it drain
  csync();
  if (tid == 0) {
    s_flag = static_cast<int>(k_ring);
    __threadfence_block();
    s_stop = 1;
  }
}

}  // namespace c2s
