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
  int out_type, n_layers, F, kvd, vocab;  // F, kvd: this rank's rows (the model's on one GPU)
  int qrows, vrows;                        // this rank's attn_q rows and vocabulary rows
  int nphase, n_steps;
  int nslot;
  int lng;  // phases with many rows per CTA: the compute warps form 2^lng groups (kWarps >> lng warps each)
  int off_full, off_empty, off_abar, off_act;
  int off_xn, off_limbs, off_q8, off_y, yrows;  // relative to off_act
  int slot_bytes, slot_alloc;  // weight ring: payload per slot, slot stride
  int H, n_heads, n_kv, hd, max_tokens, max_splits, split_len, rope_len;
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
  int phase0;           // 0: a step starts with logits + selection; 1: with the forward
                        // of the token in DevState (the last phase is then logits)
  unsigned long long *trace;  // optional: [step][phase][cta][kTraceFields], see k_persistent
  // tensor parallel over `world` GPUs (world == 1: everything below unused).
  // n_kv is then this rank's kv heads (global ids tp_g0 ..), q rows start at
  // query head tp_h0, vocabulary rows at tp_v0; qpk = the model's query heads
  // per kv head.  Exchanges between ranks are tagged 64-bit words (tag << 32 |
  // value bits) stored straight into every rank's buffers over NVLink: a
  // reader polls the words themselves until each carries the expected tag, so
  // no barrier or fence crosses GPUs.  Tags count the exchanges over the
  // engine's lifetime (DevState::xbar), so buffers are never reset.
  //   recv   [2][world][H]       o-proj / down partial rows (parity: o-proj 0, down 1)
  //   argbuf [2][world][G][2]    per-CTA argmax (value, id) of the logits (parity: step)
  // The next normed phase adds the received partials to the residual
  // xbuf[2][H] (each CTA stores its share of the new residual).
  int world, rank, qpk, tp_h0, tp_h1, tp_g0, tp_v0;
  // 1: o-proj / down hand their output rows to the next phase as tagged words
  // instead of a grid barrier and X (the tensor-parallel exchange; on one GPU
  // the barrier is faster)
  int ll;
  float *xbuf;
  const unsigned long long *recv, *argbuf;
  unsigned long long *peer_recv[8], *peer_arg[8];
  // dataflow hand-off (one GPU): no grid barrier between phases.  Every
  // phase writes its output as tagged 64-bit words (tag << 32 | value bits)
  // with the tag of its phase, tag(kp) = tag0 + kp + 1 (kp counts the
  // launch's phases; the host advances tag0 past every tag a launch can
  // write, so a stale word never matches), and the next phase polls the
  // words it reads until they carry the previous phase's tag.  Each phase
  // reads the output of the phase just before it, so the poll is the only
  // wait.  Buffers: tX[H] residual (o-proj, down), tq/tk/tv (QKV), tatt
  // (attention), th[F] (gate/up: SwiGLU output), tsel[0] the selected
  // token (logits), tsel[1] the forward's commit (down of the last layer,
  // CTA 0), which also publishes the state it wrote before it.
  int df;
  unsigned tag0;
  unsigned long long *tX, *tq, *tk, *tv, *tatt, *th, *tsel;
};
constexpr int kMaxRanks = 8;

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

__device__ __forceinline__ Seg pseg(const uint8_t *w, int type, int rows, int cols, const float *bias, float *out,
                                    int slot_bytes) {
  Seg s;
  s.w = w;
  s.type = type;
  s.rows = rows;
  s.row_bytes = qrow_bytes(type, cols);
  s.units = (type == T_Q4_K || type == T_Q6_K) ? (cols / 256) * 4 : cols / 32;
  s.rows_per_chunk = max(1, slot_bytes / s.row_bytes);
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

// tagged words: single-copy atomic 64-bit stores / loads at system scope
__device__ __forceinline__ void st_tagged(unsigned long long *p, unsigned tag, uint32_t bits) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"((static_cast<unsigned long long>(tag) << 32) | bits)
               : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Sum over ranks (in rank order) of element i .. i+3 of the tagged partial
// rows recv[par][r][*], polling until every word carries `tag`.  Bounded
// (~2 s): on expiry sets the error flag and returns zeros with *ok cleared.
__device__ __forceinline__ float4 sum_tagged4(const PParams &P, int par, int i, unsigned tag, unsigned *err,
                                              bool &ok) {
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  const unsigned long long *base = P.recv + static_cast<size_t>(par) * P.world * P.H + i;
  for (int r0 = 0; r0 < P.world; r0 += 2) {
    const int nr = min(2, P.world - r0);
    unsigned long long w[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) w[j][e] = j < nr ? ld_tagged(base + static_cast<size_t>(r0 + j) * P.H + e) : 0ull;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
      bool all = true;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (j < nr && static_cast<unsigned>(w[j][e] >> 32) != tag) {
            all = false;
            w[j][e] = ld_tagged(base + static_cast<size_t>(r0 + j) * P.H + e);
          }
      if (all) break;
      if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
        atomicOr(err, kErrCounter);
        ok = false;
        return make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (j < nr) {
        if (r0 + j == 0) {
          o = make_float4(__uint_as_float(static_cast<uint32_t>(w[j][0])), __uint_as_float(static_cast<uint32_t>(w[j][1])),
                          __uint_as_float(static_cast<uint32_t>(w[j][2])), __uint_as_float(static_cast<uint32_t>(w[j][3])));
        } else {
          o.x = __fadd_rn(o.x, __uint_as_float(static_cast<uint32_t>(w[j][0])));
          o.y = __fadd_rn(o.y, __uint_as_float(static_cast<uint32_t>(w[j][1])));
          o.z = __fadd_rn(o.z, __uint_as_float(static_cast<uint32_t>(w[j][2])));
          o.w = __fadd_rn(o.w, __uint_as_float(static_cast<uint32_t>(w[j][3])));
        }
      }
  }
  return o;
}

// Q8_K of a global vector straight into shared memory: warp w quantises
// superblocks w, w + kWarps, ..., kPer at a time, the loads of the next kPer
// in flight while the current ones are quantised.
__device__ __forceinline__ void build_q8k_global(const float *src, int cols, int8_t *qs, float *d, int32_t *bsum) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = cols / 256;
  constexpr int kPer = 4;  // superblocks per warp per round
  float4 a[kPer], b[kPer];
  auto load = [&](int base) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int sb = base + warp + k * kWarps;
      a[k] = b[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (sb < nsb) {
        a[k] = __ldcg(reinterpret_cast<const float4 *>(src + sb * 256 + lane * 8));
        b[k] = __ldcg(reinterpret_cast<const float4 *>(src + sb * 256 + lane * 8 + 4));
      }
    }
  };
  load(0);
  for (int base = 0; base < nsb; base += kPer * kWarps) {
    float x[kPer][8];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      x[k][0] = a[k].x, x[k][1] = a[k].y, x[k][2] = a[k].z, x[k][3] = a[k].w;
      x[k][4] = b[k].x, x[k][5] = b[k].y, x[k][6] = b[k].z, x[k][7] = b[k].w;
    }
    if (base + kPer * kWarps < nsb) load(base + kPer * kWarps);
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int sb = base + warp + k * kWarps;
      if (sb >= nsb) break;
      quantize_sb_warp(x[k], d + sb, bsum + sb * 16, [&](int ln, const int (&q)[8]) {
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

// Q8_K of a tagged global vector (the dataflow hand-off of h) into shared
// memory: warp w quantises superblocks w, w + kWarps, ..., each polled until
// every word carries `tag`.  False if a poll gave up (error flag set).
__device__ __noinline__ bool build_q8k_tagged(const unsigned long long *src, unsigned tag, int cols, int8_t *qs,
                                              float *d, int32_t *bsum, unsigned *err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsb = cols / 256;
  bool ok = true;
  for (int sb = warp; sb < nsb; sb += kWarps) {
    float x[8];
    ok = poll_block8(src + sb * 256 + lane * 8, tag, x, err) && ok;
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
  return ok;
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
    ph.seg[0] = pseg(P.out_w, P.out_type, P.vrows, P.H, nullptr, P.logits, P.slot_bytes);
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
      ph.seg[0] = pseg(L.q, L.tq, P.qrows, P.H, L.qb, P.q, P.slot_bytes);
      ph.seg[1] = pseg(L.k, L.tk, P.kvd, P.H, L.kb, P.k, P.slot_bytes);
      ph.seg[2] = pseg(L.v, L.tv, P.kvd, P.H, L.vb, P.v, P.slot_bytes);
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
      ph.cols = P.qrows;
      ph.seg[0] = pseg(L.o, L.to, P.H, P.qrows, nullptr, P.X, P.slot_bytes);
      ph.x_in = P.attn_out;
      break;
    case 3:
      ph.kind = K_FFN_UP;
      ph.nseg = 2;
      ph.cols = P.H;
      ph.seg[0] = pseg(L.gate, L.tg, P.F, P.H, nullptr, nullptr, P.slot_bytes);
      ph.seg[1] = pseg(L.up, L.tu, P.F, P.H, nullptr, nullptr, P.slot_bytes);
      ph.norm_w = L.ffn_norm;
      break;
    default:
      ph.kind = K_FFN_DOWN;
      ph.nseg = 1;
      ph.cols = P.F;
      ph.seg[0] = pseg(L.down, L.td, P.H, P.F, nullptr, P.X, P.slot_bytes);
      ph.x_in = P.h;
      ph.commit_here = (l == P.n_layers - 1);
      break;
  }
  needs();
}

// ---------------------------------------------------------------------------
// attention: CTA c takes item c = (kv head g, split s) of the step's position
// (read, with its RoPE row, during the logits phase).  Splits are fixed
// position ranges, so the CTA that stores a cache row is the one that reads
// it in later steps.
// ---------------------------------------------------------------------------
template <bool DF>
__device__ bool p_attention(const PParams &P, const PPhase &ph, float *asmem, uint64_t *abar, uint32_t (&uses)[kAttnBufs],
                            int item, int pos, const float *rope_row, unsigned tag_in, unsigned tag_out,
                            const unsigned *cbase) {
  DevState *st = P.st;
  if (pos < 0 || pos >= P.max_tokens) {
    if (threadIdx.x == 0 && item == 0) atomicOr(&st->err, kErrPos);
    return true;
  }
  const int hd = P.hd;
  const AttnLayout AL = attn_layout(pos, P.split_len, P.n_kv, P.tp_h1 - P.tp_h0, static_cast<int>(gridDim.x));
  if (item >= AL.n_items) return true;
  // item = (unit x, split s), split-major
  const int nx = AL.per_head ? P.tp_h1 - P.tp_h0 : P.n_kv;
  const int x = item % nx, s = item / nx;
  AttnJob J;
  if (!attn_unit(AL, x, P.qpk, P.tp_h0, P.tp_h1, P.tp_g0, st->attn_counter, J)) return true;
  const size_t head_stride = static_cast<size_t>(P.max_tokens) * hd;
  const size_t off = (static_cast<size_t>(ph.layer) * P.n_kv + J.g) * head_stride;
  J.q = P.q + static_cast<size_t>(J.h0) * hd;
  J.k = P.k + J.g * hd;
  J.v = P.v + J.g * hd;
  J.q_norm = ph.q_norm;
  J.k_norm = ph.k_norm;
  J.kc = P.kcache + off;
  J.vc = P.vcache + off;
  J.rope_cs = pos < P.rope_len ? rope_row : nullptr;
  J.rope_sn = pos < P.rope_len ? rope_row + hd / 2 : nullptr;
  J.out = P.attn_out;
  J.part = P.part;
  J.dist = 1;  // cooperative launch: all CTAs are resident
  J.s = s;
  J.nsplit = AL.nsplit;
  J.p0 = s * P.split_len;
  J.p1 = min(pos + 1, J.p0 + P.split_len);
  J.pos = pos;
  J.hd = hd;
  J.max_splits = P.max_splits;
  J.eps = P.eps;
  J.scale = P.scale;
  if (DF) {  // inputs and outputs as tagged words; split arrivals counted over the launch
    J.tq = P.tq + static_cast<size_t>(J.h0) * hd;
    J.tk = P.tk + J.g * hd;
    J.tv = P.tv + J.g * hd;
    J.tout = P.tatt;
    J.tag_in = tag_in;
    J.tag_out = tag_out;
    J.cnt_base = cbase[x];
  }
  return attend(J, asmem, abar, uses, &st->err);
}

// ---------------------------------------------------------------------------
// one matvec phase on the compute warps; weights arrive through the ring
// ---------------------------------------------------------------------------
struct PhaseRows {
  int r0[kMaxSegs], r1[kMaxSegs];
  // packed: the rows of all segments fit one ring slot and travel as one
  // chunk (one copy per segment, segment s at byte off[s] of the slot)
  int packed, total;
  int off[kMaxSegs];
};

// 16-B aligned byte span [a0, a1) of rows r0 .. r1-1 of a segment
__device__ __forceinline__ void seg_span(const Seg &S, int r0, int r1, uintptr_t &a0, uintptr_t &a1) {
  const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(r0) * S.row_bytes;
  a0 = src & ~uintptr_t(15);
  a1 = (src + static_cast<uintptr_t>(r1 - r0) * S.row_bytes + 15) & ~uintptr_t(15);
}

// chunk i of the phase for this CTA: segment, first row, row count, offset
// of the first row in the CTA's rows of that segment (same enumeration on
// both sides of the ring)
struct PChunk {
  int seg, r0, nr, lr0;
};

__device__ __forceinline__ int phase_rows(const PPhase &ph, int c, int G, int slot_bytes, PhaseRows &R) {
  int n = 0, total = 0;
#pragma unroll
  for (int s = 0; s < kMaxSegs; ++s) {
    R.r0[s] = R.r1[s] = 0;
    R.off[s] = total;
    if (s < ph.nseg) {
      seg_rows(ph.seg[s].rows, c, G, R.r0[s], R.r1[s]);
      const int cpr = ph.seg[s].rows_per_chunk;
      n += (R.r1[s] - R.r0[s] + cpr - 1) / cpr;
      if (R.r1[s] > R.r0[s]) {
        uintptr_t a0, a1;
        seg_span(ph.seg[s], R.r0[s], R.r1[s], a0, a1);
        total += static_cast<int>(a1 - a0);
      }
    }
  }
  R.total = total;
  R.packed = (ph.nseg > 1 && n > 1 && total <= slot_bytes) ? 1 : 0;
  return R.packed ? 1 : n;
}

__device__ __forceinline__ PChunk phase_chunk(const PPhase &ph, const PhaseRows &R, int i) {
  PChunk c{0, 0, 0, 0};
  bool found = false;
#pragma unroll
  for (int s = 0; s < kMaxSegs; ++s) {
    if (!found && s < ph.nseg) {
      const int cpr = ph.seg[s].rows_per_chunk;
      const int nch = (R.r1[s] - R.r0[s] + cpr - 1) / cpr;
      if (i < nch) {
        c.seg = s;
        c.lr0 = i * cpr;
        c.r0 = R.r0[s] + c.lr0;
        c.nr = min(R.r1[s], c.r0 + cpr) - c.r0;
        found = true;
      } else {
        i -= nch;
      }
    }
  }
  return c;
}

__device__ __forceinline__ void issue_chunk_rows(const Seg &S, const PChunk &c, uint8_t *slot, uint64_t *bar) {
  const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(c.r0) * S.row_bytes;
  const uintptr_t end = src + static_cast<uintptr_t>(c.nr) * S.row_bytes;
  const uintptr_t a0 = src & ~uintptr_t(15);
  const uintptr_t a1 = (end + 15) & ~uintptr_t(15);
  const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s(slot, reinterpret_cast<const void *>(a0), bytes, bar);
}

// bounded wait of one warp on a ring slot; false on timeout (error flag set)
__device__ __forceinline__ bool warp_wait_full(uint64_t *bar, uint32_t parity, unsigned *err) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_bounded(bar, parity, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <bool DF>
__device__ bool p_matvec(const PParams &P, const PPhase &ph, uint8_t *smem, uint32_t &k_ring, float (*red)[kWarps],
                         float *scratch, int *s_flag, int *s_pos, float *s_rope, unsigned long long *tr,
                         unsigned &xb, bool from_X, unsigned tag_in, unsigned tag_out, int step, int *s_halt) {
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  DevState *st = P.st;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.off_full);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + P.off_empty);
  uint8_t *act = smem + P.off_act;
  const int cols = ph.cols, nb = cols / 32, nsb = cols / 256;
  float *xn = reinterpret_cast<float *>(act + P.off_xn);
  int *la = reinterpret_cast<int *>(act + P.off_limbs);
  int *lb = la + 8 * nb, *lc = lb + 8 * nb;
  float *ls = reinterpret_cast<float *>(lc + 8 * nb);
  int8_t *q8qs = reinterpret_cast<int8_t *>(act + P.off_q8);
  float *q8d = reinterpret_cast<float *>(act + P.off_q8 + q8_qs_bytes(cols));
  int32_t *q8bs = reinterpret_cast<int32_t *>(act + P.off_q8 + q8_qs_bytes(cols) + ((4 * nsb + 15) & ~15));
  float *ybuf = reinterpret_cast<float *>(act + P.off_y);
  const LimbsView LV{la, lb, lc, ls, nb};
  const Q8KView q8{q8qs, q8d, q8bs};
  PhaseRows R;
  const int nchunks = phase_rows(ph, c, G, P.slot_bytes, R);
  // the attention's split arrivals of this layer: every split has finished
  // waiting on them before the grid barrier this phase follows (dataflow:
  // the counters accumulate over the launch instead)
  if (!DF && ph.kind == K_OPROJ && tid == 0 && c < 64) st->attn_counter[c] = 0;
  // dataflow: this phase's input is the previous phase's tagged output (the
  // first phase of a launch reads the plain buffers the host or the last
  // launch left)
  const bool dfi = DF && !from_X;
  const bool residual = ph.kind == K_OPROJ || ph.kind == K_FFN_DOWN;
  const bool normed = ph.kind == K_QKV || ph.kind == K_FFN_UP || ph.kind == K_LOGITS;
  // ---- loads the epilogue needs, requested first
  float xres = 0.f, bias[kMaxSegs] = {0.f, 0.f, 0.f};
  // (the dataflow kernel is the one-GPU specialisation: no tensor-parallel paths)
  const bool tp = !DF && P.world > 1, ll = !DF && P.ll != 0;
  if (residual && !ll && R.r0[0] + tid < R.r1[0]) xres = __ldcg(P.X + R.r0[0] + tid);
#pragma unroll
  for (int s = 0; s < kMaxSegs; ++s)
    if (s < ph.nseg && ph.seg[s].bias && R.r0[s] + tid < R.r1[s]) bias[s] = __ldg(ph.seg[s].bias + R.r0[s] + tid);
  __shared__ int win[kThreads];
  __shared__ int s_fail, s_tok;
  auto read_window = [&]() {
    // SeqLen = the position this step forwards; the penalty window's ids and
    // the RoPE row of that position (kept in shared memory for the step)
    const int wpos = ldst(&st->seq_len);
    const int wlen = max(0, min(st->window, wpos));
    if (tid < wlen) win[tid] = ldst(P.token_ids + wpos - wlen + tid);
    if (tid == 0) *s_pos = wpos;
    const int half = P.hd / 2;
    if (wpos >= 0 && wpos < P.rope_len && tid < P.hd)
      s_rope[tid] = __ldg((tid < half ? P.rope_cos : P.rope_sin) + static_cast<size_t>(wpos) * half + (tid % half));
  };
  if (ph.kind == K_LOGITS && !dfi) read_window();
  // the flag is clear between phases (a phase that set it ended the loop);
  // the first phase of a launch clears it before anything can set it
  if (from_X && tid == 0) s_fail = 0;
  if (from_X) csync();
  // ---- input vector: 4 values per thread per float4 slot (cols <= 16 * kThreads)
  const int n4 = cols >> 2;
  if (normed) {
    float4 xv[4], wv[4];
    const float4 *x4 = reinterpret_cast<const float4 *>(P.X);
    const float4 *w4 = reinterpret_cast<const float4 *>(ph.norm_w);
    const bool embed = ph.kind == K_QKV && ph.do_embed;
    if (embed) {
      if (dfi) {  // the token the previous step's logits phase selected
        if (tid == 0) {
          uint32_t bits = 0;
          if (!poll_tag1(P.tsel, tag_in, bits, &st->err)) s_fail = 1;
          fence_gpu();  // the selection's state and every CTA's earlier K/V rows
          s_tok = static_cast<int>(bits);
        }
      } else if (tid == 0) {
        s_tok = ldst(&st->fwd_token);
      }
      csync();
      int tok = s_tok;
      if (tok < 0 || tok >= st->vocab) tok = 0;  // engine/model.go:222-224
      dequant_row_cta(P.embd_type, P.embd_w + static_cast<size_t>(tok) * P.embd_row_bytes, xn, cols);
      csync();
      if (DF) {  // the residual rows this CTA owns in o-proj / down (same thread)
        int a, b;
        seg_rows(P.H, c, G, a, b);
        if (a + tid < b) P.X[a + tid] = xn[a + tid];
      }
    }
    // tensor parallel: X = residual + the partials every rank sent (rank
    // order), from xbuf[par]; this CTA stores its share of the new X in
    // xbuf[1 - par] for the next reduction.  gate/up follows o-proj's
    // reduction (par 0); qkv (layers > 0) and logits follow down's (par 1).
    // The first phase of a launch reads the residual the per-phase kernels
    // left in X (from_X).
    const int par = ph.kind == K_FFN_UP ? 0 : 1;
    const bool reduce = ll && !embed && !from_X;
    const float4 *xs4 = reduce ? reinterpret_cast<const float4 *>(P.xbuf + static_cast<size_t>(par) * P.H) : x4;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = tid + k * kThreads;
      xv[k] = wv[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n4) {
        wv[k] = __ldg(w4 + i);
        if (!(dfi && !embed)) xv[k] = embed ? reinterpret_cast<const float4 *>(xn)[i] : __ldcg(xs4 + i);
      }
    }
    if (dfi && !embed) {  // the residual of the previous phase, as tagged words (via xn)
      if (!poll_to_smem(P.tX, cols, xn, nullptr, 0, nullptr, nullptr, 0, nullptr, tag_in, &st->err)) s_fail = 1;
      csync();
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (tid + k * kThreads < n4) xv[k] = reinterpret_cast<const float4 *>(xn)[tid + k * kThreads];
      if (ph.kind == K_LOGITS) {  // the forward's commit: SeqLen, TokenIDs, the stop flag
        if (tid == 0) {
          uint32_t bits = 0;
          if (!poll_tag1(P.tsel + 1, tag_in, bits, &st->err)) s_fail = 1;
          fence_gpu();
          s_tok = ldst(&st->halted);
        }
        csync();
        if (s_tok) {  // the stop token was forwarded: a normal end
          *s_halt = 1;
          return true;
        }
        read_window();
      }
    }
    if (reduce) {  // the exchange this phase follows is number xb
      bool got = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = tid + k * kThreads;
        if (i < n4 && got) {
          const float4 o = sum_tagged4(P, par, 4 * i, xb, &st->err, got);
          xv[k] = make_float4(__fadd_rn(xv[k].x, o.x), __fadd_rn(xv[k].y, o.y), __fadd_rn(xv[k].z, o.z),
                              __fadd_rn(xv[k].w, o.w));
        }
      }
      if (!got) *reinterpret_cast<volatile int *>(&s_fail) = 1;
    }
    if (ll && (embed || reduce)) {  // this CTA's share of the new residual (logits: back in X)
      float4 *xd = ph.kind == K_LOGITS ? reinterpret_cast<float4 *>(P.X)
                                       : reinterpret_cast<float4 *>(P.xbuf + static_cast<size_t>(embed ? 0 : 1 - par) * P.H);
      const int a = static_cast<int>((static_cast<unsigned>(c) * n4) / G);
      const int b = static_cast<int>((static_cast<unsigned>(c + 1) * n4) / G);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = tid + k * kThreads;
        if (i >= a && i < b) xd[i] = xv[k];
      }
    } else if (embed && c == 0) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (tid + k * kThreads < n4) reinterpret_cast<float4 *>(P.X)[tid + k * kThreads] = xv[k];
    }
    // RMSNorm (tensor/ops.go:207-218)
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      ss = fmaf(xv[k].x, xv[k].x, ss);
      ss = fmaf(xv[k].y, xv[k].y, ss);
      ss = fmaf(xv[k].z, xv[k].z, ss);
      ss = fmaf(xv[k].w, xv[k].w, ss);
    }
    ss = block_sum(ss, scratch);
    const float mean = __fadd_rn(__fdiv_rn(ss, static_cast<float>(cols)), P.eps);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(mean)));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xv[k].x = __fmul_rn(__fmul_rn(xv[k].x, inv), wv[k].x);
      xv[k].y = __fmul_rn(__fmul_rn(xv[k].y, inv), wv[k].y);
      xv[k].z = __fmul_rn(__fmul_rn(xv[k].z, inv), wv[k].z);
      xv[k].w = __fmul_rn(__fmul_rn(xv[k].w, inv), wv[k].w);
    }
    if (ph.kind == K_LOGITS && c == 0)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (tid + k * kThreads < n4) reinterpret_cast<float4 *>(P.normx)[tid + k * kThreads] = xv[k];
    if (ph.need_f32)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k * kThreads < n4) put_limbs(xv[k], tid + k * kThreads, tid + k * kThreads < n4, la, lb, lc, ls, nb);
    if (ph.need_q8k) {
      if (embed) csync();  // xn held the embedding row
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (tid + k * kThreads < n4) reinterpret_cast<float4 *>(xn)[tid + k * kThreads] = xv[k];
      csync();
      build_q8k(xn, cols, q8qs, q8d, q8bs);
    }
  } else {
    // o-proj: the attention output; down: the SwiGLU output
    const unsigned long long *tin = ph.kind == K_OPROJ ? P.tatt : P.th;
    if (ph.need_f32) {
      const float4 *x4 = reinterpret_cast<const float4 *>(ph.x_in);
      if (dfi) {  // via xn (cols <= H)
        if (!poll_to_smem(tin, cols, xn, nullptr, 0, nullptr, nullptr, 0, nullptr, tag_in, &st->err)) s_fail = 1;
        csync();
        x4 = reinterpret_cast<const float4 *>(xn);
      }
      for (int i0 = 0; i0 < n4; i0 += kThreads) {
        const int i = i0 + tid;
        const float4 v = i < n4 ? (dfi ? x4[i] : __ldcg(x4 + i)) : make_float4(0.f, 0.f, 0.f, 0.f);
        put_limbs(v, i, i < n4, la, lb, lc, ls, nb);
      }
    }
    if (ph.need_q8k) {
      if (dfi) {
        if (!build_q8k_tagged(tin, tag_in, cols, q8qs, q8d, q8bs, &st->err)) s_fail = 1;
      } else {
        build_q8k_global(ph.x_in, cols, q8qs, q8d, q8bs);
      }
    }
  }
  csync();
  if (tr) tr[1] = globaltimer_ns();
  // ---- chunks from the ring.  Few rows: every warp takes rows
  // j = warp (mod kWarps) of each chunk.  Many rows in as many chunks as
  // ring slots or more: the warps split into ng groups of ws; group g takes
  // chunks g, g + ng, ... and its warps rows j = warp (mod ws) of them, so
  // that each warp evaluates larger row groups against one activation load.
  // Each chunk's slot is released by kWarps arrivals either way.
  long long wait_cyc = 0;
  const long long loop_t0 = tr ? clock64() : 0;
  int my_rows = 0;
#pragma unroll
  for (int s = 0; s < kMaxSegs; ++s) my_rows += R.r1[s] - R.r0[s];
  const int lng = (nchunks >= P.nslot && my_rows >= 16 * kWarps) ? P.lng : 0;
  const int ng = 1 << lng, lws = 3 - lng, ws = kWarps >> lng;  // kWarps = 8
  const int grp = warp >> lws, wig = warp & (ws - 1);
  static_assert(kWarps == 8, "warp groups assume 8 compute warps");
  int jbase = 0;
  for (int i = grp; i < nchunks; i += ng) {
    const uint32_t k = k_ring + static_cast<uint32_t>(i);
    const int slot = static_cast<int>(k % static_cast<uint32_t>(P.nslot));
    const uint32_t parity = (k / static_cast<uint32_t>(P.nslot)) & 1u;
    const long long w0 = tr ? clock64() : 0;
    if (*reinterpret_cast<volatile int *>(&s_fail) || !warp_wait_full(&full[slot], parity, &st->err)) {
      s_fail = 1;
      break;
    }
    if (tr) wait_cyc += clock64() - w0;
    // the chunk's pieces: every segment of a packed chunk, else one piece
    const int npiece = R.packed ? ph.nseg : 1;
    for (int pc = 0; pc < npiece; ++pc) {
      PChunk ch;
      int off;
      if (R.packed) {
        ch.seg = pc;
        ch.r0 = R.r0[pc];
        ch.nr = R.r1[pc] - R.r0[pc];
        ch.lr0 = 0;
        off = R.off[pc];
      } else {
        ch = phase_chunk(ph, R, i);
        off = 0;
      }
      if (ch.nr <= 0) continue;
      const Seg &S = ph.seg[ch.seg];
      const uintptr_t src = reinterpret_cast<uintptr_t>(S.w) + static_cast<uintptr_t>(ch.r0) * S.row_bytes;
      const uint8_t *rows = smem + static_cast<size_t>(slot) * P.slot_alloc + off + (src & 15);
      const int first = (wig - jbase) & (ws - 1);
      if (first < ch.nr) {
        const int cnt = (ch.nr - first + ws - 1) >> lws;
        float *y = ybuf + ch.seg * P.yrows + ch.lr0;
        switch (S.type) {
          case T_Q8_0: warp_rows<T_Q8_0>(rows, S.row_bytes, S.units, first, cnt, LV, q8, y, ws); break;
          case T_Q5_0: warp_rows<T_Q5_0>(rows, S.row_bytes, S.units, first, cnt, LV, q8, y, ws); break;
          case T_Q4_K: warp_rows<T_Q4_K>(rows, S.row_bytes, S.units, first, cnt, LV, q8, y, ws); break;
          case T_Q6_K: warp_rows<T_Q6_K>(rows, S.row_bytes, S.units, first, cnt, LV, q8, y, ws); break;
          default: break;
        }
      }
      jbase += ch.nr;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_n(&empty[slot], static_cast<uint32_t>(ng));
  }
  k_ring += static_cast<uint32_t>(nchunks);
  csync();
  if (s_fail) return false;
  if (tr) {
    tr[2] = globaltimer_ns();
    tr[4] = static_cast<unsigned long long>(wait_cyc);
    tr[6] = static_cast<unsigned long long>(clock64() - loop_t0);
  }
  // ---- epilogue
  if (ph.kind == K_QKV) {
#pragma unroll
    for (int s = 0; s < kMaxSegs; ++s)
      if (s < ph.nseg && R.r0[s] + tid < R.r1[s]) {
        const float v = __fadd_rn(ybuf[s * P.yrows + tid], bias[s]);
        if (DF)
          st_tag((s == 0 ? P.tq : s == 1 ? P.tk : P.tv) + R.r0[s] + tid, tag_out, v);
        else
          ph.seg[s].out[R.r0[s] + tid] = v;
      }
  } else if (residual) {
    if (ll) {  // partial rows to every rank, tagged as exchange xb + 1 (summed by the next normed phase)
      const int par = ph.kind == K_OPROJ ? 0 : 1;
      if (R.r0[0] + tid < R.r1[0]) {
        const uint32_t v = __float_as_uint(ybuf[tid]);
        const size_t at = (static_cast<size_t>(par) * P.world + P.rank) * P.H + R.r0[0] + tid;
        for (int r = 0; r < P.world; ++r) st_tagged(P.peer_recv[r] + at, xb + 1, v);
      }
    } else if (R.r0[0] + tid < R.r1[0]) {
      const float v = __fadd_rn(xres, ybuf[tid]);
      P.X[R.r0[0] + tid] = v;
      if (DF) st_tag(P.tX + R.r0[0] + tid, tag_out, v);
    }
    if (ph.kind == K_FFN_DOWN && ph.commit_here && c == 0 && tid == 0) {
      if (ldst(&st->commit)) {
        const int pos = ldst(&st->fwd_pos);
        if (pos >= 0 && pos < st->out_cap) P.token_ids[pos] = ldst(&st->fwd_token);  // KVCache.StoreTokenID
        st->seq_len = pos + 1;
        if (ldst(&st->halt_pending)) {
          st->halted = 1;
          st->halt_pending = 0;
        }
      }
      // bench rewind: SeqLen returns to the prompt every rewind_period steps
      if (P.rewind_period > 0 && (step + 1) % P.rewind_period == 0) st->seq_len = P.rewind_base;
      if (DF) {  // publish the commit (and the state above) to the next logits phase
        fence_gpu();
        st_tag(P.tsel + 1, tag_out, 0.f);
      }
    }
  } else if (ph.kind == K_FFN_UP) {
    // SwiGLU (internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19), float64 exp
    if (R.r0[0] + tid < R.r1[0]) {
      const double g = static_cast<double>(ybuf[tid]);
      const float silu = static_cast<float>(g / (1.0 + exp(-g)));
      const float v = __fmul_rn(silu, ybuf[P.yrows + tid]);
      if (DF)
        st_tag(P.th + R.r0[0] + tid, tag_out, v);
      else
        P.h[R.r0[0] + tid] = v;
    }
  } else if (ph.kind == K_LOGITS) {
    const int lo = R.r0[0], n = R.r1[0] - lo;
    for (int r = tid; r < n; r += kThreads) P.logits[lo + r] = ybuf[r];
    const int glo = P.tp_v0 + lo;  // vocabulary id of this CTA's first row
    // repetition penalty on this CTA's rows (c2slm.go:156-170): every
    // occurrence in the window applies the factor once; the thread holding a
    // token's first occurrence applies all of them, in place
    const int pos = *s_pos, wlen = max(0, min(st->window, pos));
    const float pen = st->penalty;
    auto penalise = [&](float &v, int times) {
      for (int q = 0; q < times; ++q) v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
    };
    auto eligible = [&](int tok) {
      return tok >= 0 && tok < st->vocab && tok != st->im_end && tok != st->eos && tok >= glo && tok < glo + n;
    };
    csync();  // logits stored before ybuf is penalised
    if (wlen <= kThreads) {
      if (tid < wlen) {
        const int tok = win[tid];
        if (eligible(tok)) {
          bool first = true;
          int times = 0;
          for (int q = 0; q < wlen; ++q)
            if (win[q] == tok) {
              first = first && q >= tid;
              ++times;
            }
          if (first) penalise(ybuf[tok - glo], times);
        }
      }
    } else if (tid == 0) {
      for (int p = pos - wlen; p < pos; ++p) {
        const int tok = ldst(P.token_ids + p);
        if (eligible(tok)) penalise(ybuf[tok - glo], 1);
      }
    }
    csync();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int r = tid; r < n; r += kThreads) {
      const float v = ybuf[r];
      if (v > bv || (v == bv && glo + r < bi)) {
        bv = v;
        bi = glo + r;
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
    if (lane == 0) {
      red[0][warp] = bv;
      red[1][warp] = __int_as_float(bi);
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
      if (tp) {  // to every rank, tagged as exchange xb + 1: each one reduces all ranks' partials
        const size_t at = ((static_cast<size_t>((xb + 1) & 1u) * P.world + P.rank) * G + c) * 2;
        for (int r = 0; r < P.world; ++r) {
          st_tagged(P.peer_arg[r] + at, xb + 1, __float_as_uint(bv));
          st_tagged(P.peer_arg[r] + at + 1, xb + 1, static_cast<uint32_t>(bi));
        }
      } else {
        P.amax_part[c] = make_float2(bv, __int_as_float(bi));
        __threadfence();
        const unsigned t = atomicAdd(&st->logits_counter, 1u);
        *s_flag = (t == static_cast<unsigned>(G - 1)) ? 1 : 0;
      }
    }
    csync();
    if (tp) {
      xb += 1;
      *s_flag = c == 0 ? 1 : 0;  // CTA 0 of every rank selects (the same id on all ranks)
      csync();
    }
    const int nparts = tp ? P.world * G : G;
    const unsigned long long *tagged = P.argbuf + static_cast<size_t>(xb & 1u) * P.world * G * 2;
    if (*s_flag) {  // the selecting CTA reduces the partials (ties: lowest id)
      __threadfence();
      float best_v = -INFINITY;
      int best_i = 0x7fffffff;
      for (int kk = tid; kk < nparts; kk += kThreads) {
        float2 pv;
        if (tp) {  // poll until both words of the partial carry the exchange's tag (bounded)
          unsigned long long a = ld_tagged(tagged + 2 * kk), b = ld_tagged(tagged + 2 * kk + 1);
          const long long t0 = clock64();
          for (uint32_t it = 0; static_cast<unsigned>(a >> 32) != xb || static_cast<unsigned>(b >> 32) != xb; ++it) {
            if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
              atomicOr(&st->err, kErrCounter);
              *reinterpret_cast<volatile int *>(&s_fail) = 1;
              break;
            }
            a = ld_tagged(tagged + 2 * kk);
            b = ld_tagged(tagged + 2 * kk + 1);
          }
          pv = make_float2(__uint_as_float(static_cast<uint32_t>(a)), __int_as_float(static_cast<int>(static_cast<uint32_t>(b))));
        } else {
          pv = __ldcg(P.amax_part + kk);
        }
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
      if (lane == 0) {
        red[0][warp] = best_v;
        red[1][warp] = __int_as_float(best_i);
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
      if (DF) {  // publish the selection (and the state above) to the next forward
        fence_gpu();
        st_tag(P.tsel, tag_out, __int_as_float(best_i));
      }
    }
  }
  return true;
}

// DF: the one-GPU dataflow specialisation (PParams::df); otherwise grid
// barriers between phases and the tensor-parallel exchanges.
template <bool DF>
__global__ void __launch_bounds__(kPThreads, 1) k_persistent(const PParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kWarps][kWarps];
  __shared__ float scratch[kWarps];
  __shared__ int s_flag, s_ok;
  __shared__ volatile int s_stop;
  __shared__ PPhase s_ph, s_pph;  // current phase: compute side / producer side
  __shared__ int s_pos;           // position forwarded by the current step
  __shared__ float s_rope[256];   // its RoPE row: cos[hd/2], sin[hd/2]
  __shared__ unsigned s_cbase[64];  // dataflow: split arrivals counted so far per attention unit
  __shared__ int s_halt;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + P.off_full);
  uint64_t *empty = reinterpret_cast<uint64_t *>(smem + P.off_empty);
  uint64_t *abar = reinterpret_cast<uint64_t *>(smem + P.off_abar);
  const int G = gridDim.x, c = blockIdx.x, tid = threadIdx.x;
  DevState *st = P.st;
  if (tid == 0) {
    for (int i = 0; i < P.nslot; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWarps);  // every compute warp releases the slot
    }
    for (int i = 0; i < kAttnBufs; ++i) mbar_init(&abar[i], 1);
    fence_mbar_init();
    // split arrivals start from zero (a launch that stopped on an error may
    // have left counts); the first attention phase follows a grid barrier.
    // Dataflow: no barrier orders this store, so the host clears them.
    if (!DF && c < 64) st->attn_counter[c] = 0;
    s_stop = 0;
  }
  __syncthreads();

  if (tid >= kThreads) {
    // ------------------------------------------------------------ producer
    if (tid != kThreads) return;
    uint32_t k = 0;
    bool stopped = false;
    const int total = P.n_steps * P.nphase;
    for (int kp = 0; kp < total && !stopped; ++kp) {
      {
        const int pi = (P.phase0 + kp) % P.nphase;
        build_phase(P, pi, s_pph);
        const PPhase &ph = s_pph;
        if (ph.kind == K_ATTN) continue;
        PhaseRows R;
        const int nch = phase_rows(ph, c, G, P.slot_bytes, R);
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
          uint8_t *dst = smem + static_cast<size_t>(slot) * P.slot_alloc;
          if (R.packed) {  // every segment's rows into the one slot
            mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(R.total));
#pragma unroll
            for (int sg = 0; sg < kMaxSegs; ++sg)
              if (sg < ph.nseg && R.r1[sg] > R.r0[sg]) {
                uintptr_t a0, a1;
                seg_span(ph.seg[sg], R.r0[sg], R.r1[sg], a0, a1);
                bulk_g2s(dst + R.off[sg], reinterpret_cast<const void *>(a0), static_cast<uint32_t>(a1 - a0), &full[slot]);
              }
          } else {
            const PChunk ch = phase_chunk(ph, R, i);
            issue_chunk_rows(ph.seg[ch.seg], ch, dst, &full[slot]);
          }
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
  uint32_t abar_uses[kAttnBufs] = {};
  unsigned bar_target = 0;
  bool ok = true;
  unsigned xb = static_cast<unsigned>(ldst(reinterpret_cast<const int *>(&st->xbar)));  // cross-GPU barriers so far
  bool crossed = false;  // the previous phase ended with a cross-GPU barrier
  int last_kind = -1;    // kind of the last phase completed
  if (tid == 0) s_pos = ldst(&st->fwd_pos);  // the forward's position when phase0 == 1
  if (tid < 64) s_cbase[tid] = 0;
  if (tid == 0) s_halt = 0;
  if (tid < P.hd && P.phase0 == 1) {
    const int pos0 = ldst(&st->fwd_pos), half = P.hd / 2;
    if (pos0 >= 0 && pos0 < P.rope_len)
      s_rope[tid] = __ldg((tid < half ? P.rope_cos : P.rope_sin) + static_cast<size_t>(pos0) * half + (tid % half));
  }
  const int total = P.n_steps * P.nphase;
  for (int kp = 0; kp < total && ok; ++kp) {
    {
      const int step = (P.phase0 + kp) / P.nphase, pi = (P.phase0 + kp) % P.nphase;
      if (tid == 0) build_phase(P, pi, s_ph);
      csync();
      const PPhase &ph = s_ph;
      const long long b0 = P.trace ? clock64() : 0;
      if (kp > 0 && !DF && !(crossed && pi != 0)) {
        bar_target += 1;
        if (!grid_barrier(P.gbar, bar_target, &st->err, &s_ok)) { ok = false; break; }
      }
      crossed = false;
      // stop token forwarded: a normal end (dataflow: the logits phase reads
      // the flag once the forward's commit is published)
      if (pi == 0 && (!DF || kp == 0) && ldst(&st->halted)) break;
      const unsigned tag_in = P.tag0 + static_cast<unsigned>(kp), tag_out = tag_in + 1u;
      unsigned long long *tr =
          (P.trace && tid == 0)
              ? P.trace + (static_cast<size_t>(kp) * G + c) * kTraceFields
              : nullptr;
      if (tr) {
        const long long b1 = clock64();
        tr[0] = globaltimer_ns();
        tr[5] = static_cast<unsigned long long>(b1 - b0);
        tr[7] = static_cast<unsigned long long>(b1);
      }
      if (ph.kind == K_ATTN) {
        if (!p_attention<DF>(P, ph, reinterpret_cast<float *>(smem + P.off_act), abar, abar_uses, c, s_pos, s_rope,
                         tag_in, tag_out, s_cbase)) {
          ok = false;
          break;
        }
        if (DF && s_pos >= 0 && s_pos < P.max_tokens) {
          // every unit's splits arrived once each when there was more than
          // one (the layout is the same on every CTA)
          csync();
          const AttnLayout AL = attn_layout(s_pos, P.split_len, P.n_kv, P.tp_h1 - P.tp_h0, G);
          if (AL.nsplit > 1 && tid < (AL.per_head ? P.tp_h1 - P.tp_h0 : P.n_kv))
            s_cbase[tid] += static_cast<unsigned>(AL.nsplit);
        }
      } else {
        if (!p_matvec<DF>(P, ph, smem, k_ring, red, scratch, &s_flag, &s_pos, s_rope, tr, xb, kp == 0, tag_in, tag_out,
                      step, &s_halt)) {
          ok = false;
          break;
        }
        if (s_halt) break;
      }
      csync();
      if (tr) tr[3] = globaltimer_ns();
      // tensor parallel: o-proj / down sent exchange xb + 1; the next phase
      // polls its tagged words instead of waiting at a grid barrier (except
      // logits, which reads the state the down phase committed)
      if (!DF && P.ll && (ph.kind == K_OPROJ || ph.kind == K_FFN_DOWN)) {
        xb += 1;
        crossed = true;
      }
      last_kind = ph.kind;
    }
  }
  if (!DF && P.ll && ok && last_kind == K_FFN_DOWN) {
    // the launch ends after a forward: leave its residual in X for the
    // per-phase kernels and the next launch (X = xbuf[1] + the down partials)
    const int n4 = P.H / 4;
    const int a = static_cast<int>((static_cast<unsigned>(c) * n4) / G);
    const int b = static_cast<int>((static_cast<unsigned>(c + 1) * n4) / G);
    const float4 *xs = reinterpret_cast<const float4 *>(P.xbuf + P.H);
    bool got = true;
    for (int i = a + tid; i < b && got; i += kThreads) {
      const float4 o = sum_tagged4(P, 1, 4 * i, xb, &st->err, got);
      const float4 x = __ldcg(xs + i);
      reinterpret_cast<float4 *>(P.X)[i] =
          make_float4(__fadd_rn(x.x, o.x), __fadd_rn(x.y, o.y), __fadd_rn(x.z, o.z), __fadd_rn(x.w, o.w));
    }
  }
  // exchanges done; after a failure, jump far past every tag already written
  // so that no later exchange can match a stale word
  if (c == 0 && tid == 0) st->xbar = ok ? xb : xb + (1u << 24);
  // tell the producer where consumption stopped, then let it drain
  csync();
  if (tid == 0) {
    s_flag = static_cast<int>(k_ring);
    __threadfence_block();
    s_stop = 1;
  }
}

}  // namespace c2s
