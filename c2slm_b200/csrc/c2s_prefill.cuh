// c2s_prefill.cuh -- multi-token prefill (IngestFrom of a prompt) on the
// 5th-generation tensor cores.
//
// The reference ingests a prompt as one engine.Forward per token
// (c2slm.go:92-115): every token's activations are quantised to Q8_K on their
// own and its attention is causal.  Here the tokens of a chunk go through
// each layer together: the K-quant projections become int8 GEMMs of the
// tokens' Q8_K rows against the weights on tcgen05 (kind::i8, accumulators in
// TMEM), the rest (norms, RoPE, attention, SwiGLU) runs per token.
//
// Integer contract of a K-quant row dot (A8/A9): per superblock, Q4_K adds
//   sum_j d*d8*sc_j*dot_j - dmin*d8*m_j*bsum_j   (j: 8 sub-blocks of 32)
// and Q6_K adds d6*d8*sum_g sc_g*(dot_g - 32*bsum_g).  The tensor cores see
// the scale folded into the weight byte: v = q*sc (Q4_K 0..945, Q6_K
// (q-32)*sc) is split into int8 digits v = 128*hi + lo, lo in [0, 127], so
// that per superblock
//   sum_j sc_j*dot_j = 128*MMA(q8, hi) + MMA(q8, lo)        (exact int32)
// and Q4_K's min term sum_j m_j*bsum_j = MMA(q8, m) with m_j repeated over
// its 32 elements.  Each superblock then takes one float step per (token,
// row): acc += f(isum)*(d*d8) - f(msum)*(dmin*d8) -- the same integers as the
// reference, with fewer float roundings.
#pragma once
#include "c2s_kernels.cuh"

namespace c2s {

// ---------------------------------------------------------------------------
// tcgen05 / TMEM wrappers
// ---------------------------------------------------------------------------
// shared-memory matrix descriptor: K-major, no swizzle ("interleaved" core
// matrices of 8 rows x 16 B), lbo = byte distance of the two 16-B halves of
// a 32-B K step, sbo = byte distance of consecutive 8-row groups
__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version of sm_100
  return d;
}

// instruction descriptor of kind::i8: s32 accumulator, signed A and B,
// both K-major, M x N
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// K-quant x Q8_K GEMM: out[t][r] (+)= sum_k W[r][k] x[t][k] for a tile of
// 128 tokens x 64 weight rows per CTA, one superblock (K = 256) per round:
//   A (tokens' Q8_K bytes)   8 K-steps x [128 rows x 32 B]   32 KB
//   B planes hi, lo (, m)    8 K-steps x [64 rows x 32 B]    16 KB each
//   TMEM accumulators        hi | lo | m, 64 columns each
// ---------------------------------------------------------------------------
constexpr int kPfM = 128, kPfN = 64, kPfThreads = 128;
constexpr int kPfAStep = kPfM * 32, kPfBStep = kPfN * 32;
constexpr int kPfABytes = 8 * kPfAStep, kPfBPlane = 8 * kPfBStep;
constexpr int kPfSmem = kPfABytes + 3 * kPfBPlane + 2 * kPfN * 4 + 1024;

enum PfMode { PF_STORE = 0, PF_ADD = 1 };

struct PfGemm {
  const uint8_t *w;  // weight rows (GGML blocks), row_bytes each
  int type, rows, cols, row_bytes;
  const int8_t *aq;  // tokens' Q8_K bytes [M][lda]
  const float *ad;   // tokens' superblock scales [M][ldd]
  int lda, ldd, M;
  float *out;        // [M][ldo]
  int ldo, mode;
  const float *bias;  // [rows] or null (PF_STORE)
  unsigned *err;
};

// byte offset of (row r, byte kb of a 32-B K step) in one K step of the
// interleaved layout
__device__ __forceinline__ int pf_off(int r, int kb) { return (r >> 3) * 256 + (kb >> 4) * 128 + (r & 7) * 16 + (kb & 15); }

// 16 int8 digits (hi, lo) of v = q * s for 16 weights of one row
__device__ __forceinline__ void pf_digits16(const int (&v)[16], uint4 &hi, uint4 &lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    h[w] = l[w] = 0u;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int x = v[4 * w + b];
      h[w] |= (static_cast<uint32_t>(x >> 7) & 0xFFu) << (8 * b);  // floor(x / 128)
      l[w] |= (static_cast<uint32_t>(x) & 0x7Fu) << (8 * b);        // x mod 128
    }
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int TYPE>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(const PfGemm G) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t s_tmem;
  constexpr int NPL = TYPE == T_Q4_K ? 3 : 2;  // digit planes (+ min plane)
  uint8_t *sA = smem;
  uint8_t *sB = smem + kPfABytes;  // plane p at sB + p * kPfBPlane
  float *rowd = reinterpret_cast<float *>(sB + 3 * kPfBPlane);
  float *rowdm = rowd + kPfN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * kPfN, t0 = blockIdx.y * kPfM;
  const int nsb = G.cols / 256;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {  // 4 x 64 columns: hi, lo, m (and one spare)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(smem_addr(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
  const int tok = t0 + tid;  // this thread's token in the epilogue (TMEM lane tid)
  float acc[kPfN];
#pragma unroll
  for (int r = 0; r < kPfN; ++r) acc[r] = 0.f;
  bool ok = true;
  for (int s = 0; s < nsb && ok; ++s) {
    // ---- A: 128 tokens x 256 Q8_K bytes of superblock s (zeros past M)
    for (int i = tid; i < kPfM * 16; i += kPfThreads) {
      const int r = i >> 4, c = i & 15;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (t0 + r < G.M)
        v = __ldg(reinterpret_cast<const uint4 *>(G.aq + static_cast<size_t>(t0 + r) * G.lda + s * 256 + c * 16));
      *reinterpret_cast<uint4 *>(sA + (c >> 1) * kPfAStep + pf_off(r, (c & 1) * 16)) = v;
    }
    // ---- B: 64 rows of superblock s as digit planes
    if constexpr (TYPE == T_Q4_K) {
      // task (row rr, sub-block pair p): sub-blocks 2p (low nibbles), 2p+1 (high)
      for (int task = tid; task < kPfN * 4; task += kPfThreads) {
        const int rr = task >> 2, p = task & 3;
        const bool valid = r0 + rr < G.rows;
        const uint8_t *blk = G.w + static_cast<size_t>(valid ? r0 + rr : 0) * G.row_bytes + s * 144;
        const uint4 hd = __ldg(reinterpret_cast<const uint4 *>(blk));
        const uint4 qa = __ldg(reinterpret_cast<const uint4 *>(blk + 16 + 32 * p));
        const uint4 qb = __ldg(reinterpret_cast<const uint4 *>(blk + 32 + 32 * p));
        // 6-bit scales / mins of sub-blocks 2p, 2p+1 (tensor/ops.go:354-361)
        const uint32_t sc8[3] = {hd.y, hd.z, hd.w};
        auto sbyte = [&](int i) { return static_cast<int>((sc8[i >> 2] >> (8 * (i & 3))) & 0xFFu); };
        int sc[2], mn[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = 2 * p + u;
          if (j < 4) {
            sc[u] = sbyte(j) & 63;
            mn[u] = sbyte(j + 4) & 63;
          } else {
            sc[u] = (sbyte(j + 4) & 15) | ((sbyte(j - 4) >> 6) << 4);
            mn[u] = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
          }
          if (!valid) sc[u] = mn[u] = 0;
        }
        const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = 2 * p + u;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            int v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const uint32_t byte = (qw[half * 4 + (e >> 2)] >> (8 * (e & 3))) & 0xFFu;
              v[e] = static_cast<int>(u == 0 ? (byte & 15u) : (byte >> 4)) * sc[u];
            }
            uint4 hi, lo;
            pf_digits16(v, hi, lo);
            const int off = j * kPfBStep + pf_off(rr, half * 16);
            *reinterpret_cast<uint4 *>(sB + off) = hi;
            *reinterpret_cast<uint4 *>(sB + kPfBPlane + off) = lo;
            const uint32_t m4 = static_cast<uint32_t>(mn[u]) * 0x01010101u;
            *reinterpret_cast<uint4 *>(sB + 2 * kPfBPlane + off) = make_uint4(m4, m4, m4, m4);
          }
        }
        if (p == 0) {
          const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
          rowd[rr] = valid ? dd.x : 0.f;
          rowdm[rr] = valid ? dd.y : 0.f;
        }
      }
    } else {
      // Q6_K task (row rr, half n, quarter k): K step j = 4n + k, elements
      // l = 0..31 of q6u = low 4 bits | 2 high bits << 4, group scale
      // sc[8n + 2k + l / 16] (c2_tensor_gemv2_q6_k_q8_k_nosimd_gen.go:80-237)
      for (int task = tid; task < kPfN * 8; task += kPfThreads) {
        const int rr = task >> 3, n = (task >> 2) & 1, k = task & 3;
        const bool valid = r0 + rr < G.rows;
        const uint8_t *blk = G.w + static_cast<size_t>(valid ? r0 + rr : 0) * G.row_bytes + s * 210;
        uint32_t ql[8], qh[8];
        ld_window<8>(blk + 64 * n + 32 * (k & 1), ql);
        ld_window<8>(blk + 128 + 32 * n, qh);
        const int g0 = 8 * n + 2 * k;
        const int s0 = valid ? static_cast<int8_t>(blk[192 + g0]) : 0;
        const int s1 = valid ? static_cast<int8_t>(blk[192 + g0 + 1]) : 0;
        const int j = 4 * n + k;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          int v[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int w = half * 4 + (e >> 2), b = e & 3;
            const uint32_t lb = (ql[w] >> (8 * b)) & 0xFFu, hb = (qh[w] >> (8 * b)) & 0xFFu;
            const int q6 = static_cast<int>(((k >> 1) ? (lb >> 4) : (lb & 15u)) | (((hb >> (2 * k)) & 3u) << 4));
            v[e] = (q6 - 32) * (half ? s1 : s0);
          }
          uint4 hi, lo;
          pf_digits16(v, hi, lo);
          const int off = j * kPfBStep + pf_off(rr, half * 16);
          *reinterpret_cast<uint4 *>(sB + off) = hi;
          *reinterpret_cast<uint4 *>(sB + kPfBPlane + off) = lo;
        }
        if (n == 0 && k == 0) rowd[rr] = valid ? h2f(ld16(blk + 208)) : 0.f;
      }
    }
    // ---- the MMAs of this superblock (one thread), then the epilogue
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    if (tid == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(kPfM, kPfN);
#pragma unroll
      for (int pl = 0; pl < NPL; ++pl)
        for (int j = 0; j < 8; ++j)
          umma_i8(tmem + pl * kPfN, umma_sdesc(smem_addr(sA + j * kPfAStep), 128, 256),
                  umma_sdesc(smem_addr(sB + pl * kPfBPlane + j * kPfBStep), 128, 256), idesc, j > 0 ? 1u : 0u);
      umma_commit(&bar);
    }
    ok = mbar_wait_bounded(&bar, static_cast<uint32_t>(s & 1), G.err);
    tmem_fence_after();
    if (ok) {
      const float d8 = tok < G.M ? __ldg(G.ad + static_cast<size_t>(tok) * G.ldd + s) : 0.f;
#pragma unroll
      for (int c0 = 0; c0 < kPfN; c0 += 16) {
        uint32_t hi[16], lo[16], mm[16];
        tmem_ld16(tmem + lane_base + c0, hi);
        tmem_ld16(tmem + lane_base + kPfN + c0, lo);
        if constexpr (TYPE == T_Q4_K) tmem_ld16(tmem + lane_base + 2 * kPfN + c0, mm);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = c0 + i;
          const int isum = static_cast<int>(hi[i]) * 128 + static_cast<int>(lo[i]);
          const float dd = __fmul_rn(rowd[r], d8);
          float t = __fmul_rn(static_cast<float>(isum), dd);
          if constexpr (TYPE == T_Q4_K)
            t = __fsub_rn(t, __fmul_rn(static_cast<float>(static_cast<int>(mm[i])), __fmul_rn(rowdm[r], d8)));
          acc[r] = __fadd_rn(acc[r], t);
        }
      }
    }
    tmem_fence_before();
    __syncthreads();  // smem and TMEM free for the next superblock
    tmem_fence_after();
  }
  if (ok && tok < G.M) {
    float *o = G.out + static_cast<size_t>(tok) * G.ldo + r0;
#pragma unroll
    for (int r = 0; r < kPfN; ++r)
      if (r0 + r < G.rows) {
        if (G.mode == PF_ADD)
          o[r] = __fadd_rn(o[r], acc[r]);
        else
          o[r] = G.bias ? __fadd_rn(acc[r], __ldg(G.bias + r0 + r)) : acc[r];
      }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

// ---------------------------------------------------------------------------
// per-token kernels of a prefill chunk (n tokens at positions p0 .. p0+n-1)
// ---------------------------------------------------------------------------
// EmbedToken of each token (engine/model.go:221-247): x[t] = row(tok[t])
__global__ void __launch_bounds__(kThreads) k_pf_embed(const int *tok, int n, int vocab, int type, const uint8_t *w,
                                                       int row_bytes, float *x, int H) {
  const int t = blockIdx.x;
  if (t >= n) return;
  int id = tok[t];
  if (id < 0 || id >= vocab) id = 0;  // engine/model.go:222-224
  dequant_row_cta(type, w + static_cast<size_t>(id) * row_bytes, x + static_cast<size_t>(t) * H, H);
}

// One token's row x[t][0..K) -> optional RMSNorm with weight nw (tensor/ops.go:
// 207-218) -> Q8_K (internal/simd/c2_quantize_q8_k_gen.go:11-91): bytes
// q[t][0..K), superblock scales d[t][0..K/256).  xn (optional) receives the
// normalised f32 row.
__global__ void __launch_bounds__(kThreads) k_pf_norm_q8k(const float *x, int ldx, const float *nw, float eps, int K,
                                                          int n, int8_t *q, int ldq, float *d, int ldd, float *xn) {
  __shared__ float scratch[kWarps];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (t >= n) return;
  const float *xr = x + static_cast<size_t>(t) * ldx;
  float inv = 1.f;
  if (nw) {
    float ss = 0.f;
    for (int i = tid * 4; i < K; i += kThreads * 4) {
      const float4 v = *reinterpret_cast<const float4 *>(xr + i);
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
    ss = block_sum(ss, scratch);
    const float mean = __fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps);
    inv = static_cast<float>(1.0 / sqrt(static_cast<double>(mean)));
  }
  for (int sb = warp; sb < K / 256; sb += kWarps) {
    float v[8];
    const float4 a = *reinterpret_cast<const float4 *>(xr + sb * 256 + lane * 8);
    const float4 b = *reinterpret_cast<const float4 *>(xr + sb * 256 + lane * 8 + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    if (nw) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __ldg(nw + sb * 256 + lane * 8 + i));
    }
    if (xn) {
      float *o = xn + static_cast<size_t>(t) * ldx + sb * 256 + lane * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[i];
    }
    int32_t bs[16];
    quantize_sb_warp(v, d + static_cast<size_t>(t) * ldd + sb, bs, [&](int ln, const int (&qv)[8]) {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w0 |= (static_cast<uint32_t>(qv[k]) & 0xFFu) << (8 * k);
        w1 |= (static_cast<uint32_t>(qv[4 + k]) & 0xFFu) << (8 * k);
      }
      *reinterpret_cast<uint2 *>(q + static_cast<size_t>(t) * ldq + sb * 256 + ln * 8) = make_uint2(w0, w1);
    });
  }
}

// q, k of each token: QK-norm (Qwen3, engine/forward.go:80-91), NeoX RoPE of
// position p0 + t (tensor/ops.go:228-286); q back in place, k and v into the
// layer's cache rows (KVCache.StoreKV, engine/kvcache.go:143-158).
__global__ void __launch_bounds__(kThreads) k_pf_rope_store(float *q, const float *k, const float *v, int ldq,
                                                            int ldkv, int n, int p0, int nqh, int nkv, int hd,
                                                            const float *rope_cos, const float *rope_sin,
                                                            int rope_len, const float *q_norm, const float *k_norm,
                                                            float eps, float *kc, float *vc, size_t head_stride) {
  extern __shared__ __align__(16) float buf[];  // [nqh + nkv][hd]
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5;
  if (t >= n) return;
  const int pos = p0 + t, half = hd / 2;
  float *qt = q + static_cast<size_t>(t) * ldq;
  const float *kt = k + static_cast<size_t>(t) * ldkv;
  for (int i = tid; i < nqh * hd; i += kThreads) buf[i] = qt[i];
  for (int i = tid; i < nkv * hd; i += kThreads) buf[nqh * hd + i] = kt[i];
  csync();
  if (q_norm || k_norm) {
    for (int h = warp; h < nqh + nkv; h += kWarps) {
      const float *w = h < nqh ? q_norm : k_norm;
      if (w) head_rmsnorm_warp(buf + h * hd, w, hd, eps);
    }
    csync();
  }
  if (pos < rope_len) {
    const float *cs = rope_cos + static_cast<size_t>(pos) * half, *sn = rope_sin + static_cast<size_t>(pos) * half;
    for (int i = tid; i < (nqh + nkv) * half; i += kThreads) {
      const int h = i / half, j = i - h * half;
      float *r = buf + h * hd;
      const float x0 = r[j], x1 = r[j + half], c = cs[j], s = sn[j];
      r[j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      r[j + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    csync();
  }
  for (int i = tid; i < nqh * hd; i += kThreads) qt[i] = buf[i];
  for (int i = tid; i < nkv * hd; i += kThreads) {
    const int g = i / hd, j = i - g * hd;
    kc[g * head_stride + static_cast<size_t>(pos) * hd + j] = buf[nqh * hd + i];
    vc[g * head_stride + static_cast<size_t>(pos) * hd + j] = v[static_cast<size_t>(t) * ldkv + i];
  }
}

// Causal attention of token t (position p0 + t) for the query heads of kv
// group blockIdx.x, over cache rows 0 .. p0 + t (rows already stored and
// rotated): the decode attention of one split, no RoPE, no store.
struct PfAttn {
  const float *q;  // [n][ldq] rotated
  float *out;      // [n][ldq]
  float *kc, *vc;  // this layer's planes: group g row p at [g * head_stride + p * hd]
  size_t head_stride;
  int ldq, n, p0, n_kv, qpk, n_heads, hd, max_splits;
  float scale, eps;
  unsigned *err;
};

__global__ void __launch_bounds__(kThreads) k_pf_attention(const PfAttn A) {
  extern __shared__ __align__(128) float asmem[];
  __shared__ __align__(8) uint64_t bars[kAttnBufs];
  const int tid = threadIdx.x, g = blockIdx.x, t = blockIdx.y;
  if (tid == 0) {
    for (int i = 0; i < kAttnBufs; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (t >= A.n) return;
  const int pos = A.p0 + t, hd = A.hd;
  AttnJob J;
  J.g = g;
  J.h0 = g * A.qpk;
  J.qpk = min(A.qpk, A.n_heads - J.h0);
  J.store_kv = 0;
  J.counter = nullptr;
  J.q = A.q + static_cast<size_t>(t) * A.ldq + static_cast<size_t>(J.h0) * hd;
  J.k = A.kc + g * A.head_stride + static_cast<size_t>(pos) * hd;
  J.v = A.vc + g * A.head_stride + static_cast<size_t>(pos) * hd;
  J.q_norm = J.k_norm = nullptr;
  J.kc = A.kc + g * A.head_stride;
  J.vc = A.vc + g * A.head_stride;
  J.rope_cs = J.rope_sn = nullptr;
  J.out = A.out + static_cast<size_t>(t) * A.ldq;
  J.part = nullptr;
  J.dist = 0;
  J.s = 0;
  J.nsplit = 1;
  J.p0 = 0;
  J.p1 = pos + 1;
  J.pos = pos;
  J.hd = hd;
  J.max_splits = A.max_splits;
  J.eps = A.eps;
  J.scale = A.scale;
  uint32_t uses[kAttnBufs] = {};
  attend(J, asmem, bars, uses, A.err);
}

// SwiGLU in place (internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19)
__global__ void __launch_bounds__(kThreads) k_pf_swiglu(float *g, const float *u, size_t count) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * kThreads) {
    const double x = static_cast<double>(g[i]);
    g[i] = __fmul_rn(static_cast<float>(x / (1.0 + exp(-x))), u[i]);
  }
}

// the chunk's bookkeeping on the device: TokenIDs, SeqLen and the forward
// inputs of its last token (as the per-token path leaves them)
__global__ void k_pf_commit(DevState *st, int *token_ids, const int *tok, int n, int p0, int cap) {
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (p0 + i < cap) token_ids[p0 + i] = tok[i];
  if (threadIdx.x == 0) {
    st->fwd_token = tok[n - 1];
    st->fwd_pos = p0 + n - 1;
    st->seq_len = p0 + n;
  }
}

}  // namespace c2s
