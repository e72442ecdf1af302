// c2s_prefill.cuh -- multi-token prefill (IngestFrom of a prompt) on the
// 5th-generation tensor cores.
//
// The reference ingests a prompt as one engine.Forward per token
// (c2slm.go:92-115): every token's activations are quantised to Q8_K on their
// own and its attention is causal.  Here the tokens of a chunk go through
// each layer together: the K-quant projections become int8 GEMMs of the
// tokens' Q8_K rows against the weights on tcgen05 (kind::i8, accumulators in
// TMEM); norms, RoPE and SwiGLU run per token, the causal attention as a
// tiled kernel over the chunk's query vectors.
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

// instruction descriptor of kind::tf32: f32 accumulator, tf32 A and B, both
// K-major, M x N
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// kind::tf32, A and B in shared memory
__device__ __forceinline__ void umma_tf32_ss(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

// kind::tf32, A in tensor memory (M lanes x K columns, one element a column),
// B in shared memory
__device__ __forceinline__ void umma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 8 consecutive 32-bit columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes <- registers
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// K-quant x Q8_K GEMM: out[t][r] (+)= sum_k W[r][k] x[t][k], one CTA per tile
// of 128 weight rows (the MMA's M, TMEM lanes) x 128 tokens (N, columns),
// one superblock (K = 256) per round.
//
// Operands sit in HBM already in the tensor cores' shared-memory layout
// (K-major, no swizzle: core matrices of 8 rows x 16 B; per 32-B K step the
// two 16-B halves 128 B apart, 8-row groups 256 B apart), so a round is a few
// 1-D bulk copies:
//   weight planes [row tile][superblock][hi, lo] 8 K steps x [128 x 32 B]  64 KB
//   token tile    [token tile][superblock]       8 K steps x [128 x 32 B]  32 KB
//   token scales  d8 [token tile][superblock][128] f32, sub-block sums
//                 bs [token tile][superblock][128][8] int16
// (planes by k_pf_planes once per weight matrix, tokens by k_pf_norm_q8k).
// Per row the block scales (d, dmin) and the 6-bit mins m_j come from a
// table rowinfo[row][superblock]; the Q4_K min term sum_j m_j * bs_j is an
// integer dot on the CUDA cores.
// Warps 0-7: epilogue (warp w: TMEM lanes 32 (w % 4) .. (the rows), tokens
// 64 (w / 4) ..), warp 8 lane 0: copies, warp 9 lane 0: MMAs.  Two
// shared-memory operand stages (planes + token tile; freed by the MMAs'
// commit), a ring of four token-scale slots (freed by the epilogue) and two
// TMEM accumulator sets overlap the copies of round s+1, the MMAs of round s
// and the epilogue of round s-1.
// ---------------------------------------------------------------------------
constexpr int kPfM = 128, kPfN = 128, kPfThreads = 320;
constexpr int kPfKStep = 128 * 32, kPfPlane = 8 * kPfKStep;  // per superblock: 32 KB
constexpr int kPfTokTile = kPfPlane;                          // token tile per superblock
constexpr int kPfD8Bytes = kPfN * 4, kPfBsBytes = kPfN * 16;
constexpr int kPfStage = 2 * kPfPlane + kPfTokTile;  // operands of one superblock
// token scales of a superblock (d8, sub-block sums) in a ring of their own:
// the epilogue reads them after the MMAs are done with the operand stage,
// which is then free for the next copy without waiting for the epilogue
constexpr int kPfScale = kPfD8Bytes + kPfBsBytes, kPfScaleSlots = 4;
constexpr int kPfStages = 2;
constexpr int kPfSmem = kPfStages * kPfStage + kPfScaleSlots * kPfScale + 128;

enum PfMode { PF_STORE = 0, PF_ADD = 1 };

struct PfGemm {
  const uint8_t *planes;  // [row tile][superblock][2][32 KB]
  const uint4 *rowinfo;   // [row tile * 128 + r][superblock]: d, dmin (f32 bits), m[8] bytes
  int type, rows, cols;
  const uint8_t *a;    // token tiles [token tile][superblock][32 KB]
  const float *ad;     // [token tile][superblock][128]
  const int16_t *abs;  // [token tile][superblock][128][8]
  int M;
  float *out;  // [M][ldo]
  int ldo, mode;
  const float *bias;  // [rows] or null (PF_STORE)
  unsigned *err;
};

// byte offset of (row r, byte kb of a 32-B K step) in one K step of the
// interleaved layout
__host__ __device__ __forceinline__ int pf_off(int r, int kb) {
  return (r >> 3) * 256 + (kb >> 4) * 128 + (r & 7) * 16 + (kb & 15);
}

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

// Digit planes and row table of one weight matrix: CTA (row tile, superblock).
// Rows past the matrix are zero.
template <int TYPE>
__global__ void __launch_bounds__(128) k_pf_planes(const uint8_t *w, int rows, int row_bytes, int nsb, uint8_t *planes,
                                                   uint4 *rowinfo) {
  const int R = blockIdx.x, s = blockIdx.y, r0 = R * kPfM;
  uint8_t *dst = planes + (static_cast<size_t>(R) * nsb + s) * 2 * kPfPlane;
  if constexpr (TYPE == T_Q4_K) {
    // task (row rr, sub-block pair p): sub-blocks 2p (low nibbles), 2p+1 (high)
    for (int task = threadIdx.x; task < kPfM * 4; task += 128) {
      const int rr = task >> 2, p = task & 3;
      const bool valid = r0 + rr < rows;
      const uint8_t *blk = w + static_cast<size_t>(valid ? r0 + rr : 0) * row_bytes + s * 144;
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
          const int off = j * kPfKStep + pf_off(rr, half * 16);
          *reinterpret_cast<uint4 *>(dst + off) = hi;
          *reinterpret_cast<uint4 *>(dst + kPfPlane + off) = lo;
        }
      }
      uint8_t *ri = reinterpret_cast<uint8_t *>(rowinfo + (static_cast<size_t>(r0) + rr) * nsb + s);
      ri[8 + 2 * p] = static_cast<uint8_t>(mn[0]);
      ri[9 + 2 * p] = static_cast<uint8_t>(mn[1]);
      if (p == 0) {
        const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
        reinterpret_cast<float *>(ri)[0] = valid ? dd.x : 0.f;
        reinterpret_cast<float *>(ri)[1] = valid ? dd.y : 0.f;
      }
    }
  } else {
    // Q6_K task (row rr, half n, quarter k): K step j = 4n + k, elements
    // l = 0..31 of q6u = low 4 bits | 2 high bits << 4, group scale
    // sc[8n + 2k + l / 16] (c2_tensor_gemv2_q6_k_q8_k_nosimd_gen.go:80-237)
    for (int task = threadIdx.x; task < kPfM * 8; task += 128) {
      const int rr = task >> 3, n = (task >> 2) & 1, k = task & 3;
      const bool valid = r0 + rr < rows;
      const uint8_t *blk = w + static_cast<size_t>(valid ? r0 + rr : 0) * row_bytes + s * 210;
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
          const int wi = half * 4 + (e >> 2), b = e & 3;
          const uint32_t lb = (ql[wi] >> (8 * b)) & 0xFFu, hb = (qh[wi] >> (8 * b)) & 0xFFu;
          const int q6 = static_cast<int>(((k >> 1) ? (lb >> 4) : (lb & 15u)) | (((hb >> (2 * k)) & 3u) << 4));
          v[e] = (q6 - 32) * (half ? s1 : s0);
        }
        uint4 hi, lo;
        pf_digits16(v, hi, lo);
        const int off = j * kPfKStep + pf_off(rr, half * 16);
        *reinterpret_cast<uint4 *>(dst + off) = hi;
        *reinterpret_cast<uint4 *>(dst + kPfPlane + off) = lo;
      }
      if (n == 0 && k == 0) {
        const float d6 = valid ? h2f(ld16(blk + 208)) : 0.f;
        rowinfo[(static_cast<size_t>(r0) + rr) * nsb + s] = make_uint4(__float_as_uint(d6), 0u, 0u, 0u);
      }
    }
  }
}

// One CTA's tile (row tile R, token tile T) of G; smem: kPfSmem bytes.
template <int TYPE>
__device__ __forceinline__ void pf_gemm_tile(const PfGemm &G, const int R, const int T, uint8_t *smem) {
  __shared__ __align__(8) uint64_t full[kPfStages], empty[kPfStages], tfull[2], tempty[2], sfull[kPfScaleSlots],
      sempty[kPfScaleSlots];
  __shared__ uint32_t s_tmem;
  constexpr uint32_t kStageBytes = kPfStage;
  uint8_t *sscale = smem + kPfStages * kPfStage;  // [kPfScaleSlots][d8 | bs]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = R * kPfM, t0 = T * kPfN;
  const int nsb = G.cols / 256;
  if (tid == 0) {
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);  // the MMAs' commit
    }
    for (int i = 0; i < kPfScaleSlots; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], 8);  // the eight epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);
    }
    fence_mbar_init();
  }
  if (warp == 0) {  // two accumulator sets of hi | lo, 128 columns each
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = s_tmem;
  bool ok = true;
  if (warp == 8) {
    // ---------------------------------------------------------- copies
    if (lane == 0) {
      const uint8_t *pw = G.planes + static_cast<size_t>(R) * nsb * 2 * kPfPlane;
      const size_t tb0 = static_cast<size_t>(T) * nsb;
      for (int s = 0; s < nsb && ok; ++s) {
        const int st = s % kPfStages;
        if (s >= kPfStages) ok = mbar_wait_bounded(&empty[st], static_cast<uint32_t>((s / kPfStages - 1) & 1), G.err);
        if (!ok) break;
        uint8_t *dst = smem + st * kPfStage;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        bulk_g2s(dst, pw + static_cast<size_t>(s) * 2 * kPfPlane, 2 * kPfPlane, &full[st]);
        bulk_g2s(dst + 2 * kPfPlane, G.a + (tb0 + s) * kPfTokTile, kPfTokTile, &full[st]);
        const int ss = s % kPfScaleSlots;
        if (s >= kPfScaleSlots)
          ok = mbar_wait_bounded(&sempty[ss], static_cast<uint32_t>((s / kPfScaleSlots - 1) & 1), G.err);
        if (!ok) break;
        uint8_t *sd = sscale + ss * kPfScale;
        mbar_arrive_expect_tx(&sfull[ss], kPfScale);
        bulk_g2s(sd, G.ad + (tb0 + s) * kPfN, kPfD8Bytes, &sfull[ss]);
        bulk_g2s(sd + kPfD8Bytes, G.abs + (tb0 + s) * kPfN * 8, kPfBsBytes, &sfull[ss]);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMAs
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(kPfM, kPfN);
      for (int s = 0; s < nsb && ok; ++s) {
        const int st = s % kPfStages, tb = s & 1;
        ok = mbar_wait_bounded(&full[st], static_cast<uint32_t>((s / kPfStages) & 1), G.err);
        if (ok && s >= 2) ok = mbar_wait_bounded(&tempty[tb], static_cast<uint32_t>(((s >> 1) - 1) & 1), G.err);
        if (!ok) break;
        tmem_fence_after();
        const uint8_t *sw = smem + st * kPfStage, *sx = sw + 2 * kPfPlane;
        const uint32_t td = tmem + static_cast<uint32_t>(tb * 2 * kPfN);
#pragma unroll
        for (int pl = 0; pl < 2; ++pl)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            umma_i8(td + pl * kPfN, umma_sdesc(smem_addr(sw + pl * kPfPlane + j * kPfKStep), 128, 256),
                    umma_sdesc(smem_addr(sx + j * kPfKStep), 128, 256), idesc, j > 0 ? 1u : 0u);
        umma_commit(&empty[st]);  // the stage's operands are read
        umma_commit(&tfull[tb]);  // the accumulators are complete
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int quad = warp & 3, th = warp >> 2;  // rows 32 quad + lane, tokens 64 th ..
    const int row = r0 + 32 * quad + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quad) << 16;
    float acc[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) acc[i] = 0.f;
    const uint4 *ri = G.rowinfo + static_cast<size_t>(row) * nsb;
    uint4 rin = __ldg(ri);  // this row's table entry, one superblock ahead
    for (int s = 0; s < nsb && ok; ++s) {
      const int ss = s % kPfScaleSlots, tb = s & 1;
      const uint4 rv = rin;
      if (s + 1 < nsb) rin = __ldg(ri + s + 1);
      ok = mbar_wait_bounded(&tfull[tb], static_cast<uint32_t>((s >> 1) & 1), G.err) &&
           mbar_wait_bounded(&sfull[ss], static_cast<uint32_t>((s / kPfScaleSlots) & 1), G.err);
      {  // ok made uniform over the epilogue warps (all leave together)
        uint32_t all;
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 2, 256, q;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(all) : "r"(ok ? 1u : 0u) : "memory");
        ok = all != 0;
      }
      if (!ok) break;
      tmem_fence_after();
      const float dr = __uint_as_float(rv.x), dmr = __uint_as_float(rv.y);
      const uint8_t *stg = sscale + ss * kPfScale;
      const float *sd8 = reinterpret_cast<const float *>(stg);
      const uint4 *sbs = reinterpret_cast<const uint4 *>(stg + kPfD8Bytes);
      const uint32_t ta = tmem + lane_base + static_cast<uint32_t>(tb * 2 * kPfN + 64 * th);
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 8) {
        uint32_t hi[8], lo[8];
        tmem_ld8(ta + c0, hi);
        tmem_ld8(ta + kPfN + c0, lo);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tk = 64 * th + c0 + i;
          // token scales four at a time (one broadcast load)
          const float4 d84 = *reinterpret_cast<const float4 *>(sd8 + (tk & ~3));
          const float d8i = (i & 3) == 0 ? d84.x : (i & 3) == 1 ? d84.y : (i & 3) == 2 ? d84.z : d84.w;
          const int isum = static_cast<int>(hi[i]) * 128 + static_cast<int>(lo[i]);
          if constexpr (TYPE == T_Q4_K) {
            const uint4 b = sbs[tk];  // sub-block sums 0..7 as int16 pairs
            int msum = __dp2a_lo(static_cast<int>(b.x), static_cast<int>(rv.z), 0);
            msum = __dp2a_hi(static_cast<int>(b.y), static_cast<int>(rv.z), msum);
            msum = __dp2a_lo(static_cast<int>(b.z), static_cast<int>(rv.w), msum);
            msum = __dp2a_hi(static_cast<int>(b.w), static_cast<int>(rv.w), msum);
            // d8 (d isum - dmin msum): the integer dots are exact; the float
            // terms are those of the per-token matvec, associated differently
            const float u = fmaf(dr, static_cast<float>(isum), -__fmul_rn(dmr, static_cast<float>(msum)));
            acc[c0 + i] = fmaf(d8i, u, acc[c0 + i]);
          } else {
            acc[c0 + i] = fmaf(__fmul_rn(dr, d8i), static_cast<float>(isum), acc[c0 + i]);
          }
        }
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[tb]);
        mbar_arrive(&sempty[ss]);
      }
    }
    if (ok && row < G.rows) {
      float *o = G.out + static_cast<size_t>(t0 + 64 * th) * G.ldo + row;
      const int nt = min(64, G.M - (t0 + 64 * th));
      if (G.mode == PF_ADD) {
        // residual add in batches of 16: all loads of a batch before its
        // stores (one memory round trip per batch, not one per token)
#pragma unroll
        for (int i0 = 0; i0 < 64; i0 += 16) {
          float old[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) old[i] = i0 + i < nt ? o[static_cast<size_t>(i0 + i) * G.ldo] : 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (i0 + i < nt) o[static_cast<size_t>(i0 + i) * G.ldo] = __fadd_rn(old[i], acc[i0 + i]);
        }
      } else {
        const float bias = G.bias ? __ldg(G.bias + row) : 0.f;
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < nt) o[static_cast<size_t>(i) * G.ldo] = G.bias ? __fadd_rn(acc[i], bias) : acc[i];
      }
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

// Up to three GEMMs of one weight type over the same token tiles in one
// launch (the q, k and v projections, whose narrow k / v matrices alone would
// occupy 16 CTAs): blockIdx.x runs over the row tiles of job 0, then of job
// 1, ...
struct PfGemmSet {
  PfGemm g[3];
  int tiles[3];  // row tiles of each job
  int n;         // jobs
};

template <int TYPE>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(const __grid_constant__ PfGemmSet S) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ PfGemm sG;  // this CTA's job (read from shared memory, not kept in registers)
  __shared__ int sR;     // its row tile in the job
  if (threadIdx.x == 0) {
    const int R = blockIdx.x, t0 = S.tiles[0], t1 = S.tiles[1];
    if (R < t0 || S.n == 1) {
      sG = S.g[0];
      sR = R;
    } else if (R < t0 + t1 || S.n == 2) {
      sG = S.g[1];
      sR = R - t0;
    } else {
      sG = S.g[2];
      sR = R - t0 - t1;
    }
  }
  __syncthreads();
  pf_gemm_tile<TYPE>(sG, sR, blockIdx.y, smem);
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
// 207-218) -> Q8_K (internal/simd/c2_quantize_q8_k_gen.go:11-91), written for
// the GEMM: bytes into the token tiles q [token tile][superblock][32 KB],
// superblock scales d [token tile][superblock][128], sub-block sums bs
// [token tile][superblock][128][8] (int16).  xn (optional) receives the
// normalised f32 row.  With u (the FFN's up projection, same layout as x = its
// gate), the row quantised is SwiGLU(x, u) instead
// (internal/simd/c2_tensor_swiglu_nosimd_gen.go:11-19; no norm then).
__global__ void __launch_bounds__(kThreads) k_pf_norm_q8k(const float *x, int ldx, const float *nw, float eps, int K,
                                                          int n, uint8_t *q, float *d, int16_t *bs, float *xn,
                                                          const float *u = nullptr) {
  __shared__ float scratch[kWarps];
  __shared__ int32_t s_bsum[kWarps][16];
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (t >= n) return;
  const int nsb = K / 256, T = t / kPfN, tr = t % kPfN;
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
  for (int sb = warp; sb < nsb; sb += kWarps) {
    float v[8];
    const float4 a = *reinterpret_cast<const float4 *>(xr + sb * 256 + lane * 8);
    const float4 b = *reinterpret_cast<const float4 *>(xr + sb * 256 + lane * 8 + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    if (u) {
      const float *ur = u + static_cast<size_t>(t) * ldx + sb * 256 + lane * 8;
      const float4 ua = *reinterpret_cast<const float4 *>(ur), ub = *reinterpret_cast<const float4 *>(ur + 4);
      const float uv[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const double g = static_cast<double>(v[i]);
        v[i] = __fmul_rn(static_cast<float>(g / (1.0 + exp(-g))), uv[i]);
      }
    }
    if (nw) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), __ldg(nw + sb * 256 + lane * 8 + i));
    }
    if (xn) {
      float *o = xn + static_cast<size_t>(t) * ldx + sb * 256 + lane * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = v[i];
    }
    const size_t tile = static_cast<size_t>(T) * nsb + sb;
    quantize_sb_warp(v, d + tile * kPfN + tr, s_bsum[warp], [&](int ln, const int (&qv)[8]) {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w0 |= (static_cast<uint32_t>(qv[k]) & 0xFFu) << (8 * k);
        w1 |= (static_cast<uint32_t>(qv[4 + k]) & 0xFFu) << (8 * k);
      }
      // 8 bytes = elements 8ln .. 8ln+7: K step ln / 4, bytes (ln % 4) * 8 of it
      *reinterpret_cast<uint2 *>(q + tile * kPfTokTile + (ln >> 2) * kPfKStep + pf_off(tr, (ln & 3) * 8)) =
          make_uint2(w0, w1);
    });
    __syncwarp();
    if (lane < 8)  // sub-block sums: two 16-element sums each (|sum| <= 4064)
      bs[(tile * kPfN + tr) * 8 + lane] = static_cast<int16_t>(s_bsum[warp][2 * lane] + s_bsum[warp][2 * lane + 1]);
    __syncwarp();
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

// x += d over n values (tensor parallel: the residual plus the ranks' summed
// o-proj / down rows of the chunk)
__global__ void k_pf_add(float *x, const float *d, size_t n) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    x[i] = __fadd_rn(x[i], d[i]);
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

// ---------------------------------------------------------------------------
// Causal attention of a prefill chunk, tiled: CTA (kv group g, block of 128
// query vectors v = token * qpk + head of the group's heads, key split s; the
// blocks of the latest tokens, which see the most keys, are scheduled first).
// A block's keys 0 .. kall-1 are cut into splits of split_keys (a multiple
// of the 128-key tile) so that the grid's CTAs carry similar work.  Per key
// tile (K transposed and V staged in shared memory):
//   S = Q K^T * scale   (8 queries x 8 keys per thread, f32)
//   online softmax per query (exp in float64 as tensor.Softmax,
//                        tensor/ops.go:317-339; keys past the query's position
//                        excluded)
//   O = O * alpha + P V (8 queries x HD/16 dims per thread)
// and O / l at the end (engine/forward.go:143-155 per head and position).
// Shared-memory loads move 16 B per lane and cost one wavefront per 8 lanes
// whether or not lanes share an address, so the 8 x 8 register tiles (4 FMA
// per loaded float) are what keeps the FMA pipe, not shared memory, the bound.
// A block of one split writes O / l; otherwise each split writes its
// (m, l, O) and the last split of the block to arrive combines them in split
// order (weights exp(m_s - max m) in float64) and clears the block's counter.
// ---------------------------------------------------------------------------
struct PfFlash {
  const float *q;        // [n][ldq] rotated queries
  float *out;            // [n][ldq]
  const float *kc, *vc;  // this layer's planes: group g row p at [g * head_stride + p * hd]
  size_t head_stride;
  int ldq, n, p0, qpk, n_heads;
  // tensor-parallel shard: this rank's query heads are global heads
  // [hbase, hbase + n_heads) and its kv groups start at global group gbase;
  // the CTA of local group g takes the group's heads the rank holds (a
  // group may straddle ranks).  One GPU: 0, 0.
  int hbase, gbase;
  float scale;
  float *part;           // [group][block][max_splits][kFqN][hd + 2]: (m, l, O) of a split
  unsigned *count;       // [group][block]: arrivals of the block's splits (0 between launches)
  int split_keys, max_splits;
  // tensor-core kernel (k_pf_attn): the layer's K/V tiles (k_pf_kv_tiles),
  // tiles per group, and the status word its bounded waits report to
  const uint8_t *tiles;
  int tiles_per_group;
  unsigned *err;
};

constexpr int kFqN = 128, kFkN = 128;
// probabilities [key][query], rows of kFqN + 16 floats: the S tile stores
// (8 lanes on 32 consecutive queries) and the softmax reads (lane = query +
// 16 x key parity) are conflict-free
constexpr int kFps = kFqN + 16;

// shared memory of k_pf_flash<HD>, in floats: Qt [HD][kFqN] | Kt [HD][kFkN]
// sharing its space with Pt [kFkN][kFps] | Vs [kFkN][HD] | s_m, s_l,
// s_alpha, s_lim [kFqN]
__host__ __device__ constexpr int pf_flash_kp(int hd) { return hd * kFkN > kFkN * kFps ? hd * kFkN : kFkN * kFps; }
__host__ __device__ constexpr size_t pf_flash_smem(int hd) {
  return (static_cast<size_t>(hd) * kFqN + pf_flash_kp(hd) + static_cast<size_t>(kFkN) * hd + 4 * kFqN) * 4;
}

// Split partials of a query block: per split and query row, (m, l, -, -,
// O[HD]) -- rows of pf_part_width(HD) floats, O 16-byte aligned.
__host__ __device__ constexpr int pf_part_width(int hd) { return hd + 4; }

// The last-arriving split of a query block combines the block's nsplit
// partials in split order: per query M = max m_s, w_s = exp(m_s - M) in
// float64, L = sum w_s l_s, out = (sum w_s O_s) / L.  Four output columns a
// task, every split's value loaded before the ordered sum.  s_w: shared
// [nsplit][kFqN], s_l: shared [kFqN]; all nthreads threads call it.
template <int HD>
__device__ __forceinline__ void pf_split_combine(const PfFlash &A, const float *pblk, int nsplit, int v0, int nv,
                                                 int qg, int h0, float *s_w, float *s_l, int tid, int nthreads) {
  constexpr int PW = pf_part_width(HD);
  if (tid < kFqN) {
    float M = -INFINITY;
    for (int j = 0; j < nsplit; ++j) M = fmaxf(M, __ldcg(pblk + (static_cast<size_t>(j) * kFqN + tid) * PW));
    float L = 0.f;
    for (int j = 0; j < nsplit; ++j) {
      const float mj = __ldcg(pblk + (static_cast<size_t>(j) * kFqN + tid) * PW);
      const float w = mj == -INFINITY ? 0.f : static_cast<float>(exp(static_cast<double>(__fsub_rn(mj, M))));
      s_w[j * kFqN + tid] = w;
      L = __fadd_rn(L, __fmul_rn(w, __ldcg(pblk + (static_cast<size_t>(j) * kFqN + tid) * PW + 1)));
    }
    s_l[tid] = L;
  }
  __syncthreads();
  for (int i = tid; i < kFqN * (HD / 4); i += nthreads) {
    const int qi = i / (HD / 4), d4 = (i - qi * (HD / 4)) * 4, v = v0 + qi;
    if (v >= nv) continue;
    float4 x[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nsplit)
        x[j] = __ldcg(reinterpret_cast<const float4 *>(pblk + (static_cast<size_t>(j) * kFqN + qi) * PW + 4 + d4));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < nsplit) {
        const float w = s_w[j * kFqN + qi];
        acc.x = __fadd_rn(acc.x, __fmul_rn(w, x[j].x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(w, x[j].y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(w, x[j].z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(w, x[j].w));
      }
    const float L = s_l[qi];
    const int t = v / qg, h = v - t * qg;
    *reinterpret_cast<float4 *>(A.out + static_cast<size_t>(t) * A.ldq + (h0 + h) * HD + d4) =
        make_float4(acc.x / L, acc.y / L, acc.z / L, acc.w / L);
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) k_pf_flash(const PfFlash A) {
  extern __shared__ __align__(16) float fsm[];
  float *Qt = fsm;                         // [HD][kFqN]
  float *Kt = Qt + HD * kFqN, *Pt = Kt;    // [HD][kFkN], then [kFkN][kFps]
  float *Vs = Kt + pf_flash_kp(HD);        // [kFkN][HD]
  float *s_m = Vs + kFkN * HD, *s_l = s_m + kFqN, *s_alpha = s_l + kFqN;
  int *s_lim = reinterpret_cast<int *>(s_alpha + kFqN);  // last key position of each query
  const int tid = threadIdx.x, g = blockIdx.x;
  const int nblk = gridDim.y, blk = nblk - 1 - blockIdx.y, sp = blockIdx.z;
  // this group's query heads on this rank: local heads [h0, h0 + qg)
  const int gg = A.gbase + g;
  const int hlo = max(A.hbase, gg * A.qpk), hhi = min(A.hbase + A.n_heads, (gg + 1) * A.qpk);
  const int qg = hhi - hlo, h0 = hlo - A.hbase;
  if (qg <= 0) return;
  const int nv = A.n * qg, v0 = blk * kFqN;
  if (v0 >= nv) return;
  const int vlast = min(nv, v0 + kFqN) - 1;
  const int kall = A.p0 + vlast / qg + 1;  // the block's keys 0 .. kall-1
  const int nsplit = (kall + A.split_keys - 1) / A.split_keys;
  if (sp >= nsplit) return;  // this block has fewer splits
  const int kbeg = sp * A.split_keys, kend = min(kall, kbeg + A.split_keys);  // this split's keys
  // ---- queries of the block, transposed (a warp: 32 queries of one d4); causal limits
  for (int i = tid; i < kFqN * (HD / 4); i += kThreads) {
    const int qi = i % kFqN, d4 = (i / kFqN) * 4, v = v0 + qi;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (v < nv) {
      const int t = v / qg, h = v - t * qg;
      x = *reinterpret_cast<const float4 *>(A.q + static_cast<size_t>(t) * A.ldq + (h0 + h) * HD + d4);
    }
    Qt[(d4 + 0) * kFqN + qi] = x.x;
    Qt[(d4 + 1) * kFqN + qi] = x.y;
    Qt[(d4 + 2) * kFqN + qi] = x.z;
    Qt[(d4 + 3) * kFqN + qi] = x.w;
  }
  if (tid < kFqN) {
    const int v = v0 + tid;
    s_lim[tid] = v < nv ? A.p0 + v / qg : -1;
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.f;
  }
  // thread tiles: queries tq*4 + e and 64 + tq*4 + e (S and O); keys tk*4 + e
  // and 64 + tk*4 + e (S); dims tk*4 + 64 c + e (O)
  const int tq = tid & 15, tk = tid >> 4;
  constexpr int OD = HD / 16;
  auto qof = [&](int a) { return (a < 4 ? 0 : 64) + tq * 4 + (a & 3); };
  auto dof = [&](int b) { return tk * 4 + 16 * (b & ~3) + (b & 3); };
  float o[8][OD];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < OD; ++b) o[a][b] = 0.f;
  const float *kg = A.kc + g * A.head_stride, *vg = A.vc + g * A.head_stride;
  for (int kb = kbeg; kb < kend; kb += kFkN) {
    const int nk = min(kFkN, kend - kb);
    __syncthreads();  // Pt and Vs of the previous tile consumed
    for (int i = tid; i < kFkN * (HD / 4); i += kThreads) {
      {  // K transposed: a warp covers 32 keys of one d4 (conflict-free stores)
        const int kr = i % kFkN, d4 = (i / kFkN) * 4;
        float4 kx = make_float4(0.f, 0.f, 0.f, 0.f);
        if (kr < nk) kx = __ldcg(reinterpret_cast<const float4 *>(kg + static_cast<size_t>(kb + kr) * HD + d4));
        Kt[(d4 + 0) * kFkN + kr] = kx.x;
        Kt[(d4 + 1) * kFkN + kr] = kx.y;
        Kt[(d4 + 2) * kFkN + kr] = kx.z;
        Kt[(d4 + 3) * kFkN + kr] = kx.w;
      }
      {  // V as rows
        const int vr = i / (HD / 4), v4 = (i % (HD / 4)) * 4;
        float4 vx = make_float4(0.f, 0.f, 0.f, 0.f);
        if (vr < nk) vx = __ldcg(reinterpret_cast<const float4 *>(vg + static_cast<size_t>(kb + vr) * HD + v4));
        *reinterpret_cast<float4 *>(Vs + vr * HD + v4) = vx;
      }
    }
    __syncthreads();
    // ---- S = Q K^T for the thread's 8 x 8 tile
    float sacc[8][8];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) sacc[a][b] = 0.f;
#pragma unroll 2
    for (int d = 0; d < HD; ++d) {
      const float4 q0 = *reinterpret_cast<const float4 *>(Qt + d * kFqN + tq * 4);
      const float4 q1 = *reinterpret_cast<const float4 *>(Qt + d * kFqN + 64 + tq * 4);
      const float4 k0 = *reinterpret_cast<const float4 *>(Kt + d * kFkN + tk * 4);
      const float4 k1 = *reinterpret_cast<const float4 *>(Kt + d * kFkN + 64 + tk * 4);
      const float qa[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      const float ka[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
      for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) sacc[a][b] = fmaf(qa[a], ka[b], sacc[a][b]);
    }
    __syncthreads();  // every thread is done with Kt: Pt takes its space
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const int kl = (b < 4 ? 0 : 64) + tk * 4 + (b & 3), key = kb + kl;
#pragma unroll
      for (int hq = 0; hq < 2; ++hq) {
        float w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int a = 4 * hq + e;
          w[e] = (kl < nk && key <= s_lim[qof(a)]) ? __fmul_rn(sacc[a][b], A.scale) : -INFINITY;
        }
        *reinterpret_cast<float4 *>(Pt + kl * kFps + 64 * hq + tq * 4) = make_float4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncthreads();
    // ---- online softmax: 2 threads per query, keys 2 j + part
    {
      const int qi = tid >> 1, part = tid & 1;
      float mx = -INFINITY;
#pragma unroll 8
      for (int j = 0; j < kFkN / 2; ++j) mx = fmaxf(mx, Pt[(2 * j + part) * kFps + qi]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      const float m_old = s_m[qi], m_new = fmaxf(m_old, mx);
      float ls = 0.f;
#pragma unroll 4
      for (int j = 0; j < kFkN / 2; ++j) {  // four exponentials in flight
        float *pp = Pt + (2 * j + part) * kFps + qi;
        const float sv = *pp;
        const float e = sv == -INFINITY ? 0.f : static_cast<float>(exp(static_cast<double>(__fsub_rn(sv, m_new))));
        *pp = e;
        ls += e;
      }
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      if (part == 0) {
        const float alpha = m_new == -INFINITY ? 1.f : static_cast<float>(exp(static_cast<double>(m_old - m_new)));
        s_alpha[qi] = alpha;
        s_l[qi] = __fadd_rn(__fmul_rn(s_l[qi], alpha), ls);
        s_m[qi] = m_new;
      }
    }
    __syncthreads();
    // ---- O = O * alpha + P V for the thread's 8 queries x OD dims
    {
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        const float al = s_alpha[qof(a)];
#pragma unroll
        for (int b = 0; b < OD; ++b) o[a][b] *= al;
      }
#pragma unroll 2
      for (int k = 0; k < nk; ++k) {
        const float4 p0 = *reinterpret_cast<const float4 *>(Pt + k * kFps + tq * 4);
        const float4 p1 = *reinterpret_cast<const float4 *>(Pt + k * kFps + 64 + tq * 4);
        const float pa[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        float vv[OD];
#pragma unroll
        for (int b = 0; b < OD; b += 4) {
          const float4 x = *reinterpret_cast<const float4 *>(Vs + k * HD + tk * 4 + 16 * b);
          vv[b] = x.x, vv[b + 1] = x.y, vv[b + 2] = x.z, vv[b + 3] = x.w;
        }
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
          for (int b = 0; b < OD; ++b) o[a][b] = fmaf(pa[a], vv[b], o[a][b]);
      }
    }
  }
  __syncthreads();
  if (nsplit == 1) {
#pragma unroll
    for (int a = 0; a < 8; ++a) {
      const int q = qof(a), v = v0 + q;
      if (v < nv) {
        const int t = v / qg, h = v - t * qg;
        const float l = s_l[q];
        float *dst = A.out + static_cast<size_t>(t) * A.ldq + (h0 + h) * HD;
#pragma unroll
        for (int b = 0; b < OD; ++b) dst[dof(b)] = o[a][b] / l;
      }
    }
    return;
  }
  // ---- partial (m, l, O) of this split; the block's last split combines
  constexpr int PW = pf_part_width(HD);
  float *pblk = A.part + (static_cast<size_t>(g) * nblk + blk) * A.max_splits * kFqN * PW;
  {
    float *pp = pblk + static_cast<size_t>(sp) * kFqN * PW;
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < OD; ++b) pp[qof(a) * PW + 4 + dof(b)] = o[a][b];
    if (tid < kFqN) {
      pp[tid * PW] = s_m[tid];
      pp[tid * PW + 1] = s_l[tid];
    }
  }
  __threadfence();
  __syncthreads();
  int *s_last = s_lim;  // the causal limits are no longer needed
  if (tid == 0) {
    unsigned *cnt = A.count + static_cast<size_t>(g) * nblk + blk;
    const unsigned prev = atomicAdd(cnt, 1u);
    const int last = prev == static_cast<unsigned>(nsplit - 1) ? 1 : 0;
    if (last) *cnt = 0u;  // for the next launch (every split of this one has arrived)
    *s_last = last;
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  pf_split_combine<HD>(A, pblk, nsplit, v0, nv, qg, h0, Pt, s_l, tid, kThreads);
}

// ---------------------------------------------------------------------------
// Causal attention of a prefill chunk on the tensor cores (kind::tf32).
//
// FP32 products from TF32 operands: each f32 operand x is split into
// hi = x with its 13 low mantissa bits cleared (a TF32 value) and
// lo = x - hi (exact), and a product is taken as hi*hi' + hi*lo' + lo*hi'
// (lo read as TF32 in turn; the lo*lo' term, below 2^-20 of the product, is
// dropped), accumulated in the MMA's f32 accumulator.  Against float64
// attention from the same q, k and v this is as close as the FP32 kernel
// (k_pf_flash): the error of both is set by the f32 rounding of large,
// peaked scores, not by the split.
//
// CTA: kv group g, block of 128 query vectors (as k_pf_flash: v = token *
// qg + head, the latest tokens' blocks first), key split sp; keys in tiles
// of 64.  Two passes over the split's key tiles, as the reference's Softmax
// (tensor/ops.go:317-339) takes the maximum of all scores before any
// exponential:
//   pass 1  S = Q K^T (TMEM), row maxima of S * scale over the causal keys;
//   pass 2  S again, p = exp(S * scale - m) (exp_nonpos: f32 on the FMA pipe;
//           the float64 exponential's conversions made the multi-function
//           unit the kernel's bound), l += p in key order, O += P V (TMEM).
// O / l at the end, or the split's (m, l, O) for the last-arriving split to
// combine (the FP32 kernel's combine, in split order).
// Warps 0-3: one query row per thread (TMEM lane): Q into TMEM, softmax,
// epilogue.  Warp 4 lane 0: MMAs (and the TMEM allocation).  Warp 5 lane 0:
// bulk copies of the K / V tiles.
// TMEM columns: Q hi [0, HD), Q lo [HD, 2 HD), two S buffers of 64,
// O [2 HD + 128, 3 HD + 128) -- 512 columns at HD = 128.
// Shared memory: K hi | lo, V^T hi | lo of one tile (4 planes of 64 x HD
// f32), P hi | lo (2 x 128 x 64 f32), all in the no-swizzle K-major
// core-matrix layout of the GEMM (per 32-B K step: 8-row groups 256 B apart,
// 16-B halves 128 B apart).
// ---------------------------------------------------------------------------
constexpr int kTaK = 64;          // keys per tile
constexpr int kTaThreads = 192;
__host__ __device__ constexpr int ta_plane(int hd) { return kTaK * hd * 4; }
__host__ __device__ constexpr size_t ta_tile_bytes(int hd) { return 4 * static_cast<size_t>(ta_plane(hd)); }
constexpr int kTaPPlane = 128 * kTaK * 4;
__host__ __device__ constexpr size_t ta_smem(int hd) { return ta_tile_bytes(hd) + 2 * kTaPPlane; }

// e^x for x <= 0 in f32 with FMA-pipe arithmetic only: Cody-Waite reduction
// x = k ln2 + r, |r| <= ln2 / 2, with ln2 split into a head cut to 15
// significant bits (k * head exact for |k| < 512) and the remainder; e^r by
// its Taylor series to degree 7 in Horner form (truncation below 6e-9
// relative); 2^k from the exponent bits.  Against the f32 rounding of the
// float64 e^x (the reference's Softmax value) over [-87, 0]: within 1 ulp,
// equal for ~94 % of arguments (200,000 uniform samples).  Returns 0
// below e^-87 (under the smallest normal f32: next to the row maximum's
// probability 1 such a term cannot change a sum or a weighted mean).
__device__ __forceinline__ float exp_nonpos(float x) {
  if (!(x > -87.f)) return 0.f;  // also -inf
  const float k = rintf(x * 1.44269504088896341f);  // log2(e)
  float r = fmaf(k, -0.693145751953125f, x);        // ln2 head
  r = fmaf(k, -1.42860682030941723e-6f, r);         // ln2 - head
  float p = 1.f / 5040.f;
  p = fmaf(p, r, 1.f / 720.f);
  p = fmaf(p, r, 1.f / 120.f);
  p = fmaf(p, r, 1.f / 24.f);
  p = fmaf(p, r, 1.f / 6.f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.f);
  p = fmaf(p, r, 1.f);
  return p * __int_as_float((static_cast<int>(k) + 127) << 23);
}

// x = hi + lo: hi = x with the 13 low mantissa bits cleared (a TF32 value),
// lo = x - hi (exact; the tensor cores read it as TF32 too)
__device__ __forceinline__ void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
  hi = __float_as_uint(x) & 0xFFFFE000u;
  lo = __float_as_uint(__fsub_rn(x, __uint_as_float(hi)));
}

// K and V rows 0 .. nkeys-1 of every kv group of a layer -> the tiles the
// tensor-core attention copies: per group and tile of 64 keys, four planes
// [K hi | K lo | V^T hi | V^T lo], each 64 x HD f32.  K planes: the B
// operand of Q K^T (rows = keys, K-major over dims); V^T planes: the B
// operand of P V (rows = dims, K-major over keys).  Task i writes the 16
// bytes at 16 i of a plane (coalesced stores).  Keys past nkeys are zero.
template <int HD>
__global__ void __launch_bounds__(256) k_pf_kv_tiles(const float *kc, const float *vc, size_t head_stride, int nkeys,
                                                     uint8_t *tiles, int tiles_per_group) {
  constexpr int PL = ta_plane(HD);
  const int t = blockIdx.x, g = blockIdx.y, kb = t * kTaK;
  uint8_t *dst = tiles + (static_cast<size_t>(g) * tiles_per_group + t) * 4 * PL;
  const float *kg = kc + g * head_stride, *vg = vc + g * head_stride;
  for (int i = threadIdx.x; i < kTaK * HD / 4; i += blockDim.x) {
    uint4 h, l;
    {  // K: row r = 8 grp + r8 (key), dims 8 s + 4 half ..
      const int r8 = i & 7, half = (i >> 3) & 1, grp = (i >> 4) & 7, ks = i >> 7;
      const int r = grp * 8 + r8, d4 = ks * 8 + half * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kb + r < nkeys) x = __ldcg(reinterpret_cast<const float4 *>(kg + static_cast<size_t>(kb + r) * HD + d4));
      tf32_split(x.x, h.x, l.x);
      tf32_split(x.y, h.y, l.y);
      tf32_split(x.z, h.z, l.z);
      tf32_split(x.w, h.w, l.w);
      *reinterpret_cast<uint4 *>(dst + 16 * i) = h;
      *reinterpret_cast<uint4 *>(dst + PL + 16 * i) = l;
    }
    {  // V^T: row n = 8 ng + n8 (dim), keys 8 ks + 4 half ..
      const int n8 = i & 7, half = (i >> 3) & 1, ng = (i >> 4) % (HD / 8), ks = (i >> 4) / (HD / 8);
      const int n = ng * 8 + n8, k0 = kb + ks * 8 + half * 4;
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = k0 + e < nkeys ? __ldcg(vg + static_cast<size_t>(k0 + e) * HD + n) : 0.f;
      tf32_split(x[0], h.x, l.x);
      tf32_split(x[1], h.y, l.y);
      tf32_split(x[2], h.z, l.z);
      tf32_split(x[3], h.w, l.w);
      *reinterpret_cast<uint4 *>(dst + 2 * PL + 16 * i) = h;
      *reinterpret_cast<uint4 *>(dst + 3 * PL + 16 * i) = l;
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(kTaThreads, 1) k_pf_attn(const PfFlash A) {
  extern __shared__ __align__(128) uint8_t tsm[];
  constexpr int PL = ta_plane(HD);
  uint8_t *sK = tsm, *sV = tsm + 2 * PL, *sP = tsm + 4 * PL;  // each: hi plane, then lo plane
  __shared__ __align__(8) uint64_t k_full, k_empty, v_full, v_empty, s_full[2], s_empty[2], p_full, p_empty, q_ready,
      o_full;
  __shared__ uint32_t s_tmem;
  __shared__ float s_l[kFqN];
  __shared__ int s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = blockIdx.x, nblk = gridDim.y, blk = nblk - 1 - blockIdx.y, sp = blockIdx.z;
  // this group's query heads on this rank: local heads [h0, h0 + qg)
  const int gg = A.gbase + g;
  const int hlo = max(A.hbase, gg * A.qpk), hhi = min(A.hbase + A.n_heads, (gg + 1) * A.qpk);
  const int qg = hhi - hlo, h0 = hlo - A.hbase;
  if (qg <= 0) return;
  const int nv = A.n * qg, v0 = blk * kFqN;
  if (v0 >= nv) return;
  const int vlast = min(nv, v0 + kFqN) - 1;
  const int kall = A.p0 + vlast / qg + 1;  // the block's keys 0 .. kall-1
  const int nsplit = (kall + A.split_keys - 1) / A.split_keys;
  if (sp >= nsplit) return;  // this block has fewer splits
  const int kbeg = sp * A.split_keys, kend = min(kall, kbeg + A.split_keys);  // this split's keys
  const int kt0 = kbeg / kTaK, nt = (kend - kbeg + kTaK - 1) / kTaK;
  if (tid == 0) {
    mbar_init(&k_full, 1);
    mbar_init(&k_empty, 1);
    mbar_init(&v_full, 1);
    mbar_init(&v_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    mbar_init(&p_full, 4);
    mbar_init(&p_empty, 1);
    mbar_init(&q_ready, 4);
    mbar_init(&o_full, 1);
    fence_mbar_init();
  }
  if (warp == 4) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_addr(&s_tmem)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = s_tmem;
  constexpr uint32_t cQh = 0, cQl = HD, cS = 2 * HD, cO = 2 * HD + 2 * kTaK;
  bool ok = true;
  if (warp == 5) {
    // ------------------------------------------------------------ copies
    if (lane == 0) {
      const uint8_t *tg = A.tiles + static_cast<size_t>(g) * A.tiles_per_group * 4 * PL;
      int ku = 0, vu = 0;
      for (int pass = 0; pass < 2 && ok; ++pass)
        for (int j = 0; j < nt && ok; ++j) {
          const uint8_t *src = tg + static_cast<size_t>(kt0 + j) * 4 * PL;
          if (ku > 0 && !(ok = mbar_wait_bounded(&k_empty, static_cast<uint32_t>((ku - 1) & 1), A.err))) break;
          mbar_arrive_expect_tx(&k_full, 2 * PL);
          bulk_g2s(sK, src, 2 * PL, &k_full);
          ++ku;
          if (pass == 1) {
            if (vu > 0 && !(ok = mbar_wait_bounded(&v_empty, static_cast<uint32_t>((vu - 1) & 1), A.err))) break;
            mbar_arrive_expect_tx(&v_full, 2 * PL);
            bulk_g2s(sV, src + 2 * PL, 2 * PL, &v_full);
            ++vu;
          }
        }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMAs
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_tf32(128, kTaK), idO = umma_idesc_tf32(128, HD);
      int ku = 0, su = 0, vu = 0, pu = 0;
      // S(b) = Q K^T: the two cross terms, then hi x hi
      auto issue_s = [&]() -> bool {
        if (!mbar_wait_bounded(&k_full, static_cast<uint32_t>(ku & 1), A.err)) return false;
        const int b = su & 1;
        if (su >= 2 && !mbar_wait_bounded(&s_empty[b], static_cast<uint32_t>(((su >> 1) - 1) & 1), A.err))
          return false;
        tmem_fence_after();
        const uint32_t d = tmem + cS + static_cast<uint32_t>(b * kTaK);
#pragma unroll 1
        for (int ks = 0; ks < HD / 8; ++ks) {
          const uint64_t bl = umma_sdesc(smem_addr(sK + PL + ks * (kTaK * 32)), 128, 256);
          const uint64_t bh = umma_sdesc(smem_addr(sK + ks * (kTaK * 32)), 128, 256);
          umma_tf32_ts(d, tmem + cQh + 8 * ks, bl, idS, ks > 0 ? 1u : 0u);
          umma_tf32_ts(d, tmem + cQl + 8 * ks, bh, idS, 1u);
        }
#pragma unroll 1
        for (int ks = 0; ks < HD / 8; ++ks)
          umma_tf32_ts(d, tmem + cQh + 8 * ks, umma_sdesc(smem_addr(sK + ks * (kTaK * 32)), 128, 256), idS, 1u);
        umma_commit(&k_empty);
        umma_commit(&s_full[b]);
        ++ku, ++su;
        return true;
      };
      // O += P V: the two cross terms, then hi x hi
      auto issue_pv = [&](bool first) -> bool {
        if (!mbar_wait_bounded(&v_full, static_cast<uint32_t>(vu & 1), A.err)) return false;
        if (!mbar_wait_bounded(&p_full, static_cast<uint32_t>(pu & 1), A.err)) return false;
        tmem_fence_after();
        const uint32_t d = tmem + cO;
#pragma unroll 1
        for (int ks = 0; ks < kTaK / 8; ++ks) {
          const uint64_t ah = umma_sdesc(smem_addr(sP + ks * 4096), 128, 256);
          const uint64_t al = umma_sdesc(smem_addr(sP + kTaPPlane + ks * 4096), 128, 256);
          const uint64_t bh = umma_sdesc(smem_addr(sV + ks * (HD * 32)), 128, 256);
          const uint64_t bl = umma_sdesc(smem_addr(sV + PL + ks * (HD * 32)), 128, 256);
          umma_tf32_ss(d, ah, bl, idO, (first && ks == 0) ? 0u : 1u);
          umma_tf32_ss(d, al, bh, idO, 1u);
        }
#pragma unroll 1
        for (int ks = 0; ks < kTaK / 8; ++ks)
          umma_tf32_ss(d, umma_sdesc(smem_addr(sP + ks * 4096), 128, 256),
                       umma_sdesc(smem_addr(sV + ks * (HD * 32)), 128, 256), idO, 1u);
        umma_commit(&v_empty);
        umma_commit(&p_empty);
        ++vu, ++pu;
        return true;
      };
      ok = mbar_wait_bounded(&q_ready, 0u, A.err);
      for (int j = 0; j < nt && ok; ++j) ok = issue_s();  // pass 1
      if (ok) ok = issue_s();                               // pass 2: S of the next tile before P V of this one
      for (int j = 0; j < nt && ok; ++j) {
        if (j + 1 < nt) ok = issue_s();
        if (ok) ok = issue_pv(j == 0);
      }
      if (ok) umma_commit(&o_full);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int r = tid;  // query row of the block = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    const int v = v0 + r;
    const bool valid = v < nv;
    const int t = valid ? v / qg : 0, hh = valid ? v - t * qg : 0;
    const int lim = valid ? A.p0 + t : -1;  // last key position of this query
    {  // Q row -> TMEM, hi and lo
      const float *qrow = A.q + static_cast<size_t>(t) * A.ldq + (h0 + hh) * HD;
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t qh[32], ql[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (valid) x = *reinterpret_cast<const float4 *>(qrow + c0 + i);
          tf32_split(x.x, qh[i], ql[i]);
          tf32_split(x.y, qh[i + 1], ql[i + 1]);
          tf32_split(x.z, qh[i + 2], ql[i + 2]);
          tf32_split(x.w, qh[i + 3], ql[i + 3]);
        }
        tmem_st32(tmem + lane_base + cQh + c0, qh);
        tmem_st32(tmem + lane_base + cQl + c0, ql);
      }
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_ready);
    }
    float m = -INFINITY, l = 0.f;
    int su = 0, pu = 0;
    // scores of tile j into sv (the S buffer is released once they are in registers)
    auto load_s = [&](uint32_t (&s0)[32], uint32_t (&s1)[32]) -> bool {
      const int b = su & 1;
      bool w = mbar_wait_bounded(&s_full[b], static_cast<uint32_t>((su >> 1) & 1), A.err);
      w = __all_sync(0xffffffffu, w);
      if (!w) return false;
      tmem_fence_after();
      tmem_ld32(tmem + lane_base + cS + static_cast<uint32_t>(b * kTaK), s0);
      tmem_ld32(tmem + lane_base + cS + static_cast<uint32_t>(b * kTaK + 32), s1);
      tmem_wait_ld();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      ++su;
      return true;
    };
#pragma unroll 1
    for (int j = 0; j < nt && ok; ++j) {  // pass 1: maxima
      uint32_t s0[32], s1[32];
      if (!(ok = load_s(s0, s1))) break;
      const int kb = kbeg + j * kTaK;
#pragma unroll
      for (int c = 0; c < kTaK; ++c)
        if (kb + c < kend && kb + c <= lim)
          m = fmaxf(m, __fmul_rn(__uint_as_float(c < 32 ? s0[c] : s1[c - 32]), A.scale));
    }
#pragma unroll 1
    for (int j = 0; j < nt && ok; ++j) {  // pass 2: probabilities, P to shared memory
      uint32_t s0[32], s1[32];
      if (!(ok = load_s(s0, s1))) break;
      if (pu > 0) {
        bool w = mbar_wait_bounded(&p_empty, static_cast<uint32_t>((pu - 1) & 1), A.err);
        if (!(ok = __all_sync(0xffffffffu, w))) break;
      }
      const int kb = kbeg + j * kTaK;
      uint8_t *prow = sP + (r >> 3) * 256 + (r & 7) * 16;
#pragma unroll
      for (int c4 = 0; c4 < kTaK / 4; ++c4) {
        uint32_t ph[4], pl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = 4 * c4 + e, key = kb + c;
          const float sc = __uint_as_float(c < 32 ? s0[c] : s1[c - 32]);
          float p = 0.f;
          if (key < kend && key <= lim)
            p = exp_nonpos(__fsub_rn(__fmul_rn(sc, A.scale), m));
          l = __fadd_rn(l, p);
          tf32_split(p, ph[e], pl[e]);
        }
        const int off = (c4 >> 1) * 4096 + (c4 & 1) * 128;
        *reinterpret_cast<uint4 *>(prow + off) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
        *reinterpret_cast<uint4 *>(prow + kTaPPlane + off) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor cores
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full);
      ++pu;
    }
    if (ok) {
      bool w = mbar_wait_bounded(&o_full, 0u, A.err);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tmem_fence_after();
      constexpr int PW = pf_part_width(HD);
      float *pp = nsplit == 1 ? nullptr
                              : A.part + ((static_cast<size_t>(g) * nblk + blk) * A.max_splits + sp) * kFqN * PW +
                                    static_cast<size_t>(r) * PW;
      float *dst = A.out + static_cast<size_t>(t) * A.ldq + (h0 + hh) * HD;
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + cO + c0, o);
        tmem_wait_ld();
        if (nsplit == 1) {
          if (valid)
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4 *>(dst + c0 + i) =
                  make_float4(__uint_as_float(o[i]) / l, __uint_as_float(o[i + 1]) / l, __uint_as_float(o[i + 2]) / l,
                              __uint_as_float(o[i + 3]) / l);
        } else {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4 *>(pp + 4 + c0 + i) = make_float4(
                __uint_as_float(o[i]), __uint_as_float(o[i + 1]), __uint_as_float(o[i + 2]), __uint_as_float(o[i + 3]));
        }
      }
      if (nsplit > 1) {
        pp[0] = m;
        pp[1] = l;
        __threadfence();
      }
    }
  }
  tmem_fence_before();
  const int all_ok = __syncthreads_and(ok ? 1 : 0);
  if (warp == 4) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  if (nsplit == 1) return;
  // ---- the block's last split to arrive combines the splits in order
  float *pblk = A.part + (static_cast<size_t>(g) * nblk + blk) * A.max_splits * kFqN * pf_part_width(HD);
  if (tid == 0) {
    unsigned *cnt = A.count + static_cast<size_t>(g) * nblk + blk;
    const unsigned prev = atomicAdd(cnt, 1u);
    const int last = prev == static_cast<unsigned>(nsplit - 1) ? 1 : 0;
    if (last) *cnt = 0u;  // for the next launch (every split of this one has arrived)
    s_last = last;
  }
  __syncthreads();
  if (!s_last || !all_ok) return;
  __threadfence();
  pf_split_combine<HD>(A, pblk, nsplit, v0, nv, qg, h0, reinterpret_cast<float *>(sP), s_l, tid, kTaThreads);
}

}  // namespace c2s
