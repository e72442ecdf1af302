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
// shared-memory stages and two TMEM accumulator sets overlap the copies of
// round s+1, the MMAs of round s and the epilogue of round s-1.
// ---------------------------------------------------------------------------
constexpr int kPfM = 128, kPfN = 128, kPfThreads = 320;
constexpr int kPfKStep = 128 * 32, kPfPlane = 8 * kPfKStep;  // per superblock: 32 KB
constexpr int kPfTokTile = kPfPlane;                          // token tile per superblock
constexpr int kPfD8Bytes = kPfN * 4, kPfBsBytes = kPfN * 16;
constexpr int kPfStage = 2 * kPfPlane + kPfTokTile + kPfD8Bytes + kPfBsBytes;
constexpr int kPfStages = 2;
constexpr int kPfSmem = kPfStages * kPfStage + 128;

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
  __shared__ __align__(8) uint64_t full[kPfStages], empty[kPfStages], tfull[2], tempty[2];
  __shared__ uint32_t s_tmem;
  constexpr uint32_t kStageBytes = kPfStage;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = R * kPfM, t0 = T * kPfN;
  const int nsb = G.cols / 256;
  if (tid == 0) {
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1 + 8);  // the MMAs' commit and the eight epilogue warps
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
        bulk_g2s(dst + 2 * kPfPlane + kPfTokTile, G.ad + (tb0 + s) * kPfN, kPfD8Bytes, &full[st]);
        bulk_g2s(dst + 2 * kPfPlane + kPfTokTile + kPfD8Bytes, G.abs + (tb0 + s) * kPfN * 8, kPfBsBytes, &full[st]);
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
      const int st = s % kPfStages, tb = s & 1;
      const uint4 rv = rin;
      if (s + 1 < nsb) rin = __ldg(ri + s + 1);
      ok = mbar_wait_bounded(&tfull[tb], static_cast<uint32_t>((s >> 1) & 1), G.err);
      {  // ok made uniform over the epilogue warps (all leave together)
        uint32_t all;
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, 2, 256, q;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(all) : "r"(ok ? 1u : 0u) : "memory");
        ok = all != 0;
      }
      if (!ok) break;
      tmem_fence_after();
      const float dr = __uint_as_float(rv.x), dmr = __uint_as_float(rv.y);
      const uint8_t *stg = smem + st * kPfStage + 2 * kPfPlane + kPfTokTile;
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
        mbar_arrive(&empty[st]);
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
  constexpr int PW = HD + 2;
  float *pblk = A.part + (static_cast<size_t>(g) * nblk + blk) * A.max_splits * kFqN * PW;
  {
    float *pp = pblk + static_cast<size_t>(sp) * kFqN * PW;
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < OD; ++b) pp[qof(a) * PW + 2 + dof(b)] = o[a][b];
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
  // weights of the splits for each query: w_s = exp(m_s - M) (float64), over s in order
  float *s_w = Pt;  // [max_splits][kFqN]
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
  for (int i = tid; i < kFqN * HD; i += kThreads) {
    const int qi = i / HD, dd = i - qi * HD, v = v0 + qi;
    if (v >= nv) continue;
    float acc = 0.f;
    for (int j = 0; j < nsplit; ++j)
      acc = __fadd_rn(acc, __fmul_rn(s_w[j * kFqN + qi], __ldcg(pblk + (static_cast<size_t>(j) * kFqN + qi) * PW + 2 + dd)));
    const int t = v / qg, h = v - t * qg;
    A.out[static_cast<size_t>(t) * A.ldq + (h0 + h) * HD + dd] = acc / s_l[qi];
  }
}

}  // namespace c2s
