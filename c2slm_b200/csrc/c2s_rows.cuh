// c2s_rows.cuh -- warp-level row groups of the quantized matvecs.
//
// A warp owns a set of rows of a staged weight chunk and evaluates them in
// groups of up to 8: each lane takes one "unit" of every row (a 32-value
// Q5_0/Q8_0 block, or a 64-value K-quant unit), loads the activation of that
// unit into registers once, and reuses it across the rows of the group.  The
// per-lane partial sums of a group are reduced across the warp with a
// transposing butterfly (8 rows in 9 shuffles).  Every row is summed by the
// same lane tree whatever its group, so results do not depend on how rows
// are spread over warps.
//
// Weight blocks in shared memory keep their GGML layouts (Q5_0 22 B, Q8_0
// 34 B, Q6_K 210 B are only 2-byte aligned); they are read as aligned
// 32-bit windows recombined with funnel shifts.
#pragma once
#include "c2s_device.cuh"

namespace c2s {

// ---------------------------------------------------------------------------
// f32 activation of one 32-value block split into three int8 limbs:
//   x = s * (a + b/254 + c/254^2),  s = max|x|/127,  a, b, c in [-127, 127]
// (reconstruction error <= ~6.2e-8 * max|x|).  A Q8_0 / Q5_0 block dot is
// then three int8 dp4a chains and one f32 combine.
// ---------------------------------------------------------------------------
struct XLimbs {
  int a[8], b[8], c[8];
  float s;
};

__device__ __forceinline__ void make_limbs(const float (&x)[32], XLimbs &L) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
  L.s = amax / 127.f;
  const float inv = amax > 0.f ? 127.f / amax : 0.f;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    uint32_t wa = 0, wb = 0, wc = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float y = x[4 * t + e] * inv;
      const float a = rintf(y);
      const float r1 = __fmul_rn(y - a, 254.f);
      const float b = rintf(r1);
      const float c = rintf(__fmul_rn(r1 - b, 254.f));
      wa |= (static_cast<uint32_t>(static_cast<int>(a)) & 0xFFu) << (8 * e);
      wb |= (static_cast<uint32_t>(static_cast<int>(b)) & 0xFFu) << (8 * e);
      wc |= (static_cast<uint32_t>(static_cast<int>(c)) & 0xFFu) << (8 * e);
    }
    L.a[t] = static_cast<int>(wa);
    L.b[t] = static_cast<int>(wb);
    L.c[t] = static_cast<int>(wc);
  }
}

__device__ __forceinline__ float limbs_combine(int A, int B, int C, float s) {
  const float k = 1.f / 254.f;
  return s * fmaf(fmaf(static_cast<float>(C), k, static_cast<float>(B)), k, static_cast<float>(A));
}



// n 32-bit words starting at a 2-byte aligned shared-memory address: n + 1
// aligned loads (the word after the range must be readable).
template <int N>
__device__ __forceinline__ void ld_window(const uint8_t *p, uint32_t (&out)[N]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  uint32_t prev = w[0];
#pragma unroll
  for (int t = 0; t < N; ++t) {
    const uint32_t nxt = w[t + 1];
    out[t] = __funnelshift_rc(prev, nxt, sh);
    prev = nxt;
  }
}

// the n aligned words covering [p & ~3, (p & ~3) + 4n)
template <int N>
__device__ __forceinline__ void ld_aligned(const uint8_t *p, uint32_t (&out)[N]) {
  const uint32_t *w = reinterpret_cast<const uint32_t *>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
#pragma unroll
  for (int t = 0; t < N; ++t) out[t] = w[t];
}

// ---------------------------------------------------------------------------
// activations in shared memory
//   limbs (Q5_0 / Q8_0): x of block b = s[b] * (a + b/254 + c/254^2), the
//     three int8 limbs packed 4 per word, word t of block b at [t*nb + b]
//   Q8_K (Q4_K / Q6_K): the split layout of Q8KView
// ---------------------------------------------------------------------------
struct LimbsView {
  const int *a, *b, *c;
  const float *s;
  int nb;
};

__device__ __forceinline__ void load_limbs(const LimbsView &V, int u, bool ok, XLimbs &L) {
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    L.a[t] = ok ? V.a[t * V.nb + u] : 0;
    L.b[t] = ok ? V.b[t * V.nb + u] : 0;
    L.c[t] = ok ? V.c[t * V.nb + u] : 0;
  }
  L.s = ok ? V.s[u] : 0.f;
}

// Limbs of the f32 activation held 4 values per thread: the thread with
// float4 index i holds word t = i % 8 of block i / 8.  All lanes of the warp
// must call it (the 8 threads of a block exchange their max).
__device__ __forceinline__ void put_limbs(const float4 v, int i, bool valid, int *la, int *lb, int *lc, float *ls,
                                          int nb) {
  float amax = valid ? fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))) : 0.f;
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (!valid) return;
  const int blk = i >> 3, t = i & 7;
  const float inv = amax > 0.f ? 127.f / amax : 0.f;
  const float x[4] = {v.x, v.y, v.z, v.w};
  uint32_t wa = 0, wb = 0, wc = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float y = x[e] * inv;
    const float a = rintf(y);
    const float r1 = __fmul_rn(y - a, 254.f);
    const float b = rintf(r1);
    const float c = rintf(__fmul_rn(r1 - b, 254.f));
    wa |= (static_cast<uint32_t>(static_cast<int>(a)) & 0xFFu) << (8 * e);
    wb |= (static_cast<uint32_t>(static_cast<int>(b)) & 0xFFu) << (8 * e);
    wc |= (static_cast<uint32_t>(static_cast<int>(c)) & 0xFFu) << (8 * e);
  }
  la[t * nb + blk] = static_cast<int>(wa);
  lb[t * nb + blk] = static_cast<int>(wb);
  lc[t * nb + blk] = static_cast<int>(wc);
  if (t == 0) ls[blk] = amax / 127.f;
}

// ---------------------------------------------------------------------------
// unit dots against register-resident activations
// ---------------------------------------------------------------------------
// Q8_0 block (fp16 d, 32 int8) at a 2-byte aligned address: 9 aligned
// words cover it; sh = 0 or 16 is the block's offset in the first word.
__device__ __forceinline__ float limbs_dot_q8_0(const uint8_t *blk, const XLimbs &L) {
  uint32_t w[9];
  ld_aligned<9>(blk, w);
  const uint32_t sh = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(blk) & 3u) * 8u;
  const float d = h2f(static_cast<uint16_t>((w[0] >> sh) & 0xffffu));
  int A = 0, B = 0, C = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int q = static_cast<int>(__funnelshift_rc(w[t], w[t + 1], 16u + sh));
    A = __dp4a(q, L.a[t], A);
    B = __dp4a(q, L.b[t], B);
    C = __dp4a(q, L.c[t], C);
  }
  return d * limbs_combine(A, B, C, L.s);
}

// Q5_0 block (fp16 d, u32 qh, 16 B nibbles) at a 2-byte aligned address;
// int8(q - 16) = nibble | (high bit ? 0 : 0xF0)
__device__ __forceinline__ float limbs_dot_q5_0(const uint8_t *blk, const XLimbs &L) {
  uint32_t w[6];
  ld_aligned<6>(blk, w);
  const uint32_t sh = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(blk) & 3u) * 8u;
  const float d = h2f(static_cast<uint16_t>((w[0] >> sh) & 0xffffu));
  const uint32_t qh = __funnelshift_rc(w[0], w[1], 16u + sh);
  int A = 0, B = 0, C = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t q = __funnelshift_rc(w[1 + t], w[2 + t], 16u + sh);
    const uint32_t hl = spread4((qh >> (4 * t)) & 0xFu) ^ 0x01010101u;
    const uint32_t hh = spread4((qh >> (16 + 4 * t)) & 0xFu) ^ 0x01010101u;
    const int lo = static_cast<int>((q & 0x0F0F0F0Fu) | (hl * 0xF0u));
    const int hi = static_cast<int>(((q >> 4) & 0x0F0F0F0Fu) | (hh * 0xF0u));
    A = __dp4a(lo, L.a[t], A);
    B = __dp4a(lo, L.b[t], B);
    C = __dp4a(lo, L.c[t], C);
    A = __dp4a(hi, L.a[4 + t], A);
    B = __dp4a(hi, L.b[4 + t], B);
    C = __dp4a(hi, L.c[4 + t], C);
  }
  return d * limbs_combine(A, B, C, L.s);
}

// 4-way dot of unsigned bytes (a) and signed bytes (b), plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Q4_K unit (superblock sb, sub-block pair j): activation of the unit
struct Q4Act {
  int4 xa, xb, xc, xd;
  float d8, bs01, bs23;
};

__device__ __forceinline__ void load_q4act(const Q8KView &x, int u, bool ok, Q4Act &A) {
  const int sb = u >> 2, j = u & 3;
  if (!ok) {
    A.xa = A.xb = A.xc = A.xd = make_int4(0, 0, 0, 0);
    A.d8 = A.bs01 = A.bs23 = 0.f;
    return;
  }
  const int8_t *q8 = x.qs + q8_pad_index(sb * 256 + 64 * j);
  A.xa = *reinterpret_cast<const int4 *>(q8);
  A.xb = *reinterpret_cast<const int4 *>(q8 + 16);
  A.xc = *reinterpret_cast<const int4 *>(q8 + 32);
  A.xd = *reinterpret_cast<const int4 *>(q8 + 48);
  A.d8 = x.d[sb];
  const int4 bs = *reinterpret_cast<const int4 *>(x.bsum + sb * 16 + 4 * j);
  A.bs01 = static_cast<float>(bs.x + bs.y);
  A.bs23 = static_cast<float>(bs.z + bs.w);
}

// Per-lane constants of the Q4_K unit a lane evaluates: sub-block pair
// j = lane & 3 of its superblock (every row pass starts at a multiple of 32
// units, so j is fixed for the lane).
struct Q4Lane {
  uint32_t sel_ab, sel_c;  // byte_perm selectors of the 6-bit scale/min bytes of pair j
  uint32_t hi;             // j >= 2: scales split over the low and high bytes
  int qoff;                // offset of the pair's 32 quant bytes
};

__device__ __forceinline__ Q4Lane q4_lane() {
  const int j = threadIdx.x & 3;
  Q4Lane K;
  K.sel_ab = (j & 1) ? 0x7632u : 0x5410u;
  K.sel_c = (j & 1) ? 0x3232u : 0x1010u;
  K.hi = j >= 2 ? 1u : 0u;
  K.qoff = 16 + 32 * j;
  return K;
}

// f32 term of one Q4_K sub-block pair (internal/simd/
// c2_tensor_dot_q4_k_q8_k_nosimd_gen.go:20-68); blk is 16-B aligned.
// The 6-bit scales and mins of sub-blocks 2j, 2j+1 (tensor/ops.go:354-361)
// are unpacked together: W = [sc0, sc1, m0, m1] as bytes.
__device__ __forceinline__ float unit_q4k_reg(const uint8_t *blk, const Q4Lane &K, const Q4Act &A) {
  const uint4 h = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, scales[0..11]
  const float2 dmn = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
  const float d = dmn.x, dmin = dmn.y;
  // AB = s[2k], s[2k+1], s[4+2k], s[5+2k]; CC = s[8+2k], s[9+2k] twice (k = j & 1)
  const uint32_t AB = __byte_perm(h.y, h.z, K.sel_ab);
  const uint32_t CC = __byte_perm(h.w, 0u, K.sel_c);
  const uint32_t lowW = AB & 0x3F3F3F3Fu;
  const uint32_t highW = (CC & 0x00000F0Fu) | ((CC >> 4) & 0x0F0F0000u) | ((AB >> 2) & 0x30303030u);
  const uint32_t W = K.hi ? highW : lowW;
  const int sc0 = static_cast<int>(W & 0xFFu), sc1 = static_cast<int>((W >> 8) & 0xFFu);
  const int m0 = static_cast<int>((W >> 16) & 0xFFu), m1 = static_cast<int>(W >> 24);
  const uint4 wa = *reinterpret_cast<const uint4 *>(blk + K.qoff);
  const uint4 wb = *reinterpret_cast<const uint4 *>(blk + K.qoff + 16);
  const uint32_t m4 = 0x0F0F0F0Fu, h4 = 0xF0F0F0F0u;
  // low nibbles as they are; high nibbles in place (16 x the nibble, an
  // unsigned byte) -- their dot is exactly 16 x the nibble dot
  int lo = 0, hi16 = 0;
  lo = __dp4a(static_cast<int>(wa.x & m4), A.xa.x, lo);
  lo = __dp4a(static_cast<int>(wa.y & m4), A.xa.y, lo);
  lo = __dp4a(static_cast<int>(wa.z & m4), A.xa.z, lo);
  lo = __dp4a(static_cast<int>(wa.w & m4), A.xa.w, lo);
  lo = __dp4a(static_cast<int>(wb.x & m4), A.xb.x, lo);
  lo = __dp4a(static_cast<int>(wb.y & m4), A.xb.y, lo);
  lo = __dp4a(static_cast<int>(wb.z & m4), A.xb.z, lo);
  lo = __dp4a(static_cast<int>(wb.w & m4), A.xb.w, lo);
  hi16 = dp4a_us(wa.x & h4, A.xc.x, hi16);
  hi16 = dp4a_us(wa.y & h4, A.xc.y, hi16);
  hi16 = dp4a_us(wa.z & h4, A.xc.z, hi16);
  hi16 = dp4a_us(wa.w & h4, A.xc.w, hi16);
  hi16 = dp4a_us(wb.x & h4, A.xd.x, hi16);
  hi16 = dp4a_us(wb.y & h4, A.xd.y, hi16);
  hi16 = dp4a_us(wb.z & h4, A.xd.z, hi16);
  hi16 = dp4a_us(wb.w & h4, A.xd.w, hi16);
  const int hi = hi16 >> 4;  // exact: a multiple of 16
  const float dd = __fmul_rn(d, A.d8), dm = __fmul_rn(dmin, A.d8);
  const float t0 = __fsub_rn(__fmul_rn(static_cast<float>(lo), __fmul_rn(dd, static_cast<float>(sc0))),
                             __fmul_rn(A.bs01, __fmul_rn(dm, static_cast<float>(m0))));
  const float t1 = __fsub_rn(__fmul_rn(static_cast<float>(hi), __fmul_rn(dd, static_cast<float>(sc1))),
                             __fmul_rn(A.bs23, __fmul_rn(dm, static_cast<float>(m1))));
  return __fadd_rn(t0, t1);
}

// Q6_K unit (sb, n, kp): quarters ka = kp and kb = kp + 2 of half n
struct Q6Act {
  int xa[8], xb[8];
  int bsa0, bsa1, bsb0, bsb1;
  float d8;
};

__device__ __forceinline__ void load_q6act(const Q8KView &x, int u, bool ok, Q6Act &A) {
  const int sb = u >> 2, n = (u >> 1) & 1, kp = u & 1;
  if (!ok) {
#pragma unroll
    for (int t = 0; t < 8; ++t) A.xa[t] = A.xb[t] = 0;
    A.bsa0 = A.bsa1 = A.bsb0 = A.bsb1 = 0;
    A.d8 = 0.f;
    return;
  }
  const int4 *qa = reinterpret_cast<const int4 *>(x.qs + q8_pad_index(sb * 256 + 128 * n + 32 * kp));
  const int4 *qb = reinterpret_cast<const int4 *>(x.qs + q8_pad_index(sb * 256 + 128 * n + 32 * (kp + 2)));
  const int4 a0 = qa[0], a1 = qa[1], b0 = qb[0], b1 = qb[1];
  A.xa[0] = a0.x; A.xa[1] = a0.y; A.xa[2] = a0.z; A.xa[3] = a0.w;
  A.xa[4] = a1.x; A.xa[5] = a1.y; A.xa[6] = a1.z; A.xa[7] = a1.w;
  A.xb[0] = b0.x; A.xb[1] = b0.y; A.xb[2] = b0.z; A.xb[3] = b0.w;
  A.xb[4] = b1.x; A.xb[5] = b1.y; A.xb[6] = b1.z; A.xb[7] = b1.w;
  const int32_t *bs = x.bsum + sb * 16 + 8 * n;
  A.bsa0 = bs[2 * kp];
  A.bsa1 = bs[2 * kp + 1];
  A.bsb0 = bs[2 * kp + 4];
  A.bsb1 = bs[2 * kp + 5];
  A.d8 = x.d[sb];
}

// this unit's share of the superblock's int32 isum
// (internal/simd/c2_tensor_gemv2_q6_k_q8_k_nosimd_gen.go:80-237)
__device__ __forceinline__ int unit_q6k_reg(const uint8_t *blk, int n, int kp, const Q6Act &A) {
  uint32_t l[8], h[8];
  ld_window<8>(blk + 64 * n + 32 * kp, l);
  ld_window<8>(blk + 128 + 32 * n, h);
  const uint32_t sca = ld16(blk + 192 + 8 * n + 2 * kp);
  const uint32_t scb = ld16(blk + 192 + 8 * n + 2 * kp + 4);
  // 6-bit quants of quarters ka = kp and kb = kp + 2: low nibble | 2 high
  // bits (qh >> 2k) at bits 4-5, i.e. qh << (4 - 2ka) and qh >> (2kb - 4)
  const uint32_t sha = 4u - 2u * static_cast<uint32_t>(kp), shb = 2u * static_cast<uint32_t>(kp);
  int sa0 = 0, sa1 = 0, sb0 = 0, sb1 = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t va = (l[t] & 0x0F0F0F0Fu) | ((h[t] << sha) & 0x30303030u);
    const uint32_t vb = ((l[t] >> 4) & 0x0F0F0F0Fu) | ((h[t] >> shb) & 0x30303030u);
    if (t < 4) {
      sa0 = __dp4a(static_cast<int>(va), A.xa[t], sa0);
      sb0 = __dp4a(static_cast<int>(vb), A.xb[t], sb0);
    } else {
      sa1 = __dp4a(static_cast<int>(va), A.xa[t], sa1);
      sb1 = __dp4a(static_cast<int>(vb), A.xb[t], sb1);
    }
  }
  const int sa_0 = static_cast<int8_t>(sca & 0xFFu), sa_1 = static_cast<int8_t>(sca >> 8);
  const int sb_0 = static_cast<int8_t>(scb & 0xFFu), sb_1 = static_cast<int8_t>(scb >> 8);
  return ((sa0 - 32 * A.bsa0) * sa_0 + (sa1 - 32 * A.bsa1) * sa_1) +
         ((sb0 - 32 * A.bsb0) * sb_0 + (sb1 - 32 * A.bsb1) * sb_1);
}

// ---------------------------------------------------------------------------
// transposing butterfly over NR rows (NR a power of two <= 32): after it,
// lane l holds the warp sum of row (l >> (5 - log2 NR)) in the return value
// ---------------------------------------------------------------------------
template <int NR>
__device__ __forceinline__ float reduce_rows(float (&v)[NR]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = NR / 2, o = 16; h >= 1; h >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? v[i] : v[i + h];
      const float keep = up ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = 32 / NR / 2; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

template <int NR>
__device__ __forceinline__ int reduced_row_of_lane() {
  return NR == 1 ? 0 : ((threadIdx.x & 31) >> (NR == 2 ? 4 : NR == 4 ? 3 : NR == 8 ? 2 : NR == 16 ? 1 : 0));
}

// NR rows at base, base + rstep, ... (all valid) -> y[0], y[ystep], ...
// Lanes past the last unit evaluate a clamped unit and discard it, so the
// row loop has no branches and the rows interleave.
template <int TYPE, int NR>
__device__ __forceinline__ void row_group(const uint8_t *base, size_t rstep, int U, const LimbsView &LV,
                                          const Q8KView &q8, float *y, int ystep) {
  const int lane = threadIdx.x & 31;
  float acc[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) acc[i] = 0.f;
  for (int ub = 0; ub < U; ub += 32) {
    const bool ok = ub + lane < U;
    const int u = ok ? ub + lane : U - 1;
    if constexpr (TYPE == T_Q8_0 || TYPE == T_Q5_0) {
      XLimbs L;
      load_limbs(LV, u, true, L);
      const int boff = u * (TYPE == T_Q8_0 ? 34 : 22);
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const uint8_t *blk = base + i * rstep + boff;
        const float t = TYPE == T_Q8_0 ? limbs_dot_q8_0(blk, L) : limbs_dot_q5_0(blk, L);
        acc[i] += ok ? t : 0.f;
      }
    } else if constexpr (TYPE == T_Q4_K) {
      Q4Act A;
      load_q4act(q8, u, true, A);
      const int boff = (u >> 2) * 144;
      const Q4Lane K = q4_lane();
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const float t = unit_q4k_reg(base + i * rstep + boff, K, A);
        acc[i] += ok ? t : 0.f;
      }
    } else if constexpr (TYPE == T_Q6_K) {
      Q6Act A;
      load_q6act(q8, u, true, A);
      const int boff = (u >> 2) * 210;
#pragma unroll
      for (int i = 0; i < NR; ++i) {  // the 4 lanes of a superblock combine
        const uint8_t *blk = base + i * rstep + boff;
        int is = unit_q6k_reg(blk, (u >> 1) & 1, u & 1, A);
        is += __shfl_xor_sync(0xffffffffu, is, 1);
        is += __shfl_xor_sync(0xffffffffu, is, 2);
        const float t = __fmul_rn(static_cast<float>(is), __fmul_rn(h2f(ld16(blk + 208)), A.d8));
        acc[i] += (ok && (u & 3) == 0) ? t : 0.f;
      }
    }
  }
  const float v = reduce_rows<NR>(acc);
  const int r = reduced_row_of_lane<NR>();
  if ((lane & (32 / NR - 1)) == 0) y[r * ystep] = v;
}

// Rows first, first + ws, ... (cnt of them) of a staged chunk -> y[local
// row], in groups of 8 (Q5_0 / Q8_0; 4 for the K-quants, whose larger
// per-row register state makes 8-row groups slower), 4, 2 and 1 rows.  U
// units per row; ws warps share the chunk.
template <int TYPE>
__device__ __forceinline__ void warp_rows(const uint8_t *rows, int row_bytes, int U, int first, int cnt,
                                          const LimbsView &LV, const Q8KView &q8, float *y, int ws = kWarps) {
  const size_t rstep = static_cast<size_t>(ws) * row_bytes;
  const uint8_t *base = rows + static_cast<size_t>(first) * row_bytes;
  float *yp = y + first;
  int left = cnt;
  if constexpr (TYPE == T_Q4_K || TYPE == T_Q6_K) {
    for (; left >= 4; left -= 4, base += 4 * rstep, yp += 4 * ws)
      row_group<TYPE, 4>(base, rstep, U, LV, q8, yp, ws);
  } else {
    for (; left >= 8; left -= 8, base += 8 * rstep, yp += 8 * ws)
      row_group<TYPE, 8>(base, rstep, U, LV, q8, yp, ws);
  }
  if (left >= 4) {
    row_group<TYPE, 4>(base, rstep, U, LV, q8, yp, ws);
    left -= 4, base += 4 * rstep, yp += 4 * ws;
  }
  if (left >= 2) {
    row_group<TYPE, 2>(base, rstep, U, LV, q8, yp, ws);
    left -= 2, base += 2 * rstep, yp += 2 * ws;
  }
  if (left >= 1) row_group<TYPE, 1>(base, rstep, U, LV, q8, yp, ws);
}

}  // namespace c2s
