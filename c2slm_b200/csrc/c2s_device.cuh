// c2s_device.cuh -- device building blocks of the sm_100a token loop.
//
// Block layouts are GGML's, read in place from HBM/shared memory
// (tensor/ops.go:11-22): Q5_0 22 B, Q8_0 34 B, Q4_K 144 B, Q6_K 210 B per
// block, Q8_K activations 292 B per 256 values.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace c2s {

constexpr int kThreads = 256;              // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;                 // weight staging ring depth
constexpr int kStageBytes = 16384;         // payload per stage
constexpr int kStageAlloc = kStageBytes + 64;  // + alignment slack
constexpr int kMaxSegs = 3;
constexpr int kMaxSplits = 148;            // attention KV splits per kv head (upper bound)
constexpr int kMinSplitLen = 32;           // positions per split before splitting further

// device-side error flags (DevState::err)
constexpr unsigned kErrMbarTimeout = 1u;
constexpr unsigned kErrBadType = 2u;
constexpr unsigned kErrPos = 4u;
constexpr unsigned kErrCounter = 8u;

// GGML ids (gguf/reader.go:21-37)
constexpr int T_F32 = 0, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14;

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// n arrivals on a barrier in one operation
__device__ __forceinline__ void mbar_arrive_n(uint64_t *bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait budget for every bounded spin: ~2 s at the B200's ~2 GHz SM clock,
// measured with the SM-local cycle counter (cheap to read, unlike
// %globaltimer).
constexpr long long kSpinCycles = 4000000000LL;

// Bounded wait: gives up after kSpinCycles, sets *err and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, unsigned *err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) break;
  }
  atomicOr(err, kErrMbarTimeout);
  return false;
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map), completion
// tracked by the mbarrier's transaction count.  dst/src 16-B aligned, bytes
// a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Programmatic dependent launch (sm_90+): the wait blocks until the previous
// grid in the stream has completed and its writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// scalar helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint16_t ld16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }

// 32-bit load from a 2-byte aligned shared/global address (reads the next
// aligned word too; buffers carry slack for it).
__device__ __forceinline__ uint32_t ld32u(const uint8_t *p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
  return __funnelshift_r(w[0], w[1], static_cast<uint32_t>(a & 3u) * 8u);
}

// bit t of b (t<4) -> bit 8t of the result
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return (b * 0x00204081u) & 0x01010101u; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Barrier over the kThreads compute threads of a CTA (named barrier 1).  In
// the persistent kernel a producer warp runs beside them and must not be
// waited for; in the per-phase kernels these are all the threads.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory"); }

// Block-wide sum with a fixed reduction tree (deterministic).  `scratch`
// holds kWarps floats.  All compute threads get the result.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  csync();
  if (l == 0) scratch[w] = v;
  csync();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) r += scratch[i];
  return r;
}

// ---------------------------------------------------------------------------
// Q8_K activation in shared memory (split layout)
//   qs   : int8 [cols], padded 16 B after every 64 values (bank spread)
//   d    : f32 [nsb]
//   bsum : int32 [nsb*16]
// ---------------------------------------------------------------------------
__host__ __device__ constexpr int q8_pad_index(int e) { return e + (e >> 6) * 16; }
__host__ __device__ constexpr int q8_qs_bytes(int cols) { return q8_pad_index(cols) + 64; }

struct Q8KView {
  const int8_t *qs;
  const float *d;
  const int32_t *bsum;
};

// Quantises one 256-value superblock exactly as C2_quantize_row_q8_k
// (internal/simd/c2_quantize_q8_k_gen.go:11-91): amax; d = amax/127;
// q = trunc(x*(127/amax) +- 0.5) clamped to +-127; bsum of each 16.  Every
// float op is explicitly rounded (no FMA contraction).  Executed by one warp:
// lane l owns x[8l .. 8l+7]; bsum j = lanes 2j, 2j+1.
// Writes q (256 int8 in natural order through `put_q`), d and bsums.
template <class PutQ>
__device__ __forceinline__ void quantize_sb_warp(const float (&x)[8], float *d_out, int32_t *bsum_out,
                                                 PutQ put_q) {
  const int lane = threadIdx.x & 31;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = x[i];
    const float a = v < 0.f ? -v : v;
    amax = a > amax ? a : amax;
  }
  amax = warp_max(amax);
  int q[8];
  if (amax == 0.f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
    if (lane == 0) *d_out = 0.f;
  } else {
    const float iscale = __fdiv_rn(127.f, amax);
    if (lane == 0) *d_out = __fdiv_rn(amax, 127.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = __fmul_rn(x[i], iscale);
      const float r = v >= 0.f ? __fadd_rn(v, 0.5f) : __fsub_rn(v, 0.5f);
      int qi = static_cast<int>(r);  // truncation toward zero, like Go's int(float32)
      qi = qi > 127 ? 127 : qi;
      qi = qi < -127 ? -127 : qi;
      q[i] = qi;
    }
  }
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += q[i];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  if ((lane & 1) == 0) bsum_out[lane >> 1] = s;
  put_q(lane, q);
}

// ---------------------------------------------------------------------------
// Per-unit dot products.  A "unit" is the work one lane does on one row:
//   Q4_K : (superblock, j)      64 values, 4 units per superblock
//   Q6_K : (superblock, n, kp)  64 values, 4 units per superblock
//   Q5_0 : one 32-value block
//   Q8_0 : one 32-value block
// ---------------------------------------------------------------------------

// Q4_K x Q8_K sub-block pair j of superblock sb (internal/simd/
// c2_tensor_dot_q4_k_q8_k_nosimd_gen.go:20-68).  `blk` is 16-B aligned.
// Returns the f32 term the reference adds for this j; lo/hi receive the
// int32 sub-block dots (the bit-exact contract).
__device__ __forceinline__ float unit_q4k(const uint8_t *blk, int sb, int j, const Q8KView &x, int &lo_out,
                                          int &hi_out) {
  const uint32_t dh = *reinterpret_cast<const uint32_t *>(blk);
  const float d = h2f(static_cast<uint16_t>(dh & 0xffffu));
  const float dmin = h2f(static_cast<uint16_t>(dh >> 16));
  const uint8_t *s = blk + 4;
  // 6-bit scale / min unpack (tensor/ops.go:354-361)
  const int i0 = 2 * j, i1 = 2 * j + 1;
  int sc0, m0, sc1, m1;
  if (j < 2) {
    sc0 = s[i0] & 63;
    m0 = s[i0 + 4] & 63;
    sc1 = s[i1] & 63;
    m1 = s[i1 + 4] & 63;
  } else {
    sc0 = (s[i0 + 4] & 15) | ((s[i0 - 4] >> 6) << 4);
    m0 = (s[i0 + 4] >> 4) | ((s[i0] >> 6) << 4);
    sc1 = (s[i1 + 4] & 15) | ((s[i1 - 4] >> 6) << 4);
    m1 = (s[i1 + 4] >> 4) | ((s[i1] >> 6) << 4);
  }
  const uint4 wa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * j);
  const uint4 wb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * j);
  const int8_t *q8 = x.qs + q8_pad_index(sb * 256 + 64 * j);
  const int4 xa = *reinterpret_cast<const int4 *>(q8);
  const int4 xb = *reinterpret_cast<const int4 *>(q8 + 16);
  const int4 xc = *reinterpret_cast<const int4 *>(q8 + 32);
  const int4 xd = *reinterpret_cast<const int4 *>(q8 + 48);
  const uint32_t m4 = 0x0F0F0F0Fu;
  int lo = 0, hi = 0;
  lo = __dp4a(static_cast<int>(wa.x & m4), xa.x, lo);
  lo = __dp4a(static_cast<int>(wa.y & m4), xa.y, lo);
  lo = __dp4a(static_cast<int>(wa.z & m4), xa.z, lo);
  lo = __dp4a(static_cast<int>(wa.w & m4), xa.w, lo);
  lo = __dp4a(static_cast<int>(wb.x & m4), xb.x, lo);
  lo = __dp4a(static_cast<int>(wb.y & m4), xb.y, lo);
  lo = __dp4a(static_cast<int>(wb.z & m4), xb.z, lo);
  lo = __dp4a(static_cast<int>(wb.w & m4), xb.w, lo);
  hi = __dp4a(static_cast<int>((wa.x >> 4) & m4), xc.x, hi);
  hi = __dp4a(static_cast<int>((wa.y >> 4) & m4), xc.y, hi);
  hi = __dp4a(static_cast<int>((wa.z >> 4) & m4), xc.z, hi);
  hi = __dp4a(static_cast<int>((wa.w >> 4) & m4), xc.w, hi);
  hi = __dp4a(static_cast<int>((wb.x >> 4) & m4), xd.x, hi);
  hi = __dp4a(static_cast<int>((wb.y >> 4) & m4), xd.y, hi);
  hi = __dp4a(static_cast<int>((wb.z >> 4) & m4), xd.z, hi);
  hi = __dp4a(static_cast<int>((wb.w >> 4) & m4), xd.w, hi);
  lo_out = lo;
  hi_out = hi;
  const float d8 = x.d[sb];
  const float dd = __fmul_rn(d, d8), dm = __fmul_rn(dmin, d8);
  const int32_t *bs = x.bsum + sb * 16 + 4 * j;
  const float bs01 = static_cast<float>(bs[0] + bs[1]);
  const float bs23 = static_cast<float>(bs[2] + bs[3]);
  const float t0 = __fsub_rn(__fmul_rn(static_cast<float>(lo), __fmul_rn(dd, static_cast<float>(sc0))),
                             __fmul_rn(bs01, __fmul_rn(dm, static_cast<float>(m0))));
  const float t1 = __fsub_rn(__fmul_rn(static_cast<float>(hi), __fmul_rn(dd, static_cast<float>(sc1))),
                             __fmul_rn(bs23, __fmul_rn(dm, static_cast<float>(m1))));
  return __fadd_rn(t0, t1);
}

// Q6_K x Q8_K unit (sb, n, kp): quarters k = kp and kp+2 of half n
// (internal/simd/c2_tensor_gemv2_q6_k_q8_k_nosimd_gen.go:80-237).  Returns
// this unit's share of the superblock's int32 isum; the 4 units of a
// superblock sum exactly (integer) before the f32 scale.
__device__ __forceinline__ int unit_q6k_isum(const uint8_t *blk, int sb, int n, int kp, const Q8KView &x) {
  const uint8_t *ql = blk + 64 * n + 32 * kp;
  const uint8_t *qh = blk + 128 + 32 * n;
  const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * n);
  const int ka = kp, kb = kp + 2;
  const int8_t *q8a = x.qs + q8_pad_index(sb * 256 + 128 * n + 32 * ka);
  const int8_t *q8b = x.qs + q8_pad_index(sb * 256 + 128 * n + 32 * kb);
  int sa0 = 0, sa1 = 0, sb0 = 0, sb1 = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t l4 = ld32u(ql + 4 * t);
    const uint32_t h4 = ld32u(qh + 4 * t);
    const uint32_t va = (l4 & 0x0F0F0F0Fu) | (((h4 >> (2 * ka)) & 0x03030303u) << 4);
    const uint32_t vb = ((l4 >> 4) & 0x0F0F0F0Fu) | (((h4 >> (2 * kb)) & 0x03030303u) << 4);
    const int xa = *reinterpret_cast<const int *>(q8a + 4 * t);
    const int xb = *reinterpret_cast<const int *>(q8b + 4 * t);
    if (t < 4) {
      sa0 = __dp4a(static_cast<int>(va), xa, sa0);
      sb0 = __dp4a(static_cast<int>(vb), xb, sb0);
    } else {
      sa1 = __dp4a(static_cast<int>(va), xa, sa1);
      sb1 = __dp4a(static_cast<int>(vb), xb, sb1);
    }
  }
  const int32_t *bs = x.bsum + sb * 16 + 8 * n;
  return ((sa0 - 32 * bs[2 * ka]) * sc[2 * ka] + (sa1 - 32 * bs[2 * ka + 1]) * sc[2 * ka + 1]) +
         ((sb0 - 32 * bs[2 * kb]) * sc[2 * kb] + (sb1 - 32 * bs[2 * kb + 1]) * sc[2 * kb + 1]);
}

// Q5_0 block . f32 x (tensor/ops.go:40-74).  `xt` points at element 0 of the
// block in the transposed x layout (element i at xt[i*stride]).
__device__ __forceinline__ float unit_q5_0(const uint8_t *blk, const float *xt, int stride) {
  const float d = h2f(ld16(blk));
  const uint32_t qh = static_cast<uint32_t>(ld16(blk + 2)) | (static_cast<uint32_t>(ld16(blk + 4)) << 16);
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t w = ld32u(blk + 6 + 4 * t);
    const uint32_t lo = (w & 0x0F0F0F0Fu) | (spread4((qh >> (4 * t)) & 0xFu) << 4);
    const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) | (spread4((qh >> (16 + 4 * t)) & 0xFu) << 4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sum = fmaf(static_cast<float>(static_cast<int>((lo >> (8 * e)) & 0xFFu) - 16), xt[(4 * t + e) * stride], sum);
      sum = fmaf(static_cast<float>(static_cast<int>((hi >> (8 * e)) & 0xFFu) - 16), xt[(16 + 4 * t + e) * stride],
                 sum);
    }
  }
  return d * sum;
}

// Q8_0 block . f32 x (internal/simd/c2_tensor_dot_q8_0_nosimd_gen.go:68-91).
__device__ __forceinline__ float unit_q8_0(const uint8_t *blk, const float *xt, int stride) {
  const float d = h2f(ld16(blk));
  float sum = 0.f;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const uint32_t w = ld32u(blk + 2 + 4 * t);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int q = static_cast<int>(static_cast<int8_t>((w >> (8 * e)) & 0xFFu));
      sum = fmaf(static_cast<float>(q), xt[(4 * t + e) * stride], sum);
    }
  }
  return d * sum;
}

// ---------------------------------------------------------------------------
// Row dequantisation (EmbedToken, engine/model.go:221-247; Q6_K per
// tensor/oracle_q6_k_test.go:62-94).  Thread t of the CTA writes elements
// t, t+blockDim, ... of out.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void dequant_row_cta(int type, const uint8_t *row, float *out, int cols) {
  for (int i = threadIdx.x; i < cols; i += kThreads) {
    float v = 0.f;
    if (type == T_Q8_0) {
      const uint8_t *b = row + (i >> 5) * 34;
      v = h2f(ld16(b)) * static_cast<float>(static_cast<int8_t>(b[2 + (i & 31)]));
    } else if (type == T_Q5_0) {
      const uint8_t *b = row + (i >> 5) * 22;
      const int e = i & 31, k = e & 15;
      const uint32_t qh = static_cast<uint32_t>(ld16(b + 2)) | (static_cast<uint32_t>(ld16(b + 4)) << 16);
      const uint8_t byte = b[6 + k];
      const int nib = e < 16 ? (byte & 15) : (byte >> 4);
      const int hb = (qh >> (e < 16 ? k : k + 16)) & 1;
      v = h2f(ld16(b)) * static_cast<float>((nib | (hb << 4)) - 16);
    } else if (type == T_Q4_K) {
      const uint8_t *b = row + (i >> 8) * 144;
      const int e = i & 255, sbi = e >> 6, l = e & 31, hi = (e >> 5) & 1;
      const uint8_t *s = b + 4;
      const int idx = 2 * sbi + hi;
      int sc, m;
      if (idx < 4) {
        sc = s[idx] & 63;
        m = s[idx + 4] & 63;
      } else {
        sc = (s[idx + 4] & 15) | ((s[idx - 4] >> 6) << 4);
        m = (s[idx + 4] >> 4) | ((s[idx] >> 6) << 4);
      }
      const uint8_t q = b[16 + sbi * 32 + l];
      const float dd = __fmul_rn(h2f(ld16(b)), static_cast<float>(sc));
      const float dm = __fmul_rn(h2f(ld16(b + 2)), static_cast<float>(m));
      v = __fsub_rn(__fmul_rn(dd, static_cast<float>(hi ? (q >> 4) : (q & 15))), dm);
    } else if (type == T_Q6_K) {
      const uint8_t *b = row + (i >> 8) * 210;
      const int e = i & 255, n = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
      const uint8_t qlb = b[64 * n + l + ((quarter & 1) ? 32 : 0)];
      const uint8_t qhb = b[128 + 32 * n + l];
      const int q = ((quarter < 2) ? (qlb & 15) : (qlb >> 4)) | (((qhb >> (2 * quarter)) & 3) << 4);
      const int8_t sc = static_cast<int8_t>(b[192 + 8 * n + (l >> 4) + 2 * quarter]);
      v = __fmul_rn(__fmul_rn(h2f(ld16(b + 208)), static_cast<float>(sc)), static_cast<float>(q - 32));
    } else if (type == T_F32) {
      v = reinterpret_cast<const float *>(row)[i];
    }
    out[i] = v;
  }
}

// ---- tagged words of the one-GPU dataflow hand-off (gpu scope) ----------
__device__ __forceinline__ void st_tag(unsigned long long *p, unsigned tag, float v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p),
               "l"((static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v))
               : "memory");
}
// two consecutive words (16-B aligned), each single-copy atomic
__device__ __forceinline__ ulonglong2 ld_tag2(const unsigned long long *p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned tag_of(unsigned long long w) { return static_cast<unsigned>(w >> 32); }
__device__ __forceinline__ float val_of(unsigned long long w) { return __uint_as_float(static_cast<uint32_t>(w)); }
// acquire side of a hand-off that also publishes plain data (fence after
// the poll observed the writer's word; the writer fenced before storing it)
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Polls tagged words into shared memory as floats: up to three segments
// (src[k][0 .. n[k]), n[k] % 4 == 0, 16-B aligned) into dst[k], every
// compute thread taking groups of 4 words, two groups in flight, until each
// word carries `tag`.  Bounded (~2 s): on expiry sets the error flag and
// returns false.  The caller synchronises the CTA before reading dst.
__device__ __noinline__ bool poll_to_smem(const unsigned long long *s0, int n0, float *d0,
                                          const unsigned long long *s1, int n1, float *d1,
                                          const unsigned long long *s2, int n2, float *d2, unsigned tag,
                                          unsigned *err) {
  const int g0n = n0 / 4, g1n = n1 / 4, ng = g0n + g1n + n2 / 4;
  auto at = [&](int g, const unsigned long long *&src, float *&dst) {
    if (g < g0n) {
      src = s0 + 4 * g;
      dst = d0 + 4 * g;
    } else if (g < g0n + g1n) {
      src = s1 + 4 * (g - g0n);
      dst = d1 + 4 * (g - g0n);
    } else {
      src = s2 + 4 * (g - g0n - g1n);
      dst = d2 + 4 * (g - g0n - g1n);
    }
  };
  bool ok = true;
  for (int base = 0; base < ng; base += 2 * kThreads) {
    const int ga = base + threadIdx.x, gb = ga + kThreads;
    const unsigned long long *pa = nullptr, *pb = nullptr;
    float *da = nullptr, *db = nullptr;
    ulonglong2 a0, a1, b0, b1;
    if (ga < ng) {
      at(ga, pa, da);
      a0 = ld_tag2(pa);
      a1 = ld_tag2(pa + 2);
    }
    if (gb < ng) {
      at(gb, pb, db);
      b0 = ld_tag2(pb);
      b1 = ld_tag2(pb + 2);
    }
    long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
      bool all = true;
      if (ga < ng && (tag_of(a0.x) != tag || tag_of(a0.y) != tag || tag_of(a1.x) != tag || tag_of(a1.y) != tag)) {
        all = false;
        a0 = ld_tag2(pa);
        a1 = ld_tag2(pa + 2);
      }
      if (gb < ng && (tag_of(b0.x) != tag || tag_of(b0.y) != tag || tag_of(b1.x) != tag || tag_of(b1.y) != tag)) {
        all = false;
        b0 = ld_tag2(pb);
        b1 = ld_tag2(pb + 2);
      }
      if (all) break;
      if (it == 0) {
        t0 = clock64();
      } else if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
        atomicOr(err, kErrCounter);
        ok = false;
        break;
      }
    }
    if (ga < ng) *reinterpret_cast<float4 *>(da) = make_float4(val_of(a0.x), val_of(a0.y), val_of(a1.x), val_of(a1.y));
    if (gb < ng) *reinterpret_cast<float4 *>(db) = make_float4(val_of(b0.x), val_of(b0.y), val_of(b1.x), val_of(b1.y));
    if (!ok) break;
  }
  return ok;
}

// Polls the 8 tagged words x[8*lane .. 8*lane+7] of one 256-value block
// (16-B aligned) until each carries `tag`; bounded like poll_to_smem.
__device__ __forceinline__ bool poll_block8(const unsigned long long *p, unsigned tag, float (&x)[8], unsigned *err) {
  ulonglong2 w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = ld_tag2(p + 2 * j);
  long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    bool all = true;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (tag_of(w[j].x) != tag || tag_of(w[j].y) != tag) all = false;
    if (all) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) w[j] = ld_tag2(p + 2 * j);
    if (it == 0) {
      t0 = clock64();
    } else if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
      atomicOr(err, kErrCounter);
      return false;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x[2 * j] = val_of(w[j].x);
    x[2 * j + 1] = val_of(w[j].y);
  }
  return true;
}

// one tagged word, polled until it carries `tag` (bounded); its value bits
__device__ __forceinline__ bool poll_tag1(const unsigned long long *p, unsigned tag, uint32_t &bits, unsigned *err) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  const long long t0 = clock64();
  for (uint32_t it = 0; tag_of(w) != tag; ++it) {
    if ((it & 15u) == 15u && clock64() - t0 > kSpinCycles) {
      atomicOr(err, kErrCounter);
      return false;
    }
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  }
  bits = static_cast<uint32_t>(w);
  return true;
}

}  // namespace c2s
