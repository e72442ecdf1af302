// c2s_engine.cu -- host side of the sm_100a token loop and its C ABI.
//
// Replaces engine.LoadModel / Forward / ComputeLogits and c2slm.Engine's
// generate loop (see include/c2slm_b200.h for the per-function mapping).
// Model tensors are uploaded once, in their GGML block layouts, into one HBM
// arena; a decode step is a CUDA graph of 5 kernels per layer plus one logits
// kernel, chained with programmatic dependent launch.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <nccl.h>  // types only: the library is loaded with dlopen when a tensor-parallel engine is created
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <array>
#include <initializer_list>
#include <vector>

#include "../../include/c2slm_b200.h"
#include "c2s_persistent.cuh"
#include "c2s_prefill.cuh"

using namespace c2s;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                                  \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return fail(C2S_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

constexpr int kMaxContext = 16384;  // engine.MaxContextLen (engine/kvcache.go:11)

size_t row_bytes_of(int type, int64_t cols) {
  switch (type) {
    case T_Q5_0: return static_cast<size_t>(cols / 32) * 22;
    case T_Q8_0: return static_cast<size_t>(cols / 32) * 34;
    case T_Q4_K: return static_cast<size_t>(cols / 256) * 144;
    case T_Q6_K: return static_cast<size_t>(cols / 256) * 210;
    case T_F32: return static_cast<size_t>(cols) * 4;
    default: return 0;
  }
}

bool is_kquant(int t) { return t == T_Q4_K || t == T_Q6_K; }
bool is_f32x(int t) { return t == T_Q5_0 || t == T_Q8_0; }

int check_matrix(int type, int64_t rows, int64_t cols, const char *what) {
  if (!(is_kquant(type) || is_f32x(type)))
    return fail(C2S_ERR_UNSUPPORTED, "%s: GGML type %d is not a supported matrix type", what, type);
  if (rows <= 0 || cols <= 0) return fail(C2S_ERR_ARG, "%s: bad shape %lld x %lld", what, (long long)rows, (long long)cols);
  if (rows > (1 << 24)) return fail(C2S_ERR_UNSUPPORTED, "%s: more than 2^24 rows", what);  // 32-bit row split
  if (is_kquant(type) && cols % 256) return fail(C2S_ERR_UNSUPPORTED, "%s: K-quant needs cols %% 256 == 0 (cols=%lld)", what, (long long)cols);
  if (is_f32x(type) && cols % 32) return fail(C2S_ERR_UNSUPPORTED, "%s: cols %% 32 != 0", what);
  if (row_bytes_of(type, cols) > static_cast<size_t>(kStageBytes))
    return fail(C2S_ERR_UNSUPPORTED, "%s: row of %zu bytes exceeds the %d-byte staging slot", what,
                row_bytes_of(type, cols), kStageBytes);
  return C2S_OK;
}

int units_of(int type, int cols) { return is_kquant(type) ? (cols / 256) * 4 : cols / 32; }

// ---------------------------------------------------------------------------
// launch helper (programmatic dependent launch attribute)
// ---------------------------------------------------------------------------
bool g_use_pdl = [] {
  const char *e = getenv("C2S_NO_PDL");
  return !(e && *e && *e != '0');
}();

template <class P>
cudaError_t launch(void (*kernel)(P), dim3 grid, dim3 block, size_t smem, cudaStream_t s, const P &params) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_use_pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, params);
}

// same, for kernels with several arguments
template <class... KArgs, class... Args>
cudaError_t launchv(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_use_pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// shared-memory layout of one k_matvec launch
void layout_matvec(MatParams &P, int grid) {
  auto a16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  int yr = 1;
  for (int s = 0; s < P.nseg; ++s) yr = std::max(yr, (P.seg[s].rows + grid - 1) / grid + 1);
  P.ybuf_rows = yr;
  size_t off = static_cast<size_t>(kStages) * kStageAlloc;
  P.off_bars = static_cast<int>(off);
  off += 64;
  const bool normed = P.kind == K_QKV || P.kind == K_FFN_UP || P.kind == K_NORM ||
                      (P.kind == K_LOGITS && P.x_in == nullptr);
  P.off_nw = static_cast<int>(off);
  if (normed) off += a16(static_cast<size_t>(P.cols) * 4);
  bool bias = false;
  for (int s = 0; s < P.nseg; ++s) bias = bias || P.seg[s].bias != nullptr;
  P.off_bias = static_cast<int>(off);
  if (bias) off += a16(static_cast<size_t>(P.nseg) * yr * 4);
  P.off_xn = static_cast<int>(off);
  off += a16(static_cast<size_t>(P.cols) * 4);
  P.off_xt = static_cast<int>(off);  // limbs of the f32 activation (25 words per 32-value block)
  if (P.need_f32) off += a16(static_cast<size_t>(P.cols / 32) * 25 * 4);
  P.off_q8 = static_cast<int>(off);
  if (P.need_q8k) {
    const int nsb = P.cols / 256;
    off += a16(static_cast<size_t>(q8_qs_bytes(P.cols))) + a16(4 * static_cast<size_t>(nsb)) + 64 * nsb;
  }
  P.off_y = static_cast<int>(off);
  off += static_cast<size_t>(std::max(P.nseg, 1)) * yr * 4;
  P.smem_bytes = static_cast<int>(off);
}

Seg make_seg(const uint8_t *w, int type, int rows, int cols, const float *bias, float *out) {
  Seg s{};
  s.w = w;
  s.type = type;
  s.rows = rows;
  s.row_bytes = static_cast<int>(row_bytes_of(type, cols));
  s.units = units_of(type, cols);
  s.rows_per_chunk = std::max(1, kStageBytes / std::max(1, s.row_bytes));
  s.bias = bias;
  s.out = out;
  return s;
}

void finish_needs(MatParams &P) {
  P.need_f32 = 0;
  P.need_q8k = 0;
  for (int s = 0; s < P.nseg; ++s) {
    if (is_f32x(P.seg[s].type)) P.need_f32 = 1;
    if (is_kquant(P.seg[s].type)) P.need_q8k = 1;
  }
}

// ---------------------------------------------------------------------------
// GGUF (gguf/reader.go:394-546), host side
// ---------------------------------------------------------------------------
struct GTensor {
  std::string name;
  int type = 0;
  int n_dims = 0;
  int64_t dims[4] = {0, 0, 0, 0};
  const uint8_t *data = nullptr;
  uint64_t nbytes = 0;
};

struct GFile {
  uint8_t *map = nullptr;
  size_t size = 0;
  std::vector<GTensor> tensors;
  struct KV {
    std::string key;
    uint32_t vt;
    uint64_t u;
    int64_t i;
    double f;
  };
  std::vector<KV> kvs;
  int32_t im_end = 0, eos = 0;
  ~GFile() {
    if (map) munmap(map, size);
  }
  bool u32(const char *k, uint32_t *out) const {  // GetUint32, gguf/reader.go:559-576
    for (auto &kv : kvs)
      if (kv.key == k) {
        if (kv.vt == 4 || kv.vt == 10) { *out = static_cast<uint32_t>(kv.u); return true; }
        if (kv.vt == 5 || kv.vt == 11) { *out = static_cast<uint32_t>(kv.i); return true; }
        return false;
      }
    return false;
  }
  bool f32(const char *k, float *out) const {  // GetFloat32, gguf/reader.go:579-592
    for (auto &kv : kvs)
      if (kv.key == k) {
        if (kv.vt == 6 || kv.vt == 12) { *out = static_cast<float>(kv.f); return true; }
        return false;
      }
    return false;
  }
};

struct Rd {
  const uint8_t *p;
  size_t n, pos = 0;
  bool bad = false;
  bool need(size_t k) {
    if (pos + k > n) bad = true;
    return !bad;
  }
  uint8_t u8() { return need(1) ? p[pos++] : 0; }
  uint16_t u16() { if (!need(2)) return 0; uint16_t v; memcpy(&v, p + pos, 2); pos += 2; return v; }
  uint32_t u32() { if (!need(4)) return 0; uint32_t v; memcpy(&v, p + pos, 4); pos += 4; return v; }
  uint64_t u64() { if (!need(8)) return 0; uint64_t v; memcpy(&v, p + pos, 8); pos += 8; return v; }
  bool str(std::string *s) {
    const uint64_t l = u64();
    if (bad || !need(l)) return false;
    if (s) s->assign(reinterpret_cast<const char *>(p + pos), l);
    pos += l;
    return true;
  }
};

bool skip_value(Rd &r, uint32_t vt, GFile::KV *kv, int depth) {
  switch (vt) {
    case 0: case 7: { uint8_t v = r.u8(); if (kv) kv->u = v; } break;
    case 1: { int8_t v = static_cast<int8_t>(r.u8()); if (kv) kv->i = v; } break;
    case 2: { uint16_t v = r.u16(); if (kv) kv->u = v; } break;
    case 3: { int16_t v = static_cast<int16_t>(r.u16()); if (kv) kv->i = v; } break;
    case 4: { uint32_t v = r.u32(); if (kv) kv->u = v; } break;
    case 5: { int32_t v = static_cast<int32_t>(r.u32()); if (kv) kv->i = v; } break;
    case 6: { uint32_t b = r.u32(); float f; memcpy(&f, &b, 4); if (kv) kv->f = f; } break;
    case 8: if (!r.str(nullptr)) return false; break;
    case 9: {
      if (depth > 4) return false;
      const uint32_t et = r.u32();
      const uint64_t n = r.u64();
      for (uint64_t i = 0; i < n && !r.bad; ++i)
        if (!skip_value(r, et, nullptr, depth + 1)) return false;
    } break;
    case 10: { uint64_t v = r.u64(); if (kv) kv->u = v; } break;
    case 11: { int64_t v = static_cast<int64_t>(r.u64()); if (kv) kv->i = v; } break;
    case 12: { uint64_t b = r.u64(); double d; memcpy(&d, &b, 8); if (kv) kv->f = d; } break;
    default: return false;
  }
  return !r.bad;
}

uint64_t tensor_nbytes(int type, const int64_t *dims, int nd) {  // gguf/reader.go:513-546
  if (nd == 0) return 0;
  uint64_t n = 1;
  for (int i = 0; i < nd; ++i) n *= static_cast<uint64_t>(dims[i]);
  switch (type) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 2: return (n / 32) * 18;
    case 6: return (n / 32) * 22;
    case 8: return (n / 32) * 34;
    case 12: return (n / 256) * 144;
    case 14: return (n / 256) * 210;
    default: return n * 4;
  }
}

int gguf_open(const char *path, std::unique_ptr<GFile> &out) {
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(C2S_ERR_ARG, "gguf open %s: %s", path, strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return fail(C2S_ERR_FORMAT, "gguf: file too small");
  }
  void *m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_SHARED | MAP_POPULATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return fail(C2S_ERR_FORMAT, "gguf mmap failed");
  auto f = std::make_unique<GFile>();
  f->map = static_cast<uint8_t *>(m);
  f->size = static_cast<size_t>(st.st_size);
  Rd r{f->map, f->size};
  if (r.u32() != 0x46554747u) return fail(C2S_ERR_FORMAT, "invalid GGUF magic");
  const uint32_t ver = r.u32();
  if (ver < 2 || ver > 3) return fail(C2S_ERR_FORMAT, "unsupported GGUF version %u", ver);
  const uint64_t nt = r.u64(), nkv = r.u64();
  if (r.bad || nt > (1u << 20) || nkv > (1u << 20)) return fail(C2S_ERR_FORMAT, "bad GGUF header");
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nkv; ++i) {
    GFile::KV kv{};
    if (!r.str(&kv.key)) return fail(C2S_ERR_FORMAT, "metadata key truncated");
    kv.vt = r.u32();
    if (kv.vt == 9 && kv.key == "tokenizer.ggml.tokens") {
      const uint32_t et = r.u32();
      const uint64_t n = r.u64();
      if (et != 8) return fail(C2S_ERR_FORMAT, "tokenizer.ggml.tokens is not a string array");
      std::string s;
      for (uint64_t t = 0; t < n && !r.bad; ++t) {
        if (!r.str(&s)) break;
        if (s == "<|im_end|>") f->im_end = static_cast<int32_t>(t);        // tokenizer/bpe.go:284-289
        if (s == "<|endoftext|>") f->eos = static_cast<int32_t>(t);
      }
    } else if (!skip_value(r, kv.vt, &kv, 0)) {
      return fail(C2S_ERR_FORMAT, "metadata[%s] unreadable", kv.key.c_str());
    }
    if (kv.key == "general.alignment" && (kv.vt == 4 || kv.vt == 10) && kv.u) alignment = kv.u;
    if (r.bad) return fail(C2S_ERR_FORMAT, "metadata truncated");
    f->kvs.push_back(kv);
  }
  std::vector<uint64_t> offs;
  for (uint64_t i = 0; i < nt; ++i) {
    GTensor t;
    if (!r.str(&t.name)) return fail(C2S_ERR_FORMAT, "tensor name truncated");
    t.n_dims = static_cast<int>(r.u32());
    if (t.n_dims > 4) return fail(C2S_ERR_FORMAT, "tensor %s has %d dims", t.name.c_str(), t.n_dims);
    for (int d = 0; d < t.n_dims; ++d) t.dims[d] = static_cast<int64_t>(r.u64());
    t.type = static_cast<int>(r.u32());
    offs.push_back(r.u64());
    if (r.bad) return fail(C2S_ERR_FORMAT, "tensor infos truncated");
    f->tensors.push_back(t);
  }
  size_t pos = r.pos;
  if (pos % alignment) pos += alignment - pos % alignment;
  for (size_t i = 0; i < f->tensors.size(); ++i) {
    GTensor &t = f->tensors[i];
    t.nbytes = tensor_nbytes(t.type, t.dims, t.n_dims);
    if (pos + offs[i] + t.nbytes > f->size) return fail(C2S_ERR_FORMAT, "tensor[%s] data out of range", t.name.c_str());
    t.data = f->map + pos + offs[i];
  }
  out = std::move(f);
  return C2S_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Engine
// ---------------------------------------------------------------------------
struct LayerDev {
  const uint8_t *q, *k, *v, *o, *gate, *up, *down;
  int tq, tk, tv, to, tgate, tup, tdown;
  const float *attn_norm, *ffn_norm, *qb, *kb, *vb, *qn, *kn;
};

struct HostFwdIn {
  int token, pos, commit;
};

// Tensor-parallel shard of one rank (one GPU): query heads [h0, h1) in units
// of whole 256-column superblocks of attn_output's input (pairs of heads at
// head_dim 128), the kv heads [g0, g1) they use, FFN rows [f0, f1) in
// superblocks of 256, vocabulary rows [v0, v1) of an even split padded to
// vpad rows per rank.  One GPU: the whole model.
struct TpPlan {
  int rank = 0, world = 1;
  int h0 = 0, h1 = 0, g0 = 0, g1 = 0, f0 = 0, f1 = 0, v0 = 0, v1 = 0, vpad = 0;
};

int tp_plan(const c2s_model_desc &d, int rank, int world, TpPlan &p, std::string &why) {
  p = TpPlan{};
  p.rank = rank;
  p.world = world;
  const int hd = d.head_dim > 0 ? d.head_dim : d.embd / d.n_heads;
  const int qpk = d.n_heads / d.n_kv_heads;
  if (world <= 1) {
    p.h1 = d.n_heads;
    p.g1 = d.n_kv_heads;
    p.f1 = d.ffn / 256;
    p.v1 = p.vpad = d.vocab;
    return 0;
  }
  if (hd <= 0 || 256 % hd != 0 || d.n_heads % (256 / hd) != 0) {
    why = "tensor parallel: heads must group into 256-column superblocks";
    return -1;
  }
  if (d.ffn % 256) {
    why = "tensor parallel: ffn must be a multiple of 256";
    return -1;
  }
  auto split = [](int n, int parts, int r, int &a, int &b) {  // first n % parts parts get one more
    const int q = n / parts, m = n % parts;
    a = r * q + std::min(r, m);
    b = a + q + (r < m ? 1 : 0);
  };
  const int upb = 256 / hd, units = d.n_heads / upb;
  if (units < world || d.ffn / 256 < world) {
    why = "tensor parallel: fewer head groups or FFN superblocks than ranks";
    return -1;
  }
  int u0, u1;
  split(units, world, rank, u0, u1);
  p.h0 = u0 * upb;
  p.h1 = u1 * upb;
  p.g0 = p.h0 / qpk;
  p.g1 = (p.h1 + qpk - 1) / qpk;
  split(d.ffn / 256, world, rank, p.f0, p.f1);
  p.vpad = (d.vocab + world - 1) / world;
  p.v0 = std::min(d.vocab, rank * p.vpad);
  p.v1 = std::min(d.vocab, p.v0 + p.vpad);
  return 0;
}

// NCCL entry points, resolved from libnccl.so.2 at first use
struct NcclApi {
  decltype(&ncclGetUniqueId) get_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) err_str = nullptr;
};

struct c2s_engine {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  c2s_model_desc d{};
  int tok_type = 0, out_type = 0;
  const uint8_t *tok_embd = nullptr, *output = nullptr;
  const float *out_norm = nullptr;
  std::vector<LayerDev> layers;
  // device memory
  uint8_t *weights = nullptr;
  size_t weights_bytes = 0;
  float *kv = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  float *X = nullptr, *normx = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn_out = nullptr,
        *h = nullptr, *logits = nullptr, *part = nullptr, *scratch_x = nullptr;
  float2 *amax_part = nullptr;
  int *token_ids = nullptr, *out_tokens = nullptr, *rows_idx = nullptr;
  DevState *st = nullptr;
  // pinned host mirrors
  HostFwdIn *h_in = nullptr;  // ring of forward inputs
  int h_in_next = 0;
  float *h_buf = nullptr;     // staging for normx/logits
  // multi-token prefill on the tensor cores (c2s_prefill.cuh): buffers for a
  // chunk of up to pf_cap tokens, allocated on first use
  int pf_ok = 0, pf_cap = 0, pf_kmax = 0;
  float *pf_x = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_att = nullptr, *pf_g = nullptr,
        *pf_u = nullptr, *pf_d8 = nullptr;
  uint8_t *pf_q8 = nullptr;   // tokens' Q8_K bytes in the GEMM's A-tile layout
  int *pf_tok = nullptr;
  int16_t *pf_bs = nullptr;   // tokens' Q8_K sub-block sums
  uint8_t *pf_planes = nullptr;  // every layer projection's digit planes and row tables
  float *pf_fpart = nullptr;     // attention split partials (PfFlash::part)
  float *pf_delta = nullptr;     // tensor parallel: the chunk's partial o-proj / down rows, allreduced
  unsigned *pf_fcount = nullptr; // attention split arrivals (PfFlash::count)
  int pf_fsplit = 0, pf_fns = 0; // keys per attention split, most splits of a block
  uint8_t *pf_kvt = nullptr;     // one layer's K/V tiles of the tensor-core attention (k_pf_kv_tiles)
  int pf_kvt_tpg = 0;            // tiles per kv group
  int pf_attn_fp32 = 0;          // test switch (C2S_PF_ATTN=fp32): the FP32 attention kernel instead
  std::vector<std::array<const uint8_t *, 7>> pf_pl;  // per layer: q, k, v, o, gate, up, down
  std::vector<std::array<const uint4 *, 7>> pf_ri;
  DevState *h_st = nullptr;
  int *h_tokens = nullptr;
  int host_seq = 0;
  int max_splits = 1, split_len = 256;
  size_t attn_smem = 0;
  int kernels_per_step = 0;
  cudaGraphExec_t g_forward = nullptr, g_step = nullptr, g_logits = nullptr, g_fwd_select = nullptr;
  std::vector<MatParams> mp_cache;
  uint64_t algorithmic_bytes = 0;
  // persistent decode kernel
  PPhase *d_phases = nullptr;
  int nphase = 0;
  unsigned *gbar = nullptr;
  unsigned long long *df_words = nullptr;  // tagged hand-off buffers of the one-GPU persistent kernel
  size_t df_nwords = 0;
  unsigned df_tag = 0;                     // tag base of the next launch (advanced past every tag used)
  PParams pp{};
  size_t p_smem = 0;
  bool use_persistent = true;
  // tensor parallel (world > 1)
  TpPlan plan;
  ncclComm_t comm = nullptr;
  float *delta = nullptr;        // this rank's partial o-proj / down output, allreduced in place
  float *logits_full = nullptr;  // gathered logits [world * vpad]
  // persistent decode across the group: tagged words recv [2][world][H] | argbuf [2][world][G][2],
  // mapped into every rank (peer_shared[r] = rank r's region, this rank's own included)
  uint8_t *tp_shared = nullptr;
  uint8_t *peer_shared[8] = {};
  float *xbuf = nullptr;         // [2][H] residual stream
  bool tp_persist_ok = false;    // the persistent kernel fits; enabled once the peers are mapped
};

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// libnccl.so.2 is opened on the first tensor-parallel call only; a process
// that already loaded it (e.g. through torch.distributed) shares that copy.
int nccl_api(const NcclApi **out) {
  static NcclApi api;
  static std::string why;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      why = dlerror() ? dlerror() : "dlopen(libnccl.so.2) failed";
      return;
    }
    api.get_id = reinterpret_cast<decltype(api.get_id)>(dlsym(h, "ncclGetUniqueId"));
    api.init_rank = reinterpret_cast<decltype(api.init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.destroy = reinterpret_cast<decltype(api.destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.err_str = reinterpret_cast<decltype(api.err_str)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_id || !api.init_rank || !api.destroy || !api.all_reduce || !api.all_gather || !api.err_str) {
      why = "libnccl.so.2 lacks an expected symbol";
      api = NcclApi{};
    }
  });
  if (!api.get_id) return fail(C2S_ERR_UNSUPPORTED, "NCCL unavailable: %s", why.c_str());
  *out = &api;
  return C2S_OK;
}

const c2s_tensor_desc *find_t(const c2s_tensor_desc *ts, int n, const std::string &name) {
  for (int i = 0; i < n; ++i)
    if (ts[i].name && name == ts[i].name) return &ts[i];
  return nullptr;
}

int64_t t_cols(const c2s_tensor_desc *t) { return t->n_dims > 0 ? t->dims[0] : 0; }
int64_t t_rows(const c2s_tensor_desc *t) { return t->n_dims > 1 ? t->dims[1] : 1; }

int matvec_params_common(c2s_engine *e, MatParams &P) {
  P.eps = e->d.eps;
  P.X = e->X;
  P.st = e->st;
  P.token_ids = e->token_ids;
  P.out_tokens = e->out_tokens;
  P.part = e->amax_part;
  finish_needs(P);
  layout_matvec(P, e->num_sms);
  return C2S_OK;
}

// Builds the kernel sequence of one forward (L layers) on `s`.
// Optional per-kernel timing (eager launches only): events[k] brackets
// kernel k of the sequence; kind_of[k] receives its stage id.
struct KTimer {
  std::vector<cudaEvent_t> *ev = nullptr;
  std::vector<int> *kind = nullptr;
};

cudaError_t mark(KTimer *t, cudaStream_t s, int kind) {
  if (!t || !t->ev) return cudaSuccess;
  cudaEvent_t ev;
  cudaError_t err = cudaEventCreate(&ev);
  if (err) return err;
  t->ev->push_back(ev);
  if (kind >= 0) t->kind->push_back(kind);
  return cudaEventRecord(ev, s);
}

// allreduce (sum) of this rank's partial in e->delta, then X += delta on every
// rank (and the commit of the forwarded token after the last layer)
cudaError_t enqueue_tp_reduce(c2s_engine *e, cudaStream_t s, bool commit_here, bool check_halt) {
  const NcclApi *nc = nullptr;
  if (nccl_api(&nc)) return cudaErrorUnknown;
  const ncclResult_t r = nc->all_reduce(e->delta, e->delta, e->d.embd, ncclFloat32, ncclSum, e->comm, s);
  if (r != ncclSuccess) {
    fail(C2S_ERR_CUDA, "ncclAllReduce: %s", nc->err_str(r));
    return cudaErrorUnknown;
  }
  const int blocks = (e->d.embd + kThreads - 1) / kThreads;
  return launchv(k_residual_add, dim3(blocks), dim3(kThreads), 0, s, e->X, static_cast<const float *>(e->delta),
                e->d.embd, e->st, e->token_ids, commit_here ? 1 : 0, check_halt ? 1 : 0);
}

cudaError_t enqueue_forward(c2s_engine *e, cudaStream_t s, bool check_halt, bool final_norm, KTimer *tm = nullptr) {
  const int L = e->d.n_layers, H = e->d.embd, hd = e->d.head_dim;
  const TpPlan &pl = e->plan;
  const bool tp = pl.world > 1;
  // this rank's rows: query heads, kv heads, FFN (the whole model on one GPU)
  const int nq = (pl.h1 - pl.h0) * hd, kvd = (pl.g1 - pl.g0) * hd;
  const int F = tp ? (pl.f1 - pl.f0) * 256 : e->d.ffn;
  const int G = e->num_sms;
  cudaError_t err = cudaSuccess;
  for (int l = 0; l < L && err == cudaSuccess; ++l) {
    const LayerDev &Ld = e->layers[l];
    // QKV (+ embedding on layer 0)
    MatParams P{};
    P.kind = K_QKV;
    P.nseg = 3;
    P.cols = H;
    P.seg[0] = make_seg(Ld.q, Ld.tq, nq, H, Ld.qb, e->q);
    P.seg[1] = make_seg(Ld.k, Ld.tk, kvd, H, Ld.kb, e->k);
    P.seg[2] = make_seg(Ld.v, Ld.tv, kvd, H, Ld.vb, e->v);
    P.norm_w = Ld.attn_norm;
    P.do_embed = (l == 0);
    P.embd_w = e->tok_embd;
    P.embd_type = e->tok_type;
    P.embd_row_bytes = static_cast<int>(row_bytes_of(e->tok_type, H));
    P.check_halt = check_halt;
    matvec_params_common(e, P);
    if ((err = mark(tm, s, -1))) break;
    err = launch(k_matvec, dim3(G), dim3(kThreads), P.smem_bytes, s, P);
    if (err || (err = mark(tm, s, K_QKV))) break;
    // attention
    AttnParams A{};
    A.layer = l;
    A.n_heads = e->d.n_heads;
    A.n_kv = pl.g1 - pl.g0;
    A.qpk = e->d.n_heads / e->d.n_kv_heads;
    A.tp_h0 = pl.h0;
    A.tp_h1 = pl.h1;
    A.tp_g0 = pl.g0;
    A.hd = hd;
    A.max_tokens = e->d.max_tokens;
    A.max_splits = e->max_splits;
    A.rope_len = kMaxContext;
    A.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));  // engine/forward.go:59
    A.eps = e->d.eps;
    A.q = e->q;
    A.k = e->k;
    A.v = e->v;
    const size_t plane = static_cast<size_t>(L) * (pl.g1 - pl.g0) * e->d.max_tokens * hd;
    A.kcache = e->kv;
    A.vcache = e->kv + plane;
    A.rope_cos = e->rope_cos;
    A.rope_sin = e->rope_sin;
    A.q_norm = Ld.qn;
    A.k_norm = Ld.kn;
    A.part = e->part;
    A.out = e->attn_out;
    A.st = e->st;
    A.check_halt = check_halt;
    A.split_len = e->split_len;
    A.items_cap = e->num_sms;  // the persistent kernel's grid
    if ((err = mark(tm, s, -1))) break;
    err = launch(k_attention, dim3(std::max(pl.g1 - pl.g0, pl.h1 - pl.h0), e->max_splits), dim3(kThreads),
                 e->attn_smem, s, A);
    if (err || (err = mark(tm, s, 7))) break;
    // o_proj + residual (tensor parallel: this rank's heads' columns, then an allreduce)
    P = MatParams{};
    P.kind = tp ? K_RAW : K_OPROJ;
    P.nseg = 1;
    P.cols = nq;
    P.seg[0] = make_seg(Ld.o, Ld.to, H, nq, nullptr, tp ? e->delta : e->X);
    P.x_in = e->attn_out;
    P.check_halt = check_halt;
    matvec_params_common(e, P);
    if ((err = mark(tm, s, -1))) break;
    err = launch(k_matvec, dim3(G), dim3(kThreads), P.smem_bytes, s, P);
    if (!err && tp) err = enqueue_tp_reduce(e, s, false, check_halt);
    if (err || (err = mark(tm, s, K_OPROJ))) break;
    // gate/up + SwiGLU
    P = MatParams{};
    P.kind = K_FFN_UP;
    P.nseg = 2;
    P.cols = H;
    P.seg[0] = make_seg(Ld.gate, Ld.tgate, F, H, nullptr, nullptr);
    P.seg[1] = make_seg(Ld.up, Ld.tup, F, H, nullptr, nullptr);
    P.norm_w = Ld.ffn_norm;
    P.h_out = e->h;
    P.check_halt = check_halt;
    matvec_params_common(e, P);
    if ((err = mark(tm, s, -1))) break;
    err = launch(k_matvec, dim3(G), dim3(kThreads), P.smem_bytes, s, P);
    if (err || (err = mark(tm, s, K_FFN_UP))) break;
    // down + residual (+ commit on the last layer); tensor parallel: this
    // rank's FFN columns, then an allreduce
    P = MatParams{};
    P.kind = tp ? K_RAW : K_FFN_DOWN;
    P.nseg = 1;
    P.cols = F;
    P.seg[0] = make_seg(Ld.down, Ld.tdown, H, F, nullptr, tp ? e->delta : e->X);
    P.x_in = e->h;
    P.commit_here = (l == L - 1);
    P.check_halt = check_halt;
    matvec_params_common(e, P);
    if ((err = mark(tm, s, -1))) break;
    err = launch(k_matvec, dim3(G), dim3(kThreads), P.smem_bytes, s, P);
    if (!err && tp) err = enqueue_tp_reduce(e, s, l == L - 1, check_halt);
    if (err || (err = mark(tm, s, K_FFN_DOWN))) break;
  }
  if (err == cudaSuccess && final_norm) {
    MatParams P{};
    P.kind = K_NORM;
    P.nseg = 0;
    P.cols = H;
    P.norm_w = e->out_norm;
    P.normx_out = e->normx;
    P.check_halt = check_halt;
    matvec_params_common(e, P);
    err = launch(k_matvec, dim3(1), dim3(kThreads), P.smem_bytes, s, P);
  }
  return err;
}

cudaError_t enqueue_logits(c2s_engine *e, cudaStream_t s, bool select, bool from_normx, bool check_halt,
                           KTimer *tm = nullptr) {
  const TpPlan &pl = e->plan;
  const bool tp = pl.world > 1;
  MatParams P{};
  P.kind = K_LOGITS;
  P.nseg = 1;
  P.cols = e->d.embd;
  P.seg[0] = make_seg(e->output, e->out_type, pl.v1 - pl.v0, e->d.embd, nullptr, e->logits);
  P.norm_w = e->out_norm;
  P.x_in = from_normx ? e->normx : nullptr;
  P.normx_out = from_normx ? nullptr : e->normx;
  P.select = select && !tp;
  P.check_halt = check_halt;
  matvec_params_common(e, P);
  cudaError_t err = mark(tm, s, -1);
  if (!err) err = launch(k_matvec, dim3(e->num_sms), dim3(kThreads), P.smem_bytes, s, P);
  if (!err && tp) {
    // every rank gathers the whole vocabulary (rows of rank r at r * vpad),
    // then selects from it with the same rules: identical ids on all ranks
    const NcclApi *nc = nullptr;
    if (nccl_api(&nc)) return cudaErrorUnknown;
    const ncclResult_t r = nc->all_gather(e->logits, e->logits_full, pl.vpad, ncclFloat32, e->comm, s);
    if (r != ncclSuccess) {
      fail(C2S_ERR_CUDA, "ncclAllGather: %s", nc->err_str(r));
      return cudaErrorUnknown;
    }
    if (select) {
      const size_t smem = (static_cast<size_t>(e->d.vocab) / e->num_sms + 2) * 4;
      err = launchv(k_select, dim3(e->num_sms), dim3(kThreads), smem, s, static_cast<const float *>(e->logits_full),
                   e->d.vocab, e->st, static_cast<const int *>(e->token_ids), e->out_tokens, e->amax_part,
                   check_halt ? 1 : 0);
    }
  }
  if (!err) err = mark(tm, s, K_LOGITS);
  return err;
}

int capture(c2s_engine *e, cudaGraphExec_t *out, int which) {
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t err = cudaSuccess;
  switch (which) {
    case 0: err = enqueue_forward(e, e->stream, false, true); break;          // Forward + NormX
    case 1:                                                                    // decode step
      err = enqueue_logits(e, e->stream, true, false, true);
      if (!err) err = enqueue_forward(e, e->stream, true, false);
      break;
    case 2: err = enqueue_logits(e, e->stream, false, true, false); break;   // ComputeLogits(NormX)
    case 3:                                                                    // forward then select
      err = enqueue_forward(e, e->stream, false, false);
      if (!err) err = enqueue_logits(e, e->stream, true, false, false);
      break;
  }
  cudaError_t e2 = cudaStreamEndCapture(e->stream, &g);
  if (err != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return fail(C2S_ERR_CUDA, "kernel launch during capture: %s", cudaGetErrorString(err));
  }
  if (e2 != cudaSuccess) return fail(C2S_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(e2));
  cudaError_t e3 = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e3 != cudaSuccess) return fail(C2S_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e3));
  return C2S_OK;
}

int read_status(c2s_engine *e) {
  // Reads back the device state (sync point); reports bounded-wait failures.
  CK(cudaMemcpyAsync(e->h_st, e->st, sizeof(DevState), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  if (e->h_st->err) {
    const unsigned code = e->h_st->err;
    CK(cudaMemsetAsync(&e->st->err, 0, sizeof(unsigned), e->stream));
    CK(cudaStreamSynchronize(e->stream));
    return fail(C2S_ERR_TIMEOUT, "device reported error flags 0x%x (bounded wait expired or bad position)", code);
  }
  e->host_seq = e->h_st->seq_len;
  return C2S_OK;
}

int set_fwd_input(c2s_engine *e, int token, int pos, int commit) {
  HostFwdIn *slot = &e->h_in[e->h_in_next];
  e->h_in_next = (e->h_in_next + 1) % (e->d.max_tokens + 8);
  slot->token = token;
  slot->pos = pos;
  slot->commit = commit;
  CK(cudaMemcpyAsync(e->st, slot, sizeof(HostFwdIn), cudaMemcpyHostToDevice, e->stream));
  return C2S_OK;
}

// ---------------------------------------------------------------------------
// persistent decode kernel: phase table, shared-memory layout, launch
// ---------------------------------------------------------------------------

// Warp groups of the many-row matvec phases (2^lng of them): group g
// consumes ring chunks g, g + ng, ... and chunk k sits in slot k % nslot.  A
// slot must belong to one group only -- two groups waiting on one slot's
// full barrier at different uses would see the older phase's parity as
// complete, read a chunk that has not arrived and over-release the slot --
// so ng must divide nslot (then chunks k and k + nslot have the same group).
int ring_groups_log2(int nslot, int lng) {
  lng = std::max(0, std::min(3, lng));
  while (lng > 0 && (nslot < (1 << lng) || nslot % (1 << lng) != 0)) --lng;
  return lng;
}

int persistent_setup(c2s_engine *e) {
  const c2s_model_desc &d = e->d;
  const TpPlan &pl = e->plan;
  const bool tp = pl.world > 1;
  // this rank's rows (the model's on one GPU)
  const int L = d.n_layers, H = d.embd, hd = d.head_dim;
  const int F = tp ? (pl.f1 - pl.f0) * 256 : d.ffn, kvd = (pl.g1 - pl.g0) * hd, nq = (pl.h1 - pl.h0) * hd;
  const int V = pl.v1 - pl.v0;
  const int G = e->num_sms;
  if (tp && pl.world > kMaxRanks) return fail(C2S_ERR_UNSUPPORTED, "persistent decode: more than %d ranks", kMaxRanks);
  std::vector<PPhase> ph;
  auto mk = [&](int kind, int layer) {
    PPhase p{};
    p.kind = kind;
    p.layer = layer;
    return p;
  };
  auto needs = [](PPhase &p) {
    p.need_f32 = 0;
    p.need_q8k = 0;
    for (int s = 0; s < p.nseg; ++s) {
      if (is_f32x(p.seg[s].type)) p.need_f32 = 1;
      if (is_kquant(p.seg[s].type)) p.need_q8k = 1;
    }
  };
  {
    PPhase p = mk(K_LOGITS, -1);
    p.nseg = 1;
    p.cols = H;
    p.seg[0] = make_seg(e->output, e->out_type, V, H, nullptr, e->logits);
    p.norm_w = e->out_norm;
    needs(p);
    ph.push_back(p);
  }
  for (int l = 0; l < L; ++l) {
    const LayerDev &Ld = e->layers[l];
    PPhase q = mk(K_QKV, l);
    q.nseg = 3;
    q.cols = H;
    q.seg[0] = make_seg(Ld.q, Ld.tq, nq, H, Ld.qb, e->q);
    q.seg[1] = make_seg(Ld.k, Ld.tk, kvd, H, Ld.kb, e->k);
    q.seg[2] = make_seg(Ld.v, Ld.tv, kvd, H, Ld.vb, e->v);
    q.norm_w = Ld.attn_norm;
    q.do_embed = (l == 0);
    needs(q);
    ph.push_back(q);
    PPhase a = mk(K_ATTN, l);
    a.q_norm = Ld.qn;
    a.k_norm = Ld.kn;
    ph.push_back(a);
    PPhase o = mk(K_OPROJ, l);
    o.nseg = 1;
    o.cols = H;
    o.cols = nq;
    o.seg[0] = make_seg(Ld.o, Ld.to, H, nq, nullptr, e->X);
    o.x_in = e->attn_out;
    needs(o);
    ph.push_back(o);
    PPhase u = mk(K_FFN_UP, l);
    u.nseg = 2;
    u.cols = H;
    u.seg[0] = make_seg(Ld.gate, Ld.tgate, F, H, nullptr, nullptr);
    u.seg[1] = make_seg(Ld.up, Ld.tup, F, H, nullptr, nullptr);
    u.norm_w = Ld.ffn_norm;
    needs(u);
    ph.push_back(u);
    PPhase w = mk(K_FFN_DOWN, l);
    w.nseg = 1;
    w.cols = F;
    w.seg[0] = make_seg(Ld.down, Ld.tdown, H, F, nullptr, e->X);
    w.x_in = e->h;
    w.commit_here = (l == L - 1);
    needs(w);
    ph.push_back(w);
  }
  // shared memory: weight ring | mbarriers | activation region (union of the
  // matvec and attention working sets)
  auto a16 = [](size_t v) { return (v + 15) & ~size_t(15); };
  int limb_cap = 0, q8_cap = 0, yrows = 1;
  for (auto &p : ph) {
    if (p.kind == K_ATTN) continue;
    for (int s = 0; s < p.nseg; ++s) {
      const int per = (p.seg[s].rows + G - 1) / G + 1;
      yrows = std::max(yrows, per);
      if (p.kind != K_LOGITS && per > kThreads)
        return fail(C2S_ERR_UNSUPPORTED, "persistent decode: more than %d rows per CTA", kThreads);
    }
    if (p.need_f32) limb_cap = std::max(limb_cap, p.cols);
    if (p.need_q8k) q8_cap = std::max(q8_cap, p.cols);
  }
  PParams &P = e->pp;
  P.off_xn = 0;  // f32 input vector (embedding row, normalised x for Q8_K)
  P.off_limbs = static_cast<int>(a16(static_cast<size_t>(H) * 4));
  P.off_q8 = P.off_limbs + static_cast<int>(a16(static_cast<size_t>(limb_cap / 32) * 25 * 4));
  const size_t q8b = q8_cap ? a16(static_cast<size_t>(q8_qs_bytes(q8_cap))) + a16(4 * static_cast<size_t>(q8_cap / 256)) +
                                  64 * static_cast<size_t>(q8_cap / 256)
                            : 0;
  P.off_y = P.off_q8 + static_cast<int>(a16(q8b));
  P.yrows = yrows;
  const size_t mv_act = static_cast<size_t>(P.off_y) + static_cast<size_t>(kMaxSegs) * yrows * 4;
  const int qpk = d.n_heads / d.n_kv_heads;
  const size_t at_act = attn_smem_bytes(hd, qpk);
  const size_t act = a16(std::max(mv_act, at_act));
  const size_t budget = 227 * 1024 - 8192;  // dynamic smem; static smem of the kernel is < 8 KB
  // weight ring: a few large slots (each warp consumes many rows per slot).
  // Measured per step: three 48 KB slots with one warp group at the 0.5B
  // width (F 4864); three 40 KB slots at the 1.5B width (F 8960: 1476 vs
  // 1517 us); 32 KB slots with two groups where phases have hundreds of rows
  // per CTA (the 7B width, F > 12288: 2.86 vs 2.96 ms)
  const bool wide = F > 12288;
  int slot_kb = wide ? 32 : F > 6144 ? 40 : 48;
  if (const char *sk = getenv("C2S_SLOT_KB")) slot_kb = std::max(8, std::min(96, atoi(sk)));
  size_t max_row = 0;
  for (auto &p : ph)
    for (int s = 0; s < p.nseg; ++s) max_row = std::max(max_row, static_cast<size_t>(p.seg[s].row_bytes));
  if (budget < act + 1024) return fail(C2S_ERR_UNSUPPORTED, "persistent decode: activation set too large for shared memory");
  const size_t ring = budget - act - 1024;
  size_t slot_bytes = static_cast<size_t>(slot_kb) * 1024;
  while (slot_bytes > 16384 && ring / (slot_bytes + 64) < 3) slot_bytes -= 8192;
  if (slot_bytes < max_row) slot_bytes = (max_row + 1023) & ~size_t(1023);
  int nslot = static_cast<int>(ring / (slot_bytes + 64));
  nslot = std::min(nslot, 8);
  if (nslot < 2) return fail(C2S_ERR_UNSUPPORTED, "persistent decode: activation set too large for shared memory");
  P.nslot = nslot;
  // warp groups of the many-row phases: each group holds one slot while it
  // computes, so fewer groups than slots leave slots to fill meanwhile
  int lng = wide ? 1 : nslot >= 8 ? 3 : nslot >= 4 ? 2 : nslot >= 2 ? 1 : 0;
  if (const char *lg = getenv("C2S_LNG")) lng = atoi(lg);
  P.lng = ring_groups_log2(nslot, lng);
  P.slot_bytes = static_cast<int>(slot_bytes);
  P.slot_alloc = static_cast<int>(slot_bytes + 64);
  size_t off = static_cast<size_t>(nslot) * P.slot_alloc;
  P.off_full = static_cast<int>(off);
  off += 8 * nslot;
  P.off_empty = static_cast<int>(off);
  off += 8 * nslot;
  P.off_abar = static_cast<int>(off);
  off += 8 * kAttnBufs;
  off = (off + 127) & ~size_t(127);
  P.off_act = static_cast<int>(off);
  e->p_smem = off + act;
  // parameters: the layer table travels in the kernel's parameter space
  if (L > kMaxLayers) return fail(C2S_ERR_UNSUPPORTED, "persistent decode: more than %d layers", kMaxLayers);
  if (H > 16 * kThreads) return fail(C2S_ERR_UNSUPPORTED, "persistent decode: embd above %d", 16 * kThreads);
  static_assert(sizeof(PParams) < 32000, "kernel parameter space");
  for (int l = 0; l < L; ++l) {
    const LayerDev &Ld = e->layers[l];
    PLayer &y = P.layers[l];
    y.q = Ld.q; y.k = Ld.k; y.v = Ld.v; y.o = Ld.o; y.gate = Ld.gate; y.up = Ld.up; y.down = Ld.down;
    y.attn_norm = Ld.attn_norm; y.ffn_norm = Ld.ffn_norm;
    y.qb = Ld.qb; y.kb = Ld.kb; y.vb = Ld.vb; y.qn = Ld.qn; y.kn = Ld.kn;
    y.tq = static_cast<int8_t>(Ld.tq); y.tk = static_cast<int8_t>(Ld.tk); y.tv = static_cast<int8_t>(Ld.tv);
    y.to = static_cast<int8_t>(Ld.to); y.tg = static_cast<int8_t>(Ld.tgate); y.tu = static_cast<int8_t>(Ld.tup);
    y.td = static_cast<int8_t>(Ld.tdown);
  }
  P.out_w = e->output;
  P.out_norm = e->out_norm;
  P.out_type = e->out_type;
  P.n_layers = L;
  P.F = F;
  P.kvd = kvd;
  P.vocab = d.vocab;
  P.qrows = nq;
  P.vrows = V;
  P.world = pl.world;
  P.rank = pl.rank;
  P.qpk = d.n_heads / d.n_kv_heads;
  P.tp_h0 = pl.h0;
  P.tp_h1 = pl.h1;
  P.tp_g0 = pl.g0;
  P.tp_v0 = pl.v0;  // the exchange buffers of a tensor-parallel group are set by tp_exchange_setup
  e->nphase = static_cast<int>(ph.size());
  CK(cudaMalloc(&e->gbar, 4 * static_cast<size_t>(G) + 64));
  CK(cudaMemset(e->gbar, 0, 4 * static_cast<size_t>(G) + 64));
  P.nphase = e->nphase;
  P.H = H;
  P.n_heads = d.n_heads;
  P.n_kv = pl.g1 - pl.g0;
  P.hd = hd;
  P.max_tokens = d.max_tokens;
  P.max_splits = e->max_splits;
  P.split_len = e->split_len;
  P.rope_len = kMaxContext;
  P.eps = d.eps;
  P.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));  // engine/forward.go:59
  P.X = e->X;
  P.normx = e->normx;
  P.q = e->q;
  P.k = e->k;
  P.v = e->v;
  P.attn_out = e->attn_out;
  P.h = e->h;
  P.logits = e->logits;
  P.part = e->part;
  P.amax_part = e->amax_part;
  const size_t plane = static_cast<size_t>(L) * (pl.g1 - pl.g0) * d.max_tokens * hd;
  P.kcache = e->kv;
  P.vcache = e->kv + plane;
  P.rope_cos = e->rope_cos;
  P.rope_sin = e->rope_sin;
  P.embd_w = e->tok_embd;
  P.embd_type = e->tok_type;
  P.embd_row_bytes = static_cast<int>(row_bytes_of(e->tok_type, H));
  P.st = e->st;
  P.token_ids = e->token_ids;
  P.out_tokens = e->out_tokens;
  P.gbar = e->gbar;
  P.ll = tp ? 1 : 0;  // tensor parallel: the cross-GPU exchange of o-proj / down partial rows
  // one GPU: phases hand off through tagged words, without grid barriers,
  // where the phases are latency-bound (measured: 0.5B 6 %, 1.5B 2.5 % faster
  // per step); at the 7B width every CTA's tagged copy of the 18,944-value
  // SwiGLU output costs more than the barrier it replaces (1.7 % slower)
  P.df = (!tp && F <= 12288) ? 1 : 0;
  if (P.df) {
    const size_t nw[7] = {static_cast<size_t>(H), static_cast<size_t>(nq), static_cast<size_t>(kvd),
                          static_cast<size_t>(kvd), static_cast<size_t>(nq), static_cast<size_t>(F), 2};
    size_t tot = 0;
    for (size_t w : nw) tot += (w + 3) & ~size_t(3);  // 32-byte aligned regions
    CK(cudaMalloc(&e->df_words, tot * 8));
    CK(cudaMemsetAsync(e->df_words, 0, tot * 8, e->stream));  // ordered before every launch on the stream
    e->df_nwords = tot;
    e->df_tag = 0;
    unsigned long long *w = e->df_words;
    unsigned long long **dst[7] = {&P.tX, &P.tq, &P.tk, &P.tv, &P.tatt, &P.th, &P.tsel};
    for (int i = 0; i < 7; ++i) {
      *dst[i] = w;
      w += (nw[i] + 3) & ~size_t(3);
    }
  }
  const void *kfn = P.df ? reinterpret_cast<const void *>(k_persistent<true>)
                         : reinterpret_cast<const void *>(k_persistent<false>);
  CK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(e->p_smem)));
  int blocks = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kfn, kPThreads, e->p_smem));
  const char *mode = getenv("C2S_DECODE");
  e->use_persistent = blocks >= 1 && !(mode && strcmp(mode, "graph") == 0);
  return C2S_OK;
}

// n_steps decode steps (logits+select+forward) in one cooperative launch
int launch_persistent(c2s_engine *e, int n_steps, int rewind_period, int rewind_base,
                      unsigned long long *trace = nullptr, int phase0 = 0) {
  PParams P = e->pp;
  P.trace = trace;
  P.phase0 = phase0;
  P.n_steps = n_steps;
  P.rewind_period = rewind_period;
  P.rewind_base = rewind_base;
  if (!P.df) CK(cudaMemsetAsync(e->gbar, 0, 4 * static_cast<size_t>(e->num_sms), e->stream));  // grid barriers only
  if (P.df) {
    // tags of this launch: tag0 + 1 .. tag0 + phases; the next launch starts
    // past them, so no word left by this one (finished or stopped) can match
    const unsigned phases = static_cast<unsigned>(n_steps) * static_cast<unsigned>(e->nphase);
    if (static_cast<unsigned long long>(e->df_tag) + phases + 2 >= 0x7fffffffull) {  // restart the tag space
      CK(cudaMemsetAsync(e->df_words, 0, e->df_nwords * 8, e->stream));
      e->df_tag = 0;
    }
    P.tag0 = e->df_tag;
    e->df_tag += phases + 2;
    // the attention's split arrivals accumulate from zero over the launch
    CK(cudaMemsetAsync(e->st->attn_counter, 0, sizeof(e->st->attn_counter), e->stream));
  }
  void *args[] = {&P};
  const void *kfn = P.df ? reinterpret_cast<const void *>(k_persistent<true>)
                         : reinterpret_cast<const void *>(k_persistent<false>);
  CK(cudaLaunchCooperativeKernel(kfn, dim3(e->num_sms), dim3(kPThreads),
                                 args, e->p_smem, e->stream));
  return C2S_OK;
}

int engine_build(c2s_engine *e, const c2s_model_desc *desc, const c2s_tensor_desc *ts, int n) {
  c2s_model_desc d = *desc;
  if (d.embd <= 0 || d.n_layers <= 0 || d.n_heads <= 0 || d.n_kv_heads <= 0 || d.ffn <= 0)
    return fail(C2S_ERR_ARG, "model desc: non-positive dimension");
  if (d.head_dim <= 0) d.head_dim = d.embd / d.n_heads;  // engine/model.go:137
  if (d.n_heads % d.n_kv_heads) return fail(C2S_ERR_UNSUPPORTED, "n_heads %% n_kv_heads != 0");
  if (d.head_dim % 4 || d.head_dim > 256 || d.head_dim % 2)
    return fail(C2S_ERR_UNSUPPORTED, "head_dim %d not supported", d.head_dim);
  if (d.n_kv_heads > 64) return fail(C2S_ERR_UNSUPPORTED, "more than 64 kv heads");
  if (d.max_tokens <= 0) d.max_tokens = kMaxContext;
  if (d.max_tokens > kMaxContext) return fail(C2S_ERR_ARG, "max_tokens above %d", kMaxContext);
  if (d.rope_base == 0) d.rope_base = 1000000.0f;
  if (d.eps == 0) d.eps = 1e-6f;
  const c2s_tensor_desc *te = find_t(ts, n, "token_embd.weight");
  if (!te || te->n_dims < 2) return fail(C2S_ERR_FORMAT, "missing token_embd.weight");
  if (d.vocab <= 0) d.vocab = static_cast<int32_t>(t_rows(te));  // engine/model.go:118
  const c2s_tensor_desc *on = find_t(ts, n, "output_norm.weight");
  if (!on) return fail(C2S_ERR_FORMAT, "missing output_norm.weight");
  const c2s_tensor_desc *ow = find_t(ts, n, "output.weight");
  if (!ow) ow = te;  // tied fallback (engine/model.go:126-130)
  const int H = d.embd, hd = d.head_dim;
  if (d.n_heads * hd != H) return fail(C2S_ERR_UNSUPPORTED, "n_heads*head_dim != embd");
  if (H % 256 && (is_kquant(te->type))) return fail(C2S_ERR_UNSUPPORTED, "embedding type needs embd %% 256 == 0");
  if (e->plan.world <= 1) {
    std::string why;
    tp_plan(d, 0, 1, e->plan, why);
  }
  const TpPlan &pl = e->plan;
  // this engine's rows (tensor parallel: the rank's shard; else the model)
  const int nq = (pl.h1 - pl.h0) * hd, kvd = (pl.g1 - pl.g0) * hd;
  const int F = pl.world > 1 ? (pl.f1 - pl.f0) * 256 : d.ffn;
  const int V = pl.v1 - pl.v0;
  if (int rc = check_matrix(ow->type, V, H, "output")) return rc;
  if (!(te->type == T_Q8_0 || te->type == T_Q5_0 || te->type == T_Q4_K || te->type == T_Q6_K || te->type == T_F32))
    return fail(C2S_ERR_UNSUPPORTED, "token_embd type %d", te->type);
  if (H > 16384 || F > 65536) return fail(C2S_ERR_UNSUPPORTED, "dimensions too large");

  // ---- collect the tensors to upload, with their arena offsets
  struct Up {
    const c2s_tensor_desc *t;
    size_t off;
  };
  std::vector<Up> ups;
  size_t total = 0;
  auto add = [&](const c2s_tensor_desc *t) -> size_t {
    for (auto &u : ups)
      if (u.t == t) return u.off;
    const size_t off = total;
    ups.push_back({t, off});
    total += (t->nbytes + 64 + 255) & ~size_t(255);
    return off;
  };
  struct LOff {
    size_t q, k, v, o, gate, up, down, an, fn, qb, kb, vb, qn, kn;
    int tq, tk, tv, to, tg, tu, td;
    bool hqb, hkb, hvb, hqn, hkn;
  };
  std::vector<LOff> lo(d.n_layers);
  char nm[128];
  for (int l = 0; l < d.n_layers; ++l) {
    auto T = [&](const char *s) {
      snprintf(nm, sizeof nm, "blk.%d.%s", l, s);
      return find_t(ts, n, nm);
    };
    const c2s_tensor_desc *an = T("attn_norm.weight"), *q = T("attn_q.weight"), *k = T("attn_k.weight"),
                          *v = T("attn_v.weight"), *o = T("attn_output.weight"), *fn = T("ffn_norm.weight"),
                          *g = T("ffn_gate.weight"), *u = T("ffn_up.weight"), *dn = T("ffn_down.weight");
    if (!an || !q || !k || !v || !o || !fn || !g || !u || !dn)
      return fail(C2S_ERR_FORMAT, "blk.%d is missing a projection or norm tensor", l);
    int rc;
    if ((rc = check_matrix(q->type, nq, H, "attn_q")) || (rc = check_matrix(k->type, kvd, H, "attn_k")) ||
        (rc = check_matrix(v->type, kvd, H, "attn_v")) || (rc = check_matrix(o->type, H, nq, "attn_output")) ||
        (rc = check_matrix(g->type, F, H, "ffn_gate")) || (rc = check_matrix(u->type, F, H, "ffn_up")) ||
        (rc = check_matrix(dn->type, H, F, "ffn_down")))
      return rc;
    if (t_cols(q) != H || t_rows(q) != nq || t_cols(k) != H || t_rows(k) != kvd || t_cols(v) != H ||
        t_rows(v) != kvd || t_cols(o) != nq || t_rows(o) != H || t_cols(g) != H || t_rows(g) != F ||
        t_cols(u) != H || t_rows(u) != F || t_cols(dn) != F || t_rows(dn) != H)
      return fail(C2S_ERR_FORMAT, "blk.%d tensor shapes do not match the hyper-parameters", l);
    LOff &x = lo[l];
    x.an = add(an); x.q = add(q); x.k = add(k); x.v = add(v); x.o = add(o);
    x.fn = add(fn); x.gate = add(g); x.up = add(u); x.down = add(dn);
    x.tq = q->type; x.tk = k->type; x.tv = v->type; x.to = o->type; x.tg = g->type; x.tu = u->type; x.td = dn->type;
    const c2s_tensor_desc *qb = T("attn_q.bias"), *kb = T("attn_k.bias"), *vb = T("attn_v.bias");
    const c2s_tensor_desc *qn = T("attn_q_norm.weight"), *kn = T("attn_k_norm.weight");
    x.hqb = qb; x.hkb = kb; x.hvb = vb; x.hqn = qn; x.hkn = kn;
    if (qb) { if (qb->nbytes < static_cast<uint64_t>(nq) * 4) return fail(C2S_ERR_FORMAT, "attn_q.bias too short"); x.qb = add(qb); }
    if (kb) { if (kb->nbytes < static_cast<uint64_t>(kvd) * 4) return fail(C2S_ERR_FORMAT, "attn_k.bias too short"); x.kb = add(kb); }
    if (vb) { if (vb->nbytes < static_cast<uint64_t>(kvd) * 4) return fail(C2S_ERR_FORMAT, "attn_v.bias too short"); x.vb = add(vb); }
    if (qn) x.qn = add(qn);
    if (kn) x.kn = add(kn);
  }
  const size_t off_te = add(te), off_on = add(on), off_ow = add(ow);

  // ---- device memory
  e->d = d;
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, e->device));
  e->num_sms = prop.multiProcessorCount;
  CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  if (cudaMalloc(&e->weights, total) != cudaSuccess) return fail(C2S_ERR_OOM, "weights: cudaMalloc(%zu) failed", total);
  e->weights_bytes = total;
  CK(cudaMemset(e->weights, 0, total));
  for (auto &u : ups) CK(cudaMemcpy(e->weights + u.off, u.t->data, u.t->nbytes, cudaMemcpyHostToDevice));
  const uint8_t *W = e->weights;
  e->tok_embd = W + off_te;
  e->tok_type = te->type;
  e->output = W + off_ow;
  e->out_type = ow->type;
  e->out_norm = reinterpret_cast<const float *>(W + off_on);
  e->layers.resize(d.n_layers);
  for (int l = 0; l < d.n_layers; ++l) {
    LayerDev &Ld = e->layers[l];
    const LOff &x = lo[l];
    Ld.q = W + x.q; Ld.k = W + x.k; Ld.v = W + x.v; Ld.o = W + x.o;
    Ld.gate = W + x.gate; Ld.up = W + x.up; Ld.down = W + x.down;
    Ld.tq = x.tq; Ld.tk = x.tk; Ld.tv = x.tv; Ld.to = x.to; Ld.tgate = x.tg; Ld.tup = x.tu; Ld.tdown = x.td;
    Ld.attn_norm = reinterpret_cast<const float *>(W + x.an);
    Ld.ffn_norm = reinterpret_cast<const float *>(W + x.fn);
    Ld.qb = x.hqb ? reinterpret_cast<const float *>(W + x.qb) : nullptr;
    Ld.kb = x.hkb ? reinterpret_cast<const float *>(W + x.kb) : nullptr;
    Ld.vb = x.hvb ? reinterpret_cast<const float *>(W + x.vb) : nullptr;
    Ld.qn = x.hqn ? reinterpret_cast<const float *>(W + x.qn) : nullptr;
    Ld.kn = x.hkn ? reinterpret_cast<const float *>(W + x.kn) : nullptr;
  }
  // RoPE table over MaxContextLen, angles in float64 (tensor/ops.go:237-257)
  {
    const int half = hd / 2;
    std::vector<float> c(static_cast<size_t>(kMaxContext) * half), s(c.size());
    for (int p = 0; p < kMaxContext; ++p)
      for (int i = 0; i < half; ++i) {
        const double freq = 1.0 / pow(static_cast<double>(d.rope_base), static_cast<double>(2 * i) / hd);
        const double val = static_cast<double>(p) * freq;
        c[static_cast<size_t>(p) * half + i] = static_cast<float>(cos(val));
        s[static_cast<size_t>(p) * half + i] = static_cast<float>(sin(val));
      }
    CK(cudaMalloc(&e->rope_cos, c.size() * 4));
    CK(cudaMalloc(&e->rope_sin, s.size() * 4));
    CK(cudaMemcpy(e->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(e->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
  }
  // KV cache [2][L][KVH][max_tokens][hd] fp32 (engine/kvcache.go:31); a
  // tensor-parallel rank keeps its kv heads only
  const size_t kvn = static_cast<size_t>(2) * d.n_layers * (pl.g1 - pl.g0) * d.max_tokens * hd;
  if (cudaMalloc(&e->kv, kvn * 4) != cudaSuccess) return fail(C2S_ERR_OOM, "KV cache: cudaMalloc(%zu) failed", kvn * 4);
  CK(cudaMemset(e->kv, 0, kvn * 4));
  e->max_splits = std::max(1, std::min(kMaxSplits, e->num_sms / d.n_kv_heads));
  // positions per attention split, fixed for the engine so that position p
  // always belongs to split p / split_len: at least 64 KB of K per split, and
  // few enough splits for max_tokens
  e->split_len = std::max(16384 / hd, (d.max_tokens + e->max_splits - 1) / e->max_splits);
  const int qpk = d.n_heads / d.n_kv_heads;
  if (qpk > 8) return fail(C2S_ERR_UNSUPPORTED, "more than 8 query heads per kv head");
  if (hd != 64 && hd != 128) return fail(C2S_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  e->attn_smem = attn_smem_bytes(hd, qpk);
  if (e->attn_smem > 200 * 1024) return fail(C2S_ERR_UNSUPPORTED, "attention smem %zu too large", e->attn_smem);
  auto dalloc = [&](void **p, size_t bytes) -> int {
    if (cudaMalloc(p, bytes) != cudaSuccess) return fail(C2S_ERR_OOM, "cudaMalloc(%zu) failed", bytes);
    if (cudaMemset(*p, 0, bytes) != cudaSuccess) return fail(C2S_ERR_CUDA, "cudaMemset failed");
    return C2S_OK;
  };
  int rc;
  if ((rc = dalloc(reinterpret_cast<void **>(&e->X), H * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->normx), H * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->q), H * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->k), kvd * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->v), kvd * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->attn_out), H * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->h), static_cast<size_t>(F) * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->logits), static_cast<size_t>(d.vocab) * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->part),
                   static_cast<size_t>(d.n_heads) * e->max_splits * (hd + 2) * 4)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->amax_part), static_cast<size_t>(e->num_sms) * sizeof(float2))) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->token_ids), static_cast<size_t>(d.max_tokens) * 4)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->out_tokens), static_cast<size_t>(d.max_tokens) * 4 + 64)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->rows_idx), static_cast<size_t>(d.vocab) * 4)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->scratch_x), static_cast<size_t>(d.vocab) * 4)) ||
      (rc = dalloc(reinterpret_cast<void **>(&e->st), sizeof(DevState))))
    return rc;
  if (pl.world > 1) {
    if ((rc = dalloc(reinterpret_cast<void **>(&e->delta), static_cast<size_t>(H) * 4 + 64)) ||
        (rc = dalloc(reinterpret_cast<void **>(&e->logits_full),
                     static_cast<size_t>(pl.world) * pl.vpad * 4 + 64)))
      return rc;
    // rows past this rank's share of the padded split never win the argmax
    if (V < pl.vpad) {
      std::vector<float> ninf(static_cast<size_t>(pl.vpad - V), -INFINITY);
      CK(cudaMemcpy(e->logits + V, ninf.data(), ninf.size() * 4, cudaMemcpyHostToDevice));
    }
  }
  CK(cudaMallocHost(&e->h_in, sizeof(HostFwdIn) * (d.max_tokens + 8)));
  CK(cudaMallocHost(&e->h_buf, static_cast<size_t>(std::max(d.vocab, H)) * 4 + 64));
  CK(cudaMallocHost(&e->h_st, sizeof(DevState)));
  CK(cudaMallocHost(&e->h_tokens, static_cast<size_t>(d.max_tokens) * 4 + 64));
  DevState s0{};
  s0.penalty = 1.15f;  // c2slm.go:165-167
  s0.window = 64;      // c2slm.go:157
  s0.stop_on_special = 1;
  s0.out_cap = d.max_tokens;
  s0.im_end = d.im_end;
  s0.eos = d.eos;
  s0.vocab = d.vocab;
  CK(cudaMemcpy(e->st, &s0, sizeof s0, cudaMemcpyHostToDevice));

  // ---- kernels: shared-memory limits, graphs
  CK(cudaFuncSetAttribute(k_matvec, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  CK(cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  CK(cudaFuncSetAttribute(k_pf_flash<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pf_flash_smem(128))));
  CK(cudaFuncSetAttribute(k_pf_flash<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pf_flash_smem(64))));
  CK(cudaFuncSetAttribute(k_pf_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ta_smem(128))));
  CK(cudaFuncSetAttribute(k_pf_attn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ta_smem(64))));
  CK(cudaFuncSetAttribute(k_pf_gemm<T_Q4_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
  CK(cudaFuncSetAttribute(k_pf_gemm<T_Q6_K>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem));
  {  // prefill on the tensor cores: one GPU, every layer projection a K-quant, superblock-aligned widths
    bool okp = d.embd % 256 == 0 && d.ffn % 256 == 0 && (hd == 64 || hd == 128);
    for (int l = 0; l < d.n_layers && okp; ++l) {
      const LayerDev &Ld = e->layers[l];
      for (int t : {Ld.tq, Ld.tk, Ld.tv, Ld.to, Ld.tgate, Ld.tup, Ld.tdown}) okp = okp && is_kquant(t);
    }
    const char *pe = getenv("C2S_PREFILL");
    e->pf_ok = okp && !(pe && strcmp(pe, "0") == 0) ? 1 : 0;
    const char *pa = getenv("C2S_PF_ATTN");
    e->pf_attn_fp32 = pa && strcmp(pa, "fp32") == 0 ? 1 : 0;
  }
  if ((rc = capture(e, &e->g_forward, 0)) || (rc = capture(e, &e->g_step, 1)) ||
      (rc = capture(e, &e->g_logits, 2)) || (rc = capture(e, &e->g_fwd_select, 3))) {
    if (!g_use_pdl) return rc;
    // graphs with programmatic edges refused: capture plain launches instead
    fprintf(stderr, "c2slm_b200: PDL capture failed (%s); using plain launches\n", g_err.c_str());
    cudaGetLastError();
    g_use_pdl = false;
    for (cudaGraphExec_t *gx : {&e->g_forward, &e->g_step, &e->g_logits, &e->g_fwd_select})
      if (*gx) { cudaGraphExecDestroy(*gx); *gx = nullptr; }
    if ((rc = capture(e, &e->g_forward, 0)) || (rc = capture(e, &e->g_step, 1)) ||
        (rc = capture(e, &e->g_logits, 2)) || (rc = capture(e, &e->g_fwd_select, 3)))
      return rc;
  }
  e->kernels_per_step = 5 * d.n_layers + 1;
  if (pl.world > 1) e->kernels_per_step = 7 * d.n_layers + 2;  // + a residual add after each allreduce, + selection
  if ((rc = persistent_setup(e))) return rc;
  if (pl.world > 1) {  // until tp_exchange_setup has mapped the peers' buffers
    e->tp_persist_ok = e->use_persistent;
    e->use_persistent = false;
  }
  // every set-up copy and memset (some on the legacy stream, which the
  // engine's non-blocking stream does not wait for) completes here
  CK(cudaDeviceSynchronize());
  return C2S_OK;
}

// Persistent decode across a tensor-parallel group: every rank allocates one
// exchange region of tagged 64-bit words (partial rows [2][world][H], argmax
// partials [2][world][G][2]), zeroed, and maps every other
// rank's region through CUDA IPC; the handles travel through an NCCL
// all-gather, which also guarantees that every rank has zeroed its region
// before any rank starts decoding.
int tp_exchange_setup(c2s_engine *e) {
  const TpPlan &pl = e->plan;
  const int W = pl.world, G = e->num_sms, H = e->d.embd;
  if (W > kMaxRanks) return fail(C2S_ERR_UNSUPPORTED, "more than %d ranks", kMaxRanks);
  const NcclApi *nc = nullptr;
  if (int rc = nccl_api(&nc)) return rc;
  auto a256 = [](size_t v) { return (v + 255) & ~size_t(255); };
  // tagged words: recv [2][W][H], argbuf [2][W][G][2]; zero = tag 0, never expected
  const size_t off_arg = a256(static_cast<size_t>(2) * W * H * 8);
  const size_t bytes = off_arg + a256(static_cast<size_t>(2) * W * G * 2 * 8);
  CK(cudaMalloc(&e->tp_shared, bytes));
  CK(cudaMemset(e->tp_shared, 0, bytes));
  CK(cudaMalloc(&e->xbuf, static_cast<size_t>(2) * H * 4 + 64));
  CK(cudaMemset(e->xbuf, 0, static_cast<size_t>(2) * H * 4 + 64));
  CK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t mine;
  CK(cudaIpcGetMemHandle(&mine, e->tp_shared));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  uint8_t *dh = nullptr;
  CK(cudaMalloc(&dh, static_cast<size_t>(64) * W));
  CK(cudaMemcpy(dh + 64 * pl.rank, &mine, 64, cudaMemcpyHostToDevice));
  const ncclResult_t r = nc->all_gather(dh + 64 * pl.rank, dh, 64, ncclUint8, e->comm, e->stream);
  if (r != ncclSuccess) {
    cudaFree(dh);
    return fail(C2S_ERR_CUDA, "ncclAllGather (IPC handles): %s", nc->err_str(r));
  }
  std::vector<cudaIpcMemHandle_t> hs(W);
  CK(cudaStreamSynchronize(e->stream));
  CK(cudaMemcpy(hs.data(), dh, static_cast<size_t>(64) * W, cudaMemcpyDeviceToHost));
  cudaFree(dh);
  for (int k = 0; k < W; ++k) {
    if (k == pl.rank) {
      e->peer_shared[k] = e->tp_shared;
      continue;
    }
    void *p = nullptr;
    const cudaError_t er = cudaIpcOpenMemHandle(&p, hs[k], cudaIpcMemLazyEnablePeerAccess);
    if (er != cudaSuccess) return fail(C2S_ERR_CUDA, "cudaIpcOpenMemHandle (rank %d): %s", k, cudaGetErrorString(er));
    e->peer_shared[k] = static_cast<uint8_t *>(p);
  }
  PParams &P = e->pp;
  P.ll = 1;
  P.xbuf = e->xbuf;
  P.recv = reinterpret_cast<const unsigned long long *>(e->tp_shared);
  P.argbuf = reinterpret_cast<const unsigned long long *>(e->tp_shared + off_arg);
  for (int k = 0; k < W; ++k) {
    P.peer_recv[k] = reinterpret_cast<unsigned long long *>(e->peer_shared[k]);
    P.peer_arg[k] = reinterpret_cast<unsigned long long *>(e->peer_shared[k] + off_arg);
  }
  e->use_persistent = e->tp_persist_ok;
  return C2S_OK;
}

// Copies of the tensors one tensor-parallel rank holds: rows of attn_q /
// attn_k / attn_v (+ biases), ffn_gate / ffn_up and the output projection
// (the tied token_embd serves as output.weight), columns of attn_output and
// ffn_down (whole blocks of every row).  Row slices point into the caller's
// memory; column slices are gathered into `own`.
int tp_slice(const c2s_model_desc &d, const TpPlan &pl, const c2s_tensor_desc *ts, int n,
             std::vector<c2s_tensor_desc> &out, std::vector<std::vector<uint8_t>> &own,
             std::vector<std::string> &names) {
  const int hd = d.head_dim;
  out.clear();
  own.clear();
  names.clear();
  names.reserve(static_cast<size_t>(n) + 1);
  auto rows = [&](const c2s_tensor_desc &t, int64_t r0, int64_t r1) -> int {
    const bool vec = t.n_dims < 2;  // a bias: its elements are the rows
    const int64_t cols = vec ? 1 : t_cols(&t), nr = vec ? t.dims[0] : t_rows(&t);
    if (vec && t.type != T_F32) return fail(C2S_ERR_FORMAT, "%s: 1-D tensor of type %d", t.name, t.type);
    const size_t rb = t.type == T_F32 ? static_cast<size_t>(cols) * 4 : row_bytes_of(t.type, cols);
    if (r1 > nr || r0 < 0 || r0 > r1) return fail(C2S_ERR_FORMAT, "%s: rows %lld..%lld of %lld", t.name, (long long)r0, (long long)r1, (long long)nr);
    c2s_tensor_desc c = t;
    c.data = static_cast<const uint8_t *>(t.data) + static_cast<size_t>(r0) * rb;
    c.nbytes = static_cast<uint64_t>(r1 - r0) * rb;
    if (t.n_dims >= 2) c.dims[1] = r1 - r0; else c.dims[0] = r1 - r0;
    out.push_back(c);
    return C2S_OK;
  };
  auto cols = [&](const c2s_tensor_desc &t, int64_t c0, int64_t c1) -> int {
    const int64_t nc = t_cols(&t), nr = t_rows(&t);
    const int blk = is_kquant(t.type) ? 256 : 32;
    const size_t bb = row_bytes_of(t.type, blk);
    if (!(is_kquant(t.type) || is_f32x(t.type)) || c0 % blk || c1 % blk || c1 > nc)
      return fail(C2S_ERR_UNSUPPORTED, "%s: column slice %lld..%lld of type %d", t.name, (long long)c0, (long long)c1, t.type);
    const size_t rb = row_bytes_of(t.type, nc), sb = static_cast<size_t>((c1 - c0) / blk) * bb;
    own.emplace_back(static_cast<size_t>(nr) * sb);
    std::vector<uint8_t> &buf = own.back();
    const uint8_t *src = static_cast<const uint8_t *>(t.data);
    for (int64_t r = 0; r < nr; ++r)
      memcpy(buf.data() + r * sb, src + r * rb + static_cast<size_t>(c0 / blk) * bb, sb);
    c2s_tensor_desc c = t;
    c.data = buf.data();
    c.nbytes = buf.size();
    c.dims[0] = c1 - c0;
    out.push_back(c);
    return C2S_OK;
  };
  own.reserve(static_cast<size_t>(2 * d.n_layers) + 1);
  bool has_output = false;
  for (int i = 0; i < n; ++i) {
    const c2s_tensor_desc &t = ts[i];
    const std::string nm = t.name ? t.name : "";
    auto ends = [&](const char *suf) {
      const size_t k = strlen(suf);
      return nm.size() >= k && nm.compare(nm.size() - k, k, suf) == 0;
    };
    int rc = C2S_OK;
    if (ends(".attn_q.weight") || ends(".attn_q.bias")) rc = rows(t, int64_t(pl.h0) * hd, int64_t(pl.h1) * hd);
    else if (ends(".attn_k.weight") || ends(".attn_k.bias") || ends(".attn_v.weight") || ends(".attn_v.bias"))
      rc = rows(t, int64_t(pl.g0) * hd, int64_t(pl.g1) * hd);
    else if (ends(".attn_output.weight")) rc = cols(t, int64_t(pl.h0) * hd, int64_t(pl.h1) * hd);
    else if (ends(".ffn_gate.weight") || ends(".ffn_up.weight")) rc = rows(t, int64_t(pl.f0) * 256, int64_t(pl.f1) * 256);
    else if (ends(".ffn_down.weight")) rc = cols(t, int64_t(pl.f0) * 256, int64_t(pl.f1) * 256);
    else if (nm == "output.weight") {
      rc = rows(t, pl.v0, pl.v1);
      has_output = true;
    } else out.push_back(t);
    if (rc) return rc;
  }
  if (!has_output) {  // tied embeddings: the rank's vocabulary rows of token_embd project the logits
    const c2s_tensor_desc *te = find_t(ts, n, "token_embd.weight");
    if (!te) return fail(C2S_ERR_FORMAT, "missing token_embd.weight");
    if (int rc = rows(*te, pl.v0, pl.v1)) return rc;
    names.push_back("output.weight");
    out.back().name = names.back().c_str();
  }
  return C2S_OK;
}

void engine_free(c2s_engine *e) {
  if (!e) return;
  DeviceGuard g(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (cudaGraphExec_t *gx : {&e->g_forward, &e->g_step, &e->g_logits, &e->g_fwd_select})
    if (*gx) cudaGraphExecDestroy(*gx);
  for (void *p : {static_cast<void *>(e->weights), static_cast<void *>(e->kv), static_cast<void *>(e->rope_cos),
                  static_cast<void *>(e->rope_sin), static_cast<void *>(e->X), static_cast<void *>(e->normx),
                  static_cast<void *>(e->q), static_cast<void *>(e->k), static_cast<void *>(e->v),
                  static_cast<void *>(e->attn_out), static_cast<void *>(e->h), static_cast<void *>(e->logits),
                  static_cast<void *>(e->part), static_cast<void *>(e->amax_part), static_cast<void *>(e->token_ids),
                  static_cast<void *>(e->out_tokens), static_cast<void *>(e->rows_idx),
                  static_cast<void *>(e->scratch_x), static_cast<void *>(e->st),
                  static_cast<void *>(e->gbar), static_cast<void *>(e->delta),
                  static_cast<void *>(e->logits_full), static_cast<void *>(e->df_words)})
    if (p) cudaFree(p);
  for (void *p : {static_cast<void *>(e->pf_x), static_cast<void *>(e->pf_q), static_cast<void *>(e->pf_k),
                  static_cast<void *>(e->pf_v), static_cast<void *>(e->pf_att), static_cast<void *>(e->pf_g),
                  static_cast<void *>(e->pf_u), static_cast<void *>(e->pf_d8), static_cast<void *>(e->pf_q8),
                  static_cast<void *>(e->pf_tok), static_cast<void *>(e->pf_planes), static_cast<void *>(e->pf_bs),
                  static_cast<void *>(e->pf_fpart), static_cast<void *>(e->pf_fcount), static_cast<void *>(e->pf_delta),
                  static_cast<void *>(e->pf_kvt)})
    if (p) cudaFree(p);
  for (int k = 0; k < 8; ++k)
    if (e->peer_shared[k] && e->peer_shared[k] != e->tp_shared) cudaIpcCloseMemHandle(e->peer_shared[k]);
  for (void *p : {static_cast<void *>(e->tp_shared), static_cast<void *>(e->xbuf)})
    if (p) cudaFree(p);
  if (e->comm) {
    const NcclApi *nc = nullptr;
    if (nccl_api(&nc) == C2S_OK) nc->destroy(e->comm);
  }
  for (void *p : {static_cast<void *>(e->h_in), static_cast<void *>(e->h_buf), static_cast<void *>(e->h_st),
                  static_cast<void *>(e->h_tokens)})
    if (p) cudaFreeHost(p);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

// per-device context for the op-level entry points
struct OpCtx {
  cudaStream_t stream = nullptr;
  DevState *st = nullptr;
  bool ready = false;
};
std::mutex g_op_mu;
OpCtx g_op[64];

int op_ctx(int device, OpCtx **out) {
  if (device < 0 || device >= 64) return fail(C2S_ERR_ARG, "device %d out of range", device);
  std::lock_guard<std::mutex> lk(g_op_mu);
  OpCtx &c = g_op[device];
  if (!c.ready) {
    CK(cudaSetDevice(device));
    CK(cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&c.st, sizeof(DevState)));
    CK(cudaMemset(c.st, 0, sizeof(DevState)));
    CK(cudaFuncSetAttribute(k_matvec, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    c.ready = true;
  }
  *out = &c;
  return C2S_OK;
}

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

// RAW matvec launch on device pointers
int gemv_launch(OpCtx *c, int type, const void *dw, const float *dx, float *dy, int rows, int cols, int32_t *dbg) {
  if (int rc = check_matrix(type, rows, cols, "gemv")) return rc;
  int nsm = 148;
  int dev = current_device();
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  MatParams P{};
  P.kind = K_RAW;
  P.nseg = 1;
  P.cols = cols;
  P.seg[0] = make_seg(static_cast<const uint8_t *>(dw), type, rows, cols, nullptr, dy);
  P.x_in = dx;
  P.st = c->st;
  P.dbg = dbg;
  finish_needs(P);
  layout_matvec(P, nsm);
  CK(launch(k_matvec, dim3(nsm), dim3(kThreads), P.smem_bytes, c->stream, P));
  return C2S_OK;
}

template <class T>
struct DevBuf {
  T *p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  // zeroed on the op's stream: the op streams are non-blocking, so a memset
  // on the legacy default stream would not be ordered before the kernels
  int alloc(size_t n, cudaStream_t s) {
    if (cudaMalloc(&p, n * sizeof(T) + 64) != cudaSuccess) return fail(C2S_ERR_OOM, "cudaMalloc failed");
    if (cudaMemsetAsync(p, 0, n * sizeof(T) + 64, s) != cudaSuccess) return fail(C2S_ERR_CUDA, "cudaMemsetAsync failed");
    return C2S_OK;
  }
};

int op_finish(OpCtx *c) {
  CK(cudaStreamSynchronize(c->stream));
  unsigned err = 0;
  CK(cudaMemcpy(&err, &c->st->err, sizeof err, cudaMemcpyDeviceToHost));
  if (err) {
    cudaMemset(&c->st->err, 0, sizeof(unsigned));
    return fail(C2S_ERR_TIMEOUT, "device reported error flags 0x%x", err);
  }
  return C2S_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char *c2s_last_error(void) { return g_err.c_str(); }
const char *c2s_version(void) { return "c2slm_b200 0.1 sm_100a"; }

int c2s_engine_create(const c2s_model_desc *desc, const c2s_tensor_desc *tensors, int n_tensors, int device,
                      c2s_engine **out) {
  if (!desc || !tensors || n_tensors <= 0 || !out) return fail(C2S_ERR_ARG, "null argument");
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(C2S_ERR_CUDA, "no CUDA device");
  if (device < 0 || device >= ndev) return fail(C2S_ERR_ARG, "device %d of %d", device, ndev);
  DeviceGuard g(device);
  auto *e = new c2s_engine();
  e->device = device;
  const int rc = engine_build(e, desc, tensors, n_tensors);
  if (rc != C2S_OK) {
    const std::string msg = g_err;
    engine_free(e);
    g_err = msg;
    return rc;
  }
  *out = e;
  return C2S_OK;
}

// hyper-parameters and tensor table of an opened GGUF, as engine.LoadModel reads them
static void gguf_descs(GFile *f, int max_tokens, c2s_model_desc &d, std::vector<c2s_tensor_desc> &ts) {
  // engine/model.go:64-112: qwen2.* keys, then qwen3.*, then defaults
  d = c2s_model_desc{};
  uint32_t u;
  auto hp = [&](const char *k2, const char *k3, int dflt) {
    u = 0;
    f->u32(k2, &u);
    if (u == 0) f->u32(k3, &u);
    if (u == 0) u = static_cast<uint32_t>(dflt);
    return static_cast<int32_t>(u);
  };
  d.embd = hp("qwen2.embedding_length", "qwen3.embedding_length", 896);
  d.n_layers = hp("qwen2.block_count", "qwen3.block_count", 24);
  d.n_heads = hp("qwen2.attention.head_count", "qwen3.attention.head_count", 14);
  d.n_kv_heads = hp("qwen2.attention.head_count_kv", "qwen3.attention.head_count_kv", 2);
  d.ffn = hp("qwen2.feed_forward_length", "qwen3.feed_forward_length", 4864);
  float fv = 0;
  f->f32("qwen2.rope.freq_base", &fv);
  if (fv == 0) f->f32("qwen3.rope.freq_base", &fv);
  d.rope_base = fv == 0 ? 1000000.0f : fv;
  fv = 0;
  f->f32("qwen2.attention.layer_norm_rms_epsilon", &fv);
  if (fv == 0) f->f32("qwen3.attention.layer_norm_rms_epsilon", &fv);
  d.eps = fv == 0 ? 1e-6f : fv;
  d.max_tokens = max_tokens > 0 ? max_tokens : kMaxContext;
  d.im_end = f->im_end;
  d.eos = f->eos;
  ts.assign(f->tensors.size(), c2s_tensor_desc{});
  for (size_t i = 0; i < ts.size(); ++i) {
    const GTensor &t = f->tensors[i];
    ts[i].name = t.name.c_str();
    ts[i].type = t.type;
    ts[i].n_dims = t.n_dims;
    for (int k = 0; k < 4; ++k) ts[i].dims[k] = t.dims[k];
    ts[i].data = t.data;
    ts[i].nbytes = t.nbytes;
  }
}

int c2s_engine_open(const char *path, int device, int max_tokens, c2s_engine **out) {
  if (!path || !out) return fail(C2S_ERR_ARG, "null argument");
  std::unique_ptr<GFile> f;
  if (int rc = gguf_open(path, f)) return rc;
  c2s_model_desc d;
  std::vector<c2s_tensor_desc> ts;
  gguf_descs(f.get(), max_tokens, d, ts);
  return c2s_engine_create(&d, ts.data(), static_cast<int>(ts.size()), device, out);
}

int c2s_engine_open_tp(const char *path, int device, int max_tokens, int rank, int world, const uint8_t *nccl_id,
                       c2s_engine **out) {
  if (!path || !out) return fail(C2S_ERR_ARG, "null argument");
  std::unique_ptr<GFile> f;
  if (int rc = gguf_open(path, f)) return rc;
  c2s_model_desc d;
  std::vector<c2s_tensor_desc> ts;
  gguf_descs(f.get(), max_tokens, d, ts);
  return c2s_engine_create_tp(&d, ts.data(), static_cast<int>(ts.size()), device, rank, world, nccl_id, out);
}

int c2s_nccl_unique_id(uint8_t *id_out) {
  if (!id_out) return fail(C2S_ERR_ARG, "null argument");
  const NcclApi *nc = nullptr;
  if (int rc = nccl_api(&nc)) return rc;
  ncclUniqueId id;
  const ncclResult_t r = nc->get_id(&id);
  if (r != ncclSuccess) return fail(C2S_ERR_CUDA, "ncclGetUniqueId: %s", nc->err_str(r));
  static_assert(sizeof(ncclUniqueId) == C2S_NCCL_ID_BYTES, "NCCL unique id size");
  memcpy(id_out, &id, sizeof id);
  return C2S_OK;
}

int c2s_tp_plan(const c2s_model_desc *desc, int rank, int world, int32_t *plan_out) {
  if (!desc || !plan_out) return fail(C2S_ERR_ARG, "null argument");
  if (world < 1 || rank < 0 || rank >= world) return fail(C2S_ERR_ARG, "rank %d of %d", rank, world);
  c2s_model_desc d = *desc;
  if (d.head_dim <= 0 && d.n_heads > 0) d.head_dim = d.embd / d.n_heads;
  if (d.n_heads <= 0 || d.n_kv_heads <= 0 || d.n_heads % d.n_kv_heads || d.vocab <= 0)
    return fail(C2S_ERR_ARG, "model desc: heads / vocab");
  TpPlan p;
  std::string why;
  if (tp_plan(d, rank, world, p, why)) return fail(C2S_ERR_UNSUPPORTED, "%s", why.c_str());
  const int32_t v[9] = {p.h0, p.h1, p.g0, p.g1, p.f0, p.f1, p.v0, p.v1, p.vpad};
  memcpy(plan_out, v, sizeof v);
  return C2S_OK;
}

int c2s_engine_create_tp(const c2s_model_desc *desc, const c2s_tensor_desc *tensors, int n_tensors, int device,
                         int rank, int world, const uint8_t *nccl_id, c2s_engine **out) {
  if (!desc || !tensors || n_tensors <= 0 || !out || !nccl_id) return fail(C2S_ERR_ARG, "null argument");
  if (world < 2 || rank < 0 || rank >= world) return fail(C2S_ERR_ARG, "rank %d of world %d", rank, world);
  *out = nullptr;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(C2S_ERR_CUDA, "no CUDA device");
  if (device < 0 || device >= ndev) return fail(C2S_ERR_ARG, "device %d of %d", device, ndev);
  // the dimensions LoadModel derives (engine/model.go:118,137)
  c2s_model_desc d = *desc;
  if (d.n_heads <= 0 || d.n_kv_heads <= 0 || d.embd <= 0) return fail(C2S_ERR_ARG, "model desc: non-positive dimension");
  if (d.head_dim <= 0) d.head_dim = d.embd / d.n_heads;
  const c2s_tensor_desc *te = find_t(tensors, n_tensors, "token_embd.weight");
  if (!te || te->n_dims < 2) return fail(C2S_ERR_FORMAT, "missing token_embd.weight");
  if (d.vocab <= 0) d.vocab = static_cast<int32_t>(t_rows(te));
  TpPlan plan;
  std::string why;
  if (tp_plan(d, rank, world, plan, why)) return fail(C2S_ERR_UNSUPPORTED, "%s", why.c_str());
  std::vector<c2s_tensor_desc> shard;
  std::vector<std::vector<uint8_t>> own;
  std::vector<std::string> names;
  if (int rc = tp_slice(d, plan, tensors, n_tensors, shard, own, names)) return rc;
  const NcclApi *nc = nullptr;
  if (int rc = nccl_api(&nc)) return rc;
  DeviceGuard g(device);
  auto *e = new c2s_engine();
  e->device = device;
  e->plan = plan;
  ncclUniqueId id;
  memcpy(&id, nccl_id, sizeof id);
  const ncclResult_t r = nc->init_rank(&e->comm, world, id, rank);
  if (r != ncclSuccess) {
    e->comm = nullptr;
    engine_free(e);
    return fail(C2S_ERR_CUDA, "ncclCommInitRank: %s", nc->err_str(r));
  }
  int rc = engine_build(e, &d, shard.data(), static_cast<int>(shard.size()));
  if (rc == C2S_OK) rc = tp_exchange_setup(e);
  if (rc != C2S_OK) {
    const std::string msg = g_err;
    engine_free(e);
    g_err = msg;
    return rc;
  }
  *out = e;
  return C2S_OK;
}

void c2s_engine_close(c2s_engine *e) { engine_free(e); }

int c2s_engine_desc(const c2s_engine *e, c2s_model_desc *out) {
  if (!e || !out) return fail(C2S_ERR_ARG, "null argument");
  *out = e->d;
  return C2S_OK;
}

int c2s_forward(c2s_engine *e, int32_t token, int32_t pos, float *normx_out) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (pos < 0 || pos >= e->d.max_tokens) return fail(C2S_ERR_ARG, "pos %d outside [0, %d)", pos, e->d.max_tokens);
  DeviceGuard g(e->device);
  if (int rc = set_fwd_input(e, token, pos, 0)) return rc;
  CK(cudaGraphLaunch(e->g_forward, e->stream));
  if (normx_out) CK(cudaMemcpyAsync(e->h_buf, e->normx, e->d.embd * 4, cudaMemcpyDeviceToHost, e->stream));
  if (int rc = read_status(e)) return rc;
  if (normx_out) memcpy(normx_out, e->h_buf, e->d.embd * 4);
  return C2S_OK;
}

int c2s_compute_logits(c2s_engine *e, const float *normx_in, const int32_t *targets, int n_targets,
                       float *logits_out) {
  if (!e || !logits_out) return fail(C2S_ERR_ARG, "null argument");
  if (n_targets < 0) return fail(C2S_ERR_ARG, "n_targets < 0");
  DeviceGuard g(e->device);
  if (normx_in) {
    memcpy(e->h_buf, normx_in, e->d.embd * 4);
    CK(cudaMemcpyAsync(e->normx, e->h_buf, e->d.embd * 4, cudaMemcpyHostToDevice, e->stream));
  }
  if (targets && n_targets > 0 && e->plan.world > 1) {
    // tensor parallel: the vocabulary is spread over the ranks; project it
    // whole (a collective every rank makes) and keep the targets
    std::vector<float> all(static_cast<size_t>(e->d.vocab));
    if (int rc = c2s_compute_logits(e, nullptr, nullptr, 0, all.data())) return rc;
    for (int i = 0; i < n_targets; ++i) {
      const int t = targets[i];
      if (t >= 0 && t < e->d.vocab) logits_out[t] = all[t];  // engine/forward.go:177-179
    }
    return C2S_OK;
  }
  if (targets && n_targets > 0) {
    if (n_targets > e->d.vocab) return fail(C2S_ERR_ARG, "too many targets");
    memcpy(e->h_tokens, targets, static_cast<size_t>(n_targets) * 4);
    CK(cudaMemcpyAsync(e->rows_idx, e->h_tokens, static_cast<size_t>(n_targets) * 4, cudaMemcpyHostToDevice,
                       e->stream));
    k_dot_rows_f32x<<<n_targets, kThreads, 0, e->stream>>>(e->out_type, e->output,
                                                           static_cast<int>(row_bytes_of(e->out_type, e->d.embd)),
                                                           e->normx, e->rows_idx, n_targets, e->scratch_x,
                                                           e->d.vocab, e->d.embd);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(e->h_buf, e->scratch_x, static_cast<size_t>(n_targets) * 4, cudaMemcpyDeviceToHost,
                       e->stream));
    CK(cudaStreamSynchronize(e->stream));
    for (int i = 0; i < n_targets; ++i) {
      const int t = targets[i];
      if (t < 0 || t >= e->d.vocab) continue;  // engine/forward.go:177-179
      logits_out[t] = e->h_buf[i];
    }
    return C2S_OK;
  }
  CK(cudaGraphLaunch(e->g_logits, e->stream));
  CK(cudaMemcpyAsync(e->h_buf, e->plan.world > 1 ? e->logits_full : e->logits, static_cast<size_t>(e->d.vocab) * 4,
                     cudaMemcpyDeviceToHost, e->stream));
  if (int rc = read_status(e)) return rc;
  memcpy(logits_out, e->h_buf, static_cast<size_t>(e->d.vocab) * 4);
  return C2S_OK;
}

int c2s_kv_seq_len(const c2s_engine *e) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  return e->host_seq;
}

int c2s_kv_set_seq_len(c2s_engine *e, int seq_len) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (seq_len < 0 || seq_len > e->d.max_tokens) return fail(C2S_ERR_ARG, "seq_len %d out of range", seq_len);
  DeviceGuard g(e->device);
  e->h_st->seq_len = seq_len;
  CK(cudaMemcpyAsync(&e->st->seq_len, &e->h_st->seq_len, sizeof(int), cudaMemcpyHostToDevice, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  e->host_seq = seq_len;
  return C2S_OK;
}

int c2s_kv_reset(c2s_engine *e) { return c2s_kv_set_seq_len(e, 0); }

int c2s_kv_rewind(c2s_engine *e, int n) {  // engine/kvcache.go:109-117
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (n < 0) n = 0;
  if (n > e->host_seq) n = e->host_seq;
  return c2s_kv_set_seq_len(e, e->host_seq - n);
}

int c2s_kv_store_token_id(c2s_engine *e, int pos, int32_t token) {  // engine/kvcache.go:120-125
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (pos < 0 || pos >= e->d.max_tokens) return C2S_OK;  // ignored like the reference
  DeviceGuard g(e->device);
  e->h_tokens[0] = token;
  CK(cudaMemcpyAsync(e->token_ids + pos, e->h_tokens, 4, cudaMemcpyHostToDevice, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return C2S_OK;
}

int c2s_kv_token_ids(const c2s_engine *e, int32_t *out, int n) {
  if (!e || !out) return fail(C2S_ERR_ARG, "null argument");
  if (n < 0 || n > e->d.max_tokens) return fail(C2S_ERR_ARG, "n out of range");
  DeviceGuard g(e->device);
  CK(cudaMemcpy(out, e->token_ids, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost));
  return C2S_OK;
}

int c2s_kv_get(const c2s_engine *e, int is_value, int layer, int kv_head, int pos, float *out) {
  if (!e || !out) return fail(C2S_ERR_ARG, "null argument");
  if (layer < 0 || layer >= e->d.n_layers || kv_head < 0 || kv_head >= e->d.n_kv_heads || pos < 0 ||
      pos >= e->d.max_tokens)
    return fail(C2S_ERR_ARG, "kv index out of range");
  // a tensor-parallel rank holds kv heads [g0, g1)
  const int nkv = e->plan.g1 - e->plan.g0, g = kv_head - e->plan.g0;
  if (g < 0 || g >= nkv) return fail(C2S_ERR_ARG, "kv head %d is not held by this rank", kv_head);
  DeviceGuard dg(e->device);
  const size_t hd = e->d.head_dim;
  const size_t plane = static_cast<size_t>(e->d.n_layers) * nkv * e->d.max_tokens * hd;
  const size_t off = (is_value ? plane : 0) +
                     ((static_cast<size_t>(layer) * nkv + g) * e->d.max_tokens + pos) * hd;
  CK(cudaMemcpy(out, e->kv + off, hd * 4, cudaMemcpyDeviceToHost));
  return C2S_OK;
}

int c2s_prefill_debug(const c2s_engine *e, int which, float *out, int n_floats) {
  if (!e || !out || n_floats < 0 || which < 0 || which > 1) return fail(C2S_ERR_ARG, "bad argument");
  if (!e->pf_att) return fail(C2S_ERR_STATE, "no tensor-core prefill has run on this engine");
  const int nqh = e->plan.world > 1 ? e->plan.h1 - e->plan.h0 : e->d.n_heads;
  if (static_cast<size_t>(n_floats) > static_cast<size_t>(e->pf_cap) * nqh * e->d.head_dim)
    return fail(C2S_ERR_ARG, "n_floats %d exceeds the prefill chunk's buffers", n_floats);
  DeviceGuard dg(e->device);
  CK(cudaStreamSynchronize(e->stream));
  CK(cudaMemcpy(out, which == 0 ? e->pf_att : e->pf_q, static_cast<size_t>(n_floats) * 4, cudaMemcpyDeviceToHost));
  return C2S_OK;
}

// ---------------------------------------------------------------------------
// prefill: chunks of up to pf_cap tokens through every layer together
// ---------------------------------------------------------------------------
static int pf_alloc(c2s_engine *e) {
  if (e->pf_cap) return C2S_OK;
  const c2s_model_desc &d = e->d;
  const TpPlan &pl = e->plan;
  const bool tp = pl.world > 1;
  // this rank's shard (the whole model on one GPU)
  const int nqh = tp ? pl.h1 - pl.h0 : d.n_heads, nkv = tp ? pl.g1 - pl.g0 : d.n_kv_heads;
  const int cap = 1024, H = d.embd, F = tp ? (pl.f1 - pl.f0) * 256 : d.ffn, nq = nqh * d.head_dim,
            kvd = nkv * d.head_dim;
  const int kmax = std::max(std::max(H, F), nq);
  auto al = [&](void **p, size_t bytes) -> int {
    if (cudaMalloc(p, bytes) != cudaSuccess) return fail(C2S_ERR_OOM, "prefill buffers: cudaMalloc(%zu) failed", bytes);
    return C2S_OK;
  };
  const size_t c = cap;
  int rc;
  if ((rc = al(reinterpret_cast<void **>(&e->pf_x), c * H * 4)) || (rc = al(reinterpret_cast<void **>(&e->pf_q), c * nq * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_k), c * kvd * 4)) || (rc = al(reinterpret_cast<void **>(&e->pf_v), c * kvd * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_att), c * nq * 4)) || (rc = al(reinterpret_cast<void **>(&e->pf_g), c * F * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_u), c * F * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_d8), c * (kmax / 256) * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_q8), c * kmax)) || (rc = al(reinterpret_cast<void **>(&e->pf_tok), c * 4)) ||
      (rc = al(reinterpret_cast<void **>(&e->pf_bs), c * (kmax / 256) * 16)))
    return rc;
  if (tp && (rc = al(reinterpret_cast<void **>(&e->pf_delta), c * H * 4))) return rc;
  // attention splits: keys of a query block in splits of pf_fsplit (a
  // multiple of both kernels' key tiles, at least 512: the 2048-token prefill
  // took 26.6 ms at 256, 25.2 at 384, 24.6-24.8 at 512, 26.5 at 768, 25.4 at
  // 1024), at most 16 per block at max_tokens
  {
    const int mt = d.max_tokens, hd = d.head_dim;
    e->pf_fsplit = std::max(4 * kFkN, ((mt + 15) / 16 + kFkN - 1) / kFkN * kFkN);
    e->pf_fns = (mt + e->pf_fsplit - 1) / e->pf_fsplit;
    const size_t nblk = (c * (d.n_heads / d.n_kv_heads) + kFqN - 1) / kFqN;
    const size_t blocks = static_cast<size_t>(nkv) * nblk;
    if ((rc = al(reinterpret_cast<void **>(&e->pf_fpart), blocks * e->pf_fns * kFqN * pf_part_width(hd) * 4)) ||
        (rc = al(reinterpret_cast<void **>(&e->pf_fcount), blocks * 4)))
      return rc;
    CK(cudaMemsetAsync(e->pf_fcount, 0, blocks * 4, e->stream));
    // K/V tiles of the tensor-core attention: one layer, every position
    e->pf_kvt_tpg = (mt + kTaK - 1) / kTaK;
    if ((rc = al(reinterpret_cast<void **>(&e->pf_kvt), static_cast<size_t>(nkv) * e->pf_kvt_tpg * ta_tile_bytes(hd))))
      return rc;
  }
  // the digit planes of every layer projection, converted once
  auto plane_bytes = [](int, int rows, int cols) {
    return static_cast<size_t>((rows + kPfM - 1) / kPfM) * (cols / 256) * 2 * kPfPlane;
  };
  auto info_bytes = [](int rows, int cols) {
    return static_cast<size_t>((rows + kPfM - 1) / kPfM) * kPfM * (cols / 256) * sizeof(uint4);
  };
  struct M { const uint8_t *w; int type, rows, cols; };
  std::vector<std::array<M, 7>> mats;
  size_t total = 0;
  for (int l = 0; l < d.n_layers; ++l) {
    const LayerDev &Ld = e->layers[l];
    std::array<M, 7> m = {M{Ld.q, Ld.tq, nq, H}, M{Ld.k, Ld.tk, kvd, H}, M{Ld.v, Ld.tv, kvd, H}, M{Ld.o, Ld.to, H, nq},
                          M{Ld.gate, Ld.tgate, F, H}, M{Ld.up, Ld.tup, F, H}, M{Ld.down, Ld.tdown, H, F}};
    for (auto &x : m) total += plane_bytes(x.type, x.rows, x.cols) + info_bytes(x.rows, x.cols);
    mats.push_back(m);
  }
  if ((rc = al(reinterpret_cast<void **>(&e->pf_planes), total))) return rc;
  e->pf_pl.assign(d.n_layers, {});
  e->pf_ri.assign(d.n_layers, {});
  CK(cudaMemsetAsync(e->pf_planes, 0, total, e->stream));
  size_t off = 0;
  for (int l = 0; l < d.n_layers; ++l)
    for (int i = 0; i < 7; ++i) {
      const M &x = mats[l][i];
      uint8_t *dst = e->pf_planes + off;
      uint4 *info = reinterpret_cast<uint4 *>(dst + plane_bytes(x.type, x.rows, x.cols));
      e->pf_pl[l][i] = dst;
      e->pf_ri[l][i] = info;
      const dim3 grid((x.rows + kPfM - 1) / kPfM, x.cols / 256);
      const int rb = static_cast<int>(row_bytes_of(x.type, x.cols));
      if (x.type == T_Q4_K)
        k_pf_planes<T_Q4_K><<<grid, 128, 0, e->stream>>>(x.w, x.rows, rb, x.cols / 256, dst, info);
      else
        k_pf_planes<T_Q6_K><<<grid, 128, 0, e->stream>>>(x.w, x.rows, rb, x.cols / 256, dst, info);
      CK(cudaGetLastError());
      off += plane_bytes(x.type, x.rows, x.cols) + info_bytes(x.rows, x.cols);
    }
  e->pf_cap = cap;
  e->pf_kmax = kmax;
  return C2S_OK;
}

// One K-quant GEMM of the chunk's n tokens (their Q8_K rows in pf_q8 /
// pf_d8): weight matrix `which` of layer l
struct PfJob {
  int which, type, rows, cols;
  float *out;
  int ldo, mode;
  const float *bias;
};

// The jobs of one weight type in one launch (none: nothing)
static int pf_gemm_type(c2s_engine *e, int l, int n, int type, std::initializer_list<PfJob> jobs) {
  PfGemmSet S{};
  int tiles = 0;
  for (const PfJob &j : jobs) {
    if (j.type != type) continue;
    PfGemm &G = S.g[S.n];
    G.planes = e->pf_pl[l][j.which];
    G.rowinfo = e->pf_ri[l][j.which];
    G.type = j.type;
    G.rows = j.rows;
    G.cols = j.cols;
    G.a = e->pf_q8;
    G.ad = e->pf_d8;
    G.abs = e->pf_bs;
    G.M = n;
    G.out = j.out;
    G.ldo = j.ldo;
    G.mode = j.mode;
    G.bias = j.bias;
    G.err = &e->st->err;
    S.tiles[S.n] = (j.rows + kPfM - 1) / kPfM;
    tiles += S.tiles[S.n++];
  }
  if (S.n == 0) return C2S_OK;
  const dim3 grid(tiles, (n + kPfN - 1) / kPfN);
  if (type == T_Q4_K)
    k_pf_gemm<T_Q4_K><<<grid, kPfThreads, kPfSmem, e->stream>>>(S);
  else
    k_pf_gemm<T_Q6_K><<<grid, kPfThreads, kPfSmem, e->stream>>>(S);
  CK(cudaGetLastError());
  return C2S_OK;
}

// Up to three GEMMs over the same tokens: one launch per weight type
static int pf_gemm(c2s_engine *e, int l, int n, std::initializer_list<PfJob> jobs) {
  if (jobs.size() > 3) return fail(C2S_ERR_ARG, "pf_gemm: more than three jobs");
  for (const int type : {T_Q4_K, T_Q6_K})
    if (int rc = pf_gemm_type(e, l, n, type, jobs)) return rc;
  return C2S_OK;
}

// n tokens at positions p0.. (p0 + n <= max_tokens): the forward of each, as
// engine.Forward per token would leave the KV cache, TokenIDs, SeqLen and
// the last NormX
static int pf_run(c2s_engine *e, int p0, const int32_t *tokens, int n) {
  const c2s_model_desc &d = e->d;
  const TpPlan &pl = e->plan;
  const bool tp = pl.world > 1;
  // this rank's shard (the whole model on one GPU): query heads, kv groups,
  // FFN rows; attn_output and ffn_down give partial rows, summed over the
  // ranks before the residual add
  const int H = d.embd, hd = d.head_dim, L = d.n_layers, qpk = d.n_heads / d.n_kv_heads;
  const int nqh = tp ? pl.h1 - pl.h0 : d.n_heads, nkv = tp ? pl.g1 - pl.g0 : d.n_kv_heads;
  const int F = tp ? (pl.f1 - pl.f0) * 256 : d.ffn;
  const int nq = nqh * hd, kvd = nkv * hd;
  const NcclApi *nc = nullptr;
  if (tp)
    if (int rc = nccl_api(&nc)) return rc;
  // tensor parallel: out = the chunk's partial rows -> allreduce -> x += out
  auto reduce_add = [&]() -> int {
    const size_t cnt = static_cast<size_t>(n) * H;
    const ncclResult_t r = nc->all_reduce(e->pf_delta, e->pf_delta, cnt, ncclFloat32, ncclSum, e->comm, e->stream);
    if (r != ncclSuccess) return fail(C2S_ERR_CUDA, "prefill ncclAllReduce: %s", nc->err_str(r));
    k_pf_add<<<e->num_sms * 4, kThreads, 0, e->stream>>>(e->pf_x, e->pf_delta, cnt);
    CK(cudaGetLastError());
    return C2S_OK;
  };

  const size_t head_stride = static_cast<size_t>(d.max_tokens) * hd;
  const size_t plane = static_cast<size_t>(L) * nkv * head_stride;
  cudaStream_t s = e->stream;
  CK(cudaMemcpyAsync(e->pf_tok, tokens, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, s));
  k_pf_embed<<<n, kThreads, 0, s>>>(e->pf_tok, n, d.vocab, e->tok_type, e->tok_embd,
                                     static_cast<int>(row_bytes_of(e->tok_type, H)), e->pf_x, H);
  CK(cudaGetLastError());
  for (int l = 0; l < L; ++l) {
    const LayerDev &Ld = e->layers[l];
    k_pf_norm_q8k<<<n, kThreads, 0, s>>>(e->pf_x, H, Ld.attn_norm, d.eps, H, n, e->pf_q8, e->pf_d8, e->pf_bs, nullptr);
    int rc;
    if ((rc = pf_gemm(e, l, n,
                      {{0, Ld.tq, nq, H, e->pf_q, nq, PF_STORE, Ld.qb}, {1, Ld.tk, kvd, H, e->pf_k, kvd, PF_STORE, Ld.kb},
                       {2, Ld.tv, kvd, H, e->pf_v, kvd, PF_STORE, Ld.vb}})))
      return rc;
    float *kc = e->kv + static_cast<size_t>(l) * nkv * head_stride, *vc = kc + plane;
    k_pf_rope_store<<<n, kThreads, static_cast<size_t>(nqh + nkv) * hd * 4, s>>>(
        e->pf_q, e->pf_k, e->pf_v, nq, kvd, n, p0, nqh, nkv, hd, e->rope_cos, e->rope_sin, kMaxContext, Ld.qn, Ld.kn,
        d.eps, kc, vc, head_stride);
    PfFlash A{};
    A.q = e->pf_q;
    A.out = e->pf_att;
    A.kc = kc;
    A.vc = vc;
    A.head_stride = head_stride;
    A.ldq = nq;
    A.n = n;
    A.p0 = p0;
    A.qpk = qpk;
    A.n_heads = nqh;
    A.hbase = tp ? pl.h0 : 0;
    A.gbase = tp ? pl.g0 : 0;
    A.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(hd)));  // engine/forward.go:59
    A.part = e->pf_fpart;
    A.count = e->pf_fcount;
    A.split_keys = e->pf_fsplit;
    A.max_splits = e->pf_fns;
    A.tiles = e->pf_kvt;
    A.tiles_per_group = e->pf_kvt_tpg;
    A.err = &e->st->err;
    const dim3 fgrid(nkv, (n * qpk + kFqN - 1) / kFqN, (p0 + n + e->pf_fsplit - 1) / e->pf_fsplit);
    if (e->pf_attn_fp32) {
      if (hd == 128)
        k_pf_flash<128><<<fgrid, kThreads, pf_flash_smem(128), s>>>(A);
      else
        k_pf_flash<64><<<fgrid, kThreads, pf_flash_smem(64), s>>>(A);
    } else {
      const dim3 tgrid((p0 + n + kTaK - 1) / kTaK, nkv);
      if (hd == 128) {
        k_pf_kv_tiles<128><<<tgrid, 256, 0, s>>>(kc, vc, head_stride, p0 + n, e->pf_kvt, e->pf_kvt_tpg);
        k_pf_attn<128><<<fgrid, kTaThreads, ta_smem(128), s>>>(A);
      } else {
        k_pf_kv_tiles<64><<<tgrid, 256, 0, s>>>(kc, vc, head_stride, p0 + n, e->pf_kvt, e->pf_kvt_tpg);
        k_pf_attn<64><<<fgrid, kTaThreads, ta_smem(64), s>>>(A);
      }
    }
    CK(cudaGetLastError());
    k_pf_norm_q8k<<<n, kThreads, 0, s>>>(e->pf_att, nq, nullptr, 0.f, nq, n, e->pf_q8, e->pf_d8, e->pf_bs, nullptr);
    if (tp) {
      if ((rc = pf_gemm(e, l, n, {{3, Ld.to, H, nq, e->pf_delta, H, PF_STORE, nullptr}})) || (rc = reduce_add()))
        return rc;
    } else if ((rc = pf_gemm(e, l, n, {{3, Ld.to, H, nq, e->pf_x, H, PF_ADD, nullptr}}))) {
      return rc;
    }
    k_pf_norm_q8k<<<n, kThreads, 0, s>>>(e->pf_x, H, Ld.ffn_norm, d.eps, H, n, e->pf_q8, e->pf_d8, e->pf_bs, nullptr);
    if ((rc = pf_gemm(e, l, n,
                      {{4, Ld.tgate, F, H, e->pf_g, F, PF_STORE, nullptr}, {5, Ld.tup, F, H, e->pf_u, F, PF_STORE, nullptr}})))
      return rc;
    // SwiGLU(gate, up) quantised straight into the down projection's token tiles
    k_pf_norm_q8k<<<n, kThreads, 0, s>>>(e->pf_g, F, nullptr, 0.f, F, n, e->pf_q8, e->pf_d8, e->pf_bs, nullptr,
                                         e->pf_u);
    if (tp) {
      if ((rc = pf_gemm(e, l, n, {{6, Ld.tdown, H, F, e->pf_delta, H, PF_STORE, nullptr}})) || (rc = reduce_add()))
        return rc;
    } else if ((rc = pf_gemm(e, l, n, {{6, Ld.tdown, H, F, e->pf_x, H, PF_ADD, nullptr}}))) {
      return rc;
    }
    CK(cudaGetLastError());
  }
  // the last token's residual stream (read by a following ComputeLogits /
  // generate step) and its NormX (engine/forward.go:133-137)
  CK(cudaMemcpyAsync(e->X, e->pf_x + static_cast<size_t>(n - 1) * H, static_cast<size_t>(H) * 4,
                     cudaMemcpyDeviceToDevice, s));
  k_pf_norm_q8k<<<1, kThreads, 0, s>>>(e->pf_x + static_cast<size_t>(n - 1) * H, H, e->out_norm, d.eps, H, 1,
                                       e->pf_q8, e->pf_d8, e->pf_bs, e->normx);
  k_pf_commit<<<1, kThreads, 0, s>>>(e->st, e->token_ids, e->pf_tok, n, p0, d.max_tokens);
  CK(cudaGetLastError());
  return C2S_OK;
}

int c2s_ingest_from(c2s_engine *e, int pos, const int32_t *tokens, int n, float *last_normx_out) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (n <= 0) return 0;
  if (!tokens) return fail(C2S_ERR_ARG, "null tokens");
  DeviceGuard g(e->device);
  // c2slm.go:96-104: clamp into [0, SeqLen] and rewind in place
  if (pos < 0) pos = 0;
  if (pos > e->host_seq) pos = e->host_seq;
  if (pos < e->host_seq)
    if (int rc = c2s_kv_set_seq_len(e, pos)) return rc;
  int done = 0;
  if (e->pf_ok && n > 1) {  // the tensor-core prefill, chunk by chunk
    if (int rc = pf_alloc(e)) return rc;
    const int total = std::min(n, e->d.max_tokens - pos);
    for (int c0 = 0; c0 < total; c0 += e->pf_cap) {
      const int m = std::min(e->pf_cap, total - c0);
      if (int rc = pf_run(e, pos + c0, tokens + c0, m)) return rc;
      done += m;
    }
  } else {
    for (int i = 0; i < n; ++i) {
      const int p = pos + i;
      if (p >= e->d.max_tokens) break;
      if (int rc = set_fwd_input(e, tokens[i], p, 1)) return rc;
      CK(cudaGraphLaunch(e->g_forward, e->stream));
      ++done;
    }
  }
  if (done > 0 && last_normx_out)
    CK(cudaMemcpyAsync(e->h_buf, e->normx, e->d.embd * 4, cudaMemcpyDeviceToHost, e->stream));
  if (int rc = read_status(e)) return rc;
  if (done > 0 && last_normx_out) memcpy(last_normx_out, e->h_buf, e->d.embd * 4);
  return done;
}

static int set_gen_state(c2s_engine *e, float penalty, int window, int stop_on_special) {
  // halted, halt_pending, stop_on_special, window, penalty, n_out (contiguous)
  DevState *h = e->h_st;
  h->halted = 0;
  h->halt_pending = 0;
  h->stop_on_special = stop_on_special ? 1 : 0;
  h->window = window;
  h->penalty = penalty;
  h->n_out = 0;
  const size_t off = offsetof(DevState, halted);
  const size_t len = offsetof(DevState, out_cap) - off;
  CK(cudaMemcpyAsync(reinterpret_cast<uint8_t *>(e->st) + off, reinterpret_cast<uint8_t *>(h) + off, len,
                     cudaMemcpyHostToDevice, e->stream));
  return C2S_OK;
}

int c2s_generate(c2s_engine *e, int max_new, float penalty, int window, int stop_on_special, int32_t *tokens_out,
                 int *n_out) {
  if (!e || !n_out) return fail(C2S_ERR_ARG, "null argument");
  if (max_new > 0 && !tokens_out) return fail(C2S_ERR_ARG, "null tokens_out");
  if (window < 0) return fail(C2S_ERR_ARG, "window < 0");
  *n_out = 0;
  DeviceGuard g(e->device);
  // c2slm.go:78-80 / 149-151: never past the KV capacity
  const int remaining = e->d.max_tokens - e->host_seq;
  if (max_new > remaining) max_new = remaining;
  if (max_new <= 0) return C2S_OK;
  if (e->host_seq <= 0) return fail(C2S_ERR_STATE, "generate needs a forwarded prefix (SeqLen == 0)");
  if (int rc = set_gen_state(e, penalty, window, stop_on_special)) return rc;
  if (e->use_persistent) {
    if (int rc = launch_persistent(e, max_new, 0, 0)) return rc;
  } else {
    for (int i = 0; i < max_new; ++i) CK(cudaGraphLaunch(e->g_step, e->stream));
  }
  CK(cudaMemcpyAsync(e->h_tokens, e->out_tokens, static_cast<size_t>(max_new) * 4, cudaMemcpyDeviceToHost,
                     e->stream));
  if (int rc = read_status(e)) return rc;
  const int n = std::min(e->h_st->n_out, max_new);
  memcpy(tokens_out, e->h_tokens, static_cast<size_t>(n) * 4);
  *n_out = n;
  return C2S_OK;
}

int c2s_decode_step(c2s_engine *e, int32_t token, float penalty, int window, int32_t *next_out) {
  if (!e || !next_out) return fail(C2S_ERR_ARG, "null argument");
  if (e->host_seq >= e->d.max_tokens) return fail(C2S_ERR_STATE, "KV cache full");
  DeviceGuard g(e->device);
  if (int rc = set_gen_state(e, penalty, window, 0)) return rc;
  if (int rc = set_fwd_input(e, token, e->host_seq, 1)) return rc;
  if (e->use_persistent) {  // forward of `token`, then logits + selection
    if (int rc = launch_persistent(e, 1, 0, 0, nullptr, 1)) return rc;
  } else {
    CK(cudaGraphLaunch(e->g_fwd_select, e->stream));
  }
  CK(cudaMemcpyAsync(e->h_tokens, e->out_tokens, 4, cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  *next_out = e->h_tokens[0];
  e->host_seq += 1;
  return C2S_OK;
}

int c2s_engine_sync(c2s_engine *e) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  DeviceGuard g(e->device);
  return read_status(e);
}

int c2s_bench_decode(c2s_engine *e, int n_steps, float penalty, int window) {
  if (!e) return fail(C2S_ERR_ARG, "null engine");
  if (n_steps > e->d.max_tokens - e->host_seq) return fail(C2S_ERR_ARG, "n_steps exceeds KV capacity");
  DeviceGuard g(e->device);
  if (int rc = set_gen_state(e, penalty, window, 0)) return rc;
  if (e->use_persistent) {
    if (int rc = launch_persistent(e, n_steps, 0, 0)) return rc;
  } else {
    for (int i = 0; i < n_steps; ++i) CK(cudaGraphLaunch(e->g_step, e->stream));
  }
  e->host_seq += n_steps;  // confirmed by the next read_status
  return C2S_OK;
}

int c2s_kernels_per_step(const c2s_engine *e) { return e ? e->kernels_per_step : 0; }

int c2s_decode_launches(const c2s_engine *e, int n_steps) {
  if (!e || n_steps <= 0) return 0;
  return e->use_persistent ? 1 : e->kernels_per_step * n_steps;
}

int c2s_bench_decode_timed(c2s_engine *e, int n_steps, float penalty, int window, int period, float *ms_out) {
  if (!e || !ms_out) return fail(C2S_ERR_ARG, "null argument");
  const int span = period > 0 ? std::min(period, n_steps) : n_steps;
  if (n_steps <= 0 || span > e->d.max_tokens - e->host_seq) return fail(C2S_ERR_ARG, "n_steps out of range");
  DeviceGuard g(e->device);
  if (int rc = set_gen_state(e, penalty, window, 0)) return rc;
  // every `period` steps SeqLen is rewound to its value at entry (KVCache.Rewind:
  // no copy), so the decoded positions stay in [base, base + period)
  e->h_st->fwd_token = e->host_seq;  // pinned source for the rewinds
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  CK(cudaEventRecord(a, e->stream));
  if (e->use_persistent) {
    if (int rc = launch_persistent(e, n_steps, period, e->host_seq)) return rc;
  } else {
    for (int i = 0; i < n_steps; ++i) {
      if (period > 0 && i > 0 && i % period == 0)
        CK(cudaMemcpyAsync(&e->st->seq_len, &e->h_st->fwd_token, sizeof(int), cudaMemcpyHostToDevice, e->stream));
      CK(cudaGraphLaunch(e->g_step, e->stream));
    }
  }
  CK(cudaEventRecord(b, e->stream));
  CK(cudaEventSynchronize(b));
  CK(cudaEventElapsedTime(ms_out, a, b));
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return read_status(e);
}

int c2s_trace_decode(c2s_engine *e, int n_steps, float penalty, int window, uint64_t *trace_out, int *nphase_out) {
  if (!e || !trace_out || !nphase_out) return fail(C2S_ERR_ARG, "null argument");
  if (!e->use_persistent) return fail(C2S_ERR_STATE, "persistent decode kernel not in use");
  if (n_steps <= 0 || n_steps > e->d.max_tokens - e->host_seq) return fail(C2S_ERR_ARG, "n_steps out of range");
  DeviceGuard g(e->device);
  if (int rc = set_gen_state(e, penalty, window, 0)) return rc;
  const size_t n = static_cast<size_t>(n_steps) * e->nphase * e->num_sms * c2s::kTraceFields;
  unsigned long long *dtr = nullptr;
  CK(cudaMalloc(&dtr, n * 8));
  CK(cudaMemsetAsync(dtr, 0, n * 8, e->stream));
  int rc = launch_persistent(e, n_steps, 0, 0, dtr);
  if (rc == C2S_OK) {
    cudaMemcpyAsync(trace_out, dtr, n * 8, cudaMemcpyDeviceToHost, e->stream);
    rc = read_status(e);
  }
  cudaFree(dtr);
  *nphase_out = e->nphase;
  return rc;
}

int c2s_profile_step(c2s_engine *e, int n_steps, float penalty, int window, float *stage_ms, int *stage_launches) {
  if (!e || !stage_ms || !stage_launches) return fail(C2S_ERR_ARG, "null argument");
  if (n_steps <= 0 || n_steps > e->d.max_tokens - e->host_seq) return fail(C2S_ERR_ARG, "n_steps out of range");
  DeviceGuard g(e->device);
  if (int rc = set_gen_state(e, penalty, window, 0)) return rc;
  std::vector<cudaEvent_t> ev;
  std::vector<int> kind;
  KTimer tm{&ev, &kind};
  cudaError_t err = cudaSuccess;
  for (int i = 0; i < n_steps && !err; ++i) {
    err = enqueue_logits(e, e->stream, true, false, true, &tm);
    if (!err) err = enqueue_forward(e, e->stream, true, false, &tm);
  }
  if (err) return fail(C2S_ERR_CUDA, "profile launch: %s", cudaGetErrorString(err));
  CK(cudaStreamSynchronize(e->stream));
  for (int k = 0; k < 8; ++k) {
    stage_ms[k] = 0.f;
    stage_launches[k] = 0;
  }
  for (size_t i = 0; i < kind.size(); ++i) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, ev[2 * i], ev[2 * i + 1]));
    stage_ms[kind[i]] += ms;
    stage_launches[kind[i]] += 1;
  }
  for (auto x : ev) cudaEventDestroy(x);
  return read_status(e);
}

int c2s_ring_groups(int nslot, int lng) { return ring_groups_log2(nslot, lng); }

// ---- op-level entry points ------------------------------------------------
int c2s_quantize_row_q8_k(const float *x, uint8_t *y, int cols) {
  if (!x || !y) return fail(C2S_ERR_ARG, "null argument");
  if (cols <= 0 || cols % 256) return fail(C2S_ERR_ARG, "cols must be a positive multiple of 256");
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  DevBuf<float> dx;
  DevBuf<uint8_t> dy;
  const size_t ybytes = static_cast<size_t>(cols / 256) * 292;
  if (int rc = dx.alloc(cols, c->stream)) return rc;
  if (int rc = dy.alloc(ybytes, c->stream)) return rc;
  CK(cudaMemcpyAsync(dx.p, x, cols * 4, cudaMemcpyHostToDevice, c->stream));
  const int nsb = cols / 256;
  k_quantize_q8k<<<(nsb + kWarps - 1) / kWarps, kThreads, 0, c->stream>>>(dx.p, dy.p, cols);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(y, dy.p, ybytes, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

int c2s_gemv(int type, const void *weight, const float *x, float *y, int rows, int cols) {
  if (!weight || !x || !y) return fail(C2S_ERR_ARG, "null argument");
  if (int rc = check_matrix(type, rows, cols, "gemv")) return rc;
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  const size_t wb = row_bytes_of(type, cols) * rows;
  DevBuf<uint8_t> dw;
  DevBuf<float> dx, dy;
  if (int rc = dw.alloc(wb, c->stream)) return rc;
  if (int rc = dx.alloc(cols, c->stream)) return rc;
  if (int rc = dy.alloc(rows, c->stream)) return rc;
  CK(cudaMemcpyAsync(dw.p, weight, wb, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(dx.p, x, static_cast<size_t>(cols) * 4, cudaMemcpyHostToDevice, c->stream));
  if (int rc = gemv_launch(c, type, dw.p, dx.p, dy.p, rows, cols, nullptr)) return rc;
  CK(cudaMemcpyAsync(y, dy.p, static_cast<size_t>(rows) * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

// ---------------------------------------------------------------------------
// c2s_gemv_noalloc: c2s_gemv with every device byte it touches in one
// file-scope array.  Some callers cannot allocate device memory at the
// moment they need a matvec: a host whose free HBM is held by another
// allocator (a framework's caching pool) gets out-of-memory from cudaMalloc
// although nothing is in use, and a latency-critical loop cannot afford the
// device-wide synchronisation that cudaFree performs.  This entry point makes
// neither call: it stages the operands in kNoAllocScratchBytes of statically
// reserved device memory, runs the same kernel as c2s_gemv on the calling
// thread's default stream, and copies y back.
//
//   - The first call on a device does the set-up (it looks up the array's
//     device address, which may load this library's device code onto that
//     device); make that first call before any stream capture.
//   - Weights + x + y + 1.5 KB must fit in the array (4 MiB); larger calls are
//     rejected with C2S_ERR_ARG before any device work.
//   - The array starts with the kernel's status block (a DevState, padded to
//     a 256-byte boundary), whose error word must be zero when a call
//     starts: it is zero when the library loads, and a call that finds it
//     set clears it before returning.
//     Nothing else needs an initial value (each call writes x and the
//     weights before the kernel reads them).
//   - All calls on one device share the array: calls that overlap in time
//     (from several host threads) race on it and must be serialised by the
//     caller.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
// the status block must stay small next to the array (x starts after it)
static_assert(sizeof(DevState) <= 512, "c2s_gemv_noalloc: status block outgrew its reservation");
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static uint8_t *g_noalloc_base[64];  // device address of the array, per device (set-up done)
static std::mutex g_noalloc_mu;

int c2s_gemv_device(int device, int type, const void *d_weight, const float *d_x, float *d_y, int rows, int cols) {
  if (!d_weight || !d_x || !d_y) return fail(C2S_ERR_ARG, "null argument");
  if (reinterpret_cast<uintptr_t>(d_weight) & 255) return fail(C2S_ERR_ARG, "d_weight must be 256-byte aligned");
  OpCtx *c;
  if (int rc = op_ctx(device, &c)) return rc;
  DeviceGuard g(device);
  return gemv_launch(c, type, d_weight, d_x, d_y, rows, cols, nullptr);
}

int c2s_bench_gemv(int device, int type, const void *d_weight, size_t copy_stride, int n_copies, const float *d_x,
                   float *d_y, int rows, int cols, int reps, float *ms_out) {
  if (!d_weight || !d_x || !d_y || !ms_out) return fail(C2S_ERR_ARG, "null argument");
  if (n_copies < 1 || reps < 1) return fail(C2S_ERR_ARG, "n_copies and reps must be positive");
  if (reps % 1000 && reps > 4000) return fail(C2S_ERR_ARG, "reps must be a multiple of 1000 or at most 4000");
  if (n_copies > 1 && (copy_stride & 255)) return fail(C2S_ERR_ARG, "copy_stride must be a multiple of 256");
  if (reinterpret_cast<uintptr_t>(d_weight) & 255) return fail(C2S_ERR_ARG, "d_weight must be 256-byte aligned");
  if (int rc = check_matrix(type, rows, cols, "bench_gemv")) return rc;
  OpCtx *c;
  if (int rc = op_ctx(device, &c)) return rc;
  DeviceGuard g(device);
  const int per = reps % 1000 == 0 ? 1000 : reps, replays = reps / per;
  const uint8_t *w0 = static_cast<const uint8_t *>(d_weight);
  // one graph of `per` launches, launch i on copy i % n_copies
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int rc = C2S_OK;
  for (int i = 0; i < per && rc == C2S_OK; ++i)
    rc = gemv_launch(c, type, w0 + static_cast<size_t>(i % n_copies) * copy_stride, d_x, d_y, rows, cols, nullptr);
  const cudaError_t ec = cudaStreamEndCapture(c->stream, &graph);
  if (rc) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (ec != cudaSuccess) return fail(C2S_ERR_CUDA, "bench_gemv capture: %s", cudaGetErrorString(ec));
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) return fail(C2S_ERR_CUDA, "bench_gemv instantiate: %s", cudaGetErrorString(ei));
  cudaEvent_t a, b;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&b));
  cudaError_t er = cudaGraphLaunch(exec, c->stream);  // warm-up
  if (!er) er = cudaEventRecord(a, c->stream);
  for (int r = 0; r < replays && !er; ++r) er = cudaGraphLaunch(exec, c->stream);
  if (!er) er = cudaEventRecord(b, c->stream);
  if (!er) er = cudaEventSynchronize(b);
  if (!er) er = cudaEventElapsedTime(ms_out, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaGraphExecDestroy(exec);
  if (er) return fail(C2S_ERR_CUDA, "bench_gemv: %s", cudaGetErrorString(er));
  return op_finish(c);
}

int c2s_gemv_noalloc(int type, const void *weight, const float *x, float *y, int rows, int cols) {
  if (!weight || !x || !y) return fail(C2S_ERR_ARG, "null argument");
  if (int rc = check_matrix(type, rows, cols, "gemv_noalloc")) return rc;
  auto a256 = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t wb = row_bytes_of(type, cols) * rows;
  // [status block | x | y | weights], each 256-byte aligned, 64 B of slack after each
  const size_t off_x = a256(sizeof(DevState)), off_y = off_x + a256(static_cast<size_t>(cols) * 4 + 64);
  const size_t off_w = off_y + a256(static_cast<size_t>(rows) * 4 + 64);
  const size_t need = off_w + a256(wb + 64);
  if (need > kNoAllocScratchBytes)
    return fail(C2S_ERR_ARG, "gemv_noalloc: needs %zu bytes of scratch (weights %zu), the static scratch holds %zu",
                need, wb, kNoAllocScratchBytes);
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return fail(C2S_ERR_CUDA, "gemv_noalloc: no current CUDA device");
  uint8_t *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {  // set-up, once per device, with that device current
      void *p = nullptr;
      const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (rc != cudaSuccess)
        return fail(C2S_ERR_CUDA, "gemv_noalloc set-up: cudaGetSymbolAddress: %s", cudaGetErrorString(rc));
      CK(cudaFuncSetAttribute(k_matvec, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      g_noalloc_base[dev] = static_cast<uint8_t *>(p);
    }
    base = g_noalloc_base[dev];
  }
  OpCtx c;  // no stream or status block is created: both come from the caller / the array
  c.stream = cudaStreamPerThread;
  c.st = reinterpret_cast<DevState *>(base);
  CK(cudaMemcpyAsync(base + off_w, weight, wb, cudaMemcpyHostToDevice, c.stream));
  CK(cudaMemcpyAsync(base + off_x, x, static_cast<size_t>(cols) * 4, cudaMemcpyHostToDevice, c.stream));
  if (int rc = gemv_launch(&c, type, base + off_w, reinterpret_cast<const float *>(base + off_x),
                           reinterpret_cast<float *>(base + off_y), rows, cols, nullptr))
    return rc;
  CK(cudaMemcpyAsync(y, base + off_y, static_cast<size_t>(rows) * 4, cudaMemcpyDeviceToHost, c.stream));
  unsigned err = 0;
  CK(cudaMemcpyAsync(&err, &c.st->err, sizeof err, cudaMemcpyDeviceToHost, c.stream));
  CK(cudaStreamSynchronize(c.stream));
  if (err) {
    CK(cudaMemsetAsync(&c.st->err, 0, sizeof(unsigned), c.stream));
    CK(cudaStreamSynchronize(c.stream));
    return fail(C2S_ERR_TIMEOUT, "gemv_noalloc: device reported error flags 0x%x", err);
  }
  return C2S_OK;
}

int c2s_kquant_partials(int type, const void *weight, const float *x, int32_t *dots, int rows, int cols) {
  if (!weight || !x || !dots) return fail(C2S_ERR_ARG, "null argument");
  if (!is_kquant(type)) return fail(C2S_ERR_ARG, "partials exist for Q4_K and Q6_K only");
  if (int rc = check_matrix(type, rows, cols, "partials")) return rc;
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  const size_t wb = row_bytes_of(type, cols) * rows;
  const size_t nd = static_cast<size_t>(rows) * (cols / 256) * (type == T_Q4_K ? 8 : 1);
  DevBuf<uint8_t> dw;
  DevBuf<float> dx, dy;
  DevBuf<int32_t> dd;
  if (int rc = dw.alloc(wb, c->stream)) return rc;
  if (int rc = dx.alloc(cols, c->stream)) return rc;
  if (int rc = dy.alloc(rows, c->stream)) return rc;
  if (int rc = dd.alloc(nd, c->stream)) return rc;
  CK(cudaMemcpyAsync(dw.p, weight, wb, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(dx.p, x, static_cast<size_t>(cols) * 4, cudaMemcpyHostToDevice, c->stream));
  if (int rc = gemv_launch(c, type, dw.p, dx.p, dy.p, rows, cols, dd.p)) return rc;
  CK(cudaMemcpyAsync(dots, dd.p, nd * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

int c2s_dot_rows_f32x(int type, const void *weight, const float *x, const int32_t *rows_idx, int n, float *out,
                      int rows, int cols) {
  if (!weight || !x || !rows_idx || !out) return fail(C2S_ERR_ARG, "null argument");
  if (int rc = check_matrix(type, rows, cols, "dot_rows")) return rc;
  if (n <= 0) return C2S_OK;
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  const size_t wb = row_bytes_of(type, cols) * rows;
  DevBuf<uint8_t> dw;
  DevBuf<float> dx, dout;
  DevBuf<int> di;
  if (int rc = dw.alloc(wb, c->stream)) return rc;
  if (int rc = dx.alloc(cols, c->stream)) return rc;
  if (int rc = dout.alloc(n, c->stream)) return rc;
  if (int rc = di.alloc(n, c->stream)) return rc;
  CK(cudaMemcpyAsync(dw.p, weight, wb, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(dx.p, x, static_cast<size_t>(cols) * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(di.p, rows_idx, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, c->stream));
  k_dot_rows_f32x<<<n, kThreads, 0, c->stream>>>(type, dw.p, static_cast<int>(row_bytes_of(type, cols)), dx.p, di.p,
                                                  n, dout.p, rows, cols);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(out, dout.p, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

int c2s_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
  if (!out || !x || !w || n <= 0) return fail(C2S_ERR_ARG, "bad argument");
  if (n > 48 * 1024) return fail(C2S_ERR_ARG, "n too large");
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  DevBuf<float> dx, dw, dout;
  if (int rc = dx.alloc(n, c->stream)) return rc;
  if (int rc = dw.alloc(n, c->stream)) return rc;
  if (int rc = dout.alloc(n, c->stream)) return rc;
  CK(cudaMemcpyAsync(dx.p, x, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(dw.p, w, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaFuncSetAttribute(k_rmsnorm_op, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  k_rmsnorm_op<<<1, kThreads, static_cast<size_t>(n) * 4, c->stream>>>(dout.p, dx.p, dw.p, n, eps);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(out, dout.p, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

int c2s_swiglu(float *out, const float *gate, const float *up, int n) {
  if (!out || !gate || !up || n <= 0) return fail(C2S_ERR_ARG, "bad argument");
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  DevBuf<float> dg, du, dout;
  if (int rc = dg.alloc(n, c->stream)) return rc;
  if (int rc = du.alloc(n, c->stream)) return rc;
  if (int rc = dout.alloc(n, c->stream)) return rc;
  CK(cudaMemcpyAsync(dg.p, gate, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, c->stream));
  CK(cudaMemcpyAsync(du.p, up, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, c->stream));
  k_swiglu_op<<<(n + 255) / 256, 256, 0, c->stream>>>(dout.p, dg.p, du.p, n);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(out, dout.p, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

int c2s_dequant_row(int type, const void *row, float *out, int cols) {
  if (!row || !out || cols <= 0) return fail(C2S_ERR_ARG, "bad argument");
  const size_t rb = row_bytes_of(type, cols);
  if (!rb) return fail(C2S_ERR_UNSUPPORTED, "type %d", type);
  OpCtx *c;
  if (int rc = op_ctx(current_device(), &c)) return rc;
  DevBuf<uint8_t> dr;
  DevBuf<float> dout;
  if (int rc = dr.alloc(rb, c->stream)) return rc;
  if (int rc = dout.alloc(cols, c->stream)) return rc;
  CK(cudaMemcpyAsync(dr.p, row, rb, cudaMemcpyHostToDevice, c->stream));
  k_dequant_op<<<1, kThreads, 0, c->stream>>>(type, dr.p, dout.p, cols);
  CK(cudaGetLastError());
  CK(cudaMemcpyAsync(out, dout.p, static_cast<size_t>(cols) * 4, cudaMemcpyDeviceToHost, c->stream));
  return op_finish(c);
}

}  // extern "C"
