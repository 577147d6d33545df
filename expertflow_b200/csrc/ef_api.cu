// ef_api.cu -- host side of the C ABI declared in include/efmoe.h.
//
// Validates arguments, lays out the caller's workspace, encodes the TMA tensor
// maps of the weight stacks and enqueues the kernel sequence on the caller's
// stream:  router logits -> top-k -> permute -> activation prep -> gate/up
// (+SwiGLU) -> down -> combine.  Nothing here allocates device memory.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/efmoe.h"
#include "ef_common.cuh"

namespace ef {
cudaError_t launch_router_logits(const uint16_t* x, int x_bf16, const uint16_t* wg, int w_bf16, int T, int E, int H,
                                 float* logits, cudaStream_t st,
                                 const uint16_t* wg2 = nullptr, float* logits2 = nullptr,
                                 const uint16_t* wg3 = nullptr, float* logits3 = nullptr);
cudaError_t launch_router_select(const float* logits, const float* e_bias, int T, int E, int k, int mode,
                                 int norm_topk, int n_group, int topk_group, float scaling, int* inds, float* wts,
                                 cudaStream_t st,
                                 const float* logits2 = nullptr, const float* e_bias2 = nullptr,
                                 int* inds2 = nullptr, float* wts2 = nullptr, const float* logits3 = nullptr,
                                 const float* e_bias3 = nullptr, int* inds3 = nullptr, float* wts3 = nullptr);
cudaError_t launch_permute(const int* entries, int n_ent, int k, int n_exp, int n_sh, int seg_chunk,
                           const PermBufs& pb, cudaStream_t st);
cudaError_t launch_prep_act(const uint16_t* act, const int* row_src, int is_bf16, int n, int K, int bits,
                            uint16_t* out, float* sums, cudaStream_t st, const int* n_dev = nullptr,
                            int max_blocks = 0);
cudaError_t launch_combine(const float* rows, const int* inv, const float* wts, int T, int k, int H, int sh_base,
                           void* out, int out_dtype, cudaStream_t st, const uint32_t* wait_flags = nullptr,
                           int n_wait = 0, const uint32_t* epoch = nullptr);
cudaError_t launch_qmv(int bits, int mode, const QmvParams& p, int n_sm, cudaStream_t st, int min_segments = 0);
size_t qmv_smem_required(int bits, int mode, int K);
cudaError_t launch_qgemm(int bits, int mode, const GemmParams& p, int n_sm, cudaStream_t st);
cudaError_t launch_qgemm2(int bits, int mode, const GemmParams& p, int n_sm, cudaStream_t st);
size_t qgemm_smem_required(int bits);
cudaError_t launch_dequantize(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int cols, int bits,
                              void* out, int out_dtype, cudaStream_t st);
}  // namespace ef

using namespace ef;

namespace {

thread_local std::string g_last_msg;

ef_status fail(ef_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_msg = buf;
  return s;
}

#define EF_LAUNCH(name, call)                                                               \
  do {                                                                                      \
    TraceScope _ts(st, name);                                                               \
    cudaError_t _e = (call);                                                                \
    if (_e != cudaSuccess) return fail(EF_ERR_CUDA, "%s: %s", name, cudaGetErrorString(_e)); \
  } while (0)

#define EF_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t _e = (call);                                                                  \
    if (_e != cudaSuccess) return fail(EF_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e)); \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- tracing: CUDA events around each launch (off by default)
struct TraceRec {
  const char* name;
  cudaEvent_t a, b;
};
std::mutex g_trace_mu;
bool g_trace_on = false;
std::vector<TraceRec> g_trace;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t trace_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

struct TraceScope {
  cudaStream_t st;
  TraceRec rec{nullptr, nullptr, nullptr};
  TraceScope(cudaStream_t s, const char* name) : st(s) {
    if (!g_trace_on) return;
    std::lock_guard<std::mutex> lk(g_trace_mu);
    rec = {name, trace_event(), trace_event()};
    cudaEventRecord(rec.a, st);
  }
  ~TraceScope() {
    if (!rec.name) return;
    cudaEventRecord(rec.b, st);
    std::lock_guard<std::mutex> lk(g_trace_mu);
    g_trace.push_back(rec);
  }
};

// ---- tensor-map encoder from the driver (no link-time libcuda dependency)
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t get_encoder() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

// A tensor map depends only on (base, shape, box, swizzle), which repeat call
// after call for a layer's weights and workspaces, while an encode costs
// microseconds of host time: a small per-thread cache of encoded 2-D maps keeps
// the encodes off the launch path.
static CUresult encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, const cuuint64_t* dims,
                          const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw,
                          CUtensorMapL2promotion l2) {
  struct Entry {
    CUtensorMap map;
    const void* base;
    cuuint64_t d0, d1, s0;
    cuuint32_t b0, b1;
    int dt, sw, l2;
    bool valid;
  };
  static thread_local Entry cache[256];
  uint64_t h = reinterpret_cast<uintptr_t>(base) * 0x9E3779B97F4A7C15ull;
  h ^= (dims[0] * 0x100000001B3ull) ^ (dims[1] * 0xC2B2AE3D27D4EB4Full) ^ ((uint64_t)box[1] << 40) ^
       ((uint64_t)box[0] << 48) ^ ((uint64_t)dt << 56) ^ ((uint64_t)sw << 60);
  Entry& e = cache[(h ^ (h >> 29)) & 255];
  if (e.valid && e.base == base && e.d0 == dims[0] && e.d1 == dims[1] && e.s0 == strides[0] && e.b0 == box[0] &&
      e.b1 == box[1] && e.dt == (int)dt && e.sw == (int)sw && e.l2 == (int)l2) {
    *m = e.map;
    return CUDA_SUCCESS;
  }
  PFN_encodeTiled_t enc = get_encoder();
  if (!enc) return CUDA_ERROR_NOT_INITIALIZED;
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    e.map = *m;
    e.base = base;
    e.d0 = dims[0]; e.d1 = dims[1]; e.s0 = strides[0];
    e.b0 = box[0]; e.b1 = box[1];
    e.dt = (int)dt; e.sw = (int)sw; e.l2 = (int)l2;
    e.valid = true;
  }
  return r;
}

// 2-D map over packed codes [rows, words], box = 32 words x 64 rows, 128-B swizzle.
ef_status encode_codes_map(CUtensorMap* m, const uint32_t* w, long long rows, int words) {
  if (!get_encoder()) return fail(EF_ERR_NOT_READY, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)words, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)words * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)kRowTile};
  CUresult r = encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (r != CUDA_SUCCESS) return fail(EF_ERR_INVALID, "tensor map encode failed (%d)", (int)r);
  return EF_OK;
}

// 2-D map over fp16 activation rows [rows, K]: box 64 columns x 8 rows, 128-B swizzle.
ef_status encode_act_map(CUtensorMap* m, const uint16_t* act, long long rows, int K) {
  if (!get_encoder()) return fail(EF_ERR_NOT_READY, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)(rows > 0 ? rows : 1)};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kTokChunk};
  CUresult r = encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (r != CUDA_SUCCESS) return fail(EF_ERR_INVALID, "activation tensor map encode failed (%d)", (int)r);
  return EF_OK;
}

// fp16 scales or biases [rows, ng] for the decode GEMV's scale chunks: box 32
// groups x 64 rows, 64-byte swizzle.  Needs 16-byte rows (ng % 8 == 0) and a
// 16-byte-aligned base; false (nothing recorded) when the map cannot be made.
static bool encode_scales_map(CUtensorMap* m, const uint16_t* a, long long rows, int ng) {
  if (!get_encoder() || !a || ng % 8 || !aligned16(a) || rows < kRowTile) return false;
  cuuint64_t dims[2] = {(cuuint64_t)ng, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ng * 2};
  cuuint32_t box[2] = {32, (cuuint32_t)kRowTile};
  return encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, a, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B) == CUDA_SUCCESS;
}

// Chunked scale streaming for a GEMV launch whose scale pointers are set:
// maps over the routed arrays (rows = E * R) and the shared expert's (rows =
// shared_rows); whole-item scale slots when any map cannot be made.
static void set_scale_maps(QmvParams& p, long long rows, long long shared_rows) {
  p.sb_chunked = 0;
  const uint16_t* arr[8] = {p.s0, p.b0, p.s1 ? p.s1 : p.s0, p.b1 ? p.b1 : p.b0,
                            p.ss0, p.sb0, p.ss1 ? p.ss1 : p.ss0, p.sb1 ? p.sb1 : p.sb0};
  for (int i = 0; i < 8; ++i)
    if (!encode_scales_map(&p.tm_sc[i], arr[i], i < 4 ? rows : shared_rows, p.K / 64)) return;
  p.sb_chunked = 1;
}

// Code tiles for the grouped GEMM: box (chunk of 64 columns) x box_rows rows,
// swizzle matching the 64-byte (8-bit) / 32-byte (4-bit) row chunk.
ef_status encode_gemm_codes_map(CUtensorMap* m, const uint32_t* w, long long rows, int words, int bits, int box_rows) {
  if (!get_encoder()) return fail(EF_ERR_NOT_READY, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)words, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)words * 4};
  cuuint32_t box[2] = {(cuuint32_t)(64 * bits / 32), (cuuint32_t)box_rows};
  CUresult r = encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, dims, strides, box,
                         bits == 8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (r != CUDA_SUCCESS) return fail(EF_ERR_INVALID, "GEMM code tensor map encode failed (%d)", (int)r);
  return EF_OK;
}

// Activation rows for the grouped GEMM: box 64 columns x box_rows rows, 128-B swizzle.
ef_status encode_gemm_act_map(CUtensorMap* m, const uint16_t* act, long long rows, int K, int box_rows = 32) {
  if (!get_encoder()) return fail(EF_ERR_NOT_READY, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  CUresult r = encode_2d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (r != CUDA_SUCCESS) return fail(EF_ERR_INVALID, "GEMM activation tensor map encode failed (%d)", (int)r);
  return EF_OK;
}

// SM count of the current device, cached per device index (host threads may
// race on a first fill; they store the same value).
int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// ---- workspace carving
struct Carver {
  uint8_t* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

struct FfnBufs {
  PermBufs pb;
  uint16_t* x16;
  float* xsum;
  uint16_t* h16;
  float* hsum;
  float* yrows;
  int* ids;
};

// Routed rows (n_rows = entries + shared rows) carry their own gathered copy of
// the activation row (x16), so segments are contiguous for the GEMV tiles.
void carve_ffn(Carver& c, int n_ent, int n_bins, int n_rows, int H, int I, FfnBufs& f) {
  const int max_segs = (n_rows + kTokChunk - 1) / kTokChunk + n_bins + 2;
  f.pb.counts = c.take<int>(n_bins + 1);
  f.pb.offsets = c.take<int>(n_bins + 2);
  f.pb.row_src = c.take<int>(n_rows + 1);
  f.pb.inv = c.take<int>(n_ent + 1);
  f.pb.seg_expert = c.take<int>(max_segs);
  f.pb.seg_row0 = c.take<int>(max_segs);
  f.pb.seg_nrows = c.take<int>(max_segs);
  f.pb.n_seg = c.take<int>(1);
  f.x16 = c.take<uint16_t>((size_t)n_rows * H);
  f.xsum = c.take<float>((size_t)n_rows * sum_ld(H));
  f.h16 = c.take<uint16_t>((size_t)n_rows * I);
  f.hsum = c.take<float>((size_t)n_rows * sum_ld(I));
  f.yrows = c.take<float>((size_t)n_rows * H);
}

ef_status check_cfg(const ef_moe_cfg* c) {
  if (!c) return fail(EF_ERR_INVALID, "cfg is NULL");
  if (c->bits != 4 && c->bits != 8) return fail(EF_ERR_UNSUPPORTED, "bits must be 4 or 8 (got %d)", c->bits);
  if (c->group_size != 64) return fail(EF_ERR_UNSUPPORTED, "group_size must be 64 (got %d)", c->group_size);
  if (c->hidden <= 0 || c->hidden % 64) return fail(EF_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  if (c->inter <= 0 || c->inter % 64) return fail(EF_ERR_UNSUPPORTED, "inter must be a positive multiple of 64");
  if (c->n_experts < 1 || c->n_experts > 512) return fail(EF_ERR_UNSUPPORTED, "n_experts must be in 1..512");
  if (c->top_k < 1 || c->top_k > 16 || c->top_k > c->n_experts)
    return fail(EF_ERR_UNSUPPORTED, "top_k must be in 1..min(16, n_experts)");
  if (c->router_mode != EF_ROUTER_SOFTMAX && c->router_mode != EF_ROUTER_SIGMOID_GROUP)
    return fail(EF_ERR_INVALID, "unknown router_mode");
  if (c->router_mode == EF_ROUTER_SIGMOID_GROUP) {
    if (c->n_group < 1 || c->n_group > 32 || c->n_experts % c->n_group)
      return fail(EF_ERR_UNSUPPORTED, "n_group must divide n_experts and be <= 32");
    if (c->topk_group < 1 || c->topk_group > c->n_group) return fail(EF_ERR_INVALID, "topk_group out of range");
    if (c->n_group > 1 && c->topk_group * (c->n_experts / c->n_group) < c->top_k)
      return fail(EF_ERR_INVALID, "kept groups hold fewer than top_k experts");
  }
  if (c->n_shared < 0 || c->n_shared > 1) return fail(EF_ERR_UNSUPPORTED, "n_shared must be 0 or 1");
  if (c->n_shared && c->shared_inter != c->inter)
    return fail(EF_ERR_UNSUPPORTED, "shared_inter must equal inter");
  if (c->act_dtype != EF_DT_BF16 && c->act_dtype != EF_DT_F16) return fail(EF_ERR_UNSUPPORTED, "act_dtype");
  if (c->gate_dtype != EF_DT_BF16 && c->gate_dtype != EF_DT_F16) return fail(EF_ERR_UNSUPPORTED, "gate_dtype");
  return EF_OK;
}

ef_status check_qw(const ef_qweight& q, const char* name) {
  if (!q.w || !q.scales || !q.biases) return fail(EF_ERR_INVALID, "%s: null pointer", name);
  if (!aligned16(q.w) || !aligned16(q.scales) || !aligned16(q.biases))
    return fail(EF_ERR_INVALID, "%s: pointers must be 16-byte aligned", name);
  return EF_OK;
}

QmvParams make_params_common() {
  QmvParams p;
  memset(&p, 0, sizeof(p));
  return p;
}

// Where the down projection of an expert-parallel forward stores its rows
// (see QmvParams::ret_rank).
struct EpReturn {
  const int* rank;
  const int* row;
  float* const* base;
  uint32_t* const* flag;
  const uint32_t* epoch;
  uint32_t* ctr;
  int ranks, rows;
};

// gate/up (mode 0) then down (mode 1) over permuted rows already described by
// f.pb; with `ret`, the down rows go to the expert-parallel return regions.
ef_status run_experts(const ef_moe_cfg* c, const FfnBufs& f, int n_rows, const ef_qweight& gate,
                      const ef_qweight& up, const ef_qweight& down, const ef_qweight* sg, const ef_qweight* su,
                      const ef_qweight* sd, cudaStream_t st, const EpReturn* ret = nullptr) {
  const int H = c->hidden, I = c->inter, E = c->n_experts, bits = c->bits;
  const int nsm = sm_count();
  ef_status s;
  // mode 0: K = H, R = I
  QmvParams p0 = make_params_common();
  p0.w0 = gate.w; p0.w1 = up.w; p0.sw0 = sg ? sg->w : gate.w; p0.sw1 = su ? su->w : up.w;
  if ((s = encode_codes_map(&p0.tm_w0, gate.w, (long long)E * I, H * bits / 32))) return s;
  if ((s = encode_codes_map(&p0.tm_w1, up.w, (long long)E * I, H * bits / 32))) return s;
  if (sg) {
    if ((s = encode_codes_map(&p0.tm_sw0, sg->w, I, H * bits / 32))) return s;
    if ((s = encode_codes_map(&p0.tm_sw1, su->w, I, H * bits / 32))) return s;
    p0.ss0 = sg->scales; p0.sb0 = sg->biases; p0.ss1 = su->scales; p0.sb1 = su->biases;
  } else {
    p0.tm_sw0 = p0.tm_w0; p0.tm_sw1 = p0.tm_w1;
    p0.ss0 = gate.scales; p0.sb0 = gate.biases; p0.ss1 = up.scales; p0.sb1 = up.biases;
  }
  p0.s0 = gate.scales; p0.b0 = gate.biases; p0.s1 = up.scales; p0.b1 = up.biases;
  if ((s = encode_act_map(&p0.tm_act, f.x16, n_rows, H))) return s;
  p0.act_sum = f.xsum;
  p0.seg_expert = f.pb.seg_expert; p0.seg_row0 = f.pb.seg_row0; p0.seg_nrows = f.pb.seg_nrows; p0.n_seg = f.pb.n_seg;
  p0.K = H; p0.R = I; p0.n_experts = E;
  set_scale_maps(p0, (long long)E * I, sg ? I : (long long)E * I);
  p0.h_out = f.h16; p0.hsum_out = f.hsum; p0.y_out = nullptr;
  EF_LAUNCH("qmv_gate_up", launch_qmv(bits, 0, p0, nsm, st));
  // mode 1: K = I, R = H
  QmvParams p1 = make_params_common();
  p1.w0 = down.w; p1.w1 = down.w; p1.sw0 = sd ? sd->w : down.w; p1.sw1 = p1.sw0;
  if ((s = encode_codes_map(&p1.tm_w0, down.w, (long long)E * H, I * bits / 32))) return s;
  if (sd) {
    if ((s = encode_codes_map(&p1.tm_sw0, sd->w, H, I * bits / 32))) return s;
    p1.ss0 = sd->scales; p1.sb0 = sd->biases;
  } else {
    p1.tm_sw0 = p1.tm_w0; p1.ss0 = down.scales; p1.sb0 = down.biases;
  }
  p1.tm_w1 = p1.tm_w0; p1.tm_sw1 = p1.tm_sw0;
  p1.s0 = down.scales; p1.b0 = down.biases;
  if ((s = encode_act_map(&p1.tm_act, f.h16, n_rows, I))) return s;
  p1.act_sum = f.hsum;
  p1.seg_expert = f.pb.seg_expert; p1.seg_row0 = f.pb.seg_row0; p1.seg_nrows = f.pb.seg_nrows; p1.n_seg = f.pb.n_seg;
  p1.K = I; p1.R = H; p1.n_experts = E;
  set_scale_maps(p1, (long long)E * H, sd ? H : (long long)E * H);
  p1.y_out = f.yrows;
  if (ret) {
    p1.ret_rank = ret->rank;
    p1.ret_row = ret->row;
    p1.ret_base = ret->base;
    p1.ret_flag = ret->flag;
    p1.ep_epoch = ret->epoch;
    p1.ep_ctr = ret->ctr;
    p1.ep_ranks = ret->ranks;
    p1.ret_rows = ret->rows;
  }
  // each expert with rows makes at least one segment
  const int min_segs = std::min(n_rows, E + (sd ? 1 : 0));
  EF_LAUNCH("qmv_down", launch_qmv(bits, 1, p1, nsm, st, min_segs));
  return EF_OK;
}

// Grouped-GEMM (tcgen05) version of run_experts; segments of <= kGemmSegRows rows.
ef_status run_experts_gemm(const ef_moe_cfg* c, const FfnBufs& f, int n_rows, const ef_qweight& gate,
                           const ef_qweight& up, const ef_qweight& down, const ef_qweight* sg, const ef_qweight* su,
                           const ef_qweight* sd, cudaStream_t st) {
  const int H = c->hidden, I = c->inter, E = c->n_experts, bits = c->bits;
  const int nsm = sm_count();
  // single-SM kernel unless the SM-pair kernel (cta_group::2) is requested:
  // both tile 256 weight rows x <= 192 token rows per tile, so the pair loads
  // the same activation bytes and dequantises the same codes per FLOP, and its
  // cross-SM handshakes made it slower on B200 (4.5 ms vs 3.2 ms for the
  // 4096-token DeepSeek-V3-shaped gate_up)
  const bool pairs = c->path == EF_PATH_GEMM_PAIR && nsm >= 2;
  const int cb0 = pairs ? 64 : 128, cb1 = 128, ab = pairs ? 16 : 32;
  ef_status s;
  GemmParams g0;
  memset(&g0, 0, sizeof(g0));
  if ((s = encode_gemm_codes_map(&g0.tm_c0, gate.w, (long long)E * I, H * bits / 32, bits, cb0))) return s;
  if ((s = encode_gemm_codes_map(&g0.tm_c1, up.w, (long long)E * I, H * bits / 32, bits, cb0))) return s;
  if (sg) {
    if ((s = encode_gemm_codes_map(&g0.tm_sc0, sg->w, I, H * bits / 32, bits, cb0))) return s;
    if ((s = encode_gemm_codes_map(&g0.tm_sc1, su->w, I, H * bits / 32, bits, cb0))) return s;
    g0.ss0 = sg->scales; g0.sb0 = sg->biases; g0.ss1 = su->scales; g0.sb1 = su->biases;
  } else {
    g0.tm_sc0 = g0.tm_c0; g0.tm_sc1 = g0.tm_c1;
    g0.ss0 = gate.scales; g0.sb0 = gate.biases; g0.ss1 = up.scales; g0.sb1 = up.biases;
  }
  g0.s0 = gate.scales; g0.b0 = gate.biases; g0.s1 = up.scales; g0.b1 = up.biases;
  if ((s = encode_gemm_act_map(&g0.tm_act, f.x16, n_rows, H, ab))) return s;
  g0.seg_expert = f.pb.seg_expert; g0.seg_row0 = f.pb.seg_row0; g0.seg_nrows = f.pb.seg_nrows; g0.n_seg = f.pb.n_seg;
  g0.K = H; g0.R = I; g0.n_experts = E; g0.h_out = f.h16;
  EF_LAUNCH("qgemm_gate_up", pairs ? launch_qgemm2(bits, 0, g0, nsm, st) : launch_qgemm(bits, 0, g0, nsm, st));
  GemmParams g1;
  memset(&g1, 0, sizeof(g1));
  if ((s = encode_gemm_codes_map(&g1.tm_c0, down.w, (long long)E * H, I * bits / 32, bits, cb1))) return s;
  if (sd) {
    if ((s = encode_gemm_codes_map(&g1.tm_sc0, sd->w, H, I * bits / 32, bits, cb1))) return s;
    g1.ss0 = sd->scales; g1.sb0 = sd->biases;
  } else {
    g1.tm_sc0 = g1.tm_c0; g1.ss0 = down.scales; g1.sb0 = down.biases;
  }
  g1.tm_c1 = g1.tm_c0; g1.tm_sc1 = g1.tm_sc0;
  g1.s0 = down.scales; g1.b0 = down.biases;
  if ((s = encode_gemm_act_map(&g1.tm_act, f.h16, n_rows, I, ab))) return s;
  g1.seg_expert = f.pb.seg_expert; g1.seg_row0 = f.pb.seg_row0; g1.seg_nrows = f.pb.seg_nrows; g1.n_seg = f.pb.n_seg;
  g1.K = I; g1.R = H; g1.n_experts = E; g1.y_out = f.yrows;
  EF_LAUNCH("qgemm_down", pairs ? launch_qgemm2(bits, 1, g1, nsm, st) : launch_qgemm(bits, 1, g1, nsm, st));
  return EF_OK;
}

// Grouped GEMM for many tokens per expert, decode GEMV otherwise.
bool use_gemm(const ef_moe_cfg* c, int n_rows, int n_ent) {
  // code boxes are 128 rows tall: both projections need at least that many rows
  if (n_rows < 128 || c->inter < 128 || c->hidden < 128) return false;
  if (c->path == EF_PATH_GEMM || c->path == EF_PATH_GEMM_PAIR) return true;
  if (c->path == EF_PATH_GEMV) return false;
  return (long long)n_ent >= 32LL * c->n_experts;  // >= 32 routed rows per expert on average
}

size_t smem_check(int bits, int H, int I) {
  size_t a = qmv_smem_required(bits, 0, H), b = qmv_smem_required(bits, 1, I);
  return a > b ? a : b;
}

}  // namespace

// =====================================================================================
extern "C" {

const char* ef_version(void) { return "efmoe 0.1.0 (sm_100a)"; }

const char* ef_status_string(ef_status s) {
  switch (s) {
    case EF_OK: return "ok";
    case EF_ERR_INVALID: return "invalid argument";
    case EF_ERR_UNSUPPORTED: return "unsupported configuration";
    case EF_ERR_CUDA: return "CUDA error";
    case EF_ERR_WORKSPACE: return "workspace too small";
    case EF_ERR_TIMEOUT: return "device wait timed out";
    case EF_ERR_SLOT_MISS: return "expert not resident";
    case EF_ERR_RANGE: return "value out of range";
    case EF_ERR_NOT_READY: return "not ready";
    case EF_ERR_IO: return "file read failed";
    default: return "unknown status";
  }
}

const char* ef_last_error_message(void) { return g_last_msg.c_str(); }

ef_status ef_trace_enable(int on) {
  std::lock_guard<std::mutex> lk(g_trace_mu);
  g_trace_on = on != 0;
  return EF_OK;
}

int ef_trace_read(ef_trace_rec* recs, int max_recs) {
  std::lock_guard<std::mutex> lk(g_trace_mu);
  int n = 0;
  for (const TraceRec& r : g_trace) {
    float ms = -1.0f;
    if (cudaEventSynchronize(r.b) == cudaSuccess) cudaEventElapsedTime(&ms, r.a, r.b);
    if (recs && n < max_recs) recs[n] = ef_trace_rec{r.name, ms};
    ++n;
    g_event_pool.push_back(r.a);
    g_event_pool.push_back(r.b);
  }
  g_trace.clear();
  return recs ? (n < max_recs ? n : max_recs) : n;
}

ef_status ef_get_device_error(void* stream, int* code) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0, zero = 0;
  EF_CUDA(cudaMemcpyFromSymbolAsync(&v, g_ef_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
  EF_CUDA(cudaStreamSynchronize(st));
  EF_CUDA(cudaMemcpyToSymbolAsync(g_ef_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st));
  EF_CUDA(cudaStreamSynchronize(st));
  if (code) *code = v;
  if (v >= 1000 && v < 2000) return EF_ERR_TIMEOUT;
  if (v >= 2000) return EF_ERR_RANGE;
  return EF_OK;
}

size_t ef_router_workspace_size(const ef_moe_cfg* cfg, int T) {
  if (!cfg || T < 0) return 0;
  Carver c{nullptr};
  c.take<float>((size_t)T * cfg->n_experts);
  return c.off + 256;
}

ef_status ef_router_topk(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w, const float* e_bias,
                         int32_t* inds, float* weights, float* logits_out, void* workspace, size_t ws_bytes,
                         void* stream) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!x || !gate_w || !inds || !weights) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x) || !aligned16(gate_w)) return fail(EF_ERR_INVALID, "x and gate_w must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* logits = logits_out;
  if (!logits) {
    if (ws_bytes < ef_router_workspace_size(cfg, T) || !workspace) return fail(EF_ERR_WORKSPACE, "workspace too small");
    Carver c{static_cast<uint8_t*>(workspace)};
    logits = c.take<float>((size_t)T * cfg->n_experts);
  }
  EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), cfg->act_dtype == EF_DT_BF16,
                               static_cast<const uint16_t*>(gate_w), cfg->gate_dtype == EF_DT_BF16, T, cfg->n_experts,
                               cfg->hidden, logits, st));
  EF_LAUNCH("router_select", launch_router_select(logits, e_bias, T, cfg->n_experts, cfg->top_k, cfg->router_mode, cfg->norm_topk,
                               cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->n_group : 1, cfg->topk_group,
                               cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->routed_scaling : 1.0f, inds,
                               weights, st));
  return EF_OK;
}

size_t ef_permute_workspace_size(int n_entries, int n_experts, int n_shared_rows, int seg_rows) {
  if (n_entries < 0 || n_experts < 1 || n_shared_rows < 0 || seg_rows < 1) return 0;
  Carver c{nullptr};
  const int max_segs = (n_entries + n_shared_rows + seg_rows - 1) / seg_rows + n_experts + 3;
  c.take<int>(max_segs);
  c.take<int>(max_segs);
  c.take<int>(max_segs);
  c.take<int>(1);
  return c.off + 256;
}

ef_status ef_permute(const int32_t* entries, int n_entries, int k, int n_experts, int n_shared_rows, int seg_rows,
                     int32_t* counts, int32_t* offsets, int32_t* row_src, int32_t* inv, void* workspace,
                     size_t ws_bytes, void* stream) {
  if (n_entries < 0 || k < 1 || n_experts < 1 || n_experts > 512 || n_shared_rows < 0 || seg_rows < 1)
    return fail(EF_ERR_INVALID, "bad permute arguments (n_entries %d, k %d, n_experts %d, shared rows %d, seg %d)",
                n_entries, k, n_experts, n_shared_rows, seg_rows);
  if (n_entries % k) return fail(EF_ERR_INVALID, "n_entries must be a multiple of k");
  if (n_entries + n_shared_rows == 0) return EF_OK;
  if (!entries || !counts || !offsets || !row_src || !inv) return fail(EF_ERR_INVALID, "null pointer");
  if (!workspace || ws_bytes < ef_permute_workspace_size(n_entries, n_experts, n_shared_rows, seg_rows))
    return fail(EF_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  const int max_segs = (n_entries + n_shared_rows + seg_rows - 1) / seg_rows + n_experts + 3;
  PermBufs pb;
  pb.counts = counts;
  pb.offsets = offsets;
  pb.row_src = row_src;
  pb.inv = inv;
  pb.seg_expert = c.take<int>(max_segs);
  pb.seg_row0 = c.take<int>(max_segs);
  pb.seg_nrows = c.take<int>(max_segs);
  pb.n_seg = c.take<int>(1);
  EF_LAUNCH("permute", launch_permute(entries, n_entries, k, n_experts, n_shared_rows, seg_rows, pb, st));
  return EF_OK;
}

ef_status ef_combine(const float* rows, const int32_t* inv, const float* wts, int T, int k, int H, int shared_base,
                     void* y, int out_dtype, void* stream) {
  if (T < 0 || k < 1 || H <= 0 || H % 4) return fail(EF_ERR_INVALID, "bad combine shape (T %d, k %d, H %d)", T, k, H);
  if (out_dtype < EF_DT_BF16 || out_dtype > EF_DT_F32) return fail(EF_ERR_UNSUPPORTED, "out_dtype");
  if (T == 0) return EF_OK;
  if (!rows || !inv || !y) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(rows) || !aligned16(y)) return fail(EF_ERR_INVALID, "rows and y must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  EF_LAUNCH("combine", launch_combine(rows, inv, wts, T, k, H, shared_base, y, out_dtype, st));
  return EF_OK;
}

// permute -> gather -> experts -> weighted combine for T tokens routed by
// inds [T, k] (ids in [0, cfg->n_experts)) with weights wts [T, k].
static ef_status moe_tail(const ef_moe_cfg* cfg, const void* x, int T, const int* inds, const float* wts,
                          const ef_qweight& gate, const ef_qweight& up, const ef_qweight& down, const ef_qweight* sg,
                          const ef_qweight* su, const ef_qweight* sd, const FfnBufs& f, void* y, cudaStream_t st) {
  ef_status s;
  const int H = cfg->hidden, E = cfg->n_experts, k = cfg->top_k;
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  const int n_sh = cfg->n_shared ? T : 0;
  const bool gemm = use_gemm(cfg, T * k + n_sh, T * k);
  EF_LAUNCH("permute", launch_permute(inds, T * k, k, E, n_sh, gemm ? kGemmSegRows : kSegRows, f.pb, st));
  EF_LAUNCH("prep_act", launch_prep_act(static_cast<const uint16_t*>(x), f.pb.row_src, bf, T * k + n_sh, H, cfg->bits,
                                        f.x16, f.xsum, st));
  if (gemm) {
    if ((s = run_experts_gemm(cfg, f, T * k + n_sh, gate, up, down, cfg->n_shared ? sg : nullptr,
                              cfg->n_shared ? su : nullptr, cfg->n_shared ? sd : nullptr, st)))
      return s;
  } else if ((s = run_experts(cfg, f, T * k + n_sh, gate, up, down, cfg->n_shared ? sg : nullptr,
                              cfg->n_shared ? su : nullptr, cfg->n_shared ? sd : nullptr, st))) {
    return s;
  }
  // shared rows start at offsets[E] == T*k
  EF_LAUNCH("combine", launch_combine(f.yrows, f.pb.inv, wts, T, k, H, cfg->n_shared ? T * k : -1, y,
                         cfg->out_f32 ? EF_DT_F32 : (bf ? EF_DT_BF16 : EF_DT_F16), st));
  return EF_OK;
}

static size_t moe_ws(const ef_moe_cfg* cfg, int T, Carver& c, float** logits, int** inds, float** wts, FfnBufs* f) {
  const int E = cfg->n_experts, k = cfg->top_k;
  const int n_ent = T * k, n_rows = n_ent + (cfg->n_shared ? T : 0);
  *logits = c.take<float>((size_t)T * E);
  *inds = c.take<int>((size_t)n_ent);
  *wts = c.take<float>((size_t)n_ent);
  carve_ffn(c, n_ent, E + 1, n_rows, cfg->hidden, cfg->inter, *f);
  return c.off;
}

size_t ef_moe_workspace_size(const ef_moe_cfg* cfg, int T) {
  if (!cfg || T < 0) return 0;
  Carver c{nullptr};
  float* l;
  int* i;
  float* w;
  FfnBufs f;
  return moe_ws(cfg, T, c, &l, &i, &w, &f) + 256;
}

ef_status ef_moe_forward(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w, const float* e_bias,
                         ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* sg, const ef_qweight* su,
                         const ef_qweight* sd, void* y, int32_t* inds_out, float* wts_out, void* workspace,
                         size_t ws_bytes, void* stream) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!x || !gate_w || !y) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x) || !aligned16(gate_w) || !aligned16(y)) return fail(EF_ERR_INVALID, "x/gate_w/y must be 16-byte aligned");
  if ((s = check_qw(gate, "gate")) || (s = check_qw(up, "up")) || (s = check_qw(down, "down"))) return s;
  if (cfg->n_shared) {
    if (!sg || !su || !sd) return fail(EF_ERR_INVALID, "n_shared=1 needs shared_gate/up/down");
    if ((s = check_qw(*sg, "shared_gate")) || (s = check_qw(*su, "shared_up")) || (s = check_qw(*sd, "shared_down")))
      return s;
  }
  if (ws_bytes < ef_moe_workspace_size(cfg, T) || !workspace || !aligned16(workspace))
    return fail(EF_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, ef_moe_workspace_size(cfg, T));
  if (smem_check(cfg->bits, cfg->hidden, cfg->inter) > 227 * 1024)
    return fail(EF_ERR_UNSUPPORTED, "hidden/inter too large for the decode kernel");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  float* logits;
  int* inds;
  float* wts;
  FfnBufs f;
  moe_ws(cfg, T, c, &logits, &inds, &wts, &f);
  if (inds_out) inds = inds_out;
  if (wts_out) wts = wts_out;
  const int H = cfg->hidden, E = cfg->n_experts, k = cfg->top_k;
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), bf, static_cast<const uint16_t*>(gate_w),
                               cfg->gate_dtype == EF_DT_BF16, T, E, H, logits, st));
  EF_LAUNCH("router_select", launch_router_select(logits, e_bias, T, E, k, cfg->router_mode, cfg->norm_topk,
                               cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->n_group : 1, cfg->topk_group,
                               cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->routed_scaling : 1.0f, inds, wts,
                               st));
  return moe_tail(cfg, x, T, inds, wts, gate, up, down, sg, su, sd, f, y, st);
}

size_t ef_experts_workspace_size(const ef_moe_cfg* cfg, int N) {
  if (!cfg || N < 0) return 0;
  Carver c{nullptr};
  FfnBufs f;
  carve_ffn(c, N, cfg->n_experts + 1, N, cfg->hidden, cfg->inter, f);
  return c.off + 256;
}

ef_status ef_moe_experts_forward(const ef_moe_cfg* cfg, const void* x_rows, int N, const int32_t* row_expert,
                                 ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* sg,
                                 const ef_qweight* su, const ef_qweight* sd, float* y_rows, void* workspace,
                                 size_t ws_bytes, void* stream) {
  (void)sg; (void)su; (void)sd;
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (N < 0) return fail(EF_ERR_INVALID, "N < 0");
  if (N == 0) return EF_OK;
  if (!x_rows || !row_expert || !y_rows) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x_rows) || !aligned16(y_rows)) return fail(EF_ERR_INVALID, "x_rows/y_rows must be 16-byte aligned");
  if ((s = check_qw(gate, "gate")) || (s = check_qw(up, "up")) || (s = check_qw(down, "down"))) return s;
  if (ws_bytes < ef_experts_workspace_size(cfg, N) || !workspace) return fail(EF_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  FfnBufs f;
  carve_ffn(c, N, cfg->n_experts + 1, N, cfg->hidden, cfg->inter, f);
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  const bool gemm = use_gemm(cfg, N, N);
  EF_LAUNCH("permute", launch_permute(row_expert, N, 1, cfg->n_experts, 0, gemm ? kGemmSegRows : kSegRows, f.pb, st));
  EF_LAUNCH("prep_act", launch_prep_act(static_cast<const uint16_t*>(x_rows), f.pb.row_src, bf, N, cfg->hidden,
                                        cfg->bits, f.x16, f.xsum, st));
  if (gemm) {
    if ((s = run_experts_gemm(cfg, f, N, gate, up, down, nullptr, nullptr, nullptr, st))) return s;
  } else if ((s = run_experts(cfg, f, N, gate, up, down, nullptr, nullptr, nullptr, st))) {
    return s;
  }
  EF_LAUNCH("combine", launch_combine(f.yrows, f.pb.inv, nullptr, N, 1, cfg->hidden, -1, y_rows, EF_DT_F32, st));
  return EF_OK;
}

// ---- single-matrix ops (mode 1 of the GEMV kernel with one "expert")
static size_t qmm_ws(int M, int k, int n_exp, int out_dim, int in_dim, Carver& c, FfnBufs& f, int n_rows_x) {
  const int n_ent = M * k;
  const int max_segs = (n_ent + kTokChunk - 1) / kTokChunk + n_exp + 2;
  f.pb.counts = c.take<int>(n_exp + 1);
  f.pb.offsets = c.take<int>(n_exp + 2);
  f.pb.row_src = c.take<int>(n_ent + 1);
  f.pb.inv = c.take<int>(n_ent + 1);
  f.pb.seg_expert = c.take<int>(max_segs);
  f.pb.seg_row0 = c.take<int>(max_segs);
  f.pb.seg_nrows = c.take<int>(max_segs);
  f.pb.n_seg = c.take<int>(1);
  (void)n_rows_x;
  f.x16 = c.take<uint16_t>((size_t)n_ent * in_dim);
  f.xsum = c.take<float>((size_t)n_ent * sum_ld(in_dim));
  f.yrows = c.take<float>((size_t)n_ent * out_dim);
  f.ids = c.take<int>((size_t)M);  // expert ids (all zero) for the single-matrix case
  return c.off;
}

static ef_status check_qmm(int out_dim, int in_dim, int bits, int group) {
  if (bits != 4 && bits != 8) return fail(EF_ERR_UNSUPPORTED, "bits must be 4 or 8");
  if (group != 64) return fail(EF_ERR_UNSUPPORTED, "group_size must be 64");
  if (in_dim <= 0 || in_dim % 64) return fail(EF_ERR_UNSUPPORTED, "in_dim must be a positive multiple of 64");
  if (out_dim <= 0 || out_dim % 64) return fail(EF_ERR_UNSUPPORTED, "out_dim must be a positive multiple of 64");
  if (qmv_smem_required(bits, 1, in_dim) > 227 * 1024) return fail(EF_ERR_UNSUPPORTED, "in_dim too large");
  return EF_OK;
}

static ef_status run_single_matrix(const ef_qweight& w, int n_exp, int out_dim, int in_dim, int bits,
                                   const FfnBufs& f, int n_rows, cudaStream_t st) {
  QmvParams p = make_params_common();
  ef_status s;
  p.w0 = w.w; p.w1 = w.w; p.sw0 = w.w; p.sw1 = w.w;
  if ((s = encode_codes_map(&p.tm_w0, w.w, (long long)n_exp * out_dim, in_dim * bits / 32))) return s;
  p.tm_w1 = p.tm_w0; p.tm_sw0 = p.tm_w0; p.tm_sw1 = p.tm_w0;
  p.s0 = w.scales; p.b0 = w.biases; p.ss0 = w.scales; p.sb0 = w.biases;
  if ((s = encode_act_map(&p.tm_act, f.x16, n_rows, in_dim))) return s;
  p.act_sum = f.xsum;
  p.seg_expert = f.pb.seg_expert; p.seg_row0 = f.pb.seg_row0; p.seg_nrows = f.pb.seg_nrows; p.n_seg = f.pb.n_seg;
  p.K = in_dim; p.R = out_dim; p.n_experts = n_exp;
  set_scale_maps(p, (long long)n_exp * out_dim, (long long)n_exp * out_dim);
  p.y_out = f.yrows;
  EF_LAUNCH("qmv_down", launch_qmv(bits, 1, p, sm_count(), st, std::min(n_rows, n_exp)));
  return EF_OK;
}

size_t ef_quantized_matmul_workspace_size(int M, int out_dim, int in_dim) {
  if (M < 0) return 0;
  Carver c{nullptr};
  FfnBufs f;
  return qmm_ws(M, 1, 1, out_dim, in_dim, c, f, M) + 256;
}

ef_status ef_quantized_matmul(const void* x, int act_dtype, int M, const uint32_t* w, const uint16_t* scales,
                              const uint16_t* biases, int out_dim, int in_dim, int bits, int group_size, void* y,
                              void* workspace, size_t ws_bytes, void* stream) {
  ef_status s = check_qmm(out_dim, in_dim, bits, group_size);
  if (s) return s;
  if (act_dtype != EF_DT_BF16 && act_dtype != EF_DT_F16) return fail(EF_ERR_UNSUPPORTED, "act_dtype");
  if (M < 0) return fail(EF_ERR_INVALID, "M < 0");
  if (M == 0) return EF_OK;
  ef_qweight q{w, scales, biases};
  if ((s = check_qw(q, "w"))) return s;
  if (!x || !y || !aligned16(x) || !aligned16(y)) return fail(EF_ERR_INVALID, "x/y null or misaligned");
  if (!workspace || ws_bytes < ef_quantized_matmul_workspace_size(M, out_dim, in_dim))
    return fail(EF_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  FfnBufs f;
  qmm_ws(M, 1, 1, out_dim, in_dim, c, f, M);
  int* ids = f.ids;
  EF_CUDA(cudaMemsetAsync(ids, 0, sizeof(int) * (size_t)M, st));
  EF_LAUNCH("permute", launch_permute(ids, M, 1, 1, 0, kSegRows, f.pb, st));
  EF_LAUNCH("prep_act", launch_prep_act(static_cast<const uint16_t*>(x), f.pb.row_src, act_dtype == EF_DT_BF16, M,
                                        in_dim, bits, f.x16, f.xsum, st));
  if ((s = run_single_matrix(q, 1, out_dim, in_dim, bits, f, M, st))) return s;
  EF_LAUNCH("combine", launch_combine(f.yrows, f.pb.inv, nullptr, M, 1, out_dim, -1, y, act_dtype, st));
  return EF_OK;
}

size_t ef_gather_qmm_workspace_size(int T, int k, int n_experts, int out_dim, int in_dim) {
  if (T < 0 || k < 1) return 0;
  Carver c{nullptr};
  FfnBufs f;
  return qmm_ws(T, k, n_experts, out_dim, in_dim, c, f, T) + 256;
}

ef_status ef_gather_qmm(const void* x, int act_dtype, int T, const int32_t* indices, int k, ef_qweight w,
                        int n_experts, int out_dim, int in_dim, int bits, int group_size, void* y, void* workspace,
                        size_t ws_bytes, void* stream) {
  ef_status s = check_qmm(out_dim, in_dim, bits, group_size);
  if (s) return s;
  if (act_dtype != EF_DT_BF16 && act_dtype != EF_DT_F16) return fail(EF_ERR_UNSUPPORTED, "act_dtype");
  if (T < 0 || k < 1 || n_experts < 1 || n_experts > 512) return fail(EF_ERR_INVALID, "bad T/k/n_experts");
  if (T == 0) return EF_OK;
  if ((s = check_qw(w, "w"))) return s;
  if (!x || !y || !indices || !aligned16(x) || !aligned16(y)) return fail(EF_ERR_INVALID, "x/y/indices");
  if (!workspace || ws_bytes < ef_gather_qmm_workspace_size(T, k, n_experts, out_dim, in_dim))
    return fail(EF_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  FfnBufs f;
  qmm_ws(T, k, n_experts, out_dim, in_dim, c, f, T);
  EF_LAUNCH("permute", launch_permute(indices, T * k, k, n_experts, 0, kSegRows, f.pb, st));
  EF_LAUNCH("prep_act", launch_prep_act(static_cast<const uint16_t*>(x), f.pb.row_src, act_dtype == EF_DT_BF16,
                                        T * k, in_dim, bits, f.x16, f.xsum, st));
  if ((s = run_single_matrix(w, n_experts, out_dim, in_dim, bits, f, T * k, st))) return s;
  EF_LAUNCH("combine", launch_combine(f.yrows, f.pb.inv, nullptr, T * k, 1, out_dim, -1, y, act_dtype, st));
  return EF_OK;
}

ef_status ef_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int rows, int cols,
                        int bits, int group_size, void* out, int out_dtype, void* stream) {
  if (bits != 4 && bits != 8) return fail(EF_ERR_UNSUPPORTED, "bits must be 4 or 8");
  if (group_size != 64) return fail(EF_ERR_UNSUPPORTED, "group_size must be 64");
  if (rows < 0 || cols < 0 || cols % 64) return fail(EF_ERR_INVALID, "cols must be a multiple of 64");
  if (out_dtype < EF_DT_BF16 || out_dtype > EF_DT_F32) return fail(EF_ERR_UNSUPPORTED, "out_dtype");
  if (rows == 0 || cols == 0) return EF_OK;
  if (!w || !scales || !biases || !out) return fail(EF_ERR_INVALID, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  EF_LAUNCH("dequantize", launch_dequantize(w, scales, biases, rows, cols, bits, out, out_dtype, st));
  return EF_OK;
}

}  // extern "C"
