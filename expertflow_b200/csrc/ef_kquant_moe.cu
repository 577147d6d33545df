// ef_kquant_moe.cu -- MoE layer whose experts are GGUF K-quant matrices
// (Q2_K / Q3_K / Q4_K), the form in which the reference streams DeepSeek
// GGUF models: ExpertMmapLoader.load_expert_dequantized (ef_deepseek_mmap.py:
// 570-593) decodes an expert's gate / up / down slices of the stacked
// blk.{i}.ffn_{gate,up,down}_exps tensors to fp16, and the MoE forward runs
// silu(x Wg^T) * (x Wu^T) Wd^T per routed (token, k) with the score-weighted
// sum in k order plus the shared expert (ef_deepseek_mmap.py:1563-1660).
//
// Router, permutation and combine are the 4/8-bit layer's.  The experts run
// on two routed K-quant GEMV kernels, work item = (segment of <= 8 rows of one
// expert) x (16 weight rows), one warp per item: blocks are decoded straight
// into mma.sync A fragments (the decoders of ef_kquant.cu: the same fp16 values
// as the reference's dequantisation), activations are fp16 in the format's
// permuted order, products accumulate in fp32.
//   gate/up: h = silu(g) * u per (row, output), fp32;
//   down:    y rows, fp32, for the combine.
#include "ef_common.cuh"

namespace ef {

// out[r][K] fp16 in the K-quant GEMV's permuted order for TYPE (see
// kquant_prep_kernel) = in[row_src[r]] (or in[r]); in: bf16 / fp16 / fp32 rows
// of K values (in_dtype EF_DT_*).  n_dev (or null): row count on the device.
// Q4_K also the sums of each 32-element sub-block of the rounded values, xs
// fp32 [n][K / 32], in element order.
template <int TYPE>
__global__ void kq_rows_prep_kernel(const void* __restrict__ in, int in_dtype, const int* __restrict__ row_src,
                                    int n, const int* __restrict__ n_dev, int K, uint16_t* __restrict__ out,
                                    float* __restrict__ xs) {
  pdl_wait();
  if (n_dev) n = min(n, max(0, *n_dev));
  const long long total = (long long)n * K;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / K), kk = (int)(i % K);
    const int kb = kk >> 8, pp = kk & 255;
    const int q = pp >> 5, c = (pp >> 3) & 3, rr = pp & 7;
    const int src = 256 * kb + kq_elem(TYPE, c, 2 * q + (rr >> 2), rr & 3);
    const long long sr = row_src ? __ldg(row_src + r) : r;
    float v;
    if (in_dtype == 2) {
      v = static_cast<const float*>(in)[sr * K + src];
    } else {
      v = act_to_f32(static_cast<const uint16_t*>(in)[sr * K + src], in_dtype == 0);
    }
    if (!(fabsf(v) <= 65504.0f)) ef_set_error(kDevErrRange);
    out[i] = f32_to_h16_sat(v);
  }
  if (TYPE == kKqQ4) {
    const int nsb = K >> 5;
    const long long tsum = (long long)n * nsb;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < tsum;
         i += (long long)gridDim.x * blockDim.x) {
      const int r = (int)(i / nsb), sb = (int)(i % nsb);
      const long long sr = row_src ? __ldg(row_src + r) : r;
      float sum = 0.0f;
      for (int e = 0; e < 32; ++e) {
        const size_t o = (size_t)sr * K + 32 * sb + e;
        const float v = in_dtype == 2 ? static_cast<const float*>(in)[o]
                                      : act_to_f32(static_cast<const uint16_t*>(in)[o], in_dtype == 0);
        sum += h16_to_f32(f32_to_h16_sat(v));
      }
      xs[i] = sum;
    }
  }
}

struct KqMoeParams {
  const uint8_t* w0;   // gate (mode 0) or down (mode 1): expert 0's first block
  const uint8_t* w1;   // up (mode 0)
  long long stride0;   // bytes from one expert's matrix to the next
  long long stride1;
  const uint8_t* sw0;  // the shared expert's matrices (expert id == n_experts)
  const uint8_t* sw1;
  const uint16_t* xp;  // permuted fp16 activation rows [n_rows][K]
  const float* xs;     // Q4_K: their sub-block sums [n_rows][K / 32]
  const int* seg_expert;
  const int* seg_row0;
  const int* seg_nrows;
  const int* n_seg;
  int K, R, n_experts;
  float* out;          // mode 0: h [rows][R]; mode 1: y [rows][R] (fp32)
};

template <int TYPE, int MODE>
__global__ void __launch_bounds__(kKqWarps * 32, MODE == 0 ? 1 : 2) kq_moe_kernel(const __grid_constant__ KqMoeParams p) {
  pdl_wait();
  constexpr int BB = kq_block_bytes(TYPE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int nb = p.K >> 8;
  const int n_rt = p.R >> 4;
  const int n_items = (*p.n_seg) * n_rt;
  const size_t row_bytes = (size_t)nb * BB;
  for (int item = blockIdx.x * kKqWarps + warp; item < n_items; item += gridDim.x * kKqWarps) {
    const int seg = item / n_rt, rt = item - seg * n_rt;
    const int e = __ldg(p.seg_expert + seg), row0 = __ldg(p.seg_row0 + seg), nrows = __ldg(p.seg_nrows + seg);
    const bool sh = e >= p.n_experts;
    const uint8_t* b0 = sh ? p.sw0 : p.w0 + (size_t)e * p.stride0;
    const uint8_t* g0 = b0 + (size_t)(16 * rt + g) * row_bytes;  // rows g and g + 8 of the tile
    const uint8_t* g1 = g0 + 8 * row_bytes;
    const uint8_t* u0 = nullptr;
    const uint8_t* u1 = nullptr;
    if (MODE == 0) {
      const uint8_t* b1 = sh ? p.sw1 : p.w1 + (size_t)e * p.stride1;
      u0 = b1 + (size_t)(16 * rt + g) * row_bytes;
      u1 = u0 + 8 * row_bytes;
    }
    // lane g's token column: a row of the segment (rows past its end repeat
    // the last one; their outputs are not stored)
    const size_t tok_off[1] = {(size_t)(row0 + min(g, nrows - 1)) * p.K};
    // Q4_K sub-block sums of the accumulator's tokens 2c, 2c + 1 (the same repeat)
    const size_t xs_off[1][2] = {{(size_t)(row0 + min(2 * c, nrows - 1)) * (size_t)(p.K >> 5),
                                  (size_t)(row0 + min(2 * c + 1, nrows - 1)) * (size_t)(p.K >> 5)}};
    const uint16_t* xl = p.xp + 8 * c;
    float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    float accu[1][4] = {{0.f, 0.f, 0.f, 0.f}};
    KqRow<TYPE> ra, rb;
    ra.load(g0, c);
    rb.load(g1, c);
    for (int kb = 0; kb < nb; ++kb) {
      KqRow<TYPE> na, nbr;
      if (kb + 1 < nb) {  // next block's rows in flight while this one is decoded
        na.load(g0 + (size_t)(kb + 1) * BB, c);
        nbr.load(g1 + (size_t)(kb + 1) * BB, c);
      }
      if constexpr (TYPE == kKqQ4)
        kq_block_q4<1>(ra, rb, c, xl + (size_t)kb * 256, tok_off, p.xs + (size_t)kb * 8, xs_off, acc);
      else
        kq_block_mma<TYPE, 1>(ra, rb, c, xl + (size_t)kb * 256, tok_off, acc);
      if (MODE == 0) {
        KqRow<TYPE> ua, ub;
        ua.load(u0 + (size_t)kb * BB, c);
        ub.load(u1 + (size_t)kb * BB, c);
        if constexpr (TYPE == kKqQ4)
          kq_block_q4<1>(ua, ub, c, xl + (size_t)kb * 256, tok_off, p.xs + (size_t)kb * 8, xs_off, accu);
        else
          kq_block_mma<TYPE, 1>(ua, ub, c, xl + (size_t)kb * 256, tok_off, accu);
      }
      if (kb + 1 < nb) {
        ra = na;
        rb = nbr;
      }
    }
    // accumulator: rows g / g + 8 of the tile, tokens 2c, 2c + 1
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = 2 * c + (i & 1);
      const int row = 16 * rt + g + ((i & 2) ? 8 : 0);
      if (tok < nrows) {
        float v = acc[0][i];
        if (MODE == 0) v = __fdividef(v, 1.0f + __expf(-v)) * accu[0][i];
        p.out[(size_t)(row0 + tok) * p.R + row] = v;
      }
    }
  }
}

template <int TYPE>
cudaError_t launch_kq_rows_prep_t(const void* in, int in_dtype, const int* row_src, int n, const int* n_dev, int K,
                                  uint16_t* out, float* xs, int n_sm, cudaStream_t st) {
  const long long total = (long long)n * K;
  if (total == 0) return cudaSuccess;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)n_sm * 16);
  return launch_pdl(kq_rows_prep_kernel<TYPE>, grid, 256, 0, st, in, in_dtype, row_src, n, n_dev, K, out, xs);
}

cudaError_t launch_kq_rows_prep(int type, const void* in, int in_dtype, const int* row_src, int n, const int* n_dev,
                                int K, uint16_t* out, float* xs, int n_sm, cudaStream_t st) {
  if (type == kKqQ2) return launch_kq_rows_prep_t<kKqQ2>(in, in_dtype, row_src, n, n_dev, K, out, xs, n_sm, st);
  if (type == kKqQ3) return launch_kq_rows_prep_t<kKqQ3>(in, in_dtype, row_src, n, n_dev, K, out, xs, n_sm, st);
  return launch_kq_rows_prep_t<kKqQ4>(in, in_dtype, row_src, n, n_dev, K, out, xs, n_sm, st);
}

// Grid: enough CTAs for the item count of the worst case (rows / 8 segments
// plus one per expert), capped at two waves of resident CTAs.
cudaError_t launch_kq_moe(int type, int mode, const KqMoeParams& p, int max_items, int n_sm, cudaStream_t st) {
  const int grid = std::max(1, std::min((max_items + kKqWarps - 1) / kKqWarps, 4 * n_sm));
  if (mode == 0) {
    if (type == kKqQ2) return launch_pdl(kq_moe_kernel<kKqQ2, 0>, grid, kKqWarps * 32, 0, st, p);
    if (type == kKqQ3) return launch_pdl(kq_moe_kernel<kKqQ3, 0>, grid, kKqWarps * 32, 0, st, p);
    return launch_pdl(kq_moe_kernel<kKqQ4, 0>, grid, kKqWarps * 32, 0, st, p);
  }
  if (type == kKqQ2) return launch_pdl(kq_moe_kernel<kKqQ2, 1>, grid, kKqWarps * 32, 0, st, p);
  if (type == kKqQ3) return launch_pdl(kq_moe_kernel<kKqQ3, 1>, grid, kKqWarps * 32, 0, st, p);
  return launch_pdl(kq_moe_kernel<kKqQ4, 1>, grid, kKqWarps * 32, 0, st, p);
}

}  // namespace ef

namespace {

struct KqWs {
  float* logits;
  int* inds;
  float* wts;
  PermBufs pb;
  uint16_t* xp;   // routed rows, permuted for the gate / up type [n_rows][H]
  float* xs;      // Q4_K gate / up: their sub-block sums [n_rows][H / 32]
  float* h;       // [n_rows][I]
  uint16_t* hp;   // h permuted for the down type [n_rows][I]
  float* hs;      // Q4_K down: its sub-block sums [n_rows][I / 32]
  float* yrows;   // [n_rows][H]
};

size_t kq_ws(const ef_moe_cfg* cfg, int T, Carver& c, KqWs& w) {
  const int E = cfg->n_experts, k = cfg->top_k, H = cfg->hidden, I = cfg->inter;
  const int n_ent = T * k, n_rows = n_ent + (cfg->n_shared ? T : 0), nb = E + 1;
  const int max_segs = (n_rows + kTokChunk - 1) / kTokChunk + nb + 2;
  w.logits = c.take<float>((size_t)T * E);
  w.inds = c.take<int>((size_t)n_ent);
  w.wts = c.take<float>((size_t)n_ent);
  w.pb.counts = c.take<int>(nb + 1);
  w.pb.offsets = c.take<int>(nb + 2);
  w.pb.row_src = c.take<int>(n_rows + 1);
  w.pb.inv = c.take<int>(n_ent + 1);
  w.pb.seg_expert = c.take<int>(max_segs);
  w.pb.seg_row0 = c.take<int>(max_segs);
  w.pb.seg_nrows = c.take<int>(max_segs);
  w.pb.n_seg = c.take<int>(1);
  w.xp = c.take<uint16_t>((size_t)n_rows * H);
  w.xs = c.take<float>((size_t)n_rows * (H / 32));
  w.h = c.take<float>((size_t)n_rows * I);
  w.hp = c.take<uint16_t>((size_t)n_rows * I);
  w.hs = c.take<float>((size_t)n_rows * (I / 32));
  w.yrows = c.take<float>((size_t)n_rows * H);
  return c.off;
}

bool kq_type_ok(int t) { return t == ef::kKqQ2 || t == ef::kKqQ3 || t == ef::kKqQ4; }

ef_status check_kqw(const ef_kqweight& q, const char* name, int N, int K) {
  if (!q.blocks) return fail(EF_ERR_INVALID, "%s: null pointer", name);
  if (!kq_type_ok(q.type))
    return fail(EF_ERR_UNSUPPORTED, "%s: K-quant type must be Q2_K (10), Q3_K (11) or Q4_K (12), got %d", name,
                q.type);
  const long long matrix = (long long)N * (K / 256) * ef::kq_block_bytes(q.type);
  if (q.expert_stride < matrix)
    return fail(EF_ERR_INVALID, "%s: expert_stride %lld is smaller than one expert's matrix (%lld bytes)", name,
                q.expert_stride, matrix);
  const uintptr_t a = q.type == ef::kKqQ4 ? 15 : (q.type == ef::kKqQ2 ? 3 : 1);
  if ((reinterpret_cast<uintptr_t>(q.blocks) & a) || (q.expert_stride & (long long)a))
    return fail(EF_ERR_INVALID, "%s: blocks and expert_stride must be %d-byte aligned", name, (int)a + 1);
  return EF_OK;
}

}  // namespace

extern "C" {

size_t ef_kquant_moe_workspace_size(const ef_moe_cfg* cfg, int T) {
  if (!cfg || T < 0) return 0;
  Carver c{nullptr};
  KqWs w;
  return kq_ws(cfg, T, c, w) + 256;
}

ef_status ef_kquant_moe_forward(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w,
                                const float* e_bias, ef_kqweight gate, ef_kqweight up, ef_kqweight down,
                                const ef_kqweight* sg, const ef_kqweight* su, const ef_kqweight* sd, void* y,
                                int32_t* inds_out, float* wts_out, void* workspace, size_t ws_bytes, void* stream) {
  if (!cfg) return fail(EF_ERR_INVALID, "cfg is NULL");
  const int H = cfg->hidden, I = cfg->inter, E = cfg->n_experts, k = cfg->top_k;
  if (H <= 0 || H % 256 || I <= 0 || I % 256)
    return fail(EF_ERR_UNSUPPORTED, "hidden and inter must be positive multiples of 256 (K-quant blocks)");
  // routing and layout checks of the 4/8-bit layer (bits / group do not apply to K-quant experts)
  ef_moe_cfg rc = *cfg;
  rc.bits = 4;
  rc.group_size = 64;
  ef_status s = check_cfg(&rc);
  if (s) return s;
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!x || !gate_w || !y) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x) || !aligned16(gate_w) || !aligned16(y)) return fail(EF_ERR_INVALID, "x/gate_w/y must be 16-byte aligned");
  if ((s = check_kqw(gate, "gate", I, H)) || (s = check_kqw(up, "up", I, H)) || (s = check_kqw(down, "down", H, I)))
    return s;
  if (up.type != gate.type) return fail(EF_ERR_UNSUPPORTED, "gate and up must share a K-quant type");
  if (cfg->n_shared) {
    if (!sg || !su || !sd) return fail(EF_ERR_INVALID, "n_shared=1 needs shared_gate/up/down");
    if ((s = check_kqw(*sg, "shared_gate", I, H)) || (s = check_kqw(*su, "shared_up", I, H)) ||
        (s = check_kqw(*sd, "shared_down", H, I)))
      return s;
    if (sg->type != gate.type || su->type != gate.type || sd->type != down.type)
      return fail(EF_ERR_UNSUPPORTED, "the shared expert's K-quant types must match the routed experts'");
  }
  if (!workspace || !aligned16(workspace) || ws_bytes < ef_kquant_moe_workspace_size(cfg, T))
    return fail(EF_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, ef_kquant_moe_workspace_size(cfg, T));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  KqWs w;
  kq_ws(cfg, T, c, w);
  int* inds = inds_out ? inds_out : w.inds;
  float* wts = wts_out ? wts_out : w.wts;
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  const int n_sh = cfg->n_shared ? T : 0, n_rows = T * k + n_sh;
  const int nsm = sm_count();
  EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), bf, static_cast<const uint16_t*>(gate_w),
                                                  cfg->gate_dtype == EF_DT_BF16, T, E, H, w.logits, st));
  EF_LAUNCH("router_select", launch_router_select(w.logits, e_bias, T, E, k, cfg->router_mode, cfg->norm_topk,
                                                  cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->n_group : 1,
                                                  cfg->topk_group,
                                                  cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->routed_scaling : 1.0f,
                                                  inds, wts, st));
  EF_LAUNCH("permute", launch_permute(inds, T * k, k, E, n_sh, kTokChunk, w.pb, st));
  EF_LAUNCH("kq_prep_x", launch_kq_rows_prep(gate.type, x, bf ? EF_DT_BF16 : EF_DT_F16, w.pb.row_src, n_rows,
                                             nullptr, H, w.xp, w.xs, nsm, st));
  const int max_items_gu = ((n_rows + kTokChunk - 1) / kTokChunk + E + 1) * (I / 16);
  KqMoeParams p0;
  memset(&p0, 0, sizeof(p0));
  p0.w0 = static_cast<const uint8_t*>(gate.blocks);
  p0.w1 = static_cast<const uint8_t*>(up.blocks);
  p0.stride0 = gate.expert_stride;
  p0.stride1 = up.expert_stride;
  p0.sw0 = sg ? static_cast<const uint8_t*>(sg->blocks) : p0.w0;
  p0.sw1 = su ? static_cast<const uint8_t*>(su->blocks) : p0.w1;
  p0.xp = w.xp;
  p0.xs = w.xs;
  p0.seg_expert = w.pb.seg_expert; p0.seg_row0 = w.pb.seg_row0; p0.seg_nrows = w.pb.seg_nrows; p0.n_seg = w.pb.n_seg;
  p0.K = H; p0.R = I; p0.n_experts = E; p0.out = w.h;
  EF_LAUNCH("kq_gate_up", launch_kq_moe(gate.type, 0, p0, max_items_gu, nsm, st));
  EF_LAUNCH("kq_prep_h", launch_kq_rows_prep(down.type, w.h, EF_DT_F32, nullptr, n_rows, nullptr, I, w.hp, w.hs, nsm, st));
  KqMoeParams p1 = p0;
  p1.w0 = static_cast<const uint8_t*>(down.blocks);
  p1.w1 = nullptr;
  p1.stride0 = down.expert_stride;
  p1.stride1 = 0;
  p1.sw0 = sd ? static_cast<const uint8_t*>(sd->blocks) : p1.w0;
  p1.sw1 = nullptr;
  p1.xp = w.hp;
  p1.xs = w.hs;
  p1.K = I; p1.R = H; p1.out = w.yrows;
  const int max_items_d = ((n_rows + kTokChunk - 1) / kTokChunk + E + 1) * (H / 16);
  EF_LAUNCH("kq_down", launch_kq_moe(down.type, 1, p1, max_items_d, nsm, st));
  EF_LAUNCH("combine", launch_combine(w.yrows, w.pb.inv, wts, T, k, H, cfg->n_shared ? T * k : -1, y,
                                      cfg->out_f32 ? EF_DT_F32 : (bf ? EF_DT_BF16 : EF_DT_F16), st));
  return EF_OK;
}

}  // extern "C"
