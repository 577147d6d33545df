// ef_ep.cu -- device side of expert-parallel MoE (experts sharded by rank).
//
// Expert e lives on rank e / (E / n_ranks); the router and the shared expert
// are replicated.  A rank's forward is
//   dispatch : route its tokens, sort the routed entries by expert (the
//              counting sort of ef_permute.cu, so the rows for rank r form one
//              contiguous run), gather the token rows in that order with the
//              destination's local expert id, and count the rows per rank;
//   exchange : all-to-all of the counts, then of the rows (NCCL, host side);
//   experts  : ef_moe_experts_forward on the received rows;
//   exchange : the reverse all-to-all of the fp32 expert outputs;
//   combine  : y[t] = sum_j w[t, j] * back[inv[t, j]] (+ the shared row t).
// The reference runs every expert on one host (ef_engine.py:678-703); the
// partitioning follows the expert-parallel layout of its DeepSeek-V3 target.
#include "ef_common.cuh"

namespace ef {

// send_rows[p] = x[row_src[p]] (H act-dtype columns), p < n_ent;
// send_eid[inv[i]] = entries[i] % e_local.
__global__ void ep_pack_kernel(const uint4* __restrict__ x, int h16, const int* __restrict__ row_src,
                               const int* __restrict__ entries, const int* __restrict__ inv, int n_ent, int e_local,
                               uint4* __restrict__ send_rows, int* __restrict__ send_eid) {
  const long long total = (long long)n_ent * h16;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / h16;
    const long long c = i - p * h16;
    send_rows[i] = x[(long long)__ldg(row_src + p) * h16 + c];
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_ent; i += gridDim.x * blockDim.x)
    send_eid[__ldg(inv + i)] = __ldg(entries + i) % e_local;
}

// counts[r] = rows sorted to rank r's experts
__global__ void ep_counts_kernel(const int* __restrict__ offsets, int n_ranks, int e_local, int* __restrict__ counts) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < n_ranks) counts[r] = offsets[(r + 1) * e_local] - offsets[r * e_local];
}

}  // namespace ef

namespace {

struct EpWs {
  float* logits;
  int* inds;
  PermBufs pb;
};
size_t ep_ws(const ef_moe_cfg* cfg, int T, Carver& c, EpWs& w) {
  const int E = cfg->n_experts, k = cfg->top_k, n_ent = T * k;
  w.logits = c.take<float>((size_t)T * E);
  w.inds = c.take<int>((size_t)n_ent);
  const int max_segs = n_ent / kTokChunk + E + 3;
  w.pb.counts = c.take<int>(E + 1);
  w.pb.offsets = c.take<int>(E + 2);
  w.pb.row_src = c.take<int>(n_ent + 1);
  w.pb.inv = c.take<int>(n_ent + 1);
  w.pb.seg_expert = c.take<int>(max_segs);
  w.pb.seg_row0 = c.take<int>(max_segs);
  w.pb.seg_nrows = c.take<int>(max_segs);
  w.pb.n_seg = c.take<int>(1);
  return c.off;
}

}  // namespace

extern "C" {

size_t ef_ep_dispatch_workspace_size(const ef_moe_cfg* cfg, int T) {
  if (!cfg || T < 0) return 0;
  Carver c{nullptr};
  EpWs w;
  return ep_ws(cfg, T, c, w) + 256;
}

ef_status ef_ep_dispatch(const ef_moe_cfg* cfg, int n_ranks, const void* x, int T, const void* gate_w,
                         const float* e_bias, void* send_rows, int32_t* send_expert, int32_t* send_counts,
                         int32_t* inv_out, float* wts_out, int32_t* inds_out, void* workspace, size_t ws_bytes,
                         void* stream) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (n_ranks < 1 || cfg->n_experts % n_ranks != 0)
    return fail(EF_ERR_INVALID, "n_ranks must divide n_experts (%d, %d)", n_ranks, cfg->n_experts);
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    if (send_counts && cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * n_ranks, st) != cudaSuccess)
      return fail(EF_ERR_CUDA, "memset failed");
    return EF_OK;
  }
  if (!x || !gate_w || !send_rows || !send_expert || !send_counts || !inv_out || !wts_out)
    return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x) || !aligned16(send_rows) || !aligned16(gate_w))
    return fail(EF_ERR_INVALID, "x, gate_w and send_rows must be 16-byte aligned");
  if (ws_bytes < ef_ep_dispatch_workspace_size(cfg, T) || !workspace) return fail(EF_ERR_WORKSPACE, "workspace too small");
  Carver c{static_cast<uint8_t*>(workspace)};
  EpWs w;
  ep_ws(cfg, T, c, w);
  const int E = cfg->n_experts, k = cfg->top_k, H = cfg->hidden, n_ent = T * k;
  int* inds = inds_out ? inds_out : w.inds;
  w.pb.inv = inv_out;
  EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), cfg->act_dtype == EF_DT_BF16,
                                                  static_cast<const uint16_t*>(gate_w), cfg->gate_dtype == EF_DT_BF16, T,
                                                  E, H, w.logits, st));
  EF_LAUNCH("router_select",
            launch_router_select(w.logits, e_bias, T, E, k, cfg->router_mode, cfg->norm_topk,
                                 cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->n_group : 1, cfg->topk_group,
                                 cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->routed_scaling : 1.0f, inds,
                                 wts_out, st));
  EF_LAUNCH("permute", launch_permute(inds, n_ent, k, E, 0, kTokChunk, w.pb, st));
  const int e_local = E / n_ranks;
  const int h16 = H / 8;
  const long long total = (long long)n_ent * h16;
  const int blocks = (int)std::min<long long>((total + 255) / 256, (long long)sm_count() * 8);
  EF_LAUNCH("ep_pack", (ef::ep_pack_kernel<<<std::max(blocks, 1), 256, 0, st>>>(
                            static_cast<const uint4*>(x), h16, w.pb.row_src, inds, inv_out, n_ent, e_local,
                            static_cast<uint4*>(send_rows), send_expert),
                        cudaGetLastError()));
  EF_LAUNCH("ep_counts", (ef::ep_counts_kernel<<<(n_ranks + 127) / 128, 128, 0, st>>>(w.pb.offsets, n_ranks, e_local,
                                                                                       send_counts),
                          cudaGetLastError()));
  return EF_OK;
}

ef_status ef_ep_combine(const ef_moe_cfg* cfg, const float* back_rows, const int32_t* inv, const float* wts, int T,
                        int with_shared, void* y, void* stream) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!back_rows || !inv || !wts || !y) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(back_rows) || !aligned16(y)) return fail(EF_ERR_INVALID, "back_rows and y must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int k = cfg->top_k;
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  EF_LAUNCH("combine", launch_combine(back_rows, inv, wts, T, k, cfg->hidden, with_shared ? T * k : -1, y,
                                      cfg->out_f32 ? EF_DT_F32 : (bf ? EF_DT_BF16 : EF_DT_F16), st));
  return EF_OK;
}

}  // extern "C"
