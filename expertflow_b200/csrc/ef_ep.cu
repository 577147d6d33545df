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

// =====================================================================================
// Expert parallelism over NVLink peer memory.
//
// Every rank owns one exchange buffer with the same layout (EpLayout); peers
// map it through CUDA IPC.  Per forward, with epoch e (a device counter that
// the dispatch kernel advances):
//   ep_dispatch_kernel : sorted routed row p of this rank goes to rank d =
//                        expert / e_local, slot q = p - first row for d, as
//                        bf16/fp16 row + (local expert, p) into d's receive
//                        region for this source; the last CTA stores each
//                        destination's row count and releases its flag = e.
//   ep_recv_kernel     : one CTA; waits for every source's flag (bounded),
//                        sorts the received rows by local expert (+ the
//                        shared bin of this rank's own rows) into the FFN's
//                        permutation and records each row's return address.
//   (prep + GEMV/GEMM of the local experts, unchanged)
//   ep_return_kernel   : fp32 output row -> its source's return region at the
//                        source's sorted row p; the last CTA releases the
//                        source's done flag = e.
//   ep_wait_kernel     : waits for every rank's done flag, then the usual
//                        combine reads the return region in k order.
// Buffer reuse needs no extra handshake: a source's next dispatch follows its
// combine, which waited for every destination's done flag, and a destination
// raises it only after its gather of the received rows has completed.
namespace ef {

constexpr int kEpMaxRanks = EF_EP_MAX_RANKS;

struct EpPeers {
  uint8_t* base[kEpMaxRanks];
};

// Byte offsets inside an exchange buffer (identical on every rank) and the
// shape of the exchange.
struct EpGeom {
  int P, rank, el, k, H, T, rmax, max_tokens, has_shared, max_recv;
  unsigned long long off_flags, off_done, off_counts, off_meta, off_rows, off_back, off_local;
  uint32_t* epoch;  // this rank's epoch counter
  uint32_t* ctr;    // [2] last-CTA counters of dispatch and return
};

EF_DEV uint32_t* slot_u32(uint8_t* base, unsigned long long off, int i) {
  return reinterpret_cast<uint32_t*>(base + off + (size_t)i * 64);
}

// One warp copies n16 16-byte units src -> dst (dst may be a peer GPU's
// memory): each lane issues kCopyBatch independent loads before its stores,
// so a row's loads overlap instead of waiting one round trip each.
constexpr int kCopyBatch = 8;
constexpr int kRowParts = 4;  // warps per copied row
EF_DEV void warp_copy16(uint4* dst, const uint4* src, int n16, int lane) {
  for (int c0 = lane; c0 < n16; c0 += 32 * kCopyBatch) {
    uint4 v[kCopyBatch];
#pragma unroll
    for (int u = 0; u < kCopyBatch; ++u)
      if (c0 + 32 * u < n16) v[u] = src[c0 + 32 * u];
#pragma unroll
    for (int u = 0; u < kCopyBatch; ++u)
      if (c0 + 32 * u < n16) dst[c0 + 32 * u] = v[u];
  }
}

// The last CTA of a grid to get here returns true (all CTAs' earlier global
// stores, peer stores included, are then visible system-wide); counter reset.
EF_DEV bool last_cta(uint32_t* ctr, int* s_last) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    *s_last = atomicAdd(ctr, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!*s_last) return false;
  __threadfence_system();
  if (threadIdx.x == 0) *ctr = 0;
  return true;
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __grid_constant__ EpPeers peers, EpGeom g,
                                                          const uint16_t* __restrict__ x,
                                                          const int* __restrict__ row_src,
                                                          const int* __restrict__ offsets) {
  pdl_wait();
  __shared__ int s_off[513];
  __shared__ int s_last;
  const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(g.epoch) + 1u;
  const int E = g.el * g.P;
  const int n = g.T * g.k;
  if (n > 0)
    for (int i = threadIdx.x; i <= E; i += blockDim.x) s_off[i] = offsets[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int h16 = g.H / 8;
  const int part16 = (h16 + kRowParts - 1) / kRowParts;  // 16-byte units per warp's part of a row
  const uint4* xs = reinterpret_cast<const uint4*>(x);
  const size_t row_bytes = (size_t)g.H * 2;
  // work unit = (sorted routed row p, part) and then (own token t, part)
  for (int wu = blockIdx.x * wpb + warp; wu < n * kRowParts; wu += gridDim.x * wpb) {
    const int p = wu / kRowParts, part = wu - p * kRowParts;
    int lo = 0, hi = E;  // the expert of sorted row p: s_off[lo] <= p < s_off[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_off[mid] <= p) lo = mid; else hi = mid;
    }
    const int d = lo / g.el, le = lo - d * g.el;
    const int q = p - s_off[d * g.el];
    if (q >= g.rmax) {  // cannot happen for distinct experts per token
      if (lane == 0) ef_set_error(kDevErrRecvOverflow);
      continue;
    }
    uint8_t* db = peers.base[d];
    uint4* dst = reinterpret_cast<uint4*>(db + g.off_rows + ((size_t)g.rank * g.rmax + q) * row_bytes);
    const uint4* src = xs + (size_t)__ldg(row_src + p) * h16;
    const int c0 = part * part16;
    warp_copy16(dst + c0, src + c0, min(part16, h16 - c0), lane);
    if (lane == 0 && part == 0)
      reinterpret_cast<int2*>(db + g.off_meta)[(size_t)g.rank * g.rmax + q] = make_int2(le, p);
  }
  if (g.has_shared) {  // this rank's own tokens, for its shared-expert bin
    uint8_t* ob = peers.base[g.rank];
    for (int wu = blockIdx.x * wpb + warp; wu < g.T * kRowParts; wu += gridDim.x * wpb) {
      const int t = wu / kRowParts, part = wu - t * kRowParts;
      uint4* dst = reinterpret_cast<uint4*>(ob + g.off_rows + ((size_t)g.P * g.rmax + t) * row_bytes);
      const uint4* src = xs + (size_t)t * h16;
      const int c0 = part * part16;
      warp_copy16(dst + c0, src + c0, min(part16, h16 - c0), lane);
    }
  }
  if (!last_cta(&g.ctr[0], &s_last)) return;
  if (threadIdx.x < g.P) {
    const int d = threadIdx.x;
    const int cnt = n > 0 ? min(s_off[(d + 1) * g.el] - s_off[d * g.el], g.rmax) : 0;
    uint8_t* db = peers.base[d];
    *reinterpret_cast<volatile int*>(slot_u32(db, g.off_counts, g.rank)) = cnt;
    st_release_sys(slot_u32(db, g.off_flags, g.rank), ep);
  }
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(g.epoch) = ep;
}

}  // namespace ef

namespace ef {

// One CTA of kPermThreads.  Received row i (over the sources in rank order)
// is row j of source s's region; it is sorted by local expert into pb (bins
// 0..el-1, then this rank's T own rows as the shared bin when has_shared).
// row_src = row of the receive buffer, ret_rank/ret_row = where its output
// goes (source rank, the source's sorted row; shared rows: this rank, T*k+t).
__global__ void __launch_bounds__(kPermThreads) ep_recv_kernel(EpGeom g, const uint8_t* own,
                                                               int seg_chunk, PermBufs pb, int* __restrict__ ret_rank,
                                                               int* __restrict__ ret_row, int* __restrict__ n_rows) {
  pdl_wait();
  extern __shared__ int s_hist[];
  __shared__ int s_warp[32];
  __shared__ int s_total;
  __shared__ int s_pre[kEpMaxRanks + 1];
  const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(g.epoch);
  if (threadIdx.x < g.P) {
    const int s = threadIdx.x;
    const bool ok = wait_flag_sys(slot_u32(const_cast<uint8_t*>(own), g.off_flags, s), ep);
    int c = ok ? *reinterpret_cast<const volatile int*>(slot_u32(const_cast<uint8_t*>(own), g.off_counts, s)) : 0;
    s_pre[s + 1] = min(max(c, 0), g.rmax);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_pre[0] = 0;
    for (int s = 0; s < g.P; ++s) s_pre[s + 1] += s_pre[s];
    if (s_pre[g.P] > g.max_recv) ef_set_error(kDevErrRecvOverflow);
  }
  __syncthreads();
  const int N = min(s_pre[g.P], g.max_recv);
  // peer-written: plain (coherent) loads after the acquire, not the read-only path
  const volatile int2* meta = reinterpret_cast<const volatile int2*>(own + g.off_meta);
  const int P = g.P, rmax = g.rmax, pmax = g.max_tokens * g.k;
  auto src_row = [&](int i) {  // row of the receive regions holding received row i
    int lo = 0, hi = P;        // s_pre[lo] <= i < s_pre[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_pre[mid] <= i) lo = mid; else hi = mid;
    }
    return lo * rmax + (i - s_pre[lo]);
  };
  counting_sort_cta(
      N, g.el, g.has_shared ? g.T : 0, seg_chunk, pb, s_hist, s_warp, &s_total,
      [&](int i) { return meta[src_row(i)].x; },
      [&](int i, int pos) {
        const int r = src_row(i);
        int p = meta[r].y;
        if (p < 0 || p >= pmax) {
          ef_set_error(kDevErrRange);
          p = 0;
        }
        pb.row_src[pos] = r;
        ret_rank[pos] = r / rmax;
        ret_row[pos] = p;
      },
      [&](int t, int pos) {
        pb.row_src[pos] = P * rmax + t;
        ret_rank[pos] = g.rank;
        ret_row[pos] = g.T * g.k + t;
      });
  if (threadIdx.x == 0) *n_rows = N + (g.has_shared ? g.T : 0);
}

// Output row q (fp32, sorted local order) -> source ret_rank[q]'s return
// region at row ret_row[q]; the last CTA raises every source's done flag.
__global__ void __launch_bounds__(256) ep_return_kernel(const __grid_constant__ EpPeers peers, EpGeom g,
                                                        const float* __restrict__ yrows,
                                                        const int* __restrict__ ret_rank,
                                                        const int* __restrict__ ret_row,
                                                        const int* __restrict__ n_rows_dev, int max_rows) {
  pdl_wait();
  __shared__ int s_last;
  const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(g.epoch);
  const int n = min(max(*n_rows_dev, 0), max_rows);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int h16 = g.H / 4;  // 16-byte units of an fp32 row
  const int part16 = (h16 + kRowParts - 1) / kRowParts;
  const int back_rows = g.max_tokens * g.k + g.max_tokens;
  for (int wu = blockIdx.x * wpb + warp; wu < n * kRowParts; wu += gridDim.x * wpb) {
    const int q = wu / kRowParts, part = wu - q * kRowParts;
    const int s = __ldg(ret_rank + q), p = __ldg(ret_row + q);
    if (s < 0 || s >= g.P || p < 0 || p >= back_rows) continue;  // recorded by ep_recv_kernel
    uint4* dst = reinterpret_cast<uint4*>(peers.base[s] + g.off_back + (size_t)p * g.H * 4);
    const uint4* src = reinterpret_cast<const uint4*>(yrows + (size_t)q * g.H);
    const int c0 = part * part16;
    warp_copy16(dst + c0, src + c0, min(part16, h16 - c0), lane);
  }
  if (!last_cta(&g.ctr[1], &s_last)) return;
  if (threadIdx.x < g.P) st_release_sys(slot_u32(peers.base[threadIdx.x], g.off_done, g.rank), ep);
}

// Waits until every rank has returned this rank's rows for the current epoch.
__global__ void ep_wait_kernel(EpGeom g, const uint8_t* own) {
  pdl_wait();
  const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(g.epoch);
  if (threadIdx.x < g.P) wait_flag_sys(slot_u32(const_cast<uint8_t*>(own), g.off_done, threadIdx.x), ep);
}

}  // namespace ef

struct ef_ep_group {
  ef_moe_cfg cfg;
  int dev = 0, rank = 0, P = 1, max_tokens = 0, rmax = 0, max_recv = 0;
  ef::EpGeom geom;  // T filled per forward
  uint8_t* base = nullptr;
  size_t bytes = 0;
  ef::EpPeers peers;
  uint8_t* mapped[ef::kEpMaxRanks];
  bool opened = false;
};

namespace {

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t kEpLocalTables = 64;  // offset of the pointer tables in the local area

// Layout of an exchange buffer: flags, done flags and counts (64 bytes per
// source rank), the receive metadata and rows ([P][rmax], then this rank's own
// rows for its shared expert), the return region ([max_tokens * k] routed rows
// in the source's sorted order, then max_tokens shared rows) and this rank's
// epoch and last-CTA counters.
size_t ep_layout(ef::EpGeom& g) {
  size_t o = 0;
  g.off_flags = o;
  o = align256(o + (size_t)g.P * 64);
  g.off_done = o;
  o = align256(o + (size_t)g.P * 64);
  g.off_counts = o;
  o = align256(o + (size_t)g.P * 64);
  g.off_meta = o;
  o = align256(o + (size_t)g.P * g.rmax * 8);
  g.off_rows = o;
  o = align256(o + ((size_t)g.P * g.rmax + g.max_tokens) * g.H * 2);
  g.off_back = o;
  o = align256(o + ((size_t)g.max_tokens * g.k + g.max_tokens) * g.H * 4);
  g.off_local = o;  // epoch, 3 last-CTA counters, then the return-region and done-flag tables
  o = align256(o + kEpLocalTables + 2 * kEpMaxRanks * sizeof(void*));
  return o;
}

struct EpWork {
  float* logits;
  int* inds;
  float* wts;
  PermBufs own;      // this rank's entries sorted by (global) expert
  FfnBufs f;         // the received rows' FFN
  int* ret_rank;
  int* ret_row;
  int* n_rows;
};

int ep_rows_max(const ef_ep_group* g) { return g->max_recv + g->max_tokens; }

size_t ep_carve(const ef_ep_group* g, int T, Carver& c, EpWork& w) {
  const int E = g->cfg.n_experts, k = g->cfg.top_k, n_ent = T * k;
  const int el = E / g->P, nr = ep_rows_max(g);
  w.logits = c.take<float>((size_t)T * E);
  w.inds = c.take<int>((size_t)n_ent);
  w.wts = c.take<float>((size_t)n_ent);
  const int own_segs = n_ent / kTokChunk + E + 3;
  w.own.counts = c.take<int>(E + 1);
  w.own.offsets = c.take<int>(E + 2);
  w.own.row_src = c.take<int>(n_ent + 1);
  w.own.inv = c.take<int>(n_ent + 1);
  w.own.seg_expert = c.take<int>(own_segs);
  w.own.seg_row0 = c.take<int>(own_segs);
  w.own.seg_nrows = c.take<int>(own_segs);
  w.own.n_seg = c.take<int>(1);
  carve_ffn(c, 1, el + 1, nr, g->cfg.hidden, g->cfg.inter, w.f);
  w.ret_rank = c.take<int>(nr);
  w.ret_row = c.take<int>(nr);
  w.n_rows = c.take<int>(1);
  return c.off;
}

}  // namespace

extern "C" {

ef_status ef_ep_group_create(const ef_moe_cfg* cfg, int rank, int n_ranks, int max_tokens, int max_recv_rows,
                             ef_ep_group** out) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (!out) return fail(EF_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (n_ranks < 1 || n_ranks > ef::kEpMaxRanks || cfg->n_experts % n_ranks)
    return fail(EF_ERR_INVALID, "n_ranks must divide n_experts and be in 1..%d", ef::kEpMaxRanks);
  if (rank < 0 || rank >= n_ranks) return fail(EF_ERR_INVALID, "rank out of range");
  if (max_tokens < 1 || max_recv_rows < 0) return fail(EF_ERR_INVALID, "max_tokens >= 1, max_recv_rows >= 0");
  if (cfg->n_shared && cfg->shared_inter != cfg->inter) return fail(EF_ERR_UNSUPPORTED, "shared_inter must equal inter");
  const int el = cfg->n_experts / n_ranks;
  const long long rmax = (long long)max_tokens * std::min(cfg->top_k, el);
  const long long worst = rmax * n_ranks;
  if (worst > (1 << 26)) return fail(EF_ERR_UNSUPPORTED, "max_tokens too large for the exchange");
  ef_ep_group* g = new ef_ep_group();
  g->cfg = *cfg;
  g->rank = rank;
  g->P = n_ranks;
  g->max_tokens = max_tokens;
  g->rmax = (int)rmax;
  g->max_recv = max_recv_rows > 0 ? (int)std::min<long long>(max_recv_rows, worst) : (int)worst;
  for (int i = 0; i < ef::kEpMaxRanks; ++i) {
    g->peers.base[i] = nullptr;
    g->mapped[i] = nullptr;
  }
  ef::EpGeom& G = g->geom;
  memset(&G, 0, sizeof(G));
  G.P = n_ranks;
  G.rank = rank;
  G.el = el;
  G.k = cfg->top_k;
  G.H = cfg->hidden;
  G.rmax = g->rmax;
  G.max_tokens = max_tokens;
  G.has_shared = cfg->n_shared ? 1 : 0;
  G.max_recv = g->max_recv;
  g->bytes = ep_layout(G);
  cudaError_t e = cudaGetDevice(&g->dev);
  if (e == cudaSuccess) e = cudaMalloc(&g->base, g->bytes);
  if (e == cudaSuccess) e = cudaMemset(g->base, 0, g->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    const size_t bytes = g->bytes;
    if (g->base) cudaFree(g->base);
    delete g;
    return fail(EF_ERR_CUDA, "exchange buffer (%zu bytes): %s", bytes, cudaGetErrorString(e));
  }
  G.epoch = reinterpret_cast<uint32_t*>(g->base + G.off_local);
  G.ctr = G.epoch + 1;  // [0] dispatch, [1] return kernel, [2] the down GEMV's fused return
  g->peers.base[rank] = g->base;
  *out = g;
  return EF_OK;
}

ef_status ef_ep_group_handle(const ef_ep_group* g, void* handle) {
  if (!g || !handle) return fail(EF_ERR_INVALID, "null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == EF_EP_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  EF_CUDA(cudaIpcGetMemHandle(&h, g->base));
  memcpy(handle, &h, sizeof(h));
  return EF_OK;
}

ef_status ef_ep_group_open(ef_ep_group* g, const void* handles) {
  if (!g || !handles) return fail(EF_ERR_INVALID, "null pointer");
  if (g->opened) return fail(EF_ERR_INVALID, "group already opened");
  const uint8_t* hs = static_cast<const uint8_t*>(handles);
  for (int s = 0; s < g->P; ++s) {
    if (s == g->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hs + (size_t)s * EF_EP_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < s; ++r)
        if (g->mapped[r]) {
          cudaIpcCloseMemHandle(g->mapped[r]);
          g->mapped[r] = nullptr;
          g->peers.base[r] = nullptr;
        }
      return fail(EF_ERR_CUDA, "opening rank %d's exchange buffer: %s", s, cudaGetErrorString(e));
    }
    g->mapped[s] = static_cast<uint8_t*>(p);
    g->peers.base[s] = g->mapped[s];
  }
  // tables the down GEMV's fused return reads: every rank's return region and
  // this rank's done flag in every rank's buffer
  std::vector<uintptr_t> tab(2 * (size_t)g->P);
  for (int s = 0; s < g->P; ++s) {
    tab[s] = reinterpret_cast<uintptr_t>(g->peers.base[s] + g->geom.off_back);
    tab[g->P + s] = reinterpret_cast<uintptr_t>(g->peers.base[s] + g->geom.off_done + (size_t)g->rank * 64);
  }
  const cudaError_t e = cudaMemcpy(g->base + g->geom.off_local + kEpLocalTables, tab.data(),
                                   tab.size() * sizeof(uintptr_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(EF_ERR_CUDA, "return tables: %s", cudaGetErrorString(e));
  g->opened = true;
  return EF_OK;
}

size_t ef_ep_workspace_size(const ef_ep_group* g, int T) {
  if (!g || T < 0) return 0;
  Carver c{nullptr};
  EpWork w;
  return ep_carve(g, T, c, w) + 256;
}

ef_status ef_ep_group_destroy(ef_ep_group* g) {
  if (!g) return EF_OK;
  for (int s = 0; s < ef::kEpMaxRanks; ++s)
    if (g->mapped[s]) cudaIpcCloseMemHandle(g->mapped[s]);
  if (g->base) cudaFree(g->base);
  delete g;
  return EF_OK;
}

}  // extern "C"

extern "C" ef_status ef_ep_forward(ef_ep_group* g, const void* x, int T, const void* gate_w, const float* e_bias,
                                   ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* sg,
                                   const ef_qweight* su, const ef_qweight* sd, void* y, int out_dtype,
                                   int32_t* inds_out, float* wts_out, void* workspace, size_t ws_bytes,
                                   void* stream) {
  if (!g) return fail(EF_ERR_INVALID, "group is NULL");
  if (!g->opened) return fail(EF_ERR_NOT_READY, "ef_ep_group_open has not been called");
  const ef_moe_cfg* cfg = &g->cfg;
  ef_status s;
  if (T < 0 || T > g->max_tokens) return fail(EF_ERR_INVALID, "T=%d outside 0..max_tokens=%d", T, g->max_tokens);
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != g->dev)
    return fail(EF_ERR_INVALID, "the group lives on device %d, the current device is %d", g->dev, dev);
  if (T > 0 && (!x || !gate_w || !y)) return fail(EF_ERR_INVALID, "null pointer");
  if (out_dtype != EF_DT_F32 && out_dtype != cfg->act_dtype)
    return fail(EF_ERR_UNSUPPORTED, "out_dtype must be EF_DT_F32 or the activation dtype");
  if ((x && !aligned16(x)) || (gate_w && !aligned16(gate_w)) || (y && !aligned16(y)))
    return fail(EF_ERR_INVALID, "x/gate_w/y must be 16-byte aligned");
  if ((s = check_qw(gate, "gate")) || (s = check_qw(up, "up")) || (s = check_qw(down, "down"))) return s;
  if (cfg->n_shared) {
    if (!sg || !su || !sd) return fail(EF_ERR_INVALID, "n_shared=1 needs shared_gate/up/down");
    if ((s = check_qw(*sg, "shared_gate")) || (s = check_qw(*su, "shared_up")) || (s = check_qw(*sd, "shared_down")))
      return s;
  }
  if (!workspace || !aligned16(workspace) || ws_bytes < ef_ep_workspace_size(g, T))
    return fail(EF_ERR_WORKSPACE, "workspace too small (%zu < %zu)", ws_bytes, ef_ep_workspace_size(g, T));
  if (smem_check(cfg->bits, cfg->hidden, cfg->inter) > 227 * 1024)
    return fail(EF_ERR_UNSUPPORTED, "hidden/inter too large for the decode kernel");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c{static_cast<uint8_t*>(workspace)};
  EpWork w;
  ep_carve(g, T, c, w);
  int* inds = inds_out ? inds_out : w.inds;
  float* wts = wts_out ? wts_out : w.wts;
  const int H = cfg->hidden, E = cfg->n_experts, k = cfg->top_k, el = E / g->P;
  const bool bf = cfg->act_dtype == EF_DT_BF16;
  const int nsm = sm_count();
  // the local FFN: el experts (+ the shared bin); grouped GEMM when the rows
  // this rank sends (about what it receives) fill the experts
  ef_moe_cfg lc = *cfg;
  lc.n_experts = el;
  const int nr_max = ep_rows_max(g);
  const int rows_expect = T * k + (cfg->n_shared ? T : 0);
  const bool gemm = nr_max >= 128 && use_gemm(&lc, std::max(rows_expect, 128), T * k);
  ef::EpGeom G = g->geom;
  G.T = T;
  if (T > 0) {
    EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), bf,
                                                    static_cast<const uint16_t*>(gate_w),
                                                    cfg->gate_dtype == EF_DT_BF16, T, E, H, w.logits, st));
    EF_LAUNCH("router_select",
              launch_router_select(w.logits, e_bias, T, E, k, cfg->router_mode, cfg->norm_topk,
                                   cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->n_group : 1, cfg->topk_group,
                                   cfg->router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg->routed_scaling : 1.0f, inds, wts,
                                   st));
    EF_LAUNCH("permute", launch_permute(inds, T * k, k, E, 0, kTokChunk, w.own, st));
  }
  {
    const int rows = T * k + (cfg->n_shared ? T : 0);
    const int blocks = std::max(1, std::min((rows * ef::kRowParts + 7) / 8, 4 * nsm));
    EF_LAUNCH("ep_dispatch", launch_pdl(ef::ep_dispatch_kernel, blocks, 256, 0, st, g->peers, G,
                                        static_cast<const uint16_t*>(x), (const int*)w.own.row_src,
                                        (const int*)w.own.offsets));
  }
  {
    const size_t smem = sizeof(int) * (size_t)ef::kPermWarps * (el + 1);
    static std::atomic<bool> attr_set[64];
    EF_LAUNCH("ep_recv", (set_max_smem_once(ef::ep_recv_kernel, 160 * 1024, attr_set) != cudaSuccess
                              ? cudaGetLastError()
                              : launch_pdl(ef::ep_recv_kernel, 1, ef::kPermThreads, smem, st, G,
                                           (const uint8_t*)g->base, gemm ? kGemmSegRows : kSegRows, w.f.pb,
                                           w.ret_rank, w.ret_row, w.n_rows)));
  }
  const uint16_t* recv_rows = reinterpret_cast<const uint16_t*>(g->base + G.off_rows);
  EF_LAUNCH("prep_act", launch_prep_act(recv_rows, w.f.pb.row_src, bf, nr_max, H, cfg->bits, w.f.x16, w.f.xsum, st,
                                        w.n_rows, 4 * nsm));
  const ef_qweight* lsg = cfg->n_shared ? sg : nullptr;
  const ef_qweight* lsu = cfg->n_shared ? su : nullptr;
  const ef_qweight* lsd = cfg->n_shared ? sd : nullptr;
  if (gemm) {
    if ((s = run_experts_gemm(&lc, w.f, nr_max, gate, up, down, lsg, lsu, lsd, st))) return s;
    const int blocks = std::max(1, std::min((nr_max * ef::kRowParts + 7) / 8, 4 * nsm));
    EF_LAUNCH("ep_return", launch_pdl(ef::ep_return_kernel, blocks, 256, 0, st, g->peers, G,
                                      (const float*)w.f.yrows, (const int*)w.ret_rank, (const int*)w.ret_row,
                                      (const int*)w.n_rows, nr_max));
  } else {
    // the down GEMV stores each output row into its source rank's return
    // region itself and its last CTA releases the done flags
    uint8_t* tabs = g->base + G.off_local + kEpLocalTables;
    EpReturn er;
    er.rank = w.ret_rank;
    er.row = w.ret_row;
    er.base = reinterpret_cast<float* const*>(tabs);
    er.flag = reinterpret_cast<uint32_t* const*>(tabs + (size_t)g->P * sizeof(void*));
    er.epoch = G.epoch;
    er.ctr = G.ctr + 2;
    er.ranks = g->P;
    er.rows = g->max_tokens * k + g->max_tokens;
    if ((s = run_experts(&lc, w.f, nr_max, gate, up, down, lsg, lsu, lsd, st, &er))) return s;
  }
  if (T > 0) {  // the combine waits for every rank's done flag itself
    const float* back = reinterpret_cast<const float*>(g->base + G.off_back);
    EF_LAUNCH("combine", launch_combine(back, w.own.inv, wts, T, k, H, cfg->n_shared ? T * k : -1, y, out_dtype,
                                        st, reinterpret_cast<const uint32_t*>(g->base + G.off_done), g->P,
                                        G.epoch));
  } else {  // nothing to combine, but the next dispatch must follow every rank's return
    EF_LAUNCH("ep_wait", launch_pdl(ef::ep_wait_kernel, 1, 64, 0, st, G, (const uint8_t*)g->base));
  }
  return EF_OK;
}
