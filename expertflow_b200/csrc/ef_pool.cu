// ef_pool.cu -- expert residency for streaming decode.
//
// (1) CachePolicy: the reference's FrequencyWeightedCache (ef_engine.py:48-104)
//     restated over integer keys: get() on a hit adds 1.0 to the key's score,
//     put() inserts with score + 1.0, trim() evicts the minimum-score key
//     (first inserted among equal scores, as min() over an insertion-ordered
//     dict does) until size <= budget and then multiplies every score by the
//     decay.  Scores are doubles, so the arithmetic is bit-identical to the
//     Python floats.  An LRU variant evicts the least recently touched key.
// (2) ef_slot_pool: the expert pool lives in pinned host memory; at creation
//     the pool repacks the caller's stacked MLX arrays ([E, ...] per layer)
//     into one contiguous blob per (layer, expert), so a miss is ONE large
//     host-to-device copy (about 50 GB/s on this link, against about 32 GB/s
//     for the nine separate arrays).  Every layer owns `budget + headroom` HBM
//     slots, stored as stacked per-projection arrays so the expert kernels read
//     them like any stacked layer.  A layer forward routes, copies each
//     non-resident expert's blob into a staging ring on the pool's copy stream,
//     scatters the staged blobs into their slots with one kernel, makes the
//     compute stream wait, and runs the experts on slot ids (read by the
//     permute kernel straight from pinned memory, so no small copy queues
//     behind the expert copies).  The optional next-layer gate predicts the
//     next layer's experts from the current input
//     (experiments/ef_v16_prefetch.py:92-113) and their copies are issued
//     right after this layer's expert kernels, so both the host work and the
//     copies overlap those kernels.  trim() runs once per token
//     (ef_pool_end_token), as the reference trims after each token; the
//     headroom slots hold the token's misses until then.
// (3) A pool over an ef_expert_store (ef_pool_create_from_store) keeps only a
//     bounded number of pinned host blobs, the least recently used replaced;
//     an expert in neither HBM nor the host tier is read from the model files
//     by the store's reader threads.  The step starts its own reads and waits
//     for them before it changes any residency state; after this layer's
//     expert kernels, the lookahead starts the reads of the next layer's
//     predicted experts (they run while this layer computes, and their copies
//     into HBM follow when that layer runs).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <set>
#include <thread>
#include <unordered_map>
#include <vector>

namespace ef {

// Learned eviction scorer of the reference's BeladyExpertCache
// (ef_engine.py:107-161): 3 -> H -> H -> 1, SiLU between layers, input
// [1/recency, count/max_count, gap_ema/max_gap]; the cached key with the
// highest score is evicted.  Evaluated in double precision.
struct BeladyNet {
  int hidden = 0;
  bool trained = false;
  std::vector<double> w1, b1, w2, b2, w3;  // w1 [3][H], w2 [H][H], w3 [H]
  double b3 = 0.0;
  static double silu(double x) {
    const double c = std::min(20.0, std::max(-20.0, x));
    return x / (1.0 + std::exp(-c));
  }
  double score(const float (&f)[3]) const {
    std::vector<double> h1(hidden), h2(hidden);
    for (int j = 0; j < hidden; ++j) {
      double z = b1[j];
      for (int i = 0; i < 3; ++i) z += (double)f[i] * w1[(size_t)i * hidden + j];
      h1[j] = silu(z);
    }
    for (int j = 0; j < hidden; ++j) {
      double z = b2[j];
      for (int i = 0; i < hidden; ++i) z += h1[i] * w2[(size_t)i * hidden + j];
      h2[j] = silu(z);
    }
    double sc = b3;
    for (int i = 0; i < hidden; ++i) sc += h2[i] * w3[i];
    return sc;
  }
};

class CachePolicy {
 public:
  CachePolicy(int kind, int budget, double decay) : kind_(kind), budget_(budget), decay_(decay) {}

  bool get(long long key) {
    auto it = ents_.find(key);
    if (it == ents_.end()) return false;
    it->second.score += 1.0;
    it->second.last = ++clock_;
    if (kind_ == EF_POLICY_BELADY) touch(key);
    return true;
  }
  void put(long long key) {
    auto it = ents_.find(key);
    if (it != ents_.end()) {  // a put of a resident key only refreshes it (the dict keeps its place)
      it->second.score += 1.0;
      it->second.last = ++clock_;
    } else {
      Ent e;
      e.score = 1.0;
      e.seq = ++seq_;
      e.last = ++clock_;
      ents_.emplace(key, e);
    }
    if (kind_ == EF_POLICY_BELADY) touch(key);
  }
  bool contains(long long key) const { return ents_.count(key) != 0; }
  int size() const { return (int)ents_.size(); }
  // Evicts down to the budget, then decays (FREQ: scores; BELADY: access
  // counts, truncated to integers); returns the evicted keys in order.
  std::vector<long long> trim() {
    std::vector<long long> out;
    if (kind_ == EF_POLICY_BELADY) {
      while ((int)ents_.size() > budget_) {
        const long long v = belady_victim(nullptr);
        out.push_back(v);
        ents_.erase(v);
      }
      for (auto& kv : recs_) kv.second.count = (long long)((double)kv.second.count * decay_);
      return out;
    }
    while ((int)ents_.size() > budget_) {
      auto victim = ents_.begin();
      for (auto it = ents_.begin(); it != ents_.end(); ++it) {
        if (kind_ == EF_POLICY_LRU) {
          if (it->second.last < victim->second.last) victim = it;
        } else if (it->second.score < victim->second.score ||
                   (it->second.score == victim->second.score && it->second.seq < victim->second.seq)) {
          victim = it;
        }
      }
      out.push_back(victim->first);
      ents_.erase(victim);
    }
    if (kind_ == EF_POLICY_FREQ)
      for (auto& kv : ents_) kv.second.score *= decay_;
    return out;
  }
  // Advances the token clock of the learned policy (BeladyExpertCache.end_token).
  void end_token() { ++token_; }
  // Resident keys, ascending.
  std::vector<long long> keys() const {
    std::vector<long long> k;
    k.reserve(ents_.size());
    for (const auto& kv : ents_) k.push_back(kv.first);
    std::sort(k.begin(), k.end());
    return k;
  }
  // FREQ/LRU: the key's score; BELADY: its eviction score (the predictor's
  // output, or count * decay^recency when untrained).
  double score(long long key) const {
    if (kind_ == EF_POLICY_BELADY) {
      if (!ents_.count(key)) return 0.0;
      if (net_.trained) {
        float f[3];
        features(key, f);
        return net_.score(f);
      }
      return fallback_score(key);
    }
    auto it = ents_.find(key);
    return it == ents_.end() ? 0.0 : it->second.score;
  }
  // Lowest-priority resident key not in `keep` (or -1): the victim an
  // immediate eviction would take.
  long long victim_excluding(const std::vector<char>& keep) const {
    if (kind_ == EF_POLICY_BELADY) return belady_victim(&keep);
    long long best = -1;
    const Ent* be = nullptr;
    for (const auto& kv : ents_) {
      if (kv.first >= 0 && kv.first < (long long)keep.size() && keep[kv.first]) continue;
      const Ent& e = kv.second;
      bool better;
      if (!be) better = true;
      else if (kind_ == EF_POLICY_LRU) better = e.last < be->last;
      else better = e.score < be->score || (e.score == be->score && e.seq < be->seq);
      if (better) {
        best = kv.first;
        be = &e;
      }
    }
    return best;
  }
  void erase(long long key) { ents_.erase(key); }
  void set_net(BeladyNet n) { net_ = std::move(n); }

 private:
  struct Ent {
    double score;
    unsigned long long seq;   // insertion order
    unsigned long long last;  // recency
  };
  struct Rec {  // BeladyExpertCache.access_records entry
    long long last = 0, count = 0;
    double gap_ema = 0.0;
  };
  // BeladyExpertCache._update_access (ef_engine.py:211-220)
  void touch(long long key) {
    Rec& r = recs_[key];
    if (r.count > 0) {
      const double a = 0.7 * r.gap_ema;
      const double b = 0.3 * (double)(token_ - r.last);
      r.gap_ema = a + b;
      max_gap_ = std::max(max_gap_, r.gap_ema);
    }
    r.last = token_;
    r.count += 1;
    max_freq_ = std::max(max_freq_, r.count);
  }
  // BeladyExpertCache._build_features (ef_engine.py:231-241), float32 like the reference
  void features(long long key, float (&f)[3]) const {
    auto it = recs_.find(key);
    const Rec r = it == recs_.end() ? Rec{} : it->second;
    const long long rec = token_ - r.last;
    f[0] = (float)(1.0 / (double)std::max(rec, 1LL));
    f[1] = (float)((double)r.count / (double)std::max(max_freq_, 1LL));
    f[2] = (float)(r.gap_ema / std::max(max_gap_, 1.0));
  }
  double fallback_score(long long key) const {  // count * decay^recency (ef_engine.py:256-260)
    auto it = recs_.find(key);
    const Rec r = it == recs_.end() ? Rec{} : it->second;
    return (double)r.count * std::pow(decay_, (double)(token_ - r.last));
  }
  // BeladyExpertCache.trim's choice (ef_engine.py:243-261): among the
  // resident keys in insertion order, the first with the highest predictor
  // score (trained, more than one key) or the lowest fallback score.
  long long belady_victim(const std::vector<char>* keep) const {
    std::vector<std::pair<unsigned long long, long long>> order;
    order.reserve(ents_.size());
    for (const auto& kv : ents_) {
      if (keep && kv.first >= 0 && kv.first < (long long)keep->size() && (*keep)[kv.first]) continue;
      order.push_back({kv.second.seq, kv.first});
    }
    if (order.empty()) return -1;
    std::sort(order.begin(), order.end());
    const bool learned = net_.trained && ents_.size() > 1;
    long long best = -1;
    double bs = 0.0;
    for (const auto& o : order) {
      double sc;
      if (learned) {
        float f[3];
        features(o.second, f);
        sc = net_.score(f);
      } else {
        sc = fallback_score(o.second);
      }
      if (best < 0 || (learned ? sc > bs : sc < bs)) {
        best = o.second;
        bs = sc;
      }
    }
    return best;
  }
  int kind_, budget_;
  double decay_;
  unsigned long long seq_ = 0, clock_ = 0;
  std::unordered_map<long long, Ent> ents_;
  // learned policy state
  std::unordered_map<long long, Rec> recs_;
  long long token_ = 0, max_freq_ = 1;
  double max_gap_ = 1.0;
  BeladyNet net_;
};

}  // namespace ef

struct ef_cache_policy {
  ef::CachePolicy p;
};

// ------------------------------------------------------------------------------ slot pool
namespace ef {

struct ProjGeom {
  int rows, words, groups;  // per expert
  size_t wbytes() const { return (size_t)rows * words * 4; }
  size_t sbytes() const { return (size_t)rows * groups * 2; }
};

struct LayerSlots {
  uint8_t* base = nullptr;                 // device, n_slots experts (9 arrays each)
  std::vector<int> slot_expert;            // -1: free
  std::vector<int> expert_slot;            // -1: not in HBM
  std::vector<char> staged;                // copied by the lookahead, not yet in the policy
  CachePolicy policy;
  cudaEvent_t ready[2] = {nullptr, nullptr};  // per copy lane: after its last copy into this layer
  cudaEvent_t last_use = nullptr;             // compute stream: after this layer's last expert kernels
  bool has_ready[2] = {false, false}, has_use = false;
  explicit LayerSlots(int kind, int budget, double decay) : policy(kind, budget, decay) {}
};

struct CopyTimer {
  cudaEvent_t a = nullptr, b = nullptr;
  bool stall = false;  // a compute-stream stall on copies, not a copy interval
};

// Staged blobs -> slot arrays.  Blob layout: for each projection j, w then
// scales then biases (9 arrays, each 16-byte aligned); array a of blob i goes
// to dst[a] + slot[i] * bytes[a].
constexpr int kScatterMax = 16;
constexpr int kScatterThreads = 64;
struct ScatterParams {
  const uint8_t* stage;
  size_t blob_bytes;
  int n;
  int slot[kScatterMax];
  uint8_t* dst[9];
  size_t off[10];   // array a starts at off[a] of a blob (16-byte aligned), off[9] = used bytes
  size_t size[9];   // bytes of array a (its stride between slots)
};
__global__ void __launch_bounds__(kScatterThreads) pool_scatter_kernel(const __grid_constant__ ScatterParams p) {
  const int i = blockIdx.y;
  if (i >= p.n) return;
  const uint4* src = reinterpret_cast<const uint4*>(p.stage + (size_t)i * p.blob_bytes);
  const size_t n16 = p.off[9] / 16;
  for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < n16; v += (size_t)gridDim.x * blockDim.x) {
    const size_t o = v * 16;
    int a = 0;
#pragma unroll
    for (int k = 1; k < 9; ++k) a += o >= p.off[k] ? 1 : 0;
    const size_t r = o - p.off[a];
    if (r < p.size[a]) *reinterpret_cast<uint4*>(p.dst[a] + (size_t)p.slot[i] * p.size[a] + r) = src[v];
  }
}

// r[t] += y[t] (when y), then x[t] = r[t] / sqrt(mean(r[t]^2) + eps) in the
// activation dtype (when x): the residual stream and pre-MoE norm between the
// stacked layers of a decode step.  One CTA per token, fixed reduction order.
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ r, const float* __restrict__ y,
                                                                   int H, float eps, int act_bf16,
                                                                   uint16_t* __restrict__ x) {
  pdl_wait();
  pdl_launch_next();
  const size_t base = (size_t)blockIdx.x * H;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    float v = r[base + i];
    if (y) {
      v += y[base + i];
      r[base + i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  if (!x) return;
  __shared__ float part[kNormThreads / 32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += part[w];
  const float inv = rsqrtf(tot / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    const float v = r[base + i] * inv;
    x[base + i] = act_bf16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
  }
}

}  // namespace ef

namespace ef {
// The routed (and predicted) expert ids of a pool step -> mapped pinned host
// memory, then `seq` into the host flag once they are visible there.
__global__ void publish_ids_kernel(const int* __restrict__ inds, const int* __restrict__ pred,
                                   const int* __restrict__ pred2, int n, int* h_inds, int* h_pred, int* h_pred2,
                                   uint32_t* h_flag, uint32_t seq) {
  pdl_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    h_inds[i] = inds[i];
    if (pred) h_pred[i] = pred[i];
    if (pred2) h_pred2[i] = pred2[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(h_flag, seq);
  }
}
}  // namespace ef

struct ef_slot_pool {
  ef_moe_cfg cfg;
  ef_pool_cfg pc;
  int dev = 0;
  int n_slots = 0;
  ef::ProjGeom geom[3];                    // gate, up, down
  size_t expert_bytes = 0;
  std::vector<ef_qweight> host[3];         // caller's stacked arrays, read during ef_pool_create only
  size_t blob_bytes = 0;                   // one expert, 9 arrays
  size_t blob_off[10] = {0};               // array offsets within a blob
  uint8_t* host_blobs = nullptr;           // pinned [n_layers][E] blobs
  // copy lanes: 0 = the step's own misses, 1 = lookahead prefetch; each has its
  // stream, staging ring and scatter batch, so neither waits behind the other
  struct Lane {
    cudaStream_t stream = nullptr;
    uint8_t* stage = nullptr;  // device staging ring, kScatterMax blobs
    int n_staged = 0;
    ef::ScatterParams scat{};
  } lane[2];
  ef::ScatterParams scat{};                // blob layout, copied into each lane's batch
  std::vector<ef::LayerSlots> layers;
  uint8_t* dev_mem = nullptr;
  int32_t* h_inds = nullptr;               // mapped pinned staging: routed ids, predicted ids, slot ids, flag
  int32_t* h_pred = nullptr;
  int32_t* h_slot = nullptr;
  int32_t* h_pred2 = nullptr;
  // the expert kernels of a layer step (permute .. combine) as CUDA graphs,
  // one per (layer, tokens, buffers); run eagerly the first time, captured
  // on cap_stream the second, replayed from then on
  struct TailGraph {
    int layer, T, out_f32;
    const void* x;
    const void* y;
    const void* wts;
    const void* ws;
    int uses;
    cudaGraphExec_t exec;
  };
  std::vector<TailGraph> tails;
  cudaStream_t cap_stream = nullptr;
  int32_t* d_inds = nullptr;               // the same staging as the device addresses it
  uint32_t* h_flag = nullptr;              // sequence number of the last published routing
  uint32_t h_seq = 0;
  int h_cap = 0;
  ef_pool_stats st{};
  // routing trace (ef_pool_record_routing): (layer, expert) pairs in routing
  // order and, per ended token, the number of pairs recorded up to its end
  bool rec_on = false;
  std::vector<int32_t> rec_pairs;
  std::vector<long long> rec_tok_end;
  std::vector<ef::CopyTimer> timers;       // one per copy batch, folded into st.copy_ms on demand
  std::vector<ef::CopyTimer> spare;
  // host tier over a store: host_blobs then holds host_n blobs, replaced
  // least recently used first, instead of every expert of every layer
  ef_expert_store* store = nullptr;
  int host_n = 0;
  std::vector<long long> host_key;             // layer * E + expert, -1: free
  std::vector<unsigned long long> host_last;   // recency
  std::vector<unsigned long long> host_pin;    // the step that needs the blob (not replaced during it)
  std::unique_ptr<ef::ReadTicket[]> host_ticket;
  std::vector<cudaEvent_t> host_copied;        // after the last copy out of the blob
  std::vector<char> host_has_copy;
  std::vector<int> host_free;
  std::set<std::pair<unsigned long long, int>> host_lru;  // (recency, blob) of the occupied blobs
  std::unordered_map<long long, int> host_where;
  unsigned long long host_clock = 0, epoch = 0;
};

namespace {

using ef::CopyTimer;
using ef::LayerSlots;

// device view of slot s of a layer: the 9 arrays at fixed offsets
struct SlotView {
  uint8_t* w[3];
  uint8_t* s[3];
  uint8_t* b[3];
};
SlotView slot_arrays(const ef_slot_pool* P, const LayerSlots& L) {
  // layout per layer: for each projection, [n_slots] w, then [n_slots] s, then [n_slots] b
  SlotView v;
  uint8_t* p = L.base;
  for (int j = 0; j < 3; ++j) {
    v.w[j] = p;
    p += (size_t)P->n_slots * P->geom[j].wbytes();
    v.s[j] = p;
    p += (size_t)P->n_slots * P->geom[j].sbytes();
    v.b[j] = p;
    p += (size_t)P->n_slots * P->geom[j].sbytes();
  }
  return v;
}

void fold_timers(ef_slot_pool* P, bool all) {
  size_t keep_from = 0;
  for (size_t i = 0; i < P->timers.size(); ++i) {
    CopyTimer& t = P->timers[i];
    if (!all && cudaEventQuery(t.b) != cudaSuccess) {
      keep_from = i;
      break;
    }
    if (all) cudaEventSynchronize(t.b);
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, t.a, t.b) == cudaSuccess) (t.stall ? P->st.copy_wait_ms : P->st.copy_ms) += ms;
    P->spare.push_back(t);
    keep_from = i + 1;
  }
  P->timers.erase(P->timers.begin(), P->timers.begin() + keep_from);
}

CopyTimer timer_begin(ef_slot_pool* P, cudaStream_t cs) {
  if (P->timers.size() > 256) fold_timers(P, false);
  CopyTimer t;
  if (!P->spare.empty()) {
    t = P->spare.back();
    P->spare.pop_back();
  } else {
    cudaEventCreate(&t.a);
    cudaEventCreate(&t.b);
  }
  t.stall = false;
  cudaEventRecord(t.a, cs);
  return t;
}

// Scatter the staged blobs into their slots (one kernel on the copy stream).
ef_status flush_stage(ef_slot_pool* P, int ln) {
  auto& C = P->lane[ln];
  if (C.n_staged == 0) return EF_OK;
  C.scat.n = C.n_staged;
  // 64-thread blocks (2,048 registers) fit beside two decode-GEMV CTAs on an
  // SM (4,096 registers left), so the scatter runs while the experts of the
  // current layer compute instead of waiting for them to finish
  dim3 grid(256, C.n_staged);
  ef::pool_scatter_kernel<<<grid, ef::kScatterThreads, 0, C.stream>>>(C.scat);
  C.n_staged = 0;
  if (cudaGetLastError() != cudaSuccess) return fail(EF_ERR_CUDA, "slot scatter launch failed");
  return EF_OK;
}

// Copy expert e of layer l into slot s: one blob copy into the staging ring
// (the scatter into the slot arrays follows in flush_stage).  h: the expert's
// host-tier blob in a pool over a store (read complete), else -1.
ef_status copy_expert(ef_slot_pool* P, int ln, int l, int e, int s, int h) {
  LayerSlots& L = P->layers[l];
  auto& C = P->lane[ln];
  if (C.n_staged == ef::kScatterMax) {
    ef_status st = flush_stage(P, ln);
    if (st) return st;
  }
  if (C.n_staged == 0) {  // the ring now holds this layer's blobs
    const SlotView v = slot_arrays(P, L);
    for (int j = 0; j < 3; ++j) {
      C.scat.dst[3 * j] = v.w[j];
      C.scat.dst[3 * j + 1] = v.s[j];
      C.scat.dst[3 * j + 2] = v.b[j];
    }
  }
  const uint8_t* src = P->host_blobs + (h >= 0 ? (size_t)h : (size_t)l * P->cfg.n_experts + e) * P->blob_bytes;
  if (cudaMemcpyAsync(C.stage + (size_t)C.n_staged * P->blob_bytes, src, P->blob_bytes, cudaMemcpyHostToDevice,
                      C.stream) != cudaSuccess)
    return fail(EF_ERR_CUDA, "expert copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  if (h >= 0) {
    cudaEventRecord(P->host_copied[h], C.stream);
    P->host_has_copy[h] = 1;
  }
  C.scat.slot[C.n_staged++] = s;
  L.slot_expert[s] = e;
  L.expert_slot[e] = s;
  P->st.h2d_bytes += (double)P->expert_bytes;
  return EF_OK;
}

// A free slot of layer l, else the slot of a staged (prefetched, unused)
// expert not in `keep` (then *from_staged is set); -1 when neither exists.
int take_slot(ef_slot_pool* P, int l, const std::vector<char>& keep, bool* from_staged = nullptr) {
  LayerSlots& L = P->layers[l];
  for (int s = 0; s < P->n_slots; ++s)
    if (L.slot_expert[s] < 0) return s;
  for (int s = 0; s < P->n_slots; ++s) {
    const int e = L.slot_expert[s];
    if (L.staged[e] && !keep[e]) {
      if (from_staged) *from_staged = true;
      L.staged[e] = 0;
      L.expert_slot[e] = -1;
      L.slot_expert[s] = -1;
      return s;
    }
  }
  return -1;
}

// ---- host tier (pools over a store)
int host_find(const ef_slot_pool* P, int l, int e) {
  auto it = P->host_where.find((long long)l * P->cfg.n_experts + e);
  return it == P->host_where.end() ? -1 : it->second;
}

void host_touch(ef_slot_pool* P, int h) {
  P->host_lru.erase({P->host_last[h], h});
  P->host_last[h] = ++P->host_clock;
  P->host_lru.insert({P->host_last[h], h});
  P->host_pin[h] = P->epoch;
}

void host_drop(ef_slot_pool* P, int h) {
  P->host_where.erase(P->host_key[h]);
  P->host_lru.erase({P->host_last[h], h});
  P->host_key[h] = -1;
  P->host_free.push_back(h);
}

// Expert e of layer l in the host tier, pinned for this step: found, or its
// read from the files started into a free or the least recently used blob
// that this step does not need.  Returns the blob, or -1 when none can be
// replaced.
int host_fetch(ef_slot_pool* P, int l, int e, bool ahead) {
  int h = host_find(P, l, e);
  if (h >= 0) {
    host_touch(P, h);
    P->st.host_hits++;
    return h;
  }
  if (!P->host_free.empty()) {
    h = P->host_free.back();
    P->host_free.pop_back();
  } else {
    for (const auto& it : P->host_lru) {
      const int c = it.second;
      if (P->host_pin[c] != P->epoch && ef::store_done(&P->host_ticket[c])) {
        h = c;
        break;
      }
    }
    if (h < 0 && !ahead) {  // only reads in flight are left to replace: take the oldest once it lands
      for (const auto& it : P->host_lru) {
        if (P->host_pin[it.second] != P->epoch) {
          h = it.second;
          ef::store_wait(P->store, &P->host_ticket[h], 0, 0);
          break;
        }
      }
    }
    if (h < 0) return -1;
    host_drop(P, h);
    P->host_free.pop_back();
    P->st.host_evictions++;
  }
  if (P->host_has_copy[h]) {  // a copy out of the blob may still be in flight
    cudaEventSynchronize(P->host_copied[h]);
    P->host_has_copy[h] = 0;
  }
  const long long key = (long long)l * P->cfg.n_experts + e;
  P->host_key[h] = key;
  P->host_where[key] = h;
  P->host_last[h] = ++P->host_clock;
  P->host_lru.insert({P->host_last[h], h});
  P->host_pin[h] = P->epoch;
  ef::store_submit(P->store, l, e, P->host_blobs + (size_t)h * P->blob_bytes, &P->host_ticket[h]);
  P->st.host_reads++;
  if (ahead) P->st.host_reads_ahead++;
  return h;
}

// Waits for blob h's read; a failed read leaves the tier (the next request reads again).
ef_status host_ready(ef_slot_pool* P, int h, int l, int e) {
  ef::ReadTicket* t = &P->host_ticket[h];
  ef_status s;
  if (!ef::store_done(t)) {
    const auto t0 = std::chrono::steady_clock::now();
    s = ef::store_wait(P->store, t, l, e);
    P->st.read_wait_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  } else {
    s = ef::store_wait(P->store, t, l, e);
  }
  if (s) host_drop(P, h);
  return s;
}

void copies_begin(ef_slot_pool* P, int ln, LayerSlots& L) {
  // a slot may still be read by the layer's previous expert kernels
  if (L.has_use) cudaStreamWaitEvent(P->lane[ln].stream, L.last_use, 0);
}

std::vector<int> distinct_sorted(const int32_t* ids, int n, int E) {
  std::vector<int> d;
  d.reserve(n);
  for (int i = 0; i < n; ++i)
    if (ids[i] >= 0 && ids[i] < E) d.push_back(ids[i]);
  std::sort(d.begin(), d.end());
  d.erase(std::unique(d.begin(), d.end()), d.end());
  return d;
}

struct PoolWs {
  float* logits;
  int* inds;
  float* wts;
  float* plogits[2];  // lookahead predictions: the next layer, the one after it
  int* pinds[2];
  float* pwts[2];
  FfnBufs f;
};
size_t pool_ws(const ef_slot_pool* P, int T, Carver& c, PoolWs& w) {
  const ef_moe_cfg& cfg = P->cfg;
  const int E = cfg.n_experts, k = cfg.top_k;
  const int n_ent = T * k, n_rows = n_ent + (cfg.n_shared ? T : 0);
  w.logits = c.take<float>((size_t)T * E);
  w.inds = c.take<int>((size_t)n_ent);
  w.wts = c.take<float>((size_t)n_ent);
  for (int a = 0; a < 2; ++a) {
    w.plogits[a] = c.take<float>((size_t)T * E);
    w.pinds[a] = c.take<int>((size_t)n_ent);
    w.pwts[a] = c.take<float>((size_t)n_ent);
  }
  carve_ffn(c, n_ent, P->n_slots + 1, n_rows, cfg.hidden, cfg.inter, w.f);
  return c.off;
}

// Routes x through gate gw (and, when gw2 / gw3, the next layers' gates in the
// same two launches: those routings are the lookahead predictions).
// Polls the host flag until the routing of step `seq` is published (bounded:
// the stream's errors are checked every millisecond or so, and 30 s without
// the flag is an error).
ef_status wait_published(const uint32_t* flag, uint32_t seq, cudaStream_t st) {
  const auto t0 = std::chrono::steady_clock::now();
  for (uint32_t i = 0;; ++i) {
    if ((int)(*reinterpret_cast<const volatile uint32_t*>(flag) - seq) >= 0) break;
    if ((i & 4095u) == 4095u) {
      const cudaError_t e = cudaStreamQuery(st);
      if (e != cudaSuccess && e != cudaErrorNotReady) return fail(EF_ERR_CUDA, "routing failed: %s", cudaGetErrorString(e));
      if (e == cudaSuccess && (int)(*reinterpret_cast<const volatile uint32_t*>(flag) - seq) < 0)
        return fail(EF_ERR_CUDA, "routing finished without publishing its ids");
      if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(30))
        return fail(EF_ERR_TIMEOUT, "routing ids not published within 30 s");
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  return EF_OK;
}

ef_status pool_route(const ef_moe_cfg& cfg, const void* x, int T, const void* gw, const float* eb, float* logits, int* inds,
                     float* wts, const void* gw2, const float* eb2, float* logits2, int* inds2, float* wts2,
                     const void* gw3, const float* eb3, float* logits3, int* inds3, float* wts3, cudaStream_t st) {
  const bool bf = cfg.act_dtype == EF_DT_BF16;
  EF_LAUNCH("router_logits", launch_router_logits(static_cast<const uint16_t*>(x), bf, static_cast<const uint16_t*>(gw),
                                                  cfg.gate_dtype == EF_DT_BF16, T, cfg.n_experts, cfg.hidden, logits, st,
                                                  static_cast<const uint16_t*>(gw2), gw2 ? logits2 : nullptr,
                                                  static_cast<const uint16_t*>(gw3), gw3 ? logits3 : nullptr));
  EF_LAUNCH("router_select",
            launch_router_select(logits, eb, T, cfg.n_experts, cfg.top_k, cfg.router_mode, cfg.norm_topk,
                                 cfg.router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg.n_group : 1, cfg.topk_group,
                                 cfg.router_mode == EF_ROUTER_SIGMOID_GROUP ? cfg.routed_scaling : 1.0f, inds, wts, st,
                                 gw2 ? logits2 : nullptr, eb2, inds2, wts2, gw3 ? logits3 : nullptr, eb3, inds3, wts3));
  return EF_OK;
}

ef_status make_net(int hidden, const float* w1, const float* b1, const float* w2, const float* b2, const float* w3,
                   const float* b3, int trained, ef::BeladyNet& n) {
  if (hidden < 1 || hidden > 4096) return fail(EF_ERR_INVALID, "hidden must be in 1..4096");
  if (!w1 || !b1 || !w2 || !b2 || !w3 || !b3) return fail(EF_ERR_INVALID, "null predictor weight");
  const size_t H = (size_t)hidden;
  n.hidden = hidden;
  n.trained = trained != 0;
  n.w1.assign(w1, w1 + 3 * H);
  n.b1.assign(b1, b1 + H);
  n.w2.assign(w2, w2 + H * H);
  n.b2.assign(b2, b2 + H);
  n.w3.assign(w3, w3 + H);
  n.b3 = b3[0];
  return EF_OK;
}

ef_status check_pool_cfg(const ef_moe_cfg* cfg, const ef_pool_cfg* pc) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (!pc) return fail(EF_ERR_INVALID, "null pointer");
  if (pc->n_layers <= 0 || pc->budget < 0 || pc->headroom < cfg->top_k)
    return fail(EF_ERR_INVALID, "need n_layers > 0, budget >= 0, headroom >= top_k");
  if (pc->policy != EF_POLICY_FREQ && pc->policy != EF_POLICY_LRU && pc->policy != EF_POLICY_BELADY)
    return fail(EF_ERR_INVALID, "unknown policy");
  if (cfg->n_shared) return fail(EF_ERR_UNSUPPORTED, "the slot pool streams routed experts only (n_shared = 0)");
  return EF_OK;
}

// The pool without its host contents: HBM slots, the two copy lanes (stream
// + staging ring), n_host_blobs pinned host blobs and the per-layer state.
ef_status pool_alloc(const ef_moe_cfg* cfg, const ef_pool_cfg* pc, size_t n_host_blobs, ef_slot_pool** out) {
  const int E = cfg->n_experts;
  const int n_slots = std::min(E, pc->budget + pc->headroom);
  ef_slot_pool* P = new ef_slot_pool();
  P->cfg = *cfg;
  P->pc = *pc;
  P->n_slots = n_slots;
  cudaGetDevice(&P->dev);
  const int H = cfg->hidden, I = cfg->inter, b = cfg->bits;
  P->geom[0] = {I, H * b / 32, H / 64};
  P->geom[1] = P->geom[0];
  P->geom[2] = {H, I * b / 32, I / 64};
  for (int j = 0; j < 3; ++j) P->expert_bytes += P->geom[j].wbytes() + 2 * P->geom[j].sbytes();
  const ef::BlobLayout lay = ef::blob_layout(*cfg);
  for (int a = 0; a < 10; ++a) P->blob_off[a] = P->scat.off[a] = lay.off[a];
  for (int a = 0; a < 9; ++a) P->scat.size[a] = lay.size[a];
  P->blob_bytes = P->scat.blob_bytes = lay.bytes;
  const size_t per_layer = (size_t)n_slots * P->expert_bytes;
  if (cudaMalloc(&P->dev_mem, per_layer * pc->n_layers) != cudaSuccess ||
      cudaMalloc(&P->lane[0].stage, (size_t)ef::kScatterMax * P->blob_bytes) != cudaSuccess ||
      cudaMalloc(&P->lane[1].stage, (size_t)ef::kScatterMax * P->blob_bytes) != cudaSuccess) {
    cudaGetLastError();
    ef_pool_destroy(P);
    return fail(EF_ERR_CUDA, "slot pool: cannot allocate %zu bytes of HBM", per_layer * pc->n_layers);
  }
  const size_t host_bytes = n_host_blobs * P->blob_bytes;
  if (cudaMallocHost(&P->host_blobs, host_bytes) != cudaSuccess) {
    cudaGetLastError();
    P->host_blobs = nullptr;
    ef_pool_destroy(P);
    return fail(EF_ERR_CUDA, "slot pool: cannot pin %zu bytes of host memory", host_bytes);
  }
  for (int ln = 0; ln < 2; ++ln) {
    P->lane[ln].scat = P->scat;
    P->lane[ln].scat.stage = P->lane[ln].stage;
    if (cudaStreamCreateWithFlags(&P->lane[ln].stream, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      ef_pool_destroy(P);
      return fail(EF_ERR_CUDA, "slot pool: stream creation failed");
    }
  }
  P->layers.reserve(pc->n_layers);
  for (int l = 0; l < pc->n_layers; ++l) {
    P->layers.emplace_back(pc->policy, pc->budget, pc->decay);
    LayerSlots& L = P->layers.back();
    L.base = P->dev_mem + per_layer * l;
    L.slot_expert.assign(n_slots, -1);
    L.expert_slot.assign(E, -1);
    L.staged.assign(E, 0);
    cudaEventCreateWithFlags(&L.ready[0], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&L.ready[1], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&L.last_use, cudaEventDisableTiming);
  }
  *out = P;
  return EF_OK;
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- policy (host only)
ef_status ef_policy_create(int kind, int budget, double decay, ef_cache_policy** out) {
  if (!out) return fail(EF_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (kind != EF_POLICY_FREQ && kind != EF_POLICY_LRU && kind != EF_POLICY_BELADY)
    return fail(EF_ERR_INVALID, "unknown policy %d", kind);
  if (budget < 0) return fail(EF_ERR_INVALID, "budget < 0");
  *out = new ef_cache_policy{ef::CachePolicy(kind, budget, decay)};
  return EF_OK;
}
int ef_policy_get(ef_cache_policy* p, long long key) { return p && p->p.get(key) ? 1 : 0; }
void ef_policy_put(ef_cache_policy* p, long long key) {
  if (p) p->p.put(key);
}
int ef_policy_trim(ef_cache_policy* p, long long* evicted, int cap) {
  if (!p) return -1;
  const std::vector<long long> ev = p->p.trim();
  for (int i = 0; i < (int)ev.size() && i < cap && evicted; ++i) evicted[i] = ev[i];
  return (int)ev.size();
}
int ef_policy_size(const ef_cache_policy* p) { return p ? p->p.size() : -1; }
int ef_policy_keys(const ef_cache_policy* p, long long* keys, int cap) {
  if (!p) return -1;
  const std::vector<long long> k = p->p.keys();
  for (int i = 0; i < (int)k.size() && i < cap && keys; ++i) keys[i] = k[i];
  return (int)k.size();
}
double ef_policy_score(const ef_cache_policy* p, long long key) { return p ? p->p.score(key) : 0.0; }
void ef_policy_end_token(ef_cache_policy* p) {
  if (p) p->p.end_token();
}
ef_status ef_policy_set_predictor(ef_cache_policy* p, int hidden, const float* w1, const float* b1, const float* w2,
                                  const float* b2, const float* w3, const float* b3, int trained) {
  if (!p) return fail(EF_ERR_INVALID, "policy is NULL");
  ef::BeladyNet n;
  ef_status s = make_net(hidden, w1, b1, w2, b2, w3, b3, trained, n);
  if (s) return s;
  p->p.set_net(std::move(n));
  return EF_OK;
}
void ef_policy_destroy(ef_cache_policy* p) { delete p; }

// ---------------------------------------------------------------- slot pool
ef_status ef_pool_create(const ef_moe_cfg* cfg, const ef_pool_cfg* pc, const ef_qweight* host_gate,
                         const ef_qweight* host_up, const ef_qweight* host_down, ef_slot_pool** out) {
  if (!out) return fail(EF_ERR_INVALID, "out is NULL");
  *out = nullptr;
  ef_status s = check_pool_cfg(cfg, pc);
  if (s) return s;
  if (!host_gate || !host_up || !host_down) return fail(EF_ERR_INVALID, "null pointer");
  const int E = cfg->n_experts;
  for (int l = 0; l < pc->n_layers; ++l) {
    const ef_qweight* qs[3] = {&host_gate[l], &host_up[l], &host_down[l]};
    for (int j = 0; j < 3; ++j) {
      if (!qs[j]->w || !qs[j]->scales || !qs[j]->biases) return fail(EF_ERR_INVALID, "layer %d: null host array", l);
      for (const void* ptr : {(const void*)qs[j]->w, (const void*)qs[j]->scales, (const void*)qs[j]->biases}) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
          cudaGetLastError();
          return fail(EF_ERR_INVALID, "layer %d: cannot query an expert array pointer", l);
        }
        if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged)
          return fail(EF_ERR_INVALID, "layer %d: expert pool arrays must be host memory", l);
      }
    }
  }
  ef_slot_pool* P = nullptr;
  if ((s = pool_alloc(cfg, pc, (size_t)pc->n_layers * E, &P))) return s;
  for (int j = 0; j < 3; ++j) P->host[j].assign((j == 0 ? host_gate : j == 1 ? host_up : host_down),
                                                 (j == 0 ? host_gate : j == 1 ? host_up : host_down) + pc->n_layers);
  {  // repack the stacked arrays into per-expert blobs, layers in parallel
    const int nt = std::max(1, std::min(16, (int)std::thread::hardware_concurrency()));
    std::vector<std::thread> th;
    for (int t = 0; t < nt; ++t) {
      th.emplace_back([P, t, nt, E]() {
        for (int l = t; l < P->pc.n_layers; l += nt) {
          for (int e = 0; e < E; ++e) {
            uint8_t* dst = P->host_blobs + ((size_t)l * E + e) * P->blob_bytes;
            for (int j = 0; j < 3; ++j) {
              const ef_qweight& h = P->host[j][l];
              const ef::ProjGeom& g = P->geom[j];
              memcpy(dst + P->blob_off[3 * j], reinterpret_cast<const uint8_t*>(h.w) + (size_t)e * g.wbytes(), g.wbytes());
              memcpy(dst + P->blob_off[3 * j + 1], reinterpret_cast<const uint8_t*>(h.scales) + (size_t)e * g.sbytes(), g.sbytes());
              memcpy(dst + P->blob_off[3 * j + 2], reinterpret_cast<const uint8_t*>(h.biases) + (size_t)e * g.sbytes(), g.sbytes());
            }
          }
        }
      });
    }
    for (auto& x : th) x.join();
  }
  for (int j = 0; j < 3; ++j) P->host[j].clear();  // the caller's arrays are not read again
  *out = P;
  return EF_OK;
}

ef_status ef_pool_create_from_store(const ef_moe_cfg* cfg, const ef_pool_cfg* pc, ef_expert_store* store,
                                    int host_blobs, ef_slot_pool** out) {
  if (!out) return fail(EF_ERR_INVALID, "out is NULL");
  *out = nullptr;
  ef_status s = check_pool_cfg(cfg, pc);
  if (s) return s;
  if (!store) return fail(EF_ERR_INVALID, "store is NULL");
  const ef_moe_cfg& sc = store->cfg;
  if (sc.hidden != cfg->hidden || sc.inter != cfg->inter || sc.bits != cfg->bits || sc.n_experts != cfg->n_experts)
    return fail(EF_ERR_INVALID, "the store's layer shape differs from cfg");
  if (store->n_layers != pc->n_layers) return fail(EF_ERR_INVALID, "the store holds %d layers, the pool %d",
                                                   store->n_layers, pc->n_layers);
  if (host_blobs < 2 * cfg->top_k) return fail(EF_ERR_INVALID, "host_blobs must be >= 2 * top_k");
  host_blobs = (int)std::min<long long>(host_blobs, (long long)pc->n_layers * cfg->n_experts);
  ef_slot_pool* P = nullptr;
  if ((s = pool_alloc(cfg, pc, (size_t)host_blobs, &P))) return s;
  P->store = store;
  P->host_n = host_blobs;
  P->host_key.assign(host_blobs, -1);
  P->host_last.assign(host_blobs, 0);
  P->host_pin.assign(host_blobs, 0);
  P->host_ticket.reset(new ef::ReadTicket[host_blobs]);
  P->host_copied.assign(host_blobs, nullptr);
  P->host_has_copy.assign(host_blobs, 0);
  for (int h = host_blobs - 1; h >= 0; --h) P->host_free.push_back(h);
  for (int h = 0; h < host_blobs; ++h) {
    if (cudaEventCreateWithFlags(&P->host_copied[h], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      ef_pool_destroy(P);
      return fail(EF_ERR_CUDA, "slot pool: event creation failed");
    }
  }
  *out = P;
  return EF_OK;
}

size_t ef_pool_workspace_size(const ef_slot_pool* P, int T) {
  if (!P || T < 0) return 0;
  Carver c{nullptr};
  PoolWs w;
  return pool_ws(P, T, c, w) + 256;
}

namespace {
void drop_tail_graphs(ef_slot_pool* P) {
  for (auto& g : P->tails)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  P->tails.clear();
}

// The layer step's expert kernels on the slot arrays (slot ids in the pinned
// staging, which the host rewrites before each launch): replayed from a CUDA
// graph once the same layer has run with the same buffers, so the host issues
// one launch instead of five kernel launches and their tensor-map encodes.
ef_status run_tail(ef_slot_pool* P, int layer, const ef_moe_cfg& sc, const void* x, int T, const float* wts,
                   const ef_qweight& qg, const ef_qweight& qu, const ef_qweight& qd, const FfnBufs& f, void* y,
                   const void* ws, cudaStream_t st) {
  if (g_trace_on)  // traced launches record events per kernel: run them eagerly
    return moe_tail(&sc, x, T, P->h_slot, wts, qg, qu, qd, nullptr, nullptr, nullptr, f, y, st);
  ef_slot_pool::TailGraph* g = nullptr;
  for (auto& t : P->tails)
    if (t.layer == layer && t.T == T && t.out_f32 == sc.out_f32 && t.x == x && t.y == y && t.wts == wts && t.ws == ws) {
      g = &t;
      break;
    }
  if (!g) {
    if (P->tails.size() >= 4096) drop_tail_graphs(P);  // buffers keep changing: start over
    P->tails.push_back({layer, T, sc.out_f32, x, y, wts, ws, 0, nullptr});
    g = &P->tails.back();
  }
  if (!g->exec && g->uses++ == 0)
    return moe_tail(&sc, x, T, P->h_slot, wts, qg, qu, qd, nullptr, nullptr, nullptr, f, y, st);
  if (!g->exec) {
    if (!P->cap_stream && cudaStreamCreateWithFlags(&P->cap_stream, cudaStreamNonBlocking) != cudaSuccess)
      return fail(EF_ERR_CUDA, "slot pool: capture stream creation failed");
    if (cudaStreamBeginCapture(P->cap_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
      return fail(EF_ERR_CUDA, "slot pool: stream capture failed to start");
    const ef_status s = moe_tail(&sc, x, T, P->h_slot, wts, qg, qu, qd, nullptr, nullptr, nullptr, f, y, P->cap_stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(P->cap_stream, &graph);
    if (s) {
      if (graph) cudaGraphDestroy(graph);
      return s;
    }
    if (e != cudaSuccess || !graph) return fail(EF_ERR_CUDA, "slot pool: capture failed: %s", cudaGetErrorString(e));
    const cudaError_t ei = cudaGraphInstantiate(&g->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) {
      g->exec = nullptr;
      return fail(EF_ERR_CUDA, "slot pool: graph instantiation failed: %s", cudaGetErrorString(ei));
    }
  }
  if (cudaGraphLaunch(g->exec, st) != cudaSuccess)
    return fail(EF_ERR_CUDA, "slot pool: graph launch failed: %s", cudaGetErrorString(cudaGetLastError()));
  return EF_OK;
}

// Copies ahead the experts predicted for layer nl that are not in its slots
// (staged: they enter the policy only when a step uses them).  In a pool over
// a store, an expert not yet in the host tier has its read started instead,
// and is copied when a later prediction or its layer finds it there.
ef_status stage_ahead(ef_slot_pool* P, int nl, const int32_t* pred_ids, int n) {
  const int E = P->cfg.n_experts;
  LayerSlots& N = P->layers[nl];
  const std::vector<int> pred = distinct_sorted(pred_ids, n, E);
  std::vector<char> nkeep(E, 0);
  for (int e : pred) nkeep[e] = 1;
  bool any = false;
  CopyTimer t{};
  ef_status s;
  for (int e : pred) {
    if (N.expert_slot[e] >= 0) continue;
    int h = -1;
    if (P->store) {
      h = host_find(P, nl, e);
      if (h < 0) {
        host_fetch(P, nl, e, true);  // -1 (no blob to replace): the prediction is only a hint
        continue;
      }
      if (!ef::store_done(&P->host_ticket[h]) || P->host_ticket[h].err.load()) continue;
      host_touch(P, h);
      P->st.host_hits++;
    }
    const int sl = take_slot(P, nl, nkeep);
    if (sl < 0) break;  // no free slot: the prediction is only a hint
    if (!any) {
      copies_begin(P, 1, N);
      t = timer_begin(P, P->lane[1].stream);
      any = true;
    }
    if ((s = copy_expert(P, 1, nl, e, sl, h))) return s;
    N.staged[e] = 1;
    P->st.copies_prefetch++;
  }
  if (any) {
    if ((s = flush_stage(P, 1))) return s;
    cudaEventRecord(t.b, P->lane[1].stream);
    P->timers.push_back(t);
    cudaEventRecord(N.ready[1], P->lane[1].stream);
    N.has_ready[1] = true;
  }
  return EF_OK;
}

// One streamed layer.  ahead_w / ahead_b: the gates of the next n_ahead
// layers (0..2), routed on this layer's input as the lookahead predictions.
ef_status pool_layer(ef_slot_pool* P, int layer, const void* x, int T, const void* gate_w, const float* e_bias,
                     int n_ahead, const void* const* ahead_w, const float* const* ahead_b, void* y, int out_f32,
                     int32_t* inds_out, float* wts_out, void* workspace, cudaStream_t st) {
  using clk = std::chrono::steady_clock;
  const auto h0 = clk::now();
  const ef_moe_cfg& cfg = P->cfg;
  const int E = cfg.n_experts, k = cfg.top_k, n = T * k;
  Carver c{static_cast<uint8_t*>(workspace)};
  PoolWs w;
  pool_ws(P, T, c, w);
  ef_status s;
  int* inds = inds_out ? inds_out : w.inds;
  float* wts = wts_out ? wts_out : w.wts;
  const void* gw[2] = {n_ahead > 0 ? ahead_w[0] : nullptr, n_ahead > 1 ? ahead_w[1] : nullptr};
  const float* gb[2] = {n_ahead > 0 && ahead_b ? ahead_b[0] : nullptr, n_ahead > 1 && ahead_b ? ahead_b[1] : nullptr};
  // 1. route this layer, and predict the next layers' experts from the same input
  if ((s = pool_route(cfg, x, T, gate_w, e_bias, w.logits, inds, wts, gw[0], gb[0], w.plogits[0], w.pinds[0],
                      w.pwts[0], gw[1], gb[1], w.plogits[1], w.pinds[1], w.pwts[1], st)))
    return s;
  if (n > P->h_cap) {
    if (P->h_inds) {
      cudaStreamSynchronize(st);  // no earlier layer still reads the old staging
      cudaFreeHost(P->h_inds);
    }
    drop_tail_graphs(P);  // they read the old slot-id staging
    P->h_cap = std::max(n, 256);
    if (cudaHostAlloc(reinterpret_cast<void**>(&P->h_inds), 4 * sizeof(int32_t) * P->h_cap + 64,
                      cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void**>(&P->d_inds), P->h_inds, 0) != cudaSuccess) {
      if (P->h_inds) cudaFreeHost(P->h_inds);
      P->h_inds = nullptr;
      P->h_cap = 0;
      return fail(EF_ERR_CUDA, "mapped pinned staging allocation failed");
    }
    P->h_flag = reinterpret_cast<uint32_t*>(P->h_inds + 4 * P->h_cap);
    *reinterpret_cast<volatile uint32_t*>(P->h_flag) = P->h_seq;
  }
  P->h_pred = P->h_inds + P->h_cap;
  P->h_slot = P->h_inds + 2 * P->h_cap;
  P->h_pred2 = P->h_inds + 3 * P->h_cap;
  // the routing reaches the host through the mapped staging: a one-CTA kernel
  // stores the ids there and then the step's sequence number, which this
  // thread polls (no copy launch, no stream synchronisation)
  const uint32_t seq = ++P->h_seq;
  EF_LAUNCH("publish_ids", launch_pdl(ef::publish_ids_kernel, 1, 256, 0, st, (const int*)inds,
                                      (const int*)(gw[0] ? w.pinds[0] : nullptr),
                                      (const int*)(gw[1] ? w.pinds[1] : nullptr), n, P->d_inds, P->d_inds + P->h_cap,
                                      P->d_inds + 3 * P->h_cap, reinterpret_cast<uint32_t*>(P->d_inds + 4 * P->h_cap),
                                      seq));
  const auto h1 = clk::now();
  if ((s = wait_published(P->h_flag, seq, st))) return s;
  const auto h2 = clk::now();
  P->st.route_wait_ms += std::chrono::duration<double, std::milli>(h2 - h1).count();
  P->st.host_ms += std::chrono::duration<double, std::milli>(h1 - h0).count();
  if (P->rec_on)  // the reference records each routed entry in (token, k) order (ef_engine.py:640-646)
    for (int i = 0; i < n; ++i) {
      P->rec_pairs.push_back(layer);
      P->rec_pairs.push_back(P->h_inds[i]);
    }
  const std::vector<int> need = distinct_sorted(P->h_inds, n, E);
  std::vector<char> keep(E, 0);
  for (int e : need) keep[e] = 1;
  LayerSlots& L = P->layers[layer];
  ++P->epoch;
  if (P->store) {  // start the file reads of this layer's experts missing in HBM and the host tier first
    for (int e : need)
      if (L.expert_slot[e] < 0 && host_fetch(P, layer, e, false) < 0)
        return fail(EF_ERR_SLOT_MISS, "layer %d: the host tier (%d blobs) cannot hold one step's experts", layer,
                    P->host_n);
  }
  // this layer's file reads must be complete before its state changes (a
  // failed read leaves the pool as it was)
  if (P->store) {
    for (int e : need) {
      if (L.expert_slot[e] >= 0) continue;
      const int h = host_find(P, layer, e);
      if (h < 0) return fail(EF_ERR_SLOT_MISS, "layer %d expert %d left the host tier", layer, e);
      if ((s = host_ready(P, h, layer, e))) return s;
    }
  }
  // 2. resolve this layer's experts (ef_engine.py:650-675): policy get, put on a miss
  bool any = false;
  CopyTimer t{};
  for (int e : need) {
    P->st.accesses++;
    if (L.policy.get(e)) {
      P->st.hits++;
      if (L.expert_slot[e] < 0) return fail(EF_ERR_SLOT_MISS, "policy/slot state diverged (layer %d expert %d)", layer, e);
      continue;
    }
    P->st.misses++;
    L.policy.put(e);
    if (L.expert_slot[e] >= 0) {  // staged by the lookahead
      if (L.staged[e]) P->st.prefetch_used++;
      L.staged[e] = 0;
      continue;
    }
    bool from_staged = false;
    int sl = take_slot(P, layer, keep, &from_staged);
    if (sl < 0) {  // full: evict now the lowest-priority resident expert this step does not use
      const long long v = L.policy.victim_excluding(keep);
      if (v < 0) return fail(EF_ERR_SLOT_MISS, "layer %d: no slot for expert %d (raise headroom)", layer, e);
      L.policy.erase(v);
      sl = L.expert_slot[v];
      L.expert_slot[v] = -1;
      L.slot_expert[sl] = -1;
      P->st.evictions++;
    }
    if (!any) {
      copies_begin(P, 0, L);
      t = timer_begin(P, P->lane[0].stream);
      any = true;
    }
    // a slot taken from an unused prefetch may still be written by the
    // prefetch lane: this lane's scatter into it goes after that lane's
    if (from_staged && L.has_ready[1]) cudaStreamWaitEvent(P->lane[0].stream, L.ready[1], 0);
    if ((s = copy_expert(P, 0, layer, e, sl, P->store ? host_find(P, layer, e) : -1))) return s;
    P->st.copies_sync++;
  }
  if (any) {
    if ((s = flush_stage(P, 0))) return s;
    cudaEventRecord(t.b, P->lane[0].stream);
    P->timers.push_back(t);
    cudaEventRecord(L.ready[0], P->lane[0].stream);
    L.has_ready[0] = true;
  }
  // this layer's experts wait for both lanes' copies into its slots (the
  // stall is timed on the compute stream)
  bool pending[2];
  for (int ln = 0; ln < 2; ++ln) pending[ln] = L.has_ready[ln] && cudaEventQuery(L.ready[ln]) != cudaSuccess;
  if (pending[0] || pending[1]) {
    CopyTimer wt = timer_begin(P, st);
    wt.stall = true;
    for (int ln = 0; ln < 2; ++ln)
      if (pending[ln]) cudaStreamWaitEvent(st, L.ready[ln], 0);
    cudaEventRecord(wt.b, st);
    P->timers.push_back(wt);
  }
  // 3. experts on slot ids
  // slot ids stay in pinned memory: the permute kernel reads them over the
  // link (n ints) instead of a copy that would queue behind the expert copies
  for (int i = 0; i < n; ++i) P->h_slot[i] = L.expert_slot[P->h_inds[i]];
  ef_moe_cfg sc = cfg;
  sc.n_experts = P->n_slots;
  sc.out_f32 = out_f32 ? 1 : 0;
  const SlotView v = slot_arrays(P, L);
  const ef_qweight qg{reinterpret_cast<uint32_t*>(v.w[0]), reinterpret_cast<uint16_t*>(v.s[0]), reinterpret_cast<uint16_t*>(v.b[0])};
  const ef_qweight qu{reinterpret_cast<uint32_t*>(v.w[1]), reinterpret_cast<uint16_t*>(v.s[1]), reinterpret_cast<uint16_t*>(v.b[1])};
  const ef_qweight qd{reinterpret_cast<uint32_t*>(v.w[2]), reinterpret_cast<uint16_t*>(v.s[2]), reinterpret_cast<uint16_t*>(v.b[2])};
  if ((s = run_tail(P, layer, sc, x, T, wts, qg, qu, qd, w.f, y, workspace, st))) return s;
  cudaEventRecord(L.last_use, st);
  L.has_use = true;
  // 4. lookahead copies for the next layers, issued after this layer's expert
  //    kernels so that the host work and the copies overlap them (the step
  //    synchronised once, for the routing; host time before the launches is
  //    idle GPU time); the nearer layer's copies are queued first
  for (int a = 0; a < n_ahead; ++a)
    if ((s = stage_ahead(P, layer + 1 + a, a ? P->h_pred2 : P->h_pred, n))) return s;
  P->st.host_ms += std::chrono::duration<double, std::milli>(clk::now() - h2).count();
  return EF_OK;
}
}  // namespace

ef_status ef_pool_moe_forward(ef_slot_pool* P, int layer, const void* x, int T, const void* gate_w,
                              const float* e_bias, const void* next_gate_w, const float* next_e_bias, void* y,
                              int out_f32, int32_t* inds_out, float* wts_out, void* workspace, size_t ws_bytes,
                              void* stream) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  if (layer < 0 || layer >= P->pc.n_layers) return fail(EF_ERR_RANGE, "layer %d out of range", layer);
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!x || !gate_w || !y) return fail(EF_ERR_INVALID, "null pointer");
  if (!aligned16(x) || !aligned16(gate_w) || !aligned16(y)) return fail(EF_ERR_INVALID, "x/gate_w/y must be 16-byte aligned");
  if (next_gate_w && layer + 1 >= P->pc.n_layers) return fail(EF_ERR_RANGE, "no layer after %d to predict", layer);
  if (ws_bytes < ef_pool_workspace_size(P, T) || !workspace) return fail(EF_ERR_WORKSPACE, "workspace too small");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != P->dev) return fail(EF_ERR_INVALID, "pool belongs to device %d, current device is %d", P->dev, dev);
  const float* nb = next_e_bias;
  return pool_layer(P, layer, x, T, gate_w, e_bias, next_gate_w ? 1 : 0, &next_gate_w, &nb, y, out_f32, inds_out,
                    wts_out, workspace, static_cast<cudaStream_t>(stream));
}

size_t ef_pool_decode_workspace_size(const ef_slot_pool* P, int T) {
  if (!P || T < 0) return 0;
  const size_t H = P->cfg.hidden;
  return ((size_t)T * H * 2 + 255) / 256 * 256 + ((size_t)T * H * 4 + 255) / 256 * 256 + ef_pool_workspace_size(P, T) +
         256;
}

ef_status ef_pool_decode_step(ef_slot_pool* P, float* r, int T, const void* const* gate_w,
                              const float* const* e_bias, int lookahead, float eps, void* workspace, size_t ws_bytes,
                              void* stream) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (!r || !gate_w) return fail(EF_ERR_INVALID, "null pointer");
  if (lookahead < 0 || lookahead > 2) return fail(EF_ERR_INVALID, "lookahead must be 0, 1 or 2 layers");
  if (ws_bytes < ef_pool_decode_workspace_size(P, T) || !workspace) return fail(EF_ERR_WORKSPACE, "workspace too small");
  const int H = P->cfg.hidden, L = P->pc.n_layers;
  for (int l = 0; l < L; ++l)
    if (!gate_w[l] || !aligned16(gate_w[l])) return fail(EF_ERR_INVALID, "gate_w[%d] null or not 16-byte aligned", l);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != P->dev) return fail(EF_ERR_INVALID, "pool belongs to device %d, current device is %d", P->dev, dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int bf = P->cfg.act_dtype == EF_DT_BF16;
  Carver c{static_cast<uint8_t*>(workspace)};
  uint16_t* x = c.take<uint16_t>((size_t)T * H);
  float* y = c.take<float>((size_t)T * H);
  void* fws = c.take<uint8_t>(ef_pool_workspace_size(P, T));
  const size_t fws_bytes = ef_pool_workspace_size(P, T);
  ef_status s;
  for (int l = 0; l < L; ++l) {
    EF_LAUNCH("add_rmsnorm", launch_pdl(ef::add_rmsnorm_kernel, T, ef::kNormThreads, 0, st, r,
                                            l ? static_cast<const float*>(y) : nullptr, H, eps, bf, x));
    const int n_ahead = std::min(lookahead, L - 1 - l);
    if ((s = pool_layer(P, l, x, T, gate_w[l], e_bias ? e_bias[l] : nullptr, n_ahead, gate_w + l + 1,
                        e_bias ? e_bias + l + 1 : nullptr, y, 1, nullptr, nullptr, fws, st)))
      return s;
  }
  EF_LAUNCH("add_rmsnorm", launch_pdl(ef::add_rmsnorm_kernel, T, ef::kNormThreads, 0, st, r,
                                          static_cast<const float*>(y), H, eps, bf, static_cast<uint16_t*>(nullptr)));
  return ef_pool_end_token(P);
}

ef_status ef_pool_end_token(ef_slot_pool* P) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  for (auto& L : P->layers) {
    for (long long e : L.policy.trim()) {
      const int sl = L.expert_slot[e];
      if (sl >= 0) L.slot_expert[sl] = -1;
      L.expert_slot[e] = -1;
      P->st.evictions++;
    }
    L.policy.end_token();  // trim, then end_token, as the reference's decode loop does
  }
  P->st.tokens++;
  if (P->rec_on) P->rec_tok_end.push_back((long long)(P->rec_pairs.size() / 2));
  return EF_OK;
}

ef_status ef_pool_record_routing(ef_slot_pool* P, int on) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  if (on && !P->rec_on) {
    P->rec_pairs.clear();
    P->rec_tok_end.clear();
  }
  P->rec_on = on != 0;
  return EF_OK;
}

ef_status ef_pool_routing_trace(const ef_slot_pool* P, int32_t* pairs, long long pair_cap, long long* n_pairs,
                                long long* token_ends, long long tok_cap, long long* n_tokens) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  const long long np = (long long)(P->rec_pairs.size() / 2), nt = (long long)P->rec_tok_end.size();
  if (n_pairs) *n_pairs = np;
  if (n_tokens) *n_tokens = nt;
  if (pairs)
    for (long long i = 0; i < std::min(np, pair_cap) * 2; ++i) pairs[i] = P->rec_pairs[(size_t)i];
  if (token_ends)
    for (long long i = 0; i < std::min(nt, tok_cap); ++i) token_ends[i] = P->rec_tok_end[(size_t)i];
  return EF_OK;
}

ef_status ef_pool_set_predictor(ef_slot_pool* P, int hidden, const float* w1, const float* b1, const float* w2,
                                const float* b2, const float* w3, const float* b3, int trained) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  ef::BeladyNet n;
  ef_status s = make_net(hidden, w1, b1, w2, b2, w3, b3, trained, n);
  if (s) return s;
  for (auto& L : P->layers) L.policy.set_net(n);
  return EF_OK;
}

ef_status ef_pool_resident(const ef_slot_pool* P, int layer, int32_t* experts, int cap, int* n) {
  if (!P || !n) return fail(EF_ERR_INVALID, "null pointer");
  if (layer < 0 || layer >= P->pc.n_layers) return fail(EF_ERR_RANGE, "layer out of range");
  const std::vector<long long> k = P->layers[layer].policy.keys();
  *n = (int)k.size();
  for (int i = 0; i < (int)k.size() && i < cap && experts; ++i) experts[i] = (int32_t)k[i];
  return EF_OK;
}

ef_status ef_pool_get_stats(ef_slot_pool* P, ef_pool_stats* out) {
  if (!P || !out) return fail(EF_ERR_INVALID, "null pointer");
  for (auto& C : P->lane) cudaStreamSynchronize(C.stream);
  fold_timers(P, true);
  *out = P->st;
  return EF_OK;
}

ef_status ef_pool_reset_stats(ef_slot_pool* P) {
  if (!P) return fail(EF_ERR_INVALID, "pool is NULL");
  for (auto& C : P->lane) cudaStreamSynchronize(C.stream);
  fold_timers(P, true);
  P->st = ef_pool_stats{};
  return EF_OK;
}

ef_status ef_pool_destroy(ef_slot_pool* P) {
  if (!P) return EF_OK;
  for (auto& C : P->lane)
    if (C.stream) cudaStreamSynchronize(C.stream);
  for (int h = 0; h < P->host_n && P->host_ticket; ++h)  // reads still writing into the host blobs
    if (!ef::store_done(&P->host_ticket[h])) ef::store_wait(P->store, &P->host_ticket[h], 0, 0);
  fold_timers(P, true);
  for (auto& t : P->spare) {
    cudaEventDestroy(t.a);
    cudaEventDestroy(t.b);
  }
  drop_tail_graphs(P);
  if (P->cap_stream) cudaStreamDestroy(P->cap_stream);
  for (auto& L : P->layers) {
    cudaEventDestroy(L.ready[0]);
    cudaEventDestroy(L.ready[1]);
    cudaEventDestroy(L.last_use);
  }
  for (cudaEvent_t ev : P->host_copied)
    if (ev) cudaEventDestroy(ev);
  for (auto& C : P->lane) {
    if (C.stream) cudaStreamDestroy(C.stream);
    if (C.stage) cudaFree(C.stage);
  }
  if (P->dev_mem) cudaFree(P->dev_mem);
  if (P->host_blobs) cudaFreeHost(P->host_blobs);
  if (P->h_inds) cudaFreeHost(P->h_inds);
  delete P;
  return EF_OK;
}

}  // extern "C"
