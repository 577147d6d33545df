/*
 * efmoe.h -- C ABI of libefmoe.so, the B200 (sm_100a) implementation of the
 * ExpertFlow MoE-layer hot path.
 *
 * Conventions
 *   - Every tensor argument is a DEVICE pointer owned by the caller; sizes are
 *     plain ints.  No call allocates device memory: scratch space is the
 *     caller's `workspace` (size from ef_moe_workspace_size).
 *   - Every compute call is asynchronous on `stream` (a cudaStream_t, passed as
 *     void*; NULL = legacy default stream) and returns EF_OK or a negative
 *     EF_ERR_* code.  Argument checks happen on the host before any launch.
 *   - Quantised weights use the MLX affine layout (uint32-packed codes,
 *     LSB-first; fp16 scale and bias per 64-column group), stacked per expert:
 *       w      uint32 [n_experts, out_dim, in_dim * bits / 32]
 *       scales fp16   [n_experts, out_dim, in_dim / 64]
 *       biases fp16   [n_experts, out_dim, in_dim / 64]
 *     dequant(w)[o, i] = scales[o, i/64] * q[o, i] + biases[o, i/64].
 *   - Routing: indices are bit-exact with the CPU oracle (fp32 logits in a
 *     fixed lane-interleaved order, top-k by (score desc, index asc)).
 *   - Handles are not thread-safe; use one per stream.
 *
 * Reference interfaces replaced (paths relative to the reference checkout):
 *   ef_moe_forward        streaming_moe_forward(moe_module, x, expert_cache)  ef_engine.py:598-706
 *   ef_router_topk        moe_module.gate(x) + argpartition/softmax        ef_engine.py:609-619
 *   ef_quantized_matmul   mx.quantized_matmul(x, w, s, b, transpose=True)  ef_engine.py:689-694
 *   ef_dequantize         mx.dequantize(w, s, b, group_size, bits)         ef_cpu_fast.py:70-75
 *   ef_gather_qmm         QuantizedSwitchLinear.__call__(x, indices)        ef_engine_v4.py:52-64
 *   ef_moe_experts_forward  per-(row, expert) SwiGLU loop                  ef_engine.py:678-695
 *   ef_permute            unique-expert grouping of the routed entries     ef_engine.py:640-647
 *   ef_combine            score-weighted sum over k (+ shared)             ef_engine.py:695-703
 *   ef_ep_forward         the per-(token, k) expert loop, experts sharded   ef_engine.py:678-703
 *                         across the GPUs of one box (no reference counterpart for the split)
 *   ef_slotpool_*         FrequencyWeightedCache get/put/trim              ef_engine.py:48-104
 *                         + mmap page-in of misses                        ef_engine.py:650-675
 *   ef_kquant_*           GGUF Q2_K/Q3_K/Q4_K decode (+ GEMV)              ef_deepseek_mmap.py:330-378,655-773
 *   ef_kquant_moe_forward the MoE layer over GGUF K-quant experts          ef_deepseek_mmap.py:570-593,1563-1660
 *   ef_store_*            expert byte ranges read out of the checkpoint     ef_deepseek_mmap.py:431-570,
 *                         files on reader threads                          experiments/ef_v18_prefetch2.py:76-200
 */
#ifndef EFMOE_H
#define EFMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ef_status;
#define EF_OK 0
#define EF_ERR_INVALID (-1)     /* bad shape, null or misaligned pointer */
#define EF_ERR_UNSUPPORTED (-2) /* bits / group / dtype / size not supported */
#define EF_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define EF_ERR_WORKSPACE (-4)   /* workspace too small */
#define EF_ERR_TIMEOUT (-5)     /* a bounded device-side wait ran out */
#define EF_ERR_SLOT_MISS (-6)   /* expert not resident in the slot pool */
#define EF_ERR_RANGE (-7)       /* activation outside the fp16 range */
#define EF_ERR_NOT_READY (-8)   /* no CUDA device / extension not initialised */
#define EF_ERR_IO (-9)          /* a file read failed, or read a value the format cannot carry */

enum { EF_DT_BF16 = 0, EF_DT_F16 = 1, EF_DT_F32 = 2 };
enum { EF_ROUTER_SOFTMAX = 0, EF_ROUTER_SIGMOID_GROUP = 1 };
enum { EF_PATH_AUTO = 0, EF_PATH_GEMV = 1, EF_PATH_GEMM = 2, EF_PATH_GEMM_PAIR = 3 };

/* One stack of quantised projections (see layout above). */
typedef struct {
  const uint32_t* w;
  const uint16_t* scales;
  const uint16_t* biases;
} ef_qweight;

/* Layer configuration: the attributes the reference reads from an mlx_lm MoE
 * module (num_experts_per_tok, switch_mlp.*.bits/group_size, shared_experts)
 * plus the gate's routing parameters. */
typedef struct {
  int hidden;         /* H, multiple of 64 */
  int inter;          /* I (per routed expert), multiple of 64 */
  int n_experts;      /* E, 1..512 */
  int top_k;          /* k, 1..16 */
  int bits;           /* 4 or 8 */
  int group_size;     /* 64 */
  int router_mode;    /* EF_ROUTER_* */
  int norm_topk;      /* softmax: renormalise over k; sigmoid: divide by the sum */
  int n_group;        /* sigmoid_group: expert groups (1 = no group limit), <= 32 */
  int topk_group;     /* sigmoid_group: groups kept */
  float routed_scaling;
  int n_shared;       /* 0 or 1 shared expert (always-on, weight 1.0) */
  int shared_inter;   /* I of the shared expert */
  int act_dtype;      /* EF_DT_BF16 or EF_DT_F16 (x and y) */
  int gate_dtype;     /* EF_DT_F16 or EF_DT_BF16 (router weight) */
  int path;           /* EF_PATH_AUTO / GEMV (decode kernels) / GEMM (tcgen05 grouped GEMM, one SM per tile) /
                         GEMM_PAIR (the same contraction on SM pairs, cta_group::2) */
  int out_f32;        /* 1: y is fp32 (the combine's accumulator); 0: y has act_dtype */
} ef_moe_cfg;

/* ---- library ---------------------------------------------------------- */
const char* ef_version(void);
const char* ef_status_string(ef_status s);
/* Detail of the last error returned on the calling host thread. */
const char* ef_last_error_message(void);
/* Reads and clears the device-side error word (set by bounded waits that ran
 * out, or by an out-of-range activation); synchronises `stream`. */
ef_status ef_get_device_error(void* stream, int* code);

/* ---- tracing ------------------------------------------------------------ */
/* When enabled, every kernel the library launches is bracketed by two CUDA
 * events recorded on the launching stream.  ef_trace_read waits for the
 * recorded events, writes up to max_recs (name, milliseconds) records in launch
 * order, returns how many were written and clears the trace.  The reference
 * times its phases with time.time() buckets (experiments/ef_profile_moe.py). */
typedef struct {
  const char* name;
  float ms;
} ef_trace_rec;
ef_status ef_trace_enable(int on);
int ef_trace_read(ef_trace_rec* recs, int max_recs);

/* ---- whole layer ------------------------------------------------------ */
/* Bytes of workspace ef_moe_forward needs for T tokens (256-byte aligned). */
size_t ef_moe_workspace_size(const ef_moe_cfg* cfg, int T);

/* y[T, H] = sum_k w[t,k] * SwiGLU_{e[t,k]}(x[t]) (+ shared(x[t])), routing by
 * the gate (gate_w fp16/bf16 [E, H], e_bias fp32 [E] or NULL).  inds_out
 * [T, k] int32 and wts_out [T, k] fp32 are optional (NULL to skip).
 * Replaces streaming_moe_forward, ef_engine.py:598-706. */
ef_status ef_moe_forward(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w, const float* e_bias,
                         ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* shared_gate,
                         const ef_qweight* shared_up, const ef_qweight* shared_down, void* y, int32_t* inds_out,
                         float* wts_out, void* workspace, size_t workspace_bytes, void* stream);

/* Same as ef_moe_forward, for callers that cannot allocate device memory (an
 * FFI host without a CUDA allocator of its own, or a decode loop that must not
 * call cudaMalloc): no workspace argument; the scratch is a fixed array of
 * EF_NOALLOC_SCRATCH_BYTES held in device memory by every GPU that loads the
 * library.  Returns EF_ERR_WORKSPACE when ef_moe_workspace_size(cfg, T) is
 * larger.  The first call on each device resolves the array's address (make
 * it before any stream capture).  All calls share the array: calls that
 * overlap on the GPU race and must be serialised by the caller.
 * No counterpart in the reference. */
#define EF_NOALLOC_SCRATCH_BYTES (64u << 20)
ef_status ef_moe_forward_noalloc(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w,
                                 const float* e_bias, ef_qweight gate, ef_qweight up, ef_qweight down,
                                 const ef_qweight* shared_gate, const ef_qweight* shared_up,
                                 const ef_qweight* shared_down, void* y, int32_t* inds_out, float* wts_out,
                                 void* stream);

/* ---- router ----------------------------------------------------------- */
/* inds [T, k] int32 in rank order, weights [T, k] fp32.  Replaces
 * moe_module.gate(x) + argpartition/take_along_axis/softmax, ef_engine.py:609-619. */
size_t ef_router_workspace_size(const ef_moe_cfg* cfg, int T);
ef_status ef_router_topk(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w, const float* e_bias,
                         int32_t* inds, float* weights, float* logits_out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---- permutation and combine ------------------------------------------------ */
/* Stable counting sort of routed entries by expert (order (expert, entry)),
 * atomic-free.  entries [n_entries] hold expert ids in [0, n_experts); entry i
 * belongs to token i / k.  n_shared_rows > 0 adds bin n_experts holding rows
 * for tokens 0..n_shared_rows-1 (the shared expert) after all routed rows.
 * Outputs: counts [n_bins] rows per bin, offsets [n_bins + 1] first sorted row
 * of each bin, row_src [n_entries + n_shared_rows] token of each sorted row,
 * inv [n_entries] sorted row of each entry; n_bins = n_experts (+1 with shared
 * rows).  The workspace holds the segments of <= seg_rows rows the expert
 * kernels consume.  Replaces the unique-expert grouping of ef_engine.py:640-647
 * and expertflow_final.py:94-113. */
size_t ef_permute_workspace_size(int n_entries, int n_experts, int n_shared_rows, int seg_rows);
ef_status ef_permute(const int32_t* entries, int n_entries, int k, int n_experts, int n_shared_rows, int seg_rows,
                     int32_t* counts, int32_t* offsets, int32_t* row_src, int32_t* inv, void* workspace,
                     size_t workspace_bytes, void* stream);
/* y[t, :] = sum_j wts[t, j] * rows[inv[t*k + j], :] in j order (wts NULL: unit
 * weights), + rows[shared_base + t, :] when shared_base >= 0; rows fp32
 * [*, H], y [T, H] in out_dtype (EF_DT_*).  Replaces the score-weighted sum of
 * ef_engine.py:695-703. */
ef_status ef_combine(const float* rows, const int32_t* inv, const float* wts, int T, int k, int H, int shared_base,
                     void* y, int out_dtype, void* stream);

/* ---- experts on routed rows --------------------------------------------- */
/* Rows x[N, H] (act dtype), row_expert[N] in [0, n_experts) (or n_experts for
 * the shared expert when shared_* is given); y_rows[N, H] fp32 = expert(x row).
 * The per-(row, expert) SwiGLU of ef_engine.py:678-695 without the weighting;
 * used by expert-parallel dispatch (rows received from peers). */
size_t ef_experts_workspace_size(const ef_moe_cfg* cfg, int N);
ef_status ef_moe_experts_forward(const ef_moe_cfg* cfg, const void* x_rows, int N, const int32_t* row_expert,
                                 ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* shared_gate,
                                 const ef_qweight* shared_up, const ef_qweight* shared_down, float* y_rows,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* ---- MLX op equivalents ------------------------------------------------- */
/* y[M, out] = x[M, in] @ dequant(w)^T  (x, y act dtype).  Replaces
 * mx.quantized_matmul(x, w, s, b, transpose=True, group_size, bits). */
size_t ef_quantized_matmul_workspace_size(int M, int out_dim, int in_dim);
ef_status ef_quantized_matmul(const void* x, int act_dtype, int M, const uint32_t* w, const uint16_t* scales,
                              const uint16_t* biases, int out_dim, int in_dim, int bits, int group_size, void* y,
                              void* workspace, size_t workspace_bytes, void* stream);

/* out[rows, cols] (EF_DT_F32 / F16 / BF16) = dequant(w).  Replaces mx.dequantize. */
ef_status ef_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int rows, int cols,
                        int bits, int group_size, void* out, int out_dtype, void* stream);

/* y[T, k, out] = x[t] @ dequant(w[indices[t, j]])^T.  Replaces gather_qmm
 * (QuantizedSwitchLinear.__call__, ef_engine_v4.py:52-64). */
size_t ef_gather_qmm_workspace_size(int T, int k, int n_experts, int out_dim, int in_dim);
ef_status ef_gather_qmm(const void* x, int act_dtype, int T, const int32_t* indices, int k, ef_qweight w,
                        int n_experts, int out_dim, int in_dim, int bits, int group_size, void* y, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ---- expert parallelism (experts sharded across ranks) --------------------- */
/* Expert e lives on rank e / (E / n_ranks); router and shared expert are
 * replicated; each rank routes its own T tokens.  The exchange steps are
 * NCCL all-to-alls issued by the host between these calls:
 *   ef_ep_dispatch -> all-to-all(send_counts) -> all-to-all(send_rows,
 *   send_expert) -> ef_moe_experts_forward (local experts) -> all-to-all of
 *   the fp32 outputs back -> ef_ep_combine.
 * Replaces the single-host per-(token, k) expert loop of ef_engine.py:678-703. */
size_t ef_ep_dispatch_workspace_size(const ef_moe_cfg* cfg, int T);
/* Route x [T, H]; send_rows [T*k, H] (act dtype) = the routed token rows sorted
 * by expert (so by destination rank), send_expert [T*k] = the destination's
 * local expert id, send_counts [n_ranks] = rows per rank, inv_out [T*k] =
 * sorted row of entry (t, j), wts_out [T*k] = routing weights, inds_out
 * [T*k] = global expert ids (or NULL). */
ef_status ef_ep_dispatch(const ef_moe_cfg* cfg, int n_ranks, const void* x, int T, const void* gate_w,
                         const float* e_bias, void* send_rows, int32_t* send_expert, int32_t* send_counts,
                         int32_t* inv_out, float* wts_out, int32_t* inds_out, void* workspace,
                         size_t workspace_bytes, void* stream);
/* y[t] = sum_j wts[t, j] * back_rows[inv[t, j]] (+ back_rows[T*k + t] when
 * with_shared), in j order; back_rows fp32 [T*k (+T), H]. */
ef_status ef_ep_combine(const ef_moe_cfg* cfg, const float* back_rows, const int32_t* inv, const float* wts, int T,
                        int with_shared, void* y, void* stream);

/* ---- expert parallelism over NVLink peer memory -------------------------------------- */
/* The same split (expert e on rank e / (E / n_ranks); router and shared expert
 * replicated; each rank routes its own tokens), exchanged by the kernels
 * themselves through the peers' memory instead of host-issued all-to-alls:
 *   - each rank owns one exchange buffer (receive regions for every source
 *     rank, a row-return region for its own tokens, arrival flags); the
 *     buffers are shared once through CUDA IPC handles;
 *   - ef_ep_forward routes and sorts this rank's tokens, and one kernel stores
 *     every routed token row straight into its destination rank's receive
 *     region and raises that rank's arrival flag (release at system scope);
 *   - a one-CTA kernel waits (bounded) for every source's flag, then sorts the
 *     received rows by local expert; this rank's shared expert is one more bin;
 *     the local experts run on the decode GEMV or the grouped GEMM;
 *   - one kernel stores each fp32 output row back into its source rank's
 *     return region (the row the source sorted the entry to) and raises the
 *     source's done flag; the source waits for every rank's done flag and
 *     combines in k order.
 * The combine is the single-GPU layer's, over the same fp32 rows, so the output
 * equals ef_moe_forward's whenever both run the same expert kernels.  Nothing
 * in a forward waits on the host: a device-side epoch numbers the flags, so a
 * forward can be captured in a CUDA graph.  Every rank must issue the same
 * sequence of forwards (T may differ per rank, 0 included); a rank that stops
 * makes the others' bounded waits run out (EF_ERR_TIMEOUT from
 * ef_get_device_error), after which the group must be destroyed and created
 * again.  No TMA reads peer memory.  Replaces the single-host per-(token, k)
 * expert loop of ef_engine.py:678-703 (the reference has no multi-device path). */
#define EF_EP_HANDLE_BYTES 64
#define EF_EP_MAX_RANKS 64
typedef struct ef_ep_group ef_ep_group;
/* This rank's exchange buffer on the current device, for forwards of up to
 * max_tokens tokens per rank; max_recv_rows (0 = the worst case, n_ranks *
 * max_tokens * min(top_k, E / n_ranks)) bounds the rows one rank receives per
 * forward (a forward that receives more reports EF_ERR_RANGE on the device and
 * drops the excess).  Allocates device memory (cudaMalloc) here only. */
ef_status ef_ep_group_create(const ef_moe_cfg* cfg, int rank, int n_ranks, int max_tokens, int max_recv_rows,
                             ef_ep_group** out);
/* The exchange buffer's IPC handle (EF_EP_HANDLE_BYTES bytes) for the other ranks. */
ef_status ef_ep_group_handle(const ef_ep_group* g, void* handle);
/* Maps every peer's buffer from the gathered handles [n_ranks][EF_EP_HANDLE_BYTES]
 * (this rank's own entry is not used).  Every rank calls it before its first forward. */
ef_status ef_ep_group_open(ef_ep_group* g, const void* handles);
size_t ef_ep_workspace_size(const ef_ep_group* g, int T);
/* y[T, H] (out_dtype: EF_DT_F32, or the activation dtype) for this rank's T
 * tokens (T <= max_tokens; cfg->act_dtype as given at creation).  gate/up/down: this
 * rank's local experts [E / n_ranks, ...]; shared_*: the replicated shared
 * expert when cfg->n_shared.  inds_out / wts_out [T, k] optional. */
ef_status ef_ep_forward(ef_ep_group* g, const void* x, int T, const void* gate_w, const float* e_bias,
                        ef_qweight gate, ef_qweight up, ef_qweight down, const ef_qweight* shared_gate,
                        const ef_qweight* shared_up, const ef_qweight* shared_down, void* y, int out_dtype,
                        int32_t* inds_out, float* wts_out, void* workspace, size_t workspace_bytes, void* stream);
/* Unmaps the peers and frees the buffer; call only when no rank has a forward
 * in flight (e.g. after a barrier). */
ef_status ef_ep_group_destroy(ef_ep_group* g);

/* ---- expert residency: cache policy and HBM slot pool ------------------------------ */
/* Eviction policies.  EF_POLICY_FREQ is the reference's FrequencyWeightedCache
 * (ef_engine.py:48-104): a hit adds 1 to the key's score, a put inserts with
 * score + 1, trim() evicts the lowest score (earliest inserted among equals)
 * down to the budget and multiplies every score by `decay`.  EF_POLICY_LRU
 * evicts the least recently used key and does not decay. */
#define EF_POLICY_FREQ 0
#define EF_POLICY_LRU 1
/* EF_POLICY_BELADY is the reference's BeladyExpertCache (ef_engine.py:163-279):
 * per key it records the last access token, an access count and an EMA of the
 * gap between accesses; trim() evicts, among the resident keys in insertion
 * order, the first with the highest learned score (a 3 -> H -> H -> 1 SiLU
 * network on [1/recency, count/max_count, gap/max_gap], weights from
 * ef_policy_set_predictor) or, while the predictor is untrained, the first
 * with the lowest count * decay^recency; then every count becomes
 * floor(count * decay).  ef_policy_end_token advances its token clock (the
 * reference calls trim, then end_token, once per token). */
#define EF_POLICY_BELADY 2
typedef struct ef_cache_policy ef_cache_policy;
ef_status ef_policy_create(int kind, int budget, double decay, ef_cache_policy** out);
int ef_policy_get(ef_cache_policy* p, long long key);  /* 1 on a hit (FrequencyWeightedCache.get) */
void ef_policy_put(ef_cache_policy* p, long long key);  /* FrequencyWeightedCache.put */
/* FrequencyWeightedCache.trim: returns the number evicted, their keys (in
 * eviction order) in evicted[0..cap). */
int ef_policy_trim(ef_cache_policy* p, long long* evicted, int cap);
int ef_policy_size(const ef_cache_policy* p);
int ef_policy_keys(const ef_cache_policy* p, long long* keys, int cap); /* resident keys, ascending */
double ef_policy_score(const ef_cache_policy* p, long long key);
void ef_policy_end_token(ef_cache_policy* p);
/* Predictor weights (row-major, the reference's BeladyPredictor layout):
 * w1 [3][hidden], b1 [hidden], w2 [hidden][hidden], b2 [hidden], w3 [hidden],
 * b3 [1]; trained = 0 keeps the frequency fallback. Copied. */
ef_status ef_policy_set_predictor(ef_cache_policy* p, int hidden, const float* w1, const float* b1, const float* w2,
                                  const float* b2, const float* w3, const float* b3, int trained);
void ef_policy_destroy(ef_cache_policy* p);

/* Streaming-decode expert pool: the experts of n_layers MoE layers live in
 * pinned host memory (the pool copies the caller's per-layer stacked MLX
 * arrays [E, ...], pinned or pageable, into its own pinned store of one
 * contiguous blob per expert); each layer owns min(E, budget + headroom) HBM
 * slots.  `budget` experts per layer stay
 * resident across tokens (the policy's budget); `headroom` (>= top_k x tokens
 * per step) holds a token's misses until ef_pool_end_token trims, as the
 * reference trims once per token.  Replaces the expert_cache argument of
 * streaming_moe_forward (ef_engine.py:650-675) and the lookahead prefetch of
 * experiments/ef_v16_prefetch.py:92-113. */
typedef struct {
  int n_layers;
  int budget;    /* experts per layer kept across tokens */
  int headroom;  /* extra slots per layer for one step's misses */
  int policy;    /* EF_POLICY_FREQ | EF_POLICY_LRU | EF_POLICY_BELADY */
  double decay;  /* EF_POLICY_FREQ score decay per token (reference: 0.95) */
} ef_pool_cfg;
typedef struct {
  long long accesses;        /* distinct (layer, expert) resolutions */
  long long hits;            /* policy hits (FrequencyWeightedCache.get semantics) */
  long long misses;          /* policy misses */
  long long copies_sync;     /* misses copied on demand (the step waits for them) */
  long long copies_prefetch; /* experts copied ahead by the lookahead */
  long long prefetch_used;   /* prefetched experts the next layer then used */
  long long evictions;
  long long tokens;          /* ef_pool_end_token calls */
  double h2d_bytes;          /* expert bytes copied host -> HBM */
  double copy_ms;            /* copy-stream time spent in those copies */
  /* pools over an ef_expert_store (zero otherwise): */
  long long host_hits;       /* experts found in the pinned host tier when asked for */
  long long host_reads;      /* experts read from the files (on demand + ahead) */
  long long host_reads_ahead;/* of those, reads started by the lookahead */
  long long host_evictions;  /* host-tier blobs replaced */
  double read_wait_ms;       /* host time the pool waited for file reads */
  double copy_wait_ms;       /* compute-stream time stalled on copies into a layer's slots */
  double route_wait_ms;      /* host time spent waiting for the routing to be published */
  double host_ms;            /* other host time in the pool's layer steps (decisions, launches) */
} ef_pool_stats;
typedef struct ef_slot_pool ef_slot_pool;
/* cfg: the layer configuration (n_shared must be 0); host_*: n_layers entries of
 * host arrays (read once, during the call).  The pool allocates its HBM
 * slots, a staging ring, its pinned store and a copy stream on the current
 * device. */
ef_status ef_pool_create(const ef_moe_cfg* cfg, const ef_pool_cfg* pool_cfg, const ef_qweight* host_gate,
                         const ef_qweight* host_up, const ef_qweight* host_down, ef_slot_pool** out);
size_t ef_pool_workspace_size(const ef_slot_pool* pool, int T);
/* One MoE layer of a streaming decode step: route x (gate_w, e_bias), copy
 * the weights of experts not in HBM, run the experts, y = weighted combine
 * (fp32 when out_f32, else the activation dtype).  next_gate_w / next_e_bias
 * (or NULL): the next layer's gate; its predicted experts are copied ahead on
 * the pool's stream while this layer computes.  Synchronises `stream` once
 * (the routing decides the copies). */
ef_status ef_pool_moe_forward(ef_slot_pool* pool, int layer, const void* x, int T, const void* gate_w,
                              const float* e_bias, const void* next_gate_w, const float* next_e_bias, void* y,
                              int out_f32, int32_t* inds_out, float* wts_out, void* workspace,
                              size_t workspace_bytes, void* stream);
ef_status ef_pool_end_token(ef_slot_pool* pool); /* trim + decay every layer (once per token) */
/* One decode step through all n_layers pooled layers: for each layer,
 * r += y (from the previous layer), x = r / sqrt(mean(r^2) + eps) in the
 * activation dtype (the pre-MoE norm), y = ef_pool_moe_forward(layer, x) with
 * the gates of the next `lookahead` layers (0, 1 or 2) routed on x as the
 * lookahead predictions (the nearer layer's copies are queued first); finally
 * r += y and ef_pool_end_token.  r [T, H] fp32 (the residual stream) is updated in place;
 * gate_w / e_bias: n_layers device pointers (e_bias may be NULL, or hold NULLs). */
size_t ef_pool_decode_workspace_size(const ef_slot_pool* pool, int T);
ef_status ef_pool_decode_step(ef_slot_pool* pool, float* r, int T, const void* const* gate_w,
                              const float* const* e_bias, int lookahead, float eps, void* workspace,
                              size_t workspace_bytes, void* stream);
ef_status ef_pool_resident(const ef_slot_pool* pool, int layer, int32_t* experts, int cap, int* n);
/* Routing trace for offline training of the learned eviction predictor (the
 * reference's record_routing / end_token / routing_trace, ef_engine.py:222-229,
 * called at :643-646): while on, every ef_pool_moe_forward records (layer,
 * expert) for each routed entry in (token, k) order and every
 * ef_pool_end_token closes a token.  Turning it on clears the trace. */
ef_status ef_pool_record_routing(ef_slot_pool* pool, int on);
/* pairs [n_pairs][2] (layer, expert) in recording order; token_ends[i] = pairs
 * recorded up to the end of token i.  Copies up to pair_cap pairs and tok_cap
 * ends; n_pairs / n_tokens receive the full counts. */
ef_status ef_pool_routing_trace(const ef_slot_pool* pool, int32_t* pairs, long long pair_cap, long long* n_pairs,
                                long long* token_ends, long long tok_cap, long long* n_tokens);
/* The learned policy's predictor for every layer of a pool created with
 * policy EF_POLICY_BELADY (same layout as ef_policy_set_predictor). */
ef_status ef_pool_set_predictor(ef_slot_pool* pool, int hidden, const float* w1, const float* b1, const float* w2,
                                const float* b2, const float* w3, const float* b3, int trained);

/* ---- GGUF K-quants ------------------------------------------------------------------ */
/* Blocks of 256 elements as the reference decodes them (ef_deepseek_mmap.py:330-378,
 * 655-773): Q2_K 84 B, Q3_K 110 B, Q4_K 144 B per block; value = RN16(d*sc*q - dmin*mn).
 * The reference's Q2_K and Q4_K element orders and Q4_K scale packing are its own
 * (they differ from ggml's); these calls follow the reference. */
#define EF_GGML_Q2_K 10
#define EF_GGML_Q3_K 11
#define EF_GGML_Q4_K 12
/* out fp16 [n_blocks * 256] (16-byte aligned) = the decode of n_blocks consecutive
 * blocks (4-byte aligned), bit-identical to the reference's decoders. */
ef_status ef_kquant_dequantize(int type, const void* blocks, long long n_blocks, void* out, void* stream);
/* Decode GEMV: y fp32 [T, N] = x [T, K] . W^T, W [N, K] stored as N rows of K/256
 * blocks (row r = blocks [r K/256, (r+1) K/256)), i.e. one GGML tensor of shape
 * (K, N) or one expert's slice of a stacked (K, N, E) tensor.  T <= 32, N % 16 == 0,
 * K % 256 == 0; blocks 16-byte (Q4_K) or 4-byte aligned.  Weights are decoded to the
 * same fp16 values as ef_kquant_dequantize, products accumulated in fp32. */
size_t ef_kquant_matmul_workspace_size(int T, int K);
ef_status ef_kquant_matmul(const void* x, int act_dtype, int T, const void* blocks, int type, int N, int K, float* y,
                           void* workspace, size_t workspace_bytes, void* stream);

/* One stacked K-quant projection of a MoE layer: expert e's matrix (N rows of
 * K/256 blocks, i.e. its slice of a GGML (K, N, E) tensor such as
 * blk.{i}.ffn_gate_exps) starts at blocks + e * expert_stride bytes.  blocks
 * and expert_stride 16-byte (Q4_K), 4-byte (Q2_K) or 2-byte (Q3_K) aligned. */
typedef struct {
  const void* blocks;
  int type;                 /* EF_GGML_Q2_K / Q3_K / Q4_K */
  long long expert_stride;  /* bytes; >= N * K / 256 * block bytes */
} ef_kqweight;
/* ef_moe_forward for experts stored as GGUF K-quant blocks (the reference's
 * DeepSeek GGUF models): same router, permutation and combine; each routed
 * (token, k) runs silu(x Wg^T) * (x Wu^T) Wd^T on the fp16 weights the
 * reference's decoders give (ExpertMmapLoader.load_expert_dequantized,
 * ef_deepseek_mmap.py:570-593; MoE forward :1563-1660), decoded inside the GEMV
 * with fp32 accumulation.  cfg->bits / group_size are not used; hidden and
 * inter must be multiples of 256; gate and up share one type, the shared
 * expert's types match the routed ones.  Decode-size batches (the weights
 * are streamed once per 8 routed rows of an expert). */
size_t ef_kquant_moe_workspace_size(const ef_moe_cfg* cfg, int T);
ef_status ef_kquant_moe_forward(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w,
                                const float* e_bias, ef_kqweight gate, ef_kqweight up, ef_kqweight down,
                                const ef_kqweight* shared_gate, const ef_kqweight* shared_up,
                                const ef_kqweight* shared_down, void* y, int32_t* inds_out, float* wts_out,
                                void* workspace, size_t workspace_bytes, void* stream);

/* ---- cold tier: expert blobs read from the model files ----------------------------- */
/* Expert e's copy of one stacked array (w, scales or biases of gate, up or
 * down) occupies bytes [offset + e * stride, offset + e * stride + size) of
 * file `file`, size fixed by the layer shape (MLX safetensors store a stacked
 * tensor [E, ...] contiguously, so stride = size).  bf16 != 0 (scales and
 * biases only): the file holds bf16, converted to fp16 on read; a value fp16
 * cannot hold exactly fails that read with EF_ERR_IO. */
typedef struct {
  int file;
  int bf16;
  long long offset;
  long long stride;
} ef_file_array;
typedef struct ef_expert_store ef_expert_store;
typedef struct {
  size_t blob_bytes;   /* one expert's blob */
  size_t offsets[10];  /* array a (3 * projection + {w, scales, biases}) starts at offsets[a]; [9] = used bytes */
  int n_layers;
  int n_readers;
  int direct;          /* files opened with O_DIRECT */
  long long reads;     /* expert blobs read so far */
  double file_bytes;   /* bytes read so far */
} ef_store_info;
/* Opens n_files files (read-only; direct != 0: O_DIRECT, page cache bypassed)
 * and starts n_readers reader threads (<= 0: 4 x cores, between 8 and 64).  arrays:
 * [n_layers][9] entries in the order gate w, s, b, up w, s, b, down w, s, b;
 * every expert's range is checked against the file size here.  Host only: no
 * CUDA call. */
ef_status ef_store_open(const ef_moe_cfg* cfg, int n_layers, const char* const* paths, int n_files,
                        const ef_file_array* arrays, int n_readers, int direct, ef_expert_store** out);
ef_status ef_store_get_info(const ef_expert_store* store, ef_store_info* out);
/* Reads n expert blobs (layer layers[i], expert experts[i]) into host buffers
 * dst[i] of blob_bytes each, in parallel on the reader threads; returns when
 * all are done (the first error, if any). */
ef_status ef_store_read(ef_expert_store* store, int n, const int32_t* layers, const int32_t* experts,
                        void* const* dst);
ef_status ef_store_close(ef_expert_store* store);
/* A slot pool whose host tier is host_blobs pinned expert blobs (all layers
 * together, least recently used replaced) over `store`: a miss in HBM that
 * is also a miss in the host tier reads the expert from the files; the
 * lookahead starts the reads of the next layer's predicted experts, which
 * overlap this layer's compute.  The store must outlive the pool.  host_blobs
 * >= 2 * top_k; one step needs at most host_blobs distinct experts. */
ef_status ef_pool_create_from_store(const ef_moe_cfg* cfg, const ef_pool_cfg* pool_cfg, ef_expert_store* store,
                                    int host_blobs, ef_slot_pool** out);
ef_status ef_pool_get_stats(ef_slot_pool* pool, ef_pool_stats* out);
ef_status ef_pool_reset_stats(ef_slot_pool* pool);
ef_status ef_pool_destroy(ef_slot_pool* pool);

#ifdef __cplusplus
}
#endif
#endif /* EFMOE_H */
