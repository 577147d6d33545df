// ef_permute.cu -- token permutation, activation staging and weighted combine.
//
// Replaces the per-token / per-k Python loops of ef_engine.py:636-704:
//   * permute: routed entries (t, j) are grouped by expert with a stable
//     counting sort (order (expert, t*k + j)) computed without atomics: warps
//     histogram their slice with __match_any_sync leaders, one CTA scans, the
//     same warps scatter; the shared expert (ef_engine.py:628-631) is an extra
//     bin holding every token.  It also cuts each expert's rows into segments
//     for the grouped kernels.
//   * prep: activations -> fp16 in "pair order" (per 8 columns: c0 c4 c1 c5
//     c2 c6 c3 c7, the order in which the GEMV kernel unpacks nibble pairs),
//     plus fp32 sums per 64-column group (for the affine bias term).
//   * combine: y[t] = sum_j w[t, j] * rows[inv[t, j]] in j order, + shared row
//     (ef_engine.py:695-703).
#include "ef_common.cuh"

namespace ef {

constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;

// Block-wide exclusive scan of one value per thread (1024 threads).
__device__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
    int ws = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, ws, off);
      if (lane >= off) ws += y;
    }
    s_warp[lane] = ws - w;  // exclusive warp base
    if (lane == 31) *total = ws;
  }
  __syncthreads();
  int r = s_warp[warp] + x - v;
  __syncthreads();
  return r;
}

// Stable counting sort of n_ent entries into bins by one CTA of kPermThreads
// threads, without atomics: warps histogram their slice of the entries with
// __match_any_sync leaders, one block scan gives each bin's first row and each
// warp's base within it, the same warps scatter in entry order.  bin_of(j)
// returns entry j's bin in [0, n_bin) (out-of-range ids are reported in the
// device error word and sorted into bin 0); emit(j, pos) records that entry j
// landed on sorted row pos.  n_sh > 0 appends bin n_bin with n_sh rows,
// emit_shared(t, pos) for t < n_sh.  Writes pb.counts / offsets and segments of
// at most seg_chunk rows.  s_hist: kPermWarps * (n_bin + 1) ints of shared memory.
template <class BinOf, class Emit, class EmitShared>
__device__ void counting_sort_cta(int n_ent, int n_bin, int n_sh, int seg_chunk, const PermBufs& pb, int* s_hist,
                                  int* s_warp, int* s_total, BinOf bin_of, Emit emit, EmitShared emit_shared) {
  const int nb = n_bin + (n_sh > 0 ? 1 : 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kPermWarps * nb; i += kPermThreads) s_hist[i] = 0;
  __syncthreads();
  int per = (n_ent + kPermWarps - 1) / kPermWarps;
  per = (per + 31) & ~31;
  const int beg = warp * per, end = min(n_ent, beg + per);
  int* hist = s_hist + warp * nb;
  // phase 1: per-warp histogram
  for (int base = beg; base < end; base += 32) {
    const int j = base + lane;
    const bool valid = j < end;
    int e = valid ? bin_of(j) : -1;
    if (valid && (e < 0 || e >= n_bin)) {
      ef_set_error(kDevErrRange);
      e = 0;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (valid && lane == __ffs(peers) - 1) hist[e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // phase 2: totals, offsets, per-warp bases
  int cnt = 0;
  const int b = threadIdx.x;
  if (b < nb) {
    if (b < n_bin) {
      for (int w = 0; w < kPermWarps; ++w) cnt += s_hist[w * nb + b];
    } else {
      cnt = n_sh;
    }
  }
  const int off = block_exclusive_scan(b < nb ? cnt : 0, s_warp, s_total);
  if (b < nb) {
    pb.counts[b] = cnt;
    pb.offsets[b] = off;
    if (b == nb - 1) pb.offsets[nb] = off + cnt;
    if (b < n_bin) {
      int run = off;
      for (int w = 0; w < kPermWarps; ++w) {
        const int c = s_hist[w * nb + b];
        s_hist[w * nb + b] = run;
        run += c;
      }
    }
  }
  __syncthreads();
  // phase 3: stable scatter
  for (int base = beg; base < end; base += 32) {
    const int j = base + lane;
    const bool valid = j < end;
    int e = valid ? bin_of(j) : -1;
    if (valid && (e < 0 || e >= n_bin)) e = 0;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (valid) emit(j, hist[e] + __popc(peers & ((1u << lane) - 1u)));
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) hist[e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  if (n_sh > 0) {
    const int base = pb.offsets[n_bin];
    for (int t = threadIdx.x; t < n_sh; t += kPermThreads) emit_shared(t, base + t);
  }
  // phase 4: segments of at most seg_chunk rows
  const int nseg = (b < nb) ? (cnt + seg_chunk - 1) / seg_chunk : 0;
  const int sbase = block_exclusive_scan(nseg, s_warp, s_total);
  if (b < nb) {
    for (int q = 0; q < nseg; ++q) {
      pb.seg_expert[sbase + q] = b;
      pb.seg_row0[sbase + q] = off + q * seg_chunk;
      pb.seg_nrows[sbase + q] = min(seg_chunk, cnt - q * seg_chunk);
    }
  }
  if (threadIdx.x == 0) *pb.n_seg = *s_total;
}

// entries: n_ent routed entries (expert id per entry; token = entry / k).
// n_sh: rows of the shared bin (0 or T), bin index n_exp.
__global__ void __launch_bounds__(kPermThreads) permute_kernel(const int* __restrict__ entries, int n_ent, int k,
                                                               int n_exp, int n_sh, int seg_chunk, PermBufs pb) {
  pdl_wait();
  pdl_launch_next();
  extern __shared__ int s_hist[];  // [kPermWarps][nb]
  __shared__ int s_warp[32];
  __shared__ int s_total;
  counting_sort_cta(
      n_ent, n_exp, n_sh, seg_chunk, pb, s_hist, s_warp, &s_total, [&](int j) { return entries[j]; },
      [&](int j, int pos) {
        pb.row_src[pos] = j / k;
        pb.inv[j] = pos;
      },
      [&](int t, int pos) { pb.row_src[pos] = t; });
}

// ---------------------------------------------------------------- prep
// Output row j = act[row_src[j]] (or act[j] when row_src is null), converted
// to fp16 in the GEMV activation layout (act_pos for `bits`), plus the sums
// [n, sum_ld(K)] of each 64-column group.  Gathering the routed rows here makes
// every segment's rows contiguous for the GEMV kernel's tile loads.  n_dev
// (or null): the row count in device memory (at most n), for callers whose
// row count is only known on the device; the grid then strides over the rows.
__global__ void prep_act_kernel(const uint16_t* __restrict__ act, const int* __restrict__ row_src, int is_bf16, int n,
                                const int* __restrict__ n_dev, int K, int bits, uint16_t* __restrict__ out,
                                float* __restrict__ sums) {
  pdl_wait();  // its successor, a persistent GEMV / GEMM, launches at its completion
  const int nblk = K >> 3;
  if (n_dev) n = min(n, max(0, *n_dev));
  const long long total = (long long)n * nblk;
  const long long stride = (long long)gridDim.x * blockDim.x;
  // uniform trip count across the block: the group-sum shuffles need every lane
  for (long long base = (long long)blockIdx.x * blockDim.x; base < total; base += stride) {
    const long long gid = base + threadIdx.x;
    const bool valid = gid < total;
    const long long g = valid ? gid : 0;
    const long long orow = g / nblk;
    const long long irow = row_src ? __ldg(row_src + orow) : orow;
    const uint4 v = reinterpret_cast<const uint4*>(act)[irow * nblk + (g - orow * nblk)];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = act_to_f32(static_cast<uint16_t>(w[i] & 0xffffu), is_bf16);
      f[2 * i + 1] = act_to_f32(static_cast<uint16_t>(w[i] >> 16), is_bf16);
    }
    uint16_t h[8];
    float s = 0.0f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!(fabsf(f[i]) <= 65504.0f)) bad = true;
      const __half hv = __float2half_rn(f[i]);
      h[i] = __half_as_ushort(hv);
      s += __half2float(hv);
    }
    if (valid && bad) ef_set_error(kDevErrRange);
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      o[q] = (uint32_t)h[act_col(2 * q, bits)] | ((uint32_t)h[act_col(2 * q + 1, bits)] << 16);
    if (valid) reinterpret_cast<uint4*>(out)[g] = make_uint4(o[0], o[1], o[2], o[3]);
    // 8 consecutive threads cover one 64-column group (nblk is a multiple of 8)
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (valid && (gid & 7) == 0) {
      const long long row = gid / nblk;
      const int grp = (int)((gid - row * nblk) >> 3);
      sums[row * sum_ld(K) + grp] = s;
    }
  }
}

// ---------------------------------------------------------------- combine
// out[t, c] = sum_j wts[t, j] * rows[inv[t*k + j], c]  (+ rows[sh_base + t, c])
// wts == nullptr means unit weights.  out dtype: 0 bf16, 1 fp16, 2 fp32.
// wait_flags (or null): the rows are written by peer GPUs; every CTA first
// waits (bounded) until flags 0..n_wait-1 (64 bytes apart) reach *epoch.
__global__ void combine_kernel(const float* rows, const int* __restrict__ inv, const float* __restrict__ wts, int T,
                               int k, int H, int sh_base, void* __restrict__ out, int out_dtype,
                               const uint32_t* wait_flags, int n_wait, const uint32_t* epoch) {
  pdl_wait();
  if (wait_flags) {
    const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(epoch);
    if ((int)threadIdx.x < n_wait) wait_flag_sys(wait_flags + threadIdx.x * 16, ep);
    __syncthreads();
  }
  pdl_launch_next();
  const int t = blockIdx.y;
  const int c4 = blockIdx.x * blockDim.x + threadIdx.x;  // index of a 4-column quad
  if (t >= T || c4 * 4 >= H) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  // unrolled so that several rows' loads are in flight (the sum stays in j order)
#pragma unroll 4
  for (int j = 0; j < k; ++j) {
    int r = inv[(size_t)t * k + j];
    float w = wts ? wts[(size_t)t * k + j] : 1.0f;
    float4 v = reinterpret_cast<const float4*>(rows + (size_t)r * H)[c4];
    if (j == 0) {
      acc = make_float4(v.x * w, v.y * w, v.z * w, v.w * w);
    } else {
      acc.x += v.x * w; acc.y += v.y * w; acc.z += v.z * w; acc.w += v.w * w;
    }
  }
  if (sh_base >= 0) {
    float4 v = reinterpret_cast<const float4*>(rows + (size_t)(sh_base + t) * H)[c4];
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  size_t o = (size_t)t * H + (size_t)c4 * 4;
  if (out_dtype == 2) {
    reinterpret_cast<float4*>(static_cast<float*>(out) + o)[0] = acc;
  } else if (out_dtype == 1) {
    __half2 a = __floats2half2_rn(acc.x, acc.y), b = __floats2half2_rn(acc.z, acc.w);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + o) = u;
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y), b = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + o) = u;
  }
}

// ---------------------------------------------------------------- launchers
cudaError_t launch_permute(const int* entries, int n_ent, int k, int n_exp, int n_sh, int seg_chunk,
                           const PermBufs& pb, cudaStream_t st) {
  const int nb = n_exp + (n_sh > 0 ? 1 : 0);
  size_t smem = sizeof(int) * (size_t)kPermWarps * nb;
  static std::atomic<bool> attr_set[64];
  const cudaError_t e = set_max_smem_once(permute_kernel, 160 * 1024, attr_set);
  if (e != cudaSuccess) return e;
  return launch_pdl(permute_kernel, 1, kPermThreads, smem, st, entries, n_ent, k, n_exp, n_sh, seg_chunk, pb);
}

// n_dev (or null): the device-side row count (<= n); the grid is then capped
// at max_blocks and strides over the rows.
cudaError_t launch_prep_act(const uint16_t* act, const int* row_src, int is_bf16, int n, int K, int bits,
                            uint16_t* out, float* sums, cudaStream_t st, const int* n_dev, int max_blocks) {
  long long total = (long long)n * (K / 8);
  if (total == 0) return cudaSuccess;
  int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (n_dev && max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
  return launch_pdl(prep_act_kernel, (unsigned)blocks, threads, 0, st, act, row_src, is_bf16, n, n_dev, K, bits, out,
                    sums);
}

cudaError_t launch_combine(const float* rows, const int* inv, const float* wts, int T, int k, int H, int sh_base,
                           void* out, int out_dtype, cudaStream_t st, const uint32_t* wait_flags, int n_wait,
                           const uint32_t* epoch) {
  if (T == 0) return cudaSuccess;
  int quads = H / 4;
  int threads = quads < 256 ? ((quads + 31) / 32) * 32 : 256;
  if (wait_flags && threads < n_wait) threads = ((n_wait + 31) / 32) * 32;
  dim3 grid((quads + threads - 1) / threads, T);
  return launch_pdl(combine_kernel, grid, threads, 0, st, rows, inv, wts, T, k, H, sh_base, out, out_dtype,
                    wait_flags, n_wait, epoch);
}

}  // namespace ef
