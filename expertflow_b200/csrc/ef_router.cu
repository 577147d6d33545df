// ef_router.cu -- router logits and top-k selection (sm_100a).
//
// Replaces moe_module.gate(x) and the argpartition / take_along_axis / softmax
// of ef_engine.py:609-619 (and the mlx_lm MoEGate variants the reference calls
// there).  Indices are bit-exact with the CPU oracle:
//   * logits: each 8-element chunk c of the hidden dim belongs to slot c % 128;
//     a CTA's warp w owns slots 32w..32w+31, lane l accumulates its chunks in
//     increasing order (16x16-bit products are exact in fp32, so FMA and
//     mul+add agree), the 32 lanes reduce by xor butterfly, the 4 warp totals
//     combine as (G0 + G1) + (G2 + G3);
//   * selection: top-k by (score desc, index asc) with warp arg-max rounds;
//   * exp / sigmoid: only correctly rounded IEEE operations (see det_expf).
#include "ef_common.cuh"

namespace ef {

__device__ int g_router_dummy;

// ---------------------------------------------------------------- deterministic exp
// Cody-Waite: x = n*ln2 + r, ln2 = LN2_HI (16 significant bits) + LN2_LO, so
// n*LN2_HI is exact for |n| < 256; e^r by its degree-7 Taylor polynomial
// (|r| <= ln2/2, truncation < 1e-8 relative) in Horner form; then an exact
// multiplication by 2^n (two steps when the result is subnormal).
#define EF_LOG2E 1.44269502162933349609375f
#define EF_LN2_HI 0.693145751953125f
#define EF_LN2_LO 1.428606765330187045e-06f

EF_DEV float pow2f(int n) { return __int_as_float((n + 127) << 23); }

EF_DEV float det_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228393554688f) return __int_as_float(0x7f800000);
  if (x < -103.972084045410f) return 0.0f;
  float n = rintf(__fmul_rn(x, EF_LOG2E));
  float r = __fsub_rn(x, __fmul_rn(n, EF_LN2_HI));
  r = __fsub_rn(r, __fmul_rn(n, EF_LN2_LO));
  float p = 1.98412698412698412698e-04f;
  p = __fadd_rn(__fmul_rn(p, r), 1.38888888888888888889e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 8.33333333333333333333e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 4.16666666666666666667e-02f);
  p = __fadd_rn(__fmul_rn(p, r), 1.66666666666666666667e-01f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  int ni = static_cast<int>(n);
  if (ni > 127) { p = __fmul_rn(p, pow2f(127)); ni -= 127; }
  if (ni < -126) { p = __fmul_rn(p, pow2f(-64)); ni += 64; }
  if (ni < -126) { p = __fmul_rn(p, pow2f(-64)); ni += 64; }
  return __fmul_rn(p, pow2f(ni));
}

EF_DEV float det_sigmoidf(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-x))); }

// ---------------------------------------------------------------- logits
EF_DEV void cvt8(const uint4& v, int is_bf16, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (is_bf16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 ff = __half22float2(h);
      f[2 * i] = ff.x;
      f[2 * i + 1] = ff.y;
    }
  }
}

// CTA = 4 warps computes logits for TT tokens x TE experts.  blockIdx.z = 1
// and 2 take a second and third gate (wg2 -> logits2, wg3 -> logits3) over the
// same tokens, so a layer's routing and the predictions of the next layers
// share one launch.
template <int TT, int TE>
__global__ void __launch_bounds__(128) router_logits_kernel(const uint16_t* __restrict__ x, int x_bf16,
                                                            const uint16_t* __restrict__ wg, int w_bf16,
                                                            int T, int E, int H, float* __restrict__ logits,
                                                            const uint16_t* __restrict__ wg2,
                                                            float* __restrict__ logits2,
                                                            const uint16_t* __restrict__ wg3,
                                                            float* __restrict__ logits3) {
  pdl_wait();
  pdl_launch_next();
  if (blockIdx.z == 1) {
    wg = wg2;
    logits = logits2;
  } else if (blockIdx.z == 2) {
    wg = wg3;
    logits = logits3;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
  const int nch = H >> 3;
  float acc[TT][TE];
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < TE; ++b) acc[a][b] = 0.0f;

  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const uint4* wv = reinterpret_cast<const uint4*>(wg);
  // small tiles: several iterations' loads in flight per thread (a thread's
  // FMA order over c is unchanged)
#pragma unroll(TT * TE <= 4 ? 4 : 1)
  for (int c = warp * 32 + lane; c < nch; c += 128) {
    float xf[TT][8], wf[TE][8];
#pragma unroll
    for (int a = 0; a < TT; ++a) {
      int t = min(t0 + a, T - 1);
      uint4 v = __ldg(xv + (size_t)t * nch + c);
      cvt8(v, x_bf16, xf[a]);
    }
#pragma unroll
    for (int b = 0; b < TE; ++b) {
      int e = min(e0 + b, E - 1);
      uint4 v = __ldg(wv + (size_t)e * nch + c);
      cvt8(v, w_bf16, wf[b]);
    }
#pragma unroll
    for (int a = 0; a < TT; ++a)
#pragma unroll
      for (int b = 0; b < TE; ++b)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[a][b] = __fmaf_rn(xf[a][i], wf[b][i], acc[a][b]);  // exact product: one rounding either way
  }
  __shared__ float part[4][TT][TE];
#pragma unroll
  for (int a = 0; a < TT; ++a)
#pragma unroll
    for (int b = 0; b < TE; ++b) {
      float v = acc[a][b];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
      if (lane == 0) part[warp][a][b] = v;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < TT * TE; i += blockDim.x) {
    int a = i / TE, b = i % TE;
    int t = t0 + a, e = e0 + b;
    if (t < T && e < E) {
      float v = __fadd_rn(__fadd_rn(part[0][a][b], part[1][a][b]), __fadd_rn(part[2][a][b], part[3][a][b]));
      logits[(size_t)t * E + e] = v;
    }
  }
}

// ---------------------------------------------------------------- selection
struct SelCfg {
  int E, k, mode, norm_topk, n_group, topk_group;
  float scaling;
};

EF_DEV bool ranks_before(float va, int ia, float vb, int ib) { return (va > vb) || (va == vb && ia < ib); }

// Order-preserving unsigned key of a float (larger float -> larger key; -0
// and +0 map to the same key, as they compare equal).
EF_DEV uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));  // -0 + 0 = +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Warp-wide arg-max by (value desc, index asc) from each lane's candidate
// (key 0 and index 0x7fffffff for none): the largest key, then the smallest
// index among the lanes that hold it -- two warp reductions.
EF_DEV int warp_argmax_key(uint32_t key, int idx) {
  const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
  return (int)__reduce_min_sync(0xffffffffu, key == kmax ? (uint32_t)idx : 0x7fffffffu);
}

// warp-wide arg-max by (value desc, index asc)
EF_DEV void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, off);
    int oi = __shfl_xor_sync(0xffffffffu, i, off);
    if (ranks_before(ov, oi, v, i)) { v = ov; i = oi; }
  }
}

constexpr int kMaxE = 512;
constexpr int kSelWarps = 4;

// One warp per token.  Scores live in shared memory (E <= 512).  blockIdx.y = 1
// and 2 select the second and third gate's logits / bias / outputs (see
// router_logits_kernel).
// PER: score keys per lane (E <= 32 PER); the picks do not depend on it.
template <int PER>
__global__ void __launch_bounds__(kSelWarps * 32) router_select_kernel(const float* __restrict__ logits,
                                                                       const float* __restrict__ e_bias, int T,
                                                                       SelCfg cfg, int* __restrict__ inds,
                                                                       float* __restrict__ wts,
                                                                       const float* __restrict__ logits2,
                                                                       const float* __restrict__ e_bias2,
                                                                       int* __restrict__ inds2,
                                                                       float* __restrict__ wts2,
                                                                       const float* __restrict__ logits3,
                                                                       const float* __restrict__ e_bias3,
                                                                       int* __restrict__ inds3,
                                                                       float* __restrict__ wts3) {
  pdl_wait();
  pdl_launch_next();
  if (blockIdx.y == 1) {
    logits = logits2;
    e_bias = e_bias2;
    inds = inds2;
    wts = wts2;
  } else if (blockIdx.y == 2) {
    logits = logits3;
    e_bias = e_bias3;
    inds = inds3;
    wts = wts3;
  }
  __shared__ float s_score[kSelWarps][kMaxE];  // selection score
  __shared__ float s_keep[kSelWarps][kMaxE];   // sigmoid value / logit for weights
  __shared__ float s_gs[kSelWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kSelWarps + warp;
  if (t >= T) return;
  const int E = cfg.E, k = cfg.k;
  float* sc = s_score[warp];
  float* kv = s_keep[warp];
  const float* l = logits + (size_t)t * E;
  if (cfg.mode == 0) {
    for (int e = lane; e < E; e += 32) {
      float v = l[e];
      if (e_bias) v = __fadd_rn(v, e_bias[e]);
      sc[e] = v;
      kv[e] = v;
    }
  } else {
    for (int e = lane; e < E; e += 32) {
      float s = det_sigmoidf(l[e]);
      kv[e] = s;
      sc[e] = e_bias ? __fadd_rn(s, e_bias[e]) : s;
    }
  }
  __syncwarp();
  if (cfg.mode == 1 && cfg.n_group > 1) {
    const int G = cfg.n_group, gsz = E / G;
    if (lane < G) {
      float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll 8
      for (int e = lane * gsz; e < (lane + 1) * gsz; ++e) {
        float v = sc[e];
        if (v > m1) { m2 = m1; m1 = v; }
        else if (v > m2) { m2 = v; }
      }
      s_gs[warp][lane] = __fadd_rn(m1, m2);
    }
    __syncwarp();
    // keep the top `topk_group` groups by (score desc, group asc)
    unsigned keep = 0u;
    float gv = lane < G ? s_gs[warp][lane] : -INFINITY;
    int gi = lane < G ? lane : 0x7fffffff;
    for (int r = 0; r < cfg.topk_group; ++r) {
      float bv = ((keep >> lane) & 1u) ? -INFINITY : gv;
      int bi = ((keep >> lane) & 1u) ? 0x7fffffff : gi;
      warp_argmax(bv, bi);
      keep |= 1u << bi;
    }
    for (int e = lane; e < E; e += 32)
      if (!((keep >> (e / gsz)) & 1u)) sc[e] = 0.0f;
    __syncwarp();
  }
  // top-k over sc by (value desc, index asc); each lane keeps the keys of its
  // elements e = lane + 32 r, a taken element's key drops to 0.  Lane j < k
  // keeps the j-th pick (no per-thread arrays indexed by j: they would live
  // in local memory).
  constexpr int kPerLane = PER;
  uint32_t keys[kPerLane];
#pragma unroll
  for (int r = 0; r < kPerLane; ++r) keys[r] = lane + 32 * r < E ? order_key(sc[lane + 32 * r]) : 0u;
  int my_sel = 0;
  for (int j = 0; j < k; ++j) {
    uint32_t bk = 0u;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < kPerLane; ++r)
      if (keys[r] > bk) {  // strict: the lane's lower index wins ties
        bk = keys[r];
        bi = lane + 32 * r;
      }
    const int win = warp_argmax_key(bk, bi);
    if (lane == j) my_sel = win;
    const bool own = (win & 31) == lane;
    const int wr = win >> 5;
#pragma unroll
    for (int r = 0; r < kPerLane; ++r) keys[r] = (own && r == wr) ? 0u : keys[r];
  }
  // weights of the picks, lane j for pick j; sums over the picks run in j
  // order (shuffles bring the values to every lane), as the oracle adds them
  const bool mine = lane < k;
  float w = 0.0f;
  if (cfg.mode == 0) {
    const float m = kv[__shfl_sync(0xffffffffu, my_sel, 0)];
    if (cfg.norm_topk) {
      w = mine ? det_expf(__fsub_rn(kv[my_sel], m)) : 0.0f;
      float s = __shfl_sync(0xffffffffu, w, 0);
      for (int j = 1; j < k; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, w, j));
      w = __fdiv_rn(w, s);
    } else {
      float z = 0.0f;
      for (int e = lane; e < E; e += 32) z = __fadd_rn(z, det_expf(__fsub_rn(kv[e], m)));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) z = __fadd_rn(z, __shfl_xor_sync(0xffffffffu, z, off));
      w = mine ? __fdiv_rn(det_expf(__fsub_rn(kv[my_sel], m)), z) : 0.0f;
    }
  } else {
    w = mine ? kv[my_sel] : 0.0f;
    float s = __shfl_sync(0xffffffffu, w, 0);
    for (int j = 1; j < k; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, w, j));
    if (cfg.norm_topk && k > 1) w = __fdiv_rn(w, s);
    w = __fmul_rn(w, cfg.scaling);
  }
  if (mine) {
    inds[(size_t)t * k + lane] = my_sel;
    wts[(size_t)t * k + lane] = w;
  }
}

// ---------------------------------------------------------------- launchers
// wg2 / logits2, wg3 / logits3 (optional, wg3 only with wg2): further gates
// routed over the same tokens in the same launch.
cudaError_t launch_router_logits(const uint16_t* x, int x_bf16, const uint16_t* wg, int w_bf16, int T, int E,
                                 int H, float* logits, cudaStream_t st, const uint16_t* wg2, float* logits2,
                                 const uint16_t* wg3, float* logits3) {
  const int nz = wg2 ? (wg3 ? 3 : 2) : 1;
  if (T >= 64) {
    dim3 grid((T + 7) / 8, (E + 7) / 8, nz);
    return launch_pdl(router_logits_kernel<8, 8>, grid, 128, 0, st, x, x_bf16, wg, w_bf16, T, E, H, logits, wg2,
                      logits2, wg3, logits3);
  } else if (T >= 4) {
    dim3 grid((T + 3) / 4, (E + 3) / 4, nz);
    return launch_pdl(router_logits_kernel<4, 4>, grid, 128, 0, st, x, x_bf16, wg, w_bf16, T, E, H, logits, wg2,
                      logits2, wg3, logits3);
  } else {
    int te = (E >= 256) ? 2 : 1;
    dim3 grid(T, (E + te - 1) / te, nz);
    if (te == 2)
      return launch_pdl(router_logits_kernel<1, 2>, grid, 128, 0, st, x, x_bf16, wg, w_bf16, T, E, H, logits, wg2,
                        logits2, wg3, logits3);
    else
      return launch_pdl(router_logits_kernel<1, 1>, grid, 128, 0, st, x, x_bf16, wg, w_bf16, T, E, H, logits, wg2,
                        logits2, wg3, logits3);
  }
  return cudaGetLastError();
}

cudaError_t launch_router_select(const float* logits, const float* e_bias, int T, int E, int k, int mode,
                                 int norm_topk, int n_group, int topk_group, float scaling, int* inds, float* wts,
                                 cudaStream_t st, const float* logits2, const float* e_bias2, int* inds2,
                                 float* wts2, const float* logits3, const float* e_bias3, int* inds3, float* wts3) {
  SelCfg c{E, k, mode, norm_topk, n_group, topk_group, scaling};
  dim3 grid((T + kSelWarps - 1) / kSelWarps, logits2 ? (logits3 ? 3 : 2) : 1);
  if (E <= 128)
    return launch_pdl(router_select_kernel<4>, grid, kSelWarps * 32, 0, st, logits, e_bias, T, c, inds, wts, logits2,
                      e_bias2, inds2, wts2, logits3, e_bias3, inds3, wts3);
  if (E <= 256)
    return launch_pdl(router_select_kernel<8>, grid, kSelWarps * 32, 0, st, logits, e_bias, T, c, inds, wts, logits2,
                      e_bias2, inds2, wts2, logits3, e_bias3, inds3, wts3);
  return launch_pdl(router_select_kernel<kMaxE / 32>, grid, kSelWarps * 32, 0, st, logits, e_bias, T, c, inds, wts, logits2, e_bias2,
                    inds2, wts2, logits3, e_bias3, inds3, wts3);
}

}  // namespace ef
