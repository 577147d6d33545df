// ef_qgemm.cu -- prefill-size grouped quantised GEMM on tcgen05 / TMEM (sm_100a).
//
// Replaces the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694
// when an expert receives many tokens (prefill): the expert matmuls become a
// dense grouped contraction  Y[tokens, out] = X[tokens, K] . dequant(W)[out, K]^T
// per expert, run on the 5th-generation tensor cores with fp32 accumulation in
// tensor memory.
//
// Work item = (segment of <= 128 rows routed to one expert) x (128 weight rows);
// for the gate/up pass the 128 rows are 64 gate rows + the same 64 up rows, so
// the SwiGLU pairs meet in one accumulator.  One persistent CTA per SM:
//   warp 0      TMA: per 64-column K chunk, the code tile(s) (swizzled) and the
//               activation tile [128 rows x 64 cols] fp16 (128-B swizzle, which
//               is the UMMA K-major canonical layout) into a 4-deep ring
//   warp 1      TMEM allocation; lane 0 issues tcgen05.mma (M=128, N<=128,
//               K=16) into one of two TMEM accumulators and commits
//   warps 2-5   dequantise: codes -> exact fp16 q (mantissa trick + one fp16
//               FMA) -> fp16 s*q + b (one fp16 FMA, single rounding) written as
//               the UMMA A tile (K-major, 128-B swizzle)
//   warps 6-9   epilogue: tcgen05.ld of the accumulator; gate/up pass:
//               h = silu(g) * u -> fp16 rows; down pass: fp32 rows
// The activation columns carry the same within-block permutation as the GEMV
// path (act_pos), and the dequantised A rows are written in that order, so the
// contraction over K is unchanged.  Every wait is bounded; TMEM is released on
// every exit path.
#include "ef_common.cuh"

namespace ef {

constexpr int kGemmM = 128;          // weight rows per item (UMMA M)
constexpr int kGemmN = 128;          // routed rows per segment (max UMMA N used)
constexpr int kGemmKC = 64;          // K columns per chunk (one quantisation group)
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 320;    // 10 warps
constexpr int kTmemCols = 256;       // two accumulators of kGemmN fp32 columns
constexpr int kExchPitch = kGemmN + 1;  // floats; odd pitch keeps the exchange conflict-free

template <int BITS>
struct GemmShape {
  static constexpr int CROW = kGemmKC * BITS / 8;          // code bytes per row per chunk (64 / 32)
  static constexpr int CODE_BYTES = kGemmM * CROW;          // 8 KB / 4 KB
  static constexpr int A_BYTES = kGemmM * kGemmKC * 2;      // 16 KB fp16
  static constexpr int B_BYTES = kGemmN * kGemmKC * 2;      // 16 KB fp16
  static constexpr int CODE_OFF = 0;
  static constexpr int A_OFF = (CODE_BYTES + 1023) / 1024 * 1024;
  static constexpr int B_OFF = A_OFF + A_BYTES;
  static constexpr int STAGE = B_OFF + B_BYTES;
};

constexpr size_t gemm_smem_bytes(int bits) {
  return 1024 + (size_t)kGemmStages * (bits == 4 ? GemmShape<4>::STAGE : GemmShape<8>::STAGE) +
         64 * kExchPitch * 4 /* up-half exchange */ + 512 /* barriers + tmem addr */;
}

struct GemmParams {
  CUtensorMap tm_c0, tm_c1;    // routed codes (gate/up or down), 2-D [E*R, K*bits/32]
  CUtensorMap tm_sc0, tm_sc1;  // shared-expert codes
  CUtensorMap tm_act;          // activation rows [n_rows, K] fp16, box 64 x 128, 128-B swizzle
  const uint16_t* s0; const uint16_t* b0; const uint16_t* s1; const uint16_t* b1;
  const uint16_t* ss0; const uint16_t* sb0; const uint16_t* ss1; const uint16_t* sb1;
  const int* seg_expert; const int* seg_row0; const int* seg_nrows; const int* n_seg;
  int K;              // input dim
  int R;              // output rows per expert (gate/up pass: I, down pass: H)
  int n_experts;      // expert id == n_experts selects the shared expert
  uint16_t* h_out;    // gate/up pass: fp16 [n_rows, R] in the activation layout
  float* y_out;       // down pass: fp32 [n_rows, R]
};

// ---------------------------------------------------------------- tcgen05 helpers
EF_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                  // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                  // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                  // 128-byte swizzle
  return d;
}
EF_DEV uint32_t umma_idesc_f16_f32(int M, int N) {
  return (1u << 4)                         // D = f32
         | (0u << 7) | (0u << 10)          // A, B = f16
         | (0u << 15) | (0u << 16)         // both K-major
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
EF_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
EF_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
EF_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
EF_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
EF_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
EF_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct GemmItem {
  int expert, row0_seg, nrows, rt;
};
EF_DEV GemmItem gemm_item(const GemmParams& p, int w, int n_rt) {
  GemmItem it;
  const int seg = w / n_rt;
  it.rt = w - seg * n_rt;
  it.expert = __ldg(p.seg_expert + seg);
  it.row0_seg = __ldg(p.seg_row0 + seg);
  it.nrows = __ldg(p.seg_nrows + seg);
  return it;
}

// fp16 pair (1 + qa/1024, 1 + qb/1024) -> (s qa + b, s qb + b), exact q then one rounding
EF_DEV uint32_t dq_pair(uint32_t v, __half2 s2, __half2 b2) {
  const __half2 q = __hfma2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1024.0f),
                            __float2half2_rn(-1024.0f));
  const __half2 w = __hfma2(q, s2, b2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

template <int BITS, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) qgemm_kernel(const __grid_constant__ GemmParams p) {
  using S = GemmShape<BITS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* exch = reinterpret_cast<float*>(smem + (size_t)kGemmStages * S::STAGE);  // [64][kExchPitch]
  uint64_t* bars = reinterpret_cast<uint64_t*>(exch + 64 * kExchPitch + 2);  // 8-byte aligned
  uint64_t* full = bars;                       // [stages] TMA landed
  uint64_t* aready = bars + kGemmStages;       // [stages] A tile written (4 dequant warps)
  uint64_t* sfree = bars + 2 * kGemmStages;    // [stages] MMAs of the stage done (commit)
  uint64_t* accf = bars + 3 * kGemmStages;     // [2] accumulator full (commit)
  uint64_t* acce = accf + 2;                   // [2] accumulator drained (4 epilogue warps)
  uint64_t* exb = acce + 2;                    // [2] exchange written / consumed
  uint64_t* drain = exb + 2;                   // final MMA drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemmStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&aready[i], 4);
      mbar_init(&sfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 4);
      mbar_init(&exb[i], 4);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  if (warp == 1) {  // TMEM allocation (whole warp)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_rt = MODE == 0 ? p.R / (kGemmM / 2) : p.R / kGemmM;
  const int n_work = (*p.n_seg) * n_rt;
  const int nk = p.K / kGemmKC;
  const int ng = p.K / 64;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&p.tm_c0);
      prefetch_tmap(&p.tm_act);
      uint32_t f = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const bool shared = it.expert >= p.n_experts;
        const int e = shared ? 0 : it.expert;
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % kGemmStages;
          if (f >= (uint32_t)kGemmStages &&
              !mbar_wait(&sfree[st], ((f / kGemmStages) - 1) & 1u, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* stage = smem + (size_t)st * S::STAGE;
          mbar_arrive_expect_tx(&full[st], S::CODE_BYTES + S::B_BYTES);
          const int kw = kc * (kGemmKC * BITS / 32);
          if (MODE == 0) {
            const int r0 = e * p.R + it.rt * (kGemmM / 2);
            tma_load_2d(stage + S::CODE_OFF, shared ? &p.tm_sc0 : &p.tm_c0, kw, r0, &full[st]);
            tma_load_2d(stage + S::CODE_OFF + S::CODE_BYTES / 2, shared ? &p.tm_sc1 : &p.tm_c1, kw, r0, &full[st]);
          } else {
            tma_load_2d(stage + S::CODE_OFF, shared ? &p.tm_sc0 : &p.tm_c0, kw, e * p.R + it.rt * kGemmM, &full[st]);
          }
          tma_load_2d(stage + S::B_OFF, &p.tm_act, kc * kGemmKC, it.row0_seg, &full[st]);
        }
      }
      for (uint32_t i = (f > (uint32_t)kGemmStages ? f - kGemmStages : 0); i < f; ++i)
        mbar_wait(&full[i % kGemmStages], (i / kGemmStages) & 1u, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t f = 0, item = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++item) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const int N = (it.nrows + 15) & ~15;
        const uint32_t idesc = umma_idesc_f16_f32(kGemmM, N);
        const int buf = item & 1;
        // wait until the epilogue drained this accumulator (two items ago)
        if (item >= 2 && !mbar_wait(&acce[buf], ((item >> 1) - 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(buf * kGemmN);
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % kGemmStages;
          if (!mbar_wait(&aready[st], (f / kGemmStages) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
          tc_fence_after();
          const uint8_t* stage = smem + (size_t)st * S::STAGE;
          const uint64_t ad = umma_desc_sw128(smem_u32(stage + S::A_OFF));
          const uint64_t bd = umma_desc_sw128(smem_u32(stage + S::B_OFF));
#pragma unroll
          for (int k = 0; k < kGemmKC / 16; ++k)  // K advance inside the 128-B swizzle atom: 32 B per step
            umma_f16(tmem_d, ad + (uint64_t)((k * 32) >> 4), bd + (uint64_t)((k * 32) >> 4), idesc,
                     (kc > 0 || k > 0) ? 1u : 0u);
          umma_commit(&sfree[st]);  // frees the stage when these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&accf[buf]);  // accumulator complete
      }
      // drain any MMAs still in flight before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, kDevErrTimeoutTc);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ dequantisers
    const int d = threadIdx.x - 64;  // A row 0..127
    uint32_t f = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
      const GemmItem it = gemm_item(p, w, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const int e = shared ? 0 : it.expert;
      const uint16_t* sp;
      const uint16_t* bp;
      size_t row;
      if (MODE == 0) {
        const bool up = d >= 64;
        sp = up ? (shared ? p.ss1 : p.s1) : (shared ? p.ss0 : p.s0);
        bp = up ? (shared ? p.sb1 : p.b1) : (shared ? p.sb0 : p.b0);
        row = (size_t)e * p.R + (size_t)it.rt * (kGemmM / 2) + (d & 63);
      } else {
        sp = shared ? p.ss0 : p.s0;
        bp = shared ? p.sb0 : p.b0;
        row = (size_t)e * p.R + (size_t)it.rt * kGemmM + d;
      }
      const uint16_t* srow = sp + row * ng;
      const uint16_t* brow = bp + row * ng;
      uint16_t s_next = __ldg(srow), b_next = __ldg(brow);
      for (int kc = 0; kc < nk; ++kc, ++f) {
        const uint16_t s_cur = s_next, b_cur = b_next;
        if (kc + 1 < nk) {
          s_next = __ldg(srow + kc + 1);
          b_next = __ldg(brow + kc + 1);
        }
        const int st = f % kGemmStages;
        if (!mbar_wait(&full[st], (f / kGemmStages) & 1u, kDevErrTimeoutFull)) { ok = false; break; }
        uint8_t* stage = smem + (size_t)st * S::STAGE;
        const __half2 s2 = __half2half2(__ushort_as_half(s_cur));
        const __half2 b2 = __half2half2(__ushort_as_half(b_cur));
        uint8_t* arow = stage + S::A_OFF + (d >> 3) * 1024 + (d & 7) * 128;
        const uint8_t* crow = stage + S::CODE_OFF + d * S::CROW;
        if constexpr (BITS == 8) {
          uint32_t wv[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // 64-byte rows, 64-byte swizzle: chunk q at q ^ ((d >> 1) & 3)
            const uint4 v = *reinterpret_cast<const uint4*>(crow + ((q ^ ((d >> 1) & 3)) << 4));
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int b = 0; b < 8; ++b) {  // block b: words (2b, 2b+1) = columns 8b..8b+7
            const uint32_t wa = wv[2 * b], wb = wv[2 * b + 1];
            uint4 o;
            o.x = dq_pair(lop3_and_or(wa, 0x00FF00FFu, 0x3C003C00u), s2, b2);       // (c0, c2)
            o.y = dq_pair(lop3_and_or(wb, 0x00FF00FFu, 0x3C003C00u), s2, b2);       // (c4, c6)
            o.z = dq_pair(lop3_and_or(wa >> 8, 0x00FF00FFu, 0x3C003C00u), s2, b2);  // (c1, c3)
            o.w = dq_pair(lop3_and_or(wb >> 8, 0x00FF00FFu, 0x3C003C00u), s2, b2);  // (c5, c7)
            *reinterpret_cast<uint4*>(arow + ((b ^ (d & 7)) << 4)) = o;
          }
        } else {
          uint32_t wv[8];
#pragma unroll
          for (int q = 0; q < 2; ++q) {  // 32-byte rows, 32-byte swizzle: chunk q at q ^ ((d >> 2) & 1)
            const uint4 v = *reinterpret_cast<const uint4*>(crow + ((q ^ ((d >> 2) & 1)) << 4));
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int b = 0; b < 8; ++b) {  // block b = word b: nibble pairs (s, s+4)
            const uint32_t wd = wv[b];
            uint4 o;
            o.x = dq_pair(lop3_and_or(wd, 0x000F000Fu, 0x3C003C00u), s2, b2);
            o.y = dq_pair(lop3_and_or(wd >> 4, 0x000F000Fu, 0x3C003C00u), s2, b2);
            o.z = dq_pair(lop3_and_or(wd >> 8, 0x000F000Fu, 0x3C003C00u), s2, b2);
            o.w = dq_pair(lop3_and_or(wd >> 12, 0x000F000Fu, 0x3C003C00u), s2, b2);
            *reinterpret_cast<uint4*>(arow + ((b ^ (d & 7)) << 4)) = o;
          }
        }
        fence_proxy_async();  // generic-proxy A writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[st]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int lrow = q * 32 + lane;  // accumulator row (= TMEM lane)
    uint32_t item = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++item) {
      const GemmItem it = gemm_item(p, w, n_rt);
      const int buf = item & 1;
      if (!mbar_wait(&accf[buf], (item >> 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kGemmN);
      const int ncols = (it.nrows + 15) & ~15;
      if constexpr (MODE == 1) {
        float* yrow = p.y_out + (size_t)it.row0_seg * p.R + (size_t)it.rt * kGemmM + lrow;
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < it.nrows) yrow[(size_t)(c0 + j) * p.R] = __uint_as_float(r[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
      } else {
        // rows 0-63: gate, 64-127: up (same output rows).  Up warps hand their
        // values to the gate warps through shared memory.
        if (q >= 2) {
          for (int c0 = 0; c0 < ncols; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(taddr + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) exch[(lrow - 64) * kExchPitch + c0 + j] = __uint_as_float(r[j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&exb[0]);
        if (!mbar_wait(&exb[0], item & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        if (q < 2) {
          const int orow = it.rt * (kGemmM / 2) + lrow;  // output column of h
          const size_t col = (size_t)(orow & ~7) + act_pos(orow & 7, BITS);
          for (int c0 = 0; c0 < ncols; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(taddr + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < it.nrows) {
                const float g = __uint_as_float(r[j]);
                const float u = exch[lrow * kExchPitch + c0 + j];
                const float h = g / (1.0f + expf(-g)) * u;
                p.h_out[(size_t)(it.row0_seg + c0 + j) * p.R + col] = f32_to_h16_sat(h);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acce[buf]);
          mbar_arrive(&exb[1]);
        }
        // exchange buffer free before the next item writes it
        if (!mbar_wait(&exb[1], item & 1u, kDevErrTimeoutTc)) { ok = false; break; }
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

size_t qgemm_smem_required(int bits) { return gemm_smem_bytes(bits); }

template <int BITS, int MODE>
static cudaError_t launch_qgemm_t(const GemmParams& p, int n_sm, cudaStream_t st) {
  const size_t smem = gemm_smem_bytes(BITS);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<BITS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  qgemm_kernel<BITS, MODE><<<n_sm, kGemmThreads, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qgemm(int bits, int mode, const GemmParams& p, int n_sm, cudaStream_t st) {
  if (bits == 4) return mode == 0 ? launch_qgemm_t<4, 0>(p, n_sm, st) : launch_qgemm_t<4, 1>(p, n_sm, st);
  return mode == 0 ? launch_qgemm_t<8, 0>(p, n_sm, st) : launch_qgemm_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
