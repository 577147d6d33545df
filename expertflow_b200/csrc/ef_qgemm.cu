// ef_qgemm.cu -- prefill-size grouped quantised GEMM on tcgen05 / TMEM (sm_100a).
//
// Replaces the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694
// when an expert receives many tokens (prefill): the expert matmuls become a
// dense grouped contraction  Y[tokens, out] = X[tokens, K] . dequant(W)[out, K]^T
// per expert, run on the 5th-generation tensor cores with fp32 accumulation in
// tensor memory.
//
// Work item = (segment of <= 192 rows routed to one expert) x (256 weight rows,
// issued as two M=128 UMMA tiles that share the activation tile).  In the
// gate/up pass tile 0 holds 128 gate rows and tile 1 the same 128 up rows, so a
// SwiGLU pair lands in the same TMEM lane of the two accumulators.  The
// dequantised weights never touch shared memory: they are written to TMEM and
// consumed there as the UMMA A operand (tcgen05.mma ... [d], [a_tmem], b_desc).
// One persistent CTA per SM, 19 warps:
//   warp 0      TMA: code tiles (2 x 128 rows x one 64-column group, swizzled)
//               into a code ring; prefetches code tiles 8 chunks ahead into L2
//   warp 18     TMA: activation rows of the segment (32-row boxes, 128-B
//               swizzle = the UMMA K-major canonical layout) into an act ring
//   warp 1      TMEM allocation (512 columns); lane 0 issues tcgen05.mma
//               (M=128, N = segment rows rounded to 16, K=16) and commits
//   warps 2-9   dequantise one weight row each: codes -> fp16 1024 + q under
//               the exponent of 1024 (8-bit: one byte permute per pair; 4-bit:
//               LOP3 + shift) -> exact q (one fp16 subtraction) -> fp16 s*q + b
//               (one fp16 FMA, single rounding) -> tcgen05.st into the A tile
//   warps 10-17 epilogue (two per TMEM lane quarter, alternate 32-column
//               blocks): tcgen05.ld of both accumulators; gate/up pass:
//               h = silu(g) * u -> fp16 rows; down pass: fp32 rows
// TMEM columns: accumulator 0 [0, 192), accumulator 1 [192, 384), A tiles
// [384, 512) = 2 buffers x 2 tiles x 32 columns (64 fp16 per lane).
// The activation columns carry the same within-block permutation as the GEMV
// path (act_pos), and the dequantised A rows are written in that order, so the
// contraction over K is unchanged.  Every wait is bounded; TMEM is released on
// every exit path.
#include "ef_common.cuh"

namespace ef {

// Pipeline depths (compile-time; the TMEM and shared-memory budgets are checked below)
#ifndef EF_GEMM_ABUFS
#define EF_GEMM_ABUFS 2
#endif
#ifndef EF_GEMM_EPI_WARPS
#define EF_GEMM_EPI_WARPS 8
#endif
#ifndef EF_GEMM_CSTAGES8
#define EF_GEMM_CSTAGES8 6
#endif
#ifndef EF_GEMM_ASTAGES8
#define EF_GEMM_ASTAGES8 4
#endif
#ifndef EF_GEMM_CSTAGES4
#define EF_GEMM_CSTAGES4 8
#endif
#ifndef EF_GEMM_ASTAGES4
#define EF_GEMM_ASTAGES4 5
#endif
constexpr int kGemmTileM = 128;             // rows per UMMA tile
constexpr int kGemmItemRows = 256;          // weight rows per work item (two tiles)
constexpr int kGemmNMax = kGemmSegRows;     // routed rows per segment (UMMA N)
constexpr int kGemmKC = 64;                 // K columns per chunk (one quantisation group)
constexpr int kActBoxRows = 32;             // activation TMA box height
constexpr int kGemmABufs = EF_GEMM_ABUFS;   // A tile pairs in TMEM
constexpr int kGemmPrefetch = 8;            // code tiles prefetched into L2 ahead of the ring
constexpr int kGemmDqWarps = 8;
constexpr int kGemmEpiWarps = EF_GEMM_EPI_WARPS;  // 4 or 8 (one or two per TMEM lane quarter)
constexpr int kGemmEpiWarp0 = 2 + kGemmDqWarps;
constexpr int kGemmActWarp = kGemmEpiWarp0 + kGemmEpiWarps;
constexpr int kGemmThreads = (kGemmActWarp + 1) * 32;
constexpr int kTmemCols = 512;
constexpr int kAccCols = kGemmNMax;         // columns per accumulator
constexpr int kAColBase = 2 * kAccCols;     // first A-tile column
static_assert(kGemmNMax % 32 == 0 && kGemmNMax <= 256, "segment rows: whole activation boxes, UMMA N <= 256");
static_assert(kAColBase + kGemmABufs * 2 * (kGemmKC / 2) <= kTmemCols, "TMEM budget");
static_assert(kGemmEpiWarps == 4 || kGemmEpiWarps == 8, "epilogue warps");

template <int BITS>
struct GemmShape {
  static constexpr int CROW = kGemmKC * BITS / 8;               // code bytes per row per chunk (64 / 32)
  static constexpr int CODE_BYTES = kGemmItemRows * CROW;        // 16 KB / 8 KB
  static constexpr int CODE_STAGES = BITS == 8 ? EF_GEMM_CSTAGES8 : EF_GEMM_CSTAGES4;
  static constexpr int ACT_BYTES = kGemmNMax * kGemmKC * 2;      // fp16 rows x 128 B
  static constexpr int ACT_STAGES = BITS == 8 ? EF_GEMM_ASTAGES8 : EF_GEMM_ASTAGES4;
  static constexpr int ACT_BASE = CODE_STAGES * CODE_BYTES;      // 1024-aligned
  static constexpr int BAR_BASE = ACT_BASE + ACT_STAGES * ACT_BYTES;
};

constexpr size_t gemm_smem_bytes(int bits) {
  return 1024 + (size_t)(bits == 4 ? GemmShape<4>::BAR_BASE : GemmShape<8>::BAR_BASE) + 512;
}
static_assert(gemm_smem_bytes(8) <= 232448 && gemm_smem_bytes(4) <= 232448, "shared memory budget");

struct GemmParams {
  CUtensorMap tm_c0, tm_c1;    // routed codes (gate/up or down), 2-D [E*R, K*bits/32], box 128 rows
  CUtensorMap tm_sc0, tm_sc1;  // shared-expert codes
  CUtensorMap tm_act;          // activation rows [n_rows, K] fp16, box 64 x 32, 128-B swizzle
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
// D[tmem] (+)= A[tmem] . B[smem]^T ; A is M x 16 fp16 (lane = row, 2 per column)
EF_DEV void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
EF_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
EF_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
EF_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
EF_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
EF_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
EF_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
EF_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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
  if (it.nrows > kGemmNMax) {  // segments are cut to kGemmNMax rows by the permute step
    ef_set_error(kDevErrRange);
    it.nrows = kGemmNMax;
  }
  return it;
}

// 16-bit element j (0..7) of a 16-byte register block, without local memory
EF_DEV uint16_t pick16(const uint4& v, int j) {
  const uint32_t w = (j & 4) ? ((j & 2) ? v.w : v.z) : ((j & 2) ? v.y : v.x);
  return (uint16_t)(w >> ((j & 1) * 16));
}
// Scales (or biases) of 8 consecutive groups blk*8 .. blk*8+7 of one weight row;
// groups past the row end read as 0.  16-byte aligned rows whose length is a
// multiple of 8 groups use one vector load.
EF_DEV uint4 load_group_block(const uint16_t* row, int blk, int ng) {
  if (row == nullptr) return make_uint4(0, 0, 0, 0);
  if ((ng & 7) == 0 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0)
    return __ldg(reinterpret_cast<const uint4*>(row) + blk);
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int g = blk * 8 + 2 * j;
    const uint32_t lo = g < ng ? __ldg(row + g) : 0u;
    const uint32_t hi = g + 1 < ng ? __ldg(row + g + 1) : 0u;
    w[j] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// fp16 pair (1 + qa/1024, 1 + qb/1024) -> (s qa + b, s qb + b), exact q then one rounding
// fp16 pair (1024 + q0, 1024 + q1) -> the weights (s q0 + b, s q1 + b): the
// subtraction is exact, the FMA rounds once.
EF_DEV uint32_t dq_pair(uint32_t v, __half2 s2, __half2 b2) {
  const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&v), __float2half2_rn(1024.0f));
  const __half2 w = __hfma2(q, s2, b2);
  return *reinterpret_cast<const uint32_t*>(&w);
}
// Bytes of v picked by `sel` (0x4240: 0, 2; 0x4341: 1, 3) under the high byte
// 0x64: the fp16 pair (1024 + b, 1024 + b').
EF_DEV uint32_t code_pair8(uint32_t v, uint32_t sel) { return prmt(v, 0x64646464u, sel); }

template <int BITS, int MODE>
__global__ void __launch_bounds__(kGemmThreads, 1) qgemm_kernel(const __grid_constant__ GemmParams p) {
  using S = GemmShape<BITS>;
  constexpr int CS = S::CODE_STAGES, AS = S::ACT_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* codes = smem;                       // [CS][256 rows][CROW], swizzled
  uint8_t* acts = smem + S::ACT_BASE;          // [AS][kGemmNMax rows][128 B], 128-B swizzle
  uint64_t* cfull = reinterpret_cast<uint64_t*>(smem + S::BAR_BASE);  // [CS] code tile landed
  uint64_t* cfree = cfull + CS;                // [CS] code tile consumed (8 dequant warps)
  uint64_t* bfull = cfree + CS;                // [AS] activation tile landed
  uint64_t* bfree = bfull + AS;                // [AS] MMAs reading it done (commit)
  uint64_t* aready = bfree + AS;               // [ABUFS] A tiles written to TMEM (8 dequant warps)
  uint64_t* afree = aready + kGemmABufs;       // [ABUFS] MMAs reading them done (commit)
  uint64_t* accf = afree + kGemmABufs;         // accumulators complete (commit)
  uint64_t* acce = accf + 1;                   // accumulators drained (epilogue warps)
  uint64_t* drain = acce + 1;                  // final MMA drain
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < CS; ++i) {
      mbar_init(&cfull[i], 1);
      mbar_init(&cfree[i], kGemmDqWarps);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bfree[i], 1);
    }
    for (int i = 0; i < kGemmABufs; ++i) {
      mbar_init(&aready[i], kGemmDqWarps);
      mbar_init(&afree[i], 1);
    }
    mbar_init(accf, 1);
    mbar_init(acce, kGemmEpiWarps);
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
  pdl_wait();  // the segments and activations of the previous kernels
  // (no early launch of the successor: its CTAs would wait on SMs this
  // persistent grid fills)

  const int n_rt = MODE == 0 ? (p.R + kGemmTileM - 1) / kGemmTileM : (p.R + kGemmItemRows - 1) / kGemmItemRows;
  const int n_work = (*p.n_seg) * n_rt;
  const int nk = p.K / kGemmKC;
  const int ng = p.K / 64;

  if (warp == 0) {
    // ------------------------------------------------------------------ code tiles
    if (lane == 0) {
      prefetch_tmap(&p.tm_c0);
      prefetch_tmap(&p.tm_c1);
      uint32_t f = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const bool shared = it.expert >= p.n_experts;
        const int e = shared ? 0 : it.expert;
        const CUtensorMap* cm0 = shared ? &p.tm_sc0 : &p.tm_c0;
        const CUtensorMap* cm1 = MODE == 0 ? (shared ? &p.tm_sc1 : &p.tm_c1) : cm0;
        const int r0 = e * p.R + it.rt * (MODE == 0 ? kGemmTileM : kGemmItemRows);
        const int r1 = MODE == 0 ? r0 : r0 + kGemmTileM;
        auto prefetch_codes = [&](int kc) {
          const int kw = kc * (kGemmKC * BITS / 32);
          prefetch_tile_l2(cm0, kw, r0);
          prefetch_tile_l2(cm1, kw, r1);
        };
        for (int kc = 0; kc < kGemmPrefetch && kc < nk; ++kc) prefetch_codes(kc);
        for (int kc = 0; kc < nk; ++kc, ++f) {
          if (kc + kGemmPrefetch < nk) prefetch_codes(kc + kGemmPrefetch);
          const int st = f % CS;
          if (f >= (uint32_t)CS && !mbar_wait(&cfree[st], ((f / CS) - 1) & 1u, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* dst = codes + (size_t)st * S::CODE_BYTES;
          const int kw = kc * (kGemmKC * BITS / 32);
          mbar_arrive_expect_tx(&cfull[st], S::CODE_BYTES);
          tma_load_2d(dst, cm0, kw, r0, &cfull[st]);
          tma_load_2d(dst + S::CODE_BYTES / 2, cm1, kw, r1, &cfull[st]);
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (uint32_t i = (f > (uint32_t)CS ? f - CS : 0); i < f; ++i)
        mbar_wait(&cfull[i % CS], (i / CS) & 1u, kDevErrTimeoutFull);
    }
  } else if (warp == kGemmActWarp) {
    // ------------------------------------------------------------------ activation tiles
    if (lane == 0) {
      prefetch_tmap(&p.tm_act);
      uint32_t f = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const int nb = (it.nrows + kActBoxRows - 1) / kActBoxRows;
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % AS;
          if (f >= (uint32_t)AS && !mbar_wait(&bfree[st], ((f / AS) - 1) & 1u, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* dst = acts + (size_t)st * S::ACT_BYTES;
          mbar_arrive_expect_tx(&bfull[st], (uint32_t)nb * kActBoxRows * kGemmKC * 2);
          for (int j = 0; j < nb; ++j)
            tma_load_2d(dst + j * kActBoxRows * kGemmKC * 2, &p.tm_act, kc * kGemmKC, it.row0_seg + j * kActBoxRows,
                        &bfull[st]);
        }
      }
      for (uint32_t i = (f > (uint32_t)AS ? f - AS : 0); i < f; ++i)
        mbar_wait(&bfull[i % AS], (i / AS) & 1u, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t f = 0, item = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++item) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const int N = (it.nrows + 15) & ~15;
        const uint32_t idesc = umma_idesc_f16_f32(kGemmTileM, N);
        // the epilogue must have drained the previous item's accumulators
        if (item >= 1 && !mbar_wait(acce, (item - 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        tc_fence_after();
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % AS, ab = f % kGemmABufs;
          if (!mbar_wait(&bfull[st], (f / AS) & 1u, kDevErrTimeoutFull)) { ok = false; break; }
          if (!mbar_wait(&aready[ab], (f / kGemmABufs) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bd = umma_desc_sw128(smem_u32(acts + (size_t)st * S::ACT_BYTES));
          const uint32_t a0 = tmem_base + (uint32_t)(kAColBase + ab * kGemmKC);
#pragma unroll
          for (int k = 0; k < kGemmKC / 16; ++k) {  // K=16 per step: 8 TMEM columns, 32 B of the swizzle atom
            const uint32_t acc = (kc > 0 || k > 0) ? 1u : 0u;
            umma_f16_ts(tmem_base, a0 + k * 8, bd + (uint64_t)((k * 32) >> 4), idesc, acc);
            umma_f16_ts(tmem_base + kAccCols, a0 + kGemmKC / 2 + k * 8, bd + (uint64_t)((k * 32) >> 4), idesc, acc);
          }
          umma_commit(&bfree[st]);  // frees the activation tile once read
          umma_commit(&afree[ab]);  // frees the A tiles once read
        }
        if (!ok) break;
        umma_commit(accf);  // accumulators complete
      }
      // drain any MMAs still in flight before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, kDevErrTimeoutTc);
    }
  } else if (warp < 2 + kGemmDqWarps) {
    // ------------------------------------------------------------------ dequantisers
    // Warp w writes TMEM lane quarter w % 4 of tile (w - 2) / 4: one A row per thread.
    // Scales/biases arrive 8 groups at a time, one block ahead of use (the next
    // block may belong to the next work item), so global-load latency stays off
    // the per-chunk path.
    const int tile = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int lr = quarter * 32 + lane;          // row within the tile = TMEM lane
    const int d = tile * kGemmTileM + lr;        // row within the item's code tile
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(kAColBase + tile * (kGemmKC / 2));
    const int nblk = (ng + 7) >> 3;
    auto item_rows = [&](int w, const uint16_t*& srow, const uint16_t*& brow) {
      const GemmItem it = gemm_item(p, w, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const int e = shared ? 0 : it.expert;
      const uint16_t* sp;
      const uint16_t* bp;
      int orow;
      if (MODE == 0) {
        sp = tile ? (shared ? p.ss1 : p.s1) : (shared ? p.ss0 : p.s0);
        bp = tile ? (shared ? p.sb1 : p.b1) : (shared ? p.sb0 : p.b0);
        orow = it.rt * kGemmTileM + lr;
      } else {
        sp = shared ? p.ss0 : p.s0;
        bp = shared ? p.sb0 : p.b0;
        orow = it.rt * kGemmItemRows + d;
      }
      if (orow < p.R) {
        const size_t row = (size_t)e * p.R + orow;
        srow = sp + row * ng;
        brow = bp + row * ng;
      } else {  // rows past the projection end: zero weights, never stored
        srow = nullptr;
        brow = nullptr;
      }
    };
    int pw = blockIdx.x, pblk = 0;  // prefetch cursor: block held in (sn, bn)
    const uint16_t* psrow = nullptr;
    const uint16_t* pbrow = nullptr;
    uint4 sn = make_uint4(0, 0, 0, 0), bn = sn, sc = sn, bc = sn;
    if (pw < n_work) {
      item_rows(pw, psrow, pbrow);
      sn = load_group_block(psrow, 0, ng);
      bn = load_group_block(pbrow, 0, ng);
    }
    uint32_t f = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
      for (int kc = 0; kc < nk; ++kc, ++f) {
        if ((kc & 7) == 0) {  // take the prefetched block, fetch the one after it
          sc = sn;
          bc = bn;
          if (++pblk == nblk) {
            pblk = 0;
            pw += gridDim.x;
            if (pw < n_work) item_rows(pw, psrow, pbrow);
          }
          if (pw < n_work) {
            sn = load_group_block(psrow, pblk, ng);
            bn = load_group_block(pbrow, pblk, ng);
          }
        }
        const __half2 s2 = __half2half2(__ushort_as_half(pick16(sc, kc & 7)));
        const __half2 b2 = __half2half2(__ushort_as_half(pick16(bc, kc & 7)));
        const int st = f % CS, ab = f % kGemmABufs;
        if (!mbar_wait(&cfull[st], (f / CS) & 1u, kDevErrTimeoutFull)) { ok = false; break; }
        const uint8_t* crow = codes + (size_t)st * S::CODE_BYTES + d * S::CROW;
        uint32_t wv[BITS * 2];  // this row's codes for the chunk (16 / 8 words)
        if constexpr (BITS == 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // 64-byte rows, 64-byte swizzle: chunk q at q ^ ((d >> 1) & 3)
            const uint4 v = *reinterpret_cast<const uint4*>(crow + ((q ^ ((d >> 1) & 3)) << 4));
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 2; ++q) {  // 32-byte rows, 32-byte swizzle: chunk q at q ^ ((d >> 2) & 1)
            const uint4 v = *reinterpret_cast<const uint4*>(crow + ((q ^ ((d >> 2) & 1)) << 4));
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
        }
        uint32_t a[32];  // fp16 pairs of K positions (2c, 2c+1), c = 0..31
        if constexpr (BITS == 8) {
#pragma unroll
          for (int b = 0; b < 8; ++b) {  // block b: words (2b, 2b+1) = columns 8b..8b+7
            const uint32_t wa = wv[2 * b], wb = wv[2 * b + 1];
            a[4 * b + 0] = dq_pair(code_pair8(wa, 0x4240u), s2, b2);  // (c0, c2)
            a[4 * b + 1] = dq_pair(code_pair8(wb, 0x4240u), s2, b2);  // (c4, c6)
            a[4 * b + 2] = dq_pair(code_pair8(wa, 0x4341u), s2, b2);  // (c1, c3)
            a[4 * b + 3] = dq_pair(code_pair8(wb, 0x4341u), s2, b2);  // (c5, c7)
          }
        } else {
#pragma unroll
          for (int b = 0; b < 8; ++b) {  // block b = word b: nibble pairs (s, s+4)
            const uint32_t wd = wv[b];
            a[4 * b + 0] = dq_pair(lop3_and_or(wd, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 1] = dq_pair(lop3_and_or(wd >> 4, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 2] = dq_pair(lop3_and_or(wd >> 8, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 3] = dq_pair(lop3_and_or(wd >> 12, 0x000F000Fu, 0x64006400u), s2, b2);
          }
        }
        if (f >= (uint32_t)kGemmABufs &&
            !mbar_wait(&afree[ab], ((f / kGemmABufs) - 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(t_lane + (uint32_t)(ab * kGemmKC), a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        // The code tile is released only here: an mbarrier arrive does not wait
        // for the thread's outstanding shared-memory loads, whereas the completed
        // tcgen05.st has consumed every lane's loaded words.
        if (lane == 0) {
          mbar_arrive(&cfree[st]);
          mbar_arrive(&aready[ab]);
        }
      }
    }
  } else if (warp < kGemmActWarp) {
    // ------------------------------------------------------------------ epilogue
    // Warp (quarter, half): TMEM lane quarter warp % 4; with 8 epilogue warps the
    // two warps of a quarter take alternate 32-column blocks.
    const int quarter = warp & 3;
    const int half = kGemmEpiWarps == 8 ? (warp - kGemmEpiWarp0) >> 2 : 0;
    constexpr int kColStep = 32 * (kGemmEpiWarps / 4);
    const int lr = quarter * 32 + lane;    // accumulator row (= TMEM lane)
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16);
    uint32_t item = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++item) {
      const GemmItem it = gemm_item(p, w, n_rt);
      if (!mbar_wait(accf, item & 1u, kDevErrTimeoutTc)) { ok = false; break; }
      tc_fence_after();
      if constexpr (MODE == 1) {
        const int o0 = it.rt * kGemmItemRows + lr, o1 = o0 + kGemmTileM;
        float* yrow = p.y_out + (size_t)it.row0_seg * p.R;
        for (int c0 = half * 32; c0 < it.nrows; c0 += kColStep) {
          uint32_t r0[32], r1[32];
          tmem_ld32(t_lane + c0, r0);
          tmem_ld32(t_lane + kAccCols + c0, r1);
          tmem_wait_ld();
          const int nc = min(32, it.nrows - c0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < nc) {
              if (o0 < p.R) yrow[(size_t)(c0 + j) * p.R + o0] = __uint_as_float(r0[j]);
              if (o1 < p.R) yrow[(size_t)(c0 + j) * p.R + o1] = __uint_as_float(r1[j]);
            }
          }
        }
      } else {
        // accumulator 0: gate row orow, accumulator 1: up row orow (same lane)
        const int orow = it.rt * kGemmTileM + lr;
        const bool valid = orow < p.R;
        const size_t col = (size_t)(orow & ~7) + act_pos(orow & 7, BITS);
        uint16_t* hrow = p.h_out + (size_t)it.row0_seg * p.R + col;
        for (int c0 = half * 32; c0 < it.nrows; c0 += kColStep) {
          uint32_t g[32], u[32];
          tmem_ld32(t_lane + c0, g);
          tmem_ld32(t_lane + kAccCols + c0, u);
          tmem_wait_ld();
          const int nc = valid ? min(32, it.nrows - c0) : 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < nc) {
              const float gv = __uint_as_float(g[j]);
              const float h = gv / (1.0f + expf(-gv)) * __uint_as_float(u[j]);
              hrow[(size_t)(c0 + j) * p.R] = f32_to_h16_sat(h);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce);
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
  static std::atomic<bool> attr_set[64];
  if (const cudaError_t e = set_max_smem_once(qgemm_kernel<BITS, MODE>, (int)smem, attr_set)) return e;
  return launch_pdl(qgemm_kernel<BITS, MODE>, n_sm, kGemmThreads, smem, st, p);
}

cudaError_t launch_qgemm(int bits, int mode, const GemmParams& p, int n_sm, cudaStream_t st) {
  if (bits == 4) return mode == 0 ? launch_qgemm_t<4, 0>(p, n_sm, st) : launch_qgemm_t<4, 1>(p, n_sm, st);
  return mode == 0 ? launch_qgemm_t<8, 0>(p, n_sm, st) : launch_qgemm_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
