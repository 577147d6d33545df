// ef_qgemm2.cu -- prefill grouped quantised GEMM on SM pairs (tcgen05 cta_group::2).
//
// The same contraction as ef_qgemm.cu (Y[tokens, out] = X . dequant(W)^T per
// expert, the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694),
// issued as 2-SM UMMA: a cluster of two CTAs on two SMs computes an M=256 x N
// tile per instruction.  Each CTA holds 128 weight rows of A (dequantised into
// its own TMEM) and half of the N activation rows of B (its own shared
// memory); each CTA's TMEM receives its 128 rows of the result.  Per SM this
// halves the activation traffic and the accumulator footprint, which leaves
// TMEM room for double-buffered accumulators (the epilogue of one item
// overlaps the next item's MMAs) and three A buffers.
//
// Work item = (segment of <= 192 rows routed to one expert) x (output rows):
//   gate/up pass: 128 output rows (h columns); CTA r holds gate rows
//     [64 r, 64 r + 64) of the item in TMEM lanes 0-63 and the same up rows in
//     lanes 64-127, so SwiGLU pairs meet through a shared-memory exchange;
//   down pass: 256 output rows; CTA r holds rows [128 r, 128 r + 128).
// Roles per CTA (15 warps): warp 0 code TMA (local ring, L2 prefetch ahead);
// warp 14 activation TMA (the CTA's half of the segment rows; transaction
// bytes counted on CTA 0's barrier); warp 1 TMEM allocation, and in CTA 0 the
// MMA issuer (tcgen05.mma.cta_group::2, commits multicast to both CTAs);
// warps 2-9 dequantise (one half row each, written with tcgen05.st);
// warps 10-13 epilogue.  CTA 1's dequant and epilogue warps arrive on CTA 0's
// barriers (mapa + mbarrier.arrive.release.cluster).  Every wait is bounded;
// no thread leaves before the final cluster barrier, so neither CTA exits
// while its peer may still touch its shared memory or TMEM.
#include "ef_common.cuh"

namespace ef {

constexpr int kG2Tile = 128;                  // weight rows per CTA (UMMA M = 256 per pair)
constexpr int kG2NMax = kGemmSegRows;         // segment rows (UMMA N, a multiple of 32)
constexpr int kG2HalfMax = kG2NMax / 2;       // activation rows per CTA
constexpr int kG2BoxRows = 16;
constexpr int kG2ABufs = 3;
constexpr int kG2DqWarps = 8;
constexpr int kG2EpiWarp0 = 2 + kG2DqWarps;   // 10
constexpr int kG2ActWarp = kG2EpiWarp0 + 4;   // 14
constexpr int kG2Threads = (kG2ActWarp + 1) * 32;
constexpr int kG2AccCols = kG2NMax;
constexpr int kG2AColBase = 2 * kG2AccCols;   // 384
constexpr int kG2ExchPitch = kG2NMax + 1;
static_assert(kG2NMax % 32 == 0 && kG2HalfMax % kG2BoxRows == 0, "segment rows");
static_assert(kG2AColBase + kG2ABufs * (kGemmKC / 2) <= kTmemCols, "TMEM budget");

template <int BITS>
struct G2Shape {
  static constexpr int CROW = kGemmKC * BITS / 8;            // 64 / 32 bytes
  static constexpr int CODE_BYTES = kG2Tile * CROW;           // 8 KB / 4 KB
  static constexpr int CODE_STAGES = BITS == 8 ? 8 : 10;
  static constexpr int ACT_BYTES = kG2HalfMax * kGemmKC * 2;  // 12 KB
  static constexpr int ACT_STAGES = 6;
  static constexpr int ACT_BASE = CODE_STAGES * CODE_BYTES;
  static constexpr int EXCH_BASE = ACT_BASE + ACT_STAGES * ACT_BYTES;
  static constexpr int BAR_BASE = EXCH_BASE + 64 * kG2ExchPitch * 4;
};

constexpr size_t g2_smem_bytes(int bits) {
  return 1024 + (size_t)(bits == 4 ? G2Shape<4>::BAR_BASE : G2Shape<8>::BAR_BASE) + 512;
}
static_assert(g2_smem_bytes(8) <= 232448 && g2_smem_bytes(4) <= 232448, "shared memory budget");

// ---------------------------------------------------------------- cluster helpers
EF_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs; the warp reconverges first (.aligned barrier).
EF_DEV void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same offset in CTA `rank` of the cluster
EF_DEV uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
// Arrive on another CTA's barrier.  The data it guards is TMEM (ordered by
// tcgen05.wait::st and the tcgen05 fences) or already counted by the barrier's
// transaction bytes, so the default (CTA-scope) semantics suffice; a
// cluster-scope release here would fence every prior memory operation.
EF_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Bounded wait on a barrier that the other CTA also arrives on (remote
// arrive, multicast commit, transaction bytes of the peer's copy).
EF_DEV bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int code) { return mbar_wait(bar, parity, code); }
// Activation tile of this CTA; the transaction bytes complete on CTA 0's barrier.
EF_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, uint32_t bar_cta0) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cta0)
      : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T over the CTA pair (M = 256)
EF_DEV void umma2_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n}\n" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0),
      "r"(0)
      : "memory");
}
// Completion of this thread's prior MMAs arrives on `bar` in both CTAs.
EF_DEV void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
EF_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

template <int BITS, int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kG2Threads, 1)
    qgemm2_kernel(const __grid_constant__ GemmParams p) {
  using S = G2Shape<BITS>;
  constexpr int CS = S::CODE_STAGES, AS = S::ACT_STAGES, NA = kG2ABufs;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* codes = smem;
  uint8_t* acts = smem + S::ACT_BASE;
  float* exch = reinterpret_cast<float*>(smem + S::EXCH_BASE);
  uint64_t* cfull = reinterpret_cast<uint64_t*>(smem + S::BAR_BASE);  // [CS] local
  uint64_t* cfree = cfull + CS;        // [CS] local (8 dequant warps)
  uint64_t* bfull = cfree + CS;        // [AS] CTA 0: both halves landed
  uint64_t* bfree = bfull + AS;        // [AS] both CTAs: MMAs done with the stage (multicast commit)
  uint64_t* aready = bfree + AS;       // [NA] CTA 0: 16 dequant warps of the pair
  uint64_t* afree = aready + NA;       // [NA] both CTAs (multicast commit)
  uint64_t* accf = afree + NA;         // [2] both CTAs (multicast commit)
  uint64_t* acce = accf + 2;           // [2] CTA 0: 8 epilogue warps of the pair
  uint64_t* exb = acce + 2;            // [2] local exchange handshake (gate/up pass)
  uint64_t* drain = exb + 2;           // CTA 0
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < CS; ++i) {
      mbar_init(&cfull[i], 1);
      mbar_init(&cfree[i], kG2DqWarps);
    }
    for (int i = 0; i < AS; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bfree[i], 1);
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(&aready[i], 2 * kG2DqWarps);
      mbar_init(&afree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 8);
      mbar_init(&exb[i], 4);
    }
    mbar_init(drain, 1);
    mbar_fence_init();
  }
  cluster_sync_all();  // barriers initialised in both CTAs before any remote arrive
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_pairs = gridDim.x >> 1, pair = blockIdx.x >> 1;
  const int out_tile = MODE == 0 ? kG2Tile : 2 * kG2Tile;  // output rows per item
  const int n_rt = (p.R + out_tile - 1) / out_tile;
  const int n_work = (*p.n_seg) * n_rt;
  const int nk = p.K / kGemmKC;
  const int ng = p.K / 64;

  if (warp == 0) {
    // ------------------------------------------------------------------ code tiles (local)
    if (lane == 0) {
      prefetch_tmap(&p.tm_c0);
      prefetch_tmap(&p.tm_c1);
      uint32_t f = 0;
      bool ok = true;
      for (int w = pair; w < n_work && ok; w += n_pairs) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const bool shared = it.expert >= p.n_experts;
        const int e = shared ? 0 : it.expert;
        const CUtensorMap* cm0 = shared ? &p.tm_sc0 : &p.tm_c0;
        const CUtensorMap* cm1 = MODE == 0 ? (shared ? &p.tm_sc1 : &p.tm_c1) : cm0;
        // gate/up: gate rows then up rows of this CTA's 64 output rows; down: 128 rows
        const int r0 = e * p.R + it.rt * out_tile + (int)crank * (MODE == 0 ? 64 : kG2Tile);
        auto prefetch_codes = [&](int kc) {
          const int kw = kc * (kGemmKC * BITS / 32);
          prefetch_tile_l2(cm0, kw, r0);
          if (MODE == 0) prefetch_tile_l2(cm1, kw, r0);
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
          if (MODE == 0) tma_load_2d(dst + S::CODE_BYTES / 2, cm1, kw, r0, &cfull[st]);
        }
      }
      for (uint32_t i = (f > (uint32_t)CS ? f - CS : 0); i < f; ++i)
        mbar_wait(&cfull[i % CS], (i / CS) & 1u, kDevErrTimeoutFull);
    }
  } else if (warp == kG2ActWarp) {
    // ------------------------------------------------------------------ activation half-tiles
    if (lane == 0) {
      prefetch_tmap(&p.tm_act);
      uint32_t f = 0;
      bool ok = true;
      for (int w = pair; w < n_work && ok; w += n_pairs) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const int N = (it.nrows + 31) & ~31;
        const int half = N / 2;
        const int nb = (half + kG2BoxRows - 1) / kG2BoxRows;
        const int row0 = it.row0_seg + (int)crank * half;
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % AS;
          if (f >= (uint32_t)AS && !mbar_wait_cluster(&bfree[st], ((f / AS) - 1) & 1u, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* dst = acts + (size_t)st * S::ACT_BYTES;
          const uint32_t bar0 = map_to_rank(&bfull[st], 0);
          if (leader) mbar_arrive_expect_tx(&bfull[st], 2u * nb * kG2BoxRows * kGemmKC * 2);
          for (int j = 0; j < nb; ++j)
            tma_load_2d_pair(dst + j * kG2BoxRows * kGemmKC * 2, &p.tm_act, kc * kGemmKC, row0 + j * kG2BoxRows, bar0);
        }
      }
      // the last stages' loads are counted on CTA 0's barriers; wait for this
      // CTA's own stages to be released by the final MMAs instead
      for (uint32_t i = (f > (uint32_t)AS ? f - AS : 0); i < f; ++i)
        mbar_wait_cluster(&bfree[i % AS], (i / AS) & 1u, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (CTA 0)
    if (leader && lane == 0) {
      uint32_t f = 0, item = 0;
      bool ok = true;
      for (int w = pair; w < n_work && ok; w += n_pairs, ++item) {
        const GemmItem it = gemm_item(p, w, n_rt);
        const int N = (it.nrows + 31) & ~31;
        const uint32_t idesc = umma_idesc_f16_f32(2 * kG2Tile, N);
        const int buf = item & 1;
        if (item >= 2 && !mbar_wait_cluster(&acce[buf], ((item >> 1) - 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(buf * kG2AccCols);
        for (int kc = 0; kc < nk; ++kc, ++f) {
          const int st = f % AS, ab = f % NA;
          if (!mbar_wait_cluster(&bfull[st], (f / AS) & 1u, kDevErrTimeoutFull)) { ok = false; break; }
          if (!mbar_wait_cluster(&aready[ab], (f / NA) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
          tc_fence_after();
          const uint64_t bd = umma_desc_sw128(smem_u32(acts + (size_t)st * S::ACT_BYTES));
          const uint32_t a0 = tmem_base + (uint32_t)(kG2AColBase + ab * (kGemmKC / 2));
#pragma unroll
          for (int k = 0; k < kGemmKC / 16; ++k)
            umma2_f16_ts(tmem_d, a0 + k * 8, bd + (uint64_t)((k * 32) >> 4), idesc, (kc > 0 || k > 0) ? 1u : 0u);
          umma2_commit_both(&bfree[st]);
          umma2_commit_both(&afree[ab]);
        }
        if (!ok) break;
        umma2_commit_both(&accf[buf]);
      }
      umma2_commit_both(drain);
      mbar_wait(drain, 0, kDevErrTimeoutTc);
    }
  } else if (warp < kG2EpiWarp0) {
    // ------------------------------------------------------------------ dequantisers
    // warp -> (TMEM lane quarter, K half): thread = one A row, 32 of the 64 columns
    const int quarter = warp & 3;
    const int khalf = (warp - 2) >> 2;
    const int lr = quarter * 32 + lane;  // row of this CTA's A tile (TMEM lane)
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(kG2AColBase + khalf * 16);
    const int nblk = (ng + 7) >> 3;
    auto item_rows = [&](int w, const uint16_t*& srow, const uint16_t*& brow) {
      const GemmItem it = gemm_item(p, w, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const int e = shared ? 0 : it.expert;
      const uint16_t* sp;
      const uint16_t* bp;
      int orow;
      if (MODE == 0) {
        const bool up = lr >= 64;
        sp = up ? (shared ? p.ss1 : p.s1) : (shared ? p.ss0 : p.s0);
        bp = up ? (shared ? p.sb1 : p.b1) : (shared ? p.sb0 : p.b0);
        orow = it.rt * out_tile + (int)crank * 64 + (lr & 63);
      } else {
        sp = shared ? p.ss0 : p.s0;
        bp = shared ? p.sb0 : p.b0;
        orow = it.rt * out_tile + (int)crank * kG2Tile + lr;
      }
      if (orow < p.R) {
        const size_t row = (size_t)e * p.R + orow;
        srow = sp + row * ng;
        brow = bp + row * ng;
      } else {
        srow = nullptr;
        brow = nullptr;
      }
    };
    int pw = pair, pblk = 0;
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
    for (int w = pair; w < n_work && ok; w += n_pairs) {
      for (int kc = 0; kc < nk; ++kc, ++f) {
        if ((kc & 7) == 0) {
          sc = sn;
          bc = bn;
          if (++pblk == nblk) {
            pblk = 0;
            pw += n_pairs;
            if (pw < n_work) item_rows(pw, psrow, pbrow);
          }
          if (pw < n_work) {
            sn = load_group_block(psrow, pblk, ng);
            bn = load_group_block(pbrow, pblk, ng);
          }
        }
        const __half2 s2 = __half2half2(__ushort_as_half(pick16(sc, kc & 7)));
        const __half2 b2 = __half2half2(__ushort_as_half(pick16(bc, kc & 7)));
        const int st = f % CS, ab = f % NA;
        if (!mbar_wait(&cfull[st], (f / CS) & 1u, kDevErrTimeoutFull)) { ok = false; break; }
        const uint8_t* crow = codes + (size_t)st * S::CODE_BYTES + lr * S::CROW;
        uint32_t a[16];  // fp16 pairs of K positions 32 khalf + (2c, 2c+1), c = 0..15
        if constexpr (BITS == 8) {
          uint32_t wv[8];
#pragma unroll
          for (int q = 0; q < 2; ++q) {  // 64-byte rows, 64-byte swizzle: chunk q at q ^ ((lr >> 1) & 3)
            const int qq = 2 * khalf + q;
            const uint4 v = *reinterpret_cast<const uint4*>(crow + ((qq ^ ((lr >> 1) & 3)) << 4));
            wv[4 * q] = v.x; wv[4 * q + 1] = v.y; wv[4 * q + 2] = v.z; wv[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint32_t wa = wv[2 * b], wb = wv[2 * b + 1];
            a[4 * b + 0] = dq_pair(code_pair8(wa, 0x4240u), s2, b2);
            a[4 * b + 1] = dq_pair(code_pair8(wb, 0x4240u), s2, b2);
            a[4 * b + 2] = dq_pair(code_pair8(wa, 0x4341u), s2, b2);
            a[4 * b + 3] = dq_pair(code_pair8(wb, 0x4341u), s2, b2);
          }
        } else {
          // 32-byte rows, 32-byte swizzle: chunk q at q ^ ((lr >> 2) & 1); this half = chunk khalf
          const uint4 v = *reinterpret_cast<const uint4*>(crow + ((khalf ^ ((lr >> 2) & 1)) << 4));
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint32_t wd = wv[b];
            a[4 * b + 0] = dq_pair(lop3_and_or(wd, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 1] = dq_pair(lop3_and_or(wd >> 4, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 2] = dq_pair(lop3_and_or(wd >> 8, 0x000F000Fu, 0x64006400u), s2, b2);
            a[4 * b + 3] = dq_pair(lop3_and_or(wd >> 12, 0x000F000Fu, 0x64006400u), s2, b2);
          }
        }
        if (f >= (uint32_t)NA && !mbar_wait_cluster(&afree[ab], ((f / NA) - 1) & 1u, kDevErrTimeoutTc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st16(t_lane + (uint32_t)(ab * (kGemmKC / 2)), a);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cfree[st]);  // the code words were consumed by the completed tcgen05.st
          if (leader) mbar_arrive(&aready[ab]);
          else mbar_arrive_remote(map_to_rank(&aready[ab], 0));
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 10-13)
    const int quarter = warp & 3;
    const int lr = quarter * 32 + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)(quarter * 32) << 16);
    uint32_t item = 0;
    bool ok = true;
    for (int w = pair; w < n_work && ok; w += n_pairs, ++item) {
      const GemmItem it = gemm_item(p, w, n_rt);
      const int buf = item & 1;
      if (!mbar_wait_cluster(&accf[buf], (item >> 1) & 1u, kDevErrTimeoutTc)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tacc = t_lane + (uint32_t)(buf * kG2AccCols);
      if constexpr (MODE == 1) {
        const int orow = it.rt * out_tile + (int)crank * kG2Tile + lr;
        float* yrow = p.y_out + (size_t)it.row0_seg * p.R + orow;
        for (int c0 = 0; c0 < it.nrows; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tacc + c0, r);
          tmem_wait_ld();
          const int nc = min(32, it.nrows - c0);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < nc && orow < p.R) yrow[(size_t)(c0 + j) * p.R] = __uint_as_float(r[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&acce[buf]);
          else mbar_arrive_remote(map_to_rank(&acce[buf], 0));
        }
      } else {
        // lanes 64-127 hold up rows: copy them to the exchange buffer
        if (quarter >= 2) {
          for (int c0 = 0; c0 < it.nrows; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tacc + c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) exch[(lr - 64) * kG2ExchPitch + c0 + j] = __uint_as_float(r[j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&exb[0]);
        if (!mbar_wait(&exb[0], item & 1u, kDevErrTimeoutTc)) { ok = false; break; }
        uint32_t g[32];
        if (quarter < 2) {
          const int orow = it.rt * out_tile + (int)crank * 64 + lr;  // h column
          const bool valid = orow < p.R;
          const size_t col = (size_t)(orow & ~7) + act_pos(orow & 7, BITS);
          uint16_t* hrow = p.h_out + (size_t)it.row0_seg * p.R + col;
          for (int c0 = 0; c0 < it.nrows; c0 += 32) {
            tmem_ld32(tacc + c0, g);
            tmem_wait_ld();
            const int nc = valid ? min(32, it.nrows - c0) : 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < nc) {
                const float gv = __uint_as_float(g[j]);
                const float h = gv / (1.0f + expf(-gv)) * exch[lr * kG2ExchPitch + c0 + j];
                hrow[(size_t)(c0 + j) * p.R] = f32_to_h16_sat(h);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&acce[buf]);
          else mbar_arrive_remote(map_to_rank(&acce[buf], 0));
          mbar_arrive(&exb[1]);
        }
        if (!mbar_wait(&exb[1], item & 1u, kDevErrTimeoutTc)) { ok = false; break; }  // exchange free again
      }
    }
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  cluster_sync_all();  // both CTAs done: no remote arrive, MMA or copy can touch either CTA any more
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
  cluster_sync_all();
}

size_t qgemm2_smem_required(int bits) { return g2_smem_bytes(bits); }

template <int BITS, int MODE>
static cudaError_t launch_qgemm2_t(const GemmParams& p, int n_sm, cudaStream_t st) {
  const size_t smem = g2_smem_bytes(BITS);
  static std::atomic<bool> attr_set[64];
  if (const cudaError_t e = set_max_smem_once(qgemm2_kernel<BITS, MODE>, (int)smem, attr_set)) return e;
  qgemm2_kernel<BITS, MODE><<<(n_sm / 2) * 2, kG2Threads, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qgemm2(int bits, int mode, const GemmParams& p, int n_sm, cudaStream_t st) {
  if (bits == 4) return mode == 0 ? launch_qgemm2_t<4, 0>(p, n_sm, st) : launch_qgemm2_t<4, 1>(p, n_sm, st);
  return mode == 0 ? launch_qgemm2_t<8, 0>(p, n_sm, st) : launch_qgemm2_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
