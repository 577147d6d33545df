// ef_qmv.cu -- decode-size grouped quantised GEMV (sm_100a).
//
// Replaces the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694
// (gate, up, silu*up, down) for small token counts, where the layer is bound by
// HBM bandwidth on the packed weights.
//
// Work item = (segment of <= 32 rows routed to one expert) x (64 weight rows).
// A CTA is 4 compute warps + 1 producer warp and loops over work items
// (persistent).  The producer streams, per 256-column (4-bit) / 128-column
// (8-bit) stage, the 64-row code tile(s) with a 2-D TMA load (128-byte
// swizzle) and the segment's activation rows with 1-D bulk copies into a
// 4-deep mbarrier ring; per work item it also bulk-loads the tile's fp16
// scales/biases and the rows' group sums.
//
// Dot products run on the tensor cores with exact operands: a code q is
// unpacked into the fp16 value 1 + q/16 (4-bit: nibble moved to mantissa bits
// 6..9 with one shift and one LOP3 per pair) or 1 + q/1024 (8-bit: byte into
// bits 0..7 with PRMT + LOP3), activations are fp16, products accumulate in
// fp32 per 64-column group:
//     D_g = sum_i x_i (1 + q_i / Q)
//     y  += (Q s_g) D_g + (b_g - Q s_g) sum_i x_i        (= sum_i x_i (s_g q_i + b_g))
// The k order inside mma.m16n8k16 is permuted consistently for codes and
// activations (activations are stored in "pair order"), which leaves every
// dot product unchanged.
//
// mode 0: gate and up tiles together, epilogue h = silu(g) * u stored as fp16
//         pair-ordered rows + group sums (input of mode 1).
// mode 1: down projection, fp32 rows for the combine.
#include "ef_common.cuh"

namespace ef {

template <int BITS, int MODE>
struct QmvShape {
  static constexpr int KT = BITS == 4 ? 256 : 128;   // columns per stage
  static constexpr int GPS = KT / 64;                 // groups per stage
  static constexpr int ROWB = KT * BITS / 8;          // bytes per code row per stage (128)
  static constexpr int NMAT = MODE == 0 ? 2 : 1;
  static constexpr int CODE_BYTES = NMAT * kRowTile * ROWB;
  static constexpr int ACT_PITCH = KT * 2 + kActPad;
  static constexpr int ACT_BYTES = kTokChunk * ACT_PITCH;
  static constexpr int STAGE_BYTES = ((CODE_BYTES + ACT_BYTES) + 1023) / 1024 * 1024;
  static constexpr float Q = BITS == 4 ? 16.0f : 1024.0f;
};

template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_smem_bytes(int K) {
  using S = QmvShape<BITS, MODE>;
  const int ng = K / 64;
  size_t b = 1024;  // alignment slack
  b += (size_t)kStages * S::STAGE_BYTES;
  b += (size_t)S::NMAT * 2 * kRowTile * ng * 2;  // scales + biases
  b += (size_t)kTokChunk * sum_ld(K) * 4;       // activation group sums
  b += (size_t)kTokChunk * kRowTile * 2;         // h staging (mode 0)
  b += 128;                                      // barriers
  return b;
}

EF_DEV uint32_t pair4(uint32_t w, int s) {
  // nibbles s and s+4 -> fp16 pair (1 + q_s/16, 1 + q_{s+4}/16)
  uint32_t v = (s == 0) ? (w << 6) : (s == 1) ? (w << 2) : (s == 2) ? (w >> 2) : (w >> 6);
  return lop3_and_or(v, 0x03C003C0u, 0x3C003C00u);
}
EF_DEV uint32_t pair8(uint32_t a, uint32_t b, int s) {
  // byte s of a and byte s of b -> fp16 pair (1 + qa/1024, 1 + qb/1024)
  return lop3_and_or(prmt(a, b, (uint32_t)(s | ((4 + s) << 8))), 0x00FF00FFu, 0x3C003C00u);
}

struct WorkItem {
  int expert, row0_seg, nrows, rt;
};

EF_DEV WorkItem decode_work(const QmvParams& p, int w, int n_rt) {
  WorkItem it;
  int seg = w / n_rt;
  it.rt = w - seg * n_rt;
  it.expert = p.seg_expert[seg];
  it.row0_seg = p.seg_row0[seg];
  it.nrows = p.seg_nrows[seg];
  return it;
}

template <int BITS, int MODE, int NT>
EF_DEV bool qmv_consume(const QmvParams& p, const WorkItem& it, uint8_t* stage_base, const uint16_t* s_sb,
                        const float* s_xs, uint16_t* s_h, uint64_t* full, uint64_t* empty, uint64_t* sb_empty,
                        uint64_t* epi, uint32_t item, uint32_t& fill_it) {
  using S = QmvShape<BITS, MODE>;
  const int lane = threadIdx.x & 31, cw = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ng = p.K / 64;
  const int xs_ld = sum_ld(p.K);
  const int nstages = (p.K + S::KT - 1) / S::KT;
  const int rA = cw * 16 + g, rB = rA + 8;
  float y[S::NMAT][NT][4];
#pragma unroll
  for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) y[m][n][i] = 0.0f;

  for (int st = 0; st < nstages; ++st, ++fill_it) {
    const int slot = fill_it % kStages;
    const uint32_t parity = (fill_it / kStages) & 1u;
    if (!mbar_wait(&full[slot], parity, kDevErrTimeoutFull)) return false;
    const uint8_t* codes = stage_base + (size_t)slot * S::STAGE_BYTES;
    const uint8_t* act = codes + S::CODE_BYTES;
    const int gvalid = min(S::GPS, ng - st * S::GPS);  // last stage may be partial
#pragma unroll
    for (int G = 0; G < S::GPS; ++G) {
      if (G >= gvalid) break;
      const int Gabs = st * S::GPS + G;
      // ---- B operands (activation rows nt*8 + g)
      uint4 blk0[NT], blk1[NT];
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint8_t* ar = act + (size_t)(n * 8 + g) * S::ACT_PITCH + (size_t)(8 * G + 2 * t) * 16;
        blk0[n] = *reinterpret_cast<const uint4*>(ar);
        blk1[n] = *reinterpret_cast<const uint4*>(ar + 16);
      }
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m) {
        const uint8_t* cm = codes + (size_t)m * kRowTile * S::ROWB;
        float D[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) D[n][i] = 0.0f;
        if constexpr (BITS == 4) {
          const int chunk = 2 * G + (t >> 1);
          const uint2 wa = *reinterpret_cast<const uint2*>(cm + rA * 128 + ((chunk ^ (rA & 7)) << 4) + 8 * (t & 1));
          const uint2 wb = *reinterpret_cast<const uint2*>(cm + rB * 128 + ((chunk ^ (rB & 7)) << 4) + 8 * (t & 1));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t ga = (j >> 1) ? wa.y : wa.x;
            const uint32_t gb = (j >> 1) ? wb.y : wb.x;
            const int s0 = 2 * (j & 1);
            uint32_t a[4] = {pair4(ga, s0), pair4(gb, s0), pair4(ga, s0 + 1), pair4(gb, s0 + 1)};
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              const uint4& bk = (j >> 1) ? blk1[n] : blk0[n];
              mma_16816(D[n], a, (j & 1) ? bk.z : bk.x, (j & 1) ? bk.w : bk.y);
            }
          }
        } else {
          const int chunk = 4 * G + t;
          const uint4 wa = *reinterpret_cast<const uint4*>(cm + rA * 128 + ((chunk ^ (rA & 7)) << 4));
          const uint4 wb = *reinterpret_cast<const uint4*>(cm + rB * 128 + ((chunk ^ (rB & 7)) << 4));
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t aA = (j >> 1) ? wa.z : wa.x, aB = (j >> 1) ? wa.w : wa.y;
            const uint32_t bA = (j >> 1) ? wb.z : wb.x, bB = (j >> 1) ? wb.w : wb.y;
            const int s0 = 2 * (j & 1);
            uint32_t a[4] = {pair8(aA, aB, s0), pair8(bA, bB, s0), pair8(aA, aB, s0 + 1), pair8(bA, bB, s0 + 1)};
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              const uint4& bk = (j >> 1) ? blk1[n] : blk0[n];
              mma_16816(D[n], a, (j & 1) ? bk.z : bk.x, (j & 1) ? bk.w : bk.y);
            }
          }
        }
        // ---- per-group affine epilogue
        const uint16_t* sm = s_sb + (size_t)m * 2 * kRowTile * ng;
        const uint16_t* bm = sm + (size_t)kRowTile * ng;
        const float sA = h16_to_f32(sm[rA * ng + Gabs]) * S::Q, sB = h16_to_f32(sm[rB * ng + Gabs]) * S::Q;
        const float bA = h16_to_f32(bm[rA * ng + Gabs]) - sA, bB = h16_to_f32(bm[rB * ng + Gabs]) - sB;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const float x0 = s_xs[(n * 8 + 2 * t) * xs_ld + Gabs], x1 = s_xs[(n * 8 + 2 * t + 1) * xs_ld + Gabs];
          y[m][n][0] = fmaf(sA, D[n][0], fmaf(bA, x0, y[m][n][0]));
          y[m][n][1] = fmaf(sA, D[n][1], fmaf(bA, x1, y[m][n][1]));
          y[m][n][2] = fmaf(sB, D[n][2], fmaf(bB, x0, y[m][n][2]));
          y[m][n][3] = fmaf(sB, D[n][3], fmaf(bB, x1, y[m][n][3]));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(sb_empty);

  const int row0 = it.rt * kRowTile;
  if constexpr (MODE == 0) {
    // h = silu(g) * u -> fp16 staging [32][64] in pair order
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (i < 2) ? rA : rB;
        const int tok = n * 8 + 2 * t + (i & 1);
        const float gv = y[0][n][i], uv = y[1][n][i];
        const float h = gv / (1.0f + expf(-gv)) * uv;
        s_h[tok * kRowTile + (r & ~7) + pair_pos(r & 7)] = f32_to_h16_sat(h);
      }
    // all four warps' h values staged (bounded mbarrier sync, not bar.sync)
    __syncwarp();
    if (lane == 0) mbar_arrive(&epi[0]);
    if (!mbar_wait(&epi[0], item & 1u, kDevErrTimeoutFull)) return false;
    const int R = p.R;
    for (int c = threadIdx.x; c < it.nrows * 8; c += kComputeWarps * 32) {
      const int tok = c >> 3, part = c & 7;
      const uint4 v = reinterpret_cast<const uint4*>(s_h + tok * kRowTile)[part];
      reinterpret_cast<uint4*>(p.h_out + (size_t)(it.row0_seg + tok) * R + row0)[part] = v;
    }
    if (threadIdx.x < it.nrows) {
      const int tok = threadIdx.x;
      float s = 0.0f;
      for (int c = 0; c < kRowTile; ++c) s += h16_to_f32(s_h[tok * kRowTile + c]);
      p.hsum_out[(size_t)(it.row0_seg + tok) * sum_ld(R) + it.rt] = s;
    }
    // staging buffer free again before the next item writes it
    __syncwarp();
    if (lane == 0) mbar_arrive(&epi[1]);
    if (!mbar_wait(&epi[1], item & 1u, kDevErrTimeoutFull)) return false;
  } else {
    const int R = p.R;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (i < 2) ? rA : rB;
        const int tok = n * 8 + 2 * t + (i & 1);
        if (tok < it.nrows) p.y_out[(size_t)(it.row0_seg + tok) * R + row0 + r] = y[0][n][i];
      }
  }
  return true;
}

template <int BITS, int MODE>
__global__ void __launch_bounds__(kQmvThreads, 1) qmv_kernel(const __grid_constant__ QmvParams p) {
  using S = QmvShape<BITS, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ng = p.K / 64;
  uint8_t* stage_base = smem;
  uint16_t* s_sb = reinterpret_cast<uint16_t*>(stage_base + (size_t)kStages * S::STAGE_BYTES);
  const int xs_ld = sum_ld(p.K);
  float* s_xs = reinterpret_cast<float*>(s_sb + (size_t)S::NMAT * 2 * kRowTile * ng);
  uint16_t* s_h = reinterpret_cast<uint16_t*>(s_xs + (size_t)kTokChunk * xs_ld);
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_h + (size_t)kTokChunk * kRowTile);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* sb_full = bars + 2 * kStages;
  uint64_t* sb_empty = sb_full + 1;
  uint64_t* epi = sb_full + 2;  // two epilogue syncs among the compute warps

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kComputeWarps);
    }
    mbar_init(sb_full, 1);
    mbar_init(sb_empty, kComputeWarps);
    mbar_init(&epi[0], kComputeWarps);
    mbar_init(&epi[1], kComputeWarps);
    mbar_fence_init();
  }
  __syncthreads();

  const int n_rt = p.R / kRowTile;
  const int n_work = (*p.n_seg) * n_rt;
  const int nstages = (p.K + S::KT - 1) / S::KT;

  if (warp == kComputeWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&p.tm_w0);
      if (MODE == 0) prefetch_tmap(&p.tm_w1);
      uint32_t fill_it = 0, item = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x, ++item) {
        const WorkItem it = decode_work(p, w, n_rt);
        const bool shared = it.expert >= p.n_experts;
        const size_t rowg = (size_t)(shared ? 0 : it.expert) * p.R + (size_t)it.rt * kRowTile;
        // scales / biases / group sums for this item
        if (item > 0 && !mbar_wait(sb_empty, (item - 1) & 1u, kDevErrTimeoutScales)) { ok = false; break; }
        const uint32_t sb_bytes = (uint32_t)(kRowTile * ng * 2);
        const uint32_t xs_bytes = (uint32_t)(xs_ld * 4);
        mbar_arrive_expect_tx(sb_full, S::NMAT * 2 * sb_bytes + it.nrows * xs_bytes);
        const uint16_t* src_s0 = shared ? p.ss0 : p.s0;
        const uint16_t* src_b0 = shared ? p.sb0 : p.b0;
        bulk_load(s_sb, src_s0 + rowg * ng, sb_bytes, sb_full);
        bulk_load(s_sb + kRowTile * ng, src_b0 + rowg * ng, sb_bytes, sb_full);
        if (MODE == 0) {
          const uint16_t* src_s1 = shared ? p.ss1 : p.s1;
          const uint16_t* src_b1 = shared ? p.sb1 : p.b1;
          bulk_load(s_sb + 2 * kRowTile * ng, src_s1 + rowg * ng, sb_bytes, sb_full);
          bulk_load(s_sb + 3 * kRowTile * ng, src_b1 + rowg * ng, sb_bytes, sb_full);
        }
        for (int r = 0; r < it.nrows; ++r) {
          const int src_row = p.row_src ? p.row_src[it.row0_seg + r] : it.row0_seg + r;
          bulk_load(s_xs + r * xs_ld, p.act_sum + (size_t)src_row * xs_ld, xs_bytes, sb_full);
        }
        const CUtensorMap* m0 = shared ? &p.tm_sw0 : &p.tm_w0;
        const CUtensorMap* m1 = shared ? &p.tm_sw1 : &p.tm_w1;
        for (int st = 0; st < nstages; ++st, ++fill_it) {
          const int slot = fill_it % kStages;
          if (fill_it >= (uint32_t)kStages &&
              !mbar_wait(&empty[slot], ((fill_it / kStages) - 1) & 1u, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* dst = stage_base + (size_t)slot * S::STAGE_BYTES;
          const int kcols = min(S::KT, p.K - st * S::KT);  // partial last stage: TMA zero-fills codes
          mbar_arrive_expect_tx(&full[slot], S::CODE_BYTES + it.nrows * kcols * 2);
          const int kw = st * (S::KT * BITS / 32);
          tma_load_2d(dst, m0, kw, (int)rowg, &full[slot]);
          if (MODE == 0) tma_load_2d(dst + kRowTile * S::ROWB, m1, kw, (int)rowg, &full[slot]);
          uint8_t* adst = dst + S::CODE_BYTES;
          for (int r = 0; r < it.nrows; ++r) {
            const int src_row = p.row_src ? p.row_src[it.row0_seg + r] : it.row0_seg + r;
            bulk_load(adst + r * S::ACT_PITCH, p.act + (size_t)src_row * p.K + (size_t)st * S::KT, kcols * 2,
                      &full[slot]);
          }
        }
      }
      // drain: wait (bounded) for the copies this thread issued last
      const uint32_t n_issued = fill_it;
      for (uint32_t i = (n_issued > (uint32_t)kStages ? n_issued - kStages : 0); i < n_issued; ++i)
        mbar_wait(&full[i % kStages], (i / kStages) & 1u, kDevErrTimeoutFull);
    }
    return;
  }
  // -------------------------------------------------------------- consumers
  uint32_t fill_it = 0, item = 0;
  for (int w = blockIdx.x; w < n_work; w += gridDim.x, ++item) {
    const WorkItem it = decode_work(p, w, n_rt);
    if (!mbar_wait(sb_full, item & 1u, kDevErrTimeoutScales)) return;
    const int nt = (it.nrows + 7) >> 3;
    bool ok;
    switch (nt) {
      case 1: ok = qmv_consume<BITS, MODE, 1>(p, it, stage_base, s_sb, s_xs, s_h, full, empty, sb_empty, epi, item, fill_it); break;
      case 2: ok = qmv_consume<BITS, MODE, 2>(p, it, stage_base, s_sb, s_xs, s_h, full, empty, sb_empty, epi, item, fill_it); break;
      case 3: ok = qmv_consume<BITS, MODE, 3>(p, it, stage_base, s_sb, s_xs, s_h, full, empty, sb_empty, epi, item, fill_it); break;
      default: ok = qmv_consume<BITS, MODE, 4>(p, it, stage_base, s_sb, s_xs, s_h, full, empty, sb_empty, epi, item, fill_it); break;
    }
    if (!ok) return;
  }
}

template <int BITS, int MODE>
static cudaError_t launch_qmv_t(const QmvParams& p, int n_sm, cudaStream_t st) {
  size_t smem = qmv_smem_bytes<BITS, MODE>(p.K);
  cudaError_t e = cudaFuncSetAttribute(qmv_kernel<BITS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  qmv_kernel<BITS, MODE><<<n_sm, kQmvThreads, smem, st>>>(p);
  return cudaGetLastError();
}

size_t qmv_smem_required(int bits, int mode, int K) {
  if (bits == 4) return mode == 0 ? qmv_smem_bytes<4, 0>(K) : qmv_smem_bytes<4, 1>(K);
  return mode == 0 ? qmv_smem_bytes<8, 0>(K) : qmv_smem_bytes<8, 1>(K);
}

cudaError_t launch_qmv(int bits, int mode, const QmvParams& p, int n_sm, cudaStream_t st) {
  if (bits == 4) return mode == 0 ? launch_qmv_t<4, 0>(p, n_sm, st) : launch_qmv_t<4, 1>(p, n_sm, st);
  return mode == 0 ? launch_qmv_t<8, 0>(p, n_sm, st) : launch_qmv_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
