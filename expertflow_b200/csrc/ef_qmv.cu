// ef_qmv.cu -- decode-size grouped quantised GEMV (sm_100a).
//
// Replaces the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694
// (gate, up, silu*up, down) for small token counts, where the layer is bound by
// HBM bandwidth on the packed weights.
//
// Work item = (segment of <= 8 rows routed to one expert) x (64 weight rows).
// A CTA has 4 compute warps (16 rows each), a TMA producer warp and a scale
// producer warp, and loops over work items (persistent; two CTAs per SM when
// shared memory allows).  The TMA warp streams, per 256-column (4-bit) /
// 128-column (8-bit) stage, the 64-row code tile of each matrix with a 2-D TMA
// load (128-byte swizzle) and the segment's activation rows with 1-D bulk
// copies into an mbarrier ring.  The scale warp bulk-loads, per work item, the
// tile's fp16 scales/biases (row pitch padded against bank conflicts when the
// row length allows) and the rows' group sums into one of two slots, so the
// next item's loads overlap this item's math.
//
// Dot products run on the tensor cores with exact operands: a code q becomes
// the fp16 value 1 + q/1024 by masking it into the low mantissa bits (one LOP3
// per pair of codes plus one shift per nibble/byte position); activations are
// fp16; products accumulate in fp32 per 64-column group in two independent MMA
// chains per matrix:
//     D_g = sum_i x_i (1 + q_i / 1024)
//     y  += (1024 s_g) D_g + (b_g - 1024 s_g) sum_i x_i    (= sum_i x_i (s_g q_i + b_g))
// The k order inside mma.m16n8k16 is permuted consistently for codes and
// activations (see act_pos), which leaves every dot product unchanged.
//
// mode 0: gate and up tiles together, epilogue h = silu(g) * u stored as fp16
//         rows in the activation layout + group sums (input of mode 1).
// mode 1: down projection, fp32 rows for the combine.
#include "ef_common.cuh"

namespace ef {

constexpr int kTmaWarp = kComputeWarps;
constexpr int kScaleWarp = kComputeWarps + 1;

template <int BITS, int MODE>
struct QmvShape {
  static constexpr int KT = BITS == 4 ? 256 : 128;   // columns per stage
  static constexpr int GPS = KT / 64;                 // groups per stage
  static constexpr int ROWB = KT * BITS / 8;          // bytes per code row per stage (128)
  static constexpr int NMAT = MODE == 0 ? 2 : 1;
  static constexpr int CODE_BYTES = NMAT * kRowTile * ROWB;
  static constexpr int ACT_BOX = kTokChunk * 128;     // one 64-column group of 8 activation rows
  static constexpr int ACT_BYTES = GPS * ACT_BOX;
  static constexpr int STAGE_BYTES = ((CODE_BYTES + ACT_BYTES) + 1023) / 1024 * 1024;
};
constexpr float kQ = 1024.0f;

// Group sums and scales/biases are copied as contiguous blocks (one copy per
// array per item): their shared-memory row pitch is the global one.
__host__ __device__ inline int xs_pitch(int K) { return sum_ld(K); }
__host__ __device__ inline int sb_pitch(int K) { return K / 64; }

template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_sb_bytes(int K) {  // scales + biases of one item
  return (size_t)QmvShape<BITS, MODE>::NMAT * 2 * kRowTile * sb_pitch(K) * 2;
}
__host__ __device__ inline size_t qmv_xs_bytes(int K) { return (size_t)kTokChunk * xs_pitch(K) * 4; }
template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_slot_bytes(int K) {
  return (qmv_sb_bytes<BITS, MODE>(K) + 127) / 128 * 128 + (qmv_xs_bytes(K) + 127) / 128 * 128;
}

// Shared memory: `ns` pipeline stages, two per-item slots (scales/biases and
// group sums), the h staging tile and the barriers.
template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_smem_bytes(int K, int ns) {
  using S = QmvShape<BITS, MODE>;
  size_t b = 1024;  // alignment slack
  b += (size_t)ns * S::STAGE_BYTES;
  b += 2 * qmv_slot_bytes<BITS, MODE>(K);
  b += (size_t)kTokChunk * kRowTile * 2;  // h staging (mode 0)
  b += 256;                               // barriers
  return b;
}

EF_DEV uint32_t mag(uint32_t v, uint32_t mask) { return lop3_and_or(v, mask, 0x3C003C00u); }

struct WorkItem {
  int expert, row0_seg, nrows, rt;
};

EF_DEV WorkItem decode_work(const QmvParams& p, int w, int n_rt) {
  WorkItem it;
  int seg = w / n_rt;
  it.rt = w - seg * n_rt;
  it.expert = __ldg(p.seg_expert + seg);
  it.row0_seg = __ldg(p.seg_row0 + seg);
  it.nrows = __ldg(p.seg_nrows + seg);
  return it;
}

// Bounded barrier among the compute warps built from an mbarrier.
EF_DEV bool warps_sync(uint64_t* bar, uint32_t parity) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  return mbar_wait(bar, parity, kDevErrTimeoutFull);
}

struct QmvSmem {
  uint8_t* stage_base;
  uint8_t* slot_base;
  uint16_t* s_h;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* sb_full;   // [2]
  uint64_t* sb_empty;  // [2]
  uint64_t* sync;      // [2] epilogue staging
};

// The code words of one 64-column group for rows rA, rB (8 bytes of each row at
// 4 bits, 16 at 8 bits), read from a 128-byte-swizzled stage tile.
template <int BITS>
struct GroupCodes {
  uint4 a, b;  // 4 bits: .x/.y used
};
template <int BITS>
EF_DEV GroupCodes<BITS> load_group_codes(const uint8_t* cm, int G, int rA, int rB, int t) {
  GroupCodes<BITS> c;
  if constexpr (BITS == 4) {
    const int chunk = 2 * G + (t >> 1);
    const uint2 va = *reinterpret_cast<const uint2*>(cm + rA * 128 + ((chunk ^ (rA & 7)) << 4) + 8 * (t & 1));
    const uint2 vb = *reinterpret_cast<const uint2*>(cm + rB * 128 + ((chunk ^ (rB & 7)) << 4) + 8 * (t & 1));
    c.a = make_uint4(va.x, va.y, 0u, 0u);
    c.b = make_uint4(vb.x, vb.y, 0u, 0u);
  } else {
    const int chunk = 4 * G + t;
    c.a = *reinterpret_cast<const uint4*>(cm + rA * 128 + ((chunk ^ (rA & 7)) << 4));
    c.b = *reinterpret_cast<const uint4*>(cm + rB * 128 + ((chunk ^ (rB & 7)) << 4));
  }
  return c;
}

// Dot products of one 64-column group for rows rA, rB of matrix m and the
// segment's 8 tokens; folds the group's affine scale into y.
template <int BITS, int MODE>
EF_DEV void qmv_group_regs(const GroupCodes<BITS>& cw, const uint4 (&blk)[2], float sA, float sB, float bA, float bB,
                           float x0, float x1, float (&y)[4]) {
  float D[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  if constexpr (BITS == 4) {
    const uint2 va = make_uint2(cw.a.x, cw.a.y), vb = make_uint2(cw.b.x, cw.b.y);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wa = h ? va.y : va.x, wb = h ? vb.y : vb.x;
      // nibble pairs (s, s+4): P_s = ((w >> 4s) & 0x000F000F) | 1.0h
      const uint32_t a0[4] = {mag(wa, 0x000F000Fu), mag(wb, 0x000F000Fu), mag(wa >> 4, 0x000F000Fu),
                              mag(wb >> 4, 0x000F000Fu)};
      const uint32_t a1[4] = {mag(wa >> 8, 0x000F000Fu), mag(wb >> 8, 0x000F000Fu), mag(wa >> 12, 0x000F000Fu),
                              mag(wb >> 12, 0x000F000Fu)};
      mma_16816(D[0], a0, blk[h].x, blk[h].y);
      mma_16816(D[1], a1, blk[h].z, blk[h].w);
    }
  } else {
    const uint4 va = cw.a, vb = cw.b;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wa0 = h ? va.z : va.x, wa1 = h ? va.w : va.y;  // row A: cols 0-3, 4-7 of block h
      const uint32_t wb0 = h ? vb.z : vb.x, wb1 = h ? vb.w : vb.y;
      // bytes (0,2) and (1,3) of a word: ((w >> 8k) & 0x00FF00FF) | 1.0h
      const uint32_t a0[4] = {mag(wa0, 0x00FF00FFu), mag(wb0, 0x00FF00FFu), mag(wa1, 0x00FF00FFu),
                              mag(wb1, 0x00FF00FFu)};
      const uint32_t a1[4] = {mag(wa0 >> 8, 0x00FF00FFu), mag(wb0 >> 8, 0x00FF00FFu), mag(wa1 >> 8, 0x00FF00FFu),
                              mag(wb1 >> 8, 0x00FF00FFu)};
      mma_16816(D[0], a0, blk[h].x, blk[h].y);
      mma_16816(D[1], a1, blk[h].z, blk[h].w);
    }
  }
  y[0] = fmaf(sA, D[0][0] + D[1][0], fmaf(bA, x0, y[0]));
  y[1] = fmaf(sA, D[0][1] + D[1][1], fmaf(bA, x1, y[1]));
  y[2] = fmaf(sB, D[0][2] + D[1][2], fmaf(bB, x0, y[2]));
  y[3] = fmaf(sB, D[0][3] + D[1][3], fmaf(bB, x1, y[3]));
}

template <int BITS, int MODE>
EF_DEV void qmv_group(const uint8_t* cm, const uint4 (&blk)[2], int G, int rA, int rB, int t, float sA, float sB,
                      float bA, float bB, float x0, float x1, float (&y)[4]) {
  qmv_group_regs<BITS, MODE>(load_group_codes<BITS>(cm, G, rA, rB, t), blk, sA, sB, bA, bB, x0, x1, y);
}

// One work item for one compute warp.  Returns false after a failed wait.
template <int BITS, int MODE>
EF_DEV bool qmv_item(const QmvParams& p, const WorkItem& it, const QmvSmem& sm, int q, uint32_t item,
                     uint32_t fill_base, int ns) {
  using S = QmvShape<BITS, MODE>;
  const int lane = threadIdx.x & 31, cw = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ng = p.K / 64;
  const int xp = xs_pitch(p.K), sp = sb_pitch(p.K);
  const int nstages = (p.K + S::KT - 1) / S::KT;
  const int rA = cw * 16 + g, rB = rA + 8;
  const uint8_t* slot = sm.slot_base + (size_t)q * qmv_slot_bytes<BITS, MODE>(p.K);
  const uint16_t* s_sb = reinterpret_cast<const uint16_t*>(slot);
  const float* s_xs = reinterpret_cast<const float*>(slot + (qmv_sb_bytes<BITS, MODE>(p.K) + 127) / 128 * 128);
  const bool vec_ok = (ng & 3) == 0;  // stage groups 8-byte aligned in the scale rows

  float y[S::NMAT][4];
#pragma unroll
  for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[m][i] = 0.0f;

  for (int st = 0; st < nstages; ++st) {
    const uint32_t f = fill_base + st;
    const int slot_i = f % ns;
    if (!mbar_wait(&sm.full[slot_i], (f / ns) & 1u, kDevErrTimeoutFull)) return false;
    const uint8_t* codes = sm.stage_base + (size_t)slot_i * S::STAGE_BYTES;
    // activation box of group G: [8 rows][128 B], 16-byte chunk c of row r at chunk c ^ r
    const uint8_t* act = codes + S::CODE_BYTES + (size_t)g * 128;
    const int gvalid = min(S::GPS, ng - st * S::GPS);  // last stage may be partial
    const int g0 = st * S::GPS;
    if (gvalid == S::GPS && vec_ok) {
      // ---- full stage: all loads of the stage issued up front, groups unguarded
      float xa[S::GPS], xb[S::GPS];
      if constexpr (S::GPS == 4) {
        const float4 u = *reinterpret_cast<const float4*>(s_xs + (2 * t) * xp + g0);
        const float4 v = *reinterpret_cast<const float4*>(s_xs + (2 * t + 1) * xp + g0);
        xa[0] = u.x; xa[1] = u.y; xa[2] = u.z; xa[3] = u.w;
        xb[0] = v.x; xb[1] = v.y; xb[2] = v.z; xb[3] = v.w;
      } else {
        const float2 u = *reinterpret_cast<const float2*>(s_xs + (2 * t) * xp + g0);
        const float2 v = *reinterpret_cast<const float2*>(s_xs + (2 * t + 1) * xp + g0);
        xa[0] = u.x; xa[1] = u.y;
        xb[0] = v.x; xb[1] = v.y;
      }
      uint4 blk[S::GPS][2];
#pragma unroll
      for (int G = 0; G < S::GPS; ++G) {
        blk[G][0] = *reinterpret_cast<const uint4*>(act + G * S::ACT_BOX + (((2 * t) ^ g) << 4));
        blk[G][1] = *reinterpret_cast<const uint4*>(act + G * S::ACT_BOX + (((2 * t + 1) ^ g) << 4));
      }
      // every code word of the stage up front: the shared-memory latencies
      // overlap instead of serialising group by group
      GroupCodes<BITS> cw[S::NMAT][S::GPS];
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
        for (int G = 0; G < S::GPS; ++G)
          cw[m][G] = load_group_codes<BITS>(codes + (size_t)m * kRowTile * S::ROWB, G, rA, rB, t);
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m) {
        const uint16_t* ms = s_sb + (size_t)m * 2 * kRowTile * sp;
        const uint16_t* mb = ms + (size_t)kRowTile * sp;
        uint16_t hsA[S::GPS], hsB[S::GPS], hbA[S::GPS], hbB[S::GPS];
        if constexpr (S::GPS == 4) {
          const uint2 a = *reinterpret_cast<const uint2*>(ms + rA * sp + g0);
          const uint2 b = *reinterpret_cast<const uint2*>(ms + rB * sp + g0);
          const uint2 c = *reinterpret_cast<const uint2*>(mb + rA * sp + g0);
          const uint2 d = *reinterpret_cast<const uint2*>(mb + rB * sp + g0);
          const uint32_t wa[2] = {a.x, a.y}, wb[2] = {b.x, b.y}, wc[2] = {c.x, c.y}, wd[2] = {d.x, d.y};
#pragma unroll
          for (int G = 0; G < 4; ++G) {
            hsA[G] = (uint16_t)(wa[G >> 1] >> (16 * (G & 1)));
            hsB[G] = (uint16_t)(wb[G >> 1] >> (16 * (G & 1)));
            hbA[G] = (uint16_t)(wc[G >> 1] >> (16 * (G & 1)));
            hbB[G] = (uint16_t)(wd[G >> 1] >> (16 * (G & 1)));
          }
        } else {
          const uint32_t a = *reinterpret_cast<const uint32_t*>(ms + rA * sp + g0);
          const uint32_t b = *reinterpret_cast<const uint32_t*>(ms + rB * sp + g0);
          const uint32_t c = *reinterpret_cast<const uint32_t*>(mb + rA * sp + g0);
          const uint32_t d = *reinterpret_cast<const uint32_t*>(mb + rB * sp + g0);
#pragma unroll
          for (int G = 0; G < 2; ++G) {
            hsA[G] = (uint16_t)(a >> (16 * G));
            hsB[G] = (uint16_t)(b >> (16 * G));
            hbA[G] = (uint16_t)(c >> (16 * G));
            hbB[G] = (uint16_t)(d >> (16 * G));
          }
        }
#pragma unroll
        for (int G = 0; G < S::GPS; ++G) {
          const float sA = h16_to_f32(hsA[G]) * kQ, sB = h16_to_f32(hsB[G]) * kQ;
          qmv_group_regs<BITS, MODE>(cw[m][G], blk[G], sA, sB, h16_to_f32(hbA[G]) - sA, h16_to_f32(hbB[G]) - sB,
                                     xa[G], xb[G], y[m]);
        }
      }
    } else {
#pragma unroll
      for (int G = 0; G < S::GPS; ++G) {
        if (G < gvalid) {
          const int Gabs = g0 + G;
          const uint4 blk[2] = {*reinterpret_cast<const uint4*>(act + G * S::ACT_BOX + (((2 * t) ^ g) << 4)),
                                *reinterpret_cast<const uint4*>(act + G * S::ACT_BOX + (((2 * t + 1) ^ g) << 4))};
          const float x0 = s_xs[(2 * t) * xp + Gabs], x1 = s_xs[(2 * t + 1) * xp + Gabs];
#pragma unroll
          for (int m = 0; m < S::NMAT; ++m) {
            const uint16_t* ms = s_sb + (size_t)m * 2 * kRowTile * sp;
            const uint16_t* mb = ms + (size_t)kRowTile * sp;
            const float sA = h16_to_f32(ms[rA * sp + Gabs]) * kQ, sB = h16_to_f32(ms[rB * sp + Gabs]) * kQ;
            const float bA = h16_to_f32(mb[rA * sp + Gabs]) - sA, bB = h16_to_f32(mb[rB * sp + Gabs]) - sB;
            qmv_group<BITS, MODE>(codes + (size_t)m * kRowTile * S::ROWB, blk, G, rA, rB, t, sA, sB, bA, bB, x0,
                                  x1, y[m]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot_i]);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&sm.sb_empty[q]);  // slot may be reloaded

  const int row0 = it.rt * kRowTile;
  const int R = p.R;
  if constexpr (MODE == 0) {
    // h = silu(g) * u -> fp16 staging [8][64] in the activation layout
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (i < 2) ? rA : rB;
      const int tok = 2 * t + (i & 1);
      const float gv = y[0][i], uv = y[1][i];
      const float h = gv / (1.0f + expf(-gv)) * uv;
      sm.s_h[tok * kRowTile + (r & ~7) + act_pos(r & 7, BITS)] = f32_to_h16_sat(h);
    }
    if (!warps_sync(&sm.sync[0], item & 1u)) return false;
    for (int c = threadIdx.x; c < it.nrows * 8; c += kComputeWarps * 32) {
      const int tok = c >> 3, part = c & 7;
      const uint4 v = reinterpret_cast<const uint4*>(sm.s_h + tok * kRowTile)[part];
      reinterpret_cast<uint4*>(p.h_out + (size_t)(it.row0_seg + tok) * R + row0)[part] = v;
    }
    if ((int)threadIdx.x < it.nrows) {
      const int tok = threadIdx.x;
      float s = 0.0f;
      for (int c = 0; c < kRowTile; ++c) s += h16_to_f32(sm.s_h[tok * kRowTile + c]);
      p.hsum_out[(size_t)(it.row0_seg + tok) * sum_ld(R) + it.rt] = s;
    }
    if (!warps_sync(&sm.sync[1], item & 1u)) return false;  // staging free for the next item
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (i < 2) ? rA : rB;
      const int tok = 2 * t + (i & 1);
      if (tok < it.nrows) p.y_out[(size_t)(it.row0_seg + tok) * R + row0 + r] = y[0][i];
    }
  }
  return true;
}

template <int BITS, int MODE>
__global__ void __launch_bounds__(kQmvThreads, 2) qmv_kernel(const __grid_constant__ QmvParams p) {
  using S = QmvShape<BITS, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int ns = p.n_stages;
  const int ng = p.K / 64;
  QmvSmem sm;
  sm.stage_base = smem;
  sm.slot_base = sm.stage_base + (size_t)ns * S::STAGE_BYTES;
  sm.s_h = reinterpret_cast<uint16_t*>(sm.slot_base + 2 * qmv_slot_bytes<BITS, MODE>(p.K));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm.s_h + (size_t)kTokChunk * kRowTile);
  sm.full = bars;
  sm.empty = bars + ns;
  sm.sb_full = bars + 2 * ns;
  sm.sb_empty = sm.sb_full + 2;
  sm.sync = sm.sb_full + 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kComputeWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.sb_full[i], 1);
      mbar_init(&sm.sb_empty[i], kComputeWarps);
      mbar_init(&sm.sync[i], kComputeWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  const int n_rt = p.R / kRowTile;
  const int n_work = (*p.n_seg) * n_rt;
  const int nstages = (p.K + S::KT - 1) / S::KT;

  if (warp == kTmaWarp) {
    if (lane != 0) return;
    // ---------------------------------------------------- stage ring (codes + activation rows)
    prefetch_tmap(&p.tm_w0);
    if (MODE == 0) prefetch_tmap(&p.tm_w1);
    prefetch_tmap(&p.tm_act);
    uint32_t fill_it = 0;
    bool ok = true;
    int w = blockIdx.x;
    WorkItem nxt = w < n_work ? decode_work(p, w, n_rt) : WorkItem{0, 0, 0, 0};
    for (; w < n_work && ok; w += gridDim.x) {
      const WorkItem it = nxt;
      if (w + (int)gridDim.x < n_work) nxt = decode_work(p, w + gridDim.x, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const int rowg = (shared ? 0 : it.expert) * p.R + it.rt * kRowTile;
      const CUtensorMap* m0 = shared ? &p.tm_sw0 : &p.tm_w0;
      const CUtensorMap* m1 = shared ? &p.tm_sw1 : &p.tm_w1;
      for (int st = 0; st < nstages; ++st, ++fill_it) {
        const int slot = fill_it % ns;
        if (fill_it >= (uint32_t)ns && !mbar_wait(&sm.empty[slot], ((fill_it / ns) - 1) & 1u, kDevErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint8_t* dst = sm.stage_base + (size_t)slot * S::STAGE_BYTES;
        // partial last stage: the code box past the row end is zero-filled by TMA
        const int gv = min(S::GPS, ng - st * S::GPS);
        mbar_arrive_expect_tx(&sm.full[slot], S::CODE_BYTES + gv * S::ACT_BOX);
        const int kw = st * (S::KT * BITS / 32);
        tma_load_2d(dst, m0, kw, rowg, &sm.full[slot]);
        if (MODE == 0) tma_load_2d(dst + kRowTile * S::ROWB, m1, kw, rowg, &sm.full[slot]);
        uint8_t* adst = dst + S::CODE_BYTES;
        for (int G = 0; G < gv; ++G)
          tma_load_2d(adst + G * S::ACT_BOX, &p.tm_act, st * S::KT + 64 * G, it.row0_seg, &sm.full[slot]);
      }
    }
    // drain: wait (bounded) for the copies issued last
    for (uint32_t i = (fill_it > (uint32_t)ns ? fill_it - ns : 0); i < fill_it; ++i)
      mbar_wait(&sm.full[i % ns], (i / ns) & 1u, kDevErrTimeoutFull);
    return;
  }
  if (warp == kScaleWarp) {
    if (lane != 0) return;
    // ---------------------------------------------------- per-item scales/biases and group sums
    const int xs_ld = sum_ld(p.K), sp = sb_pitch(p.K);
    uint32_t item = 0;
    int w = blockIdx.x;
    WorkItem nxt = w < n_work ? decode_work(p, w, n_rt) : WorkItem{0, 0, 0, 0};
    for (; w < n_work; w += gridDim.x, ++item) {
      const WorkItem it = nxt;
      if (w + (int)gridDim.x < n_work) nxt = decode_work(p, w + gridDim.x, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const size_t rowg = (size_t)(shared ? 0 : it.expert) * p.R + (size_t)it.rt * kRowTile;
      const int q = item & 1;
      if (item >= 2 && !mbar_wait(&sm.sb_empty[q], ((item >> 1) - 1) & 1u, kDevErrTimeoutScales)) break;
      uint8_t* slot = sm.slot_base + (size_t)q * qmv_slot_bytes<BITS, MODE>(p.K);
      uint16_t* s_sb = reinterpret_cast<uint16_t*>(slot);
      float* s_xs = reinterpret_cast<float*>(slot + (qmv_sb_bytes<BITS, MODE>(p.K) + 127) / 128 * 128);
      const uint32_t row_bytes = (uint32_t)(ng * 2);
      const uint32_t xs_bytes = (uint32_t)(it.nrows * xs_ld * 4);
      mbar_arrive_expect_tx(&sm.sb_full[q], S::NMAT * 2 * kRowTile * row_bytes + xs_bytes);
      const uint16_t* srcs[4] = {shared ? p.ss0 : p.s0, shared ? p.sb0 : p.b0, shared ? p.ss1 : p.s1,
                                 shared ? p.sb1 : p.b1};
#pragma unroll
      for (int a = 0; a < 2 * S::NMAT; ++a) {
        const uint16_t* gsrc = srcs[a] + rowg * ng;
        uint16_t* dst = s_sb + (size_t)a * kRowTile * sp;
        bulk_load(dst, gsrc, kRowTile * row_bytes, &sm.sb_full[q]);
      }
      bulk_load(s_xs, p.act_sum + (size_t)it.row0_seg * xs_ld, xs_bytes, &sm.sb_full[q]);
    }
    if (item > 0) mbar_wait(&sm.sb_full[(item - 1) & 1], ((item - 1) >> 1) & 1u, kDevErrTimeoutScales);
    return;
  }
  // -------------------------------------------------------------- compute warps
  uint32_t fill_base = 0, item = 0;
  int w = blockIdx.x;
  WorkItem nxt = w < n_work ? decode_work(p, w, n_rt) : WorkItem{0, 0, 0, 0};
  for (; w < n_work; w += gridDim.x, ++item) {
    const WorkItem it = nxt;
    if (w + (int)gridDim.x < n_work) nxt = decode_work(p, w + gridDim.x, n_rt);
    const int q = item & 1;
    if (!mbar_wait(&sm.sb_full[q], (item >> 1) & 1u, kDevErrTimeoutScales)) return;
    if (!qmv_item<BITS, MODE>(p, it, sm, q, item, fill_base, ns)) return;
    fill_base += nstages;
  }
}

// Ring depth and CTAs per SM: two CTAs per SM with >= 3 stages each when they
// fit in half of the shared memory, else one CTA with the deepest ring.
template <int BITS, int MODE>
static int qmv_pick(int K, int* ctas_per_sm) {
  if (K > 16384) return 0;
  for (int ns = 6; ns >= 3; --ns)
    if (qmv_smem_bytes<BITS, MODE>(K, ns) <= 113 * 1024) { *ctas_per_sm = 2; return ns; }
  for (int ns = 6; ns >= 2; --ns)
    if (qmv_smem_bytes<BITS, MODE>(K, ns) <= 227 * 1024) { *ctas_per_sm = 1; return ns; }
  return 0;
}

template <int BITS, int MODE>
static cudaError_t launch_qmv_t(const QmvParams& p_in, int n_sm, cudaStream_t st) {
  QmvParams p = p_in;
  int per_sm = 1;
  p.n_stages = qmv_pick<BITS, MODE>(p.K, &per_sm);
  if (p.n_stages == 0) return cudaErrorInvalidValue;
  const size_t smem = qmv_smem_bytes<BITS, MODE>(p.K, p.n_stages);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(qmv_kernel<BITS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  qmv_kernel<BITS, MODE><<<n_sm * per_sm, kQmvThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// SIZE_MAX when the decode kernel cannot hold a K-wide item in shared memory.
size_t qmv_smem_required(int bits, int mode, int K) {
  int per = 1, ns;
  if (bits == 4) {
    ns = mode == 0 ? qmv_pick<4, 0>(K, &per) : qmv_pick<4, 1>(K, &per);
    if (!ns) return ~size_t(0);
    return mode == 0 ? qmv_smem_bytes<4, 0>(K, ns) : qmv_smem_bytes<4, 1>(K, ns);
  }
  ns = mode == 0 ? qmv_pick<8, 0>(K, &per) : qmv_pick<8, 1>(K, &per);
  if (!ns) return ~size_t(0);
  return mode == 0 ? qmv_smem_bytes<8, 0>(K, ns) : qmv_smem_bytes<8, 1>(K, ns);
}

cudaError_t launch_qmv(int bits, int mode, const QmvParams& p, int n_sm, cudaStream_t st) {
  if (bits == 4) return mode == 0 ? launch_qmv_t<4, 0>(p, n_sm, st) : launch_qmv_t<4, 1>(p, n_sm, st);
  return mode == 0 ? launch_qmv_t<8, 0>(p, n_sm, st) : launch_qmv_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
