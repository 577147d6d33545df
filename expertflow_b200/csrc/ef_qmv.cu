// ef_qmv.cu -- decode-size grouped quantised GEMV (sm_100a).
//
// Replaces the per-(token, k) mx.quantized_matmul calls of ef_engine.py:689-694
// (gate, up, silu*up, down) for small token counts, where the layer is bound by
// HBM bandwidth on the packed weights.
//
// Work item = (segment of <= 16 rows routed to one expert) x (64 weight rows);
// a segment of more than 8 rows is two MMA n-tiles that share every unpacked
// code, so the expert's weights pass through the SM once for up to 16 tokens.
// A CTA has 4 compute warps (16 rows each), a TMA producer warp and a scale
// producer warp, and loops over work items (persistent; two CTAs per SM).
//  * The TMA warp streams, per 256-column (4-bit) / 128-column (8-bit) stage,
//    the 64-row code tile of each matrix (2-D TMA, 128-byte swizzle) and the
//    segment's activation rows into an mbarrier ring.
//  * The scale warp streams the tile's fp16 scales and biases in chunks of 32
//    groups (2-D TMA boxes of 32 groups x 64 rows, 64-byte swizzle, so that a
//    chunk slot is 16 KB whatever K is and the compute warps' reads are free
//    of bank conflicts) together with the rows' group sums, into a ring of
//    slots a chunk or more ahead of the compute warps.  When the row length
//    is not a multiple of 8 groups (16 bytes) the slot holds a whole item's
//    scales instead, copied as contiguous blocks.  In mode 0 the same warp
//    also copies each finished item's h tile from shared memory to h_out, so
//    the compute warps go straight on to the next item.
//
// Dot products run on the tensor cores with exact operands: a code q becomes
// the fp16 value 1024 + q, placed in the low mantissa bits under the exponent
// of 1024 (4-bit: one LOP3 per pair of codes plus one shift per nibble
// position; 8-bit: one byte permute per pair); activations are fp16; products
// accumulate in fp32 per 64-column group in one MMA chain per matrix:
//     D_g = sum_i x_i (1024 + q_i)
//     y  += s_g D_g + (b_g - 1024 s_g) sum_i x_i    (= sum_i x_i (s_g q_i + b_g))
// The k order inside mma.m16n8k16 is permuted consistently for codes and
// activations (see act_pos), which leaves every dot product unchanged.  The
// 16 weight rows of an MMA block are taken in the order row_of_lane(), so that
// the swizzled code words and scales a warp loads fall in distinct banks.
//
// mode 0: gate and up tiles together, epilogue h = silu(g) * u stored as fp16
//         rows in the activation layout + group sums (input of mode 1).
// mode 1: down projection, fp32 rows for the combine.
// mode 2: mode 1 with 128-row items, taken as two 64-row tiles of the same
//         matrix in the two-matrix path of mode 0 (twice the work per stage
//         and per item, one activation tile for both).
#include "ef_common.cuh"

namespace ef {

constexpr int kTmaWarp = kComputeWarps;
constexpr int kScaleWarp = kComputeWarps + 1;

template <int BITS, int MODE>
struct QmvShape {
  static constexpr int KT = BITS == 4 ? 256 : 128;   // columns per stage
  static constexpr int GPS = KT / 64;                 // groups per stage
  static constexpr int ROWB = KT * BITS / 8;          // bytes per code row per stage (128)
  static constexpr int NMAT = MODE == 1 ? 1 : 2;
  static constexpr int ITEM_ROWS = MODE == 2 ? 2 * kRowTile : kRowTile;  // weight rows per work item
  static constexpr int CODE_BYTES = NMAT * kRowTile * ROWB;
  static constexpr int ACT_BOX = kTokChunk * 128;     // one 64-column group of 8 activation rows (a TMA box)
  static constexpr int ACT_GROUP = kSegRows * 128;    // a group's rows of both n-tiles
  static constexpr int ACT_BYTES = GPS * ACT_GROUP;
  static constexpr int STAGE_BYTES = ((CODE_BYTES + ACT_BYTES) + 1023) / 1024 * 1024;
};
constexpr float kQ = 1024.0f;

// Weight row (within a 16-row MMA block, first half) held by the lanes of group
// g = lane / 4.  The code tile's 16-byte units are swizzled by row % 8; with
// 8-byte code loads a half-warp (g = 0..3) then reads rows 0, 2, 4, 6 and
// covers all 32 banks, with 16-byte loads each 8-lane phase reads rows r and
// r + 4.
template <int BITS>
__host__ __device__ constexpr int row_of_lane(int g) {
  return BITS == 4 ? 2 * (g & 3) + (g >> 2) : (g >> 1) + 4 * (g & 1);
}

// ---- scale slots
// Chunked: [2 * NMAT arrays][64 rows][32 groups] fp16 in the TMA's 64-byte
// swizzle (a 4 KB box per array), then the group sums [16 tokens][32] fp32.
// Whole item: [2 * NMAT][64][K / 64] fp16 and [16][sum_ld(K)] fp32, both as
// contiguous copies.
constexpr int kSbChunk = 32;                          // groups per chunk
constexpr int kSbBox = kRowTile * kSbChunk * 2;       // bytes of one array's box
constexpr int kXsPitchChunk = kSbChunk;               // floats (unpadded: the smem budget has no room for a pad)

template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_slot_bytes(int K, bool chunked) {
  constexpr int NM = QmvShape<BITS, MODE>::NMAT;
  size_t sb, xs;
  if (chunked) {
    sb = (size_t)2 * NM * kSbBox;
    xs = (size_t)kSegRows * kXsPitchChunk * 4;
  } else {
    sb = (size_t)2 * NM * kRowTile * (K / 64) * 2;
    xs = (size_t)kSegRows * sum_ld(K) * 4;
  }
  const size_t b = (sb + 127) / 128 * 128 + (xs + 127) / 128 * 128;
  return (b + 1023) / 1024 * 1024;  // slots stay 1024-byte aligned (swizzle atoms)
}

// Shared memory: `ns` pipeline stages, `nq` scale slots, in mode 0 the
// double-buffered h staging tile and its per-warp sums, and the barriers.
// The dynamic shared memory starts 1024-byte aligned (checked by the kernel),
// so no alignment slack is reserved: three 24 KB stages must fit beside the
// scale slots in the 113 KB a CTA has at two CTAs per SM.
template <int BITS, int MODE>
__host__ __device__ inline size_t qmv_smem_bytes(int K, int ns, int nq, bool chunked) {
  using S = QmvShape<BITS, MODE>;
  size_t b = 0;
  b += (size_t)ns * S::STAGE_BYTES;
  b += (size_t)nq * qmv_slot_bytes<BITS, MODE>(K, chunked);
  if (MODE == 0) {
    b += (size_t)2 * kSegRows * kRowTile * 2;       // h staging
    b += (size_t)2 * kComputeWarps * kSegRows * 4;  // h sums
  }
  b += 256;                                         // barriers: 2 ns + 2 nq + 4
  return b;
}

// Index (in fp16 words, within one array of a slot) of row r, slot-relative
// group gc.  Chunked slots follow the 64-byte TMA swizzle: 16-byte unit u of
// the 64-byte row r sits at unit u ^ ((r >> 1) & 3).
EF_DEV int sb_word(bool chunked, int r, int gc, int row_len) {
  if (!chunked) return r * row_len + gc;
  return r * kSbChunk + ((((gc >> 3) ^ ((r >> 1) & 3)) << 3) | (gc & 7));
}

// (v & mask) | 1024.0h in both halves: the fp16 pair (1024 + q_lo, 1024 + q_hi)
EF_DEV uint32_t mag(uint32_t v, uint32_t mask) { return lop3_and_or(v, mask, 0x64006400u); }
// Bytes of v picked by `sel` (0x4240: bytes 0, 2; 0x4341: bytes 1, 3) as the low
// bytes of two fp16 halves whose high byte is 0x64: the pair (1024 + b, 1024 + b').
EF_DEV uint32_t mag8(uint32_t v, uint32_t sel) { return prmt(v, 0x64646464u, sel); }

// N consecutive floats / fp16 words from shared memory (N * size aligned).
template <int N>
EF_DEV void load_f32s(const float* p, float (&v)[N]) {
  if constexpr (N == 4) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
  } else if constexpr (N == 2) {
    const float2 u = *reinterpret_cast<const float2*>(p);
    v[0] = u.x; v[1] = u.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = p[i];
  }
}
template <int N>
EF_DEV void load_h16s(const uint16_t* p, uint16_t (&h)[N]) {
  if constexpr (N == 4) {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    h[0] = (uint16_t)a.x; h[1] = (uint16_t)(a.x >> 16); h[2] = (uint16_t)a.y; h[3] = (uint16_t)(a.y >> 16);
  } else if constexpr (N == 2) {
    const uint32_t a = *reinterpret_cast<const uint32_t*>(p);
    h[0] = (uint16_t)a; h[1] = (uint16_t)(a >> 16);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) h[i] = p[i];
  }
}

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

struct QmvSmem {
  uint8_t* stage_base;
  uint8_t* slot_base;
  uint16_t* s_h;       // [2][8][64] h staging (mode 0)
  float* hsum;         // [2][kComputeWarps][8] per-warp h sums (mode 0)
  uint64_t* full;
  uint64_t* empty;
  uint64_t* sb_full;   // [n_slots]
  uint64_t* sb_empty;  // [n_slots]
  uint64_t* h_ready;   // [2] mode 0: h tile staged (compute warps)
  uint64_t* h_free;    // [2] mode 0: h tile copied out (scale warp)
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
// segment's tokens 0..7 (blk) and, when `two`, its tokens 8..15 (blk2): the
// codes are unpacked once and feed both n-tiles.  Folds the group's affine
// scale into y / y2 (sA, sB: scales; bA, bB: bias - 1024 * scale; x0, x1: the
// group sums of tokens 2t, 2t + 1; x2, x3: of tokens 8 + 2t, 9 + 2t).  `two`
// is uniform across the warp.
template <int BITS>
EF_DEV void qmv_group_regs(const GroupCodes<BITS>& cw, const uint4 (&blk)[2], const uint4 (&blk2)[2], bool two,
                           float sA, float sB, float bA, float bB, float x0, float x1, float x2, float x3,
                           float (&y)[4], float (&y2)[4]) {
  float D[4] = {0.f, 0.f, 0.f, 0.f};
  float E[4] = {0.f, 0.f, 0.f, 0.f};
  if constexpr (BITS == 4) {
    const uint2 va = make_uint2(cw.a.x, cw.a.y), vb = make_uint2(cw.b.x, cw.b.y);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wa = h ? va.y : va.x, wb = h ? vb.y : vb.x;
      // nibble pairs (s, s+4): P_s = ((w >> 4s) & 0x000F000F) | 1024.0h
      const uint32_t a0[4] = {mag(wa, 0x000F000Fu), mag(wb, 0x000F000Fu), mag(wa >> 4, 0x000F000Fu),
                              mag(wb >> 4, 0x000F000Fu)};
      const uint32_t a1[4] = {mag(wa >> 8, 0x000F000Fu), mag(wb >> 8, 0x000F000Fu), mag(wa >> 12, 0x000F000Fu),
                              mag(wb >> 12, 0x000F000Fu)};
      mma_16816(D, a0, blk[h].x, blk[h].y);
      mma_16816(D, a1, blk[h].z, blk[h].w);
      if (two) {
        mma_16816(E, a0, blk2[h].x, blk2[h].y);
        mma_16816(E, a1, blk2[h].z, blk2[h].w);
      }
    }
  } else {
    const uint4 va = cw.a, vb = cw.b;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t wa0 = h ? va.z : va.x, wa1 = h ? va.w : va.y;  // row A: cols 0-3, 4-7 of block h
      const uint32_t wb0 = h ? vb.z : vb.x, wb1 = h ? vb.w : vb.y;
      // bytes (0,2) and (1,3) of a word under the high byte 0x64 of 1024.0h,
      // one byte permute per pair
      const uint32_t a0[4] = {mag8(wa0, 0x4240u), mag8(wb0, 0x4240u), mag8(wa1, 0x4240u), mag8(wb1, 0x4240u)};
      const uint32_t a1[4] = {mag8(wa0, 0x4341u), mag8(wb0, 0x4341u), mag8(wa1, 0x4341u), mag8(wb1, 0x4341u)};
      mma_16816(D, a0, blk[h].x, blk[h].y);
      mma_16816(D, a1, blk[h].z, blk[h].w);
      if (two) {
        mma_16816(E, a0, blk2[h].x, blk2[h].y);
        mma_16816(E, a1, blk2[h].z, blk2[h].w);
      }
    }
  }
  y[0] = fmaf(sA, D[0], fmaf(bA, x0, y[0]));
  y[1] = fmaf(sA, D[1], fmaf(bA, x1, y[1]));
  y[2] = fmaf(sB, D[2], fmaf(bB, x0, y[2]));
  y[3] = fmaf(sB, D[3], fmaf(bB, x1, y[3]));
  if (two) {
    y2[0] = fmaf(sA, E[0], fmaf(bA, x2, y2[0]));
    y2[1] = fmaf(sA, E[1], fmaf(bA, x3, y2[1]));
    y2[2] = fmaf(sB, E[2], fmaf(bB, x2, y2[2]));
    y2[3] = fmaf(sB, E[3], fmaf(bB, x3, y2[3]));
  }
}

// fp16 word G of N packed consecutive fp16 values (N = 4: a uint2; N = 2: in .x)
template <int N>
EF_DEV uint16_t h16_at(const uint2& v, int G) {
  const uint32_t w = (N == 4 && G >= 2) ? v.y : v.x;
  return (uint16_t)(w >> ((G & 1) * 16));
}
template <int N>
EF_DEV uint2 load_h16_pack(const uint16_t* p) {
  if constexpr (N == 4) return *reinterpret_cast<const uint2*>(p);
  else return make_uint2(*reinterpret_cast<const uint32_t*>(p), 0u);
}

// Scale warp, mode 0: copy item e's staged h tile to h_out and its per-token
// sums (over the compute warps, in warp order) to hsum_out, then free the
// staging buffer.  Returns false after a failed wait.
template <int BITS, int MODE>
EF_DEV bool qmv_h_out(const QmvParams& p, const QmvSmem& sm, const WorkItem& it, uint32_t e) {
  const int lane = threadIdx.x & 31;
  const uint32_t b = e & 1u;
  bool ok = true;
  if (lane == 0) ok = mbar_wait(&sm.h_ready[b], (e >> 1) & 1u, kDevErrTimeoutFull);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return false;
  const uint16_t* s_h = sm.s_h + (size_t)b * kSegRows * kRowTile;
  const float* s_hs = sm.hsum + (size_t)b * kComputeWarps * kSegRows;
  const int R = p.R, row0 = it.rt * kRowTile;
  for (int c = lane; c < it.nrows * 8; c += 32) {
    const int tok = c >> 3, part = c & 7;
    const uint4 v = reinterpret_cast<const uint4*>(s_h + tok * kRowTile)[part];
    reinterpret_cast<uint4*>(p.h_out + (size_t)(it.row0_seg + tok) * R + row0)[part] = v;
  }
  if (lane < it.nrows) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) s += s_hs[w * kSegRows + lane];
    p.hsum_out[(size_t)(it.row0_seg + lane) * sum_ld(R) + it.rt] = s;
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&sm.h_free[b]);
  return true;
}

// Scale-slot bookkeeping shared by the producer and the compute warps.
struct SbGeom {
  bool chunked;
  int spc;      // stages per scale chunk
  int row_len;  // groups per slot row
  int xp;       // floats per token row of the slot's group sums
};
template <int BITS, int MODE>
EF_DEV SbGeom sb_geom(const QmvParams& p, int nstages) {
  SbGeom g;
  g.chunked = p.sb_chunked != 0;
  g.spc = g.chunked ? kSbChunk / QmvShape<BITS, MODE>::GPS : nstages;
  g.row_len = g.chunked ? kSbChunk : p.K / 64;
  g.xp = g.chunked ? kXsPitchChunk : sum_ld(p.K);
  return g;
}

// One work item for one compute warp; `cc` counts the scale chunks consumed.
// A segment of more than 8 rows runs its tokens 8..15 as a second n-tile on
// the same unpacked codes (`two`, uniform across the CTA).  Returns false after
// a failed wait.
template <int BITS, int MODE>
EF_DEV bool qmv_item(const QmvParams& p, const WorkItem& it, const QmvSmem& sm, uint32_t item, uint32_t fill_base,
                     uint32_t& cc, int ns, int nq) {
  using S = QmvShape<BITS, MODE>;
  constexpr int GPS = S::GPS;
  const int lane = threadIdx.x & 31, cw = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int ng = p.K / 64;
  const int nstages = (p.K + S::KT - 1) / S::KT;
  const SbGeom geo = sb_geom<BITS, MODE>(p, nstages);
  const size_t slot_bytes = qmv_slot_bytes<BITS, MODE>(p.K, geo.chunked);
  const size_t arr_words = geo.chunked ? (size_t)kRowTile * kSbChunk : (size_t)kRowTile * ng;
  const size_t xs_off =
      geo.chunked ? (size_t)2 * S::NMAT * kSbBox : ((size_t)2 * S::NMAT * arr_words * 2 + 127) / 128 * 128;
  const int rA = cw * 16 + row_of_lane<BITS>(g), rB = rA + 8;
  const bool vec_ok = geo.chunked || (ng & 3) == 0;  // a stage's groups aligned in the scale rows
  const bool two = it.nrows > kTokChunk;

  float y[S::NMAT][4], y2[S::NMAT][4];
#pragma unroll
  for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[m][i] = y2[m][i] = 0.0f;

  const uint16_t* s_sb = nullptr;
  const float* s_xs = nullptr;
  int q = 0, sc = 0, cg0 = 0;  // slot, stage within the chunk, first group of the chunk
  int slot_i = (int)(fill_base % (uint32_t)ns);
  uint32_t phase = (fill_base / (uint32_t)ns) & 1u;
  const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
  for (int st = 0; st < nstages; ++st) {
    if (sc == 0) {  // a new scale chunk
      q = (int)(cc % (uint32_t)nq);
      if (!mbar_wait(&sm.sb_full[q], (cc / (uint32_t)nq) & 1u, kDevErrTimeoutScales)) return false;
      const uint8_t* slot = sm.slot_base + (size_t)q * slot_bytes;
      s_sb = reinterpret_cast<const uint16_t*>(slot);
      s_xs = reinterpret_cast<const float*>(slot + xs_off);
      cg0 = st * GPS;
    }
    if (!mbar_wait(&sm.full[slot_i], phase, kDevErrTimeoutFull)) return false;
    const uint8_t* codes = sm.stage_base + (size_t)slot_i * S::STAGE_BYTES;
    // activation rows of group G: [16 rows][128 B] (rows 8..15 loaded only for
    // two n-tiles), 16-byte chunk c of row r at chunk c ^ (r % 8)
    const uint8_t* act = codes + S::CODE_BYTES + (size_t)g * 128;
    const uint8_t* act2 = act + (size_t)kTokChunk * 128;
    const int gvalid = min(GPS, ng - st * GPS);  // last stage may be partial
    const int gc = st * GPS - cg0;               // slot-relative first group of the stage
    if (gvalid == GPS && vec_ok && !two) {
      // ---- full stage, one n-tile: every load of the stage issued up front
      // (their shared-memory latencies overlap), groups unguarded
      float xa[GPS], xb[GPS];
      load_f32s<GPS>(s_xs + (2 * t) * geo.xp + gc, xa);
      load_f32s<GPS>(s_xs + (2 * t + 1) * geo.xp + gc, xb);
      uint4 blk[GPS][2];
#pragma unroll
      for (int G = 0; G < GPS; ++G) {
        blk[G][0] = *reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t) ^ g) << 4));
        blk[G][1] = *reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t + 1) ^ g) << 4));
      }
      GroupCodes<BITS> cwd[S::NMAT][GPS];
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
        for (int G = 0; G < GPS; ++G)
          cwd[m][G] = load_group_codes<BITS>(codes + (size_t)m * kRowTile * S::ROWB, G, rA, rB, t);
      const int wA = sb_word(geo.chunked, rA, gc, geo.row_len), wB = sb_word(geo.chunked, rB, gc, geo.row_len);
      const uint4 none[2] = {zero4, zero4};
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m) {
        const uint16_t* ms = s_sb + (size_t)m * 2 * arr_words;
        const uint16_t* mb = ms + arr_words;
        uint16_t hsA[GPS], hsB[GPS], hbA[GPS], hbB[GPS];
        load_h16s<GPS>(ms + wA, hsA);
        load_h16s<GPS>(ms + wB, hsB);
        load_h16s<GPS>(mb + wA, hbA);
        load_h16s<GPS>(mb + wB, hbB);
#pragma unroll
        for (int G = 0; G < GPS; ++G) {
          const float sA = h16_to_f32(hsA[G]), sB = h16_to_f32(hsB[G]);
          qmv_group_regs<BITS>(cwd[m][G], blk[G], none, false, sA, sB, fmaf(-kQ, sA, h16_to_f32(hbA[G])),
                               fmaf(-kQ, sB, h16_to_f32(hbB[G])), xa[G], xb[G], 0.0f, 0.0f, y[m], y2[m]);
        }
      }
    } else if (gvalid == GPS && vec_ok) {
      // ---- full stage, two n-tiles: sums, code words and scales of the stage
      // up front, each group's activation rows of both n-tiles as the group
      // comes up (fewer live registers), groups unguarded
      float xa[GPS], xb[GPS], xc[GPS], xd[GPS];
      load_f32s<GPS>(s_xs + (2 * t) * geo.xp + gc, xa);
      load_f32s<GPS>(s_xs + (2 * t + 1) * geo.xp + gc, xb);
      load_f32s<GPS>(s_xs + (kTokChunk + 2 * t) * geo.xp + gc, xc);
      load_f32s<GPS>(s_xs + (kTokChunk + 2 * t + 1) * geo.xp + gc, xd);
      GroupCodes<BITS> cwd[S::NMAT][GPS];
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
        for (int G = 0; G < GPS; ++G)
          cwd[m][G] = load_group_codes<BITS>(codes + (size_t)m * kRowTile * S::ROWB, G, rA, rB, t);
      const int wA = sb_word(geo.chunked, rA, gc, geo.row_len), wB = sb_word(geo.chunked, rB, gc, geo.row_len);
      uint2 hsA[S::NMAT], hsB[S::NMAT], hbA[S::NMAT], hbB[S::NMAT];  // fp16 scales / biases of the GPS groups
#pragma unroll
      for (int m = 0; m < S::NMAT; ++m) {
        const uint16_t* ms = s_sb + (size_t)m * 2 * arr_words;
        const uint16_t* mb = ms + arr_words;
        hsA[m] = load_h16_pack<GPS>(ms + wA);
        hsB[m] = load_h16_pack<GPS>(ms + wB);
        hbA[m] = load_h16_pack<GPS>(mb + wA);
        hbB[m] = load_h16_pack<GPS>(mb + wB);
      }
#pragma unroll
      for (int G = 0; G < GPS; ++G) {
        const uint4 blk[2] = {*reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t) ^ g) << 4)),
                              *reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t + 1) ^ g) << 4))};
        const uint4 blk2[2] = {*reinterpret_cast<const uint4*>(act2 + G * S::ACT_GROUP + (((2 * t) ^ g) << 4)),
                               *reinterpret_cast<const uint4*>(act2 + G * S::ACT_GROUP + (((2 * t + 1) ^ g) << 4))};
#pragma unroll
        for (int m = 0; m < S::NMAT; ++m) {
          const float sA = h16_to_f32(h16_at<GPS>(hsA[m], G)), sB = h16_to_f32(h16_at<GPS>(hsB[m], G));
          qmv_group_regs<BITS>(cwd[m][G], blk, blk2, true, sA, sB, fmaf(-kQ, sA, h16_to_f32(h16_at<GPS>(hbA[m], G))),
                               fmaf(-kQ, sB, h16_to_f32(h16_at<GPS>(hbB[m], G))), xa[G], xb[G], xc[G], xd[G], y[m],
                               y2[m]);
        }
      }
    } else {
#pragma unroll
      for (int G = 0; G < GPS; ++G) {
        if (G < gvalid) {
          const uint4 blk[2] = {*reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t) ^ g) << 4)),
                                *reinterpret_cast<const uint4*>(act + G * S::ACT_GROUP + (((2 * t + 1) ^ g) << 4))};
          uint4 blk2[2] = {zero4, zero4};
          float x2 = 0.0f, x3 = 0.0f;
          if (two) {
            blk2[0] = *reinterpret_cast<const uint4*>(act2 + G * S::ACT_GROUP + (((2 * t) ^ g) << 4));
            blk2[1] = *reinterpret_cast<const uint4*>(act2 + G * S::ACT_GROUP + (((2 * t + 1) ^ g) << 4));
            x2 = s_xs[(kTokChunk + 2 * t) * geo.xp + gc + G];
            x3 = s_xs[(kTokChunk + 2 * t + 1) * geo.xp + gc + G];
          }
          const float x0 = s_xs[(2 * t) * geo.xp + gc + G], x1 = s_xs[(2 * t + 1) * geo.xp + gc + G];
          const int wA = sb_word(geo.chunked, rA, gc + G, geo.row_len);
          const int wB = sb_word(geo.chunked, rB, gc + G, geo.row_len);
#pragma unroll
          for (int m = 0; m < S::NMAT; ++m) {
            const uint16_t* ms = s_sb + (size_t)m * 2 * arr_words;
            const uint16_t* mb = ms + arr_words;
            const float sA = h16_to_f32(ms[wA]), sB = h16_to_f32(ms[wB]);
            const float bA = fmaf(-kQ, sA, h16_to_f32(mb[wA])), bB = fmaf(-kQ, sB, h16_to_f32(mb[wB]));
            qmv_group_regs<BITS>(load_group_codes<BITS>(codes + (size_t)m * kRowTile * S::ROWB, G, rA, rB, t), blk,
                                 blk2, two, sA, sB, bA, bB, x0, x1, x2, x3, y[m], y2[m]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot_i]);
    if (++slot_i == ns) {
      slot_i = 0;
      phase ^= 1u;
    }
    if (++sc == geo.spc || st == nstages - 1) {  // chunk done: its slot may be reloaded
      if (lane == 0) mbar_arrive(&sm.sb_empty[q]);
      sc = 0;
      ++cc;
    }
  }

  if constexpr (MODE == 0) {
    // h = silu(g) * u -> fp16 staging [16][64] in the activation layout, and
    // each token's sum of the 64 rounded h values (the group sum the down
    // projection folds its biases with): per thread over rows rA, rB, over the
    // 8 lane groups by shuffles, over the warps by the scale warp, which also
    // copies the tile out.  Staging and sums are double-buffered by item
    // parity; a buffer is rewritten (item + 2) only after its copy-out.
    const uint32_t hb_i = item & 1u;
    uint16_t* s_h = sm.s_h + (size_t)hb_i * kSegRows * kRowTile;
    float* s_hs = sm.hsum + (size_t)hb_i * kComputeWarps * kSegRows;
    if (item >= 2 && !mbar_wait(&sm.h_free[hb_i], ((item >> 1) - 1) & 1u, kDevErrTimeoutFull)) return false;
    float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      if (n == 1 && !two) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (i < 2) ? rA : rB;
        const int tok = n * kTokChunk + 2 * t + (i & 1);
        const float gv = n ? y2[0][i] : y[0][i], uv = n ? y2[1][i] : y[1][i];
        const float h = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
        const uint16_t hb = f32_to_h16_sat(h);
        s_h[tok * kRowTile + (r & ~7) + act_pos(r & 7, BITS)] = hb;
        part[2 * n + (i & 1)] += h16_to_f32(hb);
      }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[j] += __shfl_xor_sync(0xffffffffu, part[j], o);
    if (g == 0) {
      s_hs[cw * kSegRows + 2 * t] = part[0];
      s_hs[cw * kSegRows + 2 * t + 1] = part[1];
      s_hs[cw * kSegRows + kTokChunk + 2 * t] = part[2];
      s_hs[cw * kSegRows + kTokChunk + 2 * t + 1] = part[3];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.h_ready[hb_i]);
  } else {
    const int R = p.R;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      if (n == 1 && !two) break;
#pragma unroll
      for (int tb = 0; tb < 2; ++tb) {  // tokens 2t, 2t + 1 of n-tile n
        const int tok = n * kTokChunk + 2 * t + tb;
        if (tok >= it.nrows) continue;
        const int q = it.row0_seg + tok;
        float* yrow = p.y_out + (size_t)q * R;
        if (p.ret_rank) {  // straight into the source rank's return region
          const int rk = __ldg(p.ret_rank + q), rr = __ldg(p.ret_row + q);
          if (rk < 0 || rk >= p.ep_ranks || rr < 0 || rr >= p.ret_rows) continue;  // recorded by the receiver
          yrow = p.ret_base[rk] + (size_t)rr * R;
        }
#pragma unroll
        for (int m = 0; m < S::NMAT; ++m)
#pragma unroll
          for (int i = tb; i < 4; i += 2) {
            const int r = (i < 2) ? rA : rB;
            const int row = it.rt * S::ITEM_ROWS + m * kRowTile + r;
            yrow[row] = n ? y2[m][i] : y[m][i];
          }
      }
    }
  }
  return true;
}

template <int BITS, int MODE>
__global__ void __launch_bounds__(kQmvThreads, 2) qmv_kernel(const __grid_constant__ QmvParams p) {
  using S = QmvShape<BITS, MODE>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // the 128-byte swizzle of the stage tiles needs 1024-byte aligned stages and
  // the launch reserves no slack for aligning up: a base that is not aligned
  // ends the kernel before any shared-memory access, with an error recorded
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) ef_set_error(kDevErrSmemAlign);
    return;
  }
  uint8_t* smem = smem_raw;
  const int ns = p.n_stages, nq = p.n_slots;
  const int ng = p.K / 64;
  const int nstages = (p.K + S::KT - 1) / S::KT;
  const SbGeom geo = sb_geom<BITS, MODE>(p, nstages);
  const size_t slot_bytes = qmv_slot_bytes<BITS, MODE>(p.K, geo.chunked);
  QmvSmem sm;
  sm.stage_base = smem;
  sm.slot_base = sm.stage_base + (size_t)ns * S::STAGE_BYTES;
  sm.s_h = reinterpret_cast<uint16_t*>(sm.slot_base + (size_t)nq * slot_bytes);
  sm.hsum = reinterpret_cast<float*>(sm.s_h + (MODE == 0 ? (size_t)2 * kSegRows * kRowTile : 0));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm.hsum + (MODE == 0 ? (size_t)2 * kComputeWarps * kSegRows : 0));
  sm.full = bars;
  sm.empty = bars + ns;
  sm.sb_full = bars + 2 * ns;
  sm.sb_empty = sm.sb_full + nq;
  sm.h_ready = sm.sb_empty + nq;
  sm.h_free = sm.h_ready + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kComputeWarps);
    }
    for (int i = 0; i < nq; ++i) {
      mbar_init(&sm.sb_full[i], 1);
      mbar_init(&sm.sb_empty[i], kComputeWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.h_ready[i], kComputeWarps);
      mbar_init(&sm.h_free[i], 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the segments, activations and sums of the previous kernels
  // (no early launch of the successor: its CTAs would wait on SMs this
  // persistent grid fills)

  const int n_rt = p.R / S::ITEM_ROWS;
  const int n_work = (*p.n_seg) * n_rt;

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
      const int rowg = (shared ? 0 : it.expert) * p.R + it.rt * S::ITEM_ROWS;
      const CUtensorMap* m0 = shared ? &p.tm_sw0 : &p.tm_w0;
      // second tile: up (mode 0), or the next 64 rows of the same matrix (mode 2)
      const CUtensorMap* m1 = MODE == 2 ? m0 : (shared ? &p.tm_sw1 : &p.tm_w1);
      const int rowg1 = MODE == 2 ? rowg + kRowTile : rowg;
      for (int st = 0; st < nstages; ++st, ++fill_it) {
        const int slot = fill_it % ns;
        if (fill_it >= (uint32_t)ns && !mbar_wait(&sm.empty[slot], ((fill_it / ns) - 1) & 1u, kDevErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        uint8_t* dst = sm.stage_base + (size_t)slot * S::STAGE_BYTES;
        // partial last stage: the code box past the row end is zero-filled by TMA
        const int gv = min(S::GPS, ng - st * S::GPS);
        // the segment's rows 8..15 only when it has them (a second n-tile)
        const int n_boxes = it.nrows > kTokChunk ? 2 : 1;
        mbar_arrive_expect_tx(&sm.full[slot], S::CODE_BYTES + gv * n_boxes * S::ACT_BOX);
        const int kw = st * (S::KT * BITS / 32);
        tma_load_2d(dst, m0, kw, rowg, &sm.full[slot]);
        if (S::NMAT == 2) tma_load_2d(dst + kRowTile * S::ROWB, m1, kw, rowg1, &sm.full[slot]);
        uint8_t* adst = dst + S::CODE_BYTES;
        for (int G = 0; G < gv; ++G)
          for (int bx = 0; bx < n_boxes; ++bx)
            tma_load_2d(adst + G * S::ACT_GROUP + bx * S::ACT_BOX, &p.tm_act, st * S::KT + 64 * G,
                        it.row0_seg + bx * kTokChunk, &sm.full[slot]);
      }
    }
    // drain: wait (bounded) for the copies issued last
    for (uint32_t i = (fill_it > (uint32_t)ns ? fill_it - ns : 0); i < fill_it; ++i)
      mbar_wait(&sm.full[i % ns], (i / ns) & 1u, kDevErrTimeoutFull);
    return;
  }
  if (warp == kScaleWarp) {
    // ---------------------------------------------------- scale chunks (lane 0); mode 0: h copy-out (warp)
    const int xs_ld = sum_ld(p.K);
    const int nck = geo.chunked ? (ng + kSbChunk - 1) / kSbChunk : 1;
    const size_t arr_bytes = geo.chunked ? (size_t)kSbBox : (size_t)kRowTile * ng * 2;
    const size_t xs_off =
        geo.chunked ? (size_t)2 * S::NMAT * kSbBox : ((size_t)2 * S::NMAT * arr_bytes + 127) / 128 * 128;
    if (lane == 0 && geo.chunked)
      for (int a = 0; a < 2 * S::NMAT; ++a) prefetch_tmap(&p.tm_sc[a]);
    uint32_t item = 0, cc = 0;
    bool ok = true;
    int w = blockIdx.x;
    WorkItem nxt = w < n_work ? decode_work(p, w, n_rt) : WorkItem{0, 0, 0, 0};
    for (; w < n_work && ok; w += gridDim.x, ++item) {
      const WorkItem it = nxt;
      if (w + (int)gridDim.x < n_work) nxt = decode_work(p, w + gridDim.x, n_rt);
      const bool shared = it.expert >= p.n_experts;
      const size_t rowg = (size_t)(shared ? 0 : it.expert) * p.R + (size_t)it.rt * S::ITEM_ROWS;
      for (int ck = 0; ck < nck && ok; ++ck, ++cc) {
        const int q = (int)(cc % (uint32_t)nq);
        if (lane == 0)
          ok = cc < (uint32_t)nq || mbar_wait(&sm.sb_empty[q], ((cc / nq) - 1) & 1u, kDevErrTimeoutScales);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        // item - 2 has left its stages (the freed slot held a later chunk)
        if (MODE == 0 && ck == 0 && item >= 2) {
          ok = qmv_h_out<BITS, MODE>(p, sm, decode_work(p, w - 2 * (int)gridDim.x, n_rt), item - 2);
          if (!ok) break;
        }
        if (lane != 0) continue;
        uint8_t* slot = sm.slot_base + (size_t)q * slot_bytes;
        float* s_xs = reinterpret_cast<float*>(slot + xs_off);
        if (geo.chunked) {
          const int g0 = ck * kSbChunk;
          const int xs_n = min(kSbChunk, xs_ld - g0);  // multiple of 4
          mbar_arrive_expect_tx(&sm.sb_full[q], (uint32_t)(2 * S::NMAT * kSbBox + it.nrows * xs_n * 4));
          // arrays s, b of tile 0, then of tile 1 (mode 0: up; mode 2: the next 64 rows)
#pragma unroll
          for (int a = 0; a < 2 * S::NMAT; ++a)
            tma_load_2d(slot + (size_t)a * kSbBox, &p.tm_sc[(shared ? 4 : 0) + (MODE == 2 ? (a & 1) : a)], g0,
                        (int)rowg + (MODE == 2 ? (a >> 1) * kRowTile : 0), &sm.sb_full[q]);
          for (int tok = 0; tok < it.nrows; ++tok)
            bulk_load(s_xs + tok * kXsPitchChunk, p.act_sum + (size_t)(it.row0_seg + tok) * xs_ld + g0,
                      (uint32_t)xs_n * 4, &sm.sb_full[q]);
        } else {
          const uint32_t row_bytes = (uint32_t)(ng * 2);
          const uint32_t xs_bytes = (uint32_t)(it.nrows * xs_ld * 4);
          mbar_arrive_expect_tx(&sm.sb_full[q], S::NMAT * 2 * kRowTile * row_bytes + xs_bytes);
          const uint16_t* s0 = shared ? p.ss0 : p.s0;
          const uint16_t* b0 = shared ? p.sb0 : p.b0;
          const uint16_t* srcs[4] = {s0, b0, MODE == 2 ? s0 + (size_t)kRowTile * ng : (shared ? p.ss1 : p.s1),
                                     MODE == 2 ? b0 + (size_t)kRowTile * ng : (shared ? p.sb1 : p.b1)};
#pragma unroll
          for (int a = 0; a < 2 * S::NMAT; ++a)
            bulk_load(slot + (size_t)a * arr_bytes, srcs[a] + rowg * ng, kRowTile * row_bytes, &sm.sb_full[q]);
          bulk_load(s_xs, p.act_sum + (size_t)it.row0_seg * xs_ld, xs_bytes, &sm.sb_full[q]);
        }
      }
    }
    // the last items' h tiles
    if (MODE == 0)
      for (uint32_t e = item > 2u ? item - 2 : 0; e < item && ok; ++e)
        ok = qmv_h_out<BITS, MODE>(p, sm, decode_work(p, blockIdx.x + (int)e * (int)gridDim.x, n_rt), e);
    if (lane == 0 && cc > 0) mbar_wait(&sm.sb_full[(cc - 1) % nq], ((cc - 1) / nq) & 1u, kDevErrTimeoutScales);
    return;
  }
  // -------------------------------------------------------------- compute warps
  uint32_t fill_base = 0, item = 0, cc = 0;
  int w = blockIdx.x;
  WorkItem nxt = w < n_work ? decode_work(p, w, n_rt) : WorkItem{0, 0, 0, 0};
  for (; w < n_work; w += gridDim.x, ++item) {
    const WorkItem it = nxt;
    if (w + (int)gridDim.x < n_work) nxt = decode_work(p, w + gridDim.x, n_rt);
    if (!qmv_item<BITS, MODE>(p, it, sm, item, fill_base, cc, ns, nq)) break;
    fill_base += nstages;
  }
  if (MODE != 0 && p.ret_rank) {
    // expert-parallel return: every compute warp of the CTA has stored its
    // rows; the grid's last CTA releases the done flags (also after a failed
    // wait, recorded in the error word, so that no peer waits for a dead rank)
    asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32) : "memory");
    if (threadIdx.x == 0) {
      __threadfence_system();
      if (atomicAdd(p.ep_ctr, 1u) == gridDim.x - 1) {
        __threadfence_system();
        const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(p.ep_epoch);
        for (int r = 0; r < p.ep_ranks; ++r) st_release_sys(p.ret_flag[r], ep);
        *p.ep_ctr = 0;
      }
    }
  }
}

// Ring depth, scale slots and CTAs per SM: two CTAs per SM with >= 3 stages
// each when they fit in half of the shared memory, else one CTA with the
// deepest ring.  Scale chunks of few stages get four slots, so that a chunk's
// scales are requested several chunks before its first stage.
template <int BITS, int MODE>
static int qmv_pick(int K, bool chunked, int* ctas_per_sm, int* n_slots) {
  if (K > 16384) return 0;
  const int nstages = (K + QmvShape<BITS, MODE>::KT - 1) / QmvShape<BITS, MODE>::KT;
  const int spc = chunked ? kSbChunk / QmvShape<BITS, MODE>::GPS : nstages;
  const int nq = spc <= 4 ? 4 : 2;
  for (int q = nq; q >= 2; q -= 2) {
    *n_slots = q;
    for (int ns = 6; ns >= 3; --ns)
      if (qmv_smem_bytes<BITS, MODE>(K, ns, q, chunked) <= 113 * 1024) { *ctas_per_sm = 2; return ns; }
  }
  *n_slots = 2;
  for (int ns = 12; ns >= 2; --ns)
    if (qmv_smem_bytes<BITS, MODE>(K, ns, 2, chunked) <= 227 * 1024) { *ctas_per_sm = 1; return ns; }
  return 0;
}

template <int BITS, int MODE>
static cudaError_t launch_qmv_t(const QmvParams& p_in, int n_sm, cudaStream_t st) {
  QmvParams p = p_in;
  int per_sm = 1;
  const bool chunked = p.sb_chunked != 0;
  p.n_stages = qmv_pick<BITS, MODE>(p.K, chunked, &per_sm, &p.n_slots);
  if (p.n_stages == 0) return cudaErrorInvalidValue;
  const size_t smem = qmv_smem_bytes<BITS, MODE>(p.K, p.n_stages, p.n_slots, chunked);
  static std::atomic<bool> attr_set[64];
  if (const cudaError_t e = set_max_smem_once(qmv_kernel<BITS, MODE>, 227 * 1024, attr_set)) return e;
  return launch_pdl(qmv_kernel<BITS, MODE>, n_sm * per_sm, kQmvThreads, smem, st, p);
}

// SIZE_MAX when the decode kernel cannot hold a K-wide item in shared memory
// (whole-item scale slots: the larger of the two layouts).
size_t qmv_smem_required(int bits, int mode, int K) {
  int per = 1, nq = 2, ns;
  if (bits == 4) {
    ns = mode == 0 ? qmv_pick<4, 0>(K, false, &per, &nq) : qmv_pick<4, 1>(K, false, &per, &nq);
    if (!ns) return ~size_t(0);
    return mode == 0 ? qmv_smem_bytes<4, 0>(K, ns, nq, false) : qmv_smem_bytes<4, 1>(K, ns, nq, false);
  }
  ns = mode == 0 ? qmv_pick<8, 0>(K, false, &per, &nq) : qmv_pick<8, 1>(K, false, &per, &nq);
  if (!ns) return ~size_t(0);
  return mode == 0 ? qmv_smem_bytes<8, 0>(K, ns, nq, false) : qmv_smem_bytes<8, 1>(K, ns, nq, false);
}

// mode 1 runs as mode 2 (128-row items) when the output rows allow it and
// the segments (at least min_segments of them) give every CTA an item.
cudaError_t launch_qmv(int bits, int mode, const QmvParams& p, int n_sm, cudaStream_t st, int min_segments) {
  if (mode == 1 && p.R % (2 * kRowTile) == 0 && (long long)min_segments * (p.R / (2 * kRowTile)) >= 2LL * n_sm)
    mode = 2;
  if (bits == 4) {
    if (mode == 0) return launch_qmv_t<4, 0>(p, n_sm, st);
    return mode == 2 ? launch_qmv_t<4, 2>(p, n_sm, st) : launch_qmv_t<4, 1>(p, n_sm, st);
  }
  if (mode == 0) return launch_qmv_t<8, 0>(p, n_sm, st);
  return mode == 2 ? launch_qmv_t<8, 2>(p, n_sm, st) : launch_qmv_t<8, 1>(p, n_sm, st);
}

}  // namespace ef
