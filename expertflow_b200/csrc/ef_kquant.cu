// ef_kquant.cu -- GGUF K-quant blocks (Q2_K, Q3_K, Q4_K): decode to fp16 and
// the decode GEMV y = x . W^T over rows stored as such blocks.
//
// Formats, as the reference's decoders read them (256 elements per block;
// value = RN16(d*sc*q - dmin*mn) with the products exact in fp32):
//   Q2_K  84 B: scales[16] @0 (sc = lo nibble, mn = hi nibble of group i/16),
//               qs[64] @16 (element i: bits 2(i%4) of byte i/4), d @80, dmin @82
//               (ef_deepseek_mmap.py:330-378)
//   Q3_K 110 B: hmask[32] @0, qs[64] @32, scales[12] @96, d @108; element
//               i = 128h + 32s + b: q = ((qs[32h+b] >> 2s) & 3) - 4 (hmask bit
//               4h+s of byte b clear); 6-bit group scale (low nibble of byte
//               g%8, >> 4 for g >= 8; high 2 bits from byte 8 + g%4, shifted
//               2(g/4)) minus 32 (ef_deepseek_mmap.py:717-773)
//   Q4_K 144 B: d @0, dmin @2, scales[12] @4, qs[128] @16; elements 0..127 the
//               low nibbles, 128..255 the high nibbles; sub-block j = i/32:
//               sc = s[j] & 63, mn = s[8+j] & 63 (j < 4) or
//               (s[j-4] >> 6) | ((s[j+4] >> 2) & 0x30) (ef_deepseek_mmap.py:655-714)
// Every product d*sc*q and dmin*mn fits in fp32's 24-bit significand, so one
// fused multiply-add gives exactly the reference's RN32(d*sc*q - dmin*mn); the
// fp16 conversion rounds to nearest-even as numpy's astype does.
//
// GEMV (decode): mma.sync m16n8k16 with fp32 accumulation.  A warp owns 16
// rows; lane (g = lane/4, c = lane%4) decodes rows g and g+8 straight into its
// A fragments.  Q2_K and Q3_K fragments are the reference's fp16 weights
// (RN16 of the exact value); Q4_K codes go into the MMA exactly, as the fp16
// values 1024 + q (one LOP3 per pair), each MMA's 16 reduction indices inside
// one 32-element sub-block, and the sub-block's scale and min are folded in
// fp32 afterwards:  y += A D - (1024 A + B) X,  D = sum (1024 + q) x,  X = sum x
// (A = d sc, B = dmin mn), which is sum (A q - B) x without the fp16 rounding of
// each weight.  Within each 256-element block the reduction index is permuted
// so that lane c's 64 elements of a row sit in whole code words of the block
// (the order depends on the format); the activations are permuted the same
// way by kquant_prep_kernel, so every MMA pairs matching weights and inputs.
// Permuted activations: xp[token][256 kb + 8 (4 q + c) + r] holds
// x[token][256 kb + elem(c, 2q + r/4, r%4)], so lane c reads 16 bytes per two
// MMAs.  Warps of a CTA share one 16-row tile when the matrix is too small to
// fill the GPU (split over the blocks of K, reduced through shared memory in
// a fixed order, so results do not depend on timing).

namespace ef {

constexpr int kKqQ2 = 10, kKqQ3 = 11, kKqQ4 = 12;
constexpr int kKqWarps = 8;  // warps per GEMV CTA

__host__ __device__ constexpr int kq_block_bytes(int type) {
  return type == kKqQ2 ? 84 : type == kKqQ3 ? 110 : 144;
}

// Element (0..255) of a block that lane c's slot t (0..3) of MMA j (0..15) carries.
__host__ __device__ inline int kq_elem(int type, int c, int j, int t) {
  if (type == kKqQ2) return 64 * c + 16 * (j >> 2) + (j & 3) + 4 * t;
  if (type == kKqQ3) {
    const int h = j >> 3, s = (j >> 1) & 3, u = j & 1;
    return 128 * h + 32 * s + 8 * c + 4 * u + t;
  }
  // Q4_K: MMA j = 4J + 2h + u takes the low (h = 0: sub-block J) or high
  // (h = 1: sub-block 4 + J) nibbles of qs word 32J + 8c + 4u; slots t0, t1
  // are its bytes 0 and 2, t2, t3 its bytes 1 and 3
  const int J = j >> 2, h = (j >> 1) & 1, u = j & 1;
  return 32 * (J + 4 * h) + 8 * c + 4 * u + ((t & 1) << 1) + (t >> 1);
}

EF_DEV float kq_f16(const uint8_t* p) {  // fp16 field (2-byte aligned)
  return __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(p)));
}
EF_DEV float code_f32(uint32_t q) {  // exact float of a small unsigned code
  return __uint_as_float(0x4B000000u | q) - 8388608.0f;
}
// 32-bit word at a 2-byte aligned address (two aligned loads + funnel shift).
EF_DEV uint32_t ld_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  if ((a & 3) == 0) return __ldg(w);
  return __funnelshift_r(__ldg(w), __ldg(w + 1), 16);
}
EF_DEV uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One row's data for lane c of one block, and its per-MMA fp16 pairs.
template <int TYPE>
struct KqRow;

template <>
struct KqRow<kKqQ2> {
  uint32_t qw[4];  // qs bytes 16c .. 16c+15: word w is group 4c + w (element 16w' + e at bits 2e)
  uint32_t sc;     // scale bytes 4c .. 4c+3
  uint32_t dd;     // d | dmin << 16
  EF_DEV void load(const uint8_t* blk, int c) {
    const uint32_t* q = reinterpret_cast<const uint32_t*>(blk + 16 + 16 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) qw[i] = __ldg(q + i);
    sc = __ldg(reinterpret_cast<const uint32_t*>(blk + 4 * c));
    dd = __ldg(reinterpret_cast<const uint32_t*>(blk + 80));
  }
  EF_DEV void prep(int) {}
  // A group takes only four values, RN16(A q - B) for q = 0..3 (exactly the
  // reference's rounding); they sit as halves 0..3 of (L01, L23) and each
  // pair of codes selects its two halves with one byte permute.  MMA
  // j = 4W + m carries the group's elements m, m+4 (t0, t1) and m+8, m+12 (t2, t3).
  template <int W>
  EF_DEV void frags(int, uint32_t (&lo)[4], uint32_t (&hi)[4]) const {
    const float d = __half2float(__ushort_as_half((uint16_t)dd));
    const float m = __half2float(__ushort_as_half((uint16_t)(dd >> 16)));
    const uint32_t s = (sc >> (8 * W)) & 0xffu;
    const float A = d * (float)(s & 15u), B = m * (float)(s >> 4);
    const uint32_t L01 = pack_h2(fmaf(A, 0.0f, -B), fmaf(A, 1.0f, -B));
    const uint32_t L23 = pack_h2(fmaf(A, 2.0f, -B), fmaf(A, 3.0f, -B));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t r4 = (qw[W] >> (2 * e)) & 0x03030303u;  // codes of elements e, e+4, e+8, e+12
      const uint32_t S = r4 * 0x22u + 0x10101010u;           // byte pair (2q, 2q+1) per code
      lo[e] = prmt(L01, L23, S);
      hi[e] = prmt(L01, L23, S >> 16);
    }
  }
};

template <>
struct KqRow<kKqQ3> {
  uint32_t qw[4];  // [2h + u]: qs bytes 32h + 8c + 4u .. +3
  uint32_t hw[2];  // [u]: hmask bytes 8c + 4u .. +3
  float A[8];      // [2h + s/... ] scale of group 8h + 2s + c/2, times d: index 4h + s
  EF_DEV void load(const uint8_t* blk, int c) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int u = 0; u < 2; ++u) qw[2 * h + u] = ld_u32_a2(blk + 32 + 32 * h + 8 * c + 4 * u);
    hw[0] = ld_u32_a2(blk + 8 * c);
    hw[1] = ld_u32_a2(blk + 8 * c + 4);
    const uint32_t s0 = ld_u32_a2(blk + 96), s1 = ld_u32_a2(blk + 100), s2 = ld_u32_a2(blk + 104);
    const float d = kq_f16(blk + 108);
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int g = 8 * h + 2 * s + (c >> 1);
        const int lb = g & 7;
        const uint32_t lw = lb < 4 ? s0 : s1;
        const uint32_t lo = ((lw >> (8 * (lb & 3))) >> (g >= 8 ? 4 : 0)) & 15u;
        const uint32_t hi = ((s2 >> (8 * (g & 3))) >> (2 * (g >> 2))) & 3u;
        A[4 * h + s] = d * ((float)(lo | (hi << 4)) - 32.0f);
      }
  }
  EF_DEV void prep(int) {}
  // MMAs j = 4QQ .. 4QQ+3.  A group takes eight values, a (u - 4) for
  // u = q + 4 in 0..7 (exact products, then RN16): halves 0..3 of (L0, L1)
  // for the codes whose hmask bit is clear, of (L2, L3) for those with it
  // set.  Each pair of 2-bit codes selects from both tables with one byte
  // permute each; the hmask bits, moved to the top of their bytes, become a
  // per-half mask (sign-replicating permute) that picks between the two.
  template <int QQ>
  EF_DEV void frags(int, uint32_t (&lo)[4], uint32_t (&hi)[4]) const {
    constexpr int H = QQ >> 1;
#pragma unroll
    for (int sp = 0; sp < 2; ++sp) {
      const int s = 2 * (QQ & 1) + sp;
      const float a = A[4 * H + s];
      const uint32_t L0 = pack_h2(a * -4.0f, a * -3.0f), L1 = pack_h2(a * -2.0f, a * -1.0f);
      const uint32_t L2 = pack_h2(a * 0.0f, a), L3 = pack_h2(a * 2.0f, a * 3.0f);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j4 = 2 * sp + u;
        const uint32_t r4 = (qw[2 * H + u] >> (2 * s)) & 0x03030303u;  // 2-bit codes of bytes 0..3
        const uint32_t S = r4 * 0x22u + 0x10101010u;
        const uint32_t hs = hw[u] << (7 - (4 * H + s));               // hmask bit -> bit 7 of its byte
        const uint32_t m01 = prmt(hs, 0u, 0x9988u), m23 = prmt(hs, 0u, 0xBBAAu);
        const uint32_t lo_n = prmt(L0, L1, S), lo_p = prmt(L2, L3, S);
        const uint32_t hi_n = prmt(L0, L1, S >> 16), hi_p = prmt(L2, L3, S >> 16);
        lo[j4] = (lo_n & ~m01) | (lo_p & m01);
        hi[j4] = (hi_n & ~m23) | (hi_p & m23);
      }
    }
  }
};

template <>
struct KqRow<kKqQ4> {
  uint2 qw[4];     // [J]: qs bytes 32J + 8c .. 32J + 8c + 7
  uint32_t s[3];   // scales[12]
  uint32_t dd;     // d | dmin << 16
  float A[2], C[2];  // after prep(): sub-blocks 2c, 2c + 1: A = d sc, C = 1024 A + dmin mn
  EF_DEV void load(const uint8_t* blk, int c) {
#pragma unroll
    for (int J = 0; J < 4; ++J) qw[J] = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 32 * J + 8 * c));
    const uint32_t* w = reinterpret_cast<const uint32_t*>(blk);
    dd = __ldg(w);
    s[0] = __ldg(w + 1);
    s[1] = __ldg(w + 2);
    s[2] = __ldg(w + 3);
  }
  // the same words from a block staged in shared memory
  EF_DEV void load_shared(const uint8_t* blk, int c) {
#pragma unroll
    for (int J = 0; J < 4; ++J) qw[J] = *reinterpret_cast<const uint2*>(blk + 16 + 32 * J + 8 * c);
    const uint4 h = *reinterpret_cast<const uint4*>(blk);
    dd = h.x;
    s[0] = h.y;
    s[1] = h.z;
    s[2] = h.w;
  }
  // byte i of scales[12] (i is lane-dependent: selects, not an indexed load,
  // keep the words in registers)
  EF_DEV uint32_t sbyte(int i) const {
    const uint32_t w = i < 4 ? s[0] : (i < 8 ? s[1] : s[2]);
    return (w >> (8 * (i & 3))) & 0xffu;
  }
  // sub-block j: sc = s[j] & 63; mn = s[8 + j] & 63 (j < 4), else
  // (s[j - 4] >> 6) | ((s[j + 4] >> 2) & 0x30) (the reference's decode)
  EF_DEV void prep(int c) {
    const float d = __half2float(__ushort_as_half((uint16_t)dd));
    const float m = __half2float(__ushort_as_half((uint16_t)(dd >> 16)));
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = 2 * c + i;
      const uint32_t sc = sbyte(j) & 63u;
      const uint32_t mn = j < 4 ? (sbyte(8 + j) & 63u) : ((sbyte(j - 4) >> 6) | ((sbyte(j + 4) >> 2) & 0x30u));
      A[i] = d * (float)sc;
      C[i] = fmaf(1024.0f, A[i], m * (float)mn);
    }
  }
};

// Permute and convert the activations: xp fp16 [n_tok8][K] (tokens >= T zero);
// Q4_K also the sums of each 32-element sub-block of the rounded values, xs
// fp32 [n_tok8][K / 32], in element order.
template <int TYPE>
__global__ void kquant_prep_kernel(const uint16_t* __restrict__ x, int act_bf16, int T, int K, int n_tok8,
                                   uint16_t* __restrict__ xp, float* __restrict__ xs) {
  const long long total = (long long)n_tok8 * K;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int tok = (int)(i / K), kk = (int)(i % K);
    const int kb = kk >> 8, p = kk & 255;
    const int q = p >> 5, c = (p >> 3) & 3, r = p & 7;
    const int src = 256 * kb + kq_elem(TYPE, c, 2 * q + (r >> 2), r & 3);
    uint16_t out = 0;
    if (tok < T) {
      const float v = act_to_f32(x[(size_t)tok * K + src], act_bf16);
      if (!(fabsf(v) <= 65504.0f)) ef_set_error(kDevErrRange);
      out = __half_as_ushort(__float2half_rn(v));
    }
    xp[i] = out;
  }
  if (TYPE == kKqQ4) {
    const int nsb = K >> 5;
    const long long tsum = (long long)n_tok8 * nsb;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < tsum;
         i += (long long)gridDim.x * blockDim.x) {
      const int tok = (int)(i / nsb), sb = (int)(i % nsb);
      float sum = 0.0f;
      if (tok < T)
        for (int e = 0; e < 32; ++e)
          sum += __half2float(__float2half_rn(act_to_f32(x[(size_t)tok * K + 32 * sb + e], act_bf16)));
      xs[i] = sum;
    }
  }
}

// One lane's contribution of one block for one 16-row tile: per quarter of
// the block, decode 4 MMAs' fragments of both rows, then run them for every
// token group.
template <int TYPE, int NT, int QQ>
EF_DEV void kq_quarter_mma(const KqRow<TYPE>& r0, const KqRow<TYPE>& r1, int c, const uint16_t* __restrict__ xrow,
                           const size_t (&tok_off)[NT], float (&acc)[NT][4]) {
  uint32_t a0l[4], a0h[4], a1l[4], a1h[4];
  r0.template frags<QQ>(c, a0l, a0h);
  r1.template frags<QQ>(c, a1l, a1h);
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const uint16_t* xr = xrow + tok_off[n] + 64 * QQ;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(xr + 32 * h));
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        const int j = 2 * h + v;
        const uint32_t a[4] = {a0l[j], a1l[j], a0h[j], a1h[j]};
        mma_16816(acc[n], a, v ? b.z : b.x, v ? b.w : b.y);
      }
    }
  }
}

template <int TYPE, int NT>
EF_DEV void kq_block_mma(KqRow<TYPE>& r0, KqRow<TYPE>& r1, int c, const uint16_t* __restrict__ xrow,
                         const size_t (&tok_off)[NT], float (&acc)[NT][4]) {
  // xrow: column 256 kb + 8 c of the permuted activations; tok_off[n]: this
  // lane's token row of token group n
  r0.prep(c);
  r1.prep(c);
  kq_quarter_mma<TYPE, NT, 0>(r0, r1, c, xrow, tok_off, acc);
  kq_quarter_mma<TYPE, NT, 1>(r0, r1, c, xrow, tok_off, acc);
  kq_quarter_mma<TYPE, NT, 2>(r0, r1, c, xrow, tok_off, acc);
  kq_quarter_mma<TYPE, NT, 3>(r0, r1, c, xrow, tok_off, acc);
}

// Q4_K: one block of both rows.  Per sub-block: two MMAs on the exact codes
// into a fresh accumulator, then the fold with the sub-block's A and C of each
// row (decoded by the quad's lane that owns the sub-block, passed by shuffle)
// and the tokens' sub-block sums.  xs_blk: the sums of this block (xs + 8 kb);
// xs_off[n][i]: the row offset of token 8n + 2c + i in xs.
template <int NT>
EF_DEV void kq_block_q4(KqRow<kKqQ4>& r0, KqRow<kKqQ4>& r1, int c, const uint16_t* __restrict__ xrow,
                        const size_t (&tok_off)[NT], const float* __restrict__ xs_blk,
                        const size_t (&xs_off)[NT][2], float (&acc)[NT][4]) {
  r0.prep(c);
  r1.prep(c);
  const int qbase = (threadIdx.x & 31) & ~3;
#pragma unroll
  for (int J = 0; J < 4; ++J)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int sb = J + 4 * h;
      uint32_t a[2][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t w0 = u ? r0.qw[J].y : r0.qw[J].x, w1 = u ? r1.qw[J].y : r1.qw[J].x;
        a[u][0] = lop3_and_or(w0 >> (4 * h), 0x000F000Fu, 0x64006400u);
        a[u][1] = lop3_and_or(w1 >> (4 * h), 0x000F000Fu, 0x64006400u);
        a[u][2] = lop3_and_or(w0 >> (8 + 4 * h), 0x000F000Fu, 0x64006400u);
        a[u][3] = lop3_and_or(w1 >> (8 + 4 * h), 0x000F000Fu, 0x64006400u);
      }
      const int src = qbase + (sb >> 1);
      const float A0 = __shfl_sync(0xffffffffu, r0.A[sb & 1], src);
      const float C0 = __shfl_sync(0xffffffffu, r0.C[sb & 1], src);
      const float A1 = __shfl_sync(0xffffffffu, r1.A[sb & 1], src);
      const float C1 = __shfl_sync(0xffffffffu, r1.C[sb & 1], src);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(xrow + tok_off[n] + 64 * J + 32 * h));
        float D[4] = {0.f, 0.f, 0.f, 0.f};
        mma_16816(D, a[0], b.x, b.y);
        mma_16816(D, a[1], b.z, b.w);
        const float X0 = __ldg(xs_blk + xs_off[n][0] + sb), X1 = __ldg(xs_blk + xs_off[n][1] + sb);
        acc[n][0] = fmaf(A0, D[0], fmaf(-C0, X0, acc[n][0]));
        acc[n][1] = fmaf(A0, D[1], fmaf(-C0, X1, acc[n][1]));
        acc[n][2] = fmaf(A1, D[2], fmaf(-C1, X0, acc[n][2]));
        acc[n][3] = fmaf(A1, D[3], fmaf(-C1, X1, acc[n][3]));
      }
    }
}

// Blocks in flight per warp (register ring depth).  Deeper rings cost
// occupancy and measured slower.
constexpr int kKqDepth = 2;

// y [T, N] fp32.  Grid: ceil(n_tiles / tiles_per_cta) CTAs of kKqWarps warps;
// `split` warps share a tile (each a contiguous range of blocks).
template <int TYPE, int NT>
__global__ void __launch_bounds__(kKqWarps * 32, (NT == 1 && TYPE == kKqQ2) ? 3 : 2) kquant_gemv_kernel(const uint8_t* __restrict__ w,
                                                                   const uint16_t* __restrict__ xp,
                                                                   const float* __restrict__ xs, int T, int N,
                                                                   int K, int split, float* __restrict__ y) {
  constexpr int BB = kq_block_bytes(TYPE);
  __shared__ float red[kKqWarps][32][NT * 4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tiles_per_cta = kKqWarps / split;
  const int tile = blockIdx.x * tiles_per_cta + warp / split;
  const int part = warp % split;
  const int nb = K >> 8;
  const int n_tiles = N >> 4;
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
  if (tile < n_tiles) {
    const int kb0 = (int)((long long)nb * part / split), kb1 = (int)((long long)nb * (part + 1) / split);
    const size_t row_bytes = (size_t)nb * BB;
    const uint8_t* row0 = w + (size_t)(16 * tile + g) * row_bytes;
    const uint8_t* row1 = row0 + 8 * row_bytes;
    const size_t tok_stride = (size_t)K;
    const uint16_t* xl = xp + 8 * c;
    // token rows past T hold zeros: every lane whose token is one of them
    // reads row T, so those loads collapse into one broadcast per warp
    size_t tok_off[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) tok_off[n] = (size_t)(8 * n + g < T ? 8 * n + g : T) * tok_stride;
    // Q4_K sub-block sums of the accumulator's tokens 8n + 2c, 8n + 2c + 1
    // (rows past T hold zeros)
    size_t xs_off[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 2; ++i) xs_off[n][i] = (size_t)(8 * n + 2 * c + i) * (size_t)(K >> 5);
    // ring of D blocks in flight per warp: the load of block kb + D is issued
    // as soon as block kb has been consumed
    constexpr int D = kKqDepth;
    KqRow<TYPE> b0[D], b1[D];
#pragma unroll
    for (int i = 0; i < D; ++i)
      if (kb0 + i < kb1) {
        b0[i].load(row0 + (size_t)(kb0 + i) * BB, c);
        b1[i].load(row1 + (size_t)(kb0 + i) * BB, c);
      }
    for (int kb = kb0; kb < kb1; kb += D) {
#pragma unroll
      for (int i = 0; i < D; ++i) {
        if (kb + i < kb1) {
          if constexpr (TYPE == kKqQ4)
            kq_block_q4<NT>(b0[i], b1[i], c, xl + (size_t)(kb + i) * 256, tok_off, xs + (size_t)(kb + i) * 8, xs_off,
                            acc);
          else
            kq_block_mma<TYPE, NT>(b0[i], b1[i], c, xl + (size_t)(kb + i) * 256, tok_off, acc);
          if (kb + i + D < kb1) {
            b0[i].load(row0 + (size_t)(kb + i + D) * BB, c);
            b1[i].load(row1 + (size_t)(kb + i + D) * BB, c);
          }
        }
      }
    }
  }
  if (split > 1) {
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][lane][4 * n + i] = acc[n][i];
    __syncthreads();
    if (part != 0) return;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float sum = 0.0f;
        for (int p = 0; p < split; ++p) sum += red[warp + p][lane][4 * n + i];
        acc[n][i] = sum;
      }
  }
  if (tile >= n_tiles) return;
  // accumulator (row g / g+8, tokens 2c, 2c+1 of each group of 8)
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = 8 * n + 2 * c + (i & 1);
      const int row = 16 * tile + g + ((i & 2) ? 8 : 0);
      if (tok < T) y[(size_t)tok * N + row] = acc[n][i];
    }
}

// Q4_K GEMV fed through shared memory: each warp streams its tile's 16 rows
// through a private ring of kKq4Stages stages of kKq4SB blocks per row (one
// bulk copy per row per stage, completion on the stage's mbarrier), so a warp
// has up to kKq4Stages * 16 * kKq4SB * 144 bytes in flight and its lanes read
// the staged words from shared memory (two CTAs per SM).  Same tiles, split
// and reduction as kquant_gemv_kernel; every wait is bounded and after a
// failed one the warp waits (bounded) for the copies it has issued.
constexpr int kKq4Stages = 2;
constexpr int kKq4SB = 2;
constexpr int kKq4RowBytes = kKq4SB * 144;               // one row's share of a stage
constexpr int kKq4StageBytes = 16 * kKq4RowBytes;         // a stage of the warp's 16 rows
constexpr int kKq4WarpBytes = kKq4Stages * kKq4StageBytes;

template <int NT>
__global__ void __launch_bounds__(kKqWarps * 32, 2) kq4_bulk_gemv_kernel(const uint8_t* __restrict__ w,
                                                                         const uint16_t* __restrict__ xp,
                                                                         const float* __restrict__ xs, int T, int N,
                                                                         int K, int split, float* __restrict__ y) {
  extern __shared__ __align__(128) uint8_t kq4_smem[];
  __shared__ __align__(8) uint64_t bars[kKqWarps][kKq4Stages];
  __shared__ float red[kKqWarps][32][NT * 4];
  constexpr int BB = 144;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int tiles_per_cta = kKqWarps / split;
  const int tile = blockIdx.x * tiles_per_cta + warp / split;
  const int part = warp % split;
  const int nb = K >> 8;
  const int n_tiles = N >> 4;
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
  if (tile < n_tiles) {
    const int kb0 = (int)((long long)nb * part / split), kb1 = (int)((long long)nb * (part + 1) / split);
    const size_t row_bytes = (size_t)nb * BB;
    const uint8_t* rows = w + (size_t)(16 * tile) * row_bytes;  // the tile's first row
    uint8_t* ring = kq4_smem + (size_t)warp * kKq4WarpBytes;
    uint64_t* bar = bars[warp];
    if (lane == 0) {
      for (int i = 0; i < kKq4Stages; ++i) mbar_init(&bar[i], 1);
      mbar_fence_init();
    }
    __syncwarp();
    // stage st covers blocks [kb0 + st * SB, + SB) of every row
    const int n_st = (kb1 - kb0 + kKq4SB - 1) / kKq4SB;
    auto issue = [&](int st) {
      const int kb = kb0 + st * kKq4SB, nblk = min(kKq4SB, kb1 - kb);
      uint64_t* b = &bar[st % kKq4Stages];
      uint8_t* dst = ring + (size_t)(st % kKq4Stages) * kKq4StageBytes;
      mbar_arrive_expect_tx(b, (uint32_t)(16 * nblk * BB));
      for (int r = 0; r < 16; ++r)
        bulk_load(dst + r * kKq4RowBytes, rows + (size_t)r * row_bytes + (size_t)kb * BB, (uint32_t)(nblk * BB), b);
    };
    if (lane == 0)
      for (int st = 0; st < min(kKq4Stages, n_st); ++st) issue(st);
    const uint16_t* xl = xp + 8 * c;
    size_t tok_off[NT];
#pragma unroll
    for (int n = 0; n < NT; ++n) tok_off[n] = (size_t)(8 * n + g < T ? 8 * n + g : T) * (size_t)K;
    size_t xs_off[NT][2];
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 2; ++i) xs_off[n][i] = (size_t)(8 * n + 2 * c + i) * (size_t)(K >> 5);
    int st = 0;
    bool ok = true;
    for (; st < n_st; ++st) {
      if (!mbar_wait(&bar[st % kKq4Stages], (uint32_t)(st / kKq4Stages) & 1u, kDevErrTimeoutFull)) {
        ok = false;
        break;
      }
      const uint8_t* stage = ring + (size_t)(st % kKq4Stages) * kKq4StageBytes;
      const int kb = kb0 + st * kKq4SB, nblk = min(kKq4SB, kb1 - kb);
#pragma unroll
      for (int i = 0; i < kKq4SB; ++i) {
        if (i < nblk) {
          KqRow<kKqQ4> r0, r1;
          r0.load_shared(stage + g * kKq4RowBytes + i * BB, c);
          r1.load_shared(stage + (g + 8) * kKq4RowBytes + i * BB, c);
          kq_block_q4<NT>(r0, r1, c, xl + (size_t)(kb + i) * 256, tok_off, xs + (size_t)(kb + i) * 8, xs_off, acc);
        }
      }
      __syncwarp();
      if (lane == 0 && st + kKq4Stages < n_st) {
        fence_proxy_async();  // this stage's shared-memory reads before the copy that overwrites it
        issue(st + kKq4Stages);
      }
    }
    if (!ok && lane == 0)  // stages issued but not consumed: wait (bounded) for their copies before leaving
      for (int d = st; d < min(n_st, st + kKq4Stages); ++d)
        mbar_wait(&bar[d % kKq4Stages], (uint32_t)(d / kKq4Stages) & 1u, kDevErrTimeoutFull);
  }
  if (split > 1) {
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][lane][4 * n + i] = acc[n][i];
    __syncthreads();
    if (part != 0) return;
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float sum = 0.0f;
        for (int q = 0; q < split; ++q) sum += red[warp + q][lane][4 * n + i];
        acc[n][i] = sum;
      }
  }
  if (tile >= n_tiles) return;
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = 8 * n + 2 * c + (i & 1);
      const int row = 16 * tile + g + ((i & 2) ? 8 : 0);
      if (tok < T) y[(size_t)tok * N + row] = acc[n][i];
    }
}

// fp16 out[n_blocks * 256]: the reference's decode, one thread per 16 elements.
template <int TYPE>
__global__ void kquant_dequant_kernel(const uint8_t* __restrict__ blocks, long long n_blocks,
                                      uint16_t* __restrict__ out) {
  constexpr int BB = kq_block_bytes(TYPE);
  const long long n16 = n_blocks * 16;
  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < n16;
       u += (long long)gridDim.x * blockDim.x) {
    const uint8_t* b = blocks + (u >> 4) * BB;
    const int e0 = (int)(u & 15) * 16;  // elements e0 .. e0+15 of the block
    float v[16];
    if (TYPE == kKqQ2) {
      const int grp = e0 >> 4;
      const float A = kq_f16(b + 80) * (float)(b[grp] & 15), B = kq_f16(b + 82) * (float)(b[grp] >> 4);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = fmaf(A, (float)((b[16 + ((e0 + i) >> 2)] >> (2 * ((e0 + i) & 3))) & 3), -B);
    } else if (TYPE == kKqQ3) {
      const int grp = e0 >> 4;
      const uint32_t lo = (grp < 8 ? b[96 + grp] : (b[96 + grp - 8] >> 4)) & 15u;
      const uint32_t hi = (b[104 + (grp & 3)] >> (2 * (grp >> 2))) & 3u;
      const float A = kq_f16(b + 108) * ((float)(lo | (hi << 4)) - 32.0f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int e = e0 + i, h = e >> 7, s = (e >> 5) & 3, bb = e & 31;
        const int q = (int)((b[32 + 32 * h + bb] >> (2 * s)) & 3) - (((b[bb] >> (4 * h + s)) & 1) ? 0 : 4);
        v[i] = fmaf(A, (float)q, -0.0f);
      }
    } else {
      const int e = e0 & 127, j = (e0 >> 7) * 4 + (e >> 5);  // sub-block of these 16 elements
      const uint8_t* s = b + 4;
      const uint32_t sc = s[j] & 63u;
      const uint32_t mn = j < 4 ? (s[8 + j] & 63u) : (uint32_t)((s[j - 4] >> 6) | ((s[j + 4] >> 2) & 0x30));
      const float A = kq_f16(b) * (float)sc, B = kq_f16(b + 2) * (float)mn;
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = fmaf(A, (float)((b[16 + e + i] >> (e0 >= 128 ? 4 : 0)) & 15), -B);
    }
    uint4 o[2];
    uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) ow[i] = pack_h2(v[2 * i], v[2 * i + 1]);
    uint4* dst = reinterpret_cast<uint4*>(out + u * 16);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

template <int TYPE>
cudaError_t launch_kquant_gemv_t(const uint8_t* w, const uint16_t* xp, const float* xs, int T, int N, int K,
                                 int split, float* y, cudaStream_t st) {
  const int n_tiles = N >> 4, tiles_per_cta = kKqWarps / split;
  const int grid = (n_tiles + tiles_per_cta - 1) / tiles_per_cta;
  const int nt = (T + 7) / 8;
  if constexpr (TYPE == kKqQ4) {
    // up to 16 tokens through shared memory; 17..32 (four token groups) in
    // registers (the shared-memory kernel spills there and measured slower)
    if (nt <= 2) {
      constexpr int smem = kKqWarps * kKq4WarpBytes;
      static std::atomic<bool> a1[64], a2[64];
      cudaError_t e;
      if (nt == 1) {
        if ((e = set_max_smem_once(kq4_bulk_gemv_kernel<1>, smem, a1))) return e;
        kq4_bulk_gemv_kernel<1><<<grid, kKqWarps * 32, smem, st>>>(w, xp, xs, T, N, K, split, y);
      } else {
        if ((e = set_max_smem_once(kq4_bulk_gemv_kernel<2>, smem, a2))) return e;
        kq4_bulk_gemv_kernel<2><<<grid, kKqWarps * 32, smem, st>>>(w, xp, xs, T, N, K, split, y);
      }
      return cudaGetLastError();
    }
  }
  if (nt == 1) kquant_gemv_kernel<TYPE, 1><<<grid, kKqWarps * 32, 0, st>>>(w, xp, xs, T, N, K, split, y);
  else if (nt == 2) kquant_gemv_kernel<TYPE, 2><<<grid, kKqWarps * 32, 0, st>>>(w, xp, xs, T, N, K, split, y);
  else kquant_gemv_kernel<TYPE, 4><<<grid, kKqWarps * 32, 0, st>>>(w, xp, xs, T, N, K, split, y);
  return cudaGetLastError();
}

}  // namespace ef

namespace {

int kq_split(int N, int K, int n_sm) {
  // warps sharing a tile: enough (tile, block range) units for about four
  // waves of resident warps, so the last wave's tail stays short
  const int n_tiles = N >> 4, nb = K >> 8;
  int split = 1;
  while (split < ef::kKqWarps && (long long)n_tiles * split < 96LL * n_sm && split * 2 <= nb) split *= 2;
  return split;
}

// Q4_K up to 16 tokens (shared-memory kernel, two CTAs of kKqWarps warps per
// SM): warps share a tile only while the tiles give fewer than one wave of
// resident warps, so each warp streams long row ranges through its ring.
int kq4_split(int N, int K, int n_sm) {
  const int n_tiles = N >> 4, nb = K >> 8;
  int split = 1;
  while (split < ef::kKqWarps && (long long)n_tiles * split < 2LL * ef::kKqWarps * n_sm && split * 2 <= nb) split *= 2;
  return split;
}

ef_status check_kquant(int type, int N, int K) {
  if (type != ef::kKqQ2 && type != ef::kKqQ3 && type != ef::kKqQ4)
    return fail(EF_ERR_UNSUPPORTED, "K-quant type must be Q2_K (10), Q3_K (11) or Q4_K (12), got %d", type);
  if (N <= 0 || N % 16) return fail(EF_ERR_UNSUPPORTED, "N must be a positive multiple of 16 (got %d)", N);
  if (K <= 0 || K % 256) return fail(EF_ERR_UNSUPPORTED, "K must be a positive multiple of 256 (got %d)", K);
  return EF_OK;
}

}  // namespace

extern "C" {

ef_status ef_kquant_dequantize(int type, const void* blocks, long long n_blocks, void* out, void* stream) {
  if (type != ef::kKqQ2 && type != ef::kKqQ3 && type != ef::kKqQ4)
    return fail(EF_ERR_UNSUPPORTED, "K-quant type must be Q2_K (10), Q3_K (11) or Q4_K (12), got %d", type);
  if (n_blocks < 0) return fail(EF_ERR_INVALID, "n_blocks < 0");
  if (n_blocks == 0) return EF_OK;
  if (!blocks || !out) return fail(EF_ERR_INVALID, "null pointer");
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(blocks) & 3))
    return fail(EF_ERR_INVALID, "out must be 16-byte and blocks 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n16 = n_blocks * 16;
  const int grid = (int)std::min<long long>((n16 + 255) / 256, 148LL * 64);
  const uint8_t* b = static_cast<const uint8_t*>(blocks);
  uint16_t* o = static_cast<uint16_t*>(out);
  if (type == ef::kKqQ2) ef::kquant_dequant_kernel<ef::kKqQ2><<<grid, 256, 0, st>>>(b, n_blocks, o);
  else if (type == ef::kKqQ3) ef::kquant_dequant_kernel<ef::kKqQ3><<<grid, 256, 0, st>>>(b, n_blocks, o);
  else ef::kquant_dequant_kernel<ef::kKqQ4><<<grid, 256, 0, st>>>(b, n_blocks, o);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EF_ERR_CUDA, "kquant_dequant: %s", cudaGetErrorString(e));
  return EF_OK;
}

size_t ef_kquant_matmul_workspace_size(int T, int K) {
  if (T < 0 || K < 0) return 0;
  const int nt = (T + 7) / 8;
  const size_t rows = (size_t)(nt <= 2 ? nt : 4) * 8;  // token groups the kernel reads: 1, 2 or 4
  return (rows * K * 2 + 255) / 256 * 256 + rows * (K / 32) * 4 + 256;  // permuted rows, Q4_K sub-block sums
}

ef_status ef_kquant_matmul(const void* x, int act_dtype, int T, const void* blocks, int type, int N, int K, float* y,
                           void* workspace, size_t ws_bytes, void* stream) {
  ef_status s = check_kquant(type, N, K);
  if (s) return s;
  if (act_dtype != EF_DT_BF16 && act_dtype != EF_DT_F16) return fail(EF_ERR_UNSUPPORTED, "act_dtype");
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  if (T == 0) return EF_OK;
  if (T > 32) return fail(EF_ERR_UNSUPPORTED, "T must be <= 32 for the K-quant GEMV (decode)");
  if (!x || !blocks || !y || !workspace) return fail(EF_ERR_INVALID, "null pointer");
  const uintptr_t need_align = type == ef::kKqQ4 ? 15 : 3;  // Q4_K rows are read in 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(blocks) & need_align) || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(EF_ERR_INVALID, "blocks must be %d-byte aligned, workspace 16-byte aligned", (int)need_align + 1);
  if (ws_bytes < ef_kquant_matmul_workspace_size(T, K)) return fail(EF_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nt = (T + 7) / 8;
  const int n_tok_k = (nt <= 2 ? nt : 4) * 8;  // token rows the kernel reads (zero beyond T)
  uint16_t* xp = static_cast<uint16_t*>(workspace);
  float* xsum = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((size_t)n_tok_k * K * 2 + 255) / 256 * 256);
  const int n_sm = sm_count();
  const int pgrid = (int)std::min<long long>(((long long)n_tok_k * K + 255) / 256, (long long)n_sm * 16);
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  const int bf = act_dtype == EF_DT_BF16;
  if (type == ef::kKqQ2) ef::kquant_prep_kernel<ef::kKqQ2><<<pgrid, 256, 0, st>>>(xs, bf, T, K, n_tok_k, xp, xsum);
  else if (type == ef::kKqQ3) ef::kquant_prep_kernel<ef::kKqQ3><<<pgrid, 256, 0, st>>>(xs, bf, T, K, n_tok_k, xp, xsum);
  else ef::kquant_prep_kernel<ef::kKqQ4><<<pgrid, 256, 0, st>>>(xs, bf, T, K, n_tok_k, xp, xsum);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EF_ERR_CUDA, "kquant_prep: %s", cudaGetErrorString(e));
  const int split = type == ef::kKqQ4 && T <= 16 ? kq4_split(N, K, n_sm) : kq_split(N, K, n_sm);
  const uint8_t* w = static_cast<const uint8_t*>(blocks);
  if (type == ef::kKqQ2) e = ef::launch_kquant_gemv_t<ef::kKqQ2>(w, xp, xsum, T, N, K, split, y, st);
  else if (type == ef::kKqQ3) e = ef::launch_kquant_gemv_t<ef::kKqQ3>(w, xp, xsum, T, N, K, split, y, st);
  else e = ef::launch_kquant_gemv_t<ef::kKqQ4>(w, xp, xsum, T, N, K, split, y, st);
  if (e != cudaSuccess) return fail(EF_ERR_CUDA, "kquant_gemv: %s", cudaGetErrorString(e));
  return EF_OK;
}

}  // extern "C"
