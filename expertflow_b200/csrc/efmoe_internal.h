// efmoe_internal.h -- structures shared by the host API and the kernels.
#pragma once
#include <cuda.h>
#include <stdint.h>
#include <cuda_runtime.h>

namespace ef {

// ---- quantised grouped GEMV (decode path) ----
constexpr int kRowTile = 64;        // weight rows per work item (4 warps x 16 rows)
constexpr int kTokChunk = 8;        // rows (tokens) of one MMA n-tile / activation box
constexpr int kSegRows = 16;        // rows per decode-GEMV segment: up to two n-tiles share each weight pass
#ifndef EF_GEMM_NMAX
#define EF_GEMM_NMAX 192
#endif
constexpr int kGemmSegRows = EF_GEMM_NMAX;  // rows (tokens) per segment of the grouped GEMM (UMMA N)
constexpr int kComputeWarps = 4;    // 4 x 16 rows
constexpr int kQmvThreads = (kComputeWarps + 2) * 32;  // + TMA producer warp + scale producer warp

// Row stride (floats) of the per-64-column group sums of a K-wide activation:
// padded to 4 groups so that every row is a whole number of 16-byte units.
__host__ __device__ inline int sum_ld(int K) { return ((K / 64) + 3) & ~3; }

// error codes written to the device error word
constexpr int kDevErrTimeoutFull = 1001;
constexpr int kDevErrTimeoutEmpty = 1002;
constexpr int kDevErrTimeoutScales = 1003;
constexpr int kDevErrRange = 2001;
constexpr int kDevErrTimeoutTc = 1004;
constexpr int kDevErrSmemAlign = 2003;  // dynamic shared memory not 1024-byte aligned
constexpr int kDevErrTimeoutPeer = 1005;  // a peer rank's flag never arrived
constexpr int kDevErrRecvOverflow = 2002; // more rows received than the exchange holds

// Output of the permutation (all device pointers into the workspace).
struct PermBufs {
  int* counts;      // [n_bins]            rows per expert (bin n_experts = shared expert)
  int* offsets;     // [n_bins + 1]        first sorted row of each expert
  int* row_src;     // [n_rows]            source row (token) of each sorted row
  int* inv;         // [n_entries]         sorted row of each routed entry (t*k + j)
  int* seg_expert;  // [max_segs]
  int* seg_row0;    // [max_segs]
  int* seg_nrows;   // [max_segs]
  int* n_seg;       // [1]
};

struct QmvParams {
  CUtensorMap tm_w0;    // routed codes: gate (mode 0) or down (mode 1), 2-D [E*R, K*bits/32]
  CUtensorMap tm_w1;    // routed codes: up (mode 0)
  CUtensorMap tm_sw0;   // shared expert codes
  CUtensorMap tm_sw1;
  const uint32_t* w0;   // raw code pointers of the four maps (for L2 prefetch of whole items)
  const uint32_t* w1;
  const uint32_t* sw0;
  const uint32_t* sw1;
  const uint16_t* s0;   // routed scales/biases [E*R, K/64]
  const uint16_t* b0;
  const uint16_t* s1;
  const uint16_t* b1;
  const uint16_t* ss0;  // shared expert scales/biases [R, K/64]
  const uint16_t* sb0;
  const uint16_t* ss1;
  const uint16_t* sb1;
  CUtensorMap tm_act;       // fp16 activation rows [n_rows, K] in routed-row order and the GEMV
                            // layout (act_pos); 2-D, box 64 columns x 8 rows, 128-byte swizzle
  const float* act_sum;     // [n_rows, sum_ld(K)] group sums of the activation rows
  const int* seg_expert;
  const int* seg_row0;
  const int* seg_nrows;
  const int* n_seg;
  int K;                    // input dim
  int R;                    // output rows per expert
  int n_experts;            // expert id == n_experts selects the shared expert
  uint16_t* h_out;          // mode 0: fp16 pair-ordered [n_rows, R]
  float* hsum_out;          // mode 0: [n_rows, sum_ld(R)] group sums of h
  float* y_out;             // mode 1: fp32 [n_rows, R]
  CUtensorMap tm_sc[8];     // scales/biases as [rows, K/64] fp16, box 32 groups x 64 rows, 64-byte swizzle:
                            // s0, b0, s1, b1, then the shared expert's ss0, sb0, ss1, sb1 (valid if sb_chunked)
  int sb_chunked;           // 1: scales streamed in 32-group chunks through tm_sc (K / 64 a multiple of 8)
  int n_stages;             // TMA ring depth (set by the launcher)
  int n_slots;              // scale slots (set by the launcher)
  // expert-parallel return (modes 1 / 2, ret_rank non-null): output row q goes
  // to rank ret_rank[q]'s return region at row ret_row[q] (peer stores), and
  // the grid's last CTA releases this rank's done flag in every rank's buffer
  // (value *ep_epoch) once every row is written
  const int* ret_rank;
  const int* ret_row;
  float* const* ret_base;      // device [ep_ranks]: each rank's return region
  uint32_t* const* ret_flag;   // device [ep_ranks]: this rank's done flag in each rank's buffer
  const uint32_t* ep_epoch;
  uint32_t* ep_ctr;            // last-CTA counter (zero between launches)
  int ep_ranks;
  int ret_rows;                // rows of a return region (bound of ret_row)
};

}  // namespace ef
