// ef_dequant.cu -- MLX affine dequantisation (replaces mx.dequantize,
// ef_cpu_fast.py:70-75): out[o, i] = s[o, i/64] * q[o, i] + b[o, i/64].
// s*q is exact in fp32 (11-bit x 8-bit significands), so the single rounding
// of the fma equals the oracle's multiply-then-add.
#include "ef_common.cuh"

namespace ef {

template <int BITS>
__global__ void dequant_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ s,
                               const uint16_t* __restrict__ b, int rows, int cols, void* __restrict__ out,
                               int out_dtype) {
  constexpr int PER = 32 / BITS;
  const int wpr = cols / PER;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)rows * wpr) return;
  const int o = (int)(gid / wpr), wi = (int)(gid % wpr);
  const uint32_t word = w[gid];
  const int col0 = wi * PER;
  const int g = col0 / 64, ng = cols / 64;
  const float sc = h16_to_f32(s[(size_t)o * ng + g]);
  const float bi = h16_to_f32(b[(size_t)o * ng + g]);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const float q = (float)((word >> (BITS * j)) & ((1u << BITS) - 1u));
    const float v = fmaf(sc, q, bi);
    const size_t idx = (size_t)o * cols + col0 + j;
    if (out_dtype == 2) static_cast<float*>(out)[idx] = v;
    else if (out_dtype == 1) static_cast<__half*>(out)[idx] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  }
}

cudaError_t launch_dequantize(const uint32_t* w, const uint16_t* s, const uint16_t* b, int rows, int cols, int bits,
                              void* out, int out_dtype, cudaStream_t st) {
  const long long words = (long long)rows * cols * bits / 32;
  const int threads = 256;
  const unsigned blocks = (unsigned)((words + threads - 1) / threads);
  if (bits == 4)
    dequant_kernel<4><<<blocks, threads, 0, st>>>(w, s, b, rows, cols, out, out_dtype);
  else
    dequant_kernel<8><<<blocks, threads, 0, st>>>(w, s, b, rows, cols, out, out_dtype);
  return cudaGetLastError();
}

}  // namespace ef
