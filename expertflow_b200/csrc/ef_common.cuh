// ef_common.cuh -- device helpers shared by the sm_100a kernels of libefmoe.
//
// Every wait on an mbarrier is bounded: after EF_WAIT_LIMIT polls the waiting
// thread records an error code in the device error word and returns false, so a
// lost copy ends the kernel with a status instead of a hang.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>

#include "efmoe_internal.h"

#define EF_DEV __device__ __forceinline__

#ifndef EF_WAIT_LIMIT
#define EF_WAIT_LIMIT (1u << 26)
#endif

// Device error word (one per process; read and cleared by ef_get_device_error).
__device__ int g_ef_dev_error = 0;

EF_DEV void ef_set_error(int code) { atomicCAS(&g_ef_dev_error, 0, code); }
EF_DEV bool ef_error_seen() { return *(volatile int*)&g_ef_dev_error != 0; }

EF_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---------------------------------------------------------------- mbarrier
EF_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
EF_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
EF_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

EF_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
EF_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
EF_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false (and records `code`) if the phase never completed
// or another thread already reported an error.
EF_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  for (uint32_t i = 0; i < EF_WAIT_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u && ef_error_seen()) return false;
  }
  ef_set_error(code);
  return false;
}

// ---------------------------------------------------------------- flags shared with peer GPUs
// A wait on a peer's flag ends after kPeerWaitNs of the GPU's global timer
// or kPeerWaitPolls polls, whichever comes first: ranks may start a forward
// seconds apart (host-side work between layers), a dead rank must not hang
// the others.
constexpr unsigned long long kPeerWaitNs = 20ull * 1000 * 1000 * 1000;
constexpr uint32_t kPeerWaitPolls = 1u << 28;
EF_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
EF_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait until *flag has reached `want` (flags only grow, mod 2^32);
// false (error word set) when it never does or another wait already failed.
EF_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
EF_DEV bool wait_flag_sys(const uint32_t* flag, uint32_t want) {
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0; i < kPeerWaitPolls; ++i) {
    if ((int)(ld_acquire_sys(flag) - want) >= 0) return true;
    if ((i & 255u) == 255u && (ef_error_seen() || global_ns() - t0 > kPeerWaitNs)) break;
    __nanosleep(i < 1024 ? 32 : 256);
  }
  if (!ef_error_seen()) ef_set_error(ef::kDevErrTimeoutPeer);
  return false;
}

// ---------------------------------------------------------------- programmatic dependent launch
// The kernels of one forward are launched with programmatic stream
// serialisation: each waits for its predecessor's completion and memory
// (pdl_wait) before its first global-memory access, then lets its successor
// be scheduled (pdl_launch_next), so the stream order of the data is kept
// while launch latency and prologues overlap the predecessor's tail.  Letting
// the successor launch only after the wait keeps the early launches to one
// kernel ahead: a chain of waiting grids would hold the SMs' registers and
// shared memory.  Kernels followed by a persistent grid (the decode GEMV and
// the grouped GEMM fill every SM) do not launch it early -- its CTAs would
// start late on SMs still busy with the predecessor -- it then launches at
// the predecessor's completion, which still saves the launch gap.  Without a
// programmatic predecessor both are no-ops.
EF_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
EF_DEV void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// EF_PDL=0 in the environment launches without the attribute.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("EF_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Raises a kernel's dynamic shared-memory limit once per device (the attribute
// belongs to the device's context); host threads may race on a first call,
// which only repeats the idempotent attribute call.
template <typename Kern>
inline cudaError_t set_max_smem_once(Kern* kern, int bytes, std::atomic<bool> (&done)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < 64) done[dev].store(true, std::memory_order_release);
  return e;
}

// ---------------------------------------------------------------- TMA / bulk copies
// 2-D tiled tensor load, completion counted on `bar` (bytes).
EF_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
// Prefetch the box of a 2-D tensor map at (c0, c1) into L2.
EF_DEV void prefetch_tile_l2(const CUtensorMap* map, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1)
               : "memory");
}
// 1-D bulk copy global -> shared; dst/src 16-byte aligned, bytes % 16 == 0.
EF_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
EF_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- bit tricks
EF_DEV uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {  // (a & b) | c
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
EF_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// mma.sync m16n8k16, fp16 inputs, fp32 accumulate.
EF_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

EF_DEV float h16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
EF_DEV float bf16_to_f32(uint16_t h) { return __uint_as_float(static_cast<uint32_t>(h) << 16); }
EF_DEV float act_to_f32(uint16_t v, int is_bf16) { return is_bf16 ? bf16_to_f32(v) : h16_to_f32(v); }

// Saturating fp32 -> fp16 (returns bits).
EF_DEV uint16_t f32_to_h16_sat(float v) {
  v = fminf(fmaxf(v, -65504.0f), 65504.0f);
  return __half_as_ushort(__float2half_rn(v));
}

// Activation layout seen by the GEMV kernel: each 8-column block is stored
// permuted so that the pairs of codes unpacked into one 32-bit register meet
// the matching 32-bit pair of activations.
//   4-bit codes: [c0 c4 c1 c5 c2 c6 c3 c7]   (nibbles s and s+4 of a word)
//   8-bit codes: [c0 c2 c4 c6 c1 c3 c5 c7]   (bytes 0/2 and 1/3 of a word)
// act_pos: position of column c (0..7) in its block; act_col: the inverse.
__host__ __device__ __forceinline__ int act_pos(int c, int bits) {
  return bits == 4 ? (((c & 3) << 1) | ((c >> 2) & 1)) : (((c & 1) << 2) | (c >> 1));
}
__host__ __device__ __forceinline__ int act_col(int p, int bits) {
  return bits == 4 ? ((p >> 1) | ((p & 1) << 2)) : (((p & 3) << 1) | (p >> 2));
}
