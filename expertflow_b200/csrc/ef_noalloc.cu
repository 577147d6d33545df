// ef_noalloc.cu -- ef_moe_forward_noalloc: the layer forward for callers that
// cannot allocate device memory.
//
// Who needs it: a host that binds this library through a plain FFI (ctypes,
// cgo, JNI) and has no CUDA allocator of its own to size and own the
// workspace that ef_moe_forward asks for, or a serving process whose device
// memory is owned up front by another framework's pool and whose decode loop
// must not call cudaMalloc (which can synchronise the device) between layers.
//
// The scratch lives in one file-scope __device__ array of a fixed size
// (EF_NOALLOC_SCRATCH_BYTES); every GPU that loads the library holds it until
// the process exits, whether or not this entry point is ever called (the
// array is part of the library's one module).  Host code never dereferences
// the array's name: the first call on each device resolves the array's device
// address with cudaGetSymbolAddress (with that device current) and caches it
// for that device's context, so the first call per device should come before
// any stream capture.  Every call shares
// the array and it keeps the previous call's contents: nothing in it needs to
// start at zero (each region the kernels read is written earlier in the same
// call), but calls that overlap on the GPU (other streams, other host threads)
// race on it and must be serialised by the caller.
#include <mutex>

#include "../../include/efmoe.h"
#include "ef_common.cuh"

static __device__ __align__(256) unsigned char g_ef_noalloc_scratch[EF_NOALLOC_SCRATCH_BYTES];

namespace {

// The array's address belongs to the CUDA context that loaded the module: a
// cudaDeviceReset (or a released and re-created primary context) loads it
// again, possibly at another address.  Each device's cached address is kept
// with the unique id of the context it was resolved in (cuCtxGetId) and
// resolved again when the current context's id differs.
typedef CUresult (*PFN_ctxGetCurrent_t)(CUcontext*);
typedef CUresult (*PFN_ctxGetId_t)(CUcontext, unsigned long long*);

struct NoallocSlot {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;
  bool ready = false;
};

std::mutex g_noalloc_mu;
NoallocSlot g_noalloc[64];

// Unique id of the calling thread's current context (0 when there is none or
// the driver lacks the call).
unsigned long long current_ctx_id() {
  static PFN_ctxGetCurrent_t get_cur = nullptr;
  static PFN_ctxGetId_t get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PFN_ctxGetCurrent_t>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_ctxGetId_t>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_cur && get_id && get_cur(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS) return id;
  return 0;
}

// Device address of the scratch array on the current device (set up once per
// device and context).
ef_status noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(EF_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(EF_ERR_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc[dev];
  const unsigned long long id = current_ctx_id();
  if (!slot.ready || id == 0 || id != slot.ctx_id) {
    void* p = nullptr;
    // also makes the device's primary context current when none is yet
    e = cudaGetSymbolAddress(&p, g_ef_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(EF_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    slot.ptr = p;
    slot.ctx_id = current_ctx_id();
    slot.ready = slot.ctx_id != 0;  // without a context id, resolve on every call
  }
  *out = slot.ptr;
  return EF_OK;
}

}  // namespace

extern "C" ef_status ef_moe_forward_noalloc(const ef_moe_cfg* cfg, const void* x, int T, const void* gate_w,
                                             const float* e_bias, ef_qweight gate, ef_qweight up, ef_qweight down,
                                             const ef_qweight* shared_gate, const ef_qweight* shared_up,
                                             const ef_qweight* shared_down, void* y, int32_t* inds_out,
                                             float* wts_out, void* stream) {
  ef_status s = check_cfg(cfg);
  if (s) return s;
  if (T < 0) return fail(EF_ERR_INVALID, "T < 0");
  const size_t need = ef_moe_workspace_size(cfg, T);
  if (need > (size_t)EF_NOALLOC_SCRATCH_BYTES)
    return fail(EF_ERR_WORKSPACE,
                "T=%d needs %zu bytes of scratch; ef_moe_forward_noalloc holds %zu bytes (use ef_moe_forward "
                "with a caller workspace, or split the batch)",
                T, need, (size_t)EF_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if ((s = noalloc_scratch(&scratch))) return s;
  return ef_moe_forward(cfg, x, T, gate_w, e_bias, gate, up, down, shared_gate, shared_up, shared_down, y, inds_out,
                        wts_out, scratch, (size_t)EF_NOALLOC_SCRATCH_BYTES, stream);
}
