// dsm_router_noalloc: the router for callers that cannot allocate device memory.
//
// Some callers of this router cannot hand it a workspace: an inference engine that has
// planned every byte of device memory up front (its arena owns the GPU and it cannot size
// or grant extra buffers per call), or a latency-critical decode loop that must not go
// through an allocator at all. This entry point takes the same inputs and outputs as
// dsm_router and uses, as scratch, a fixed array that lives in the library's own device
// memory. Limits and sharing rules:
//
//   - The array holds kNoAllocScratchBytes (8 MiB) on every GPU that loads the library,
//     until the process exits. A call whose dsm_router_workspace_bytes() exceeds it is
//     rejected with DSM_ERR_WORKSPACE before any GPU work.
//   - The first call on a device resolves the array's device address there (once per
//     device, with that device current); make that first call before any stream capture.
//     The address is cached together with the unique id of the CUDA context it belongs to.
//     cudaDeviceReset destroys that context and the array with it; the first call after a
//     reset sees a new context id and resolves the address again (again: before any
//     capture), so a stale address is never passed to a kernel.
//   - Every call shares the one array and leaves its contents behind. The router overwrites
//     every scratch cell it reads, so nothing has to start at zero; but two calls that can
//     overlap on the GPU (different streams without ordering between them) race on it.
//   - Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace dsm {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static_assert(kNoAllocScratchBytes == DSM_ROUTER_NOALLOC_MAX_SCRATCH_BYTES, "header and library disagree");

static __device__ __align__(256) unsigned char g_router_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  void* addr = nullptr;
  unsigned long long ctx_id = 0;  // unique id of the context the address belongs to
};
std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices];

// The driver's current-context queries, reached through the runtime (no libcuda link).
struct CtxFns {
  PFN_cuCtxGetCurrent_v4000 current = nullptr;
  PFN_cuCtxGetId_v12000 id = nullptr;
};
const CtxFns& ctx_fns() {
  static CtxFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  return f;
}

// Unique id of the calling thread's current context, 0 when there is none yet.
unsigned long long current_ctx_id() {
  const CtxFns& f = ctx_fns();
  if (!f.current || !f.id) return 0;
  CUcontext c = nullptr;
  if (f.current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  unsigned long long id = 0;
  return f.id(c, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of g_router_scratch on the current device: resolved on the first call on a
// device, and again whenever the device's context has changed since (after cudaDeviceReset).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSM_ERR_CUDA, std::string("dsm_router_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(DSM_ERR_UNSUPPORTED, "dsm_router_noalloc: device ordinal >= 64");
  if (!ctx_fns().current || !ctx_fns().id)
    return fail(DSM_ERR_CUDA, "dsm_router_noalloc: cuCtxGetCurrent / cuCtxGetId unavailable");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long id = current_ctx_id();
  if (!slot.addr || id == 0 || id != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_router_scratch);  // makes the device's primary context current
    if (e != cudaSuccess || p == nullptr)
      return fail(DSM_ERR_CUDA, std::string("dsm_router_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    slot.addr = p;
    slot.ctx_id = current_ctx_id();
  }
  *out = slot.addr;
  return DSM_OK;
}

}  // namespace
}  // namespace dsm

extern "C" int dsm_router_noalloc(const void* x, int x_dtype, int64_t n_tokens, int dim, const float* gate_weight,
                                  int n_experts, const float* gate_bias, const int32_t* tid2eid, int64_t vocab,
                                  const void* input_ids, int ids_dtype, int64_t n_ids, int topk, int score_func,
                                  float route_scale, float* weights_out, int32_t* indices_out, void* stream) {
  using namespace dsm;
  if (n_tokens > 0 && dim > 0 && n_experts > 0) {
    const size_t need = dsm_router_workspace_bytes(n_tokens, dim, n_experts);
    if (need > kNoAllocScratchBytes)
      return fail(DSM_ERR_WORKSPACE, "dsm_router_noalloc: this call needs " + std::to_string(need) +
                                         " bytes of scratch, more than the fixed " +
                                         std::to_string(kNoAllocScratchBytes) +
                                         "; use dsm_router with a caller-provided workspace");
  }
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  return dsm_router(x, x_dtype, n_tokens, dim, gate_weight, n_experts, gate_bias, tid2eid, vocab, input_ids, ids_dtype,
                    n_ids, topk, score_func, route_scale, scratch, weights_out, indices_out, stream);
}
