// Fused MLP entry point that allocates nothing, for callers that may not call
// cudaMalloc (or may not have the library allocate on their behalf): plugin
// hosts that own every byte of device memory, inference servers that reserve
// the GPU's memory up front, and real-time loops that cannot afford the device
// synchronisation an allocation can cause. Such a caller passes inputs and the
// output; the hidden activation block lives in a fixed device array of this
// file instead of a caller-provided workspace.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds TFB200_NOALLOC_SCRATCH_BYTES of it until the process exits.
// With CUDA's lazy module loading (the default since CUDA 12.2) that memory is
// committed when this file's module first loads on a device, which is inside
// the first call's cudaGetSymbolAddress; a host that reserves all of the GPU's
// memory should make its first call before that (or run with
// CUDA_MODULE_LOADING=EAGER). Host code cannot use the array's name as a device
// address (it names a host stand-in), so the device address is fetched once per
// device and context with cudaGetSymbolAddress, with that device current, on the
// first call made on it. That first call should therefore come before any stream
// capture. A new context on the device (after cudaDeviceReset) is noticed and
// the address fetched again. All calls on a device share the array and it keeps
// the last call's contents: two calls whose kernels overlap on the GPU
// (different streams without ordering between them) race on it. Nothing in it
// has to start at zero: the staging pass and the up-projection write every
// element that the later kernels read, and when the problem's full workspace
// (with the GEMMs' tail-split region) fits the scratch, the staging launch of
// every call clears the split's flags before the GEMMs read them.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <string>

#include "../../include/tfb200.h"
#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[TFB200_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct ScratchEntry {
  std::atomic<void*> ptr{nullptr};
  std::atomic<CUcontext> ctx{nullptr};
};

// The calling thread's current context (CUDA driver, looked up once).
CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 get = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuCtxGetCurrent_v4000>(nullptr);
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }();
  CUcontext c = nullptr;
  if (get && get(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

void* scratch_address(std::string* err) {
  static ScratchEntry entries[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = "no current CUDA device";
    return nullptr;
  }
  ScratchEntry& e = entries[dev];
  // Fast path: the address is known for the context this thread runs in.
  const CUcontext ctx = current_context();
  void* p = e.ptr.load(std::memory_order_acquire);
  if (p && ctx && e.ctx.load(std::memory_order_acquire) == ctx) return p;
  // First call on this device (or a new context): look the address up.
  std::lock_guard<std::mutex> lock(mu);
  void* q = nullptr;
  const cudaError_t rc = cudaGetSymbolAddress(&q, g_noalloc_scratch);
  if (rc != cudaSuccess || q == nullptr) {
    *err = std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(rc);
    return nullptr;
  }
  e.ctx.store(current_context(), std::memory_order_release);
  e.ptr.store(q, std::memory_order_release);
  return q;
}

}  // namespace

extern "C" int tfb200_fused_mlp_noalloc(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1,
                                        const void* b1, const tfb200_mat* w2, const tfb200_mat* residual,
                                        float eps, int gelu_mode, tfb200_mat* y, void* stream) {
  // The size limit applies to problems whose shapes chain; anything else is
  // left to tfb200_fused_mlp, which reports the shape error itself.
  if (x && w1 && w2 && w1->rows == x->cols && w2->rows == w1->cols) {
    const size_t need = tfb200::mlp_workspace_min_bytes(x->rows, x->cols, w1->cols, w2->cols);
    if (need > TFB200_NOALLOC_SCRATCH_BYTES) {
      tfb200::set_last_error("tfb200_fused_mlp_noalloc: the problem needs " + std::to_string(need) +
                             " bytes of scratch for its hidden block and staging; the fixed scratch holds " +
                             std::to_string(static_cast<size_t>(TFB200_NOALLOC_SCRATCH_BYTES)) +
                             ". Use tfb200_fused_mlp with a workspace, or fewer rows per call.");
      return TFB200_EINVAL;
    }
  }
  std::string err;
  void* scratch = scratch_address(&err);
  if (!scratch) {
    tfb200::set_last_error("tfb200_fused_mlp_noalloc: " + err);
    return TFB200_ECUDA;
  }
  return tfb200_fused_mlp(x, gamma, w1, b1, w2, residual, eps, gelu_mode, y, stream, scratch,
                          TFB200_NOALLOC_SCRATCH_BYTES);
}
