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
// Host code cannot use the array's name as a device address (it names a host
// stand-in), so the device address is fetched once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on it.
// That first call should therefore come before any stream capture. All calls on
// a device share the array and it keeps the last call's contents: two calls
// whose kernels overlap on the GPU (different streams without ordering between
// them) race on it. Nothing in it has to start at zero: the staging pass and
// the up-projection write every element that the later kernels read.
#include <mutex>
#include <string>

#include "../../include/tfb200.h"
#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[TFB200_NOALLOC_SCRATCH_BYTES];

void* scratch_address(std::string* err) {
  static void* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = "no current CUDA device";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *err = std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e);
      return nullptr;
    }
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace

extern "C" int tfb200_fused_mlp_noalloc(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1,
                                        const void* b1, const tfb200_mat* w2, const tfb200_mat* residual,
                                        float eps, int gelu_mode, tfb200_mat* y, void* stream) {
  if (x && w1 && w2) {
    const size_t need = tfb200_fused_mlp_workspace_size(x->rows, x->cols, w1->cols, w2->cols);
    if (need > TFB200_NOALLOC_SCRATCH_BYTES) {
      tfb200::set_last_error("tfb200_fused_mlp_noalloc: the workspace needs " + std::to_string(need) +
                             " bytes (tfb200_fused_mlp_workspace_size); the fixed scratch holds " +
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
