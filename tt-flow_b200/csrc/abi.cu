// C ABI of libtfb200 (declared in include/tfb200.h): argument validation, error
// reporting and dispatch to the sm_100a kernels.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/tfb200.h"
#include "internal.h"
#include "pair_sched.h"
#include "sm100_ptx.cuh"

namespace tfb200 {

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
std::atomic<uint64_t> g_wait_ns{2000000000ull};

// Per-device status word written by kernels whose bounded waits ran out.
__device__ int g_device_status;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

__global__ void k_fill_zero_bf16(bf16* c, int64_t rows, int64_t cols, int64_t ld) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, cc = i - r * cols;
    c[r * ld + cc] = __float2bfloat16_rn(0.0f);
  }
}

// Waits on an mbarrier that nothing arrives on; the bounded wait gives up after
// limit_ns and records the timeout in the status word.
__global__ void k_wait_selftest(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    abort = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(smem_u32(&bar), 0, &abort, limit_ns)) atomicExch(status, kDevTimeout);
}

bool mat_ok(const tfb200_mat* m, const char* name, std::string* err) {
  if (!m) {
    *err = std::string(name) + ": null descriptor";
    return false;
  }
  if (m->dtype != TFB200_BF16) {
    *err = std::string(name) + ": dtype must be TFB200_BF16";
    return false;
  }
  if (m->rows < 0 || m->cols < 0) {
    *err = std::string(name) + ": negative shape";
    return false;
  }
  if (m->ld < m->cols || m->ld < 1) {
    *err = std::string(name) + ": leading dimension smaller than the column count";
    return false;
  }
  if (!m->data && m->rows > 0 && m->cols > 0) {
    *err = std::string(name) + ": null data";
    return false;
  }
  return true;
}

const bf16* as_bf16(const void* p) { return static_cast<const bf16*>(p); }

// Largest dimension the size functions accept: products of three such values
// and small constants stay far inside size_t.
constexpr int64_t kMaxDim = int64_t(1) << 30;
constexpr size_t kTooBig = ~size_t(0);

size_t al256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

int64_t pair_tiles(int64_t m, int64_t n) { return ((m + 255) / 256) * ((n + 255) / 256); }

// The fused MLP's tail-split region (pair_sched.h): flags of the up- and the
// down-projection, then slots shared by both launches (the down-projection runs
// after the up-projection has completed).
size_t mlp_split_bytes(int64_t m, int64_t h, int64_t n) {
  if (m <= cfg::kTileM) return 0;
  const int64_t t = std::max(pair_tiles(m, h), pair_tiles(m, n));
  return static_cast<size_t>(2 * sched::flag_bytes() + sched::slot_count(t) * sched::kSlotBytes);
}

}  // namespace

// Workspace the fused MLP cannot run without: the bf16 hidden block and the
// RMSNorm staging (or the streamed path's buffers for few rows). A workspace
// of tfb200_fused_mlp_workspace_size() bytes adds the tail-split region.
size_t mlp_workspace_min_bytes(int64_t m, int64_t k, int64_t h, int64_t n) {
  if (m <= 0 || h <= 0 || k <= 0) return 0;
  if (m > kMaxDim || k > kMaxDim || h > kMaxDim || n > kMaxDim) return kTooBig;
  size_t need = al256(static_cast<size_t>(m) * static_cast<size_t>(h) * 2) + rms_prep_bytes(m, k);
  if (m <= kStreamMaxRows && n > 0) need = std::max(need, decode_mlp_bytes(m, k, h, n));
  return need;
}

int* device_status_ptr(std::string* err) {
  static int* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    if (err) *err = "no current CUDA device";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) {
      if (err) *err = std::string("cudaGetSymbolAddress(status): ") + cudaGetErrorString(e);
      return nullptr;
    }
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int sm_count() {
  static std::atomic<int> counts[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int c = counts[dev].load(std::memory_order_relaxed);
  if (!c) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    c = n > 0 ? n : 148;
    counts[dev].store(c, std::memory_order_relaxed);
  }
  return c;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

uint64_t launches() { return g_launches.load(); }
void count_launch(uint64_t n) { g_launches.fetch_add(n); }
uint64_t wait_limit_ns() { return g_wait_ns.load(); }
void set_wait_limit_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : 1); }

}  // namespace tfb200

using namespace tfb200;

extern "C" {

int tfb200_version(void) { return TFB200_ABI_VERSION; }

const char* tfb200_last_error(void) { return g_last_error.c_str(); }

uint64_t tfb200_launch_count(void) { return launches(); }

void tfb200_set_wait_limit_ns(uint64_t ns) { set_wait_limit_ns(ns); }

int tfb200_device_status(void) {
  std::string err;
  int* p = device_status_ptr(&err);
  if (!p) return fail(TFB200_ECUDA, err);
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("status read: ") + cudaGetErrorString(e));
  return v == kDevOk ? TFB200_OK : TFB200_ETIMEOUT;
}

int tfb200_clear_device_status(void) {
  std::string err;
  int* p = device_status_ptr(&err);
  if (!p) return fail(TFB200_ECUDA, err);
  int zero = 0;
  cudaError_t e = cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("status clear: ") + cudaGetErrorString(e));
  return TFB200_OK;
}

int tfb200_matmul(const tfb200_mat* a, const tfb200_mat* b, tfb200_mat* c, void* stream) {
  std::string err;
  if (!mat_ok(a, "a", &err) || !mat_ok(b, "b", &err) || !mat_ok(c, "c", &err))
    return fail(TFB200_EINVAL, "tfb200_matmul: " + err);
  if (a->cols != b->rows || c->rows != a->rows || c->cols != b->cols)
    return fail(TFB200_EINVAL, "tfb200_matmul: shapes do not agree (A[M,K] @ B[K,N] -> C[M,N])");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (c->rows == 0 || c->cols == 0) return TFB200_OK;
  if (a->cols == 0) {
    const int64_t n = c->rows * c->cols;
    const int blocks = static_cast<int>(n / 256 + 1 < 4096 ? n / 256 + 1 : 4096);
    k_fill_zero_bf16<<<blocks, 256, 0, s>>>(static_cast<bf16*>(c->data), c->rows, c->cols, c->ld);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("tfb200_matmul: ") + cudaGetErrorString(e));
    count_launch();
    return TFB200_OK;
  }
  GemmProblem g;
  g.M = a->rows;
  g.N = b->cols;
  g.K = a->cols;
  g.A = as_bf16(a->data);
  g.lda = a->ld;
  g.B = as_bf16(b->data);
  g.ldb = b->ld;
  g.C = static_cast<bf16*>(c->data);
  g.ldc = c->ld;
  int rc = run_gemm(g, s, &err);
  return rc ? fail(rc, "tfb200_matmul: " + err) : TFB200_OK;
}

size_t tfb200_fused_rmsnorm_matmul_workspace_size(int64_t m, int64_t k, int64_t n) {
  if (m <= 0 || k <= 0) return 0;
  if (m > kMaxDim || k > kMaxDim || n > kMaxDim) return kTooBig;
  return rms_prep_bytes(m, k) + pair_split_bytes(m, n);
}

int tfb200_fused_rmsnorm_matmul(const tfb200_mat* x, const void* gamma, const tfb200_mat* w, float eps,
                                tfb200_mat* y, void* stream, void* workspace, size_t workspace_bytes) {
  std::string err;
  if (!mat_ok(x, "x", &err) || !mat_ok(w, "w", &err) || !mat_ok(y, "y", &err))
    return fail(TFB200_EINVAL, "tfb200_fused_rmsnorm_matmul: " + err);
  if (x->cols != w->rows || y->rows != x->rows || y->cols != w->cols)
    return fail(TFB200_EINVAL, "tfb200_fused_rmsnorm_matmul: shapes do not agree (X[M,K], W[K,N] -> Y[M,N])");
  if (!(eps >= 0.0f)) return fail(TFB200_EINVAL, "tfb200_fused_rmsnorm_matmul: eps must be >= 0");
  if (y->rows == 0 || y->cols == 0) return TFB200_OK;
  if (x->cols == 0) return fail(TFB200_EINVAL, "tfb200_fused_rmsnorm_matmul: RMSNorm over an empty dimension");
  if (!gamma) return fail(TFB200_EINVAL, "tfb200_fused_rmsnorm_matmul: null gamma");
  const size_t base = rms_prep_bytes(x->rows, x->cols);
  if (!workspace || workspace_bytes < base)
    return fail(TFB200_EWORKSPACE,
                "tfb200_fused_rmsnorm_matmul: workspace smaller than the staging block it needs "
                "(tfb200_fused_rmsnorm_matmul_workspace_size() bytes give the fastest schedule)");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(TFB200_EWORKSPACE, "tfb200_fused_rmsnorm_matmul: workspace must be 256-byte aligned");
  // With the full workspace the GEMM may split the tail of its last wave; the
  // split's flags are cleared by the staging launch.
  const size_t split = pair_split_bytes(x->rows, w->cols);
  const bool use_split = split && workspace_bytes - base >= split;
  char* sp = static_cast<char*>(workspace) + base;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bf16* a = nullptr;
  int64_t lda = 0;
  float* inv = nullptr;
  int rc = run_rms_prep(as_bf16(x->data), x->ld, as_bf16(gamma), x->rows, x->cols, eps, workspace, &a, &lda, &inv,
                        s, &err, use_split ? sp : nullptr, use_split ? static_cast<size_t>(sched::flag_bytes()) : 0);
  if (rc) return fail(rc, "tfb200_fused_rmsnorm_matmul: " + err);
  GemmProblem g;
  g.M = x->rows;
  g.N = w->cols;
  g.K = x->cols;
  g.A = a;
  g.lda = lda;
  g.B = as_bf16(w->data);
  g.ldb = w->ld;
  g.C = static_cast<bf16*>(y->data);
  g.ldc = y->ld;
  g.row_scale = inv;
  g.b_stable = true;  // preceded by the staging pass, which writes only the workspace
  if (use_split) {
    g.sk_flags = reinterpret_cast<int*>(sp);
    g.sk_slots = reinterpret_cast<float*>(sp + sched::flag_bytes());
    g.sk_max_slots = static_cast<int>(sched::slot_count(pair_tiles(g.M, g.N)));
  }
  rc = run_gemm(g, s, &err);
  return rc ? fail(rc, "tfb200_fused_rmsnorm_matmul: " + err) : TFB200_OK;
}

size_t tfb200_fused_mlp_workspace_size(int64_t m, int64_t k, int64_t h, int64_t n) {
  const size_t base = mlp_workspace_min_bytes(m, k, h, n);
  if (base == 0 || base == kTooBig) return base;
  return base + mlp_split_bytes(m, h, n);
}

int tfb200_fused_mlp(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1, const void* b1,
                     const tfb200_mat* w2, const tfb200_mat* residual, float eps, int gelu_mode, tfb200_mat* y,
                     void* stream, void* workspace, size_t workspace_bytes) {
  std::string err;
  if (!mat_ok(x, "x", &err) || !mat_ok(w1, "w1", &err) || !mat_ok(w2, "w2", &err) ||
      !mat_ok(residual, "residual", &err) || !mat_ok(y, "y", &err))
    return fail(TFB200_EINVAL, "tfb200_fused_mlp: " + err);
  const int64_t M = x->rows, K = x->cols, H = w1->cols, N = w2->cols;
  if (w1->rows != K || w2->rows != H || y->rows != M || y->cols != N || residual->rows != M ||
      residual->cols != N)
    return fail(TFB200_EINVAL,
                "tfb200_fused_mlp: shapes do not agree (X[M,K], W1[K,H], W2[H,N], R[M,N] -> Y[M,N])");
  if (gelu_mode != TFB200_GELU_ERF && gelu_mode != TFB200_GELU_TANH)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp: gelu_mode must be TFB200_GELU_ERF or TFB200_GELU_TANH");
  if (!(eps >= 0.0f)) return fail(TFB200_EINVAL, "tfb200_fused_mlp: eps must be >= 0");
  if (M == 0 || N == 0) return TFB200_OK;
  if (K == 0) return fail(TFB200_EINVAL, "tfb200_fused_mlp: RMSNorm over an empty dimension");
  if (!gamma) return fail(TFB200_EINVAL, "tfb200_fused_mlp: null gamma");
  if (H == 0) return fail(TFB200_EUNSUPPORTED, "tfb200_fused_mlp: empty hidden dimension");
  const size_t need = mlp_workspace_min_bytes(M, K, H, N);
  if (!workspace || workspace_bytes < need)
    return fail(TFB200_EWORKSPACE,
                "tfb200_fused_mlp: workspace smaller than the hidden block and staging it needs "
                "(tfb200_fused_mlp_workspace_size() bytes give the fastest schedule)");
  if (reinterpret_cast<uintptr_t>(workspace) & 255u)
    return fail(TFB200_EWORKSPACE, "tfb200_fused_mlp: workspace must be 256-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (decode_eligible(M, w1->data, w1->ld, w2->data, w2->ld) && H % 8 == 0) {
    // Few rows: stream the weights through every SM (swap-AB, split K).
    int rc = run_decode_mlp(as_bf16(x->data), x->ld, as_bf16(gamma), as_bf16(w1->data), w1->ld, as_bf16(b1),
                            as_bf16(w2->data), w2->ld, as_bf16(residual->data), residual->ld, eps,
                            gelu_mode == TFB200_GELU_ERF ? kGeluErf : kGeluTanh, static_cast<bf16*>(y->data), y->ld,
                            nullptr, 0, M, K, H, N, workspace, s, &err);
    return rc ? fail(rc, "tfb200_fused_mlp (streamed): " + err) : TFB200_OK;
  }
  bf16* hid = static_cast<bf16*>(workspace);
  const size_t hid_bytes = al256(static_cast<size_t>(M) * static_cast<size_t>(H) * 2);
  const size_t base = hid_bytes + rms_prep_bytes(M, K);
  // With the full workspace both GEMMs may split the tail of their last wave;
  // the split's flags are cleared by the staging launch.
  const size_t split = mlp_split_bytes(M, H, N);
  const bool use_split = split && workspace_bytes >= base && workspace_bytes - base >= split;
  char* sp = static_cast<char*>(workspace) + base;
  bf16* a = nullptr;
  int64_t lda = 0;
  float* inv = nullptr;
  int rc = run_rms_prep(as_bf16(x->data), x->ld, as_bf16(gamma), M, K, eps, static_cast<char*>(workspace) + hid_bytes,
                        &a, &lda, &inv, s, &err, use_split ? sp : nullptr,
                        use_split ? static_cast<size_t>(2 * sched::flag_bytes()) : 0);
  if (rc) return fail(rc, "tfb200_fused_mlp: " + err);
  GemmProblem g1;
  g1.M = M;
  g1.N = H;
  g1.K = K;
  g1.A = a;
  g1.lda = lda;
  g1.B = as_bf16(w1->data);
  g1.ldb = w1->ld;
  g1.C = hid;
  g1.ldc = H;
  g1.row_scale = inv;
  g1.bias = as_bf16(b1);
  g1.gelu = gelu_mode == TFB200_GELU_ERF ? kGeluErf : kGeluTanh;
  float* slots = reinterpret_cast<float*>(sp + 2 * sched::flag_bytes());
  g1.b_stable = true;  // preceded by the staging pass, which writes only the workspace
  if (use_split) {
    g1.sk_flags = reinterpret_cast<int*>(sp);
    g1.sk_slots = slots;
    g1.sk_max_slots = static_cast<int>(sched::slot_count(pair_tiles(M, H)));
  }
  rc = run_gemm(g1, s, &err);
  if (rc) return fail(rc, "tfb200_fused_mlp (up projection): " + err);
  GemmProblem g2;
  g2.M = M;
  g2.N = N;
  g2.K = H;
  g2.A = hid;
  g2.lda = H;
  g2.B = as_bf16(w2->data);
  g2.ldb = w2->ld;
  g2.C = static_cast<bf16*>(y->data);
  g2.ldc = y->ld;
  g2.residual = as_bf16(residual->data);
  g2.ldr = residual->ld;
  g2.b_stable = true;  // preceded by the up-projection, which writes only the hidden block
  if (use_split) {
    g2.sk_flags = reinterpret_cast<int*>(sp + sched::flag_bytes());
    g2.sk_slots = slots;
    g2.sk_max_slots = static_cast<int>(sched::slot_count(pair_tiles(M, N)));
  }
  rc = run_gemm(g2, s, &err);
  if (rc) return fail(rc, "tfb200_fused_mlp (down projection): " + err);
  return TFB200_OK;
}

size_t tfb200_fused_mlp_partial_workspace_size(int64_t m, int64_t k, int64_t h, int64_t n) {
  if (m <= 0 || k <= 0 || h <= 0 || n <= 0) return 0;
  return decode_core_bytes(m, k, h, n);
}

int tfb200_fused_mlp_partial(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1, const void* b1,
                             const tfb200_mat* w2, float eps, int gelu_mode, float* partial, int64_t ld_partial,
                             void* stream, void* workspace, size_t workspace_bytes) {
  std::string err;
  if (!mat_ok(x, "x", &err) || !mat_ok(w1, "w1", &err) || !mat_ok(w2, "w2", &err))
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: " + err);
  const int64_t M = x->rows, K = x->cols, H = w1->cols, N = w2->cols;
  if (w1->rows != K || w2->rows != H)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: shapes do not chain (X[M,K], W1[K,H], W2[H,N])");
  if (gelu_mode != TFB200_GELU_ERF && gelu_mode != TFB200_GELU_TANH)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: bad gelu_mode");
  if (!(eps >= 0.0f)) return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: eps must be >= 0");
  if (M == 0 || N == 0) return TFB200_OK;
  if (!partial || ld_partial < N) return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: bad partial buffer");
  if (!gamma || K == 0) return fail(TFB200_EINVAL, "tfb200_fused_mlp_partial: null gamma or empty K");
  if (!decode_eligible(M, w1->data, w1->ld, w2->data, w2->ld) || H % 8 != 0)
    return fail(TFB200_EUNSUPPORTED,
                "tfb200_fused_mlp_partial: needs M <= 64, 16-byte aligned weights with ld % 8 == 0, H % 8 == 0");
  const size_t need = tfb200_fused_mlp_partial_workspace_size(M, K, H, N);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(TFB200_EWORKSPACE, "tfb200_fused_mlp_partial: workspace missing, small or not 256-byte aligned");
  const int rc = run_decode_mlp(as_bf16(x->data), x->ld, as_bf16(gamma), as_bf16(w1->data), w1->ld, as_bf16(b1),
                                as_bf16(w2->data), w2->ld, nullptr, 0, eps,
                                gelu_mode == TFB200_GELU_ERF ? kGeluErf : kGeluTanh, nullptr, 0, partial, ld_partial,
                                M, K, H, N, workspace, static_cast<cudaStream_t>(stream), &err);
  return rc ? fail(rc, "tfb200_fused_mlp_partial: " + err) : TFB200_OK;
}

int tfb200_residual_add(const float* partial, int64_t ld_partial, const tfb200_mat* residual, tfb200_mat* y,
                        void* stream) {
  std::string err;
  if (!mat_ok(residual, "residual", &err) || !mat_ok(y, "y", &err))
    return fail(TFB200_EINVAL, "tfb200_residual_add: " + err);
  if (residual->rows != y->rows || residual->cols != y->cols)
    return fail(TFB200_EINVAL, "tfb200_residual_add: residual and y shapes differ");
  if (y->rows == 0 || y->cols == 0) return TFB200_OK;
  if (!partial || ld_partial < y->cols) return fail(TFB200_EINVAL, "tfb200_residual_add: bad partial buffer");
  const int rc = launch_residual_add(partial, ld_partial, as_bf16(residual->data), residual->ld,
                                     static_cast<bf16*>(y->data), y->ld, y->rows, y->cols,
                                     static_cast<cudaStream_t>(stream), &err);
  return rc ? fail(rc, "tfb200_residual_add: " + err) : TFB200_OK;
}

int tfb200_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  std::string err;
  int* st = device_status_ptr(&err);
  if (!st) return fail(TFB200_ECUDA, err);
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(TFB200_EINVAL, "tfb200_selftest_bounded_wait: limit must be in (0, 10 s]");
  k_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(st, limit_ns);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("selftest launch: ") + cudaGetErrorString(e));
  count_launch();
  return TFB200_OK;
}

static size_t al256b(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

}  // extern "C"

namespace tfb200 {
TpLayout tp_layout(int64_t max_rows, int64_t n, int world) {
  TpLayout l{};
  const size_t rows_n = static_cast<size_t>(max_rows) * static_cast<size_t>(n);
  const size_t blocks = static_cast<size_t>((n + 127) / 128);
  l.acc = 0;
  l.local_cnt = l.acc + al256b(rows_n * 4);
  l.slots = l.local_cnt + al256b(blocks * 4);
  l.arrive = l.slots + static_cast<size_t>(world) * al256b(rows_n * 4);
  l.out = l.arrive + al256b(blocks * 4);
  l.done = l.out + al256b(rows_n * 2);
  l.total = l.done + 256;
  return l;
}
}  // namespace tfb200

extern "C" {

size_t tfb200_tp_buffer_bytes(int64_t max_rows, int64_t n, int32_t world) {
  if (max_rows <= 0 || max_rows > kStreamMaxRows || n <= 0 || world < 1 || world > TFB200_MAX_TP) return 0;
  return tp_layout(max_rows, n, world).total;
}

int tfb200_fused_mlp_tp(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1, const void* b1,
                        const tfb200_mat* w2, const tfb200_mat* residual, float eps, int gelu_mode,
                        const tfb200_tp_comm* comm, void* stream, void* workspace, size_t workspace_bytes) {
  std::string err;
  if (!mat_ok(x, "x", &err) || !mat_ok(w1, "w1", &err) || !mat_ok(w2, "w2", &err) ||
      !mat_ok(residual, "residual", &err))
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: " + err);
  if (!comm || comm->world < 1 || comm->world > TFB200_MAX_TP || comm->rank < 0 || comm->rank >= comm->world)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: bad communicator (rank / world)");
  const int64_t M = x->rows, K = x->cols, H = w1->cols, N = w2->cols;
  if (w1->rows != K || w2->rows != H || residual->rows != M || residual->cols != N)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: shapes do not chain (X[M,K], W1[K,H], W2[H,N], R[M,N])");
  if (gelu_mode != TFB200_GELU_ERF && gelu_mode != TFB200_GELU_TANH)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: bad gelu_mode");
  if (!(eps >= 0.0f) || !gamma || K == 0) return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: bad eps / gamma / K");
  if (M == 0 || N == 0) return TFB200_OK;
  if (M > comm->max_rows || comm->max_rows > kStreamMaxRows)
    return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: more rows than the buffers were sized for (max_rows <= 64)");
  for (int r = 0; r < comm->world; ++r)
    if (!comm->peer_buf[r] || (reinterpret_cast<uintptr_t>(comm->peer_buf[r]) & 255u))
      return fail(TFB200_EINVAL, "tfb200_fused_mlp_tp: missing or unaligned peer buffer");
  if (!decode_eligible(M, w1->data, w1->ld, w2->data, w2->ld) || H % 8 != 0 || N % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(residual->data) & 15u) || residual->ld % 8 != 0)
    return fail(TFB200_EUNSUPPORTED,
                "tfb200_fused_mlp_tp: needs 16-byte aligned weights and residual with leading dimensions % 8 == 0, "
                "H % 8 == 0 and N % 8 == 0");
  const size_t need = tfb200_fused_mlp_partial_workspace_size(M, K, H, N);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(TFB200_EWORKSPACE, "tfb200_fused_mlp_tp: workspace missing, small or not 256-byte aligned");
  const TpLayout l = tp_layout(comm->max_rows, N, comm->world);
  TpPeers tp;
  tp.rank = comm->rank;
  tp.world = comm->world;
  tp.slot_stride = comm->max_rows * N;
  char* own = static_cast<char*>(comm->peer_buf[comm->rank]);
  tp.acc = reinterpret_cast<float*>(own + l.acc);
  tp.local_cnt = reinterpret_cast<int*>(own + l.local_cnt);
  for (int r = 0; r < comm->world; ++r) {
    char* b = static_cast<char*>(comm->peer_buf[r]);
    tp.slots[r] = reinterpret_cast<float*>(b + l.slots);
    tp.arrive[r] = reinterpret_cast<unsigned*>(b + l.arrive);
    tp.out[r] = reinterpret_cast<bf16*>(b + l.out);
    tp.done[r] = reinterpret_cast<unsigned*>(b + l.done);
  }
  const int rc = run_decode_mlp(as_bf16(x->data), x->ld, as_bf16(gamma), as_bf16(w1->data), w1->ld, as_bf16(b1),
                                as_bf16(w2->data), w2->ld, as_bf16(residual->data), residual->ld, eps,
                                gelu_mode == TFB200_GELU_ERF ? kGeluErf : kGeluTanh, nullptr, 0, nullptr, 0, M, K, H,
                                N, workspace, static_cast<cudaStream_t>(stream), &err, &tp);
  return rc ? fail(rc, "tfb200_fused_mlp_tp: " + err) : TFB200_OK;
}

int tfb200_tp_output(const tfb200_tp_comm* comm, int64_t n, void** out) {
  if (!comm || !out || comm->world < 1 || comm->world > TFB200_MAX_TP || comm->rank < 0 ||
      comm->rank >= comm->world || !comm->peer_buf[comm->rank] || n <= 0)
    return fail(TFB200_EINVAL, "tfb200_tp_output: bad communicator");
  *out = static_cast<char*>(comm->peer_buf[comm->rank]) + tp_layout(comm->max_rows, n, comm->world).out;
  return TFB200_OK;
}

int tfb200_ipc_get(const void* ptr, void* handle64, size_t* offset) {
  if (!ptr || !handle64) return fail(TFB200_EINVAL, "tfb200_ipc_get: null argument");
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  if (!range_fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(TFB200_ECUDA, "tfb200_ipc_get: cuMemGetAddressRange unavailable");
    range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(TFB200_ECUDA, "tfb200_ipc_get: pointer is not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(handle64, &h, sizeof(h));
  if (offset) *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return TFB200_OK;
}

int tfb200_ipc_open(const void* handle64, void** base) {
  if (!handle64 || !base) return fail(TFB200_EINVAL, "tfb200_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return TFB200_OK;
}

int tfb200_ipc_close(void* base) {
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(TFB200_ECUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return TFB200_OK;
}

}  // extern "C"
