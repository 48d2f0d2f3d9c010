// Host-side interfaces shared by the CUDA translation units of libtfb200.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace tfb200 {

using bf16 = __nv_bfloat16;

enum GeluMode : int { kGeluNone = 0, kGeluErf = 1, kGeluTanh = 2 };

// One GEMM with the fused epilogue options of this backend:
//   C[M,N] = epi( row_scale[m] * (A[M,K] @ B[K,N]) )
// epi(v) = gelu(v + bias[n]) (each part optional), then + residual[m,n].
// row_scale (fp32, optional) carries the RMSNorm inverse RMS when A is the
// bf16(x * gamma) block staged by run_rms_prep.
// All matrices are bf16, row-major, with leading dimensions in elements.
struct GemmProblem {
  int64_t M = 0, N = 0, K = 0;
  const bf16* A = nullptr;
  int64_t lda = 0;
  const bf16* B = nullptr;
  int64_t ldb = 0;
  bf16* C = nullptr;
  int64_t ldc = 0;
  const float* row_scale = nullptr;
  const bf16* bias = nullptr;
  int gelu = kGeluNone;
  const bf16* residual = nullptr;
  int64_t ldr = 0;
};

// Launch the persistent tcgen05 GEMM. Returns 0 or a negative TFB200_E* code with
// a message in *err.
int run_gemm(const GemmProblem& p, cudaStream_t stream, std::string* err);

// RMSNorm staging pass (rmsnorm_prep.cu): writes bf16(x * gamma) with leading
// dimension staged_ld(K) and inv[m] = 1/sqrt(mean_k(x^2) + eps) into `ws`
// (rms_prep_bytes(M, K) bytes, 256-byte aligned).
int64_t staged_ld(int64_t k);
size_t rms_prep_bytes(int64_t m, int64_t k);
int run_rms_prep(const bf16* x, int64_t ldx, const bf16* gamma, int64_t M, int64_t K, float eps, void* ws,
                 bf16** a_out, int64_t* lda_out, float** inv_out, cudaStream_t stream, std::string* err);

// Device status word (per device): set by kernels whose bounded waits ran out.
int* device_status_ptr(std::string* err);

// Set the message tfb200_last_error() returns on this thread.
void set_last_error(const std::string& msg);

// SM count of the current device (cached).
int sm_count();

// Per-kernel launch counter (host side, for the benchmark's launch accounting).
uint64_t launches();
void count_launch(uint64_t n = 1);

// Wait-limit (ns) given to kernels' bounded waits.
uint64_t wait_limit_ns();
void set_wait_limit_ns(uint64_t ns);

}  // namespace tfb200
