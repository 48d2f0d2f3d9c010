// RMSNorm staging pass of the fused RMSNorm+MatMul and fused MLP paths.
//
// One warp per row reads the activation row once from HBM, computes
// sum(x^2) in fp32, and writes
//   inv[m]   = 1 / sqrt(sum_k x[m,k]^2 / K + eps)            (fp32)
//   a[m, k]  = bf16(x[m,k] * gamma[k])                       (bf16, one rounding)
// The GEMM that follows consumes `a` as its A operand and multiplies each
// accumulator row by inv[m] in its epilogue, using
//   rmsnorm(x) @ W = diag(inv) * ((x * gamma) @ W).
// This replaces the RMSNorm part of the Tensix fused compute kernels
// (tensixflow lib/tensixflow/Codegen/EmitCompute.cpp:172-213 square / reduce /
// rsqrt / scale, :437-492 in the MLP kernel). `a` is written with a leading
// dimension that is a multiple of 8 elements so that TMA can always describe it,
// whatever the alignment of x.
//
// The pass is HBM-bound: 2*M*K bytes read, 2*M*K + 4*M written. The second read
// of each row (to apply gamma after the sum is known) hits L1/L2.
#include "internal.h"
#include "sm100_ptx.cuh"

namespace tfb200 {

namespace {

constexpr int kWarps = 8;

// Clears `n` 16-byte words at `zero` with all threads of the grid (the flags of
// the GEMM that follows; a few KiB).
__device__ __forceinline__ void clear_words(uint4* __restrict__ zero, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    zero[i] = make_uint4(0u, 0u, 0u, 0u);
}

template <bool VEC>
__global__ void __launch_bounds__(kWarps * 32) k_rms_prep(const bf16* __restrict__ x, int64_t ldx,
                                                          const bf16* __restrict__ gamma, int M, int K, float eps,
                                                          bf16* __restrict__ a, int64_t lda,
                                                          float* __restrict__ inv, uint4* __restrict__ zero,
                                                          int64_t zero_vecs) {
  // Launched with programmatic serialization: wait for the preceding grid (which
  // may still read `a` or write `x`), then let the GEMM that follows place its
  // CTAs and run its prologue beside this pass's last CTAs.
  grid_dep_wait();
  grid_dep_launch();
  clear_words(zero, zero_vecs);
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < M; row += stride) {
    const bf16* xr = x + row * ldx;
    bf16* ar = a + row * lda;
    float ss = 0.0f;
    if (VEC) {
      const uint4* xv = reinterpret_cast<const uint4*>(xr);
      const int nchunk = K / 8;
      uint64_t ss2 = 0;
#pragma unroll 4
      for (int c = lane; c < nchunk; c += 32) {
        const uint4 v = __ldg(xv + c);
        ss2 = sq_acc_bf16x2(ss2, v.x);
        ss2 = sq_acc_bf16x2(ss2, v.y);
        ss2 = sq_acc_bf16x2(ss2, v.z);
        ss2 = sq_acc_bf16x2(ss2, v.w);
      }
      ss = __uint_as_float(static_cast<uint32_t>(ss2)) + __uint_as_float(static_cast<uint32_t>(ss2 >> 32));
    } else {
      for (int k = lane; k < K; k += 32) {
        const float v = __bfloat162float(xr[k]);
        ss = fmaf(v, v, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) inv[row] = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
    if (VEC) {
      const uint4* xv = reinterpret_cast<const uint4*>(xr);
      const uint4* gv = reinterpret_cast<const uint4*>(gamma);
      uint4* av = reinterpret_cast<uint4*>(ar);
      const int nchunk = K / 8;
#pragma unroll 4
      for (int c = lane; c < nchunk; c += 32) {
        const uint4 v = __ldg(xv + c);
        const uint4 g = __ldg(gv + c);
        av[c] = make_uint4(mul_bf16x2(v.x, g.x), mul_bf16x2(v.y, g.y), mul_bf16x2(v.z, g.z), mul_bf16x2(v.w, g.w));
      }
    } else {
      for (int k = lane; k < K; k += 32)
        ar[k] = __float2bfloat16_rn(__bfloat162float(xr[k]) * __bfloat162float(gamma[k]));
    }
  }
}

// Rows of up to kRegChunks * 32 * 8 elements (K <= 4096): the warp holds its
// row in registers, so x is read from HBM once and all of a lane's 16-byte loads
// are in flight together. Same arithmetic and summation order as k_rms_prep.
constexpr int kRegChunks = 16;

__global__ void __launch_bounds__(kWarps * 32) k_rms_prep_reg(const bf16* __restrict__ x, int64_t ldx,
                                                              const bf16* __restrict__ gamma, int M, int K, float eps,
                                                              bf16* __restrict__ a, int64_t lda,
                                                              float* __restrict__ inv, uint4* __restrict__ zero,
                                                              int64_t zero_vecs) {
  grid_dep_wait();
  grid_dep_launch();
  clear_words(zero, zero_vecs);
  const int lane = threadIdx.x & 31;
  const int nchunk = K / 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); row < M; row += stride) {
    const uint4* xv = reinterpret_cast<const uint4*>(x + row * ldx);
    uint4 v[kRegChunks];
#pragma unroll
    for (int i = 0; i < kRegChunks; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < nchunk ? __ldg(xv + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    uint64_t ss2 = 0;
#pragma unroll
    for (int i = 0; i < kRegChunks; ++i) {
      if (lane + 32 * i < nchunk) {
        ss2 = sq_acc_bf16x2(ss2, v[i].x);
        ss2 = sq_acc_bf16x2(ss2, v[i].y);
        ss2 = sq_acc_bf16x2(ss2, v[i].z);
        ss2 = sq_acc_bf16x2(ss2, v[i].w);
      }
    }
    float ss = __uint_as_float(static_cast<uint32_t>(ss2)) + __uint_as_float(static_cast<uint32_t>(ss2 >> 32));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) inv[row] = 1.0f / sqrtf(ss / static_cast<float>(K) + eps);
    const uint4* gv = reinterpret_cast<const uint4*>(gamma);
    uint4* av = reinterpret_cast<uint4*>(a + row * lda);
#pragma unroll
    for (int i = 0; i < kRegChunks; ++i) {
      const int c = lane + 32 * i;
      if (c < nchunk) {
        const uint4 g = __ldg(gv + c);
        av[c] = make_uint4(mul_bf16x2(v[i].x, g.x), mul_bf16x2(v[i].y, g.y), mul_bf16x2(v[i].z, g.z),
                           mul_bf16x2(v[i].w, g.w));
      }
    }
  }
}

// Few rows: a whole CTA per row so the row's loads are all in flight at once,
// and CTAs past the last row clear `zero` (the streamed GEMMs' fp32
// accumulators and counters) with 16-byte stores.
constexpr int kRowThreads = 256;
constexpr int kRowChunks = 4;  // 16-byte chunks per thread held in registers: rows of up to 8192 elements

__global__ void __launch_bounds__(kRowThreads) k_rms_prep_rows(const bf16* __restrict__ x, int64_t ldx,
                                                               const bf16* __restrict__ gamma, int M, int K,
                                                               float eps, bf16* __restrict__ a, int64_t lda,
                                                               float* __restrict__ inv, uint4* __restrict__ zero,
                                                               int64_t zero_vecs) {
  // Launched with programmatic serialization, like k_rms_prep.
  grid_dep_wait();
  grid_dep_launch();
  if (blockIdx.x >= M) {
    const int64_t stride = static_cast<int64_t>(gridDim.x - M) * kRowThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x - M) * kRowThreads + threadIdx.x; i < zero_vecs; i += stride)
      zero[i] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const int64_t row = blockIdx.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * ldx);
  const uint4* gv = reinterpret_cast<const uint4*>(gamma);
  uint4* av = reinterpret_cast<uint4*>(a + row * lda);
  const int nchunk = K / 8;
  uint64_t ss2 = 0;
  const bool in_regs = nchunk <= kRowChunks * kRowThreads;
  if (in_regs) {
    // The row and gamma in registers, all loads in flight together; bf16(x *
    // gamma) does not depend on the sum, so it is written at once (one memory
    // round trip on the decode step's critical path instead of two).
    uint4 xr[kRowChunks], gr[kRowChunks];
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nchunk) {
        xr[i] = __ldg(xv + c);
        gr[i] = __ldg(gv + c);
      }
    }
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nchunk) {
        const uint4 v = xr[i], g = gr[i];
        av[c] = make_uint4(mul_bf16x2(v.x, g.x), mul_bf16x2(v.y, g.y), mul_bf16x2(v.z, g.z), mul_bf16x2(v.w, g.w));
        ss2 = sq_acc_bf16x2(ss2, v.x);
        ss2 = sq_acc_bf16x2(ss2, v.y);
        ss2 = sq_acc_bf16x2(ss2, v.z);
        ss2 = sq_acc_bf16x2(ss2, v.w);
      }
    }
  } else {
#pragma unroll 4
    for (int c = threadIdx.x; c < nchunk; c += kRowThreads) {
      const uint4 v = __ldg(xv + c);
      ss2 = sq_acc_bf16x2(ss2, v.x);
      ss2 = sq_acc_bf16x2(ss2, v.y);
      ss2 = sq_acc_bf16x2(ss2, v.z);
      ss2 = sq_acc_bf16x2(ss2, v.w);
    }
  }
  float ss = __uint_as_float(static_cast<uint32_t>(ss2)) + __uint_as_float(static_cast<uint32_t>(ss2 >> 32));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[kRowThreads / 32];
  __shared__ float s_inv;
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < kRowThreads / 32; ++w) t += part[w];
    s_inv = 1.0f / sqrtf(t / static_cast<float>(K) + eps);
    inv[row] = s_inv;
  }
  if (in_regs) return;
#pragma unroll 4
  for (int c = threadIdx.x; c < nchunk; c += kRowThreads) {
    const uint4 v = __ldg(xv + c);
    const uint4 g = __ldg(gv + c);
    av[c] = make_uint4(mul_bf16x2(v.x, g.x), mul_bf16x2(v.y, g.y), mul_bf16x2(v.z, g.z), mul_bf16x2(v.w, g.w));
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int64_t staged_ld(int64_t k) { return (k + 7) / 8 * 8; }

size_t rms_prep_bytes(int64_t m, int64_t k) {
  const size_t a = static_cast<size_t>(m) * static_cast<size_t>(staged_ld(k)) * 2;
  const size_t i = static_cast<size_t>(m) * 4;
  return ((a + 255) & ~size_t(255)) + ((i + 255) & ~size_t(255));
}

int run_rms_prep(const bf16* x, int64_t ldx, const bf16* gamma, int64_t M, int64_t K, float eps, void* ws,
                 bf16** a_out, int64_t* lda_out, float** inv_out, cudaStream_t stream, std::string* err,
                 void* zero, size_t zero_bytes) {
  const int64_t lda = staged_ld(K);
  bf16* a = static_cast<bf16*>(ws);
  const size_t abytes = (static_cast<size_t>(M) * lda * 2 + 255) & ~size_t(255);
  float* inv = reinterpret_cast<float*>(static_cast<char*>(ws) + abytes);
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && al16(x) && al16(gamma) && al16(a);
  *a_out = a;
  *lda_out = lda;
  *inv_out = inv;
  if (vec && M <= 1024 && (zero_bytes % 16) == 0 && al16(zero)) {
    // Few rows: one CTA per row, plus CTAs that clear `zero`.
    const int64_t zvec = static_cast<int64_t>(zero_bytes / 16);
    const int zblocks = zvec ? static_cast<int>(zvec / (kRowThreads * 8) + 1 < 512 ? zvec / (kRowThreads * 8) + 1 : 512)
                             : 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(M) + static_cast<unsigned>(zblocks), 1, 1);
    cfg.blockDim = dim3(kRowThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_rms_prep_rows, x, ldx, gamma, static_cast<int>(M), static_cast<int>(K),
                                       eps, a, lda, inv, static_cast<uint4*>(zero), zvec);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
      if (err) *err = std::string("rmsnorm staging launch: ") + cudaGetErrorString(e);
      return -3;
    }
    count_launch();
    return 0;
  }
  int64_t zvec = 0;
  if (zero_bytes && (zero_bytes % 16) == 0 && al16(zero) && zero_bytes <= (1u << 20)) {
    zvec = static_cast<int64_t>(zero_bytes / 16);  // small regions: cleared by the staging kernel itself
  } else if (zero_bytes) {
    const cudaError_t e = cudaMemsetAsync(zero, 0, zero_bytes, stream);
    if (e != cudaSuccess) {
      if (err) *err = std::string("accumulator clear: ") + cudaGetErrorString(e);
      return -3;
    }
  }
  uint4* zw = zvec ? static_cast<uint4*>(zero) : nullptr;
  const int64_t blocks64 = (M + kWarps - 1) / kWarps;
  const int blocks = static_cast<int>(blocks64 < 65535 * 8 ? blocks64 : 65535 * 8);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int Mi = static_cast<int>(M), Ki = static_cast<int>(K);
  cudaError_t e = vec && K <= kRegChunks * 32 * 8
                      ? cudaLaunchKernelEx(&cfg, k_rms_prep_reg, x, ldx, gamma, Mi, Ki, eps, a, lda, inv, zw, zvec)
                  : vec ? cudaLaunchKernelEx(&cfg, k_rms_prep<true>, x, ldx, gamma, Mi, Ki, eps, a, lda, inv, zw, zvec)
                        : cudaLaunchKernelEx(&cfg, k_rms_prep<false>, x, ldx, gamma, Mi, Ki, eps, a, lda, inv, zw,
                                             zvec);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    if (err) *err = std::string("rmsnorm staging launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

}  // namespace tfb200
