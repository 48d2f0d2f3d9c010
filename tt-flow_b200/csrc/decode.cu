// Decode-shaped fused MLP (few token rows, weights streamed from HBM) and the
// tensor-parallel pieces built on it.
//
//   staging   bf16(x * gamma) and 1/rms per row          (rmsnorm_prep.cu)
//   up        h   = bf16(gelu(inv * (xg @ W1) + b1))     (stream_sm100.cu, kStreamFinishUp)
//   down      y   = bf16(h @ W2 + residual)              (kStreamFinishDown)
//
// Tensor parallel over G GPUs (W1 split by columns, b1 alongside, W2 split by
// rows): every GPU runs staging + up on its shard, then either
//   * the down-projection with the cross-GPU reduction in the same kernel
//     (kStreamTpReduce, tfb200_fused_mlp_tp): each column block is summed on its
//     owner GPU from the ranks' 16-byte pushes and written to every GPU, or
//   * the down-projection as a kStreamPartial into an fp32 [M, N] buffer, one
//     all-reduce across GPUs, and tfb200_residual_add: y = bf16(sum + residual).
#include <string>

#include "../../include/tfb200.h"
#include "internal.h"

namespace tfb200 {

namespace {

size_t al256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

__global__ void k_residual_add(const float* __restrict__ part, int64_t ldp, const bf16* __restrict__ res, int64_t ldr,
                               bf16* __restrict__ y, int64_t ldy, int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    y[m * ldy + n] = __float2bfloat16_rn(part[m * ldp + n] + __bfloat162float(res[m * ldr + n]));
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Workspace of the streamed MLP: hidden block, staging, fp32 up accumulator and
// the up / down column-block counters (the down accumulator is separate).
size_t decode_core_bytes(int64_t m, int64_t k, int64_t h, int64_t n) {
  return al256(static_cast<size_t>(m) * h * 2) + rms_prep_bytes(m, k) + al256(static_cast<size_t>(m) * h * 4) +
         al256(stream_counter_bytes(h)) + al256(stream_counter_bytes(n));
}

size_t decode_mlp_bytes(int64_t m, int64_t k, int64_t h, int64_t n) {
  return decode_core_bytes(m, k, h, n) + al256(static_cast<size_t>(m) * n * 4);
}

bool decode_eligible(int64_t m, const void* w1, int64_t ldw1, const void* w2, int64_t ldw2) {
  return m >= 1 && m <= kStreamMaxRows && al16(w1) && al16(w2) && ldw1 % 8 == 0 && ldw2 % 8 == 0;
}

// Streamed MLP. With out_partial != nullptr the down-projection leaves its fp32
// sum there (ld ldp) instead of adding the residual and rounding.
int run_decode_mlp(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* w1, int64_t ldw1, const bf16* b1,
                   const bf16* w2, int64_t ldw2, const bf16* residual, int64_t ldr, float eps, int gelu, bf16* y,
                   int64_t ldy, float* out_partial, int64_t ldp, int64_t M, int64_t K, int64_t H, int64_t N,
                   void* ws, cudaStream_t s, std::string* err, const TpPeers* tp) {
  char* base = static_cast<char*>(ws);
  bf16* hid = reinterpret_cast<bf16*>(base);
  base += al256(static_cast<size_t>(M) * H * 2);
  void* prep = base;
  base += rms_prep_bytes(M, K);
  float* acc1 = reinterpret_cast<float*>(base);
  base += al256(static_cast<size_t>(M) * H * 4);
  int* cnt1 = reinterpret_cast<int*>(base);
  base += al256(stream_counter_bytes(H));
  int* cnt2 = reinterpret_cast<int*>(base);
  base += al256(stream_counter_bytes(N));
  float* acc2 = out_partial ? out_partial : reinterpret_cast<float*>(base);
  const int64_t ld2 = out_partial ? ldp : N;

  // The fp32 accumulators and the column-block counters start at zero: the
  // staging launch clears the workspace region; a caller's partial buffer with
  // padding between rows is cleared separately.
  const size_t clear_bytes = static_cast<size_t>(reinterpret_cast<char*>(cnt2) - reinterpret_cast<char*>(acc1)) +
                             al256(stream_counter_bytes(N)) +
                             ((out_partial || tp) ? 0 : al256(static_cast<size_t>(M) * N * 4));
  if (out_partial && !tp) {
    const cudaError_t e = ld2 == N ? cudaMemsetAsync(acc2, 0, static_cast<size_t>(M) * N * 4, s)
                                   : cudaMemset2DAsync(acc2, ld2 * 4, 0, N * 4, M, s);
    if (e != cudaSuccess) {
      *err = std::string("decode MLP clear: ") + cudaGetErrorString(e);
      return -3;
    }
  }
  bf16* a = nullptr;
  int64_t lda = 0;
  float* inv = nullptr;
  int rc = run_rms_prep(x, ldx, gamma, M, K, eps, prep, &a, &lda, &inv, s, err, acc1, clear_bytes);
  if (rc) return rc;
  StreamProblem up;
  up.M = M;
  up.N = H;
  up.K = K;
  up.A = a;
  up.lda = lda;
  up.W = w1;
  up.ldw = ldw1;
  up.acc = acc1;
  up.counters = cnt1;
  up.mode = kStreamFinishUp;
  up.col_scale = inv;
  up.bias = b1;
  up.gelu = gelu;
  up.out = hid;
  up.ldo = H;
  rc = run_stream(up, s, err);
  if (rc) return rc;
  if (H % 8 != 0) {
    *err = "decode MLP: hidden width must be a multiple of 8";
    return -2;
  }
  StreamProblem dn;
  dn.M = M;
  dn.N = N;
  dn.K = H;
  dn.A = hid;
  dn.lda = H;
  dn.W = w2;
  dn.ldw = ldw2;
  dn.acc = acc2;
  dn.counters = cnt2;
  if (tp) {
    // Down-projection and the cross-GPU reduction in one kernel. Its local
    // sums and counters live in the tensor-parallel buffer and are returned to
    // zero by the kernel, so nothing to clear here.
    dn.mode = kStreamTpReduce;
    dn.tp = *tp;
    dn.acc = tp->acc;
    dn.counters = tp->local_cnt;
    dn.residual = residual;
    dn.ldr = ldr;
    dn.ldo = N;
  } else if (out_partial) {
    dn.mode = kStreamPartial;
  } else {
    dn.mode = kStreamFinishDown;
    dn.residual = residual;
    dn.ldr = ldr;
    dn.out = y;
    dn.ldo = ldy;
  }
  // The counters and the fp32 accumulator of this pass must not be the ones the
  // up pass used: they are separate regions of the workspace (or the caller's
  // partial buffer).
  if (dn.mode == kStreamFinishDown && ld2 != N) {
    *err = "decode MLP: internal accumulator layout";
    return -3;
  }
  rc = run_stream(dn, s, err);
  return rc;
}

int launch_residual_add(const float* part, int64_t ldp, const bf16* res, int64_t ldr, bf16* y, int64_t ldy,
                        int64_t M, int64_t N, cudaStream_t s, std::string* err) {
  const int64_t total = M * N;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  k_residual_add<<<static_cast<int>(blocks), 256, 0, s>>>(part, ldp, res, ldr, y, ldy, M, N);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string("residual add launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

}  // namespace tfb200
