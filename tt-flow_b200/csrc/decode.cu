// Decode-shaped fused MLP (few token rows, weights streamed from HBM) and the
// tensor-parallel pieces built on it.
//
//   staging   bf16(x * gamma) and 1/rms per row          (rmsnorm_prep.cu)
//   one launch of the weight-streaming kernel (stream_sm100.cu), two phases:
//   up        h   = bf16(gelu(inv * (xg @ W1) + b1))     (kStreamFinishUp)
//   down      y   = bf16(h @ W2 + residual)              (kStreamFinishDown)
//
// Tensor parallel over G GPUs (W1 split by columns, b1 alongside, W2 split by
// rows): every GPU runs staging + up on its shard, then either
//   * the down-projection with the cross-GPU reduction in the same kernel
//     (kStreamTpReduce, tfb200_fused_mlp_tp): each column block is summed on its
//     owner GPU from the ranks' 16-byte pushes and written to every GPU, or
//   * the down-projection as a kStreamPartial into an fp32 [M, N] buffer, one
//     all-reduce across GPUs, and tfb200_residual_add: y = bf16(sum + residual).
#include <cstdlib>
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

// The streamed MLP runs as two launches (up, then down) unless
// TFB200_STREAM_LAUNCHES=1 asks for the single two-phase launch.
bool two_launches() {
  static const bool two = [] {
    const char* v = std::getenv("TFB200_STREAM_LAUNCHES");
    return !(v && v[0] == '1');
  }();
  return two;
}

// Units (64 x 128 weight tiles, 16 KiB) per CTA of the down-projection's
// weights prefetched into L2 while the up-projection drains: 32 x 16 KiB x 148
// CTAs = 78 MB, inside the 126 MB L2. Measured on B200 at 32 x 8192 x 28672
// (us per step, two runs each): none 171.9 / 172.6, 24 units 166.7 / 166.8,
// 32 units 166.3 / 166.4, 48 units 167.5 / 167.7, 64 units 170.3 / 170.6 (the
// prefetched tiles no longer fit beside the stream); after the finisher
// changes of the streaming kernel, 16 units 157.8 / 158.2, 24 units 156.1 /
// 156.2, 32 units 155.9 / 155.9, 40 units 156.4 / 156.5. TFB200_STREAM_PREFETCH
// overrides it (0 turns it off).
int prefetch_units() {
  static const int n = [] {
    const char* v = std::getenv("TFB200_STREAM_PREFETCH");
    return v ? std::atoi(v) : 32;
  }();
  return n;
}

}  // namespace

// Workspace of the streamed MLP: hidden block, staging, the partial-sum slots
// of the streaming kernel, then the up / down column-block counters and the
// phase barrier (one region, cleared by the staging launch).
size_t decode_core_bytes(int64_t m, int64_t k, int64_t h, int64_t n) {
  return al256(static_cast<size_t>(m) * h * 2) + rms_prep_bytes(m, k) + al256(stream_slot_bytes(m, h > n ? h : n)) +
         al256(stream_counter_bytes(h) + stream_counter_bytes(n) + sizeof(int));
}

size_t decode_mlp_bytes(int64_t m, int64_t k, int64_t h, int64_t n) { return decode_core_bytes(m, k, h, n); }

bool decode_eligible(int64_t m, const void* w1, int64_t ldw1, const void* w2, int64_t ldw2) {
  return m >= 1 && m <= kStreamMaxRows && al16(w1) && al16(w2) && ldw1 % 8 == 0 && ldw2 % 8 == 0;
}

// Streamed MLP: the staging launch, then one launch of the weight-streaming
// kernel running the up-projection and the down-projection as its two phases.
// With out_partial != nullptr the down-projection leaves its fp32 sum there
// (ld ldp) instead of adding the residual and rounding.
int run_decode_mlp(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* w1, int64_t ldw1, const bf16* b1,
                   const bf16* w2, int64_t ldw2, const bf16* residual, int64_t ldr, float eps, int gelu, bf16* y,
                   int64_t ldy, float* out_partial, int64_t ldp, int64_t M, int64_t K, int64_t H, int64_t N,
                   void* ws, cudaStream_t s, std::string* err, const TpPeers* tp) {
  if (H % 8 != 0) {
    *err = "decode MLP: hidden width must be a multiple of 8";
    return -2;
  }
  char* base = static_cast<char*>(ws);
  bf16* hid = reinterpret_cast<bf16*>(base);
  base += al256(static_cast<size_t>(M) * H * 2);
  void* prep = base;
  base += rms_prep_bytes(M, K);
  float* slots = reinterpret_cast<float*>(base);
  base += al256(stream_slot_bytes(M, H > N ? H : N));
  int* cnt1 = reinterpret_cast<int*>(base);
  int* cnt2 = cnt1 + (H + 127) / 128;
  int* bar = cnt2 + (N + 127) / 128;
  const size_t clear_bytes = al256(stream_counter_bytes(H) + stream_counter_bytes(N) + sizeof(int));

  // The counters and the phase barrier start at zero: the staging launch clears
  // them. Slots, hidden block and outputs are written whole by the kernel.
  bf16* a = nullptr;
  int64_t lda = 0;
  float* inv = nullptr;
  int rc = run_rms_prep(x, ldx, gamma, M, K, eps, prep, &a, &lda, &inv, s, err, cnt1, clear_bytes);
  if (rc) return rc;
  StreamProblem sp;
  sp.M = M;
  sp.nphases = 2;
  sp.slots = slots;
  sp.grid_bar = bar;
  StreamPhase& up = sp.ph[0];
  up.N = H;
  up.K = K;
  up.A = a;
  up.lda = lda;
  up.W = w1;
  up.ldw = ldw1;
  up.counters = cnt1;
  up.mode = kStreamFinishUp;
  up.col_scale = inv;
  up.bias = b1;
  up.gelu = gelu;
  up.out = hid;
  up.ldo = H;
  StreamPhase& dn = sp.ph[1];
  dn.N = N;
  dn.K = H;
  dn.A = hid;
  dn.lda = H;
  dn.W = w2;
  dn.ldw = ldw2;
  dn.counters = cnt2;
  if (tp) {
    // Down-projection and the cross-GPU reduction in the same launch. Its local
    // sums and counters live in the tensor-parallel buffer; the counters are
    // returned to zero by the kernel.
    dn.mode = kStreamTpReduce;
    sp.tp = *tp;
    dn.part = tp->acc;
    dn.counters = tp->local_cnt;
    dn.residual = residual;
    dn.ldr = ldr;
    dn.ldo = N;
  } else if (out_partial) {
    dn.mode = kStreamPartial;
    dn.part = out_partial;
    dn.ldp = ldp;
  } else {
    dn.mode = kStreamFinishDown;
    dn.residual = residual;
    dn.ldr = ldr;
    dn.out = y;
    dn.ldo = ldy;
  }
  sp.prefetch_units = prefetch_units();
  if (!two_launches()) return run_stream(sp, s, err);
  // The two phases as two launches (chained with programmatic dependent
  // launch): the down-projection's launch waits for the up-projection's grid.
  StreamProblem a1 = sp, a2 = sp;
  a1.nphases = 1;
  a2.nphases = 1;
  a2.ph[0] = sp.ph[1];
  a1.next = sp.ph[1];
  a2.prefetch_units = 0;
  rc = run_stream(a1, s, err);
  if (rc) return rc;
  return run_stream(a2, s, err);
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
