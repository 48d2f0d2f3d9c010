// Host-side interfaces shared by the CUDA translation units of libtfb200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kernel_config.h"

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
  // Tail split of the CTA-pair kernel's last wave (pair_sched.h): slots for
  // up to sk_max_slots fp32 partial accumulators and their flags (zero on
  // entry; the kernel returns them to zero). sk_max_slots = 0: no split.
  float* sk_slots = nullptr;
  int* sk_flags = nullptr;
  int sk_max_slots = 0;
  // B is not written by the kernel that precedes this GEMM in the stream (true
  // in the fused paths, where that kernel is the library's own staging pass or
  // up-projection): the pair kernel then requests its first stages of B before
  // it waits for that kernel to complete.
  bool b_stable = false;
};

// Launch the persistent tcgen05 GEMM. Returns 0 or a negative TFB200_E* code with
// a message in *err.
int run_gemm(const GemmProblem& p, cudaStream_t stream, std::string* err);

// Weight-streaming fused MLP for few rows (stream_sm100.cu): one persistent
// launch runs one or two phases, each acc[M,N] = A[M,K] @ W[K,N] split over all
// SMs (partial sums in per-CTA slots, added in CTA order by the CTA that
// completes a 128-column block), then a per-column-block finishing epilogue;
// a grid barrier separates the phases (phase 1 reads what phase 0 wrote).
enum StreamMode : int { kStreamPartial = 0, kStreamFinishUp = 1, kStreamFinishDown = 2, kStreamTpReduce = 3 };
constexpr int kMaxTp = 8;
// Tensor-parallel reduction fused into the down-projection (kStreamTpReduce).
// Each rank first sums its CTAs' partials for a 128-column block (slots added
// in CTA order) into its local buffer. On a rank that does not own the block
// (owner = nb % world), the CTA that completes it locally pushes it, M x 128
// fp32 in 16-byte stores, into its slot on the owner and arrives on the
// owner's counter. On the owner, that CTA waits for the other ranks' arrivals,
// adds the slots and its own sums in rank order plus the residual, rounds,
// writes the block to every rank's output and bumps every rank's done counter.
// Counters are returned to zero by the CTAs done with them.
struct TpPeers {
  int rank = 0, world = 1;
  int64_t slot_stride = 0;          // elements between two source slots (rows capacity x N)
  float* acc = nullptr;             // this rank: fp32 [M, N] local sums
  int* local_cnt = nullptr;         // this rank: per-block local arrivals
  float* slots[kMaxTp] = {};        // per rank: `world` fp32 [M, N] slots, one per source rank
  unsigned int* arrive[kMaxTp] = {};  // per rank: per-block arrivals of the ranks
  bf16* out[kMaxTp] = {};           // per rank: bf16 [M, N] result
  unsigned int* done[kMaxTp] = {};  // per rank: blocks finished for it in this call
};
// Byte offsets of one rank's tensor-parallel buffer (all 256-byte aligned).
struct TpLayout {
  size_t acc, local_cnt, slots, arrive, out, done, total;
};
TpLayout tp_layout(int64_t max_rows, int64_t n, int world);
struct StreamPhase {
  int64_t N = 0, K = 0;
  const bf16* A = nullptr;  // [M, K] tokens (phase 1: the block phase 0 writes)
  int64_t lda = 0;
  const bf16* W = nullptr;  // [K, N] weights
  int64_t ldw = 0;
  int mode = kStreamPartial;
  int* counters = nullptr;           // ceil(N / 128) ints, zero on entry
  const float* col_scale = nullptr;  // [M] (kStreamFinishUp)
  const bf16* bias = nullptr;        // [N] (kStreamFinishUp)
  int gelu = kGeluNone;
  const bf16* residual = nullptr;    // [M, N] (kStreamFinishDown, kStreamTpReduce)
  int64_t ldr = 0;
  bf16* out = nullptr;               // kStreamFinishUp / kStreamFinishDown
  int64_t ldo = 0;
  float* part = nullptr;             // kStreamPartial: fp32 result; kStreamTpReduce: this rank's sums [M, N]
  int64_t ldp = 0;
};
struct StreamProblem {
  int64_t M = 0;
  StreamPhase ph[2];
  int nphases = 1;
  float* slots = nullptr;   // stream_slot_bytes(M, largest N of the phases)
  int* grid_bar = nullptr;  // one int, zero on entry (two phases)
  TpPeers tp;               // kStreamTpReduce
  // Optional, one phase: the weights of the streaming launch that follows on
  // the same stream (only next.W, ldw, N, K are read). Once a CTA has issued its
  // own weight stream it prefetches into L2 the first prefetch_units units of
  // the range the same CTA of that launch will stream, so HBM stays busy while
  // this launch drains. With two phases, prefetch_units units of phase 1 past
  // the shared-memory ring are prefetched before the phase barrier.
  StreamPhase next;
  int prefetch_units = 0;
};
int run_stream(const StreamProblem& p, cudaStream_t stream, std::string* err);
int stream_mpad(int64_t m);
size_t stream_counter_bytes(int64_t n);
size_t stream_slot_bytes(int64_t m, int64_t n_max);

// Streamed (decode-shaped) fused MLP, decode.cu. Used for M <= kStreamMaxRows.
constexpr int64_t kStreamMaxRows = cfg::kStreamMaxRows;
size_t decode_core_bytes(int64_t m, int64_t k, int64_t h, int64_t n);
size_t decode_mlp_bytes(int64_t m, int64_t k, int64_t h, int64_t n);
bool decode_eligible(int64_t m, const void* w1, int64_t ldw1, const void* w2, int64_t ldw2);
int run_decode_mlp(const bf16* x, int64_t ldx, const bf16* gamma, const bf16* w1, int64_t ldw1, const bf16* b1,
                   const bf16* w2, int64_t ldw2, const bf16* residual, int64_t ldr, float eps, int gelu, bf16* y,
                   int64_t ldy, float* out_partial, int64_t ldp, int64_t M, int64_t K, int64_t H, int64_t N,
                   void* ws, cudaStream_t s, std::string* err, const TpPeers* tp = nullptr);
int launch_residual_add(const float* part, int64_t ldp, const bf16* res, int64_t ldr, bf16* y, int64_t ldy,
                        int64_t M, int64_t N, cudaStream_t s, std::string* err);

// Tensor map of a row-major bf16 matrix [rows, cols] (leading dimension ld),
// box of 64 columns x box_rows rows, 128-byte swizzle, zero fill outside.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_rows,
              std::string* err);
bool make_map_box(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                  uint32_t box_rows, CUtensorMapSwizzle swizzle, std::string* err);

// RMSNorm staging pass (rmsnorm_prep.cu): writes bf16(x * gamma) with leading
// dimension staged_ld(K) and inv[m] = 1/sqrt(mean_k(x^2) + eps) into `ws`
// (rms_prep_bytes(M, K) bytes, 256-byte aligned). The same launch clears
// `zero_bytes` bytes at `zero` (accumulators of the streamed GEMMs).
int64_t staged_ld(int64_t k);
size_t rms_prep_bytes(int64_t m, int64_t k);
int run_rms_prep(const bf16* x, int64_t ldx, const bf16* gamma, int64_t M, int64_t K, float eps, void* ws,
                 bf16** a_out, int64_t* lda_out, float** inv_out, cudaStream_t stream, std::string* err,
                 void* zero = nullptr, size_t zero_bytes = 0);

// Minimum workspace of tfb200_fused_mlp (without the tail-split region).
size_t mlp_workspace_min_bytes(int64_t m, int64_t k, int64_t h, int64_t n);

// Workspace region of the pair kernel's tail split for a GEMM of M x N output:
// 0 when the pair kernel does not run (M <= 128). Laid out as
// [flags: sched::flag_bytes()][slots], 256-byte aligned.
size_t pair_split_bytes(int64_t m, int64_t n);

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
