/*
 * tfb200.h -- C ABI of the B200 (sm_100a) backend for tt-flow's fused hot path:
 * fused RMSNorm+MatMul, fused MLP block (RMSNorm, MatMul+bias+GELU, MatMul,
 * residual add) and plain tiled MatMul.
 *
 * The reference (tensixflow) has no linked ABI for this path: its boundary is
 * the op semantics of python/tensixflow/golden.py:97-122 (checked by the
 * harness, python/tensixflow/harness.py:146-181) and the generated TT-Metalium
 * host program, whose kernels the entry points below replace
 * (lib/tensixflow/Codegen/EmitHost.cpp:100-575 matmul, :581-978 fused
 * RMSNorm+MatMul, :980-1502 fused MLP). Each entry point cites the item it
 * replaces.
 *
 * Conventions
 *  - Matrices are row-major bf16 in device memory, described by tfb200_mat
 *    (ld = leading dimension in elements, >= cols). Vectors (gamma, b1) are
 *    contiguous bf16 device arrays.
 *  - The caller owns every buffer; the library calls no device allocator and
 *    never frees caller memory. The only device memory it holds is static: a
 *    status word and the fixed scratch of tfb200_fused_mlp_noalloc.
 *  - Calls are asynchronous and ordered on `stream` (a cudaStream_t; NULL is the
 *    legacy default stream). Distinct host threads may call concurrently on
 *    distinct streams.
 *  - Return value: TFB200_OK (0) or a negative TFB200_E* code; the message of the
 *    last failure on the calling thread is in tfb200_last_error().
 *  - Device-side waits are bounded. A kernel whose wait runs out returns early and
 *    records TFB200_ETIMEOUT in a per-device status word read by
 *    tfb200_device_status().
 *  - No C++ exception crosses this boundary.
 */
#ifndef TFB200_H_
#define TFB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TFB200_ABI_VERSION 1

enum tfb200_status {
  TFB200_OK = 0,
  TFB200_EINVAL = -1,       /* bad argument: null pointer, shape mismatch, bad ld */
  TFB200_EUNSUPPORTED = -2, /* valid request this backend does not implement */
  TFB200_ECUDA = -3,        /* a CUDA runtime / driver call failed */
  TFB200_ETIMEOUT = -4,     /* a bounded device wait ran out */
  TFB200_EWORKSPACE = -5,   /* workspace missing or smaller than required */
  TFB200_ENOSPC = -6        /* output buffer (text) too small */
};

enum tfb200_dtype { TFB200_BF16 = 0, TFB200_F32 = 1 };

enum tfb200_gelu { TFB200_GELU_ERF = 0, TFB200_GELU_TANH = 1 };

/* A row-major matrix view: data[r * ld + c], r < rows, c < cols. */
typedef struct tfb200_mat {
  void* data;
  int64_t rows;
  int64_t cols;
  int64_t ld;
  int32_t dtype; /* enum tfb200_dtype; the kernels take TFB200_BF16 */
} tfb200_mat;

/* ABI version (TFB200_ABI_VERSION of the built library). */
int tfb200_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* tfb200_last_error(void);

/* C = A @ B, fp32 accumulation, bf16 output (round to nearest even).
 * A [M,K], B [K,N], C [M,N]. Replaces the blocked-reuse / output-tile matmul
 * kernels (EmitCompute.cpp:257-329, :560-650) and the matmul host program
 * (EmitHost.cpp:100-575); semantics of golden.matmul (golden.py:56-60).
 * K == 0 writes zeros; M == 0 or N == 0 is a no-op. */
int tfb200_matmul(const tfb200_mat* a, const tfb200_mat* b, tfb200_mat* c, void* stream);

/* Bytes of device workspace tfb200_fused_rmsnorm_matmul takes for M rows of
 * width K and N outputs: the staged bf16(x * gamma) block and the per-row
 * inverse RMS, plus the fp32 slots and flags of the GEMM's tail split (a short
 * last wave of tiles spread over idle CTA pairs). A workspace that holds only
 * the first part is accepted and runs without the split. */
size_t tfb200_fused_rmsnorm_matmul_workspace_size(int64_t m, int64_t k, int64_t n);

/* Y = rmsnorm(X, gamma, eps) @ W with rmsnorm(x) = x / sqrt(mean_k(x^2) + eps) * gamma.
 * X [M,K], gamma [K], W [K,N], Y [M,N]. One HBM-bound pass stages
 * bf16(x * gamma) and 1/rms per row in `workspace` (>=
 * tfb200_fused_rmsnorm_matmul_workspace_size bytes, 256-byte aligned); the
 * tcgen05 GEMM consumes the staged block and scales each fp32 accumulator row
 * by 1/rms in its epilogue.
 * Replaces the fused RMSNorm+MatMul compute kernel (EmitCompute.cpp:60-255) and
 * host program (EmitHost.cpp:581-978); semantics of golden.fused_rmsnorm_matmul
 * (golden.py:97-102) and of the dialect op tensixflow.fused_rmsnorm_matmul
 * (TensixflowOps.td:230-253; verifier TensixflowOps.cpp:197-278). */
int tfb200_fused_rmsnorm_matmul(const tfb200_mat* x, const void* gamma, const tfb200_mat* w, float eps,
                                tfb200_mat* y, void* stream, void* workspace, size_t workspace_bytes);

/* Bytes of device workspace tfb200_fused_mlp takes for M rows, K model width,
 * H hidden width and N output width: the bf16 hidden activation block, the
 * RMSNorm staging, and the tail-split slots of the two GEMMs (M > 64) or the
 * partial-sum slots and counters of the weight-streaming kernel (M <= 64). For
 * M > 64 a workspace without the tail-split slots is accepted and runs without
 * the split. */
size_t tfb200_fused_mlp_workspace_size(int64_t m, int64_t k, int64_t h, int64_t n);

/* Y = gelu(rmsnorm(X, gamma, eps) @ W1 + b1) @ W2 + R.
 * X [M,K], gamma [K], W1 [K,H], b1 [H] (or NULL for no bias), W2 [H,N],
 * R [M,N] (residual; may alias X when N == K), Y [M,N]. gelu_mode is
 * TFB200_GELU_ERF (the reference's exact form) or TFB200_GELU_TANH.
 * The hidden block is kept as bf16 in `workspace` (>= tfb200_fused_mlp_workspace_size
 * bytes, 256-byte aligned), next to the RMSNorm staging.
 * Replaces the fused MLP compute kernel (EmitCompute.cpp:331-558) and host
 * program (EmitHost.cpp:980-1502); semantics of golden.fused_mlp
 * (golden.py:105-122) and of tensixflow.fused_mlp (TensixflowOps.td:259-285;
 * verifier TensixflowOps.cpp:284-413, which accepts a 1-D [H] bias). */
int tfb200_fused_mlp(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1, const void* b1,
                     const tfb200_mat* w2, const tfb200_mat* residual, float eps, int gelu_mode, tfb200_mat* y,
                     void* stream, void* workspace, size_t workspace_bytes);

/* Tensor-parallel fused MLP, one shard per GPU (the decode-shaped case, M <= 64):
 * partial[M,N] (fp32, leading dimension ld_partial) =
 *     gelu(rmsnorm(X, gamma, eps) @ W1s + b1s) @ W2s
 * where W1s [K, H/G] is this GPU's column shard of W1, b1s the matching slice of
 * b1 and W2s [H/G, N] the matching row shard of W2. Summing `partial` over the G
 * GPUs (one all-reduce) and calling tfb200_residual_add gives tfb200_fused_mlp's
 * result. RMSNorm is computed redundantly on every GPU from the full X. The
 * reference has no multi-device path (its n300 second chip exists only in the
 * planner's arithmetic); this splits the same op (golden.py:105-122). */
size_t tfb200_fused_mlp_partial_workspace_size(int64_t m, int64_t k, int64_t h_shard, int64_t n);
int tfb200_fused_mlp_partial(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1_shard,
                             const void* b1_shard, const tfb200_mat* w2_shard, float eps, int gelu_mode,
                             float* partial, int64_t ld_partial, void* stream, void* workspace,
                             size_t workspace_bytes);

/* Tensor-parallel fused MLP with the all-reduce fused into the down-projection
 * kernel (NVLink peer memory instead of a separate collective). W1 is split by
 * columns (b1 alongside) and W2 by rows; every rank passes the full X, gamma
 * and residual. Each rank sums its partial products for a 128-column block in
 * its own buffer; on the other ranks the CTA completing the block pushes it
 * (fp32, 16-byte stores) into its slot on the block's owner (rank block % world)
 * and arrives there; the owner waits for them, adds the ranks' sums in rank
 * order and the residual, rounds to bf16 and writes the block to every rank's
 * output. The call returns
 * (stream-ordered) once every block has reached this rank; the result is this
 * rank's output buffer (tfb200_tp_output), valid until the next call.
 * Every rank allocates one buffer of tfb200_tp_buffer_bytes(max_rows, n, world)
 * bytes, 256-byte aligned and zero-filled before the first call, shares it
 * (tfb200_ipc_*), and fills `peer_buf` with every rank's buffer as mapped in
 * this process. The kernels return the buffers to zero after each call. All
 * ranks make the same calls with the same shapes, in the same order. Waits are
 * bounded: a timeout sets TFB200_ETIMEOUT in the device status word and leaves
 * the buffers to be zero-filled again. Needs M <= max_rows <= 64, N % 8 == 0,
 * H % 8 == 0 and 16-byte aligned weights and residual with leading dimensions
 * % 8 == 0. No counterpart in the reference, which has no multi-device path. */
#define TFB200_MAX_TP 8
typedef struct tfb200_tp_comm {
  int32_t rank;
  int32_t world;
  int64_t max_rows;                  /* rows the buffers were sized for */
  void* peer_buf[TFB200_MAX_TP];     /* each rank's buffer, as mapped in this process */
} tfb200_tp_comm;
size_t tfb200_tp_buffer_bytes(int64_t max_rows, int64_t n, int32_t world);
/* This rank's bf16 [M, n] result inside its buffer (leading dimension n). */
int tfb200_tp_output(const tfb200_tp_comm* comm, int64_t n, void** out);
int tfb200_fused_mlp_tp(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1_shard, const void* b1_shard,
                        const tfb200_mat* w2_shard, const tfb200_mat* residual, float eps, int gelu_mode,
                        const tfb200_tp_comm* comm, void* stream, void* workspace, size_t workspace_bytes);

/* CUDA IPC of a device buffer between the processes of one node:
 * tfb200_ipc_get writes a 64-byte handle of the allocation holding `ptr` and the
 * offset of `ptr` in it; tfb200_ipc_open maps a peer's handle and returns the
 * peer allocation's base (add the offset); tfb200_ipc_close unmaps it. */
int tfb200_ipc_get(const void* ptr, void* handle64, size_t* offset);
int tfb200_ipc_open(const void* handle64, void** base);
int tfb200_ipc_close(void* base);

/* y = bf16(partial + residual): the last step of the tensor-parallel MLP, after
 * the partial sums have been reduced across GPUs (the residual add of
 * golden.py:122). partial is fp32 with leading dimension ld_partial. */
int tfb200_residual_add(const float* partial, int64_t ld_partial, const tfb200_mat* residual, tfb200_mat* y,
                        void* stream);

/* Size of the fixed device scratch behind tfb200_fused_mlp_noalloc (8 MiB). */
#define TFB200_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

/* tfb200_fused_mlp for callers that cannot allocate device memory -- plugin
 * hosts and inference servers that own every byte of the GPU's memory, or
 * latency-critical loops that must not risk the synchronisation of an
 * allocation. Same arguments and result as tfb200_fused_mlp, minus the
 * workspace: the workspace tfb200_fused_mlp_workspace_size reports (the hidden
 * block and the RMSNorm staging) lives in a fixed TFB200_NOALLOC_SCRATCH_BYTES
 * device array that the library
 * holds on every GPU that loads it, until the process exits. With CUDA's lazy
 * module loading (the default since CUDA 12.2) the array's memory is committed
 * when the module loads on a device, at the latest inside the first call there;
 * a host that reserves all of the GPU's memory makes that first call before it
 * does (or runs with CUDA_MODULE_LOADING=EAGER). Larger problems are
 * refused with TFB200_EINVAL and a message, before any launch. The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture. All calls on a device share the array:
 * calls whose kernels may overlap on the GPU race on it and must be ordered by
 * the caller. Allocates nothing and calls no allocating routine.
 * This entry point has no counterpart in the reference. */
int tfb200_fused_mlp_noalloc(const tfb200_mat* x, const void* gamma, const tfb200_mat* w1, const void* b1,
                             const tfb200_mat* w2, const tfb200_mat* residual, float eps, int gelu_mode,
                             tfb200_mat* y, void* stream);

/* The tensixflow front end of this backend on IR text: parse the dialect
 * subset of the fused path, apply `args` in order (the tensixflow-opt flags
 * --tensixflow-device=b200, --tensixflow-fuse-rmsnorm-matmul,
 * --tensixflow-plan-noc-sharding, --tensixflow-allocate-circular-buffers, or
 * --tensixflow-to-json for the plan JSON of tensixflow-translate) and write the
 * printed IR or JSON, NUL-terminated, to `out`. *needed (if not NULL) receives
 * the size the output needs; TFB200_ENOSPC when `cap` is smaller. Host-only: no
 * device is touched. Replaces tensixflow-opt's pass pipeline for these flags
 * (FuseRmsnormMatmulPass.cpp:203-234, PlanNocShardingPass.cpp:135-304,
 * AllocateCircularBuffersPass.cpp:63-104) and tensixflow-translate's
 * --tensixflow-to-json (tensixflow-translate.cpp:75-222, 291-297), with the B200
 * planner in place of the Tensix planner. */
int tfb200_opt(const char* text, const char* args, char* out, size_t cap, size_t* needed);

/* Re-plan a plan document for the B200: `plan_json_in` is a plan JSON of
 * schema/plan.schema.json written for any device (tensixflow-translate
 * --tensixflow-to-json, tools/tensixflow-translate/tensixflow-translate.cpp:75-222,
 * or tfb200_opt); its `tensors` and `fusion` give the problem. Writes the B200
 * plan JSON (device b200, mapping, CTAs, shared-memory stages, fused_feasible,
 * HBM bytes, time estimate) to `out`; `needed` as for tfb200_opt. Malformed
 * documents give TFB200_EINVAL with the line and column in tfb200_last_error().
 * No counterpart in the reference, which re-plans only from IR. */
int tfb200_plan(const char* plan_json_in, char* out, size_t cap, size_t* needed);

/* Device status word of the current device: TFB200_OK, or TFB200_ETIMEOUT if a
 * kernel's bounded wait ran out since the last clear. Synchronises the device. */
int tfb200_device_status(void);
/* Reset the current device's status word to TFB200_OK. */
int tfb200_clear_device_status(void);

/* Failure-detection self-test: launches one kernel that waits on a device
 * barrier nothing completes. Its bounded wait gives up after limit_ns (at most
 * 10 s) and sets the status word to TFB200_ETIMEOUT; the context stays usable.
 * No counterpart in the reference (its failure handling is host-side exit codes,
 * scripts/run_generated.sh:17-23). */
int tfb200_selftest_bounded_wait(uint64_t limit_ns, void* stream);

/* Wall-time limit of every bounded device wait, in nanoseconds (default 2e9). */
void tfb200_set_wait_limit_ns(uint64_t ns);

/* Number of kernels this library has launched in this process. */
uint64_t tfb200_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* TFB200_H_ */
