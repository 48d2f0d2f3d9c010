// Persistent, warp-specialised tcgen05 GEMM for sm_100a with the fused RMSNorm
// prologue and the bias / GELU / residual epilogue of the tt-flow hot path.
//
// This replaces the Tensix compute kernels that the reference emits as strings:
// the fused RMSNorm+MatMul compute (tensixflow lib/tensixflow/Codegen/
// EmitCompute.cpp:60-255), the fused MLP compute (:331-558) and the plain tiled
// matmul compute (:257-329, :560-650), together with their reader and writer
// kernels (EmitReader.cpp, EmitWriter.cpp).
//
// One CTA per SM walks output tiles of 128 x 256 (grid-stride over a grouped
// raster so that concurrently running tiles share A and B panels in L2).
// Warp roles:
//   warp 0      TMA producer: A tile [128 x 64] (K-major) and B tile [64 x 256]
//               (N-major, four 64-column boxes), 128-byte swizzle, S stages.
//   warp 1      MMA issuer: one thread issues tcgen05.mma 128x256x16 into a
//               double-buffered fp32 accumulator in TMEM (2 x 256 columns).
//   warp 2      TMEM allocator.
//   warps 4-7   epilogue: tcgen05.ld 32 columns at a time, row scale (the
//               RMSNorm inverse RMS), bias, GELU, residual, bf16 round, store.
//   warps 8-11  (only for operands TMA cannot describe: leading dimensions that
//               are not multiples of 8 elements or unaligned pointers) plain-load
//               producer that writes the same swizzled stage layout.
// For the fused RMSNorm paths A is the bf16(x * gamma) block staged by
// rmsnorm_prep.cu and the row scale is its 1/rms vector. (An in-mainloop
// variant that rewrote each TMA-staged A tile in shared memory measured 35%
// slower at 8192x4096x6144: the hand-off, async-proxy fences, gamma loads and
// shared-memory traffic all contend with the MMA pipeline, while the staging
// pass costs one extra HBM round trip of X, 6% of that GEMM.)
// Every wait is bounded; when one runs out the kernel records kDevTimeout in the
// device status word, drains what it issued and returns.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "internal.h"
#include "kernel_config.h"
#include "pair_sched.h"
#include "sm100_ptx.cuh"

namespace tfb200 {

namespace {

constexpr int BM = cfg::kTileM;
constexpr int BN = cfg::kTileN;
constexpr int BK = cfg::kTileK;
constexpr int STAGES = cfg::kStages;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;  // 16 KiB
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;  // 32 KiB
constexpr uint32_t TMEM_COLS = 2 * BN;           // two accumulators
constexpr int GROUP_M = cfg::kGroupM;            // raster group (tiles of M)

struct KParams {
  int M, N, K;
  const bf16* A;
  int64_t lda;
  const bf16* B;
  int64_t ldb;
  bf16* C;
  int64_t ldc;
  const float* row_scale;
  const bf16* bias;
  int gelu;
  const bf16* residual;
  int64_t ldr;
  int vec_ok;     // C / residual / bias allow 16-byte accesses
  int tma_store;  // the pair kernel stores C through shared memory with TMA
  int* status;
  uint64_t timeout_ns;
  // CTA-pair kernel only: the work schedule (pair_sched.h) and, for its tail
  // split, the caller's slots (fp32 partial accumulators) and their flags.
  sched::PairSched ps;
  float* sk_slots;
  int* sk_flags;
  // The preceding kernel in the stream does not write B (the fused paths, where
  // it is this library's staging pass or up-projection): the pair kernel may
  // request its first stages of B before waiting for that kernel.
  int b_prefetch;
};

struct SmemCtl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

static_assert(sizeof(SmemCtl) == cfg::kGemmCtlBytes, "planner's control-block size");

constexpr size_t smem_bytes() {
  return 1024 /*alignment slack*/ + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + sizeof(SmemCtl);
}

// Grouped raster: tiles run down `group` row tiles before moving one column
// tile right, so concurrently running tiles share A and B panels in L2.
template <int GROUP>
__device__ __forceinline__ void tile_coords_g(int t, int num_m, int num_n, int& tm, int& tn) {
  const int per_group = GROUP * num_n;
  const int g = t / per_group;
  const int first_m = g * GROUP;
  const int gsize = min(num_m - first_m, GROUP);
  const int local = t - g * per_group;
  tm = first_m + local % gsize;
  tn = local / gsize;
}
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  tile_coords_g<GROUP_M>(t, num_m, num_n, tm, tn);
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
// tanh form of GELU with the hardware tanh (tanh.approx.f32, relative error
// about 2^-11): well inside the bf16 rounding (2^-9) of the value it produces.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.0f + tanh_approx(u));
}

__device__ __forceinline__ void raise_abort(SmemCtl* ctl, int* status) {
  ctl->abort = 1;
  atomicExch(status, kDevTimeout);
}

// Warp-uniform bounded wait (every lane waits; the warp agrees on the outcome).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, SmemCtl* ctl, const KParams& p) {
  bool ok = mbar_wait(bar, parity, &ctl->abort, p.timeout_ns);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && (threadIdx.x & 31) == 0) raise_abort(ctl, p.status);
  return ok;
}

// GELU (tanh form) on an fp32 pair: with c1 = sqrt(2/pi) and c2 = c1 * 0.044715,
// u = x * (c1 + c2 * x^2) and gelu = h + h * tanh(u) with h = x / 2: three
// packed ops for u, two for the result, tanh per element.
__device__ __forceinline__ uint64_t gelu_tanh2(uint64_t x) {
  const uint64_t c1 = f2(0.7978845608028654f, 0.7978845608028654f);
  const uint64_t c2 = f2(0.035677408136300125f, 0.035677408136300125f);
  const uint64_t half = f2(0.5f, 0.5f);
  const uint64_t u = f2_mul(x, f2_fma(f2_mul(x, x), c2, c1));
  float u0, u1;
  f2_split(u, u0, u1);
  const uint64_t t = f2(tanh_approx(u0), tanh_approx(u1));
  const uint64_t h = f2_mul(x, half);
  return f2_fma(h, t, h);
}

// Row scale, bias, GELU and residual on 32 accumulator columns of one row
// (columns col0 .. col0+31 of `row`), in fp32.
__device__ __forceinline__ void epilogue_values(const KParams& p, const uint32_t (&v)[32], float scale, int64_t row,
                                                int col0, float (&f)[32]) {
  if (p.vec_ok && col0 + 32 <= p.N && p.gelu == kGeluTanh && p.bias && !p.residual) {
    // The MLP up-projection's epilogue on fp32 pairs: scale, bias, GELU.
    const uint64_t s2 = f2(scale, scale);
    const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 b = __ldg(bp + u);
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = u * 8 + 2 * e;
        uint64_t x = f2_mul(f2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), s2);
        x = gelu_tanh2(f2_add(x, f2_from_bf16x2(bw[e])));
        f2_split(x, f[j], f[j + 1]);
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) * scale;
  const bool full = p.vec_ok && (col0 + 32 <= p.N);
  if (p.bias) {
    if (full) {
      const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 b = __ldg(bp + u);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          f[u * 8 + 2 * e] += bf16_lo(bw[e]);
          f[u * 8 + 2 * e + 1] += bf16_hi(bw[e]);
        }
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) f[j] += __bfloat162float(p.bias[col0 + j]);
    }
  }
  if (p.gelu == kGeluErf) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = gelu_erf(f[j]);
  } else if (p.gelu == kGeluTanh) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = gelu_tanh(f[j]);
  }
  if (p.residual) {
    const bf16* rp = p.residual + row * p.ldr + col0;
    if (full) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 b = *reinterpret_cast<const uint4*>(rp + u * 8);
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          f[u * 8 + 2 * e] += bf16_lo(bw[e]);
          f[u * 8 + 2 * e + 1] += bf16_hi(bw[e]);
        }
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) f[j] += __bfloat162float(rp[j]);
    }
  }
}

// epilogue_values, then bf16 round and direct 16-byte stores.
__device__ __forceinline__ void epilogue_chunk(const KParams& p, const uint32_t (&v)[32], float scale, int64_t row,
                                               int col0) {
  float f[32];
  epilogue_values(p, v, scale, row, col0, f);
  const bool full = p.vec_ok && (col0 + 32 <= p.N);
  bf16* cp = p.C + row * p.ldc + col0;
  if (full) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint4 o;
      o.x = pack_bf16(f[u * 8 + 0], f[u * 8 + 1]);
      o.y = pack_bf16(f[u * 8 + 2], f[u * 8 + 3]);
      o.z = pack_bf16(f[u * 8 + 4], f[u * 8 + 5]);
      o.w = pack_bf16(f[u * 8 + 6], f[u * 8 + 7]);
      *reinterpret_cast<uint4*>(cp + u * 8) = o;
    }
  } else {
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) cp[j] = __float2bfloat16_rn(f[j]);
  }
}

template <bool MANUAL>
struct Roles {
  static constexpr int kLoadWarp0 = 8;
  static constexpr int kThreads = 256 + (MANUAL ? 128 : 0);
};

template <bool MANUAL>
__global__ void __launch_bounds__(Roles<MANUAL>::kThreads, 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(sB + STAGES * B_STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int kLoadWarp0 = Roles<MANUAL>::kLoadWarp0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), MANUAL ? 128 : 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl->tfull[b]), 1);
      mbar_init(smem_u32(&ctl->tempty[b]), 128);
    }
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    if (!MANUAL) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
    }
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(&ctl->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;

  const int num_m = (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int total = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (warp == 0 && !MANUAL) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;  // stages with loads in flight (for the drain)
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
  int tm, tn;
  tile_coords(t, num_m, num_n, tm, tn);
  for (int kb = 0; kb < kblocks; ++kb) {
    if (!mbar_wait(smem_u32(&ctl->empty[stage]), phase ^ 1u, &ctl->abort, p.timeout_ns)) {
      raise_abort(ctl, p.status);
      ok = false;
      break;
    }
    const uint32_t fb = smem_u32(&ctl->full[stage]);
    mbar_arrive_expect_tx(fb, A_STAGE_BYTES + B_STAGE_BYTES);
    tma_load_2d(smem_u32(sA + stage * A_STAGE_BYTES), &tmA, fb, kb * BK, tm * BM);
#pragma unroll
    for (int j = 0; j < BN / 64; ++j)
      tma_load_2d(smem_u32(sB + stage * B_STAGE_BYTES + j * 8192), &tmB, fb, tn * BN + j * 64, kb * BK);
    armed |= 1u << stage;
    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
      }
      if (!ok) {
  // Let the copies already issued land before the CTA's shared memory goes away.
  for (int s = 0; s < STAGES; ++s)
    if (armed & (1u << s)) {
      const uint64_t t0 = global_ns();
      while (!mbar_test(smem_u32(&ctl->full[s]), (armed_phase >> s) & 1u) &&
             global_ns() - t0 < p.timeout_ns) {
      }
    }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int i = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
  const int acc = i & 1;
  const uint32_t use = static_cast<uint32_t>(i >> 1);
  if (!mbar_wait(smem_u32(&ctl->tempty[acc]), (use & 1u) ^ 1u, &ctl->abort, p.timeout_ns)) {
    raise_abort(ctl, p.status);
    ok = false;
    break;
  }
  tc_fence_after();
  const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
  for (int kb = 0; kb < kblocks && ok; ++kb) {
    if (!mbar_wait(smem_u32(&ctl->full[stage]), phase, &ctl->abort, p.timeout_ns)) {
      raise_abort(ctl, p.status);
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t a0 = smem_u32(sA + stage * A_STAGE_BYTES);
    const uint32_t b0 = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
    for (int k = 0; k < BK / 16; ++k) {
      const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);
      const uint64_t bd = sdesc_sw128(b0 + k * 2048, 8192, 1024);
      mma_bf16(d, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
    }
    if (!ok) break;
    mma_commit(smem_u32(&ctl->empty[stage]));
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
  if (ok) mma_commit(smem_u32(&ctl->tfull[acc]));
      }
      // Wait until every MMA this thread issued has finished (TMEM is freed below).
      mma_commit(smem_u32(&ctl->drain));
      const uint64_t t0 = global_ns();
      while (!mbar_test(smem_u32(&ctl->drain), 0) && global_ns() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = q * 32 + lane;
    int i = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      const int acc = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      if (!warp_wait(smem_u32(&ctl->tfull[acc]), use & 1u, ctl, p)) break;
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * BM + r;
      const float scale = (p.row_scale && row < p.M) ? __ldg(p.row_scale + row) : 1.0f;
      for (int c = 0; c < BN / 32; ++c) {
  const int col0 = tn * BN + c * 32;
  if (col0 >= p.N) break;  // warp-uniform
  uint32_t v[32];
  tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + c * 32),
                 v);
  tmem_wait_ld();
  if (row < p.M) epilogue_chunk(p, v, scale, row, col0);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->tempty[acc]));
    }
  } else if (MANUAL && warp >= kLoadWarp0 && warp < kLoadWarp0 + 4) {
    // ------------------------------------------------- plain-load producer
    const int tid = threadIdx.x - kLoadWarp0 * 32;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      for (int kb = 0; kb < kblocks; ++kb) {
  if (!warp_wait(smem_u32(&ctl->empty[stage]), phase ^ 1u, ctl, p)) {
    ok = false;
    break;
  }
  // A: thread tid owns row tid of the tile.
  {
    const int64_t gm = static_cast<int64_t>(tm) * BM + tid;
    uint8_t* rowp = sA + stage * A_STAGE_BYTES + tid * 128;
    for (int c = 0; c < 8; ++c) {
      uint32_t w[4];
      for (int e = 0; e < 4; ++e) {
        const int k = kb * BK + c * 8 + 2 * e;
        float lo = 0.f, hi = 0.f;
        if (gm < p.M && k < p.K) lo = __bfloat162float(p.A[gm * p.lda + k]);
        if (gm < p.M && k + 1 < p.K) hi = __bfloat162float(p.A[gm * p.lda + k + 1]);
        w[e] = pack_bf16(lo, hi);
      }
      *reinterpret_cast<uint4*>(rowp + ((c ^ (tid & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  // B: thread tid owns k-row tid/2 and 128 of the 256 columns.
  {
    const int kr = tid >> 1;
    const int64_t gk = static_cast<int64_t>(kb) * BK + kr;
    for (int cc = 0; cc < 16; ++cc) {
      const int nl = (tid & 1) * 128 + cc * 8;
      uint32_t w[4];
      for (int e = 0; e < 4; ++e) {
        const int64_t n = static_cast<int64_t>(tn) * BN + nl + 2 * e;
        float lo = 0.f, hi = 0.f;
        if (gk < p.K && n < p.N) lo = __bfloat162float(p.B[gk * p.ldb + n]);
        if (gk < p.K && n + 1 < p.N) hi = __bfloat162float(p.B[gk * p.ldb + n + 1]);
        w[e] = pack_bf16(lo, hi);
      }
      uint8_t* dst = sB + stage * B_STAGE_BYTES + (nl >> 6) * 8192 + kr * 128 +
                     ((((nl & 63) >> 3) ^ (kr & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  fence_proxy_async_smem();
  mbar_arrive(smem_u32(&ctl->full[stage]));
  if (++stage == STAGES) {
    stage = 0;
    phase ^= 1u;
  }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ----------------------------------------------------------- CTA-pair kernel
//
// Same contract as k_gemm, with a 256 x 256 output tile per pair of CTAs
// (cluster of 2) and tcgen05.mma.cta_group::2: each CTA stages its own 128 rows
// of A and its own 128 columns of B per 64-deep k block (16 + 16 KiB), the
// leader CTA issues one 256x256x16 MMA over both CTAs' shared memory, and each
// CTA's TMEM receives its 128 rows of the fp32 accumulator. Halving the B bytes
// staged per CTA frees shared memory for six stages instead of four.
// Barriers: both CTAs' TMA loads complete on the leader's `full` barrier (armed
// by the leader with both CTAs' bytes); the leader's MMA thread signals each
// CTA's `empty` and `tfull` barrier; both CTAs' epilogue warps arrive on the
// leader's `tempty` barrier. Every wait is bounded.
constexpr int PSTAGES = cfg::kPairStages;
constexpr int PBM = 2 * BM;                       // rows per pair tile
constexpr uint32_t PB_STAGE_BYTES = BM * BK * 2;  // this CTA's 128 of the 256 B columns

struct PairCtl {
  uint64_t full[PSTAGES];
  uint64_t empty[PSTAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// Epilogue staging for TMA stores: per epilogue warp two 32 x 32 bf16 buffers.
constexpr int PEPI = cfg::kPairEpiWarps;  // epilogue warps 4 .. 4 + PEPI - 1
constexpr int PCHUNKS = BN / 32 / (PEPI / 4);  // 32-column chunks per epilogue warp
constexpr uint32_t C_STAGE_BYTES = 32 * 32 * 2;
constexpr uint32_t C_STAGING_BYTES = PEPI * 2 * C_STAGE_BYTES;
static_assert(PEPI == 8 && PCHUNKS == 4, "two epilogue warps per TMEM lane quadrant");
static_assert(C_STAGING_BYTES == cfg::kPairStagingBytes, "planner's epilogue staging size");
static_assert(sizeof(PairCtl) == cfg::kPairCtlBytes, "planner's pair control-block size");
static_assert(PBM == cfg::kPairTileM, "planner's pair tile");

constexpr size_t pair_smem_bytes() {
  return 1024 + PSTAGES * (A_STAGE_BYTES + PB_STAGE_BYTES) + C_STAGING_BYTES + sizeof(PairCtl);
}

__device__ __forceinline__ void raise_abort_pair(PairCtl* ctl, int* status) {
  ctl->abort = 1;
  atomicExch(status, kDevTimeout);
}

// GROUP: raster group (row tiles) of the pair tiles; see launch_pair.
template <int GROUP>
__global__ void __launch_bounds__(cfg::kPairThreads, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + PSTAGES * A_STAGE_BYTES;
  uint8_t* sC = sB + PSTAGES * PB_STAGE_BYTES;
  PairCtl* ctl = reinterpret_cast<PairCtl*>(sC + C_STAGING_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl->tfull[b]), 1);
      mbar_init(smem_u32(&ctl->tempty[b]), 2 * PEPI);  // the epilogue warps of both CTAs
    }
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (p.tma_store) tma_prefetch_desc(&tmC);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_u32(&ctl->tmem_base), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // Programmatic dependent launch: the next grid in the stream may place its CTAs
  // as this grid's CTAs exit (its prologue overlaps this grid's tail); this grid
  // touches no global memory before the preceding grid has completed.
  grid_dep_launch();
  if (warp != 0) grid_dep_wait();  // the producer waits below, after its weight prefetch

  const int pair = blockIdx.x >> 1;
  const sched::PairSched& ps = p.ps;  // ps.pairs == gridDim.x / 2 (the launcher sets it)
  const int nwork = sched::work_count(ps, pair);
  const int num_m = (p.M + PBM - 1) / PBM;
  const int num_n = (p.N + BN - 1) / BN;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // Weight prefetch: the first item's first stages of B (which the preceding
      // kernel does not write) are requested while that kernel finishes; their
      // stages are armed for A and B now, and A follows after the wait. The
      // stages are fresh, so no `empty` wait precedes them.
      int npre = 0;
      if (p.b_prefetch && nwork > 0) {
        const sched::Work w = sched::work_item(ps, pair, 0);
        int tm, tn;
        tile_coords_g<GROUP>(w.tile, num_m, num_n, tm, tn);
        npre = min(PSTAGES, w.k1 - w.k0);
        for (int s = 0; s < npre; ++s) {
          const uint32_t fb = mapa_shared(smem_u32(&ctl->full[s]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&ctl->full[s]), 2 * (A_STAGE_BYTES + PB_STAGE_BYTES));
#pragma unroll
          for (int j = 0; j < 2; ++j)
            tma_load_2d_pair(smem_u32(sB + s * PB_STAGE_BYTES + j * 8192), &tmB, fb,
                             tn * BN + static_cast<int>(rank) * 128 + j * 64, (w.k0 + s) * BK);
        }
      }
      grid_dep_wait();
      for (int i = 0; i < nwork && ok; ++i) {
        const sched::Work w = sched::work_item(ps, pair, i);
        int tm, tn;
        tile_coords_g<GROUP>(w.tile, num_m, num_n, tm, tn);
        for (int kb = w.k0; kb < w.k1; ++kb) {
          const bool pre = i == 0 && kb - w.k0 < npre;  // armed, B in flight
          if (!pre && !mbar_wait(smem_u32(&ctl->empty[stage]), phase ^ 1u, &ctl->abort, p.timeout_ns)) {
            raise_abort_pair(ctl, p.status);
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&ctl->full[stage]), 0);
          if (leader && !pre)
            mbar_arrive_expect_tx(smem_u32(&ctl->full[stage]), 2 * (A_STAGE_BYTES + PB_STAGE_BYTES));
          tma_load_2d_pair(smem_u32(sA + stage * A_STAGE_BYTES), &tmA, fb, kb * BK,
                           tm * PBM + static_cast<int>(rank) * BM);
          if (!pre) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              tma_load_2d_pair(smem_u32(sB + stage * PB_STAGE_BYTES + j * 8192), &tmB, fb,
                               tn * BN + static_cast<int>(rank) * 128 + j * 64, kb * BK);
          }
          if (++stage == PSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Copies already issued land within microseconds; give them time before
        // the cluster tears down.
        const uint64_t t0 = global_ns();
        while (global_ns() - t0 < 1000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------- MMA issuer (leader)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16(PBM, BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < nwork && ok; ++i) {
        const sched::Work w = sched::work_item(ps, pair, i);
        const int acc = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!mbar_wait(smem_u32(&ctl->tempty[acc]), (use & 1u) ^ 1u, &ctl->abort, p.timeout_ns)) {
          raise_abort_pair(ctl, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = w.k0; kb < w.k1 && ok; ++kb) {
          if (!mbar_wait(smem_u32(&ctl->full[stage]), phase, &ctl->abort, p.timeout_ns)) {
            raise_abort_pair(ctl, p.status);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * PB_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b0 + k * 2048, 8192, 1024);
            mma_bf16_pair(d, ad, bd, idesc, (kb != w.k0 || k != 0) ? 1u : 0u);
          }
          mma_commit_pair_both(smem_u32(&ctl->empty[stage]), 0x3);
          if (++stage == PSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) {
          mma_commit_pair_both(smem_u32(&ctl->tfull[acc]), 0x3);
        }
      }
      mma_commit_pair(smem_u32(&ctl->drain));
      const uint64_t t0 = global_ns();
      while (!mbar_test(smem_u32(&ctl->drain), 0) && global_ns() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------- epilogue (both CTAs)
    // Warp w reads TMEM lane quadrant q = w % 4 (rows q*32 .. q*32+31 of this
    // CTA's 128) and the column chunks [c0, c0 + PCHUNKS) of the tile.
    const int q = warp & 3;
    const int ew = warp - 4;                 // epilogue warp 0 .. PEPI-1
    const int c0 = (ew >> 2) * PCHUNKS;      // first of this warp's 32-column chunks
    const int r = q * 32 + lane;
    for (int i = 0; i < nwork; ++i) {
      const sched::Work w = sched::work_item(ps, pair, i);
      int tm, tn;
      tile_coords_g<GROUP>(w.tile, num_m, num_n, tm, tn);
      const int acc = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      bool ok = mbar_wait(smem_u32(&ctl->tfull[acc]), use & 1u, &ctl->abort, p.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) raise_abort_pair(ctl, p.status);
        break;
      }
      tc_fence_after();
      const int64_t row0 = static_cast<int64_t>(tm) * PBM + static_cast<int64_t>(rank) * BM + q * 32;
      const int64_t row = row0 + lane;
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (w.role == sched::kPart) {
        // Helper part of a split tile: this warp's 32 rows of the fp32
        // accumulator go to the part's slot (layout [chunk][column / 4][row][4],
        // so each warp-wide 16-byte store covers 512 contiguous bytes), then the
        // warp's flag is raised. Warps whose rows are all past the matrix skip
        // both, as the main pair's matching warp skips the wait.
        if (row0 < p.M) {
          float4* slot = reinterpret_cast<float4*>(p.sk_slots + (static_cast<int64_t>(w.slot) * 2 + rank) * (BM * BN)) + r;
          int* flag = p.sk_flags + ((w.slot * 2 + static_cast<int>(rank)) * PEPI + ew) * PCHUNKS;
          for (int c = c0; c < c0 + PCHUNKS; ++c) {
            if (tn * BN + c * 32 >= p.N) break;  // warp-uniform
            uint32_t v[32];
            tmem_ld_32cols(tacc + static_cast<uint32_t>(c * 32), v);
            tmem_wait_ld();
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4)
              __stcg(slot + (c * 8 + j4) * BM, make_float4(__uint_as_float(v[4 * j4]), __uint_as_float(v[4 * j4 + 1]),
                                                          __uint_as_float(v[4 * j4 + 2]),
                                                          __uint_as_float(v[4 * j4 + 3])));
            // Each lane publishes its row of the chunk: the chunk's counter
            // reaches 32 once every row is in L2 (release covers the lane's stores).
            red_add_release_gpu(flag + (c - c0), 1);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const uint32_t te = smem_u32(&ctl->tempty[acc]);
          if (leader)
            mbar_arrive(te);
          else
            mbar_arrive_cluster(mapa_shared(te, 0));
        }
        continue;
      }
      const bool fix = w.role == sched::kMain && row0 < p.M;
      bool fix_ok = true;
      const float scale = (p.row_scale && row < p.M) ? __ldg(p.row_scale + row) : 1.0f;
      for (int c = c0; c < c0 + PCHUNKS; ++c) {
        const int col0 = tn * BN + c * 32;
        if (col0 >= p.N || row0 >= p.M) break;  // warp-uniform: nothing of this block is in the matrix
        uint32_t v[32];
        tmem_ld_32cols(tacc + static_cast<uint32_t>(c * 32), v);
        tmem_wait_ld();
        if (fix) {
          // Own k-blocks [0, kc) first, then the parts in k order: a fixed order.
          // Each lane waits for its row of the part's chunk (the helper lane that
          // wrote it released the chunk's counter).
          for (int j = 0; j < ps.parts && fix_ok; ++j) {
            const int* f = p.sk_flags + (((w.slot + j) * 2 + static_cast<int>(rank)) * PEPI + ew) * PCHUNKS + (c - c0);
            if (ld_acquire_gpu(f) != 32) {
              const uint64_t t0 = global_ns();
              while (ld_acquire_gpu(f) != 32) {
                if (ctl->abort || global_ns() - t0 > p.timeout_ns) {
                  fix_ok = false;
                  break;
                }
              }
            }
            if (!__all_sync(0xffffffffu, fix_ok)) {
              fix_ok = false;
              break;
            }
            const float4* slot =
                reinterpret_cast<const float4*>(p.sk_slots + (static_cast<int64_t>(w.slot + j) * 2 + rank) * (BM * BN)) +
                r + c * 8 * BM;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 a = __ldcg(slot + j4 * BM);
              v[4 * j4] = __float_as_uint(__uint_as_float(v[4 * j4]) + a.x);
              v[4 * j4 + 1] = __float_as_uint(__uint_as_float(v[4 * j4 + 1]) + a.y);
              v[4 * j4 + 2] = __float_as_uint(__uint_as_float(v[4 * j4 + 2]) + a.z);
              v[4 * j4 + 3] = __float_as_uint(__uint_as_float(v[4 * j4 + 3]) + a.w);
            }
          }
          if (!fix_ok) {
            if (lane == 0) raise_abort_pair(ctl, p.status);
            break;
          }
        }
        if (!p.tma_store) {
          if (row < p.M) epilogue_chunk(p, v, scale, row, col0);
          continue;
        }
        // Stage the warp's 32 x 32 bf16 block (64-byte swizzle: 16-byte chunk u
        // of row r sits at chunk u ^ ((r >> 1) & 3), conflict-free for 8 rows)
        // and store it with one TMA; rows / columns past the matrix are clipped.
        float f[32];
        if (row < p.M) {
          epilogue_values(p, v, scale, row, col0, f);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = 0.0f;
        }
        if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
        __syncwarp();
        const uint32_t buf = smem_u32(sC) + static_cast<uint32_t>((ew * 2 + (c & 1)) * C_STAGE_BYTES);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t a = buf + static_cast<uint32_t>(lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4));
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pack_bf16(f[u * 8 + 0], f[u * 8 + 1])),
                       "r"(pack_bf16(f[u * 8 + 2], f[u * 8 + 3])), "r"(pack_bf16(f[u * 8 + 4], f[u * 8 + 5])),
                       "r"(pack_bf16(f[u * 8 + 6], f[u * 8 + 7]))
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf, col0, static_cast<int32_t>(row0));
          bulk_commit();
        }
      }
      if (!fix_ok) break;
      if (fix) {
        // The parts are consumed: return the counters to zero for the next launch.
        __syncwarp();
        if (lane < ps.parts * PCHUNKS)
          st_relaxed_gpu(p.sk_flags + (((w.slot + lane / PCHUNKS) * 2 + static_cast<int>(rank)) * PEPI + ew) * PCHUNKS +
                             lane % PCHUNKS,
                         0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t te = smem_u32(&ctl->tempty[acc]);
        if (leader)
          mbar_arrive(te);
        else
          mbar_arrive_cluster(mapa_shared(te, 0));
      }
    }
  }
  if (warp >= 4 && lane == 0 && p.tma_store) bulk_wait_all();  // staged stores have left shared memory
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers or shared memory
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn(std::string* err) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn && err) *err = "cuTensorMapEncodeTiled is unavailable from the CUDA driver";
  return fn;
}

}  // namespace

// Row-major bf16 matrix [rows, cols] with leading dimension ld: box of
// 64 (cols) x box_rows, 128-byte swizzle, zero fill outside the matrix.
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_rows,
              std::string* err) {
  return make_map_box(m, base, rows, cols, ld, 64, box_rows, CU_TENSOR_MAP_SWIZZLE_128B, err);
}

bool make_map_box(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, uint32_t box_cols,
                  uint32_t box_rows, CUtensorMapSwizzle swizzle, std::string* err) {
  auto fn = encode_fn(err);
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err) *err = "cuTensorMapEncodeTiled failed (CUresult " + std::to_string(static_cast<int>(r)) + ")";
    return false;
  }
  return true;
}

namespace {

// The pair kernel splits the tail of its last wave (pair_sched.h) when the
// caller's workspace holds the slots and the split shortens the busiest pair's
// work by at least 2 %. TFB200_GEMM_SCHED=dp turns the split off, =split takes
// it for any gain (both for measurements).
int split_min_gain_permille() {
  static const int v = [] {  // initialised once, thread-safe
    const char* e = std::getenv("TFB200_GEMM_SCHED");
    if (e && std::string(e) == "dp") return -1;
    if (e && std::string(e) == "split") return 0;
    return 20;
  }();
  return v;
}

// Most tail parts one helper pair takes (pair_sched.h plan()); 1 unless
// TFB200_GEMM_PARTS_PER_HELPER says otherwise (for measurements).
int parts_per_helper() {
  static const int v = [] {
    const char* e = std::getenv("TFB200_GEMM_PARTS_PER_HELPER");
    const int n = e ? std::atoi(e) : 1;
    return n >= 1 ? n : 1;
  }();
  return v;
}

template <bool MANUAL>
int launch(const KParams& kp, const CUtensorMap& ta, const CUtensorMap& tb, int grid, cudaStream_t s,
           std::string* err) {
  auto kern = k_gemm<MANUAL>;
  // Per-device first-call setup; calls may come from several host threads.
  static std::mutex mu;
  static std::atomic<bool> ready[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = smem_bytes();
  if (dev >= 0 && dev < 64 && !ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev].load(std::memory_order_relaxed)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) {
        if (err) *err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
        return -3;
      }
      ready[dev].store(true, std::memory_order_release);
    }
  }
  kern<<<grid, Roles<MANUAL>::kThreads, smem, s>>>(ta, tb, kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    if (err) *err = std::string("gemm launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

template <int GROUP>
int launch_pair_g(const KParams& kp_in, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  int pair_tiles, int max_slots, cudaStream_t s, std::string* err) {
  const auto kern = k_gemm_pair<GROUP>;
  // Per-device first-call setup; calls may come from several host threads.
  static std::mutex mu;
  static std::atomic<bool> ready[64];
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = pair_smem_bytes();
  if (dev < 0 || dev >= 64) {
    if (err) *err = "device index out of range";
    return -3;
  }
  std::unique_lock<std::mutex> lock(mu, std::defer_lock);
  if (!ready[dev].load(std::memory_order_acquire)) lock.lock();
  if (!ready[dev].load(std::memory_order_relaxed)) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e != cudaSuccess) {
      if (err) *err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
      return -3;
    }
    // Persistent pairs: launch no more clusters than can be resident at once.
    cudaLaunchConfig_t q{};
    q.gridDim = dim3(static_cast<unsigned>(sm_count()), 1, 1);
    q.blockDim = dim3(cfg::kPairThreads, 1, 1);
    q.dynamicSmemBytes = smem;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &q);
    if (e != cudaSuccess || n <= 0) {
      if (err) *err = std::string("cudaOccupancyMaxActiveClusters: ") + cudaGetErrorString(e);
      return -3;
    }
    max_clusters[dev] = n;
    ready[dev].store(true, std::memory_order_release);
  }
  if (lock.owns_lock()) lock.unlock();
  // The tail split is planned over every resident pair (the helpers are the
  // pairs a short last wave leaves idle); without it, no more pairs than tiles.
  KParams kp = kp_in;
  const int kblocks = (kp.K + BK - 1) / BK;
  const int gain = split_min_gain_permille();
  kp.ps = sched::plan(pair_tiles, kblocks, max_clusters[dev], gain >= 0 ? max_slots : 0, gain >= 0 ? gain : 0,
                      parts_per_helper());
  if (kp.ps.rem == 0) {
    const int used = pair_tiles < max_clusters[dev] ? pair_tiles : max_clusters[dev];
    kp.ps = sched::plan(pair_tiles, kblocks, used, 0);
  }
  const int pairs = kp.ps.pairs;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(cfg::kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, kp);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    if (err) *err = std::string("pair gemm launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

// Long-K products (K >= 8192, such as the MLP down-projection) run with raster
// groups of 8 row tiles, the rest with 16. In a burst A/B on one GPU, groups of
// 8 ran the 8192x16384x4096 down-projection 1.1 % faster; the 8192x4096x16384
// up-projection keeps 16.
int launch_pair(const KParams& kp, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                int pair_tiles, int max_slots, cudaStream_t s, std::string* err) {
  return kp.K >= 8192 ? launch_pair_g<8>(kp, ta, tb, tc, pair_tiles, max_slots, s, err)
                      : launch_pair_g<GROUP_M>(kp, ta, tb, tc, pair_tiles, max_slots, s, err);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernel choice for TMA-describable operands: the CTA-pair kernel unless
// TFB200_GEMM_KERNEL=single, or when the problem has too few rows to fill a
// 256-row pair tile.
// Stores through shared memory and TMA unless TFB200_GEMM_STORE=direct.
bool tma_store_enabled() {
  static const bool on = [] {  // initialised once, thread-safe
    const char* v = std::getenv("TFB200_GEMM_STORE");
    return !(v && std::string(v) == "direct");
  }();
  return on;
}

bool use_pair(int64_t M) {
  static const bool pair = [] {  // initialised once, thread-safe
    const char* v = std::getenv("TFB200_GEMM_KERNEL");
    return !(v && std::string(v) == "single");
  }();
  return pair && M > BM;
}

}  // namespace

int run_gemm(const GemmProblem& g, cudaStream_t stream, std::string* err) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) {
    if (err) *err = "run_gemm: empty problem";
    return -1;
  }
  if (g.M > (1ll << 31) / 2 || g.N > (1ll << 31) / 2 || g.K > (1ll << 31) / 2) {
    if (err) *err = "run_gemm: dimension too large";
    return -2;
  }
  int* status = device_status_ptr(err);
  if (!status) return -3;
  KParams kp{};
  kp.M = static_cast<int>(g.M);
  kp.N = static_cast<int>(g.N);
  kp.K = static_cast<int>(g.K);
  kp.A = g.A;
  kp.lda = g.lda;
  kp.B = g.B;
  kp.ldb = g.ldb;
  kp.C = g.C;
  kp.ldc = g.ldc;
  kp.row_scale = g.row_scale;
  kp.bias = g.bias;
  kp.gelu = g.gelu;
  kp.residual = g.residual;
  kp.ldr = g.ldr;
  kp.vec_ok = (g.ldc % 8 == 0) && aligned16(g.C) && (!g.residual || (g.ldr % 8 == 0 && aligned16(g.residual))) &&
              (!g.bias || aligned16(g.bias));
  kp.status = status;
  kp.timeout_ns = wait_limit_ns();

  // TMA needs 16-byte aligned bases and row strides.
  const bool tma_ok = aligned16(g.A) && aligned16(g.B) && (g.lda % 8 == 0) && (g.ldb % 8 == 0);
  const int num_tiles = static_cast<int>(((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN));
  const int grid = num_tiles < sm_count() ? num_tiles : sm_count();

  CUtensorMap ta{}, tb{};
  if (tma_ok) {
    if (!make_map(&ta, g.A, g.M, g.K, g.lda, BM, err)) return -3;
    if (!make_map(&tb, g.B, g.K, g.N, g.ldb, BK, err)) return -3;
    if (use_pair(g.M)) {
      const int pair_tiles = static_cast<int>(((g.M + PBM - 1) / PBM) * ((g.N + BN - 1) / BN));
      CUtensorMap tc{};
      kp.tma_store = aligned16(g.C) && g.ldc % 8 == 0 && tma_store_enabled();
      if (kp.tma_store && !make_map_box(&tc, g.C, g.M, g.N, g.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B, err)) return -3;
      kp.b_prefetch = g.b_stable ? 1 : 0;
      int max_slots = 0;
      if (g.sk_slots && g.sk_flags && g.sk_max_slots > 0) {
        kp.sk_slots = g.sk_slots;
        kp.sk_flags = g.sk_flags;
        max_slots = g.sk_max_slots;
      }
      return launch_pair(kp, ta, tb, tc, pair_tiles, max_slots, stream, err);
    }
    return launch<false>(kp, ta, tb, grid, stream, err);
  }
  return launch<true>(kp, ta, tb, grid, stream, err);
}

size_t pair_split_bytes(int64_t m, int64_t n) {
  if (m <= BM || n <= 0) return 0;
  const int64_t tiles = ((m + PBM - 1) / PBM) * ((n + BN - 1) / BN);
  return static_cast<size_t>(sched::region_bytes(tiles));
}

}  // namespace tfb200
