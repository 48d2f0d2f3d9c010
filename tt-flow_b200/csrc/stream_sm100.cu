// Weight-streaming (decode-shaped) GEMM for sm_100a: few token rows, large
// weights. HBM-bound: the job is to stream W at full bandwidth from every SM.
//
// Computes acc[M, N] = A[M, K] @ W[K, N] with M <= 64 (tokens) through the
// transposed product acc^T = W^T A^T ("swap AB"): the MMA's M side is 128 output
// features (W columns, read N-major straight from row-major W) and its N side is
// the token count rounded up to 32, so no MMA row is wasted on padding tokens.
// Work units are (128-column block, 64-deep k block) pairs; the U units are cut
// into gridDim.x contiguous ranges of equal length (stream-K), so every SM
// streams the same number of weight bytes whatever the wave count. A CTA
// accumulates each column block it touches in TMEM, then adds its fp32 partial
// into `acc` in global memory (L2 atomics). The CTA that completes a column
// block (a per-block arrival counter) applies the epilogue for that block:
//   mode kFinishUp:   out = bf16(gelu(acc * col_scale[m] + bias[n]))
//   mode kFinishDown: out = bf16(acc + residual[m, n])
//   mode kPartial:    nothing (acc is the result, e.g. a tensor-parallel partial
//                     sum reduced across GPUs afterwards)
//   mode kTpReduce:   the partial goes into the owning GPU's accumulator over
//                     NVLink; the last contributor across GPUs adds the residual
//                     and writes the block to every GPU (TpPeers).
// `acc` and the counters must be zero on entry (the RMSNorm staging pass clears
// them). Launched with programmatic stream serialization: the prologue and the
// first ring of weight tiles overlap the preceding grid's tail.
//
// Warp roles: warp 0 TMA producer (W tile 64k x 128n as two 64-column boxes,
// A tile Mpad x 64k), warp 1 MMA issuer (tcgen05.mma 128 x Mpad x 16, kAcc TMEM
// accumulators), warp 2 TMEM allocator, warps 4-7 partial-sum and finishing
// epilogue. All waits are bounded (kDevTimeout in the status word).
//
// This is the small-M form of the MLP compute the reference emits
// (tensixflow lib/tensixflow/Codegen/EmitCompute.cpp:331-558).
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "internal.h"
#include "kernel_config.h"
#include "sm100_ptx.cuh"

namespace tfb200 {

namespace {

constexpr int SBN = cfg::kStreamN;  // output features per unit (MMA M)
constexpr int SBK = cfg::kStreamK;  // k per unit
constexpr uint32_t W_STAGE = SBN * SBK * 2;  // 16 KiB
constexpr int kMaxStages = cfg::kStreamMaxStages;

struct SParams {
  int M, N, K, Mpad;
  int units, kblocks, nblocks;
  float* acc;
  int* counters;
  int mode;
  const float* col_scale;
  const bf16* bias;
  int gelu;
  const bf16* residual;
  int64_t ldr;
  bf16* out;
  int64_t ldo;
  int stages;
  uint32_t tmem_cols;
  int* status;
  uint64_t timeout_ns;
  TpPeers tp;
};

// TMEM accumulators in rotation: the MMA may run kAcc-1 segments ahead of the
// epilogue.
constexpr int kAcc = cfg::kStreamAcc;

struct SCtl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[kAcc];
  uint64_t tempty[kAcc];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int finisher;
};

static_assert(sizeof(SCtl) == cfg::kStreamCtlBytes, "planner's control-block size");

__device__ __forceinline__ int64_t unit_start(int c, int units, int grid) {
  return static_cast<int64_t>(c) * units / grid;
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(int64_t u, int units, int grid) {
  return static_cast<int>(((u + 1) * grid + units - 1) / units - 1);
}

// A CTA's unit range [u0, u1) cut at column-block boundaries gives its
// segments, one TMEM accumulation and epilogue each, taken in order. (Taking
// the column blocks a CTA covers whole first measured 1-3 us slower.)
struct Segs {
  int64_t u0, u1;
  int kb;
  int first_blk, n;  // column blocks touched
};
__device__ __forceinline__ Segs make_segs(int64_t u0, int64_t u1, int kb) {
  Segs g;
  g.u0 = u0;
  g.u1 = u1;
  g.kb = kb;
  g.first_blk = u1 > u0 ? static_cast<int>(u0 / kb) : 0;
  g.n = u1 > u0 ? static_cast<int>((u1 - 1) / kb) - g.first_blk + 1 : 0;
  return g;
}
__device__ __forceinline__ void seg_range(const Segs& g, int i, int64_t* s, int64_t* e, int* nb) {
  *nb = g.first_blk + i;
  *s = max(g.u0, static_cast<int64_t>(*nb) * g.kb);
  *e = min(g.u1, static_cast<int64_t>(*nb + 1) * g.kb);
}

__device__ __forceinline__ void raise_abort(SCtl* ctl, int* status) {
  ctl->abort = 1;
  atomicExch(status, kDevTimeout);
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// AND of `ok` over the 128 epilogue threads (named barrier 1): every epilogue
// warp takes the same branch, so none is left waiting at a later epi_bar().
__device__ __forceinline__ bool epi_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(ok ? 1u : 0u)
      : "memory");
  return r != 0;
}

// Bounded wait by all 128 epilogue threads with a common outcome.
__device__ __forceinline__ bool epi_wait(uint32_t bar, uint32_t parity, SCtl* ctl, const SParams& p) {
  const bool ok = epi_all(mbar_wait(bar, parity, &ctl->abort, p.timeout_ns));
  if (!ok && threadIdx.x == 128) raise_abort(ctl, p.status);
  return ok;
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }
// tanh form of GELU with the hardware tanh (tanh.approx.f32, relative error
// about 2^-11): well inside the bf16 rounding (2^-9) of the value it produces.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.0f + tanh_approx(u));
}

// The residual column a finishing thread needs, read into registers (bf16
// pairs) when its segment starts, before the accumulator is ready: read at
// finishing time these loads miss L2 (the weight stream has evicted the
// residual) and cost more than the rest of the finish.
constexpr int kResRegs = static_cast<int>(kStreamMaxRows / 2);
__device__ __forceinline__ void load_residual(const SParams& p, int nf, uint32_t (&res)[kResRegs]) {
  const unsigned short* r = reinterpret_cast<const unsigned short*>(p.residual);
#pragma unroll
  for (int i = 0; i < kResRegs; ++i) {
    const int m = 2 * i;
    const uint32_t lo = m < p.M ? r[static_cast<int64_t>(m) * p.ldr + nf] : 0u;
    const uint32_t hi = m + 1 < p.M ? r[static_cast<int64_t>(m + 1) * p.ldr + nf] : 0u;
    res[i] = lo | (hi << 16);
  }
}
__device__ __forceinline__ float residual_at(const uint32_t (&res)[kResRegs], int m) {
  return __uint_as_float((m & 1) ? (res[m >> 1] & 0xFFFF0000u) : (res[m >> 1] << 16));
}

// Element i of a per-rank pointer array in the kernel parameters, read with
// constant indices only: a runtime index into a parameter array makes the
// compiler go through a local copy on every access.
template <typename T>
__device__ __forceinline__ T* tp_pick(T* const (&arr)[kMaxTp], int i) {
  T* r = arr[0];
#pragma unroll
  for (int k = 1; k < kMaxTp; ++k)
    if (i == k) r = arr[k];
  return r;
}

// Tensor-parallel finish mapping: epilogue thread et covers the 8 columns
// nb*128 + (et % 16)*8 .. +8 of rows et/16 + 8k, so every access is a 16-byte
// vector. Its residual values, bf16 pairs: res[4k + i] = columns 2i, 2i+1 of
// row et/16 + 8k.
__device__ __forceinline__ void load_residual_tp(const SParams& p, int nb, int et, uint32_t (&res)[kResRegs]) {
  const int r0 = et >> 4;
  const int c = nb * SBN + (et & 15) * 8;
#pragma unroll
  for (int k = 0; k < kStreamMaxRows / 8; ++k) {
    const int m = r0 + 8 * k;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < p.M && c < p.N) v = __ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(m) * p.ldr + c));
    res[4 * k + 0] = v.x;
    res[4 * k + 1] = v.y;
    res[4 * k + 2] = v.z;
    res[4 * k + 3] = v.w;
  }
}

__device__ __forceinline__ float4 ld_relaxed_sys_v4(const float* ptr) {
  float4 v;
  asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(ptr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return a | (b << 16);
}
__device__ __forceinline__ float bf16_lo_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi_f(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// Called by the 128 epilogue threads of the CTA that completed column block nb
// on this rank. Another rank pushes its sums into its slot on the block's
// owner and arrives there (release); the owner waits until the other ranks
// have arrived (acquire, bounded), adds their slots and its own sums in rank
// order plus the residual, writes the block to every rank and counts it done
// there (release). One thread arrives or waits for the CTA, after a barrier.
__device__ __forceinline__ void tp_push_and_finish(const SParams& p, SCtl* ctl, int nb, int et,
                                                   const uint32_t (&res)[kResRegs]) {
  const int owner = nb % p.tp.world;
  const int r0 = et >> 4;
  const int c = nb * SBN + (et & 15) * 8;
  const bool col_ok = c < p.N;
  constexpr int kRows = kStreamMaxRows / 8;
  if (owner != p.tp.rank) {
    float* slot = tp_pick(p.tp.slots, owner) + static_cast<int64_t>(p.tp.rank) * p.tp.slot_stride;
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int m = r0 + 8 * k;
      if (m < p.M && col_ok) {
        float* src = p.acc + static_cast<int64_t>(m) * p.N + c;
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
        float* dst = slot + static_cast<int64_t>(m) * p.N + c;
        *reinterpret_cast<float4*>(dst) = a;
        *reinterpret_cast<float4*>(dst + 4) = b;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(src) = z;  // ready for the next call
        *reinterpret_cast<float4*>(src + 4) = z;
      }
    }
    epi_bar();
    if (et == 0) {
      p.counters[nb] = 0;  // every local contribution is in: ready for the next call
      red_add_release_sys(tp_pick(p.tp.arrive, owner) + nb, 1u);  // the slot before the arrival
    }
    return;
  }
  // Owner: its own sums, read before the wait.
  float own[kRows][8];
#pragma unroll
  for (int k = 0; k < kRows; ++k) {
    const int m = r0 + 8 * k;
    if (m < p.M && col_ok) {
      float* src = p.acc + static_cast<int64_t>(m) * p.N + c;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
      own[k][0] = a.x; own[k][1] = a.y; own[k][2] = a.z; own[k][3] = a.w;
      own[k][4] = b.x; own[k][5] = b.y; own[k][6] = b.z; own[k][7] = b.w;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(src) = z;  // ready for the next call
      *reinterpret_cast<float4*>(src + 4) = z;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) own[k][i] = 0.f;
    }
  }
  if (et == 0) {
    p.counters[nb] = 0;
    unsigned* arr = tp_pick(p.tp.arrive, owner) + nb;
    const unsigned want = static_cast<unsigned>(p.tp.world - 1);
    const uint64_t t0 = global_ns();
    bool ok = true;
    while (ld_acquire_sys(arr) < want) {
      if (global_ns() - t0 > p.timeout_ns) {
        atomicExch(p.status, kDevTimeout);
        ok = false;
        break;
      }
    }
    if (ok) st_relaxed_sys(arr, 0u);  // every rank is in: ready for the next call
    ctl->finisher = ok;
  }
  epi_bar();
  if (!ctl->finisher) return;
  const float* slots = tp_pick(p.tp.slots, owner);
  bf16* outs[kMaxTp];
#pragma unroll
  for (int r = 0; r < kMaxTp; ++r) outs[r] = r < p.tp.world ? p.tp.out[r] : nullptr;
#pragma unroll
  for (int k = 0; k < kRows; ++k) {
    const int m = r0 + 8 * k;
    if (m < p.M && col_ok) {
      // The ranks' sums in rank order (the same on every run), then the residual.
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < kMaxTp; ++r) {
        if (r >= p.tp.world) break;
        if (r == owner) {
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += own[k][i];
        } else {
          const float* src = slots + static_cast<int64_t>(r) * p.tp.slot_stride + static_cast<int64_t>(m) * p.N + c;
          const float4 a = ld_relaxed_sys_v4(src);
          const float4 b = ld_relaxed_sys_v4(src + 4);
          acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
          acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
        }
      }
      uint4 o;
      o.x = pack2_bf16(acc[0] + bf16_lo_f(res[4 * k + 0]), acc[1] + bf16_hi_f(res[4 * k + 0]));
      o.y = pack2_bf16(acc[2] + bf16_lo_f(res[4 * k + 1]), acc[3] + bf16_hi_f(res[4 * k + 1]));
      o.z = pack2_bf16(acc[4] + bf16_lo_f(res[4 * k + 2]), acc[5] + bf16_hi_f(res[4 * k + 2]));
      o.w = pack2_bf16(acc[6] + bf16_lo_f(res[4 * k + 3]), acc[7] + bf16_hi_f(res[4 * k + 3]));
#pragma unroll
      for (int r = 0; r < kMaxTp; ++r)
        if (r < p.tp.world) *reinterpret_cast<uint4*>(outs[r] + static_cast<int64_t>(m) * p.ldo + c) = o;
    }
  }
  epi_bar();
  if (et == 0) {
    // Release: the block's rows on every rank before its done counts.
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r)
      if (r < p.tp.world) red_add_release_sys(p.tp.done[r], 1u);
  }
}

__global__ void __launch_bounds__(256, 1)
    k_stream(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA, const SParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t a_stage = static_cast<uint32_t>(p.Mpad) * SBK * 2;
  uint8_t* sW = smem;
  uint8_t* sA = smem + p.stages * W_STAGE;
  SCtl* ctl = reinterpret_cast<SCtl*>(sA + p.stages * a_stage);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(smem_u32(&ctl->tfull[b]), 1);
      mbar_init(smem_u32(&ctl->tempty[b]), 128);
    }
    mbar_init(smem_u32(&ctl->drain), 1);
    ctl->abort = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmA);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(&ctl->tmem_base), p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;

  const int G = gridDim.x;
  const int64_t u0 = unit_start(blockIdx.x, p.units, G);
  const int64_t u1 = unit_start(blockIdx.x + 1, p.units, G);

  const Segs segs = make_segs(u0, u1, p.kblocks);
  // The next grid in the stream (launched with programmatic serialization) may
  // start its prologue as soon as SMs free up; it still waits for this grid to
  // complete before it reads anything this grid writes.
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_phase = 0;
      bool ok = true;
      // The first ring of weight tiles is requested before waiting for the
      // preceding grid (the RMSNorm staging or the up-projection, which never
      // write the weights); their token tiles follow once it has completed.
      bool waited = false;
      int pre = 0;
      int pre_kb[kMaxStages];
      for (int si = 0; si < segs.n && ok; ++si) {
        int64_t s0, e0;
        int nb;
        seg_range(segs, si, &s0, &e0, &nb);
        for (int64_t u = s0; u < e0; ++u) {
          const int kb = static_cast<int>(u - static_cast<int64_t>(nb) * p.kblocks);
          if (!waited && pre == p.stages) {
            grid_dep_wait();
            for (int i = 0; i < pre; ++i)
              tma_load_2d(smem_u32(sA + i * a_stage), &tmA, smem_u32(&ctl->full[i]), pre_kb[i] * SBK, 0);
            waited = true;
          }
          if (!mbar_wait(smem_u32(&ctl->empty[stage]), phase ^ 1u, &ctl->abort, p.timeout_ns)) {
            raise_abort(ctl, p.status);
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&ctl->full[stage]);
          mbar_arrive_expect_tx(fb, W_STAGE + a_stage);
          tma_load_2d(smem_u32(sW + stage * W_STAGE), &tmW, fb, nb * SBN, kb * SBK);
          tma_load_2d(smem_u32(sW + stage * W_STAGE + 8192), &tmW, fb, nb * SBN + 64, kb * SBK);
          if (waited)
            tma_load_2d(smem_u32(sA + stage * a_stage), &tmA, fb, kb * SBK, 0);
          else
            pre_kb[pre++] = kb;  // stage == pre here
          armed |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!waited) {
        grid_dep_wait();
        for (int i = 0; i < pre; ++i)
          tma_load_2d(smem_u32(sA + i * a_stage), &tmA, smem_u32(&ctl->full[i]), pre_kb[i] * SBK, 0);
      }
      if (!ok) {
        for (int s = 0; s < p.stages; ++s)
          if (armed & (1u << s)) {
            const uint64_t t0 = global_ns();
            while (!mbar_test(smem_u32(&ctl->full[s]), (armed_phase >> s) & 1u) &&
                   global_ns() - t0 < p.timeout_ns) {
            }
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(SBN, p.Mpad, true, false);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int si = 0; si < segs.n && ok; ++si) {
        int64_t s0, e0;
        int nb;
        seg_range(segs, si, &s0, &e0, &nb);
        const int acc = si % kAcc;
        const uint32_t use = static_cast<uint32_t>(si / kAcc);
        if (!mbar_wait(smem_u32(&ctl->tempty[acc]), (use & 1u) ^ 1u, &ctl->abort, p.timeout_ns)) {
          raise_abort(ctl, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * p.Mpad);
        bool first = true;
        for (int64_t u = s0; u < e0; ++u) {
          if (!mbar_wait(smem_u32(&ctl->full[stage]), phase, &ctl->abort, p.timeout_ns)) {
            raise_abort(ctl, p.status);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w0 = smem_u32(sW + stage * W_STAGE);
          const uint32_t a0 = smem_u32(sA + stage * a_stage);
#pragma unroll
          for (int k = 0; k < SBK / 16; ++k) {
            const uint64_t wd = sdesc_sw128(w0 + k * 2048, 8192, 1024);  // MN-major W^T
            const uint64_t ad = sdesc_sw128(a0 + k * 32, 16, 1024);      // K-major tokens
            mma_bf16(d, wd, ad, idesc, (first && k == 0) ? 0u : 1u);
          }
          first = false;
          mma_commit(smem_u32(&ctl->empty[stage]));
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) mma_commit(smem_u32(&ctl->tfull[acc]));
      }
      mma_commit(smem_u32(&ctl->drain));
      const uint64_t t0 = global_ns();
      while (!mbar_test(smem_u32(&ctl->drain), 0) && global_ns() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp >= 4) {
    const int q = warp & 3;
    const int et = threadIdx.x - 128;  // 0..127
    grid_dep_wait();  // the accumulators, counters and row scales come from the preceding grids
    for (int si = 0; si < segs.n; ++si) {
      int64_t s0, e0;
      int nb;
      seg_range(segs, si, &s0, &e0, &nb);
      const int acc = si % kAcc;
      const uint32_t use = static_cast<uint32_t>(si / kAcc);
      // What a finisher of this column block reads besides the accumulator,
      // loaded while the block's MMAs run.
      const int nf = nb * SBN + et;
      uint32_t res[kResRegs];
      float bias = 0.0f;
      if (p.mode == kStreamFinishDown && nf < p.N) {
        load_residual(p, nf, res);
      } else if (p.mode == kStreamTpReduce) {
        load_residual_tp(p, nb, et, res);
      } else {
#pragma unroll
        for (int i = 0; i < kResRegs; ++i) res[i] = 0u;
        if (p.mode == kStreamFinishUp && p.bias && nf < p.N) bias = __bfloat162float(p.bias[nf]);
      }
      if (!epi_wait(smem_u32(&ctl->tfull[acc]), use & 1u, ctl, p)) break;
      tc_fence_after();
      const int n = nb * SBN + q * 32 + lane;
      for (int c0 = 0; c0 < p.Mpad; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * p.Mpad + c0),
                       v);
        tmem_wait_ld();
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = c0 + j;
            if (m < p.M) atomicAdd(p.acc + static_cast<int64_t>(m) * p.N + n, __uint_as_float(v[j]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->tempty[acc]));
      if (p.mode == kStreamPartial) continue;
      // Arrive on the column block's counter; the last contributor finishes it.
      // One thread arrives for the CTA after a barrier.
      epi_bar();
      if (et == 0) {
        const int64_t first_u = static_cast<int64_t>(nb) * p.kblocks;
        const int contributors =
            cta_of(first_u + p.kblocks - 1, p.units, G) - cta_of(first_u, p.units, G) + 1;
        // Release: the block's atomics before the arrival; acquire: every
        // contributor's atomics before the finisher's reads.
        const int prev = atom_add_acq_rel_gpu(p.counters + nb, 1);
        ctl->finisher = prev == contributors - 1;
      }
      epi_bar();
      if (p.mode == kStreamTpReduce) {
        if (ctl->finisher) tp_push_and_finish(p, ctl, nb, et, res);
        continue;
      }
      if (ctl->finisher) {
        if (nf < p.N) {
          // Thirty-two rows per step so their loads are in flight together (one
          // L2 round trip for up to 32 tokens).
#pragma unroll
          for (int m0 = 0; m0 < kStreamMaxRows; m0 += 32) {
            if (m0 >= p.M) break;
            float val[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + j;
              val[j] = m < p.M ? __ldcg(p.acc + static_cast<int64_t>(m) * p.N + nf) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + j;
              if (m >= p.M) break;
              float v = val[j];
              if (p.mode == kStreamFinishUp) {
                v = v * __ldg(p.col_scale + m) + bias;
                v = p.gelu == kGeluErf ? gelu_erf(v) : (p.gelu == kGeluTanh ? gelu_tanh(v) : v);
              } else {
                v += residual_at(res, m);
              }
              p.out[static_cast<int64_t>(m) * p.ldo + nf] = __float2bfloat16_rn(v);
            }
          }
        }
        epi_bar();
      }
    }
  }

  // Tensor-parallel: the call is complete on this rank once every column block
  // (finished on whichever rank) has landed here. One thread waits, bounded,
  // then returns the counter to zero for the next call.
  if (p.mode == kStreamTpReduce && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned* done = tp_pick(p.tp.done, p.tp.rank);
    const unsigned target = static_cast<unsigned>(p.nblocks);
    const uint64_t t0 = global_ns();
    bool ok = true;
    while (ld_acquire_sys(done) < target) {
      if (global_ns() - t0 > p.timeout_ns) {
        atomicExch(p.status, kDevTimeout);
        ok = false;
        break;
      }
    }
    if (ok) st_relaxed_sys(done, 0u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace

int stream_mpad(int64_t m) { return static_cast<int>((m + 31) / 32 * 32); }

size_t stream_counter_bytes(int64_t n) { return static_cast<size_t>((n + SBN - 1) / SBN) * sizeof(int); }

int run_stream(const StreamProblem& sp, cudaStream_t stream, std::string* err) {
  if (sp.M <= 0 || sp.M > kStreamMaxRows || sp.N <= 0 || sp.K <= 0) {
    if (err) *err = "weight-streaming GEMM: needs 1 <= M <= 64 and N, K > 0";
    return -2;
  }
  if ((reinterpret_cast<uintptr_t>(sp.A) & 15u) || (reinterpret_cast<uintptr_t>(sp.W) & 15u) || sp.lda % 8 ||
      sp.ldw % 8) {
    if (err) *err = "weight-streaming GEMM: operands must be 16-byte aligned with leading dimensions % 8 == 0";
    return -2;
  }
  int* status = device_status_ptr(err);
  if (!status) return -3;
  SParams p{};
  p.M = static_cast<int>(sp.M);
  p.N = static_cast<int>(sp.N);
  p.K = static_cast<int>(sp.K);
  p.Mpad = stream_mpad(sp.M);
  p.kblocks = static_cast<int>((sp.K + SBK - 1) / SBK);
  p.nblocks = static_cast<int>((sp.N + SBN - 1) / SBN);
  p.units = p.kblocks * p.nblocks;
  p.acc = sp.acc;
  p.counters = sp.counters;
  p.mode = sp.mode;
  p.col_scale = sp.col_scale;
  p.bias = sp.bias;
  p.gelu = sp.gelu;
  p.residual = sp.residual;
  p.ldr = sp.ldr;
  p.out = sp.out;
  p.ldo = sp.ldo;
  p.tp = sp.tp;
  if (sp.mode == kStreamTpReduce && (sp.tp.world < 1 || sp.tp.world > kMaxTp || sp.tp.rank < 0 ||
                                     sp.tp.rank >= sp.tp.world)) {
    if (err) *err = "weight-streaming GEMM: bad tensor-parallel rank / world";
    return -1;
  }
  p.status = status;
  p.timeout_ns = wait_limit_ns();
  const uint32_t a_stage = static_cast<uint32_t>(p.Mpad) * SBK * 2;
  const size_t budget = cfg::kStreamBudget;
  int stages = static_cast<int>(budget / (W_STAGE + a_stage));
  p.stages = stages > kMaxStages ? kMaxStages : stages;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(kAcc * p.Mpad)) cols <<= 1;
  p.tmem_cols = cols;
  const size_t smem = 1024 + static_cast<size_t>(p.stages) * (W_STAGE + a_stage) + sizeof(SCtl);

  CUtensorMap tw{}, ta{};
  if (!make_map(&tw, sp.W, sp.K, sp.N, sp.ldw, SBK, err)) return -3;
  if (!make_map(&ta, sp.A, sp.M, sp.K, sp.lda, static_cast<uint32_t>(p.Mpad), err)) return -3;
  // Per-device first-call setup; calls may come from several host threads.
  static std::mutex mu;
  static std::atomic<bool> ready[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !ready[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(mu);
    if (!ready[dev].load(std::memory_order_relaxed)) {
      cudaError_t e = cudaFuncSetAttribute(k_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e != cudaSuccess) {
        if (err) *err = std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
        return -3;
      }
      ready[dev].store(true, std::memory_order_release);
    }
  }
  const int grid = p.units < sm_count() ? p.units : sm_count();
  // Programmatic dependent launch: this grid's prologue and first ring of
  // weight tiles overlap the tail of the preceding grid (TFB200_PDL=0 turns it off).
  static const bool pdl = [] {
    const char* v = std::getenv("TFB200_PDL");
    return !(v && v[0] == '0');
  }();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_stream, tw, ta, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    if (err) *err = std::string("weight-streaming GEMM launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

}  // namespace tfb200
