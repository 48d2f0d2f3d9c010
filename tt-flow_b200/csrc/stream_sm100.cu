// Weight-streaming (decode-shaped) fused MLP for sm_100a: few token rows, large
// weights. HBM-bound: the job is to stream the weights at full bandwidth from
// every SM.
//
// One persistent launch runs one GEMM, or the MLP's two GEMMs as two phases,
//   phase 0: h   = epi0(A0[M, K0] @ W0[K0, N0])   (up-projection, h in HBM/L2)
//   phase 1: out = epi1(h[M, N0]  @ W1[N0, N1])   (down-projection)
// with a grid-wide barrier between them (a counter the RMSNorm staging pass
// zeroes; one CTA per SM, launched cooperatively so that every CTA is resident
// together whatever else runs on the GPU). The decode MLP (decode.cu) runs the
// two GEMMs as two one-phase launches by default, which measured faster; the
// two-phase launch gives the same bits. Each GEMM is computed as the
// transposed product acc^T = W^T A^T ("swap AB"): the MMA's M side is 128
// output features (W columns, read N-major straight from row-major W) and its
// N side is the token count rounded up to 32. Work units are (128-column block,
// 64-deep k block) pairs; the U units of a phase are cut into gridDim.x
// contiguous ranges of equal length, so every SM streams the same number of
// weight bytes. A CTA accumulates each column block its range touches in TMEM
// (one segment), and writes that partial sum, fp32 [M, 128], to its own slot
// in the workspace: the slot of (column block nb, CTA c) is nb + c, unique
// because the ranges are contiguous. The CTA that completes a column block (a
// per-block arrival counter) adds the slots of its contributors in CTA order --
// a fixed order, so results do not depend on timing -- and applies the phase's
// epilogue:
//   kStreamFinishUp:   out = bf16(gelu(sum * col_scale[m] + bias[n]))
//   kStreamFinishDown: out = bf16(sum + residual[m, n])
//   kStreamPartial:    part = sum (fp32; e.g. a tensor-parallel partial sum
//                      reduced across GPUs afterwards)
//   kStreamTpReduce:   part (this rank's sums) goes to the block's owner GPU
//                      over NVLink; the owner adds the ranks' sums in rank
//                      order and the residual and writes the block to every
//                      GPU (TpPeers).
// Only the arrival counters and the phase barrier must be zero on entry (the
// staging pass clears them); slots, hidden block and outputs are written
// whole. The phase-1 weight tiles that fit the shared-memory ring are
// requested before the barrier; the hidden block follows once every CTA has
// arrived. Launched with programmatic stream serialization: the prologue and
// the first ring of weight tiles overlap the preceding grid's tail. A CTA that
// has issued its whole weight stream also prefetches into L2 the first units of
// the range it (or the same CTA of the next launch) streams next, so that HBM
// keeps streaming while the slowest CTAs and the finishers drain.
//
// Warp roles: warp 0 TMA producer (W tile 64k x 128n as two 64-column boxes,
// A tile Mpad x 64k), warp 1 MMA issuer (tcgen05.mma 128 x Mpad x 16, kAcc TMEM
// accumulators in rotation across both phases), warp 2 TMEM allocator, warps
// 4-7 slot writes and finishing epilogue. All waits are bounded (kDevTimeout in
// the status word).
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

struct SPhase {
  int N, K, kblocks, nblocks, units;
  int mode;
  const float* col_scale;
  const bf16* bias;
  int gelu;
  const bf16* residual;
  int64_t ldr;
  bf16* out;
  int64_t ldo;
  float* part;
  int64_t ldp;
  int* counters;
};

struct SParams {
  int M, Mpad, nph;
  SPhase ph[2];
  float* slots;   // (nblocks + gridDim.x - 1) slots of fp32 [M, 128]
  int* grid_bar;  // phase barrier: arrivals of the CTAs
  int stages;
  uint32_t tmem_cols;
  int* status;
  uint64_t timeout_ns;
  TpPeers tp;
  // L2 prefetch of the weights streamed next (tmW1): pf_units units of the
  // range this CTA streams there, after skipping pf_skip of them.
  int pf_units, pf_skip, pf_kblocks, pf_total;
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
template <int PH>
__device__ __forceinline__ Segs phase_segs(const SParams& p) {
  const SPhase& f = p.ph[PH];
  return make_segs(unit_start(blockIdx.x, f.units, gridDim.x), unit_start(blockIdx.x + 1, f.units, gridDim.x),
                   f.kblocks);
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

// Generic-proxy global writes (the hidden block) against async-proxy (TMA)
// reads of the same memory in another CTA.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
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
__device__ __forceinline__ void load_residual(const SParams& p, const SPhase& f, int nf,
                                              uint32_t (&res)[kResRegs]) {
  const unsigned short* r = reinterpret_cast<const unsigned short*>(f.residual);
#pragma unroll
  for (int i = 0; i < kResRegs; ++i) {
    const int m = 2 * i;
    const uint32_t lo = m < p.M ? r[static_cast<int64_t>(m) * f.ldr + nf] : 0u;
    const uint32_t hi = m + 1 < p.M ? r[static_cast<int64_t>(m + 1) * f.ldr + nf] : 0u;
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
__device__ __forceinline__ void load_residual_tp(const SParams& p, const SPhase& f, int nb, int et,
                                                 uint32_t (&res)[kResRegs]) {
  const int r0 = et >> 4;
  const int c = nb * SBN + (et & 15) * 8;
#pragma unroll
  for (int k = 0; k < kStreamMaxRows / 8; ++k) {
    const int m = r0 + 8 * k;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < p.M && c < f.N)
      v = __ldg(reinterpret_cast<const uint4*>(f.residual + static_cast<int64_t>(m) * f.ldr + c));
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
// on this rank, after this rank's sums of the block are in f.part ([M, N]).
// Another rank pushes its sums into its slot on the block's owner and arrives
// there (release); the owner waits until the other ranks have arrived
// (acquire, bounded), adds their slots and its own sums in rank order plus the
// residual, writes the block to every rank and counts it done there (release).
// One thread arrives or waits for the CTA, after a barrier.
__device__ __forceinline__ void tp_push_and_finish(const SParams& p, const SPhase& f, SCtl* ctl, int nb, int et,
                                                   const uint32_t (&res)[kResRegs]) {
  const int owner = nb % p.tp.world;
  const int r0 = et >> 4;
  const int c = nb * SBN + (et & 15) * 8;
  const bool col_ok = c < f.N;
  constexpr int kRows = kStreamMaxRows / 8;
  if (owner != p.tp.rank) {
    float* slot = tp_pick(p.tp.slots, owner) + static_cast<int64_t>(p.tp.rank) * p.tp.slot_stride;
#pragma unroll
    for (int k = 0; k < kRows; ++k) {
      const int m = r0 + 8 * k;
      if (m < p.M && col_ok) {
        const float* src = f.part + static_cast<int64_t>(m) * f.N + c;
        const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
        const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
        float* dst = slot + static_cast<int64_t>(m) * f.N + c;
        *reinterpret_cast<float4*>(dst) = a;
        *reinterpret_cast<float4*>(dst + 4) = b;
      }
    }
    epi_bar();
    if (et == 0) {
      f.counters[nb] = 0;  // every local contribution is in: ready for the next call
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
      const float* src = f.part + static_cast<int64_t>(m) * f.N + c;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(src));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(src + 4));
      own[k][0] = a.x; own[k][1] = a.y; own[k][2] = a.z; own[k][3] = a.w;
      own[k][4] = b.x; own[k][5] = b.y; own[k][6] = b.z; own[k][7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) own[k][i] = 0.f;
    }
  }
  if (et == 0) {
    f.counters[nb] = 0;
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
          const float* src = slots + static_cast<int64_t>(r) * p.tp.slot_stride + static_cast<int64_t>(m) * f.N + c;
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
        if (r < p.tp.world) *reinterpret_cast<uint4*>(outs[r] + static_cast<int64_t>(m) * f.ldo + c) = o;
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

// ---------------------------------------------------------------- producer

// Ring state of the TMA producer, carried across the phases. A stage armed
// before its phase's gate opened (the preceding grid for phase 0, the phase
// barrier for phase 1) has its weight tile in flight and its token tile
// pending; `pend` lists those stages.
struct Ring {
  int stage;
  uint32_t phase;
  uint32_t armed, armed_phase;
  int npend;
  int pend_stage[kMaxStages];
  int pend_kb[kMaxStages];
};

// Wait for every CTA to arrive at the phase barrier (bounded).
__device__ __forceinline__ bool wait_phase_barrier(const SParams& p, SCtl* ctl) {
  const int want = static_cast<int>(gridDim.x);
  const uint64_t t0 = global_ns();
  while (ld_acquire_gpu(p.grid_bar) < want) {
    if (ctl->abort || global_ns() - t0 > p.timeout_ns) return false;
  }
  fence_proxy_async_global();
  return true;
}

template <int PH>
__device__ __forceinline__ bool produce(const SParams& p, SCtl* ctl, const CUtensorMap* tmW, const CUtensorMap* tmA,
                                       uint8_t* sW, uint8_t* sA, uint32_t a_stage, Ring& ring) {
  const SPhase& f = p.ph[PH];
  const Segs segs = phase_segs<PH>(p);
  // The weights are read exactly once: evict them first, so that the partial
  // sums, the hidden block and the residual the finishers read stay in L2 (the
  // weight stream replaces all of L2 every ~20 us).
  const uint64_t evict_first = l2_policy_evict_first();
  bool open = false;  // the gate of this phase's token tiles
  ring.npend = 0;
  auto open_gate = [&]() -> bool {
    if (PH == 0) {
      grid_dep_wait();
    } else if (!wait_phase_barrier(p, ctl)) {
      raise_abort(ctl, p.status);
      return false;
    }
    for (int i = 0; i < ring.npend; ++i)
      tma_load_2d(smem_u32(sA + ring.pend_stage[i] * a_stage), tmA, smem_u32(&ctl->full[ring.pend_stage[i]]),
                  ring.pend_kb[i] * SBK, 0);
    open = true;
    return true;
  };
  for (int si = 0; si < segs.n; ++si) {
    int64_t s0, e0;
    int nb;
    seg_range(segs, si, &s0, &e0, &nb);
    for (int64_t u = s0; u < e0; ++u) {
      const int kb = static_cast<int>(u - static_cast<int64_t>(nb) * f.kblocks);
      if (!open && ring.npend == p.stages && !open_gate()) return false;
      if (!mbar_wait(smem_u32(&ctl->empty[ring.stage]), ring.phase ^ 1u, &ctl->abort, p.timeout_ns)) {
        raise_abort(ctl, p.status);
        return false;
      }
      const uint32_t fb = smem_u32(&ctl->full[ring.stage]);
      mbar_arrive_expect_tx(fb, W_STAGE + a_stage);
      tma_load_2d_hint(smem_u32(sW + ring.stage * W_STAGE), tmW, fb, nb * SBN, kb * SBK, evict_first);
      tma_load_2d_hint(smem_u32(sW + ring.stage * W_STAGE + 8192), tmW, fb, nb * SBN + 64, kb * SBK, evict_first);
      if (open) {
        tma_load_2d(smem_u32(sA + ring.stage * a_stage), tmA, fb, kb * SBK, 0);
      } else {
        ring.pend_stage[ring.npend] = ring.stage;
        ring.pend_kb[ring.npend] = kb;
        ++ring.npend;
      }
      ring.armed |= 1u << ring.stage;
      ring.armed_phase = (ring.armed_phase & ~(1u << ring.stage)) | (ring.phase << ring.stage);
      if (++ring.stage == p.stages) {
        ring.stage = 0;
        ring.phase ^= 1u;
      }
    }
  }
  if (!open && !open_gate()) return false;
  return true;
}

// Units [u0 + skip, u0 + skip + pf_units) of the range [u0, u1) this CTA
// streams from tmW next (the next launch's weights, or phase 1), brought into
// L2 with the same unit -> (column block, k block) order as produce().
__device__ __forceinline__ void prefetch_next_weights(const SParams& p, const CUtensorMap* tmW) {
  const int64_t u0 = unit_start(blockIdx.x, p.pf_total, gridDim.x);
  const int64_t u1 = unit_start(blockIdx.x + 1, p.pf_total, gridDim.x);
  int64_t e = u0 + p.pf_skip + p.pf_units;
  if (e > u1) e = u1;
  for (int64_t u = u0 + p.pf_skip; u < e; ++u) {
    const int nb = static_cast<int>(u / p.pf_kblocks);
    const int kb = static_cast<int>(u - static_cast<int64_t>(nb) * p.pf_kblocks);
    tma_prefetch_l2_2d(tmW, nb * SBN, kb * SBK);
    tma_prefetch_l2_2d(tmW, nb * SBN + 64, kb * SBK);
  }
}

// -------------------------------------------------------------- MMA issuer

template <int PH>
__device__ __forceinline__ bool mma_phase(const SParams& p, SCtl* ctl, uint8_t* sW, uint8_t* sA, uint32_t a_stage,
                                          uint32_t tmem_base, int& gseg, int& stage, uint32_t& phase) {
  const Segs segs = phase_segs<PH>(p);
  const uint32_t idesc = idesc_bf16(SBN, p.Mpad, true, false);
  for (int si = 0; si < segs.n; ++si, ++gseg) {
    int64_t s0, e0;
    int nb;
    seg_range(segs, si, &s0, &e0, &nb);
    const int acc = gseg % kAcc;
    const uint32_t use = static_cast<uint32_t>(gseg / kAcc);
    if (!mbar_wait(smem_u32(&ctl->tempty[acc]), (use & 1u) ^ 1u, &ctl->abort, p.timeout_ns)) {
      raise_abort(ctl, p.status);
      return false;
    }
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * p.Mpad);
    bool first = true;
    for (int64_t u = s0; u < e0; ++u) {
      if (!mbar_wait(smem_u32(&ctl->full[stage]), phase, &ctl->abort, p.timeout_ns)) {
        raise_abort(ctl, p.status);
        return false;
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
    mma_commit(smem_u32(&ctl->tfull[acc]));
  }
  return true;
}

// ---------------------------------------------------------------- epilogue

// Sum of the slots of contributors c_first .. c_last for rows m0 .. m0+R-1 of
// feature et, added in CTA order (a fixed order). The loads of four
// contributors are issued together: each group is one L2 round trip.
constexpr int kSumRows = 16;
__device__ __forceinline__ void sum_slots(const SParams& p, int nb, int c_first, int c_last, int et, int m0,
                                          float (&acc)[kSumRows]) {
  const int64_t slot_elems = static_cast<int64_t>(p.M) * SBN;
#pragma unroll
  for (int j = 0; j < kSumRows; ++j) acc[j] = 0.0f;
  for (int cg = c_first; cg <= c_last; cg += 4) {
    float v[4][kSumRows];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float* sl = p.slots + static_cast<int64_t>(nb + cg + k) * slot_elems + et;
#pragma unroll
      for (int j = 0; j < kSumRows; ++j) {
        const int m = m0 + j;
        v[k][j] = (cg + k <= c_last && m < p.M) ? __ldcg(sl + static_cast<int64_t>(m) * SBN) : 0.0f;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int j = 0; j < kSumRows; ++j) acc[j] += v[k][j];
  }
}

// The 128 epilogue threads (et = feature within the column block) run one
// phase's segments: slot writes, arrivals, and the finish of completed blocks.
template <int PH>
__device__ __forceinline__ bool epilogue_phase(const SParams& p, SCtl* ctl, uint32_t tmem_base, int& gseg) {
  const SPhase& f = p.ph[PH];
  const Segs segs = phase_segs<PH>(p);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int et = threadIdx.x - 128;  // 0..127
  const int64_t slot_elems = static_cast<int64_t>(p.M) * SBN;
  // The finishers' row scales (1/rms), staged once per phase in shared memory:
  // read from global memory at finishing time they cost an L2 round trip.
  float* s_scale = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ctl) + sizeof(SCtl));
  if (f.mode == kStreamFinishUp) {
    if (et < p.M) s_scale[et] = __ldg(f.col_scale + et);
    epi_bar();
  }
  for (int si = 0; si < segs.n; ++si, ++gseg) {
    int64_t s0, e0;
    int nb;
    seg_range(segs, si, &s0, &e0, &nb);
    const int acc = gseg % kAcc;
    const uint32_t use = static_cast<uint32_t>(gseg / kAcc);
    // What a finisher of this column block reads besides the slots, loaded
    // while the block's MMAs run.
    const int nf = nb * SBN + et;
    uint32_t res[kResRegs];
    float bias = 0.0f;
    if (f.mode == kStreamFinishDown && nf < f.N) {
      load_residual(p, f, nf, res);
    } else if (f.mode == kStreamTpReduce) {
      load_residual_tp(p, f, nb, et, res);
    } else {
#pragma unroll
      for (int i = 0; i < kResRegs; ++i) res[i] = 0u;
      if (f.mode == kStreamFinishUp && f.bias && nf < f.N) bias = __bfloat162float(f.bias[nf]);
    }
    if (!epi_wait(smem_u32(&ctl->tfull[acc]), use & 1u, ctl, p)) return false;
    tc_fence_after();
    // This CTA's partial sum of block nb: feature et (TMEM lane), tokens in
    // TMEM columns; slot layout [m][128], so a warp's store covers 128 bytes.
    float* slot = p.slots + static_cast<int64_t>(nb + static_cast<int>(blockIdx.x)) * slot_elems;
    const int n_local = q * 32 + lane;
    for (int c0 = 0; c0 < p.Mpad; c0 += 32) {
      uint32_t v[32];
      tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * p.Mpad + c0), v);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int m = c0 + j;
        if (m < p.M) __stcg(slot + static_cast<int64_t>(m) * SBN + n_local, __uint_as_float(v[j]));
      }
    }
    tc_fence_before();
    mbar_arrive(smem_u32(&ctl->tempty[acc]));
    // Arrive on the column block's counter; the last contributor finishes it.
    // One thread arrives for the CTA after a barrier (release: the CTA's slot
    // before the arrival; acquire: every contributor's slot before the reads).
    epi_bar();
    const int64_t first_u = static_cast<int64_t>(nb) * f.kblocks;
    const int c_first = cta_of(first_u, f.units, gridDim.x);
    const int c_last = cta_of(first_u + f.kblocks - 1, f.units, gridDim.x);
    if (et == 0) {
      const int prev = atom_add_acq_rel_gpu(f.counters + nb, 1);
      ctl->finisher = prev == c_last - c_first;
    }
    epi_bar();
    if (!ctl->finisher) continue;
    // The contributors' slots in CTA order (the same order on every run).
    const bool col_ok = nf < f.N;
    if (f.mode == kStreamTpReduce) {
      // This rank's sums of the block into f.part, then the cross-GPU finish.
#pragma unroll 1
      for (int m0 = 0; m0 < p.M; m0 += kSumRows) {
        float val[kSumRows];
        sum_slots(p, nb, c_first, c_last, et, m0, val);
#pragma unroll
        for (int j = 0; j < kSumRows; ++j)
          if (col_ok && m0 + j < p.M) f.part[static_cast<int64_t>(m0 + j) * f.N + nf] = val[j];
      }
      epi_bar();
      tp_push_and_finish(p, f, ctl, nb, et, res);
      continue;
    }
    // Every row batch's slot loads are issued before the first store: a store
    // may alias the slots, so loads placed after one wait for it, and a
    // load-store chain per batch cost about 3 us of the up-projection's finish
    // (measured with per-CTA timestamps on B200 at 32 x 8192 x 28672: step
    // 166 -> 159 us together with the staged row scales). The batch loop is
    // unrolled, so the residual registers are indexed with constants.
    constexpr int kBatches = static_cast<int>(kStreamMaxRows / kSumRows);
    float vals[kBatches][kSumRows];
#pragma unroll
    for (int b = 0; b < kBatches; ++b)
      if (b * kSumRows < p.M) sum_slots(p, nb, c_first, c_last, et, b * kSumRows, vals[b]);
#pragma unroll
    for (int m0 = 0; m0 < kStreamMaxRows; m0 += kSumRows) {
      if (m0 >= p.M) break;
      if (!col_ok) continue;
#pragma unroll
      for (int j = 0; j < kSumRows; ++j) {
        const int m = m0 + j;
        if (m >= p.M) break;
        float v = vals[m0 / kSumRows][j];
        if (f.mode == kStreamPartial) {
          f.part[static_cast<int64_t>(m) * f.ldp + nf] = v;
          continue;
        }
        if (f.mode == kStreamFinishUp) {
          v = v * s_scale[m] + bias;
          v = f.gelu == kGeluErf ? gelu_erf(v) : (f.gelu == kGeluTanh ? gelu_tanh(v) : v);
        } else {
          v += residual_at(res, m);
        }
        f.out[static_cast<int64_t>(m) * f.ldo + nf] = __float2bfloat16_rn(v);
      }
    }
    epi_bar();
  }
  return true;
}

__global__ void __launch_bounds__(256, 1)
    k_stream(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmA0,
             const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmA1, const SParams p) {
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
    tma_prefetch_desc(&tmW0);
    tma_prefetch_desc(&tmA0);
    if (p.nph > 1) {
      tma_prefetch_desc(&tmW1);
      tma_prefetch_desc(&tmA1);
    } else if (p.pf_units > 0) {
      tma_prefetch_desc(&tmW1);
    }
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(&ctl->tmem_base), p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // The next grid in the stream (launched with programmatic serialization) may
  // start its prologue as soon as SMs free up; it still waits for this grid to
  // complete before it reads anything this grid writes.
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // The first ring of weight tiles is requested before waiting for the
      // preceding grid (the RMSNorm staging, which never writes the weights);
      // their token tiles follow once it has completed. In the same way the
      // phase-1 weight tiles that fit the ring are requested before the phase
      // barrier.
      Ring ring{};
      bool ok = produce<0>(p, ctl, &tmW0, &tmA0, sW, sA, a_stage, ring);
      if (ok && p.pf_units > 0) prefetch_next_weights(p, &tmW1);
      if (ok && p.nph > 1) ok = produce<1>(p, ctl, &tmW1, &tmA1, sW, sA, a_stage, ring);
      if (!ok) {
        for (int s = 0; s < p.stages; ++s)
          if (ring.armed & (1u << s)) {
            const uint64_t t0 = global_ns();
            while (!mbar_test(smem_u32(&ctl->full[s]), (ring.armed_phase >> s) & 1u) &&
                   global_ns() - t0 < p.timeout_ns) {
            }
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int gseg = 0, stage = 0;
      uint32_t phase = 0;
      bool ok = mma_phase<0>(p, ctl, sW, sA, a_stage, tmem_base, gseg, stage, phase);
      if (ok && p.nph > 1) mma_phase<1>(p, ctl, sW, sA, a_stage, tmem_base, gseg, stage, phase);
      mma_commit(smem_u32(&ctl->drain));
      const uint64_t t0 = global_ns();
      while (!mbar_test(smem_u32(&ctl->drain), 0) && global_ns() - t0 < p.timeout_ns) {
      }
    }
  } else if (warp >= 4) {
    grid_dep_wait();  // row scales, counters and the residual come from the preceding grids
    int gseg = 0;
    bool ok = epilogue_phase<0>(p, ctl, tmem_base, gseg);
    if (p.nph > 1) {
      // Phase barrier: this CTA's finished blocks of the hidden block are
      // written; one thread arrives for the CTA (release after the barrier).
      epi_bar();
      if (threadIdx.x == 128) {
        fence_proxy_async_global();
        red_add_release_gpu(p.grid_bar, 1);
      }
      if (ok) epilogue_phase<1>(p, ctl, tmem_base, gseg);
    }
  }

  // Tensor-parallel: the call is complete on this rank once every column block
  // (finished on whichever rank) has landed here. One thread waits, bounded,
  // then returns the counter to zero for the next call.
  if (p.ph[p.nph - 1].mode == kStreamTpReduce && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned* done = tp_pick(p.tp.done, p.tp.rank);
    const unsigned target = static_cast<unsigned>(p.ph[p.nph - 1].nblocks);
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

SPhase make_phase(const StreamPhase& s) {
  SPhase f{};
  f.N = static_cast<int>(s.N);
  f.K = static_cast<int>(s.K);
  f.kblocks = static_cast<int>((s.K + SBK - 1) / SBK);
  f.nblocks = static_cast<int>((s.N + SBN - 1) / SBN);
  f.units = f.kblocks * f.nblocks;
  f.mode = s.mode;
  f.col_scale = s.col_scale;
  f.bias = s.bias;
  f.gelu = s.gelu;
  f.residual = s.residual;
  f.ldr = s.ldr;
  f.out = s.out;
  f.ldo = s.ldo;
  f.part = s.part;
  f.ldp = s.ldp;
  f.counters = s.counters;
  return f;
}

}  // namespace

int stream_mpad(int64_t m) { return static_cast<int>((m + 31) / 32 * 32); }

size_t stream_counter_bytes(int64_t n) { return static_cast<size_t>((n + SBN - 1) / SBN) * sizeof(int); }

size_t stream_slot_bytes(int64_t m, int64_t n_max) {
  const int64_t slots = (n_max + SBN - 1) / SBN + cfg::kStreamMaxGrid - 1;
  return static_cast<size_t>(slots) * static_cast<size_t>(m) * SBN * 4;
}

int run_stream(const StreamProblem& sp, cudaStream_t stream, std::string* err) {
  if (sp.M <= 0 || sp.M > kStreamMaxRows || sp.nphases < 1 || sp.nphases > 2) {
    if (err) *err = "weight-streaming MLP: needs 1 <= M <= 64 and one or two phases";
    return -2;
  }
  for (int i = 0; i < sp.nphases; ++i) {
    const StreamPhase& f = sp.ph[i];
    if (f.N <= 0 || f.K <= 0 || (reinterpret_cast<uintptr_t>(f.A) & 15u) || (reinterpret_cast<uintptr_t>(f.W) & 15u) ||
        f.lda % 8 || f.ldw % 8 || !f.counters) {
      if (err) *err = "weight-streaming MLP: operands must be 16-byte aligned with leading dimensions % 8 == 0";
      return -2;
    }
  }
  if (!sp.slots || (sp.nphases > 1 && !sp.grid_bar)) {
    if (err) *err = "weight-streaming MLP: missing slots or phase barrier";
    return -2;
  }
  int* status = device_status_ptr(err);
  if (!status) return -3;
  SParams p{};
  p.M = static_cast<int>(sp.M);
  p.Mpad = stream_mpad(sp.M);
  p.nph = sp.nphases;
  p.ph[0] = make_phase(sp.ph[0]);
  if (sp.nphases > 1) p.ph[1] = make_phase(sp.ph[1]);
  p.slots = sp.slots;
  p.grid_bar = sp.grid_bar;
  p.tp = sp.tp;
  const int last_mode = sp.ph[sp.nphases - 1].mode;
  if (last_mode == kStreamTpReduce &&
      (sp.tp.world < 1 || sp.tp.world > kMaxTp || sp.tp.rank < 0 || sp.tp.rank >= sp.tp.world)) {
    if (err) *err = "weight-streaming MLP: bad tensor-parallel rank / world";
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
  const size_t smem =
      1024 + static_cast<size_t>(p.stages) * (W_STAGE + a_stage) + sizeof(SCtl) + cfg::kStreamScaleBytes;

  CUtensorMap tw0{}, ta0{}, tw1{}, ta1{};
  const StreamPhase& f0 = sp.ph[0];
  if (!make_map(&tw0, f0.W, f0.K, f0.N, f0.ldw, SBK, err)) return -3;
  if (!make_map(&ta0, f0.A, sp.M, f0.K, f0.lda, static_cast<uint32_t>(p.Mpad), err)) return -3;
  if (sp.nphases > 1) {
    const StreamPhase& f1 = sp.ph[1];
    if (!make_map(&tw1, f1.W, f1.K, f1.N, f1.ldw, SBK, err)) return -3;
    if (!make_map(&ta1, f1.A, sp.M, f1.K, f1.lda, static_cast<uint32_t>(p.Mpad), err)) return -3;
  } else if (sp.prefetch_units > 0 && sp.next.W) {
    if (!make_map(&tw1, sp.next.W, sp.next.K, sp.next.N, sp.next.ldw, SBK, err)) return -3;
    ta1 = ta0;
  } else {
    tw1 = tw0;
    ta1 = ta0;
  }
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
  // One CTA per SM (every CTA resident: the phase barrier waits for all of
  // them), no more CTAs than the smallest phase has units.
  int grid = sm_count() < cfg::kStreamMaxGrid ? sm_count() : cfg::kStreamMaxGrid;
  for (int i = 0; i < p.nph; ++i)
    if (p.ph[i].units < grid) grid = p.ph[i].units;
  // L2 prefetch of the weights streamed next. For the next launch this holds
  // only when that launch gets the same grid (the same CTA -> range map).
  if (sp.prefetch_units > 0) {
    if (p.nph > 1) {
      p.pf_units = sp.prefetch_units;
      p.pf_skip = p.stages;  // phase 1's first ring is loaded before the phase barrier
      p.pf_kblocks = p.ph[1].kblocks;
      p.pf_total = p.ph[1].units;
    } else if (sp.next.W) {
      const SPhase nx = make_phase(sp.next);
      int grid_next = sm_count() < cfg::kStreamMaxGrid ? sm_count() : cfg::kStreamMaxGrid;
      if (nx.units < grid_next) grid_next = nx.units;
      if (grid_next == grid) {
        p.pf_units = sp.prefetch_units;
        p.pf_skip = 0;
        p.pf_kblocks = nx.kblocks;
        p.pf_total = nx.units;
      }
    }
  }
  // Programmatic dependent launch: this grid's prologue and first ring of
  // weight tiles overlap the tail of the preceding grid (TFB200_PDL=0 turns it off).
  static const bool pdl = [] {
    const char* v = std::getenv("TFB200_PDL");
    return !(v && v[0] == '0');
  }();
  // Cooperative launch: the grid's CTAs are scheduled together, so the phase
  // barrier cannot wait on a CTA that another kernel on another stream keeps
  // off the GPU. Combined with programmatic serialization where the driver
  // accepts both (checked once per process).
  static std::atomic<int> pdl_with_coop{1};
  static const bool coop = [] {  // TFB200_STREAM_COOP=0: plain launch (for measurements)
    const char* v = std::getenv("TFB200_STREAM_COOP");
    return !(v && v[0] == '0');
  }();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = (coop && p.nph > 1) ? 1 : 0;  // only the phase barrier needs it
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_with_coop.load()) ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_stream, tw0, ta0, tw1, ta1, p);
  if (e != cudaSuccess && cfg.numAttrs == 2) {
    (void)cudaGetLastError();  // the refused launch's error; nothing was enqueued
    pdl_with_coop.store(0);
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, k_stream, tw0, ta0, tw1, ta1, p);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    if (err) *err = std::string("weight-streaming MLP launch: ") + cudaGetErrorString(e);
    return -3;
  }
  count_launch();
  return 0;
}

}  // namespace tfb200
