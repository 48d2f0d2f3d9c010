// Tile, stage and shared-memory geometry of the kernels in this library. The
// kernels (gemm_sm100.cu, stream_sm100.cu) and the B200 planner
// (front/plan.cpp) both take it from here, so a plan describes exactly what the
// library launches; the kernels check their control-block sizes against it at
// compile time. Plain C++ (the planner is host code).
#pragma once

namespace tfb200::cfg {

// One CTA (k_gemm, up to 128 rows): 128 x 256 output tiles, 64-deep k blocks,
// 4 shared-memory stages.
constexpr int kTileM = 128, kTileN = 256, kTileK = 64, kStages = 4;
constexpr int kGemmCtlBytes = 112;  // k_gemm's barriers, TMEM address and abort flag

// CTA pair (k_gemm_pair, more than 128 rows): 256 x 256 tiles per pair of CTAs
// (cta_group::2), 6 stages of 16 KiB A + 16 KiB B per CTA, 8 epilogue warps
// (two per TMEM lane quadrant, each taking half of the tile's columns) with
// two 32 x 32 bf16 staging buffers each.
constexpr int kPairEpiWarps = 8;
constexpr int kPairThreads = (4 + kPairEpiWarps) * 32;
constexpr int kPairTileM = 2 * kTileM, kPairStages = 6, kPairStagingBytes = kPairEpiWarps * 2 * 32 * 32 * 2;
constexpr int kPairCtlBytes = 144;
constexpr int kGroupM = 16;  // raster group of both tiled kernels (row tiles)

// Weight-streaming kernel (k_stream, at most kStreamMaxRows token rows): units
// of 128 weight columns x 64 k, up to 12 stages within 200 KiB of shared memory,
// kStreamAcc TMEM accumulators in rotation.
constexpr int kStreamMaxRows = 64;
constexpr int kStreamN = 128, kStreamK = 64, kStreamMaxStages = 12, kStreamBudget = 200 * 1024;
constexpr int kStreamAcc = 4;
// Most CTAs of the weight-streaming kernel (one per SM; sizes its partial-sum slots).
constexpr int kStreamMaxGrid = 160;
constexpr int kStreamCtlBytes = 280;
// Row scales (1/rms) the up-projection's finishers read, staged after the control block.
constexpr int kStreamScaleBytes = kStreamMaxRows * 4;

}  // namespace tfb200::cfg
