// RUN: tensixflow-opt --tensixflow-device=b200 --tensixflow-fuse-rmsnorm-matmul --tensixflow-plan-noc-sharding --tensixflow-allocate-circular-buffers %s | FileCheck %s
// RUN: tensixflow-opt --tensixflow-device=b200 --tensixflow-plan-noc-sharding %s | FileCheck %s --check-prefix=PLAN

// The QKV projection workload (8192 x 4096 x 6144, bf16). The single-use
// rmsnorm -> matmul fuses; the B200 planner maps it onto 74 persistent CTA pairs
// (148 CTAs, cta_group::2) of 256 x 256 tiles (768 tiles, at most 11 per pair),
// six 32 KiB shared-memory stages per CTA (its 128 rows of A and its 128 columns
// of B, 16 KiB each) and two TMEM accumulators of 128 x 256 fp32 per CTA, which
// fit the 227 KiB / 512-column budget: fused_feasible.
// The normalised row is staged once in HBM as bf16(x * gamma), so no traffic
// is saved on it.

// CHECK: module attributes {tensixflow.device = "b200", tensixflow.emission = #tensixflow.emission<mapping "persistent-cta-pair-tiles", cores_used 148, max_tiles_per_core 11, dram_read 184557568, dram_write 167804928, fused_stage_tiles 96, fused_feasible true>, tensixflow.fusion_report = 1 : i64, tensixflow.schedule = #tensixflow.schedule<grid 2x74, act "row-major", weight "replicate", storage "HBM", fusion "fused_rmsnorm_matmul", cbs [0:6:16384, 1:6:16384, 16:2:131072]
// CHECK-SAME: multicast 0, saved_read 0, saved_write 0, saved_intermediate 0>}
// CHECK: tensixflow.fused_rmsnorm_matmul %arg0, %arg1, %arg2 {epsilon = 1.0e-05 : f32, tensixflow.eliminated_bytes = 67108864 : i64, tensixflow.eliminated_tensors = 1 : i64}

// Without the fusion pass the planner still plans the pair as fused, and the
// buffer list stays empty until --tensixflow-allocate-circular-buffers runs.
// PLAN: fusion "fused_rmsnorm_matmul", cbs []
// PLAN: tensixflow.rmsnorm
// PLAN: tensixflow.matmul
tensixflow.func @qkv(%x: tensor<8192x4096xbf16>, %gamma: tensor<4096xbf16>, %w: tensor<4096x6144xbf16>) -> tensor<8192x6144xbf16> {
  %0 = tensixflow.rmsnorm %x, %gamma {epsilon = 1.0e-05 : f32} : tensor<8192x4096xbf16>, tensor<4096xbf16> -> tensor<8192x4096xbf16>
  %1 = tensixflow.matmul %0, %w : tensor<8192x4096xbf16> x tensor<4096x6144xbf16> -> tensor<8192x6144xbf16>
  tensixflow.return %1 : tensor<8192x6144xbf16>
}
