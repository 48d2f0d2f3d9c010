// RUN: tensixflow-opt --tensixflow-fuse-rmsnorm-matmul --tensixflow-plan-noc-sharding --tensixflow-allocate-circular-buffers %s | FileCheck %s

// The fused MLP block at 8192 tokens x 4096 x 16384. The whole chain fuses
// (five intermediates, 939524096 bytes). Two tiled GEMMs: 4096 tiles for the
// up-projection (28 per CTA) and 1024 for the down-projection. The bias-add,
// GELU and residual-add never reach HBM: matmul1 out and add1 out
// (8192 x 16384 each) and matmul2 out (8192 x 4096), 603979776 bytes saved.

// CHECK: tensixflow.emission = #tensixflow.emission<mapping "persistent-cta-pair-tiles", cores_used 148, max_tiles_per_core 28, dram_read 738238464, dram_write 402685952, fused_stage_tiles 96, fused_feasible true>
// CHECK-SAME: tensixflow.fusion_report = 1 : i64
// CHECK-SAME: fusion "fused_mlp", cbs [0:6:16384, 1:6:16384, 16:2:131072]
// CHECK-SAME: saved_read 603979776, saved_write 603979776, saved_intermediate 603979776>
// CHECK: tensixflow.fused_mlp %arg0, %arg1, %arg2, %arg3, %arg4, %arg5 {epsilon = 1.0e-05 : f32, tensixflow.eliminated_bytes = 939524096 : i64, tensixflow.eliminated_tensors = 5 : i64}
// CHECK-NOT: tensixflow.gelu
tensixflow.func @mlp(%x: tensor<1x8192x4096xbf16>, %gamma: tensor<4096xbf16>, %w1: tensor<4096x16384xbf16>, %b1: tensor<1x8192x16384xbf16>, %w2: tensor<16384x4096xbf16>, %residual: tensor<1x8192x4096xbf16>) -> tensor<1x8192x4096xbf16> {
  %0 = tensixflow.rmsnorm %x, %gamma {epsilon = 1.0e-05 : f32} : tensor<1x8192x4096xbf16>, tensor<4096xbf16> -> tensor<1x8192x4096xbf16>
  %1 = tensixflow.matmul %0, %w1 : tensor<1x8192x4096xbf16> x tensor<4096x16384xbf16> -> tensor<1x8192x16384xbf16>
  %2 = tensixflow.add %1, %b1 : tensor<1x8192x16384xbf16>
  %3 = tensixflow.gelu %2 : tensor<1x8192x16384xbf16>
  %4 = tensixflow.matmul %3, %w2 : tensor<1x8192x16384xbf16> x tensor<16384x4096xbf16> -> tensor<1x8192x4096xbf16>
  %5 = tensixflow.add %4, %residual : tensor<1x8192x4096xbf16>
  tensixflow.return %5 : tensor<1x8192x4096xbf16>
}
