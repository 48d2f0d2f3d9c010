// RUN: tensixflow-opt --allow-unregistered-dialect --tensixflow-import-ttir %s | FileCheck %s --check-prefix=IMPORT
// RUN: tensixflow-opt --allow-unregistered-dialect --tensixflow-import-ttir --tensixflow-device=b200 --tensixflow-fuse-rmsnorm-matmul --tensixflow-plan-noc-sharding --tensixflow-allocate-circular-buffers %s | FileCheck %s --check-prefix=PLAN

// Bare-tensor TTIR of the QKV projection (rms_norm -> matmul, 8192 x 4096 x
// 6144) imported and planned for the B200: the importer rebuilds the pair in the
// tensixflow dialect (the f32 epsilon prints as the reference prints it), the
// fusion pass folds it into one fused_rmsnorm_matmul and the planner maps it
// onto the persistent CTA-tile GEMM.

// IMPORT-LABEL: tensixflow.func @qkv
// IMPORT: %0 = tensixflow.rmsnorm %arg0, %arg1 {epsilon = 9.99999974E-6 : f32} : tensor<8192x4096xbf16>, tensor<4096xbf16> -> tensor<8192x4096xbf16>
// IMPORT: %1 = tensixflow.matmul %0, %arg2 : tensor<8192x4096xbf16> x tensor<4096x6144xbf16> -> tensor<8192x6144xbf16>
// IMPORT: tensixflow.return %1 : tensor<8192x6144xbf16>

// PLAN: tensixflow.emission = #tensixflow.emission<mapping "persistent-cta-pair-tiles", cores_used 148, max_tiles_per_core 11
// PLAN-SAME: fused_feasible true>
// PLAN-SAME: fusion "fused_rmsnorm_matmul"
// PLAN: tensixflow.fused_rmsnorm_matmul %arg0, %arg1, %arg2 {epsilon = 9.99999974E-6 : f32
func.func @qkv(%arg0: tensor<8192x4096xbf16>, %arg1: tensor<4096xbf16>, %arg2: tensor<4096x6144xbf16>) -> tensor<8192x6144xbf16> {
  %0 = "ttir.rms_norm"(%arg0, %arg1) <{epsilon = 1.000000e-05 : f32, normalized_shape = array<i64: 4096>, operandSegmentSizes = array<i32: 1, 1, 0>}> : (tensor<8192x4096xbf16>, tensor<4096xbf16>) -> tensor<8192x4096xbf16>
  %1 = "ttir.matmul"(%0, %arg2) : (tensor<8192x4096xbf16>, tensor<4096x6144xbf16>) -> tensor<8192x6144xbf16>
  return %1 : tensor<8192x6144xbf16>
}
