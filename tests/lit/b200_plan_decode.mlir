// RUN: tensixflow-opt --tensixflow-plan-noc-sharding --tensixflow-allocate-circular-buffers %s | FileCheck %s
// RUN: tensixflow-opt --tensixflow-to-json %s | FileCheck %s --check-prefix=JSON

// The decode-shaped MLP (32 tokens, 8192 -> 28672 -> 8192) written directly as
// a fused_mlp with the 1-D [H] bias the verifier accepts. Few rows: the planner
// picks the weight-streaming split-K kernel (weight columns on the MMA's
// 128-row side, 32 tokens on its N side), which streams a disjoint slice of the
// weights through each of the 148 CTAs ("shard"). Ten 20 KiB stages and a
// 64-column TMEM double buffer fit; the model is HBM-bound.

// CHECK: tensixflow.emission = #tensixflow.emission<mapping "stream-k-swap-ab", cores_used 148, max_tiles_per_core 388, dram_read 943005696, dram_write 2883712, fused_stage_tiles 100, fused_feasible true>
// CHECK-SAME: weight "shard", storage "HBM", fusion "fused_mlp", cbs [0:10:4096, 1:10:16384, 16:4:16384]
// JSON: "graph_id": "decode"
// JSON: "weight_strategy": "shard"
// JSON: "mapping": "stream-k-swap-ab"
// JSON: "fused_feasible": true
// JSON: "bottleneck": "dram"
tensixflow.func @decode(%x: tensor<32x8192xbf16>, %gamma: tensor<8192xbf16>, %w1: tensor<8192x28672xbf16>, %b1: tensor<28672xbf16>, %w2: tensor<28672x8192xbf16>, %residual: tensor<32x8192xbf16>) -> tensor<32x8192xbf16> {
  %0 = tensixflow.fused_mlp %x, %gamma, %w1, %b1, %w2, %residual {epsilon = 1.0e-05 : f32} : tensor<32x8192xbf16>, tensor<8192xbf16>, tensor<8192x28672xbf16>, tensor<28672xbf16>, tensor<28672x8192xbf16>, tensor<32x8192xbf16> -> tensor<32x8192xbf16>
  tensixflow.return %0 : tensor<32x8192xbf16>
}
