// RUN: split-file %s %t
// RUN: not tensixflow-opt --tensixflow-device=n150 --tensixflow-plan-noc-sharding %t/ok.mlir 2>&1 | FileCheck %t/ok.mlir --check-prefix=DEV
// RUN: tensixflow-opt -verify-diagnostics %t/b1.mlir
// RUN: tensixflow-opt -verify-diagnostics %t/w2.mlir
// RUN: tensixflow-opt -verify-diagnostics %t/residual.mlir

//--- ok.mlir
// The B200 backend plans for b200 only; a Tensix device name is refused.
// DEV: unknown device 'n150'; valid devices: b200
tensixflow.func @mm(%a: tensor<128x64xbf16>, %b: tensor<64x32xbf16>) -> tensor<128x32xbf16> {
  %0 = tensixflow.matmul %a, %b : tensor<128x64xbf16> x tensor<64x32xbf16> -> tensor<128x32xbf16>
  tensixflow.return %0 : tensor<128x32xbf16>
}

//--- b1.mlir
tensixflow.func @bad_bias(%x: tensor<32x64xbf16>, %g: tensor<64xbf16>, %w1: tensor<64x128xbf16>, %b1: tensor<96xbf16>, %w2: tensor<128x64xbf16>, %r: tensor<32x64xbf16>) -> tensor<32x64xbf16> {
  // expected-error @below {{b1 last dimension (96) must match w1's hidden dimension (128)}}
  %0 = tensixflow.fused_mlp %x, %g, %w1, %b1, %w2, %r : tensor<32x64xbf16>, tensor<64xbf16>, tensor<64x128xbf16>, tensor<96xbf16>, tensor<128x64xbf16>, tensor<32x64xbf16> -> tensor<32x64xbf16>
  tensixflow.return %0 : tensor<32x64xbf16>
}

//--- w2.mlir
tensixflow.func @bad_w2(%x: tensor<32x64xbf16>, %g: tensor<64xbf16>, %w1: tensor<64x128xbf16>, %b1: tensor<128xbf16>, %w2: tensor<96x64xbf16>, %r: tensor<32x64xbf16>) -> tensor<32x64xbf16> {
  // expected-error @below {{mismatched hidden dimensions: w1 H = 128 but w2 H = 96}}
  %0 = tensixflow.fused_mlp %x, %g, %w1, %b1, %w2, %r : tensor<32x64xbf16>, tensor<64xbf16>, tensor<64x128xbf16>, tensor<128xbf16>, tensor<96x64xbf16>, tensor<32x64xbf16> -> tensor<32x64xbf16>
  tensixflow.return %0 : tensor<32x64xbf16>
}

//--- residual.mlir
tensixflow.func @bad_residual(%x: tensor<32x64xbf16>, %g: tensor<64xbf16>, %w1: tensor<64x128xbf16>, %b1: tensor<128xbf16>, %w2: tensor<128x64xbf16>, %r: tensor<16x64xbf16>) -> tensor<16x64xbf16> {
  // expected-error @below {{residual shape must equal the output shape}}
  %0 = tensixflow.fused_mlp %x, %g, %w1, %b1, %w2, %r : tensor<32x64xbf16>, tensor<64xbf16>, tensor<64x128xbf16>, tensor<128xbf16>, tensor<128x64xbf16>, tensor<16x64xbf16> -> tensor<16x64xbf16>
  tensixflow.return %0 : tensor<16x64xbf16>
}
