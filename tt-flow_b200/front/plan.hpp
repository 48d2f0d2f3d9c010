// B200 planner: replaces the reference's Tensix core-grid / circular-buffer
// planner (tensixflow lib/tensixflow/Scheduler/{GridPlanner,WeightPlanner,
// CBAllocator,NoCEstimator,EmissionEstimator,PlanReport}.cpp) and its roofline
// model (lib/tensixflow/Analysis/PerfModel.cpp:162-260) with a CTA-tile,
// shared-memory and TMEM budget planner for the kernels of libtfb200, keeping the
// reference's outputs: the schedule and emission attributes (with
// fused_feasible) and the plan JSON of schema/plan.schema.json.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace tfb200::front {

// The B200 entry of spec/devices.json (the reference's device-table layout);
// tests/test_device_spec.py holds these values and the time model to it.
struct B200Device {
  std::string name = "b200";
  std::string arch = "blackwell_sm100a";
  int64_t dies = 2;                     // grid_y
  int64_t sms_per_die = 74;             // grid_x
  int64_t smem_per_cta = 232448;        // 227 KiB opt-in dynamic shared memory
  int64_t tmem_columns = 512;           // x 128 lanes x 32 bit per SM
  int64_t l2_bytes = 126ll << 20;
  int64_t bf16_flops_per_clk_per_sm = 8192;  // dense tcgen05 kind::f16
  int64_t hbm_bytes_per_s = 7700000000000ll;  // HBM3e, HGX figure
  double sm_clock_hz = 1.965e9;
  // Measured on this pool's B200s (copy bandwidth, cuBLAS bf16 burst); the
  // model's time estimates use these.
  double measured_hbm_bytes_per_s = 6534.5e9;
  double measured_bf16_flops_per_s = 1635.3e12;
  int64_t sms() const { return dies * sms_per_die; }
};

const B200Device& b200();

struct PlanTensor {
  std::string name;
  std::vector<int64_t> shape;
  std::string dtype;
  std::string placement;  // "DRAM" (HBM) or "L1" (on-chip: smem / TMEM)
};

struct CbSpec {
  int64_t index, depth, tile_bytes;
};

// What the graph asks for, independent of the device.
struct PlanRequest {
  std::string graph_id;
  std::string fusion;  // "fused_rmsnorm_matmul" | "fused_mlp" | "none"
  bool already_fused = false;
  int64_t M = 0, K = 0, N = 0, H = 0;  // rows (leading dims flattened), widths
  int bpe = 2;
  std::vector<PlanTensor> tensors;
};

struct B200Plan {
  PlanRequest req;
  // kernel mapping
  std::string mapping;  // "persistent-cta-pair-tiles" | "persistent-cta-tiles" | "stream-k-swap-ab"
  int64_t tile_m = 0, tile_n = 0, tile_k = 0, stages = 0;
  int64_t tiles = 0, ctas = 0, max_tiles_per_cta = 0;
  int64_t smem_bytes = 0, tmem_columns = 0;
  int64_t fused_stage_tiles = 0;  // 32x32 bf16 tiles staged per CTA (all stages)
  bool fused_feasible = false;
  std::string infeasible_reason;
  // layout
  std::string act = "row-major", weight = "replicate", storage = "DRAM";
  std::vector<CbSpec> cbs;
  // traffic (bytes)
  int64_t dram_read = 0, dram_write = 0, l1_bytes = 0, multicast = 0;
  int64_t saved_read = 0, saved_write = 0, saved_intermediate = 0;
  // model
  int64_t flops = 0;
  int64_t launches = 0;
  int64_t est_cycles = 0;
  double compute_util = 0;
  double est_seconds = 0;
  std::string bottleneck;
  std::vector<std::string> suggestions;
};

B200Plan plan_b200(const PlanRequest& r);

// Textual attribute values in the dialect's syntax.
std::string schedule_attr(const B200Plan& p, bool with_cbs);
std::string emission_attr(const B200Plan& p);
// Plan JSON (fields and nesting of plan.schema.json), pretty-printed.
std::string plan_json(const B200Plan& p);
// One-paragraph human summary (the reference prints "Chosen layout" to stderr).
std::string plan_report(const B200Plan& p);

}  // namespace tfb200::front
