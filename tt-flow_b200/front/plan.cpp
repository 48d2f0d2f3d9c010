// B200 planner, roofline model and plan JSON (see plan.hpp).
#include "plan.hpp"

#include "../csrc/kernel_config.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <sstream>

namespace tfb200::front {

namespace {

int64_t cdiv(int64_t a, int64_t b) { return b > 0 ? (a + b - 1) / b : 0; }

// Tile geometry of the kernels in libtfb200, from the header the kernels use
// (csrc/kernel_config.h): one CTA (k_gemm, up to 128 rows), the CTA pair
// (k_gemm_pair, more than 128 rows; at most 74 resident pairs) and the
// weight-streaming kernel (k_stream, at most kStreamMaxRows rows).
constexpr int64_t kTileM = cfg::kTileM, kTileN = cfg::kTileN, kTileK = cfg::kTileK, kStages = cfg::kStages;
constexpr int64_t kGemmCtlBytes = cfg::kGemmCtlBytes;
constexpr int64_t kPairTileM = cfg::kPairTileM, kPairStages = cfg::kPairStages;
constexpr int64_t kPairStagingBytes = cfg::kPairStagingBytes, kPairCtlBytes = cfg::kPairCtlBytes;
constexpr int64_t kMaxPairs = 74;
constexpr int64_t kStreamCtlBytes = cfg::kStreamCtlBytes;
constexpr int64_t kStreamMaxRows = cfg::kStreamMaxRows;
constexpr int64_t kStreamN = cfg::kStreamN, kStreamK = cfg::kStreamK, kStreamMaxStages = cfg::kStreamMaxStages;
constexpr int64_t kStreamBudget = cfg::kStreamBudget, kStreamAcc = cfg::kStreamAcc;
constexpr double kLaunchSeconds = 3e-6;  // per kernel launch boundary (ramp up / drain)
// Fractions of the measured peaks the kernels sustain, measured on B200 with
// CUDA events: the tcgen05 GEMM ran the fused MLP 8192x4096x16384 at
// 1356-1460 TFLOP/s (82-88 % of 1662.2) and the fused RMSNorm+MatMul
// 8192x4096x6144 at 1384-1411 TFLOP/s (83-85 %); the weight-streaming kernels
// ran the decode MLP 32x8192x28672 at 5961-6108 GB/s (91-93.5 % of 6534.5).
// (spec/devices.json "model" records both with their basis.)
constexpr double kTensorEfficiency = 0.87;
constexpr double kHbmEfficiency = 0.93;

std::string q(const std::string& s) { return "\"" + s + "\""; }

struct Gemm {
  int64_t M, N, K;
};

void add_tiled(B200Plan& p, const Gemm& g, bool pair) {
  const B200Device& d = b200();
  const int64_t tm = pair ? kPairTileM : kTileM;
  const int64_t tiles = cdiv(g.M, tm) * cdiv(g.N, kTileN);
  p.tiles += tiles;
  // A pair's two CTAs share one tile; max_tiles_per_cta counts tiles per pair then.
  const int64_t workers = std::min<int64_t>(pair ? kMaxPairs : d.sms(), tiles);
  p.ctas = std::max(p.ctas, pair ? 2 * workers : workers);
  p.max_tiles_per_cta = std::max(p.max_tiles_per_cta, cdiv(tiles, workers));
  // every staged A/B byte is written by TMA and read by the MMA once
  p.l1_bytes += 2 * tiles * cdiv(g.K, kTileK) * (tm + kTileN) * kTileK * 2;
  p.launches += 1;
}

}  // namespace

const B200Device& b200() {
  static const B200Device d;
  return d;
}

B200Plan plan_b200(const PlanRequest& r) {
  const B200Device& d = b200();
  B200Plan p;
  p.req = r;
  const int64_t M = r.M, K = r.K, N = r.N, H = r.H, b = r.bpe;
  const int64_t Kst = cdiv(K, 8) * 8;  // staged leading dimension
  const bool mlp = r.fusion == "fused_mlp";
  const bool rms = mlp || r.fusion == "fused_rmsnorm_matmul";
  if (M <= 0 || K <= 0 || N <= 0 || (mlp && H <= 0)) {
    p.infeasible_reason = "empty or dynamic dimension";
    p.mapping = "none";
    return p;
  }
  const bool stream = mlp && M <= kStreamMaxRows;
  if (stream) {
    // Weight-streaming swap-AB split-K kernel: 128 weight columns x 64 k per unit.
    const int64_t mpad = cdiv(M, 32) * 32;
    const int64_t a_stage = mpad * kStreamK * 2, w_stage = kStreamN * kStreamK * 2;
    p.mapping = "stream-k-swap-ab";
    p.tile_m = kStreamN;
    p.tile_n = mpad;
    p.tile_k = kStreamK;
    p.stages = std::min<int64_t>(kStreamMaxStages, kStreamBudget / (w_stage + a_stage));
    p.smem_bytes = 1024 + p.stages * (w_stage + a_stage) + kStreamCtlBytes + cfg::kStreamScaleBytes;
    int64_t cols = 32;
    while (cols < kStreamAcc * mpad) cols <<= 1;
    p.tmem_columns = cols;
    const int64_t units_up = cdiv(H, kStreamN) * cdiv(K, kStreamK);
    const int64_t units_dn = cdiv(N, kStreamN) * cdiv(H, kStreamK);
    p.tiles = units_up + units_dn;
    p.ctas = std::min<int64_t>(d.sms(), std::max(units_up, units_dn));
    p.max_tiles_per_cta = cdiv(units_up, std::min<int64_t>(d.sms(), units_up)) +
                          cdiv(units_dn, std::min<int64_t>(d.sms(), units_dn));
    p.l1_bytes = 2 * (units_up + units_dn) * (w_stage + a_stage);
    p.fused_stage_tiles = p.stages * (w_stage + a_stage) / 2048;
    p.weight = "shard";  // every CTA streams a disjoint slice of the weights
    p.cbs = {{0, p.stages, a_stage}, {1, p.stages, w_stage}, {16, kStreamAcc, mpad * 128 * 4}};
    p.launches = 3;
    p.fused_feasible = p.smem_bytes <= d.smem_per_cta && p.tmem_columns <= d.tmem_columns && mpad <= 256;
    if (!p.fused_feasible) p.infeasible_reason = "streamed stages exceed shared memory or TMEM";
  } else if (M > kTileM) {
    // What the library launches for more than 128 rows: the CTA-pair kernel.
    p.mapping = "persistent-cta-pair-tiles";
    p.tile_m = kPairTileM;
    p.tile_n = kTileN;
    p.tile_k = kTileK;
    p.stages = kPairStages;
    const int64_t a_stage = kTileM * kTileK * 2, b_stage = (kTileN / 2) * kTileK * 2;  // per CTA
    p.smem_bytes = 1024 + kPairStages * (a_stage + b_stage) + kPairStagingBytes + kPairCtlBytes;
    p.tmem_columns = 2 * kTileN;  // double-buffered 128 x 256 fp32 accumulator per CTA
    if (mlp) {
      add_tiled(p, {M, H, K}, true);
      add_tiled(p, {M, N, H}, true);
    } else {
      add_tiled(p, {M, N, K}, true);
    }
    if (rms) p.launches += 1;  // staging pass
    p.fused_stage_tiles = kPairStages * (a_stage + b_stage) / 2048;
    p.cbs = {{0, kPairStages, a_stage}, {1, kPairStages, b_stage}, {16, 2, kTileM * kTileN * 4}};
    p.fused_feasible = p.smem_bytes <= d.smem_per_cta && p.tmem_columns <= d.tmem_columns;
    if (!p.fused_feasible) p.infeasible_reason = "tile stages exceed shared memory or TMEM";
  } else {
    p.mapping = "persistent-cta-tiles";
    p.tile_m = kTileM;
    p.tile_n = kTileN;
    p.tile_k = kTileK;
    p.stages = kStages;
    p.smem_bytes = 1024 + kStages * (kTileM + kTileN) * kTileK * 2 + kGemmCtlBytes;
    p.tmem_columns = 2 * kTileN;  // double-buffered fp32 accumulator
    if (mlp) {
      add_tiled(p, {M, H, K}, false);
      add_tiled(p, {M, N, H}, false);
    } else {
      add_tiled(p, {M, N, K}, false);
    }
    if (rms) p.launches += 1;  // staging pass
    p.fused_stage_tiles = kStages * (kTileM + kTileN) * kTileK * 2 / 2048;
    p.cbs = {{0, kStages, kTileM * kTileK * 2}, {1, kStages, kTileK * kTileN * 2}, {16, 2, kTileM * kTileN * 4}};
    p.fused_feasible = p.smem_bytes <= d.smem_per_cta && p.tmem_columns <= d.tmem_columns;
    if (!p.fused_feasible) p.infeasible_reason = "tile stages exceed shared memory or TMEM";
  }
  // Compulsory HBM traffic of the emitted kernels (each tensor once; panels
  // re-read from HBM when L2 does not hold them are not counted).
  if (mlp) {
    const int64_t x = M * K * b, a = M * Kst * b, inv = M * 4, w1 = K * H * b, w2 = H * N * b, b1 = H * b,
                  hid = M * H * b, y = M * N * b, res = M * N * b, g = K * b;
    p.dram_read = x + g + a + w1 + b1 + hid + w2 + res;
    p.dram_write = a + inv + hid + y;
    p.flops = 2 * M * K * H + 2 * M * H * N;
    // matmul1 out, bias-add out (M x H each) and matmul2 out (M x N) never reach HBM;
    // the normalised row (staged as bf16(x*gamma)) and the GELU output do.
    p.saved_intermediate = 2 * M * H * b + M * N * b;
    p.storage = "HBM";
  } else if (rms) {
    const int64_t x = M * K * b, a = M * Kst * b, inv = M * 4, w = K * N * b, y = M * N * b, g = K * b;
    p.dram_read = x + g + a + w;
    p.dram_write = a + inv + y;
    p.flops = 2 * M * K * N;
    p.saved_intermediate = 0;  // the normalised row is staged once in HBM as bf16(x*gamma)
    p.storage = "HBM";
  } else {
    p.dram_read = (M * K + K * N) * b;
    p.dram_write = M * N * b;
    p.flops = 2 * M * K * N;
    p.storage = "DRAM";
  }
  if (r.fusion == "none") p.saved_intermediate = 0;
  p.saved_read = p.saved_intermediate;
  p.saved_write = p.saved_intermediate;
  p.multicast = 0;  // no cluster multicast anywhere: weight reuse comes from L2

  // Roofline with the measured peaks scaled by the sustained fractions above:
  // time = max(compute, HBM) + launch boundaries.
  const double t_compute = static_cast<double>(p.flops) / (d.measured_bf16_flops_per_s * kTensorEfficiency);
  const double t_hbm = static_cast<double>(p.dram_read + p.dram_write) / (d.measured_hbm_bytes_per_s * kHbmEfficiency);
  p.est_seconds = std::max(t_compute, t_hbm) + kLaunchSeconds * static_cast<double>(p.launches);
  p.est_cycles = static_cast<int64_t>(std::llround(p.est_seconds * d.sm_clock_hz));
  p.compute_util = p.est_seconds > 0 ? t_compute / p.est_seconds : 0.0;
  const double ratio = t_hbm > 0 ? t_compute / t_hbm : 1e9;
  p.bottleneck = ratio > 1.1 ? "compute" : (ratio < 0.9 ? "dram" : "balanced");
  if (stream) {
    p.suggestions.push_back("weight-bound: split W1 by columns and W2 by rows over GPUs (tensor parallel) to cut bytes per GPU");
  } else {
    if (p.tiles < d.sms())
      p.suggestions.push_back("fewer output tiles (" + std::to_string(p.tiles) +
                              ") than SMs: use smaller tiles or split K to fill the 148 SMs");
    const double waves = static_cast<double>(p.tiles) / static_cast<double>(d.sms());
    // (Not for the CTA-pair kernel: splitting its last wave into half tiles measured slower on the B200, whose
    // idle SMs in a short last wave let the busy ones clock higher under the power limit.)
    if (p.mapping != "persistent-cta-pair-tiles" && waves > 1.0 && waves - std::floor(waves) > 0 &&
        waves - std::floor(waves) < 0.5)
      p.suggestions.push_back("last wave runs " + std::to_string(static_cast<int>((waves - std::floor(waves)) * 100)) +
                              "% full: a stream-K split of the tail would balance the SMs");
    if (M % kTileM != 0) p.suggestions.push_back("M is not a multiple of 128: the last row tile is partly empty");
  }
  if (p.bottleneck == "compute" && p.mapping == "persistent-cta-tiles")
    p.suggestions.push_back("tensor-bound: 2-CTA (cta_group::2) tiles halve B-operand shared-memory traffic");
  return p;
}

std::string schedule_attr(const B200Plan& p, bool with_cbs) {
  const B200Device& d = b200();
  std::ostringstream os;
  os << "#tensixflow.schedule<grid " << d.dies << "x" << d.sms_per_die << ", act " << q(p.act) << ", weight "
     << q(p.weight) << ", storage " << q(p.storage) << ", fusion " << q(p.req.fusion) << ", cbs [";
  if (with_cbs)
    for (size_t i = 0; i < p.cbs.size(); ++i)
      os << (i ? ", " : "") << p.cbs[i].index << ":" << p.cbs[i].depth << ":" << p.cbs[i].tile_bytes;
  os << "], dram_read " << p.dram_read << ", dram_write " << p.dram_write << ", l1 " << p.l1_bytes << ", multicast "
     << p.multicast << ", saved_read " << p.saved_read << ", saved_write " << p.saved_write << ", saved_intermediate "
     << p.saved_intermediate << ">";
  return os.str();
}

std::string emission_attr(const B200Plan& p) {
  std::ostringstream os;
  os << "#tensixflow.emission<mapping " << q(p.mapping) << ", cores_used " << p.ctas << ", max_tiles_per_core "
     << p.max_tiles_per_cta << ", dram_read " << p.dram_read << ", dram_write " << p.dram_write
     << ", fused_stage_tiles " << p.fused_stage_tiles << ", fused_feasible " << (p.fused_feasible ? "true" : "false")
     << ">";
  return os.str();
}

namespace {

std::string jstr(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\';
    if (c == '\n') {
      o += "\\n";
      continue;
    }
    o += c;
  }
  return o + "\"";
}

std::string jnum(double v) {
  char buf[64];
  std::snprintf(buf, sizeof(buf), "%.6g", v);
  return buf;
}

}  // namespace

std::string plan_json(const B200Plan& p) {
  const B200Device& d = b200();
  std::ostringstream o;
  o << "{\n";
  o << "  \"graph_id\": " << jstr(p.req.graph_id) << ",\n";
  o << "  \"device\": {\n    \"name\": " << jstr(d.name) << ",\n    \"arch\": " << jstr(d.arch)
    << ",\n    \"grid_x\": " << d.sms_per_die << ",\n    \"grid_y\": " << d.dies << ",\n    \"l1_usable_bytes\": "
    << d.smem_per_cta << ",\n    \"flops_per_cycle_per_core\": " << d.bf16_flops_per_clk_per_sm
    << ",\n    \"dram_bandwidth_bytes_per_second\": " << d.hbm_bytes_per_s << "\n  },\n";
  o << "  \"activation_sharding\": " << jstr(p.act) << ",\n";
  o << "  \"weight_strategy\": " << jstr(p.weight) << ",\n";
  o << "  \"intermediate_storage\": " << jstr(p.storage) << ",\n";
  o << "  \"fusion\": " << jstr(p.req.fusion) << ",\n";
  o << "  \"estimated_dram_reads_saved\": " << p.saved_read << ",\n";
  o << "  \"estimated_intermediate_writes_saved\": " << p.saved_write << ",\n";
  o << "  \"tensors\": [";
  for (size_t i = 0; i < p.req.tensors.size(); ++i) {
    const PlanTensor& t = p.req.tensors[i];
    o << (i ? "," : "") << "\n    {\n      \"name\": " << jstr(t.name) << ",\n      \"shape\": [";
    for (size_t k = 0; k < t.shape.size(); ++k) o << (k ? ", " : "") << t.shape[k];
    o << "],\n      \"dtype\": " << jstr(t.dtype) << ",\n      \"placement\": " << jstr(t.placement) << "\n    }";
  }
  o << (p.req.tensors.empty() ? "],\n" : "\n  ],\n");
  o << "  \"layout\": {\n    \"activation_sharding\": " << jstr(p.act) << ",\n    \"weight_strategy\": "
    << jstr(p.weight) << "\n  },\n";
  o << "  \"shard_grid\": {\n    \"grid_y\": " << d.dies << ",\n    \"grid_x\": " << d.sms_per_die << "\n  },\n";
  o << "  \"cb_specs\": [";
  for (size_t i = 0; i < p.cbs.size(); ++i)
    o << (i ? "," : "") << "\n    {\n      \"index\": " << p.cbs[i].index << ",\n      \"depth\": " << p.cbs[i].depth
      << ",\n      \"tile_bytes\": " << p.cbs[i].tile_bytes << "\n    }";
  o << (p.cbs.empty() ? "],\n" : "\n  ],\n");
  o << "  \"noc\": {\n    \"dram_read_bytes\": " << p.dram_read << ",\n    \"dram_write_bytes\": " << p.dram_write
    << ",\n    \"l1_bytes\": " << p.l1_bytes << ",\n    \"multicast_bytes\": " << p.multicast << "\n  },\n";
  o << "  \"emission\": {\n    \"mapping\": " << jstr(p.mapping) << ",\n    \"cores_used\": " << p.ctas
    << ",\n    \"max_tiles_per_core\": " << p.max_tiles_per_cta << ",\n    \"dram_read_bytes\": " << p.dram_read
    << ",\n    \"dram_write_bytes\": " << p.dram_write << ",\n    \"fused_stage_tiles\": " << p.fused_stage_tiles
    << ",\n    \"fused_feasible\": " << (p.fused_feasible ? "true" : "false") << "\n  },\n";
  o << "  \"perf\": {\n    \"est_cycles\": " << p.est_cycles << ",\n    \"compute_util\": " << jnum(p.compute_util)
    << ",\n    \"bottleneck\": " << jstr(p.bottleneck == "dram" ? "dram" : p.bottleneck) << ",\n    \"suggestions\": [";
  for (size_t i = 0; i < p.suggestions.size(); ++i) o << (i ? ", " : "") << jstr(p.suggestions[i]);
  o << "]\n  },\n";
  std::ostringstream grid, shards, cbu, tl;
  grid << d.dies << " dies x " << d.sms_per_die << " SMs; " << p.ctas << " persistent CTAs";
  shards << p.mapping << ": " << p.tiles << " work units of " << p.tile_m << "x" << p.tile_n << "x" << p.tile_k
         << ", at most " << p.max_tiles_per_cta << " per CTA";
  cbu << p.stages << " shared-memory stages, " << p.smem_bytes << " B of " << d.smem_per_cta << "; TMEM "
      << p.tmem_columns << " of " << d.tmem_columns << " columns";
  tl << p.launches << " launches, " << jnum(p.est_seconds * 1e6) << " us estimated";
  o << "  \"viz\": {\n    \"core_grid\": " << jstr(grid.str()) << ",\n    \"shards\": " << jstr(shards.str())
    << ",\n    \"noc_routes\": " << jstr("none: TMA loads per CTA, weight reuse through L2, no multicast")
    << ",\n    \"cb_usage\": " << jstr(cbu.str()) << ",\n    \"timeline\": " << jstr(tl.str()) << "\n  }\n";
  o << "}\n";
  return o.str();
}

std::string plan_report(const B200Plan& p) {
  std::ostringstream os;
  os << "Chosen layout (b200): graph " << p.req.graph_id << ", fusion " << p.req.fusion << ", mapping " << p.mapping
     << ", " << p.ctas << " CTAs, " << p.stages << " stages (" << p.smem_bytes << " B smem, " << p.tmem_columns
     << " TMEM columns), fused_feasible " << (p.fused_feasible ? "true" : "false") << ", estimated "
     << p.est_seconds * 1e6 << " us (" << p.bottleneck << "-bound)\n";
  return os.str();
}

}  // namespace tfb200::front
