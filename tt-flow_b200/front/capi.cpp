// C ABI of the front end (declared in include/tfb200.h): tfb200_opt, tfb200_plan.
#include <cstring>
#include <string>

#include "../../include/tfb200.h"
#include "passes.hpp"
#include "plan.hpp"
#include "plan_in.hpp"

namespace tfb200 {
void set_last_error(const std::string& msg);
}

extern "C" int tfb200_opt(const char* text, const char* args, char* out, size_t cap, size_t* needed) {
  if (!text) {
    tfb200::set_last_error("tfb200_opt: null input text");
    return TFB200_EINVAL;
  }
  const auto r = tfb200::front::run_pipeline(text, args ? std::string(args) : std::string());
  if (!r.ok) {
    tfb200::set_last_error("tfb200_opt: " + r.diag);
    return TFB200_EINVAL;
  }
  if (needed) *needed = r.output.size() + 1;
  if (!out || cap < r.output.size() + 1) {
    tfb200::set_last_error("tfb200_opt: output buffer needs " + std::to_string(r.output.size() + 1) + " bytes");
    return TFB200_ENOSPC;
  }
  std::memcpy(out, r.output.c_str(), r.output.size() + 1);
  return TFB200_OK;
}

extern "C" int tfb200_plan(const char* plan_json_in, char* out, size_t cap, size_t* needed) {
  if (!plan_json_in) {
    tfb200::set_last_error("tfb200_plan: null plan JSON");
    return TFB200_EINVAL;
  }
  tfb200::front::PlanRequest req;
  std::string err;
  if (!tfb200::front::request_from_plan_json(plan_json_in, &req, &err)) {
    tfb200::set_last_error("tfb200_plan: " + err);
    return TFB200_EINVAL;
  }
  const std::string json = tfb200::front::plan_json(tfb200::front::plan_b200(req));
  if (needed) *needed = json.size() + 1;
  if (!out || cap < json.size() + 1) {
    tfb200::set_last_error("tfb200_plan: output buffer needs " + std::to_string(json.size() + 1) + " bytes");
    return TFB200_ENOSPC;
  }
  std::memcpy(out, json.c_str(), json.size() + 1);
  return TFB200_OK;
}
