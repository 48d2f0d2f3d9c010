// C ABI of the front end (declared in include/tfb200.h): tfb200_opt.
#include <cstring>
#include <string>

#include "../../include/tfb200.h"
#include "passes.hpp"

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
