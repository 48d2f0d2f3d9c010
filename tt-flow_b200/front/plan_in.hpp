// Plan JSON in (schema/plan.schema.json): the graph a plan document describes,
// as a PlanRequest for the B200 planner. Used by tfb200_plan.
#pragma once

#include <string>
#include <utility>
#include <vector>

#include "plan.hpp"

namespace tfb200::front {

struct JVal {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  std::string text;  // string contents, or a number's literal text
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
  const JVal* get(const std::string& key) const;
};

bool parse_json(const std::string& text, JVal* out, std::string* err);
bool request_from_plan_json(const std::string& text, PlanRequest* r, std::string* err);

}  // namespace tfb200::front
