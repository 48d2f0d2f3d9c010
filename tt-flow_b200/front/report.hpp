// Plan report for the B200 (replaces tensixflow tools/tensixflow-report for
// plans of this backend). Like the reference's report, it is the validator of a
// plan document: it re-derives the emission block from the plan's own tensors
// and fusion with the B200 planner, refuses a plan whose emission numbers or
// mapping disagree (naming the field) or that has no emission block, and only
// then renders a self-contained offline HTML page. Nothing is written for a
// plan it refuses.
#pragma once

#include <string>

namespace tfb200::front {

struct ReportResult {
  bool ok = false;
  std::string diag;  // why the plan was refused
  std::string html;  // the rendered page (ok only)
};

ReportResult report_plan(const std::string& plan_json_text);

}  // namespace tfb200::front
