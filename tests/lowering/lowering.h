// lowering.h -- compiling and calling the reference's C, and the restated
// unit tests (TEST INFRASTRUCTURE).
#pragma once
#include <functional>
#include <string>
#include <vector>

namespace kir {

// Compiles `code` (the C the renderer emitted for function `name`) with gcc
// (-O2 -ffp-contract=off, so no product is fused into an FMA, as the
// one-operation-per-statement C the reference's clang build compiles) and
// calls it; args[s] points at the buffer of parameter slot s, or at the
// value of a scalar parameter.  Programs are cached by source text.
void run_c(const std::string &code, const std::string &name, const std::vector<void *> &args);

struct Case {
  std::string name;
  std::function<void()> fn;
};
std::vector<Case> structure_cases();

}  // namespace kir
