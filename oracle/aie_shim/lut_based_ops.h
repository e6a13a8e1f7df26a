// CPU restatement of MLIR-AIE's getExpBf16 (aie_runtime_lib/AIE2/lut_based_ops,
// v1.3.4, not present here): the exact exponential of each bf16 lane, rounded
// to fp32 in the accumulator. The real function reads two lookup tables; its
// tables are not published in the reference, so this is the ideal it
// approximates. TEST INFRASTRUCTURE ONLY.
#pragma once
#include <cmath>
#include "aie_api/aie.hpp"

inline aie::accum<accfloat, 16> getExpBf16(const aie::vector<bfloat16, 16> &x) {
  aie::accum<accfloat, 16> r;
  for (int i = 0; i < 16; i++) r.v[i] = (float)std::exp((double)(float)x.v[i]);
  return r;
}
