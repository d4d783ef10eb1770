// bind_util.h - helpers of the Python bindings.
#pragma once

#include <torch/extension.h>

#include "strfmt.h"

namespace rab {

// float32 data pointer of `t`, refused with a RuntimeError (RAB_CHECK) for any
// other dtype; used instead of data_ptr<float>() so a wrong dtype raises
// through the same path as every other argument check.
inline float* f32_ptr(const torch::Tensor& t, const char* name) {
  RAB_CHECK(t.scalar_type() == torch::kFloat32, "%s must be float32", name);
  return static_cast<float*>(t.data_ptr());
}

}  // namespace rab
