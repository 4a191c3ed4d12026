// Internal hooks between the host runtime (runtime.cpp) and other translation units of the library.
#pragma once
#include <cuda_runtime.h>
#include <string>
#include "kernels.cuh"

struct gem_model;

namespace gem {

// What a kernel-level entry point needs to run the full head of a model.
struct ModelHeadView {
  MatView w;          // output matrix
  const uint32_t* row_of = nullptr;   // token -> row when the rows are in class order (null: token order)
  const uint32_t* row_tok = nullptr;  // row -> token, likewise
  bool exact = true;  // numerics mode
  cudaStream_t st = nullptr;
  int sms = 0, device = 0, d = 0;
  int* err = nullptr;  // device error word
};
bool model_head_view(const gem_model* m, ModelHeadView* out);
void set_last_error(const std::string& msg);

}  // namespace gem
