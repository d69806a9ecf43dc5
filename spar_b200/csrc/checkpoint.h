// SPARCKPT v1 checkpoint format shared by checkpoint.cpp (the format, host arrays) and trainer.cu
// (the named tensors of a config, device staging).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "spar_b200.h"

namespace spar_b200 {

struct CkptTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint64_t numel() const {
    uint64_t n = 1;
    for (uint64_t d : shape) n *= d;
    return n;
  }
};

// Named tensors (name, shape) of a Spar-family config in named-parameter order (trainer.cu).
bool checkpoint_tensors(const SparB200LMConfig& c, std::vector<CkptTensor>& out);

// One contiguous row-major host array per named tensor; m / v may be null when
// meta.adam_step == 0 (write).
SparCudaStatus checkpoint_write(const char* path, const SparB200LMConfig& c,
                                const SparB200Checkpoint& meta, const float* const* values,
                                const float* const* m, const float* const* v);
SparCudaStatus checkpoint_read(const char* path, const SparB200LMConfig& c,
                               SparB200Checkpoint& meta, float* const* values, float* const* m,
                               float* const* v);

}  // namespace spar_b200
