#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace ftb {

class CudaError : public std::runtime_error {
 public:
  explicit CudaError(const std::string &m) : std::runtime_error(m) {}
};

[[noreturn]] inline void throw_cuda(cudaError_t e, const char *what, const char *file, int line) {
  throw CudaError(std::string("CUDA error: ") + cudaGetErrorString(e) + " (" + what + " at " + file + ":" +
                  std::to_string(line) + ")");
}

}  // namespace ftb

#define CUDA_TRY(expr)                                                   \
  do {                                                                   \
    cudaError_t ft_e_ = (expr);                                          \
    if (ft_e_ != cudaSuccess) ::ftb::throw_cuda(ft_e_, #expr, __FILE__, __LINE__); \
  } while (0)
