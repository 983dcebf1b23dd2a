// Host-side CUDA error checking shared by the kernel launchers and the bindings.
#pragma once
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#define GB_CUDA_CHECK(expr)                                                                  \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                  \
  } while (0)

#define GB_LAUNCH_CHECK() GB_CUDA_CHECK(cudaGetLastError())
