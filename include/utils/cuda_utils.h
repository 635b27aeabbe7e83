// Error convention of the PowerSparse C++ API: CUDA failures become
// std::runtime_error("file:line: expr: message").  Same macro and behaviour as
// utils/cuda_utils.h:7-14 of ParCIS/PowerSparse.
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

inline void CheckCuda(cudaError_t status, const char* expression, const char* file, int line) {
  if (status != cudaSuccess)
    throw std::runtime_error(std::string(file) + ":" + std::to_string(line) + ": " + expression + ": " +
                             cudaGetErrorString(status));
}

#define CUDA_CALL(call) CheckCuda((call), #call, __FILE__, __LINE__)
