// Companion of ref_sm_shim.h (TEST INFRASTRUCTURE ONLY).
#include <cstdlib>
#include <cuda_runtime.h>

cudaError_t ps_ref_get_device_properties(cudaDeviceProp* prop, int device) {
  const cudaError_t status = cudaGetDeviceProperties(prop, device);
  const char* forced = std::getenv("PS_REF_SM_COUNT");
  if (status == cudaSuccess && forced && *forced) prop->multiProcessorCount = std::atoi(forced);
  return status;
}
