// Force-included into the reference's utils/matrix_utils.cu by oracle/Makefile
// (TEST INFRASTRUCTURE ONLY).  The reference picks its number of worksets from the
// device's SM count (utils/matrix_utils.cu:37-42).  Routing that one query through
// ps_ref_get_device_properties lets golden layouts exercise the multi-workset path
// on small matrices: PS_REF_SM_COUNT, when set, replaces multiProcessorCount.
#pragma once
#include <cuda_runtime.h>
#ifdef cudaGetDeviceProperties
#undef cudaGetDeviceProperties
#endif
cudaError_t ps_ref_get_device_properties(cudaDeviceProp* prop, int device);
#define cudaGetDeviceProperties ps_ref_get_device_properties
