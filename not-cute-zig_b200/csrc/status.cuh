// status.cuh -- the mapping of CUDA runtime errors onto the library's status
// codes (reference CudaError set, src/cuda.zig:134-151), shared by the
// flash-attention and GEMM entry points.
#pragma once
#include <cuda_runtime.h>

#include "ncz_flash.h"

namespace ncz {

inline int map_cuda_error(cudaError_t e) {
    switch (e) {
        case cudaSuccess: return NCZ_SUCCESS;
        case cudaErrorMemoryAllocation: return NCZ_ERROR_OUT_OF_MEMORY;
        case cudaErrorSharedObjectInitFailed: return NCZ_ERROR_SHARED_OBJECT_INIT_FAILED;
        case cudaErrorSymbolNotFound: return NCZ_ERROR_NOT_FOUND;
        case cudaErrorInvalidValue: return NCZ_ERROR_INVALID_VALUE;
        case cudaErrorDeviceUninitialized: return NCZ_ERROR_INVALID_CONTEXT;
        case cudaErrorInvalidDevice: return NCZ_ERROR_INVALID_DEVICE;
        case cudaErrorInvalidKernelImage:
        case cudaErrorNoKernelImageForDevice: return NCZ_ERROR_INVALID_IMAGE;
        case cudaErrorContextIsDestroyed: return NCZ_ERROR_CONTEXT_IS_DESTROYED;
        case cudaErrorLaunchFailure: return NCZ_ERROR_LAUNCH_FAILED;
        case cudaErrorLaunchOutOfResources: return NCZ_ERROR_LAUNCH_OUT_OF_RESOURCES;
        case cudaErrorLaunchTimeout: return NCZ_ERROR_LAUNCH_TIMEOUT;
        case cudaErrorIllegalAddress: return NCZ_ERROR_ILLEGAL_ADDRESS;
        case cudaErrorNoDevice: return NCZ_ERROR_NO_DEVICE;
        case cudaErrorInitializationError:
        case cudaErrorInsufficientDriver: return NCZ_ERROR_NOT_INITIALIZED;
        default: return NCZ_ERROR_UNKNOWN;
    }
}

// Driver-call table entries return the runtime's error numbers as int.
inline int map_cuda_error(int e) { return map_cuda_error(static_cast<cudaError_t>(e)); }

}  // namespace ncz
