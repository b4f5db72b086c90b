/*
 * Minimal stand-in for <hip/hip_runtime.h>, used only so that the reference's
 * host-only header asm_f4gemm/f4gemm.hpp compiles with g++ into oracle/_ref.
 * TEST INFRASTRUCTURE ONLY.  The shim never calls the module-loading or launch
 * functions below; they exist to satisfy declarations and always fail.
 */
#pragma once
#include <cstddef>
typedef int hipError_t;
static const hipError_t hipSuccess = 0;
typedef struct ihipModule_t* hipModule_t;
typedef struct ihipModuleSymbol_t* hipFunction_t;
typedef struct ihipStream_t* hipStream_t;
#define HIP_LAUNCH_PARAM_BUFFER_POINTER ((void*)0x01)
#define HIP_LAUNCH_PARAM_BUFFER_SIZE ((void*)0x02)
#define HIP_LAUNCH_PARAM_END ((void*)0x03)
static inline const char* hipGetErrorString(hipError_t) { return "hip stub: not available"; }
static inline hipError_t hipModuleLoad(hipModule_t*, const char*) { return 1; }
static inline hipError_t hipModuleGetFunction(hipFunction_t*, hipModule_t, const char*) { return 1; }
static inline hipError_t hipModuleLaunchKernel(hipFunction_t, unsigned, unsigned, unsigned, unsigned, unsigned,
                                               unsigned, unsigned, hipStream_t, void**, void**) { return 1; }
