// Test infrastructure: the part of the CUDA runtime API the library's fp32
// launchers use, for building them for the host on the SIMT emulation
// (tests/simt_host.h). Streams are opaque handles; launches run to completion
// when they are made; a launch whose threads waited on barriers that could not
// complete is reported by cudaGetLastError as a launch failure.
#pragma once

#include <chrono>

#include "cuda.h"
#include "simt_host.h"

typedef void* cudaStream_t;
enum cudaError_t { cudaSuccess = 0, cudaErrorInvalidValue = 1, cudaErrorLaunchFailure = 719 };

inline cudaError_t cudaGetLastError() {
  const bool f = simt::launch_failed();
  simt::launch_failed() = false;
  return f ? cudaErrorLaunchFailure : cudaSuccess;
}
inline cudaError_t cudaPeekAtLastError() { return simt::launch_failed() ? cudaErrorLaunchFailure : cudaSuccess; }
inline const char* cudaGetErrorString(cudaError_t e) {
  return e == cudaSuccess ? "no error" : "host emulation: threads waited on barriers that could not complete";
}
inline cudaError_t cudaGetDevice(int* d) {
  *d = 0;
  return cudaSuccess;
}

enum cudaMemcpyKind { cudaMemcpyHostToHost = 0, cudaMemcpyHostToDevice = 1, cudaMemcpyDeviceToHost = 2,
                      cudaMemcpyDeviceToDevice = 3, cudaMemcpyDefault = 4 };
inline cudaError_t cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t = nullptr) {
  std::memset(p, v, n);
  return cudaSuccess;
}
inline cudaError_t cudaMemcpyAsync(void* d, const void* s, size_t n, cudaMemcpyKind, cudaStream_t = nullptr) {
  std::memmove(d, s, n);
  return cudaSuccess;
}
// A __device__ variable is a host global here: its address is the host address.
template <class T>
inline cudaError_t cudaGetSymbolAddress(void** p, T& symbol) {
  *p = (void*)&symbol;
  return cudaSuccess;
}

enum cudaFuncAttribute { cudaFuncAttributeMaxDynamicSharedMemorySize = 8 };
template <class F>
inline cudaError_t cudaFuncSetAttribute(F, cudaFuncAttribute, int) {
  return cudaSuccess;
}

enum cudaLaunchAttributeID { cudaLaunchAttributeProgrammaticStreamSerialization = 1 };
struct cudaLaunchAttributeValue {
  int programmaticStreamSerializationAllowed;
};
struct cudaLaunchAttribute {
  cudaLaunchAttributeID id;
  cudaLaunchAttributeValue val;
};
struct cudaLaunchConfig_t {
  dim3 gridDim, blockDim;
  size_t dynamicSmemBytes;
  cudaStream_t stream;
  cudaLaunchAttribute* attrs;
  unsigned numAttrs;
};
template <class... KArgs, class... Args>
inline cudaError_t cudaLaunchKernelEx(const cudaLaunchConfig_t* c, void (*kernel)(KArgs...), Args&&... args) {
  return simt::launch(kernel, c->gridDim, c->blockDim, c->dynamicSmemBytes, static_cast<KArgs>(args)...)
             ? cudaSuccess
             : cudaErrorLaunchFailure;
}

enum cudaStreamCaptureStatus { cudaStreamCaptureStatusNone = 0, cudaStreamCaptureStatusActive = 1 };
inline cudaError_t cudaStreamIsCapturing(cudaStream_t, cudaStreamCaptureStatus* s) {
  *s = cudaStreamCaptureStatusNone;
  return cudaSuccess;
}
enum cudaDriverEntryPointQueryResult { cudaDriverEntryPointSuccess = 0, cudaDriverEntryPointSymbolNotFound = 1 };
enum { cudaEnableDefault = 0 };
// The driver entry points the library looks up: cuTensorMapEncodeTiled only.
inline cudaError_t cudaGetDriverEntryPoint(const char* name, void** fn, unsigned long long,
                                           cudaDriverEntryPointQueryResult* q) {
  if (strcmp(name, "cuTensorMapEncodeTiled") != 0) {
    *q = cudaDriverEntryPointSymbolNotFound;
    return cudaErrorInvalidValue;
  }
  *fn = reinterpret_cast<void*>(&simt::encode_tiled);
  *q = cudaDriverEntryPointSuccess;
  return cudaSuccess;
}
