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

enum cudaLaunchAttributeID { cudaLaunchAttributeClusterDimension = 4,
                             cudaLaunchAttributeProgrammaticStreamSerialization = 5 };
struct cudaLaunchAttributeValue {
  int programmaticStreamSerializationAllowed;
  struct {
    unsigned x, y, z;
  } clusterDim;
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
// A cluster dimension attribute runs the CTAs of each cluster at the same
// time (clusters along x only, as the library launches them); programmatic
// stream serialization changes nothing here (launches run to completion).
inline unsigned launch_cluster_x(const cudaLaunchConfig_t* c) {
  for (unsigned i = 0; i < c->numAttrs; ++i)
    if (c->attrs[i].id == cudaLaunchAttributeClusterDimension) {
      const auto& d = c->attrs[i].val.clusterDim;
      return d.y == 1 && d.z == 1 ? d.x : 0;
    }
  return 1;
}
template <class... KArgs, class... Args>
inline cudaError_t cudaLaunchKernelEx(const cudaLaunchConfig_t* c, void (*kernel)(KArgs...), Args&&... args) {
  const unsigned cx = launch_cluster_x(c);
  if (cx == 0 || cx > 16 || c->gridDim.x % cx) return cudaErrorInvalidValue;
  return simt::launch_cluster(kernel, c->gridDim, c->blockDim, c->dynamicSmemBytes, cx, static_cast<KArgs>(args)...)
             ? cudaSuccess
             : cudaErrorLaunchFailure;
}

// The device the emulation stands for: a B200's 148 SMs, one CTA of the
// tensor-core kernels (about 200 KB of shared memory) per SM.
enum cudaDeviceAttr { cudaDevAttrMultiProcessorCount = 16 };
inline cudaError_t cudaDeviceGetAttribute(int* v, cudaDeviceAttr a, int) {
  if (a != cudaDevAttrMultiProcessorCount) return cudaErrorInvalidValue;
  *v = 148;
  return cudaSuccess;
}
template <class F>
inline cudaError_t cudaOccupancyMaxActiveClusters(int* n, F, const cudaLaunchConfig_t* c) {
  const unsigned cx = launch_cluster_x(c);
  if (cx == 0) return cudaErrorInvalidValue;
  *n = 148 / (int)cx;
  return cudaSuccess;
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
