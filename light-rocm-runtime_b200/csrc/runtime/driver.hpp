// Lazily loaded CUDA driver API table.
//
// liblrrt.so does not link libcuda: it dlopen()s libcuda.so.1 inside lr_init()
// so the library (and every lr_* symbol) loads on machines without an NVIDIA
// driver, where lr_init() then succeeds with zero devices.
#ifndef LRRT_B200_DRIVER_HPP_
#define LRRT_B200_DRIVER_HPP_

#include <cuda.h>

namespace lrrt_b200 {

// X(name): `name` is the cuda.h spelling; the macro expansion of the header
// (e.g. cuMemAlloc -> cuMemAlloc_v2) selects the exported driver symbol.
#define LRRT_DRIVER_FUNCTIONS(X)                                               \
  X(cuInit)                                                                    \
  X(cuGetErrorName)                                                            \
  X(cuGetErrorString)                                                          \
  X(cuDeviceGetCount)                                                          \
  X(cuDeviceGet)                                                               \
  X(cuDeviceGetName)                                                           \
  X(cuDeviceGetAttribute)                                                      \
  X(cuDevicePrimaryCtxRetain)                                                  \
  X(cuDevicePrimaryCtxRelease)                                                 \
  X(cuCtxSetCurrent)                                                           \
  X(cuCtxSynchronize)                                                          \
  X(cuStreamCreate)                                                            \
  X(cuStreamDestroy)                                                           \
  X(cuStreamSynchronize)                                                       \
  X(cuStreamWaitEvent)                                                         \
  X(cuEventCreate)                                                             \
  X(cuEventDestroy)                                                            \
  X(cuEventRecord)                                                             \
  X(cuEventSynchronize)                                                        \
  X(cuEventElapsedTime)                                                        \
  X(cuMemAlloc)                                                                \
  X(cuMemFree)                                                                 \
  X(cuMemHostAlloc)                                                            \
  X(cuMemFreeHost)                                                             \
  X(cuMemcpy)                                                                  \
  X(cuMemcpyAsync)                                                             \
  X(cuMemsetD8Async)                                                           \
  X(cuModuleLoadData)                                                          \
  X(cuModuleUnload)                                                            \
  X(cuModuleGetFunction)                                                       \
  X(cuFuncGetAttribute)                                                        \
  X(cuFuncSetAttribute)                                                        \
  X(cuFuncGetParamInfo)                                                        \
  X(cuLaunchKernelEx)                                                          \
  X(cuOccupancyMaxActiveBlocksPerMultiprocessor)

struct Driver {
#define LRRT_DECLARE_DRIVER_FUNCTION(fn) decltype(&fn) fn##_ = nullptr;
  LRRT_DRIVER_FUNCTIONS(LRRT_DECLARE_DRIVER_FUNCTION)
#undef LRRT_DECLARE_DRIVER_FUNCTION
  void *library = nullptr;
  bool loaded = false;
};

// Loads libcuda.so.1 once; returns false (and leaves the table empty) when the
// library or any symbol is missing.
bool load_driver(Driver &driver);

} // namespace lrrt_b200

#endif // LRRT_B200_DRIVER_HPP_
