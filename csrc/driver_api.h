// CUDA driver-API entry points used by the extensions (tensor-map encoding,
// allocation ranges), resolved at run time through the runtime's
// cudaGetDriverEntryPoint: the libraries then do not link libcuda, so they
// import on machines without a GPU driver (builds, CPU tests) and fail with a
// clear error only when a driver call is actually made.
#pragma once

#include <cstdio>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace pd {

template <typename Fn>
inline Fn driver_entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  const cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (!(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr)) {
    char msg[256];   // one C string: see PD_CHECK in common.cuh
    snprintf(msg, sizeof(msg), "CUDA driver entry point %s is unavailable (%d, %d)", name, int(e), int(q));
    TORCH_CHECK(false, static_cast<const char*>(msg));
  }
  return reinterpret_cast<Fn>(p);
}

inline CUresult tensor_map_encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank, void* base,
                                        const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                                        const cuuint32_t* estrides, CUtensorMapInterleave interleave,
                                        CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2,
                                        CUtensorMapFloatOOBfill oob) {
  using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                          const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                          CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Fn fn = driver_entry<Fn>("cuTensorMapEncodeTiled");
  return fn(map, dtype, rank, base, dims, strides, box, estrides, interleave, swizzle, l2, oob);
}

inline CUresult mem_get_address_range(CUdeviceptr* base, size_t* size, CUdeviceptr ptr) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = driver_entry<Fn>("cuMemGetAddressRange");
  return fn(base, size, ptr);
}

}  // namespace pd
