// Host-side runtime shared by every translation unit of libkvm_sm100:
// per-device facts (SM count, the device status word), the thread-local error
// message behind kvm_sm100_last_error(), and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/kvm_sm100.h"

namespace kvm {

// Device-side status bits, OR-ed into the per-device status word by kernels.
enum DeviceStatusBits : int {
  kDevWaitTimeout = 1,   // a bounded mbarrier wait expired
  kDevBadInput = 2,      // a kernel saw an index or count outside its range
};

struct DeviceInfo {
  int sm_count = 0;
  int* status = nullptr;  // one int in device memory, zero-initialised
};

// Lazily initialised per-device info for the current device; nullptr (and the
// last error set) if the device cannot be queried.
const DeviceInfo* device_info();

// Launch `kern` on `st`; with `pdl`, programmatic dependent launch is
// allowed: the kernel may start (and run its prologue) while the previous
// kernel of the stream is finishing. Every kernel launched that way calls
// pdl_wait() (below) before it touches global memory that an earlier kernel
// of the stream writes or reads.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// Device side of programmatic dependent launch. pdl_wait(): block until the
// kernels this one may overlap have completed and their memory is visible.
// pdl_trigger(): let the next kernel of the stream start launching. Both do
// nothing in a kernel launched without the attribute.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

// Record `msg` as this thread's last error and return `code`.
int fail(int code, const std::string& msg);
int fail_cuda(cudaError_t e, const char* what);

// Encode a 2-D tiled tensor map over a row-major matrix.
//   base:   global address (16-byte aligned)
//   inner:  elements per row that exist (innermost extent)
//   outer:  rows
//   row_bytes: byte stride between rows (multiple of 16)
//   box_inner x box_outer: the tile one TMA load copies
//   elem:   CU_TENSOR_MAP_DATA_TYPE_*
// 128-byte swizzle; out-of-range elements read as zero.
int encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapDataType elem,
                   CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace kvm

#define KVM_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t kvm_e_ = (expr);                            \
    if (kvm_e_ != cudaSuccess) return ::kvm::fail_cuda(kvm_e_, #expr); \
  } while (0)
