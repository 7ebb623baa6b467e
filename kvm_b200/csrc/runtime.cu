// Per-device state, error reporting and tensor-map encoding for the C ABI.
#include "runtime.h"

#include <cudaTypedefs.h>

#include <mutex>
#include <string>

namespace kvm {
namespace {

constexpr int kMaxDevices = 64;

thread_local std::string t_last_error;
std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_ready[kMaxDevices] = {};

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int fail_cuda(cudaError_t e, const char* what) {
  return fail(KVM_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    fail(KVM_ERR_CUDA, "cudaGetDevice failed");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dev_ready[dev]) {
    DeviceInfo info;
    cudaError_t e =
        cudaDeviceGetAttribute(&info.sm_count, cudaDevAttrMultiProcessorCount,
                               dev);
    if (e != cudaSuccess) {
      fail_cuda(e, "cudaDeviceGetAttribute(SM count)");
      return nullptr;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
      fail(KVM_ERR_UNSUPPORTED,
           "libkvm_sm100 is built for sm_100a only (device is sm_" +
               std::to_string(major) + std::to_string(minor) + ")");
      return nullptr;
    }
    e = cudaMalloc(&info.status, sizeof(int));
    if (e != cudaSuccess) {
      fail_cuda(e, "cudaMalloc(status word)");
      return nullptr;
    }
    e = cudaMemset(info.status, 0, sizeof(int));
    if (e != cudaSuccess) {
      fail_cuda(e, "cudaMemset(status word)");
      return nullptr;
    }
    g_dev[dev] = info;
    g_dev_ready[dev] = true;
  }
  return &g_dev[dev];
}

int encode_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapDataType elem,
                   CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(KVM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (!aligned16(base) || (row_bytes & 15u) != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "TMA operand must be 16-byte aligned with a row stride that "
                "is a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, elem, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(KVM_ERR_CUDA,
                "cuTensorMapEncodeTiled failed with CUresult " +
                    std::to_string(static_cast<int>(r)));
  return KVM_OK;
}

}  // namespace kvm

namespace kvm {
namespace {
// An empty kernel whose attributes stand for every kernel of this library
// (all translation units are compiled with the same -gencode).
__global__ void binary_version_probe_kernel() {}
}  // namespace
}  // namespace kvm

extern "C" {

const char* kvm_sm100_last_error(void) { return kvm::t_last_error.c_str(); }

int kvm_sm100_kernel_binary_version(int* version) {
  if (!version) return kvm::fail(KVM_ERR_INVALID_ARG, "kernel_binary_version: NULL");
  cudaFuncAttributes a;
  KVM_CUDA_TRY(cudaFuncGetAttributes(&a, kvm::binary_version_probe_kernel));
  *version = a.binaryVersion;
  return KVM_OK;
}

int kvm_sm100_version(void) { return KVM_SM100_ABI_VERSION; }

int kvm_sm100_device_status(int* status_out, int clear) {
  const kvm::DeviceInfo* d = kvm::device_info();
  if (!d) return KVM_ERR_CUDA;
  int v = 0;
  KVM_CUDA_TRY(cudaDeviceSynchronize());
  KVM_CUDA_TRY(cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) KVM_CUDA_TRY(cudaMemset(d->status, 0, sizeof(int)));
  if (status_out) *status_out = v;
  if (v & kvm::kDevWaitTimeout)
    return kvm::fail(KVM_ERR_TIMEOUT, "a device-side bounded wait expired");
  if (v & kvm::kDevBadInput)
    return kvm::fail(KVM_ERR_INVALID_ARG,
                     "a kernel saw an index or count outside its range");
  return KVM_OK;
}

}  // extern "C"
