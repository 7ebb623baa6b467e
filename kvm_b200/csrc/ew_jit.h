// Fused elementwise code generation (NVRTC, sm_100a): the kernel behind
// kvm_sm100_elementwise unless KVM_SM100_EW_JIT=0 selects the interpreter.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/kvm_sm100.h"

namespace kvm {

bool ew_jit_enabled();
// Generate and compile the kernel for these arguments (no GPU needed).
int ew_jit_prepare(const kvm_ew_program& p, const kvm_ew_inputs& in, const void* out,
                   int64_t n);
// Compile if needed, load on the current device if needed, launch.
int ew_jit_launch(const kvm_ew_program& p, const kvm_ew_inputs& in, void* out, int64_t n,
                  cudaStream_t stream);

}  // namespace kvm
