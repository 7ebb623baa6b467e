// Executor: runs a KVM kernel-dialect graph on one B200 through the sm_100a
// C ABI (include/kvm_sm100.h).
//
//   kernel graph --TransformKernelToTask (the reference's pass, using the
//   sm_100a Device target)--> task graph --Prepare--> launch plan --Run-->
//
// Prepare walks the task graph once. Each task value is a global buffer, a
// view of one (task.tma.gmem_to_smem / task.lsu.gmem_to_reg), a pending
// tensor-core product (task.tc.mma / task.tc.mma_acc) or a pending ALU/SFU
// expression; stores (task.lsu.reg_to_gmem) and collectives turn them into
// launches: a tcgen05 GEMM (grouped by expert after a moe_dispatch), the
// elementwise interpreter, the MoE routing / dispatch / combine kernels. Every
// device buffer is allocated in Prepare; Run only launches (no allocation,
// no host synchronisation), so a Run can be timed or repeated.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "attr.h"
#include "dialect/dtype.h"
#include "graph.h"

namespace kvm::sm100 {

struct Buffer {
  void* ptr = nullptr;
  std::vector<int64_t> shape;
  ir::dialect::Dtype dtype = ir::dialect::Dtype::kF32;
  int64_t numel() const;
  int64_t bytes() const;
};

int64_t DtypeBytes(ir::dialect::Dtype d);

class Executor {
 public:
  // `kernel` and `attrs` come from serial::Parse; the executor lowers the
  // graph itself (TransformKernelToTask) and keeps the task graph.
  Executor(const ir::Graph& kernel, const ir::AttrMap& attrs);
  ~Executor();
  Executor(const Executor&) = delete;
  Executor& operator=(const Executor&) = delete;

  // Block arguments, in order, with their shapes and dtypes.
  const std::vector<Buffer>& inputs() const { return inputs_; }
  const std::vector<std::string>& input_names() const { return input_names_; }

  // Allocate buffers and build the launch plan. Inputs are allocated here and
  // may be filled (FillInput / CopyInput) before or after Prepare.
  void Prepare();
  void CopyInput(int index, const void* host, int64_t bytes);
  void FillInputNormal(int index, uint64_t seed, float mean, float std);
  void FillInputConst(int index, float value);

  // Launch the plan on `stream` (asynchronous). Returns a kvm_status. The
  // first Run also re-lays out per-expert weights once ([E, K, N] ->
  // [E, N, K]), so those inputs must be filled before it.
  int Run(cudaStream_t stream);

  const std::vector<Buffer>& outputs() const { return outputs_; }
  const ir::Graph& task_graph() const { return task_; }
  int launches_per_run() const { return static_cast<int>(steps_.size()); }
  const std::vector<std::string>& step_names() const { return step_names_; }

 private:
  struct Slot;
  struct Routing;
  Slot& slot(const ir::ValueNode* v);
  Buffer& Materialize(const ir::ValueNode* v);
  const Buffer& GlobalOf(const ir::ValueNode* v);
  void PlanStore(const ir::ValueNode* src, const ir::ValueNode* dst);
  void PlanGemm(const ir::ValueNode* mma, const Buffer& out);
  void PlanExpr(const ir::ValueNode* expr, const Buffer& out);
  void PlanComm(const ir::OpNode* op);
  void* Alloc(int64_t bytes);
  const ir::OpNode* KernelCommOp(const std::string& name, int nth) const;

  const ir::Graph& kernel_;
  const ir::AttrMap& attrs_;
  ir::Graph task_;
  std::vector<Buffer> inputs_;
  std::vector<std::string> input_names_;
  std::vector<Buffer> outputs_;
  std::unordered_map<const ir::ValueNode*, std::unique_ptr<Slot>> slots_;
  std::vector<std::unique_ptr<Routing>> routings_;
  std::vector<void*> allocations_;
  std::unordered_map<const void*, Routing*> routing_of_;  // logits buffer -> routing
  std::vector<std::function<int(cudaStream_t)>> once_steps_;  // weight re-layouts
  std::vector<std::function<int(cudaStream_t)>> steps_;
  std::vector<std::string> step_names_;
  bool prepared_ = false;
  bool once_done_ = false;
};

}  // namespace kvm::sm100
