// Executor: runs a KVM kernel-dialect graph on one B200 through the sm_100a
// C ABI (include/kvm_sm100.h).
//
//   kernel graph --TransformKernelToTask (the reference's pass, using the
//   sm_100a Device target)--> task graph --Prepare--> launch plan --Run-->
//
// Prepare walks the task graph in three passes:
//   analysis  each task value is a global buffer, a view of one
//             (task.tma.gmem_to_smem / task.lsu.gmem_to_reg), a pending
//             tensor-core product (task.tc.mma / task.tc.mma_acc) or a pending
//             ALU/SFU expression; uses of every global are counted;
//   fusion    single-use elementwise results are inlined into their consumer
//             (rounded to their declared dtype, so the graph's arithmetic is
//             kept); the SiLU-gate composite over two GEMMs that share A
//             becomes one gate/up GEMM with the activation in its epilogue;
//             the RMSNorm composite becomes the RMSNorm kernel; a router GEMM
//             that only feeds moe_dispatch / moe_combine becomes the fused
//             router + top-k kernel;
//   planning  stores and collectives, in program order, become launches.
// Every device buffer is allocated in Prepare; Run only launches (no
// allocation, no host synchronisation), so a Run can be timed or repeated.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "attr.h"
#include "kvm_sm100.h"
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

  // Multi-process runs: the world communicator (kvm_sm100_comm_init) of this
  // process's rank; the collectives of the graph run over it (and over
  // communicators split from it for rank subsets). Set before Prepare.
  void SetComm(kvm_comm* world);

  // Analysis and fusion only (no GPU needed); Prepare runs it first.
  void Plan();
  // Allocate buffers and build the launch plan. Inputs are allocated here and
  // may be filled (FillInput / CopyInput) after Prepare.
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
  // Fusions applied by Prepare, one line each (for reports and tests).
  const std::vector<std::string>& fusions() const { return fusions_; }

 private:
  struct Slot;
  struct Routing;
  struct SNode;
  struct SiluMatch;
  struct RmsMatch;
  Slot& slot(const ir::ValueNode* v);
  Buffer& Materialize(const ir::ValueNode* v);
  const Buffer& GlobalOf(const ir::ValueNode* v);
  const ir::ValueNode* BaseGlobal(const ir::ValueNode* v);
  void Analyze();
  void Fuse();
  SNode Resolve(const ir::ValueNode* v);
  bool MatchSilu(const ir::ValueNode* dst, SiluMatch* m);
  bool MatchRms(const ir::ValueNode* dst, RmsMatch* m);
  bool InputFill(const ir::ValueNode* v, double* value) const;
  void PlanStore(const ir::ValueNode* src, const ir::ValueNode* dst);
  void PlanGemm(const ir::ValueNode* mma, const Buffer& out);
  void PlanExpr(const ir::ValueNode* expr, const Buffer& out);
  void PlanComm(const ir::OpNode* op);
  void PlanExpertDispatch(const ir::OpNode* op, const std::vector<int>& ranks);
  Routing* PlanRoute(const ir::OpNode* op, const ir::OpNode* kop, const Buffer& x,
                     const Buffer& g);
  void PlanSilu(const ir::ValueNode* dst);
  void PlanRms(const ir::ValueNode* dst);
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
  // analysis / fusion state
  std::vector<const ir::OpNode*> actions_;  // stores and collectives, in order
  std::unordered_map<const ir::ValueNode*, const ir::ValueNode*> producer_;  // global <- stored value
  std::unordered_map<const ir::ValueNode*, int> uses_;        // global -> reads
  std::unordered_map<const ir::ValueNode*, std::vector<const ir::OpNode*>> consumers_;
  std::unordered_map<const ir::OpNode*, Routing*> routing_by_op_;
  std::unordered_map<const ir::ValueNode*, bool> inlined_;    // folded into a consumer
  std::unordered_map<const ir::ValueNode*, bool> elided_;     // produced inside a fusion
  std::unordered_map<const ir::ValueNode*, std::unique_ptr<SiluMatch>> silu_;
  std::unordered_map<const ir::ValueNode*, std::unique_ptr<RmsMatch>> rms_;
  std::unordered_map<const ir::ValueNode*, std::pair<const ir::ValueNode*, const ir::ValueNode*>>
      router_;  // logits global -> (x, router weight [H, E]) of its fused GEMM
  std::vector<std::string> fusions_;
  std::vector<std::function<int(cudaStream_t)>> once_steps_;  // weight re-layouts
  std::vector<std::function<int(cudaStream_t)>> steps_;
  kvm_comm* world_ = nullptr;
  int rank_ = 0, nranks_ = 1;
  std::map<std::vector<int>, kvm_comm*> subcomms_;  // rank set -> communicator
  kvm_comm* CommFor(const std::vector<int>& ranks, int* my_index);
  std::vector<std::string> step_names_;
  bool analyzed_ = false;
  bool prepared_ = false;
  bool once_done_ = false;
};

}  // namespace kvm::sm100
