// The sm_100a target of kvm::device::Device (declared in the reference's
// src/device/device.h:35-62): the per-kernel-op lowering hook that
// TransformKernelToTask (src/transform/kernel_to_task/kernel_to_task.cpp:47,83)
// calls for every kernel op. It replaces the reference's src/device/device.cpp
// at link time and keeps its contract:
//
//   * kernel.gemm and the collectives lower exactly as the reference lowers
//     them (device.cpp:85-121): the same task ops, operands, locations and
//     lineage names (base = operand names joined by '_' + '_' + op name with
//     '.' -> '_' + '_' + suffix), so the reference's own decomp tests hold;
//   * ops the reference leaves unlowered (device.cpp:149) gain lowerings the
//     B200 executor runs: kernel.matmul (TMA-staged operands into the tensor
//     core, tcgen05 on sm_100a) and the elementwise arithmetic, compare and
//     cast ops (register loads -> ALU/SFU op -> store; a / b is
//     sfu.rcp(b) then alu.mul, as task/dialect.cpp:36 prescribes);
//   * anything else still fails loudly (attention and kvcache ops).
#include <glog/logging.h>

#include <span>
#include <string>
#include <utility>
#include <vector>

#include "device/device.h"
#include "dialect/kernel/values.h"
#include "dialect/task/dialect.h"
#include "dialect/task/values.h"
#include "value.h"

namespace kvm::device {
namespace {

namespace kernel = ir::kernel;
namespace task = ir::task;
using ir::AnyOf;
using ir::Block;
using ir::OperationImpl;
using ir::Operator;
using ir::OpNode;
using ir::Type;
using ir::Value;
using ir::ValueNode;

const task::TensorImpl* TaskTensor(const ValueNode* v) {
  return v ? v->value().impl.as<task::TensorImpl>() : nullptr;
}
const kernel::TensorImpl* KernelTensor(const ValueNode* v) {
  return v ? v->value().impl.as<kernel::TensorImpl>() : nullptr;
}

std::string LineageBase(std::span<const std::string> input_names,
                        const std::string& op_name) {
  std::string base;
  for (const std::string& n : input_names) base += n + "_";
  for (char c : op_name) base += (c == '.') ? '_' : c;
  return base + "_";
}

// Appends single-result task ops to one block under one lineage base.
class Emitter {
 public:
  Emitter(const ir::serial::Registry& ops, Block* block, std::string base)
      : ops_(ops), block_(block), base_(std::move(base)) {}

  ValueNode* Emit(const std::string& key, AnyOf<OperationImpl> impl,
                  std::vector<ValueNode*> ins, const std::string& suffix,
                  std::vector<int> shape, task::Dtype dtype,
                  task::Location loc) {
    auto op = ops_.GetOperator(key);
    CHECK(op) << "sm100 decomp: task op '" << key << "' is not registered";
    Value out{base_ + suffix, Type{"tensor", "task"},
              task::TensorImpl{std::move(shape), {}, dtype, loc}};
    OpNode* node = block_->MakeOperation(ir::Operation{*op, std::move(impl)},
                                         std::move(ins), {std::move(out)});
    return node->results()[0];
  }

 private:
  const ir::serial::Registry& ops_;
  Block* block_;
  std::string base_;
};

// gemm: D = A.B + C -- the reference's expansion, unchanged.
std::vector<ValueNode*> LowerGemm(Emitter& em, std::span<ValueNode* const> ins,
                                  const ValueNode* kout) {
  const task::TensorImpl* a = TaskTensor(ins[0]);
  const task::TensorImpl* b = TaskTensor(ins[1]);
  const task::TensorImpl* c = TaskTensor(ins[2]);
  const kernel::TensorImpl* d = KernelTensor(kout);
  CHECK(a && b && c) << "sm100 decomp gemm: operands are not task tensors";
  CHECK(d) << "sm100 decomp gemm: result is not a kernel tensor";
  ValueNode* a_s = em.Emit("task.tma.gmem_to_smem", {}, {ins[0]}, "a_smem",
                           a->shape, a->dtype, task::Location::kShared);
  ValueNode* b_s = em.Emit("task.tma.gmem_to_smem", {}, {ins[1]}, "b_smem",
                           b->shape, b->dtype, task::Location::kShared);
  ValueNode* c_r = em.Emit("task.lsu.gmem_to_reg", {}, {ins[2]}, "c_reg",
                           c->shape, c->dtype, task::Location::kRegister);
  ValueNode* acc = em.Emit("task.tc.mma_acc", {}, {a_s, b_s, c_r}, "mma",
                           d->shape, d->dtype, task::Location::kRegister);
  return {em.Emit("task.lsu.reg_to_gmem", {}, {acc}, "out", d->shape, d->dtype,
                  task::Location::kGlobal)};
}

// matmul: D = A.B. Operands staged by TMA, the product in the tensor core
// (on sm_100a its accumulator lives in TMEM; the task dialect calls that
// location "register"), stored back to global.
std::vector<ValueNode*> LowerMatmul(Emitter& em,
                                    std::span<ValueNode* const> ins,
                                    const ValueNode* kout) {
  const task::TensorImpl* a = TaskTensor(ins[0]);
  const task::TensorImpl* b = TaskTensor(ins[1]);
  const kernel::TensorImpl* d = KernelTensor(kout);
  CHECK(a && b) << "sm100 decomp matmul: operands are not task tensors";
  CHECK(d) << "sm100 decomp matmul: result is not a kernel tensor";
  ValueNode* a_s = em.Emit("task.tma.gmem_to_smem", {}, {ins[0]}, "a_smem",
                           a->shape, a->dtype, task::Location::kShared);
  ValueNode* b_s = em.Emit("task.tma.gmem_to_smem", {}, {ins[1]}, "b_smem",
                           b->shape, b->dtype, task::Location::kShared);
  ValueNode* acc = em.Emit("task.tc.mma", {}, {a_s, b_s}, "mma", d->shape,
                           d->dtype, task::Location::kRegister);
  return {em.Emit("task.lsu.reg_to_gmem", {}, {acc}, "out", d->shape, d->dtype,
                  task::Location::kGlobal)};
}

// Elementwise op: operands loaded to registers, one (or, for div, two) task
// ALU/SFU ops, the result stored back.
std::vector<ValueNode*> LowerElementwise(Emitter& em, const std::string& name,
                                         std::span<ValueNode* const> ins,
                                         const ValueNode* kout) {
  const kernel::TensorImpl* d = KernelTensor(kout);
  CHECK(d) << "sm100 decomp " << name << ": result is not a kernel tensor";
  std::vector<ValueNode*> regs;
  const char* suffix[] = {"a_reg", "b_reg", "c_reg"};
  for (std::size_t i = 0; i < ins.size(); ++i) {
    const task::TensorImpl* t = TaskTensor(ins[i]);
    CHECK(t) << "sm100 decomp " << name << ": operand is not a task tensor";
    regs.push_back(em.Emit("task.lsu.gmem_to_reg", {}, {ins[i]}, suffix[i],
                           t->shape, t->dtype, task::Location::kRegister));
  }
  auto reg_op = [&](const std::string& key, std::vector<ValueNode*> args,
                    const std::string& sfx) {
    return em.Emit(key, {}, std::move(args), sfx, d->shape, d->dtype,
                   task::Location::kRegister);
  };
  ValueNode* r = nullptr;
  if (name == "div") {
    ValueNode* rcp = reg_op("task.sfu.rcp", {regs[1]}, "rcp");
    r = reg_op("task.alu.mul", {regs[0], rcp}, "div");
  } else if (name == "exp" || name == "log" || name == "sqrt" ||
             name == "rsqrt") {
    r = reg_op("task.sfu." + name, {regs[0]}, name);
  } else {
    std::string sfx = name;
    for (char& c : sfx)
      if (c == '.') c = '_';
    r = reg_op("task.alu." + name, regs, sfx);
  }
  return {em.Emit("task.lsu.reg_to_gmem", {}, {r}, "out", d->shape, d->dtype,
                  task::Location::kGlobal)};
}

// A collective stays one task op carrying the kernel op's rank constants
// (the reference's LowerCollective, device.cpp:108-121).
std::vector<ValueNode*> LowerCollective(Emitter& em, const OpNode* kop,
                                        std::span<ValueNode* const> ins,
                                        const ValueNode* kout) {
  const kernel::TensorImpl* out = KernelTensor(kout);
  CHECK(out) << "sm100 decomp collective: result is not a kernel tensor";
  return {em.Emit("task." + kop->op().op.name, kop->op().impl,
                  std::vector<ValueNode*>(ins.begin(), ins.end()), "out",
                  out->shape, out->dtype, task::Location::kGlobal)};
}

bool IsElementwise(const std::string& n) {
  static const char* kOps[] = {
      "add",    "sub",    "mul",    "div",    "max",       "min",
      "neg",    "exp",    "log",    "sqrt",   "rsqrt",     "abs",
      "cmp.eq", "cmp.ne", "cmp.lt", "cmp.le", "cmp.gt",    "cmp.ge",
      "cast.f16", "cast.f32", "cast.bf16", "cast.i32"};
  for (const char* k : kOps)
    if (n == k) return true;
  return false;
}

}  // namespace

Device::Device(const ir::GraphConfig& config) : config_(config) {
  task::RegisterTaskDialect(ops_);
}

std::vector<ir::ValueNode*> Device::Decomp(
    const ir::OpNode* kernel_op, std::span<ir::ValueNode* const> inputs,
    std::span<const std::string> input_names,
    std::span<const ir::ValueNode* const> kernel_outputs,
    ir::Block* block) const {
  const std::string& name = kernel_op->op().op.name;
  Emitter em(ops_, block, LineageBase(input_names, name));
  CHECK_EQ(kernel_outputs.size(), 1u)
      << "sm100 decomp " << name << ": expected 1 output";
  if (name == "gemm") return LowerGemm(em, inputs, kernel_outputs[0]);
  if (name == "matmul") return LowerMatmul(em, inputs, kernel_outputs[0]);
  if (name.rfind("comm.", 0) == 0)
    return LowerCollective(em, kernel_op, inputs, kernel_outputs[0]);
  if (IsElementwise(name))
    return LowerElementwise(em, name, inputs, kernel_outputs[0]);
  CHECK(false) << "sm100 decomp: no lowering for kernel op '" << name << "'";
  return {};
}

}  // namespace kvm::device
