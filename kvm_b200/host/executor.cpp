// Executor implementation: task graph -> launch plan over the sm_100a C ABI.
#include "executor.h"

#include <algorithm>
#include <any>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "dialect/kernel/ops.h"
#include "dialect/task/values.h"
#include "kvm_sm100.h"
#include "node.h"
#include "transform/kernel_to_task/kernel_to_task.h"

namespace kvm::sm100 {
namespace {

using ir::dialect::Dtype;

[[noreturn]] void Fail(const std::string& msg) {
  throw std::runtime_error("kvm executor: " + msg);
}

void Check(int rc, const char* what) {
  if (rc != KVM_OK)
    Fail(std::string(what) + ": " + kvm_sm100_last_error());
}

int EwDtype(Dtype d) {
  switch (d) {
    case Dtype::kBf16: return KVM_EW_BF16;
    case Dtype::kF16: return KVM_EW_F16;
    case Dtype::kI32: return KVM_EW_I32;
    case Dtype::kF32: return KVM_EW_F32;
    default: Fail("dtype " + ir::dialect::DtypeName(d) + " is not executable");
  }
}

const ir::task::TensorImpl& TaskTensorOf(const ir::ValueNode* v) {
  const auto* t = v->value().impl.as<ir::task::TensorImpl>();
  if (!t) Fail("value %" + v->value().name + " is not a task tensor");
  return *t;
}

std::string OpKey(const ir::OpNode* op) {
  const ir::Operator& o = op->op().op;
  return o.dialect.empty() ? o.name : o.dialect + "." + o.name;
}

bool StartsWith(const std::string& s, const char* p) { return s.rfind(p, 0) == 0; }

// Numpy-style broadcast of `in` to `out` as the interpreter's (size, div): the
// input's non-1 dimensions, right-aligned, must be one contiguous run of the
// output's dimensions; size = their product, div = product of the output
// dimensions after them.
void Broadcast(const std::vector<int64_t>& in, const std::vector<int64_t>& out,
               int64_t* size, int64_t* div) {
  const std::size_t r = out.size();
  if (in.size() > r) Fail("elementwise operand has more dimensions than the result");
  std::vector<int64_t> s(r, 1);
  for (std::size_t i = 0; i < in.size(); ++i) s[r - in.size() + i] = in[i];
  int first = -1, last = -1;
  for (std::size_t d = 0; d < r; ++d) {
    if (s[d] != 1 && s[d] != out[d]) Fail("elementwise operand does not broadcast");
    if (s[d] != 1) {
      if (first < 0) first = int(d);
      else if (last != int(d) - 1) Fail("unsupported broadcast pattern");
      last = int(d);
    }
  }
  *size = 1;
  *div = 1;
  if (first < 0) return;  // scalar
  for (int d = first; d <= last; ++d) *size *= out[d];
  for (std::size_t d = last + 1; d < r; ++d) *div *= out[d];
}

}  // namespace

int64_t DtypeBytes(Dtype d) {
  switch (d) {
    case Dtype::kI16: case Dtype::kF16: case Dtype::kBf16: return 2;
    case Dtype::kBool: return 1;
    default: return 4;
  }
}

int64_t Buffer::numel() const {
  int64_t n = 1;
  for (int64_t s : shape) n *= s;
  return n;
}

int64_t Buffer::bytes() const { return numel() * DtypeBytes(dtype); }

struct Executor::Routing {
  int T = 0, E = 0, k = 0;
  int32_t* idx = nullptr;
  float* w = nullptr;
  int32_t* offsets = nullptr;
  int32_t* pos = nullptr;
  int32_t* src = nullptr;
  void* ws = nullptr;
  // Expert parallelism over the op's ranks (P > 1): this rank (position me in
  // the rank set) owns experts [me*epr, (me+1)*epr); rows routed to them from
  // every rank arrive in `recv` (cap = T*k*P rows), expert outputs go to `y`;
  // both are mapped into every member (CUDA IPC).
  int P = 1, me = 0, epr = 0;
  int64_t cap = 0;
  kvm_ep_peers peers{};
  int32_t* send_base = nullptr;
  int32_t* loc_off = nullptr;
  uint32_t* done = nullptr;
  uint32_t epoch = 0;  // per Run, the same on every member
  kvm_comm* comm = nullptr;
  std::vector<void*> own_ipc, opened_ipc;
};

struct Executor::Slot {
  enum Kind { kGlobal, kView, kMma, kExpr } kind = kGlobal;
  Buffer buf;                             // kGlobal (ptr null until planned)
  const ir::ValueNode* base = nullptr;    // kView: the viewed global value
  std::vector<const ir::ValueNode*> args; // kMma (a, b[, c]) / kExpr operands
  std::string op;                         // kExpr: "alu.add", "sfu.exp", ...
  Routing* group = nullptr;               // rows grouped by a moe_dispatch
};

// Semantic view of an expression for pattern matching: loads and inlined
// globals are looked through, a * rcp(b) reads as div(a, b).
struct Executor::SNode {
  std::string op;                        // "" for a leaf
  std::vector<SNode> args;
  const ir::ValueNode* leaf = nullptr;   // the global a leaf reads
  bool is(const char* o) const { return op == o; }
};

struct Executor::SiluMatch {
  const ir::ValueNode* g = nullptr;  // gate GEMM result (not materialised)
  const ir::ValueNode* u = nullptr;  // up GEMM result (not materialised)
};

struct Executor::RmsMatch {
  const ir::ValueNode* x = nullptr;
  const ir::ValueNode* gamma = nullptr;  // may be null
  float eps = 0.f;
};

Executor::Executor(const ir::Graph& kernel, const ir::AttrMap& attrs)
    : kernel_(kernel), attrs_(attrs) {
  transform::TransformKernelToTask(kernel_, task_);
  for (const ir::ValueNode* a : task_.root()->arguments()) {
    const auto& t = TaskTensorOf(a);
    Buffer b;
    b.shape.assign(t.shape.begin(), t.shape.end());
    b.dtype = t.dtype;
    inputs_.push_back(b);
    input_names_.push_back(a->value().name);
  }
}

Executor::~Executor() {
  // Expert-parallel peer memory: every member stops using the others' buffers
  // (a barrier over the group's communicator) before any of them is freed.
  bool any_ep = false;
  for (auto& r : routings_) any_ep = any_ep || !r->own_ipc.empty();
  if (any_ep) {
    cudaDeviceSynchronize();
    void* one = nullptr;
    if (cudaMalloc(&one, sizeof(float)) == cudaSuccess) {
      for (auto& r : routings_) {
        if (r->own_ipc.empty()) continue;
        kvm_sm100_all_reduce(r->comm, one, one, 1, KVM_EW_F32, KVM_RED_SUM, nullptr);
        cudaDeviceSynchronize();
        for (void* q : r->opened_ipc) kvm_sm100_ipc_close(q);
        kvm_sm100_all_reduce(r->comm, one, one, 1, KVM_EW_F32, KVM_RED_SUM, nullptr);
        cudaDeviceSynchronize();
        for (void* q : r->own_ipc) kvm_sm100_ipc_free(q);
      }
      cudaFree(one);
    }
  }
  for (auto& kv : subcomms_)
    if (kv.second && kv.second != world_) kvm_sm100_comm_destroy(kv.second);
  for (void* p : allocations_) cudaFree(p);
}

void Executor::SetComm(kvm_comm* world) {
  if (prepared_) Fail("SetComm must come before Prepare");
  world_ = world;
  if (world_ && kvm_sm100_comm_rank(world_, &rank_, &nranks_) != KVM_OK)
    Fail(std::string("comm: ") + kvm_sm100_last_error());
}

// The communicator of a rank set, numbered by position in `ranks` (split
// from the world communicator once; every rank makes the same splits in the
// same order, since every rank plans the same graph). Null when this rank is
// not a member.
kvm_comm* Executor::CommFor(const std::vector<int>& ranks, int* my_index) {
  *my_index = -1;
  for (std::size_t i = 0; i < ranks.size(); ++i)
    if (ranks[i] == rank_) *my_index = int(i);
  std::vector<int> all(nranks_);
  for (int i = 0; i < nranks_; ++i) all[i] = i;
  if (ranks == all) return world_;
  auto it = subcomms_.find(ranks);
  if (it != subcomms_.end()) return it->second;
  std::vector<int32_t> r(ranks.begin(), ranks.end());
  kvm_comm* sub = nullptr;
  if (kvm_sm100_comm_split(world_, r.data(), int(r.size()), &sub) != KVM_OK)
    Fail(std::string("comm split: ") + kvm_sm100_last_error());
  subcomms_[ranks] = sub;
  return sub;
}

void* Executor::Alloc(int64_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes > 0 ? bytes : 16)) != cudaSuccess)
    Fail("cudaMalloc of " + std::to_string(bytes) + " bytes failed");
  allocations_.push_back(p);
  return p;
}

Executor::Slot& Executor::slot(const ir::ValueNode* v) {
  auto it = slots_.find(v);
  if (it == slots_.end()) Fail("value %" + v->value().name + " has no producer");
  return *it->second;
}

const ir::ValueNode* Executor::BaseGlobal(const ir::ValueNode* v) {
  while (slot(v).kind == Slot::kView) v = slot(v).base;
  return v;
}

const Buffer& Executor::GlobalOf(const ir::ValueNode* v) {
  Slot& s = slot(BaseGlobal(v));
  if (s.kind != Slot::kGlobal || !s.buf.ptr)
    Fail("value %" + v->value().name + " is read before it is stored");
  return s.buf;
}

Buffer& Executor::Materialize(const ir::ValueNode* v) {
  Slot& s = slot(v);
  if (!s.buf.ptr) s.buf.ptr = Alloc(s.buf.bytes());
  return s.buf;
}

const ir::OpNode* Executor::KernelCommOp(const std::string& name, int nth) const {
  int seen = 0;
  for (const ir::OpNode* op : kernel_.root()->operations())
    if (op->op().op.name == name && seen++ == nth) return op;
  return nullptr;
}

bool Executor::InputFill(const ir::ValueNode* v, double* value) const {
  const auto& targs = task_.root()->arguments();
  for (std::size_t i = 0; i < targs.size(); ++i) {
    if (targs[i] != v) continue;
    const std::any* a = attrs_.Get(kernel_.root()->arguments()[i], "fill");
    if (!a) return false;
    if (const auto* d = std::any_cast<double>(a)) { *value = *d; return true; }
    if (const auto* n = std::any_cast<std::int64_t>(a)) { *value = double(*n); return true; }
    return false;
  }
  return false;
}

void Executor::Analyze() {
  const ir::Block* root = task_.root();
  for (std::size_t i = 0; i < root->arguments().size(); ++i) {
    auto s = std::make_unique<Slot>();
    s->kind = Slot::kGlobal;
    s->buf = inputs_[i];
    slots_[root->arguments()[i]] = std::move(s);
  }
  auto new_global = [&](const ir::ValueNode* v, Routing* group) {
    const auto& t = TaskTensorOf(v);
    auto s = std::make_unique<Slot>();
    s->kind = Slot::kGlobal;
    s->buf.shape.assign(t.shape.begin(), t.shape.end());
    s->buf.dtype = t.dtype;
    s->group = group;
    slots_[v] = std::move(s);
  };
  for (const ir::OpNode* op : root->operations()) {
    const std::string key = OpKey(op);
    const ir::ValueNode* res = op->results().empty() ? nullptr : op->results()[0];
    for (const ir::ValueNode* a : op->operands()) consumers_[a].push_back(op);
    if (key == "task.tma.gmem_to_smem" || key == "task.lsu.gmem_to_reg" ||
        key == "task.lsu.smem_to_reg") {
      const ir::ValueNode* g = BaseGlobal(op->operands()[0]);
      ++uses_[g];
      auto s = std::make_unique<Slot>();
      s->kind = Slot::kView;
      s->base = op->operands()[0];
      s->group = slot(g).group;
      slots_[res] = std::move(s);
    } else if (key == "task.tc.mma" || key == "task.tc.mma_acc") {
      auto s = std::make_unique<Slot>();
      s->kind = Slot::kMma;
      s->args.assign(op->operands().begin(), op->operands().end());
      s->group = slot(op->operands()[0]).group;
      slots_[res] = std::move(s);
    } else if (StartsWith(key, "task.alu.") || StartsWith(key, "task.sfu.")) {
      auto s = std::make_unique<Slot>();
      s->kind = Slot::kExpr;
      s->op = key.substr(5);
      s->args.assign(op->operands().begin(), op->operands().end());
      for (const ir::ValueNode* a : s->args)
        if (!s->group) s->group = slot(a).group;
      slots_[res] = std::move(s);
    } else if (key == "task.lsu.reg_to_gmem" || key == "task.tma.smem_to_gmem") {
      producer_[res] = op->operands()[0];
      new_global(res, slot(op->operands()[0]).group);
      actions_.push_back(op);
    } else if (StartsWith(key, "task.comm.")) {
      for (const ir::ValueNode* a : op->operands()) ++uses_[BaseGlobal(a)];
      Routing* group = nullptr;
      if (op->op().op.name == "comm.moe_dispatch") {
        auto r = std::make_unique<Routing>();
        group = r.get();
        routing_by_op_[op] = group;
        routings_.push_back(std::move(r));
      }
      new_global(res, group);
      actions_.push_back(op);
    } else {
      Fail("no executor rule for task op '" + key + "'");
    }
  }
  for (const ir::ValueNode* o : root->outputs()) ++uses_[BaseGlobal(o)];
}

Executor::SNode Executor::Resolve(const ir::ValueNode* v) {
  Slot& s = slot(v);
  if (s.kind == Slot::kView) return Resolve(s.base);
  if (s.kind == Slot::kGlobal) {
    auto p = producer_.find(v);
    if (inlined_.count(v) && p != producer_.end()) return Resolve(p->second);
    SNode n;
    n.leaf = v;
    return n;
  }
  SNode n;
  if (s.kind == Slot::kMma) {
    n.op = "mma";
    return n;
  }
  if (s.op == "alu.mul" && slot(s.args[1]).kind == Slot::kExpr &&
      slot(s.args[1]).op == "sfu.rcp") {
    n.op = "div";
    n.args = {Resolve(s.args[0]), Resolve(slot(s.args[1]).args[0])};
    return n;
  }
  n.op = s.op;
  for (const ir::ValueNode* a : s.args) n.args.push_back(Resolve(a));
  return n;
}

// h = mul(div(g, add(exp(neg(g)), 1)), u) with g, u products of the same A.
bool Executor::MatchSilu(const ir::ValueNode* dst, SiluMatch* m) {
  auto pit = producer_.find(dst);
  if (pit == producer_.end() || slot(pit->second).kind != Slot::kExpr) return false;
  const SNode h = Resolve(pit->second);
  if (!h.is("alu.mul") || h.args.size() != 2) return false;
  for (int side = 0; side < 2; ++side) {
    const SNode& d = h.args[side];
    const SNode& u = h.args[1 - side];
    if (!d.is("div") || !u.leaf) continue;
    const SNode& x = d.args[0];
    const SNode& den = d.args[1];
    if (!x.leaf || !den.is("alu.add")) continue;
    for (int o = 0; o < 2; ++o) {
      const SNode& ex = den.args[o];
      const SNode& one = den.args[1 - o];
      double fill = 0;
      if (!ex.is("sfu.exp") || !ex.args[0].is("alu.neg") || !one.leaf) continue;
      if (ex.args[0].args[0].leaf != x.leaf) continue;
      if (!InputFill(one.leaf, &fill) || fill != 1.0) continue;
      const ir::ValueNode* g = x.leaf;
      const ir::ValueNode* uu = u.leaf;
      auto pg = producer_.find(g), pu = producer_.find(uu);
      if (pg == producer_.end() || pu == producer_.end()) return false;
      Slot& mg = slot(pg->second);
      Slot& mu = slot(pu->second);
      if (mg.kind != Slot::kMma || mu.kind != Slot::kMma || mg.args.size() != 2 ||
          mu.args.size() != 2)
        return false;
      if (BaseGlobal(mg.args[0]) != BaseGlobal(mu.args[0])) return false;
      const Buffer& bg = slot(BaseGlobal(mg.args[1])).buf;
      const Buffer& bu = slot(BaseGlobal(mu.args[1])).buf;
      if (bg.shape != bu.shape || bg.dtype != Dtype::kBf16) return false;
      const int64_t F = bg.shape.back();
      if (F % 128 != 0 || uses_[g] != 2 || uses_[uu] != 1) return false;
      if (slot(dst).buf.dtype != Dtype::kBf16) return false;
      m->g = g;
      m->u = uu;
      return true;
    }
  }
  return false;
}

// y = mul(mul(x, r), gamma) or mul(x, r), r = rsqrt(add(ms, eps)),
// ms = matmul(sq, invh) with invh = 1/H, sq = mul(x, x).
bool Executor::MatchRms(const ir::ValueNode* dst, RmsMatch* m) {
  auto pit = producer_.find(dst);
  if (pit == producer_.end() || slot(pit->second).kind != Slot::kExpr) return false;
  SNode y = Resolve(pit->second);
  const ir::ValueNode* gamma = nullptr;
  auto find_r = [](const SNode& n, const SNode** x, const SNode** r) {
    if (!n.is("alu.mul") || n.args.size() != 2) return false;
    for (int s = 0; s < 2; ++s)
      if (n.args[s].is("sfu.rsqrt") && n.args[1 - s].leaf) {
        *x = &n.args[1 - s];
        *r = &n.args[s];
        return true;
      }
    return false;
  };
  const SNode *x = nullptr, *r = nullptr;
  if (!find_r(y, &x, &r)) {
    if (!y.is("alu.mul") || y.args.size() != 2) return false;
    for (int s = 0; s < 2 && !x; ++s)
      if (y.args[1 - s].leaf && find_r(y.args[s], &x, &r)) gamma = y.args[1 - s].leaf;
    if (!x) return false;
  }
  const SNode& add = r->args[0];
  if (!add.is("alu.add")) return false;
  for (int s = 0; s < 2; ++s) {
    const SNode& ms = add.args[s];
    const SNode& eps = add.args[1 - s];
    double ev = 0, inv = 0;
    if (!ms.leaf || !eps.leaf || !InputFill(eps.leaf, &ev)) continue;
    auto pm = producer_.find(ms.leaf);
    if (pm == producer_.end() || slot(pm->second).kind != Slot::kMma) continue;
    Slot& mm = slot(pm->second);
    if (mm.args.size() != 2) continue;
    const ir::ValueNode* sq = BaseGlobal(mm.args[0]);
    const ir::ValueNode* invh = BaseGlobal(mm.args[1]);
    const Buffer& xb = slot(x->leaf).buf;
    if (xb.shape.size() != 2 || xb.dtype != Dtype::kBf16) return false;
    const int64_t H = xb.shape[1];
    if (!InputFill(invh, &inv) || std::abs(inv * double(H) - 1.0) > 1e-2) return false;
    auto ps = producer_.find(sq);
    if (ps == producer_.end() || slot(ps->second).kind != Slot::kExpr) return false;
    const SNode sqn = Resolve(ps->second);
    if (!sqn.is("alu.mul") || sqn.args[0].leaf != x->leaf || sqn.args[1].leaf != x->leaf)
      return false;
    if (uses_[sq] != 1 || uses_[ms.leaf] != 1 || H % 8 != 0) return false;
    if (gamma) {
      const Buffer& gb = slot(gamma).buf;
      if (gb.numel() != H || gb.dtype != Dtype::kBf16) return false;
    }
    if (slot(dst).buf.dtype != Dtype::kBf16 || slot(dst).buf.numel() != xb.numel())
      return false;
    m->x = x->leaf;
    m->gamma = gamma;
    m->eps = float(ev);
    elided_[sq] = true;
    elided_[ms.leaf] = true;
    return true;
  }
  return false;
}

void Executor::Fuse() {
  // KVM_EXEC_NO_FUSION=1 keeps every kernel op a launch of its own.
  if (const char* e = std::getenv("KVM_EXEC_NO_FUSION"); e && e[0] == '1') return;
  // 1. inline single-use elementwise results into their one consumer
  for (const ir::OpNode* op : actions_) {
    if (StartsWith(OpKey(op), "task.comm.")) continue;
    const ir::ValueNode* dst = op->results()[0];
    if (slot(producer_[dst]).kind != Slot::kExpr || uses_[dst] != 1) continue;
    bool feeds_expr = false;
    for (const ir::OpNode* c : consumers_[dst]) {
      if (OpKey(c) != "task.lsu.gmem_to_reg") continue;
      feeds_expr = true;
      for (const ir::OpNode* cc : consumers_[c->results()[0]]) {
        const std::string k = OpKey(cc);
        if (!StartsWith(k, "task.alu.") && !StartsWith(k, "task.sfu.")) feeds_expr = false;
      }
    }
    if (feeds_expr) inlined_[dst] = true;
  }
  // 2. composites
  for (const ir::OpNode* op : actions_) {
    if (StartsWith(OpKey(op), "task.comm.")) continue;
    const ir::ValueNode* dst = op->results()[0];
    if (inlined_.count(dst)) continue;
    SiluMatch sm;
    RmsMatch rm;
    if (MatchSilu(dst, &sm)) {
      elided_[sm.g] = elided_[sm.u] = true;
      silu_[dst] = std::make_unique<SiluMatch>(sm);
      fusions_.push_back("silu_gate: %" + dst->value().name + " = SiLU(%" +
                         sm.g->value().name + ") * %" + sm.u->value().name);
    } else if (MatchRms(dst, &rm)) {
      rms_[dst] = std::make_unique<RmsMatch>(rm);
      fusions_.push_back("rmsnorm: %" + dst->value().name + " = RMSNorm(%" +
                         rm.x->value().name + ")");
    }
  }
  // 3. router GEMMs that only feed moe_dispatch / moe_combine
  for (const ir::OpNode* op : actions_) {
    if (StartsWith(OpKey(op), "task.comm.")) continue;
    const ir::ValueNode* dst = op->results()[0];
    Slot& src = slot(producer_[dst]);
    if (src.kind != Slot::kMma || src.args.size() != 2) continue;
    const Buffer& b = slot(BaseGlobal(src.args[1])).buf;
    const Buffer& a = slot(BaseGlobal(src.args[0])).buf;
    if (b.shape.size() != 2 || b.shape[1] > 256 || b.dtype != Dtype::kBf16 ||
        a.dtype != Dtype::kBf16 || slot(dst).buf.dtype != Dtype::kF32 ||
        a.shape.size() != 2 || a.shape[1] % 8 != 0)
      continue;
    bool ok = !consumers_[dst].empty();
    for (const ir::OpNode* c : consumers_[dst]) {
      const std::string n = c->op().op.name;
      if ((n != "comm.moe_dispatch" && n != "comm.moe_combine") || c->operands()[1] != dst ||
          c->operands()[0] == dst)
        ok = false;
    }
    for (const ir::ValueNode* o : task_.root()->outputs())
      if (BaseGlobal(o) == dst) ok = false;
    if (ok) {
      router_[dst] = {BaseGlobal(src.args[0]), BaseGlobal(src.args[1])};
      fusions_.push_back("router: %" + dst->value().name + " = router GEMM + top-k");
    }
  }
}

void Executor::Plan() {
  if (analyzed_) return;
  Analyze();
  Fuse();
  analyzed_ = true;
}

void Executor::Prepare() {
  if (prepared_) return;
  Plan();
  const ir::Block* root = task_.root();
  for (std::size_t i = 0; i < root->arguments().size(); ++i) {
    inputs_[i].ptr = Alloc(inputs_[i].bytes());
    slot(root->arguments()[i]).buf.ptr = inputs_[i].ptr;
  }
  for (const ir::OpNode* op : actions_) {
    const ir::ValueNode* res = op->results()[0];
    if (StartsWith(OpKey(op), "task.comm.")) {
      PlanComm(op);
    } else if (inlined_.count(res) || elided_.count(res)) {
      continue;  // computed inside its consumer's launch
    } else if (silu_.count(res)) {
      PlanSilu(res);
    } else if (rms_.count(res)) {
      PlanRms(res);
    } else if (router_.count(res)) {
      Materialize(res);  // logits; the fused router launches with the dispatch
    } else {
      PlanStore(producer_[res], res);
    }
  }
  for (const ir::ValueNode* o : task_.root()->outputs()) outputs_.push_back(GlobalOf(o));
  prepared_ = true;
}

void Executor::PlanSilu(const ir::ValueNode* dst) {
  const SiluMatch& m = *silu_[dst];
  Slot& mg = slot(producer_[m.g]);
  Slot& mu = slot(producer_[m.u]);
  const Buffer A = GlobalOf(mg.args[0]);
  const Buffer Wg = GlobalOf(mg.args[1]);
  const Buffer Wu = GlobalOf(mu.args[1]);
  Buffer& out = Materialize(dst);
  const int64_t K = A.shape[1], F = Wg.shape.back();
  const int64_t E = Wg.shape.size() == 3 ? Wg.shape[0] : 1;
  const int64_t M = A.shape[0];
  if (Wg.shape[Wg.shape.size() - 2] != K) Fail("SiLU-gate GEMM: B rows must equal K");
  void* w13 = Alloc(2 * E * F * K * 2);
  const void* wg = Wg.ptr;
  const void* wu = Wu.ptr;
  once_steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_pack_gate_up(wg, wu, w13, int(E), int(F), int(K), KVM_B_KN, st);
  });
  const void* a = A.ptr;
  void* d = out.ptr;
  Routing* r = slot(BaseGlobal(mg.args[0])).group;
  if (Wg.shape.size() == 3) {
    if (!r || r->E != E) Fail("per-expert SiLU-gate GEMM needs A grouped by a moe_dispatch");
    if (r->P > 1) {
      if (M != r->cap) Fail("expert-parallel GEMM rows must be the dispatch's T*top_k*ranks");
      const void* wl = static_cast<const char*>(w13) + int64_t(r->me) * r->epr * 2 * F * K * 2;
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_grouped_gemm_bf16(a, wl, d, r->loc_off, r->epr, int(M),
                                           int(2 * F), int(K), 2, st);
      });
    } else {
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_grouped_gemm_bf16(a, w13, d, r->offsets, int(E), int(M),
                                           int(2 * F), int(K), 2, st);
      });
    }
    step_names_.push_back("grouped_gemm_silu_gate");
  } else {
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_gemm_bf16_silu_gate(a, K, w13, d, F, int(M), int(F), int(K), st);
    });
    step_names_.push_back("gemm_silu_gate");
  }
}

void Executor::PlanRms(const ir::ValueNode* dst) {
  const RmsMatch& m = *rms_[dst];
  const Buffer X = GlobalOf(m.x);
  const void* g = m.gamma ? GlobalOf(m.gamma).ptr : nullptr;
  Buffer& out = Materialize(dst);
  const void* x = X.ptr;
  void* y = out.ptr;
  const int rows = int(X.shape[0]), H = int(X.shape[1]);
  const float eps = m.eps;
  steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_rmsnorm_bf16(x, g, y, rows, H, eps, st);
  });
  step_names_.push_back("rmsnorm");
}

void Executor::PlanStore(const ir::ValueNode* src, const ir::ValueNode* dst) {
  Slot& s = slot(src);
  Buffer& out = Materialize(dst);
  if (s.kind == Slot::kMma) {
    PlanGemm(src, out);
  } else if (s.kind == Slot::kExpr) {
    PlanExpr(src, out);
  } else {
    const Buffer in = GlobalOf(src);
    if (in.bytes() != out.bytes()) Fail("store of %" + dst->value().name + ": size mismatch");
    void* d = out.ptr;
    const void* p = in.ptr;
    const int64_t n = in.bytes();
    steps_.push_back([d, p, n](cudaStream_t st) {
      return cudaMemcpyAsync(d, p, n, cudaMemcpyDeviceToDevice, st) == cudaSuccess
                 ? KVM_OK : KVM_ERR_CUDA;
    });
    step_names_.push_back("copy");
  }
}

void Executor::PlanGemm(const ir::ValueNode* mma, const Buffer& out) {
  Slot& s = slot(mma);
  const Buffer A = GlobalOf(s.args[0]);
  const Buffer B = GlobalOf(s.args[1]);
  const Buffer* C = s.args.size() > 2 ? &GlobalOf(s.args[2]) : nullptr;
  if (A.dtype != Dtype::kBf16 || B.dtype != Dtype::kBf16)
    Fail("tcgen05 GEMM in this build takes bf16 operands (got " +
         ir::dialect::DtypeName(A.dtype) + ", " + ir::dialect::DtypeName(B.dtype) + ")");
  if (A.shape.size() != 2) Fail("GEMM A operand must be 2-D");
  const int64_t M = A.shape[0], K = A.shape[1];
  if (B.shape.size() == 2 && B.shape[1] == 1 && !C) {
    if (B.shape[0] != K) Fail("GEMM inner dimensions disagree");
    if (out.dtype != Dtype::kBf16 && out.dtype != Dtype::kF32)
      Fail("GEMM result must be bf16 or f32");
    const void* a = A.ptr; const void* b = B.ptr;
    void* d = out.ptr;
    const int od = out.dtype == Dtype::kF32 ? KVM_F32 : KVM_BF16;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_gemv_bf16(a, K, b, d, od, int(M), int(K), st);
    });
    step_names_.push_back("gemv_bf16");
    return;
  }
  if (B.shape.size() == 2) {
    if (B.shape[0] != K) Fail("GEMM inner dimensions disagree");
    const int64_t N = B.shape[1];
    if (out.numel() != M * N) Fail("GEMM result shape disagrees with A.B");
    if (out.dtype != Dtype::kBf16 && out.dtype != Dtype::kF32)
      Fail("GEMM result must be bf16 or f32");
    if (C && (C->dtype != out.dtype || C->numel() != out.numel()))
      Fail("gemm addend C must match the result's dtype and shape");
    const void* a = A.ptr; const void* b = B.ptr;
    const void* c = C ? C->ptr : nullptr;
    void* d = out.ptr;
    const int od = out.dtype == Dtype::kF32 ? KVM_F32 : KVM_BF16;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_gemm_bf16(a, K, b, N, KVM_B_KN, c, d, N, od, int(M), int(N),
                                 int(K), st);
    });
    step_names_.push_back("gemm_bf16");
    return;
  }
  if (B.shape.size() != 3) Fail("GEMM B operand must be 2-D or 3-D");
  if (!s.group) Fail("a 3-D (per-expert) B needs A rows grouped by a moe_dispatch");
  if (C) Fail("per-expert gemm with an addend is not supported");
  const int64_t E = B.shape[0], N = B.shape[2];
  if (B.shape[1] != K || E != s.group->E) Fail("per-expert B must be [E, K, N]");
  if (out.dtype != Dtype::kBf16) Fail("per-expert GEMM result must be bf16");
  // One-time re-layout of the expert weights [E, K, N] -> [E, N, K].
  void* bt = Alloc(B.bytes());
  const void* b = B.ptr;
  once_steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_transpose_bf16(b, bt, int(E), int(K), int(N), st);
  });
  Routing* r = s.group;
  const void* a = A.ptr;
  void* d = out.ptr;
  if (r->P > 1) {
    // this rank's experts over the rows it received
    if (M != r->cap) Fail("expert-parallel GEMM rows must be the dispatch's T*top_k*ranks");
    const void* bl = static_cast<const char*>(bt) + int64_t(r->me) * r->epr * N * K * 2;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_grouped_gemm_bf16(a, bl, d, r->loc_off, r->epr, int(M), int(N),
                                         int(K), 0, st);
    });
    step_names_.push_back("grouped_gemm_bf16");
    return;
  }
  steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_grouped_gemm_bf16(a, bt, d, r->offsets, int(E), int(M), int(N),
                                       int(K), 0, st);
  });
  step_names_.push_back("grouped_gemm_bf16");
}

void Executor::PlanExpr(const ir::ValueNode* expr, const Buffer& out) {
  kvm_ew_program prog;
  std::memset(&prog, 0, sizeof(prog));
  kvm_ew_inputs ins;
  std::memset(&ins, 0, sizeof(ins));
  std::unordered_map<const void*, int> input_of;  // buffer -> input slot
  std::unordered_map<const ir::ValueNode*, int> reg_of;
  int next_reg = 0;
  auto emit = [&](int op, int a, int b) {
    if (prog.n_instr >= KVM_EW_MAX_INSTR || next_reg >= KVM_EW_MAX_REGS)
      Fail("elementwise expression too large");
    const int s = prog.n_instr++;
    prog.op[s] = uint8_t(op);
    prog.a[s] = uint8_t(a);
    prog.b[s] = uint8_t(b);
    prog.dst[s] = uint8_t(next_reg);
    return next_reg++;
  };
  std::function<int(const ir::ValueNode*)> gen = [&](const ir::ValueNode* v) -> int {
    auto it = reg_of.find(v);
    if (it != reg_of.end()) return it->second;
    Slot& s = slot(v);
    int r;
    const ir::ValueNode* gv = s.kind == Slot::kExpr ? nullptr : BaseGlobal(v);
    if (gv && inlined_.count(gv)) {
      // the producer's expression, rounded to the inlined value's dtype
      r = gen(producer_[gv]);
      const Dtype dt = slot(gv).buf.dtype;
      if (dt == Dtype::kBf16) r = emit(KVM_EW_ROUND_BF16, r, 0);
      else if (dt == Dtype::kF16) r = emit(KVM_EW_ROUND_F16, r, 0);
      else if (dt == Dtype::kI32) r = emit(KVM_EW_TRUNC_I32, r, 0);
    } else if (s.kind != Slot::kExpr) {
      const Buffer& b = GlobalOf(v);
      auto in = input_of.find(b.ptr);
      int slot_i;
      if (in == input_of.end()) {
        if (prog.n_inputs >= KVM_EW_MAX_INPUTS) Fail("elementwise: too many inputs");
        slot_i = prog.n_inputs++;
        ins.ptr[slot_i] = b.ptr;
        prog.in_dtype[slot_i] = EwDtype(b.dtype);
        Broadcast(b.shape, out.shape, &prog.in_size[slot_i], &prog.in_div[slot_i]);
        input_of[b.ptr] = slot_i;
      } else {
        slot_i = in->second;
      }
      r = emit(KVM_EW_LOAD, slot_i, 0);
    } else {
      const std::string& op = s.op;
      // a * (1 / b) as lowered for kernel.div is the division a / b.
      if (op == "alu.mul" && slot(s.args[1]).kind == Slot::kExpr &&
          slot(s.args[1]).op == "sfu.rcp") {
        const int a = gen(s.args[0]);
        const int b = gen(slot(s.args[1]).args[0]);
        r = emit(KVM_EW_DIV, a, b);
      } else {
        static const std::unordered_map<std::string, int> kOps = {
            {"alu.add", KVM_EW_ADD}, {"alu.sub", KVM_EW_SUB}, {"alu.mul", KVM_EW_MUL},
            {"alu.max", KVM_EW_MAX}, {"alu.min", KVM_EW_MIN}, {"alu.neg", KVM_EW_NEG},
            {"alu.abs", KVM_EW_ABS}, {"sfu.rcp", KVM_EW_RCP}, {"sfu.exp", KVM_EW_EXP},
            {"sfu.log", KVM_EW_LOG}, {"sfu.sqrt", KVM_EW_SQRT},
            {"sfu.rsqrt", KVM_EW_RSQRT}, {"alu.cmp.eq", KVM_EW_CMP_EQ},
            {"alu.cmp.ne", KVM_EW_CMP_NE}, {"alu.cmp.lt", KVM_EW_CMP_LT},
            {"alu.cmp.le", KVM_EW_CMP_LE}, {"alu.cmp.gt", KVM_EW_CMP_GT},
            {"alu.cmp.ge", KVM_EW_CMP_GE}, {"alu.cast.bf16", KVM_EW_ROUND_BF16},
            {"alu.cast.f16", KVM_EW_ROUND_F16}, {"alu.cast.i32", KVM_EW_TRUNC_I32},
            {"alu.cast.f32", -1}};
        auto k = kOps.find(op);
        if (k == kOps.end()) Fail("no elementwise rule for task op '" + op + "'");
        const int a = gen(s.args[0]);
        const int b = s.args.size() > 1 ? gen(s.args[1]) : 0;
        r = k->second < 0 ? a : emit(k->second, a, b);
      }
    }
    reg_of[v] = r;
    return r;
  };
  prog.out_reg = gen(expr);
  prog.out_dtype = EwDtype(out.dtype);
  void* d = out.ptr;
  const int64_t n = out.numel();
  for (int i = 0; i < prog.n_inputs; ++i)
    if (n % (prog.in_size[i] * prog.in_div[i]) != 0)
      Fail("elementwise operand does not broadcast to the result shape");
  // generate + compile the fused kernel now, not inside the first (maybe
  // captured) run
  if (kvm_sm100_elementwise_prepare(&prog, &ins, d, n) != KVM_OK)
    Fail(std::string("elementwise: ") + kvm_sm100_last_error());
  steps_.push_back([prog, ins, d, n](cudaStream_t st) {
    return kvm_sm100_elementwise(&prog, &ins, d, n, st);
  });
  step_names_.push_back("elementwise");
}

// Routing of a moe_dispatch (one rank or several): top_k from the kernel op's
// attrs, then softmax + top-k (fused with the router GEMM when its logits feed
// only the MoE ops) and the expert-major permutation of this rank's pairs.
Executor::Routing* Executor::PlanRoute(const ir::OpNode* op, const ir::OpNode* kop,
                                       const Buffer& x, const Buffer& g) {
  if (x.shape.size() != 2 || g.shape.size() != 2 || g.shape[0] != x.shape[0])
    Fail("moe_dispatch(x [T,H], g [T,E]) shapes disagree");
  if (x.dtype != Dtype::kBf16) Fail("moe_dispatch tokens must be bf16");
  int k = 2;
  if (kop)
    if (const std::any* a = attrs_.Get(kop, "top_k"))
      if (const auto* v = std::any_cast<std::int64_t>(a)) k = int(*v);
  Routing* r = routing_by_op_.at(op);
  r->T = int(x.shape[0]);
  r->E = int(g.shape[1]);
  r->k = k;
  const int64_t n = int64_t(r->T) * k;
  r->idx = static_cast<int32_t*>(Alloc(n * 4));
  r->w = static_cast<float*>(Alloc(n * 4));
  r->offsets = static_cast<int32_t*>(Alloc((r->E + 1) * 4));
  r->pos = static_cast<int32_t*>(Alloc(n * 4));
  r->src = static_cast<int32_t*>(Alloc(n * 4));
  r->ws = Alloc(kvm_sm100_moe_permute_workspace(r->T, k, r->E));
  Routing* rp = r;
  void* gp = g.ptr;
  const int gd = EwDtype(g.dtype);
  auto rt = router_.find(BaseGlobal(op->operands()[1]));
  if (rt != router_.end()) {
    // router GEMM + softmax + top-k in one kernel; its weight [H, E] is
    // re-laid out once to [E, H]
    const Buffer& ra = GlobalOf(rt->second.first);
    const Buffer& rw = GlobalOf(rt->second.second);
    const int RH = int(rw.shape[0]), RE = int(rw.shape[1]);
    void* wt = Alloc(rw.bytes());
    const void* wsrc = rw.ptr;
    once_steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_transpose_bf16(wsrc, wt, 1, RH, RE, st);
    });
    const void* ap = ra.ptr;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_moe_router_topk(ap, wt, static_cast<float*>(gp), rp->idx, rp->w,
                                       rp->T, RH, RE, rp->k, st);
    });
    step_names_.push_back("moe_router_topk");
  } else {
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_moe_topk(gp, gd, rp->T, rp->E, rp->k, rp->idx, rp->w, st);
    });
    step_names_.push_back("moe_topk");
  }
  steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_moe_permute(rp->idx, rp->T, rp->k, rp->E, rp->offsets, rp->pos,
                                 rp->src, rp->ws, st);
  });
  step_names_.push_back("moe_permute");
  return r;
}

// moe_dispatch over several ranks: expert parallelism. The rank set's
// communicator carries a one-time exchange of CUDA IPC handles (receive rows,
// expert outputs, count matrix, flags) at Prepare; every Run then routes and
// permutes this rank's tokens, exchanges counts, stores each routed row into
// its owner's receive buffer (peer stores) and waits for every member's rows.
// The dispatch result is the receive buffer: T*top_k*ranks rows (capacity),
// expert-major then source-rank-major, of which the first loc_off[E/ranks]
// are filled; the expert GEMMs over it use this rank's experts only.
void Executor::PlanExpertDispatch(const ir::OpNode* op, const std::vector<int>& ranks) {
  int nth = 0;
  for (const ir::OpNode* o : task_.root()->operations()) {
    if (o == op) break;
    if (o->op().op.name == "comm.moe_dispatch") ++nth;
  }
  const ir::OpNode* kop = KernelCommOp("comm.moe_dispatch", nth);
  const ir::ValueNode* res = op->results()[0];
  if (!world_)
    Fail("moe_dispatch over " + std::to_string(ranks.size()) +
         " ranks needs a communicator (kvm_run --rank/--world)");
  if (ranks.size() > KVM_EP_MAX_RANKS) Fail("expert parallelism over more than 8 ranks");
  int me = -1;
  kvm_comm* comm = CommFor(ranks, &me);
  if (me < 0) Fail("this rank is not in the moe_dispatch's rank set");
  const Buffer x = GlobalOf(op->operands()[0]);
  const Buffer g = GlobalOf(op->operands()[1]);
  Routing* r = PlanRoute(op, kop, x, g);
  const int P = int(ranks.size()), E = r->E, H = int(x.shape[1]);
  if (E % P != 0) Fail("moe_dispatch: the experts must split evenly over the ranks");
  r->P = P;
  r->me = me;
  r->epr = E / P;
  r->comm = comm;
  r->cap = int64_t(r->T) * r->k * P;
  // peer buffers, mapped into every member
  const int64_t bytes[4] = {r->cap * H * 2, r->cap * H * 2, int64_t(P) * E * 4,
                            int64_t(3 + r->epr) * P * 4};
  void* own[4];
  for (int i = 0; i < 4; ++i) {
    if (kvm_sm100_ipc_alloc(bytes[i], &own[i]) != KVM_OK)
      Fail(std::string("expert parallel: ") + kvm_sm100_last_error());
    r->own_ipc.push_back(own[i]);
  }
  std::vector<char> mine(4 * 64), all(size_t(P) * 4 * 64);
  for (int i = 0; i < 4; ++i)
    if (kvm_sm100_ipc_get_handle(own[i], mine.data() + i * 64) != KVM_OK)
      Fail(std::string("expert parallel: ") + kvm_sm100_last_error());
  void* dev = Alloc(int64_t(P + 1) * 4 * 64);
  void* dev_all = static_cast<char*>(dev) + 4 * 64;
  cudaMemcpy(dev, mine.data(), mine.size(), cudaMemcpyHostToDevice);
  if (kvm_sm100_all_gather(comm, dev, dev_all, 4 * 64 / 4, KVM_EW_I32, nullptr) != KVM_OK)
    Fail(std::string("expert parallel: handle exchange: ") + kvm_sm100_last_error());
  cudaDeviceSynchronize();
  cudaMemcpy(all.data(), dev_all, all.size(), cudaMemcpyDeviceToHost);
  kvm_ep_peers& pr = r->peers;
  std::memset(&pr, 0, sizeof(pr));
  pr.rank = me;
  pr.world = P;
  pr.E = E;
  pr.H = H;
  pr.k = r->k;
  for (int q = 0; q < P; ++q) {
    void* ptr[4];
    for (int i = 0; i < 4; ++i) {
      if (q == me) {
        ptr[i] = own[i];
      } else {
        if (kvm_sm100_ipc_open_handle(all.data() + (size_t(q) * 4 + i) * 64, &ptr[i]) !=
            KVM_OK)
          Fail(std::string("expert parallel: ") + kvm_sm100_last_error());
        r->opened_ipc.push_back(ptr[i]);
      }
    }
    pr.recv[q] = ptr[0];
    pr.y[q] = ptr[1];
    pr.cnt[q] = ptr[2];
    pr.flags[q] = ptr[3];
  }
  r->send_base = static_cast<int32_t*>(Alloc(int64_t(E) * 4));
  r->loc_off = static_cast<int32_t*>(Alloc(int64_t(r->epr + 1) * 4));
  r->done = static_cast<uint32_t*>(Alloc(16));
  cudaMemset(r->done, 0, 16);
  // the dispatch result lives in the receive buffer; the expert outputs the
  // matching moe_combine reads live in the peer-visible y buffer
  Slot& rs = slot(res);
  if (rs.buf.numel() != r->cap * H || rs.buf.dtype != Dtype::kBf16)
    Fail("moe_dispatch over " + std::to_string(P) + " ranks: result must be bf16 [T*top_k*" +
         std::to_string(P) + ", H] (this rank's receive capacity)");
  rs.buf.ptr = own[0];
  for (const ir::OpNode* c : consumers_[BaseGlobal(op->operands()[1])])
    if (c->op().op.name == "comm.moe_combine") {
      Slot& ys = slot(BaseGlobal(c->operands()[0]));
      if (!ys.buf.ptr && ys.buf.numel() == r->cap * H && ys.buf.dtype == Dtype::kBf16)
        ys.buf.ptr = own[1];
    }
  Routing* rp = r;
  const kvm_ep_peers* prp = &r->peers;
  const void* xp = x.ptr;
  steps_.push_back([=](cudaStream_t st) {
    ++rp->epoch;
    return kvm_sm100_ep_counts(prp, rp->offsets, rp->send_base, rp->loc_off, rp->epoch, st);
  });
  step_names_.push_back("ep_counts");
  steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_ep_dispatch(prp, xp, rp->idx, rp->pos, rp->offsets, rp->send_base,
                                 rp->T, rp->cap, rp->done, rp->epoch, st);
  });
  step_names_.push_back("ep_dispatch");
  steps_.push_back([=](cudaStream_t st) {
    return kvm_sm100_ep_wait(prp, 1, rp->epoch, st);
  });
  step_names_.push_back("ep_wait");
  routing_of_[g.ptr] = r;
}

void Executor::PlanComm(const ir::OpNode* op) {
  const std::string name = op->op().op.name;  // "comm.moe_dispatch", ...
  int nth = 0;
  for (const ir::OpNode* o : task_.root()->operations()) {
    if (o == op) break;
    if (o->op().op.name == name) ++nth;
  }
  const ir::OpNode* kop = KernelCommOp(name, nth);
  const ir::ValueNode* res = op->results()[0];
  std::vector<int> moe_ranks;
  if (name == "comm.moe_dispatch" || name == "comm.moe_combine") {
    // Over several ranks the op is the expert-parallel exchange: the experts
    // are split evenly over the ranks (in the order of the op's rank list),
    // and the exchange runs over NVLink peer memory (ep.cu).
    if (const auto* r = op->op().impl.as<ir::kernel::MoeDispatch>()) moe_ranks = r->ranks;
    if (const auto* r = op->op().impl.as<ir::kernel::MoeCombine>()) moe_ranks = r->ranks;
    std::sort(moe_ranks.begin(), moe_ranks.end());
    moe_ranks.erase(std::unique(moe_ranks.begin(), moe_ranks.end()), moe_ranks.end());
  }
  if (name == "comm.moe_dispatch" && moe_ranks.size() > 1) {
    PlanExpertDispatch(op, moe_ranks);
    return;
  }
  if (name == "comm.moe_dispatch") {
    const Buffer x = GlobalOf(op->operands()[0]);
    const Buffer g = GlobalOf(op->operands()[1]);
    Routing* rp = PlanRoute(op, kop, x, g);
    const int64_t n = int64_t(rp->T) * rp->k;
    Buffer& out = Materialize(res);
    if (out.numel() != n * x.shape[1] || out.dtype != Dtype::kBf16)
      Fail("moe_dispatch result must be bf16 [T*top_k, H]");
    const void* xp = x.ptr;
    void* dp = out.ptr;
    const int H = int(x.shape[1]);
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_moe_scatter_rows(xp, rp->pos, dp, rp->T, rp->k, H, st);
    });
    step_names_.push_back("moe_scatter_rows");
    routing_of_[g.ptr] = rp;
    return;
  }
  if (name == "comm.moe_combine") {
    const Buffer y = GlobalOf(op->operands()[0]);
    const Buffer g = GlobalOf(op->operands()[1]);
    auto it = routing_of_.find(g.ptr);
    if (it == routing_of_.end()) Fail("moe_combine(y, g): g was never dispatched on");
    Routing* rp = it->second;
    Buffer& out = Materialize(res);
    const int H = int(y.shape.back());
    if (out.numel() != int64_t(rp->T) * H || out.dtype != Dtype::kBf16)
      Fail("moe_combine result must be bf16 [T, H]");
    if ((moe_ranks.size() > 1) != (rp->P > 1))
      Fail("moe_combine must run over the rank set of its moe_dispatch");
    if (rp->P > 1) {
      // The reverse exchange: every member's expert outputs are complete,
      // then each token's k rows are loaded from their owners (peer loads)
      // and combined as on one GPU.
      if (y.ptr != rp->peers.y[rp->me] || y.numel() != rp->cap * H)
        Fail("expert-parallel moe_combine(y, g): y must be the expert GEMM output over the "
             "dispatch's rows [T*top_k*ranks, H]");
      const kvm_ep_peers* pr = &rp->peers;
      void* o = out.ptr;
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_ep_signal(pr, 2, rp->epoch, st);
      });
      step_names_.push_back("ep_signal");
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_ep_wait(pr, 2, rp->epoch, st);
      });
      step_names_.push_back("ep_wait");
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_ep_combine(pr, rp->idx, rp->pos, rp->offsets, rp->send_base, rp->w,
                                    o, rp->T, rp->cap, st);
      });
      step_names_.push_back("ep_combine");
      return;
    }
    const void* yp = y.ptr;
    void* op_ = out.ptr;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_moe_combine(yp, rp->pos, rp->w, op_, rp->T, rp->k, H, st);
    });
    step_names_.push_back("moe_combine");
    return;
  }
  // The collectives proper (kernel/dialect.cpp:58-64). A rank outside an
  // op's rank set, and every op over a single rank, passes its input
  // through; the members exchange over NCCL (kvm_sm100_all_reduce, ...).
  std::vector<int> ranks;
  int root_rank = -1, peer_from = -1, peer_to = -1;
  if (const auto* r = op->op().impl.as<ir::kernel::AllReduceSum>()) ranks = r->ranks;
  if (const auto* r = op->op().impl.as<ir::kernel::AllReduceMax>()) ranks = r->ranks;
  if (const auto* r = op->op().impl.as<ir::kernel::AllGather>()) ranks = r->ranks;
  if (const auto* r = op->op().impl.as<ir::kernel::AllToAllOp>()) ranks = r->ranks;
  if (const auto* r = op->op().impl.as<ir::kernel::BroadcastOp>()) {
    root_rank = r->from;
    ranks = r->to;
    ranks.push_back(r->from);
    std::sort(ranks.begin(), ranks.end());
    ranks.erase(std::unique(ranks.begin(), ranks.end()), ranks.end());
  }
  if (const auto* r = op->op().impl.as<ir::kernel::SendOp>()) {
    peer_from = r->from;
    peer_to = r->to;
  }
  if (const auto* r = op->op().impl.as<ir::kernel::RecvOp>()) {
    peer_from = r->from;
    peer_to = r->to;
  }
  const Buffer in = GlobalOf(op->operands()[0]);
  const bool p2p = name == "comm.send" || name == "comm.recv";
  const bool single = p2p ? peer_from == peer_to : ranks.size() <= 1;
  if (single) {
    PlanStore(op->operands()[0], res);
    return;
  }
  if (!world_)
    Fail("'" + name + "' across ranks needs a communicator (kvm_run --rank/--world)");
  const int dt = EwDtype(in.dtype);
  const int64_t count = in.numel();
  const void* src = in.ptr;
  if (p2p) {
    if (peer_from < 0 || peer_to < 0 || peer_from >= nranks_ || peer_to >= nranks_)
      Fail("'" + name + "': rank outside the world");
    kvm_comm* w = world_;
    if (name == "comm.send" && rank_ == peer_from) {
      PlanStore(op->operands()[0], res);  // the sender keeps its value
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_send(w, src, count, dt, peer_to, st);
      });
      step_names_.push_back("comm_send");
    } else if (name == "comm.recv" && rank_ == peer_to) {
      Buffer& out = Materialize(res);
      if (out.numel() != count) Fail("comm.recv: result shape != operand shape");
      void* dst = out.ptr;
      steps_.push_back([=](cudaStream_t st) {
        return kvm_sm100_recv(w, dst, count, dt, peer_from, st);
      });
      step_names_.push_back("comm_recv");
    } else {
      PlanStore(op->operands()[0], res);
    }
    return;
  }
  for (int r : ranks)
    if (r < 0 || r >= nranks_) Fail("'" + name + "': rank outside the world");
  int me = -1;
  kvm_comm* c = CommFor(ranks, &me);
  if (me < 0 || !c) {
    PlanStore(op->operands()[0], res);
    return;
  }
  Buffer& out = Materialize(res);
  void* dst = out.ptr;
  const int P = int(ranks.size());
  if (name == "comm.all_reduce.sum" || name == "comm.all_reduce.max") {
    if (out.numel() != count) Fail(name + ": result shape != operand shape");
    const int red = name == "comm.all_reduce.sum" ? KVM_RED_SUM : KVM_RED_MAX;
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_all_reduce(c, src, dst, count, dt, red, st);
    });
  } else if (name == "comm.all_gather") {
    if (out.numel() != count * P)
      Fail("comm.all_gather: result must hold ranks x operand elements (dim 0 stacked)");
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_all_gather(c, src, dst, count, dt, st);
    });
  } else if (name == "comm.all_to_all") {
    if (out.numel() != count || count % P)
      Fail("comm.all_to_all: operand must split evenly over the ranks (dim 0)");
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_all_to_all(c, src, dst, count / P, dt, st);
    });
  } else if (name == "comm.broadcast") {
    if (out.numel() != count) Fail("comm.broadcast: result shape != operand shape");
    const int root = int(std::find(ranks.begin(), ranks.end(), root_rank) - ranks.begin());
    steps_.push_back([=](cudaStream_t st) {
      return kvm_sm100_broadcast(c, src, dst, count, dt, root, st);
    });
  } else {
    Fail("collective '" + name + "' is not supported");
  }
  std::string sn = name.substr(5);
  std::replace(sn.begin(), sn.end(), '.', '_');
  step_names_.push_back("comm_" + sn);
}

void Executor::CopyInput(int index, const void* host, int64_t bytes) {
  if (index < 0 || index >= int(inputs_.size())) Fail("input index out of range");
  if (!prepared_) Prepare();
  if (bytes != inputs_[index].bytes()) Fail("input " + input_names_[index] + ": byte count");
  if (cudaMemcpy(inputs_[index].ptr, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess)
    Fail("input copy failed");
}

void Executor::FillInputNormal(int index, uint64_t seed, float mean, float std) {
  if (!prepared_) Prepare();
  const Buffer& b = inputs_.at(index);
  Check(kvm_sm100_fill_normal(b.ptr, EwDtype(b.dtype), b.numel(), seed, mean, std,
                              nullptr), "fill_normal");
}

void Executor::FillInputConst(int index, float value) {
  if (!prepared_) Prepare();
  const Buffer& b = inputs_.at(index);
  void* scalar = Alloc(4);
  if (cudaMemcpy(scalar, &value, 4, cudaMemcpyHostToDevice) != cudaSuccess)
    Fail("constant copy failed");
  kvm_ew_program prog;
  std::memset(&prog, 0, sizeof(prog));
  prog.n_inputs = 1;
  prog.n_instr = 1;
  prog.in_dtype[0] = KVM_EW_F32;
  prog.in_size[0] = 1;
  prog.in_div[0] = 1;
  prog.out_dtype = EwDtype(b.dtype);
  kvm_ew_inputs ins;
  std::memset(&ins, 0, sizeof(ins));
  ins.ptr[0] = scalar;
  Check(kvm_sm100_elementwise(&prog, &ins, b.ptr, b.numel(), nullptr), "fill const");
}

int Executor::Run(cudaStream_t stream) {
  if (!prepared_) Prepare();
  if (!once_done_) {
    for (auto& s : once_steps_)
      if (int rc = s(stream); rc != KVM_OK) return rc;
    once_done_ = true;
  }
  for (auto& s : steps_)
    if (int rc = s(stream); rc != KVM_OK) return rc;
  return KVM_OK;
}

}  // namespace kvm::sm100
