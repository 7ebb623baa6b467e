#include "task_to_tile.h"

#include <glog/logging.h>

#include <algorithm>
#include <map>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "dialect/task/values.h"
#include "dialect/tile/dialect.h"
#include "dialect/tile/ops.h"
#include "dialect/tile/values.h"
#include "dialect/tile/verify.h"
#include "serialization/registry.h"

namespace kvm::sm100 {
namespace {

namespace task = ir::task;
namespace tile = ir::tile;
using ir::AnyOf;
using ir::Block;
using ir::Graph;
using ir::OperationImpl;
using ir::OpNode;
using ir::Type;
using ir::Value;
using ir::ValueNode;
using ir::dialect::Dtype;

constexpr int kTileM = 128;  // rows of one tcgen05 tile (one SM)
constexpr int kTileK = 16;   // K of one kind::f16 instruction

tile::Location TileLoc(task::Location l) {
  switch (l) {
    case task::Location::kShared:
      return tile::Location::kShared;
    case task::Location::kRegister:
      return tile::Location::kRegister;
    default:
      return tile::Location::kGlobal;
  }
}

const task::TensorImpl* TaskTensor(const ValueNode* v) {
  return v ? v->value().impl.as<task::TensorImpl>() : nullptr;
}

int CeilDiv(int a, int b) { return (a + b - 1) / b; }

// Name of the tile of `name` at `slice`: "name_at_r_c" (the text form
// refers to values by name, so every tile value gets its own).
std::string TileName(const std::string& name, const std::vector<int>& slice) {
  if (slice.empty()) return name;
  std::string k = name + "_at_";
  for (std::size_t i = 0; i < slice.size(); ++i)
    k += (i ? "_" : "") + std::to_string(slice[i]);
  return k;
}

// A tensor-core chain of the task graph: D = A.B [+ C], A and B staged from
// global by TMA, C loaded to registers, D stored to global by its users.
struct Chain {
  const OpNode* mma = nullptr;
  const ValueNode* a_glob = nullptr;
  const ValueNode* b_glob = nullptr;
  const ValueNode* c_glob = nullptr;  // mma_acc only
  std::vector<const OpNode*> folded;  // the TMA/LSU ops and stores it absorbs
  std::vector<const OpNode*> stores;
};

class Lowering {
 public:
  Lowering(const Graph& task, Graph& tile, const TileConfig& cfg)
      : task_(task), tile_(tile), cfg_(cfg) {
    tile::RegisterTileDialect(reg_);
  }

  TileStats Run() {
    const Block* tb = task_.root();
    CHECK(tb) << "task_to_tile: task graph has no root block";
    tile_.config() = task_.config();
    block_ = tile_.MakeRoot(tb->name());
    // Block arguments first, in order (full-shape views of the inputs).
    for (const ValueNode* arg : tb->arguments()) {
      const task::TensorImpl* t = TaskTensor(arg);
      CHECK(t) << "task_to_tile: argument %" << arg->value().name << " is not a task tensor";
      View(arg->value().name, t->shape, t->dtype, {});
    }
    for (const OpNode* op : tb->operations()) {
      Chain c;
      if (MatchChain(op, &c)) {
        chains_[op] = c;
        for (const OpNode* f : c.folded) folded_.insert(f);
      }
    }
    for (const OpNode* op : tb->operations()) {
      if (chains_.count(op)) {
        LowerChain(chains_[op]);
      } else if (!folded_.count(op)) {
        Copy(op);
      }
    }
    std::vector<ValueNode*> outs;
    for (const ValueNode* o : tb->outputs()) {
      auto st = stored_.find(o);
      if (st != stored_.end()) {
        outs.insert(outs.end(), st->second.begin(), st->second.end());
      } else {
        outs.push_back(FullValue(o));
      }
    }
    if (!outs.empty()) block_->SetOutputs(std::move(outs));
    return stats_;
  }

 private:
  // The global source of a staged operand: `v` = tma.gmem_to_smem(g) or
  // lsu.gmem_to_reg(g) with g in global memory and no other reader of v.
  const ValueNode* StagedFrom(const ValueNode* v, const char* op_name,
                              std::vector<const OpNode*>* folded) {
    const OpNode* d = v ? v->def() : nullptr;
    if (!d || d->op().op.name != op_name || d->operands().size() != 1) return nullptr;
    if (v->uses().size() != 1) return nullptr;
    const ValueNode* g = d->operands()[0];
    const task::TensorImpl* t = TaskTensor(g);
    if (!t || t->loc != task::Location::kGlobal || t->shape.size() != 2) return nullptr;
    folded->push_back(d);
    return g;
  }

  bool MatchChain(const OpNode* op, Chain* c) {
    const std::string& n = op->op().op.name;
    const bool acc = n == "tc.mma_acc";
    if (!(n == "tc.mma" || acc)) return false;
    if (op->operands().size() != (acc ? 3u : 2u) || op->results().size() != 1) return false;
    const task::TensorImpl* a = TaskTensor(op->operands()[0]);
    const task::TensorImpl* b = TaskTensor(op->operands()[1]);
    const task::TensorImpl* d = TaskTensor(op->results()[0]);
    if (!a || !b || !d || a->shape.size() != 2 || b->shape.size() != 2 ||
        d->shape.size() != 2 || a->dtype != b->dtype ||
        (a->dtype != Dtype::kBf16 && a->dtype != Dtype::kF16))
      return false;
    Chain ch;
    ch.mma = op;
    ch.a_glob = StagedFrom(op->operands()[0], "tma.gmem_to_smem", &ch.folded);
    ch.b_glob = StagedFrom(op->operands()[1], "tma.gmem_to_smem", &ch.folded);
    if (acc) ch.c_glob = StagedFrom(op->operands()[2], "lsu.gmem_to_reg", &ch.folded);
    if (!ch.a_glob || !ch.b_glob || (acc && !ch.c_glob)) return false;
    const ValueNode* dv = op->results()[0];
    if (dv->uses().empty()) return false;
    for (const ir::Use& u : dv->uses()) {
      if (u.user->op().op.name != "lsu.reg_to_gmem") return false;
      ch.stores.push_back(u.user);
      ch.folded.push_back(u.user);
    }
    *c = std::move(ch);
    return true;
  }

  ValueNode* View(const std::string& name, std::vector<int> shape, Dtype dt,
                  std::vector<int> slice) {
    const std::string key = TileName(name, slice);
    auto it = views_.find(key);
    if (it != views_.end()) return it->second;
    ValueNode* v = block_->AddArgument(
        Value{key, Type{"tensor", "tile"},
              tile::TensorImpl{std::move(shape), {}, dt, tile::Location::kGlobal,
                               std::move(slice)}});
    views_[key] = v;
    return v;
  }

  ValueNode* Emit(const std::string& op_name, AnyOf<OperationImpl> impl,
                  std::vector<ValueNode*> ins, std::string name, std::vector<int> shape,
                  Dtype dt, tile::Location loc, std::vector<int> slice) {
    auto op = reg_.GetOperator("tile." + op_name);
    CHECK(op) << "task_to_tile: tile op '" << op_name << "' is not registered";
    Value out{std::move(name), Type{"tensor", "tile"},
              tile::TensorImpl{std::move(shape), {}, dt, loc, std::move(slice)}};
    OpNode* node = block_->MakeOperation(ir::Operation{*op, std::move(impl)},
                                         std::move(ins), {std::move(out)});
    return node->results()[0];
  }

  // Tile sizes of the one-SM GEMM (kvm_sm100_gemm_bf16): 128 x 256 tiles
  // when those alone fill the SMs, else 128 x 128; a product narrower than
  // 128 columns (the router's 64 experts, a GEMV) takes N rounded up to 16.
  int TileN(int M, int N) const {
    if (N < 128) return (N + 15) & ~15;
    return static_cast<long long>(CeilDiv(M, kTileM)) * CeilDiv(N, 256) >= cfg_.sm_count
               ? 256
               : 128;
  }

  void LowerChain(const Chain& c) {
    const task::TensorImpl* a = TaskTensor(c.mma->operands()[0]);
    const task::TensorImpl* b = TaskTensor(c.mma->operands()[1]);
    const task::TensorImpl* d = TaskTensor(c.mma->results()[0]);
    const int M = a->shape[0], K = a->shape[1], N = b->shape[1];
    const int BN = TileN(M, N);
    const std::string& an = c.a_glob->value().name;
    const std::string& bn = c.b_glob->value().name;
    const std::string dn = c.mma->results()[0]->value().name;
    const int mt = CeilDiv(M, kTileM), nt = CeilDiv(N, BN), kt = CeilDiv(K, kTileK);
    std::vector<ValueNode*> dtiles;
    for (int mi = 0; mi < mt; ++mi)
      for (int ni = 0; ni < nt; ++ni) {
        const std::vector<int> dslice{mi * kTileM, ni * BN};
        ValueNode* acc = nullptr;
        if (c.c_glob) {
          const task::TensorImpl* ct = TaskTensor(c.c_glob);
          ValueNode* cv = View(c.c_glob->value().name, {kTileM, BN}, ct->dtype, dslice);
          acc = Emit("lsu.gmem_to_reg", {}, {cv}, TileName(c.c_glob->value().name + "_reg", dslice),
                     {kTileM, BN}, ct->dtype, tile::Location::kRegister, dslice);
          ++stats_.loads;
        }
        for (int kk = 0; kk < kt; ++kk) {
          const std::vector<int> as{mi * kTileM, kk * kTileK}, bs{kk * kTileK, ni * BN};
          ValueNode* av = View(an, {kTileM, kTileK}, a->dtype, as);
          ValueNode* bv = View(bn, {kTileK, BN}, b->dtype, bs);
          // one staged copy per use (each output tile stages its own operands)
          const std::string use = "_for_" + std::to_string(mi) + "_" + std::to_string(ni);
          ValueNode* at = Emit("tma.gmem_to_smem", {}, {av}, TileName(an + "_smem", as) + use,
                               {kTileM, kTileK}, a->dtype, tile::Location::kShared, as);
          ValueNode* bt = Emit("tma.gmem_to_smem", {}, {bv}, TileName(bn + "_smem", bs) + use,
                               {kTileK, BN}, b->dtype, tile::Location::kShared, bs);
          const std::string dname = TileName(dn, dslice) + "_k" + std::to_string(kk);
          stats_.loads += 2;
          if (!acc) {
            acc = Emit("tc.mma", tile::MmaOp{kTileM, BN, kTileK}, {at, bt}, dname,
                       {kTileM, BN}, d->dtype, tile::Location::kRegister, dslice);
          } else {
            acc = Emit("tc.mma_acc", tile::MmaAccOp{kTileM, BN, kTileK}, {at, bt, acc}, dname,
                       {kTileM, BN}, d->dtype, tile::Location::kRegister, dslice);
          }
          ++stats_.mma;
        }
        dtiles.push_back(acc);
      }
    for (const OpNode* st : c.stores) {
      const ValueNode* sv = st->results()[0];
      const task::TensorImpl* so = TaskTensor(sv);
      std::vector<ValueNode*>& out = stored_[sv];
      for (int mi = 0, i = 0; mi < mt; ++mi)
        for (int ni = 0; ni < nt; ++ni, ++i) {
          const std::vector<int> dslice{mi * kTileM, ni * BN};
          out.push_back(Emit("lsu.reg_to_gmem", {}, {dtiles[i]}, TileName(sv->value().name, dslice),
                             {kTileM, BN}, so->dtype, tile::Location::kGlobal, dslice));
          ++stats_.stores;
        }
    }
    stats_.tiled.push_back(dn + ": [" + std::to_string(M) + "," + std::to_string(K) +
                           "]x[" + std::to_string(K) + "," + std::to_string(N) + "] -> " +
                           std::to_string(mt * nt) + " tiles of 128x" + std::to_string(BN) +
                           ", " + std::to_string(mt * nt * kt) + " mma (k=16)");
  }

  // Full-shape tile value standing for task value v.
  ValueNode* FullValue(const ValueNode* v) {
    auto it = copied_.find(v);
    if (it != copied_.end()) return it->second;
    const task::TensorImpl* t = TaskTensor(v);
    CHECK(t) << "task_to_tile: %" << v->value().name << " is not a task tensor";
    // A global tensor (argument or stored result): its full-shape view.
    return View(v->value().name, t->shape, t->dtype, {});
  }

  void Copy(const OpNode* op) {
    std::vector<ValueNode*> ins;
    for (const ValueNode* v : op->operands()) ins.push_back(FullValue(v));
    CHECK_EQ(op->results().size(), 1u) << "task_to_tile: multi-result task op";
    const ValueNode* r = op->results()[0];
    const task::TensorImpl* t = TaskTensor(r);
    CHECK(t) << "task_to_tile: result of " << op->op().op.name << " is not a task tensor";
    ValueNode* out = Emit(op->op().op.name, op->op().impl, std::move(ins), r->value().name,
                          t->shape, t->dtype, TileLoc(t->loc), {});
    copied_[r] = out;
    ++stats_.copied;
  }

  const Graph& task_;
  Graph& tile_;
  TileConfig cfg_;
  ir::serial::Registry reg_;
  Block* block_ = nullptr;
  TileStats stats_;
  std::map<std::string, ValueNode*> views_;
  std::unordered_map<const ValueNode*, ValueNode*> copied_;
  std::unordered_map<const ValueNode*, std::vector<ValueNode*>> stored_;
  std::unordered_map<const OpNode*, Chain> chains_;
  std::unordered_set<const OpNode*> folded_;
};

const tile::TensorImpl* TileTensor(const ValueNode* v) {
  return v ? v->value().impl.as<tile::TensorImpl>() : nullptr;
}

// The executor's broadcasting (graph_ops.cu): an input is aligned with the
// output's trailing dims (numpy rule: each dim equal or 1) or, failing
// that, with its leading dims.
bool Broadcasts(const std::vector<int>& in, const std::vector<int>& out) {
  if (in == out) return true;
  if (in.size() > out.size()) return false;
  const std::size_t off = out.size() - in.size();
  bool trailing = true, leading = true;
  for (std::size_t i = 0; i < in.size(); ++i) {
    trailing = trailing && (in[i] == out[off + i] || in[i] == 1);
    leading = leading && (in[i] == out[i] || in[i] == 1);
  }
  return trailing || leading;
}

ir::VerifyResult VerifyMma(const OpNode* op, bool acc) {
  const std::string& name = op->op().op.name;
  int im = 0, in = 0, ik = 0;
  if (acc) {
    const tile::MmaAccOp* mm = op->op().impl.as<tile::MmaAccOp>();
    if (!mm) return ir::VerifyResult::Fail(name + ": missing MmaAccOp impl");
    im = mm->m; in = mm->n; ik = mm->k;
  } else {
    const tile::MmaOp* mm = op->op().impl.as<tile::MmaOp>();
    if (!mm) return ir::VerifyResult::Fail(name + ": missing MmaOp impl");
    im = mm->m; in = mm->n; ik = mm->k;
  }
  const std::size_t nin = acc ? 3 : 2;
  if (op->operands().size() != nin || op->results().size() != 1)
    return ir::VerifyResult::Fail(name + ": wrong operand/result count");
  const tile::TensorImpl* a = TileTensor(op->operands()[0]);
  const tile::TensorImpl* b = TileTensor(op->operands()[1]);
  const tile::TensorImpl* d = TileTensor(op->results()[0]);
  if (!a || !b || !d) return ir::VerifyResult::Fail(name + ": operand not a tile.tensor");
  if (a->shape.size() != 2 || b->shape.size() != 2 || d->shape.size() != 2)
    return ir::VerifyResult::Fail(name + ": operands must be 2-D");
  const int m = a->shape[0], k = a->shape[1], n = b->shape[1];
  if (b->shape[0] != k) return ir::VerifyResult::Fail(name + ": A.k != B.k");
  if (d->shape[0] != m || d->shape[1] != n)
    return ir::VerifyResult::Fail(name + ": D shape != [m,n]");
  if (m != im || n != in || k != ik)
    return ir::VerifyResult::Fail(name + ": operand shape != op (m,n,k)");
  if (b->loc != tile::Location::kShared)
    return ir::VerifyResult::Fail(name + ": B must be in shared");
  if (a->loc == tile::Location::kGlobal)
    return ir::VerifyResult::Fail(name + ": A must be in shared or the accumulator memory");
  // On sm_100a the accumulator lives in TMEM; the dialect calls it register.
  if (d->loc != tile::Location::kRegister)
    return ir::VerifyResult::Fail(name + ": D must be in register (TMEM)");
  if (acc) {
    const tile::TensorImpl* c = TileTensor(op->operands()[2]);
    if (!c || c->shape != d->shape || c->loc != tile::Location::kRegister)
      return ir::VerifyResult::Fail(name + ": C must match D in register");
  }
  if (a->dtype != b->dtype)
    return ir::VerifyResult::Fail(name + ": A and B must have one dtype");
  if (!LegalMmaTile(m, n, k, a->dtype, d->dtype))
    return ir::VerifyResult::Fail(name + ": (m=" + std::to_string(m) + ", n=" +
                                  std::to_string(n) + ", k=" + std::to_string(k) +
                                  ") is not a tcgen05 kind::f16 tile");
  return ir::VerifyResult::Ok();
}

}  // namespace

bool LegalMmaTile(int m, int n, int k, Dtype ab, Dtype d) {
  if (ab != Dtype::kBf16 && ab != Dtype::kF16) return false;
  if (d != Dtype::kF32 && d != Dtype::kF16 && d != Dtype::kBf16) return false;
  if (k != 16) return false;
  if (m == 64) return n % 8 == 0 && n >= 8 && n <= 256;
  if (m == 128 || m == 256) return n % 16 == 0 && n >= 16 && n <= 256;
  return false;
}

TileStats TransformTaskToTile(const Graph& task, Graph& tile, const TileConfig& cfg) {
  Lowering l(task, tile, cfg);
  return l.Run();
}

ir::VerifyResult VerifyTileOp(const OpNode* op) {
  const std::string& n = op->op().op.name;
  if (n == "tc.mma") return VerifyMma(op, false);
  if (n == "tc.mma_acc") return VerifyMma(op, true);
  if (n.rfind("comm.", 0) == 0 || n.rfind("warp.", 0) == 0) {
    if (op->operands().size() != op->op().op.inputs.size() ||
        op->results().size() != op->op().op.outputs.size())
      return ir::VerifyResult::Fail(n + ": wrong operand/result count");
    return ir::VerifyResult::Ok();
  }
  const bool elementwise = n.rfind("alu.", 0) == 0 || n.rfind("sfu.", 0) == 0;
  if (elementwise) {
    if (op->results().size() != 1 || op->operands().size() != op->op().op.inputs.size())
      return ir::VerifyResult::Fail(n + ": wrong operand/result count");
    const tile::TensorImpl* o = TileTensor(op->results()[0]);
    if (!o) return ir::VerifyResult::Fail(n + ": output not a tile.tensor");
    bool same = true;
    for (const ValueNode* v : op->operands()) {
      const tile::TensorImpl* t = TileTensor(v);
      if (!t) return ir::VerifyResult::Fail(n + ": input not a tile.tensor");
      if (!Broadcasts(t->shape, o->shape))
        return ir::VerifyResult::Fail(n + ": input shape neither the output's nor a "
                                          "leading/trailing block of it");
      same = same && t->shape == o->shape;
    }
    if (!same) return ir::VerifyResult::Ok();  // broadcast: the reference rule needs equal shapes
  }
  if (elementwise || n.rfind("tma.", 0) == 0 || n.rfind("lsu.", 0) == 0)
    return ir::tile::Verify(op);
  return ir::VerifyResult::Fail("tile op '" + n + "' has no sm_100a rule");
}

}  // namespace kvm::sm100
