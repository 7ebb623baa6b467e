// kvm_run: execute a .kvm kernel-dialect graph on one B200.
//
//   kvm_run GRAPH.kvm [--inputs DIR] [--out DIR] [--seed S] [--warmup W]
//                     [--iters N] [--dump-task] [--lower-only]
//                     [--tile [--dump-tile]]
//                     [--rank R --world N --comm-dir DIR]
//   kvm_run --verify-tile TILE_GRAPH.kvm
//
// The graph is parsed by the reference parser (serial::Parse), lowered by the
// reference transform with the sm_100a Device target, and executed by the
// Executor. Inputs: DIR/<arg>.bin (raw bytes of the declared dtype) when
// given, else the argument's attrs -- {fill = v} for a constant,
// {std = s} (and {mean = m}) for seeded normal values -- else N(0, 1) from
// seed S + argument index. Outputs are written to DIR/<name>.bin; a JSON
// summary (launch plan, time per run, output checksums) goes to stdout.
// --tile lowers the task graph further to the tile dialect (task_to_tile.h)
// and checks every tile op against the sm_100a rules (no GPU needed);
// --verify-tile checks a tile-dialect graph given as text.
// --rank/--world run one rank of an N-process job (one process per GPU,
// GPU R): rank 0 writes the NCCL unique id to DIR/nccl_id (the others wait
// for it, 60 s at most; DIR starts empty), the graph's comm.* ops run over NCCL, inputs come
// from <inputs>/r<R>/ and outputs go to <out>/r<R>/, and seeded inputs
// use seed S + 1000003 R + argument index ({replicated = true} arguments, such
// as expert weights, use seed S + argument index on every rank).
#include <cuda_runtime.h>

#include <any>
#include <chrono>
#include <cstdio>
#include <thread>
#include <cstring>
#include <fstream>
#include <iostream>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "dialect/kernel/dialect.h"
#include "dialect/task/dialect.h"
#include "dialect/tile/dialect.h"
#include "dialect/tile/ops.h"
#include "executor.h"
#include "kvm_sm100.h"
#include "task_to_tile.h"
#include "serialization/parser.h"
#include "serialization/registry.h"
#include "serialization/serializer.h"

namespace {

std::string ReadFile(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot read " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

bool ReadBin(const std::string& path, std::vector<char>& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  out.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

double AttrNumber(const kvm::ir::AttrMap& attrs, const kvm::ir::ValueNode* v,
                  const char* key, bool* found) {
  const std::any* a = attrs.Get(v, key);
  *found = a != nullptr;
  if (!a) return 0;
  if (const auto* d = std::any_cast<double>(a)) return *d;
  if (const auto* i = std::any_cast<std::int64_t>(a)) return double(*i);
  *found = false;
  return 0;
}

// Order-independent checksum: sum and sum of squares of the values as fp64.
void Checksum(const kvm::sm100::Buffer& b, double* sum, double* sq) {
  std::vector<char> host(b.bytes());
  cudaMemcpy(host.data(), b.ptr, host.size(), cudaMemcpyDeviceToHost);
  *sum = *sq = 0;
  const int64_t n = b.numel();
  for (int64_t i = 0; i < n; ++i) {
    double v = 0;
    switch (b.dtype) {
      case kvm::ir::dialect::Dtype::kBf16: {
        uint32_t u = uint32_t(reinterpret_cast<uint16_t*>(host.data())[i]) << 16;
        float f;
        std::memcpy(&f, &u, 4);
        v = f;
        break;
      }
      case kvm::ir::dialect::Dtype::kF32:
        v = reinterpret_cast<float*>(host.data())[i];
        break;
      case kvm::ir::dialect::Dtype::kI32:
        v = reinterpret_cast<int32_t*>(host.data())[i];
        break;
      default:
        v = 0;
    }
    *sum += v;
    *sq += v * v;
  }
}

// One rank joins an N-rank job on GPU `rank`: rank 0 makes the NCCL id and
// publishes it by rename (readers never see a partial file).
kvm_comm* JoinWorld(int rank, int world, const std::string& dir) {
  int devices = 0;
  cudaGetDeviceCount(&devices);
  if (devices <= 0) throw std::runtime_error("no CUDA device");
  cudaSetDevice(rank % devices);
  std::vector<char> id(KVM_COMM_ID_BYTES);
  const std::string path = dir + "/nccl_id";
  if (rank == 0) {
    if (kvm_sm100_comm_unique_id(id.data()) != KVM_OK)
      throw std::runtime_error(std::string("comm id: ") + kvm_sm100_last_error());
    const std::string tmp = path + ".tmp";
    {
      std::ofstream f(tmp, std::ios::binary);
      f.write(id.data(), std::streamsize(id.size()));
    }
    if (std::rename(tmp.c_str(), path.c_str()) != 0)
      throw std::runtime_error("cannot publish " + path);
  } else {
    std::vector<char> data;
    for (int waited = 0; !ReadBin(path, data) || data.size() != id.size(); waited += 10) {
      if (waited > 60000) throw std::runtime_error("rank 0 did not publish " + path);
      std::this_thread::sleep_for(std::chrono::milliseconds(10));
    }
    id = data;
  }
  kvm_comm* c = nullptr;
  if (kvm_sm100_comm_init(world, rank, id.data(), &c) != KVM_OK)
    throw std::runtime_error(std::string("comm init: ") + kvm_sm100_last_error());
  return c;
}

}  // namespace

int main(int argc, char** argv) {
  std::string graph_path, in_dir, out_dir;
  uint64_t seed = 0;
  int warmup = 1, iters = 1;
  bool dump_task = false, lower_only = false, tile = false, dump_tile = false;
  std::string verify_tile, comm_dir;
  int rank = 0, world = 1;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + a);
      return argv[++i];
    };
    if (a == "--inputs") in_dir = next();
    else if (a == "--out") out_dir = next();
    else if (a == "--seed") seed = std::stoull(next());
    else if (a == "--warmup") warmup = std::stoi(next());
    else if (a == "--iters") iters = std::stoi(next());
    else if (a == "--dump-task") dump_task = true;
    else if (a == "--lower-only") lower_only = true;
    else if (a == "--tile") tile = true;
    else if (a == "--dump-tile") dump_tile = true;
    else if (a == "--verify-tile") verify_tile = next();
    else if (a == "--rank") rank = std::stoi(next());
    else if (a == "--world") world = std::stoi(next());
    else if (a == "--comm-dir") comm_dir = next();
    else if (graph_path.empty()) graph_path = a;
    else throw std::runtime_error("unexpected argument " + a);
  }
  if (!verify_tile.empty()) {
    try {
      kvm::ir::serial::Registry reg;
      kvm::ir::tile::RegisterTileDialect(reg);
      kvm::ir::Graph g;
      kvm::ir::serial::Parse(ReadFile(verify_tile), reg, g);
      int ops = 0, bad = 0;
      std::string first;
      for (const kvm::ir::OpNode* op : g.root()->operations()) {
        ++ops;
        kvm::ir::VerifyResult r = kvm::sm100::VerifyTileOp(op);
        if (!r.ok && bad++ == 0) first = r.error;
      }
      std::cout << "{\"tile_ops\": " << ops << ", \"illegal\": " << bad
                << ", \"first_error\": \"" << first << "\"}" << std::endl;
      return bad ? 3 : 0;
    } catch (const std::exception& e) {
      std::cerr << "kvm_run: " << e.what() << std::endl;
      return 1;
    }
  }
  if (graph_path.empty()) {
    std::cerr << "usage: kvm_run GRAPH.kvm [--inputs DIR] [--out DIR] [--seed S]"
                 " [--warmup W] [--iters N] [--dump-task]\n";
    return 2;
  }
  try {
    kvm::ir::serial::Registry reg;
    kvm::ir::kernel::RegisterKernelDialect(reg);
    kvm::ir::Graph kernel;
    kvm::ir::AttrMap attrs = kvm::ir::serial::Parse(ReadFile(graph_path), reg, kernel);
    kvm_comm* comm = nullptr;
    if (world > 1 && !tile && !lower_only) {
      if (rank < 0 || rank >= world) throw std::runtime_error("--rank outside --world");
      if (comm_dir.empty()) throw std::runtime_error("--world > 1 needs --comm-dir");
      comm = JoinWorld(rank, world, comm_dir);  // selects GPU `rank` first
    }
    // The executor holds peer memory of the other ranks (expert-parallel
    // graphs) and releases it collectively, so it goes before the communicator.
    auto exec = std::make_unique<kvm::sm100::Executor>(kernel, attrs);
    kvm::sm100::Executor& ex = *exec;
    uint64_t rank_seed = seed;
    if (comm) {
      ex.SetComm(comm);
      if (!in_dir.empty()) in_dir += "/r" + std::to_string(rank);
      if (!out_dir.empty()) out_dir += "/r" + std::to_string(rank);
      rank_seed += 1000003ull * uint64_t(rank);
    }
    if (dump_task) {
      kvm::ir::serial::Registry treg;
      kvm::ir::task::RegisterTaskDialect(treg);
      std::cerr << kvm::ir::serial::Serialize(ex.task_graph(), treg);
    }
    if (tile) {  // task graph -> tile graph + sm_100a checks: no GPU needed
      kvm::ir::Graph tg;
      kvm::sm100::TileStats st = kvm::sm100::TransformTaskToTile(ex.task_graph(), tg);
      int ops = 0, bad = 0, dynamic = 0;
      std::string first;
      for (const kvm::ir::OpNode* op : tg.root()->operations()) {
        ++ops;
        // Products over routed rows (3-D expert weights) keep their task
        // shape: their tiles depend on the routing and are chosen on the GPU.
        if (op->op().op.name.rfind("tc.", 0) == 0 &&
            !op->op().impl.as<kvm::ir::tile::MmaOp>() &&
            !op->op().impl.as<kvm::ir::tile::MmaAccOp>()) {
          ++dynamic;
          continue;
        }
        kvm::ir::VerifyResult r = kvm::sm100::VerifyTileOp(op);
        if (!r.ok && bad++ == 0) first = r.error;
      }
      if (dump_tile) {
        kvm::ir::serial::Registry treg;
        kvm::ir::tile::RegisterTileDialect(treg);
        std::cerr << kvm::ir::serial::Serialize(tg, treg);
      }
      std::cout << "{\"graph\": \"" << graph_path << "\", \"tile_ops\": " << ops
                << ", \"mma\": " << st.mma << ", \"loads\": " << st.loads
                << ", \"stores\": " << st.stores << ", \"copied\": " << st.copied
                << ", \"dynamic_mma\": " << dynamic
                << ", \"arguments\": " << tg.root()->arguments().size()
                << ", \"illegal\": " << bad << ", \"first_error\": \"" << first
                << "\", \"tiled\": [";
      for (std::size_t i = 0; i < st.tiled.size(); ++i)
        std::cout << (i ? ", " : "") << "\"" << st.tiled[i] << "\"";
      std::cout << "]}" << std::endl;
      return bad ? 3 : 0;
    }
    if (lower_only) {  // parse + lower + fusion analysis only: no GPU needed
      ex.Plan();
      std::cout << "{\"graph\": \"" << graph_path << "\", \"task_ops\": "
                << ex.task_graph().root()->operations().size() << ", \"fusions\": [";
      for (std::size_t i = 0; i < ex.fusions().size(); ++i)
        std::cout << (i ? ", " : "") << "\"" << ex.fusions()[i] << "\"";
      std::cout << "]}" << std::endl;
      return 0;
    }
    ex.Prepare();
    const auto& args = kernel.root()->arguments();
    for (std::size_t i = 0; i < ex.inputs().size(); ++i) {
      const std::string& name = ex.input_names()[i];
      std::vector<char> data;
      bool f_fill = false, f_std = false, f_mean = false, f_rep = false;
      const double fill = AttrNumber(attrs, args[i], "fill", &f_fill);
      const double sd = AttrNumber(attrs, args[i], "std", &f_std);
      const double mean = AttrNumber(attrs, args[i], "mean", &f_mean);
      const std::any* rep = attrs.Get(args[i], "replicated");
      if (rep)
        if (const bool* b = std::any_cast<bool>(rep)) f_rep = *b;
      if (!in_dir.empty() && ReadBin(in_dir + "/" + name + ".bin", data))
        ex.CopyInput(int(i), data.data(), int64_t(data.size()));
      else if (f_fill)
        ex.FillInputConst(int(i), float(fill));
      else  // {replicated = true}: the same values on every rank (e.g. weights)
        ex.FillInputNormal(int(i), (f_rep ? seed : rank_seed) + i, float(mean),
                           f_std ? float(sd) : 1.0f);
    }
    cudaStream_t st;
    cudaStreamCreate(&st);
    for (int w = 0; w < warmup; ++w)
      if (int rc = ex.Run(st); rc != KVM_OK)
        throw std::runtime_error(std::string("run: ") + kvm_sm100_last_error());
    int status = 0;
    if (kvm_sm100_device_status(&status, 1) != KVM_OK)
      throw std::runtime_error(std::string("device: ") + kvm_sm100_last_error());
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    for (int it = 0; it < iters; ++it)
      if (int rc = ex.Run(st); rc != KVM_OK)
        throw std::runtime_error(std::string("run: ") + kvm_sm100_last_error());
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (kvm_sm100_device_status(&status, 1) != KVM_OK)
      throw std::runtime_error(std::string("device: ") + kvm_sm100_last_error());

    std::ostringstream js;
    js << "{\"graph\": \"" << graph_path << "\", \"launch_steps\": "
       << ex.launches_per_run() << ", \"ms_per_run\": " << (iters ? ms / iters : 0)
       << ", \"iters\": " << iters << ", \"steps\": [";
    for (std::size_t i = 0; i < ex.step_names().size(); ++i)
      js << (i ? ", " : "") << "\"" << ex.step_names()[i] << "\"";
    js << "], \"fusions\": [";
    for (std::size_t i = 0; i < ex.fusions().size(); ++i)
      js << (i ? ", " : "") << "\"" << ex.fusions()[i] << "\"";
    js << "], \"outputs\": [";
    const auto& outs = kernel.root()->outputs();
    for (std::size_t i = 0; i < ex.outputs().size(); ++i) {
      const auto& b = ex.outputs()[i];
      const std::string name = outs[i]->value().name;
      double sum, sq;
      Checksum(b, &sum, &sq);
      js << (i ? ", " : "") << "{\"name\": \"" << name << "\", \"numel\": " << b.numel()
         << ", \"dtype\": \"" << kvm::ir::dialect::DtypeName(b.dtype)
         << "\", \"sum\": " << sum << ", \"sumsq\": " << sq << "}";
      if (!out_dir.empty()) {
        std::vector<char> host(b.bytes());
        cudaMemcpy(host.data(), b.ptr, host.size(), cudaMemcpyDeviceToHost);
        std::ofstream f(out_dir + "/" + name + ".bin", std::ios::binary);
        f.write(host.data(), std::streamsize(host.size()));
      }
    }
    js << "]}";
    std::cout << js.str() << std::endl;
    cudaStreamDestroy(st);
    exec.reset();
    if (comm) kvm_sm100_comm_destroy(comm);
  } catch (const std::exception& e) {
    std::cerr << "kvm_run: " << e.what() << std::endl;
    return 1;
  }
  return 0;
}
