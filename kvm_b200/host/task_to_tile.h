// Task -> tile lowering for the sm_100a target, and the device-side checker
// of tile ops (the legal-tile table the reference's tile verifier leaves as
// CHECK(false), src/ir/dialect/tile/verify.cpp:124-126).
//
// The tile graph (src/ir/dialect/tile/) is the task graph refined to
// hardware-sized pieces: every tensor-core chain of the task graph
// (tma.gmem_to_smem A, B [+ lsu.gmem_to_reg C] -> tc.mma[_acc] ->
// lsu.reg_to_gmem) becomes one tile.tc.mma / tile.tc.mma_acc per tcgen05
// instruction the sm_100a GEMM issues (M = 128 rows, N = 128 or 256 columns
// by the same rule as kvm_sm100_gemm_bf16, K = 16), with the TMA loads of
// its A and B slices and the store of each output tile. Values carry the
// dialect's slice (origin of the block in its task tensor); global tiles
// are block arguments named "<task tensor>_at_<row>_<col>", so tensor + slice
// give the dependencies, as the dialect intends (tile/values.h). Task ops
// outside tensor-core chains are copied at full shape (tile.<same op>).
#pragma once

#include <string>
#include <vector>

#include "dialect/dtype.h"
#include "graph.h"
#include "node.h"
#include "verify_result.h"

namespace kvm::sm100 {

struct TileConfig {
  int sm_count = 148;  // SMs of the device the tile sizes are chosen for
};

struct TileStats {
  int mma = 0;          // tile.tc.mma + tile.tc.mma_acc
  int loads = 0;        // tile.tma.gmem_to_smem + tile.lsu.gmem_to_reg of tiles
  int stores = 0;       // tile.lsu.reg_to_gmem of output tiles
  int copied = 0;       // task ops copied at full shape
  std::vector<std::string> tiled;  // one line per tiled product
};

// The tcgen05.mma shapes of kind::f16 (A and B both bf16 or both f16, D
// fp32 or f16) that this target issues or accepts:
//   M = 64 (one SM):  N % 8 == 0,  8 <= N <= 256
//   M = 128 (one SM): N % 16 == 0, 16 <= N <= 256
//   M = 256 (an SM pair, cta_group::2): N % 16 == 0, 16 <= N <= 256
//   K = 16.
bool LegalMmaTile(int m, int n, int k, ir::dialect::Dtype ab, ir::dialect::Dtype d);

// Lower `task` (from TransformKernelToTask) into `tile` (empty graph).
TileStats TransformTaskToTile(const ir::Graph& task, ir::Graph& tile,
                              const TileConfig& cfg = {});

// Legality of one tile op on sm_100a: the structural rules of
// ir::tile::Verify (arity, locations, shape relations), the tcgen05 shape
// table for tc.mma / tc.mma_acc, broadcasting elementwise operands (a
// leading or trailing dimension of the output), and arity for the
// collective and warp ops the reference verifier does not cover yet.
ir::VerifyResult VerifyTileOp(const ir::OpNode* op);

}  // namespace kvm::sm100
