// Layout of the per-rank workspace of the overlapped expert-parallel layer
// (kvm_sm100_ep_prepare / _dispatch_gate_up / _down_push), shared by the
// translation units that read or write it. Every part starts on 256 bytes.
//
//   seg_ctr    [E]        rows stored so far per (local expert, peer) segment
//   done_ctr   [1]        CTAs of the down GEMM that have finished
//   seg_prefix [E + 1]    row prefix of this rank's remote segments, ordered
//                         (local expert, peer) -- segment sg = le * (P-1) + i
//                         goes to rank (me + 1 + i) mod P
//   tile_first [E]        per local expert, the token tile of the fused
//                         gate/up GEMM that holds this rank's own rows (the
//                         tile order starts there; see gemm_pair.cuh)
//   push_row   [cap_rows] for each received row: (source rank << 28) | the
//                         row's index in that rank's permuted order
#pragma once

#include <cstdint>

namespace kvm {

struct EpWorkspace {
  int* seg_ctr;
  int* done_ctr;
  int* seg_prefix;
  int* tile_first;
  int* push_row;
};

inline int64_t ep_ws_align(int64_t b) { return (b + 255) & ~int64_t(255); }

inline int64_t ep_workspace_bytes(int E, int64_t cap_rows) {
  return ep_ws_align(4ll * E) + ep_ws_align(16) + ep_ws_align(4ll * (E + 1)) +
         ep_ws_align(4ll * E) + ep_ws_align(4 * cap_rows);
}

inline EpWorkspace ep_workspace(void* base, int E, int64_t cap_rows) {
  (void)cap_rows;
  char* p = static_cast<char*>(base);
  EpWorkspace w;
  w.seg_ctr = reinterpret_cast<int*>(p);
  p += ep_ws_align(4ll * E);
  w.done_ctr = reinterpret_cast<int*>(p);
  p += ep_ws_align(16);
  w.seg_prefix = reinterpret_cast<int*>(p);
  p += ep_ws_align(4ll * (E + 1));
  w.tile_first = reinterpret_cast<int*>(p);
  p += ep_ws_align(4ll * E);
  w.push_row = reinterpret_cast<int*>(p);
  return w;
}

// Flag words per rank: counts [P], data [P], outputs [P], then one per
// (local expert, source rank): 3 * P + (E / P) * P in all.
inline int64_t ep_flag_words(int E, int P) { return 3ll * P + static_cast<int64_t>(E / P) * P; }

}  // namespace kvm
