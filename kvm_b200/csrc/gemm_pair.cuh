// Grouped bf16 GEMM on SM pairs (tcgen05.mma.cta_group::2), weights as the
// MMA's M operand and tokens as its N operand.
//
//   D[r, c] = sum_k X[r, k] * W[g*N + c, k]        rows r of group g
//
// One pair tile = 256 weight rows (128 per CTA) x TN tokens (TN/2 per CTA,
// TN a multiple of 16, <= 256). The token count of a group fixes TN: a group
// of c tokens is cut into ceil(c/256) tiles of near-equal width, so a group
// of 270 tokens runs as 2 x 144 columns instead of 3 x 128 rows with the
// third almost empty. Each CTA stages 16 KB of weights and at most 16 KB of
// tokens per K block, half the operand bytes per FLOP of a one-SM 128 x 256
// tile.
//
//   warp 0 (one lane)  TMA producer of each CTA; loads count on the even
//                      CTA's full barrier
//   warp 1 (one lane)  MMA issuer (even CTA only); commits release the
//                      stages and publish the accumulator in both CTAs
//   warps 2..9         epilogue, two sets of four warps taking alternate
//                      32-token chunks: TMEM lane = output column, TMEM
//                      column = token; a warp stores 32 columns x 32 tokens
//                      per chunk (64 contiguous bytes per token)
//
// A CTA's TN/2 token rows load as a single box (128, 64, 32, 16 or 8 rows,
// the smallest that covers them): one TMA request per operand per K block.
// Splitting them into exact boxes (64 + 8 for 72 rows) costs more TMA time
// than the extra rows, and L2 prefetch of the weights ahead of the TMA loads
// (bulk tensor prefetch or prefetch.global.L2 from a spare warp) made the
// weight stream slower, not faster, on B200. So did "wide" tiles of up to
// 512 tokens (two MMAs per K block sharing one weight stage, the second
// group of tokens in a second stage): they halve the weight bytes in flight
// per SM, and the weight stream from HBM is what bounds this kernel (a group
// of 512 tokens: 663 us as one wide tile vs 587 us as two narrow tiles whose
// second weight read hits L2).
//
// Epilogues: plain (bf16 D [+ C]) and SiLU-gate. For SiLU-gate the weight
// rows come from pack_gate_up (64-row blocks: gate f0..f0+63, then up
// f0..f0+63), so TMEM lanes 0-63 of a CTA hold gate and lanes 64-127 up for
// the same 64 f: the up warps hand their values to the gate warps through
// shared memory (mbarrier handshake, bounded waits) and the gate warps write
// H[r, f] = bf16(SiLU(g) * u).
#pragma once

#include <cuda_bf16.h>

#include "gemm_bf16.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace kvm {

constexpr int kPairEpiWarps = 8;  // two sets of four (one per TMEM lane quarter)
constexpr int kPairThreads = 32 * (2 + kPairEpiWarps);
constexpr int kPairStages = 6;
constexpr int kPairBK = 64;
constexpr int kPairMaxTN = 256;
constexpr uint32_t kPairABytes = 128 * kPairBK * 2;  // 128 weight rows
constexpr uint32_t kPairBBytes = 128 * kPairBK * 2;  // <= 128 token rows
constexpr uint32_t kPairStageBytes = kPairABytes + kPairBBytes;
constexpr uint32_t kPairTmemCols = 2 * kPairMaxTN;   // two accumulators
constexpr uint32_t kPairUBytes = 2 * 32 * 64 * 4;    // SiLU hand-off, 1 per set

// Token tensor maps: boxes of 128, 64, 32, 16 and 8 rows.
struct PairMaps {
  CUtensorMap w;
  CUtensorMap x[5];
};

struct PairParams {
  int rows;              // token rows of X (all groups)
  int N;                 // weight rows (output columns) per group
  int K;
  int num_groups;
  const int* offsets;    // [num_groups + 1] token-row offsets, or null (dense)
  void* D;               // bf16
  long long ldd;
  const void* C;         // optional bf16 addend (plain epilogue), stride ldc
  long long ldc;
  int* status;
};

// Expert-parallel forms of the kernel (kEp* below), for the layer whose
// experts are sharded over the GPUs of one node (one process per GPU, peer
// memory mapped between them):
//
// kEpDispatchGateUp -- the dispatch all-to-all fused with the gate/up GEMM.
//   Four extra warps per CTA store this rank's routed token rows into the
//   owners' receive buffers (peer stores), local expert by local expert, and
//   after each (owner, local expert) segment is complete raise that owner's
//   flag for it. The producer of every CTA waits, before the first tile of a
//   group, until every other rank has raised its flag for that group, so the
//   MMAs of expert 0 run while the rows of later experts are still crossing
//   NVLink. Rows a rank routes to its own experts are written before the
//   launch (a stream-ordered kernel), so no CTA waits on another CTA of its
//   own GPU: the only waits are on other GPUs, whose CTAs all stay resident
//   (the grid is the resident pair count).
// kEpDownPush -- the down GEMM fused with the combine all-to-all: the
//   epilogue stores each output row straight into the result rows of the rank
//   that routed the token (peer stores, at the row of its permuted order), and
//   the last CTA to finish raises every rank's outputs flag.
enum PairEpMode : int { kEpNone = 0, kEpDispatchGateUp = 1, kEpDownPush = 2 };

constexpr int kPairDispatchWarps = 4;
constexpr int pair_threads(int ep) {
  return kPairThreads + (ep == kEpDispatchGateUp ? 32 * kPairDispatchWarps : 0);
}

struct PairEp {
  int P, me, epr;                 // ranks, this rank, experts per rank
  unsigned epoch;                 // this call's epoch (flags hold epochs)
  unsigned* flags[8];             // every rank's flag words
  // kEpDispatchGateUp
  const uint4* x;                 // this rank's tokens [T, H]
  int row_vecs;                   // H / 8
  const int* src_token;           // [T*k] token of each permuted row
  const int* offsets;             // [E+1] this rank's per-expert row offsets
  const int* send_base;           // [E] first row in the owner's receive buffer
  const int* seg_prefix;          // [nseg+1] rows of the remote segments
  int nseg;                       // epr * (P - 1): segment sg = (le, k-th peer)
  int* seg_ctr;                   // [nseg] rows stored so far (zero at launch)
  void* recv[8];                  // every rank's receive buffer
  // kEpDownPush
  void* push_base[8];             // every rank's result rows [T*k, H]
  const int* push_row;            // [rows] (source rank << 28) | row there
  const int* tile_first;          // [epr] first token tile of each group
  int* done_ctr;                  // CTAs finished (zero at launch)
};

// Flag words of one rank: [0, P) counts, [P, 2P) data (whole rank),
// [2P, 3P) outputs, then [3P + le*P + src] the per-group data flags.
__device__ __forceinline__ unsigned* ep_group_flag(const PairEp& ep, int owner, int le,
                                                   int src) {
  return ep.flags[owner] + 3 * ep.P + le * ep.P + src;
}

// Bounded wait until the flags for group g of the ranks in `mask` hold this
// epoch (acquire loads), then order the TMA loads that follow after them.
// (Polling them all as relaxed loads followed by one fence.acq_rel.sys was
// measured 27% slower for the whole kernel on 2 GPUs: that fence is costly.)
__device__ __forceinline__ bool ep_wait_sources(const PairEp& ep, int g, unsigned mask,
                                                volatile int* abort) {
  const unsigned* f = ep_group_flag(ep, ep.me, g, 0);
  for (int s = 0; s < ep.P; ++s) {
    if (!((mask >> s) & 1u)) continue;
    if (ld_acquire_sys(f + s) >= ep.epoch) continue;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(f + s) < ep.epoch) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        *abort = 1;
        return false;
      }
      __nanosleep(64);
    }
  }
  fence_proxy_async_global();
  return true;
}

__device__ __forceinline__ void ep_raise_segment(const PairEp& ep, int sg) {
  const int le = sg / (ep.P - 1);
  const int d = (ep.me + 1 + sg % (ep.P - 1)) % ep.P;
  st_release_sys(ep_group_flag(ep, d, le, ep.me), ep.epoch);
}

// The dispatch warps: this rank's rows for other ranks' experts, in the
// order (local expert, owner), cut in chunks of 2 rows dealt round-robin to
// every dispatch warp of the grid. A warp copies a chunk (row by row, each
// lane 16-byte vectors), fences, then credits the rows to their segments; the
// warp that completes a segment raises the owner's flag for it. Small chunks
// keep the rows in flight at any moment (2 x the dispatch warps) to a few
// local experts' worth, so the first experts' rows arrive, and their GEMM
// tiles start, long before the whole exchange is over; the copy rate stays
// bound by NVLink, not by the fences.
__device__ void ep_dispatch_rows(const PairEp& ep, int w, int nw, int lane) {
  if (ep.P < 2) return;
  const int nseg = ep.nseg;
  const int* sp = ep.seg_prefix;
  if (w == 0)
    for (int sg = lane; sg < nseg; sg += 32)
      if (sp[sg + 1] == sp[sg]) ep_raise_segment(ep, sg);
  constexpr int RC = 2;
  const int total = sp[nseg];
  const int n_chunks = (total + RC - 1) / RC;
  const int rv = ep.row_vecs;
  for (int ch = w; ch < n_chunks; ch += nw) {
    const int q0 = ch * RC, q1 = min(total, q0 + RC);
    int lo = 0, hi = nseg - 1;  // segment of q0: largest sg with sp[sg] <= q0
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sp[mid] <= q0) lo = mid; else hi = mid - 1;
    }
    const int sg0 = lo;
    int sg = sg0;
    for (int q = q0; q < q1; ++q) {
      while (q >= sp[sg + 1]) ++sg;
      const int le = sg / (ep.P - 1);
      const int d = (ep.me + 1 + sg % (ep.P - 1)) % ep.P;
      const int e = d * ep.epr + le;
      const int j = q - sp[sg];
      const long long tok = ep.src_token[ep.offsets[e] + j];
      const uint4* src = ep.x + tok * rv;
      uint4* dst = static_cast<uint4*>(ep.recv[d]) +
                   static_cast<long long>(ep.send_base[e] + j) * rv;
      for (int v0 = 0; v0 < rv; v0 += 32 * 8) {
        uint4 buf[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < rv) buf[u] = __ldg(src + v);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int v = v0 + u * 32 + lane;
          if (v < rv) dst[v] = buf[u];
        }
      }
    }
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
      for (int s2 = sg0; s2 <= sg; ++s2) {
        const int n = min(q1, sp[s2 + 1]) - max(q0, sp[s2]);
        if (n <= 0) continue;
        if (atomicAdd(&ep.seg_ctr[s2], n) + n == sp[s2 + 1] - sp[s2]) {
          __threadfence_system();
          ep_raise_segment(ep, s2);
        }
      }
    }
    __syncwarp();
  }
}

constexpr size_t gemm_pair_smem_bytes() {
  return 1024 + static_cast<size_t>(kPairStages) * kPairStageBytes +
         kPairUBytes + (2 * kPairStages + 2 + 2 + 1 + 4) * 8 + 16 +
         5 * (kMaxGroups + 1) * 4;
}

// SiLU(g) = g * sigmoid(g) with the fast reciprocal-based divide; the
// product is rounded to bf16, far coarser than the divide's error.
__device__ __forceinline__ float silu_fast(float g) {
  return __fdividef(g, 1.0f + __expf(-g));
}

struct PairTile {
  int g, mi;
  int r0;      // first token row
  int valid;   // token rows in range
  int tn;      // MMA N (multiple of 16, >= valid)
};

template <int EPI, int EP = kEpNone>
__global__ void __launch_bounds__(pair_threads(EP), 1)
    gemm_pair_kernel(const __grid_constant__ PairMaps maps, const PairParams p,
                     const __grid_constant__ PairEp ep) {
  static_assert(EPI == kEpiBf16 || EPI == kEpiSilu, "pair GEMM epilogues");
  static_assert(EP == kEpNone || (EP == kEpDispatchGateUp && EPI == kEpiSilu) ||
                    (EP == kEpDownPush && EPI == kEpiBf16),
                "expert-parallel forms: dispatch + gate/up, down + push");
  constexpr int BK = kPairBK;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ubuf = reinterpret_cast<float*>(smem + kPairStages * kPairStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      smem + kPairStages * kPairStageBytes + kPairUBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;  // [2]
  uint64_t* tempty = tfull + 2;           // [2] (even CTA: 8 warp arrivals)
  uint64_t* drain = tempty + 2;           // [1]
  uint64_t* ufull = drain + 1;            // [2] SiLU hand-off, per set
  uint64_t* ufree = ufull + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ufree + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* g_off = reinterpret_cast<int*>(tmem_slot + 4);  // [G+1]
  int* g_pref = g_off + (kMaxGroups + 1);              // [G+1] tile prefix
  int* g_tt = g_pref + (kMaxGroups + 1);               // [G] token tiles
  int* g_tn = g_tt + (kMaxGroups + 1);                 // [G] token tile width
  int* g_tme = g_tn + (kMaxGroups + 1);                // [G] first token tile in order

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cr = cluster_ctarank();  // 0 = even CTA (issues the MMAs)
  const int G = p.num_groups;
  const int m_tiles = (p.N + 255) / 256;
  const int k_blocks = (p.K + BK - 1) / BK;

  // ---- setup: barriers, TMEM, tensor maps (no global memory: with
  // programmatic dependent launch this overlaps the previous kernel), then
  // the tile table (identical in both CTAs) from the group offsets
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kPairEpiWarps);
      mbar_init(&ufull[a], 64);
      mbar_init(&ufree[a], 64);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.w);
#pragma unroll
    for (int i = 0; i < 5; ++i) tma_prefetch_desc(&maps.x[i]);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tmem_relinquish_pair();
  }
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i <= G; i += blockDim.x) {
    g_off[i] = p.offsets ? p.offsets[i] : (i == 0 ? 0 : p.rows);
    if (EP == kEpDispatchGateUp && i < G) g_tme[i] = ep.tile_first[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    bool bad = false;
    for (int g = 0; g < G; ++g) {
      int lo = g_off[g], hi = g_off[g + 1];
      if (lo < 0 || hi < lo || hi > p.rows) {
        bad = true;
        hi = lo = 0;
      }
      const int c = hi - lo;
      const int tt = (c + kPairMaxTN - 1) / kPairMaxTN;
      g_tt[g] = tt;
      g_tn[g] = tt ? (((c + tt - 1) / tt + 15) & ~15) : 0;
      g_pref[g] = acc;
      acc += m_tiles * tt;
    }
    g_pref[G] = acc;
    if (bad && p.status && cr == 0) atomicOr(p.status, kDevBadInput);
    // Expert-parallel gate/up: a group's rows are source-rank-major, and the
    // rows of source me - 1 arrive first, then me - 2, ... (every rank sends
    // its segments to me + 1, me + 2, ... in that order). Token tiles run in
    // that order too: first the tile holding this rank's own rows (already
    // here; its index comes with the call's workspace), then downwards,
    // wrapping around.
    for (int g = 0; g < G; ++g)
      g_tme[g] = EP == kEpDispatchGateUp ? min(max(g_tme[g], 0), max(g_tt[g] - 1, 0)) : 0;
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier init and TMEM of both CTAs visible
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = g_pref[G];
  const int cl0 = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(nclusters_x());

  auto map_tile = [&](int t) {
    int lo = 0, hi = G - 1;  // largest g with g_pref[g] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (g_pref[mid] <= t) lo = mid; else hi = mid - 1;
    }
    PairTile tl;
    tl.g = lo;
    const int local = t - g_pref[lo];
    const int tt = g_tt[lo];
    tl.mi = local / tt;
    int ti = local - tl.mi * tt;
    if constexpr (EP == kEpDispatchGateUp) ti = (g_tme[lo] - ti + tt) % tt;
    const int tnb = g_tn[lo];
    tl.r0 = g_off[lo] + ti * tnb;
    tl.valid = min(tnb, g_off[lo + 1] - tl.r0);
    tl.tn = (tl.valid + 15) & ~15;
    return tl;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------- TMA producer (both CTAs)
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int ready_g = -1;           // group of ready_mask
      unsigned ready_mask = 0;    // ranks whose rows of group ready_g have arrived
      for (int t = cl0; t < total_tiles && ok; t += ncl) {
        const PairTile tl = map_tile(t);
        if constexpr (EP == kEpDispatchGateUp) {
          // wait only for the ranks whose rows this tile holds
          if (tl.g != ready_g) {
            ready_g = tl.g;
            ready_mask = 1u << ep.me;
          }
          const int s_lo = __ldg(ep.push_row + tl.r0) >> 28;
          const int s_hi = __ldg(ep.push_row + tl.r0 + tl.valid - 1) >> 28;
          const unsigned need = ((2u << s_hi) - (1u << s_lo)) & ~ready_mask;
          if (need) {
            if (!ep_wait_sources(ep, tl.g, need, abort_flag)) { ok = false; break; }
            ready_mask |= need;
          }
        }
        // rows this CTA stages: the smallest box covering tn/2 token rows
        int box = 0;
        while ((128 >> box) >= tl.tn && box < 4) ++box;
        const int R = 128 >> box;
        const int w_y = tl.g * p.N + tl.mi * 256 + static_cast<int>(cr) * 128;
        const int x_y = tl.r0 + static_cast<int>(cr) * (tl.tn / 2);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * kPairStageBytes;
          const uint32_t bar = full0 + s * 8;
          if (cr == 0)
            mbar_arrive_expect_tx(&full[s], 2u * (kPairABytes + R * 128u));
          tma_load_2d_pair(a_dst, &maps.w, bar, kb * BK, w_y);
          tma_load_2d_pair(a_dst + kPairABytes, &maps.x[box], bar, kb * BK, x_y);
          if (++s == kPairStages) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && cr == 0) {
      // ---------------------------------------------- MMA issuer (even CTA)
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = cl0; t < total_tiles && ok; t += ncl) {
        const PairTile tl = map_tile(t);
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        ++it;
        if (!mbar_wait_cluster(&tempty[acc], aph ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairMaxTN;
        const uint32_t idesc = idesc_bf16(256, tl.tn, 0, 0);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * kPairStageBytes);
          const uint32_t b_addr = a_addr + kPairABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss_pair(d_tmem, sdesc_sw128(a_addr + k * 32, 0, 1024),
                            sdesc_sw128(b_addr + k * 32, 0, 1024), idesc,
                            (kb | k) != 0);
          const uint32_t e = smem_u32(&empty[s]);
          mma_commit_pair(e);
          mma_commit_pair(mapa_shared(e, 1));
          if (++s == kPairStages) { s = 0; ph ^= 1; }
        }
        if (ok) {
          const uint32_t f = smem_u32(&tfull[acc]);
          mma_commit_pair(f);
          mma_commit_pair(mapa_shared(f, 1));
        }
      }
      // Every MMA issued above must finish before TMEM is released.
      mma_commit_pair(smem_u32(drain));
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else if (EP == kEpDispatchGateUp && warp >= 2 + kPairEpiWarps) {
    // -------------------------------------------------- dispatch warps
    ep_dispatch_rows(ep, static_cast<int>(blockIdx.x) * kPairDispatchWarps +
                             (warp - 2 - kPairEpiWarps),
                     static_cast<int>(gridDim.x) * kPairDispatchWarps, lane);
  } else {
    // -------------------------------------------------- epilogue warps
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int set = (warp - 2) >> 2;  // chunks c with c % 2 == set
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    float* ub = ubuf + set * (32 * 64);
    int it = 0;
    uint32_t chunk = 0;  // SiLU hand-offs of this set so far
    for (int t = cl0; t < total_tiles; t += ncl) {
      const PairTile tl = map_tile(t);
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      ++it;
      const bool ready = mbar_wait(&tfull[acc], aph, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             acc * kPairMaxTN;
      const int n_chunks = (tl.tn + 31) / 32;
      bool ok = true;
      if constexpr (EPI == kEpiBf16) {
        const int col = tl.mi * 256 + static_cast<int>(cr) * 128 + q * 32 + lane;
        const bool col_ok = col < p.N;
        const __nv_bfloat16* crow =
            p.C ? static_cast<const __nv_bfloat16*>(p.C) + col : nullptr;
        __nv_bfloat16* drow = static_cast<__nv_bfloat16*>(p.D) + col;
#pragma unroll 1
        for (int c = set; c < n_chunks; c += 2) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_wait_ld();
          const int nv = min(32, tl.valid - c * 32);
          if constexpr (EP == kEpDownPush) {
            // row i of the chunk goes to rank (m >> 28), row (m & 0x0FFFFFFF)
            // of its result rows: lane i forms that row's address, every lane
            // then adds its column
            uintptr_t rowp = 0;
            if (lane < nv) {
              const int m = __ldg(ep.push_row + tl.r0 + c * 32 + lane);
              rowp = reinterpret_cast<uintptr_t>(ep.push_base[m >> 28]) +
                     static_cast<uintptr_t>(m & 0x0FFFFFFF) * (p.ldd * 2);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const uintptr_t base = __shfl_sync(0xffffffffu, rowp, i);
              if (i < nv && col_ok)
                reinterpret_cast<__nv_bfloat16*>(base)[col] =
                    __float2bfloat16_rn(__uint_as_float(r[i]));
            }
          } else if (col_ok) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i < nv) {
                const long long row = tl.r0 + c * 32 + i;
                float v = __uint_as_float(r[i]);
                if (crow) v += __bfloat162float(crow[row * p.ldc]);
                drow[row * p.ldd] = __float2bfloat16_rn(v);
              }
            }
          }
        }
      } else {
        // lanes 0-63 of this CTA: gate, 64-127: up, for f = fb*64 + (q&1)*32 + lane
        const bool up = q >= 2;
        const int fl = (q & 1) * 32 + lane;  // f within the 64-block
        const int f = (tl.mi * 2 + static_cast<int>(cr)) * 64 + fl;
        __nv_bfloat16* hcol = static_cast<__nv_bfloat16*>(p.D) + f;
#pragma unroll 1
        for (int c = set; c < n_chunks; c += 2, ++chunk) {
          const uint32_t uph = chunk & 1;
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_wait_ld();
          if (up) {
            if (!mbar_wait(&ufree[set], uph ^ 1, abort_flag)) { ok = false; break; }
#pragma unroll
            for (int i = 0; i < 32; ++i) ub[i * 64 + fl] = __uint_as_float(r[i]);
            mbar_arrive(&ufull[set]);
          } else {
            if (!mbar_wait(&ufull[set], uph, abort_flag)) { ok = false; break; }
            const int nv = min(32, tl.valid - c * 32);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i < nv) {
                const long long row = tl.r0 + c * 32 + i;
                const float u = ub[i * 64 + fl];
                hcol[row * p.ldd] =
                    __float2bfloat16_rn(silu_fast(__uint_as_float(r[i])) * u);
              }
            }
            mbar_arrive(&ufree[set]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (!__all_sync(0xffffffffu, ok)) break;
      if (lane == 0) mbar_arrive_cluster(tempty0 + acc * 8);
    }
  }

  if constexpr (EP == kEpDownPush) __threadfence_system();  // this CTA's pushed rows
  __syncthreads();
  if constexpr (EP == kEpDownPush) {
    if (threadIdx.x == 0 && !*abort_flag) {
      if (atomicAdd(ep.done_ctr, 1) == static_cast<int>(gridDim.x) - 1) {
        __threadfence_system();  // every CTA's rows are out: tell every rank
        for (int r = 0; r < ep.P; ++r) st_release_sys(ep.flags[r] + 2 * ep.P + ep.me, ep.epoch);
      }
    }
  }
  if (*abort_flag) {
    // Let copies and arrivals already in flight land before the pair tears
    // down (their completion is counted on the even CTA's barriers).
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kDevWaitTimeout);
  }
  tc_fence_before();
  cluster_sync_all();  // the even CTA's MMAs have drained; no remote access follows
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

}  // namespace kvm
