// Router GEMM with fused softmax and top-k (the routing step of
// kernel.comm.moe_dispatch): logits[T, E] = x[T, H] . Wr^T in fp32 on the
// tensor cores, then per token the softmax over the E logits and the k largest.
// Two kernels: router_pair_kernel (E <= 64, SM pairs, K split in two; below)
// and router_topk_kernel (E up to 256, one SM per tile):
//
//   warp 0 (one lane)  TMA producer: per K block one box of x (TR rows) and
//                      one box of Wr (BN rows; rows past E read as zero)
//   warp 1 (one lane)  MMA issuer: tcgen05.mma kind::f16, M = 128, N = BN
//                      (128 or 256 >= E), K in ascending 64-deep blocks
//   warps 2..5         epilogue, one thread per token row: logits out, then
//                      max, the softmax sum over E and the top-k
//
// A tile is TR <= 128 token rows (the MMA is M = 128; TMEM lanes at or past TR
// are not read back), sized so the tiles cover the SMs. A token's logits are
// the same bits whichever tile, CTA or batch computes them: one accumulator,
// K always in the same order.
//
// Measured on B200 with this kernel at E = 64 (8192 tokens, H 4096; it ran
// E <= 64 too before router_pair_kernel), per
// launch, timed as 50 launches queued behind a sleep kernel: 28.0 us in all
// (25.9 us once mbarrier waits carry a suspend-time hint, ptx.cuh);
// 8.3 us with no K block at all (2.4 us of it launch and setup, the rest the
// epilogue); then ~0.28 us per 64-deep K block whatever it loads: without the
// x loads 27.1 us, without the Wr loads 28.0, 128-row tiles on 64 SMs 27.8,
// 8 or 14 stages alike, without the MMAs 21.6. Walking K from a different
// chunk in different CTAs changed nothing either.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"
#include "runtime.h"

namespace kvm {

constexpr int kRouterThreads = 192;
constexpr int kRouterBK = 64;

struct RouterParams {
  int T, E, K, top_k;
  int tile_rows;   // TR, a multiple of 8 in [8, 128]
  float* logits;   // [T, E]
  int* topk_idx;   // [T, k]
  float* topk_w;   // [T, k]
  int* status;
};

// Shared memory: a ring of stages, each the x box of the tile's TR rows
// followed by the Wr box of BN rows, packed at TR * 128 + BN * 128 bytes so
// that a short tile keeps more bytes in flight (8192 tokens: 56-row tiles, 14
// stages of 15 KB). The M = 128 MMA reads 128 A rows from each stage; rows at
// or past TR read the following bytes (their results land in TMEM lanes that
// are never read), and a pad after the last stage keeps those reads inside
// the allocation. Barriers live in static shared memory.
template <int BN>   // 128 or 256 (E <= 64 runs router_pair_kernel)
struct RouterCfg {
  static constexpr uint32_t kBBytes = BN * kRouterBK * 2;
  static constexpr int kMaxStages = 16;
  static constexpr size_t kSmem = 220 * 1024;
  __host__ __device__ static uint32_t stage_bytes(int tr) {
    return static_cast<uint32_t>(tr) * (kRouterBK * 2) + kBBytes;
  }
  __host__ __device__ static int stages(int tr) {
    const uint32_t pad = static_cast<uint32_t>(128 - tr) * (kRouterBK * 2);
    const int n = static_cast<int>((kSmem - 1024 - pad) / stage_bytes(tr));
    return n < kMaxStages ? n : kMaxStages;
  }
};

// Insert (v, i) into the descending top-k list (bv, bi) of n valid entries:
// an equal value goes after the entries already there, so ties keep the lower
// expert index first. Fully unrolled so the list stays in registers.
__device__ __forceinline__ void topk_insert(float (&bv)[8], int (&bi)[8], int& n, int k,
                                            float v, int i) {
  float kth = bv[0];  // the k-th entry, read without a dynamic register index
#pragma unroll
  for (int p = 1; p < 8; ++p)
    if (p == k - 1) kth = bv[p];
  if (n >= k && !(v > kth)) return;
  // v goes before the first smaller entry (or into the first empty slot);
  // from there on every entry moves down one slot and the last drops out.
  float cv = v;
  int ci = i;
  bool placed = false;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    if (p < k && (placed || p >= n || bv[p] < cv)) {
      const float tv = bv[p];
      const int ti = bi[p];
      bv[p] = cv;
      bi[p] = ci;
      cv = tv;
      ci = ti;
      placed = true;
    }
  }
  if (n < k) ++n;
}

template <int BN>
__global__ void __launch_bounds__(kRouterThreads, 1)
    router_topk_kernel(const __grid_constant__ CUtensorMap tmX,
                       const __grid_constant__ CUtensorMap tmW, const RouterParams p) {
  using C = RouterCfg<BN>;
  constexpr int BK = kRouterBK;
  constexpr uint32_t kIdesc = idesc_bf16(128, BN, 0, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[2 * C::kMaxStages + 3];
  __shared__ uint32_t tmem_slot[1];
  __shared__ int abort_word;
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kMaxStages;
  uint64_t* tfull = bars + 2 * C::kMaxStages;   // [1] accumulators of the tile ready
  uint64_t* tempty = tfull + 1;                 // [1] epilogue done with them
  uint64_t* drain = tempty + 1;                 // [1]
  volatile int* abort_flag = &abort_word;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int TR = p.tile_rows;
  const int STAGES = C::stages(TR);
  const uint32_t stage_bytes = C::stage_bytes(TR);
  const uint32_t a_bytes = static_cast<uint32_t>(TR) * (BK * 2);
  const int tiles = (p.T + TR - 1) / TR;
  const int kb_total = (p.K + BK - 1) / BK;
  constexpr uint32_t tmem_cols = BN;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 128);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t armed_ph[C::kMaxStages];
      bool armed[C::kMaxStages];
#pragma unroll
      for (int i = 0; i < C::kMaxStages; ++i) armed[i] = false;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int row0 = t * TR;
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          armed[s] = true;
          armed_ph[s] = ph;
          tma_load_2d(a_dst, &tmX, &full[s], kb * BK, row0);
          tma_load_2d(a_dst + a_bytes, &tmW, &full[s], kb * BK, 0);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        volatile int local_abort = 0;
        for (int i = 0; i < STAGES; ++i)
          if (armed[i]) mbar_wait(&full[i], armed_ph[i], &local_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        // one accumulator set: wait until the epilogue has read the last tile's
        if (!mbar_wait(tempty, (it & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
          const uint32_t b_addr = a_addr + a_bytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss(tmem_base, sdesc_sw128(a_addr + k * 32, 0, 1024),
                       sdesc_sw128(b_addr + k * 32, 0, 1024), kIdesc,
                       (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) mma_commit(tfull);
      }
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // -------------------------------------------------- epilogue warps
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int r_in_tile = q * 32 + lane;
    const int E = p.E, k = p.top_k;
    int it = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
      const bool ready = mbar_wait(tfull, it & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      const int row = t * TR + r_in_tile;
      const bool row_ok = row < p.T && r_in_tile < TR;
      float* lrow = p.logits + static_cast<long long>(row) * E;
      float bv[8];
      int bi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        bv[i] = -INFINITY;
        bi[i] = -1;
      }
      int n = 0;
      float mx = -INFINITY;
      float sum = 0.f;
      // pass 1: logits, max, top-k (insertion list), 32 columns at a time
#pragma unroll 1
      for (int sl = 0; sl < BN / 32; ++sl) {
        float v[32];
        {
          uint32_t r[32];
          tmem_ld32(t_row + sl * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int e = sl * 32 + i;
          if (e < E) {
            if (row_ok) lrow[e] = v[i];
            mx = fmaxf(mx, v[i]);
            topk_insert(bv, bi, n, k, v[i], e);
          }
        }
      }
      // pass 2: softmax denominator in ascending expert order
#pragma unroll 1
      for (int sl = 0; sl < BN / 32; ++sl) {
        float v[32];
        {
          uint32_t r[32];
          tmem_ld32(t_row + sl * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (sl * 32 + i < E) sum += expf(v[i] - mx);
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j < k) {
            p.topk_idx[static_cast<long long>(row) * k + j] = bi[j];
            p.topk_w[static_cast<long long>(row) * k + j] = expf(bv[j] - mx) / sum;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicOr(p.status, 1);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}


// ---------------------------------------------------------------------------
// E <= 64: the router on SM pairs, K split in two.
//
// The one-SM kernel above walks all of K per tile (~0.28 us per K block)
// and finishes each row on one thread. Here the two CTAs of a cluster share
// one token tile and each walks half of K, and the epilogue spreads a row over
// 4 threads. Measured on B200 (8192 tokens, H 4096, E 64; 50 launches queued
// behind a sleep kernel): 23.4 us per launch against 25.9 us for the one-SM
// kernel (20.7 us once launched with programmatic dependent launch, which
// overlaps one launch's prologue with the previous one's tail). Right after
// another kernel: 26.7 us after a 256 MB read, 30.7 us after a 256 MB copy
// (written lines that L2 writes back while x streams in) -- the latter is
// what it costs inside the MoE layer, after the combine's writes.
//
//   warp 0 (one lane)  TMA producer for this CTA's K half
//   warp 1 (one lane)  MMA issuer: M = 128 (the tile's rows), N = 64
//   warps 2..9         epilogue. Phase 1: each warp reads 32 columns of its
//                      TMEM lane quarter (the partial logits of this CTA's K
//                      half) and stores them to the shared memory of the CTA
//                      that owns the row (rows [0, h) CTA 0, [h, TR) CTA 1).
//                      Phase 2: per owned row 4 threads of one warp, 16
//                      logits each: logit = partial(K half 0) + partial(K
//                      half 1), then max, softmax sum and top-k with shuffles.
//
// A token's logits are the same bits in any batch: the K split depends only on
// H, each half accumulates in the tensor core in K order, and the halves are
// added in a fixed order. The softmax sum is ((s0 + s1) + (s2 + s3)) over the
// four 16-column slices, each summed in ascending expert order. The top-k
// order is (larger logit, then lower expert index), NaN below every number.
constexpr int kRouterPairThreads = 320;
constexpr int kRouterXStride = 68;   // floats per exchanged row: 64 + 4 of padding

struct RouterPairCfg {
  static constexpr uint32_t kBBytes = 64 * kRouterBK * 2;                 // Wr box, 8 KB
  static constexpr uint32_t kXHalf = 2u * 64 * kRouterXStride * 4;        // 34 KB
  static constexpr uint32_t kXBytes = 2 * kXHalf;   // two tiles in flight
  static constexpr int kMaxStages = 16;
  static constexpr size_t kSmem = 220 * 1024;
  __host__ __device__ static uint32_t stage_bytes(int tr) {
    return static_cast<uint32_t>(tr) * (kRouterBK * 2) + kBBytes;
  }
  __host__ __device__ static int stages(int tr) {
    const uint32_t pad = static_cast<uint32_t>(128 - tr) * (kRouterBK * 2);
    const int n = static_cast<int>((kSmem - 1024 - kXBytes - pad) / stage_bytes(tr));
    return n < kMaxStages ? n : kMaxStages;
  }
};

struct TopkCand {
  float v;
  int i;   // -1: none
};

// The top-k order: a valid candidate before none, a larger logit first, NaN
// after every number, equal logits by lower expert index. A strict total
// order, so every lane that merges the same candidates picks the same one.
__device__ __forceinline__ bool topk_before(TopkCand a, TopkCand b) {
  if (a.i < 0) return false;
  if (b.i < 0) return true;
  if (a.v > b.v) return true;
  if (a.v < b.v) return false;
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return bn;
  return a.i < b.i;
}

__global__ void __launch_bounds__(kRouterPairThreads, 1)
    router_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                       const __grid_constant__ CUtensorMap tmW, const RouterParams p) {
  using C = RouterPairCfg;
  constexpr int BK = kRouterBK;
  constexpr uint32_t kIdesc = idesc_bf16(128, 64, 0, 0);
  constexpr uint32_t tmem_cols = 64;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [tile parity][K half][64 rows][68]: the partial logits of the rows this
  // CTA owns. Tile i + 2 reuses tile i's buffer; every thread that writes it
  // has passed the xfull wait of tile i + 1, which needs the arrivals that
  // both CTAs' threads make only after finishing phase 2 of tile i.
  float* xbuf = reinterpret_cast<float*>(base);
  uint8_t* ring = base + C::kXBytes;
  __shared__ __align__(8) uint64_t bars[2 * C::kMaxStages + 5];
  __shared__ uint32_t tmem_slot[1];
  __shared__ int abort_word;
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kMaxStages;
  uint64_t* tfull = bars + 2 * C::kMaxStages;   // partial logits of the tile in TMEM
  uint64_t* tempty = tfull + 1;                 // TMEM read back (256 epilogue threads)
  uint64_t* drain = tempty + 1;
  // [tile parity]: both CTAs' partials of the rows this CTA owns are stored.
  // One barrier per parity: a thread's arrivals for tile i on the two CTAs'
  // barriers are ordered (release) before its arrivals for tile i + 1, so a
  // thread that has passed tile i + 1 cannot count toward tile i's phase.
  uint64_t* xfull = drain + 1;
  volatile int* abort_flag = &abort_word;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t me = cluster_ctarank();   // also the K half this CTA walks
  const uint32_t peer = me ^ 1u;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const int TR = p.tile_rows;
  const int h = (TR + 1) / 2;   // rows owned by CTA 0; CTA 1 owns [h, TR)
  const int STAGES = C::stages(TR);
  const uint32_t stage_bytes = C::stage_bytes(TR);
  const uint32_t a_bytes = static_cast<uint32_t>(TR) * (BK * 2);
  const int tiles = (p.T + TR - 1) / TR;
  const int kb_total = (p.K + BK - 1) / BK;
  const int kb_half = (kb_total + 1) / 2;
  const int kb_lo = static_cast<int>(me) * kb_half;
  const int kb_hi = kb_lo + kb_half < kb_total ? kb_lo + kb_half : kb_total;
  const bool has_k = kb_hi > kb_lo;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 256);
    mbar_init(drain, 1);
    mbar_init(&xfull[0], 512);
    mbar_init(&xfull[1], 512);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // the other CTA's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // x may still be written, and the outputs read, by the previous kernel
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t armed_ph[C::kMaxStages];
      bool armed[C::kMaxStages];
#pragma unroll
      for (int i = 0; i < C::kMaxStages; ++i) armed[i] = false;
      for (int t = pair; t < tiles && ok; t += npairs) {
        const int row0 = t * TR;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = ring + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          armed[s] = true;
          armed_ph[s] = ph;
          tma_load_2d(a_dst, &tmX, &full[s], kb * BK, row0);
          tma_load_2d(a_dst + a_bytes, &tmW, &full[s], kb * BK, 0);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        volatile int local_abort = 0;
        for (int i = 0; i < STAGES; ++i)
          if (armed[i]) mbar_wait(&full[i], armed_ph[i], &local_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += npairs, ++it) {
        if (!mbar_wait(tempty, (it & 1) ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * stage_bytes);
          const uint32_t b_addr = a_addr + a_bytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_ss(tmem_base, sdesc_sw128(a_addr + k * 32, 0, 1024),
                       sdesc_sw128(b_addr + k * 32, 0, 1024), kIdesc,
                       (kb != kb_lo || k != 0) ? 1u : 0u);
          mma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) mma_commit(tfull);
      }
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // -------------------------------------------------- epilogue warps
    const int et = threadIdx.x - 64;   // 0..255
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int ch = (warp - 2) >> 2;    // phase 1: column half (32 columns)
    const int row = q * 32 + lane;     // phase 1: row of the tile (TMEM lane)
    const int owner = row < h ? 0 : 1;
    const uint32_t dst_row = mapa_shared(
        smem_u32(xbuf + (static_cast<int>(me) * 64 + (row - owner * h)) * kRouterXStride +
                 ch * 32),
        static_cast<uint32_t>(owner));
    const uint32_t xfull_own = mapa_shared(smem_u32(xfull), me);
    const uint32_t xfull_peer = mapa_shared(smem_u32(xfull), peer);
    const int lr = et >> 2;            // phase 2: owned row
    const int sl = et & 3;             // phase 2: 16-column slice
    const int n_own = me == 0 ? h : TR - h;
    const int E = p.E, k = p.top_k;
    int it = 0;
    for (int t = pair; t < tiles; t += npairs, ++it) {
      // ---- phase 1: this CTA's partial logits -> the owning CTA
      const bool ready = mbar_wait(tfull, it & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      uint32_t r[32];
      if (has_k) {
        tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ch * 32, r);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;   // no K block in this half: +0.0
      }
      tc_fence_before();
      mbar_arrive(tempty);
      const uint32_t par = static_cast<uint32_t>(it & 1);
      if (row < TR) {
        const uint32_t dst = dst_row + par * C::kXHalf;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_cluster_v4(dst + 16 * i, r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      }
      mbar_arrive_cluster(xfull_own + 8 * par);
      mbar_arrive_cluster(xfull_peer + 8 * par);

      // ---- phase 2: the rows this CTA owns
      const bool got = mbar_wait_cluster(&xfull[par], (it >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      const long long grow = static_cast<long long>(t) * TR + static_cast<int>(me) * h + lr;
      const bool row_ok = lr < n_own && grow < p.T;
      float v[16];
      {
        const float* xb = xbuf + par * (C::kXHalf / 4);
        const float4* lo = reinterpret_cast<const float4*>(xb + lr * kRouterXStride + sl * 16);
        const float4* hi =
            reinterpret_cast<const float4*>(xb + (64 + lr) * kRouterXStride + sl * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 a = lo[i], b = hi[i];
          v[4 * i] = a.x + b.x;
          v[4 * i + 1] = a.y + b.y;
          v[4 * i + 2] = a.z + b.z;
          v[4 * i + 3] = a.w + b.w;
        }
      }
      const int c0 = sl * 16;
      if (row_ok) {
        float* lrow = p.logits + grow * E;
        if (E == 64) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<float4*>(lrow + c0)[i] =
                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c0 + i < E) lrow[c0 + i] = v[i];
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (c0 + i < E) mx = fmaxf(mx, v[i]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (c0 + i < E) sum += expf(v[i] - mx);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      uint32_t taken = 0;
      for (int j = 0; j < k; ++j) {
        TopkCand b{-INFINITY, -1};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const TopkCand c{v[i], c0 + i};
          if (c0 + i < E && ((taken >> i) & 1u) == 0 && topk_before(c, b)) b = c;
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
          TopkCand o;
          o.v = __shfl_xor_sync(0xffffffffu, b.v, off);
          o.i = __shfl_xor_sync(0xffffffffu, b.i, off);
          if (topk_before(o, b)) b = o;
        }
        if (b.i >= c0 && b.i < c0 + 16) taken |= 1u << (b.i - c0);
        if (row_ok && sl == 0) {
          p.topk_idx[grow * k + j] = b.i;
          p.topk_w[grow * k + j] = expf(b.v - mx) / sum;
        }
      }
    }
  }

  __syncthreads();
  cluster_sync_all();   // no remote store or arrive is still in flight to either CTA
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicOr(p.status, 1);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace kvm
