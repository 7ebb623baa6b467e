// Router GEMM with fused softmax and top-k (the routing step of
// kernel.comm.moe_dispatch): logits[T, E] = x[T, H] . Wr^T in fp32 on the
// tensor cores, then per token the softmax over the E logits and the k largest.
//
//   warp 0 (one lane)  TMA producer: per K block one box of x (TR rows) and
//                      one box of Wr (BN rows; rows past E read as zero)
//   warp 1 (one lane)  MMA issuer: tcgen05.mma kind::f16, M = 128, N = BN
//                      (64, 128 or 256 >= E), K in ascending 64-deep blocks
//   warps 2..5         epilogue, one thread per token row: logits out, then
//                      max, the softmax sum over E and the top-k
//
// A tile is TR <= 128 token rows (the MMA is M = 128; TMEM lanes at or past TR
// are not read back), sized so the tiles cover the SMs. A token's logits are
// the same bits whichever tile, CTA or batch computes them: one accumulator,
// K always in the same order.
//
// Measured on B200 (8192 tokens, H 4096, E 64): ~29 us per launch, of which
// streaming x at the copy rate would be ~10 us; the rest is the fixed cost
// of one tile per CTA (pipeline fill, epilogue, launch). Walking K from a
// different chunk in different CTAs (so that they do not all read the same
// router-weight lines at once) changed nothing (35.3 / 36.2 / 36.7 us per
// call with 1 / 4 / 8 chunks), so the weights' L2 lines are not the limit.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

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

template <int BN>
struct RouterCfg {
  static constexpr uint32_t kABytes = 128 * kRouterBK * 2;   // 16 KB (<= 128 rows)
  static constexpr uint32_t kBBytes = BN * kRouterBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (196608 / kStageBytes) > 8 ? 8 : (196608 / kStageBytes);
  static constexpr size_t kSmem = 1024 + size_t(kStages) * kStageBytes + (2 * kStages + 3) * 8 + 16;
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
  constexpr int STAGES = C::kStages;
  constexpr int BK = kRouterBK;
  constexpr uint32_t kIdesc = idesc_bf16(128, BN, 0, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [1] accumulators of the tile ready
  uint64_t* tempty = tfull + 1;       // [1] epilogue done with them
  uint64_t* drain = tempty + 1;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int TR = p.tile_rows;
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
      uint32_t armed_ph[STAGES];
      bool armed[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) armed[i] = false;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int row0 = t * TR;
        for (int kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * C::kStageBytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(TR + BN) * (BK * 2));
          armed[s] = true;
          armed_ph[s] = ph;
          tma_load_2d(a_dst, &tmX, &full[s], kb * BK, row0);
          tma_load_2d(a_dst + C::kABytes, &tmW, &full[s], kb * BK, 0);
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
          const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
          const uint32_t b_addr = a_addr + C::kABytes;
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
      if constexpr (BN == 64) {
        // all 64 logits of the row in registers
        float v[64];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(t_row, r0);
          tmem_ld32(t_row + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __uint_as_float(r0[i]);
            v[32 + i] = __uint_as_float(r1[i]);
          }
        }
        if (row_ok) {
          if (E == 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              reinterpret_cast<float4*>(lrow)[i] =
                  make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i < E) lrow[i] = v[i];
          }
        }
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < E) mx = fmaxf(mx, v[i]);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < E) sum += expf(v[i] - mx);
        // top-k by k selection passes over the 64 registers (the largest
        // untaken value, ties to the lower index): far fewer instructions than
        // an insertion list for k <= 8
        uint64_t taken = 0;
        for (int j = 0; j < k; ++j) {
          float best = -INFINITY;
          int b = -1;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const bool free_i = i < E && ((taken >> i) & 1ull) == 0;
            if (free_i && (b < 0 || v[i] > best)) {
              best = v[i];
              b = i;
            }
          }
          taken |= 1ull << b;
          if (row_ok) {
            p.topk_idx[static_cast<long long>(row) * k + j] = b;
            p.topk_w[static_cast<long long>(row) * k + j] = expf(best - mx) / sum;
          }
        }
      } else {
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
      }
      if (BN > 64 && row_ok) {
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

}  // namespace kvm
