// Router GEMM with fused softmax and top-k (the routing step of
// kernel.comm.moe_dispatch): logits[T, E] = x[T, H] . Wr^T in fp32 on the
// tensor cores, then per token the softmax over the E logits and the k largest.
//
// The x rows stream from HBM once; the router weights (E x H, 512 KB at E = 64,
// H = 4096) are read by every CTA. If all CTAs walked K in the same order they
// would all read the same few KB of weights at the same moment, and those L2
// lines, not HBM, would set the pace. So K is cut into NCH chunks, each
// accumulated into a TMEM accumulator of its own, and CTA b works through the
// chunks starting at chunk b mod NCH: at any moment the CTAs spread over NCH
// regions of the weights. The epilogue adds the chunk accumulators in chunk
// order (((c0 + c1) + c2) + ...), so a token's logits depend only on its own
// row and H -- not on which tile or CTA computed it, nor on the token count.
//
//   warp 0 (one lane)  TMA producer: per K block one box of x (TR rows) and
//                      one box of Wr (BN rows; rows past E read as zero)
//   warp 1 (one lane)  MMA issuer: tcgen05.mma kind::f16, M = 128, N = BN,
//                      into accumulator `chunk` of the tile
//   warps 2..5         epilogue, one thread per token row: logits out, then
//                      max, top-k and the softmax sum over E
//
// A tile is TR <= 128 token rows (the MMA is M = 128; TMEM lanes at or past TR
// are not read back), sized so the tiles cover the SMs.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace kvm {

constexpr int kRouterThreads = 192;
constexpr int kRouterBK = 64;

struct RouterParams {
  int T, E, K, top_k;
  int tile_rows;   // TR, a multiple of 8 in [8, 128]
  int nch;         // K chunks (each a TMEM accumulator of BN columns)
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
  static constexpr int kMaxChunks = 512 / BN;
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
  float cv = v;
  int ci = i;
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    if (p < k && (p >= n || bv[p] < cv)) {
      const float tv = bv[p];
      const int ti = bi[p];
      bv[p] = cv;
      bi[p] = ci;
      cv = tv;
      ci = ti;
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
  const int nch = p.nch;
  const int kpc = (kb_total + nch - 1) / nch;   // K blocks per chunk
  uint32_t tmem_cols = 32;
  while (tmem_cols < static_cast<uint32_t>(nch * BN)) tmem_cols <<= 1;

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
  const int first_chunk = static_cast<int>(blockIdx.x) % nch;

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
        for (int j = 0; j < nch && ok; ++j) {
          const int c = (first_chunk + j) % nch;
          const int kb1 = min(kb_total, (c + 1) * kpc);
          for (int kb = c * kpc; kb < kb1; ++kb) {
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
        for (int j = 0; j < nch && ok; ++j) {
          const int c = (first_chunk + j) % nch;
          const uint32_t d_tmem = tmem_base + c * BN;
          const int kb0 = c * kpc, kb1 = min(kb_total, (c + 1) * kpc);
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
            const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_f16_ss(d_tmem, sdesc_sw128(a_addr + k * 32, 0, 1024),
                         sdesc_sw128(b_addr + k * 32, 0, 1024), kIdesc,
                         (kb != kb0 || k != 0) ? 1u : 0u);
            mma_commit(&empty[s]);
            if (++s == STAGES) { s = 0; ph ^= 1; }
          }
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
      // pass 1: logits (chunk accumulators added in chunk order), max, top-k
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
#pragma unroll 1
        for (int c = 1; c < nch; ++c) {
          uint32_t r[32];
          tmem_ld32(t_row + c * BN + sl * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(r[i]);
        }
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int e = sl * 32 + i;
            if (e < E) {
              lrow[e] = v[i];
              mx = fmaxf(mx, v[i]);
              topk_insert(bv, bi, n, k, v[i], e);
            }
          }
        }
      }
      // pass 2: softmax denominator in ascending expert order
      float sum = 0.f;
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
#pragma unroll 1
        for (int c = 1; c < nch; ++c) {
          uint32_t r[32];
          tmem_ld32(t_row + c * BN + sl * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(r[i]);
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

}  // namespace kvm
