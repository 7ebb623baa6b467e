// Fused causal grouped-query attention (prefill), one persistent kernel:
// S = Q K^T and O += P V on the tensor cores (tcgen05, accumulators in
// TMEM), online softmax in registers, P handed to the second MMA through
// shared memory. Scores never reach HBM: each (batch, q head, 128-row query
// tile) reads its Q tile once and the K/V tiles up to the diagonal from L2.
//
//   warp 0 (one lane)   TMA producer: Q tile, then K_j and V_j per key tile
//                       into a two-stage ring (each tile 128 rows x 128
//                       head dims = two 128-byte-swizzled boxes of 16 KB)
//   warp 1 (one lane)   MMA issuer, in the order QK_0, QK_1, PV_0, QK_2,
//                       PV_1, ... so the softmax of tile j+1 overlaps PV_j:
//                         S_b (TMEM cols 128b)  = Q . K_j^T   (K-major B)
//                         O   (TMEM cols 256)  += P_b . V_j   (MN-major B)
//   warps 2..5          one thread per query row: tcgen05.ld of its S row,
//                       causal mask, running max m and sum l in the log2
//                       domain, P = 2^(s - m) as bf16 into shared memory
//                       (128-byte swizzled K-major rows), and at the end
//                       O / l -> bf16. O is rescaled in TMEM (ld, scale, st)
//                       only when a row's max grows by more than 2^8 over
//                       the m its P values were taken against; otherwise the
//                       stale m is kept (P <= 2^8, exact in fp32 and bf16).
//
// Work items are (query tile, batch, head) with the heaviest (last) query
// tiles first, dealt round-robin to one CTA per SM. Every mbarrier wait is
// bounded; a timeout sets the device status word and the kernel drains.
#pragma once

#include <cuda_bf16.h>

#include "gemm_bf16.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace kvm {

constexpr int kAttnThreads = 192;
constexpr uint32_t kAttnHalf = 128 * 64 * 2;      // 128 rows x 64 bf16: 16 KB
constexpr uint32_t kAttnTile = 2 * kAttnHalf;     // 128 x 128 bf16: 32 KB
constexpr uint32_t kAttnOffQ = 0;
constexpr uint32_t kAttnOffK = kAttnTile;         // [2]
constexpr uint32_t kAttnOffV = 3 * kAttnTile;     // [2]
constexpr uint32_t kAttnOffP = 5 * kAttnTile;     // [2]
constexpr uint32_t kAttnOffBar = 7 * kAttnTile;
constexpr int kAttnBars = 22;
constexpr float kAttnRescale = 8.0f;              // log2 units

constexpr size_t attn_smem_bytes() {
  return 1024 + kAttnOffBar + kAttnBars * 8 + 16;
}

struct AttnParams {
  int B, L, HQ, group;  // group = HQ / HKV (query heads per kv head)
  int q_tiles;          // ceil(L / 128)
  float scale_log2;     // softmax scale * log2(e)
  __nv_bfloat16* out;
  long long ldo;
  int* status;
};

struct AttnItem {
  int b, h, qt, n;  // n = key tiles (causal: qt + 1)
};

__device__ __forceinline__ AttnItem attn_item(const AttnParams& p, int w) {
  AttnItem it;
  const int bh_count = p.B * p.HQ;
  it.qt = p.q_tiles - 1 - w / bh_count;
  const int bh = w % bh_count;
  it.b = bh / p.HQ;
  it.h = bh % p.HQ;
  it.n = it.qt + 1;
  return it;
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAttnOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;   // [2]
  uint64_t* k_empty = bars + 4;  // [2]
  uint64_t* v_full = bars + 6;   // [2]
  uint64_t* v_empty = bars + 8;  // [2]
  uint64_t* s_full = bars + 10;  // [2]
  uint64_t* s_free = bars + 12;  // [2] 128 arrivals
  uint64_t* p_full = bars + 14;  // [2] 128 arrivals
  uint64_t* p_free = bars + 16;  // [2]
  uint64_t* o_done = bars + 18;  // every PV
  uint64_t* o_final = bars + 19; // last PV of an item
  uint64_t* o_free = bars + 20;  // 128 arrivals: O read out
  uint64_t* drain = bars + 21;   // every MMA of the CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kAttnBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_items = p.B * p.HQ * p.q_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_init(o_free, 128);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_o = tmem_base + 256;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      uint32_t ic = 0, kvc = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
        const AttnItem it = attn_item(p, w);
        const int kh = it.h / p.group;
        const int row0 = it.b * p.L;
        if (!mbar_wait(q_empty, (ic & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, kAttnTile);
        tma_load_2d(smem + kAttnOffQ, &tmQ, q_full, it.h * 128, row0 + it.qt * 128);
        tma_load_2d(smem + kAttnOffQ + kAttnHalf, &tmQ, q_full, it.h * 128 + 64,
                    row0 + it.qt * 128);
        for (int j = 0; j < it.n; ++j, ++kvc) {
          const int s = kvc & 1;
          const uint32_t ph = (kvc >> 1) & 1;
          uint8_t* kd = smem + kAttnOffK + s * kAttnTile;
          uint8_t* vd = smem + kAttnOffV + s * kAttnTile;
          if (!mbar_wait(&k_empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[s], kAttnTile);
          tma_load_2d(kd, &tmK, &k_full[s], kh * 128, row0 + j * 128);
          tma_load_2d(kd + kAttnHalf, &tmK, &k_full[s], kh * 128 + 64, row0 + j * 128);
          if (!mbar_wait(&v_empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[s], kAttnTile);
          tma_load_2d(vd, &tmV, &v_full[s], kh * 128, row0 + j * 128);
          tma_load_2d(vd + kAttnHalf, &tmV, &v_full[s], kh * 128 + 64, row0 + j * 128);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t kIdescQK = idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t kIdescPV = idesc_bf16(128, 128, 0, 1);
      const uint32_t q_addr = smem_u32(smem + kAttnOffQ);
      uint32_t ic = 0, kvc = 0, tc = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
        const AttnItem it = attn_item(p, w);
        if (!mbar_wait(q_full, ic & 1, abort_flag)) { ok = false; break; }
        for (int j = 0; j <= it.n && ok; ++j) {
          if (j < it.n) {
            // S_b = Q . K_j^T
            const uint32_t kv = kvc + j, t = tc + j;
            const int s = kv & 1, b = t & 1;
            if (!mbar_wait(&k_full[s], (kv >> 1) & 1, abort_flag) ||
                !mbar_wait(&s_free[b], ((t >> 1) & 1) ^ 1, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t k_addr = smem_u32(smem + kAttnOffK + s * kAttnTile);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t off = (kk >> 2) * kAttnHalf + (kk & 3) * 32;
              mma_f16_ss(tmem_base + b * 128, sdesc_sw128(q_addr + off, 0, 1024),
                         sdesc_sw128(k_addr + off, 0, 1024), kIdescQK, kk > 0);
            }
            mma_commit(&s_full[b]);
            mma_commit(&k_empty[s]);
            if (j == it.n - 1) mma_commit(q_empty);
          }
          if (j >= 1) {
            // O += P_b . V_i
            const int i = j - 1;
            const uint32_t kv = kvc + i, t = tc + i;
            const int s = kv & 1, b = t & 1;
            if (!mbar_wait(&v_full[s], (kv >> 1) & 1, abort_flag) ||
                !mbar_wait(&p_full[b], (t >> 1) & 1, abort_flag) ||
                (i == 0 && !mbar_wait(o_free, (ic & 1) ^ 1, abort_flag))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t p_addr = smem_u32(smem + kAttnOffP + b * kAttnTile);
            const uint32_t v_addr = smem_u32(smem + kAttnOffV + s * kAttnTile);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint32_t poff = (kk >> 2) * kAttnHalf + (kk & 3) * 32;
              mma_f16_ss(tmem_o, sdesc_sw128(p_addr + poff, 0, 1024),
                         sdesc_sw128(v_addr + kk * 2048, kAttnHalf, 1024), kIdescPV,
                         (i > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&v_empty[s]);
            mma_commit(&p_free[b]);
            mma_commit(o_done);
            if (i == it.n - 1) mma_commit(o_final);
          }
        }
        kvc += it.n;
        tc += it.n;
      }
      // Every MMA issued above must finish before TMEM is released.
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // ------------------------------------------------ softmax / epilogue
    const int q = warp & 3;                   // TMEM lane quarter
    const int r = q * 32 + lane;              // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const float sl2 = p.scale_log2;
    uint32_t ic = 0, tc = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
      const AttnItem it = attn_item(p, w);
      float m = 0.f, l = 0.f;
      for (int j = 0; j < it.n; ++j) {
        const uint32_t t = tc + j;
        const int b = t & 1;
        const bool ready = mbar_wait(&s_full[b], (t >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
        tc_fence_after();
        float s[128];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t u[32];
          tmem_ld32(tmem_base + lane_off + b * 128 + c4 * 32, u);
          tmem_wait_ld();
          // two scores per instruction (packed multiply, round to nearest)
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 v = __fmul2_rn(
                make_float2(__uint_as_float(u[i]), __uint_as_float(u[i + 1])),
                make_float2(sl2, sl2));
            s[c4 * 32 + i] = v.x;
            s[c4 * 32 + i + 1] = v.y;
          }
        }
        tc_fence_before();
        mbar_arrive(&s_free[b]);
        if (j == it.qt) {  // diagonal tile: keys after the query are masked
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > r) s[c] = -INFINITY;
        }
        // Row max as eight independent chains (max is exact in any order):
        // one warp per SM sub-partition runs this, so a single 128-long
        // dependency chain would stall it on every step.
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
        for (int c = 8; c < 128; c += 8)
#pragma unroll
          for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], s[c + i]);
        const float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        if (j == 0) {
          m = mt;
        } else if (__any_sync(0xffffffffu, mt > m + kAttnRescale)) {
          // Some row of this warp outgrew its max by more than 2^8: the whole
          // warp (tcgen05.ld/st are warp-collective) rescales its 32 rows of
          // O to the new maxima (alpha = 1 for rows whose max did not grow);
          // PV_{j-1} must have landed first.
          const float mn = fmaxf(m, mt);
          const float alpha = ex2_approx(m - mn);
          const bool done = mbar_wait(o_done, (t - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, done)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t u[32];
            tmem_ld32(tmem_o + lane_off + c4 * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
            tmem_st32(tmem_o + lane_off + c4 * 32, u);
          }
          tmem_wait_st();
          l *= alpha;
          m = mn;
        }
        // P row -> shared memory (two 128-byte-swizzled K-major halves)
        const bool freed = mbar_wait(&p_free[b], ((t >> 1) & 1) ^ 1, abort_flag);
        if (!__all_sync(0xffffffffu, freed)) { ok = false; break; }
        uint8_t* prow = smem + kAttnOffP + b * kAttnTile + r * 128;
        // The tile's row sum in eight partial sums (key c into sum c % 8),
        // added to l at the end: eight short chains instead of one long one.
        float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 16; ++c) {  // 16 chunks of 8 keys
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            e[i] = ex2_approx(s[c * 8 + i] - m);
            ls[i] += e[i];
          }
          uint4 v;
          v.x = pack_bf16x2(e[0], e[1]);
          v.y = pack_bf16x2(e[2], e[3]);
          v.z = pack_bf16x2(e[4], e[5]);
          v.w = pack_bf16x2(e[6], e[7]);
          const int half = c >> 3, ch = c & 7;
          *reinterpret_cast<uint4*>(prow + half * kAttnHalf + ((ch ^ (r & 7)) << 4)) = v;
        }
        l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        fence_async_smem();
        tc_fence_before();  // orders a rescale's tcgen05.st before the PV
        mbar_arrive(&p_full[b]);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> bf16 row of the output
      const bool fin = mbar_wait(o_final, ic & 1, abort_flag);
      if (!__all_sync(0xffffffffu, fin)) { ok = false; break; }
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = it.qt * 128 + r;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(it.b) * p.L + qrow) * p.ldo +
                            static_cast<long long>(it.h) * 128;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t u[32];
        tmem_ld32(tmem_o + lane_off + c4 * 32, u);
        tmem_wait_ld();
        if (qrow < p.L) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(u[8 * i + 0]) * inv, __uint_as_float(u[8 * i + 1]) * inv);
            v.y = pack_bf16x2(__uint_as_float(u[8 * i + 2]) * inv, __uint_as_float(u[8 * i + 3]) * inv);
            v.z = pack_bf16x2(__uint_as_float(u[8 * i + 4]) * inv, __uint_as_float(u[8 * i + 5]) * inv);
            v.w = pack_bf16x2(__uint_as_float(u[8 * i + 6]) * inv, __uint_as_float(u[8 * i + 7]) * inv);
            reinterpret_cast<uint4*>(orow + c4 * 32)[i] = v;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(o_free);
      tc += it.n;
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // Let copies already in flight land before the CTA exits.
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kDevWaitTimeout);
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace kvm
