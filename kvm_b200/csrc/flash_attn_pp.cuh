// Fused causal grouped-query attention (prefill) with two query tiles per
// CTA in ping-pong: the tiles of two query heads of the same kv head at the
// same position (so they share every K/V tile and the causal extent). While
// one softmax warpgroup turns its scores into P, the tensor core runs the
// other tile's PV and next QK, so neither waits on the other.
//
//   warp 0 (one lane)   TMA producer: Q_A and Q_B, then K_j, V_j per key tile
//                       into a three-slot ring of 32 KB tiles
//   warp 1 (one lane)   MMA issuer, per key tile j:
//                         PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1)
//                       S_X (TMEM cols 128X) = Q_X . K^T, O_X (cols 256 + 128X)
//                       += P_X . V; X in {A, B}
//   warps 2..5, 6..9    softmax of tile A, tile B: one thread per query row;
//                       the row max from a first pass over S in TMEM, then
//                       P = 2^(s - m) as bf16 into shared memory from a second
//                       pass (scores are not held in registers); O rescaled in
//                       TMEM only when a row's max grows by more than 2^8
//                       (as in flash_attn.cuh); at the end O / l -> bf16.
//                       Scores are scaled with __fmul_rn (never contracted
//                       into the exponent's subtraction), so both kernels
//                       produce the same bits.
//
// The order S_X(j+1) after PV_X(j) makes the TMEM of S_X and the shared
// memory of P_X free by construction: PV_X(j) waits for P_X(j), which the
// softmax writes after its last read of S_X(j). Every mbarrier wait is
// bounded; a timeout sets the device status word and the kernel drains.
#pragma once

#include "flash_attn.cuh"

namespace kvm {

constexpr int kPpThreads = 320;
constexpr int kPpRing = 3;                            // K/V tile slots
constexpr uint32_t kPpOffQ = 0;                       // [2] Q_A, Q_B
constexpr uint32_t kPpOffKV = 2 * kAttnTile;          // [kPpRing]
constexpr uint32_t kPpOffP = 5 * kAttnTile;           // [2] P_A, P_B
constexpr uint32_t kPpOffBar = 7 * kAttnTile;
constexpr int kPpBars = 2 + 2 * kPpRing + 2 * 6 + 1;

constexpr size_t attn_pp_smem_bytes() {
  return 1024 + kPpOffBar + kPpBars * 8 + 16;
}
static_assert(attn_pp_smem_bytes() <= 232448, "ping-pong attention shared memory");

// Items (query tile, batch, head pair), heaviest query tiles first.
struct AttnPairItem {
  int b, h0, qt, n;  // heads h0, h0 + 1; n = key tiles (causal: qt + 1)
};

__device__ __forceinline__ AttnPairItem attn_pair_item(const AttnParams& p, int w) {
  AttnPairItem it;
  const int pairs = p.HQ / 2;
  const int bh_count = p.B * pairs;
  it.qt = p.q_tiles - 1 - w / bh_count;
  const int bh = w % bh_count;
  it.b = bh / pairs;
  it.h0 = 2 * (bh % pairs);
  it.n = it.qt + 1;
  return it;
}

__device__ __forceinline__ void attn_qk(uint32_t d, uint32_t q_addr, uint32_t k_addr) {
  constexpr uint32_t kIdescQK = idesc_bf16(128, 128, 0, 0);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * kAttnHalf + (kk & 3) * 32;
    mma_f16_ss(d, sdesc_sw128(q_addr + off, 0, 1024), sdesc_sw128(k_addr + off, 0, 1024),
               kIdescQK, kk > 0);
  }
}

__device__ __forceinline__ void attn_pv(uint32_t d, uint32_t p_addr, uint32_t v_addr,
                                        bool accumulate) {
  constexpr uint32_t kIdescPV = idesc_bf16(128, 128, 0, 1);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t poff = (kk >> 2) * kAttnHalf + (kk & 3) * 32;
    mma_f16_ss(d, sdesc_sw128(p_addr + poff, 0, 1024),
               sdesc_sw128(v_addr + kk * 2048, kAttnHalf, 1024), kIdescPV,
               (accumulate || kk > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(kPpThreads, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPpOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;               // [kPpRing]
  uint64_t* kv_empty = kv_full + kPpRing;     // [kPpRing]
  uint64_t* xb = kv_empty + kPpRing;          // per tile X: 6 barriers at xb + 6X
  // xb[6X + 0] s_full   (commit after QK_X)
  // xb[6X + 1] p_full   (128 arrivals: P_X written)
  // xb[6X + 2] p_free   (commit after PV_X)
  // xb[6X + 3] o_done   (commit after PV_X)
  // xb[6X + 4] o_final  (commit after the last PV_X of an item)
  // xb[6X + 5] o_free   (128 arrivals: O_X read out)
  uint64_t* drain = xb + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPpBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int n_items = p.B * (p.HQ / 2) * p.q_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kPpRing; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&xb[6 * x + 0], 1);
      mbar_init(&xb[6 * x + 1], 128);
      mbar_init(&xb[6 * x + 2], 1);
      mbar_init(&xb[6 * x + 3], 1);
      mbar_init(&xb[6 * x + 4], 1);
      mbar_init(&xb[6 * x + 5], 128);
    }
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

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      uint32_t ic = 0, c = 0;  // items, K/V tiles loaded
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
        const AttnPairItem it = attn_pair_item(p, w);
        const int kh = it.h0 / p.group;
        const int row0 = it.b * p.L;
        if (!mbar_wait(q_empty, (ic & 1) ^ 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(q_full, 2 * kAttnTile);
        for (int x = 0; x < 2; ++x) {
          uint8_t* qd = smem + kPpOffQ + x * kAttnTile;
          tma_load_2d(qd, &tmQ, q_full, (it.h0 + x) * 128, row0 + it.qt * 128);
          tma_load_2d(qd + kAttnHalf, &tmQ, q_full, (it.h0 + x) * 128 + 64,
                      row0 + it.qt * 128);
        }
        for (int j = 0; j < it.n && ok; ++j) {
          for (int kv = 0; kv < 2; ++kv, ++c) {  // K_j, then V_j
            const int s = c % kPpRing;
            const uint32_t ph = (c / kPpRing) & 1;
            if (!mbar_wait(&kv_empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
            uint8_t* dst = smem + kPpOffKV + s * kAttnTile;
            const CUtensorMap* tm = kv ? &tmV : &tmK;
            mbar_arrive_expect_tx(&kv_full[s], kAttnTile);
            tma_load_2d(dst, tm, &kv_full[s], kh * 128, row0 + j * 128);
            tma_load_2d(dst + kAttnHalf, tm, &kv_full[s], kh * 128 + 64, row0 + j * 128);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t q_addr[2] = {smem_u32(smem + kPpOffQ), smem_u32(smem + kPpOffQ + kAttnTile)};
      const uint32_t p_addr[2] = {smem_u32(smem + kPpOffP), smem_u32(smem + kPpOffP + kAttnTile)};
      auto kv_addr = [&](uint32_t idx) {
        return smem_u32(smem + kPpOffKV + (idx % kPpRing) * kAttnTile);
      };
      auto kv_wait = [&](uint32_t idx) {
        return mbar_wait(&kv_full[idx % kPpRing], (idx / kPpRing) & 1, abort_flag);
      };
      uint32_t ic = 0, c = 0, t = 0;  // items, K/V tiles consumed, key tiles
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
        const AttnPairItem it = attn_pair_item(p, w);
        if (!mbar_wait(q_full, ic & 1, abort_flag) || !kv_wait(c)) { ok = false; break; }
        tc_fence_after();
        for (int x = 0; x < 2; ++x) {
          attn_qk(tmem_base + x * 128, q_addr[x], kv_addr(c));
          mma_commit(&xb[6 * x + 0]);
        }
        mma_commit(&kv_empty[c % kPpRing]);
        if (it.n == 1) mma_commit(q_empty);
        for (int j = 0; j < it.n && ok; ++j) {
          const uint32_t kidx = c + 2 * j, vidx = kidx + 1, tt = t + j;
          const bool more = j + 1 < it.n;
          if (!kv_wait(vidx)) { ok = false; break; }
          for (int x = 0; x < 2; ++x) {
            uint64_t* X = &xb[6 * x];
            if (!mbar_wait(&X[1], tt & 1, abort_flag) ||
                (j == 0 && !mbar_wait(&X[5], (ic & 1) ^ 1, abort_flag))) {
              ok = false;
              break;
            }
            tc_fence_after();
            attn_pv(tmem_base + 256 + x * 128, p_addr[x], kv_addr(vidx), j > 0);
            mma_commit(&X[2]);
            mma_commit(&X[3]);
            if (j == it.n - 1) mma_commit(&X[4]);
            if (x == 1) mma_commit(&kv_empty[vidx % kPpRing]);
            if (more) {
              if (x == 0 && !kv_wait(kidx + 2)) { ok = false; break; }
              tc_fence_after();
              attn_qk(tmem_base + x * 128, q_addr[x], kv_addr(kidx + 2));
              mma_commit(&X[0]);
              if (x == 1) {
                mma_commit(&kv_empty[(kidx + 2) % kPpRing]);
                if (j + 1 == it.n - 1) mma_commit(q_empty);
              }
            }
          }
        }
        c += 2 * it.n;
        t += it.n;
      }
      // Every MMA issued above must finish before TMEM is released.
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // ------------------------------------------------ softmax / epilogue
    const int x = (warp - 2) >> 2;            // query tile: 0 = A, 1 = B
    const int q = warp & 3;                   // TMEM lane quarter
    const int r = q * 32 + lane;              // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_col = tmem_base + lane_off + x * 128;
    const uint32_t o_col = tmem_base + lane_off + 256 + x * 128;
    uint64_t* X = &xb[6 * x];
    uint8_t* prow = smem + kPpOffP + x * kAttnTile + r * 128;
    const float sl2 = p.scale_log2;
    uint32_t ic = 0, t = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++ic) {
      const AttnPairItem it = attn_pair_item(p, w);
      float m = 0.f, l = 0.f;
      for (int j = 0; j < it.n; ++j) {
        const uint32_t tt = t + j;
        const bool diag = j == it.qt;  // keys after the query row are masked
        const bool ready = mbar_wait(&X[0], tt & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
        tc_fence_after();
        // pass 1: the row max of this key tile
        float mt = -INFINITY;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t u[32];
          tmem_ld32(s_col + c4 * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v =
                (diag && c4 * 32 + i > r) ? -INFINITY : __fmul_rn(__uint_as_float(u[i]), sl2);
            mt = fmaxf(mt, v);
          }
        }
        if (j == 0) {
          m = mt;
        } else if (__any_sync(0xffffffffu, mt > m + kAttnRescale)) {
          // Some row of this warp outgrew its max by more than 2^8: the warp
          // rescales its 32 rows of O_X (alpha = 1 where the max did not
          // grow); PV_X(j-1) must have landed first.
          const float mn = fmaxf(m, mt);
          const float alpha = ex2_approx(m - mn);
          const bool done = mbar_wait(&X[3], (tt - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, done)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t u[32];
            tmem_ld32(o_col + c4 * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
            tmem_st32(o_col + c4 * 32, u);
          }
          tmem_wait_st();
          l *= alpha;
          m = mn;
        }
        // pass 2: P = 2^(s - m) -> shared memory (two 128-byte-swizzled
        // K-major halves), once PV_X(j-1) has read the previous P
        const bool freed = mbar_wait(&X[2], (tt & 1) ^ 1, abort_flag);
        if (!__all_sync(0xffffffffu, freed)) { ok = false; break; }
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t u[32];
          tmem_ld32(s_col + c4 * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int g8 = 0; g8 < 4; ++g8) {
            float e[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int key = c4 * 32 + g8 * 8 + i;
              const float v =
                  (diag && key > r) ? -INFINITY : __fmul_rn(__uint_as_float(u[g8 * 8 + i]), sl2);
              e[i] = ex2_approx(v - m);
              l += e[i];
            }
            uint4 pv;
            pv.x = pack_bf16x2(e[0], e[1]);
            pv.y = pack_bf16x2(e[2], e[3]);
            pv.z = pack_bf16x2(e[4], e[5]);
            pv.w = pack_bf16x2(e[6], e[7]);
            const int cc = c4 * 4 + g8;  // 8-key chunk 0..15
            const int half = cc >> 3, ch = cc & 7;
            *reinterpret_cast<uint4*>(prow + half * kAttnHalf + ((ch ^ (r & 7)) << 4)) = pv;
          }
        }
        fence_async_smem();
        tc_fence_before();  // orders this thread's TMEM reads / a rescale before the PV
        mbar_arrive(&X[1]);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> bf16 row of the output
      const bool fin = mbar_wait(&X[4], ic & 1, abort_flag);
      if (!__all_sync(0xffffffffu, fin)) { ok = false; break; }
      tc_fence_after();
      const float inv = 1.0f / l;
      const int qrow = it.qt * 128 + r;
      __nv_bfloat16* orow = p.out + (static_cast<long long>(it.b) * p.L + qrow) * p.ldo +
                            static_cast<long long>(it.h0 + x) * 128;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t u[32];
        tmem_ld32(o_col + c4 * 32, u);
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
      mbar_arrive(&X[5]);
      t += it.n;
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
