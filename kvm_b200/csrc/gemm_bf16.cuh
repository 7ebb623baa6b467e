// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores.
//
//   warp 0 (one lane)  TMA producer: A and B tiles -> shared-memory ring
//   warp 1 (one lane)  MMA issuer:   tcgen05.mma kind::f16, M=128 x N=BN x K=16
//                      per instruction, accumulator in TMEM (two buffers so the
//                      epilogue of tile i overlaps the main loop of tile i+1)
//   warps 2..5         epilogue:     tcgen05.ld TMEM -> registers -> fused
//                      elementwise work -> global memory
//
// Tiles are 128 x BN x 64 (bf16, 128-byte rows, 128-byte swizzle). The same
// kernel serves a dense GEMM (one group) and the grouped expert GEMM of the
// MoE layer (group g owns rows [off[g], off[g+1]) of A and D and weight
// matrix g of B). Tile order inside a group is N-tile major, so consecutive
// CTAs share the weight tile in L2.
#pragma once

#include <cuda_bf16.h>

#include "ptx.cuh"

namespace kvm {

enum GemmEpilogue : int {
  kEpiBf16 = 0,    // D = bf16(acc [+ C])
  kEpiF32 = 1,     // D = acc [+ C] (fp32)
  kEpiSilu = 2,    // per 128 tile cols: 64 gate, then the 64 up of the same
                   // f (pack_gate_up layout) -> bf16 SiLU(g)*u
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kMaxGroups = 256;

struct GemmParams {
  int M;                 // rows of A / D (dense) or total permuted rows
  int N;                 // columns of the product (per group)
  int K;
  int num_groups;        // 1 for dense
  const int* offsets;    // [num_groups + 1] row offsets (grouped) or null
  int b_group_rows;      // rows of B per group in the B tensor map
  void* D;
  long long ldd;         // elements
  const void* C;         // optional addend (same dtype as D), row stride ldc
  long long ldc;
  int* status;           // device status word
  int split_tiles;       // the last split_tiles tiles run as two half-width
                         // items each (BN >= 128; 0: none)
};

// Where one output tile's operands and results live.
struct GemmTile {
  int row0, row_end, col0;  // rows [row0, row_end) valid; columns from col0
  int a_x, a_y;             // A box at K block kb: (a_x + kb*BK, a_y)
  int b_x, b_y;             // B: K-major (b_x + kb*BK, b_y); MN-major (b_x, b_y + kb*BK)
  int g;
  int nb;                   // columns of this item: BN, or BN / 2 for a half
};

template <int BN>
struct GemmSmem {
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr uint32_t kBBytes = BN * kGemmBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
};

template <int BN, int STAGES>
constexpr size_t gemm_smem_bytes() {
  return 1024 + static_cast<size_t>(STAGES) * GemmSmem<BN>::kStageBytes +
         (2 * STAGES + 5) * 8 + 16 + 3 * (kMaxGroups + 1) * 4;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float bf16_lo(uint32_t v) {
  return __uint_as_float(v << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t v) {
  return __uint_as_float(v & 0xFFFF0000u);
}

__device__ __forceinline__ float silu_f(float g) {
  return g / (1.0f + __expf(-g));
}

// Store 32 consecutive fp32 results of one row as bf16 (or fp32), adding an
// optional C row. `n_valid` (<= 32) columns are in range.
template <bool F32_OUT>
__device__ __forceinline__ void store_row32(void* dst, const void* crow,
                                            const float (&v)[32],
                                            int n_valid) {
  float w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = v[i];
  if (F32_OUT) {
    float* d = static_cast<float*>(dst);
    const float* c = static_cast<const float*>(crow);
    if (n_valid == 32) {
      if (c) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float4 cv = reinterpret_cast<const float4*>(c)[i];
          w[4 * i] += cv.x; w[4 * i + 1] += cv.y;
          w[4 * i + 2] += cv.z; w[4 * i + 3] += cv.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(d)[i] =
            make_float4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n_valid) d[i] = w[i] + (c ? c[i] : 0.0f);
    }
  } else {
    __nv_bfloat16* d = static_cast<__nv_bfloat16*>(dst);
    const __nv_bfloat16* c = static_cast<const __nv_bfloat16*>(crow);
    if (n_valid == 32) {
      if (c) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 cv = reinterpret_cast<const uint4*>(c)[i];
          uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            w[8 * i + 2 * j] += bf16_lo(cw[j]);
            w[8 * i + 2 * j + 1] += bf16_hi(cw[j]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 o;
        o.x = pack_bf16x2(w[8 * i + 0], w[8 * i + 1]);
        o.y = pack_bf16x2(w[8 * i + 2], w[8 * i + 3]);
        o.z = pack_bf16x2(w[8 * i + 4], w[8 * i + 5]);
        o.w = pack_bf16x2(w[8 * i + 6], w[8 * i + 7]);
        reinterpret_cast<uint4*>(d)[i] = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n_valid)
          d[i] = __float2bfloat16_rn(w[i] + (c ? __bfloat162float(c[i]) : 0.f));
    }
  }
}

// Work items: tile t for t below the split point; past it, each remaining
// tile as two items of BN / 2 columns (first half, then second). When the
// last wave of whole tiles would occupy at most half of the SMs, splitting it
// lets the CTAs finish together. tmB2 is B's tensor map with BN / 2-row boxes
// (K-major B; MN-major B loads 64-column boxes and ignores it).
template <int BN, int STAGES, bool B_MN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmB2,
                     const GemmParams p) {
  using S = GemmSmem<BN>;
  constexpr int BM = kGemmBM, BK = kGemmBK;
  constexpr uint32_t kIdesc = idesc_bf16(BM, BN, 0, B_MN ? 1 : 0);
  constexpr uint32_t kIdescHalf = idesc_bf16(BM, BN / 2, 0, B_MN ? 1 : 0);
  constexpr bool kCanSplit = BN >= 128;
  constexpr int TR = BM;  // rows per tile

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;   // [2]
  uint64_t* tempty = tfull + 2;       // [2]
  uint64_t* drain = tempty + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* g_off = reinterpret_cast<int*>(tmem_slot + 4);   // [G+1]
  int* g_pref = g_off + (kMaxGroups + 1);               // [G+1] tile prefix
  int* g_mt = g_pref + (kMaxGroups + 1);                // [G] m-tiles

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int G = p.num_groups;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int k_blocks = (p.K + BK - 1) / BK;

  // ---- setup: group table, barriers, TMEM
  if (threadIdx.x == 0) *abort_flag = 0;
  for (int i = threadIdx.x; i <= G; i += blockDim.x)
    g_off[i] = p.offsets ? p.offsets[i] : (i == 0 ? 0 : p.M);
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    bool bad = false;
    for (int g = 0; g < G; ++g) {
      int lo = g_off[g], hi = g_off[g + 1];
      if (lo < 0 || hi < lo || hi > p.M) {
        bad = true;
        hi = lo = 0;
      }
      int mt = (hi - lo + TR - 1) / TR;
      g_mt[g] = mt;
      g_pref[g] = acc;
      acc += mt * n_tiles;
    }
    g_pref[G] = acc;
    if (bad && p.status) atomicOr(p.status, 2);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (!B_MN && kCanSplit && p.split_tiles > 0) tma_prefetch_desc(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = g_pref[G];
  const int split_first =
      kCanSplit ? total_tiles - min(max(p.split_tiles, 0), total_tiles) : total_tiles;
  const int total_items = 2 * total_tiles - split_first;

  auto map_tile = [&](int t) {
    int lo = 0, hi = G - 1;  // largest g with g_pref[g] <= t
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (g_pref[mid] <= t) lo = mid; else hi = mid - 1;
    }
    const int g = lo;
    const int local = t - g_pref[g];
    const int mt = g_mt[g];
    const int nt = local / mt;
    const int mi = local - nt * mt;
    GemmTile tl;
    tl.g = g;
    tl.row0 = g_off[g] + mi * TR;
    tl.row_end = g_off[g + 1];
    tl.col0 = nt * BN;
    tl.a_x = 0;
    tl.a_y = tl.row0;
    tl.b_x = B_MN ? tl.col0 : 0;
    tl.b_y = g * p.b_group_rows + (B_MN ? 0 : tl.col0);
    tl.nb = BN;
    return tl;
  };
  auto map_item = [&](int i) {
    if (i < split_first) return map_tile(i);
    const int u = i - split_first;
    GemmTile tl = map_tile(split_first + (u >> 1));
    tl.nb = BN / 2;
    if (u & 1) {
      tl.col0 += BN / 2;
      if (B_MN) tl.b_x += BN / 2; else tl.b_y += BN / 2;
    }
    return tl;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int s = 0;
      uint32_t ph = 0;
      uint32_t armed_ph[STAGES];
      bool armed[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) armed[i] = false;
      bool ok = true;
      for (int t = blockIdx.x; t < total_items && ok; t += gridDim.x) {
        const GemmTile tl = map_item(t);
        const bool whole = tl.nb == BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * S::kStageBytes;
          uint8_t* b_dst = a_dst + S::kABytes;
          mbar_arrive_expect_tx(&full[s], TR * (BK * 2) + tl.nb * (BK * 2));
          armed[s] = true;
          armed_ph[s] = ph;
          tma_load_2d(a_dst, &tmA, &full[s], tl.a_x + kb * BK, tl.a_y);
          if (!B_MN) {
            tma_load_2d(b_dst, whole ? &tmB : &tmB2, &full[s], tl.b_x + kb * BK, tl.b_y);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              if (j * 64 < tl.nb)
                tma_load_2d(b_dst + j * (64 * BK * 2), &tmB, &full[s],
                            tl.b_x + j * 64, tl.b_y + kb * BK);
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        // Let copies already in flight land before the CTA exits.
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
      for (int t = blockIdx.x; t < total_items && ok; t += gridDim.x) {
        const uint32_t idesc = t < split_first ? kIdesc : kIdescHalf;
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        ++it;
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * S::kStageBytes);
          const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = sdesc_sw128(a_addr + k * 32, 0, 1024);
            const uint64_t bdesc =
                B_MN ? sdesc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024)
                     : sdesc_sw128(b_addr + k * 32, 0, 1024);
            mma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0);
          }
          mma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) mma_commit(&tfull[acc]);
      }
      // Every MMA issued above must finish before TMEM is released.
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // -------------------------------------------------- epilogue warps
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r_in_tile = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < total_items; t += gridDim.x) {
      const GemmTile tl = map_item(t);
      const int row0 = tl.row0, row_end = tl.row_end, col0 = tl.col0;
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      ++it;
      // tcgen05.ld is warp-collective: the whole warp proceeds or stops.
      const bool ready = mbar_wait(&tfull[acc], aph, abort_flag);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                             acc * BN;
      const int row = row0 + r_in_tile;
      const bool row_ok = row < row_end;

      if constexpr (EPI == kEpiBf16 || EPI == kEpiF32) {
        constexpr bool F32 = EPI == kEpiF32;
        constexpr int ES = F32 ? 4 : 2;
#pragma unroll 1
        for (int c = 0; c < tl.nb / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_row + c * 32, r);
          tmem_wait_ld();
          const int col = col0 + c * 32;
          if (row_ok && col < p.N) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            char* dst = static_cast<char*>(p.D) +
                        (static_cast<long long>(row) * p.ldd + col) * ES;
            const char* crow =
                p.C ? static_cast<const char*>(p.C) +
                          (static_cast<long long>(row) * p.ldc + col) * ES
                    : nullptr;
            store_row32<F32>(dst, crow, v, min(32, p.N - col));
          }
        }
      } else if constexpr (EPI == kEpiSilu) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t rg[32], ru[32];
          const int gcol = (c >> 1) * 128 + (c & 1) * 32;  // gate; up is 64 on
          tmem_ld32(t_row + gcol, rg);
          tmem_ld32(t_row + gcol + 64, ru);
          tmem_wait_ld();
          const int col = col0 / 2 + c * 32;  // output column
          if (row_ok && col < p.N / 2) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i)
              v[i] = silu_f(__uint_as_float(rg[i])) * __uint_as_float(ru[i]);
            char* dst = static_cast<char*>(p.D) +
                        (static_cast<long long>(row) * p.ldd + col) * 2;
            store_row32<false>(dst, nullptr, v, min(32, p.N / 2 - col));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicOr(p.status, 1);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace kvm
