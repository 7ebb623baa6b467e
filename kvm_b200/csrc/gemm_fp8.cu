// FP8 (e4m3) W8A8 GEMM with 128x128 fp32 block scales, and the block
// quantiser that produces its operands.
//
//   D[m, n] = bf16( sum_kb s(kb) * P_kb[m, n] ),   s(kb) = sA[m/128][kb] * sW[n/128][kb]
//   P_kb    = sum_{k in block kb} Aq[m, k] * Wq[n, k]            (fp32, tensor core)
//
// Per 128-deep K block the MMA warp issues four tcgen05.mma kind::f8f6f4
// (128 x BN x 32) into one of NBUF TMEM buffers; eight epilogue warps read the
// buffer, multiply by the block's scale and add into fp32 registers
// (acc = fma(P, s, acc), blocks in ascending order), so the MMA of block kb+1
// overlaps the promotion of block kb. Scales are arbitrary fp32 values, which
// the tensor core's own block scaling (powers of two) cannot represent.
#include <cuda_bf16.h>
#include <cstdlib>
#include <cuda_fp8.h>

#include "ptx.cuh"
#include "runtime.h"

namespace kvm {
namespace {

constexpr int kF8BM = 128;
constexpr int kF8BK = 128;   // bytes == elements
// producer warp, MMA warp, EW epilogue warps (each TMEM lane quarter is read
// by EW/4 warps, one column slice each)
constexpr int f8_threads(int ew) { return 64 + 32 * ew; }

struct Fp8Params {
  int M, N, K;
  const float* sA;   // [ceil(M/128)][K/128]
  const float* sW;   // [N/128][K/128]
  __nv_bfloat16* D;
  long long ldd;
  int* status;
  // Work split. Whole tiles round-robin (CTA c: tiles c, c+G, ...; G =
  // gridDim.x) for all but the last one to two waves' worth of tiles
  // (streamk_first_tile); those are split stream-K: CTA c takes K blocks
  // [c*W/G, (c+1)*W/G) of the tail tiles' K blocks in tile order, so every
  // CTA ends with the same amount of work. Only a CTA's first and last
  // stream-K segments can be parts of a tile cut between CTAs; those are
  // written as fp32 partials (slot 2c for the first, 2c + 1 for the last)
  // and summed by fp8_streamk_reduce_kernel. stream_k == 0: round-robin only.
  int stream_k;
  float* partial;    // [G][2][128][128] fp32
};

// Operand tiles of one 128-deep K block. TN == 0: A = 128 activation rows,
// B = 128 weight rows, D[act row][weight col] in TMEM lanes x columns.
// TN > 0 (M <= TN <= 64): A = 128 weight rows, B = TN activation rows (the
// token count as the MMA's N), D^T in TMEM (lane = weight row = output
// column, column = token).
template <int STAGES, int NBUF, int TN>
struct Fp8Smem {
  static constexpr uint32_t kABytes = 128 * kF8BK;
  static constexpr uint32_t kBBytes = (TN ? TN : 128) * kF8BK;
  static constexpr uint32_t kStage = kABytes + kBBytes;
  static constexpr uint32_t kAccCols = TN ? TN : 128;
  static constexpr uint32_t kTmemCols =
      NBUF * kAccCols <= 32 ? 32 : NBUF * kAccCols <= 64 ? 64 : NBUF * kAccCols <= 128
          ? 128 : NBUF * kAccCols <= 256 ? 256 : 512;
  static constexpr size_t kTotal =
      1024 + static_cast<size_t>(STAGES) * kStage + (2 * STAGES + 2 * NBUF + 1) * 8 + 16;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// First tile of the stream-K tail: all tiles when there are fewer than two
// waves, else all but the last one to two waves (the earlier waves keep the
// round-robin order, whose concurrent tiles share weight tiles in L2).
__host__ __device__ __forceinline__ int streamk_first_tile(int tiles, int ctas) {
  return tiles >= 2 * ctas ? (tiles / ctas - 1) * ctas : 0;
}

// The segments (tile, K blocks [kb0, kb1)) a CTA works through, in order:
// round-robin whole tiles below t0, then its stream-K range of the tail.
struct Fp8Segments {
  long long x, hi;   // stream-K: next K-block index of the tail, end of the range
  int t, t0, tiles, step, kbs;
  __device__ Fp8Segments(const Fp8Params& p, int tiles_, int kbs_)
      : tiles(tiles_), step(static_cast<int>(gridDim.x)), kbs(kbs_) {
    t0 = p.stream_k ? streamk_first_tile(tiles_, step) : tiles_;
    const long long W = static_cast<long long>(tiles_ - t0) * kbs_;
    x = W * blockIdx.x / gridDim.x;
    hi = W * (blockIdx.x + 1) / gridDim.x;
    t = static_cast<int>(blockIdx.x);
  }
  // stream-K segments are the ones with tile >= t0
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (t < t0) {
      tile = t;
      kb0 = 0;
      kb1 = kbs;
      t += step;
      return true;
    }
    if (x >= hi) return false;
    const int u = static_cast<int>(x / kbs);
    tile = t0 + u;
    kb0 = static_cast<int>(x - static_cast<long long>(u) * kbs);
    kb1 = static_cast<int>(min(static_cast<long long>(kbs), kb0 + (hi - x)));
    x += kb1 - kb0;
    return true;
  }
};

template <int STAGES, int NBUF, int EW, int TN>
__global__ void __launch_bounds__(f8_threads(EW), 1)
    gemm_fp8_bs_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB,
                       const Fp8Params p) {
  using S = Fp8Smem<STAGES, NBUF, TN>;
  constexpr int BN = 128;
  static_assert(TN == 0 ? EW == 8 : EW == 4, "8 epilogue warps, or 4 in the swapped form");
  static_assert(TN % 16 == 0 && TN <= 64, "swapped form: N = 16, 32, 48 or 64 tokens");
  constexpr uint32_t kIdesc = idesc_e4m3(128, TN ? TN : BN, 0, 0);
  constexpr int COLS = TN ? TN : BN / (EW / 4);  // accumulator columns per thread

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStage);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* drain = tempty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m_tiles = (p.M + kF8BM - 1) / kF8BM;
  const int tiles = m_tiles * (p.N / BN);
  const int kbs = p.K / kF8BK;
  // tile t: N tile t / m_tiles (weight-major, so the M tiles of one weight
  // tile run back to back and share it in L2), M tile t % m_tiles

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 32 * EW);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      Fp8Segments seg(p, tiles, kbs);
      int tile, kb0, kb1;
      while (ok && seg.next(tile, kb0, kb1)) {
        const int nt = tile / m_tiles, mt = tile - (tile / m_tiles) * m_tiles;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * S::kStage;
          mbar_arrive_expect_tx(&full[s], S::kStage);
          if (TN) {  // A = weights, B = the (only) M tile of activations
            tma_load_2d(a_dst, &tmB, &full[s], kb * kF8BK, nt * BN);
            tma_load_2d(a_dst + S::kABytes, &tmA, &full[s], kb * kF8BK, 0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[s], kb * kF8BK, mt * kF8BM);
            tma_load_2d(a_dst + S::kABytes, &tmB, &full[s], kb * kF8BK, nt * BN);
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for every stage's last armed load to land.
        volatile int local_abort = 0;
        for (int i = 0; i < STAGES; ++i) {
          const uint32_t par = (i < s) ? ph : (ph ^ 1);
          mbar_wait(&full[i], par, &local_abort);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      uint32_t g = 0;  // K blocks issued so far (selects the TMEM buffer)
      bool ok = true;
      Fp8Segments seg(p, tiles, kbs);
      int tile, kb0, kb1;
      while (ok && seg.next(tile, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const uint32_t b = g % NBUF, bph = (g / NBUF) & 1;
          if (!mbar_wait(&tempty[b], bph ^ 1, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * S::kStage);
          const uint32_t b_addr = a_addr + S::kABytes;
          const uint32_t d = tmem_base + b * S::kAccCols;
#pragma unroll
          for (int k = 0; k < kF8BK / 32; ++k)
            mma_f8_ss(d, sdesc_sw128(a_addr + k * 32, 0, 1024),
                      sdesc_sw128(b_addr + k * 32, 0, 1024), kIdesc, k != 0);
          mma_commit(&empty[s]);
          mma_commit(&tfull[b]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // epilogue: warp quarter q owns TMEM lanes [32q, 32q+32); slice h owns
    // accumulator columns [h*COLS, (h+1)*COLS).
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int r_in = q * 32 + lane;  // TMEM lane: activation row, or weight row if TN
    uint32_t g = 0;
    bool ok = true;
    Fp8Segments seg(p, tiles, kbs);
    int tile, kb0, kb1, si = 0;  // si: stream-K segments so far
    while (ok && seg.next(tile, kb0, kb1)) {
      const int nt = tile / m_tiles, mt = tile - nt * m_tiles;
      float acc[COLS];
#pragma unroll
      for (int j = 0; j < COLS; ++j) acc[j] = 0.f;
      const float* sa = p.sA + static_cast<long long>(mt) * kbs;
      const float* sw = p.sW + static_cast<long long>(nt) * kbs;
      // The tile's block scales s(kb) = sA * sW, 32 K blocks at a time: lane l
      // loads block kb0 + 32c + l before the wait, a shuffle hands each block
      // its scale (no global-load latency inside the loop).
      float sc_lane = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int j32 = (kb - kb0) & 31;
        if (j32 == 0) {
          const int kk = kb + lane;
          sc_lane = kk < kb1 ? __ldg(sa + kk) * __ldg(sw + kk) : 0.f;
        }
        const uint32_t b = g % NBUF, bph = (g / NBUF) & 1;
        const bool ready = mbar_wait(&tfull[b], bph, abort_flag);
        if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               b * S::kAccCols + h * COLS;
        uint32_t v[COLS];
        if constexpr (COLS % 32 == 0) {
#pragma unroll
          for (int c = 0; c < COLS / 32; ++c)
            tmem_ld32(taddr + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&v[32 * c]));
        } else {
#pragma unroll
          for (int c = 0; c < COLS / 16; ++c)
            tmem_ld16(taddr + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(&v[16 * c]));
        }
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&tempty[b]);
        const float sc = __shfl_sync(0xffffffffu, sc_lane, j32);
        // Two columns per instruction (packed fp32 FMA, round to nearest:
        // the same result as two scalar fmaf_rn).
        const float2 sc2 = make_float2(sc, sc);
#pragma unroll
        for (int j = 0; j < COLS; j += 2) {
          const float2 r = __ffma2_rn(
              make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), sc2,
              make_float2(acc[j], acc[j + 1]));
          acc[j] = r.x;
          acc[j + 1] = r.y;
        }
      }
      if (!ok) break;
      const bool whole = kb0 == 0 && kb1 == kbs;
      float* part = whole ? nullptr
                          : p.partial + (static_cast<long long>(blockIdx.x) * 2 + (si ? 1 : 0)) *
                                            (kF8BM * BN);
      if (tile >= seg.t0) ++si;
      if (TN) {
        // thread = output column nt*128 + r_in; acc[m] = token m (M <= TN)
        const int col = nt * BN + r_in;
#pragma unroll
        for (int m = 0; m < COLS; ++m) {
          if (m >= p.M) break;
          if (whole)
            p.D[static_cast<long long>(m) * p.ldd + col] = __float2bfloat16_rn(acc[m]);
          else
            part[m * BN + r_in] = acc[m];
        }
      } else {
        const int row = mt * kF8BM + r_in;
        if (row < p.M) {
          if (!whole) {  // fp32 partial [128 rows][128 cols], valid rows only
            float4* dst = reinterpret_cast<float4*>(part + r_in * BN + h * COLS);
#pragma unroll
            for (int i = 0; i < COLS / 4; ++i)
              dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
          } else {
            uint4* dst = reinterpret_cast<uint4*>(
                p.D + static_cast<long long>(row) * p.ldd + nt * BN + h * COLS);
#pragma unroll
            for (int i = 0; i < COLS / 8; ++i)
              dst[i] = make_uint4(pack_bf16x2(acc[8 * i], acc[8 * i + 1]),
                                  pack_bf16x2(acc[8 * i + 2], acc[8 * i + 3]),
                                  pack_bf16x2(acc[8 * i + 4], acc[8 * i + 5]),
                                  pack_bf16x2(acc[8 * i + 6], acc[8 * i + 7]));
          }
        }
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicOr(p.status, kDevWaitTimeout);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// The CTA whose stream-K range holds K-block index x (of W over G CTAs).
__device__ __forceinline__ int streamk_cta(long long x, long long W, int G) {
  return static_cast<int>(((x + 1) * G - 1) / W);
}

// Tiles cut between CTAs: sum the CTAs' fp32 partials in CTA order (= K
// order), round to bf16. One thread per 8 outputs; tiles held whole by one
// CTA were written by the GEMM and are skipped.
__global__ void fp8_streamk_reduce_kernel(const float* __restrict__ partial,
                                          __nv_bfloat16* __restrict__ D, long long ldd,
                                          int M, int N, int kbs, int G) {
  const long long i = (blockIdx.x * 256ll + threadIdx.x) * 8;
  if (i >= static_cast<long long>(M) * N) return;
  const int row = static_cast<int>(i / N), col = static_cast<int>(i % N);
  const int m_tiles = (M + kF8BM - 1) / kF8BM;
  const int tiles = m_tiles * (N / 128);
  const int t0 = streamk_first_tile(tiles, G);
  const long long u = static_cast<long long>(col / 128) * m_tiles + row / kF8BM - t0;
  if (u < 0) return;  // a round-robin tile
  const long long W = static_cast<long long>(tiles - t0) * kbs;
  const int c_lo = streamk_cta(u * kbs, W, G);
  const int c_hi = streamk_cta(u * kbs + kbs - 1, W, G);
  if (c_lo == c_hi) return;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int c = c_lo; c <= c_hi; ++c) {
    const long long first = (W * c / G) / kbs;  // first tail tile of CTA c
    const long long slot = static_cast<long long>(c) * 2 + (u == first ? 0 : 1);
    const float* src = partial + (slot * kF8BM + row % kF8BM) * 128 + col % 128;
    const float4 x = reinterpret_cast<const float4*>(src)[0];
    const float4 y = reinterpret_cast<const float4*>(src)[1];
    a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
    a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
  }
  *reinterpret_cast<uint4*>(D + static_cast<long long>(row) * ldd + col) =
      make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                 pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
}

// Whether stream-K over `ctas` CTAs cuts any tile of the tail (tiles from
// streamk_first_tile on) between two CTAs (then partials and a reduction
// are needed).
bool streamk_cuts(int tiles_all, int kbs, int ctas) {
  const long long tiles = tiles_all - streamk_first_tile(tiles_all, ctas);
  const long long W = tiles * kbs;
  for (int c = 1; c < ctas; ++c)
    if ((W * c / ctas) % kbs != 0) return true;
  return false;
}

// 128x128 block quantiser: one block of 256 threads per 128x128 tile.
// s = amax / 448 (1 when the tile is all zeros); q = e4m3_rn_satfinite(x / s)
// with an IEEE (correctly rounded) division.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__global__ void __launch_bounds__(256)
    quantize_e4m3_block128_kernel(const T* __restrict__ x, uint8_t* __restrict__ q,
                                  float* __restrict__ scales, int R, int C) {
  __shared__ float red[8];
  const int br = blockIdx.y, bc = blockIdx.x;
  const int sc_cols = (C + 127) / 128;
  const int r0 = br * 128, c0 = bc * 128;
  float amax = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < R && c < C)
      amax = fmaxf(amax, fabsf(to_f32(x[static_cast<long long>(r) * C + c])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  const float s = m > 0.f ? __fdiv_rn(m, 448.0f) : 1.0f;
  if (threadIdx.x == 0) scales[static_cast<long long>(br) * sc_cols + bc] = s;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < R && c < C) {
      const long long o = static_cast<long long>(r) * C + c;
      const float v = __fdiv_rn(to_f32(x[o]), s);
      q[o] = static_cast<uint8_t>(
          __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
    }
  }
}

__global__ void transpose_u8_kernel(const uint8_t* __restrict__ in,
                                    uint8_t* __restrict__ out, int R, int C) {
  __shared__ uint8_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = in[static_cast<long long>(r) * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) out[static_cast<long long>(c) * R + r] = tile[threadIdx.x][i];
  }
}

__global__ void transpose_f32_kernel(const float* __restrict__ in,
                                     float* __restrict__ out, int R, int C) {
  const long long i = blockIdx.x * 256ll + threadIdx.x;
  if (i < static_cast<long long>(R) * C) {
    const long long r = i / C, c = i % C;
    out[c * R + r] = in[i];
  }
}

#define KVM_TRY(expr)                      \
  do {                                     \
    int kvm_rc_ = (expr);                  \
    if (kvm_rc_ != KVM_OK) return kvm_rc_; \
  } while (0)

}  // namespace
}  // namespace kvm

using namespace kvm;

namespace kvm {
namespace {

// Launch geometry of one FP8 GEMM: the swapped form for M <= 64, stream-K
// over min(SMs, K blocks) CTAs.
struct Fp8Plan {
  int tn;         // 0, or the swapped form's token tile (16, 32, 64)
  int tiles, kbs, ctas;
  bool use_sk;        // stream-K at all (else whole tiles round-robin)
  bool cuts;          // stream-K cuts tiles: partials + reduction
  int64_t workspace;  // bytes of fp32 partials stream-K needs (0: none)
};

Fp8Plan fp8_plan(int M, int N, int K, int sms) {
  Fp8Plan pl;
  pl.tn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 0;
  pl.tiles = ((M + kF8BM - 1) / kF8BM) * (N / 128);
  pl.kbs = K / kF8BK;
  const long long W = static_cast<long long>(pl.tiles) * pl.kbs;
  pl.ctas = static_cast<int>(W < sms ? W : sms);
  // The swapped form always balances its K blocks stream-K (its CTAs stream
  // weights at a rate set by their bytes in flight, so equal shares pay);
  // the 128-row form only when its tiles do not fill the SMs: measured at
  // M = 128 (224 tiles), round-robin 64.4 us against 66.2 us stream-K.
  pl.use_sk = pl.tn != 0 || pl.tiles < pl.ctas;
  pl.cuts = pl.use_sk && streamk_cuts(pl.tiles, pl.kbs, pl.ctas);
  pl.workspace = pl.cuts ? static_cast<int64_t>(pl.ctas) * 2 * kF8BM * 128 * 4 : 0;
  return pl;
}

template <int STAGES, int NBUF, int EW, int TN>
int launch_fp8(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8Params& p, int grid,
               cudaStream_t stream) {
  auto kern = gemm_fp8_bs_kernel<STAGES, NBUF, EW, TN>;
  constexpr size_t smem = Fp8Smem<STAGES, NBUF, TN>::kTotal;
  static_assert(smem <= 227 * 1024, "shared memory");
  KVM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  kern<<<grid, f8_threads(EW), smem, stream>>>(ta, tb, p);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int64_t kvm_sm100_gemm_fp8_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 128 != 0) return 0;
  const DeviceInfo* dev = device_info();
  return fp8_plan(M, N, K, dev ? dev->sm_count : 148).workspace;
}

extern "C" int kvm_sm100_gemm_fp8_blockscaled(const void* Aq, const float* sA,
                                              const void* Wq, const float* sW,
                                              void* D, int64_t ldd, int M,
                                              int N, int K, void* workspace,
                                              int64_t workspace_bytes,
                                              kvm_stream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 128 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "fp8 gemm: need M > 0, K % 128 == 0 and N % 128 == 0");
  if (!Aq || !Wq || !sA || !sW || !D || !aligned16(Aq) || !aligned16(Wq) ||
      !aligned16(D) || ldd < N || (ldd * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG, "fp8 gemm: NULL or unaligned operand");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Fp8Plan pl = fp8_plan(M, N, K, dev->sm_count);
  // Stream-K needs room for the partials; without it each CTA takes whole
  // tiles in turn.
  const bool stream_k = pl.use_sk && (!pl.cuts || (workspace && workspace_bytes >= pl.workspace &&
                                                    aligned16(workspace)));
  Fp8Params p{M, N, K, sA, sW, static_cast<__nv_bfloat16*>(D), ldd, dev->status,
              stream_k ? 1 : 0, static_cast<float*>(workspace)};
  const int grid = stream_k ? pl.ctas : (pl.tiles < dev->sm_count ? pl.tiles : dev->sm_count);
  const int a_rows = pl.tn ? pl.tn : kF8BM;  // activation rows one TMA box holds
  CUtensorMap ta, tb;
  KVM_TRY(encode_tmap_2d(&ta, Aq, K, M, K, kF8BK, a_rows,
                         CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tb, Wq, K, N, K, kF8BK, 128,
                         CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
  int rc;
  switch (pl.tn) {
    case 16: rc = launch_fp8<11, 8, 4, 16>(ta, tb, p, grid, st); break;
    case 32: rc = launch_fp8<10, 8, 4, 32>(ta, tb, p, grid, st); break;
    case 64: rc = launch_fp8<8, 4, 4, 64>(ta, tb, p, grid, st); break;
    default: rc = launch_fp8<6, 4, 8, 0>(ta, tb, p, grid, st); break;
  }
  if (rc != KVM_OK) return rc;
  if (stream_k && pl.cuts) {
    const long long n8 = (static_cast<long long>(M) * N) / 8;
    fp8_streamk_reduce_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, st>>>(
        static_cast<const float*>(workspace), static_cast<__nv_bfloat16*>(D), ldd, M, N,
        pl.kbs, grid);
    KVM_CUDA_TRY(cudaGetLastError());
  }
  return KVM_OK;
}

extern "C" int kvm_sm100_quantize_e4m3_block128(const void* x, int x_dtype,
                                                void* q, float* scales, int R,
                                                int C, kvm_stream_t stream) {
  if (R <= 0 || C <= 0 || !x || !q || !scales)
    return fail(KVM_ERR_INVALID_ARG, "quantize: bad shape or NULL pointer");
  dim3 grid((C + 127) / 128, (R + 127) / 128);
  if (grid.y > 65535) return fail(KVM_ERR_INVALID_ARG, "quantize: too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == KVM_F32)
    quantize_e4m3_block128_kernel<float><<<grid, 256, 0, st>>>(
        static_cast<const float*>(x), static_cast<uint8_t*>(q), scales, R, C);
  else if (x_dtype == KVM_BF16)
    quantize_e4m3_block128_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<uint8_t*>(q), scales, R, C);
  else
    return fail(KVM_ERR_INVALID_ARG, "quantize: x_dtype must be bf16 or f32");
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_transpose_u8(const void* in, void* out, int R, int C,
                                      kvm_stream_t stream) {
  if (R <= 0 || C <= 0 || !in || !out)
    return fail(KVM_ERR_INVALID_ARG, "transpose_u8: bad shape or NULL pointer");
  dim3 grid((C + 31) / 32, (R + 31) / 32);
  transpose_u8_kernel<<<grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(in), static_cast<uint8_t*>(out), R, C);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_transpose_f32(const float* in, float* out, int R, int C,
                                       kvm_stream_t stream) {
  if (R <= 0 || C <= 0 || !in || !out)
    return fail(KVM_ERR_INVALID_ARG, "transpose_f32: bad shape or NULL pointer");
  const long long n = static_cast<long long>(R) * C;
  transpose_f32_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(in, out, R, C);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
