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
#include <cuda_fp8.h>

#include "ptx.cuh"
#include "runtime.h"

namespace kvm {
namespace {

constexpr int kF8BM = 128;
constexpr int kF8BK = 128;   // bytes == elements
constexpr int kF8Threads = 320;  // producer, MMA, 8 epilogue warps

struct Fp8Params {
  int M, N, K;
  const float* sA;   // [ceil(M/128)][K/128]
  const float* sW;   // [N/128][K/128]
  __nv_bfloat16* D;
  long long ldd;
  int* status;
  int splits;        // > 1: the K blocks of each tile are split over `splits`
  float* partial;    //      work units; each writes an fp32 partial tile here
};

template <int BN, int STAGES, int NBUF>
struct Fp8Smem {
  static constexpr uint32_t kABytes = kF8BM * kF8BK;
  static constexpr uint32_t kBBytes = BN * kF8BK;
  static constexpr uint32_t kStage = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = NBUF * BN;
  static constexpr size_t kTotal =
      1024 + static_cast<size_t>(STAGES) * kStage + (2 * STAGES + 2 * NBUF + 1) * 8 + 16;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int BN, int STAGES, int NBUF>
__global__ void __launch_bounds__(kF8Threads, 1)
    gemm_fp8_bs_kernel(const __grid_constant__ CUtensorMap tmA,
                       const __grid_constant__ CUtensorMap tmB,
                       const Fp8Params p) {
  using S = Fp8Smem<BN, STAGES, NBUF>;
  static_assert(BN == 128, "scales assume one 128-column block per tile");
  constexpr uint32_t kIdesc = idesc_e4m3(kF8BM, BN, 0, 0);
  constexpr int HALF = BN / 2;

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
  const int n_tiles = p.N / BN;
  const int splits = p.splits > 1 ? p.splits : 1;
  const int total = m_tiles * n_tiles * splits;
  const int kbs = p.K / kF8BK;
  // unit t: tile t / splits (N-tile major), K blocks [kb0, kb1) of split t % splits
  auto unit = [&](int t, int& nt, int& mt, int& kb0, int& kb1) {
    const int tile = t / splits, sp = t - tile * splits;
    nt = tile / m_tiles;
    mt = tile - nt * m_tiles;
    kb0 = static_cast<int>(static_cast<long long>(sp) * kbs / splits);
    kb1 = static_cast<int>(static_cast<long long>(sp + 1) * kbs / splits);
  };

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 256);
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
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int nt, mt, kb0, kb1;
        unit(t, nt, mt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) { ok = false; break; }
          uint8_t* a_dst = smem + s * S::kStage;
          mbar_arrive_expect_tx(&full[s], S::kStage);
          tma_load_2d(a_dst, &tmA, &full[s], kb * kF8BK, mt * kF8BM);
          tma_load_2d(a_dst + S::kABytes, &tmB, &full[s], kb * kF8BK, nt * BN);
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
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int nt, mt, kb0, kb1;
        unit(t, nt, mt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const uint32_t b = g % NBUF, bph = (g / NBUF) & 1;
          if (!mbar_wait(&tempty[b], bph ^ 1, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&full[s], ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * S::kStage);
          const uint32_t b_addr = a_addr + S::kABytes;
          const uint32_t d = tmem_base + b * BN;
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
    // epilogue: warp quarter q owns TMEM lanes [32q, 32q+32); half h owns
    // columns [h*BN/2, (h+1)*BN/2).
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int r_in = q * 32 + lane;
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int nt, mt, kb0, kb1;
      unit(t, nt, mt, kb0, kb1);
      const int row = mt * kF8BM + r_in;
      float acc[HALF];
#pragma unroll
      for (int j = 0; j < HALF; ++j) acc[j] = 0.f;
      const float* sa = p.sA + static_cast<long long>(mt) * kbs;
      const float* sw = p.sW + static_cast<long long>(nt) * kbs;
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const uint32_t b = g % NBUF, bph = (g / NBUF) & 1;
        const bool ready = mbar_wait(&tfull[b], bph, abort_flag);
        if (!__all_sync(0xffffffffu, ready)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               b * BN + h * HALF;
        uint32_t v[HALF];
        uint32_t (&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[0]);
        uint32_t (&v1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&v[32]);
        tmem_ld32(taddr, v0);
        tmem_ld32(taddr + 32, v1);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&tempty[b]);
        const float sc = __ldg(sa + kb) * __ldg(sw + kb);
#pragma unroll
        for (int j = 0; j < HALF; ++j)
          acc[j] = __fmaf_rn(__uint_as_float(v[j]), sc, acc[j]);
      }
      if (!ok) break;
      if (splits > 1) {
        if (row < p.M) {  // fp32 partial [unit][128 rows][BN], valid rows only
          float4* dst = reinterpret_cast<float4*>(
              p.partial + (static_cast<long long>(t) * kF8BM + r_in) * BN + h * HALF);
#pragma unroll
          for (int i = 0; i < HALF / 4; ++i)
            dst[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
        }
      } else if (row < p.M) {
        uint4* dst = reinterpret_cast<uint4*>(
            p.D + static_cast<long long>(row) * p.ldd + nt * BN + h * HALF);
#pragma unroll
        for (int i = 0; i < HALF / 8; ++i)
          dst[i] = make_uint4(pack_bf16x2(acc[8 * i], acc[8 * i + 1]),
                              pack_bf16x2(acc[8 * i + 2], acc[8 * i + 3]),
                              pack_bf16x2(acc[8 * i + 4], acc[8 * i + 5]),
                              pack_bf16x2(acc[8 * i + 6], acc[8 * i + 7]));
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

// Sum of the split partials in split order, to bf16: one thread per 8 outputs.
__global__ void fp8_split_reduce_kernel(const float* __restrict__ partial,
                                        __nv_bfloat16* __restrict__ D, long long ldd,
                                        int M, int N, int m_tiles, int splits, int BN) {
  const long long i = (blockIdx.x * 256ll + threadIdx.x) * 8;
  if (i >= static_cast<long long>(M) * N) return;
  const int row = static_cast<int>(i / N), col = static_cast<int>(i % N);
  const int nt = col / BN, mt = row / kF8BM;
  const long long tile = static_cast<long long>(nt) * m_tiles + mt;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int sp = 0; sp < splits; ++sp) {
    const float* src = partial + ((tile * splits + sp) * kF8BM + row % kF8BM) * BN + col % BN;
    const float4 x = reinterpret_cast<const float4*>(src)[0];
    const float4 y = reinterpret_cast<const float4*>(src)[1];
    a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
    a[4] += y.x; a[5] += y.y; a[6] += y.z; a[7] += y.w;
  }
  *reinterpret_cast<uint4*>(D + static_cast<long long>(row) * ldd + col) =
      make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                 pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
}

// K splits so that every SM gets a work unit when there are fewer output
// tiles than SMs; with at least one tile per SM the partial traffic costs more
// than the balance gains (measured at M = 16 and 128 with N = 28672).
int choose_splits(int tiles, int kbs, int sms) {
  if (tiles >= sms) return 1;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 8 && kbs / s >= 4; ++s) {
    const long long units = static_cast<long long>(tiles) * s;
    const long long waves = (units + sms - 1) / sms;
    const double eff = static_cast<double>(units) / (waves * sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
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

extern "C" int64_t kvm_sm100_gemm_fp8_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 128 != 0) return 0;
  const DeviceInfo* dev = device_info();
  const int sms = dev ? dev->sm_count : 148;
  const int tiles = ((M + kF8BM - 1) / kF8BM) * (N / 128);
  const int splits = choose_splits(tiles, K / kF8BK, sms);
  return splits > 1 ? static_cast<int64_t>(tiles) * splits * kF8BM * 128 * 4 : 0;
}

extern "C" int kvm_sm100_gemm_fp8_blockscaled(const void* Aq, const float* sA,
                                              const void* Wq, const float* sW,
                                              void* D, int64_t ldd, int M,
                                              int N, int K, void* workspace,
                                              int64_t workspace_bytes,
                                              kvm_stream_t stream) {
  constexpr int BN = 128, STAGES = 6, NBUF = 4;
  if (M <= 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % BN != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "fp8 gemm: need M > 0, K % 128 == 0 and N % 128 == 0");
  if (!Aq || !Wq || !sA || !sW || !D || !aligned16(Aq) || !aligned16(Wq) ||
      !aligned16(D) || ldd < N || (ldd * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG, "fp8 gemm: NULL or unaligned operand");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  CUtensorMap ta, tb;
  KVM_TRY(encode_tmap_2d(&ta, Aq, K, M, K, kF8BK, kF8BM,
                         CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tb, Wq, K, N, K, kF8BK, BN,
                         CU_TENSOR_MAP_DATA_TYPE_UINT8, CU_TENSOR_MAP_SWIZZLE_128B));
  const int m_tiles = (M + kF8BM - 1) / kF8BM;
  const int tiles = m_tiles * (N / BN);
  int splits = choose_splits(tiles, K / kF8BK, dev->sm_count);
  const int64_t need = static_cast<int64_t>(tiles) * splits * kF8BM * BN * 4;
  if (splits > 1 && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    splits = 1;  // no room for partials: one unit per tile
  Fp8Params p{M, N, K, sA, sW, static_cast<__nv_bfloat16*>(D), ldd, dev->status,
              splits, static_cast<float*>(workspace)};
  const int units = tiles * splits;
  const int grid = units < dev->sm_count ? units : dev->sm_count;
  auto kern = gemm_fp8_bs_kernel<BN, STAGES, NBUF>;
  constexpr size_t smem = Fp8Smem<BN, STAGES, NBUF>::kTotal;
  KVM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  kern<<<grid, kF8Threads, smem, static_cast<cudaStream_t>(stream)>>>(ta, tb, p);
  KVM_CUDA_TRY(cudaGetLastError());
  if (splits > 1) {
    const long long n8 = (static_cast<long long>(M) * N) / 8;
    fp8_split_reduce_kernel<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0,
                              static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(workspace), static_cast<__nv_bfloat16*>(D), ldd, M, N,
        m_tiles, splits, BN);
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
