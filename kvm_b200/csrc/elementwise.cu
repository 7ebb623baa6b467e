// Bandwidth-bound kernels: RMSNorm, SiLU(g)*u, and the one-time weight
// re-layouts (transpose, gate/up packing) that feed the tcgen05 GEMMs.
// All loads and stores are 16-byte vectors over contiguous rows.
#include <cuda_bf16.h>

#include "runtime.h"

namespace kvm {
namespace {

__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]),
                    pack2(f[6], f[7]));
}

constexpr int kNormThreads = 256;
constexpr int kNormMaxVecs = 4;  // row cached in registers up to 8192 bf16

// One block per row. Sum of squares in fp32 (per-thread partials, then warp
// shuffles, then across warps), scale = rsqrt(sum / H + eps).
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const uint4* __restrict__ x, const uint4* __restrict__ gamma,
                   uint4* __restrict__ y, int row_vecs, float inv_h,
                   float eps) {
  __shared__ float partial[kNormThreads / 32];
  const long long row = blockIdx.x;
  const uint4* xr = x + row * row_vecs;
  uint4 cache[kNormMaxVecs];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVecs; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < row_vecs) {
      cache[i] = __ldg(xr + v);
      float f[8];
      unpack8(cache[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fmaf_rn(f[j], f[j], ss);
    }
  }
  for (int v = threadIdx.x + kNormMaxVecs * kNormThreads; v < row_vecs;
       v += kNormThreads) {
    float f[8];
    unpack8(__ldg(xr + v), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __fmaf_rn(f[j], f[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) partial[threadIdx.x / 32] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += partial[w];
  const float scale = rsqrtf(tot * inv_h + eps);

  uint4* yr = y + row * row_vecs;
  auto emit = [&](int v, uint4 xv) {
    float f[8];
    unpack8(xv, f);
    if (gamma) {
      float g[8];
      unpack8(__ldg(gamma + v), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * scale * g[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * scale;
    }
    yr[v] = pack8(f);
  };
#pragma unroll
  for (int i = 0; i < kNormMaxVecs; ++i) {
    const int v = threadIdx.x + i * kNormThreads;
    if (v < row_vecs) emit(v, cache[i]);
  }
  for (int v = threadIdx.x + kNormMaxVecs * kNormThreads; v < row_vecs;
       v += kNormThreads)
    emit(v, __ldg(xr + v));
}

__global__ void __launch_bounds__(256)
    silu_mul_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u,
                    uint4* __restrict__ h, long long n_vecs) {
  for (long long v = blockIdx.x * 256ll + threadIdx.x; v < n_vecs;
       v += static_cast<long long>(gridDim.x) * 256) {
    float gf[8], uf[8], o[8];
    unpack8(__ldg(g + v), gf);
    unpack8(__ldg(u + v), uf);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = gf[j] / (1.0f + __expf(-gf[j])) * uf[j];
    h[v] = pack8(o);
  }
}

// Transpose G matrices in[g] [R, C] -> out[g] rows, out row of input column c
// given by out_row(c). 32x32 tiles through shared memory; both the global
// reads (along C) and the writes (along R) are coalesced.
//   mode 0: out_row(c) = c,            out rows per group = C
//   mode 1: gate/up interleave: out_row(c) = (c/64)*128 + which*64 + c%64,
//           out rows per group = 2C
__global__ void transpose_kernel(const uint16_t* __restrict__ in,
                                 uint16_t* __restrict__ out, int R, int C,
                                 int mode, int which, long long out_group) {
  __shared__ uint16_t tile[32][33];
  const int g = blockIdx.z;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const uint16_t* src = in + static_cast<long long>(g) * R * C;
  uint16_t* dst = out + g * out_group;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = src[static_cast<long long>(r) * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) {
      const long long orow =
          mode == 0 ? c : (c / 64) * 128 + which * 64 + (c % 64);
      dst[orow * R + r] = tile[threadIdx.x][i];
    }
  }
}

// Gate/up interleave for weights already stored [G, F, K]: row copies.
__global__ void pack_rows_kernel(const uint4* __restrict__ wg,
                                 const uint4* __restrict__ wu,
                                 uint4* __restrict__ out, int F, int row_vecs,
                                 long long total_vecs) {
  for (long long v = blockIdx.x * 256ll + threadIdx.x; v < total_vecs;
       v += static_cast<long long>(gridDim.x) * 256) {
    const long long orow = v / row_vecs;  // row of out, over all groups
    const int col = static_cast<int>(v - orow * row_vecs);
    const long long g = orow / (2ll * F);
    const int r = static_cast<int>(orow - g * 2ll * F);
    const int blk = r / 128, i = r % 128;
    const int f = blk * 64 + (i % 64);
    const uint4* src = i < 64 ? wg : wu;
    out[v] = __ldg(src + (g * F + f) * row_vecs + col);
  }
}

int grid_for(long long n_vecs, int sm_count) {
  long long b = (n_vecs + 255) / 256;
  long long cap = static_cast<long long>(sm_count) * 16;
  return static_cast<int>(b < cap ? (b > 0 ? b : 1) : cap);
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int kvm_sm100_rmsnorm_bf16(const void* x, const void* gamma,
                                      void* y, int rows, int H, float eps,
                                      kvm_stream_t stream) {
  if (rows <= 0 || H <= 0 || H % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "rmsnorm: need rows > 0 and H % 8 == 0");
  if (!x || !y || !aligned16(x) || !aligned16(y) ||
      (gamma && !aligned16(gamma)))
    return fail(KVM_ERR_INVALID_ARG, "rmsnorm: NULL or unaligned pointer");
  rmsnorm_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), static_cast<const uint4*>(gamma),
      static_cast<uint4*>(y), H / 8, 1.0f / static_cast<float>(H), eps);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_silu_mul_bf16(const void* g, const void* u, void* h,
                                       int64_t n, kvm_stream_t stream) {
  if (n <= 0 || n % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "silu_mul: n must be a positive multiple of 8");
  if (!g || !u || !h || !aligned16(g) || !aligned16(u) || !aligned16(h))
    return fail(KVM_ERR_INVALID_ARG, "silu_mul: NULL or unaligned pointer");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const long long nv = n / 8;
  silu_mul_kernel<<<grid_for(nv, dev->sm_count), 256, 0,
                    static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(g), static_cast<const uint4*>(u),
      static_cast<uint4*>(h), nv);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_transpose_bf16(const void* in, void* out, int G,
                                        int R, int C, kvm_stream_t stream) {
  if (G <= 0 || R <= 0 || C <= 0 || G > 65535)
    return fail(KVM_ERR_INVALID_ARG, "transpose: bad shape");
  if (!in || !out) return fail(KVM_ERR_INVALID_ARG, "transpose: NULL pointer");
  dim3 grid((C + 31) / 32, (R + 31) / 32, G);
  transpose_kernel<<<grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), R, C, 0, 0,
      static_cast<long long>(R) * C);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_pack_gate_up(const void* Wg, const void* Wu,
                                      void* out, int G, int F, int K,
                                      int w_layout, kvm_stream_t stream) {
  if (G <= 0 || F <= 0 || K <= 0 || F % 128 != 0 || K % 8 != 0 || G > 65535)
    return fail(KVM_ERR_INVALID_ARG,
                "pack_gate_up: need F % 128 == 0 and K % 8 == 0");
  if (!Wg || !Wu || !out)
    return fail(KVM_ERR_INVALID_ARG, "pack_gate_up: NULL pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_layout == KVM_B_NK) {
    if (!aligned16(Wg) || !aligned16(Wu) || !aligned16(out))
      return fail(KVM_ERR_INVALID_ARG, "pack_gate_up: unaligned pointer");
    const DeviceInfo* dev = device_info();
    if (!dev) return KVM_ERR_CUDA;
    const long long total = 2ll * G * F * (K / 8);
    pack_rows_kernel<<<grid_for(total, dev->sm_count), 256, 0, st>>>(
        static_cast<const uint4*>(Wg), static_cast<const uint4*>(Wu),
        static_cast<uint4*>(out), F, K / 8, total);
    KVM_CUDA_TRY(cudaGetLastError());
    return KVM_OK;
  }
  if (w_layout != KVM_B_KN)
    return fail(KVM_ERR_INVALID_ARG, "pack_gate_up: unknown w_layout");
  // [G, K, F] inputs: transpose each into its interleaved rows.
  dim3 grid((F + 31) / 32, (K + 31) / 32, G);
  for (int which = 0; which < 2; ++which) {
    transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(
        static_cast<const uint16_t*>(which == 0 ? Wg : Wu),
        static_cast<uint16_t*>(out), K, F, 1, which, 2ll * F * K);
    KVM_CUDA_TRY(cudaGetLastError());
  }
  return KVM_OK;
}
