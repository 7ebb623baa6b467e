// Kernels the graph executor needs beyond the fused hot-path kernels:
//   * top-k + softmax over router logits that a graph computed itself
//     (kernel.comm.moe_dispatch(x, g) with g an arbitrary tensor),
//   * a generic elementwise interpreter for the kernel dialect's arithmetic,
//     compare and cast ops (src/ir/dialect/kernel/dialect.cpp:43-55) with
//     trailing-dimension broadcasting (the reference semantics for the
//     generated kernels of ew_jit.cu, and their A/B partner:
//     KVM_SM100_EW_JIT=0 selects it),
//   * a seeded normal fill for graph inputs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ew_jit.h"
#include "runtime.h"

namespace kvm {
namespace {

__device__ __forceinline__ float load_any(const void* p, int dtype, long long i) {
  switch (dtype) {
    case KVM_EW_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case KVM_EW_F16:
      return __half2float(static_cast<const __half*>(p)[i]);
    case KVM_EW_I32:
      return static_cast<float>(static_cast<const int*>(p)[i]);
    default:
      return static_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void store_any(void* p, int dtype, long long i, float v) {
  switch (dtype) {
    case KVM_EW_BF16:
      static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
      break;
    case KVM_EW_F16:
      static_cast<__half*>(p)[i] = __float2half_rn(v);
      break;
    case KVM_EW_I32:
      static_cast<int*>(p)[i] = static_cast<int>(v);  // toward zero
      break;
    default:
      static_cast<float*>(p)[i] = v;
  }
}

__global__ void __launch_bounds__(256)
    elementwise_kernel(const kvm_ew_program prog, const kvm_ew_inputs in, void* out,
                       long long n) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * 256) {
    float r[KVM_EW_MAX_REGS];
#pragma unroll 1
    for (int s = 0; s < prog.n_instr; ++s) {
      const int op = prog.op[s], a = prog.a[s], b = prog.b[s];
      float v;
      switch (op) {
        case KVM_EW_LOAD:
          v = load_any(in.ptr[a], prog.in_dtype[a], (i / prog.in_div[a]) % prog.in_size[a]);
          break;
        case KVM_EW_ADD: v = r[a] + r[b]; break;
        case KVM_EW_SUB: v = r[a] - r[b]; break;
        case KVM_EW_MUL: v = r[a] * r[b]; break;
        case KVM_EW_DIV: v = __fdiv_rn(r[a], r[b]); break;
        case KVM_EW_MAX: v = fmaxf(r[a], r[b]); break;
        case KVM_EW_MIN: v = fminf(r[a], r[b]); break;
        case KVM_EW_NEG: v = -r[a]; break;
        case KVM_EW_EXP: v = expf(r[a]); break;
        case KVM_EW_LOG: v = logf(r[a]); break;
        case KVM_EW_SQRT: v = sqrtf(r[a]); break;
        case KVM_EW_RSQRT: v = rsqrtf(r[a]); break;
        case KVM_EW_ABS: v = fabsf(r[a]); break;
        case KVM_EW_RCP: v = __frcp_rn(r[a]); break;
        case KVM_EW_CMP_EQ: v = r[a] == r[b] ? 1.f : 0.f; break;
        case KVM_EW_CMP_NE: v = r[a] != r[b] ? 1.f : 0.f; break;
        case KVM_EW_CMP_LT: v = r[a] < r[b] ? 1.f : 0.f; break;
        case KVM_EW_CMP_LE: v = r[a] <= r[b] ? 1.f : 0.f; break;
        case KVM_EW_CMP_GT: v = r[a] > r[b] ? 1.f : 0.f; break;
        case KVM_EW_CMP_GE: v = r[a] >= r[b] ? 1.f : 0.f; break;
        case KVM_EW_ROUND_BF16: v = __bfloat162float(__float2bfloat16_rn(r[a])); break;
        case KVM_EW_ROUND_F16: v = __half2float(__float2half_rn(r[a])); break;
        case KVM_EW_TRUNC_I32: v = truncf(r[a]); break;
        default: v = r[a];
      }
      r[prog.dst[s]] = v;
    }
    store_any(out, prog.out_dtype, i, r[prog.out_reg]);
  }
}

// One warp per row: y[m] = sum_k A[m,k] x[k], lanes over k with 16-byte loads,
// then a shuffle reduction.
__global__ void __launch_bounds__(256)
    gemv_kernel(const __nv_bfloat16* __restrict__ A, long long lda,
                const __nv_bfloat16* __restrict__ x, void* y, int out_dtype, int M,
                int K) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= M) return;
  const __nv_bfloat16* row = A + static_cast<long long>(warp) * lda;
  float s = 0.f;
  for (int k = lane * 8; k < K; k += 32 * 8) {
    if (k + 8 <= K) {
      const uint4 av = *reinterpret_cast<const uint4*>(row + k);
      const uint4 xv = *reinterpret_cast<const uint4*>(x + k);
      const uint32_t au[4] = {av.x, av.y, av.z, av.w}, xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s = __fmaf_rn(__uint_as_float(au[j] << 16), __uint_as_float(xu[j] << 16), s);
        s = __fmaf_rn(__uint_as_float(au[j] & 0xFFFF0000u),
                      __uint_as_float(xu[j] & 0xFFFF0000u), s);
      }
    } else {
      for (int j = k; j < K; ++j)
        s = __fmaf_rn(__bfloat162float(row[j]), __bfloat162float(x[j]), s);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) store_any(y, out_dtype == KVM_F32 ? KVM_EW_F32 : KVM_EW_BF16, warp, s);
}

// One thread per token: softmax + top-k over E logits (same selection and
// weights as the fused router epilogue: largest logit first, ties to the lower
// expert, p = exp(l - max) / sum exp(l - max) with the sum in index order).
__global__ void topk_kernel(const void* __restrict__ logits, int dtype, int T, int E,
                            int k, int* __restrict__ idx, float* __restrict__ w) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const long long base = static_cast<long long>(t) * E;
  float mx = load_any(logits, dtype, base);
  for (int e = 1; e < E; ++e) mx = fmaxf(mx, load_any(logits, dtype, base + e));
  float sum = 0.f;
  for (int e = 0; e < E; ++e) sum += expf(load_any(logits, dtype, base + e) - mx);
  int prev_i = -1;
  float prev_v = INFINITY;
  for (int j = 0; j < k; ++j) {
    // next best after (prev_v, prev_i) in the order (value desc, index asc)
    int bi = -1;
    float best = -INFINITY;
    for (int e = 0; e < E; ++e) {
      const float v = load_any(logits, dtype, base + e);
      const bool after_prev = v < prev_v || (v == prev_v && e > prev_i);
      if (after_prev && (bi < 0 || v > best)) {
        best = v;
        bi = e;
      }
    }
    idx[static_cast<long long>(t) * k + j] = bi;
    w[static_cast<long long>(t) * k + j] = expf(best - mx) / sum;
    prev_i = bi;
    prev_v = best;
  }
}

// splitmix64 of (seed, index) -> two uniforms -> Box-Muller.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(void* out, int dtype, long long n, uint64_t seed,
                                   float mean, float std) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * 256) {
    const uint64_t h = mix64(seed * 0x100000001B3ull + static_cast<uint64_t>(i));
    const float u1 = (static_cast<float>(h >> 40) + 1.0f) * (1.0f / 16777217.0f);
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    store_any(out, dtype, i, mean + std * z);
  }
}

int grid_of(long long n, int sms) {
  long long b = (n + 255) / 256;
  const long long cap = static_cast<long long>(sms) * 16;
  return static_cast<int>(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace
}  // namespace kvm

using namespace kvm;

namespace {

int check_program(const kvm_ew_program* prog, const kvm_ew_inputs* inputs, const void* out,
                  int64_t n) {
  if (!prog || !inputs || !out || n <= 0)
    return fail(KVM_ERR_INVALID_ARG, "elementwise: NULL argument or n <= 0");
  if (prog->n_instr < 1 || prog->n_instr > KVM_EW_MAX_INSTR || prog->n_inputs < 0 ||
      prog->n_inputs > KVM_EW_MAX_INPUTS || prog->out_reg < 0 ||
      prog->out_reg >= KVM_EW_MAX_REGS || prog->out_dtype < KVM_EW_BF16 ||
      prog->out_dtype > KVM_EW_I32)
    return fail(KVM_ERR_INVALID_ARG, "elementwise: program out of bounds");
  for (int s = 0; s < prog->n_instr; ++s) {
    const int op = prog->op[s];
    if (prog->dst[s] >= KVM_EW_MAX_REGS || op < 0 || op > KVM_EW_TRUNC_I32)
      return fail(KVM_ERR_INVALID_ARG, "elementwise: bad instruction");
    if (op == KVM_EW_LOAD) {
      if (prog->a[s] >= prog->n_inputs)
        return fail(KVM_ERR_INVALID_ARG, "elementwise: load of a missing input");
    } else if (prog->a[s] >= KVM_EW_MAX_REGS || prog->b[s] >= KVM_EW_MAX_REGS) {
      return fail(KVM_ERR_INVALID_ARG, "elementwise: register out of range");
    }
  }
  for (int i = 0; i < prog->n_inputs; ++i) {
    if (!inputs->ptr[i] || prog->in_size[i] <= 0 || prog->in_div[i] <= 0 ||
        n % (prog->in_size[i] * prog->in_div[i]) != 0)
      return fail(KVM_ERR_INVALID_ARG,
                  "elementwise: each input's size x divisor must divide the output size");
    if (prog->in_dtype[i] < KVM_EW_BF16 || prog->in_dtype[i] > KVM_EW_I32)
      return fail(KVM_ERR_INVALID_ARG, "elementwise: bad input dtype");
  }
  return KVM_OK;
}

}  // namespace

extern "C" int kvm_sm100_elementwise(const kvm_ew_program* prog,
                                     const kvm_ew_inputs* inputs, void* out,
                                     int64_t n, kvm_stream_t stream) {
  if (int rc = check_program(prog, inputs, out, n); rc != KVM_OK) return rc;
  if (ew_jit_enabled())
    return ew_jit_launch(*prog, *inputs, out, n, static_cast<cudaStream_t>(stream));
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  elementwise_kernel<<<grid_of(n, dev->sm_count), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(*prog, *inputs, out, n);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_elementwise_prepare(const kvm_ew_program* prog,
                                             const kvm_ew_inputs* inputs, const void* out,
                                             int64_t n) {
  if (int rc = check_program(prog, inputs, out, n); rc != KVM_OK) return rc;
  return ew_jit_enabled() ? ew_jit_prepare(*prog, *inputs, out, n) : KVM_OK;
}

extern "C" int kvm_sm100_gemv_bf16(const void* A, int64_t lda, const void* x, void* y,
                                   int out_dtype, int M, int K, kvm_stream_t stream) {
  if (!A || !x || !y || M <= 0 || K <= 0 || lda < K || !aligned16(A) || !aligned16(x) ||
      (lda * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG, "gemv: bad argument or unaligned rows");
  if (out_dtype != KVM_BF16 && out_dtype != KVM_F32)
    return fail(KVM_ERR_INVALID_ARG, "gemv: out_dtype must be bf16 or f32");
  const long long threads = static_cast<long long>(M) * 32;
  gemv_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(x), y,
      out_dtype, M, K);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_moe_topk(const void* logits, int logits_dtype, int T, int E,
                                  int k, int32_t* topk_idx, float* topk_w,
                                  kvm_stream_t stream) {
  if (!logits || !topk_idx || !topk_w || T <= 0 || E <= 0 || k < 1 || k > E)
    return fail(KVM_ERR_INVALID_ARG, "moe_topk: bad argument");
  topk_kernel<<<(T + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, logits_dtype, T, E, k, topk_idx, topk_w);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_fill_normal(void* out, int dtype, int64_t n, uint64_t seed,
                                     float mean, float std, kvm_stream_t stream) {
  if (!out || n <= 0) return fail(KVM_ERR_INVALID_ARG, "fill_normal: bad argument");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  fill_normal_kernel<<<grid_of(n, dev->sm_count), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(out, dtype, n, seed, mean,
                                                            std);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
