// Causal grouped-query attention (prefill) and rotary position embedding:
// the kernel.attn.prefill / kernel.attn.rope ops
// (src/ir/dialect/kernel/dialect.cpp:38-40) for the tensor-parallel decoder
// layer.
//
// Attention runs as three launches per chunk of heads of one batch element:
//   1. S = Q . K^T            tcgen05 GEMM, batched over heads, fp32 out,
//                             tiles entirely above the diagonal skipped
//   2. P = softmax(scale*S)   causal, fp32 statistics, bf16 out; zeros up to
//                             the end of each row's 128-row tile
//   3. O = P . V              tcgen05 GEMM, batched over heads, V read in
//                             place (N-contiguous B), K loop stopped at the
//                             diagonal, bf16 out written into the head's
//                             columns of O
// Grouped-query heads map q head h to kv head h / (HQ / HKV).
#include <cuda_bf16.h>

#include "gemm_bf16.cuh"
#include "runtime.h"

namespace kvm {
namespace {

constexpr int kSoftmaxThreads = 256;

#define KVM_TRY(expr)                      \
  do {                                     \
    int kvm_rc_ = (expr);                  \
    if (kvm_rc_ != KVM_OK) return kvm_rc_; \
  } while (0)

// One block per score row: row r of head g keeps keys 0..r.
__global__ void __launch_bounds__(kSoftmaxThreads)
    causal_softmax_kernel(const float* __restrict__ S, __nv_bfloat16* __restrict__ P,
                          int L, float scale) {
  __shared__ float red[kSoftmaxThreads / 32];
  __shared__ float bcast;
  const long long row = blockIdx.x;            // over heads x L
  const int r = static_cast<int>(row % L);
  const float* s = S + row * L;
  __nv_bfloat16* p = P + row * L;
  const int valid = r + 1;
  const int width = min(L, (r / kGemmBM + 1) * kGemmBM);  // K extent the P.V tile reads
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < valid; c += kSoftmaxThreads) mx = fmaxf(mx, s[c] * scale);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < kSoftmaxThreads / 32; ++w) m = fmaxf(m, red[w]);
    bcast = m;
  }
  __syncthreads();
  mx = bcast;
  float sum = 0.f;
  for (int c = threadIdx.x; c < valid; c += kSoftmaxThreads) sum += expf(s[c] * scale - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kSoftmaxThreads / 32; ++w) t += red[w];
    bcast = 1.0f / t;
  }
  __syncthreads();
  const float inv = bcast;
  for (int c = threadIdx.x; c < width; c += kSoftmaxThreads)
    p[c] = __float2bfloat16_rn(c < valid ? expf(s[c] * scale - mx) * inv : 0.f);
}

// Rotary embedding, rotate-half form: for each head vector x[0..hd) at
// sequence position pos and i < hd/2, theta = pos * base^(-2i/hd):
//   y[i] = x[i] cos - x[i + hd/2] sin,  y[i + hd/2] = x[i + hd/2] cos + x[i] sin.
// Rows are tokens b*L + pos; heads are consecutive hd-wide column blocks.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, long long ld, int rows, int L,
                            int heads, int hd, float base) {
  const int half = hd / 2;
  const long long total = static_cast<long long>(rows) * heads * half;
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * 256) {
    const int j = static_cast<int>(i % half);
    const long long rh = i / half;
    const int h = static_cast<int>(rh % heads);
    const long long row = rh / heads;
    const int pos = static_cast<int>(row % L);
    const float inv_freq = powf(base, -2.0f * j / hd);
    float sn, cs;
    sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
    __nv_bfloat16* v = x + row * ld + static_cast<long long>(h) * hd;
    const float a = __bfloat162float(v[j]), b = __bfloat162float(v[j + half]);
    v[j] = __float2bfloat16_rn(a * cs - b * sn);
    v[j + half] = __float2bfloat16_rn(b * cs + a * sn);
  }
}

template <int BN, int STAGES, bool B_MN, int EPI>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                int grid, cudaStream_t st) {
  auto kern = gemm_bf16_kernel<BN, STAGES, B_MN, EPI>;
  constexpr size_t smem = gemm_smem_bytes<BN, STAGES>();
  KVM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  kern<<<grid, kGemmThreads, smem, st>>>(ta, tb, p);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

int heads_per_chunk(int HQ, int group) {
  int hc = HQ < 16 ? HQ : 16;
  hc -= hc % group;
  return hc < group ? group : hc;
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int64_t kvm_sm100_attention_workspace(int B, int L, int HQ, int HKV) {
  if (B <= 0 || L <= 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0) return 0;
  const int hc = heads_per_chunk(HQ, HQ / HKV);
  const int64_t sq = static_cast<int64_t>(L) * L;
  return hc * sq * 4 + hc * sq * 2 + 256;
}

extern "C" int kvm_sm100_attention_prefill_bf16(
    const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
    void* out, int64_t ldo, int B, int L, int HQ, int HKV, int hd, float scale,
    void* workspace, int64_t workspace_bytes, kvm_stream_t stream) {
  if (B <= 0 || L <= 0 || HQ <= 0 || HKV <= 0 || HQ % HKV != 0 || hd != 128)
    return fail(KVM_ERR_INVALID_ARG,
                "attention: need B, L > 0, HQ % HKV == 0 and head_dim 128");
  if (L % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "attention: sequence length must be a multiple of 8");
  if (!q || !k || !v || !out || !workspace || !aligned16(q) || !aligned16(k) ||
      !aligned16(v) || !aligned16(out) || !aligned16(workspace))
    return fail(KVM_ERR_INVALID_ARG, "attention: NULL or unaligned pointer");
  if (ldq < int64_t(HQ) * hd || ldo < int64_t(HQ) * hd || ldk < int64_t(HKV) * hd ||
      ldv < int64_t(HKV) * hd || (ldq * 2) % 16 || (ldk * 2) % 16 || (ldv * 2) % 16 ||
      (ldo * 2) % 16)
    return fail(KVM_ERR_INVALID_ARG, "attention: bad row strides");
  if (workspace_bytes < kvm_sm100_attention_workspace(B, L, HQ, HKV))
    return fail(KVM_ERR_INVALID_ARG, "attention: workspace too small");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int group = HQ / HKV;
  const int hc = heads_per_chunk(HQ, group);
  const int64_t sq = static_cast<int64_t>(L) * L;
  float* S = static_cast<float*>(workspace);
  __nv_bfloat16* P = reinterpret_cast<__nv_bfloat16*>(S + hc * sq);
  if (scale <= 0.f) scale = 1.0f / sqrtf(static_cast<float>(hd));
  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kbp = static_cast<const __nv_bfloat16*>(k);
  const auto* vb = static_cast<const __nv_bfloat16*>(v);
  auto* ob = static_cast<__nv_bfloat16*>(out);

  for (int b = 0; b < B; ++b) {
    for (int h0 = 0; h0 < HQ; h0 += hc) {
      const int nh = HQ - h0 < hc ? HQ - h0 : hc;
      // ---- S = Q K^T (heads h0 .. h0+nh of batch b), fp32 [nh, L, L]
      CUtensorMap ta, tb;
      const __nv_bfloat16* qh = qb + static_cast<int64_t>(b) * L * ldq + int64_t(h0) * hd;
      const __nv_bfloat16* kh =
          kbp + static_cast<int64_t>(b) * L * ldk + int64_t(h0 / group) * hd;
      KVM_TRY(encode_tmap_2d(&ta, qh, int64_t(nh) * hd, L, ldq * 2, kGemmBK, kGemmBM,
                             CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
      const int nkh = (nh + group - 1) / group;
      KVM_TRY(encode_tmap_2d(&tb, kh, int64_t(nkh) * hd, L, ldk * 2, kGemmBK, 256,
                             CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
      GemmParams p{};
      p.M = L; p.N = L; p.K = hd;
      p.num_groups = nh;
      p.D = S; p.ldd = L;
      p.status = dev->status;
      p.bh_heads = nh; p.bh_group = group;
      p.a_h_cols = hd;
      p.b_h_cols = hd;
      p.d_h = sq;
      p.causal = 1;
      const int tiles = nh * ((L + 127) / 128) * ((L + 255) / 256);
      KVM_TRY((launch_gemm<256, 4, false, kEpiF32>(ta, tb, p,
                                                   tiles < dev->sm_count ? tiles : dev->sm_count, st)));
      // ---- P = causal softmax
      causal_softmax_kernel<<<static_cast<unsigned>(nh * static_cast<int64_t>(L)),
                              kSoftmaxThreads, 0, st>>>(S, P, L, scale);
      KVM_CUDA_TRY(cudaGetLastError());
      // ---- O = P V (V read in place: [keys, hd] rows, N-contiguous)
      const __nv_bfloat16* vh =
          vb + static_cast<int64_t>(b) * L * ldv + int64_t(h0 / group) * hd;
      KVM_TRY(encode_tmap_2d(&ta, P, L, int64_t(nh) * L, int64_t(L) * 2, kGemmBK, kGemmBM,
                             CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
      KVM_TRY(encode_tmap_2d(&tb, vh, int64_t(nkh) * hd, L, ldv * 2, 64, kGemmBK,
                             CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
      GemmParams o{};
      o.M = L; o.N = hd; o.K = L;
      o.num_groups = nh;
      o.D = ob + static_cast<int64_t>(b) * L * ldo + int64_t(h0) * hd;
      o.ldd = ldo;
      o.status = dev->status;
      o.bh_heads = nh; o.bh_group = group;
      o.a_h_rows = L;
      o.b_h_cols = hd;
      o.d_h = hd;
      o.causal = 2;
      const int otiles = nh * ((L + 127) / 128);
      KVM_TRY((launch_gemm<128, 6, true, kEpiBf16>(ta, tb, o,
                                                   otiles < dev->sm_count ? otiles : dev->sm_count, st)));
    }
  }
  return KVM_OK;
}

extern "C" int kvm_sm100_rope_bf16(void* x, int64_t ld, int rows, int L, int heads,
                                   int hd, float base, kvm_stream_t stream) {
  if (!x || rows <= 0 || L <= 0 || heads <= 0 || hd <= 0 || hd % 2 || ld < int64_t(heads) * hd)
    return fail(KVM_ERR_INVALID_ARG, "rope: bad argument");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const long long total = static_cast<long long>(rows) * heads * (hd / 2);
  long long blocks = (total + 255) / 256;
  if (blocks > dev->sm_count * 16ll) blocks = dev->sm_count * 16ll;
  rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), ld, rows, L, heads, hd, base > 0 ? base : 10000.f);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
