// Causal grouped-query attention (prefill) and rotary position embedding:
// the kernel.attn.prefill / kernel.attn.rope ops
// (src/ir/dialect/kernel/dialect.cpp:38-40) for the tensor-parallel decoder
// layer.
//
// Attention runs as one fused kernel (flash_attn.cuh): S and O in TMEM,
// online softmax in registers, P through shared memory; scores never reach
// HBM. (An earlier form ran S = QK^T, a softmax pass and PV as three
// launches through an L x L fp32 workspace: 3.7 ms and 74 TF/s on the
// decoder layer's attention, against 0.45 ms and 609 TF/s fused.)
// Grouped-query heads map q head h to kv head h / (HQ / HKV).
#include <cuda_bf16.h>

#include <cmath>

#include "flash_attn.cuh"
#include "gemm_bf16.cuh"
#include "runtime.h"

namespace kvm {
namespace {

#define KVM_TRY(expr)                      \
  do {                                     \
    int kvm_rc_ = (expr);                  \
    if (kvm_rc_ != KVM_OK) return kvm_rc_; \
  } while (0)

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

}  // namespace
}  // namespace kvm

using namespace kvm;

// The fused kernel needs no scratch memory.
extern "C" int64_t kvm_sm100_attention_workspace(int B, int L, int HQ, int HKV) {
  (void)B; (void)L; (void)HQ; (void)HKV;
  return 0;
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
  (void)workspace;
  (void)workspace_bytes;
  if (!q || !k || !v || !out || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      !aligned16(out))
    return fail(KVM_ERR_INVALID_ARG, "attention: NULL or unaligned pointer");
  if (ldq < int64_t(HQ) * hd || ldo < int64_t(HQ) * hd || ldk < int64_t(HKV) * hd ||
      ldv < int64_t(HKV) * hd || (ldq * 2) % 16 || (ldk * 2) % 16 || (ldv * 2) % 16 ||
      (ldo * 2) % 16)
    return fail(KVM_ERR_INVALID_ARG, "attention: bad row strides");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int group = HQ / HKV;
  if (scale <= 0.f) scale = 1.0f / sqrtf(static_cast<float>(hd));
  CUtensorMap tq, tk, tv;
  KVM_TRY(encode_tmap_2d(&tq, q, int64_t(HQ) * hd, int64_t(B) * L, ldq * 2, 64, 128,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tk, k, int64_t(HKV) * hd, int64_t(B) * L, ldk * 2, 64, 128,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tv, v, int64_t(HKV) * hd, int64_t(B) * L, ldv * 2, 64, 128,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_128B));
  AttnParams ap{};
  ap.B = B; ap.L = L; ap.HQ = HQ; ap.group = group;
  ap.q_tiles = (L + 127) / 128;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.out = static_cast<__nv_bfloat16*>(out);
  ap.ldo = ldo;
  ap.status = dev->status;
  const long long items = static_cast<long long>(B) * HQ * ap.q_tiles;
  if (items > (1ll << 30))
    return fail(KVM_ERR_INVALID_ARG, "attention: too many (batch, head, tile) items");
  const int grid = items < dev->sm_count ? int(items) : dev->sm_count;
  constexpr size_t smem = attn_smem_bytes();
  KVM_CUDA_TRY(cudaFuncSetAttribute(attn_fwd_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  attn_fwd_kernel<<<grid, kAttnThreads, smem, st>>>(tq, tk, tv, ap);
  KVM_CUDA_TRY(cudaGetLastError());
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
