// Host launchers of the bf16 tcgen05 GEMM: dense GEMM (kernel.matmul /
// kernel.gemm), the fused SiLU-gate GEMM, the grouped expert GEMM and the
// router GEMM with fused softmax/top-k.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "ep_layout.h"
#include "gemm_bf16.cuh"
#include "gemm_pair.cuh"
#include "router.cuh"
#include "runtime.h"

namespace kvm {
namespace {

// tb2: B's map with BN / 2-row boxes, read only for half-width items of a
// K-major B (p.split_tiles > 0); other launches pass tb again.
template <int BN, int STAGES, bool B_MN, int EPI>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2,
           const GemmParams& p, int grid, cudaStream_t st) {
  auto kern = gemm_bf16_kernel<BN, STAGES, B_MN, EPI>;
  constexpr size_t smem = gemm_smem_bytes<BN, STAGES>();
  KVM_CUDA_TRY(cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  kern<<<grid, kGemmThreads, smem, st>>>(ta, tb, tb2, p);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

// SM pairs that can be resident at once for the pair kernel (clusters of 2
// need two free SMs of one GPC), cached per device and epilogue.
template <int EPI, int EP = kEpNone>
int pair_clusters(int* out) {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  KVM_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *out = cached[dev];
    return KVM_OK;
  }
  auto kern = gemm_pair_kernel<EPI, EP>;
  constexpr size_t smem = gemm_pair_smem_bytes();
  KVM_CUDA_TRY(cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const DeviceInfo* d = device_info();
  if (!d) return KVM_ERR_CUDA;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (d->sm_count / 2));
  cfg.blockDim = dim3(pair_threads(EP));
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  KVM_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
  if (n <= 0) return fail(KVM_ERR_UNSUPPORTED, "pair GEMM: no SM pair can be resident");
  if (n > d->sm_count / 2) n = d->sm_count / 2;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  *out = n;
  return KVM_OK;
}

// Launch the pair kernel on min(resident pairs, upper bound of pair tiles).
template <int EPI, int EP = kEpNone>
int launch_pair(const PairMaps& maps, const PairParams& p, long long max_tiles,
                cudaStream_t st, const PairEp& ep = PairEp{}) {
  int ncl = 0;
  int rc = pair_clusters<EPI, EP>(&ncl);
  if (rc != KVM_OK) return rc;
  if (max_tiles < ncl) ncl = int(max_tiles > 0 ? max_tiles : 1);
  auto kern = gemm_pair_kernel<EPI, EP>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * ncl);
  cfg.blockDim = dim3(pair_threads(EP));
  cfg.dynamicSmemBytes = gemm_pair_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch for the single-GPU forms: the prologue
  // (barriers, TMEM, tensor maps) overlaps the previous kernel's tail
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = EP == kEpNone ? 2 : 1;
  KVM_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, maps, p, ep));
  return KVM_OK;
}

// Tensor maps of the pair kernel: weights [G*N, K] in 128-row boxes, tokens
// [rows, K] (row stride lda) in boxes of 128, 64, 32, 16 and 8 rows.
int encode_pair_maps(PairMaps* m, const void* X, long long lda, int rows,
                     const void* W, long long wrows, int K) {
  int rc = encode_tmap_2d(&m->w, W, K, wrows, (uint64_t)K * 2, kPairBK, 128,
                          CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != KVM_OK) return rc;
  for (int i = 0; i < 5; ++i) {
    rc = encode_tmap_2d(&m->x[i], X, K, rows, (uint64_t)lda * 2, kPairBK,
                        128u >> i, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != KVM_OK) return rc;
  }
  return KVM_OK;
}

// The SM-pair kernel serves the grouped and SiLU-gate GEMMs unless
// KVM_SM100_PAIR_GEMM=0 selects the one-SM kernel (for comparison).
bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KVM_SM100_PAIR_GEMM");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

int check_ptr(const void* p, const char* what) {
  if (!p) return fail(KVM_ERR_INVALID_ARG, std::string(what) + " is NULL");
  if (!aligned16(p))
    return fail(KVM_ERR_INVALID_ARG,
                std::string(what) + " must be 16-byte aligned");
  return KVM_OK;
}

#define KVM_TRY(expr)             \
  do {                            \
    int kvm_rc_ = (expr);         \
    if (kvm_rc_ != KVM_OK) return kvm_rc_; \
  } while (0)

int cdiv(long long a, long long b) { return int((a + b - 1) / b); }

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int kvm_sm100_gemm_bf16(const void* A, int64_t lda, const void* B,
                                   int64_t ldb, int b_layout, const void* C,
                                   void* D, int64_t ldd, int out_dtype, int M,
                                   int N, int K, kvm_stream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0)
    return fail(KVM_ERR_INVALID_ARG, "gemm: M, N, K must be positive");
  if (b_layout != KVM_B_NK && b_layout != KVM_B_KN)
    return fail(KVM_ERR_INVALID_ARG, "gemm: unknown b_layout");
  if (out_dtype != KVM_BF16 && out_dtype != KVM_F32)
    return fail(KVM_ERR_INVALID_ARG, "gemm: out_dtype must be bf16 or f32");
  KVM_TRY(check_ptr(A, "gemm: A"));
  KVM_TRY(check_ptr(B, "gemm: B"));
  KVM_TRY(check_ptr(D, "gemm: D"));
  if (C) KVM_TRY(check_ptr(C, "gemm: C"));
  const int es = out_dtype == KVM_F32 ? 4 : 2;
  if (lda < K || (lda * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG, "gemm: lda must be >= K and a multiple of 8");
  const long long b_inner = b_layout == KVM_B_NK ? K : N;
  if (ldb < b_inner || (ldb * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "gemm: ldb must cover B's contiguous extent and be a multiple of 8");
  if (ldd < N || (ldd * es) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "gemm: ldd must be >= N with 16-byte aligned rows");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;

  GemmParams p{};
  p.M = M; p.N = N; p.K = K;
  p.num_groups = 1; p.offsets = nullptr; p.b_group_rows = 0;
  p.D = D; p.ldd = ldd; p.C = C; p.ldc = ldd;
  p.status = dev->status;

  // Output tile width: 256 when those tiles still fill the SMs, 64 when even
  // 128-wide tiles would leave over half of the SMs idle (small, latency-bound
  // products: more CTAs each stream fewer bytes), else 128.
  const int m_tiles = cdiv(M, kGemmBM);
  const bool wide = (long long)m_tiles * cdiv(N, 256) >= dev->sm_count;
  const bool narrow = !wide && 2LL * m_tiles * cdiv(N, 128) <= dev->sm_count;
  const int BN = wide ? 256 : narrow ? 64 : 128;
  const int tiles = m_tiles * cdiv(N, BN);
  // A last wave of whole tiles on at most half of the SMs runs as twice as
  // many half-width items instead (4096 x 4096 outputs in 128 x 256 tiles:
  // 512 tiles = 3 waves + 68, so 3.5 tile times instead of 4).
  const int tail = tiles % dev->sm_count;
  if (BN >= 128 && tiles > dev->sm_count && tail > 0 && 2 * tail <= dev->sm_count)
    p.split_tiles = tail;
  const int grid = tiles < dev->sm_count ? tiles : dev->sm_count;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  CUtensorMap ta, tb, tb2;
  KVM_TRY(encode_tmap_2d(&ta, A, K, M, lda * 2, kGemmBK, kGemmBM,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  if (b_layout == KVM_B_NK) {
    KVM_TRY(encode_tmap_2d(&tb, B, K, N, ldb * 2, kGemmBK, BN,
                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           CU_TENSOR_MAP_SWIZZLE_128B));
    tb2 = tb;
    if (p.split_tiles > 0)
      KVM_TRY(encode_tmap_2d(&tb2, B, K, N, ldb * 2, kGemmBK, BN / 2,
                             CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    if (N % 8 != 0)
      return fail(KVM_ERR_INVALID_ARG, "gemm: [K,N] B needs N % 8 == 0");
    KVM_TRY(encode_tmap_2d(&tb, B, N, K, ldb * 2, 64, kGemmBK,
                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                           CU_TENSOR_MAP_SWIZZLE_128B));
    tb2 = tb;
  }
  const bool mn = b_layout == KVM_B_KN;
  const bool f32 = out_dtype == KVM_F32;
  if (wide) {
    if (!mn && !f32) return launch<256, 4, false, kEpiBf16>(ta, tb, tb2, p, grid, st);
    if (!mn && f32) return launch<256, 4, false, kEpiF32>(ta, tb, tb2, p, grid, st);
    if (mn && !f32) return launch<256, 4, true, kEpiBf16>(ta, tb, tb2, p, grid, st);
    return launch<256, 4, true, kEpiF32>(ta, tb, tb2, p, grid, st);
  }
  if (narrow) {
    if (!mn && !f32) return launch<64, 8, false, kEpiBf16>(ta, tb, tb2, p, grid, st);
    if (!mn && f32) return launch<64, 8, false, kEpiF32>(ta, tb, tb2, p, grid, st);
    if (mn && !f32) return launch<64, 8, true, kEpiBf16>(ta, tb, tb2, p, grid, st);
    return launch<64, 8, true, kEpiF32>(ta, tb, tb2, p, grid, st);
  }
  if (!mn && !f32) return launch<128, 6, false, kEpiBf16>(ta, tb, tb2, p, grid, st);
  if (!mn && f32) return launch<128, 6, false, kEpiF32>(ta, tb, tb2, p, grid, st);
  if (mn && !f32) return launch<128, 6, true, kEpiBf16>(ta, tb, tb2, p, grid, st);
  return launch<128, 6, true, kEpiF32>(ta, tb, tb2, p, grid, st);
}

// Shared body of the dense and grouped SiLU-gate / plain grouped launches.
static int grouped_impl(const void* A, long long lda, const void* B, void* D,
                        long long ldd, const int32_t* offsets, int G, int rows,
                        int N, int K, int epilogue, cudaStream_t st) {
  if (rows < 0 || N <= 0 || K <= 0 || G <= 0 || G > kMaxGroups)
    return fail(KVM_ERR_INVALID_ARG,
                "grouped gemm: need rows >= 0, N, K > 0 and 1 <= G <= 256");
  if (epilogue != kEpiBf16 && epilogue != kEpiSilu)
    return fail(KVM_ERR_INVALID_ARG, "grouped gemm: epilogue must be 0 or 2");
  if (epilogue == kEpiSilu && N % 256 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "SiLU-gate gemm: 2F must be a multiple of 256 (F % 128 == 0)");
  KVM_TRY(check_ptr(A, "grouped gemm: A"));
  KVM_TRY(check_ptr(B, "grouped gemm: B"));
  KVM_TRY(check_ptr(D, "grouped gemm: D"));
  if ((lda * 2) % 16 != 0 || lda < K)
    return fail(KVM_ERR_INVALID_ARG, "grouped gemm: K must be a multiple of 8");
  if (rows == 0) return KVM_OK;
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;

  GemmParams p{};
  p.M = rows; p.N = N; p.K = K;
  p.num_groups = G; p.offsets = offsets; p.b_group_rows = N;
  p.D = D; p.ldd = ldd; p.C = nullptr; p.ldc = 0;
  p.status = dev->status;

  if (pair_enabled()) {
    PairParams pp{};
    pp.rows = rows; pp.N = N; pp.K = K;
    pp.num_groups = G; pp.offsets = offsets;
    pp.D = D; pp.ldd = ldd; pp.C = nullptr; pp.ldc = 0;
    pp.status = dev->status;
    PairMaps maps;
    KVM_TRY(encode_pair_maps(&maps, A, lda, rows, B, (long long)N * G, K));
    // every group has at most rows/256 + 1 token tiles
    const long long ub = (long long)(cdiv(rows, kPairMaxTN) + G) * cdiv(N, 256);
    if (epilogue == kEpiSilu) return launch_pair<kEpiSilu>(maps, pp, ub, st);
    return launch_pair<kEpiBf16>(maps, pp, ub, st);
  }

  // One-SM kernel, 128 x 256 tiles (two 64-row gate blocks and their up
  // blocks for SiLU-gate).
  constexpr int BN = 256;
  const long long ub = (long long)(cdiv(rows, kGemmBM) + G) * cdiv(N, BN);
  const int grid = ub < dev->sm_count ? int(ub) : dev->sm_count;
  CUtensorMap ta, tb;
  KVM_TRY(encode_tmap_2d(&ta, A, K, rows, lda * 2, kGemmBK, kGemmBM,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tb, B, K, (uint64_t)N * G, (uint64_t)K * 2, kGemmBK,
                         BN, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  if (epilogue == kEpiSilu)
    return launch<BN, 4, false, kEpiSilu>(ta, tb, tb, p, grid, st);
  return launch<BN, 4, false, kEpiBf16>(ta, tb, tb, p, grid, st);
}

extern "C" int kvm_sm100_gemm_bf16_silu_gate(const void* A, int64_t lda,
                                             const void* W13, void* H,
                                             int64_t ldh, int M, int F, int K,
                                             kvm_stream_t stream) {
  if (M <= 0 || F <= 0 || F % 128 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "silu-gate gemm: M > 0 and F a positive multiple of 128");
  if (ldh < F || (ldh * 2) % 16 != 0 || !aligned16(H))
    return fail(KVM_ERR_INVALID_ARG, "silu-gate gemm: bad H / ldh");
  // A dense SiLU-gate GEMM is a grouped one with a single group.
  return grouped_impl(A, lda, W13, H, ldh, nullptr, 1, M, 2 * F, K, kEpiSilu,
                      static_cast<cudaStream_t>(stream));
}

extern "C" int kvm_sm100_grouped_gemm_bf16(const void* A, const void* B,
                                           void* D, const int32_t* offsets,
                                           int G, int rows, int N, int K,
                                           int epilogue,
                                           kvm_stream_t stream) {
  if (!offsets)
    return fail(KVM_ERR_INVALID_ARG, "grouped gemm: offsets is NULL");
  const long long ldd = epilogue == kEpiSilu ? N / 2 : N;
  if ((ldd * 2) % 16 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "grouped gemm: output rows must be 16-byte multiples");
  return grouped_impl(A, K, B, D, ldd, offsets, G, rows, N, K, epilogue,
                      static_cast<cudaStream_t>(stream));
}

namespace kvm {
namespace {

template <int BN>
int launch_router(const CUtensorMap& tx, const CUtensorMap& tw, const RouterParams& p,
                  int grid, cudaStream_t st) {
  auto kern = router_topk_kernel<BN>;
  constexpr size_t smem = RouterCfg<BN>::kSmem;
  KVM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  kern<<<grid, kRouterThreads, smem, st>>>(tx, tw, p);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

// Launch configuration of the pair router: clusters of 2 and (`pdl`)
// programmatic dependent launch; `attr` must hold 2 entries.
cudaLaunchConfig_t router_pair_config(int pairs, cudaStream_t st, cudaLaunchAttribute* attr,
                                      bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kRouterPairThreads);
  cfg.dynamicSmemBytes = RouterPairCfg::kSmem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cfg;
}

// SM pairs on which the pair router can be resident (cached per device).
int router_pairs(const DeviceInfo* d, int* out) {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  KVM_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *out = cached[dev];
    return KVM_OK;
  }
  KVM_CUDA_TRY(cudaFuncSetAttribute(router_pair_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(RouterPairCfg::kSmem)));
  cudaLaunchAttribute attr[2];
  cudaLaunchConfig_t cfg = router_pair_config(d->sm_count / 2, nullptr, attr, false);
  int n = 0;
  KVM_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, router_pair_kernel, &cfg));
  if (n <= 0) return fail(KVM_ERR_UNSUPPORTED, "router: no SM pair can be resident");
  if (n > d->sm_count / 2) n = d->sm_count / 2;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  *out = n;
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

extern "C" int kvm_sm100_moe_router_topk(const void* x, const void* Wr,
                                         float* logits, int32_t* topk_idx,
                                         float* topk_w, int T, int H, int E,
                                         int k, kvm_stream_t stream) {
  if (E < 1 || E > 256)
    return fail(KVM_ERR_UNSUPPORTED, "router: this build supports 1 <= E <= 256");
  if (T <= 0 || H <= 0 || H % 8 != 0 || k < 1 || k > 8 || k > E)
    return fail(KVM_ERR_INVALID_ARG,
                "router: need T > 0, H % 8 == 0 and 1 <= k <= min(8, E)");
  KVM_TRY(check_ptr(x, "router: x"));
  KVM_TRY(check_ptr(Wr, "router: Wr"));
  KVM_TRY(check_ptr(logits, "router: logits"));
  if (!topk_idx || !topk_w)
    return fail(KVM_ERR_INVALID_ARG, "router: outputs are NULL");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const int BN = E <= 64 ? 64 : E <= 128 ? 128 : 256;
  RouterParams p{};
  p.T = T; p.E = E; p.K = H; p.top_k = k;
  p.logits = logits; p.topk_idx = topk_idx; p.topk_w = topk_w;
  p.status = dev->status;
  // Rows per tile: enough tiles to give every SM (E > 64) or SM pair (E <= 64)
  // one (8192 tokens: 147 tiles of 56 rows, or 74 pair tiles of 112), at
  // least 32 rows and at most 128.
  int pairs = 0;
  if (BN == 64) KVM_TRY(router_pairs(dev, &pairs));
  int tr = (cdiv(T, BN == 64 ? pairs : dev->sm_count) + 7) & ~7;
  tr = tr < 32 ? 32 : tr > 128 ? 128 : tr;
  p.tile_rows = tr;
  const int tiles = cdiv(T, tr);
  const int grid = tiles < dev->sm_count ? tiles : dev->sm_count;
  CUtensorMap tx, tw;
  KVM_TRY(encode_tmap_2d(&tx, x, H, T, (uint64_t)H * 2, kRouterBK, tr,
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  KVM_TRY(encode_tmap_2d(&tw, Wr, H, E, (uint64_t)H * 2, kRouterBK, BN,  // rows >= E read 0
                         CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (BN == 64) {
    KVM_CUDA_TRY(cudaFuncSetAttribute(router_pair_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(RouterPairCfg::kSmem)));
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg =
        router_pair_config(tiles < pairs ? tiles : pairs, st, attr, true);
    KVM_CUDA_TRY(cudaLaunchKernelEx(&cfg, router_pair_kernel, tx, tw, p));
    return KVM_OK;
  }
  if (BN == 128) return launch_router<128>(tx, tw, p, grid, st);
  return launch_router<256>(tx, tw, p, grid, st);
}

// ------------------------------------------- overlapped expert parallel ---
// The dispatch all-to-all fused with the gate/up GEMM, and the down GEMM
// fused with the combine all-to-all (gemm_pair.cuh, kEpDispatchGateUp /
// kEpDownPush), over the peer buffers of an expert-parallel group.

namespace kvm {
namespace {

int ep_common(const kvm_ep_peers* pr, int64_t cap_rows, const void* workspace,
              uint32_t epoch, PairEp* ep) {
  if (!pr || pr->world < 1 || pr->world > KVM_EP_MAX_RANKS || pr->rank < 0 ||
      pr->rank >= pr->world || pr->E < 1 || pr->E % pr->world != 0 || pr->H % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "ep gemm: bad peer table");
  if (!workspace || cap_rows <= 0 || cap_rows >= (1ll << 28) || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep gemm: NULL workspace, bad cap_rows or epoch 0");
  if (pr->E / pr->world > kMaxGroups)
    return fail(KVM_ERR_UNSUPPORTED, "ep gemm: more than 256 experts per rank");
  *ep = PairEp{};
  ep->P = pr->world;
  ep->me = pr->rank;
  ep->epr = pr->E / pr->world;
  ep->epoch = epoch;
  for (int r = 0; r < pr->world; ++r) {
    if (!pr->recv[r] || !pr->y[r] || !pr->flags[r])
      return fail(KVM_ERR_INVALID_ARG, "ep gemm: missing peer buffer");
    ep->flags[r] = static_cast<unsigned*>(pr->flags[r]);
    ep->recv[r] = pr->recv[r];
    ep->push_base[r] = pr->y[r];
  }
  const EpWorkspace ws = ep_workspace(const_cast<void*>(workspace), pr->E, cap_rows);
  ep->seg_ctr = ws.seg_ctr;
  ep->seg_prefix = ws.seg_prefix;
  ep->nseg = ep->epr * (pr->world - 1);
  ep->push_row = ws.push_row;
  ep->tile_first = ws.tile_first;
  ep->done_ctr = ws.done_ctr;
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

extern "C" int kvm_sm100_ep_dispatch_gate_up(const kvm_ep_peers* pr, const void* x,
                                             const int32_t* src_token,
                                             const int32_t* offsets,
                                             const int32_t* send_base,
                                             const int32_t* local_offsets,
                                             const void* W13, void* Hout, int F,
                                             int64_t cap_rows, void* workspace,
                                             uint32_t epoch, kvm_stream_t stream) {
  PairEp ep;
  KVM_TRY(ep_common(pr, cap_rows, workspace, epoch, &ep));
  if (F <= 0 || F % 128 != 0)
    return fail(KVM_ERR_INVALID_ARG, "ep dispatch gate/up: F must be a multiple of 128");
  if (!src_token || !offsets || !send_base || !local_offsets)
    return fail(KVM_ERR_INVALID_ARG, "ep dispatch gate/up: NULL index array");
  KVM_TRY(check_ptr(x, "ep dispatch gate/up: x"));
  KVM_TRY(check_ptr(W13, "ep dispatch gate/up: W13"));
  KVM_TRY(check_ptr(Hout, "ep dispatch gate/up: H"));
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const int H = pr->H, G = ep.epr, N = 2 * F;
  ep.x = static_cast<const uint4*>(x);
  ep.row_vecs = H / 8;
  ep.src_token = src_token;
  ep.offsets = offsets;
  ep.send_base = send_base;
  PairParams pp{};
  pp.rows = static_cast<int>(cap_rows); pp.N = N; pp.K = H;
  pp.num_groups = G; pp.offsets = local_offsets;
  pp.D = Hout; pp.ldd = F; pp.C = nullptr; pp.ldc = 0;
  pp.status = dev->status;
  PairMaps maps;
  KVM_TRY(encode_pair_maps(&maps, pr->recv[pr->rank], H, pp.rows, W13, (long long)N * G, H));
  // Every resident pair is launched: the dispatch warps of all CTAs must run
  // whatever the number of GEMM tiles.
  return launch_pair<kEpiSilu, kEpDispatchGateUp>(maps, pp, 1ll << 30,
                                                   static_cast<cudaStream_t>(stream), ep);
}

extern "C" int kvm_sm100_ep_down_push(const kvm_ep_peers* pr, const void* Hact,
                                      const void* W2, const int32_t* local_offsets, int F,
                                      int64_t cap_rows, void* workspace, uint32_t epoch,
                                      kvm_stream_t stream) {
  PairEp ep;
  KVM_TRY(ep_common(pr, cap_rows, workspace, epoch, &ep));
  if (F <= 0 || F % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "ep down push: F must be a multiple of 8");
  if (!local_offsets) return fail(KVM_ERR_INVALID_ARG, "ep down push: NULL offsets");
  KVM_TRY(check_ptr(Hact, "ep down push: H"));
  KVM_TRY(check_ptr(W2, "ep down push: W2"));
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const int H = pr->H, G = ep.epr;
  PairParams pp{};
  pp.rows = static_cast<int>(cap_rows); pp.N = H; pp.K = F;
  pp.num_groups = G; pp.offsets = local_offsets;
  pp.D = nullptr; pp.ldd = H; pp.C = nullptr; pp.ldc = 0;
  pp.status = dev->status;
  PairMaps maps;
  KVM_TRY(encode_pair_maps(&maps, Hact, F, pp.rows, W2, (long long)H * G, F));
  // All resident pairs, so that the last CTA to finish raises the flags.
  return launch_pair<kEpiBf16, kEpDownPush>(maps, pp, 1ll << 30,
                                             static_cast<cudaStream_t>(stream), ep);
}
