// MoE dispatch / combine data movement:
//   permute  -- deterministic expert-major order of the (token, slot) pairs
//   scatter  -- token rows -> permuted rows (the dispatch copy)
//   combine  -- weighted sum of each token's expert outputs
//
// The permutation orders pairs by (expert, token, slot). Counting uses shared
// atomics (order-independent); every position is computed from prefix sums
// and warp match masks, so the result is identical run to run and equal to a
// stable sort of the pairs by expert.
#include <cuda_bf16.h>

#include "runtime.h"

#include <mutex>
#include <string>

namespace kvm {
namespace {

constexpr int kPermChunk = 256;  // pairs per block in the permute kernels
constexpr int kMaxExperts = 1024;

// Per-chunk expert histogram: counts[chunk][e].
__global__ void __launch_bounds__(kPermChunk)
    permute_count_kernel(const int* __restrict__ idx, int n, int E,
                         int* __restrict__ counts, int* status) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int i = blockIdx.x * kPermChunk + threadIdx.x;
  if (i < n) {
    const int e = idx[i];
    if (e >= 0 && e < E)
      atomicAdd(&hist[e], 1);
    else
      atomicOr(status, kDevBadInput);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    counts[static_cast<long long>(blockIdx.x) * E + e] = hist[e];
}

// Exclusive scans: base[chunk][e] = offsets[e] + sum_{c' < chunk} counts[c'][e]
// and offsets[e] = sum_{e' < e} total[e'].  One block, one thread per expert.
__global__ void permute_scan_kernel(const int* __restrict__ counts,
                                    int n_chunks, int E, int* __restrict__ base,
                                    int* __restrict__ offsets) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int tot[];
  const int e = threadIdx.x;
  int run = 0;
  if (e < E) {
    for (int c = 0; c < n_chunks; ++c) {
      const long long o = static_cast<long long>(c) * E + e;
      base[o] = run;
      run += counts[o];
    }
    tot[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int x = 0; x < E; ++x) {
      const int t = tot[x];
      tot[x] = acc;
      acc += t;
    }
    offsets[E] = acc;
  }
  __syncthreads();
  if (e < E) {
    const int off = tot[e];
    offsets[e] = off;
    for (int c = 0; c < n_chunks; ++c) base[static_cast<long long>(c) * E + e] += off;
  }
}

// Rank of each pair among the same-expert pairs before it in its chunk, plus
// the chunk base: pos[i]; src_token[pos[i]] = i / k.
//
// FUSED: `base` is the count matrix instead, and every block derives its own
// chunk bases and the expert offsets from it (the scans of
// permute_scan_kernel; block 0 also writes `offsets`), which saves a launch
// and a single-block pass when the matrix is small (n_chunks * E <= 16 K).
template <bool FUSED>
__global__ void __launch_bounds__(kPermChunk)
    permute_rank_kernel(const int* __restrict__ idx, int n, int k, int E,
                        const int* __restrict__ base, int* __restrict__ pos,
                        int* __restrict__ src_token, int n_chunks,
                        int* __restrict__ offsets) {
  pdl_trigger();
  pdl_wait();
  constexpr int kWarps = kPermChunk / 32;
  // [kWarps][E], then (FUSED) cbase [E], tot [E], two [max(kPermChunk, E)]
  extern __shared__ int wcount[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // this thread's pair, loaded before the prologue so the load overlaps it
  const int i = blockIdx.x * kPermChunk + threadIdx.x;
  int e = -1;
  if (i < n) {
    e = idx[i];
    if (e < 0 || e >= E) e = -1;
  }
  for (int x = threadIdx.x; x < kWarps * E; x += blockDim.x) wcount[x] = 0;
  int* cbase = wcount + kWarps * E;  // this chunk's base per expert
  if constexpr (FUSED) {
    int* tot = cbase + E;
    int* part_before = tot + E;
    int* part_all = part_before + (E > kPermChunk ? E : kPermChunk);
    // Column sums of the count matrix by G row groups x E experts, so every
    // thread of the block loads (G = kPermChunk / E rows apart), then the G
    // partial sums per expert are added (integers: any order is exact).
    const int G = E <= kPermChunk ? kPermChunk / E : 1;
    for (int x = threadIdx.x; x < G * E; x += blockDim.x) {
      const int ex = x % E, g = x / E;
      int before = 0, all = 0;
#pragma unroll 8
      for (int c = g; c < n_chunks; c += G) {
        const int v = base[static_cast<long long>(c) * E + ex];
        before += c < static_cast<int>(blockIdx.x) ? v : 0;
        all += v;
      }
      part_before[x] = before;
      part_all[x] = all;
    }
    __syncthreads();
    for (int ex = threadIdx.x; ex < E; ex += blockDim.x) {
      int before = 0, all = 0;
      for (int g = 0; g < G; ++g) {
        before += part_before[g * E + ex];
        all += part_all[g * E + ex];
      }
      cbase[ex] = before;
      tot[ex] = all;
    }
    __syncthreads();
    // exclusive scan of the expert totals, in place (Hillis-Steele on E <= 1024)
    for (int d = 1; d < E; d <<= 1) {
      int add[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ex = threadIdx.x + j * kPermChunk;
        add[j] = (ex < E && ex >= d) ? tot[ex - d] : 0;
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int ex = threadIdx.x + j * kPermChunk;
        if (ex < E) tot[ex] += add[j];
      }
      __syncthreads();
    }
    // tot is now inclusive: offsets[e] = tot[e - 1]
    for (int ex = threadIdx.x; ex < E; ex += blockDim.x) {
      const int off = ex > 0 ? tot[ex - 1] : 0;
      cbase[ex] += off;
      if (blockIdx.x == 0) offsets[ex] = off;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) offsets[E] = tot[E - 1];
  }
  __syncthreads();
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const unsigned lt = (1u << lane) - 1u;
  const int rank_in_warp = __popc(peers & lt);
  if (e >= 0 && rank_in_warp == 0) wcount[warp * E + e] = __popc(peers);
  __syncthreads();
  if (e >= 0) {
    int r = rank_in_warp;
    for (int w = 0; w < warp; ++w) r += wcount[w * E + e];
    const int p = (FUSED ? cbase[e] : base[static_cast<long long>(blockIdx.x) * E + e]) + r;
    pos[i] = p;
    src_token[p] = i / k;
  } else if (i < n) {
    pos[i] = -1;
  }
}

// Rows of TOK tokens per block: every thread first loads all its 16-byte
// vectors of the TOK rows (TOK x VPT loads in flight per thread, enough to
// cover HBM latency at full occupancy), then writes each to the token's k
// destination rows. VPT = vectors per thread per row (row_vecs <= 256 VPT).
constexpr int kScatterTok = 4;
constexpr int kRowThreads = 256;

template <int VPT>
__global__ void __launch_bounds__(kRowThreads)
    scatter_rows_kernel(const uint4* __restrict__ x, const int* __restrict__ pos,
                        uint4* __restrict__ xp, int T, int k, int row_vecs,
                        long long n_rows_out, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x * kScatterTok;
  uint4 val[kScatterTok][VPT];
#pragma unroll
  for (int i = 0; i < kScatterTok; ++i) {
    const int t = t0 + i;
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int v = threadIdx.x + c * kRowThreads;
      if (t < T && v < row_vecs) val[i][c] = __ldg(x + static_cast<long long>(t) * row_vecs + v);
    }
  }
#pragma unroll
  for (int i = 0; i < kScatterTok; ++i) {
    const int t = t0 + i;
    if (t >= T) break;
    for (int j = 0; j < k; ++j) {
      int d = pos[static_cast<long long>(t) * k + j];
      if (d < 0 || d >= n_rows_out) {
        if (threadIdx.x == 0) atomicOr(status, kDevBadInput);
        continue;
      }
      uint4* dst = xp + static_cast<long long>(d) * row_vecs;
#pragma unroll
      for (int c = 0; c < VPT; ++c) {
        const int v = threadIdx.x + c * kRowThreads;
        if (v < row_vecs) dst[v] = val[i][c];
      }
    }
  }
}

__device__ __forceinline__ void acc_bf16x8(float (&a)[8], uint4 v, float w) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[2 * i] = __fmaf_rn(w, __uint_as_float(u[i] << 16), a[2 * i]);
    a[2 * i + 1] = __fmaf_rn(w, __uint_as_float(u[i] & 0xFFFF0000u), a[2 * i + 1]);
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// TOK tokens per block: out[t] = sum_j w[t,j] * Y[pos[t,j]] in fp32, j in
// order, each step one fused multiply-add (a = fma(w, y, a)) starting from
// a = 0. Every thread loads its vectors of the first KL sources of its TOK
// tokens before the arithmetic (further sources, k > KL, load as they go).
constexpr int kCombineTok = 1;
constexpr int kCombineKL = 2;

template <int VPT>
__global__ void __launch_bounds__(kRowThreads)
    combine_kernel(const uint4* __restrict__ Y, const int* __restrict__ pos,
                   const float* __restrict__ w, uint4* __restrict__ out, int T, int k,
                   int row_vecs, long long n_rows_y, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t0 = blockIdx.x * kCombineTok;
  int src[kCombineTok][8];
  float wt[kCombineTok][8];
#pragma unroll
  for (int i = 0; i < kCombineTok; ++i) {
    const int t = t0 + i;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool on = t < T && j < k;
      src[i][j] = on ? pos[static_cast<long long>(t) * k + j] : -1;
      wt[i][j] = on ? w[static_cast<long long>(t) * k + j] : 0.f;
      if (on && (src[i][j] < 0 || src[i][j] >= n_rows_y)) {
        if (threadIdx.x == 0) atomicOr(status, kDevBadInput);
        src[i][j] = -1;
      }
    }
  }
  uint4 y[kCombineTok][kCombineKL][VPT];
#pragma unroll
  for (int i = 0; i < kCombineTok; ++i)
#pragma unroll
    for (int j = 0; j < kCombineKL; ++j)
#pragma unroll
      for (int c = 0; c < VPT; ++c) {
        const int v = threadIdx.x + c * kRowThreads;
        if (src[i][j] >= 0 && v < row_vecs)
          y[i][j][c] = __ldg(Y + static_cast<long long>(src[i][j]) * row_vecs + v);
      }
#pragma unroll
  for (int i = 0; i < kCombineTok; ++i) {
    const int t = t0 + i;
    if (t >= T) break;
#pragma unroll
    for (int c = 0; c < VPT; ++c) {
      const int v = threadIdx.x + c * kRowThreads;
      if (v >= row_vecs) continue;
      float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (src[i][j] < 0) continue;
        const uint4 yv = j < kCombineKL
                             ? y[i][j < kCombineKL ? j : 0][c]
                             : __ldg(Y + static_cast<long long>(src[i][j]) * row_vecs + v);
        acc_bf16x8(a, yv, wt[i][j]);
      }
      uint4 o;
      o.x = pack2(a[0], a[1]);
      o.y = pack2(a[2], a[3]);
      o.z = pack2(a[4], a[5]);
      o.w = pack2(a[6], a[7]);
      out[static_cast<long long>(t) * row_vecs + v] = o;
    }
  }
}

int n_chunks_of(int T, int k) {
  return static_cast<int>((static_cast<long long>(T) * k + kPermChunk - 1) /
                          kPermChunk);
}

// The permutation's launches: histogram, then either the scans as their own
// single-block pass and the ranks, or (small count matrices) the ranks with
// the scans folded in.
// `pdl`: launch with programmatic dependent launch (the workspace entry point;
// the allocation-free one launches plainly).
int launch_permute(const int32_t* topk_idx, int n, int k, int E, int nc, int* counts,
                   int* base, int32_t* expert_offsets, int32_t* pos, int32_t* src_token,
                   int* status, cudaStream_t st, bool pdl) {
  KVM_CUDA_TRY(launch_ex(pdl, permute_count_kernel, dim3(nc), dim3(kPermChunk),
                         E * sizeof(int), st, topk_idx, n, E, counts, status));
  const size_t rank_smem = (kPermChunk / 32) * E * sizeof(int);
  if (static_cast<long long>(nc) * E <= 16 * 1024) {
    const size_t smem =
        rank_smem + (2 * E + 2 * (E > kPermChunk ? E : kPermChunk)) * sizeof(int);
    if (smem > 48 * 1024)
      KVM_CUDA_TRY(cudaFuncSetAttribute(permute_rank_kernel<true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(smem)));
    KVM_CUDA_TRY(launch_ex(pdl, permute_rank_kernel<true>, dim3(nc), dim3(kPermChunk), smem,
                           st, topk_idx, n, k, E, static_cast<const int*>(counts), pos,
                           src_token, nc, expert_offsets));
    return KVM_OK;
  }
  const int scan_threads = ((E + 31) / 32) * 32;
  KVM_CUDA_TRY(launch_ex(pdl, permute_scan_kernel, dim3(1), dim3(scan_threads),
                         E * sizeof(int), st, static_cast<const int*>(counts), nc, E, base,
                         expert_offsets));
  if (rank_smem > 48 * 1024)
    KVM_CUDA_TRY(cudaFuncSetAttribute(permute_rank_kernel<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(rank_smem)));
  KVM_CUDA_TRY(launch_ex(pdl, permute_rank_kernel<false>, dim3(nc), dim3(kPermChunk),
                         rank_smem, st, topk_idx, n, k, E, static_cast<const int*>(base), pos,
                         src_token, nc, expert_offsets));
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}


}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int64_t kvm_sm100_moe_permute_workspace(int T, int k, int E) {
  if (T <= 0 || k <= 0 || E <= 0) return 0;
  // counts and bases: n_chunks x E ints each.
  return 2ll * n_chunks_of(T, k) * E * static_cast<int64_t>(sizeof(int));
}

extern "C" int kvm_sm100_moe_permute(const int32_t* topk_idx, int T, int k,
                                     int E, int32_t* expert_offsets,
                                     int32_t* pos, int32_t* src_token,
                                     void* workspace, kvm_stream_t stream) {
  if (T <= 0 || k < 1 || k > 8 || E < 1 || E > kMaxExperts)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_permute: need T > 0, 1 <= k <= 8, 1 <= E <= 1024");
  if (static_cast<long long>(T) * k > (1ll << 30))
    return fail(KVM_ERR_INVALID_ARG, "moe_permute: T*k too large");
  if (!topk_idx || !expert_offsets || !pos || !src_token || !workspace)
    return fail(KVM_ERR_INVALID_ARG, "moe_permute: NULL pointer");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = T * k;
  const int nc = n_chunks_of(T, k);
  int* counts = static_cast<int*>(workspace);
  int* base = counts + static_cast<long long>(nc) * E;
  return launch_permute(topk_idx, n, k, E, nc, counts, base, expert_offsets, pos, src_token,
                        dev->status, st, true);
}

extern "C" int kvm_sm100_moe_scatter_rows(const void* x, const int32_t* pos,
                                          void* xp, int T, int k, int H,
                                          kvm_stream_t stream) {
  if (T <= 0 || k < 1 || k > 8 || H <= 0 || H % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_scatter_rows: need T > 0, 1 <= k <= 8, H % 8 == 0");
  if (!x || !pos || !xp || !aligned16(x) || !aligned16(xp))
    return fail(KVM_ERR_INVALID_ARG,
                "moe_scatter_rows: NULL or unaligned pointer");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const int row_vecs = H / 8;
  const unsigned blocks = static_cast<unsigned>((T + kScatterTok - 1) / kScatterTok);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n_out = static_cast<long long>(T) * k;
  const uint4* xv = static_cast<const uint4*>(x);
  uint4* xpv = static_cast<uint4*>(xp);
  if (row_vecs <= kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, scatter_rows_kernel<1>, dim3(blocks), dim3(kRowThreads), 0, st, xv, pos, xpv, T, k, row_vecs, n_out, dev->status));
  else if (row_vecs <= 2 * kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, scatter_rows_kernel<2>, dim3(blocks), dim3(kRowThreads), 0, st, xv, pos, xpv, T, k, row_vecs, n_out, dev->status));
  else if (row_vecs <= 4 * kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, scatter_rows_kernel<4>, dim3(blocks), dim3(kRowThreads), 0, st, xv, pos, xpv, T, k, row_vecs, n_out, dev->status));
  else
    return fail(KVM_ERR_UNSUPPORTED, "moe_scatter_rows: rows wider than 8192 elements");
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_moe_combine(const void* Y, const int32_t* pos,
                                     const float* w, void* out, int T, int k,
                                     int H, kvm_stream_t stream) {
  if (T <= 0 || k < 1 || k > 8 || H <= 0 || H % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_combine: need T > 0, 1 <= k <= 8, H % 8 == 0");
  if (!Y || !pos || !w || !out || !aligned16(Y) || !aligned16(out))
    return fail(KVM_ERR_INVALID_ARG, "moe_combine: NULL or unaligned pointer");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const int row_vecs = H / 8;
  const unsigned blocks = static_cast<unsigned>((T + kCombineTok - 1) / kCombineTok);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long n_y = static_cast<long long>(T) * k;
  const uint4* yv = static_cast<const uint4*>(Y);
  uint4* ov = static_cast<uint4*>(out);
  if (row_vecs <= kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, combine_kernel<1>, dim3(blocks), dim3(kRowThreads), 0, st, yv, pos, w, ov, T, k, row_vecs, n_y, dev->status));
  else if (row_vecs <= 2 * kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, combine_kernel<2>, dim3(blocks), dim3(kRowThreads), 0, st, yv, pos, w, ov, T, k, row_vecs, n_y, dev->status));
  else if (row_vecs <= 4 * kRowThreads)
    KVM_CUDA_TRY(launch_ex(true, combine_kernel<4>, dim3(blocks), dim3(kRowThreads), 0, st, yv, pos, w, ov, T, k, row_vecs, n_y, dev->status));
  else
    return fail(KVM_ERR_UNSUPPORTED, "moe_combine: rows wider than 8192 elements");
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free permute.
//
// Some callers cannot allocate GPU memory when they route tokens: a host
// program that loads this library through its FFI and owns every device
// buffer through its own memory pool (an allocation outside the pool breaks
// its accounting and can push the process past its HBM budget), or a serving
// loop that may not call cudaMalloc/cudaFree because they synchronise the
// device. For them the permute's scratch (per-chunk expert counts and bases)
// lives in the fixed array below instead of a caller-provided workspace.
//
// Every GPU that loads this library holds the array (512 KiB + 256 B) until
// the process exits. All calls on a device share it and it keeps the last
// call's contents: each call overwrites every cell it reads before reading it,
// so nothing has to start at zero. Calls whose kernels overlap on the GPU
// (two streams, or two host threads) race on the array and must not be issued.
namespace kvm {
namespace {

constexpr int kNoAllocMaxCells = KVM_SM100_NOALLOC_PERMUTE_MAX_CELLS;
// [0, cells): counts; [cells, 2*cells): bases; then the status word of this
// entry point (bit kDevBadInput: a pair named an expert outside [0, E)),
// read and cleared by kvm_sm100_moe_permute_noalloc_status.
static __device__ __align__(256) int g_permute_scratch[2 * kNoAllocMaxCells + 64];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
int* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_permute_scratch for the current device, looked up once
// per device (host code may not use the symbol itself: in host code its name
// is only a host-side stand-in).
int noalloc_scratch(int** out) {
  int dev = 0;
  KVM_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(KVM_ERR_UNSUPPORTED, "moe_permute_noalloc: device id too large");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_permute_scratch);
    if (e != cudaSuccess)
      return fail_cuda(e, "cudaGetSymbolAddress(g_permute_scratch)");
    g_noalloc_ptr[dev] = static_cast<int*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

extern "C" int kvm_sm100_moe_permute_noalloc_status(int* status_out, int clear) {
  int* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch); rc != KVM_OK) return rc;
  int* word = scratch + 2 * kNoAllocMaxCells;
  int v = 0;
  // Plain copies into and out of the static array: nothing is allocated.
  KVM_CUDA_TRY(cudaDeviceSynchronize());
  KVM_CUDA_TRY(cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear) {
    const int zero = 0;
    KVM_CUDA_TRY(cudaMemcpy(word, &zero, sizeof(int), cudaMemcpyHostToDevice));
  }
  if (status_out) *status_out = v;
  if (v & kDevBadInput)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_permute_noalloc: an expert index was outside [0, E)");
  return KVM_OK;
}

extern "C" int kvm_sm100_moe_permute_noalloc(const int32_t* topk_idx, int T,
                                             int k, int E,
                                             int32_t* expert_offsets,
                                             int32_t* pos, int32_t* src_token,
                                             kvm_stream_t stream) {
  if (T <= 0 || k < 1 || k > 8 || E < 1 || E > kMaxExperts)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_permute_noalloc: need T > 0, 1 <= k <= 8, 1 <= E <= 1024");
  if (static_cast<long long>(T) * k > (1ll << 30))
    return fail(KVM_ERR_INVALID_ARG, "moe_permute_noalloc: T*k too large");
  const long long nc = n_chunks_of(T, k);
  if (nc * E > kNoAllocMaxCells)
    return fail(KVM_ERR_INVALID_ARG,
                "moe_permute_noalloc: ceil(T*k/256) * E = " +
                    std::to_string(nc * E) + " exceeds the static scratch of " +
                    std::to_string(kNoAllocMaxCells) +
                    " cells; use kvm_sm100_moe_permute with a workspace");
  if (!topk_idx || !expert_offsets || !pos || !src_token)
    return fail(KVM_ERR_INVALID_ARG, "moe_permute_noalloc: NULL pointer");
  int* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch); rc != KVM_OK) return rc;
  int* counts = scratch;
  int* base = scratch + kNoAllocMaxCells;
  int* status = scratch + 2 * kNoAllocMaxCells;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = T * k;
  return launch_permute(topk_idx, n, k, E, static_cast<int>(nc), counts, base, expert_offsets,
                        pos, src_token, status, st, false);
}
