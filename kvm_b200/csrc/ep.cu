// Expert-parallel MoE exchange over NVLink peer memory.
//
// The ranks of one node map each other's receive buffers, expert-output
// buffers, count matrices and flag words (CUDA IPC). One layer call:
//
//   ep_counts    every rank stores its per-expert pair counts into every
//                rank's count matrix [P][E] (peer stores), raises a flag, waits
//                for all P flags, then derives on the device: the group
//                offsets of its local experts (rows arrive expert-major, then
//                source-rank-major) and, for every global expert, the row where
//                this rank's pairs start in the owner's receive buffer.
//   ep_dispatch  the scatter of moe_dispatch fused with the all-to-all: each
//                token row is read once and stored straight into the owner's
//                receive buffer (peer stores); the last block raises the
//                data-ready flags.
//   ep_wait      (before the grouped GEMMs) waits for every source's flag.
//   ep_signal    (after the grouped GEMMs) raises the outputs-ready flags.
//   ep_combine   moe_combine fused with the reverse all-to-all: each pair's
//                expert output row is loaded from the owner's output buffer
//                (peer loads) at the row the dispatch wrote its input to.
//
// Flags hold the call's epoch (1, 2, ...), so no flag is ever reset. Every
// wait is bounded (kWaitTimeoutNs); a timeout sets the status word and the
// kernel returns. Peer data is written before a system-scope fence and a
// release store of the flag; readers acquire the flag before reading.
#include <cuda_bf16.h>

#include <cstring>

#include "ptx.cuh"
#include "runtime.h"

namespace kvm {
namespace {

enum FlagSlot { kFlagCounts = 0, kFlagData = 1, kFlagOutputs = 2 };

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *flag >= epoch (epochs only grow). False on timeout.
__device__ bool wait_flag(const unsigned* flag, unsigned epoch) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys(flag) >= epoch) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) return false;
    __nanosleep(64);
  }
}

__device__ __forceinline__ unsigned* flag_of(const kvm_ep_peers& pr, int owner,
                                             int slot, int src) {
  return reinterpret_cast<unsigned*>(pr.flags[owner]) + slot * pr.world + src;
}

// One block. Publishes counts, waits for everyone's, derives the layout.
__global__ void ep_counts_kernel(const kvm_ep_peers pr, const int* __restrict__ off,
                                 int* __restrict__ send_base,
                                 int* __restrict__ loc_off, unsigned epoch,
                                 int* status) {
  extern __shared__ int tot[];  // [E]
  const int P = pr.world, E = pr.E, me = pr.rank, epr = E / P;
  for (int i = threadIdx.x; i < P * E; i += blockDim.x) {
    const int d = i / E, e = i - d * E;
    reinterpret_cast<int*>(pr.cnt[d])[me * E + e] = off[e + 1] - off[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < P) st_release_sys(flag_of(pr, threadIdx.x, kFlagCounts, me), epoch);
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < P &&
      !wait_flag(flag_of(pr, me, kFlagCounts, threadIdx.x), epoch)) {
    atomicOr(status, kDevWaitTimeout);
    failed = 1;
  }
  __syncthreads();
  if (failed) return;
  const int* cnt = reinterpret_cast<const int*>(pr.cnt[me]);  // [P][E], all rows in
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int r = 0; r < P; ++r) s += cnt[r * E + e];
    tot[e] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int le = 0; le < epr; ++le) {
      loc_off[le] = acc;
      acc += tot[me * epr + le];
    }
    loc_off[epr] = acc;
    for (int d = 0; d < P; ++d) {
      int run = 0;  // start of local expert le inside rank d's receive buffer
      for (int le = 0; le < epr; ++le) {
        const int e = d * epr + le;
        int before = 0;  // rows of expert e from sources ranked below me
        for (int r = 0; r < me; ++r) before += cnt[r * E + e];
        send_base[e] = run + before;
        run += tot[e];
      }
    }
  }
}

// One block per token: the row is read once and stored to each pair's slot in
// the owner's receive buffer. The last block to finish raises the data flags.
__global__ void __launch_bounds__(256)
    ep_dispatch_kernel(const kvm_ep_peers pr, const uint4* __restrict__ x,
                       const int* __restrict__ idx, const int* __restrict__ pos,
                       const int* __restrict__ off, const int* __restrict__ send_base,
                       unsigned* done, unsigned epoch, long long cap_rows,
                       int* status) {
  const int t = blockIdx.x, k = pr.k, epr = pr.E / pr.world;
  const int row_vecs = pr.H / 8;
  uint4* dst[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    dst[j] = nullptr;
    if (j < k) {
      const int e = idx[static_cast<long long>(t) * k + j];
      if (e >= 0 && e < pr.E) {
        const int d = e / epr;
        const long long row =
            send_base[e] + (pos[static_cast<long long>(t) * k + j] - off[e]);
        if (row >= 0 && row < cap_rows)
          dst[j] = reinterpret_cast<uint4*>(pr.recv[d]) + row * row_vecs;
        else if (threadIdx.x == 0)
          atomicOr(status, kDevBadInput);
      } else if (threadIdx.x == 0) {
        atomicOr(status, kDevBadInput);
      }
    }
  }
  const uint4* src = x + static_cast<long long>(t) * row_vecs;
  for (int v = threadIdx.x; v < row_vecs; v += blockDim.x) {
    const uint4 val = __ldg(src + v);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (dst[j]) dst[j][v] = val;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {  // every block's stores are fenced
      *done = 0;
      __threadfence_system();
      for (int d = 0; d < pr.world; ++d)
        st_release_sys(flag_of(pr, d, kFlagData, pr.rank), epoch);
    }
  }
}

__global__ void ep_wait_kernel(const kvm_ep_peers pr, int slot, unsigned epoch,
                               int* status) {
  if (threadIdx.x < pr.world &&
      !wait_flag(flag_of(pr, pr.rank, slot, threadIdx.x), epoch))
    atomicOr(status, kDevWaitTimeout);
}

__global__ void ep_signal_kernel(const kvm_ep_peers pr, int slot, unsigned epoch) {
  __threadfence_system();
  if (threadIdx.x < pr.world)
    st_release_sys(flag_of(pr, threadIdx.x, slot, pr.rank), epoch);
}

__device__ __forceinline__ void acc8(float (&a)[8], uint4 v, float w) {
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

// One block per token: out[t] = sum_j w[t,j] * Y_owner[row(t,j)], fp32, one
// fused multiply-add per slot in slot order (same arithmetic as the
// single-GPU combine).
__global__ void __launch_bounds__(256)
    ep_combine_kernel(const kvm_ep_peers pr, const int* __restrict__ idx,
                      const int* __restrict__ pos, const int* __restrict__ off,
                      const int* __restrict__ send_base, const float* __restrict__ w,
                      uint4* __restrict__ out, long long cap_rows, int* status) {
  const int t = blockIdx.x, k = pr.k, epr = pr.E / pr.world;
  const int row_vecs = pr.H / 8;
  const uint4* src[8];
  float wt[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    src[j] = nullptr;
    wt[j] = 0.f;
    if (j < k) {
      const int e = idx[static_cast<long long>(t) * k + j];
      wt[j] = w[static_cast<long long>(t) * k + j];
      if (e >= 0 && e < pr.E) {
        const long long row =
            send_base[e] + (pos[static_cast<long long>(t) * k + j] - off[e]);
        if (row >= 0 && row < cap_rows)
          src[j] = reinterpret_cast<const uint4*>(pr.y[e / epr]) + row * row_vecs;
        else if (threadIdx.x == 0)
          atomicOr(status, kDevBadInput);
      } else if (threadIdx.x == 0) {
        atomicOr(status, kDevBadInput);
      }
    }
  }
  for (int v = threadIdx.x; v < row_vecs; v += blockDim.x) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (src[j]) acc8(a, src[j][v], wt[j]);
    out[static_cast<long long>(t) * row_vecs + v] =
        make_uint4(pack2(a[0], a[1]), pack2(a[2], a[3]), pack2(a[4], a[5]),
                   pack2(a[6], a[7]));
  }
}

int check_peers(const kvm_ep_peers* pr) {
  if (!pr) return fail(KVM_ERR_INVALID_ARG, "ep: NULL peer table");
  if (pr->world < 1 || pr->world > KVM_EP_MAX_RANKS || pr->rank < 0 ||
      pr->rank >= pr->world)
    return fail(KVM_ERR_INVALID_ARG, "ep: bad rank / world");
  if (pr->E < 1 || pr->E > 1024 || pr->E % pr->world != 0)
    return fail(KVM_ERR_INVALID_ARG, "ep: E must be 1..1024 and divisible by world");
  if (pr->k < 1 || pr->k > 8 || pr->H <= 0 || pr->H % 8 != 0)
    return fail(KVM_ERR_INVALID_ARG, "ep: need 1 <= k <= 8 and H % 8 == 0");
  for (int r = 0; r < pr->world; ++r)
    if (!pr->recv[r] || !pr->y[r] || !pr->cnt[r] || !pr->flags[r])
      return fail(KVM_ERR_INVALID_ARG, "ep: missing peer buffer");
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int kvm_sm100_ipc_alloc(int64_t bytes, void** ptr) {
  if (bytes <= 0 || !ptr) return fail(KVM_ERR_INVALID_ARG, "ipc_alloc: bad size");
  KVM_CUDA_TRY(cudaMalloc(ptr, static_cast<size_t>(bytes)));
  KVM_CUDA_TRY(cudaMemset(*ptr, 0, static_cast<size_t>(bytes)));
  return KVM_OK;
}

extern "C" int kvm_sm100_ipc_free(void* ptr) {
  KVM_CUDA_TRY(cudaFree(ptr));
  return KVM_OK;
}

extern "C" int kvm_sm100_ipc_get_handle(const void* ptr, void* handle64) {
  if (!ptr || !handle64) return fail(KVM_ERR_INVALID_ARG, "ipc_get_handle: NULL");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  KVM_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  memcpy(handle64, &h, 64);
  return KVM_OK;
}

extern "C" int kvm_sm100_ipc_open_handle(const void* handle64, void** peer_ptr) {
  if (!handle64 || !peer_ptr) return fail(KVM_ERR_INVALID_ARG, "ipc_open: NULL");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  KVM_CUDA_TRY(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return KVM_OK;
}

extern "C" int kvm_sm100_ipc_close(void* peer_ptr) {
  KVM_CUDA_TRY(cudaIpcCloseMemHandle(peer_ptr));
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_counts(const kvm_ep_peers* pr, const int32_t* offsets,
                                   int32_t* send_base, int32_t* local_offsets,
                                   uint32_t epoch, kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (!offsets || !send_base || !local_offsets || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_counts: NULL pointer or epoch 0");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  ep_counts_kernel<<<1, 1024, pr->E * sizeof(int), static_cast<cudaStream_t>(stream)>>>(
      *pr, offsets, send_base, local_offsets, epoch, dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_dispatch(const kvm_ep_peers* pr, const void* x,
                                     const int32_t* topk_idx, const int32_t* pos,
                                     const int32_t* offsets, const int32_t* send_base,
                                     int T, int64_t cap_rows, uint32_t* done,
                                     uint32_t epoch, kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (T <= 0 || !x || !aligned16(x) || !topk_idx || !pos || !offsets || !send_base ||
      !done || cap_rows <= 0 || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_dispatch: bad argument");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  ep_dispatch_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      *pr, static_cast<const uint4*>(x), topk_idx, pos, offsets, send_base, done, epoch,
      cap_rows, dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_wait(const kvm_ep_peers* pr, int slot, uint32_t epoch,
                                 kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (slot < 0 || slot > 2 || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_wait: bad slot or epoch 0");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  ep_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*pr, slot, epoch,
                                                                  dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_signal(const kvm_ep_peers* pr, int slot, uint32_t epoch,
                                   kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (slot < 0 || slot > 2 || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_signal: bad slot or epoch 0");
  ep_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*pr, slot, epoch);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_combine(const kvm_ep_peers* pr, const int32_t* topk_idx,
                                    const int32_t* pos, const int32_t* offsets,
                                    const int32_t* send_base, const float* topk_w,
                                    void* out, int T, int64_t cap_rows,
                                    kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (T <= 0 || !out || !aligned16(out) || !topk_idx || !pos || !offsets ||
      !send_base || !topk_w || cap_rows <= 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_combine: bad argument");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  ep_combine_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      *pr, topk_idx, pos, offsets, send_base, topk_w, static_cast<uint4*>(out), cap_rows,
      dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
