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

#include "ep_layout.h"
#include "ptx.cuh"
#include "runtime.h"

namespace kvm {
namespace {

enum FlagSlot { kFlagCounts = 0, kFlagData = 1, kFlagOutputs = 2 };

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

// ------------------------------------------- overlapped expert parallel ---
//
// ep_prepare: the count exchange of ep_counts, then, for the fused kernels of
// the call (gemm_pair.cuh, kEpDispatchGateUp / kEpDownPush): zeroed segment
// and CTA counters, the row prefix of this rank's remote segments in
// (local expert, peer) order, and for every row this rank will receive the
// rank and row its result goes back to. One block.
__global__ void ep_prepare_kernel(const kvm_ep_peers pr, const int* __restrict__ off,
                                  int* __restrict__ send_base, int* __restrict__ loc_off,
                                  EpWorkspace ws, long long cap_rows, unsigned epoch,
                                  int* status) {
  // tot [E], src_off [P][E], the count matrix [P][E], this rank's offsets
  // [E+1] and the first received row of each local expert [E/P], all in
  // shared memory: the scans below read no global memory
  extern __shared__ int sm[];
  int* tot = sm;
  int* src_off = sm + pr.E;
  int* scnt = src_off + pr.world * pr.E;
  int* soff = scnt + pr.world * pr.E;
  int* gstart = soff + pr.E + 1;
  const int P = pr.world, E = pr.E, me = pr.rank, epr = E / P;
  for (int i = threadIdx.x; i < P * E; i += blockDim.x) {
    const int d = i / E, e = i - d * E;
    reinterpret_cast<int*>(pr.cnt[d])[me * E + e] = off[e + 1] - off[e];
  }
  for (int i = threadIdx.x; i < E; i += blockDim.x) ws.seg_ctr[i] = 0;
  if (threadIdx.x == 0) *ws.done_ctr = 0;
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
  {
    const int* gcnt = reinterpret_cast<const int*>(pr.cnt[me]);  // [P][E], all rows in
    for (int i = threadIdx.x; i < P * E; i += blockDim.x) scnt[i] = gcnt[i];
    for (int i = threadIdx.x; i <= E; i += blockDim.x) soff[i] = off[i];
  }
  __syncthreads();
  const int* cnt = scnt;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int r = 0; r < P; ++r) s += cnt[r * E + e];
    tot[e] = s;
  }
  if (threadIdx.x < P) {  // every source's permuted offsets
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      src_off[threadIdx.x * E + e] = acc;
      acc += cnt[threadIdx.x * E + e];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int le = 0; le < epr; ++le) {
      loc_off[le] = acc;
      gstart[le] = acc;
      acc += tot[me * epr + le];
    }
    loc_off[epr] = acc;
    if (acc > cap_rows) atomicOr(status, kDevBadInput);
    int q = 0;  // remote segments of this rank's rows, (local expert, peer) order
    const int nseg = epr * (P - 1);
    for (int sg = 0; sg < nseg; ++sg) {
      ws.seg_prefix[sg] = q;
      const int le = sg / (P - 1);
      const int d = (me + 1 + sg % (P - 1)) % P;
      const int e = d * epr + le;
      q += soff[e + 1] - soff[e];
    }
    ws.seg_prefix[nseg] = q;
  }
  // token tile (of the fused gate/up GEMM's split of each local expert's rows
  // into ceil(rows / 256) tiles of equal width rounded up to 16) that holds
  // this rank's own rows: the GEMM starts each expert there
  for (int le = threadIdx.x; le < epr; le += blockDim.x) {
    const int e = me * epr + le;
    const int c = tot[e];
    const int tt = (c + 255) / 256;
    int first = 0;
    if (tt >= 2) {
      const int tn = ((c + tt - 1) / tt + 15) & ~15;
      int before = 0;
      for (int r = 0; r < me; ++r) before += cnt[r * E + e];
      first = min(tt - 1, before / tn);
    }
    ws.tile_first[le] = first;
  }
  // where this rank's rows of expert e start in the owner's receive buffer:
  // after the owner's earlier local experts, then after lower source ranks
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / epr, le = e - d * epr;
    int run = 0, before = 0;
    for (int x = 0; x < le; ++x) run += tot[d * epr + x];
    for (int r = 0; r < me; ++r) before += cnt[r * E + e];
    send_base[e] = run + before;
  }
  __syncthreads();
  // where each received row's result goes: rank s, row src_off[s][e] + j
  for (int le = 0; le < epr; ++le) {
    const int e = me * epr + le;
    int row = gstart[le];  // first received row of (le, source 0)
    for (int s = 0; s < P; ++s) {
      const int n = cnt[s * E + e];
      const int so = src_off[s * E + e];
      for (int j = threadIdx.x; j < n; j += blockDim.x)
        if (row + j < cap_rows) ws.push_row[row + j] = (s << 28) | (so + j);
      row += n;
    }
  }
}

// The rows this rank routes to its own experts, copied into its own receive
// buffer (the fused dispatch kernel sends only the other ranks' rows). These
// rows are a contiguous range of the permuted order (the local experts'
// groups); one warp per row, lanes on 16-byte vectors with every load of a
// pass issued before its stores.
__global__ void __launch_bounds__(256)
    ep_scatter_local_kernel(const kvm_ep_peers pr, const uint4* __restrict__ x,
                            const int* __restrict__ src_token, const int* __restrict__ off,
                            const int* __restrict__ send_base, long long cap_rows,
                            int* status) {
  const int epr = pr.E / pr.world, e0 = pr.rank * epr;
  const int r0 = off[e0], r1 = off[e0 + epr];
  const int lane = threadIdx.x % 32;
  const int r = r0 + static_cast<int>(blockIdx.x) * 8 + static_cast<int>(threadIdx.x / 32);
  if (r >= r1) return;
  int lo = e0, hi = e0 + epr - 1;  // local expert of row r: largest e with off[e] <= r
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= r) lo = mid; else hi = mid - 1;
  }
  const long long row = send_base[lo] + (r - off[lo]);
  if (row < 0 || row >= cap_rows) {
    if (lane == 0) atomicOr(status, kDevBadInput);
    return;
  }
  const int rv = pr.H / 8;
  const uint4* src = x + static_cast<long long>(src_token[r]) * rv;
  uint4* dst = reinterpret_cast<uint4*>(pr.recv[pr.rank]) + row * rv;
  for (int v0 = 0; v0 < rv; v0 += 32 * 8) {
    uint4 buf[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int v = v0 + u * 32 + lane;
      if (v < rv) buf[u] = __ldg(src + v);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int v = v0 + u * 32 + lane;
      if (v < rv) dst[v] = buf[u];
    }
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

extern "C" int64_t kvm_sm100_ep_overlap_workspace(int E, int64_t cap_rows) {
  if (E <= 0 || cap_rows <= 0) return 0;
  return ep_workspace_bytes(E, cap_rows);
}

extern "C" int kvm_sm100_ep_prepare(const kvm_ep_peers* pr, const int32_t* offsets,
                                    int32_t* send_base, int32_t* local_offsets,
                                    void* workspace, int64_t cap_rows, uint32_t epoch,
                                    kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (!offsets || !send_base || !local_offsets || !workspace || cap_rows <= 0 ||
      cap_rows >= (1ll << 28) || epoch == 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_prepare: NULL pointer, cap_rows or epoch 0");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const EpWorkspace ws = ep_workspace(workspace, pr->E, cap_rows);
  const size_t smem = sizeof(int) * (static_cast<size_t>(pr->E) * (1 + 2 * pr->world) +
                                     pr->E + 1 + pr->E / pr->world);
  if (smem > 48 * 1024)
    KVM_CUDA_TRY(cudaFuncSetAttribute(ep_prepare_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
  ep_prepare_kernel<<<1, 1024, smem, static_cast<cudaStream_t>(stream)>>>(
      *pr, offsets, send_base, local_offsets, ws, cap_rows, epoch, dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_ep_scatter_local(const kvm_ep_peers* pr, const void* x,
                                          const int32_t* src_token, const int32_t* offsets,
                                          const int32_t* send_base, int T, int64_t cap_rows,
                                          kvm_stream_t stream) {
  if (int rc = check_peers(pr); rc != KVM_OK) return rc;
  if (T <= 0 || !x || !aligned16(x) || !src_token || !offsets || !send_base ||
      cap_rows <= 0)
    return fail(KVM_ERR_INVALID_ARG, "ep_scatter_local: bad argument");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  const long long rows = static_cast<long long>(T) * pr->k;  // at most this many local
  ep_scatter_local_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0,
                            static_cast<cudaStream_t>(stream)>>>(
      *pr, static_cast<const uint4*>(x), src_token, offsets, send_base, cap_rows,
      dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
