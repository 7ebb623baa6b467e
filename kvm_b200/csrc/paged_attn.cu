// Paged KV cache and decode attention: kernel.kvcache.write / kvcache.read
// (src/ir/dialect/kernel/dialect.cpp:69-70) and kernel.attn.decode
// (dialect.cpp:39) over the paged layout KVMeta describes
// (src/ir/graph_config.h:20-39): pages of block_size token slots, each slot
// holding K (or V) for all kv heads of one layer, located by element strides
// (page, layer, kv, token) so page_first and layer_first pools share one
// kernel.
//
// Decode attention is split over the key axis (flash-decoding): a work item
// is (sequence, kv head, group of query rows, chunk of 1024 keys); it writes
// an unnormalised partial (O, running max m, sum l per query column) and a
// combine kernel merges the chunks. Inside an item the math runs on the
// tensor cores with the query rows x heads as the MMA's N (at most 32):
//   S^T = K . Q^T     M = 128 keys,  N = rows*heads, K = 128 dims
//   O^T += V^T . P^T  M = 128 dims,  N = rows*heads, K = 128 keys
// K and V pages land in shared memory by TMA straight from the page table
// (one box per page half), so the cache is never gathered in HBM.
//
//   warp 0             TMA producer: the warp reads an item's page ids into
//                      shared memory, then per 128-key tile one lane per
//                      page issues its K and V boxes into two 3-stage rings
//   warp 1 (one lane)  MMA issuer: S_0, then S_{j+1} before PV_j (S and P
//                      double-buffered), so softmax j overlaps the next S
//   warps 2..5         thread = key (S^T lanes) and = head dim (O^T lanes):
//                      causal mask, per-column max by a warp transpose
//                      reduction + one shared-memory exchange per tile,
//                      P = 2^(s - m) into shared memory, sums kept per
//                      thread until the item ends; O rescaled in TMEM only
//                      when a column's max grows by more than 2^8.
#include <cuda_bf16.h>

#include "gemm_bf16.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace kvm {
namespace {

#define KVM_TRY(expr)                      \
  do {                                     \
    int kvm_rc_ = (expr);                  \
    if (kvm_rc_ != KVM_OK) return kvm_rc_; \
  } while (0)

constexpr int kDecThreads = 192;
constexpr int kDecMaxN = 32;           // query rows x heads per item
constexpr int kDecStages = 3;          // K ring and V ring, 3 tiles each
constexpr int kDecChunk = 1024;        // at most this many keys per item
constexpr uint32_t kDecHalf = 128 * 64 * 2;    // 128 keys x 64 dims: 16 KB
constexpr uint32_t kDecTile = 2 * kDecHalf;    // 128 keys x 128 dims: 32 KB
constexpr uint32_t kDecOffK = 0;
constexpr uint32_t kDecOffV = kDecStages * kDecTile;
constexpr uint32_t kDecOffQ = 2 * kDecStages * kDecTile;
constexpr uint32_t kDecQBytes = 2 * kDecMaxN * 128;   // 2 atoms x 32 rows: 8 KB
constexpr uint32_t kDecOffP = kDecOffQ + kDecQBytes;  // [2] P^T buffers
constexpr uint32_t kDecOffRed = kDecOffP + 2 * kDecQBytes;  // [2][4][32] floats
constexpr uint32_t kDecOffPages = kDecOffRed + 2 * 4 * 32 * 4;  // page ids of an item
constexpr int kDecMaxPages = kDecChunk / 16 + 1;
constexpr uint32_t kDecOffBar = kDecOffPages + ((kDecMaxPages * 4 + 15) & ~15);
constexpr int kDecBars = 4 * kDecStages + 15;  // == kBarCount
constexpr float kDecRescale = 8.0f;

constexpr size_t dec_smem_bytes() { return 1024 + kDecOffBar + kDecBars * 8 + 16; }

// Keys of a group are split into nch = ceil(need / 1024) chunks of equal
// size (a multiple of 128): chunk c covers [c * size, min((c+1) * size, need)).
__host__ __device__ __forceinline__ int dec_chunks(int need) {
  return (need + kDecChunk - 1) / kDecChunk;
}
__host__ __device__ __forceinline__ int dec_chunk_size(int need) {
  const int n = dec_chunks(need);
  return n ? (((need + n - 1) / n + 127) & ~127) : 0;
}

struct DecParams {
  const __nv_bfloat16* q;
  long long ldq;
  int S, HKV, group;   // group = query heads per kv head
  int nqg;             // query rows per item (kDecMaxN / group)
  int QG, C;           // query-row groups and key chunks per (sequence, kv head)
  const int* q_off;
  const int* q_pos;
  const int* bt;
  const int* bt_off;
  int block_size, box_rows, num_pages;
  long long page_rows, layer_rows, kv_rows;  // strides in token slots
  int layer;
  float scale_log2;
  float* ws_o;   // [items][32][128]
  float* ws_ml;  // [items][2][32]
  int* status;
};

struct DecItem {
  int s, kh, qg, c;
  int r_begin, nq;   // query rows [r_begin, r_begin + nq)
  int pos0;          // position of query row r_begin
  int need;          // keys the group attends to: pos0 + nq
  int t_begin, t_end;
};

__device__ __forceinline__ DecItem dec_item(const DecParams& p, int w) {
  DecItem it;
  it.c = w % p.C;
  int rest = w / p.C;
  it.qg = rest % p.QG;
  rest /= p.QG;
  it.kh = rest % p.HKV;
  it.s = rest / p.HKV;
  const int q0 = p.q_off[it.s], q1 = p.q_off[it.s + 1];
  it.r_begin = q0 + it.qg * p.nqg;
  it.nq = min(p.nqg, q1 - it.r_begin);
  it.pos0 = p.q_pos[it.s] + (it.r_begin - q0);
  it.need = it.nq > 0 ? it.pos0 + it.nq : 0;
  const int csz = dec_chunk_size(it.need);
  it.t_begin = it.c < dec_chunks(it.need) ? it.c * csz : it.need;
  it.t_end = min(it.t_begin + csz, it.need);
  return it;
}

// Column reduction over a warp: v[NC] holds this lane's values of NC
// columns; on return lane l holds the reduction over all 32 lanes of column
// l % NC (fold the lanes that carry the same columns, then a transpose
// reduction: 31 shuffles for NC = 32 or 16).
template <int NC, bool MAX>
__device__ __forceinline__ float warp_columns(float (&v)[NC], int lane) {
#pragma unroll
  for (int o = 16; o >= NC; o >>= 1) {
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const float r = __shfl_xor_sync(0xffffffffu, v[i], o);
      v[i] = MAX ? fmaxf(v[i], r) : v[i] + r;
    }
  }
#pragma unroll
  for (int o = NC / 2; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, o);
      v[i] = MAX ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return v[0];
}

template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[NC]) {
  if constexpr (NC == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
}
template <int NC>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[NC]) {
  if constexpr (NC == 32) tmem_st32(taddr, r); else tmem_st16(taddr, r);
}

// Barrier slots in shared memory (kDecOffBar): K ring full/empty, V ring
// full/empty (kDecStages each), then the named singles below.
enum DecBar : int {
  kBarKFull = 0,
  kBarKEmpty = kDecStages,
  kBarVFull = 2 * kDecStages,
  kBarVEmpty = 3 * kDecStages,
  kBarQFull = 4 * kDecStages,  // 128 arrivals
  kBarQEmpty,
  kBarSFull,                   // [2]
  kBarSFree = kBarSFull + 2,   // [2] 128 arrivals
  kBarPFull = kBarSFree + 2,   // [2] 128 arrivals
  kBarPFree = kBarPFull + 2,   // [2]
  kBarODone = kBarPFree + 2,   // every PV
  kBarOFinal,                  // last PV of an item
  kBarOFree,                   // 128 arrivals: O read out
  kBarRed,                     // 128 arrivals
  kBarDrain,
  kBarCount
};

// The tiles of one item with NC (16 or 32) query columns, then the item's
// partial. Returns false when a wait gave up.
template <int NC>
__device__ __forceinline__ bool dec_softmax_item(const DecParams& p, uint8_t* smem,
                                                 volatile int* abort_flag,
                                                 uint32_t tmem_base, int qw, int lane,
                                                 const DecItem& it, int w, uint32_t& kt,
                                                 uint32_t& rb, uint32_t ic) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecOffBar);
  float* red = reinterpret_cast<float*>(smem + kDecOffRed);
  const int t = qw * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
  const uint32_t tmem_o = tmem_base + 64;
  const int ncol = it.nq * p.group;
  const int n_tiles = (it.t_end - it.t_begin + 127) / 128;
  float mref[NC], lsum[NC];
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    mref[i] = -INFINITY;
    lsum[i] = 0.f;
  }
  for (int j = 0; j < n_tiles; ++j) {
    const uint32_t tt = kt + j;
    const int b = tt & 1;
    const int t0 = it.t_begin + j * 128;
    const bool ready = mbar_wait(&(bars + kBarSFull)[b], (tt >> 1) & 1, abort_flag);
    if (!__all_sync(0xffffffffu, ready)) return false;
    tc_fence_after();
    float s[NC];
    {
      uint32_t u[NC];
      tmem_ld_cols<NC>(tmem_base + lane_off + b * 32, u);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < NC; ++i) s[i] = __uint_as_float(u[i]);
    }
    tc_fence_before();
    mbar_arrive(&(bars + kBarSFree)[b]);
    // Column n = query row n / group: key visible iff key <= pos0 + n / group,
    // i.e. n >= (key - pos0) * group.
    const int key = t0 + t;
    const int thr = key > it.pos0 ? min((key - it.pos0) * p.group, NC) : 0;
#pragma unroll
    for (int n = 0; n < NC; ++n)
      s[n] = (n >= thr && n < ncol) ? s[n] * p.scale_log2 : -INFINITY;
    // Keys past the last written one (only in the last tile): zero their
    // V rows, once V has landed, so 0 * stale data cannot poison P.V.
    if (t0 + 128 > it.need) {
      const int st = tt % kDecStages;
      const bool vin = mbar_wait(&(bars + kBarVFull)[st], (tt / kDecStages) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, vin)) return false;
      if (key >= it.need) {
        uint8_t* vrow = smem + kDecOffV + st * kDecTile + t * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          *reinterpret_cast<uint4*>(vrow + q * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vrow + kDecHalf + q * 16) = make_uint4(0, 0, 0, 0);
        }
      }
    }
    // ---- tile max per column: warp reduction, then across the 4 warps
    float tmp[NC];
#pragma unroll
    for (int n = 0; n < NC; ++n) tmp[n] = s[n];
    float* rbuf = red + (rb & 1) * 128;
    rbuf[qw * 32 + lane] = warp_columns<NC, true>(tmp, lane);
    mbar_arrive((bars + kBarRed));
    const bool synced = mbar_wait((bars + kBarRed), rb & 1, abort_flag);
    ++rb;
    if (!__all_sync(0xffffffffu, synced)) return false;
    const float mcol = fmaxf(fmaxf(rbuf[lane], rbuf[32 + lane]),
                             fmaxf(rbuf[64 + lane], rbuf[96 + lane]));
    // lane l owns column l % NC: rescale when any column outgrew its reference
    float my_ref = -INFINITY;
#pragma unroll
    for (int n = 0; n < NC; ++n)
      if (n == (lane & (NC - 1))) my_ref = mref[n];
    const bool grow = j == 0 ? (mcol > -INFINITY) : (mcol > my_ref + kDecRescale);
    if (__any_sync(0xffffffffu, grow)) {
      const float mnew = fmaxf(my_ref, mcol);
      const float alpha = (my_ref == -INFINITY) ? 0.f : ex2_approx(my_ref - mnew);
      if (j > 0) {
        // PV_{j-1} must have landed (PV_{j-2} has: S_j was issued after it)
        const bool done = mbar_wait((bars + kBarODone), (tt - 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, done)) return false;
        tc_fence_after();
        uint32_t u[NC];
        tmem_ld_cols<NC>(tmem_o + lane_off, u);
        tmem_wait_ld();
#pragma unroll
        for (int n = 0; n < NC; ++n)
          u[n] = __float_as_uint(__uint_as_float(u[n]) * __shfl_sync(0xffffffffu, alpha, n));
        tmem_st_cols<NC>(tmem_o + lane_off, u);
        tmem_wait_st();
      }
#pragma unroll
      for (int n = 0; n < NC; ++n) {
        lsum[n] *= __shfl_sync(0xffffffffu, alpha, n);
        mref[n] = __shfl_sync(0xffffffffu, mnew, n);
      }
    }
    // ---- P^T: row n, key t (two 128-byte-swizzled halves of 64 keys)
    const bool pfree = mbar_wait(&(bars + kBarPFree)[b], ((tt >> 1) & 1) ^ 1, abort_flag);
    if (!__all_sync(0xffffffffu, pfree)) return false;
    uint8_t* pbase = smem + kDecOffP + b * kDecQBytes + (t >> 6) * (kDecQBytes / 2);
    const int kb = (t & 63) * 2;
    const int kq = kb >> 4, kr = kb & 15;
#pragma unroll
    for (int n = 0; n < NC; ++n) {
      const float e = s[n] == -INFINITY ? 0.f : ex2_approx(s[n] - mref[n]);
      lsum[n] += e;
      *reinterpret_cast<__nv_bfloat16*>(pbase + n * 128 + ((kq ^ (n & 7)) << 4) + kr) =
          __float2bfloat16_rn(e);
    }
    fence_async_smem();
    tc_fence_before();
    mbar_arrive(&(bars + kBarPFull)[b]);
  }
  kt += n_tiles;
  // ---- item partial: O^T (unnormalised), m and l per column
  const bool fin = mbar_wait((bars + kBarOFinal), ic & 1, abort_flag);
  if (!__all_sync(0xffffffffu, fin)) return false;
  tc_fence_after();
  {
    uint32_t u[NC];
    tmem_ld_cols<NC>(tmem_o + lane_off, u);
    tmem_wait_ld();
    float* o = p.ws_o + static_cast<long long>(w) * 32 * 128 + t;
#pragma unroll
    for (int n = 0; n < NC; ++n)
      if (n < ncol) o[n * 128] = __uint_as_float(u[n]);
  }
  tc_fence_before();
  mbar_arrive((bars + kBarOFree));
  // l: sum over the 128 threads, column l on lane l
  float* rbuf = red + (rb & 1) * 128;
  rbuf[qw * 32 + lane] = warp_columns<NC, false>(lsum, lane);
  mbar_arrive((bars + kBarRed));
  const bool synced = mbar_wait((bars + kBarRed), rb & 1, abort_flag);
  ++rb;
  if (!__all_sync(0xffffffffu, synced)) return false;
  if (qw == 0 && lane < NC) {
    float my_ref = -INFINITY;
#pragma unroll
    for (int n = 0; n < NC; ++n)
      if (n == lane) my_ref = mref[n];
    p.ws_ml[static_cast<long long>(w) * 64 + lane] = my_ref;
    p.ws_ml[static_cast<long long>(w) * 64 + 32 + lane] =
        rbuf[lane] + rbuf[32 + lane] + rbuf[64 + lane] + rbuf[96 + lane];
  }
  return true;
}

// NC = 16 when every item has at most 16 query columns (decode of one or two
// rows at 8 query heads per kv head), else 32.
template <int NC>
__global__ void __launch_bounds__(kDecThreads, 1)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmKV,
                       const __grid_constant__ DecParams p,
                       int n_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + kDecOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kDecOffBar);
  uint64_t* k_full = bars + kBarKFull;
  uint64_t* k_empty = bars + kBarKEmpty;
  uint64_t* v_full = bars + kBarVFull;
  uint64_t* v_empty = bars + kBarVEmpty;
  uint64_t* q_full = bars + kBarQFull;
  uint64_t* q_empty = bars + kBarQEmpty;
  uint64_t* s_full = bars + kBarSFull;
  uint64_t* s_free = bars + kBarSFree;
  uint64_t* p_full = bars + kBarPFull;
  uint64_t* p_free = bars + kBarPFree;
  uint64_t* o_done = bars + kBarODone;
  uint64_t* o_final = bars + kBarOFinal;
  uint64_t* o_free = bars + kBarOFree;
  uint64_t* red_bar = bars + kBarRed;
  uint64_t* drain = bars + kBarDrain;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kDecBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(q_full, 128);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    mbar_init(o_free, 128);
    mbar_init(red_bar, 128);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmKV);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;    // S^T buffers: cols [0,32), [32,64)
  const uint32_t tmem_o = tmem_base + 64;   // O^T: cols [64,96)

  if (warp == 0) {
    // -------------------------------------------------- TMA producer
    // The whole warp reads the item's page ids into shared memory (off the
    // load path), then issues each tile's boxes, K before V.
    int* page_ids = reinterpret_cast<int*>(smem + kDecOffPages);
    uint32_t kt = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const DecItem it = dec_item(p, w);
      if (it.t_begin >= it.t_end) continue;
      const int pg0 = it.t_begin / p.block_size;
      const int npg = (it.t_end - 1) / p.block_size - pg0 + 1;
      const int bt0 = p.bt_off[it.s], bt_n = p.bt_off[it.s + 1] - bt0;
      for (int i = lane; i < npg; i += 32) {
        const int idx = pg0 + i;
        const int page = idx < bt_n ? p.bt[bt0 + idx] : -1;
        // Pages outside the pool or the table are reported and skipped
        // (their keys then hold stale data: the result is undefined but
        // every access stays inside the pool).
        const bool good = page >= 0 && page < p.num_pages;
        if (!good && p.status) atomicOr(p.status, kDevBadInput);
        page_ids[i] = good ? page : -1;
      }
      __syncwarp();
      // Lane 0 claims the ring slot and sets the byte count; lane sg then
      // issues page segment sg's boxes (up to 8 per 128-key tile), so small
      // pages do not serialise on one issuing thread.
      for (int t0 = it.t_begin; t0 < it.t_end && ok; t0 += 128, ++kt) {
        const int st = kt % kDecStages;
        const uint32_t eph = ((kt / kDecStages) & 1) ^ 1;
        const int t1 = min(t0 + 128, it.t_end);
        const int segs = (t1 - t0 + p.box_rows - 1) / p.box_rows;
        const int my_page =
            lane < segs ? page_ids[(t0 + lane * p.box_rows) / p.block_size - pg0] : -1;
        const uint32_t loaded = __popc(__ballot_sync(0xffffffffu, my_page >= 0));
        const uint32_t bytes = loaded * p.box_rows * 128u * 2u;
        for (int kv = 0; kv < 2 && ok; ++kv) {
          uint64_t* full = kv ? &v_full[st] : &k_full[st];
          bool got = true;
          if (lane == 0) {
            got = mbar_wait(kv ? &v_empty[st] : &k_empty[st], eph, abort_flag);
            if (got) mbar_arrive_expect_tx(full, bytes);
          }
          ok = __shfl_sync(0xffffffffu, got, 0);
          if (!ok) break;
          if (my_page >= 0) {
            const int tok = t0 + lane * p.box_rows;
            const int row = static_cast<int>(my_page * p.page_rows + p.layer * p.layer_rows +
                                             kv * p.kv_rows + tok % p.block_size);
            uint8_t* dst = smem + (kv ? kDecOffV : kDecOffK) + st * kDecTile +
                           lane * p.box_rows * 128u;
            tma_load_2d(dst, &tmKV, full, it.kh * 128, row);
            tma_load_2d(dst + kDecHalf, &tmKV, full, it.kh * 128 + 64, row);
          }
        }
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      // Order per item: S_0, then for each tile j: S_{j+1}, PV_j, so the
      // softmax of tile j overlaps the next tile's S.
      const uint32_t q_addr = smem_u32(smem + kDecOffQ);
      uint32_t kt = 0, ic = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
        const DecItem it = dec_item(p, w);
        if (it.t_begin >= it.t_end) continue;
        const int n = (it.t_end - it.t_begin + 127) / 128;
        const int npad = (it.nq * p.group + 15) & ~15;
        const uint32_t idesc_s = idesc_bf16(128, npad, 0, 0);
        const uint32_t idesc_o = idesc_bf16(128, npad, 1, 0);
        if (!mbar_wait(q_full, ic & 1, abort_flag)) { ok = false; break; }
        auto issue_s = [&](int j) -> bool {
          const uint32_t t = kt + j;
          const int st = t % kDecStages, b = t & 1;
          if (!mbar_wait(&k_full[st], (t / kDecStages) & 1, abort_flag) ||
              !mbar_wait(&s_free[b], ((t >> 1) & 1) ^ 1, abort_flag))
            return false;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + kDecOffK + st * kDecTile);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ss(tmem_base + b * 32,
                       sdesc_sw128(k_addr + (kk >> 2) * kDecHalf + (kk & 3) * 32, 0, 1024),
                       sdesc_sw128(q_addr + (kk >> 2) * (kDecQBytes / 2) + (kk & 3) * 32, 0,
                                   1024),
                       idesc_s, kk > 0);
          mma_commit(&s_full[b]);
          mma_commit(&k_empty[st]);
          if (j == n - 1) mma_commit(q_empty);
          return true;
        };
        if (!issue_s(0)) { ok = false; break; }
        for (int j = 0; j < n; ++j) {
          if (j + 1 < n && !issue_s(j + 1)) { ok = false; break; }
          const uint32_t t = kt + j;
          const int st = t % kDecStages, b = t & 1;
          if (!mbar_wait(&v_full[st], (t / kDecStages) & 1, abort_flag) ||
              !mbar_wait(&p_full[b], (t >> 1) & 1, abort_flag) ||
              (j == 0 && !mbar_wait(o_free, (ic & 1) ^ 1, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + kDecOffV + st * kDecTile);
          const uint32_t p_addr = smem_u32(smem + kDecOffP + b * kDecQBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ss(tmem_o, sdesc_sw128(v_addr + kk * 2048, kDecHalf, 1024),
                       sdesc_sw128(p_addr + (kk >> 2) * (kDecQBytes / 2) + (kk & 3) * 32, 0,
                                   1024),
                       idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&v_empty[st]);
          mma_commit(&p_free[b]);
          mma_commit(o_done);
        }
        if (!ok) break;
        mma_commit(o_final);
        kt += n;
        ++ic;
      }
      mma_commit(drain);
      volatile int local_abort = 0;
      mbar_wait(drain, 0, &local_abort);
    }
  } else {
    // ------------------------------------------------ softmax / epilogue
    const int qw = warp & 3;                    // TMEM lane quarter
    const int t = qw * 32 + lane;               // key within the tile; head dim
    const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
    uint8_t* qs = smem + kDecOffQ;
    uint32_t kt = 0, ic = 0, rb = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const DecItem it = dec_item(p, w);
      if (it.t_begin >= it.t_end) {
        // No keys for this item: an empty partial (m = -inf, l = 0).
        if (t < kDecMaxN) {
          p.ws_ml[static_cast<long long>(w) * 64 + t] = -INFINITY;
          p.ws_ml[static_cast<long long>(w) * 64 + 32 + t] = 0.f;
        }
        continue;
      }
      const int ncol = it.nq * p.group;
      // ---- Q^T operand: row n = (query row n / group, head kh*group + n % group)
      {
        const bool freed = mbar_wait(q_empty, (ic & 1) ^ 1, abort_flag);
        if (!__all_sync(0xffffffffu, freed)) { ok = false; break; }
        const int n = t >> 2, quarter = t & 3;
        uint4 v[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                      make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        if (n < ncol) {
          const __nv_bfloat16* src =
              p.q + static_cast<long long>(it.r_begin + n / p.group) * p.ldq +
              static_cast<long long>(it.kh * p.group + n % p.group) * 128 + quarter * 32;
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = reinterpret_cast<const uint4*>(src)[i];
        }
        uint8_t* dst = qs + (quarter >> 1) * (kDecQBytes / 2) + n * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ch = (quarter & 1) * 4 + i;
          *reinterpret_cast<uint4*>(dst + ((ch ^ (n & 7)) << 4)) = v[i];
        }
        fence_async_smem();
        mbar_arrive(q_full);
      }
      const bool done =
          dec_softmax_item<NC>(p, smem, abort_flag, tmem_base, qw, lane, it, w, kt, rb, ic);
      if (!done) { ok = false; break; }
      ++ic;
    }
  }

  __syncthreads();
  if (*abort_flag) {
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 1000000ull) __nanosleep(1000);
    if (threadIdx.x == 0 && p.status) atomicOr(p.status, kDevWaitTimeout);
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 128);
  }
}

// Merge the key chunks of each (sequence, kv head, query group, column):
// M = max m_c, L = sum l_c 2^(m_c - M), out = bf16(sum O_c 2^(m_c - M) / L).
__global__ void __launch_bounds__(128)
    decode_combine_kernel(const DecParams p, __nv_bfloat16* __restrict__ out,
                          long long ldo) {
  const int n = blockIdx.y;           // column: query row n / group, head n % group
  const int base = blockIdx.x;        // (s, kh, qg)
  const int qg = base % p.QG;
  const int kh = (base / p.QG) % p.HKV;
  const int s = base / (p.QG * p.HKV);
  const int q0 = p.q_off[s], q1 = p.q_off[s + 1];
  const int r_begin = q0 + qg * p.nqg;
  const int nq = min(p.nqg, q1 - r_begin);
  if (nq <= 0 || n >= nq * p.group) return;
  const int need = p.q_pos[s] + (r_begin - q0) + nq;
  const int chunks = dec_chunks(need);
  const long long w0 = static_cast<long long>(base) * p.C;
  float M = -INFINITY;
  for (int c = 0; c < chunks; ++c) M = fmaxf(M, p.ws_ml[(w0 + c) * 64 + n]);
  float L = 0.f, acc = 0.f;
  for (int c = 0; c < chunks; ++c) {
    const float m = p.ws_ml[(w0 + c) * 64 + n];
    if (m == -INFINITY) continue;
    const float f = ex2_approx(m - M);
    L += p.ws_ml[(w0 + c) * 64 + 32 + n] * f;
    acc += p.ws_o[((w0 + c) * 32 + n) * 128 + threadIdx.x] * f;
  }
  const int row = r_begin + n / p.group;
  const int h = kh * p.group + n % p.group;
  out[static_cast<long long>(row) * ldo + static_cast<long long>(h) * 128 + threadIdx.x] =
      __float2bfloat16_rn(acc / L);
}

// kvcache.write: one block per new token row; K and V rows of `width`
// elements copied as 16-byte vectors into their page slot.
__global__ void kvcache_write_kernel(__nv_bfloat16* __restrict__ cache,
                                     kvm_kv_layout L, const __nv_bfloat16* __restrict__ k,
                                     long long ldk, const __nv_bfloat16* __restrict__ v,
                                     long long ldv, const int* __restrict__ q_off,
                                     const int* __restrict__ q_pos, const int* __restrict__ bt,
                                     const int* __restrict__ bt_off, int S, int* status) {
  const int r = blockIdx.x;
  int lo = 0, hi = S - 1;  // sequence of row r: largest s with q_off[s] <= r
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q_off[mid] <= r) lo = mid; else hi = mid - 1;
  }
  const int s = lo;
  const int pos = q_pos[s] + (r - q_off[s]);
  const int idx = pos / L.block_size;
  const int page = pos >= 0 && idx < bt_off[s + 1] - bt_off[s] ? bt[bt_off[s] + idx] : -1;
  if (page < 0 || page >= L.num_pages) {
    if (threadIdx.x == 0) atomicOr(status, kDevBadInput);
    return;
  }
  const long long base = page * L.page_stride + L.layer * L.layer_stride +
                         static_cast<long long>(pos % L.block_size) * L.token_stride;
  const int vecs = L.width / 8;
  for (int i = threadIdx.x; i < 2 * vecs; i += blockDim.x) {
    const int kv = i / vecs, c = i % vecs;
    const __nv_bfloat16* src = (kv ? v + r * ldv : k + r * ldk) + c * 8;
    *reinterpret_cast<uint4*>(cache + base + kv * L.kv_stride + c * 8) =
        *reinterpret_cast<const uint4*>(src);
  }
}

// kvcache.read: one block per gathered row (sequence s, key j).
__global__ void kvcache_read_kernel(const __nv_bfloat16* __restrict__ cache,
                                    kvm_kv_layout L, __nv_bfloat16* __restrict__ k,
                                    __nv_bfloat16* __restrict__ v,
                                    const int* __restrict__ kv_off,
                                    const int* __restrict__ bt,
                                    const int* __restrict__ bt_off, int S, int* status) {
  const int r = blockIdx.x;
  int lo = 0, hi = S - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (kv_off[mid] <= r) lo = mid; else hi = mid - 1;
  }
  const int s = lo, j = r - kv_off[s];
  const int idx = j / L.block_size;
  const int page = idx < bt_off[s + 1] - bt_off[s] ? bt[bt_off[s] + idx] : -1;
  if (page < 0 || page >= L.num_pages) {
    if (threadIdx.x == 0) atomicOr(status, kDevBadInput);
    return;
  }
  const long long base = page * L.page_stride + L.layer * L.layer_stride +
                         static_cast<long long>(j % L.block_size) * L.token_stride;
  const int vecs = L.width / 8;
  for (int i = threadIdx.x; i < 2 * vecs; i += blockDim.x) {
    const int kv = i / vecs, c = i % vecs;
    __nv_bfloat16* dst = (kv ? v : k) + static_cast<long long>(r) * L.width + c * 8;
    *reinterpret_cast<uint4*>(dst) =
        *reinterpret_cast<const uint4*>(cache + base + kv * L.kv_stride + c * 8);
  }
}

int check_layout(const kvm_kv_layout* L) {
  if (!L) return fail(KVM_ERR_INVALID_ARG, "kv layout is NULL");
  if (L->block_size < 1 || L->width <= 0 || L->width % 8 || L->num_pages <= 0 ||
      L->layer < 0 || L->token_stride < L->width || L->token_stride % 8 ||
      L->page_stride % 8 || L->layer_stride % 8 || L->kv_stride % 8)
    return fail(KVM_ERR_INVALID_ARG,
                "kv layout: need block_size >= 1, width % 8 == 0, 16-byte aligned "
                "strides and token_stride >= width");
  return KVM_OK;
}

}  // namespace
}  // namespace kvm

using namespace kvm;

extern "C" int kvm_sm100_kvcache_write(void* cache, const kvm_kv_layout* L, const void* k,
                                       int64_t ldk, const void* v, int64_t ldv,
                                       const int32_t* q_offsets, const int32_t* q_positions,
                                       const int32_t* block_table, const int32_t* bt_offsets,
                                       int S, int rows, kvm_stream_t stream) {
  KVM_TRY(check_layout(L));
  if (S <= 0 || rows < 0 || !cache || !k || !v || !q_offsets || !q_positions ||
      !block_table || !bt_offsets || !aligned16(cache) || !aligned16(k) || !aligned16(v) ||
      ldk < L->width || ldv < L->width || ldk % 8 || ldv % 8)
    return fail(KVM_ERR_INVALID_ARG, "kvcache_write: bad argument");
  if (rows == 0) return KVM_OK;
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  kvcache_write_kernel<<<rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(cache), *L, static_cast<const __nv_bfloat16*>(k), ldk,
      static_cast<const __nv_bfloat16*>(v), ldv, q_offsets, q_positions, block_table,
      bt_offsets, S, dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int kvm_sm100_kvcache_read(const void* cache, const kvm_kv_layout* L, void* k,
                                      void* v, const int32_t* kv_offsets,
                                      const int32_t* block_table, const int32_t* bt_offsets,
                                      int S, int rows, kvm_stream_t stream) {
  KVM_TRY(check_layout(L));
  if (S <= 0 || rows < 0 || !cache || !k || !v || !kv_offsets || !block_table ||
      !bt_offsets || !aligned16(cache) || !aligned16(k) || !aligned16(v))
    return fail(KVM_ERR_INVALID_ARG, "kvcache_read: bad argument");
  if (rows == 0) return KVM_OK;
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  kvcache_read_kernel<<<rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(cache), *L, static_cast<__nv_bfloat16*>(k),
      static_cast<__nv_bfloat16*>(v), kv_offsets, block_table, bt_offsets, S, dev->status);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}

extern "C" int64_t kvm_sm100_attention_decode_workspace(int S, int HQ, int HKV,
                                                        int max_q_rows, int max_keys) {
  if (S <= 0 || HQ <= 0 || HKV <= 0 || HQ % HKV || HQ / HKV > kDecMaxN ||
      max_q_rows <= 0 || max_keys <= 0)
    return 0;
  const int nqg = kDecMaxN / (HQ / HKV);
  const long long QG = (max_q_rows + nqg - 1) / nqg;
  const long long C = (max_keys + kDecChunk - 1) / kDecChunk;
  const long long items = static_cast<long long>(S) * HKV * QG * C;
  return items * (32 * 128 + 64) * 4;
}

extern "C" int kvm_sm100_attention_decode_paged(
    const void* q, int64_t ldq, const void* cache, const kvm_kv_layout* L, void* out,
    int64_t ldo, const int32_t* q_offsets, const int32_t* q_positions,
    const int32_t* block_table, const int32_t* bt_offsets, int S, int HQ, int max_q_rows,
    int max_keys, float scale, void* workspace, int64_t workspace_bytes,
    kvm_stream_t stream) {
  KVM_TRY(check_layout(L));
  if (S <= 0 || HQ <= 0 || L->width % 128 || HQ % (L->width / 128))
    return fail(KVM_ERR_INVALID_ARG,
                "attention_decode: head_dim 128, width = HKV*128, HQ % HKV == 0");
  const int HKV = L->width / 128;
  const int group = HQ / HKV;
  if (group > kDecMaxN)
    return fail(KVM_ERR_UNSUPPORTED, "attention_decode: at most 32 query heads per kv head");
  const int bs = L->block_size;
  if (bs < 16 || (bs & (bs - 1)) != 0)
    return fail(KVM_ERR_UNSUPPORTED,
                "attention_decode: block_size must be a power of two >= 16");
  if (L->page_stride % L->token_stride || L->layer_stride % L->token_stride ||
      L->kv_stride % L->token_stride)
    return fail(KVM_ERR_INVALID_ARG,
                "attention_decode: page, layer and kv strides must be whole token slots");
  if (!q || !cache || !out || !q_offsets || !q_positions || !block_table || !bt_offsets ||
      !aligned16(q) || !aligned16(cache) || !aligned16(out) || ldq < int64_t(HQ) * 128 ||
      ldo < int64_t(HQ) * 128 || ldq % 8 || ldo % 8 || max_q_rows <= 0 || max_keys <= 0)
    return fail(KVM_ERR_INVALID_ARG, "attention_decode: bad argument");
  const int64_t need_ws = kvm_sm100_attention_decode_workspace(S, HQ, HKV, max_q_rows, max_keys);
  if (!workspace || workspace_bytes < need_ws || !aligned16(workspace))
    return fail(KVM_ERR_INVALID_ARG, "attention_decode: workspace too small");
  const DeviceInfo* dev = device_info();
  if (!dev) return KVM_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  DecParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.S = S; p.HKV = HKV; p.group = group;
  p.nqg = kDecMaxN / group;
  p.QG = (max_q_rows + p.nqg - 1) / p.nqg;
  p.C = (max_keys + kDecChunk - 1) / kDecChunk;
  p.q_off = q_offsets; p.q_pos = q_positions; p.bt = block_table; p.bt_off = bt_offsets;
  p.block_size = bs;
  p.box_rows = bs < 128 ? bs : 128;
  p.num_pages = L->num_pages;
  p.page_rows = L->page_stride / L->token_stride;
  p.layer_rows = L->layer_stride / L->token_stride;
  p.kv_rows = L->kv_stride / L->token_stride;
  p.layer = L->layer;
  if (scale <= 0.f) scale = 1.0f / sqrtf(128.0f);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ws_o = static_cast<float*>(workspace);
  const long long items = static_cast<long long>(S) * HKV * p.QG * p.C;
  p.ws_ml = p.ws_o + items * 32 * 128;
  p.status = dev->status;
  if (items > (1ll << 30)) return fail(KVM_ERR_INVALID_ARG, "attention_decode: too large");

  // The pool as rows of token slots: [pool_rows, width] with row stride
  // token_stride; page p, layer l, kv x, slot i is row
  // p*page_rows + l*layer_rows + x*kv_rows + i.
  const long long pool_rows = static_cast<long long>(L->num_pages) * p.page_rows +
                              static_cast<long long>(L->layer + 1) * p.layer_rows +
                              2 * p.kv_rows + bs;
  if (pool_rows >= (1ll << 31))
    return fail(KVM_ERR_UNSUPPORTED, "attention_decode: pool too large for 32-bit rows");
  CUtensorMap tkv;
  KVM_TRY(encode_tmap_2d(&tkv, cache, L->width, pool_rows, L->token_stride * 2, 64,
                         p.box_rows, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         CU_TENSOR_MAP_SWIZZLE_128B));
  const int grid = items < dev->sm_count ? int(items) : dev->sm_count;
  constexpr size_t smem = dec_smem_bytes();
  auto kern = min(max_q_rows, p.nqg) * group <= 16 ? decode_attn_kernel<16>
                                                   : decode_attn_kernel<32>;
  KVM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  kern<<<grid, kDecThreads, smem, st>>>(tkv, p, int(items));
  KVM_CUDA_TRY(cudaGetLastError());
  dim3 cgrid(static_cast<unsigned>(S * HKV * p.QG), kDecMaxN);
  decode_combine_kernel<<<cgrid, 128, 0, st>>>(p, static_cast<__nv_bfloat16*>(out), ldo);
  KVM_CUDA_TRY(cudaGetLastError());
  return KVM_OK;
}
