/*
 * kvm_sm100.h -- C ABI of the B200 (sm_100a) execution backend for KVM
 * kernel/task-dialect graphs.
 *
 * The reference toolkit (feifei-111/KVM) lowers kernel ops to task ops in
 * src/device/device.cpp but has no way to execute them. Each entry point here
 * executes one task subgraph on the GPU; the comment on each names the kernel
 * op (src/ir/dialect/kernel/dialect.cpp) and the task ops it produces
 * (src/ir/dialect/task/dialect.cpp) that the call stands in for.
 *
 * Conventions
 *  - All tensor pointers are device pointers owned by the caller; sizes are
 *    element counts; matrices are row-major with the stated row stride.
 *  - bf16 is passed as 16-bit storage (uint16_t / __nv_bfloat16).
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream).
 *  - Every call returns a kvm_status. On failure kvm_sm100_last_error() gives
 *    a message for the calling thread. Kernels never hang: device-side waits
 *    are bounded and report KVM_ERR_TIMEOUT through kvm_sm100_device_status().
 *  - Calls are asynchronous with respect to the host, like a CUDA launch.
 */
#ifndef KVM_SM100_H_
#define KVM_SM100_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVM_SM100_ABI_VERSION 1

typedef void* kvm_stream_t; /* cudaStream_t */

enum kvm_status {
  KVM_OK = 0,
  KVM_ERR_INVALID_ARG = 1, /* shape, alignment or pointer rejected */
  KVM_ERR_UNSUPPORTED = 2, /* valid request this build cannot run */
  KVM_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  KVM_ERR_TIMEOUT = 4,     /* a bounded device-side wait expired */
  KVM_ERR_NCCL = 5         /* a collective failed or timed out */
};

/* Layout of the B operand of a GEMM. */
enum kvm_b_layout {
  KVM_B_NK = 0, /* B stored [N, K] (K contiguous): the "weights" layout */
  KVM_B_KN = 1  /* B stored [K, N] (N contiguous): kernel.matmul's layout */
};

enum kvm_dtype { KVM_BF16 = 0, KVM_F32 = 1 };

/* ------------------------------------------------------------ runtime --- */

int kvm_sm100_version(void);
const char* kvm_sm100_last_error(void);

/* Synchronise the current device and read its device-side status word
 * (bit 0: a bounded wait expired; bit 1: a kernel rejected an index).
 * Returns KVM_ERR_TIMEOUT / KVM_ERR_INVALID_ARG when a bit is set. */
int kvm_sm100_device_status(int* status_out, int clear);

/* The binary architecture the current device runs this library's kernels
 * from, as cudaFuncAttributes::binaryVersion (major * 10 + minor: 100 for the
 * sm_100a cubins this library ships). Needs a device. A diagnostic with no
 * counterpart in the reference. */
int kvm_sm100_kernel_binary_version(int* version);

/* --------------------------------------------------------------- GEMM --- */

/* D[M,N] = A[M,K] . B  (+ C[M,N] when C != NULL), fp32 accumulation in TMEM.
 * A: bf16 [M, K], row stride lda; B: bf16 per b_layout with row stride ldb;
 * C (optional) and D: out_dtype, row stride ldd.
 * Replaces: kernel.matmul (src/ir/dialect/kernel/dialect.cpp:34) and
 * kernel.gemm (dialect.cpp:35), whose lowering in src/device/device.cpp:85-106
 * emits task.tma.gmem_to_smem x2, task.lsu.gmem_to_reg, task.tc.mma_acc and
 * task.lsu.reg_to_gmem (src/ir/dialect/task/dialect.cpp:33-34,56-61). */
int kvm_sm100_gemm_bf16(const void* A, int64_t lda, const void* B,
                        int64_t ldb, int b_layout, const void* C, void* D,
                        int64_t ldd, int out_dtype, int M, int N, int K,
                        kvm_stream_t stream);

/* H[M, F] = bf16( SiLU(A.Wg^T) * (A.Wu^T) ), the gated-FFN front half with
 * the activation fused into the GEMM epilogue. W13 is the packed weight from
 * kvm_sm100_pack_gate_up ([2F, K], gate/up interleaved in 64-row blocks).
 * Replaces the composite kernel.matmul x2 -> neg/exp/add/div/mul chain. */
int kvm_sm100_gemm_bf16_silu_gate(const void* A, int64_t lda, const void* W13,
                                  void* H, int64_t ldh, int M, int F, int K,
                                  kvm_stream_t stream);

/* Pack G groups of gate/up weights into the interleaved layout consumed by
 * the *_silu_gate GEMMs: out[g] = [Wg[g][0:64]; Wu[g][0:64]; Wg[g][64:128];
 * ...], each block 64 rows of K (one SM of a GEMM SM pair holds the gate and
 * the up rows of the same 64 f). w_layout says how Wg/Wu are stored:
 * KVM_B_NK = [G, F, K], KVM_B_KN = [G, K, F] (transposed while packing).
 * F must be a multiple of 128. */
int kvm_sm100_pack_gate_up(const void* Wg, const void* Wu, void* out, int G,
                           int F, int K, int w_layout, kvm_stream_t stream);

/* Transpose G row-major [R, C] bf16 matrices into [C, R] (weights given in
 * kernel.matmul's [K, N] layout are converted once to [N, K]). */
int kvm_sm100_transpose_bf16(const void* in, void* out, int G, int R, int C,
                             kvm_stream_t stream);

/* ---------------------------------------------------------------- MoE --- */

/* The router, permute (workspace form), scatter, grouped GEMMs and combine
 * below launch with programmatic dependent launch: a launch may start its
 * prologue while the previous kernel on the stream finishes, and touches
 * global memory only after that kernel has completed. Stream order is kept
 * as for any launch. */

/* Router GEMM fused with softmax and top-k. logits[T,E] = x[T,H] . Wr^T
 * (Wr stored [E, H]); probabilities p = softmax(logits) in fp32; topk_idx
 * [T,k] are the k largest logits per token (ties: lower expert index first,
 * descending order), topk_w [T,k] their probabilities (no renormalisation).
 * 1 <= E <= 256 in this build (E > 256: KVM_ERR_UNSUPPORTED); 1 <= k <= min(8, E).
 * A token's logits are the same bits in any batch: for E <= 64 the two halves
 * of K are accumulated separately (the split depends only on H) and added in
 * a fixed order; for E > 64 one accumulator walks K in order. A NaN logit
 * ranks below every number in the top-k (E <= 64).
 * The launch may overlap the tail of the previous kernel on the stream
 * (programmatic dependent launch); it reads x and writes its outputs only
 * after that kernel has completed.
 * Replaces the routing half of kernel.comm.moe_dispatch
 * (src/ir/dialect/kernel/dialect.cpp:65, passed through to
 * task.comm.moe_dispatch by src/device/device.cpp:143-147). */
int kvm_sm100_moe_router_topk(const void* x, const void* Wr, float* logits,
                              int32_t* topk_idx, float* topk_w, int T, int H,
                              int E, int k, kvm_stream_t stream);

/* Deterministic expert-major permutation of the T*k (token, slot) pairs:
 * entries are ordered by (expert, token, slot). Writes expert_offsets [E+1]
 * (exclusive prefix of per-expert counts), pos [T*k] (row of pair (t,j) in the
 * permuted order) and src_token [T*k] (token of each permuted row).
 * workspace: kvm_sm100_moe_permute_workspace(T, k, E) bytes of device memory.
 * Bit-exact: no atomics decide any position. A pair whose expert index lies
 * outside [0, E) gets pos = -1 and joins no group, so expert_offsets[E] is
 * then below T*k and src_token[expert_offsets[E]..T*k) is not written; the
 * kernel records it in the device status word (kvm_sm100_device_status). */
int64_t kvm_sm100_moe_permute_workspace(int T, int k, int E);
int kvm_sm100_moe_permute(const int32_t* topk_idx, int T, int k, int E,
                          int32_t* expert_offsets, int32_t* pos,
                          int32_t* src_token, void* workspace,
                          kvm_stream_t stream);

/* Allocation-free variant of kvm_sm100_moe_permute, with the same inputs and
 * outputs and no workspace argument. No counterpart in the reference: it exists for callers
 * that cannot allocate GPU memory while they route tokens -- a host program
 * that owns every device buffer through its own pool (an FFI host), or a
 * serving loop that must not call cudaMalloc/cudaFree because they
 * synchronise the device. The scratch lives in a static device array of
 * 2 * KVM_SM100_NOALLOC_PERMUTE_MAX_CELLS ints (512 KiB) that every GPU loading
 * the library holds until exit; sizes with ceil(T*k/256) * E above
 * KVM_SM100_NOALLOC_PERMUTE_MAX_CELLS are rejected with KVM_ERR_INVALID_ARG.
 * The first call on a device looks up that array's device address (set-up
 * done once per device, with that device current); make that first call
 * before any stream capture. All calls on a device share the array, so calls
 * whose kernels overlap on the GPU race and must not be issued. Calls no
 * cudaMalloc, cudaFree or allocating routine. Valid indices give outputs
 * bit-identical to kvm_sm100_moe_permute's. An out-of-range expert index is
 * handled as there (pos = -1, the pair joins no group), but it is recorded in
 * a status word of this entry point's own, inside the static array, not in
 * the device status word: read it with kvm_sm100_moe_permute_noalloc_status. */
#define KVM_SM100_NOALLOC_PERMUTE_MAX_CELLS 65536
int kvm_sm100_moe_permute_noalloc(const int32_t* topk_idx, int T, int k, int E,
                                  int32_t* expert_offsets, int32_t* pos,
                                  int32_t* src_token, kvm_stream_t stream);
/* Synchronise the current device and read (clear != 0: then zero) the status
 * word of kvm_sm100_moe_permute_noalloc on it; the word is sticky across calls
 * until cleared. Returns KVM_ERR_INVALID_ARG when a call saw an expert index
 * outside [0, E). Allocates nothing (two small copies to and from the static
 * array). No counterpart in the reference: it is the status half of the
 * allocation-free permute above. */
int kvm_sm100_moe_permute_noalloc_status(int* status_out, int clear);

/* xp[pos[t*k+j], :] = x[t, :] for every pair: the token scatter of
 * moe_dispatch. x: bf16 [T, H]; xp: bf16 [T*k, H]. */
int kvm_sm100_moe_scatter_rows(const void* x, const int32_t* pos, void* xp,
                               int T, int k, int H, kvm_stream_t stream);

/* Grouped expert GEMM over the permuted rows. Group g owns rows
 * [offsets[g], offsets[g+1]) of A and D (offsets live in device memory, as
 * written by kvm_sm100_moe_permute). B holds G weight matrices [N, K]
 * (K contiguous), one per group.
 *   epilogue 0: D[r, 0:N] = bf16(A[r] . B[g]^T)
 *   epilogue 2: B = packed gate/up ([G, 2F, K]); D[r, 0:F] =
 *               bf16(SiLU(gate) * up), N passed as 2F.
 * Replaces kernel.gemm on 3-D expert weights (kernel/dialect.cpp:35). */
int kvm_sm100_grouped_gemm_bf16(const void* A, const void* B, void* D,
                                const int32_t* offsets, int G, int rows,
                                int N, int K, int epilogue,
                                kvm_stream_t stream);

/* out[t, :] = bf16( sum_{j<k} w[t,j] * Y[pos[t*k+j], :] ), j in order, fp32.
 * Replaces kernel.comm.moe_combine (src/ir/dialect/kernel/dialect.cpp:66). */
int kvm_sm100_moe_combine(const void* Y, const int32_t* pos, const float* w,
                          void* out, int T, int k, int H,
                          kvm_stream_t stream);

/* -------------------------------------------- expert parallel (NVLink) --- */

/* Peer memory for the expert-parallel exchange among the `world` ranks of one
 * node (one process per GPU). Every rank allocates its own buffers with
 * kvm_sm100_ipc_alloc and exchanges their IPC handles (64 bytes each, from
 * kvm_sm100_ipc_get_handle) out of band; each rank then fills its table with
 * its own pointers at [rank] and opened peer pointers elsewhere.
 *   recv[r]  bf16 [cap_rows, H]  rows routed to rank r's experts
 *   y[r]     bf16 [cap_rows, H]  rank r's expert outputs (same rows)
 *   cnt[r]   int32 [world, E]    per-source, per-expert pair counts
 *   flags[r] uint32 [3, world]   count / data / outputs-ready epochs
 * Executes kernel.comm.moe_dispatch / moe_combine across the op's `ranks`
 * (src/ir/dialect/kernel/ops.h:87-88; the rank list survives lowering,
 * src/device/device.cpp:108-121) as peer stores and loads over NVLink. */
#define KVM_EP_MAX_RANKS 8
typedef struct kvm_ep_peers {
  int32_t rank, world, E, H, k, pad_;
  void* recv[KVM_EP_MAX_RANKS];
  void* y[KVM_EP_MAX_RANKS];
  void* cnt[KVM_EP_MAX_RANKS];
  void* flags[KVM_EP_MAX_RANKS];
} kvm_ep_peers;

int kvm_sm100_ipc_alloc(int64_t bytes, void** ptr); /* cudaMalloc + zero */
int kvm_sm100_ipc_free(void* ptr);
int kvm_sm100_ipc_get_handle(const void* ptr, void* handle64);
int kvm_sm100_ipc_open_handle(const void* handle64, void** peer_ptr);
int kvm_sm100_ipc_close(void* peer_ptr);

/* Count exchange of one call (epoch = 1, 2, ... per call, same on all ranks):
 * publishes this rank's per-expert counts (offsets [E+1] from
 * kvm_sm100_moe_permute), waits (bounded) for every rank's, and writes
 * local_offsets [E/world + 1] (group offsets of this rank's experts in its
 * receive buffer: expert-major, then source-rank-major) and send_base [E]
 * (first row of this rank's pairs of expert e in the owner's buffer). */
int kvm_sm100_ep_counts(const kvm_ep_peers* peers, const int32_t* offsets,
                        int32_t* send_base, int32_t* local_offsets,
                        uint32_t epoch, kvm_stream_t stream);

/* The dispatch all-to-all fused with the token scatter: row x[t] goes to
 * recv[owner(e)][send_base[e] + pos[t*k+j] - offsets[e]] for each pair, by
 * peer stores; then raises the data-ready flags. `done` is a zeroed uint32 in
 * this rank's device memory. */
int kvm_sm100_ep_dispatch(const kvm_ep_peers* peers, const void* x,
                          const int32_t* topk_idx, const int32_t* pos,
                          const int32_t* offsets, const int32_t* send_base, int T,
                          int64_t cap_rows, uint32_t* done, uint32_t epoch,
                          kvm_stream_t stream);

/* Bounded wait for every rank's flag `slot` (1 data, 2 outputs) to reach
 * epoch; raise this rank's flag `slot` on every rank. */
int kvm_sm100_ep_wait(const kvm_ep_peers* peers, int slot, uint32_t epoch,
                      kvm_stream_t stream);
int kvm_sm100_ep_signal(const kvm_ep_peers* peers, int slot, uint32_t epoch,
                        kvm_stream_t stream);

/* The combine all-to-all fused with the weighted combine: out[t] =
 * bf16(sum_j w[t,j] * y[owner][row of pair (t,j)]) by peer loads, fp32 with one
 * fused multiply-add per slot in slot order (bit-identical to
 * kvm_sm100_moe_combine on the same expert outputs). */
int kvm_sm100_ep_combine(const kvm_ep_peers* peers, const int32_t* topk_idx,
                         const int32_t* pos, const int32_t* offsets,
                         const int32_t* send_base, const float* topk_w, void* out,
                         int T, int64_t cap_rows, kvm_stream_t stream);

/* Overlapped form of the same exchange: the all-to-all rides inside the
 * grouped GEMMs, so NVLink transfers overlap the tensor-core work tile by
 * tile. One call of the layer on each rank (same epoch on all ranks):
 *   kvm_sm100_ep_prepare          count exchange (as kvm_sm100_ep_counts) and
 *                                 the call's segment table and return map;
 *   kvm_sm100_ep_scatter_local    rows routed to this rank's own experts;
 *   kvm_sm100_ep_dispatch_gate_up the dispatch of the other rows (peer stores
 *                                 by extra warps of the GEMM) fused with the
 *                                 grouped SiLU-gate GEMM, which starts a
 *                                 local expert's tiles as soon as every rank's
 *                                 rows for it have arrived;
 *   kvm_sm100_ep_down_push        the grouped down GEMM whose epilogue stores
 *                                 each output row straight into the result rows
 *                                 of the rank that routed the token (peer
 *                                 stores), then raises every rank's outputs flag;
 *   kvm_sm100_ep_wait(slot 2)     outputs of every rank's experts have arrived;
 *   kvm_sm100_moe_combine         on this rank's own y buffer, locally.
 * In this form y[r] holds rank r's result rows [T*k, H] in rank r's permuted
 * order (cap_rows rows suffice), and flags[r] needs 3*world + E words (one
 * per local expert and source rank after the three slots). Bit-identical to
 * kvm_sm100_moe_* on one GPU. workspace: kvm_sm100_ep_overlap_workspace(E,
 * cap_rows) bytes of this rank's device memory. Executes the same kernel ops
 * (src/ir/dialect/kernel/ops.h:87-88) as the serial exchange above. */
int64_t kvm_sm100_ep_overlap_workspace(int E, int64_t cap_rows);
int kvm_sm100_ep_prepare(const kvm_ep_peers* peers, const int32_t* offsets,
                         int32_t* send_base, int32_t* local_offsets, void* workspace,
                         int64_t cap_rows, uint32_t epoch, kvm_stream_t stream);
int kvm_sm100_ep_scatter_local(const kvm_ep_peers* peers, const void* x,
                               const int32_t* src_token, const int32_t* offsets,
                               const int32_t* send_base, int T, int64_t cap_rows,
                               kvm_stream_t stream);
int kvm_sm100_ep_dispatch_gate_up(const kvm_ep_peers* peers, const void* x,
                                  const int32_t* src_token, const int32_t* offsets,
                                  const int32_t* send_base, const int32_t* local_offsets,
                                  const void* W13, void* h, int F, int64_t cap_rows,
                                  void* workspace, uint32_t epoch, kvm_stream_t stream);
int kvm_sm100_ep_down_push(const kvm_ep_peers* peers, const void* h, const void* W2,
                           const int32_t* local_offsets, int F, int64_t cap_rows,
                           void* workspace, uint32_t epoch, kvm_stream_t stream);

/* ---------------------------------------------------------------- FP8 --- */

/* FP8 e4m3 W8A8 GEMM with 128x128 fp32 block scales, bf16 output:
 *   D[m,n] = bf16( sum_kb s * P_kb[m,n] ),  s = sA[m/128][kb] * sW[n/128][kb],
 *   P_kb = sum over the 128-deep K block kb of Aq[m,k] * Wq[n,k] (fp32),
 *   accumulated acc = fma(P_kb, s, acc) in ascending kb.
 * Aq: e4m3 [M, K] (K contiguous); sA: fp32 [ceil(M/128), K/128].
 * Wq: e4m3 [N, K] (K contiguous; weights in kernel.matmul's [K, N] layout are
 * converted once with kvm_sm100_transpose_u8 / kvm_sm100_transpose_f32);
 * sW: fp32 [N/128, K/128]. K % 128 == 0, N % 128 == 0.
 * When M is small (one or two 128-row tiles) the K blocks of each tile are
 * split over several work units so that every SM streams weights; each unit
 * then accumulates its own blocks and the units' fp32 partials are summed in
 * unit order. That needs kvm_sm100_gemm_fp8_workspace(M, N, K) bytes of
 * workspace (0 = no split; with a NULL or smaller workspace the GEMM runs
 * unsplit).
 * The reference cannot express this op (src/ir/dialect/dtype.h:13-20 has no
 * fp8); it is the sm_100a form of task.tc.mma_acc (task/dialect.cpp:34) on
 * e4m3 operands. */
int64_t kvm_sm100_gemm_fp8_workspace(int M, int N, int K);
int kvm_sm100_gemm_fp8_blockscaled(const void* Aq, const float* sA,
                                   const void* Wq, const float* sW, void* D,
                                   int64_t ldd, int M, int N, int K,
                                   void* workspace, int64_t workspace_bytes,
                                   kvm_stream_t stream);

/* Quantise x [R, C] (x_dtype KVM_BF16 or KVM_F32) to e4m3 per 128x128 block:
 * scale s = amax(|x| over the block) / 448 (1 for an all-zero block),
 * q = e4m3(x / s) with IEEE division, round-to-nearest-even, saturating to
 * +-448. scales: fp32 [ceil(R/128), ceil(C/128)]. */
int kvm_sm100_quantize_e4m3_block128(const void* x, int x_dtype, void* q,
                                     float* scales, int R, int C,
                                     kvm_stream_t stream);

/* Byte / fp32 matrix transposes [R, C] -> [C, R] (one-time weight re-layout). */
int kvm_sm100_transpose_u8(const void* in, void* out, int R, int C,
                           kvm_stream_t stream);
int kvm_sm100_transpose_f32(const float* in, float* out, int R, int C,
                            kvm_stream_t stream);

/* ------------------------------------------------------- elementwise --- */

/* y[r, :] = bf16( x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * gamma ), fp32
 * internally. gamma may be NULL (= 1). Replaces the composite
 * mul -> matmul(ones/H) -> add(eps) -> rsqrt -> mul (kernel/dialect.cpp:43-46). */
int kvm_sm100_rmsnorm_bf16(const void* x, const void* gamma, void* y,
                           int rows, int H, float eps, kvm_stream_t stream);

/* h = bf16( g * sigmoid(g) * u ) elementwise over n bf16 values. Replaces the
 * composite neg/exp/add/div/mul SiLU-gate chain (kernel/dialect.cpp:43-46). */
int kvm_sm100_silu_mul_bf16(const void* g, const void* u, void* h, int64_t n,
                            kvm_stream_t stream);

/* ---------------------------------------------------------- attention --- */

/* Causal grouped-query attention over a batch of sequences (prefill):
 * kernel.attn.prefill (src/ir/dialect/kernel/dialect.cpp:38) for equal-length
 * sequences. Tokens are rows b*L + pos; q/out hold HQ heads of 128 columns
 * each, k/v hold HKV heads (q head h reads kv head h / (HQ/HKV)); row strides
 * ldq, ldk, ldv, ldo in elements (bf16). Per head:
 *   S = scale * Q K^T (fp32), P = softmax over keys <= pos, O = P V
 *   (fp32 accumulate, bf16 out), computed in one fused pass per 128-query
 *   tile: running max and sum in fp32, unnormalised P rounded to bf16 for
 *   the P.V product, O divided by the sum at the end.
 * scale <= 0 selects 1/sqrt(head_dim). head_dim must be 128, L % 8 == 0.
 * workspace: kvm_sm100_attention_workspace(B, L, HQ, HKV) bytes (0 in this
 * build: the scores never leave the SM; workspace may then be NULL). */
int64_t kvm_sm100_attention_workspace(int B, int L, int HQ, int HKV);
int kvm_sm100_attention_prefill_bf16(const void* q, int64_t ldq, const void* k,
                                     int64_t ldk, const void* v, int64_t ldv,
                                     void* out, int64_t ldo, int B, int L, int HQ,
                                     int HKV, int head_dim, float scale,
                                     void* workspace, int64_t workspace_bytes,
                                     kvm_stream_t stream);

/* ------------------------------------------------------- collectives --- */

/* The kernel dialect's collectives (src/ir/dialect/kernel/dialect.cpp:58-64,
 * rank sets on kernel/ops.h:39-88) over NCCL on NVLink/NVSwitch, one process
 * per GPU. A communicator covers `nranks` processes; kvm_sm100_comm_split
 * derives one for a rank set (a kernel op's `ranks`). Buffers are device
 * memory of dtype KVM_EW_BF16 / F16 / F32 / I32; `count` is in elements.
 * Setup is bounded: a rank that does not join within 60 s makes init return
 * KVM_ERR_TIMEOUT. The reference has no runtime for these ops (they lower to
 * task.comm.* and stop there, src/device/device.cpp:111-121). */
typedef struct kvm_comm kvm_comm;
#define KVM_COMM_ID_BYTES 128
enum kvm_red_op { KVM_RED_SUM = 0, KVM_RED_MAX = 1 };

int kvm_sm100_comm_unique_id(void* id); /* KVM_COMM_ID_BYTES, made by one rank */
int kvm_sm100_comm_init(int nranks, int rank, const void* id, kvm_comm** comm);
/* Every rank of `parent` calls it; members of ranks[0..n) get a
 * communicator numbered by their position in `ranks`, others get NULL. */
int kvm_sm100_comm_split(kvm_comm* parent, const int32_t* ranks, int n, kvm_comm** comm);
int kvm_sm100_comm_rank(const kvm_comm* comm, int* rank, int* nranks);
int kvm_sm100_comm_destroy(kvm_comm* comm);
/* comm.all_reduce.sum / .max: recv = op over ranks of send ([count]). */
int kvm_sm100_all_reduce(kvm_comm* comm, const void* send, void* recv, int64_t count,
                         int dtype, int op, kvm_stream_t stream);
/* comm.all_gather: recv [nranks * count] = the ranks' send [count], in rank order. */
int kvm_sm100_all_gather(kvm_comm* comm, const void* send, void* recv, int64_t count,
                         int dtype, kvm_stream_t stream);
/* comm.broadcast: recv = root's send on every rank (send ignored off the root). */
int kvm_sm100_broadcast(kvm_comm* comm, const void* send, void* recv, int64_t count,
                        int dtype, int root, kvm_stream_t stream);
/* comm.send / comm.recv: point to point, matched by peer and order. */
int kvm_sm100_send(kvm_comm* comm, const void* buf, int64_t count, int dtype, int peer,
                   kvm_stream_t stream);
int kvm_sm100_recv(kvm_comm* comm, void* buf, int64_t count, int dtype, int peer,
                   kvm_stream_t stream);
/* comm.all_to_all: send [nranks * count] split in rank order; recv [nranks *
 * count] holds, at chunk p, what rank p sent to this rank. */
int kvm_sm100_all_to_all(kvm_comm* comm, const void* send, void* recv, int64_t count,
                         int dtype, kvm_stream_t stream);

/* ------------------------------------------------- paged KV cache --- */

/* A paged K/V pool as KVMeta describes it (src/ir/graph_config.h:20-39):
 * pages of block_size token slots; a slot holds `width` = layer_size
 * elements (HKV heads x head_dim, bf16) of K or of V for one layer. Element
 * (page, layer, kv, slot, e) lives at
 *   page*page_stride + layer*layer_stride + kv*kv_stride + slot*token_stride + e
 * (kv 0 = K, 1 = V), which covers layout=page_first
 * ([page][layer][kv][slot][width]) and layer_first ([layer][page][kv]...).
 * No counterpart struct in the reference: it carries KVMeta's fields plus
 * the strides they imply. */
typedef struct kvm_kv_layout {
  int64_t page_stride;
  int64_t layer_stride;
  int64_t kv_stride;
  int64_t token_stride;
  int32_t block_size;
  int32_t layer;      /* the layer this call reads or writes */
  int32_t width;      /* elements per slot: HKV * head_dim */
  int32_t num_pages;  /* pages in the pool (page ids are checked) */
} kvm_kv_layout;

/* kernel.kvcache.write (src/ir/dialect/kernel/dialect.cpp:70): S sequences;
 * the new rows q_offsets[s]..q_offsets[s+1] of k and v ([rows, width], row
 * strides ldk/ldv) sit at positions q_positions[s] + i and go to slot
 * pos % block_size of page block_table[bt_offsets[s] + pos / block_size].
 * Page ids outside [0, num_pages) are reported through the device status
 * and not written. */
int kvm_sm100_kvcache_write(void* cache, const kvm_kv_layout* layout, const void* k,
                            int64_t ldk, const void* v, int64_t ldv,
                            const int32_t* q_offsets, const int32_t* q_positions,
                            const int32_t* block_table, const int32_t* bt_offsets, int S,
                            int rows, kvm_stream_t stream);

/* kernel.kvcache.read (dialect.cpp:69): the first kv_offsets[s+1] -
 * kv_offsets[s] cached tokens of each sequence gathered in order into rows
 * kv_offsets[s].. of k and v ([rows, width], contiguous). */
int kvm_sm100_kvcache_read(const void* cache, const kvm_kv_layout* layout, void* k,
                           void* v, const int32_t* kv_offsets, const int32_t* block_table,
                           const int32_t* bt_offsets, int S, int rows, kvm_stream_t stream);

/* kernel.attn.decode (dialect.cpp:39) over the paged cache, causal: query
 * row r of sequence s (rows q_offsets[s]..) at position p = q_positions[s]
 * + (r - q_offsets[s]) attends to cached positions 0..p of s (written
 * before the call); q and out are [rows, HQ*128] (row strides ldq, ldo), q
 * head h reads kv head h / (HQ/HKV), HKV = width / 128, at most 32 query
 * heads per kv head, block_size a power of two >= 16. The keys are split in
 * chunks of 1024 over the SMs and merged; max_q_rows bounds the new rows of
 * any sequence and max_keys the keys any row attends to (both size the
 * workspace: kvm_sm100_attention_decode_workspace bytes). scale <= 0 selects
 * 1/sqrt(128). */
int64_t kvm_sm100_attention_decode_workspace(int S, int HQ, int HKV, int max_q_rows,
                                             int max_keys);
int kvm_sm100_attention_decode_paged(const void* q, int64_t ldq, const void* cache,
                                     const kvm_kv_layout* layout, void* out, int64_t ldo,
                                     const int32_t* q_offsets, const int32_t* q_positions,
                                     const int32_t* block_table, const int32_t* bt_offsets,
                                     int S, int HQ, int max_q_rows, int max_keys,
                                     float scale, void* workspace, int64_t workspace_bytes,
                                     kvm_stream_t stream);

/* Rotary position embedding in place, rotate-half form: kernel.attn.rope
 * (dialect.cpp:40). Rows are tokens b*L + pos (row stride ld elements); heads
 * are consecutive head_dim-wide column blocks; for i < head_dim/2,
 * theta = pos * base^(-2i/head_dim), (x[i], x[i+hd/2]) rotated by theta.
 * base <= 0 selects 10000. */
int kvm_sm100_rope_bf16(void* x, int64_t ld, int rows, int L, int heads,
                        int head_dim, float base, kvm_stream_t stream);

/* ------------------------------------------------ graph execution helpers --- */

/* Element types of the elementwise interpreter and kvm_sm100_moe_topk. */
enum kvm_ew_dtype { KVM_EW_BF16 = 0, KVM_EW_F32 = 1, KVM_EW_F16 = 2, KVM_EW_I32 = 3 };

/* Instructions of the elementwise interpreter (one fp32 register file per
 * element). LOAD reads input `a` at ((i / in_div[a]) mod in_size[a]) for output
 * element i, which broadcasts an input over leading dimensions (in_div 1) and
 * over trailing dimensions (in_div = their product); binary ops read
 * registers a, b. */
enum kvm_ew_op {
  KVM_EW_LOAD = 0, KVM_EW_ADD, KVM_EW_SUB, KVM_EW_MUL, KVM_EW_DIV, KVM_EW_MAX,
  KVM_EW_MIN, KVM_EW_NEG, KVM_EW_EXP, KVM_EW_LOG, KVM_EW_SQRT, KVM_EW_RSQRT,
  KVM_EW_ABS, KVM_EW_RCP, KVM_EW_CMP_EQ, KVM_EW_CMP_NE, KVM_EW_CMP_LT,
  KVM_EW_CMP_LE, KVM_EW_CMP_GT, KVM_EW_CMP_GE, KVM_EW_ROUND_BF16,
  KVM_EW_ROUND_F16, KVM_EW_TRUNC_I32
};

#define KVM_EW_MAX_INPUTS 8
#define KVM_EW_MAX_INSTR 32
#define KVM_EW_MAX_REGS 16
typedef struct kvm_ew_program {
  int32_t n_inputs, n_instr, out_reg, out_dtype;
  int32_t in_dtype[KVM_EW_MAX_INPUTS];
  int64_t in_size[KVM_EW_MAX_INPUTS]; /* element i reads (i / in_div) % in_size */
  int64_t in_div[KVM_EW_MAX_INPUTS];  /* 1 = broadcast over leading dims only */
  uint8_t op[KVM_EW_MAX_INSTR], a[KVM_EW_MAX_INSTR], b[KVM_EW_MAX_INSTR],
      dst[KVM_EW_MAX_INSTR];
} kvm_ew_program;
typedef struct kvm_ew_inputs {
  const void* ptr[KVM_EW_MAX_INPUTS];
} kvm_ew_inputs;

/* out[i] = program(inputs) for i < n, converted to out_dtype (bf16/f16 RNE).
 * Executes the kernel dialect's elementwise ops (add sub mul div max min neg
 * exp log sqrt rsqrt abs, cmp.*, cast.*: src/ir/dialect/kernel/dialect.cpp:43-55)
 * as lowered to task.alu.* / task.sfu.* (task/dialect.cpp:36-51). */
int kvm_sm100_elementwise(const kvm_ew_program* program,
                          const kvm_ew_inputs* inputs, void* out, int64_t n,
                          kvm_stream_t stream);
/* The program runs as a kernel generated for it (straight-line code, 8
 * outputs per thread with 16-byte accesses when n % 8 == 0, pointers are
 * 16-byte aligned and contiguous inputs have in_size % 8 == 0), compiled by
 * NVRTC for sm_100a on the first call with that program and those sizes and
 * cached for the process. kvm_sm100_elementwise_prepare does that compile
 * ahead (no GPU needed; call it before capturing a stream that launches the
 * program). Without libnvrtc.so.12 both return KVM_ERR_UNSUPPORTED. */
int kvm_sm100_elementwise_prepare(const kvm_ew_program* program,
                                  const kvm_ew_inputs* inputs, const void* out, int64_t n);

/* y[m] = sum_k A[m, k] * x[k] (fp32 accumulation), y of out_dtype (KVM_BF16 /
 * KVM_F32): kernel.matmul with a [K, 1] right operand (e.g. the row means of
 * the RMSNorm composite), whose [M, 1] result rows are too narrow for the
 * tensor-core GEMM's 16-byte row stores. A, x bf16. */
int kvm_sm100_gemv_bf16(const void* A, int64_t lda, const void* x, void* y,
                        int out_dtype, int M, int K, kvm_stream_t stream);

/* Softmax + top-k over router logits [T, E] of type logits_dtype
 * (KVM_EW_F32 / KVM_EW_BF16) that a graph computed itself: the routing step of
 * kernel.comm.moe_dispatch(x, g) (kernel/dialect.cpp:65). Same selection and
 * weights as kvm_sm100_moe_router_topk. */
int kvm_sm100_moe_topk(const void* logits, int logits_dtype, int T, int E, int k,
                       int32_t* topk_idx, float* topk_w, kvm_stream_t stream);

/* Seeded N(mean, std^2) fill of n elements of `dtype` (kvm_ew_dtype), from a
 * counter-based hash of (seed, index), for synthetic graph inputs. */
int kvm_sm100_fill_normal(void* out, int dtype, int64_t n, uint64_t seed,
                          float mean, float std, kvm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KVM_SM100_H_ */
