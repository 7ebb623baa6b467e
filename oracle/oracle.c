/*
 * CPU oracle for the KVM execution backend -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, as the checker; no product code path calls it.
 *
 * PARITY UNPINNED. The reference (feifei-111/KVM) has no execution path: it
 * parses .kvm graphs and lowers kernel ops to task ops
 * (src/device/device.cpp:129-151) but never computes a value, and ships no
 * golden vectors or numeric fixtures. This file restates the semantics of the
 * ops as the reference declares them:
 *   kernel.matmul  D = A.B            (src/ir/dialect/kernel/dialect.cpp:34)
 *   kernel.gemm    D = A.B + C        (dialect.cpp:35; task.tc.mma_acc
 *                                      "D = A.B + C", task/dialect.cpp:34)
 *   RMSNorm / SiLU-gate as the composites of mul/add/rsqrt and
 *                  neg/exp/add/div/mul (dialect.cpp:43-46)
 *   comm.moe_dispatch(x, g) / comm.moe_combine(y, g) (dialect.cpp:65-66),
 *                  whose routing, permutation and combine are defined by the
 *                  backend's C ABI (include/kvm_sm100.h).
 * Arithmetic: inputs bf16, fp32 accumulation (dot products in the fixed
 * 16-lane order described at gemm_f32), op outputs rounded to bf16 with
 * round-to-nearest-even.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ numerics */

static inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* fp32 -> bf16, round to nearest even; NaN stays a quiet NaN. */
static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
    return (uint16_t)((u >> 16) | 0x0040u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

uint16_t orc_f32_to_bf16(float f) { return f2bf(f); }
float orc_bf16_to_f32(uint16_t h) { return bf2f(h); }

void orc_f32_to_bf16_array(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

/* ---------------------------------------------------------------- GEMM */

/* Summation order of every dot product in this file: 16 partial sums, lane j
 * accumulating the products with k % 16 == j in ascending k (one rounded
 * multiply and one rounded add per step, no fused multiply-add), then the
 * lanes combined pairwise: ((l0+l8)+(l4+l12))+... as written in lanes_sum. */
#define LANES 16

static inline float lanes_sum(const float* l) {
  float a[8], b[4], c[2];
  for (int j = 0; j < 8; ++j) a[j] = l[j] + l[j + 8];
  for (int j = 0; j < 4; ++j) b[j] = a[j] + a[j + 4];
  for (int j = 0; j < 2; ++j) c[j] = b[j] + b[j + 2];
  return c[0] + c[1];
}

/* dot(a_f32[0:K], bf16 b[0:K]) in the order above. */
__attribute__((target_clones("avx512f", "avx2", "default"))) static float
dot_f32_bf16(const float* restrict a, const uint16_t* restrict b, int K) {
  float l[LANES] = {0};
  int k = 0;
  for (; k + LANES <= K; k += LANES)
    for (int j = 0; j < LANES; ++j) l[j] = l[j] + a[k + j] * bf2f(b[k + j]);
  for (int j = 0; k + j < K; ++j) l[j] = l[j] + a[k + j] * bf2f(b[k + j]);
  return lanes_sum(l);
}

/* acc[i][n] = sum_k A[i][k] * B(k, n) for b_kn = 0 (B stored [N][K]) or
 * b_kn = 1 (B stored [K][N]; transposed once into [N][K] first). */
static void gemm_f32(const uint16_t* A, int64_t lda, const uint16_t* B,
                     int64_t ldb, int b_kn, int M, int N, int K, float* acc) {
  const uint16_t* Bn = B;
  int64_t ldbn = ldb;
  uint16_t* Bt = NULL;
  if (b_kn) {
    Bt = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)N * (size_t)K);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n)
      for (int k = 0; k < K; ++k) Bt[(int64_t)n * K + k] = B[(int64_t)k * ldb + n];
    Bn = Bt;
    ldbn = K;
  }
  /* Work items are (row, block of 64 columns) so small-M calls still use
   * every thread; each item converts its A row once. */
  const int nb = (N + 63) / 64;
#pragma omp parallel
  {
    float* arow = (float*)malloc(sizeof(float) * (size_t)(K > 0 ? K : 1));
    int cur = -1;
#pragma omp for schedule(dynamic, 1)
    for (int64_t w = 0; w < (int64_t)M * nb; ++w) {
      const int i = (int)(w / nb), n0 = (int)(w % nb) * 64;
      if (i != cur) {
        for (int k = 0; k < K; ++k) arow[k] = bf2f(A[(int64_t)i * lda + k]);
        cur = i;
      }
      const int n1 = n0 + 64 < N ? n0 + 64 : N;
      for (int n = n0; n < n1; ++n)
        acc[(int64_t)i * N + n] = dot_f32_bf16(arow, Bn + (int64_t)n * ldbn, K);
    }
    free(arow);
  }
  free(Bt);
}

/* kernel.matmul / kernel.gemm: D = A.B (+ C). out_f32 selects fp32 output;
 * C (optional) has D's dtype and row stride. */
void orc_gemm_bf16(const uint16_t* A, int64_t lda, const uint16_t* B,
                   int64_t ldb, int b_kn, const void* C, void* D, int64_t ldd,
                   int out_f32, int M, int N, int K) {
  float* acc = (float*)malloc(sizeof(float) * (size_t)M * (size_t)N);
  gemm_f32(A, lda, B, ldb, b_kn, M, N, K, acc);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i)
    for (int n = 0; n < N; ++n) {
      float v = acc[(int64_t)i * N + n];
      int64_t o = (int64_t)i * ldd + n;
      if (out_f32) {
        if (C) v += ((const float*)C)[o];
        ((float*)D)[o] = v;
      } else {
        if (C) v += bf2f(((const uint16_t*)C)[o]);
        ((uint16_t*)D)[o] = f2bf(v);
      }
    }
  free(acc);
}

/* H[M][F] = bf16(SiLU(g) * u), g = A.Wg^T, u = A.Wu^T in fp32 (not rounded
 * between the GEMM and the activation: the fused epilogue's semantics).
 * Wg, Wu stored [F][K]. */
void orc_gemm_silu_gate(const uint16_t* A, const uint16_t* Wg,
                        const uint16_t* Wu, uint16_t* H, int M, int F, int K) {
  float* g = (float*)malloc(sizeof(float) * (size_t)M * (size_t)F);
  float* u = (float*)malloc(sizeof(float) * (size_t)M * (size_t)F);
  gemm_f32(A, K, Wg, K, 0, M, F, K, g);
  gemm_f32(A, K, Wu, K, 0, M, F, K, u);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)M * F; ++i) H[i] = f2bf(silu(g[i]) * u[i]);
  free(g);
  free(u);
}

/* Gate/up packing: out[g] rows = [Wg[g][0:64]; Wu[g][0:64]; Wg[g][64:128];
 * ...], 64-row blocks, inputs [G][F][K]. */
void orc_pack_gate_up(const uint16_t* Wg, const uint16_t* Wu, uint16_t* out,
                      int G, int F, int K) {
  for (int g = 0; g < G; ++g)
    for (int r = 0; r < 2 * F; ++r) {
      int blk = r / 128, i = r % 128;
      int f = blk * 64 + (i % 64);
      const uint16_t* src = (i < 64 ? Wg : Wu) + ((int64_t)g * F + f) * K;
      memcpy(out + ((int64_t)g * 2 * F + r) * K, src, sizeof(uint16_t) * K);
    }
}

/* ------------------------------------------------------- elementwise */

void orc_rmsnorm_bf16(const uint16_t* x, const uint16_t* gamma, uint16_t* y,
                      int rows, int H, float eps) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const uint16_t* xr = x + (int64_t)r * H;
    float ss = 0.0f;
    for (int i = 0; i < H; ++i) {
      float v = bf2f(xr[i]);
      ss += v * v;
    }
    float scale = 1.0f / sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i) {
      float v = bf2f(xr[i]) * scale;
      if (gamma) v *= bf2f(gamma[i]);
      y[(int64_t)r * H + i] = f2bf(v);
    }
  }
}

void orc_silu_mul_bf16(const uint16_t* g, const uint16_t* u, uint16_t* h,
                       int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) h[i] = f2bf(silu(bf2f(g[i])) * bf2f(u[i]));
}

/* ------------------------------------------------------------------ MoE */

/* Softmax + top-k over fp32 logits [T][E]. Experts are picked by logit
 * (softmax is monotone), largest first; among equal logits the lower expert
 * index wins. Weights are the softmax probabilities (no renormalisation):
 * p_e = exp(l_e - max) / sum_i exp(l_i - max), sum in index order. */
void orc_moe_topk(const float* logits, int T, int E, int k, int32_t* idx,
                  float* w) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t) {
    const float* l = logits + (int64_t)t * E;
    float mx = l[0];
    for (int e = 1; e < E; ++e) mx = fmaxf(mx, l[e]);
    float sum = 0.0f;
    for (int e = 0; e < E; ++e) sum += expf(l[e] - mx);
    unsigned char taken[1024];
    memset(taken, 0, (size_t)E);
    for (int j = 0; j < k; ++j) {
      int bi = -1;
      float best = -INFINITY;
      for (int e = 0; e < E; ++e)
        if (!taken[e] && (bi < 0 || l[e] > best)) {
          best = l[e];
          bi = e;
        }
      taken[bi] = 1;
      idx[(int64_t)t * k + j] = bi;
      w[(int64_t)t * k + j] = expf(best - mx) / sum;
    }
  }
}

/* Stable expert-major permutation of the T*k pairs (pair i = t*k + j):
 * offsets[e] = number of pairs with expert < e; pairs of one expert keep
 * their i order. pos[i] = permuted row of pair i; src[row] = token. */
int orc_moe_permute(const int32_t* idx, int T, int k, int E, int32_t* offsets,
                    int32_t* pos, int32_t* src) {
  int64_t n = (int64_t)T * k;
  int32_t* cursor = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
  for (int64_t i = 0; i < n; ++i) {
    if (idx[i] < 0 || idx[i] >= E) {
      free(cursor);
      return -1;
    }
    cursor[idx[i] + 1]++;
  }
  for (int e = 0; e < E; ++e) cursor[e + 1] += cursor[e];
  memcpy(offsets, cursor, sizeof(int32_t) * ((size_t)E + 1));
  for (int64_t i = 0; i < n; ++i) {
    int32_t p = cursor[idx[i]]++;
    pos[i] = p;
    src[p] = (int32_t)(i / k);
  }
  free(cursor);
  return 0;
}

void orc_moe_scatter_rows(const uint16_t* x, const int32_t* pos, uint16_t* xp,
                          int T, int k, int H) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int j = 0; j < k; ++j)
      memcpy(xp + (int64_t)pos[(int64_t)t * k + j] * H, x + (int64_t)t * H,
             sizeof(uint16_t) * H);
}

/* Grouped GEMM over permuted rows: for group g, rows [off[g], off[g+1]) of A
 * times W[g]^T (W stored [G][N][K]). silu_gate = 1: W is packed gate/up
 * ([G][2F][K], 64-row blocks) and D[r][0:F] = bf16(SiLU(g) * u). */
void orc_grouped_gemm_bf16(const uint16_t* A, const uint16_t* W, uint16_t* D,
                           const int32_t* off, int G, int N, int K,
                           int silu_gate) {
  for (int g = 0; g < G; ++g) {
    int r0 = off[g], r1 = off[g + 1];
    int M = r1 - r0;
    if (M <= 0) continue;
    const uint16_t* Wg = W + (int64_t)g * N * K;
    float* acc = (float*)malloc(sizeof(float) * (size_t)M * (size_t)N);
    gemm_f32(A + (int64_t)r0 * K, K, Wg, K, 0, M, N, K, acc);
    if (!silu_gate) {
      for (int64_t i = 0; i < (int64_t)M * N; ++i)
        D[(int64_t)r0 * N + i] = f2bf(acc[i]);
    } else {
      int F = N / 2;
#pragma omp parallel for schedule(static)
      for (int i = 0; i < M; ++i)
        for (int f = 0; f < F; ++f) {
          int blk = f / 64, c = f % 64;
          float gv = acc[(int64_t)i * N + blk * 128 + c];
          float uv = acc[(int64_t)i * N + blk * 128 + 64 + c];
          D[((int64_t)r0 + i) * F + f] = f2bf(silu(gv) * uv);
        }
    }
    free(acc);
  }
}

/* out[t] = bf16(sum_j w[t][j] * Y[pos[t*k+j]]), fp32, each step a fused
 * multiply-add in slot order starting from 0. */
void orc_moe_combine(const uint16_t* Y, const int32_t* pos, const float* w,
                     uint16_t* out, int T, int k, int H) {
#pragma omp parallel for schedule(static)
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      float a = 0.0f;
      for (int j = 0; j < k; ++j)
        a = fmaf(w[(int64_t)t * k + j],
                 bf2f(Y[(int64_t)pos[(int64_t)t * k + j] * H + h]), a);
      out[(int64_t)t * H + h] = f2bf(a);
    }
}

/* The whole MoE layer: route -> permute -> scatter -> grouped SiLU-gate GEMM
 * -> grouped down GEMM -> combine. Weights: Wr [E][H], W13 packed [E][2F][H],
 * W2 [E][H][F]. Optional outputs (NULL to skip): logits [T][E], idx, topw. */
void orc_moe_layer(const uint16_t* x, const uint16_t* Wr, const uint16_t* W13,
                   const uint16_t* W2, uint16_t* out, int T, int H, int E,
                   int F, int k, float* logits_out, int32_t* idx_out,
                   float* w_out) {
  float* logits = (float*)malloc(sizeof(float) * (size_t)T * E);
  gemm_f32(x, H, Wr, H, 0, T, E, H, logits);
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)T * k);
  float* tw = (float*)malloc(sizeof(float) * (size_t)T * k);
  orc_moe_topk(logits, T, E, k, idx, tw);
  int64_t n = (int64_t)T * k;
  int32_t* off = (int32_t*)malloc(sizeof(int32_t) * ((size_t)E + 1));
  int32_t* pos = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  int32_t* src = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  orc_moe_permute(idx, T, k, E, off, pos, src);
  uint16_t* xp = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * H);
  orc_moe_scatter_rows(x, pos, xp, T, k, H);
  uint16_t* h = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * F);
  orc_grouped_gemm_bf16(xp, W13, h, off, E, 2 * F, H, 1);
  uint16_t* y = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * H);
  orc_grouped_gemm_bf16(h, W2, y, off, E, H, F, 0);
  orc_moe_combine(y, pos, tw, out, T, k, H);
  if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)T * E);
  if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)n);
  if (w_out) memcpy(w_out, tw, sizeof(float) * (size_t)n);
  free(logits); free(idx); free(tw); free(off); free(pos); free(src);
  free(xp); free(h); free(y);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------ FP8 */

/* e4m3 ("E4M3FN" in the OCP 8-bit floating point specification): 1 sign bit,
 * 4 exponent bits with bias 7, 3 mantissa bits; exponent field 0 holds the
 * subnormals m * 2^-9; no infinities; S.1111.111 is NaN, so the largest finite
 * magnitude is 1.75 * 2^8 = 448. Conversion from fp32 rounds once to the
 * nearest representable value (ties to even mantissa) and saturates: every
 * magnitude >= 448, infinities included, becomes +-448. NaN becomes 0x7F
 * with the input's sign. */
uint8_t orc_f32_to_e4m3(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return sign | 0x7Fu;
  const float a = fabsf(x);
  if (a >= 448.0f) return sign | 0x7Eu;
  if (a < 0.015625f) { /* below 2^-6: subnormal quantum 2^-9 */
    const int m = (int)nearbyintf(a * 512.0f); /* exact scaling, one rounding */
    return sign | (uint8_t)m;                  /* m == 8 encodes 2^-6 */
  }
  int e2;
  (void)frexpf(a, &e2); /* a = f * 2^e2, f in [0.5, 1) */
  int E = e2 - 1;       /* a in [2^E, 2^(E+1)) */
  int m = (int)nearbyintf(ldexpf(a, 3 - E)); /* 8..16 */
  if (m == 16) {
    m = 8;
    E += 1;
  }
  return sign | (uint8_t)(((E + 7) << 3) | (m - 8));
}

float orc_e4m3_to_f32(uint8_t v) {
  const int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
  float r;
  if (e == 15 && m == 7) return s ? -NAN : NAN;
  if (e == 0)
    r = ldexpf((float)m, -9);
  else
    r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -r : r;
}

void orc_f32_to_e4m3_array(const float* in, uint8_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f32_to_e4m3(in[i]);
}

/* Block quantisation of x [R][C] (fp32): per 128x128 block s = amax / 448
 * (1 when amax == 0), q = e4m3(x / s); scales [ceil(R/128)][ceil(C/128)]. */
void orc_quantize_e4m3_block128(const float* x, int R, int C, uint8_t* q,
                                float* scales) {
  const int br = (R + 127) / 128, bc = (C + 127) / 128;
#pragma omp parallel for collapse(2) schedule(static)
  for (int i = 0; i < br; ++i)
    for (int j = 0; j < bc; ++j) {
      float amax = 0.0f;
      for (int r = i * 128; r < R && r < i * 128 + 128; ++r)
        for (int c = j * 128; c < C && c < j * 128 + 128; ++c)
          amax = fmaxf(amax, fabsf(x[(int64_t)r * C + c]));
      const float s = amax > 0.0f ? amax / 448.0f : 1.0f;
      scales[(int64_t)i * bc + j] = s;
      for (int r = i * 128; r < R && r < i * 128 + 128; ++r)
        for (int c = j * 128; c < C && c < j * 128 + 128; ++c)
          q[(int64_t)r * C + c] = orc_f32_to_e4m3(x[(int64_t)r * C + c] / s);
    }
}

/* D[m][n] = bf16( acc ), acc = fma(P_kb, sA[m/128][kb] * sW[n/128][kb], acc)
 * over kb ascending; P_kb = sum_{k in block} Aq[m][k] * Wq[n][k] in fp32 in
 * the 16-lane order of dot_f32_bf16 (e4m3 products are exact in fp32).
 * Aq [M][K], Wq [N][K], K % 128 == 0. */
void orc_gemm_fp8_blockscaled(const uint8_t* Aq, const float* sA,
                              const uint8_t* Wq, const float* sW, uint16_t* D,
                              int M, int N, int K) {
  const int kbs = K / 128;
  float lut[256];
  for (int v = 0; v < 256; ++v) lut[v] = orc_e4m3_to_f32((uint8_t)v);
#pragma omp parallel for schedule(dynamic, 1)
  for (int m = 0; m < M; ++m) {
    float a[128];
    for (int n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int kb = 0; kb < kbs; ++kb) {
        const uint8_t* ar = Aq + (int64_t)m * K + kb * 128;
        const uint8_t* wr = Wq + (int64_t)n * K + kb * 128;
        float l[LANES] = {0};
        for (int k = 0; k < 128; ++k) a[k] = lut[ar[k]];
        for (int k = 0; k < 128; k += LANES)
          for (int j = 0; j < LANES; ++j) l[j] = l[j] + a[k + j] * lut[wr[k + j]];
        const float s = sA[(int64_t)(m / 128) * kbs + kb] * sW[(int64_t)(n / 128) * kbs + kb];
        acc = fmaf(lanes_sum(l), s, acc);
      }
      D[(int64_t)m * N + n] = f2bf(acc);
    }
  }
}

/* ------------------------------------------------------------ attention */

/* Rotary embedding in place, rotate-half form: rows are tokens b*L + pos,
 * heads are hd-wide column blocks; theta = pos * base^(-2i/hd), i < hd/2. */
void orc_rope_bf16(uint16_t* x, int64_t ld, int rows, int L, int heads, int hd,
                   float base) {
  const int half = hd / 2;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r) {
    const int pos = r % L;
    for (int h = 0; h < heads; ++h) {
      uint16_t* v = x + (int64_t)r * ld + (int64_t)h * hd;
      for (int j = 0; j < half; ++j) {
        const float inv_freq = powf(base, -2.0f * (float)j / (float)hd);
        const float ang = (float)pos * inv_freq;
        const float sn = sinf(ang), cs = cosf(ang);
        const float a = bf2f(v[j]), b = bf2f(v[j + half]);
        v[j] = f2bf(a * cs - b * sn);
        v[j + half] = f2bf(b * cs + a * sn);
      }
    }
  }
}

/* Causal GQA attention (see kvm_sm100_attention_prefill_bf16): per (b, h),
 * s[c] = dot(q, k_c) (16-lane order) for keys c <= pos, m = max(scale*s),
 * l = sum_c exp(scale*s[c] - m) (index order), p_c = bf16(exp(scale*s[c] - m) *
 * (1/l)), out = bf16(sum_c p_c v_c) (16-lane order over c). */
void orc_attention_bf16(const uint16_t* q, int64_t ldq, const uint16_t* k,
                        int64_t ldk, const uint16_t* v, int64_t ldv, uint16_t* out,
                        int64_t ldo, int B, int L, int HQ, int HKV, int hd,
                        float scale) {
  const int group = HQ / HKV;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < HQ; ++h) {
      const int kh = h / group;
      float* qf = (float*)malloc(sizeof(float) * (size_t)hd);
      float* s = (float*)malloc(sizeof(float) * (size_t)L);
      float* pf = (float*)malloc(sizeof(float) * (size_t)L);
      for (int pos = 0; pos < L; ++pos) {
        const int64_t qr = (int64_t)(b * L + pos);
        for (int d = 0; d < hd; ++d) qf[d] = bf2f(q[qr * ldq + (int64_t)h * hd + d]);
        float m = -INFINITY;
        for (int c = 0; c <= pos; ++c) {
          const uint16_t* kr = k + (int64_t)(b * L + c) * ldk + (int64_t)kh * hd;
          s[c] = dot_f32_bf16(qf, kr, hd);
          m = fmaxf(m, s[c] * scale);
        }
        float l = 0.0f;
        for (int c = 0; c <= pos; ++c) l += expf(s[c] * scale - m);
        const float inv = 1.0f / l;
        for (int c = 0; c <= pos; ++c) pf[c] = bf2f(f2bf(expf(s[c] * scale - m) * inv));
        for (int d = 0; d < hd; ++d) {
          float lanes[LANES] = {0};
          for (int c = 0; c <= pos; ++c) {
            const float vv = bf2f(v[(int64_t)(b * L + c) * ldv + (int64_t)kh * hd + d]);
            lanes[c % LANES] = lanes[c % LANES] + pf[c] * vv;
          }
          out[qr * ldo + (int64_t)h * hd + d] = f2bf(lanes_sum(lanes));
        }
      }
      free(qf);
      free(s);
      free(pf);
    }
}

/* ---------------------------------------------------- paged KV cache --- */

/* Element offset of (page, kv, slot) in a paged cache: kv 0 = K, 1 = V. The
 * strides (elements) describe either KVMeta layout (src/ir/graph_config.h:
 * 20-39): page_first = [page][layer][kv][slot][layer_size], layer_first =
 * [layer][page][kv][slot][layer_size]. */
static int64_t kv_at(int64_t page_stride, int64_t layer_stride, int64_t kv_stride,
                     int64_t token_stride, int layer, int page, int kv, int slot) {
  return (int64_t)page * page_stride + (int64_t)layer * layer_stride +
         (int64_t)kv * kv_stride + (int64_t)slot * token_stride;
}

/* kernel.kvcache.write (src/ir/dialect/kernel/dialect.cpp:70): the new
 * tokens' K and V rows (rows q_off[s]..q_off[s+1] of sequence s, positions
 * q_pos[s] + i) go to slot pos % bs of page bt[bt_off[s] + pos / bs]. */
void orc_kvcache_write(uint16_t* cache, int64_t page_stride, int64_t layer_stride,
                       int64_t kv_stride, int64_t token_stride, int bs, int layer,
                       int width, const uint16_t* k, int64_t ldk, const uint16_t* v,
                       int64_t ldv, const int32_t* q_off, const int32_t* q_pos,
                       const int32_t* bt, const int32_t* bt_off, int S) {
  for (int s = 0; s < S; ++s)
    for (int r = q_off[s]; r < q_off[s + 1]; ++r) {
      const int pos = q_pos[s] + (r - q_off[s]);
      const int page = bt[bt_off[s] + pos / bs], slot = pos % bs;
      memcpy(cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                           page, 0, slot),
             k + (int64_t)r * ldk, sizeof(uint16_t) * (size_t)width);
      memcpy(cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                           page, 1, slot),
             v + (int64_t)r * ldv, sizeof(uint16_t) * (size_t)width);
    }
}

/* kernel.kvcache.read (dialect.cpp:69): the first kv_len[s] cached tokens of
 * each sequence, gathered into rows kv_off[s].. of k and v ([rows, width]). */
void orc_kvcache_read(const uint16_t* cache, int64_t page_stride, int64_t layer_stride,
                      int64_t kv_stride, int64_t token_stride, int bs, int layer,
                      int width, uint16_t* k, uint16_t* v, const int32_t* kv_off,
                      const int32_t* bt, const int32_t* bt_off, int S) {
  for (int s = 0; s < S; ++s)
    for (int j = 0; j < kv_off[s + 1] - kv_off[s]; ++j) {
      const int page = bt[bt_off[s] + j / bs], slot = j % bs;
      const int64_t r = kv_off[s] + j;
      memcpy(k + r * width,
             cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                           page, 0, slot),
             sizeof(uint16_t) * (size_t)width);
      memcpy(v + r * width,
             cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                           page, 1, slot),
             sizeof(uint16_t) * (size_t)width);
    }
}

/* kernel.attn.decode (dialect.cpp:39) over the paged cache: query row r of
 * sequence s sits at position p = q_pos[s] + (r - q_off[s]) and attends to
 * the cached positions 0..p of s (GQA: q head h reads kv head h / (HQ/HKV)).
 * s_j = dot(q, k_j) (16-lane order), m = max(scale*s), l = sum exp(scale*s_j
 * - m) (index order), out = bf16(sum_j exp(scale*s_j - m) v_j / l) (fp32,
 * 16-lane order over j). */
void orc_attention_decode(const uint16_t* q, int64_t ldq, const uint16_t* cache,
                          int64_t page_stride, int64_t layer_stride, int64_t kv_stride,
                          int64_t token_stride, int bs, int layer, uint16_t* out,
                          int64_t ldo, const int32_t* q_off, const int32_t* q_pos,
                          const int32_t* bt, const int32_t* bt_off, int S, int HQ,
                          int HKV, int hd, float scale) {
  const int group = HQ / HKV;
  for (int s = 0; s < S; ++s) {
    const int n = q_off[s + 1] - q_off[s];
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int i = 0; i < n; ++i)
      for (int h = 0; h < HQ; ++h) {
        const int64_t r = q_off[s] + i;
        const int pos = q_pos[s] + i, kh = h / group;
        float* qf = (float*)malloc(sizeof(float) * (size_t)hd);
        float* e = (float*)malloc(sizeof(float) * (size_t)(pos + 1));
        for (int d = 0; d < hd; ++d) qf[d] = bf2f(q[r * ldq + (int64_t)h * hd + d]);
        float m = -INFINITY;
        for (int j = 0; j <= pos; ++j) {
          const uint16_t* kr =
              cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                            bt[bt_off[s] + j / bs], 0, j % bs) + (int64_t)kh * hd;
          e[j] = dot_f32_bf16(qf, kr, hd) * scale;
          m = fmaxf(m, e[j]);
        }
        float l = 0.0f;
        for (int j = 0; j <= pos; ++j) {
          e[j] = expf(e[j] - m);
          l += e[j];
        }
        for (int d = 0; d < hd; ++d) {
          float lanes[LANES] = {0};
          for (int j = 0; j <= pos; ++j) {
            const uint16_t* vr =
                cache + kv_at(page_stride, layer_stride, kv_stride, token_stride, layer,
                              bt[bt_off[s] + j / bs], 1, j % bs) + (int64_t)kh * hd;
            lanes[j % LANES] += e[j] * bf2f(vr[d]);
          }
          out[r * ldo + (int64_t)h * hd + d] = f2bf(lanes_sum(lanes) / l);
        }
        free(qf);
        free(e);
      }
  }
}
