/*
 * oracle.c — CPU restatement of mlx-dspark's verify-path arithmetic (TEST INFRASTRUCTURE).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * this library, and only as the checker or the timed CPU baseline — never as the product.
 *
 * Restates, in plain C with OpenMP over output rows:
 *   oracle_qmm   y[M,N] = x[M,K] . (scale*q + bias)^T, MLX affine 4/8-bit g64, LSB-first
 *                packing, fp32 accumulation — the arithmetic of skinny_qmm.qmm /
 *                mx.quantized_matmul(transpose=True) (src/mlx_dspark/skinny_qmm.py:13-18,
 *                :61-160; packing per :97-99, :116-125).
 *   oracle_sdpa  softmax(scale * q.k^T + mask) . v with the verify causal rule
 *                key <= L - qL + i (src/mlx_dspark/multirow_attn.py:86, :120-124), or the
 *                tree-verify ancestor rule (:187-189), fp32 softmax, GQA head h -> kv head
 *                h / (Hq/Hk) (:85).
 * Numeric parity against MLX itself is unpinned here (MLX is not importable in this
 * environment); these functions are pinned by analytic known-answer tests instead.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf2f(uint16_t v) {
  union { uint32_t u; float f; } c;
  c.u = (uint32_t)v << 16;
  return c.f;
}

/* fp32 -> bf16, round to nearest even (finite inputs) */
static inline uint16_t f2bf(float f) {
  union { uint32_t u; float f; } c;
  c.f = f;
  return (uint16_t)((c.u + 0x7FFFu + ((c.u >> 16) & 1u)) >> 16);
}

/* IEEE binary16 -> fp32 (exact) and fp32 -> binary16 round to nearest even, through the
 * compiler's _Float16 type */
static inline float h2f(uint16_t v) {
  _Float16 h;
  memcpy(&h, &v, 2);
  return (float)h;
}
static inline float round_h(float f) { return (float)(_Float16)f; }

int oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* 8 independent fp32 lanes: the dot product vectorizes without reassociating a sum. */
#define LANES 8

static inline float lane_sum(const float* a) {
  return ((a[0] + a[4]) + (a[2] + a[6])) + ((a[1] + a[5]) + (a[3] + a[7]));
}

/* out[M,N] (fp32) = x[M,K] . dequant(W)^T. x / scales / biases are bf16 bit patterns.
 * Per weight row: dequantize w = scale*q + bias (fp32) once, then one 8-lane fp32 dot
 * product per input row. */
void oracle_qmm(const uint16_t* x, int64_t ldx, int M, int K, const uint32_t* wq,
                const uint16_t* scales, const uint16_t* biases, int N, int bits, float* out,
                int64_t ldo) {
  const int G = K / 64;
  const int wpr = K * bits / 32;
  const uint32_t mask = (1u << bits) - 1u;
  const int per = 32 / bits;
  const int wpg = 64 / per; /* words per group */
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
  for (int m = 0; m < M; ++m)
    for (int k = 0; k < K; ++k) xf[(size_t)m * K + k] = bf2f(x[(size_t)m * ldx + k]);
#pragma omp parallel
  {
    float* w = (float*)aligned_alloc(64, sizeof(float) * (size_t)((K + 15) / 16 * 16));
#pragma omp for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint32_t* row = wq + (size_t)n * wpr;
      for (int g = 0; g < G; ++g) {
        const float sc = bf2f(scales[(size_t)n * G + g]);
        const float bi = bf2f(biases[(size_t)n * G + g]);
        for (int j = 0; j < wpg; ++j) {
          const uint32_t word = row[g * wpg + j];
          float* wo = w + g * 64 + j * per;
          for (int s = 0; s < per; ++s) wo[s] = sc * (float)((word >> (bits * s)) & mask) + bi;
        }
      }
      for (int m = 0; m < M; ++m) {
        const float* xr = xf + (size_t)m * K;
        float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int k = 0; k < K; k += LANES)
          for (int l = 0; l < LANES; ++l) acc[l] += xr[k + l] * w[k + l];
        out[(size_t)m * ldo + n] = lane_sum(acc);
      }
    }
    free(w);
  }
  free(xf);
}

static inline float dot_lanes(const float* a, const float* b, int D) {
  float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  int d = 0;
  for (; d + LANES <= D; d += LANES)
    for (int l = 0; l < LANES; ++l) acc[l] += a[d + l] * b[d + l];
  float s = lane_sum(acc);
  for (; d < D; ++d) s += a[d] * b[d];
  return s;
}

/* out (fp32) [B, Hq, qL, D] contiguous. q/k/v bf16 (f16 != 0: fp16) with element strides
 * {b, h, row}. */
void oracle_sdpa_t(const uint16_t* q, const int64_t* qs, const uint16_t* k, const int64_t* ks,
                   const uint16_t* v, const int64_t* vs, int B, int Hq, int Hk, int qL, int L,
                   int D, float scale, int causal, const uint32_t* anc, int round_p, int f16,
                   float* out) {
  const int G = Hq / Hk;
#define TO_F(x) (f16 ? h2f(x) : bf2f(x))
#pragma omp parallel for collapse(2) schedule(dynamic)
  for (int b = 0; b < B; ++b) {
    for (int h = 0; h < Hq; ++h) {
      const int hk = h / G;
      float* sc = (float*)malloc(sizeof(float) * (size_t)L);
      float* qv = (float*)malloc(sizeof(float) * (size_t)D);
      float* acc = (float*)malloc(sizeof(float) * (size_t)D);
      float* kf = (float*)malloc(sizeof(float) * (size_t)L * D);
      float* vf = (float*)malloc(sizeof(float) * (size_t)L * D);
      for (int j = 0; j < L; ++j) {
        const uint16_t* kr = k + b * ks[0] + hk * ks[1] + (int64_t)j * ks[2];
        const uint16_t* vr = v + b * vs[0] + hk * vs[1] + (int64_t)j * vs[2];
        for (int d = 0; d < D; ++d) {
          kf[(size_t)j * D + d] = TO_F(kr[d]);
          vf[(size_t)j * D + d] = TO_F(vr[d]);
        }
      }
      for (int i = 0; i < qL; ++i) {
        const uint16_t* qr = q + b * qs[0] + h * qs[1] + (int64_t)i * qs[2];
        for (int d = 0; d < D; ++d) qv[d] = TO_F(qr[d]);
        float mx = -INFINITY;
        for (int j = 0; j < L; ++j) {
          int ok = 1;
          if (anc != NULL) {
            const int lo = L - qL;
            if (j >= lo) ok = (anc[b * qL + i] >> (j - lo)) & 1u;
          } else if (causal) {
            ok = j <= L - qL + i;
          }
          if (!ok) {
            sc[j] = -INFINITY;
            continue;
          }
          sc[j] = dot_lanes(qv, kf + (size_t)j * D, D) * scale;
          if (sc[j] > mx) mx = sc[j];
        }
        float den = 0.f;
        for (int d = 0; d < D; ++d) acc[d] = 0.f;
        for (int j = 0; j < L; ++j) {
          if (sc[j] == -INFINITY) continue;
          const float p = expf(sc[j] - mx);
          den += p;
          /* round_p: the reference kernel feeds P to the P.V product in the input dtype
           * (src/mlx_dspark/multirow_attn.py:136-140); the row sum stays fp32 */
          const float pv = round_p ? (f16 ? round_h(p) : bf2f(f2bf(p))) : p;
          const float* vr = vf + (size_t)j * D;
          for (int d = 0; d < D; ++d) acc[d] += pv * vr[d];
        }
        float* o = out + (((int64_t)b * Hq + h) * qL + i) * D;
        for (int d = 0; d < D; ++d) o[d] = den > 0.f ? acc[d] / den : 0.f;
      }
      free(sc);
      free(qv);
      free(acc);
      free(kf);
      free(vf);
    }
  }
}
#undef TO_F

void oracle_sdpa(const uint16_t* q, const int64_t* qs, const uint16_t* k, const int64_t* ks,
                 const uint16_t* v, const int64_t* vs, int B, int Hq, int Hk, int qL, int L,
                 int D, float scale, int causal, const uint32_t* anc, int round_p, float* out) {
  oracle_sdpa_t(q, qs, k, ks, v, vs, B, Hq, Hk, qL, L, D, scale, causal, anc, round_p, 0, out);
}
