// CPU ORACLE - TEST INFRASTRUCTURE ONLY.
//
// A C++ restatement of the reference's decode/prefill path (sensenova-loop):
// the WGSL kernels of src/shaders/{matmul,linear,attention,layers}.wgsl (with the
// Q8_FNS / Q4_FNS splices of src/gpu.rs:236-308) and the op graph of
// src/engine.rs:383-493, :653-936. Each function cites the lines it follows and
// keeps their summation order (lane-strided blocks then the shared-memory tree of
// matmul.wgsl:115-127, sequential k in the tiled matmul, 16-key tiles in attend).
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
// load this library, as the checker and the timed CPU baseline. The product path
// (libsnl_b200.so) never links or calls it.
//
// Parity status: the reference ships no golden vectors or tests for this path (its
// only tests are in src/mm.rs and src/chat.rs), and its host code cannot run here
// (Rust toolchain absent, wgpu needs a graphics stack). Its kernels can: the WGSL
// sources are translated to C++ and run on the host cores (oracle/wgsl2cpp.py,
// oracle/wgslref.py), and every kernel restated here gives their output bit for bit
// (tests/test_reference_shaders.py, and the committed golden vectors of
// tests/golden/ checked by tests/test_golden.py). The op graph of engine.rs is
// restated, not run: it is checked by the reference's own invariants (batched ==
// stepwise, rollback == never fed, snapshot/restore) in tests/test_oracle_model.py.
//
// Transcendentals (exp, log, pow, sin, cos, inverseSqrt) come from the host libm, as
// in the translated shaders; WGSL leaves their precision to the implementation, so
// the GPU is compared with both within a tolerance.
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "snl_b200.h"
#include "synth.h"
#include "synth_model.h"

#define ORC_API extern "C" __attribute__((visibility("default")))

static thread_local std::string g_err;
static int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}
ORC_API const char* orc_last_error(void) { return g_err.c_str(); }

static inline float inv_sqrt(float v) { return 1.0f / sqrtf(v); }
static inline float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

// ---------------------------------------------------------------------------
// matmul.wgsl + gpu.rs Q8_FNS / Q4_FNS
// ---------------------------------------------------------------------------

// i8x4 (matmul.wgsl:41-47): byte b of the word is element b, sign-extended.
static inline void i8x4(uint32_t w, float o[4]) {
  o[0] = (float)(int8_t)(w & 0xFF);
  o[1] = (float)(int8_t)((w >> 8) & 0xFF);
  o[2] = (float)(int8_t)((w >> 16) & 0xFF);
  o[3] = (float)(int8_t)(w >> 24);
}
// u4x4 (matmul.wgsl:49-55): four nibbles from `shift`, each minus 8.
static inline void u4x4(uint32_t w, uint32_t shift, float o[4]) {
  for (int i = 0; i < 4; i++) o[i] = (float)((w >> (shift + 4 * i)) & 15u) - 8.0f;
}
static inline float dot4(const float a[4], const float* b) {
  return a[0] * b[0] + a[1] * b[1] + a[2] * b[2] + a[3] * b[3];
}

// block_dot / block_dot_v (gpu.rs:238-252 for Q8, :278-291 for Q4): eight vec4 dots
// of one 32-element block, summed left to right.
static inline float block_dot(int dtype, const uint32_t* wb, const float* x) {
  float acc = 0.f, v[4];
  if (dtype == SNL_Q8_0) {
    for (int i = 0; i < 8; i++) {
      i8x4(wb[i], v);
      float d = dot4(v, x + 4 * i);
      acc = (i == 0) ? d : acc + d;
    }
  } else {
    for (int i = 0; i < 8; i++) {
      u4x4(wb[i / 2], (i & 1) ? 16u : 0u, v);
      float d = dot4(v, x + 4 * i);
      acc = (i == 0) ? d : acc + d;
    }
  }
  return acc;
}

// The 32-lane shared-memory tree of matmul.wgsl:87-94 / :116-127.
static inline float lane_tree(float* red) {
  for (int s = 16; s > 0; s >>= 1)
    for (int l = 0; l < s; l++) red[l] += red[l + s];
  return red[0];
}

// y for one weight row and up to 8 token rows in the order of matvec1/matvec2/matvec
// (matmul.wgsl:62-100, :129-198): lane l sums blocks l, l+32, ... (scale times the
// block dot), then the lane tree.
static void matvec_row(int dtype, const uint32_t* w, const float* ws, uint32_t row, uint32_t nb,
                       const float* const* xs, int m_rows, float* out) {
  const uint32_t bw = dtype == SNL_Q8_0 ? 8 : 4;
  for (int t = 0; t < m_rows; t++) {
    float red[32];
    for (uint32_t lane = 0; lane < 32; lane++) {
      float acc = 0.f;
      for (uint32_t b = lane; b < nb; b += 32) {
        uint64_t rb = (uint64_t)row * nb + b;
        acc += ws[rb] * block_dot(dtype, w + rb * bw, xs[t] + (uint64_t)b * 32);
      }
      red[lane] = acc;
    }
    out[t] = lane_tree(red);
  }
}

// ---- vectorized forms (AVX2), bit-identical to the scalar statements above ----------
//
// The scalar functions above are the restatement. The forms below compute the same
// expression for every output element, with the same operations in the same order
// (one rounding per multiply and per add; the build disables FMA contraction): the
// decode form runs 8 of matvec's 32 lanes per AVX register, the prefill form 8 token
// rows. They only make the checker fast enough for full-size models;
// orc_set_vector(0) switches back to the scalar statements, and a CPU test checks that
// both give identical bits.
static bool g_vector = true;
ORC_API void orc_set_vector(int on) { g_vector = on != 0; }
// Threads of the oracle's parallel loops (all host cores by default; torchrun sets
// OMP_NUM_THREADS=1 in its workers, which a caller timing the CPU baseline undoes here).
ORC_API void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
ORC_API int orc_get_threads(void) { return omp_get_max_threads(); }

// Element e of word-vector w as f32: Q8 byte e (sign-extended), or Q4 nibble at `shift`+4e
// minus 8 (i8x4 / u4x4).
static inline __m256 q8_elem(__m256i w, int e) {
  switch (e) {
    case 0: return _mm256_cvtepi32_ps(_mm256_srai_epi32(_mm256_slli_epi32(w, 24), 24));
    case 1: return _mm256_cvtepi32_ps(_mm256_srai_epi32(_mm256_slli_epi32(w, 16), 24));
    case 2: return _mm256_cvtepi32_ps(_mm256_srai_epi32(_mm256_slli_epi32(w, 8), 24));
    default: return _mm256_cvtepi32_ps(_mm256_srai_epi32(w, 24));
  }
}
static inline __m256 q4_elem(__m256i w, int sh) {
  const __m256i n = _mm256_and_si256(_mm256_srlv_epi32(w, _mm256_set1_epi32(sh)), _mm256_set1_epi32(15));
  return _mm256_sub_ps(_mm256_cvtepi32_ps(n), _mm256_set1_ps(8.0f));
}

// matvec_row for one weight row, lanes 8G..8G+7 of a round at once. xt holds each token's
// x regrouped by 8-block group: xt[((t * ngrp + g) * 32 + e) * 8 + j] = x_t[(8g + j) * 32 + e].
static void matvec_row_vec(int dtype, const uint32_t* w, const float* ws, uint32_t row, uint32_t nb,
                           const float* const* xs, const float* xt, uint32_t ngrp, int m_rows, float* out) {
  const uint32_t bw = dtype == SNL_Q8_0 ? 8 : 4;
  alignas(32) float acc[8][32];
  for (int t = 0; t < m_rows; t++)
    for (int l = 0; l < 32; l++) acc[t][l] = 0.f;
  const uint32_t* wr = w + (uint64_t)row * nb * bw;
  const float* sr = ws + (uint64_t)row * nb;
  const __m256i lane_words = _mm256_mullo_epi32(_mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7), _mm256_set1_epi32((int)bw));
  for (uint32_t r0 = 0; r0 < nb; r0 += 32) {
    for (uint32_t G = 0; G < 4; G++) {
      const uint32_t b0 = r0 + 8 * G;
      if (b0 >= nb) break;
      if (b0 + 8 > nb) {  // partial group: the valid lanes, scalar, in the same order
        for (uint32_t j = 0; b0 + j < nb; j++) {
          const uint32_t b = b0 + j;
          for (int t = 0; t < m_rows; t++)
            acc[t][8 * G + j] += sr[b] * block_dot(dtype, wr + (uint64_t)b * bw, xs[t] + (uint64_t)b * 32);
        }
        continue;
      }
      __m256i W[8];
      for (uint32_t i = 0; i < bw; i++)
        W[i] = _mm256_i32gather_epi32((const int*)(wr + (uint64_t)b0 * bw + i), lane_words, 4);
      const __m256 sv = _mm256_loadu_ps(sr + b0);
      const uint32_t g = b0 / 8;
      for (int t = 0; t < m_rows; t++) {
        const float* xg = xt + ((uint64_t)t * ngrp + g) * 32 * 8;
        __m256 bd = _mm256_setzero_ps();
        for (int i = 0; i < 8; i++) {
          __m256 v[4];
          for (int e = 0; e < 4; e++)
            v[e] = dtype == SNL_Q8_0 ? q8_elem(W[i], e) : q4_elem(W[i / 2], ((i & 1) ? 16 : 0) + 4 * e);
          const float* xe = xg + (uint64_t)(4 * i) * 8;
          __m256 d = _mm256_add_ps(_mm256_mul_ps(v[0], _mm256_loadu_ps(xe)), _mm256_mul_ps(v[1], _mm256_loadu_ps(xe + 8)));
          d = _mm256_add_ps(d, _mm256_mul_ps(v[2], _mm256_loadu_ps(xe + 16)));
          d = _mm256_add_ps(d, _mm256_mul_ps(v[3], _mm256_loadu_ps(xe + 24)));
          bd = i == 0 ? d : _mm256_add_ps(bd, d);
        }
        __m256 a = _mm256_load_ps(&acc[t][8 * G]);
        _mm256_store_ps(&acc[t][8 * G], _mm256_add_ps(a, _mm256_mul_ps(sv, bd)));
      }
    }
  }
  for (int t = 0; t < m_rows; t++) out[t] = lane_tree(acc[t]);
}

// The tiled matmul's per-element statement (c = c + w[k] * x[k] for k = 0..K-1, w the
// dequantized row) for 8 weight rows x 8 token rows per step of k. K is walked in tiles
// so a tile of every token's x stays in cache; the partial sums carry over between tiles,
// so each element still sees k in order.
static void matmul_vec(int dtype, const snl_mat_p* p, uint32_t rows_m, const float* x, const uint32_t* w,
                       const float* ws, float* y) {
  const uint32_t K = p->k, N = p->n, nb = K / 32, bw = dtype == SNL_Q8_0 ? 8 : 4;
  const uint32_t G = rows_m / 8, mv = G * 8;
  constexpr uint32_t KT = 256, RT = 8;
  std::vector<float> xT((size_t)G * K * 8);
#pragma omp parallel for schedule(static)
  for (int64_t gk = 0; gk < (int64_t)G * K; gk++) {
    const uint64_t g = (uint64_t)gk / K, k = (uint64_t)gk % K;
    for (uint32_t j = 0; j < 8; j++) xT[(uint64_t)gk * 8 + j] = x[p->x_off + (g * 8 + j) * p->x_stride + k];
  }
  std::vector<float> acc((size_t)N * mv, 0.f);
  for (uint32_t k0 = 0; k0 < K; k0 += KT) {
    const uint32_t kt = std::min(KT, K - k0);
#pragma omp parallel for schedule(static)
    for (int64_t n0 = 0; n0 < (int64_t)N; n0 += RT) {
      const uint32_t rt = (uint32_t)std::min<int64_t>(RT, N - n0);
      alignas(32) float wt[RT][KT];
      for (uint32_t r = 0; r < RT; r++) {
        for (uint32_t kk = 0; kk < kt; kk++) {
          if (r >= rt) {
            wt[r][kk] = 0.f;
            continue;
          }
          const uint64_t n = n0 + r, k = k0 + kk, b = k / 32;
          const uint32_t e = (uint32_t)(k % 32), i = e / 4, q = e % 4;
          const uint32_t* wb = w + (n * nb + b) * bw;
          float v[4];
          if (dtype == SNL_Q8_0) i8x4(wb[i], v);
          else u4x4(wb[i / 2], (i & 1) ? 16u : 0u, v);
          wt[r][kk] = v[q] * ws[n * nb + b];
        }
      }
      for (uint32_t g = 0; g < G; g++) {
        __m256 c[RT];
        for (uint32_t r = 0; r < RT; r++) c[r] = _mm256_loadu_ps(&acc[((uint64_t)n0 + (r < rt ? r : 0)) * mv + g * 8]);
        const float* xg = &xT[((uint64_t)g * K + k0) * 8];
        for (uint32_t kk = 0; kk < kt; kk++) {
          const __m256 xv = _mm256_loadu_ps(xg + (uint64_t)kk * 8);
          for (uint32_t r = 0; r < RT; r++) c[r] = _mm256_add_ps(c[r], _mm256_mul_ps(_mm256_broadcast_ss(&wt[r][kk]), xv));
        }
        for (uint32_t r = 0; r < rt; r++) _mm256_storeu_ps(&acc[((uint64_t)n0 + r) * mv + g * 8], c[r]);
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < (int64_t)N; n++) {
    for (uint32_t t = 0; t < mv; t++) y[p->y_off + (uint64_t)t * p->y_stride + p->n_off + n] = acc[(uint64_t)n * mv + t];
    if (mv == rows_m) continue;
    // token rows past the last full group of 8: the scalar statement
    std::vector<float> wrow(K);
    for (uint32_t b = 0; b < nb; b++) {
      float s = ws[(uint64_t)n * nb + b];
      const uint32_t* wb = w + ((uint64_t)n * nb + b) * bw;
      float v[4];
      for (int i = 0; i < 8; i++) {
        if (dtype == SNL_Q8_0) i8x4(wb[i], v);
        else u4x4(wb[i / 2], (i & 1) ? 16u : 0u, v);
        for (int e = 0; e < 4; e++) wrow[b * 32 + i * 4 + e] = v[e] * s;
      }
    }
    for (uint32_t m = mv; m < rows_m; m++) {
      const float* xr = x + p->x_off + (uint64_t)m * p->x_stride;
      float c = 0.f;
      for (uint32_t k = 0; k < K; k++) c = c + wrow[k] * xr[k];
      y[p->y_off + (uint64_t)m * p->y_stride + p->n_off + n] = c;
    }
  }
}

// Kernels::matmul dispatch (gpu.rs:211-218, engine.rs:967-984) and the four kernels.
ORC_API int orc_mat(int dtype, const snl_step_u* st, const snl_mat_p* p, const float* x, const void* wq,
                    const float* ws, float* y) {
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return fail(SNL_E_INVALID, "orc_mat: dtype");
  if (p->k % 32) return fail(SNL_E_INVALID, "orc_mat: k % 32");
  const uint32_t rows_m = p->m_one > 0 ? p->m_one : st->m;  // rows_m (matmul.wgsl:36-39)
  const uint32_t* w = (const uint32_t*)wq;
  const uint32_t nb = p->k / 32;
  const uint32_t bw = dtype == SNL_Q8_0 ? 8 : 4;
  if (rows_m == 0) return 0;
  if (rows_m <= 8) {
    // matvec1 (m=1), matvec2 (m=2), matvec (3..8): same per-row order.
    const int m_rows = (int)std::min<uint32_t>(rows_m, 8);
    const float* xs[8];
    for (int t = 0; t < m_rows; t++) xs[t] = x + p->x_off + (uint64_t)t * p->x_stride;
    if (g_vector) {
      const uint32_t ngrp = (nb + 7) / 8;
      std::vector<float> xt((size_t)m_rows * ngrp * 32 * 8, 0.f);
      for (int t = 0; t < m_rows; t++)
        for (uint32_t b = 0; b < nb; b++)
          for (uint32_t e = 0; e < 32; e++)
            xt[(((uint64_t)t * ngrp + b / 8) * 32 + e) * 8 + b % 8] = xs[t][(uint64_t)b * 32 + e];
#pragma omp parallel for schedule(static)
      for (int64_t row = 0; row < (int64_t)p->n; row++) {
        float out[8];
        matvec_row_vec(dtype, w, ws, (uint32_t)row, nb, xs, xt.data(), ngrp, m_rows, out);
        for (int t = 0; t < m_rows; t++) y[p->y_off + (uint64_t)t * p->y_stride + p->n_off + row] = out[t];
      }
      return 0;
    }
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)p->n; row++) {
      float out[8];
      matvec_row(dtype, w, ws, (uint32_t)row, nb, xs, m_rows, out);
      for (int t = 0; t < m_rows; t++) y[p->y_off + (uint64_t)t * p->y_stride + p->n_off + row] = out[t];
    }
    return 0;
  }
  if (g_vector) {
    matmul_vec(dtype, p, rows_m, x, w, ws, y);
    return 0;
  }
  // matmul (matmul.wgsl:242-318): dequantize to f32 (dequant8, gpu.rs:265-273 /
  // :302-307) then accumulate k = 0..K-1 sequentially, c += w * x.
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < (int64_t)p->n; n++) {
    std::vector<float> wrow(p->k);
    for (uint32_t b = 0; b < nb; b++) {
      float s = ws[(uint64_t)n * nb + b];
      const uint32_t* wb = w + ((uint64_t)n * nb + b) * bw;
      float v[4];
      for (int i = 0; i < 8; i++) {
        if (dtype == SNL_Q8_0) i8x4(wb[i], v);
        else u4x4(wb[i / 2], (i & 1) ? 16u : 0u, v);
        for (int e = 0; e < 4; e++) wrow[b * 32 + i * 4 + e] = v[e] * s;
      }
    }
    for (uint32_t m = 0; m < rows_m; m++) {
      const float* xr = x + p->x_off + (uint64_t)m * p->x_stride;
      float c = 0.f;
      for (uint32_t k = 0; k < p->k; k++) c = c + wrow[k] * xr[k];
      y[p->y_off + (uint64_t)m * p->y_stride + p->n_off + n] = c;
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// layers.wgsl
// ---------------------------------------------------------------------------

// reduce_sum (layers.wgsl:34-47): 256-lane tree.
static inline float tree256(float* red) {
  for (int s = 128; s > 0; s >>= 1)
    for (int l = 0; l < s; l++) red[l] += red[l + s];
  return red[0];
}

// branch_norm (layers.wgsl:49-76).
ORC_API int orc_branch_norm(const snl_step_u* st, const snl_layer_p* p, const float* x, const float* coef,
                            const float* w, float* out, uint32_t n_groups) {
  for (uint32_t g = 0; g < n_groups; g++) {
    uint32_t m = g + (p->last_row == 1 ? st->m - 1 : 0);
    uint64_t base = (uint64_t)m * (p->x_stride != 0 ? p->x_stride : 2 * p->h);
    float pre0 = 1.f, pre1 = 0.f;
    if (p->mode == 1) {
      pre0 = coef[m * 8];
      pre1 = coef[m * 8 + 1];
    }
    float red[256];
    for (uint32_t lid = 0; lid < 256; lid++) {
      float ss = 0.f;
      for (uint32_t i = lid; i < p->h; i += 256) {
        float v = pre0 * x[base + i];
        if (p->mode == 1) v += pre1 * x[base + p->h + i];
        ss += v * v;
      }
      red[lid] = ss;
    }
    float total = tree256(red);
    float rinv = inv_sqrt(total / (float)p->h + p->eps);
    uint64_t ob = (uint64_t)g * p->h;
    for (uint32_t i = 0; i < p->h; i++) {
      float v = pre0 * x[base + i];
      if (p->mode == 1) v += pre1 * x[base + p->h + i];
      out[ob + i] = v * rinv * (p->weight_one + w[i]);
    }
  }
  return 0;
}

// mhc_dots (layers.wgsl:78-95).
ORC_API int orc_mhc_dots(const snl_step_u* st, const snl_layer_p* p, const float* x, const float* w, float* raw) {
  uint32_t d = 2 * p->h;
  for (uint32_t m = 0; m < st->m; m++) {
    uint64_t base = (uint64_t)m * d;
    for (uint32_t o = 0; o < 9; o++) {
      float red[256];
      for (uint32_t lid = 0; lid < 256; lid++) {
        float acc = 0.f;
        if (o < 8) {
          for (uint32_t i = lid; i < d; i += 256) acc += w[(uint64_t)o * d + i] * x[base + i];
        } else {
          for (uint32_t i = lid; i < d; i += 256) {
            float v = x[base + i];
            acc += v * v;
          }
        }
        red[lid] = acc;
      }
      raw[m * 9 + o] = tree256(red);
    }
  }
  return 0;
}

static inline float lse2(float a, float b) {
  float mx = std::max(a, b);
  return mx + logf(expf(a - mx) + expf(b - mx));
}

// mhc_finish (layers.wgsl:97-132).
ORC_API int orc_mhc_finish(const snl_step_u* st, const snl_layer_p* p, const float* raw, const float* w,
                           float* coef) {
  uint32_t d = 2 * p->h;
  for (uint32_t m = 0; m < st->m; m++) {
    float rinv = inv_sqrt(raw[m * 9 + 8] / (float)d + 1e-6f);
    float lg[8];
    for (int o = 0; o < 8; o++) lg[o] = raw[m * 9 + o] * rinv + w[(uint64_t)8 * d + o];
    float a = lg[4], b = lg[5], c = lg[6], e = lg[7];
    for (uint32_t it = 0; it < p->iterations; it++) {
      float r0 = lse2(a, b), r1 = lse2(c, e);
      a -= r0;
      b -= r0;
      c -= r1;
      e -= r1;
      float c0 = lse2(a, c), c1 = lse2(b, e);
      a -= c0;
      c -= c0;
      b -= c1;
      e -= c1;
    }
    float* cb = coef + m * 8;
    cb[0] = 1.0f / (1.0f + expf(-lg[0]));
    cb[1] = 1.0f / (1.0f + expf(-lg[1]));
    cb[2] = 2.0f / (1.0f + expf(-lg[2]));
    cb[3] = 2.0f / (1.0f + expf(-lg[3]));
    cb[4] = expf(a);
    cb[5] = expf(b);
    cb[6] = expf(c);
    cb[7] = expf(e);
  }
  return 0;
}

// merge (layers.wgsl:134-164).
ORC_API int orc_merge(const snl_step_u* st, const snl_layer_p* p, float* x, const float* coef, const float* br) {
  uint64_t total = (uint64_t)st->m * p->h;
  for (uint64_t idx = 0; idx < total; idx++) {
    uint64_t m = idx / p->h, i = idx % p->h;
    uint64_t b0 = m * 2 * p->h + i, b1 = b0 + p->h;
    if (p->mode == 0) {
      x[b0] += br[idx];
      continue;
    }
    if (p->mode == 3) {
      x[b1] = x[b0];
      continue;
    }
    const float* c = coef + m * 8;
    float x0 = x[b0], x1 = x[b1], b = br[idx];
    float n0 = c[4] * x0 + c[5] * x1 + c[2] * b;
    float n1 = c[6] * x0 + c[7] * x1 + c[3] * b;
    if (p->mode == 2) {
      x[b0] = 0.5f * (n0 + n1);
    } else {
      x[b0] = n0;
      x[b1] = n1;
    }
  }
  return 0;
}

// swiglu (layers.wgsl:166-175).
ORC_API int orc_swiglu(const snl_step_u* st, const snl_layer_p* p, const float* gu, float* act) {
  uint64_t total = (uint64_t)st->m * p->inter;
  for (uint64_t idx = 0; idx < total; idx++) {
    uint64_t m = idx / p->inter, i = idx % p->inter;
    float g = gu[m * 2 * p->inter + i], u = gu[m * 2 * p->inter + p->inter + i];
    act[idx] = g / (1.0f + expf(-g)) * u;
  }
  return 0;
}

// ---------------------------------------------------------------------------
// attention.wgsl
// ---------------------------------------------------------------------------

static const uint32_t HD = 256;

// pack2x16float with round-to-nearest-even.
static inline uint32_t pack2h(float a, float b) {
  return (uint32_t)snl_f32_to_f16(a) | ((uint32_t)snl_f32_to_f16(b) << 16);
}
static inline void unpack2h(uint32_t w, float* a, float* b) {
  *a = snl_f16_to_f32((uint16_t)(w & 0xFFFF));
  *b = snl_f16_to_f32((uint16_t)(w >> 16));
}

// prep (attention.wgsl:59-127).
ORC_API int orc_attn_prep(const snl_step_u* st, const snl_attn_p* p, const float* proj, float* qbuf,
                          uint32_t* kcache, uint32_t* vcache, const float* norms, const uint32_t* rpos) {
  const uint32_t q_dim = p->n_heads * HD, kv_dim = p->n_kv * HD;
  const uint32_t slots = p->n_heads + 2 * p->n_kv;
  for (uint32_t m = 0; m < st->m; m++) {
    const uint64_t pos = st->pos0 + m;
    const uint64_t row = (uint64_t)m * p->proj_stride;
    for (uint32_t slot = 0; slot < slots; slot++) {
      float sh[HD];
      if (slot >= p->n_heads + p->n_kv) {
        uint32_t kh = slot - p->n_heads - p->n_kv;
        for (uint32_t d = 0; d < HD; d++) sh[d] = proj[row + 2 * q_dim + kv_dim + kh * HD + d];
        for (uint32_t d = 0; d < HD; d += 2) vcache[(pos * kv_dim + kh * HD + d) / 2] = pack2h(sh[d], sh[d + 1]);
        continue;
      }
      float v[HD];
      uint32_t norm_off;
      for (uint32_t d = 0; d < HD; d++) {
        v[d] = slot < p->n_heads ? proj[row + slot * 2 * HD + d] : proj[row + 2 * q_dim + (slot - p->n_heads) * HD + d];
      }
      norm_off = slot < p->n_heads ? 0 : HD;
      float red[HD];
      for (uint32_t d = 0; d < HD; d++) red[d] = v[d] * v[d];
      float total = tree256(red);
      for (uint32_t d = 0; d < HD; d++) v[d] = v[d] * inv_sqrt(total / (float)HD + p->eps) * (1.0f + norms[norm_off + d]);
      for (uint32_t d = 0; d < HD; d++) sh[d] = v[d];
      const uint32_t half_rot = p->rot_dim / 2;
      const uint32_t* rp = rpos + 4 * m;
      for (uint32_t d = 0; d < p->rot_dim; d++) {
        uint32_t fi = d % half_rot;
        float inv_freq = powf(p->rope_theta, -(float)(2 * fi) / (float)p->rot_dim);
        uint32_t rot_pos = rp[0];
        if (fi % 3 == 1 && fi < (p->mrope >> 16)) rot_pos = rp[1];
        else if (fi % 3 == 2 && fi < (p->mrope & 0xFFFF)) rot_pos = rp[2];
        float ang = (float)rot_pos * inv_freq;
        float cs = cosf(ang), sn = sinf(ang);
        if (d < half_rot) v[d] = v[d] * cs - sh[d + half_rot] * sn;
        else v[d] = v[d] * cs + sh[d - half_rot] * sn;
      }
      if (slot < p->n_heads) {
        for (uint32_t d = 0; d < HD; d++) qbuf[(uint64_t)m * q_dim + slot * HD + d] = v[d];
      } else {
        uint32_t kh = slot - p->n_heads;
        for (uint32_t d = 0; d < HD; d += 2) kcache[(pos * kv_dim + kh * HD + d) / 2] = pack2h(v[d], v[d + 1]);
      }
    }
  }
  return 0;
}

// attend (attention.wgsl:129-246): workgroup (kh, m, part), G = 4, KC = 16.
ORC_API int orc_attend(const snl_step_u* st, const snl_attn_p* p, const float* proj, const float* qbuf,
                       const uint32_t* kcache, const uint32_t* vcache, float* out, float* partial) {
  const uint32_t G = 4, KC = 16;
  const uint32_t q_dim = p->n_heads * HD, kv_dim = p->n_kv * HD;
  const uint32_t parts = st->parts;
  const int64_t n_wg = (int64_t)p->n_kv * st->m * parts;
#pragma omp parallel for schedule(dynamic)
  for (int64_t wgi = 0; wgi < n_wg; wgi++) {
    const uint32_t kh = (uint32_t)(wgi % p->n_kv);
    const uint32_t m = (uint32_t)((wgi / p->n_kv) % st->m);
    const uint32_t part = (uint32_t)(wgi / ((int64_t)p->n_kv * st->m));
    std::vector<float> qs(G * HD), acc(G * HD, 0.f);
    for (uint32_t g = 0; g < G; g++)
      for (uint32_t d = 0; d < HD; d++) qs[g * HD + d] = qbuf[(uint64_t)m * q_dim + (kh * G + g) * HD + d];
    float m_sh[4], l_sh[4], corr[4];
    for (uint32_t g = 0; g < G; g++) {
      m_sh[g] = -1e30f;
      l_sh[g] = 0.f;
    }
    const uint32_t total = st->pos0 + m + 1;
    const uint32_t chunk = (total + parts - 1) / parts;
    const uint32_t start = std::min(total, part * chunk);
    const uint32_t end = std::min(total, start + chunk);
    float pr[64], partd[256];
    for (uint32_t t0 = start; t0 < end; t0 += KC) {
      const uint32_t n_keys = std::min(KC, end - t0);
      // scores: lane lid -> (g, j) = ((lid/4)/KC, (lid/4)%KC), seg = lid%4 interleaving words.
      for (uint32_t lid = 0; lid < 256; lid++) {
        uint32_t dg = (lid / 4) / KC, dj = (lid / 4) % KC, seg = lid % 4;
        float d = 0.f;
        for (uint32_t w = 0; w < 32; w++) {
          uint32_t word = w * 4 + seg;
          uint32_t kw = dj < n_keys ? kcache[((uint64_t)(t0 + dj) * kv_dim + kh * HD) / 2 + word] : 0u;
          float kx, ky;
          unpack2h(kw, &kx, &ky);
          d += qs[dg * HD + 2 * word] * kx + qs[dg * HD + 2 * word + 1] * ky;
        }
        partd[lid] = d;
      }
      for (uint32_t lid = 0; lid < G * KC; lid++) {
        uint32_t j = lid % KC, b = lid * 4;
        float sc = -1e30f;
        if (j < n_keys) sc = (partd[b] + partd[b + 1] + partd[b + 2] + partd[b + 3]) * p->scale;
        pr[lid] = sc;
      }
      for (uint32_t g = 0; g < G; g++) {
        float mx = m_sh[g];
        for (uint32_t j = 0; j < n_keys; j++) mx = std::max(mx, pr[g * KC + j]);
        float c = expf(m_sh[g] - mx);
        float sum = 0.f;
        for (uint32_t j = 0; j < KC; j++) {
          float pe = 0.f;
          if (j < n_keys) pe = expf(pr[g * KC + j] - mx);
          pr[g * KC + j] = pe;
          sum += pe;
        }
        corr[g] = c;
        m_sh[g] = mx;
        l_sh[g] = l_sh[g] * c + sum;
      }
      for (uint32_t d = 0; d < HD; d++) {
        for (uint32_t g = 0; g < G; g++) acc[g * HD + d] *= corr[g];
        for (uint32_t j = 0; j < n_keys; j++) {
          uint32_t word = vcache[((uint64_t)(t0 + j) * kv_dim + kh * HD + d) / 2];
          float a, b;
          unpack2h(word, &a, &b);
          float v = (d % 2 == 0) ? a : b;
          for (uint32_t g = 0; g < G; g++) acc[g * HD + d] += v * pr[g * KC + j];
        }
      }
    }
    for (uint32_t g = 0; g < G; g++) {
      uint32_t h = kh * G + g;
      if (parts == 1) {
        for (uint32_t d = 0; d < HD; d++) {
          float gate = proj[(uint64_t)m * p->proj_stride + h * 2 * HD + HD + d];
          out[(uint64_t)m * q_dim + h * HD + d] = acc[g * HD + d] / l_sh[g] / (1.0f + expf(-gate));
        }
      } else {
        uint64_t pi = ((uint64_t)m * p->n_heads + h) * parts + part;
        for (uint32_t d = 0; d < HD; d++) partial[pi * (HD + 2) + d] = acc[g * HD + d];
        partial[pi * (HD + 2) + HD] = m_sh[g];
        partial[pi * (HD + 2) + HD + 1] = l_sh[g];
      }
    }
  }
  return 0;
}

// combine (attention.wgsl:248-269).
ORC_API int orc_attn_combine(const snl_step_u* st, const snl_attn_p* p, const float* proj, const float* partial,
                             float* out) {
  const uint32_t q_dim = p->n_heads * HD;
  for (uint32_t m = 0; m < st->m; m++) {
    for (uint32_t h = 0; h < p->n_heads; h++) {
      uint64_t base = ((uint64_t)m * p->n_heads + h) * st->parts;
      float mx = -1e30f;
      for (uint32_t i = 0; i < st->parts; i++) mx = std::max(mx, partial[(base + i) * (HD + 2) + HD]);
      for (uint32_t d = 0; d < HD; d++) {
        float l = 0.f, acc = 0.f;
        for (uint32_t i = 0; i < st->parts; i++) {
          uint64_t o = (base + i) * (HD + 2);
          float f = expf(partial[o + HD] - mx);
          l += partial[o + HD + 1] * f;
          acc += partial[o + d] * f;
        }
        float gate = proj[(uint64_t)m * p->proj_stride + h * 2 * HD + HD + d];
        out[(uint64_t)m * q_dim + h * HD + d] = acc / l / (1.0f + expf(-gate));
      }
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// linear.wgsl
// ---------------------------------------------------------------------------

// conv (linear.wgsl:38-66).
ORC_API int orc_conv(const snl_step_u* st, const snl_lin_p* p, const float* proj, float* conv_out, float* conv_state,
                     const float* lw, float* conv_ckpt) {
  const uint32_t cd = p->conv_dim;
  for (uint32_t c = 0; c < cd; c++) {
    float w0 = lw[c * 4], w1 = lw[c * 4 + 1], w2 = lw[c * 4 + 2], w3 = lw[c * 4 + 3];
    float r0 = conv_state[c], r1 = conv_state[cd + c], r2 = conv_state[2 * cd + c];
    for (uint32_t m = 0; m < st->m; m++) {
      float cur = proj[(uint64_t)m * p->proj_stride + c];
      float o = w0 * r0 + w1 * r1 + w2 * r2 + w3 * cur;
      conv_out[(uint64_t)m * cd + c] = o / (1.0f + expf(-o));
      r0 = r1;
      r1 = r2;
      r2 = cur;
      if (m + 1 == st->ckpt) {
        conv_ckpt[c] = r0;
        conv_ckpt[cd + c] = r1;
        conv_ckpt[2 * cd + c] = r2;
      }
    }
    conv_state[c] = r0;
    conv_state[cd + c] = r1;
    conv_state[2 * cd + c] = r2;
  }
  return 0;
}

// reduce2 (linear.wgsl:72-82): 128-lane tree of vec2.
static inline void tree128x2(float* ra, float* rb) {
  for (int s = 64; s > 0; s >>= 1)
    for (int l = 0; l < s; l++) {
      ra[l] += ra[l + s];
      rb[l] += rb[l + s];
    }
}

// delta (linear.wgsl:84-140): workgroup per value head, lane j owns state column j.
ORC_API int orc_delta(const snl_step_u* st, const snl_lin_p* p, const float* proj, const float* conv_out, float* state,
                      const float* lw, float* out, float* state_ckpt) {
  const uint32_t DK = 128, DV = 128;
  const uint32_t cd = p->conv_dim;
#pragma omp parallel for schedule(static)
  for (int64_t hh = 0; hh < (int64_t)p->n_v; hh++) {
    const uint32_t h = (uint32_t)hh;
    const uint32_t kh = h / (p->n_v / p->n_k);
    const uint32_t key_dim = p->n_k * DK;
    const uint64_t sbase = (uint64_t)h * DK * DV;
    const float a_log = lw[cd * 4 + h];
    const float dt_bias = lw[cd * 4 + p->n_v + h];
    const uint32_t z_off = cd, b_off = cd + p->n_v * DV, a_off = b_off + p->n_v;
    std::vector<float> S(DK * DV);
    for (uint32_t i = 0; i < DK; i++)
      for (uint32_t j = 0; j < DV; j++) S[i * DV + j] = state[sbase + i * DV + j];
    float qs[128], ks[128], ra[128], rb[128], o[128];
    for (uint32_t m = 0; m < st->m; m++) {
      const uint64_t crow = (uint64_t)m * cd;
      for (uint32_t j = 0; j < 128; j++) {
        float qv = conv_out[crow + kh * DK + j], kv = conv_out[crow + key_dim + kh * DK + j];
        ra[j] = qv * qv;
        rb[j] = kv * kv;
      }
      tree128x2(ra, rb);
      float sx = ra[0], sy = rb[0];
      for (uint32_t j = 0; j < 128; j++) {
        float qv = conv_out[crow + kh * DK + j], kv = conv_out[crow + key_dim + kh * DK + j];
        qs[j] = qv * inv_sqrt(sx + 1e-6f) * inv_sqrt((float)DK);
        ks[j] = kv * inv_sqrt(sy + 1e-6f);
      }
      const uint64_t prow = (uint64_t)m * p->proj_stride;
      const float beta = 1.0f / (1.0f + expf(-proj[prow + b_off + h]));
      const float araw = proj[prow + a_off + h] + dt_bias;
      float sp = araw;
      if (araw <= 20.0f) sp = logf(1.0f + expf(araw));
      const float decay = expf(-expf(a_log) * sp);
      for (uint32_t j = 0; j < DV; j++) {
        float vv = conv_out[crow + 2 * key_dim + h * DV + j];
        float kv_mem = 0.f;
        for (uint32_t i = 0; i < DK; i++) {
          S[i * DV + j] *= decay;
          kv_mem += S[i * DV + j] * ks[i];
        }
        float dlt = (vv - kv_mem) * beta;
        float oo = 0.f;
        for (uint32_t i = 0; i < DK; i++) {
          S[i * DV + j] += ks[i] * dlt;
          oo += S[i * DV + j] * qs[i];
        }
        o[j] = oo;
      }
      for (uint32_t j = 0; j < 128; j++) {
        ra[j] = o[j] * o[j];
        rb[j] = 0.f;
      }
      tree128x2(ra, rb);
      const float var_o = ra[0] / (float)DV;
      for (uint32_t j = 0; j < DV; j++) {
        float norm_w = lw[cd * 4 + 2 * p->n_v + j];
        float z = proj[prow + z_off + h * DV + j];
        out[(uint64_t)m * p->n_v * DV + h * DV + j] = o[j] * inv_sqrt(var_o + p->eps) * norm_w * (z / (1.0f + expf(-z)));
      }
      if (m + 1 == st->ckpt)
        for (uint32_t i = 0; i < DK; i++)
          for (uint32_t j = 0; j < DV; j++) state_ckpt[sbase + i * DV + j] = S[i * DV + j];
    }
    for (uint32_t i = 0; i < DK; i++)
      for (uint32_t j = 0; j < DV; j++) state[sbase + i * DV + j] = S[i * DV + j];
  }
  return 0;
}

// argmax (sampler.rs:169-177): the first maximum wins.
ORC_API uint32_t orc_argmax(const float* v, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; i++)
    if (v[i] > v[best]) best = i;
  return (uint32_t)best;
}

// Sampler::distribution + draw / verify (sampler.rs:54-167) with the caller's uniform
// draws u[] in the reference's order; the top_k_small branch (top_k 1..256) and greedy.
// out: token, accepted, draws used.
ORC_API int orc_sample(const snl_sample_p* p, float* logits, uint32_t n, const uint32_t* hist_tok,
                       const uint32_t* hist_cnt, uint32_t n_hist, const float* u, int64_t draft, uint32_t* out) {
  for (uint32_t i = 0; i < n_hist; i++) {  // sampler.rs:81-88
    if (hist_tok[i] >= n) continue;
    float& l = logits[hist_tok[i]];
    if (p->repetition_penalty != 1.0f) l = l > 0.0f ? l / p->repetition_penalty : l * p->repetition_penalty;
    l -= p->presence_penalty + p->frequency_penalty * (float)hist_cnt[i];
  }
  if (p->temperature <= 1e-5f) {  // sampler.rs:89-91
    const uint32_t t = orc_argmax(logits, n);
    out[0] = t;
    out[1] = draft >= 0 && (uint64_t)draft == t ? 1 : 0;
    out[2] = 0;
    return 0;
  }
  const size_t k = p->top_k == 0 ? n : std::min<size_t>(p->top_k, n);
  if (k > 256) return fail(-7, "orc_sample: top_k > 256 is not restated");
  // top_k_small (sampler.rs:146-164): insertion after every entry >= v.
  std::vector<std::pair<float, uint32_t>> best;
  float floor = -INFINITY;
  for (uint32_t i = 0; i < n; i++) {
    const float v = logits[i];
    if (best.size() == k && v <= floor) continue;
    size_t pos = 0;
    while (pos < best.size() && best[pos].first >= v) pos++;
    best.insert(best.begin() + pos, {v, i});
    if (best.size() > k) best.pop_back();
    if (best.size() == k) floor = best[k - 1].first;
  }
  const float mx = logits[best[0].second];  // sampler.rs:105-108
  std::vector<float> probs(k);
  float sum = 0.0f;
  for (size_t i = 0; i < k; i++) {
    probs[i] = expf((logits[best[i].second] - mx) / p->temperature);
    sum += probs[i];
  }
  for (auto& x : probs) x /= sum;
  size_t keep = k;  // sampler.rs:110-124
  if (p->min_p > 0.0f) {
    const float thresh = probs[0] * p->min_p;
    keep = 0;
    while (keep < k && probs[keep] >= thresh) keep++;
    keep = std::max<size_t>(keep, 1);
  }
  if (p->top_p < 1.0f) {
    float cum = 0.0f;
    for (size_t i = 0; i < keep; i++) {
      cum += probs[i];
      if (cum >= p->top_p) {
        keep = i + 1;
        break;
      }
    }
  }
  float total = 0.0f;
  for (size_t i = 0; i < keep; i++) total += probs[i];
  for (size_t i = 0; i < keep; i++) probs[i] /= total;
  auto draw = [&](float uu, int64_t exclude) -> uint32_t {  // sampler.rs:130-144
    float tot = 0.0f;
    for (size_t i = 0; i < keep; i++)
      if ((int64_t)best[i].second != exclude) tot += probs[i];
    float r = uu * tot;
    uint32_t last = best[0].second;
    for (size_t i = 0; i < keep; i++) {
      if ((int64_t)best[i].second == exclude) continue;
      r -= probs[i];
      last = best[i].second;
      if (r <= 0.0f) return best[i].second;
    }
    return last;
  };
  if (draft < 0) {  // sample (sampler.rs:54-59)
    out[0] = draw(u[0], -1);
    out[1] = 0;
    out[2] = 1;
    return 0;
  }
  float pd = 0.0f;  // verify (sampler.rs:62-76)
  for (size_t i = 0; i < keep; i++)
    if ((int64_t)best[i].second == draft) pd = probs[i];
  if (pd > 0.0f && u[0] < pd) {
    out[0] = (uint32_t)draft;
    out[1] = 1;
    out[2] = 1;
  } else {
    out[0] = draw(pd > 0.0f ? u[1] : u[0], draft);
    out[1] = 0;
    out[2] = pd > 0.0f ? 2 : 1;
  }
  return 0;
}

// dequant_q8_row (weights.rs:155-162).
ORC_API void orc_dequant_q8_row(const int8_t* q, const float* scales, size_t n, float* out) {
  for (size_t i = 0; i < n; i++) out[i] = (float)q[i] * scales[i / 32];
}

// ---------------------------------------------------------------------------
// Seeded synthetic tensors (the rules shared with the GPU generator, synth.h)
// ---------------------------------------------------------------------------

// Quantized tensor `name` [rows, cols]: quants into q (Q8_0: rows*cols bytes; Q4_0:
// rows*cols/2 bytes), f32 scales into s (rows*cols/32).
ORC_API void orc_gen_quant(uint64_t seed, const char* name, int dtype, size_t rows, size_t cols, void* q, float* s) {
  const uint64_t nh = snl_fnv1a(name);
  const uint64_t kq = snl_key(seed, nh, 0), ks = snl_key(seed, nh, 1);
  const int64_t n = (int64_t)rows * (int64_t)cols;
  if (dtype == SNL_Q8_0) {
    int8_t* qb = (int8_t*)q;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) qb[i] = snl_q8(snl_draw(kq, (uint64_t)i));
  } else {
    uint32_t* qw = (uint32_t*)q;
#pragma omp parallel for schedule(static)
    for (int64_t wi = 0; wi < n / 8; wi++) {
      uint32_t word = 0;
      for (int e = 0; e < 8; e++) word |= snl_nib(snl_draw(kq, (uint64_t)(wi * 8 + e))) << (4 * e);
      qw[wi] = word;
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < n / 32; b++)
    s[b] = dtype == SNL_Q8_0 ? snl_q8_scale(snl_draw(ks, (uint64_t)b)) : snl_q4_scale(snl_draw(ks, (uint64_t)b));
}

// f32 segment `sub` of tensor `name`: out[i] = offset + mult * z_i.
ORC_API void orc_gen_f32(uint64_t seed, const char* name, uint32_t sub, size_t n, float mult, float offset, float* out) {
  const uint64_t k = snl_key(seed, snl_fnv1a(name), sub);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; i++) out[i] = snl_param(snl_draw(k, (uint64_t)i), mult, offset);
}

// ---------------------------------------------------------------------------
// The model: Engine (src/engine.rs) on host memory.
// ---------------------------------------------------------------------------

namespace {

const size_t MAX_M = 512;     // engine.rs:18
const size_t SNAPSHOTS = 4;   // engine.rs:20
const size_t LOGIT_ROWS = 2;  // engine.rs:22

struct QW {  // a quantized matrix (reference layout)
  int dtype = 0;
  size_t rows = 0, cols = 0;
  std::vector<uint32_t> q;
  std::vector<float> s;
};

struct Model {
  snl_model_config cfg;
  size_t ctx = 0;
  bool has_mtp = false;
  std::map<std::string, QW> qw;
  std::map<std::string, std::vector<float>> fv;
  std::vector<size_t> plan;
  // activations (engine.rs:243-273)
  std::vector<float> x, xn, proj, act, attn_out, branch, qbuf, coef, partial, logits, hid, hlast, mhc_raw;
  std::vector<uint32_t> rpos;
  // caches (engine.rs:275-297)
  std::vector<float> lin_state, conv_state, lin_ckpt, conv_ckpt;
  std::vector<std::vector<uint32_t>> kc, vc;  // one per full-attention visit
  std::vector<std::vector<float>> snap_lin, snap_conv, snap_h;
  // MTP (engine.rs:495-580)
  std::vector<float> mx, hn, m_logits;
  std::vector<uint32_t> m_kc, m_vc;
  size_t pos = 0, hid_rows = 0, head_rows = 1, prefill_chunk = MAX_M;
  size_t state_elems = 0, conv_elems = 0;

  size_t h() const { return cfg.hidden; }
  size_t q_dim() const { return (size_t)cfg.n_heads * cfg.head_dim; }
  size_t kv_dim() const { return (size_t)cfg.n_kv_heads * cfg.head_dim; }
  size_t lin_key_dim() const { return (size_t)cfg.lin_k_heads * cfg.lin_k_dim; }
  size_t lin_value_dim() const { return (size_t)cfg.lin_v_heads * cfg.lin_v_dim; }
  size_t conv_dim() const { return 2 * lin_key_dim() + lin_value_dim(); }
  size_t lin_proj_rows() const { return conv_dim() + lin_value_dim() + 2 * cfg.lin_v_heads; }
  size_t attn_proj_rows() const { return 2 * q_dim() + 2 * kv_dim(); }
  bool is_mhc(size_t l) const { return cfg.mhc_start >= 0 && (size_t)cfg.mhc_start <= l && l < (size_t)cfg.mhc_end; }
};

snl_layer_p layer_p(const Model& M, uint32_t mode, bool last_row) {
  snl_layer_p p;
  p.h = M.cfg.hidden;
  p.mode = mode;
  p.last_row = last_row;
  p.eps = M.cfg.eps;
  p.weight_one = 1.0f;
  p.iterations = M.cfg.mhc_start >= 0 ? M.cfg.mhc_iterations : 0;
  p.inter = M.cfg.intermediate;
  p.x_stride = 0;
  return p;
}

snl_attn_p attn_p(const Model& M) {
  snl_attn_p a;
  a.n_heads = M.cfg.n_heads;
  a.n_kv = M.cfg.n_kv_heads;
  a.rot_dim = M.cfg.rot_dim;
  a.proj_stride = (uint32_t)M.attn_proj_rows();
  a.rope_theta = M.cfg.rope_theta;
  a.eps = M.cfg.eps;
  a.scale = 1.0f / sqrtf((float)M.cfg.head_dim);
  a.mrope = ((3 * M.cfg.mrope_section[1]) << 16) | (3 * M.cfg.mrope_section[2]);
  return a;
}

// mat with Rows::Step / Fixed (engine.rs:336-363): x_off 0, n_off 0 (one chunk).
void mat(const Model& M, const snl_step_u& st, const QW& w, const float* x, size_t x_stride, float* y, size_t y_stride,
         uint32_t m_one, uint32_t x_off = 0) {
  (void)M;
  snl_mat_p p;
  p.n = (uint32_t)w.rows;
  p.k = (uint32_t)w.cols;
  p.x_off = x_off;
  p.x_stride = (uint32_t)x_stride;
  p.y_off = 0;
  p.y_stride = (uint32_t)y_stride;
  p.n_off = 0;
  p.m_one = m_one;
  orc_mat(w.dtype, &st, &p, x, w.q.data(), w.s.data(), y);
}

// embed (engine.rs:777-790): stream 0 = dequantized row, stream 1 = 0.
int embed(const Model& M, const uint32_t* toks, size_t n, std::vector<float>& out) {
  const size_t h = M.h();
  const QW& e = M.qw.at("embed");
  out.assign(n * 2 * h, 0.f);
  for (size_t i = 0; i < n; i++) {
    size_t t = toks[i];
    if (t >= M.cfg.vocab) return fail(SNL_E_RANGE, "token id " + std::to_string(t) + " out of range");
    orc_dequant_q8_row((const int8_t*)e.q.data() + t * h, e.s.data() + t * h / 32, h, out.data() + i * 2 * h);
  }
  return 0;
}

void push_norm(Model& M, const snl_step_u& st, const std::vector<float>* router, const std::vector<float>& norm_w) {
  if (router) {
    snl_layer_p p0 = layer_p(M, 0, false);
    orc_mhc_dots(&st, &p0, M.x.data(), router->data(), M.mhc_raw.data());
    orc_mhc_finish(&st, &p0, M.mhc_raw.data(), router->data(), M.coef.data());
  }
  snl_layer_p p = layer_p(M, router ? 1 : 0, false);
  orc_branch_norm(&st, &p, M.x.data(), M.coef.data(), norm_w.data(), M.xn.data(), st.m);
}

// The op list of engine.rs:389-481, executed for one step.
void run_layers(Model& M, const snl_step_u& st) {
  const auto& c = M.cfg;
  const size_t h = M.h();
  size_t lin_slot = 0, full_slot = 0;
  for (size_t li : M.plan) {
    const std::string L = "l" + std::to_string(li) + ".";
    const bool mhc = M.is_mhc(li);
    if (mhc && (int32_t)li == c.mhc_start) {
      snl_layer_p p3 = layer_p(M, 3, false);
      orc_merge(&st, &p3, M.x.data(), M.coef.data(), M.branch.data());
    }
    push_norm(M, st, mhc ? &M.fv.at(L + "mhc_attn") : nullptr, M.fv.at(L + "in_ln"));
    if (c.full_attention[li]) {
      const size_t stride = M.attn_proj_rows();
      mat(M, st, M.qw.at(L + "qkv"), M.xn.data(), h, M.proj.data(), stride, 0);
      snl_attn_p ap = attn_p(M);
      orc_attn_prep(&st, &ap, M.proj.data(), M.qbuf.data(), M.kc[full_slot].data(), M.vc[full_slot].data(),
                    M.fv.at(L + "qk_norm").data(), M.rpos.data());
      orc_attend(&st, &ap, M.proj.data(), M.qbuf.data(), M.kc[full_slot].data(), M.vc[full_slot].data(),
                 M.attn_out.data(), M.partial.data());
      if (st.parts > 1) orc_attn_combine(&st, &ap, M.proj.data(), M.partial.data(), M.attn_out.data());
      mat(M, st, M.qw.at(L + "o_proj"), M.attn_out.data(), M.q_dim(), M.branch.data(), h, 0);
      full_slot++;
    } else {
      const size_t stride = M.lin_proj_rows();
      mat(M, st, M.qw.at(L + "in_proj"), M.xn.data(), h, M.proj.data(), stride, 0);
      snl_lin_p lp;
      lp.conv_dim = (uint32_t)M.conv_dim();
      lp.proj_stride = (uint32_t)stride;
      lp.n_k = c.lin_k_heads;
      lp.n_v = c.lin_v_heads;
      lp.eps = c.eps;
      lp.pad[0] = lp.pad[1] = lp.pad[2] = 0;
      float* cs = M.conv_state.data() + lin_slot * M.conv_elems;
      float* ss = M.lin_state.data() + lin_slot * M.state_elems;
      float* cc = M.conv_ckpt.data() + lin_slot * M.conv_elems;
      float* sc = M.lin_ckpt.data() + lin_slot * M.state_elems;
      const float* lw = M.fv.at(L + "lin").data();
      orc_conv(&st, &lp, M.proj.data(), M.act.data(), cs, lw, cc);
      orc_delta(&st, &lp, M.proj.data(), M.act.data(), ss, lw, M.attn_out.data(), sc);
      mat(M, st, M.qw.at(L + "out_proj"), M.attn_out.data(), M.lin_value_dim(), M.branch.data(), h, 0);
      lin_slot++;
    }
    snl_layer_p pm = layer_p(M, mhc ? 1 : 0, false);
    orc_merge(&st, &pm, M.x.data(), M.coef.data(), M.branch.data());
    push_norm(M, st, mhc ? &M.fv.at(L + "mhc_ffn") : nullptr, M.fv.at(L + "post_ln"));
    mat(M, st, M.qw.at(L + "gate_up"), M.xn.data(), h, M.proj.data(), 2 * (size_t)c.intermediate, 0);
    snl_layer_p ps = layer_p(M, 0, false);
    orc_swiglu(&st, &ps, M.proj.data(), M.act.data());
    mat(M, st, M.qw.at(L + "down"), M.act.data(), c.intermediate, M.branch.data(), h, 0);
    uint32_t mode = !mhc ? 0 : ((int32_t)(li + 1) == c.mhc_end ? 2 : 1);
    snl_layer_p pe = layer_p(M, mode, false);
    orc_merge(&st, &pe, M.x.data(), M.coef.data(), M.branch.data());
  }
}

void gen_q(Model& M, uint64_t seed, const std::string& name, int dtype, size_t rows, size_t cols) {
  QW w;
  w.dtype = dtype;
  w.rows = rows;
  w.cols = cols;
  size_t n = rows * cols;
  w.q.resize(dtype == SNL_Q8_0 ? n / 4 : n / 8);
  w.s.resize(n / 32);
  orc_gen_quant(seed, name.c_str(), dtype, rows, cols, w.q.data(), w.s.data());
  M.qw[name] = std::move(w);
}

}  // namespace

ORC_API int orc_config_validate(const snl_model_config* c) {
  // ModelConfig::validate (config.rs:195-240).
  if (c->head_dim != 256) return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: head_dim must be 256");
  if (c->lin_k_dim != 128 || c->lin_v_dim != 128)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear head dims must be 128");
  if (c->conv_kernel != 4) return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear conv kernel must be 4");
  if (c->hidden % 256) return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: hidden size must be a multiple of 256");
  if (c->n_layers == 0 || c->n_layers > SNL_MAX_LAYERS)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: layer_types length mismatch");
  if (c->n_heads != 4 * c->n_kv_heads)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: attention must have 4 query heads per KV head");
  if (c->lin_k_heads == 0 || c->lin_v_heads % c->lin_k_heads)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: linear value heads must be a multiple of key heads");
  if (c->rot_dim % 2 || c->rot_dim > c->head_dim)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: invalid rotary dim");
  if (c->mrope_section[0] + c->mrope_section[1] + c->mrope_section[2] != c->rot_dim / 2)
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: M-RoPE sections must cover the rotary dims");
  if (!(c->loop_start < c->loop_end && c->loop_end <= c->n_layers && c->loop_count >= 1))
    return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: invalid loop range");
  if (c->mhc_start >= 0) {
    if (c->mhc_streams != 2)
      return fail(SNL_E_UNSUPPORTED, "unsupported model configuration: only 2 mHC streams are supported");
    auto inside = [&](uint32_t a, uint32_t b) { return a <= (uint32_t)c->mhc_start && (uint32_t)c->mhc_end <= b; };
    if (!(inside(0, c->loop_start) || inside(c->loop_start, c->loop_end) || inside(c->loop_end, c->n_layers)))
      return fail(SNL_E_UNSUPPORTED, "mHC range crosses a loop boundary");
  }
  return 0;
}

// Create the model with seeded synthetic weights: the tensors of convert.rs:228-313
// (plan) and :205-226 (plan_mtp), with the value rules of synth.h.
ORC_API void* orc_model_create(const snl_model_config* cfg, size_t ctx, uint32_t flags, uint64_t seed, int quant) {
  if (orc_config_validate(cfg)) return nullptr;
  Model* M = new Model();
  M->cfg = *cfg;
  M->ctx = std::min<size_t>(ctx, cfg->max_position);
  M->has_mtp = (flags & SNL_ENGINE_MTP) != 0;
  const auto& c = M->cfg;
  const size_t h = c.hidden, I = c.intermediate;
  // execution_plan (config.rs:243-250)
  for (size_t i = 0; i < c.loop_start; i++) M->plan.push_back(i);
  for (size_t r = 0; r < c.loop_count; r++)
    for (size_t i = c.loop_start; i < c.loop_end; i++) M->plan.push_back(i);
  for (size_t i = c.loop_end; i < c.n_layers; i++) M->plan.push_back(i);

  snl_synth::for_each_tensor(
      c, M->has_mtp, quant,
      [&](const std::string& name, int dtype, size_t rows, size_t cols) { gen_q(*M, seed, name, dtype, rows, cols); },
      [&](const std::string& name, const snl_synth::Seg* segs, int nseg) {
        size_t total = 0;
        for (int i = 0; i < nseg; i++) total += segs[i].n;
        std::vector<float> v(total);
        size_t off = 0;
        for (int i = 0; i < nseg; i++) {
          orc_gen_f32(seed, name.c_str(), segs[i].sub, segs[i].n, segs[i].mult, segs[i].offset, v.data() + off);
          off += segs[i].n;
        }
        M->fv[name] = std::move(v);
      });

  // activations (engine.rs:243-273)
  const size_t proj_w = std::max({2 * I, M->lin_proj_rows(), M->attn_proj_rows()});
  const size_t act_w = std::max(I, M->conv_dim());
  const size_t attn_w = std::max(M->q_dim(), M->lin_value_dim());
  M->x.assign(MAX_M * 2 * h, 0.f);
  M->xn.assign(MAX_M * h, 0.f);
  M->proj.assign(MAX_M * proj_w, 0.f);
  M->act.assign(MAX_M * act_w, 0.f);
  M->attn_out.assign(MAX_M * attn_w, 0.f);
  M->branch.assign(MAX_M * h, 0.f);
  M->qbuf.assign(MAX_M * M->q_dim(), 0.f);
  M->coef.assign(MAX_M * 8, 0.f);
  M->partial.assign((size_t)c.n_heads * MAX_M * (c.head_dim + 2) * 64, 0.f);
  M->rpos.assign(MAX_M * 4, 0);
  M->logits.assign(LOGIT_ROWS * c.vocab, 0.f);
  M->hid.assign((MAX_M + 1) * h, 0.f);
  M->hlast.assign(h, 0.f);
  M->mhc_raw.assign(MAX_M * 9, 0.f);
  // caches (engine.rs:275-297)
  size_t n_full = 0;
  for (size_t l : M->plan) n_full += c.full_attention[l] ? 1 : 0;
  const size_t n_lin = M->plan.size() - n_full;
  M->state_elems = (size_t)c.lin_v_heads * c.lin_k_dim * c.lin_v_dim;
  M->conv_elems = 3 * M->conv_dim();
  M->lin_state.assign(M->state_elems * n_lin, 0.f);
  M->conv_state.assign(M->conv_elems * n_lin, 0.f);
  M->lin_ckpt.assign(M->state_elems * n_lin, 0.f);
  M->conv_ckpt.assign(M->conv_elems * n_lin, 0.f);
  const size_t kv_words = M->ctx * M->kv_dim() / 2;
  M->kc.assign(n_full, std::vector<uint32_t>(kv_words, 0));
  M->vc.assign(n_full, std::vector<uint32_t>(kv_words, 0));
  M->snap_lin.assign(SNAPSHOTS, std::vector<float>(M->lin_state.size(), 0.f));
  M->snap_conv.assign(SNAPSHOTS, std::vector<float>(M->conv_state.size(), 0.f));
  M->snap_h.assign(SNAPSHOTS, std::vector<float>(h, 0.f));
  if (M->has_mtp) {
    M->mx.assign(MAX_M * 2 * h, 0.f);
    M->hn.assign(MAX_M * h, 0.f);
    M->m_logits.assign(c.vocab, 0.f);
    M->m_kc.assign(kv_words, 0);
    M->m_vc.assign(kv_words, 0);
  }
  return M;
}

ORC_API void orc_model_destroy(void* hm) { delete (Model*)hm; }

// reset (engine.rs:652-660).
ORC_API int orc_model_reset(void* hm) {
  Model& M = *(Model*)hm;
  std::fill(M.lin_state.begin(), M.lin_state.end(), 0.f);
  std::fill(M.conv_state.begin(), M.conv_state.end(), 0.f);
  M.pos = 0;
  M.hid_rows = 0;
  return 0;
}

// snapshot / restore / rollback (engine.rs:662-697).
ORC_API int orc_model_snapshot(void* hm, size_t slot) {
  Model& M = *(Model*)hm;
  if (slot >= SNAPSHOTS) return fail(SNL_E_RANGE, "snapshot slot out of range");
  M.snap_lin[slot] = M.lin_state;
  M.snap_conv[slot] = M.conv_state;
  M.snap_h[slot] = M.hlast;
  return 0;
}
ORC_API int orc_model_restore(void* hm, size_t slot, size_t pos) {
  Model& M = *(Model*)hm;
  if (slot >= SNAPSHOTS) return fail(SNL_E_RANGE, "snapshot slot out of range");
  M.lin_state = M.snap_lin[slot];
  M.conv_state = M.snap_conv[slot];
  M.hlast = M.snap_h[slot];
  M.pos = pos;
  M.hid_rows = 0;
  return 0;
}
ORC_API int orc_model_rollback(void* hm) {
  Model& M = *(Model*)hm;
  M.lin_state = M.lin_ckpt;
  M.conv_state = M.conv_ckpt;
  std::copy(M.hid.begin() + M.h(), M.hid.begin() + 2 * M.h(), M.hlast.begin());
  M.pos -= 1;
  M.hid_rows = 1;
  return 0;
}
ORC_API size_t orc_model_pos(void* hm) { return ((Model*)hm)->pos; }
ORC_API size_t orc_model_hid_rows(void* hm) { return ((Model*)hm)->hid_rows; }
ORC_API int orc_model_read_hidden(void* hm, size_t row0, size_t rows, float* out) {
  Model& M = *(Model*)hm;
  std::copy(M.hid.begin() + row0 * M.h(), M.hid.begin() + (row0 + rows) * M.h(), out);
  return 0;
}

// Raw tensor access for tests: quants and scales of `name` (nullptr if absent).
ORC_API const void* orc_model_tensor(void* hm, const char* name, size_t* rows, size_t* cols, const float** scales) {
  Model& M = *(Model*)hm;
  auto it = M.qw.find(name);
  if (it != M.qw.end()) {
    *rows = it->second.rows;
    *cols = it->second.cols;
    *scales = it->second.s.data();
    return it->second.q.data();
  }
  auto jt = M.fv.find(name);
  if (jt != M.fv.end()) {
    *rows = 1;
    *cols = jt->second.size();
    *scales = nullptr;
    return jt->second.data();
  }
  return nullptr;
}

// The quantization of a named matrix (SNL_Q8_0 / SNL_Q4_0), or -1.
ORC_API int orc_model_tensor_dtype(void* hm, const char* name) {
  const Model& M = *(const Model*)hm;
  auto it = M.qw.find(name);
  return it == M.qw.end() ? -1 : it->second.dtype;
}

// forward_mm (engine.rs:801-936).
ORC_API int orc_model_forward_mm(void* hm, const uint32_t* tokens, size_t n, const uint32_t* pos3,
                                 const uint32_t* embed_idx, const float* embeds, size_t n_embeds, size_t logit_rows,
                                 int ckpt, float* logits_out) {
  Model& M = *(Model*)hm;
  const size_t h = M.h();
  const bool want = logit_rows > 0;
  if (logit_rows > LOGIT_ROWS || (ckpt && n != 2)) return fail(SNL_E_INVALID, "forward: unsupported logits or checkpoint request");
  if (n == 0) return fail(SNL_E_INVALID, "forward called with no tokens");
  for (size_t i = 0; i < n_embeds; i++)
    if (embed_idx[i] >= n) return fail(SNL_E_INVALID, "forward: positions or embeddings do not match the tokens");
  if (M.pos + n > M.ctx)
    return fail(SNL_E_RANGE, "context length exceeded (" + std::to_string(M.pos + n) + " > " + std::to_string(M.ctx) + ")");
  const size_t chunk = M.prefill_chunk;
  const size_t n_chunks = (n + chunk - 1) / chunk;
  size_t rows_out = 0;
  for (size_t ci = 0; ci < n_chunks; ci++) {
    const bool last = ci + 1 == n_chunks;
    const size_t c0 = ci * chunk;
    const size_t m = std::min(chunk, n - c0);
    const size_t total = M.pos + m;
    const size_t parts = m <= 4 ? std::min<size_t>(std::max<size_t>((total + 255) / 256, 1), 64) : 1;
    snl_step_u st = {(uint32_t)m, (uint32_t)M.pos, (uint32_t)parts, (uint32_t)(ckpt ? 1 : 0)};
    const size_t rows = std::min(logit_rows, m);
    if (last && want) M.head_rows = rows;
    std::vector<float> emb;
    if (int rc = embed(M, tokens + c0, m, emb)) return rc;
    for (size_t e = 0; e < n_embeds; e++) {
      size_t i = embed_idx[e];
      if (i >= c0 && i < c0 + m) std::copy(embeds + e * h, embeds + (e + 1) * h, emb.begin() + (i - c0) * 2 * h);
    }
    std::copy(emb.begin(), emb.end(), M.x.begin());
    for (size_t i = 0; i < m; i++)
      for (int k = 0; k < 4; k++)
        M.rpos[i * 4 + k] = pos3 ? (k < 3 ? pos3[(c0 + i) * 3 + k] : 0u) : (uint32_t)(M.pos + i);
    // Row 0 of hid is the hidden state of the token before this step (engine.rs:889-890).
    std::copy(M.hlast.begin(), M.hlast.end(), M.hid.begin());
    run_layers(M, st);
    snl_layer_p pf = layer_p(M, 0, false);
    orc_branch_norm(&st, &pf, M.x.data(), M.coef.data(), M.fv.at("norm").data(), M.hid.data() + h, (uint32_t)m);
    if (last && want) {
      // head (engine.rs:493, :835-842): the last `rows` rows of hid.
      mat(M, st, M.qw.at("lm_head"), M.hid.data(), h, M.logits.data(), M.cfg.vocab, (uint32_t)rows,
          (uint32_t)((m - rows + 1) * h));
      rows_out = rows;
    }
    std::copy(M.hid.begin() + m * h, M.hid.begin() + (m + 1) * h, M.hlast.begin());
    M.pos += m;
    M.hid_rows = m;
  }
  if (want && logits_out) std::copy(M.logits.begin(), M.logits.begin() + rows_out * M.cfg.vocab, logits_out);
  return 0;
}

// mtp (engine.rs:708-774).
ORC_API int orc_model_mtp(void* hm, size_t r0, const uint32_t* tokens, size_t n, const uint32_t* pos3, size_t slot0,
                          int draft, uint32_t* draft_out) {
  Model& M = *(Model*)hm;
  if (!M.has_mtp) return fail(SNL_E_STATE, "mtp: the model has no MTP head");
  if (n == 0 || r0 + n > M.hid_rows + 1) return fail(SNL_E_RANGE, "mtp: rows out of range");
  const size_t h = M.h();
  const auto& c = M.cfg;
  for (size_t c0 = 0; c0 < n; c0 += MAX_M) {
    const size_t c1 = std::min(c0 + MAX_M, n);
    const size_t m = c1 - c0;
    const size_t total = slot0 + c1;
    const size_t parts = m <= 4 ? std::min<size_t>(std::max<size_t>((total + 255) / 256, 1), 64) : 1;
    if (slot0 + c1 > M.ctx) return fail(SNL_E_RANGE, "mtp: rows out of range");
    snl_step_u st = {(uint32_t)m, (uint32_t)(slot0 + c0), (uint32_t)parts, 0};
    std::vector<float> emb;
    if (int rc = embed(M, tokens + c0, m, emb)) return rc;
    std::copy(emb.begin(), emb.end(), M.mx.begin());
    for (size_t i = 0; i < m; i++) {
      for (int k = 0; k < 3; k++) M.rpos[i * 4 + k] = pos3[(c0 + i) * 3 + k];
      M.rpos[i * 4 + 3] = 0;
    }
    const bool last = c1 == n;
    snl_layer_p p0 = layer_p(M, 0, false);
    // pre: norm_e of the embedding (engine.rs:527)
    orc_branch_norm(&st, &p0, M.mx.data(), M.coef.data(), M.fv.at("mtp.norm_e").data(), M.xn.data(), (uint32_t)m);
    // norm_h of hidden rows r0+c0.. (engine.rs:736-747), x_stride = hidden
    snl_layer_p ph = p0;
    ph.x_stride = (uint32_t)h;
    orc_branch_norm(&st, &ph, M.hid.data() + (r0 + c0) * h, M.coef.data(), M.fv.at("mtp.norm_h").data(), M.hn.data(),
                    (uint32_t)m);
    // ops (engine.rs:549-566)
    mat(M, st, M.qw.at("mtp.fc_e"), M.xn.data(), h, M.mx.data(), 2 * h, 0);
    mat(M, st, M.qw.at("mtp.fc_h"), M.hn.data(), h, M.branch.data(), h, 0);
    orc_merge(&st, &p0, M.mx.data(), M.coef.data(), M.branch.data());
    orc_branch_norm(&st, &p0, M.mx.data(), M.coef.data(), M.fv.at("mtp.in_ln").data(), M.xn.data(), (uint32_t)m);
    const size_t stride = M.attn_proj_rows();
    mat(M, st, M.qw.at("mtp.qkv"), M.xn.data(), h, M.proj.data(), stride, 0);
    snl_attn_p ap = attn_p(M);
    orc_attn_prep(&st, &ap, M.proj.data(), M.qbuf.data(), M.m_kc.data(), M.m_vc.data(), M.fv.at("mtp.qk_norm").data(),
                  M.rpos.data());
    orc_attend(&st, &ap, M.proj.data(), M.qbuf.data(), M.m_kc.data(), M.m_vc.data(), M.attn_out.data(), M.partial.data());
    if (st.parts > 1) orc_attn_combine(&st, &ap, M.proj.data(), M.partial.data(), M.attn_out.data());
    mat(M, st, M.qw.at("mtp.o_proj"), M.attn_out.data(), M.q_dim(), M.branch.data(), h, 0);
    orc_merge(&st, &p0, M.mx.data(), M.coef.data(), M.branch.data());
    orc_branch_norm(&st, &p0, M.mx.data(), M.coef.data(), M.fv.at("mtp.post_ln").data(), M.xn.data(), (uint32_t)m);
    mat(M, st, M.qw.at("mtp.gate_up"), M.xn.data(), h, M.proj.data(), 2 * (size_t)c.intermediate, 0);
    orc_swiglu(&st, &p0, M.proj.data(), M.act.data());
    mat(M, st, M.qw.at("mtp.down"), M.act.data(), c.intermediate, M.branch.data(), h, 0);
    orc_merge(&st, &p0, M.mx.data(), M.coef.data(), M.branch.data());
    if (last && draft) {
      snl_layer_p pl = layer_p(M, 0, true);
      orc_branch_norm(&st, &pl, M.mx.data(), M.coef.data(), M.fv.at("mtp.norm").data(), M.xn.data(), 1);
      mat(M, st, M.qw.at("lm_head"), M.xn.data(), h, M.m_logits.data(), c.vocab, 1);
    }
  }
  if (draft && draft_out) *draft_out = orc_argmax(M.m_logits.data(), c.vocab);
  return 0;
}

ORC_API const float* orc_model_mtp_logits(void* hm) {
  Model& M = *(Model*)hm;
  return M.has_mtp ? M.m_logits.data() : nullptr;
}

// The shared f32 <-> f16 conversions (synth.h), exported for tests against numpy.
ORC_API uint16_t orc_f32_to_f16(float f) { return snl_f32_to_f16(f); }
ORC_API float orc_f16_to_f32(uint16_t h) { return snl_f16_to_f32(h); }

// ---------------------------------------------------------------------------
// The vision tower: src/shaders/vision.wgsl and Vision::encode (src/vision.rs).
// ---------------------------------------------------------------------------

// layer_norm (vision.wgsl:40-62): per row, 256 lane-strided partial sums then the tree
// (reduce_sum, vision.wgsl:29-38) for the mean and for the centred variance.
ORC_API int orc_vis_layer_norm(const snl_vis_p* p, const float* a, float* b, const float* w) {
  const uint32_t cols = p->cols;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)p->rows; r++) {
    const float* ar = a + (uint64_t)r * cols;
    float red[256];
    for (uint32_t lid = 0; lid < 256; lid++) {
      float s = 0.f;
      for (uint32_t c = lid; c < cols; c += 256) s += ar[c];
      red[lid] = s;
    }
    const float mean = tree256(red) / (float)cols;
    for (uint32_t lid = 0; lid < 256; lid++) {
      float v = 0.f;
      for (uint32_t c = lid; c < cols; c += 256) {
        const float d = ar[c] - mean;
        v += d * d;
      }
      red[lid] = v;
    }
    const float inv = 1.0f / sqrtf(tree256(red) / (float)cols + p->eps);
    for (uint32_t c = 0; c < cols; c++) b[(uint64_t)r * cols + c] = (ar[c] - mean) * inv * w[c] + w[cols + c];
  }
  return 0;
}

static float vis_gelu_tanh(float x) {  // vision.wgsl:64-67
  float u = 0.7978845608f * (x + 0.044715f * x * x * x);
  u = u < -15.f ? -15.f : (u > 15.f ? 15.f : u);
  return 0.5f * x * (1.0f + tanhf(u));
}
static float vis_erf(float x) {  // vision.wgsl:69-75 (Abramowitz & Stegun 7.1.26)
  const float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
  const float y =
      1.0f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t *
                 expf(-x * x);
  return x >= 0.f ? y : -y;
}
static float vis_gelu_erf(float x) { return 0.5f * x * (1.0f + vis_erf(x * 0.7071067812f)); }

// epilogue (vision.wgsl:77-98).
ORC_API int orc_vis_epilogue(const snl_vis_p* p, float* a, float* b, const float* w, const float* e) {
  const uint64_t total = (uint64_t)p->rows * p->cols;
  for (uint64_t i = 0; i < total; i++) {
    float v = a[i] + w[i % p->cols];
    if (p->act == 1) v = vis_gelu_tanh(v);
    else if (p->act == 2) v = vis_gelu_erf(v);
    if (p->mode == 0) a[i] = v;
    else if (p->mode == 1) b[i] = b[i] + v;
    else b[i] = v + e[i];
  }
  return 0;
}

// rope (vision.wgsl:100-130) on [rows, 3, heads, 72].
ORC_API int orc_vis_rope(const snl_vis_p* p, float* a) {
  const uint32_t HD = 72, HALF = 36, per_token = p->heads * HALF, hidden = p->heads * HD;
  for (uint64_t i = 0; i < (uint64_t)p->rows * per_token; i++) {
    const uint32_t token = (uint32_t)(i / per_token), h = (uint32_t)(i % per_token) / HALF, j = (uint32_t)(i % HALF);
    const uint32_t mw = p->grid_w / 2, blk = token / 4, intra = token % 4;
    const uint32_t row = (blk / mw) * 2 + intra / 2, col = (blk % mw) * 2 + intra % 2;
    const uint32_t fi = j % (HALF / 2);
    const uint32_t pos = j >= HALF / 2 ? col : row;
    const float ang = (float)pos * powf(10000.0f, -(float)(2 * fi) / (float)HALF);
    const float cs = cosf(ang), sn = sinf(ang);
    for (uint32_t part = 0; part < 2; part++) {
      const uint64_t base = (uint64_t)token * 3 * hidden + part * hidden + h * HD;
      const float x1 = a[base + j], x2 = a[base + j + HALF];
      a[base + j] = x1 * cs - x2 * sn;
      a[base + j + HALF] = x2 * cs + x1 * sn;
    }
  }
  return 0;
}

// attend (vision.wgsl:137-206): per query, 16-key tiles, online softmax.
ORC_API int orc_vis_attend(const snl_vis_p* p, const float* qkv, float* out) {
  const uint32_t HD = 72, TK = 16, n = p->rows, hidden = p->heads * HD, stride = 3 * hidden;
  const float scale = 1.0f / sqrtf((float)HD);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t h = 0; h < (int64_t)p->heads; h++) {
    for (int64_t qi = 0; qi < (int64_t)n; qi++) {
      float q[72], acc[72] = {0};
      for (uint32_t d = 0; d < HD; d++) q[d] = qkv[(uint64_t)qi * stride + h * HD + d] * scale;
      float mx = -1e30f, l = 0.f, sc[16];
      for (uint32_t k0 = 0; k0 < n; k0 += TK) {
        const uint32_t cnt = std::min(TK, n - k0);
        float tmax = mx;
        for (uint32_t j = 0; j < cnt; j++) {
          const float* kr = qkv + (uint64_t)(k0 + j) * stride + hidden + h * HD;
          float s = 0.f;
          for (uint32_t d = 0; d < HD; d += 4) s += q[d] * kr[d] + q[d + 1] * kr[d + 1] + q[d + 2] * kr[d + 2] + q[d + 3] * kr[d + 3];
          sc[j] = s;
          tmax = std::max(tmax, s);
        }
        const float corr = expf(mx - tmax);
        l *= corr;
        for (uint32_t d = 0; d < HD; d++) acc[d] *= corr;
        for (uint32_t j = 0; j < cnt; j++) {
          const float* vr = qkv + (uint64_t)(k0 + j) * stride + 2 * hidden + h * HD;
          const float pj = expf(sc[j] - tmax);
          l += pj;
          for (uint32_t d = 0; d < HD; d++) acc[d] += pj * vr[d];
        }
        mx = tmax;
      }
      for (uint32_t d = 0; d < HD; d++) out[(uint64_t)qi * hidden + h * HD + d] = acc[d] / l;
    }
  }
  return 0;
}

namespace {

struct OrcVision {
  snl_vision_config c;
  std::map<std::string, QW> qw;
  std::map<std::string, std::vector<float>> fv;
};

// The synthetic tower of snl_vision_fill_synthetic: Q8_0 matrices by the shared rules,
// LayerNorm weight 1 + 0.1 z | bias 0.05 z, other biases 0.02 z, position table 0.3 z.
void vis_gen(OrcVision& V, uint64_t seed) {
  const auto& c = V.c;
  const size_t h = c.hidden, ip = c.intermediate_padded, md = (size_t)h * 4, pd = 3ull * c.temporal_patch * c.patch * c.patch;
  auto q8 = [&](const std::string& n, size_t rows, size_t cols) {
    QW w;
    w.dtype = SNL_Q8_0;
    w.rows = rows;
    w.cols = cols;
    w.q.resize(rows * cols / 4);
    w.s.resize(rows * cols / 32);
    orc_gen_quant(seed, n.c_str(), SNL_Q8_0, rows, cols, w.q.data(), w.s.data());
    V.qw[n] = std::move(w);
  };
  auto vec = [&](const std::string& n, size_t len, float mult) {
    std::vector<float> v(len);
    orc_gen_f32(seed, n.c_str(), 0, len, mult, 0.f, v.data());
    V.fv[n] = std::move(v);
  };
  auto norm = [&](const std::string& n) {
    std::vector<float> v(2 * h);
    orc_gen_f32(seed, n.c_str(), 0, h, 0.1f, 1.0f, v.data());
    orc_gen_f32(seed, n.c_str(), 1, h, 0.05f, 0.0f, v.data() + h);
    V.fv[n] = std::move(v);
  };
  q8("v.patch", h, pd);
  vec("v.patch_b", h, 0.02f);
  vec("v.pos", (size_t)c.pos_side * c.pos_side * h, 0.3f);
  for (uint32_t i = 0; i < c.depth; i++) {
    const std::string b = "v" + std::to_string(i) + ".";
    norm(b + "n1");
    norm(b + "n2");
    q8(b + "qkv", 3 * h, h);
    vec(b + "qkv_b", 3 * h, 0.02f);
    q8(b + "proj", h, h);
    vec(b + "proj_b", h, 0.02f);
    q8(b + "fc1", ip, h);
    vec(b + "fc1_b", ip, 0.02f);
    q8(b + "fc2", h, ip);
    vec(b + "fc2_b", h, 0.02f);
  }
  norm("vm.norm");
  q8("vm.fc1", md, md);
  vec("vm.fc1_b", md, 0.02f);
  q8("vm.fc2", c.out_hidden, md);
  vec("vm.fc2_b", c.out_hidden, 0.02f);
}

// Vision::pos_embed (vision.rs:141-175).
std::vector<float> vis_pos_embed(const OrcVision& V, size_t h, size_t w) {
  const size_t side = V.c.pos_side, hid = V.c.hidden, m = V.c.merge;
  auto lin = [&](size_t n) {
    std::vector<float> o(n);
    for (size_t i = 0; i < n; i++) o[i] = n == 1 ? 0.0f : (float)(side - 1) * (float)i / (float)(n - 1);
    return o;
  };
  const std::vector<float> hs = lin(h), ws = lin(w);
  const std::vector<float>& pos = V.fv.at("v.pos");
  std::vector<float> out(h * w * hid, 0.f);
  for (size_t token = 0; token < h * w; token++) {
    const size_t blk = token / (m * m), intra = token % (m * m);
    const size_t r = (blk / (w / m)) * m + intra / m, c = (blk % (w / m)) * m + intra % m;
    const size_t fh = (size_t)hs[r], fw = (size_t)ws[c];
    const size_t ch = std::min(fh + 1, side - 1), cw = std::min(fw + 1, side - 1);
    const float dh = hs[r] - (float)fh, dw = ws[c] - (float)fw;
    const size_t idx[4] = {fh * side + fw, fh * side + cw, ch * side + fw, ch * side + cw};
    const float wt[4] = {(1.0f - dh) * (1.0f - dw), (1.0f - dh) * dw, dh * (1.0f - dw), dh * dw};
    for (int k = 0; k < 4; k++)
      for (size_t j = 0; j < hid; j++) out[token * hid + j] += pos[idx[k] * hid + j] * wt[k];
  }
  return out;
}

// Kernels::matmul over `rows` token rows (vision.rs:314-343, one chunk).
void vis_mat(const QW& w, const float* x, size_t rows, float* y, size_t y_stride) {
  snl_mat_p p;
  p.n = (uint32_t)w.rows;
  p.k = (uint32_t)w.cols;
  p.x_off = 0;
  p.x_stride = (uint32_t)w.cols;
  p.y_off = 0;
  p.y_stride = (uint32_t)y_stride;
  p.n_off = 0;
  p.m_one = 0;
  snl_step_u st{(uint32_t)rows, 0, 1, 0};
  orc_mat(w.dtype, &st, &p, x, w.q.data(), w.s.data(), y);
}

}  // namespace

ORC_API void* orc_vision_create(const snl_vision_config* cfg, uint64_t seed) {
  OrcVision* V = new OrcVision();
  V->c = *cfg;
  vis_gen(*V, seed);
  return V;
}
ORC_API void orc_vision_destroy(void* hv) { delete (OrcVision*)hv; }

// Vision::encode (vision.rs:176-311), frame by frame, in the op order of :222-272.
ORC_API int orc_vision_encode(void* hv, const float* patches, size_t frames, size_t h, size_t w, float* out) {
  OrcVision& V = *(OrcVision*)hv;
  const auto& c = V.c;
  const size_t pd = 3ull * c.temporal_patch * c.patch * c.patch;
  if (h % c.merge || w % c.merge) return fail(SNL_E_INVALID, "vision input has the wrong shape");
  const size_t n = h * w, hid = c.hidden, nq = n / (c.merge * c.merge), ip = c.intermediate_padded,
               md = hid * c.merge * c.merge;
  const std::vector<float> pos = vis_pos_embed(V, h, w);
  std::vector<float> x(n * hid), xn(n * hid), tmp(n * hid), att(n * hid), qkv(std::max(n * 3 * hid, nq * c.out_hidden)),
      mlp(std::max(n * ip, nq * md)), dummy(16);
  auto norm = [&](const std::vector<float>& nw) {
    snl_vis_p p{(uint32_t)n, (uint32_t)hid, 0, 0, 1e-6f, 0, 0, 0};
    orc_vis_layer_norm(&p, x.data(), xn.data(), nw.data());
  };
  auto epi = [&](float* a, float* b, const std::vector<float>& bias, const float* e, size_t rows, size_t cols,
                 uint32_t mode, uint32_t act) {
    snl_vis_p p{(uint32_t)rows, (uint32_t)cols, mode, act, 0.f, 0, 0, 0};
    orc_vis_epilogue(&p, a, b, bias.data(), e);
  };
  for (size_t f = 0; f < frames; f++) {
    vis_mat(V.qw.at("v.patch"), patches + f * n * pd, n, tmp.data(), hid);
    epi(tmp.data(), x.data(), V.fv.at("v.patch_b"), pos.data(), n, hid, 2, 0);
    for (uint32_t i = 0; i < c.depth; i++) {
      const std::string b = "v" + std::to_string(i) + ".";
      norm(V.fv.at(b + "n1"));
      vis_mat(V.qw.at(b + "qkv"), xn.data(), n, qkv.data(), 3 * hid);
      epi(qkv.data(), dummy.data(), V.fv.at(b + "qkv_b"), nullptr, n, 3 * hid, 0, 0);
      snl_vis_p rp{(uint32_t)n, 0, 0, 0, 0.f, (uint32_t)w, c.n_heads, 0};
      orc_vis_rope(&rp, qkv.data());
      orc_vis_attend(&rp, qkv.data(), att.data());
      vis_mat(V.qw.at(b + "proj"), att.data(), n, tmp.data(), hid);
      epi(tmp.data(), x.data(), V.fv.at(b + "proj_b"), nullptr, n, hid, 1, 0);
      norm(V.fv.at(b + "n2"));
      vis_mat(V.qw.at(b + "fc1"), xn.data(), n, mlp.data(), ip);
      epi(mlp.data(), dummy.data(), V.fv.at(b + "fc1_b"), nullptr, n, ip, 0, 1);
      vis_mat(V.qw.at(b + "fc2"), mlp.data(), n, tmp.data(), hid);
      epi(tmp.data(), x.data(), V.fv.at(b + "fc2_b"), nullptr, n, hid, 1, 0);
    }
    norm(V.fv.at("vm.norm"));
    vis_mat(V.qw.at("vm.fc1"), xn.data(), nq, mlp.data(), md);
    epi(mlp.data(), dummy.data(), V.fv.at("vm.fc1_b"), nullptr, nq, md, 0, 2);
    vis_mat(V.qw.at("vm.fc2"), mlp.data(), nq, qkv.data(), c.out_hidden);
    epi(qkv.data(), dummy.data(), V.fv.at("vm.fc2_b"), nullptr, nq, c.out_hidden, 0, 0);
    memcpy(out + f * nq * c.out_hidden, qkv.data(), nq * c.out_hidden * sizeof(float));
  }
  return 0;
}

// The synthetic tower's tensors, for the GPU tests that load them through set_tensor.
ORC_API int orc_vision_tensor(void* hv, const char* name, const void** q, const float** s, size_t* rows, size_t* cols) {
  OrcVision& V = *(OrcVision*)hv;
  auto it = V.qw.find(name);
  if (it != V.qw.end()) {
    *q = it->second.q.data();
    *s = it->second.s.data();
    *rows = it->second.rows;
    *cols = it->second.cols;
    return SNL_Q8_0;
  }
  auto jt = V.fv.find(name);
  if (jt == V.fv.end()) return fail(SNL_E_INVALID, "orc_vision_tensor: unknown tensor");
  *q = jt->second.data();
  *s = nullptr;
  *rows = 1;
  *cols = jt->second.size();
  return SNL_F32;
}
