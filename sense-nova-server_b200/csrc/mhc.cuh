// The mHC router's finish (layers.wgsl:97-132, `mhc_finish`) for one token: shared by
// the norm kernel (layers.cu) and the tile GEMV's fused-norm prologue (gemv_mma.cu).
#pragma once
#include "common.cuh"

namespace snl {

__device__ __forceinline__ float lse2(float a, float b) {
  const float mx = fmaxf(a, b);
  return mx + __logf(__expf(a - mx) + __expf(b - mx));
}

// mhc_finish (layers.wgsl:97-132) for one token, with the 8 router biases given.
// The Sinkhorn normalisation of the 2x2 mixing matrix runs on exp(logits - max), where
// each half-step is a sum, one reciprocal and two products (the same iterates as the
// log-domain form, without a log per step); if any row or column sum underflows, it is
// redone in the log domain.
__device__ __forceinline__ void mhc_coef_b(const float raw[9], const float bias[8], uint32_t d, uint32_t iterations,
                                           float* __restrict__ cb) {
  const float rinv = rsqrtf(raw[8] / (float)d + 1e-6f);
  float lg[8];
#pragma unroll
  for (int o = 0; o < 8; o++) lg[o] = fmaf(raw[o], rinv, bias[o]);
  const float mx = fmaxf(fmaxf(lg[4], lg[5]), fmaxf(lg[6], lg[7]));
  float A = __expf(lg[4] - mx), B = __expf(lg[5] - mx), C = __expf(lg[6] - mx), E = __expf(lg[7] - mx);
  bool ok = true;
  for (uint32_t it = 0; it < iterations; it++) {
    const float r0 = A + B, r1 = C + E;
    ok &= r0 > 1e-30f && r1 > 1e-30f;
    const float i0 = __fdividef(1.0f, r0), i1 = __fdividef(1.0f, r1);
    A *= i0;
    B *= i0;
    C *= i1;
    E *= i1;
    const float c0 = A + C, c1 = B + E;
    ok &= c0 > 1e-30f && c1 > 1e-30f;
    const float j0 = __fdividef(1.0f, c0), j1 = __fdividef(1.0f, c1);
    A *= j0;
    C *= j0;
    B *= j1;
    E *= j1;
  }
  if (!ok) {
    float a = lg[4], b = lg[5], c = lg[6], e = lg[7];
    for (uint32_t it = 0; it < iterations; it++) {
      const float r0 = lse2(a, b), r1 = lse2(c, e);
      a -= r0;
      b -= r0;
      c -= r1;
      e -= r1;
      const float c0 = lse2(a, c), c1 = lse2(b, e);
      a -= c0;
      c -= c0;
      b -= c1;
      e -= c1;
    }
    A = __expf(a);
    B = __expf(b);
    C = __expf(c);
    E = __expf(e);
  }
  cb[0] = 1.0f / (1.0f + __expf(-lg[0]));
  cb[1] = 1.0f / (1.0f + __expf(-lg[1]));
  cb[2] = 2.0f / (1.0f + __expf(-lg[2]));
  cb[3] = 2.0f / (1.0f + __expf(-lg[3]));
  cb[4] = A;
  cb[5] = B;
  cb[6] = C;
  cb[7] = E;
}


}  // namespace snl
