// Tensor-core GEMV interface: the packed x operand ("x planes") and the epilogues.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"
#include "tp.cuh"

namespace snl {

// x planes hold x / kXPlaneScale split as hi + lo fp16 halves: plane 2t = hi, plane 2t+1
// = lo for token row t, natural k order, plane_stride halves apart (multiple of 8).
constexpr float kXPlaneScale = 16.0f;

__device__ __forceinline__ void xplane_store(__half* planes, uint32_t plane_stride, uint32_t t, uint32_t i, float v) {
  const float vs = v * (1.0f / kXPlaneScale);
  const __half hi = __float2half_rn(vs);
  const __half lo = __float2half_rn(vs - __half2float(hi));
  planes[(uint64_t)(2 * t) * plane_stride + i] = hi;
  planes[(uint64_t)(2 * t + 1) * plane_stride + i] = lo;
}

// Epilogue of one output element (token t, output row n):
//   mode 0: y[y_off + t*y_stride + n_off + n] = v
//   mode 1: residual merge into x [t, 2H] (layers.wgsl:134-164 `merge` mode `merge_mode`),
//           then optionally copy stream 0 into stream 1 (`expand`, merge mode 3).
//   mode 2: SwiGLU of gate/up row pairs (tile GEMV only, see group_finish).
struct GemvArgs {
  uint32_t n, k;
  const __half* xplanes;
  uint32_t plane_stride;
  const uint8_t* wq;
  // epilogue
  int mode;
  float* y;
  uint32_t y_off, y_stride, n_off;
  float* resid;         // mode 1: x [t, 2H]
  const float* coef;    // mode 1, merge modes 1/2: coef [t, 8]
  uint32_t h;           // mode 1: hidden size H (= n)
  int merge_mode;       // 0, 1, 2
  int expand;           // also x1 = x0 afterwards
  // mode 1, optional: the mHC router of the next norm ([8, 2H] weights, then 8 biases).
  // Each 16-row group writes its partial sums over the merged (x0 | x1) to rpart (layout
  // at merge_partials).
  const float* rnext;
  float* rpart;
  // mode 2 (SwiGLU of a pair-repacked [gate; up] matrix): the x planes of act
  // (act_stride halves per plane) and, if y is set, act itself at y[t * y_stride + i].
  __half* act_planes;
  uint32_t act_stride;
  // mode 1 under tensor parallelism (tp.size > 1): the dot is this rank's partial over
  // its K shard; each finished group trades partials with the peers (exchange site
  // tp_site, flag slot = group) and merges the rank-ordered sum.
  TpComm tp;
  uint32_t tp_site;
  // mode 1, optional: the next norm's input as x planes of both residual streams, each
  // pre-multiplied by the next norm's weight (weight_one + nw[row]): plane 4t / 4t+1 =
  // hi / lo of stream 0 of token t, 4t+2 / 4t+3 of stream 1 (nstride halves apart).
  __half* nplanes;
  uint32_t nstride;
  const float* nw;
  float weight_one;
  // Fused norm (modes 0 and 2, M = 2 x tokens): the x planes are the two weighted streams
  // of each token (as written above); the GEMV finishes the norm from the producer's
  // partials: y = rinv * (pre0 * dot(stream 0) + pre1 * dot(stream 1)), where pre0/pre1
  // come from the mHC router (nrouter, or 1 and 0 without one) and rinv from the sums of
  // squares. Block 0 also writes the router coefficients to ncoef for the later merge.
  int fused_norm;
  const float* nrpart;   // [t][groups][kRpStride] partials of the producing GEMV
  uint32_t nparts;
  const float* nrouter;  // [8, 2H] weights then 8 biases, or nullptr
  float neps;
  uint32_t niter;
  float* ncoef;
};

// Partials of a residual-merging GEMV for the next norm, summed over a group's 16 rows:
// rpart[(t * groups + group) * kRpStride + o], o = 0..7 the next mHC router's dots (when
// rnext), 8 = sum x0^2, 9 = sum x1^2, 10 = sum x0 x1 of the merged streams.

__device__ __forceinline__ void xplane4_store(__half* planes, uint32_t stride, uint32_t t, uint32_t i, float v0,
                                              float v1) {
  const float a = v0 * (1.0f / kXPlaneScale), b = v1 * (1.0f / kXPlaneScale);
  const __half ah = __float2half_rn(a), bh = __float2half_rn(b);
  planes[(uint64_t)(4 * t) * stride + i] = ah;
  planes[(uint64_t)(4 * t + 1) * stride + i] = __float2half_rn(a - __half2float(ah));
  planes[(uint64_t)(4 * t + 2) * stride + i] = bh;
  planes[(uint64_t)(4 * t + 3) * stride + i] = __float2half_rn(b - __half2float(bh));
}

// Called by all 32 lanes of a warp; lanes 16*j + r hold row r of token tt (live or not).
__device__ __forceinline__ void merge_partials(const GemvArgs& a, int tt, uint32_t row, bool live, float2 nx,
                                               uint64_t slot, bool writer) {
  if (a.mode != 1) return;
  if (a.nplanes && live) {
    const float w1 = a.weight_one + __ldg(a.nw + row);
    xplane4_store(a.nplanes, a.nstride, tt, row, nx.x * w1, nx.y * w1);
  }
  // rpart holds one slot per 16-row group of the hidden dimension: only a residual merge
  // (n = hidden) whose partials a norm consumes writes it.
  if (!a.rpart || !(a.rnext || a.nplanes)) return;
  float rs[11];
  const uint32_t d = 2 * a.h;
#pragma unroll
  for (int o = 0; o < 8; o++)
    rs[o] = live && a.rnext
                ? fmaf(__ldg(a.rnext + (uint64_t)o * d + row), nx.x, __ldg(a.rnext + (uint64_t)o * d + a.h + row) * nx.y)
                : 0.f;
  rs[8] = live ? nx.x * nx.x : 0.f;
  rs[9] = live ? nx.y * nx.y : 0.f;
  rs[10] = live ? nx.x * nx.y : 0.f;
#pragma unroll
  for (int o = 0; o < 11; o++) {
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) rs[o] += __shfl_xor_sync(0xffffffffu, rs[o], off);
  }
  if (writer) {
#pragma unroll
    for (int o = 0; o < 11; o++) a.rpart[slot * kRpStride + o] = rs[o];
  }
}

// Returns the merged (x0, x1) of element n (mode 1), for the router partials.
__device__ __forceinline__ float2 gemv_epilogue(const GemvArgs& a, uint32_t t, uint32_t n, float v) {
  if (a.mode == 0) {
    a.y[a.y_off + (uint64_t)t * a.y_stride + a.n_off + n] = v;
    return make_float2(0.f, 0.f);
  }
  float* x0 = a.resid + (uint64_t)t * 2 * a.h + n;
  float* x1 = x0 + a.h;
  float n0, n1 = *x1;
  if (a.merge_mode == 0) {
    n0 = *x0 + v;
    *x0 = n0;
  } else {
    const float* c = a.coef + t * 8;
    const float a0 = *x0, a1 = n1;
    n0 = fmaf(c[4], a0, fmaf(c[5], a1, c[2] * v));
    const float m1 = fmaf(c[6], a0, fmaf(c[7], a1, c[3] * v));
    if (a.merge_mode == 2) {
      n0 = 0.5f * (n0 + m1);
      *x0 = n0;
    } else {
      *x0 = n0;
      *x1 = m1;
      n1 = m1;
    }
  }
  if (a.expand) {
    *x1 = n0;
    n1 = n0;
  }
  return make_float2(n0, n1);
}

inline GemvArgs gemv_args_plain(const snl_mat_p& p, const __half* planes, uint32_t plane_stride, const void* wq, float* y) {
  GemvArgs a{};
  a.n = p.n;
  a.k = p.k;
  a.xplanes = planes;
  a.plane_stride = plane_stride;
  a.wq = static_cast<const uint8_t*>(wq);
  a.mode = 0;
  a.y = y;
  a.y_off = p.y_off;
  a.y_stride = p.y_stride;
  a.n_off = p.n_off;
  return a;
}

int launch_gemv_mma(int dtype, const GemvArgs& a, uint32_t m, const void* ws, int scale_f16, cudaStream_t s);
// Tile layout (see gemv_mma.cu): sizes, device repack from the reference layout, GEMV.
void tile_sizes(int dtype, uint32_t n, uint32_t k, size_t* tile_bytes, size_t* scale_floats);
// *exact = every one of the count f32 scales is an fp16 number (waits; dflag: one device
// int of scratch).
int scales_fp16_exact(const float* s, uint64_t count, int* dflag, bool* exact, cudaStream_t st);
// ts: scale_floats fp16 (ts_f16) or f32 values.
int launch_repack_tiles(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, void* tiles, void* ts,
                        int ts_f16, cudaStream_t st, uint32_t pair_half = 0);
int launch_gemv_tile(int dtype, const GemvArgs& a, uint32_t m, const void* tiles, const void* ts, int ts_f16,
                     cudaStream_t s);
int launch_xpack(const float* x, uint32_t m, uint32_t k, uint32_t x_stride, __half* planes, uint32_t plane_stride,
                 cudaStream_t s);

}  // namespace snl
