// Norm / mHC / residual / SwiGLU kernels (layers.wgsl), greedy argmax
// (sampler.rs:169-177), the device-side embedding dequant (engine.rs:777-790,
// weights.rs:155-162) and the seeded synthetic-weight generators.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"
#include "mhc.cuh"
#include "synth.h"
#include "tp.cuh"

namespace snl {
namespace {

// branch_norm (layers.wgsl:49-76): one CTA per output row.
// Generic form (any h): strided loops.
__global__ void __launch_bounds__(256) branch_norm_loop_kernel(StepRef sr, snl_layer_p p, const float* __restrict__ x,
                                                               const float* __restrict__ coef, const float* __restrict__ w,
                                                               float* __restrict__ out, XOut xo) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sh[32];
  const snl_step_u st = load_step(sr);
  const uint32_t g = blockIdx.x;
  const uint32_t m = g + (p.last_row == 1 ? st.m - 1 : 0);
  const uint64_t base = (uint64_t)m * (p.x_stride != 0 ? p.x_stride : 2 * p.h);
  float pre0 = 1.f, pre1 = 0.f;
  if (p.mode == 1) {
    pre0 = coef[m * 8];
    pre1 = coef[m * 8 + 1];
  }
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < p.h; i += blockDim.x) {
    float v = pre0 * x[base + i];
    if (p.mode == 1) v = fmaf(pre1, x[base + p.h + i], v);
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum(ss, sh);
  const float rinv = rsqrtf(total / (float)p.h + p.eps);
  const uint64_t ob = (uint64_t)g * p.h;
  for (uint32_t i = threadIdx.x; i < p.h; i += blockDim.x) {
    float v = pre0 * x[base + i];
    if (p.mode == 1) v = fmaf(pre1, x[base + p.h + i], v);
    const float o = v * rinv * (p.weight_one + w[i]);
    out[ob + i] = o;
    if (xo.planes) xout_store(xo, g, i, o);
  }
}


// Router finished inside the norm: rpart holds nparts partial router sums per token (from
// the GEMV that merged the residual); they are summed in a fixed order, the Sinkhorn
// step runs on thread 0, and coef[m] is written for the later merge.
struct NormRouter {
  const float* rpart = nullptr;
  uint32_t nparts = 0;
  const float* router = nullptr;  // [8, 2H] weights then 8 biases
  float* coef_out = nullptr;
};

// Register form (h % 4 == 0, h <= 1024 * VPT). Every load of the CTA (both streams of
// the row, the norm weight, the router partials and biases) is issued first, so the
// row costs one memory latency; the router sums take one block reduction (fixed warp
// order), the Sinkhorn step runs on thread 0, and the mixed row one more reduction.
template <int VPT>
__global__ void __launch_bounds__(256) branch_norm_kernel(StepRef sr, snl_layer_p p, const float* __restrict__ x,
                                                          const float* __restrict__ coef, const float* __restrict__ w,
                                                          float* __restrict__ out, XOut xo, NormRouter nr) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sh[32];
  __shared__ float rsh[8][9];
  __shared__ float pre_sh[2];
  const uint32_t g = blockIdx.x;
  const uint32_t m = p.last_row == 1 ? g + load_step(sr).m - 1 : g;
  const uint64_t base = (uint64_t)m * (p.x_stride != 0 ? p.x_stride : 2 * p.h);
  const uint32_t h4 = p.h / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x + base);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const bool mix = p.mode == 1;
  const bool route = mix && nr.rpart;
  float4 v[VPT], b[VPT], ww[VPT];
#pragma unroll
  for (int c = 0; c < VPT; c++) {
    const uint32_t i4 = threadIdx.x + c * 256;
    const bool in = i4 < h4;
    v[c] = in ? x4[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    b[c] = in && mix ? x4[h4 + i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    ww[c] = in ? w4[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float pre0 = 1.f, pre1 = 0.f;
  if (route) {
    float bias[8];
    if (threadIdx.x == 0) {
#pragma unroll
      for (int o = 0; o < 8; o++) bias[o] = nr.router[(uint64_t)16 * p.h + o];
    }
    float acc[9];
#pragma unroll
    for (int o = 0; o < 9; o++) acc[o] = 0.f;
    for (uint32_t i = threadIdx.x; i < nr.nparts; i += blockDim.x) {
      const float* rp = nr.rpart + ((uint64_t)m * nr.nparts + i) * kRpStride;
#pragma unroll
      for (int o = 0; o < 8; o++) acc[o] += rp[o];
      acc[8] += rp[8] + rp[9];  // sum over both streams of x^2
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 0; o < 9; o++) acc[o] = warp_sum(acc[o]);
    if (lane == 0) {
#pragma unroll
      for (int o = 0; o < 9; o++) rsh[wid][o] = acc[o];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot[9];
#pragma unroll
      for (int o = 0; o < 9; o++) {
        float t = 0.f;
        for (int k = 0; k < 8; k++) t += rsh[k][o];
        tot[o] = t;
      }
      float* cb = nr.coef_out + m * 8;
      mhc_coef_b(tot, bias, 2 * p.h, p.iterations, cb);
      pre_sh[0] = cb[0];
      pre_sh[1] = cb[1];
    }
    __syncthreads();
    pre0 = pre_sh[0];
    pre1 = pre_sh[1];
  } else if (mix) {
    pre0 = coef[m * 8];
    pre1 = coef[m * 8 + 1];
  }
  if (mix) {
#pragma unroll
    for (int c = 0; c < VPT; c++) {
      v[c].x = fmaf(pre1, b[c].x, pre0 * v[c].x);
      v[c].y = fmaf(pre1, b[c].y, pre0 * v[c].y);
      v[c].z = fmaf(pre1, b[c].z, pre0 * v[c].z);
      v[c].w = fmaf(pre1, b[c].w, pre0 * v[c].w);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < VPT; c++) ss += v[c].x * v[c].x + v[c].y * v[c].y + v[c].z * v[c].z + v[c].w * v[c].w;
  const float total = block_sum(ss, sh);
  const float rinv = rsqrtf(total / (float)p.h + p.eps);
  float4* o4 = reinterpret_cast<float4*>(out + (uint64_t)g * p.h);
#pragma unroll
  for (int c = 0; c < VPT; c++) {
    const uint32_t i4 = threadIdx.x + c * 256;
    if (i4 >= h4) break;
    float4 o;
    o.x = v[c].x * rinv * (p.weight_one + ww[c].x);
    o.y = v[c].y * rinv * (p.weight_one + ww[c].y);
    o.z = v[c].z * rinv * (p.weight_one + ww[c].z);
    o.w = v[c].w * rinv * (p.weight_one + ww[c].w);
    o4[i4] = o;
    if (xo.planes) {
      xout_store(xo, g, 4 * i4, o.x);
      xout_store(xo, g, 4 * i4 + 1, o.y);
      xout_store(xo, g, 4 * i4 + 2, o.z);
      xout_store(xo, g, 4 * i4 + 3, o.w);
    }
  }
}

// The 9 router sums of mhc_dots (layers.wgsl:78-95) for one token, in one pass
// over its two streams.
__device__ __forceinline__ void mhc_sums(const float* __restrict__ x, const float* __restrict__ w, uint32_t d,
                                         float out9[9], float* sh) {
  float acc[9];
#pragma unroll
  for (int o = 0; o < 9; o++) acc[o] = 0.f;
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = x[i];
#pragma unroll
    for (int o = 0; o < 8; o++) acc[o] = fmaf(__ldg(w + (uint64_t)o * d + i), v, acc[o]);
    acc[8] = fmaf(v, v, acc[8]);
  }
#pragma unroll
  for (int o = 0; o < 9; o++) out9[o] = block_sum(acc[o], sh);
}

__device__ __forceinline__ void mhc_coef(const float raw[9], const float* __restrict__ w, uint32_t d,
                                         uint32_t iterations, float* __restrict__ cb) {
  float bias[8];
#pragma unroll
  for (int o = 0; o < 8; o++) bias[o] = w[(uint64_t)8 * d + o];
  mhc_coef_b(raw, bias, d, iterations, cb);
}

__global__ void __launch_bounds__(256) mhc_dots_kernel(snl_layer_p p, const float* __restrict__ x,
                                                       const float* __restrict__ w, float* __restrict__ raw) {
  __shared__ float sh[32];
  const uint32_t m = blockIdx.x, d = 2 * p.h;
  float r[9];
  mhc_sums(x + (uint64_t)m * d, w, d, r, sh);
  if (threadIdx.x == 0)
    for (int o = 0; o < 9; o++) raw[m * 9 + o] = r[o];
}

__global__ void mhc_finish_kernel(StepRef sr, snl_layer_p p, const float* __restrict__ raw,
                                  const float* __restrict__ w, float* __restrict__ coef) {
  const snl_step_u st = load_step(sr);
  const uint32_t m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= st.m) return;
  float r[9];
  for (int o = 0; o < 9; o++) r[o] = raw[m * 9 + o];
  mhc_coef(r, w, 2 * p.h, p.iterations, coef + m * 8);
}

// Engine-side mHC router in two launches that use many SMs: slice s of the 2H inputs
// of token m -> part[(m * slices + s) * 9 + o]; then one warp per token sums the
// slices and finishes the Sinkhorn step (mhc_coef).
constexpr int kMhcSlices = 4;
// The 9 router sums (8 dots + sum of squares) of kMhcTok tokens over slice `blockIdx.x`
// of the 2H inputs: each thread loads the router weights of its elements once and
// applies them to the block's 8 tokens over the whole slice before any reduction; the
// 72 sums then take one warp-shuffle and one shared-memory pass per CTA.
constexpr uint32_t kMhcTok = 8;
__global__ void __launch_bounds__(256) mhc_part_kernel(snl_layer_p p, uint32_t m_rows, const float* __restrict__ x,
                                                       const float* __restrict__ w, float* __restrict__ part) {
  __shared__ float red[8][kMhcTok * 9];
  const uint32_t sl = blockIdx.x, m0 = blockIdx.y * kMhcTok, d = 2 * p.h;
  const uint32_t len = d / kMhcSlices, i0 = sl * len;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nt = min(kMhcTok, m_rows - m0);
  float acc[kMhcTok][9];
#pragma unroll
  for (uint32_t t = 0; t < kMhcTok; t++)
#pragma unroll
    for (int o = 0; o < 9; o++) acc[t][o] = 0.f;
  for (uint32_t i = i0 + threadIdx.x; i < i0 + len; i += blockDim.x) {
    float wv[8];
#pragma unroll
    for (int o = 0; o < 8; o++) wv[o] = __ldg(w + (uint64_t)o * d + i);
    float xv[kMhcTok];
#pragma unroll
    for (uint32_t t = 0; t < kMhcTok; t++) xv[t] = t < nt ? x[(uint64_t)(m0 + t) * d + i] : 0.f;
#pragma unroll
    for (uint32_t t = 0; t < kMhcTok; t++) {
#pragma unroll
      for (int o = 0; o < 8; o++) acc[t][o] = fmaf(wv[o], xv[t], acc[t][o]);
      acc[t][8] = fmaf(xv[t], xv[t], acc[t][8]);
    }
  }
#pragma unroll
  for (uint32_t t = 0; t < kMhcTok; t++)
#pragma unroll
    for (int o = 0; o < 9; o++) {
      const float v = warp_sum(acc[t][o]);
      if (lane == 0) red[warp][t * 9 + o] = v;
    }
  __syncthreads();
  if (threadIdx.x < kMhcTok * 9) {
    const uint32_t t = threadIdx.x / 9, o = threadIdx.x % 9;
    float v = 0.f;
#pragma unroll
    for (int wi = 0; wi < 8; wi++) v += red[wi][threadIdx.x];
    if (t < nt) part[((uint64_t)(m0 + t) * kMhcSlices + sl) * 9 + o] = v;
  }
}
__global__ void mhc_coef_kernel(snl_layer_p p, uint32_t m_rows, const float* __restrict__ part,
                                const float* __restrict__ w, float* __restrict__ coef) {
  const uint32_t m = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (m >= m_rows) return;
  float r[9];
#pragma unroll
  for (int o = 0; o < 9; o++) {
    float v = lane < kMhcSlices ? part[((uint64_t)m * kMhcSlices + lane) * 9 + o] : 0.f;
    r[o] = warp_sum(v);
  }
  if (lane == 0) mhc_coef(r, w, 2 * p.h, p.iterations, coef + m * 8);
}

// merge (layers.wgsl:134-164).
// Row blockIdx.y, four consecutive elements per thread (H is a multiple of 4).
__global__ void merge_kernel(snl_layer_p p, uint32_t m_rows, float* __restrict__ x, const float* __restrict__ coef,
                             const float* __restrict__ br) {
  pdl_trigger();
  pdl_wait();
  const uint32_t m = blockIdx.y, i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (m >= m_rows || i >= p.h) return;
  float4* p0 = reinterpret_cast<float4*>(x + (uint64_t)m * 2 * p.h + i);
  float4* p1 = reinterpret_cast<float4*>(x + (uint64_t)m * 2 * p.h + p.h + i);
  if (p.mode == 3) {
    *p1 = *p0;
    return;
  }
  const float4 bv = *reinterpret_cast<const float4*>(br + (uint64_t)m * p.h + i);
  float4 a0 = *p0;
  if (p.mode == 0) {
    a0.x += bv.x;
    a0.y += bv.y;
    a0.z += bv.z;
    a0.w += bv.w;
    *p0 = a0;
    return;
  }
  const float* c = coef + m * 8;
  const float4 a1 = *p1;
  const float xs0[4] = {a0.x, a0.y, a0.z, a0.w}, xs1[4] = {a1.x, a1.y, a1.z, a1.w}, bs[4] = {bv.x, bv.y, bv.z, bv.w};
  float n0[4], n1[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    n0[e] = fmaf(c[4], xs0[e], fmaf(c[5], xs1[e], c[2] * bs[e]));
    n1[e] = fmaf(c[6], xs0[e], fmaf(c[7], xs1[e], c[3] * bs[e]));
  }
  if (p.mode == 2) {
    *p0 = make_float4(0.5f * (n0[0] + n1[0]), 0.5f * (n0[1] + n1[1]), 0.5f * (n0[2] + n1[2]), 0.5f * (n0[3] + n1[3]));
  } else {
    *p0 = make_float4(n0[0], n0[1], n0[2], n0[3]);
    *p1 = make_float4(n1[0], n1[1], n1[2], n1[3]);
  }
}

// swiglu (layers.wgsl:166-175).
// Row blockIdx.y, four consecutive outputs per thread (the FFN width is a multiple of 4).
__global__ void swiglu_kernel(snl_layer_p p, uint32_t m_rows, const float* __restrict__ gu, float* __restrict__ act,
                              XOut xo) {
  pdl_trigger();
  pdl_wait();
  const uint32_t m = blockIdx.y, i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (m >= m_rows || i >= p.inter) return;
  const float4 g = *reinterpret_cast<const float4*>(gu + (uint64_t)m * 2 * p.inter + i);
  const float4 u = *reinterpret_cast<const float4*>(gu + (uint64_t)m * 2 * p.inter + p.inter + i);
  const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {u.x, u.y, u.z, u.w};
  float a[4];
#pragma unroll
  for (int e = 0; e < 4; e++) a[e] = gs[e] / (1.0f + __expf(-gs[e])) * us[e];
  *reinterpret_cast<float4*>(act + (uint64_t)m * p.inter + i) = make_float4(a[0], a[1], a[2], a[3]);
  if (xo.planes)
#pragma unroll
    for (int e = 0; e < 4; e++) xout_store(xo, m, i + e, a[e]);
}

// Greedy argmax, two passes. Key = (ordered float bits << 32) | ~index so that the
// largest key is the largest value with the smallest index (the first maximum, as
// sampler.rs:169-177, which starts at best = 0 and moves only on `x > v[best]`). So:
//   - -0.0 and +0.0 compare equal there and take the key of +0.0 (the first one wins);
//   - NaN never wins, except at index 0 of the row: with v[0] NaN, `x > v[0]` is false
//     for every x and the scan returns 0, so that element gets the largest key.
// `row_start` says whether index 0 of this scan is index 0 of the whole row (false for
// the vocabulary shards of tensor-parallel ranks other than 0).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t i, bool row_start) {
  uint32_t b = __float_as_uint(v);
  if (v != v) {
    if (row_start && i == 0) return ~0ull;
    b = 0xFF800000u;  // NaN -> -inf
  }
  if (v == 0.f) b = 0u;  // -0.0 -> +0.0
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(~i);
}

constexpr int kArgBlocks = 128;
__global__ void __launch_bounds__(512) argmax_pass1(const float* __restrict__ v, uint32_t n,
                                                    unsigned long long* __restrict__ part, int row_start) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.y;
  const float* r = v + (uint64_t)row * n;
  unsigned long long best = 0;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(__ldg(r + i), i, row_start != 0);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  __shared__ unsigned long long sh[16];
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = sh[w] > best ? sh[w] : best;
    part[(uint64_t)row * gridDim.x + blockIdx.x] = best;
  }
}
__global__ void argmax_pass2(const unsigned long long* __restrict__ part, uint32_t nparts, uint32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.x;
  unsigned long long best = 0;
  for (uint32_t i = threadIdx.x; i < nparts; i += 32) {
    const unsigned long long k = part[(uint64_t)row * nparts + i];
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if (threadIdx.x == 0) out[row] = ~(uint32_t)(best & 0xFFFFFFFFull);
}

// Tensor-parallel pass 2: the row's best key over this rank's vocabulary shard, rebased
// to the global index, is pushed into every rank's memory as two tagged words; each rank
// then takes the largest of all ranks' keys, so all agree on the token (first index on
// ties). key_set selects one of the key slot sets (kTpKeySets): each exchange kind has
// its own, so a slot is rewritten only after an exchange that every peer joined after
// reading it.
__global__ void argmax_tp_pass2(const unsigned long long* __restrict__ part, uint32_t nparts, uint32_t vl, TpComm c,
                                uint32_t site, uint32_t key_set, uint32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const uint32_t row = blockIdx.x;
  const uint32_t tag = (uint32_t)tp_epoch(c, site);
  unsigned long long best = 0;
  for (uint32_t i = threadIdx.x; i < nparts; i += 32) {
    const unsigned long long k = part[(uint64_t)row * nparts + i];
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
    best = t > best ? t : best;
  }
  if (threadIdx.x == 0) {
    const uint32_t gidx = (uint32_t)c.rank * vl + ~(uint32_t)(best & 0xFFFFFFFFull);
    const uint32_t ord = (uint32_t)(best >> 32);
    const unsigned long long key = ((unsigned long long)ord << 32) | (unsigned long long)(~gidx);
    for (int q = 0; q < c.size; q++) {
      if (q == c.rank) continue;
      unsigned long long* slot = c.llkeys[q] + (((uint64_t)key_set * kTpKeyRows + row) * kTpMax + c.rank) * 2;
      st_relaxed_sys_u64(slot, ll_word(tag, ord));
      st_relaxed_sys_u64(slot + 1, ll_word(tag, ~gidx));
    }
    unsigned long long g = key;
    for (int q = 0; q < c.size; q++) {
      if (q == c.rank) continue;
      const unsigned long long* slot = c.llkeys[c.rank] + (((uint64_t)key_set * kTpKeyRows + row) * kTpMax + q) * 2;
      const uint32_t o = ll_wait(c, slot, tag), ni = ll_wait(c, slot + 1, tag);
      const unsigned long long k = ((unsigned long long)o << 32) | ni;
      g = k > g ? k : g;
    }
    out[row] = ~(uint32_t)(g & 0xFFFFFFFFull);
  }
}

// Embedding rows (engine.rs:777-790): stream 0 = q * s of the token's Q8_0 row,
// stream 1 = 0. Ids >= vocab raise err_flag and write zeros (the host checks first).
__global__ void embed_kernel(const uint32_t* __restrict__ toks, uint32_t h, uint32_t vocab,
                             const int8_t* __restrict__ q, const float* __restrict__ s, float* __restrict__ x,
                             int* __restrict__ err, unsigned long long* __restrict__ step_ctr) {
  pdl_trigger();
  pdl_wait();
  const uint32_t m = blockIdx.y;
  // The embedding is the first kernel of every step: it advances the step counter that
  // numbers the step's tensor-parallel exchanges.
  if (step_ctr && m == 0 && blockIdx.x == 0 && threadIdx.x == 0) *step_ctr += 1;
  const uint32_t t = toks[m];
  const bool ok = t < vocab;
  if (!ok && threadIdx.x == 0 && err) *err = 1;
  // CTA x covers elements [1024 x, 1024 x + 1024) of the row, four per thread.
  const uint32_t i = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= h) return;
  float* x0 = x + (uint64_t)m * 2 * h;
  if (h % 4 == 0) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
      const uint64_t e = (uint64_t)t * h + i;
      const char4 c = *reinterpret_cast<const char4*>(q + e);
      const float sc = s[e / 32];
      v = make_float4((float)c.x * sc, (float)c.y * sc, (float)c.z * sc, (float)c.w * sc);
    }
    *reinterpret_cast<float4*>(x0 + i) = v;
    *reinterpret_cast<float4*>(x0 + h + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  for (uint32_t j = i; j < min(h, i + 4); j++) {
    x0[j] = ok ? (float)q[(uint64_t)t * h + j] * s[((uint64_t)t * h + j) / 32] : 0.f;
    x0[h + j] = 0.f;
  }
}

__global__ void gen_q8_kernel(uint64_t kq, uint64_t ks, uint64_t n, int8_t* __restrict__ q, float* __restrict__ s) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 4; i += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) w |= (uint32_t)(uint8_t)snl_q8(snl_draw(kq, i * 4 + e)) << (8 * e);
    reinterpret_cast<uint32_t*>(q)[i] = w;
    if ((i & 7) == 0) s[i / 8] = snl_q8_scale(snl_draw(ks, i / 8));
  }
}
__global__ void gen_q4_kernel(uint64_t kq, uint64_t ks, uint64_t n, uint32_t* __restrict__ q, float* __restrict__ s) {
  for (uint64_t wi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; wi < n / 8; wi += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t w = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) w |= snl_nib(snl_draw(kq, wi * 8 + e)) << (4 * e);
    q[wi] = w;
    if ((wi & 3) == 0) s[wi / 4] = snl_q4_scale(snl_draw(ks, wi / 4));
  }
}
__global__ void gen_f32_kernel(uint64_t k, uint64_t n, float mult, float offset, float* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = snl_param(snl_draw(k, i), mult, offset);
}

}  // namespace

int launch_branch_norm_router(StepRef st, const snl_layer_p& p, const float* x, float* coef, const float* w, float* out,
                              uint32_t n_groups, cudaStream_t s, XOut xo, const float* rpart, uint32_t nparts,
                              const float* router) {
  if (n_groups == 0) return SNL_OK;
  const uint32_t stride = p.x_stride != 0 ? p.x_stride : 2 * p.h;
  const bool vec = p.h % 4 == 0 && stride % 4 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 &&
                   ((uintptr_t)out % 16) == 0;
  const uint32_t vpt = (p.h / 4 + 255) / 256;
  if (!vec || vpt > 8 || p.mode != 1) return fail(SNL_E_INVALID, "branch_norm_router: unsupported shape");
  NormRouter nr;
  nr.rpart = rpart;
  nr.nparts = nparts;
  nr.router = router;
  nr.coef_out = coef;
  if (vpt <= 1) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<1>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, nr);
  else if (vpt <= 2) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<2>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, nr);
  else if (vpt <= 4) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<4>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, nr);
  else SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<8>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, nr);
  return SNL_OK;
}

int launch_branch_norm(StepRef st, const snl_layer_p& p, const float* x, const float* coef, const float* w, float* out,
                       uint32_t n_groups, cudaStream_t s, XOut xo) {
  if (n_groups == 0) return SNL_OK;
  const uint32_t stride = p.x_stride != 0 ? p.x_stride : 2 * p.h;
  const bool vec = p.h % 4 == 0 && stride % 4 == 0 && ((uintptr_t)x % 16) == 0 && ((uintptr_t)w % 16) == 0 &&
                   ((uintptr_t)out % 16) == 0;
  const uint32_t vpt = (p.h / 4 + 255) / 256;
  if (vec && vpt <= 1) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<1>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, NormRouter());
  else if (vec && vpt <= 2) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<2>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, NormRouter());
  else if (vec && vpt <= 4) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<4>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, NormRouter());
  else if (vec && vpt <= 8) SNL_PDL_LAUNCH("branch_norm_kernel", branch_norm_kernel<8>, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo, NormRouter());
  else SNL_PDL_LAUNCH("branch_norm_loop_kernel", branch_norm_loop_kernel, dim3(n_groups), dim3(256), (size_t)(0), s, st, p, x, coef, w, out, xo);
  return SNL_OK;
}
int launch_mhc_dots(StepRef st, const snl_layer_p& p, const float* x, const float* w, float* raw, uint32_t m,
                    cudaStream_t s) {
  (void)st;
  if (m == 0) return SNL_OK;
  mhc_dots_kernel<<<m, 256, 0, s>>>(p, x, w, raw);
  SNL_LAUNCH_CHECK("mhc_dots");
  return SNL_OK;
}
int launch_mhc_finish(StepRef st, const snl_layer_p& p, const float* raw, const float* w, float* coef, uint32_t m,
                      cudaStream_t s) {
  if (m == 0) return SNL_OK;
  mhc_finish_kernel<<<(m + 127) / 128, 128, 0, s>>>(st, p, raw, w, coef);
  SNL_LAUNCH_CHECK("mhc_finish");
  return SNL_OK;
}
int launch_mhc_router(const snl_layer_p& p, const float* x, const float* w, float* part, float* coef, uint32_t m,
                      cudaStream_t s) {
  if (m == 0) return SNL_OK;
  if ((2 * p.h) % kMhcSlices) return fail(SNL_E_INVALID, "mhc: 2H must divide into slices");
  mhc_part_kernel<<<dim3(kMhcSlices, (m + kMhcTok - 1) / kMhcTok), 256, 0, s>>>(p, m, x, w, part);
  SNL_LAUNCH_CHECK("mhc_part");
  mhc_coef_kernel<<<(m + 3) / 4, 128, 0, s>>>(p, m, part, w, coef);
  SNL_LAUNCH_CHECK("mhc_coef");
  return SNL_OK;
}

int launch_merge(StepRef st, const snl_layer_p& p, float* x, const float* coef, const float* br, uint32_t m,
                 cudaStream_t s) {
  (void)st;
  const uint64_t n = (uint64_t)m * p.h;
  if (n == 0) return SNL_OK;
  if (p.h % 4 || ((uintptr_t)x | (uintptr_t)br) % 16) return fail(SNL_E_INVALID, "merge: H must be a multiple of 4 and x, branch 16-byte aligned");
  SNL_PDL_LAUNCH("merge_kernel", merge_kernel, dim3((p.h / 4 + 255) / 256, m), dim3(256), (size_t)(0), s, p, m, x, coef, br);
  return SNL_OK;
}
int launch_swiglu(StepRef st, const snl_layer_p& p, const float* gu, float* act, uint32_t m, cudaStream_t s, XOut xo) {
  (void)st;
  const uint64_t n = (uint64_t)m * p.inter;
  if (n == 0) return SNL_OK;
  if (p.inter % 4 || ((uintptr_t)gu | (uintptr_t)act) % 16)
    return fail(SNL_E_INVALID, "swiglu: the FFN width must be a multiple of 4 and the buffers 16-byte aligned");
  SNL_PDL_LAUNCH("swiglu_kernel", swiglu_kernel, dim3((p.inter / 4 + 255) / 256, m), dim3(256), (size_t)(0), s, p, m, gu, act, xo);
  return SNL_OK;
}

// Per-device scratch of the two-pass argmax: rows * kArgBlocks keys, grown on demand.
static unsigned long long* argmax_scratch(uint32_t rows) {
  static thread_local unsigned long long* buf[64] = {nullptr};
  static thread_local uint32_t cap[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (cap[dev] < rows) {
    if (buf[dev]) cudaFree(buf[dev]);
    buf[dev] = nullptr;
    if (cudaMalloc(&buf[dev], sizeof(unsigned long long) * kArgBlocks * rows) != cudaSuccess) {
      cap[dev] = 0;
      return nullptr;
    }
    cap[dev] = rows;
  }
  return buf[dev];
}

int launch_argmax_with(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, unsigned long long* part,
                       cudaStream_t s) {
  if (rows == 0) return SNL_OK;
  SNL_PDL_LAUNCH("argmax_pass1", argmax_pass1, dim3(dim3(kArgBlocks, rows)), dim3(512), (size_t)(0), s, logits, n, part,
                 1);
  SNL_PDL_LAUNCH("argmax_pass2", argmax_pass2, dim3(rows), dim3(32), (size_t)(0), s, part, kArgBlocks, out_idx);
  return SNL_OK;
}

int launch_argmax_tp(const float* logits, uint32_t rows, uint32_t vl, uint32_t* out_idx, unsigned long long* part,
                     const TpComm& c, uint32_t site, cudaStream_t s, uint32_t key_set) {
  if (rows == 0) return SNL_OK;
  if (rows > kTpKeyRows || key_set >= kTpKeySets) return fail(SNL_E_RANGE, "argmax_tp: rows or key set out of range");
  SNL_PDL_LAUNCH("argmax_pass1", argmax_pass1, dim3(dim3(kArgBlocks, rows)), dim3(512), (size_t)(0), s, logits, vl, part,
                 c.rank == 0 ? 1 : 0);
  SNL_PDL_LAUNCH("argmax_tp_pass2", argmax_tp_pass2, dim3(rows), dim3(32), (size_t)(0), s, part, kArgBlocks, vl, c, site,
                 key_set, out_idx);
  return SNL_OK;
}

int launch_argmax(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, cudaStream_t s) {
  unsigned long long* part = argmax_scratch(rows);
  if (!part) return fail(SNL_E_OOM, "argmax: scratch allocation failed");
  return launch_argmax_with(logits, rows, n, out_idx, part, s);
}

int launch_embed(const uint32_t* tokens, uint32_t m, const int8_t* q, const float* s_, uint32_t h, uint32_t vocab,
                 float* x, int* err_flag, cudaStream_t s, unsigned long long* step_ctr) {
  if (m == 0) return SNL_OK;
  SNL_PDL_LAUNCH("embed_kernel", embed_kernel, dim3((h + 1023) / 1024, m), dim3(256), (size_t)(0), s, tokens, h, vocab, q,
                 s_, x, err_flag, step_ctr);
  return SNL_OK;
}

int launch_gen_quant(uint64_t seed, const char* name, int dtype, size_t rows, size_t cols, void* q, float* s,
                     cudaStream_t st) {
  const uint64_t nh = snl_fnv1a(name);
  const uint64_t kq = snl_key(seed, nh, 0), ks = snl_key(seed, nh, 1);
  const uint64_t n = (uint64_t)rows * cols;
  if (n % 32) return fail(SNL_E_INVALID, "gen_quant: size must be a multiple of 32");
  const unsigned grid = (unsigned)std::min<uint64_t>((n / 8 + 255) / 256, 148 * 64);
  if (dtype == SNL_Q8_0) gen_q8_kernel<<<grid, 256, 0, st>>>(kq, ks, n, (int8_t*)q, s);
  else gen_q4_kernel<<<grid, 256, 0, st>>>(kq, ks, n, (uint32_t*)q, s);
  SNL_LAUNCH_CHECK("gen_quant");
  return SNL_OK;
}

int launch_gen_f32(uint64_t seed, const char* name, uint32_t sub, size_t n, float mult, float offset, float* out,
                   cudaStream_t st) {
  const uint64_t k = snl_key(seed, snl_fnv1a(name), sub);
  if (n == 0) return SNL_OK;
  const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, 148 * 16);
  gen_f32_kernel<<<grid, 256, 0, st>>>(k, n, mult, offset, out);
  SNL_LAUNCH_CHECK("gen_f32");
  return SNL_OK;
}

}  // namespace snl

// ---- kernel-level C ABI (layers.wgsl entry points) ----

extern "C" int snl_branch_norm(const snl_step_u* step, const snl_layer_p* p, const float* x, const float* coef,
                               const float* w, float* out, uint32_t n_groups, void* stream) {
  if (!step || !p || !x || !w || !out) return snl::fail(SNL_E_INVALID, "snl_branch_norm: null argument");
  if (p->mode == 1 && !coef) return snl::fail(SNL_E_INVALID, "snl_branch_norm: mode 1 needs coef");
  return snl::launch_branch_norm(snl::step_val(*step), *p, x, coef, w, out, n_groups, (cudaStream_t)stream);
}
extern "C" int snl_mhc_dots(const snl_step_u* step, const snl_layer_p* p, const float* x, const float* w, float* raw,
                            void* stream) {
  if (!step || !p || !x || !w || !raw) return snl::fail(SNL_E_INVALID, "snl_mhc_dots: null argument");
  return snl::launch_mhc_dots(snl::step_val(*step), *p, x, w, raw, step->m, (cudaStream_t)stream);
}
extern "C" int snl_mhc_finish(const snl_step_u* step, const snl_layer_p* p, const float* raw, const float* w,
                              float* coef, void* stream) {
  if (!step || !p || !raw || !w || !coef) return snl::fail(SNL_E_INVALID, "snl_mhc_finish: null argument");
  return snl::launch_mhc_finish(snl::step_val(*step), *p, raw, w, coef, step->m, (cudaStream_t)stream);
}
extern "C" int snl_merge(const snl_step_u* step, const snl_layer_p* p, float* x, const float* coef, const float* branch,
                         void* stream) {
  if (!step || !p || !x) return snl::fail(SNL_E_INVALID, "snl_merge: null argument");
  if (p->mode > 3) return snl::fail(SNL_E_INVALID, "snl_merge: mode must be 0..3");
  if ((p->mode == 1 || p->mode == 2) && !coef) return snl::fail(SNL_E_INVALID, "snl_merge: modes 1 and 2 need coef");
  if (p->mode != 3 && !branch) return snl::fail(SNL_E_INVALID, "snl_merge: branch is null");
  return snl::launch_merge(snl::step_val(*step), *p, x, coef, branch, step->m, (cudaStream_t)stream);
}
extern "C" int snl_swiglu(const snl_step_u* step, const snl_layer_p* p, const float* gate_up, float* act, void* stream) {
  if (!step || !p || !gate_up || !act) return snl::fail(SNL_E_INVALID, "snl_swiglu: null argument");
  return snl::launch_swiglu(snl::step_val(*step), *p, gate_up, act, step->m, (cudaStream_t)stream);
}
extern "C" int snl_argmax(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, void* stream) {
  if (!logits || !out_idx || n == 0) return snl::fail(SNL_E_INVALID, "snl_argmax: bad argument");
  return snl::launch_argmax(logits, rows, n, out_idx, (cudaStream_t)stream);
}

extern "C" int snl_synth_quant(uint64_t seed, const char* name, int dtype, size_t rows, size_t cols, void* q, float* s,
                               void* stream) {
  if (!name || !q || !s) return snl::fail(SNL_E_INVALID, "snl_synth_quant: null argument");
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return snl::fail(SNL_E_INVALID, "snl_synth_quant: dtype");
  return snl::launch_gen_quant(seed, name, dtype, rows, cols, q, s, (cudaStream_t)stream);
}
extern "C" int snl_synth_f32(uint64_t seed, const char* name, uint32_t sub, size_t n, float mult, float offset,
                             float* out, void* stream) {
  if (!name || !out) return snl::fail(SNL_E_INVALID, "snl_synth_f32: null argument");
  return snl::launch_gen_f32(seed, name, sub, n, mult, offset, out, (cudaStream_t)stream);
}

// ---- argmax without allocation ------------------------------------------------------
//
// snl_argmax keeps its per-block partial keys in a buffer it cudaMalloc's on first use
// (and frees and re-allocates when more rows are asked for; cudaFree waits for the whole
// device). snl_argmax_noalloc serves callers that must not allocate or free device
// memory at that point: a host whose device memory is all reserved by its own pool
// allocator, or a per-token serving loop that shares the GPU and cannot afford the
// device-wide wait of a free. Its scratch is this file-scope array, sized for
// kNoAllocRows rows (16 KB), held by every GPU that loads the library until exit.
// The array's device address is looked up once per device and kept for the life of the
// process: that assumes one CUDA context per device, so a caller that destroys and
// re-creates its context (cudaDeviceReset) must not call this entry point afterwards.
namespace snl {
namespace {
constexpr uint32_t kNoAllocRows = 16;
__device__ __align__(256) unsigned long long g_argmax_noalloc_scratch[kNoAllocRows * kArgBlocks];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned long long* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device. In host code the array's
// name only stands in for it, so the address is looked up once per device (with that
// device current) and cached.
int noalloc_scratch(unsigned long long** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return snl::cuda_fail(e, "snl_argmax_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return snl::fail(SNL_E_INVALID, "snl_argmax_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_argmax_noalloc_scratch);
    if (e != cudaSuccess) return snl::cuda_fail(e, "snl_argmax_noalloc: cudaGetSymbolAddress");
    g_noalloc_addr[dev] = static_cast<unsigned long long*>(p);
  }
  *out = g_noalloc_addr[dev];
  return SNL_OK;
}
}  // namespace
}  // namespace snl

extern "C" int snl_argmax_noalloc(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, void* stream) {
  if (!logits || !out_idx || n == 0) return snl::fail(SNL_E_INVALID, "snl_argmax_noalloc: bad argument");
  if (rows > snl::kNoAllocRows)
    return snl::fail(SNL_E_RANGE, "snl_argmax_noalloc: " + std::to_string(rows) + " rows exceed the static scratch of " +
                                      std::to_string(snl::kNoAllocRows) + " rows");
  unsigned long long* part = nullptr;
  if (int rc = snl::noalloc_scratch(&part)) return rc;
  // Every partial slot the second pass reads is written by the first pass of the same
  // call, so nothing in the shared scratch has to be cleared between calls.
  return snl::launch_argmax_with(logits, rows, n, out_idx, part, (cudaStream_t)stream);
}
