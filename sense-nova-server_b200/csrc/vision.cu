// The vision tower (src/vision.rs, src/shaders/vision.wgsl) on B200.
//
// The matrix products are the Q8_0 GEMM of the language model (launch_mat: tcgen05 for
// steps of >= 8 rows). Around them, vision.wgsl has four kernels: LayerNorm, a
// bias/activation/residual epilogue, 2D RoPE and bidirectional attention. They are
// exported one to one at the kernel level (snl_vis_*). The encoder fuses the passes
// that follow one another on the same rows:
//   * patch GEMM epilogue (bias + interpolated position, vision.rs:227-229) with the first
//     LayerNorm; the interpolation (vision.rs:141-175) runs on the device per element,
//     in the reference's f32 operation order, instead of as a host table upload;
//   * every residual epilogue (mode 1) with the LayerNorm that reads its result;
//   * the qkv bias with the 2D RoPE of q and k.
// Head dimension 72 and the 2x2 merge are fixed, as vision.wgsl fixes them.
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace snl {
namespace {

constexpr uint32_t kVisHd = 72;    // vision.wgsl:22
constexpr uint32_t kVisHalf = 36;  // rotary pairs (j, j + 36)
constexpr uint32_t kVisQ = 64;     // queries per attention CTA (one per thread)
constexpr uint32_t kVisTK = 16;    // keys per shared-memory tile

__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = fminf(fmaxf(0.7978845608f * (x + 0.044715f * x * x * x), -15.f), 15.f);
  return 0.5f * x * (1.f + tanhf(u));
}

// erf by Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7), as vision.wgsl:71-75 defines it.
__device__ __forceinline__ float erf_as(float x) {
  const float t = 1.f / (1.f + 0.3275911f * fabsf(x));
  const float y =
      1.f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t *
                expf(-x * x);
  return x >= 0.f ? y : -y;
}
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erf_as(x * 0.7071067812f)); }

__device__ __forceinline__ float act_fn(float v, uint32_t act) {
  if (act == SNL_VIS_ACT_GELU_TANH) return gelu_tanh(v);
  if (act == SNL_VIS_ACT_GELU_ERF) return gelu_erf(v);
  return v;
}

// epilogue (vision.wgsl:77-98): v = act(a + bias); mode 0: a = v; 1: b += v; 2: b = v + e.
__global__ void vis_epilogue_kernel(snl_vis_p p, float* __restrict__ a, float* __restrict__ b,
                                    const float* __restrict__ w, const float* __restrict__ e) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint64_t)p.rows * p.cols) return;
  const float v = act_fn(__fadd_rn(a[i], w[i % p.cols]), p.act);
  if (p.mode == 0)
    a[i] = v;
  else if (p.mode == 1)
    b[i] = __fadd_rn(b[i], v);
  else
    b[i] = __fadd_rn(v, e[i]);
}

// The same for mode 0 on rows whose width is a multiple of 4: one float4 per thread.
__global__ void vis_bias_act4_kernel(uint32_t rows, uint32_t cols, uint32_t act, float* __restrict__ a,
                                     const float* __restrict__ w) {
  const uint32_t c4 = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t r = blockIdx.y;
  if (c4 * 4 >= cols || r >= rows) return;
  float4* pa = reinterpret_cast<float4*>(a + (uint64_t)r * cols) + c4;
  const float4 bw = reinterpret_cast<const float4*>(w)[c4];
  float4 v = *pa;
  v.x = act_fn(__fadd_rn(v.x, bw.x), act);
  v.y = act_fn(__fadd_rn(v.y, bw.y), act);
  v.z = act_fn(__fadd_rn(v.z, bw.z), act);
  v.w = act_fn(__fadd_rn(v.w, bw.w), act);
  *pa = v;
}

// The interpolated learned position of token `t` of an h x w grid, column c
// (vision.rs:141-175): linspace in f32, the four corners' weights, and their sum in
// corner order, each operation rounded once.
struct PosGrid {
  const float* table;  // [side * side, hid]
  uint32_t side, hid, h, w;
};
__device__ __forceinline__ float lin_at(uint32_t side, uint32_t n, uint32_t i) {
  if (n == 1) return 0.f;
  return __fdiv_rn(__fmul_rn((float)(side - 1), (float)i), (float)(n - 1));
}
__device__ float pos_value(const PosGrid& g, uint32_t t, uint32_t c) {
  const uint32_t blk = t / 4, intra = t % 4, mw = g.w / 2;
  const uint32_t r = (blk / mw) * 2 + intra / 2, col = (blk % mw) * 2 + intra % 2;
  const float hr = lin_at(g.side, g.h, r), wc = lin_at(g.side, g.w, col);
  const uint32_t fh = (uint32_t)hr, fw = (uint32_t)wc;
  const uint32_t ch = min(fh + 1, g.side - 1), cw = min(fw + 1, g.side - 1);
  const float dh = __fsub_rn(hr, (float)fh), dw = __fsub_rn(wc, (float)fw);
  const float odh = __fsub_rn(1.f, dh), odw = __fsub_rn(1.f, dw);
  const uint32_t idx[4] = {fh * g.side + fw, fh * g.side + cw, ch * g.side + fw, ch * g.side + cw};
  const float wt[4] = {__fmul_rn(odh, odw), __fmul_rn(odh, dw), __fmul_rn(dh, odw), __fmul_rn(dh, dw)};
  float o = 0.f;
#pragma unroll
  for (int k = 0; k < 4; k++) o = __fadd_rn(o, __fmul_rn(g.table[(uint64_t)idx[k] * g.hid + c], wt[k]));
  return o;
}

// LayerNorm of one row by one warp: mean, then the centred variance, then the output.
__device__ __forceinline__ void warp_layer_norm(const float* __restrict__ x, float* __restrict__ out,
                                                const float* __restrict__ nw, uint32_t cols, float eps, uint32_t lane) {
  float s = 0.f;
  for (uint32_t c = lane; c < cols; c += 32) s += x[c];
  const float mean = warp_sum(s) / (float)cols;
  float v = 0.f;
  for (uint32_t c = lane; c < cols; c += 32) {
    const float d = x[c] - mean;
    v += d * d;
  }
  const float inv = rsqrtf(warp_sum(v) / (float)cols + eps);
  for (uint32_t c = lane; c < cols; c += 32) out[c] = (x[c] - mean) * inv * nw[c] + nw[cols + c];
}

// layer_norm (vision.wgsl:40-62), one warp per row.
__global__ void vis_layer_norm_kernel(snl_vis_p p, const float* __restrict__ a, float* __restrict__ b,
                                      const float* __restrict__ w) {
  const uint32_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (r >= p.rows) return;
  warp_layer_norm(a + (uint64_t)r * p.cols, b + (uint64_t)r * p.cols, w, p.cols, p.eps, threadIdx.x & 31);
}

// A residual epilogue and the LayerNorm of its result, one warp per row:
//   mode 1: x += a + bias (vision.wgsl:92-93), mode 2: x = a + bias + pos (:94-95, the
//   position interpolated on the fly); then xn = LayerNorm(x) with nw.
__global__ void vis_add_norm_kernel(uint32_t rows, uint32_t cols, uint32_t mode, float eps, const float* __restrict__ a,
                                    const float* __restrict__ bias, float* __restrict__ x, float* __restrict__ xn,
                                    const float* __restrict__ nw, PosGrid pg) {
  const uint32_t r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (r >= rows) return;
  const uint32_t lane = threadIdx.x & 31;
  const float* ar = a + (uint64_t)r * cols;
  float* xr = x + (uint64_t)r * cols;
  for (uint32_t c = lane; c < cols; c += 32) {
    const float v = __fadd_rn(ar[c], bias[c]);
    xr[c] = mode == 1 ? __fadd_rn(xr[c], v) : __fadd_rn(v, pos_value(pg, r, c));
  }
  __syncwarp();
  warp_layer_norm(xr, xn + (uint64_t)r * cols, nw, cols, eps, lane);
}

// 2D rotary angle of pair j for token t (vision.wgsl:109-121): pairs j < 18 turn by the
// patch row, 18 <= j < 36 by the patch column.
__device__ __forceinline__ void rope_cs(uint32_t t, uint32_t j, uint32_t grid_w, float* cs, float* sn) {
  const uint32_t mw = grid_w / 2, blk = t / 4, intra = t % 4;
  const uint32_t row = (blk / mw) * 2 + intra / 2, col = (blk % mw) * 2 + intra % 2;
  const uint32_t fi = j % (kVisHalf / 2);
  const uint32_t pos = j >= kVisHalf / 2 ? col : row;
  const float ang = (float)pos * powf(10000.f, -(float)(2 * fi) / (float)kVisHalf);
  sincosf(ang, sn, cs);
}

// rope (vision.wgsl:100-130) on qkv [rows, 3, heads, 72]; with bias, the qkv bias is
// added first (the epilogue of vision.rs:236-237) to q, k and v.
__global__ void vis_qkv_rope_kernel(uint32_t rows, uint32_t heads, uint32_t grid_w, float* __restrict__ a,
                                    const float* __restrict__ bias) {
  const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t per_token = heads * kVisHalf;
  if (i >= (uint64_t)rows * per_token) return;
  const uint32_t t = (uint32_t)(i / per_token), h = (uint32_t)(i % per_token) / kVisHalf, j = (uint32_t)(i % kVisHalf);
  const uint32_t hidden = heads * kVisHd;
  float cs, sn;
  rope_cs(t, j, grid_w, &cs, &sn);
  for (uint32_t part = 0; part < 3; part++) {
    const uint64_t base = (uint64_t)t * 3 * hidden + part * hidden + h * kVisHd;
    float x1 = a[base + j], x2 = a[base + j + kVisHalf];
    if (bias) {
      x1 = __fadd_rn(x1, bias[part * hidden + h * kVisHd + j]);
      x2 = __fadd_rn(x2, bias[part * hidden + h * kVisHd + j + kVisHalf]);
    }
    if (part < 2) {
      a[base + j] = x1 * cs - x2 * sn;
      a[base + j + kVisHalf] = x2 * cs + x1 * sn;
    } else if (bias) {
      a[base + j] = x1;
      a[base + j + kVisHalf] = x2;
    }
  }
}

// attend (vision.wgsl:137-206): bidirectional attention over the rows of one frame. A
// CTA holds 64 queries of one head, one per thread (q and the output accumulator in
// registers); 16-key tiles of K and V are staged in shared memory and folded into an
// online softmax.
__global__ void __launch_bounds__(kVisQ) vis_attend_kernel(uint32_t n, uint32_t heads, const float* __restrict__ qkv,
                                                           float* __restrict__ out) {
  __shared__ float4 ks[kVisTK * kVisHd / 4];
  __shared__ float4 vs[kVisTK * kVisHd / 4];
  const uint32_t h = blockIdx.y;
  const uint32_t qi = blockIdx.x * kVisQ + threadIdx.x;
  const uint32_t hidden = heads * kVisHd, stride = 3 * hidden;
  const bool valid = qi < n;
  const float scale = rsqrtf((float)kVisHd);
  float4 q[kVisHd / 4], acc[kVisHd / 4];
#pragma unroll
  for (uint32_t d = 0; d < kVisHd / 4; d++) {
    acc[d] = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) v = *reinterpret_cast<const float4*>(qkv + (uint64_t)qi * stride + h * kVisHd + d * 4);
    q[d] = make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale);
  }
  float mx = -1e30f, l = 0.f;
  for (uint32_t k0 = 0; k0 < n; k0 += kVisTK) {
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < kVisTK * kVisHd / 4; t += kVisQ) {
      const uint32_t key = k0 + t / (kVisHd / 4), d = t % (kVisHd / 4);
      float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
      if (key < n) {
        const float* src = qkv + (uint64_t)key * stride + hidden + h * kVisHd + d * 4;
        kv = *reinterpret_cast<const float4*>(src);
        vv = *reinterpret_cast<const float4*>(src + hidden);
      }
      ks[t] = kv;
      vs[t] = vv;
    }
    __syncthreads();
    const uint32_t cnt = min(kVisTK, n - k0);
    float sc[kVisTK];
    float tmax = mx;
#pragma unroll
    for (uint32_t j = 0; j < kVisTK; j++) {
      float s = 0.f;
#pragma unroll
      for (uint32_t d = 0; d < kVisHd / 4; d++) {
        const float4 kk = ks[j * (kVisHd / 4) + d];
        s += q[d].x * kk.x + q[d].y * kk.y + q[d].z * kk.z + q[d].w * kk.w;
      }
      sc[j] = s;
      if (j < cnt) tmax = fmaxf(tmax, s);
    }
    const float corr = expf(mx - tmax);
    l *= corr;
#pragma unroll
    for (uint32_t d = 0; d < kVisHd / 4; d++) {
      acc[d].x *= corr;
      acc[d].y *= corr;
      acc[d].z *= corr;
      acc[d].w *= corr;
    }
#pragma unroll
    for (uint32_t j = 0; j < kVisTK; j++) {
      if (j < cnt) {
        const float pj = expf(sc[j] - tmax);
        l += pj;
#pragma unroll
        for (uint32_t d = 0; d < kVisHd / 4; d++) {
          const float4 vv = vs[j * (kVisHd / 4) + d];
          acc[d].x += pj * vv.x;
          acc[d].y += pj * vv.y;
          acc[d].z += pj * vv.z;
          acc[d].w += pj * vv.w;
        }
      }
    }
    mx = tmax;
  }
  if (!valid) return;
  float4* o = reinterpret_cast<float4*>(out + (uint64_t)qi * hidden + h * kVisHd);
  const float il = 1.f / l;
#pragma unroll
  for (uint32_t d = 0; d < kVisHd / 4; d++) o[d] = make_float4(acc[d].x * il, acc[d].y * il, acc[d].z * il, acc[d].w * il);
}

// ---- launches ------------------------------------------------------------------------

int launch_vis_layer_norm(const snl_vis_p& p, const float* a, float* b, const float* w, cudaStream_t s) {
  if (!p.rows) return SNL_OK;
  vis_layer_norm_kernel<<<(p.rows + 7) / 8, 256, 0, s>>>(p, a, b, w);
  SNL_LAUNCH_CHECK("vis_layer_norm");
  return SNL_OK;
}

int launch_vis_epilogue(const snl_vis_p& p, float* a, float* b, const float* w, const float* e, cudaStream_t s) {
  const uint64_t total = (uint64_t)p.rows * p.cols;
  if (!total) return SNL_OK;
  if (p.mode == 0 && p.cols % 4 == 0 && ((uintptr_t)a | (uintptr_t)w) % 16 == 0 && p.rows <= 65535) {
    vis_bias_act4_kernel<<<dim3((p.cols / 4 + 255) / 256, p.rows), 256, 0, s>>>(p.rows, p.cols, p.act, a, w);
  } else {
    vis_epilogue_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p, a, b, w, e);
  }
  SNL_LAUNCH_CHECK("vis_epilogue");
  return SNL_OK;
}

int launch_vis_qkv_rope(uint32_t rows, uint32_t heads, uint32_t grid_w, float* qkv, const float* bias, cudaStream_t s) {
  const uint64_t total = (uint64_t)rows * heads * kVisHalf;
  if (!total) return SNL_OK;
  vis_qkv_rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(rows, heads, grid_w, qkv, bias);
  SNL_LAUNCH_CHECK("vis_qkv_rope");
  return SNL_OK;
}

int launch_vis_attend(uint32_t n, uint32_t heads, const float* qkv, float* out, cudaStream_t s) {
  if (!n) return SNL_OK;
  if (((uintptr_t)qkv | (uintptr_t)out) % 16) return fail(SNL_E_INVALID, "vis_attend: qkv and out must be 16-byte aligned");
  vis_attend_kernel<<<dim3((n + kVisQ - 1) / kVisQ, heads), kVisQ, 0, s>>>(n, heads, qkv, out);
  SNL_LAUNCH_CHECK("vis_attend");
  return SNL_OK;
}

int launch_vis_add_norm(uint32_t rows, uint32_t cols, uint32_t mode, float eps, const float* a, const float* bias,
                        float* x, float* xn, const float* nw, const PosGrid& pg, cudaStream_t s) {
  if (!rows) return SNL_OK;
  vis_add_norm_kernel<<<(rows + 7) / 8, 256, 0, s>>>(rows, cols, mode, eps, a, bias, x, xn, nw, pg);
  SNL_LAUNCH_CHECK("vis_add_norm");
  return SNL_OK;
}

struct DevGuard {
  int prev = -1;
  explicit DevGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

constexpr float kVisEps = 1e-6f;  // vision.rs:52

}  // namespace
}  // namespace snl

using namespace snl;

// A weight of the tower on the device: Q8_0 (q int8 [rows, cols], s f32 [rows, cols/32])
// or f32 (q = n floats).
struct VisTensor {
  int dtype = SNL_F32;
  size_t rows = 0, cols = 0;
  void* q = nullptr;
  float* s = nullptr;
};

struct snl_vision {
  snl_vision_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  bool finalized = false;
  std::map<std::string, VisTensor> t;
  std::vector<void*> allocs;
  // activations of one frame, grown on demand
  size_t cap_n = 0;
  float *pin = nullptr, *x = nullptr, *xn = nullptr, *tmp = nullptr, *att = nullptr, *qkv = nullptr, *mlp = nullptr;
  float* h_out = nullptr;  // pinned staging of one frame's output
  size_t h_out_cap = 0;
};

namespace snl {
namespace {

int vis_alloc(snl_vision* v, void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, std::max<size_t>(bytes, 256));
  if (e != cudaSuccess) return cuda_fail(e, "vision: cudaMalloc");
  v->allocs.push_back(*p);
  return SNL_OK;
}

// The tensors of convert.rs:165-199 with their shapes: (name, dtype, rows, cols).
struct VisSpec {
  std::string name;
  int dtype;
  size_t rows, cols;
};
std::vector<VisSpec> vis_specs(const snl_vision_config& c) {
  const size_t h = c.hidden, ip = c.intermediate_padded, md = (size_t)c.hidden * c.merge * c.merge;
  const size_t pd = 3ull * c.temporal_patch * c.patch * c.patch;
  std::vector<VisSpec> v = {{"v.patch", SNL_Q8_0, h, pd},
                            {"v.patch_b", SNL_F32, 1, h},
                            {"v.pos", SNL_F32, (size_t)c.pos_side * c.pos_side, h}};
  for (uint32_t i = 0; i < c.depth; i++) {
    const std::string b = "v" + std::to_string(i) + ".";
    v.push_back({b + "n1", SNL_F32, 1, 2 * h});
    v.push_back({b + "n2", SNL_F32, 1, 2 * h});
    v.push_back({b + "qkv", SNL_Q8_0, 3 * h, h});
    v.push_back({b + "qkv_b", SNL_F32, 1, 3 * h});
    v.push_back({b + "proj", SNL_Q8_0, h, h});
    v.push_back({b + "proj_b", SNL_F32, 1, h});
    v.push_back({b + "fc1", SNL_Q8_0, ip, h});
    v.push_back({b + "fc1_b", SNL_F32, 1, ip});
    v.push_back({b + "fc2", SNL_Q8_0, h, ip});
    v.push_back({b + "fc2_b", SNL_F32, 1, h});
  }
  v.push_back({"vm.norm", SNL_F32, 1, 2 * h});
  v.push_back({"vm.fc1", SNL_Q8_0, md, md});
  v.push_back({"vm.fc1_b", SNL_F32, 1, md});
  v.push_back({"vm.fc2", SNL_Q8_0, c.out_hidden, md});
  v.push_back({"vm.fc2_b", SNL_F32, 1, c.out_hidden});
  return v;
}

int alloc_tensor(snl_vision* v, const VisSpec& sp, VisTensor* out) {
  VisTensor t;
  t.dtype = sp.dtype;
  t.rows = sp.rows;
  t.cols = sp.cols;
  if (sp.dtype == SNL_Q8_0) {
    SNL_TRY(vis_alloc(v, &t.q, sp.rows * sp.cols));
    SNL_TRY(vis_alloc(v, (void**)&t.s, sp.rows * sp.cols / 32 * sizeof(float)));
  } else {
    SNL_TRY(vis_alloc(v, &t.q, sp.rows * sp.cols * sizeof(float)));
  }
  *out = t;
  return SNL_OK;
}

int ensure_scratch(snl_vision* v, size_t n) {
  if (n <= v->cap_n) return SNL_OK;
  const auto& c = v->cfg;
  const size_t h = c.hidden, nq = n / 4, md = (size_t)h * 4;
  const size_t pd = 3ull * c.temporal_patch * c.patch * c.patch;
  // Old buffers stay in allocs until destroy (a request for more patches is rare).
  SNL_TRY(vis_alloc(v, (void**)&v->pin, n * pd * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->x, n * h * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->xn, n * h * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->tmp, n * h * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->att, n * h * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->qkv, std::max(n * 3 * h, nq * (size_t)c.out_hidden) * 4));
  SNL_TRY(vis_alloc(v, (void**)&v->mlp, std::max(n * (size_t)c.intermediate_padded, nq * md) * 4));
  v->cap_n = n;
  return SNL_OK;
}

// y[rows, n_out] (row stride y_stride) = x[rows, k] (row stride x_stride) . W^T.
int vis_mat(snl_vision* v, const VisTensor& w, const float* x, size_t rows, size_t x_stride, float* y, size_t y_stride) {
  snl_mat_p mp{(uint32_t)w.rows, (uint32_t)w.cols, 0, (uint32_t)x_stride, 0, (uint32_t)y_stride, 0, 0};
  snl_step_u st{(uint32_t)rows, 0, 1, 0};
  return launch_mat(SNL_Q8_0, step_val(st), mp, x, w.q, w.s, 0, y, v->stream, (uint32_t)rows);
}

const VisTensor& T(snl_vision* v, const std::string& n) { return v->t.at(n); }
const float* F(snl_vision* v, const std::string& n) { return static_cast<const float*>(v->t.at(n).q); }

// One frame (vision.rs:222-272): n = h * w patch rows in v->pin -> v->qkv [n/4, out_hidden].
int encode_frame(snl_vision* v, uint32_t gh, uint32_t gw) {
  const auto& c = v->cfg;
  const uint32_t n = gh * gw, nq = n / 4, hid = c.hidden, ip = c.intermediate_padded, md = hid * 4;
  const size_t pd = 3ull * c.temporal_patch * c.patch * c.patch;
  cudaStream_t s = v->stream;
  const PosGrid pg{F(v, "v.pos"), c.pos_side, hid, gh, gw};
  // Patch embedding; bias and the interpolated position; the first block's norm1.
  SNL_TRY(vis_mat(v, T(v, "v.patch"), v->pin, n, pd, v->tmp, hid));
  const std::string first_norm = c.depth ? "v0.n1" : "vm.norm";
  SNL_TRY(launch_vis_add_norm(n, hid, 2, kVisEps, v->tmp, F(v, "v.patch_b"), v->x, v->xn, F(v, first_norm), pg, s));
  for (uint32_t i = 0; i < c.depth; i++) {
    const std::string b = "v" + std::to_string(i) + ".";
    SNL_TRY(vis_mat(v, T(v, b + "qkv"), v->xn, n, hid, v->qkv, 3 * hid));
    SNL_TRY(launch_vis_qkv_rope(n, c.n_heads, gw, v->qkv, F(v, b + "qkv_b"), s));
    SNL_TRY(launch_vis_attend(n, c.n_heads, v->qkv, v->att, s));
    SNL_TRY(vis_mat(v, T(v, b + "proj"), v->att, n, hid, v->tmp, hid));
    SNL_TRY(launch_vis_add_norm(n, hid, 1, kVisEps, v->tmp, F(v, b + "proj_b"), v->x, v->xn, F(v, b + "n2"), pg, s));
    SNL_TRY(vis_mat(v, T(v, b + "fc1"), v->xn, n, hid, v->mlp, ip));
    snl_vis_p ep{n, ip, 0, SNL_VIS_ACT_GELU_TANH, 0.f, 0, 0, 0};
    SNL_TRY(launch_vis_epilogue(ep, v->mlp, nullptr, F(v, b + "fc1_b"), nullptr, s));
    SNL_TRY(vis_mat(v, T(v, b + "fc2"), v->mlp, n, ip, v->tmp, hid));
    const std::string next_norm = i + 1 < c.depth ? "v" + std::to_string(i + 1) + ".n1" : "vm.norm";
    SNL_TRY(launch_vis_add_norm(n, hid, 1, kVisEps, v->tmp, F(v, b + "fc2_b"), v->x, v->xn, F(v, next_norm), pg, s));
  }
  // Merger (vision.rs:261-270): each 2x2 block (4 consecutive normed rows) is one row.
  SNL_TRY(vis_mat(v, T(v, "vm.fc1"), v->xn, nq, md, v->mlp, md));
  snl_vis_p e1{nq, md, 0, SNL_VIS_ACT_GELU_ERF, 0.f, 0, 0, 0};
  SNL_TRY(launch_vis_epilogue(e1, v->mlp, nullptr, F(v, "vm.fc1_b"), nullptr, s));
  SNL_TRY(vis_mat(v, T(v, "vm.fc2"), v->mlp, nq, md, v->qkv, c.out_hidden));
  snl_vis_p e2{nq, c.out_hidden, 0, 0, 0.f, 0, 0, 0};
  SNL_TRY(launch_vis_epilogue(e2, v->qkv, nullptr, F(v, "vm.fc2_b"), nullptr, s));
  return SNL_OK;
}

}  // namespace
}  // namespace snl

// ---- C ABI -----------------------------------------------------------------------------

extern "C" int snl_vis_layer_norm(const snl_vis_p* p, const float* a, float* b, const float* w, void* stream) {
  if (!p || !a || !b || !w) return fail(SNL_E_INVALID, "snl_vis_layer_norm: null argument");
  return launch_vis_layer_norm(*p, a, b, w, (cudaStream_t)stream);
}

extern "C" int snl_vis_epilogue(const snl_vis_p* p, float* a, float* b, const float* w, const float* e, void* stream) {
  if (!p || !a || !w) return fail(SNL_E_INVALID, "snl_vis_epilogue: null argument");
  if (p->mode > 2) return fail(SNL_E_INVALID, "snl_vis_epilogue: mode must be 0..2");
  if (p->mode >= 1 && !b) return fail(SNL_E_INVALID, "snl_vis_epilogue: modes 1 and 2 need b");
  if (p->mode == 2 && !e) return fail(SNL_E_INVALID, "snl_vis_epilogue: mode 2 needs e");
  return launch_vis_epilogue(*p, a, b, w, e, (cudaStream_t)stream);
}

extern "C" int snl_vis_rope(const snl_vis_p* p, float* qkv, void* stream) {
  if (!p || !qkv) return fail(SNL_E_INVALID, "snl_vis_rope: null argument");
  if (p->grid_w == 0 || p->grid_w % 2) return fail(SNL_E_INVALID, "snl_vis_rope: grid_w must be even");
  return launch_vis_qkv_rope(p->rows, p->heads, p->grid_w, qkv, nullptr, (cudaStream_t)stream);
}

extern "C" int snl_vis_attend(const snl_vis_p* p, const float* qkv, float* out, void* stream) {
  if (!p || !qkv || !out) return fail(SNL_E_INVALID, "snl_vis_attend: null argument");
  if (p->heads == 0 || p->heads > 65535) return fail(SNL_E_INVALID, "snl_vis_attend: heads out of range");
  return launch_vis_attend(p->rows, p->heads, qkv, out, (cudaStream_t)stream);
}

extern "C" int snl_vision_create(const snl_vision_config* cfg, int device, snl_vision** out) {
  if (!cfg || !out) return fail(SNL_E_INVALID, "snl_vision_create: null argument");
  *out = nullptr;
  const auto& c = *cfg;
  if (c.n_heads == 0 || c.hidden != c.n_heads * kVisHd)
    return fail(SNL_E_UNSUPPORTED, "vision: the kernels need head_dim 72 (hidden = 72 * n_heads)");
  if (c.merge != 2) return fail(SNL_E_UNSUPPORTED, "vision: the kernels need a 2x2 merge");
  if (c.hidden % 32) return fail(SNL_E_INVALID, "vision: hidden must be a multiple of 32 (Q8_0 blocks)");
  if (c.intermediate_padded % 32 || c.intermediate_padded < c.intermediate || c.out_hidden == 0 || c.out_hidden % 4)
    return fail(SNL_E_INVALID, "vision: intermediate_padded must be a multiple of 32 >= intermediate, out_hidden of 4");
  if (c.pos_side == 0 || c.patch == 0 || c.temporal_patch == 0)
    return fail(SNL_E_INVALID, "vision: zero patch or position grid");
  if ((3ull * c.temporal_patch * c.patch * c.patch) % 32) return fail(SNL_E_INVALID, "vision: patch_dim % 32");
  snl_vision* v = new snl_vision();
  v->cfg = c;
  v->device = device;
  DevGuard g(device);
  cudaError_t e = cudaStreamCreateWithFlags(&v->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete v;
    return cuda_fail(e, "vision: stream");
  }
  for (const auto& sp : vis_specs(c)) {
    VisTensor t;
    if (int rc = alloc_tensor(v, sp, &t)) {
      snl_vision_destroy(v);
      return rc;
    }
    v->t[sp.name] = t;
  }
  *out = v;
  return SNL_OK;
}

extern "C" int snl_vision_set_tensor(snl_vision* v, const char* name, int dtype, size_t rows, size_t cols,
                                     const void* q, const void* s) {
  if (!v || !name || !q) return fail(SNL_E_INVALID, "snl_vision_set_tensor: null argument");
  auto it = v->t.find(name);
  if (it == v->t.end()) return fail(SNL_E_INVALID, std::string("vision: unknown tensor ") + name);
  VisTensor& t = it->second;
  if (t.dtype != dtype || t.rows * t.cols != rows * cols || (dtype == SNL_Q8_0 && (t.rows != rows || !s)))
    return fail(SNL_E_INVALID, std::string("vision: tensor ") + name + " has the wrong type or shape");
  DevGuard g(v->device);
  if (dtype == SNL_Q8_0) {
    SNL_CUDA_TRY(cudaMemcpy(t.q, q, rows * cols, cudaMemcpyHostToDevice));
    SNL_CUDA_TRY(cudaMemcpy(t.s, s, rows * cols / 32 * sizeof(float), cudaMemcpyHostToDevice));
  } else {
    SNL_CUDA_TRY(cudaMemcpy(t.q, q, rows * cols * sizeof(float), cudaMemcpyHostToDevice));
  }
  return SNL_OK;
}

// Seeded synthetic weights with the generator shared with the CPU checker: Q8_0 matrices
// as the language model's; LayerNorm weights 1 + 0.1 z and biases 0.05 z (sub-streams 0
// and 1); other biases 0.02 z; the position table 0.3 z.
extern "C" int snl_vision_fill_synthetic(snl_vision* v, uint64_t seed) {
  if (!v) return fail(SNL_E_INVALID, "snl_vision_fill_synthetic: null vision");
  DevGuard g(v->device);
  for (const auto& sp : vis_specs(v->cfg)) {
    VisTensor& t = v->t.at(sp.name);
    const char* nm = sp.name.c_str();
    if (sp.dtype == SNL_Q8_0) {
      SNL_TRY(snl_synth_quant(seed, nm, SNL_Q8_0, t.rows, t.cols, t.q, t.s, v->stream));
    } else if (sp.name.size() > 3 && (sp.name.compare(sp.name.size() - 3, 3, ".n1") == 0 ||
                                      sp.name.compare(sp.name.size() - 3, 3, ".n2") == 0 || sp.name == "vm.norm")) {
      const size_t h = t.cols / 2;
      SNL_TRY(snl_synth_f32(seed, nm, 0, h, 0.1f, 1.0f, static_cast<float*>(t.q), v->stream));
      SNL_TRY(snl_synth_f32(seed, nm, 1, h, 0.05f, 0.0f, static_cast<float*>(t.q) + h, v->stream));
    } else {
      const float mult = sp.name == "v.pos" ? 0.3f : 0.02f;
      SNL_TRY(snl_synth_f32(seed, nm, 0, t.rows * t.cols, mult, 0.0f, static_cast<float*>(t.q), v->stream));
    }
  }
  SNL_CUDA_TRY(cudaStreamSynchronize(v->stream));
  return SNL_OK;
}

extern "C" int snl_vision_finalize(snl_vision* v) {
  if (!v) return fail(SNL_E_INVALID, "snl_vision_finalize: null vision");
  v->finalized = true;
  return SNL_OK;
}

extern "C" int snl_vision_encode(snl_vision* v, const float* patches, size_t frames, size_t h, size_t w, float* out) {
  if (!v || !patches || !out) return fail(SNL_E_INVALID, "snl_vision_encode: null argument");
  if (!v->finalized) return fail(SNL_E_STATE, "vision: not finalized");
  const auto& c = v->cfg;
  if (h == 0 || w == 0 || h % c.merge || w % c.merge || frames == 0)
    return fail(SNL_E_INVALID, "vision input has the wrong shape");
  const size_t n = h * w, nq = n / 4;
  if (n > (1u << 22) || n * (size_t)c.intermediate_padded > (1ull << 32))
    return fail(SNL_E_RANGE, "image is too large (" + std::to_string(n) + " patches per frame)");
  const size_t pd = 3ull * c.temporal_patch * c.patch * c.patch;
  DevGuard g(v->device);
  SNL_TRY(ensure_scratch(v, n));
  const size_t out_bytes = nq * c.out_hidden * sizeof(float);
  if (out_bytes > v->h_out_cap) {
    if (v->h_out) cudaFreeHost(v->h_out);
    v->h_out = nullptr;
    v->h_out_cap = 0;
    SNL_CUDA_TRY(cudaMallocHost(&v->h_out, out_bytes));
    v->h_out_cap = out_bytes;
  }
  for (size_t f = 0; f < frames; f++) {
    SNL_CUDA_TRY(cudaMemcpyAsync(v->pin, patches + f * n * pd, n * pd * sizeof(float), cudaMemcpyHostToDevice,
                                 v->stream));
    SNL_TRY(encode_frame(v, (uint32_t)h, (uint32_t)w));
    SNL_CUDA_TRY(cudaMemcpyAsync(v->h_out, v->qkv, out_bytes, cudaMemcpyDeviceToHost, v->stream));
    SNL_CUDA_TRY(cudaStreamSynchronize(v->stream));
    memcpy(out + f * nq * c.out_hidden, v->h_out, out_bytes);
  }
  return SNL_OK;
}

extern "C" void snl_vision_destroy(snl_vision* v) {
  if (!v) return;
  DevGuard g(v->device);
  if (v->stream) cudaStreamSynchronize(v->stream);
  for (void* p : v->allocs) cudaFree(p);
  if (v->h_out) cudaFreeHost(v->h_out);
  if (v->stream) cudaStreamDestroy(v->stream);
  delete v;
}
