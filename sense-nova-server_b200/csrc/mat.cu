// Block-quantized matrix kernels: y[m, n_off + n] = sum_k x[m, k] * W[n, k].
//
// Replaces matmul.wgsl (matvec1 :129-157, matvec2 :159-198, matvec :62-100,
// matmul :242-318) and the Q8_FNS / Q4_FNS splices of gpu.rs:236-308.
// Weight layout (weights.rs:48-55): Q8_0 = int8 [n, k] row-major; Q4_0 = u32 words
// [n, k/8] with nibble i of word w = element 8w+i stored as value+8; one scale per
// 32-element block in a separate [n, k/32] array, f32 (file layout) or fp16 (the
// engine's repack, used only when every scale is fp16-exact).
//
// Decode (1-2 token rows) is HBM-bound on the weight stream: each lane issues 16-byte
// non-allocating loads of whole weight chunks, converts int8/nibbles to f32 with a
// byte-permute into the mantissa of 2^23 (exact), and the per-row sums are reduced
// with warp shuffles. Larger m goes to a tiled GEMM.
#include "common.cuh"

namespace snl {
namespace {

constexpr int kRowsPerWarp = 4;
constexpr int kWarps = 8;

template <typename ST>
__device__ __forceinline__ float load_scale(const ST* s, uint64_t i);
template <>
__device__ __forceinline__ float load_scale<float>(const float* s, uint64_t i) {
  return __ldg(s + i);
}
template <>
__device__ __forceinline__ float load_scale<__half>(const __half* s, uint64_t i) {
  return __half2float(__ldg(s + i));
}

// 4 int8 of word u -> 4 exact floats: 2^23 + (b + 128) - (2^23 + 128).
__device__ __forceinline__ void q8_word(uint32_t w, float f[4]) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
  f[1] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
  f[2] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
  f[3] = __int_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}
// 8 nibbles of word w -> 8 exact floats (nibble - 8).
__device__ __forceinline__ void q4_word(uint32_t w, float f[8]) {
#pragma unroll
  for (int i = 0; i < 8; i++) f[i] = __int_as_float(((w >> (4 * i)) & 0xFu) | 0x4B000000u) - 8388616.0f;
}

// GEMV for M (1 or 2) token rows. A warp owns kRowsPerWarp consecutive weight rows;
// lane l walks 16-byte chunks l, l+32, ... of each row (Q8: 16 elements = half a
// block; Q4: 32 elements = one block).
template <int DT, int M, typename ST>
__global__ void __launch_bounds__(256) gemv_kernel(snl_mat_p p, const float* __restrict__ x,
                                                   const uint8_t* __restrict__ wq, const ST* __restrict__ ws,
                                                   float* __restrict__ y) {
  constexpr int EPC = DT == SNL_Q8_0 ? 16 : 32;  // elements per 16-byte chunk
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t row0 = (blockIdx.x * kWarps + warp) * kRowsPerWarp;
  if (row0 >= p.n) return;
  const uint32_t K = p.k;
  const uint64_t row_bytes = DT == SNL_Q8_0 ? K : K / 2;
  const uint32_t nchunk = (uint32_t)(row_bytes / 16);
  const uint32_t nb = K / 32;
  float acc[M][kRowsPerWarp];
#pragma unroll
  for (int t = 0; t < M; t++)
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; r++) acc[t][r] = 0.f;

  for (uint32_t c = lane; c < nchunk; c += 32) {
    uint4 w[kRowsPerWarp];
    float s[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; r++) {
      const uint32_t row = row0 + r;
      if (row < p.n) {
        w[r] = ld_stream16(wq + (uint64_t)row * row_bytes + (uint64_t)c * 16);
        s[r] = load_scale<ST>(ws, (uint64_t)row * nb + (DT == SNL_Q8_0 ? c / 2 : c));
      } else {
        w[r] = make_uint4(0, 0, 0, 0);
        s[r] = 0.f;
      }
    }
    float xv[M][EPC];
#pragma unroll
    for (int t = 0; t < M; t++) {
      const float4* xp = reinterpret_cast<const float4*>(x + p.x_off + (uint64_t)t * p.x_stride + (uint64_t)c * EPC);
#pragma unroll
      for (int i = 0; i < EPC / 4; i++) {
        float4 v = __ldg(xp + i);
        xv[t][4 * i] = v.x;
        xv[t][4 * i + 1] = v.y;
        xv[t][4 * i + 2] = v.z;
        xv[t][4 * i + 3] = v.w;
      }
    }
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; r++) {
      const uint32_t wv[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
      float d[M];
#pragma unroll
      for (int t = 0; t < M; t++) d[t] = 0.f;
      if (DT == SNL_Q8_0) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float f[4];
          q8_word(wv[q], f);
#pragma unroll
          for (int t = 0; t < M; t++)
#pragma unroll
            for (int e = 0; e < 4; e++) d[t] = fmaf(f[e], xv[t][4 * q + e], d[t]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float f[8];
          q4_word(wv[q], f);
#pragma unroll
          for (int t = 0; t < M; t++)
#pragma unroll
            for (int e = 0; e < 8; e++) d[t] = fmaf(f[e], xv[t][8 * q + e], d[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < M; t++) acc[t][r] = fmaf(s[r], d[t], acc[t][r]);
    }
  }
#pragma unroll
  for (int t = 0; t < M; t++)
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; r++) acc[t][r] = warp_sum(acc[t][r]);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; r++) {
      const uint32_t row = row0 + r;
      if (row < p.n) {
#pragma unroll
        for (int t = 0; t < M; t++) y[p.y_off + (uint64_t)t * p.y_stride + p.n_off + row] = acc[t][r];
      }
    }
  }
}

// Tiled f32 GEMM for m >= 3 token rows (prefill, short tails): 64 weight rows x
// 64 tokens per CTA, K step of one 32-element block; weights are dequantized into
// shared memory (as the reference's matmul does before its f32 FMA).
constexpr int GBN = 64, GBM = 64, GBK = 32;
template <int DT, typename ST>
__global__ void __launch_bounds__(256) gemm_kernel(snl_mat_p p, uint32_t m_rows, const float* __restrict__ x,
                                                   const uint8_t* __restrict__ wq, const ST* __restrict__ ws,
                                                   float* __restrict__ y) {
  __shared__ float Wt[GBK][GBN + 4];
  __shared__ float Xt[GBK][GBM + 4];
  const int tid = threadIdx.x;
  const uint32_t n0 = blockIdx.x * GBN, m0 = blockIdx.y * GBM;
  const uint32_t K = p.k, nb = K / 32;
  const uint64_t row_bytes = DT == SNL_Q8_0 ? K : K / 2;
  const int tn = tid % 16, tm = tid / 16;  // 16 x 16 threads, 4 x 4 outputs each
  float c[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) c[i][j] = 0.f;

  for (uint32_t b = 0; b < nb; b++) {
    // W tile: 64 rows x 32 elements; thread -> (row = tid/4, 8 elements at (tid%4)*8).
    {
      const int r = tid / 4, part = tid % 4;
      const uint32_t row = n0 + r;
      float f[8];
      if (row < p.n) {
        const float s = load_scale<ST>(ws, (uint64_t)row * nb + b);
        if (DT == SNL_Q8_0) {
          const uint2 w = *reinterpret_cast<const uint2*>(wq + (uint64_t)row * row_bytes + (uint64_t)b * 32 + part * 8);
          float a[4], bb[4];
          q8_word(w.x, a);
          q8_word(w.y, bb);
#pragma unroll
          for (int e = 0; e < 4; e++) {
            f[e] = a[e] * s;
            f[4 + e] = bb[e] * s;
          }
        } else {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(wq + (uint64_t)row * row_bytes + (uint64_t)b * 16 + part * 4);
          q4_word(w, f);
#pragma unroll
          for (int e = 0; e < 8; e++) f[e] *= s;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; e++) Wt[part * 8 + e][r] = f[e];
    }
    // X tile: 64 tokens x 32 elements; thread -> (token = tid/4, 8 elements).
    {
      const int t = tid / 4, part = tid % 4;
      const uint32_t m = m0 + t;
      float f[8];
      if (m < m_rows) {
        const float4* xp = reinterpret_cast<const float4*>(x + p.x_off + (uint64_t)m * p.x_stride + (uint64_t)b * 32 + part * 8);
        float4 v0 = __ldg(xp), v1 = __ldg(xp + 1);
        f[0] = v0.x; f[1] = v0.y; f[2] = v0.z; f[3] = v0.w;
        f[4] = v1.x; f[5] = v1.y; f[6] = v1.z; f[7] = v1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; e++) Xt[part * 8 + e][t] = f[e];
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < GBK; k++) {
      const float4 a = *reinterpret_cast<const float4*>(&Wt[k][tn * 4]);
      const float4 bx = *reinterpret_cast<const float4*>(&Xt[k][tm * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {bx.x, bx.y, bx.z, bx.w};
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) c[i][j] = fmaf(av[i], bv[j], c[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint32_t m = m0 + tm * 4 + j;
    if (m >= m_rows) continue;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint32_t n = n0 + tn * 4 + i;
      if (n < p.n) y[p.y_off + (uint64_t)m * p.y_stride + p.n_off + n] = c[i][j];
    }
  }
}

template <int DT, typename ST>
int launch_mat_t(const snl_mat_p& p, uint32_t rows_m, const float* x, const void* wq, const ST* ws, float* y,
                 cudaStream_t s) {
  const uint8_t* w = static_cast<const uint8_t*>(wq);
  if (rows_m == 1) {
    dim3 grid((p.n + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp));
    gemv_kernel<DT, 1, ST><<<grid, 256, 0, s>>>(p, x, w, ws, y);
  } else if (rows_m == 2) {
    dim3 grid((p.n + kWarps * kRowsPerWarp - 1) / (kWarps * kRowsPerWarp));
    gemv_kernel<DT, 2, ST><<<grid, 256, 0, s>>>(p, x, w, ws, y);
  } else {
    dim3 grid((p.n + GBN - 1) / GBN, (rows_m + GBM - 1) / GBM);
    gemm_kernel<DT, ST><<<grid, 256, 0, s>>>(p, rows_m, x, w, ws, y);
  }
  SNL_LAUNCH_CHECK("mat");
  return SNL_OK;
}

}  // namespace

int launch_mat(int dtype, StepRef st, const snl_mat_p& p, const float* x, const void* wq, const void* ws,
               int scale_f16, float* y, cudaStream_t s, uint32_t rows_m) {
  (void)st;
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return fail(SNL_E_INVALID, "mat: dtype must be Q8_0 or Q4_0");
  if (p.k == 0 || p.k % 32) return fail(SNL_E_INVALID, "mat: k must be a positive multiple of 32");
  if ((p.x_off % 4) || (p.x_stride % 4)) return fail(SNL_E_INVALID, "mat: x_off and x_stride must be multiples of 4");
  if (((uintptr_t)x % 16) || ((uintptr_t)wq % 16)) return fail(SNL_E_INVALID, "mat: x and wq must be 16-byte aligned");
  if (rows_m == 0 || p.n == 0) return SNL_OK;
  if (dtype == SNL_Q8_0) {
    return scale_f16 ? launch_mat_t<SNL_Q8_0, __half>(p, rows_m, x, wq, (const __half*)ws, y, s)
                     : launch_mat_t<SNL_Q8_0, float>(p, rows_m, x, wq, (const float*)ws, y, s);
  }
  return scale_f16 ? launch_mat_t<SNL_Q4_0, __half>(p, rows_m, x, wq, (const __half*)ws, y, s)
                   : launch_mat_t<SNL_Q4_0, float>(p, rows_m, x, wq, (const float*)ws, y, s);
}

}  // namespace snl

extern "C" int snl_mat(int dtype, const snl_step_u* step, const snl_mat_p* p, const float* x, const void* wq,
                       const float* ws, float* y, void* stream) {
  if (!step || !p || !x || !wq || !ws || !y) return snl::fail(SNL_E_INVALID, "snl_mat: null argument");
  const uint32_t rows_m = p->m_one > 0 ? p->m_one : step->m;
  return snl::launch_mat(dtype, snl::step_val(*step), *p, x, wq, ws, 0, y, (cudaStream_t)stream, rows_m);
}
