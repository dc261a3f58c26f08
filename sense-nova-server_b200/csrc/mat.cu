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
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "ptx.cuh"

namespace snl {

// Device error word of this library's bounded waits (no allocation). Read and cleared
// by snl_device_error().
__device__ int g_dev_error;

// Device address of g_dev_error on the current device, for kernels in other files
// (looked up once per device).
int device_error_word(int** out) {
  static int* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(SNL_E_INVALID, "device ordinal out of range");
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dev_error);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_dev_error)");
    addr[dev] = static_cast<int*>(p);
  }
  *out = addr[dev];
  return SNL_OK;
}

bool pdl_on() {
  static const bool on = getenv("SNL_NO_PDL") == nullptr;
  return on;
}

int sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (!sms[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 1;
    sms[dev] = v;
  }
  return sms[dev];
}

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


// ---------------------------------------------------------------------------------
// Streaming GEMV (1-2 token rows) with bulk async copies.
//
// Each warp is an independent streaming unit: it owns groups of kSRows weight rows
// (group g = global warp id + i * total warps) and walks each group's K range in chunks
// of `chunk` bytes per row. Lanes 0..2*kSRows-1 issue one cp.async.bulk each per stage
// (a row's weight chunk, a row's scale chunk) into a per-warp ring of `stages` stages
// that completes on that stage's mbarrier, so stages * kSRows * (chunk + scales) bytes
// are in flight per warp whatever the register budget. x is staged once per CTA in
// shared memory. Weights carry an L2 evict-first policy: they are read once per token,
// while x, the KV cache and the recurrent state should stay in L2.
// ---------------------------------------------------------------------------------
constexpr int kSWarps = 8;
constexpr int kSRows = 4;
constexpr int kSMaxStages = 4;

__host__ __device__ constexpr uint32_t align16u(uint32_t v) { return (v + 15u) & ~15u; }

template <int DT, int M, typename ST>
__global__ void __launch_bounds__(kSWarps * 32, 1)
    gemv_stream_kernel(snl_mat_p p, const float* __restrict__ x, const uint8_t* __restrict__ wq,
                       const ST* __restrict__ ws, float* __restrict__ y, uint32_t chunk, uint32_t stages) {
  constexpr uint32_t EPB = DT == SNL_Q8_0 ? 1 : 2;  // elements per weight byte
  constexpr uint32_t EPC = 16 * EPB;                // elements per 16-byte chunk
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t K = p.k;
  const uint32_t row_bytes = K / EPB;
  const uint32_t nchunk = row_bytes / chunk;
  const uint32_t chunk_elems = chunk * EPB;
  const uint32_t sc_bytes = chunk_elems / 32 * (uint32_t)sizeof(ST);
  const uint32_t stage_bytes = kSRows * (chunk + sc_bytes);
  const uint32_t x_bytes = align16u(M * K * 4);
  float* xs = reinterpret_cast<float*>(smem);
  uint8_t* ring = smem + x_bytes + (uint32_t)warp * stages * stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + x_bytes + kSWarps * stages * stage_bytes) + warp * kSMaxStages;

  const uint32_t groups = (p.n + kSRows - 1) / kSRows;
  const uint32_t gw = blockIdx.x * kSWarps + warp;
  const uint32_t nw = gridDim.x * kSWarps;
  const uint32_t my_groups = gw < groups ? (groups - gw + nw - 1) / nw : 0;
  const uint32_t njobs = my_groups * nchunk;

  if (lane == 0)
    for (uint32_t s = 0; s < stages; s++) mbar_init(&bars[s], 1);
  fence_mbar_init();
  __syncwarp();
  const uint64_t pol = l2_policy_evict_first();

  auto issue = [&](uint32_t j) {
    const uint32_t s = j % stages;
    const uint32_t row0 = (gw + (j / nchunk) * nw) * kSRows;
    const uint32_t c = j % nchunk;
    const uint32_t rows = min((uint32_t)kSRows, p.n - row0);
    uint8_t* st = ring + s * stage_bytes;
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], rows * (chunk + sc_bytes));
    __syncwarp();
    if ((uint32_t)lane < rows) {
      const uint32_t r = lane;
      bulk_g2s(st + r * chunk, wq + (uint64_t)(row0 + r) * row_bytes + (uint64_t)c * chunk, chunk, &bars[s], pol);
    } else if (lane >= kSRows && (uint32_t)(lane - kSRows) < rows) {
      const uint32_t r = lane - kSRows;
      const uint8_t* src = reinterpret_cast<const uint8_t*>(ws) +
                           ((uint64_t)(row0 + r) * (K / 32) + (uint64_t)c * (chunk_elems / 32)) * sizeof(ST);
      bulk_g2s(st + kSRows * chunk + r * sc_bytes, src, sc_bytes, &bars[s], pol);
    }
  };

  const uint32_t pre = min(stages, njobs);
  for (uint32_t j = 0; j < pre; j++) issue(j);

  // Stage x (M rows of K floats) while the first weight chunks are in flight.
  {
    float4* xs4 = reinterpret_cast<float4*>(xs);
    const uint32_t k4 = K / 4;
    for (uint32_t i = threadIdx.x; i < M * k4; i += blockDim.x) {
      const uint32_t t = i / k4, e = i % k4;
      xs4[i] = __ldg(reinterpret_cast<const float4*>(x + p.x_off + (uint64_t)t * p.x_stride) + e);
    }
  }
  __syncthreads();

  float acc[M][kSRows];
#pragma unroll
  for (int t = 0; t < M; t++)
#pragma unroll
    for (int r = 0; r < kSRows; r++) acc[t][r] = 0.f;

  uint32_t j = 0;
  bool ok = true;
  for (; j < njobs; j++) {
    const uint32_t s = j % stages;
    if (!mbar_wait_bounded(&bars[s], (j / stages) & 1)) {
      ok = false;
      break;
    }
    const uint32_t row0 = (gw + (j / nchunk) * nw) * kSRows;
    const uint32_t c = j % nchunk;
    const uint32_t rows = min((uint32_t)kSRows, p.n - row0);
    const uint8_t* st = ring + s * stage_bytes;
    for (uint32_t q = lane; q < chunk / 16; q += 32) {
      const uint32_t e0 = c * chunk_elems + q * EPC;
      float xv[M][EPC];
#pragma unroll
      for (int t = 0; t < M; t++) {
        const float4* xp = reinterpret_cast<const float4*>(xs + t * K + e0);
#pragma unroll
        for (uint32_t i = 0; i < EPC / 4; i++) {
          const float4 v = xp[i];
          xv[t][4 * i] = v.x;
          xv[t][4 * i + 1] = v.y;
          xv[t][4 * i + 2] = v.z;
          xv[t][4 * i + 3] = v.w;
        }
      }
#pragma unroll
      for (int r = 0; r < kSRows; r++) {
        if ((uint32_t)r >= rows) break;
        const uint4 w = *reinterpret_cast<const uint4*>(st + r * chunk + q * 16);
        const ST* scp = reinterpret_cast<const ST*>(st + kSRows * chunk + r * sc_bytes);
        float sc;
        if constexpr (sizeof(ST) == 4) sc = scp[q * EPC / 32];
        else sc = __half2float(scp[q * EPC / 32]);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
        float d[M];
#pragma unroll
        for (int t = 0; t < M; t++) d[t] = 0.f;
#pragma unroll
        for (int qq = 0; qq < 4; qq++) {
          if constexpr (DT == SNL_Q8_0) {
            float f[4];
            q8_word(wv[qq], f);
#pragma unroll
            for (int t = 0; t < M; t++)
#pragma unroll
              for (int e = 0; e < 4; e++) d[t] = fmaf(f[e], xv[t][4 * qq + e], d[t]);
          } else {
            float f[8];
            q4_word(wv[qq], f);
#pragma unroll
            for (int t = 0; t < M; t++)
#pragma unroll
              for (int e = 0; e < 8; e++) d[t] = fmaf(f[e], xv[t][8 * qq + e], d[t]);
          }
        }
#pragma unroll
        for (int t = 0; t < M; t++) acc[t][r] = fmaf(sc, d[t], acc[t][r]);
      }
    }
    // Stage s is consumed: order the reads before the async refill, then refill it.
    fence_proxy_async_smem();
    __syncwarp();
    if (j + stages < njobs) issue(j + stages);
    if (c == nchunk - 1) {
#pragma unroll
      for (int t = 0; t < M; t++)
#pragma unroll
        for (int r = 0; r < kSRows; r++) acc[t][r] = warp_sum(acc[t][r]);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kSRows; r++) {
          if ((uint32_t)r < rows) {
#pragma unroll
            for (int t = 0; t < M; t++) y[p.y_off + (uint64_t)t * p.y_stride + p.n_off + row0 + r] = acc[t][r];
          }
        }
      }
#pragma unroll
      for (int t = 0; t < M; t++)
#pragma unroll
        for (int r = 0; r < kSRows; r++) acc[t][r] = 0.f;
    }
  }
  if (!ok) {
    // Drain the copies this warp still has in flight (bounded) before exiting.
    if (lane == 0) report_timeout(&g_dev_error);
    const uint32_t last = min(njobs, j + stages);
    for (uint32_t k = j; k < last; k++) (void)mbar_wait_bounded(&bars[k % stages], (k / stages) & 1);
  }
}

struct StreamCfg {
  uint32_t chunk, stages, smem;
};

// Chooses chunk bytes and stages for the streaming kernel, or returns false if the
// shape cannot use it (row bytes not a multiple of 256, x not fitting next to 2 stages).
template <typename ST>
bool stream_cfg(int dtype, uint32_t k, int M, StreamCfg* c) {
  const uint32_t epb = dtype == SNL_Q8_0 ? 1 : 2;
  const uint32_t row_bytes = k / epb;
  if (row_bytes % 256) return false;
  uint32_t chunk = 1024;
  while (row_bytes % chunk) chunk /= 2;
  const uint32_t sc = chunk * epb / 32 * sizeof(ST);
  const uint32_t stage = kSRows * (chunk + sc);
  const uint32_t xb = align16u(M * k * 4);
  const uint32_t limit = 227 * 1024;
  for (uint32_t s = kSMaxStages; s >= 2; s--) {
    const uint32_t total = xb + kSWarps * s * stage + kSWarps * kSMaxStages * 8;
    if (total <= limit) {
      *c = StreamCfg{chunk, s, total};
      return true;
    }
  }
  return false;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <int DT, int M, typename ST>
int launch_stream(const snl_mat_p& p, const float* x, const void* wq, const ST* ws, float* y, const StreamCfg& c,
                  cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemv_stream_kernel<DT, M, ST>;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_stream: smem attribute");
    attr_set[dev] = true;
  }
  const uint32_t groups = (p.n + kSRows - 1) / kSRows;
  const uint32_t grid = std::min<uint32_t>((groups + kSWarps - 1) / kSWarps, (uint32_t)num_sms());
  kern<<<grid, kSWarps * 32, c.smem, s>>>(p, x, static_cast<const uint8_t*>(wq), ws, y, c.chunk, c.stages);
  SNL_LAUNCH_CHECK("gemv_stream");
  return SNL_OK;
}

template <int DT, typename ST>
int launch_mat_t(const snl_mat_p& p, uint32_t rows_m, const float* x, const void* wq, const ST* ws, float* y,
                 cudaStream_t s) {
  const uint8_t* w = static_cast<const uint8_t*>(wq);
  StreamCfg sc;
  if (rows_m <= 2 && !getenv("SNL_GEMV_DIRECT") && stream_cfg<ST>(DT, p.k, (int)rows_m, &sc)) {
    return rows_m == 1 ? launch_stream<DT, 1, ST>(p, x, wq, ws, y, sc, s) : launch_stream<DT, 2, ST>(p, x, wq, ws, y, sc, s);
  }
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
               int scale_f16, float* y, cudaStream_t s, uint32_t rows_m, const __half* wplanes) {
  (void)st;
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return fail(SNL_E_INVALID, "mat: dtype must be Q8_0 or Q4_0");
  if (p.k == 0 || p.k % 32) return fail(SNL_E_INVALID, "mat: k must be a positive multiple of 32");
  if ((p.x_off % 4) || (p.x_stride % 4)) return fail(SNL_E_INVALID, "mat: x_off and x_stride must be multiples of 4");
  if (((uintptr_t)x % 16) || ((uintptr_t)wq % 16)) return fail(SNL_E_INVALID, "mat: x and wq must be 16-byte aligned");
  if (rows_m == 0 || p.n == 0) return SNL_OK;
  // Prefill-sized steps run on the tcgen05 tensor cores.
  if (rows_m >= 8 && !scale_f16 && gemm_tc_enabled())
    return launch_gemm_tc(dtype, p, rows_m, x, wq, static_cast<const float*>(ws), y, s, wplanes);
  if (dtype == SNL_Q8_0) {
    return scale_f16 ? launch_mat_t<SNL_Q8_0, __half>(p, rows_m, x, wq, (const __half*)ws, y, s)
                     : launch_mat_t<SNL_Q8_0, float>(p, rows_m, x, wq, (const float*)ws, y, s);
  }
  return scale_f16 ? launch_mat_t<SNL_Q4_0, __half>(p, rows_m, x, wq, (const __half*)ws, y, s)
                   : launch_mat_t<SNL_Q4_0, float>(p, rows_m, x, wq, (const float*)ws, y, s);
}

}  // namespace snl

extern "C" int snl_device_error(int clear) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, snl::g_dev_error, sizeof(int));
  if (e != cudaSuccess) return snl::cuda_fail(e, "snl_device_error");
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(snl::g_dev_error, &z, sizeof(int));
  }
  return v;
}

extern "C" int snl_mat(int dtype, const snl_step_u* step, const snl_mat_p* p, const float* x, const void* wq,
                       const float* ws, float* y, void* stream) {
  if (!step || !p || !x || !wq || !ws || !y) return snl::fail(SNL_E_INVALID, "snl_mat: null argument");
  const uint32_t rows_m = p->m_one > 0 ? p->m_one : step->m;
  return snl::launch_mat(dtype, snl::step_val(*step), *p, x, wq, ws, 0, y, (cudaStream_t)stream, rows_m);
}
extern "C" int snl_weight_planes(int dtype, uint32_t n, uint32_t k, const void* wq, const float* ws, void* planes,
                                 void* stream) {
  if (!wq || !ws || !planes) return snl::fail(SNL_E_INVALID, "snl_weight_planes: null argument");
  return snl::launch_weight_planes(dtype, n, k, wq, ws, static_cast<__half*>(planes), (cudaStream_t)stream);
}
extern "C" int snl_mat_wplanes(int dtype, const snl_step_u* step, const snl_mat_p* p, const float* x, const void* wq,
                               const float* ws, const void* planes, float* y, void* stream) {
  if (!step || !p || !x || !wq || !ws || !planes || !y) return snl::fail(SNL_E_INVALID, "snl_mat_wplanes: null argument");
  const uint32_t rows_m = p->m_one > 0 ? p->m_one : step->m;
  return snl::launch_mat(dtype, snl::step_val(*step), *p, x, wq, ws, 0, y, (cudaStream_t)stream, rows_m,
                         static_cast<const __half*>(planes));
}
