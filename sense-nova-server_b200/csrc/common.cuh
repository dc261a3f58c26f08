// Shared definitions of the sm_100a kernels and the C ABI.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "snl_b200.h"

namespace snl {

// Error reporting: a thread-local message behind snl_last_error().
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
void count_launch(uint64_t n = 1);

#define SNL_CUDA_TRY(expr)                                       \
  do {                                                           \
    cudaError_t _e = (expr);                                     \
    if (_e != cudaSuccess) return ::snl::cuda_fail(_e, #expr);   \
  } while (0)

// Returns a non-zero status code from the enclosing function.
#define SNL_TRY(expr)          \
  do {                         \
    int _rc = (expr);          \
    if (_rc) return _rc;       \
  } while (0)

// Checks the launch that was just issued and counts it.
#define SNL_LAUNCH_CHECK(what)                                   \
  do {                                                           \
    cudaError_t _e = cudaGetLastError();                         \
    if (_e != cudaSuccess) return ::snl::cuda_fail(_e, what);    \
    ::snl::count_launch();                                       \
  } while (0)

// A step descriptor passed to kernels: either by value (kernel-level C ABI) or
// through a device pointer (engine graphs, where pos0/parts change between replays
// while the captured launch stays the same, like the reference's `step` uniform).
// A graph is captured per (rows, checkpoint) pair, so m and ckpt of the device copy
// always equal those of the host copy passed by value: kernels take them from the
// argument and read only pos0 and parts from device memory, so a kernel's loop over the
// step's rows does not wait for that load.
struct StepRef {
  const snl_step_u* dev;
  snl_step_u val;
};
__device__ __forceinline__ snl_step_u load_step(const StepRef& s) {
  if (s.dev) {
    snl_step_u v;
    v.m = s.val.m;
    v.ckpt = s.val.ckpt;
    v.pos0 = s.dev->pos0;
    v.parts = s.dev->parts;
    return v;
  }
  return s.val;
}
inline StepRef step_val(const snl_step_u& v) { return StepRef{nullptr, v}; }
inline StepRef step_dev(const snl_step_u* d, const snl_step_u& host_copy) { return StepRef{d, host_copy}; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); every thread gets the sum.
__device__ __forceinline__ float block_sum(float v, float* sh32) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh32[wid] = v;
  __syncthreads();
  float t = lane < nw ? sh32[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

// 16-byte streaming load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Optional second output of a kernel that produces a GEMV input: the x planes of the
// tensor-core GEMV (hi/lo fp16 halves of x / 16, plane 2t = hi, 2t+1 = lo of token t).
struct XOut {
  __half* planes = nullptr;
  uint32_t stride = 0;
};
__device__ __forceinline__ void xout_store(const XOut& xo, uint32_t t, uint32_t i, float v) {
  const float vs = v * (1.0f / 16.0f);
  const __half hi = __float2half_rn(vs);
  const __half lo = __float2half_rn(vs - __half2float(hi));
  xo.planes[(uint64_t)(2 * t) * xo.stride + i] = hi;
  xo.planes[(uint64_t)(2 * t + 1) * xo.stride + i] = lo;
}

// Stride of the per-group norm partials a residual-merging GEMV writes (gemv_mma.cuh).
constexpr int kRpStride = 12;

// Device address of the library's device error word (bit 0: a bounded wait gave up).
int device_error_word(int** out);

// Launches with programmatic stream serialization (unless SNL_NO_PDL is set): the
// kernel may begin while the previous kernel on the stream finishes. Every kernel
// launched this way calls pdl_wait() before it touches anything an earlier kernel wrote.
bool pdl_on();
int sm_count();  // SMs of the current device (cached per device)
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl_on() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
#define SNL_PDL_LAUNCH(what, ...)                                \
  do {                                                           \
    cudaError_t _e = ::snl::launch_pdl(__VA_ARGS__);             \
    if (_e != cudaSuccess) return ::snl::cuda_fail(_e, what);    \
    ::snl::count_launch();                                       \
  } while (0)

// Launch helpers implemented per kernel family (internal, not part of the C ABI).
size_t sample_scratch_bytes();
int launch_sample(const snl_sample_p& p, float* logits, uint32_t n, const uint32_t* hist_tok, const uint32_t* hist_cnt,
                  uint32_t n_hist, float u0, float u1, int64_t draft, uint32_t* out, void* scratch, cudaStream_t s);
// wplanes (optional): the matrix's weight planes (launch_weight_planes) for the
// prefill GEMM.
int launch_mat(int dtype, StepRef st, const snl_mat_p& p, const float* x, const void* wq, const void* ws,
               int scale_f16, float* y, cudaStream_t s, uint32_t rows_m_host, const __half* wplanes = nullptr);
// Prefill GEMM on the tcgen05 tensor cores (gemm_tc.cu), f32 scales, m token rows.
bool gemm_tc_enabled();
int launch_gemm_tc(int dtype, const snl_mat_p& p, uint32_t m, const float* x, const void* wq, const float* ws, float* y,
                   cudaStream_t s, const __half* wplanes = nullptr);
// Weight planes [2][n][k] fp16 (hi, lo of code * scale * 256) of a Q8_0/Q4_0 matrix: the
// prefill GEMM then loads its A operand by TMA instead of dequantizing it.
int launch_weight_planes(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, __half* planes,
                         cudaStream_t st);
int launch_branch_norm(StepRef st, const snl_layer_p& p, const float* x, const float* coef, const float* w,
                       float* out, uint32_t n_groups, cudaStream_t s, XOut xo = XOut());
// branch_norm mode 1 that first finishes the mHC router from nparts partial sums per
// token (written by the residual-merging GEMV) and writes coef.
int launch_branch_norm_router(StepRef st, const snl_layer_p& p, const float* x, float* coef, const float* w,
                              float* out, uint32_t n_groups, cudaStream_t s, XOut xo, const float* rpart,
                              uint32_t nparts, const float* router);
int launch_mhc_dots(StepRef st, const snl_layer_p& p, const float* x, const float* w, float* raw, uint32_t m,
                    cudaStream_t s);
int launch_mhc_finish(StepRef st, const snl_layer_p& p, const float* raw, const float* w, float* coef, uint32_t m,
                      cudaStream_t s);
// Engine mHC router: part holds m * 16 * 9 floats of scratch.
int launch_mhc_router(const snl_layer_p& p, const float* x, const float* w, float* part, float* coef, uint32_t m,
                      cudaStream_t s);
int launch_merge(StepRef st, const snl_layer_p& p, float* x, const float* coef, const float* br, uint32_t m,
                 cudaStream_t s);
int launch_swiglu(StepRef st, const snl_layer_p& p, const float* gu, float* act, uint32_t m, cudaStream_t s,
                  XOut xo = XOut());
int launch_attn_prep(StepRef st, const snl_attn_p& p, const float* proj, float* qbuf, uint32_t* kc, uint32_t* vc,
                     const float* norms, const uint32_t* rpos, uint32_t m, cudaStream_t s);
// Keys of one split-key part of a decode step's attention: one 8-key group per warp of
// attend_kernel (12 warps).
constexpr uint32_t kAttKeysPerPart = 96;
int launch_attend(StepRef st, const snl_attn_p& p, const float* proj, const float* qbuf, const uint32_t* kc,
                  const uint32_t* vc, float* out, float* partial, uint32_t m, uint32_t parts_grid, cudaStream_t s,
                  XOut xo = XOut());
// slots: the partial layout's part count (the attend grid's); 0 = the step's.
int launch_attn_combine(StepRef st, const snl_attn_p& p, const float* proj, const float* partial, float* out,
                        uint32_t m, cudaStream_t s, uint32_t slots, XOut xo = XOut());
int launch_conv(StepRef st, const snl_lin_p& p, const float* proj, float* conv_out, float* conv_state,
                const float* lw, float* conv_ckpt, cudaStream_t s);
int launch_delta(StepRef st, const snl_lin_p& p, const float* proj, const float* conv_out, float* state,
                 const float* lw, float* out, float* state_ckpt, cudaStream_t s, XOut xo = XOut());
// conv + delta fused (engine path): no conv_out buffer.
int launch_conv_delta(StepRef st, const snl_lin_p& p, const float* proj, float* conv_state, float* state,
                      const float* lw, float* out, float* conv_ckpt, float* state_ckpt, cudaStream_t s,
                      XOut xo = XOut());
// Chunked conv + delta for prefill steps (linear.cu): host row count m, no checkpoint.
constexpr uint32_t kChunkedMinRows = 16;  // steps of at least this many rows use it
int launch_conv_delta_chunked(uint32_t m, const snl_lin_p& p, const float* proj, float* conv_state, float* state,
                              const float* lw, float* out, float* conv_out, float* scratch, cudaStream_t s);
size_t conv_delta_chunked_scratch(const snl_lin_p& p, uint32_t m);
int launch_argmax(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, cudaStream_t s);
int launch_embed(const uint32_t* tokens, uint32_t m, const int8_t* q, const float* s_, uint32_t h, uint32_t vocab,
                 float* x, int* err_flag, cudaStream_t s, unsigned long long* step_ctr = nullptr);
int launch_gen_quant(uint64_t seed, const char* name, int dtype, size_t rows, size_t cols, void* q, float* s,
                     cudaStream_t st);
int launch_gen_f32(uint64_t seed, const char* name, uint32_t sub, size_t n, float mult, float offset, float* out,
                   cudaStream_t st);

}  // namespace snl
