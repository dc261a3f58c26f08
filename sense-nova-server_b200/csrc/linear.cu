// Gated DeltaNet linear attention (linear.wgsl: conv :38-66, delta :84-140).
//
// proj rows: qkv[conv_dim] | z[n_v*128] | b[n_v] | a[n_v]; after the causal conv,
// qkv splits as q[n_k*128] | k[n_k*128] | v[n_v*128]. lw = conv w [conv_dim*4] |
// A_log[n_v] | dt_bias[n_v] | norm w[128]. The recurrent state of value head h is a
// [128 (key dim i), 128 (value dim j)] f32 matrix; column j evolves independently of
// the other columns given the head's q, k, beta and decay.
#include "common.cuh"
#include "ptx.cuh"

namespace snl {
namespace {

constexpr uint32_t DK = 128, DV = 128;

// conv: one thread per channel walking the tokens of the step.
__global__ void conv_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj, float* __restrict__ conv_out,
                            float* __restrict__ cs, const float* __restrict__ lw, float* __restrict__ ck) {
  const snl_step_u st = load_step(sr);
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t cd = p.conv_dim;
  if (c >= cd) return;
  const float4 w = *reinterpret_cast<const float4*>(lw + (uint64_t)c * 4);
  float r0 = cs[c], r1 = cs[cd + c], r2 = cs[2 * cd + c];
  for (uint32_t m = 0; m < st.m; m++) {
    const float cur = proj[(uint64_t)m * p.proj_stride + c];
    const float o = fmaf(w.w, cur, fmaf(w.z, r2, fmaf(w.y, r1, w.x * r0)));
    conv_out[(uint64_t)m * cd + c] = o / (1.0f + __expf(-o));
    r0 = r1;
    r1 = r2;
    r2 = cur;
    if (m + 1 == st.ckpt) {
      ck[c] = r0;
      ck[cd + c] = r1;
      ck[2 * cd + c] = r2;
    }
  }
  cs[c] = r0;
  cs[cd + c] = r1;
  cs[2 * cd + c] = r2;
}

// delta: CTA per value head, thread j owns state column j (128 floats in registers).
__global__ void __launch_bounds__(128) delta_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj,
                                                    const float* __restrict__ conv_out, float* __restrict__ state,
                                                    const float* __restrict__ lw, float* __restrict__ out,
                                                    float* __restrict__ state_ckpt, XOut xo) {
  __shared__ float qs[DK], ks[DK];
  __shared__ float red[32];
  const snl_step_u st = load_step(sr);
  const uint32_t h = blockIdx.x, j = threadIdx.x;
  const uint32_t kh = h / (p.n_v / p.n_k);
  const uint32_t cd = p.conv_dim, key_dim = p.n_k * DK;
  const uint64_t sbase = (uint64_t)h * DK * DV;
  const float a_log = lw[(uint64_t)cd * 4 + h];
  const float dt_bias = lw[(uint64_t)cd * 4 + p.n_v + h];
  const float norm_w = lw[(uint64_t)cd * 4 + 2 * p.n_v + j];
  const float neg_a = -__expf(a_log);
  const uint32_t z_off = cd, b_off = cd + p.n_v * DV, a_off = b_off + p.n_v;
  float S[DK];
#pragma unroll
  for (uint32_t i = 0; i < DK; i++) S[i] = state[sbase + i * DV + j];
  for (uint32_t m = 0; m < st.m; m++) {
    const uint64_t crow = (uint64_t)m * cd;
    const float qv = conv_out[crow + kh * DK + j];
    const float kv = conv_out[crow + key_dim + kh * DK + j];
    const float vv = conv_out[crow + 2 * key_dim + h * DV + j];
    const float sq = block_sum(qv * qv, red);
    const float sk = block_sum(kv * kv, red);
    qs[j] = qv * rsqrtf(sq + 1e-6f) * rsqrtf((float)DK);
    ks[j] = kv * rsqrtf(sk + 1e-6f);
    __syncthreads();
    const uint64_t prow = (uint64_t)m * p.proj_stride;
    const float beta = 1.0f / (1.0f + __expf(-proj[prow + b_off + h]));
    const float araw = proj[prow + a_off + h] + dt_bias;
    const float sp = araw <= 20.0f ? log1pf(__expf(araw)) : araw;
    const float decay = __expf(neg_a * sp);
    float kv_mem = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < DK; i++) {
      S[i] *= decay;
      kv_mem = fmaf(S[i], ks[i], kv_mem);
    }
    const float dlt = (vv - kv_mem) * beta;
    float o = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < DK; i++) {
      S[i] = fmaf(ks[i], dlt, S[i]);
      o = fmaf(S[i], qs[i], o);
    }
    const float var_o = block_sum(o * o, red) / (float)DV;
    const float z = proj[prow + z_off + h * DV + j];
    const float ov = o * rsqrtf(var_o + p.eps) * norm_w * (z / (1.0f + __expf(-z)));
    out[(uint64_t)m * p.n_v * DV + h * DV + j] = ov;
    if (xo.planes) xout_store(xo, m, h * DV + j, ov);
    if (m + 1 == st.ckpt) {
#pragma unroll
      for (uint32_t i = 0; i < DK; i++) state_ckpt[sbase + i * DV + j] = S[i];
    }
    __syncthreads();
  }
#pragma unroll
  for (uint32_t i = 0; i < DK; i++) state[sbase + i * DV + j] = S[i];
}

// conv + delta in one kernel (the engine's form of linear.wgsl:38-140): CTA per value
// head h, kCdParts x 128 threads. Thread (part, j) keeps rows [32*part, 32*part + 32) of
// state column j in registers; the four parts of a column add their partial dot
// products (kv_mem, then the output) in shared memory in part order. The causal conv +
// SiLU of the head's q, k and v channel j runs in parts 0, 1 and 2 (weights and the
// 3-token conv state in registers, no conv_out buffer); part 3 holds the output gate z
// and finishes column j (gated RMSNorm over the head's 128 outputs). The q/k channels of
// key head kh are shared by the n_v/n_k value heads of its group: the first of them owns
// their conv state and checkpoint writes.
constexpr uint32_t kCdParts = 4;
constexpr uint32_t kCdRows = DK / kCdParts;

__global__ void __launch_bounds__(DV * kCdParts) conv_delta_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj,
                                                                  float* __restrict__ conv_state, float* __restrict__ state,
                                                                  const float* __restrict__ lw, float* __restrict__ out,
                                                                  float* __restrict__ conv_ckpt,
                                                                  float* __restrict__ state_ckpt, XOut xo) {
  pdl_trigger();
  pdl_wait();
  __shared__ float raw[3][DK];             // conv outputs of q, k, v (per channel)
  __shared__ float part[2][kCdParts][DV];  // partial kv_mem, partial output
  __shared__ float scal[4];                // 1/|q|, 1/|k|, beta, decay
  __shared__ float red[4];
  const snl_step_u st = load_step(sr);
  const uint32_t h = blockIdx.x, tid = threadIdx.x, j = tid % DV, pq = tid / DV;
  const uint32_t group = p.n_v / p.n_k;
  const uint32_t kh = h / group;
  const bool owns = pq == 2 || (h % group) == 0;  // writes this thread's conv state
  const uint32_t cd = p.conv_dim, key_dim = p.n_k * DK;
  const uint32_t z_off = cd, b_off = cd + p.n_v * DV, a_off = b_off + p.n_v;
  // this thread's conv channel (parts 0..2): q, k or v channel j
  const uint32_t ch = pq == 0 ? kh * DK + j : pq == 1 ? key_dim + kh * DK + j : 2 * key_dim + h * DV + j;
  float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
  float r0 = 0.f, r1 = 0.f, r2 = 0.f;
  if (pq < 3) {
    cw = *reinterpret_cast<const float4*>(lw + (uint64_t)ch * 4);
    r0 = conv_state[ch];
    r1 = conv_state[(uint64_t)cd + ch];
    r2 = conv_state[(uint64_t)2 * cd + ch];
  }
  const uint64_t sbase = (uint64_t)h * DK * DV + (uint64_t)pq * kCdRows * DV + j;
  float S[kCdRows];
#pragma unroll
  for (uint32_t i = 0; i < kCdRows; i++) S[i] = state[sbase + i * DV];
  const float norm_w = lw[(uint64_t)cd * 4 + 2 * p.n_v + j];
  const float dt_bias = lw[(uint64_t)cd * 4 + p.n_v + h];
  const float neg_a = -__expf(lw[(uint64_t)cd * 4 + h]);
  const float inv_sqrt_dk = rsqrtf((float)DK);

  for (uint32_t m = 0; m < st.m; m++) {
    const uint64_t prow = (uint64_t)m * p.proj_stride;
    float zg = 0.f;
    if (pq < 3) {
      const float cur = proj[prow + ch];
      const float o = fmaf(cw.w, cur, fmaf(cw.z, r2, fmaf(cw.y, r1, cw.x * r0)));
      raw[pq][j] = o / (1.0f + __expf(-o));
      r0 = r1;
      r1 = r2;
      r2 = cur;
      if (m + 1 == st.ckpt && owns) {
        conv_ckpt[ch] = r0;
        conv_ckpt[(uint64_t)cd + ch] = r1;
        conv_ckpt[(uint64_t)2 * cd + ch] = r2;
      }
    } else {
      const float z = proj[prow + z_off + h * DV + j];
      zg = z / (1.0f + __expf(-z));
      if (j == 0) {
        scal[2] = 1.0f / (1.0f + __expf(-proj[prow + b_off + h]));
        const float araw = proj[prow + a_off + h] + dt_bias;
        const float sp = araw <= 20.0f ? log1pf(__expf(araw)) : araw;
        scal[3] = __expf(neg_a * sp);
      }
    }
    __syncthreads();
    // |q| and |k| over the head's 128 channels (warp 0: q, warp 4: k).
    if (tid < 32 || (tid >= DV && tid < DV + 32)) {
      const float* v = raw[tid < 32 ? 0 : 1];
      const uint32_t l = tid & 31;
      float ss = 0.f;
#pragma unroll
      for (uint32_t c = 0; c < DK / 32; c++) ss = fmaf(v[l + 32 * c], v[l + 32 * c], ss);
      ss = warp_sum(ss);
      if (l == 0) scal[tid < 32 ? 0 : 1] = rsqrtf(ss + 1e-6f);
    }
    __syncthreads();
    const float rq = scal[0] * inv_sqrt_dk, rk = scal[1], beta = scal[2], decay = scal[3];
    float kvp = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < kCdRows; i++) {
      S[i] *= decay;
      kvp = fmaf(S[i], raw[1][pq * kCdRows + i] * rk, kvp);
    }
    part[0][pq][j] = kvp;
    __syncthreads();
    const float kv_mem = ((part[0][0][j] + part[0][1][j]) + part[0][2][j]) + part[0][3][j];
    const float dlt = (raw[2][j] - kv_mem) * beta;
    float op = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < kCdRows; i++) {
      S[i] = fmaf(raw[1][pq * kCdRows + i] * rk, dlt, S[i]);
      op = fmaf(S[i], raw[0][pq * kCdRows + i] * rq, op);
    }
    part[1][pq][j] = op;
    if (m + 1 == st.ckpt) {
#pragma unroll
      for (uint32_t i = 0; i < kCdRows; i++) state_ckpt[sbase + i * DV] = S[i];
    }
    __syncthreads();
    float o = 0.f;
    if (pq == 3) {
      o = ((part[1][0][j] + part[1][1][j]) + part[1][2][j]) + part[1][3][j];
      const float w2 = warp_sum(o * o);
      if ((tid & 31) == 0) red[(tid - 3 * DV) / 32] = w2;
    }
    __syncthreads();
    if (pq == 3) {
      const float var_o = (((red[0] + red[1]) + red[2]) + red[3]) / (float)DV;
      const float ov = o * rsqrtf(var_o + p.eps) * norm_w * zg;
      out[(uint64_t)m * p.n_v * DV + h * DV + j] = ov;
      if (xo.planes) xout_store(xo, m, h * DV + j, ov);
    }
  }
  if (pq < 3 && owns) {
    conv_state[ch] = r0;
    conv_state[(uint64_t)cd + ch] = r1;
    conv_state[(uint64_t)2 * cd + ch] = r2;
  }
#pragma unroll
  for (uint32_t i = 0; i < kCdRows; i++) state[sbase + i * DV] = S[i];
}

}  // namespace

static int check_lin(const snl_lin_p& p) {
  if (p.n_k == 0 || p.n_v == 0 || p.n_v % p.n_k) return fail(SNL_E_UNSUPPORTED, "linear: n_v must be a multiple of n_k");
  if (p.conv_dim != 2 * p.n_k * DK + p.n_v * DV) return fail(SNL_E_UNSUPPORTED, "linear: conv_dim mismatch");
  return SNL_OK;
}

int launch_conv(StepRef st, const snl_lin_p& p, const float* proj, float* conv_out, float* conv_state, const float* lw,
                float* conv_ckpt, cudaStream_t s) {
  if (int rc = check_lin(p)) return rc;
  conv_kernel<<<(p.conv_dim + 255) / 256, 256, 0, s>>>(st, p, proj, conv_out, conv_state, lw, conv_ckpt);
  SNL_LAUNCH_CHECK("conv");
  return SNL_OK;
}

int launch_delta(StepRef st, const snl_lin_p& p, const float* proj, const float* conv_out, float* state,
                 const float* lw, float* out, float* state_ckpt, cudaStream_t s, XOut xo) {
  if (int rc = check_lin(p)) return rc;
  delta_kernel<<<p.n_v, DV, 0, s>>>(st, p, proj, conv_out, state, lw, out, state_ckpt, xo);
  SNL_LAUNCH_CHECK("delta");
  return SNL_OK;
}

int launch_conv_delta(StepRef st, const snl_lin_p& p, const float* proj, float* conv_state, float* state,
                      const float* lw, float* out, float* conv_ckpt, float* state_ckpt, cudaStream_t s, XOut xo) {
  if (int rc = check_lin(p)) return rc;
  SNL_PDL_LAUNCH("conv_delta_kernel", conv_delta_kernel, dim3(p.n_v), dim3(DV * kCdParts), (size_t)(0), s, st, p, proj, conv_state, state, lw, out, conv_ckpt, state_ckpt, xo);
  return SNL_OK;
}

}  // namespace snl

extern "C" int snl_conv(const snl_step_u* step, const snl_lin_p* p, const float* proj, float* conv_out,
                        float* conv_state, const float* lw, float* conv_ckpt, void* stream) {
  if (!step || !p || !proj || !conv_out || !conv_state || !lw) return snl::fail(SNL_E_INVALID, "snl_conv: null argument");
  if (step->ckpt > 0 && !conv_ckpt) return snl::fail(SNL_E_INVALID, "snl_conv: ckpt needs conv_ckpt");
  return snl::launch_conv(snl::step_val(*step), *p, proj, conv_out, conv_state, lw, conv_ckpt, (cudaStream_t)stream);
}
extern "C" int snl_delta(const snl_step_u* step, const snl_lin_p* p, const float* proj, const float* conv_out,
                         float* state, const float* lw, float* out, float* state_ckpt, void* stream) {
  if (!step || !p || !proj || !conv_out || !state || !lw || !out)
    return snl::fail(SNL_E_INVALID, "snl_delta: null argument");
  if (step->ckpt > 0 && !state_ckpt) return snl::fail(SNL_E_INVALID, "snl_delta: ckpt needs state_ckpt");
  return snl::launch_delta(snl::step_val(*step), *p, proj, conv_out, state, lw, out, state_ckpt, (cudaStream_t)stream);
}
extern "C" int snl_conv_delta(const snl_step_u* step, const snl_lin_p* p, const float* proj, float* conv_state,
                              float* state, const float* lw, float* out, float* conv_ckpt, float* state_ckpt,
                              void* stream) {
  if (!step || !p || !proj || !conv_state || !state || !lw || !out)
    return snl::fail(SNL_E_INVALID, "snl_conv_delta: null argument");
  if (step->ckpt > 0 && (!conv_ckpt || !state_ckpt)) return snl::fail(SNL_E_INVALID, "snl_conv_delta: ckpt needs buffers");
  return snl::launch_conv_delta(snl::step_val(*step), *p, proj, conv_state, state, lw, out, conv_ckpt, state_ckpt,
                                (cudaStream_t)stream);
}
