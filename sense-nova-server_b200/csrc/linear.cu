// Gated DeltaNet linear attention (linear.wgsl: conv :38-66, delta :84-140).
//
// proj rows: qkv[conv_dim] | z[n_v*128] | b[n_v] | a[n_v]; after the causal conv,
// qkv splits as q[n_k*128] | k[n_k*128] | v[n_v*128]. lw = conv w [conv_dim*4] |
// A_log[n_v] | dt_bias[n_v] | norm w[128]. The recurrent state of value head h is a
// [128 (key dim i), 128 (value dim j)] f32 matrix; column j evolves independently of
// the other columns given the head's q, k, beta and decay.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace snl {
namespace {

constexpr uint32_t DK = 128, DV = 128;

// conv (linear.wgsl:38-66), token-parallel: thread (channel c, run of kConvTok tokens)
// reads the run's inputs and the three before it (from the carried state for tokens
// before the step) and writes SiLU(w . x) per token, the same expression as the
// sequential form. The carried state and the checkpoint are written afterwards by
// conv_state_kernel, once every thread has read the old state.
constexpr uint32_t kConvTok = 8;

__global__ void __launch_bounds__(256) conv_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj,
                                                   float* __restrict__ conv_out, const float* __restrict__ cs,
                                                   const float* __restrict__ lw) {
  const snl_step_u st = load_step(sr);
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x, cd = p.conv_dim;
  const uint32_t m0 = blockIdx.y * kConvTok;
  if (c >= cd || m0 >= st.m) return;
  const float4 w = *reinterpret_cast<const float4*>(lw + (uint64_t)c * 4);
  float xv[kConvTok + 3];
#pragma unroll
  for (uint32_t j = 0; j < kConvTok + 3; j++) {
    const int t = (int)(m0 + j) - 3;
    xv[j] = t < 0 ? cs[(uint64_t)(t + 3) * cd + c] : ((uint32_t)t < st.m ? proj[(uint64_t)t * p.proj_stride + c] : 0.f);
  }
#pragma unroll
  for (uint32_t j = 0; j < kConvTok; j++) {
    const uint32_t m = m0 + j;
    if (m >= st.m) break;
    const float o = fmaf(w.w, xv[j + 3], fmaf(w.z, xv[j + 2], fmaf(w.y, xv[j + 1], w.x * xv[j])));
    conv_out[(uint64_t)m * cd + c] = o / (1.0f + __expf(-o));
  }
}

// The carried conv state after the step (the last three inputs, older ones from the
// state before it) and, if ckpt > 0, the state after token ckpt - 1.
__global__ void __launch_bounds__(256) conv_state_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj,
                                                         float* __restrict__ cs, float* __restrict__ ck) {
  const snl_step_u st = load_step(sr);
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x, cd = p.conv_dim;
  if (c >= cd || st.m == 0) return;
  const float old[3] = {cs[c], cs[(uint64_t)cd + c], cs[(uint64_t)2 * cd + c]};
  auto x = [&](int t) { return t < 0 ? old[t + 3] : proj[(uint64_t)t * p.proj_stride + c]; };
  if (st.ckpt > 0 && ck) {
    const int k = (int)st.ckpt;
    ck[c] = x(k - 3);
    ck[(uint64_t)cd + c] = x(k - 2);
    ck[(uint64_t)2 * cd + c] = x(k - 1);
  }
  const int m = (int)st.m;
  const float n0 = x(m - 3), n1 = x(m - 2), n2 = x(m - 1);
  cs[c] = n0;
  cs[(uint64_t)cd + c] = n1;
  cs[(uint64_t)2 * cd + c] = n2;
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

// conv + delta for decode steps, kCsSplit CTAs per value head: CTA c of head h owns
// state columns [32c, 32c + 32) (the columns evolve independently given q, k, beta and
// decay). One thread-block cluster holds the CTAs of all value heads of a key head
// (group = n_v / n_k heads x kCsSplit, at most 8). Each CTA runs the causal conv + SiLU
// of the 128 q and 128 k channels of its key head (threads 0-127: q, 128-255: k) and of
// its own 32 v channels; thread (part p, column j) keeps rows [16p, 16p + 16) of state
// column j in registers and the 8 parts of a column add their partial dot products in
// shared memory in part order. The gated RMSNorm over a head's 128 outputs needs the
// sums of squares of its four CTAs: each CTA publishes its partial in shared memory and,
// after a cluster barrier, adds the head's four in rank order. The q/k conv state is
// read by every CTA of the cluster and written by rank 0 after a cluster barrier; the v
// conv state by the CTA that owns the column.
constexpr uint32_t kCsCols = 32;
constexpr uint32_t kCsSplit = DV / kCsCols;
constexpr uint32_t kCsParts = 8;
constexpr uint32_t kCsRows = DK / kCsParts;
constexpr uint32_t kCsThreads = kCsCols * kCsParts;  // 256 = q and k channels of the head
static_assert(kCsThreads == 2 * DK, "one conv thread per q and k channel");

__global__ void __launch_bounds__(kCsThreads)
    conv_delta_split_kernel(StepRef sr, snl_lin_p p, const float* __restrict__ proj, float* __restrict__ conv_state,
                            float* __restrict__ state, const float* __restrict__ lw, float* __restrict__ out,
                            float* __restrict__ conv_ckpt, float* __restrict__ state_ckpt, XOut xo) {
  namespace cg = cooperative_groups;
  pdl_trigger();
  __shared__ float qk[2][DK];                 // normalised-later conv outputs of q and k
  __shared__ float vz[2][kCsCols];            // conv output of v, SiLU(z) of this CTA's columns
  __shared__ float part[2][kCsParts][kCsCols];  // partial kv_mem, partial output
  __shared__ float red[8];                    // warp sums of squares: q (0-3), k (4-7)
  __shared__ float scal[2];                   // beta, decay
  __shared__ float sq_out;                    // this CTA's sum of squared outputs (read by the cluster)
  cg::cluster_group cluster = cg::this_cluster();
  const uint32_t rank = cluster.block_rank();
  const uint32_t h = blockIdx.x / kCsSplit, c0 = (blockIdx.x % kCsSplit) * kCsCols;
  const uint32_t head_rank0 = rank - rank % kCsSplit;  // rank of this head's first CTA
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t pp = tid / kCsCols, j = tid % kCsCols;  // state part, column within the CTA
  const uint32_t group = p.n_v / p.n_k, kh = h / group;
  const uint32_t cd = p.conv_dim, key_dim = p.n_k * DK;
  const uint32_t z_off = cd, b_off = cd + p.n_v * DV, a_off = b_off + p.n_v;
  // Constants (weights) before the wait: this thread's q/k conv channel, and for threads
  // 0-31 the v conv channel of column c0 + tid.
  const uint32_t ch = tid < DK ? kh * DK + tid : key_dim + kh * DK + (tid - DK);
  const bool qk_owner = rank == 0;
  const bool has_v = tid < kCsCols;
  const uint32_t vch = 2 * key_dim + h * DV + c0 + (has_v ? tid : 0);
  const float4 cw = *reinterpret_cast<const float4*>(lw + (uint64_t)ch * 4);
  const float4 cwv = *reinterpret_cast<const float4*>(lw + (uint64_t)vch * 4);
  const float norm_w = lw[(uint64_t)cd * 4 + 2 * p.n_v + c0 + j];
  const float dt_bias = lw[(uint64_t)cd * 4 + p.n_v + h];
  const float neg_a = -__expf(lw[(uint64_t)cd * 4 + h]);
  const float inv_sqrt_dk = rsqrtf((float)DK);
  // The conv state and this thread's rows of the recurrent state are loaded before the
  // wait: only this layer's kernel of an earlier step wrote them (each step starts after
  // the previous one has finished), so they do not depend on the kernels this one waits
  // for.
  const snl_step_u st = load_step(sr);
  float r0 = conv_state[ch], r1 = conv_state[(uint64_t)cd + ch], r2 = conv_state[(uint64_t)2 * cd + ch];
  float v0 = 0.f, v1 = 0.f, v2 = 0.f;
  if (has_v) {
    v0 = conv_state[vch];
    v1 = conv_state[(uint64_t)cd + vch];
    v2 = conv_state[(uint64_t)2 * cd + vch];
  }
  const uint64_t sbase = (uint64_t)h * DK * DV + (uint64_t)pp * kCsRows * DV + c0 + j;
  float S[kCsRows];
#pragma unroll
  for (uint32_t i = 0; i < kCsRows; i++) S[i] = state[sbase + i * DV];
  pdl_wait();

  for (uint32_t m = 0; m < st.m; m++) {
    const uint64_t prow = (uint64_t)m * p.proj_stride;
    {
      const float cur = proj[prow + ch];
      const float o = fmaf(cw.w, cur, fmaf(cw.z, r2, fmaf(cw.y, r1, cw.x * r0)));
      const float so = o / (1.0f + __expf(-o));
      qk[tid / DK][tid % DK] = so;
      r0 = r1;
      r1 = r2;
      r2 = cur;
      const float ss = warp_sum(so * so);
      if (lane == 0) red[warp] = ss;
    }
    if (has_v) {
      const float cur = proj[prow + vch];
      const float o = fmaf(cwv.w, cur, fmaf(cwv.z, v2, fmaf(cwv.y, v1, cwv.x * v0)));
      vz[0][tid] = o / (1.0f + __expf(-o));
      v0 = v1;
      v1 = v2;
      v2 = cur;
    } else if (tid < 2 * kCsCols) {
      const float z = proj[prow + z_off + h * DV + c0 + (tid - kCsCols)];
      vz[1][tid - kCsCols] = z / (1.0f + __expf(-z));
    } else if (tid == 2 * kCsCols) {
      scal[0] = 1.0f / (1.0f + __expf(-proj[prow + b_off + h]));
      const float araw = proj[prow + a_off + h] + dt_bias;
      const float sp = araw <= 20.0f ? log1pf(__expf(araw)) : araw;
      scal[1] = __expf(neg_a * sp);
    }
    if (m + 1 == st.ckpt) {
      if (qk_owner) {
        conv_ckpt[ch] = r0;
        conv_ckpt[(uint64_t)cd + ch] = r1;
        conv_ckpt[(uint64_t)2 * cd + ch] = r2;
      }
      if (has_v) {
        conv_ckpt[vch] = v0;
        conv_ckpt[(uint64_t)cd + vch] = v1;
        conv_ckpt[(uint64_t)2 * cd + vch] = v2;
      }
    }
    __syncthreads();
    const float rq = rsqrtf(((red[0] + red[1]) + (red[2] + red[3])) + 1e-6f) * inv_sqrt_dk;
    const float rk = rsqrtf(((red[4] + red[5]) + (red[6] + red[7])) + 1e-6f);
    const float beta = scal[0], decay = scal[1];
    const float* kr = &qk[1][pp * kCsRows];
    const float* qr = &qk[0][pp * kCsRows];
    float kvp = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < kCsRows; i++) {
      S[i] *= decay;
      kvp = fmaf(S[i], kr[i] * rk, kvp);
    }
    part[0][pp][j] = kvp;
    __syncthreads();
    float kv_mem = 0.f;
#pragma unroll
    for (uint32_t q = 0; q < kCsParts; q++) kv_mem += part[0][q][j];
    const float dlt = (vz[0][j] - kv_mem) * beta;
    float op = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < kCsRows; i++) {
      S[i] = fmaf(kr[i] * rk, dlt, S[i]);
      op = fmaf(S[i], qr[i] * rq, op);
    }
    part[1][pp][j] = op;
    if (m + 1 == st.ckpt) {
#pragma unroll
      for (uint32_t i = 0; i < kCsRows; i++) state_ckpt[sbase + i * DV] = S[i];
    }
    __syncthreads();
    float o = 0.f;
    if (warp == 0) {
#pragma unroll
      for (uint32_t q = 0; q < kCsParts; q++) o += part[1][q][j];
      const float w2 = warp_sum(o * o);
      if (lane == 0) sq_out = w2;
    }
    cluster.sync();
    if (warp == 0) {
      float tot = 0.f;
#pragma unroll
      for (uint32_t r = 0; r < kCsSplit; r++) tot += *cluster.map_shared_rank(&sq_out, head_rank0 + r);
      const float ov = o * rsqrtf(tot / (float)DV + p.eps) * norm_w * vz[1][j];
      const uint32_t col = h * DV + c0 + j;
      out[(uint64_t)m * p.n_v * DV + col] = ov;
      if (xo.planes) xout_store(xo, m, col, ov);
    }
    cluster.sync();  // sq_out and the shared arrays are reused by the next token
  }
  if (qk_owner) {
    conv_state[ch] = r0;
    conv_state[(uint64_t)cd + ch] = r1;
    conv_state[(uint64_t)2 * cd + ch] = r2;
  }
  if (has_v) {
    conv_state[vch] = v0;
    conv_state[(uint64_t)cd + vch] = v1;
    conv_state[(uint64_t)2 * cd + vch] = v2;
  }
#pragma unroll
  for (uint32_t i = 0; i < kCsRows; i++) state[sbase + i * DV] = S[i];
}

// ---------------------------------------------------------------------------
// Chunked form of the gated delta rule (prefill steps): the same recurrence as
// delta_kernel, regrouped over chunks of kDnC tokens so that most of the work is
// matrix products that run in parallel over (head, chunk). Within a chunk starting from
// state S0 (token t: normalised q_t, k_t, v_t, beta_t, log decay l_t, Lambda_t = sum of
// l_s for s <= t in the chunk, gamma_t = exp(Lambda_t)):
//   S_t   = gamma_t S0 + sum_{s<=t} (gamma_t/gamma_s) k_s d_s^T
//   d_t   = beta_t (v_t - S~_t^T k_t),  S~_t = (decayed S_{t-1})
//   => (I + L) D = diag(beta) (V - Gamma K S0),  L[t][s] = beta_t (gamma_t/gamma_s) k_t.k_s (s < t)
//   => D = U - W S0 with T = (I + L)^-1 diag(beta), W = T Gamma K, U = T V
//   o_t  = S_t^T q_t  =>  O = P S0 + R, P = Gamma Q - M W, R = M U,
//          M[t][s] = (gamma_t/gamma_s) q_t.k_s (s <= t)
//   S_C  = gamma_C S0 + Kd^T D,  Kd[s] = (gamma_C/gamma_s) k_s.
// dn_prep_tc_kernel builds each (head, chunk)'s record in parallel: R and U as f32,
// [P; W] and Kd^T already split into the fp16 hi / lo tiles that the scan's tensor-core
// products read, gamma_C and the scale of [P; W]. dn_scan_tc_kernel carries the state
// through the chunks (each 32-column slice of a head's state is independent, so a head
// spans 4 CTAs); dn_norm_kernel applies the gated RMSNorm of the outputs. Products use
// f32 accumulation of operands split into hi + lo parts.
// ---------------------------------------------------------------------------
constexpr uint32_t kDnC = 64;                 // tokens per chunk
constexpr uint32_t kDnCols = 32;              // state columns per scan CTA
// A chunk record, in floats: R [C][128] and U [C][128] (f32); [P; W] as 4 tiles of 16 KB
// (fp16 hi K blocks 0 and 1, then lo; rows 0-63 P, 64-127 W, K = the key dimension);
// Kd^T as 2 tiles (hi, lo; rows = the key dimension, K = token); then gamma_C and the
// [P; W] scale exponent. The tiles are the scan's shared-memory image (128-byte rows,
// 16-byte chunk c of row r at c ^ (r % 8)).
constexpr uint32_t kRecTile = 128 * 128 / 4;  // floats of one 16 KB tile
constexpr uint32_t kRecR = 0, kRecU = kDnC * DV, kRecPW = 2 * kDnC * DV, kRecKd = kRecPW + 4 * kRecTile,
                   kRecScal = kRecKd + 2 * kRecTile;
constexpr uint32_t kDnChunkFloats = kRecScal + 64;

struct DnScratch {
  float* chunks;  // [n_v][n_chunks][kDnChunkFloats]
};

// 16-byte asynchronous global -> shared copies (both addresses 16-byte aligned), committed
// in groups; cp_async_wait<n> returns when at most n groups are still in flight.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 3xTF32 tensor-core products (mma.sync m16n8k8, f32 accumulate): each f32 operand is
// split into tf32 hi + lo and hi*hi + hi*lo + lo*hi are accumulated, which keeps about
// fp32 accuracy (the dropped lo*lo term is below 2^-22 of the product).
__device__ __forceinline__ uint32_t tf32_of(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_of(x);
  lo = tf32_of(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Pre-split fragments: several output tiles that share their A rows (or B columns) split
// those once per k-step, and their MMAs, into independent accumulators, interleave. Per
// tile the MMAs run in the order of mma3_tf32, so the sums are the same bits.
__device__ __forceinline__ void split_a(const float* ar, uint32_t sa, uint32_t ah[4], uint32_t al[4]) {
  const float av[4] = {ar[0], ar[8 * sa], ar[4], ar[8 * sa + 4]};
#pragma unroll
  for (int i = 0; i < 4; i++) tf32_split(av[i], ah[i], al[i]);
}
__device__ __forceinline__ void split_b(float b0, float b1, uint32_t bh[2], uint32_t bl[2]) {
  tf32_split(b0, bh[0], bl[0]);
  tf32_split(b1, bh[1], bl[1]);
}
__device__ __forceinline__ void mma3_split(float d[4], const uint32_t ah[4], const uint32_t al[4], const uint32_t bh[2],
                                           const uint32_t bl[2]) {
  mma_tf32(d, al, bh[0], bh[1]);
  mma_tf32(d, ah, bl[0], bl[1]);
  mma_tf32(d, ah, bh[0], bh[1]);
}

constexpr uint32_t kPrT = 68;  // row stride (floats) of the 64 x 64 f32 blocks

// ---------------------------------------------------------------------------
// The chunk records on the tcgen05 tensor cores (dn_prep_tc_kernel, one CTA per (chunk,
// value head)). Its large products run as tcgen05.mma (kind::f16, M = 128, f32
// accumulators in tensor memory) on operands split into fp16 hi + lo, accumulating
// hi*hi + hi*lo + lo*hi (about 22 significant bits, the same scheme as the prefill GEMM;
// the dropped lo*lo term is below 2^-22 of each product). Every operand is scaled by a
// power of two first, so hi and lo stay normal fp16 numbers: 2^14 for the unit-norm
// q, k, Gamma K and Kd rows, and 2^(14 - e) for T, M T, V, P and W, where 2^e bounds the
// block's largest magnitude. The scales are exact and are taken out of the accumulators.
//   A: [K; Q] (128 x 128) times K^T (N = 64): rows 0-63 give K K^T, rows 64-127 Q K^T.
//   Then on the CUDA cores and mma.sync: L and M with their decays, X = (I + L)^-1,
//   T = X diag(beta), MT = M T (64 x 64 x 64).
//   C: [T; MT] (128 x 64) times [Gamma K | V] (N = 2 x 128): rows 0-63 give W = T Gamma K
//   and U = T V, rows 64-127 give M W and R = M U, so P = Gamma Q - M W.
// One thread issues the MMAs; all 8 warps split the operands before and read the
// accumulators (tcgen05.ld) after, meeting at CTA barriers and commit mbarriers.
// Shared memory (~101 KB, so two CTAs share an SM and a 512-row step's 256 CTAs run in
// one wave): 16 KB tiles of [128 rows][128 B] (one K block of 64 fp16; 16-byte chunk c
// of row r stored at c ^ (r % 8)):
//   [0, 64K):   [K; Q] hi (2 K blocks) and lo (2); later [T; MT] hi, lo and
//               (Gamma K)^T hi, lo;
//   [64K, ..):  X, M (then M T) and the inverse's scratch (f32); later V^T hi and lo.
// ---------------------------------------------------------------------------
constexpr uint32_t kPtTile = 128 * 128;
constexpr uint32_t kPtF32 = 2 * kDnC * kPrT * 4 + 3 * 16 * 16 * 4;  // X, M / MT, scratch
constexpr size_t kPrepTcSmem = 4 * kPtTile + (kPtF32 > 2 * kPtTile ? kPtF32 : 2 * kPtTile) + 1024;
constexpr uint32_t kPtTmemCols = 256;
constexpr float kPtUnit = 16384.0f;  // 2^14: scale of the unit-norm operands

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((127 + e) << 23); }
// 2^(14 - e) with 2^e > max: the scale that brings magnitudes up to max below 2^14.
__device__ __forceinline__ int pt_scale_exp(float amax) {
  int e = 0;
  if (amax > 0.f) (void)frexpf(amax, &e);
  return min(max(14 - e, -100), 100);
}
__device__ __forceinline__ uint32_t ph_pair(float a, float b, bool lo) {
  const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
  if (!lo) return (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
  const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
  return (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}
// Element k of row r of a [128 rows] x (K blocks of 64) tile set, as fp16 hi and lo.
__device__ __forceinline__ void pt_store1(uint8_t* hi, uint8_t* lo, uint32_t r, uint32_t k, float v) {
  const uint32_t off = (k >> 6) * kPtTile + r * 128 + (((((k & 63) >> 3) ^ (r & 7))) << 4) + ((k & 7) << 1);
  const __half h = __float2half_rn(v);
  *reinterpret_cast<__half*>(hi + off) = h;
  *reinterpret_cast<__half*>(lo + off) = __float2half_rn(v - __half2float(h));
}
// Elements k0 .. k0 + 7 (k0 % 8 == 0) of row r: one 16-byte chunk each of hi and lo.
__device__ __forceinline__ void pt_store8(uint8_t* hi, uint8_t* lo, uint32_t r, uint32_t k0, const float* v) {
  const uint32_t off = (k0 >> 6) * kPtTile + r * 128 + ((((k0 & 63) >> 3) ^ (r & 7)) << 4);
  uint4 h, l;
  h.x = ph_pair(v[0], v[1], false);
  h.y = ph_pair(v[2], v[3], false);
  h.z = ph_pair(v[4], v[5], false);
  h.w = ph_pair(v[6], v[7], false);
  l.x = ph_pair(v[0], v[1], true);
  l.y = ph_pair(v[2], v[3], true);
  l.z = ph_pair(v[4], v[5], true);
  l.w = ph_pair(v[6], v[7], true);
  *reinterpret_cast<uint4*>(hi + off) = h;
  *reinterpret_cast<uint4*>(lo + off) = l;
}

// One split product: kbs K blocks (64 each) of A and B into the accumulator at d.
__device__ __forceinline__ void pt_mma(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                       uint32_t kbs, uint32_t idesc) {
  for (uint32_t kb = 0; kb < kbs; kb++) {
#pragma unroll
    for (uint32_t kk = 0; kk < 4; kk++) {
      const uint32_t o = kb * kPtTile + kk * 32;  // 16 fp16 along K inside the swizzled row
      const uint64_t ah = sdesc<128>(a_hi + o), al = sdesc<128>(a_lo + o);
      const uint64_t bh = sdesc<128>(b_hi + o), bl = sdesc<128>(b_lo + o);
      tc_mma(d, ah, bh, idesc, (kb | kk) != 0);
      tc_mma(d, ah, bl, idesc, 1);
      tc_mma(d, al, bh, idesc, 1);
    }
  }
}

// Largest value of v over the CTA (every thread passes its own; all get the result).
__device__ __forceinline__ float pt_block_max(float v, float* sh8) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh8[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sh8[0];
#pragma unroll
  for (int w = 1; w < 8; w++) r = fmaxf(r, sh8[w]);
  return r;
}

__global__ void __launch_bounds__(256, 2) dn_prep_tc_kernel(uint32_t m, snl_lin_p p, const float* __restrict__ proj,
                                                            const float* __restrict__ conv_out,
                                                            const float* __restrict__ lw, float* __restrict__ chunks,
                                                            int* err) {
  extern __shared__ uint8_t pt_raw[];
  uint8_t* RA = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pt_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* RB = RA + 4 * kPtTile;
  float* X = reinterpret_cast<float*>(RB);  // [C][kPrT]: L, then X = (I + L)^-1, then T
  float* Mq = X + kDnC * kPrT;              // [C][kPrT]: M, then M T
  float* tmp = Mq + kDnC * kPrT;            // [3][16][16]
  __shared__ float lam[kDnC], beta[kDnC], elam[kDnC], rq[kDnC], rk[kDnC], red[8];
  __shared__ uint64_t bar[2];
  __shared__ uint32_t tmem_sh;
  const uint32_t c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t g = lane >> 2, t4 = lane & 3;
  const uint32_t t0 = c * kDnC, ce = min(kDnC, m - t0);
  const uint32_t kh = h / (p.n_v / p.n_k), cd = p.conv_dim, key_dim = p.n_k * DK;
  const uint32_t b_off = cd + p.n_v * DV, a_off = b_off + p.n_v;
  float* rec = chunks + ((uint64_t)h * gridDim.x + c) * kDnChunkFloats;
  float* Rg = rec + kRecR;
  float* Ug = rec + kRecU;
  uint8_t* PWg = reinterpret_cast<uint8_t*>(rec + kRecPW);
  uint8_t* KdTg = reinterpret_cast<uint8_t*>(rec + kRecKd);
  const float* qsrc = conv_out + kh * DK;
  const float* ksrc = conv_out + key_dim + kh * DK;
  const float* vsrc = conv_out + 2 * key_dim + h * DV;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_sh, kPtTmemCols);
  // beta and the log decay of each token.
  if (tid < kDnC) {
    const uint32_t t = tid;
    const float neg_a = -__expf(lw[(uint64_t)cd * 4 + h]);
    const float dt_bias = lw[(uint64_t)cd * 4 + p.n_v + h];
    float bt = 0.f, lt = 0.f;
    if (t < ce) {
      const uint64_t prow = (uint64_t)(t0 + t) * p.proj_stride;
      bt = 1.0f / (1.0f + __expf(-proj[prow + b_off + h]));
      const float araw = proj[prow + a_off + h] + dt_bias;
      const float sp = araw <= 20.0f ? log1pf(__expf(araw)) : araw;
      lt = neg_a * sp;
    }
    lam[t] = lt;
    beta[t] = bt;
  }
  // 1. The chunk's k (rows 0-63) and q (rows 64-127) rows, L2-normalised (lane l sums
  //    elements l + 32 u), times 2^14, split into the A tiles. Warp w takes rows w + 8 i
  //    in two batches of 8, every load of a batch in flight before the first sum.
#pragma unroll 1
  for (uint32_t b = 0; b < 2; b++) {
    float x[8][4];
#pragma unroll
    for (uint32_t i = 0; i < 8; i++) {
      const uint32_t r = warp + 8 * (8 * b + i), t = r & (kDnC - 1);
      const float* src = (r >= kDnC ? qsrc : ksrc) + (uint64_t)(t0 + t) * cd;
#pragma unroll
      for (int u = 0; u < 4; u++) x[i][u] = t < ce ? src[lane + 32 * u] : 0.f;
    }
#pragma unroll
    for (uint32_t i = 0; i < 8; i++) {
      const uint32_t r = warp + 8 * (8 * b + i), t = r & (kDnC - 1);
      const bool isq = r >= kDnC;
      float sq = 0.f;
#pragma unroll
      for (int u = 0; u < 4; u++) sq = fmaf(x[i][u], x[i][u], sq);
      sq = warp_sum(sq);
      const float rn = isq ? rsqrtf(sq + 1e-6f) * rsqrtf((float)DK) : rsqrtf(sq + 1e-6f);
      if (lane == 0) (isq ? rq : rk)[t] = rn;
#pragma unroll
      for (int u = 0; u < 4; u++) pt_store1(RA, RA + 2 * kPtTile, r, lane + 32 * u, x[i][u] * rn * kPtUnit);
    }
  }
  fence_proxy_async_smem();  // the tiles are read by the tensor cores (async proxy)
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const uint32_t a_base = smem_u32(RA);
  if (tid == 0) {
    pt_mma(tmem, a_base, a_base + 2 * kPtTile, a_base, a_base + 2 * kPtTile, 2, tc_idesc_f16(kDnC));
    tc_commit(&bar[0]);
  } else if (tid == 32) {
    float acc = 0.f;
    for (uint32_t t = 0; t < kDnC; t++) {
      acc += lam[t];
      lam[t] = acc;
    }
  }
  __syncthreads();
  if (tid < kDnC) elam[tid] = __expf(lam[tid]);
  bool ok = __syncthreads_and(mbar_wait_bounded(&bar[0], 0));
  tc_fence_after();
  // 2. L[t][s] = beta_t e^(lam_t - lam_s) k_t.k_s (s < t) and M[t][s] = e^(lam_t - lam_s) q_t.k_s
  //    (s <= t) from the accumulator: warp w reads lanes 32 (w % 4).. (the rows), columns
  //    32 (w / 4) ..
  if (ok) {
    const uint32_t quarter = warp & 3, half = warp >> 2;
    float v[32];
    tmem_ld32(tmem + ((quarter * 32) << 16) + 32 * half, v);
    const uint32_t row = quarter * 32 + lane, t = row & (kDnC - 1);
    const float unscale = 1.0f / (kPtUnit * kPtUnit);
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const uint32_t s2 = 32 * half + j;
      const float e = s2 <= t ? __expf(lam[t] - lam[s2]) : 0.f;
      const float gv = v[j] * unscale;
      if (row < kDnC) X[t * kPrT + s2] = s2 < t ? beta[t] * e * gv : 0.f;
      else Mq[t * kPrT + s2] = s2 <= t ? e * gv : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  // 3. X = (I + L)^-1: diagonal 16-blocks by forward substitution (half a warp per
  //    block, lane c owns column c), then the off-diagonal blocks row by row,
  //    X_ij = -X_ii sum_{k=j}^{i-1} L_ik X_kj for all j < i at once.
  if (warp < 2) {
    const uint32_t bb = warp * 2 + (lane >> 4), cc = lane & 15, o = 16 * bb;
    float x[16];
#pragma unroll
    for (uint32_t r = 0; r < 16; r++) {
      float acc = 0.f;
#pragma unroll
      for (uint32_t k = 0; k < r; k++) acc = fmaf(X[(o + r) * kPrT + o + k], x[k], acc);
      x[r] = r == cc ? 1.f : (r < cc ? 0.f : -acc);
    }
    __syncwarp();
#pragma unroll
    for (uint32_t r = 0; r < 16; r++) X[(o + r) * kPrT + o + cc] = x[r];
  }
  __syncthreads();
  {
    const uint32_t r = tid >> 4, cc = tid & 15;
    for (uint32_t i = 1; i < 4; i++) {
      for (uint32_t j = 0; j < i; j++) {
        float acc = 0.f;
        for (uint32_t k = j; k < i; k++)
#pragma unroll
          for (uint32_t q = 0; q < 16; q++)
            acc = fmaf(X[(16 * i + r) * kPrT + 16 * k + q], X[(16 * k + q) * kPrT + 16 * j + cc], acc);
        tmp[(j * 16 + r) * 16 + cc] = acc;
      }
      __syncthreads();
      for (uint32_t j = 0; j < i; j++) {
        float acc = 0.f;
#pragma unroll
        for (uint32_t q = 0; q < 16; q++) acc = fmaf(X[(16 * i + r) * kPrT + 16 * i + q], tmp[(j * 16 + q) * 16 + cc], acc);
        X[(16 * i + r) * kPrT + 16 * j + cc] = -acc;
      }
      __syncthreads();
    }
  }
  float amax = 0.f;
  for (uint32_t e = tid; e < kDnC * kDnC; e += blockDim.x) {
    const uint32_t t = e / kDnC, s2 = e % kDnC;
    const float tv = s2 <= t ? X[t * kPrT + s2] * beta[s2] : 0.f;
    X[t * kPrT + s2] = tv;
    amax = fmaxf(amax, fabsf(tv));
  }
  __syncthreads();
  // 4. MT = M T (both lower triangular), 3xTF32 mma.sync: warp w takes row tile w / 2 and
  //    column tiles 4 (w % 2) .. + 3; M T replaces M once every warp has read it.
  {
    const uint32_t mt = warp >> 1, kend = 16 * (mt + 1);
    float acc[4][4] = {};
    for (uint32_t k = 0; k < kend; k += 8) {
      uint32_t ah[4], al[4];
      split_a(Mq + (16 * mt + g) * kPrT + k + t4, kPrT, ah, al);
#pragma unroll
      for (uint32_t q = 0; q < 4; q++) {
        const uint32_t nt = (warp & 1) * 4 + q;
        const float* bt = X + (k + t4) * kPrT + 8 * nt + g;
        uint32_t bh[2], bl[2];
        split_b(bt[0], bt[4 * kPrT], bh, bl);
        mma3_split(acc[q], ah, al, bh, bl);
      }
    }
    __syncthreads();
#pragma unroll
    for (uint32_t q = 0; q < 4; q++) {
      const uint32_t nt = (warp & 1) * 4 + q;
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint32_t t = 16 * mt + g + (r >= 2 ? 8 : 0), u = 8 * nt + 2 * t4 + (r & 1);
        Mq[t * kPrT + u] = acc[q][r];
        amax = fmaxf(amax, fabsf(acc[q][r]));
      }
    }
  }
  // 5. The operands of C: [T; MT] times 2^sa (tiles 0, 1 of [0, 64K)), (Gamma K)^T times
  //    2^14 (tiles 2, 3); Kd^T times 2^14 to the record.
  const int sa = pt_scale_exp(pt_block_max(amax, red));
  {
    const float scale = pow2f(sa);
    for (uint32_t e = tid; e < 2 * kDnC * (kDnC / 8); e += blockDim.x) {
      const uint32_t r = e / (kDnC / 8), k0 = 8 * (e % (kDnC / 8));
      const float* src = r < kDnC ? X + r * kPrT + k0 : Mq + (r - kDnC) * kPrT + k0;
      const float4 a = *reinterpret_cast<const float4*>(src), b = *reinterpret_cast<const float4*>(src + 4);
      const float v8[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                           b.x * scale, b.y * scale, b.z * scale, b.w * scale};
      pt_store8(RA, RA + kPtTile, r, k0, v8);
    }
  }
  const float lam_c = lam[kDnC - 1];
  {
    const uint32_t i = tid & (DK - 1), sh = tid >> 7;  // feature i, tokens 32 sh ..
    float kr[32];
#pragma unroll
    for (uint32_t u = 0; u < 32; u++) {
      const uint32_t s2 = 32 * sh + u;
      kr[u] = s2 < ce ? ksrc[(uint64_t)(t0 + s2) * cd + i] : 0.f;
    }
#pragma unroll
    for (uint32_t s0 = 0; s0 < 32; s0 += 8) {
      float gk[8], kd[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const uint32_t s2 = 32 * sh + s0 + u;
        const float kv = kr[s0 + u] * rk[s2];
        kd[u] = __expf(lam_c - lam[s2]) * kv * kPtUnit;  // Kd[s] = e^(lam_C - lam_s) k_s, times 2^14
        gk[u] = kv * elam[s2] * kPtUnit;
      }
      pt_store8(RA + 2 * kPtTile, RA + 3 * kPtTile, i, 32 * sh + s0, gk);
      pt_store8(KdTg, KdTg + kPtTile, i, 32 * sh + s0, kd);  // the scan's Kd^T tiles
    }
  }
  // V rows of the chunk (registers) and their largest magnitude.
  const uint32_t vi = tid & (DV - 1), vsh = tid >> 7;
  float vr[32], vmax = 0.f;
#pragma unroll
  for (uint32_t u = 0; u < 32; u++) {
    const uint32_t s2 = 32 * vsh + u;
    vr[u] = s2 < ce ? vsrc[(uint64_t)(t0 + s2) * cd + vi] : 0.f;
    vmax = fmaxf(vmax, fabsf(vr[u]));
  }
  fence_proxy_async_smem();
  const int sv = pt_scale_exp(pt_block_max(vmax, red));  // its barriers also publish the tiles above
  if (tid == 0) {
    tc_fence_after();
    pt_mma(tmem, a_base, a_base + kPtTile, a_base + 2 * kPtTile, a_base + 3 * kPtTile, 1, tc_idesc_f16(DK));
  }
  // V^T times 2^sv into [64K, 96K) (X and M T are no longer read) while W and M W run.
  {
    const float scale = pow2f(sv);
#pragma unroll
    for (uint32_t s0 = 0; s0 < 32; s0 += 8) {
      float v8[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v8[u] = vr[s0 + u] * scale;
      pt_store8(RB, RB + kPtTile, vi, 32 * vsh + s0, v8);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    tc_fence_after();
    pt_mma(tmem + DK, a_base, a_base + kPtTile, smem_u32(RB), smem_u32(RB) + kPtTile, 1, tc_idesc_f16(DV));
    tc_commit(&bar[1]);
  }
  ok = __syncthreads_and(ok && mbar_wait_bounded(&bar[1], 0));
  tc_fence_after();
  // 6. Accumulators: warp w reads lanes 32 (w % 4).. and columns 128 (w / 4) ..: rows
  //    0-63 hold W (columns 0-127) and U (128-255), rows 64-127 M W and M U = R, each
  //    times its operands' inverse scales. U and R go to the record as f32. P = Gamma Q -
  //    M W (rows 0-63) and W (rows 64-127) go as the scan's [P; W] tiles, times 2^spw,
  //    where 2^spw brings their largest magnitude below 2^14 (a first read finds it).
  const uint32_t quarter = warp & 3, half = warp >> 2;
  const uint32_t row = quarter * 32 + lane, t = row & (kDnC - 1);
  const bool upper = row >= kDnC;
  const float unscale = pow2f(-sa) * (half ? pow2f(-sv) : 1.0f / kPtUnit);
  const float qs = rq[t], el = elam[t];
  const float* qr = qsrc + (uint64_t)(t0 + t) * cd;
  // Column j of block cb of P (upper rows) or W, from the accumulator values v.
  auto pw_vals = [&](uint32_t cb, float* v) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 qv = upper && t < ce ? *reinterpret_cast<const float4*>(qr + 32 * cb + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float q4[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int u = 0; u < 4; u++) v[j + u] = upper ? fmaf(el, q4[u] * qs, -(v[j + u] * unscale)) : v[j + u] * unscale;
    }
  };
  float pwmax = 0.f;
  if (ok && !half) {
    for (uint32_t cb = 0; cb < 4; cb++) {
      float v[32];
      tmem_ld32(tmem + ((quarter * 32) << 16) + 32 * cb, v);
      pw_vals(cb, v);
#pragma unroll
      for (int j = 0; j < 32; j++) pwmax = fmaxf(pwmax, fabsf(v[j]));
    }
  }
  const int spw = pt_scale_exp(pt_block_max(pwmax, red));
  if (ok) {
    const float pws = pow2f(spw);
    const uint32_t prow = upper ? t : kDnC + t;  // [P; W] row
    for (uint32_t cb = 0; cb < 4; cb++) {
      float v[32];
      tmem_ld32(tmem + ((quarter * 32) << 16) + 128 * half + 32 * cb, v);
      const uint32_t i0 = 32 * cb;
      if (half) {
        float* dst = (upper ? Rg : Ug) + t * DV + i0;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(dst + j) =
              make_float4(v[j] * unscale, v[j + 1] * unscale, v[j + 2] * unscale, v[j + 3] * unscale);
      } else {
        pw_vals(cb, v);
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] *= pws;
#pragma unroll
        for (int j = 0; j < 32; j += 8) pt_store8(PWg, PWg + 2 * kPtTile, prow, i0 + j, v + j);
      }
    }
  } else if (tid == 0) {
    report_timeout(err);
  }
  if (tid == 0) {
    rec[kRecScal] = __expf(lam_c);
    rec[kRecScal + 1] = (float)spw;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kPtTmemCols);
}

// Carries one head's state slice (all 128 rows, kDnCols = 32 columns) through the chunks
// of the step on the tcgen05 tensor cores. The slice lives in registers: thread (warp
// w, lane l) holds row 32 (w % 4) + l, columns 16 (w / 4) .. + 15, which is the tensor-
// memory lane and column range that thread may read. Per chunk:
//   1. S0^T times 2^ss (2^ss brings the slice's largest magnitude below 2^14) into two
//      fp16 hi / lo B tiles; [P; W] (from the record, already split) times S0 into
//      tensor memory columns 0-31: rows 0-63 give P S0, rows 64-127 W S0.
//   2. O = P S0 + R to the outputs; D = U - W S0, times 2^sd, into the D^T tiles.
//   3. Kd^T (from the record) times D into columns 32-63; S = gamma_C S0 + Kd^T D.
// The record's [P; W] and Kd^T tiles arrive by bulk copies (one thread, mbarriers) into
// single buffers, each refilled with the next chunk's as soon as its product completed;
// this slice's columns of U and R arrive by cp.async while the state product runs.
// Shared memory: [P; W] 64 KB, Kd^T 32 KB, S0^T 16 KB (32 rows x 2 K blocks, hi and lo),
// D^T 8 KB, U and R slices 2 x 10 KB.
constexpr uint32_t kSnTile = 16384;                  // bytes of a 128-row tile
constexpr uint32_t kSnSmall = 32 * 128;              // bytes of a 32-row tile
constexpr uint32_t kScS = 40;                        // row stride (floats) of the U / R slices
constexpr uint32_t kSnPW = 0, kSnKd = 4 * kSnTile, kSnS0 = 6 * kSnTile, kSnD = kSnS0 + 4 * kSnSmall,
                   kSnU = kSnD + 2 * kSnSmall, kSnR = kSnU + kDnC * kScS * 4;
constexpr size_t kScanSmem = kSnR + kDnC * kScS * 4 + 1024;

// Element k of row r (r < 32) of the 32-row tiles, as fp16 hi and lo; K blocks of 64.
__device__ __forceinline__ void sn_store1(uint8_t* hi, uint8_t* lo, uint32_t r, uint32_t k, float v) {
  const uint32_t off = (k >> 6) * kSnSmall + r * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) + ((k & 7) << 1);
  const __half hv = __float2half_rn(v);
  *reinterpret_cast<__half*>(hi + off) = hv;
  *reinterpret_cast<__half*>(lo + off) = __float2half_rn(v - __half2float(hv));
}
// One split product with N = 32: kbs K blocks of 64; A tiles kSnTile apart, B tiles
// kSnSmall apart.
__device__ __forceinline__ void sn_mma(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo,
                                       uint32_t kbs) {
  constexpr uint32_t idesc = tc_idesc_f16(kDnCols);
  for (uint32_t kb = 0; kb < kbs; kb++) {
#pragma unroll
    for (uint32_t kk = 0; kk < 4; kk++) {
      const uint64_t ah = sdesc<128>(a_hi + kb * kSnTile + kk * 32), al = sdesc<128>(a_lo + kb * kSnTile + kk * 32);
      const uint64_t bh = sdesc<128>(b_hi + kb * kSnSmall + kk * 32), bl = sdesc<128>(b_lo + kb * kSnSmall + kk * 32);
      tc_mma(d, ah, bh, idesc, (kb | kk) != 0);
      tc_mma(d, ah, bl, idesc, 1);
      tc_mma(d, al, bh, idesc, 1);
    }
  }
}

__global__ void __launch_bounds__(256, 1) dn_scan_tc_kernel(uint32_t m, uint32_t n_chunks, snl_lin_p p,
                                                            const float* __restrict__ chunks,
                                                            float* __restrict__ state, float* __restrict__ out,
                                                            int* err) {
  extern __shared__ uint8_t sn_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sn_raw) + 1023) & ~(uintptr_t)1023);
  float* Us = reinterpret_cast<float*>(sm + kSnU);
  float* Rs = reinterpret_cast<float*>(sm + kSnR);
  __shared__ float red[8];
  __shared__ uint64_t bar[4];  // [P; W] landed, Kd^T landed, first product done, state product done
  __shared__ uint32_t tmem_sh;
  __shared__ int fail_sh;
  const uint32_t slice = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t quarter = warp & 3, jc = 16 * (warp >> 2);
  const uint32_t i = quarter * 32 + lane;  // state row = tensor-memory lane
  const uint32_t j0 = slice * kDnCols;
  float* Sg = state + (uint64_t)h * DK * DV;
  float st[16];
#pragma unroll
  for (int jj = 0; jj < 16; jj += 4) {
    const float4 v = *reinterpret_cast<const float4*>(Sg + (uint64_t)i * DV + j0 + jc + jj);
    st[jj] = v.x;
    st[jj + 1] = v.y;
    st[jj + 2] = v.z;
    st[jj + 3] = v.w;
  }
  auto rec_of = [&](uint32_t c) { return chunks + ((uint64_t)h * n_chunks + c) * kDnChunkFloats; };
  auto load_pw = [&](uint32_t c) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(rec_of(c) + kRecPW);
    mbar_arrive_expect_tx(&bar[0], 4 * kSnTile);
    for (uint32_t q = 0; q < 4; q++) bulk_g2s_plain(sm + kSnPW + q * kSnTile, src + q * kSnTile, kSnTile, &bar[0]);
  };
  auto load_kd = [&](uint32_t c) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(rec_of(c) + kRecKd);
    mbar_arrive_expect_tx(&bar[1], 2 * kSnTile);
    for (uint32_t q = 0; q < 2; q++) bulk_g2s_plain(sm + kSnKd + q * kSnTile, src + q * kSnTile, kSnTile, &bar[1]);
  };
  auto load_ur = [&](uint32_t c) {
    const float* rec = rec_of(c);
    for (uint32_t e = tid; e < 2 * kDnC * (kDnCols / 4); e += blockDim.x) {
      const uint32_t w = e / (kDnC * (kDnCols / 4)), r = (e / (kDnCols / 4)) % kDnC, q = e % (kDnCols / 4);
      cp_async16((w ? Rs : Us) + r * kScS + 4 * q, rec + (w ? kRecR : kRecU) + r * DV + j0 + 4 * q);
    }
    cp_async_commit();
  };
  if (tid == 0) {
    for (int b = 0; b < 4; b++) mbar_init(&bar[b], 1);
    fail_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&tmem_sh, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh, base = smem_u32(sm);
  if (tid == 0) {
    load_pw(0);
    load_kd(0);
  }
  load_ur(0);
  bool ok = true;
  for (uint32_t c = 0; c < n_chunks && ok; c++) {
    const uint32_t t0 = c * kDnC, ce = min(kDnC, m - t0), par = c & 1;
    const bool more = c + 1 < n_chunks;
    const float* rec = rec_of(c);
    const float gC = rec[kRecScal];
    const int spw = (int)rec[kRecScal + 1];
    // 1. S0^T into the B tiles, then [P; W] S0.
    float smax = 0.f;
#pragma unroll
    for (int jj = 0; jj < 16; jj++) smax = fmaxf(smax, fabsf(st[jj]));
    const int ss = pt_scale_exp(pt_block_max(smax, red));
    {
      const float sc = pow2f(ss);
#pragma unroll
      for (int jj = 0; jj < 16; jj++) sn_store1(sm + kSnS0, sm + kSnS0 + 2 * kSnSmall, jc + jj, i, st[jj] * sc);
    }
    cp_async_wait<0>();  // this thread's copies of U and R
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      if (mbar_wait_bounded(&bar[0], par)) {
        tc_fence_after();
        sn_mma(tmem, base + kSnPW, base + kSnPW + 2 * kSnTile, base + kSnS0, base + kSnS0 + 2 * kSnSmall, 2);
        tc_commit(&bar[2]);
      } else {
        fail_sh = 1;
      }
    }
    __syncthreads();
    ok = !fail_sh && __syncthreads_and(mbar_wait_bounded(&bar[2], par));
    tc_fence_after();
    if (!ok) break;
    if (tid == 0 && more) load_pw(c + 1);  // the product has read [P; W]
    // 2. O and D (rows 0-63 and 64-127 of the accumulator).
    float v[16];
    tmem_ld16(tmem + ((quarter * 32) << 16) + jc, v);
    const float un1 = pow2f(-spw) * pow2f(-ss);
    const uint32_t t = i & (kDnC - 1);
    float dmax = 0.f;
    if (i < kDnC) {
      if (t < ce) {
        float* o = out + (uint64_t)(t0 + t) * p.n_v * DV + h * DV + j0 + jc;
#pragma unroll
        for (int jj = 0; jj < 16; jj++) o[jj] = fmaf(v[jj], un1, Rs[t * kScS + jc + jj]);
      }
    } else {
#pragma unroll
      for (int jj = 0; jj < 16; jj++) {
        v[jj] = Us[t * kScS + jc + jj] - v[jj] * un1;
        dmax = fmaxf(dmax, fabsf(v[jj]));
      }
    }
    const int sd = pt_scale_exp(pt_block_max(dmax, red));
    if (i >= kDnC) {
      const float sc = pow2f(sd);
#pragma unroll
      for (int jj = 0; jj < 16; jj++) sn_store1(sm + kSnD, sm + kSnD + kSnSmall, jc + jj, t, v[jj] * sc);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (more) load_ur(c + 1);  // U and R of this chunk are read
    // 3. S = gamma_C S0 + Kd^T D.
    if (tid == 0) {
      if (mbar_wait_bounded(&bar[1], par)) {
        tc_fence_after();
        sn_mma(tmem + 32, base + kSnKd, base + kSnKd + kSnTile, base + kSnD, base + kSnD + kSnSmall, 1);
        tc_commit(&bar[3]);
      } else {
        fail_sh = 1;
      }
    }
    __syncthreads();
    ok = !fail_sh && __syncthreads_and(mbar_wait_bounded(&bar[3], par));
    tc_fence_after();
    if (!ok) break;
    if (tid == 0 && more) load_kd(c + 1);
    tmem_ld16(tmem + ((quarter * 32) << 16) + 32 + jc, v);
    const float un2 = pow2f(-sd) * (1.0f / kPtUnit);
#pragma unroll
    for (int jj = 0; jj < 16; jj++) st[jj] = fmaf(gC, st[jj], v[jj] * un2);
  }
  if (ok) {
#pragma unroll
    for (int jj = 0; jj < 16; jj += 4)
      *reinterpret_cast<float4*>(Sg + (uint64_t)i * DV + j0 + jc + jj) = make_float4(st[jj], st[jj + 1], st[jj + 2], st[jj + 3]);
  } else {
    // A bounded wait gave up: flag it, let the copies in flight land, stop.
    if (tid == 0) report_timeout(err);
    cp_async_wait<0>();
    if (tid == 0) {
      (void)mbar_wait_bounded(&bar[0], 0);
      (void)mbar_wait_bounded(&bar[1], 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// Gated RMSNorm of the delta outputs (linear.wgsl's tail of `delta`), in place.
__global__ void __launch_bounds__(DV) dn_norm_kernel(snl_lin_p p, const float* __restrict__ proj,
                                                     const float* __restrict__ lw, float* __restrict__ out) {
  __shared__ float red[32];
  const uint32_t t = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const uint64_t o_i = (uint64_t)t * p.n_v * DV + h * DV + j;
  const float o = out[o_i];
  const float var_o = block_sum(o * o, red) / (float)DV;
  const float z = proj[(uint64_t)t * p.proj_stride + p.conv_dim + h * DV + j];
  const float norm_w = lw[(uint64_t)p.conv_dim * 4 + 2 * p.n_v + j];
  out[o_i] = o * rsqrtf(var_o + p.eps) * norm_w * (z / (1.0f + __expf(-z)));
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
  const uint32_t m = st.val.m;  // the host copy sizes the grid
  if (m == 0) return SNL_OK;
  const dim3 grid((p.conv_dim + 255) / 256, (m + kConvTok - 1) / kConvTok);
  conv_kernel<<<grid, 256, 0, s>>>(st, p, proj, conv_out, conv_state, lw);
  SNL_LAUNCH_CHECK("conv");
  conv_state_kernel<<<(p.conv_dim + 255) / 256, 256, 0, s>>>(st, p, proj, conv_state, conv_ckpt);
  SNL_LAUNCH_CHECK("conv_state");
  return SNL_OK;
}

int launch_delta(StepRef st, const snl_lin_p& p, const float* proj, const float* conv_out, float* state,
                 const float* lw, float* out, float* state_ckpt, cudaStream_t s, XOut xo) {
  if (int rc = check_lin(p)) return rc;
  delta_kernel<<<p.n_v, DV, 0, s>>>(st, p, proj, conv_out, state, lw, out, state_ckpt, xo);
  SNL_LAUNCH_CHECK("delta");
  return SNL_OK;
}

// Chunked prefill form: conv (token-parallel) into conv_out, then the three chunked
// delta kernels. m is the host's row count; no checkpoint. scratch: the chunk records,
// n_v * ceil(m / 64) * (5 * 64 * 128 + 4) floats.
int launch_conv_delta_chunked(uint32_t m, const snl_lin_p& p, const float* proj, float* conv_state, float* state,
                              const float* lw, float* out, float* conv_out, float* scratch, cudaStream_t s) {
  if (int rc = check_lin(p)) return rc;
  if (m == 0) return SNL_OK;
  const snl_step_u sv{m, 0, 1, 0};
  if (int rc = launch_conv(step_val(sv), p, proj, conv_out, conv_state, lw, nullptr, s)) return rc;
  const uint32_t nch = (m + kDnC - 1) / kDnC;
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    SNL_CUDA_TRY(cudaFuncSetAttribute(dn_prep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrepTcSmem));
    SNL_CUDA_TRY(cudaFuncSetAttribute(dn_scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem));
    attr[dev] = true;
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  dn_prep_tc_kernel<<<dim3(nch, p.n_v), 256, kPrepTcSmem, s>>>(m, p, proj, conv_out, lw, scratch, err);
  SNL_LAUNCH_CHECK("dn_prep_tc");
  dn_scan_tc_kernel<<<dim3(DV / kDnCols, p.n_v), 256, kScanSmem, s>>>(m, nch, p, scratch, state, out, err);
  SNL_LAUNCH_CHECK("dn_scan_tc");
  dn_norm_kernel<<<dim3(m, p.n_v), DV, 0, s>>>(p, proj, lw, out);
  SNL_LAUNCH_CHECK("dn_norm");
  return SNL_OK;
}

size_t conv_delta_chunked_scratch(const snl_lin_p& p, uint32_t m) {
  return (size_t)p.n_v * ((m + kDnC - 1) / kDnC) * kDnChunkFloats;
}

int launch_conv_delta(StepRef st, const snl_lin_p& p, const float* proj, float* conv_state, float* state,
                      const float* lw, float* out, float* conv_ckpt, float* state_ckpt, cudaStream_t s, XOut xo) {
  if (int rc = check_lin(p)) return rc;
  static const bool split = getenv("SNL_CD_NOSPLIT") == nullptr;
  const uint32_t cluster = p.n_v / p.n_k * kCsSplit;
  if (split && cluster <= 8) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_v * kCsSplit);
    cfg.blockDim = dim3(kCsThreads);
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_on() ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, conv_delta_split_kernel, st, p, proj, conv_state, state, lw, out,
                                             conv_ckpt, state_ckpt, xo);
    if (e != cudaSuccess) return cuda_fail(e, "conv_delta_split_kernel");
    count_launch();
    return SNL_OK;
  }
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
namespace snl {
namespace {
// Per-device scratch of the chunked path for kernel-level callers, grown on demand.
float* chunk_scratch(size_t floats) {
  static std::mutex mu;
  static float* buf[64] = {nullptr};
  static size_t cap[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (cap[dev] < floats) {
    if (buf[dev]) cudaFree(buf[dev]);
    buf[dev] = nullptr;
    cap[dev] = 0;
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, floats * sizeof(float)) != cudaSuccess) return nullptr;
    buf[dev] = static_cast<float*>(ptr);
    cap[dev] = floats;
  }
  return buf[dev];
}
}  // namespace
}  // namespace snl

extern "C" int snl_conv_delta(const snl_step_u* step, const snl_lin_p* p, const float* proj, float* conv_state,
                              float* state, const float* lw, float* out, float* conv_ckpt, float* state_ckpt,
                              void* stream) {
  if (!step || !p || !proj || !conv_state || !state || !lw || !out)
    return snl::fail(SNL_E_INVALID, "snl_conv_delta: null argument");
  if (step->ckpt > 0 && (!conv_ckpt || !state_ckpt)) return snl::fail(SNL_E_INVALID, "snl_conv_delta: ckpt needs buffers");
  if (step->m >= snl::kChunkedMinRows && step->ckpt == 0) {
    // Prefill-sized steps: the chunked form (conv_out and chunk records in scratch).
    const size_t conv_floats = (size_t)step->m * p->conv_dim;
    float* buf = snl::chunk_scratch(conv_floats + snl::conv_delta_chunked_scratch(*p, step->m));
    if (!buf) return snl::fail(SNL_E_OOM, "snl_conv_delta: scratch");
    return snl::launch_conv_delta_chunked(step->m, *p, proj, conv_state, state, lw, out, buf, buf + conv_floats,
                                          (cudaStream_t)stream);
  }
  return snl::launch_conv_delta(snl::step_val(*step), *p, proj, conv_state, state, lw, out, conv_ckpt, state_ckpt,
                                (cudaStream_t)stream);
}
