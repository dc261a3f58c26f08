// Gated GQA attention with partial M-RoPE over an f16 KV cache
// (attention.wgsl: prep :59-127, attend :129-246, combine :248-269).
//
// Layouts are the reference's: proj rows hold per query head [q 256 | gate 256],
// then k [n_kv*256], then v [n_kv*256]; the caches hold f16 pairs packed in u32,
// cache[(pos * kv_dim + kh*256 + d) / 2]; split-K partials are
// [(m*n_heads + h)*parts + part][256 acc | max | sum].
#include <cstdlib>

#include "common.cuh"
#include "ptx.cuh"

namespace snl {
namespace {

constexpr uint32_t HD = 256;
constexpr uint32_t G = 4;  // query heads per KV head (config.rs:202)

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// prep: CTA (head slot, token), thread d = head dim. Slots [0, n_heads) queries,
// [n_heads, n_heads+n_kv) keys, then values.
__global__ void __launch_bounds__(256) prep_kernel(StepRef sr, snl_attn_p p, const float* __restrict__ proj,
                                                   float* __restrict__ qbuf, uint32_t* __restrict__ kc,
                                                   uint32_t* __restrict__ vc, const float* __restrict__ norms,
                                                   const uint32_t* __restrict__ rpos) {
  pdl_trigger();
  __shared__ float sh[HD];
  __shared__ float red[32];
  const snl_step_u st = load_step(sr);
  const uint32_t slot = blockIdx.x, m = blockIdx.y, d = threadIdx.x;
  // Before the wait: the norm weight and this dim's rotation, whose positions the host
  // wrote before the step (the projection is the only input an earlier kernel writes).
  const bool is_q = slot < p.n_heads;
  const uint32_t half_rot = p.rot_dim / 2;
  const float nw = slot < p.n_heads + p.n_kv ? 1.0f + norms[(is_q ? 0 : HD) + d] : 0.f;
  float sn = 0.f, cs = 1.f;
  if (d < p.rot_dim && m < st.m) {
    const uint32_t fi = d % half_rot;
    const float inv_freq = powf(p.rope_theta, -(float)(2 * fi) / (float)p.rot_dim);
    const uint32_t* rp = rpos + 4 * m;
    uint32_t rot_pos = rp[0];
    if (fi % 3 == 1 && fi < (p.mrope >> 16)) rot_pos = rp[1];
    else if (fi % 3 == 2 && fi < (p.mrope & 0xFFFFu)) rot_pos = rp[2];
    sincosf((float)rot_pos * inv_freq, &sn, &cs);
  }
  pdl_wait();
  if (m >= st.m) return;
  const uint64_t pos = (uint64_t)st.pos0 + m;
  const uint32_t q_dim = p.n_heads * HD, kv_dim = p.n_kv * HD;
  const uint64_t row = (uint64_t)m * p.proj_stride;
  if (slot >= p.n_heads + p.n_kv) {
    const uint32_t kh = slot - p.n_heads - p.n_kv;
    sh[d] = proj[row + 2 * q_dim + kv_dim + kh * HD + d];
    __syncthreads();
    if ((d & 1) == 0) vc[(pos * kv_dim + kh * HD + d) / 2] = pack_h2(sh[d], sh[d + 1]);
    return;
  }
  float v = is_q ? proj[row + slot * 2 * HD + d] : proj[row + 2 * q_dim + (slot - p.n_heads) * HD + d];
  const float total = block_sum(v * v, red);
  v = v * rsqrtf(total / (float)HD + p.eps) * nw;
  sh[d] = v;
  __syncthreads();
  if (d < p.rot_dim) v = d < half_rot ? v * cs - sh[d + half_rot] * sn : v * cs + sh[d - half_rot] * sn;
  if (is_q) {
    qbuf[(uint64_t)m * q_dim + slot * HD + d] = v;
  } else {
    __syncthreads();
    sh[d] = v;
    __syncthreads();
    const uint32_t kh = slot - p.n_heads;
    if ((d & 1) == 0) kc[(pos * kv_dim + kh * HD + d) / 2] = pack_h2(sh[d], sh[d + 1]);
  }
}

__device__ __forceinline__ void fa_mma(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// 16 bytes global -> shared, zero-filled when !valid (nothing is read then).
__device__ __forceinline__ void fa_cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ uint32_t fa_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// hi / lo fp16 pairs of two floats: hi = f16(v), lo = f16(v - hi)
__device__ __forceinline__ void fa_split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
  hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
  lo = fa_h2(a - __half2float(ha), b - __half2float(hb));
}

__device__ __forceinline__ void mma16808(float d[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

constexpr int kAttWarps = 12;
constexpr uint32_t kAttTcMinRows = 16;  // steps of at least this many rows use attend_tc_kernel
constexpr int kKeysPerGroup = 8;
constexpr uint32_t kAttStages = 2;  // key groups in flight per warp
static_assert(kAttKeysPerPart == kAttWarps * kKeysPerGroup, "a decode part is one key group per warp");
constexpr uint32_t kAttRowBytes = HD * 2 + 16;  // a cached K or V row (512 B) padded so ldmatrix rows hit distinct banks
constexpr uint32_t kAttGroupBytes = kKeysPerGroup * 2 * HD * 2;  // bytes copied per group: 8 keys x (K row, V row)
constexpr uint32_t kAttStageBytes = kKeysPerGroup * 2 * kAttRowBytes;
constexpr size_t kAttSmem = (size_t)kAttWarps * kAttStages * kAttStageBytes;  // 198 KB

// attend: CTA (KV head, token, part); 12 warps each take 8-key groups round-robin and
// keep their own online softmax for the G = 4 query heads. Per group, the scores
// S = Q K^T are 16 mma.sync m16n8k16 over the 256 dims (the 4 heads' queries as fp16
// hi and lo rows, K exact), and O^T += V^T P^T is 16 m16n8k8 (V exact, P as hi and lo
// columns), accumulated in f32 registers. The warps' states are merged at the end.
// Each warp streams its groups' K and V rows (16 rows of 512 contiguous bytes) into a
// ring of kAttStages groups in shared memory with bulk copies completing on one mbarrier
// per stage, so two groups per warp (192 KB per SM, one CTA) are in flight while it
// computes, instead of one load latency per group. Groups whose
// rows all precede this step's keys were written by earlier steps and are requested
// before the dependency wait; the others (the step's own keys, which the prep kernel
// writes) after it.
__global__ void __launch_bounds__(kAttWarps * 32, 1) attend_kernel(StepRef sr, snl_attn_p p, const float* __restrict__ proj,
                                                        const float* __restrict__ qbuf, const uint32_t* __restrict__ kc,
                                                        const uint32_t* __restrict__ vc, float* __restrict__ out,
                                                        float* __restrict__ partial, XOut xo, int* err) {
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t att_ring[];  // [warp][stage][8 K rows | 8 V rows], rows kAttRowBytes apart
  __shared__ uint64_t bars[kAttWarps][kAttStages];
  __shared__ float s_ml[kAttWarps][G][2];
  __shared__ __align__(16) __half q_tile[2 * G][HD + 8];  // rows of 528 B: ldmatrix rows on distinct banks
  const snl_step_u st = load_step(sr);
  const uint32_t kh = blockIdx.x, m = blockIdx.y, part = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t q_dim = p.n_heads * HD, kv_dim = p.n_kv * HD;
  const bool live = m < st.m && part < st.parts;
  const uint32_t total = st.pos0 + m + 1;
  const uint32_t chunk = (total + st.parts - 1) / st.parts;
  const uint32_t start = min(total, part * chunk);
  const uint32_t end = min(total, start + chunk);
  const uint64_t kbase = (uint64_t)kh * HD;  // in halves
  // warp-local group jj holds keys start + 8 (warp + 8 jj) ..; the part has ceil((end - start) / 8) groups
  const uint32_t ngroups = live ? (end - start + kKeysPerGroup - 1) / kKeysPerGroup : 0;
  const uint32_t my_groups = ngroups > (uint32_t)warp ? (ngroups - warp + kAttWarps - 1) / kAttWarps : 0;
  uint8_t* ring = att_ring + (size_t)warp * kAttStages * kAttStageBytes;
  if (lane == 0)
    for (uint32_t s2 = 0; s2 < kAttStages; s2++) mbar_init(&bars[warp][s2], 1);
  fence_mbar_init();
  __syncwarp();
  auto group_key0 = [&](uint32_t jj) { return start + (warp + jj * kAttWarps) * kKeysPerGroup; };
  // Rows past the part's end repeat its last key (weight 0 later), so every group is 8 KB.
  auto issue = [&](uint32_t jj) {
    const uint32_t t0 = group_key0(jj), nk = min((uint32_t)kKeysPerGroup, end - t0);
    uint64_t* bar = &bars[warp][jj % kAttStages];
    uint8_t* stg = ring + (jj % kAttStages) * kAttStageBytes;
    if (lane == 0) mbar_arrive_expect_tx(bar, kAttGroupBytes);
    __syncwarp();
    if (lane < 2 * kKeysPerGroup) {  // lanes 0-7: K rows, 8-15: V rows
      const uint32_t j = lane % kKeysPerGroup, t = t0 + min(j, nk - 1);
      const uint32_t* src = (lane < kKeysPerGroup ? kc : vc) + ((uint64_t)t * kv_dim + kbase) / 2;
      bulk_g2s_plain(stg + lane * kAttRowBytes, src, HD * 2, bar);
    }
  };
  // Requested before the wait: the leading groups whose rows all precede the step's keys.
  uint32_t issued = 0;
  while (issued < min(my_groups, kAttStages)) {
    const uint32_t t0 = group_key0(issued), last = t0 + min((uint32_t)kKeysPerGroup, end - t0) - 1;
    if (last >= st.pos0) break;
    issue(issued++);
  }
  pdl_wait();
  if (m >= st.m) return;
  if (part >= st.parts) {
    // An unused part slot of a captured step (the grid has the largest part count): a
    // partial that the merge weighs by zero.
    const uint64_t pi0 = ((uint64_t)m * p.n_heads + kh * G) * gridDim.z + part;
    for (uint32_t i = threadIdx.x; i < G * (HD + 2); i += blockDim.x) {
      const uint32_t g = i / (HD + 2), e = i % (HD + 2);
      partial[(pi0 + (uint64_t)g * gridDim.z) * (HD + 2) + e] = e == HD ? -1e30f : 0.f;
    }
    return;
  }
  for (; issued < min(my_groups, kAttStages); issued++) issue(issued);

  // The GQA group's scores and outputs as mma.sync tiles. Q is the A operand of S = Q K^T:
  // row 2h + e of the CTA's Q tile holds head h's scaled query as fp16 hi (e = 0) or lo
  // (e = 1); rows 8-15 of the MMA are zero. K and V are exact fp16 operands; all three are
  // read from shared memory with ldmatrix.
  for (uint32_t i = threadIdx.x; i < G * HD / 2; i += blockDim.x) {
    const uint32_t hq = i / (HD / 2), d2 = (i % (HD / 2)) * 2;
    const float2 x = *reinterpret_cast<const float2*>(qbuf + (uint64_t)m * q_dim + (kh * G + hq) * HD + d2);
    uint32_t hi, lo;
    fa_split2(x.x * p.scale, x.y * p.scale, hi, lo);
    *reinterpret_cast<uint32_t*>(&q_tile[2 * hq][d2]) = hi;
    *reinterpret_cast<uint32_t*>(&q_tile[2 * hq + 1][d2]) = lo;
  }
  __syncthreads();
  const uint32_t g = lane >> 2, t = lane & 3, qh = g >> 1, qhl = g & 1;
  // O^T = V^T P^T accumulators: lane (g, t) holds head t's dims 16c + g (o[c][0] from P's
  // hi half, o[c][1] from its lo half) and 16c + g + 8 (o[c][2], o[c][3]).
  float o[16][4];
#pragma unroll
  for (int c = 0; c < 16; c++)
#pragma unroll
    for (int e = 0; e < 4; e++) o[c][e] = 0.f;
  float m_run = -1e30f, l_run = 0.f;  // head qh's online softmax (equal in its 8 lanes)
  // ldmatrix x4: lane L addresses row L % 8 of matrix L / 8 = (chunk c + L / 16, dims + 8 (L / 8 % 2))
  const uint32_t lrow = lane & 7, lsel = lane >> 3;
  const uint32_t lcol = (16 * (lsel >> 1) + 8 * (lsel & 1)) * 2;
  const uint8_t* qst = reinterpret_cast<const uint8_t*>(&q_tile[lrow][0]) + lcol;

  bool ok = true;
  uint32_t jj = 0;
  for (; jj < my_groups; jj++) {
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[warp][jj % kAttStages], (jj / kAttStages) & 1))) {
      ok = false;
      break;
    }
    const uint32_t t0 = group_key0(jj), nk = min((uint32_t)kKeysPerGroup, end - t0);
    const uint8_t* kst = ring + (jj % kAttStages) * kAttStageBytes + lrow * kAttRowBytes + lcol;
    const uint8_t* vst = kst + kKeysPerGroup * kAttRowBytes;
    // S for the group's 8 keys (two accumulator chains over the 16 chunks).
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      uint32_t qa[4], kb[4];
      ldsm_x4(qa, qst + 32 * c);
      ldsm_x4(kb, kst + 32 * c);
      fa_mma(s0, qa[0], 0u, qa[1], 0u, kb[0], kb[1]);
      fa_mma(s1, qa[2], 0u, qa[3], 0u, kb[2], kb[3]);
    }
    // Head qh's scores of keys 2t and 2t + 1: its hi and lo rows (lanes g, g ^ 1) added.
    float sa = s0[0] + s1[0], sb = s0[1] + s1[1];
    sa += __shfl_xor_sync(0xffffffffu, sa, 4);
    sb += __shfl_xor_sync(0xffffffffu, sb, 4);
    const bool va_ok = 2 * t < nk, vb_ok = 2 * t + 1 < nk;
    if (!va_ok) sa = -1e30f;
    if (!vb_ok) sb = -1e30f;
    float mx = fmaxf(sa, sb);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float pa = va_ok ? __expf(sa - m_new) : 0.f;
    const float pb = vb_ok ? __expf(sb - m_new) : 0.f;
    float ls = pa + pb;
    ls += __shfl_xor_sync(0xffffffffu, ls, 1);
    ls += __shfl_xor_sync(0xffffffffu, ls, 2);
    const float corr = __expf(m_run - m_new);
    l_run = l_run * corr + ls;
    m_run = m_new;
    // P^T as the B operand: column 2h + e = head h's probabilities, fp16 hi (e = 0) or lo.
    uint32_t phi, plo;
    fa_split2(pa, pb, phi, plo);
    const uint32_t pfrag = qhl ? plo : phi;
    const float ct = __shfl_sync(0xffffffffu, corr, 8 * t);  // head t's correction (lane 8t: g = 2t)
#pragma unroll
    for (int c = 0; c < 16; c++)
#pragma unroll
      for (int e = 0; e < 4; e++) o[c][e] *= ct;
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      uint32_t va[4];
      ldsm_x4_t(va, vst + 32 * c);
      mma16808(o[c], va[0], va[1], pfrag);
      mma16808(o[c + 1], va[2], va[3], pfrag);
    }
    // The stage's rows were read by this warp's loads; the next bulk copy into it is
    // ordered after them.
    fence_proxy_async_smem();
    __syncwarp();
    if (jj + kAttStages < my_groups) issue(jj + kAttStages);
  }
  if (!ok) {
    // A bounded wait gave up: flag it and let this warp's copies still in flight land
    // before its ring is reused below (the CTA still meets at the merge barrier).
    if (lane == 0) report_timeout(err);
    for (uint32_t k2 = jj; k2 < min(my_groups, jj + kAttStages); k2++)
      (void)mbar_wait_bounded(&bars[warp][k2 % kAttStages], (k2 / kAttStages) & 1);
  }
  // This warp's accumulators go to the start of its own ring (its copies have all landed).
  float (*s_acc_w)[HD] = reinterpret_cast<float (*)[HD]>(ring);
  auto s_acc = [&](int w, int h) { return reinterpret_cast<float*>(att_ring + (size_t)w * kAttStages * kAttStageBytes) + h * HD; };
  // Publish this warp's state: head t's dims from the hi and lo halves summed.
#pragma unroll
  for (int c = 0; c < 16; c++) {
    s_acc_w[t][16 * c + g] = o[c][0] + o[c][1];
    s_acc_w[t][16 * c + g + 8] = o[c][2] + o[c][3];
  }
  if (t == 0 && qhl == 0) {
    s_ml[warp][qh][0] = m_run;
    s_ml[warp][qh][1] = l_run;
  }
  __syncthreads();
  // Merge: thread d owns head dim d for the G heads.
  const uint32_t d = threadIdx.x;
  if (d >= HD) return;
#pragma unroll
  for (int g = 0; g < (int)G; g++) {
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < kAttWarps; w++) M = fmaxf(M, s_ml[w][g][0]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kAttWarps; w++) {
      const float f = __expf(s_ml[w][g][0] - M);
      L = fmaf(s_ml[w][g][1], f, L);
      A = fmaf(s_acc(w, g)[d], f, A);
    }
    const uint32_t h = kh * G + g;
    if (gridDim.z == 1) {
      const float gate = proj[(uint64_t)m * p.proj_stride + h * 2 * HD + HD + d];
      const float o = A / L / (1.0f + __expf(-gate));
      out[(uint64_t)m * q_dim + h * HD + d] = o;
      if (xo.planes) xout_store(xo, m, h * HD + d, o);
    } else {
      // [(m * n_heads + h) * slots + part][258] with slots = the grid's part count (the
      // step's part count except in captured steps, which have the largest one).
      const uint64_t pi = ((uint64_t)m * p.n_heads + h) * gridDim.z + part;
      partial[pi * (HD + 2) + d] = A;
      if (d == 0) {
        partial[pi * (HD + 2) + HD] = M;
        partial[pi * (HD + 2) + HD + 1] = L;
      }
    }
  }
}

// combine: CTA (head, token), thread = head dim. `slots` = the partial layout's part
// count: the attend grid's, in which unused slots hold partials of weight zero; 0 = the
// step's part count (the kernel-level call, the reference's layout). All the loads (the
// first 64 parts' maxima, denominators and this thread's accumulator values) go out at
// once; each thread then adds its dim over the parts in part order, and every thread adds
// the denominator in part order from shared memory: the sequential sums of
// attention.wgsl:248-269. In a captured step nothing here waits on the step descriptor.
__global__ void __launch_bounds__(256) combine_kernel(StepRef sr, snl_attn_p p, const float* __restrict__ proj,
                                                      const float* __restrict__ partial, float* __restrict__ out,
                                                      uint32_t slots, XOut xo) {
  pdl_trigger();
  pdl_wait();
  constexpr uint32_t kPre = 64;  // parts whose values are loaded in the first round
  __shared__ float s_w[HD], s_l[HD], s_red[HD / 32];
  const uint32_t h = blockIdx.x, m = blockIdx.y, d = threadIdx.x;
  uint32_t parts = slots;
  if (slots == 0) {
    const snl_step_u st = load_step(sr);
    if (m >= st.m) return;
    parts = st.parts;
  } else if (m >= sr.val.m) {
    return;
  }
  const uint32_t q_dim = p.n_heads * HD;
  const uint64_t base = ((uint64_t)m * p.n_heads + h) * parts;
  const float* col = partial + base * (HD + 2) + d;
  const uint32_t n0 = min(parts, kPre);
  float v[kPre];
#pragma unroll
  for (uint32_t u = 0; u < kPre; u++) v[u] = col[(uint64_t)min(u, n0 - 1) * (HD + 2)];
  float mi = -1e30f, li = 0.f;
  if (d < n0) {
    mi = partial[(base + d) * (HD + 2) + HD];
    li = partial[(base + d) * (HD + 2) + HD + 1];
  }
  float mx = mi;
  for (uint32_t i = kPre + d; i < parts; i += HD) mx = fmaxf(mx, partial[(base + i) * (HD + 2) + HD]);
  mx = warp_max(mx);
  if ((d & 31) == 0) s_red[d >> 5] = mx;
  __syncthreads();
#pragma unroll
  for (uint32_t w = 0; w < HD / 32; w++) mx = fmaxf(mx, s_red[w]);
  s_w[d] = d < n0 ? __expf(mi - mx) : 0.f;  // parts past n0 add 0
  s_l[d] = li;
  __syncthreads();
  float acc = 0.f, l = 0.f;
#pragma unroll
  for (uint32_t u = 0; u < kPre; u++) acc = fmaf(v[u], s_w[u], acc);
  for (uint32_t i = 0; i < n0; i++) l = fmaf(s_l[i], s_w[i], l);
  // Parts past the first 64 (kernel-level calls only): rounds of up to 256.
  for (uint32_t c0 = kPre; c0 < parts; c0 += HD) {
    const uint32_t n = min(HD, parts - c0);
    __syncthreads();
    if (d < n) {
      const uint64_t o = (base + c0 + d) * (HD + 2);
      s_w[d] = __expf(partial[o + HD] - mx);
      s_l[d] = partial[o + HD + 1];
    }
    __syncthreads();
    for (uint32_t j = 0; j < n; j++) acc = fmaf(col[(uint64_t)(c0 + j) * (HD + 2)], s_w[j], acc);
    for (uint32_t i = 0; i < n; i++) l = fmaf(s_l[i], s_w[i], l);
  }
  const float gate = proj[(uint64_t)m * p.proj_stride + h * 2 * HD + HD + d];
  const float o = acc / l / (1.0f + __expf(-gate));
  out[(uint64_t)m * q_dim + h * HD + d] = o;
  if (xo.planes) xout_store(xo, m, h * HD + d, o);
}

// ---- prefill attention on the tensor cores ----------------------------------------
// Steps of many rows (prefill chunks) read every key once per 16 query tokens instead of
// once per token. CTA (KV head kh, block of 16 step tokens), 4 warps: warp w owns query
// head 4 kh + w for the 16 tokens, and all four share each 64-key block of K and V in
// shared memory (GQA). Per key block, FlashAttention-style (online softmax in registers):
//   S = Q K^T as mma.sync m16n8k16 (f16 in, f32 accumulate) with Q split into fp16 hi + lo
//     (K is exact: the cache holds f16), so S carries Q's ~22 bits;
//   causal and step-end masks, running max and sum per row (the S accumulator layout is
//   the next MMA's A fragment layout);
//   O += P V with P split into fp16 hi + lo (V exact), f32 accumulators in registers.
// The 64-key blocks stream in with asynchronous copies one block ahead (rows past the
// last key read as zeros). The result is the same attention as attention.wgsl:146-246
// (sequential online softmax over 16-key tiles there), in another summation order.
constexpr uint32_t kFaTok = 16;             // query tokens per CTA
constexpr uint32_t kFaKeys = 64;            // keys per block
constexpr uint32_t kFaStride = HD + 8;      // halves per smem row (528 B: ldmatrix rows on distinct banks)
constexpr size_t kFaSmem = (size_t)(2 * G * kFaTok + 4 * kFaKeys) * kFaStride * sizeof(__half);

__global__ void __launch_bounds__(128, 1) attend_tc_kernel(StepRef sr, snl_attn_p p, const float* __restrict__ proj,
                                                           const float* __restrict__ qbuf,
                                                           const uint32_t* __restrict__ kc,
                                                           const uint32_t* __restrict__ vc, float* __restrict__ out) {
  pdl_trigger();
  extern __shared__ __align__(16) __half fsm[];
  __half* Qh = fsm;                            // [G][16][kFaStride]
  __half* Ql = Qh + G * kFaTok * kFaStride;    // [G][16][kFaStride]
  __half* Kb = Ql + G * kFaTok * kFaStride;    // [2][64][kFaStride]
  __half* Vb = Kb + 2 * kFaKeys * kFaStride;   // [2][64][kFaStride]
  const snl_step_u st = load_step(sr);
  const uint32_t kh = blockIdx.x, i0 = blockIdx.y * kFaTok, tid = threadIdx.x;
  const uint32_t warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const uint32_t q_dim = p.n_heads * HD, kv_dim = p.n_kv * HD;
  pdl_wait();
  if (i0 >= st.m) return;
  const uint32_t ntok = min(kFaTok, st.m - i0);
  const uint32_t kend = st.pos0 + i0 + ntok;  // keys [0, kend) for this CTA
  const uint32_t nblk = (kend + kFaKeys - 1) / kFaKeys;
  const __half* kch = reinterpret_cast<const __half*>(kc);
  const __half* vch = reinterpret_cast<const __half*>(vc);
  auto load_block = [&](uint32_t b, uint32_t buf) {
    __half* kd = Kb + buf * kFaKeys * kFaStride;
    __half* vd = Vb + buf * kFaKeys * kFaStride;
    for (uint32_t e = tid; e < kFaKeys * (HD / 8); e += blockDim.x) {
      const uint32_t r = e / (HD / 8), c = (e % (HD / 8)) * 8;
      const uint32_t key = b * kFaKeys + r;
      const bool valid = key < kend;
      const uint64_t off = (uint64_t)(valid ? key : 0) * kv_dim + kh * HD + c;
      fa_cp16(kd + r * kFaStride + c, kch + off, valid);
      fa_cp16(vd + r * kFaStride + c, vch + off, valid);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_block(0, 0);
  // Q of the CTA's 4 heads and 16 tokens, scaled, as fp16 hi + lo (rows past the step: 0).
  for (uint32_t e = tid; e < G * kFaTok * (HD / 2); e += blockDim.x) {
    const uint32_t hh = e / (kFaTok * HD / 2), r = (e / (HD / 2)) % kFaTok, c = (e % (HD / 2)) * 2;
    float a = 0.f, b = 0.f;
    if (r < ntok) {
      const float* qp = qbuf + (uint64_t)(i0 + r) * q_dim + (kh * G + hh) * HD + c;
      a = qp[0] * p.scale;
      b = qp[1] * p.scale;
    }
    uint32_t hi, lo;
    fa_split2(a, b, hi, lo);
    *reinterpret_cast<uint32_t*>(Qh + (hh * kFaTok + r) * kFaStride + c) = hi;
    *reinterpret_cast<uint32_t*>(Ql + (hh * kFaTok + r) * kFaStride + c) = lo;
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < (int)(HD / 8); n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-1e30f, -1e30f}, lrow[2] = {0.f, 0.f};
  const __half* qh = Qh + warp * kFaTok * kFaStride;
  const __half* ql = Ql + warp * kFaTok * kFaStride;
  // ldmatrix row addresses of this lane: A (16 x 16 of Q) and B (K: keys x dims, V: keys x dims transposed)
  const uint32_t a_row = (lane & 7) + 8 * ((lane >> 3) & 1), a_col = 8 * (lane >> 4);
  const uint32_t kb_row = (lane & 7) + 8 * (lane >> 4), kb_col = 8 * ((lane >> 3) & 1);
  const uint32_t vb_row = (lane & 7) + 8 * ((lane >> 3) & 1), vb_col = 8 * (lane >> 4);
  for (uint32_t b = 0; b < nblk; b++) {
    const uint32_t buf = b & 1;
    if (b + 1 < nblk) {
      load_block(b + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const __half* kd = Kb + buf * kFaKeys * kFaStride;
    const __half* vd = Vb + buf * kFaKeys * kFaStride;
    // S = Q K^T for the warp's 16 rows x 64 keys
    float sacc[kFaKeys / 8][4];
#pragma unroll
    for (int j = 0; j < (int)(kFaKeys / 8); j++) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll 2
    for (uint32_t ks = 0; ks < HD / 16; ks++) {
      uint32_t ah[4], al[4];
      ldsm_x4(ah, qh + a_row * kFaStride + 16 * ks + a_col);
      ldsm_x4(al, ql + a_row * kFaStride + 16 * ks + a_col);
#pragma unroll
      for (int j = 0; j < (int)(kFaKeys / 8); j += 2) {
        uint32_t kb4[4];
        ldsm_x4(kb4, kd + (8 * j + kb_row) * kFaStride + 16 * ks + kb_col);
        fa_mma(sacc[j], ah[0], ah[1], ah[2], ah[3], kb4[0], kb4[1]);
        fa_mma(sacc[j], al[0], al[1], al[2], al[3], kb4[0], kb4[1]);
        fa_mma(sacc[j + 1], ah[0], ah[1], ah[2], ah[3], kb4[2], kb4[3]);
        fa_mma(sacc[j + 1], al[0], al[1], al[2], al[3], kb4[2], kb4[3]);
      }
    }
    // masks: key k is visible to row r (step token i0 + r) iff k <= pos0 + i0 + r
    const uint32_t key0 = b * kFaKeys;
    float bm[2] = {-1e30f, -1e30f};
#pragma unroll
    for (int j = 0; j < (int)(kFaKeys / 8); j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const uint32_t r = g + (e >= 2 ? 8 : 0), key = key0 + 8 * j + 2 * t + (e & 1);
        const bool vis = r < ntok && key <= st.pos0 + i0 + r;
        sacc[j][e] = vis ? sacc[j][e] : -1e30f;
        bm[e >> 1] = fmaxf(bm[e >> 1], sacc[j][e]);
      }
    }
    float corr[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; h2++) {
      bm[h2] = fmaxf(bm[h2], __shfl_xor_sync(0xffffffffu, bm[h2], 1));
      bm[h2] = fmaxf(bm[h2], __shfl_xor_sync(0xffffffffu, bm[h2], 2));
      const float mn = fmaxf(mrow[h2], bm[h2]);
      corr[h2] = __expf(mrow[h2] - mn);
      mrow[h2] = mn;
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < (int)(kFaKeys / 8); j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float pv = sacc[j][e] <= -1e29f ? 0.f : __expf(sacc[j][e] - mrow[e >> 1]);
        sacc[j][e] = pv;
        ls[e >> 1] += pv;
      }
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; h2++) {
      ls[h2] += __shfl_xor_sync(0xffffffffu, ls[h2], 1);
      ls[h2] += __shfl_xor_sync(0xffffffffu, ls[h2], 2);
      lrow[h2] = lrow[h2] * corr[h2] + ls[h2];
    }
#pragma unroll
    for (int n = 0; n < (int)(HD / 8); n++) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O += P V: P's k-step ks2 (keys 16 ks2 ..) is S tiles 2 ks2 and 2 ks2 + 1
#pragma unroll
    for (uint32_t ks2 = 0; ks2 < kFaKeys / 16; ks2++) {
      uint32_t ph[4], pl[4];
      fa_split2(sacc[2 * ks2][0], sacc[2 * ks2][1], ph[0], pl[0]);
      fa_split2(sacc[2 * ks2][2], sacc[2 * ks2][3], ph[1], pl[1]);
      fa_split2(sacc[2 * ks2 + 1][0], sacc[2 * ks2 + 1][1], ph[2], pl[2]);
      fa_split2(sacc[2 * ks2 + 1][2], sacc[2 * ks2 + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int n = 0; n < (int)(HD / 8); n += 2) {
        uint32_t vb4[4];
        ldsm_x4_t(vb4, vd + (16 * ks2 + vb_row) * kFaStride + 8 * n + vb_col);
        fa_mma(o[n], ph[0], ph[1], ph[2], ph[3], vb4[0], vb4[1]);
        fa_mma(o[n], pl[0], pl[1], pl[2], pl[3], vb4[0], vb4[1]);
        fa_mma(o[n + 1], ph[0], ph[1], ph[2], ph[3], vb4[2], vb4[3]);
        fa_mma(o[n + 1], pl[0], pl[1], pl[2], pl[3], vb4[2], vb4[3]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
  // out = O / l * sigmoid(gate) (attention.wgsl:146-246)
  const uint32_t h = kh * G + warp;
#pragma unroll
  for (int h2 = 0; h2 < 2; h2++) {
    const uint32_t r = g + 8 * h2;
    if (r >= ntok) continue;
    const uint32_t tok = i0 + r;
    const float inv_l = 1.0f / lrow[h2];
    const float* gate = proj + (uint64_t)tok * p.proj_stride + h * 2 * HD + HD;
    float* orow = out + (uint64_t)tok * q_dim + h * HD;
#pragma unroll
    for (int n = 0; n < (int)(HD / 8); n++) {
      const uint32_t d = 8 * n + 2 * t;
      const float g0 = gate[d], g1 = gate[d + 1];
      orow[d] = o[n][2 * h2] * inv_l / (1.0f + __expf(-g0));
      orow[d + 1] = o[n][2 * h2 + 1] * inv_l / (1.0f + __expf(-g1));
    }
  }
}

}  // namespace

static int check_attn(const snl_attn_p& p) {
  if (p.n_heads != G * p.n_kv || p.n_kv == 0) return fail(SNL_E_UNSUPPORTED, "attention: need 4 query heads per KV head");
  if (p.rot_dim > HD || (p.rot_dim & 1) || p.rot_dim == 0) return fail(SNL_E_UNSUPPORTED, "attention: invalid rotary dim");
  return SNL_OK;
}

int launch_attn_prep(StepRef st, const snl_attn_p& p, const float* proj, float* qbuf, uint32_t* kc, uint32_t* vc,
                     const float* norms, const uint32_t* rpos, uint32_t m, cudaStream_t s) {
  if (int rc = check_attn(p)) return rc;
  if (m == 0) return SNL_OK;
  SNL_PDL_LAUNCH("prep_kernel", prep_kernel, dim3(dim3(p.n_heads + 2 * p.n_kv, m)), dim3(HD), (size_t)(0), s, st, p, proj, qbuf, kc, vc, norms, rpos);
  return SNL_OK;
}

int launch_attend(StepRef st, const snl_attn_p& p, const float* proj, const float* qbuf, const uint32_t* kc,
                  const uint32_t* vc, float* out, float* partial, uint32_t m, uint32_t parts_grid, cudaStream_t s,
                  XOut xo) {
  if (int rc = check_attn(p)) return rc;
  if (m == 0 || parts_grid == 0) return SNL_OK;
  static const bool no_tc = getenv("SNL_NO_ATTN_TC") != nullptr;
  if (parts_grid == 1 && m >= kAttTcMinRows && !xo.planes && !no_tc) {
    // a prefill chunk: the tiled tensor-core kernel (keys read once per 16 tokens)
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
      SNL_CUDA_TRY(cudaFuncSetAttribute(attend_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaSmem));
      attr[dev] = true;
    }
    SNL_PDL_LAUNCH("attend_tc_kernel", attend_tc_kernel, dim3(p.n_kv, (m + kFaTok - 1) / kFaTok), dim3(128), kFaSmem, s,
                   st, p, proj, qbuf, kc, vc, out);
    return SNL_OK;
  }
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  static bool ring_attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !ring_attr[dev]) {
    SNL_CUDA_TRY(cudaFuncSetAttribute(attend_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttSmem));
    ring_attr[dev] = true;
  }
  SNL_PDL_LAUNCH("attend_kernel", attend_kernel, dim3(dim3(p.n_kv, m, parts_grid)), dim3(kAttWarps * 32), kAttSmem, s, st,
                 p, proj, qbuf, kc, vc, out, partial, xo, err);
  return SNL_OK;
}

int launch_attn_combine(StepRef st, const snl_attn_p& p, const float* proj, const float* partial, float* out,
                        uint32_t m, cudaStream_t s, uint32_t slots, XOut xo) {
  if (int rc = check_attn(p)) return rc;
  if (m == 0) return SNL_OK;
  SNL_PDL_LAUNCH("combine_kernel", combine_kernel, dim3(dim3(p.n_heads, m)), dim3(HD), (size_t)(0), s, st, p, proj, partial, out, slots, xo);
  return SNL_OK;
}

}  // namespace snl

extern "C" int snl_attn_prep(const snl_step_u* step, const snl_attn_p* p, const float* proj, float* qbuf,
                             uint32_t* kcache, uint32_t* vcache, const float* norms, const uint32_t* rpos,
                             void* stream) {
  if (!step || !p || !proj || !qbuf || !kcache || !vcache || !norms || !rpos)
    return snl::fail(SNL_E_INVALID, "snl_attn_prep: null argument");
  return snl::launch_attn_prep(snl::step_val(*step), *p, proj, qbuf, kcache, vcache, norms, rpos, step->m,
                               (cudaStream_t)stream);
}
extern "C" int snl_attend(const snl_step_u* step, const snl_attn_p* p, const float* proj, const float* qbuf,
                          const uint32_t* kcache, const uint32_t* vcache, float* out, float* partial, void* stream) {
  if (!step || !p || !proj || !qbuf || !kcache || !vcache) return snl::fail(SNL_E_INVALID, "snl_attend: null argument");
  if (step->parts == 0) return snl::fail(SNL_E_INVALID, "snl_attend: parts must be >= 1");
  if (step->parts == 1 ? !out : !partial) return snl::fail(SNL_E_INVALID, "snl_attend: missing output buffer");
  return snl::launch_attend(snl::step_val(*step), *p, proj, qbuf, kcache, vcache, out, partial, step->m, step->parts,
                            (cudaStream_t)stream);
}
extern "C" int snl_attn_combine(const snl_step_u* step, const snl_attn_p* p, const float* proj, const float* partial,
                                float* out, void* stream) {
  if (!step || !p || !proj || !partial || !out) return snl::fail(SNL_E_INVALID, "snl_attn_combine: null argument");
  if (step->parts == 0) return snl::fail(SNL_E_INVALID, "snl_attn_combine: parts must be >= 1");
  return snl::launch_attn_combine(snl::step_val(*step), *p, proj, partial, out, step->m, (cudaStream_t)stream, 0);
}
