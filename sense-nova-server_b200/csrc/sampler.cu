// On-device sampling (sampler.rs:54-167): repetition / presence / frequency penalties,
// temperature, top-k, min-p and top-p, then a draw, or the speculative verify of a draft.
// The host keeps the random number generator and passes its uniform draws, so a result
// is a function of (logits, history, parameters, draws), as in the reference.
//
// Supported: temperature <= 1e-5 (greedy) and top_k in [1, 256], the reference's
// top_k_small branch, whose order is defined: descending logit, ties by lower index. The
// k > 256 branch sorts with an unstable sort (tie order unspecified) and is refused.
//
// Top-k runs in two passes: kSampleParts CTAs each sort a slice of the vocabulary as
// 64-bit keys (orderable logit bits << 32 | ~index, so one descending sort gives the
// reference's order) and keep their first k; one CTA then sorts the kSampleParts * k
// candidates. That CTA's thread 0 runs the rest exactly as the reference's loops run:
// sequential f32 sums in rank order, min-p, top-p, renormalisation and the draw.
#include <cuda_fp16.h>

#include "common.cuh"
#include "ptx.cuh"

namespace snl {
namespace {

constexpr uint32_t kSampleParts = 64;     // pass-1 CTAs
constexpr uint32_t kSampleSlice = 4096;   // keys sorted per pass-1 CTA (>= ceil(n / parts))
constexpr uint32_t kSampleMaxK = 256;     // top_k_small's range (sampler.rs:98)
constexpr uint32_t kSampleThreads = 1024;

// Monotonic map of f32 to u32 (larger float -> larger key); -0 is +0 (the reference's
// comparisons treat them as equal, and equal logits rank by index).
__device__ __forceinline__ uint32_t orderable(float v) {
  uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_orderable(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}
__device__ __forceinline__ uint64_t sample_key(float v, uint32_t i) {
  return ((uint64_t)orderable(v) << 32) | (uint64_t)(~i);
}

// Bitonic sort of n (a power of two) keys in shared memory, descending.
__device__ void bitonic_desc(uint64_t* k, uint32_t n) {
  for (uint32_t size = 2; size <= n; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const uint32_t lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = k[lo], b = k[hi];
        if ((a < b) == desc) {
          k[lo] = b;
          k[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

// The penalties of Sampler::distribution (sampler.rs:81-88), one thread per token of
// the history (each token appears once, as in the reference's map).
__global__ void sample_penalty_kernel(float* __restrict__ logits, uint32_t n, const uint32_t* __restrict__ tok,
                                      const uint32_t* __restrict__ cnt, uint32_t n_hist, snl_sample_p p) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_hist || tok[i] >= n) return;
  float l = logits[tok[i]];
  if (p.repetition_penalty != 1.0f) l = l > 0.0f ? l / p.repetition_penalty : l * p.repetition_penalty;
  l -= p.presence_penalty + p.frequency_penalty * (float)cnt[i];
  logits[tok[i]] = l;
}

// Pass 1: slice `blockIdx.x` of the vocabulary -> its first k keys.
__global__ void __launch_bounds__(kSampleThreads) sample_topk_part_kernel(const float* __restrict__ logits, uint32_t n,
                                                                          uint32_t k, uint64_t* __restrict__ cand) {
  __shared__ uint64_t keys[kSampleSlice];
  const uint32_t per = (n + kSampleParts - 1) / kSampleParts;
  const uint32_t b0 = min(n, blockIdx.x * per), b1 = min(n, b0 + per);
  for (uint32_t i = threadIdx.x; i < kSampleSlice; i += blockDim.x)
    keys[i] = b0 + i < b1 ? sample_key(logits[b0 + i], b0 + i) : 0ull;
  bitonic_desc(keys, kSampleSlice);
  for (uint32_t i = threadIdx.x; i < k; i += blockDim.x) cand[(uint64_t)blockIdx.x * k + i] = keys[i];
}

// Pass 2 and the distribution / draw. out: [0] token, [1] accepted, [2] draws used.
__global__ void __launch_bounds__(kSampleThreads) sample_final_kernel(const uint64_t* __restrict__ cand, uint32_t k,
                                                                      uint32_t kpad, snl_sample_p p, float u0, float u1,
                                                                      int64_t draft, uint32_t* __restrict__ out) {
  extern __shared__ uint64_t keys[];  // [kSampleParts * kpad]
  __shared__ float prob[kSampleMaxK];
  __shared__ uint32_t tok[kSampleMaxK];
  const uint32_t total_keys = kSampleParts * kpad;
  for (uint32_t i = threadIdx.x; i < total_keys; i += blockDim.x) {
    const uint32_t part = i / kpad, j = i % kpad;
    keys[i] = j < k ? cand[(uint64_t)part * k + j] : 0ull;
  }
  bitonic_desc(keys, total_keys);
  if (threadIdx.x != 0) return;
  for (uint32_t i = 0; i < k; i++) tok[i] = ~(uint32_t)(keys[i] & 0xFFFFFFFFull);
  if (p.temperature <= 1e-5f) {  // greedy: the first maximum (argmax, sampler.rs:169-177)
    out[0] = tok[0];
    out[1] = draft >= 0 && (uint64_t)draft == tok[0] ? 1u : 0u;
    out[2] = 0;
    return;
  }
  const float mx = from_orderable((uint32_t)(keys[0] >> 32));
  float sum = 0.f;
  for (uint32_t i = 0; i < k; i++) {
    prob[i] = expf((from_orderable((uint32_t)(keys[i] >> 32)) - mx) / p.temperature);
    sum += prob[i];
  }
  for (uint32_t i = 0; i < k; i++) prob[i] /= sum;
  uint32_t keep = k;
  if (p.min_p > 0.0f) {
    const float thresh = prob[0] * p.min_p;
    keep = 0;
    while (keep < k && prob[keep] >= thresh) keep++;
    keep = max(keep, 1u);
  }
  if (p.top_p < 1.0f) {
    float cum = 0.f;
    for (uint32_t i = 0; i < keep; i++) {
      cum += prob[i];
      if (cum >= p.top_p) {
        keep = i + 1;
        break;
      }
    }
  }
  float total = 0.f;
  for (uint32_t i = 0; i < keep; i++) total += prob[i];
  for (uint32_t i = 0; i < keep; i++) prob[i] /= total;
  // draw (sampler.rs:142-156), optionally without one token.
  auto draw = [&](float u, int64_t exclude) -> uint32_t {
    float tot = 0.f;
    for (uint32_t i = 0; i < keep; i++)
      if ((int64_t)tok[i] != exclude) tot += prob[i];
    float r = u * tot;
    uint32_t last = tok[0];
    for (uint32_t i = 0; i < keep; i++) {
      if ((int64_t)tok[i] == exclude) continue;
      r -= prob[i];
      last = tok[i];
      if (r <= 0.0f) return tok[i];
    }
    return last;
  };
  if (draft < 0) {
    out[0] = draw(u0, -1);
    out[1] = 0;
    out[2] = 1;
    return;
  }
  // verify (sampler.rs:62-76): accept with probability p(draft), else redraw without it.
  float pd = 0.f;
  for (uint32_t i = 0; i < keep; i++)
    if ((int64_t)tok[i] == draft) pd = prob[i];
  if (pd > 0.0f && u0 < pd) {
    out[0] = (uint32_t)draft;
    out[1] = 1;
    out[2] = 1;
  } else {
    out[0] = draw(pd > 0.0f ? u1 : u0, draft);
    out[1] = 0;
    out[2] = pd > 0.0f ? 2 : 1;
  }
}

}  // namespace

size_t sample_scratch_bytes() { return (size_t)kSampleParts * kSampleMaxK * sizeof(uint64_t); }

int launch_sample(const snl_sample_p& p, float* logits, uint32_t n, const uint32_t* hist_tok, const uint32_t* hist_cnt,
                  uint32_t n_hist, float u0, float u1, int64_t draft, uint32_t* out, void* scratch, cudaStream_t s) {
  if (n == 0 || n > kSampleParts * kSampleSlice) return fail(SNL_E_UNSUPPORTED, "sample: vocabulary size out of range");
  const bool greedy = p.temperature <= 1e-5f;
  const uint32_t k = greedy ? 1u : (p.top_k == 0 ? n : std::min(p.top_k, n));
  if (k > kSampleMaxK)
    return fail(SNL_E_UNSUPPORTED, "sample: top_k must be 1..256 (the larger-k branch has no defined tie order)");
  if (n_hist && (!hist_tok || !hist_cnt)) return fail(SNL_E_INVALID, "sample: history arrays missing");
  if (n_hist) {
    sample_penalty_kernel<<<(n_hist + 255) / 256, 256, 0, s>>>(logits, n, hist_tok, hist_cnt, n_hist, p);
    SNL_LAUNCH_CHECK("sample_penalty");
  }
  uint64_t* cand = static_cast<uint64_t*>(scratch);
  sample_topk_part_kernel<<<kSampleParts, kSampleThreads, 0, s>>>(logits, n, k, cand);
  SNL_LAUNCH_CHECK("sample_topk_part");
  uint32_t kpad = 1;
  while (kpad < k) kpad <<= 1;
  const size_t smem = (size_t)kSampleParts * kpad * sizeof(uint64_t);
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    SNL_CUDA_TRY(cudaFuncSetAttribute(sample_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)(kSampleParts * kSampleMaxK * sizeof(uint64_t))));
    attr[dev] = true;
  }
  sample_final_kernel<<<1, kSampleThreads, smem, s>>>(cand, k, kpad, p, u0, u1, draft, out);
  SNL_LAUNCH_CHECK("sample_final");
  return SNL_OK;
}

}  // namespace snl

extern "C" size_t snl_sample_scratch_bytes(void) { return snl::sample_scratch_bytes(); }

extern "C" int snl_sample(const snl_sample_p* p, float* logits, uint32_t n, const uint32_t* hist_tok,
                          const uint32_t* hist_cnt, uint32_t n_hist, const float* u, int64_t draft, uint32_t* out,
                          void* scratch, void* stream) {
  if (!p || !logits || !u || !out || !scratch) return snl::fail(SNL_E_INVALID, "snl_sample: null argument");
  return snl::launch_sample(*p, logits, n, hist_tok, hist_cnt, n_hist, u[0], u[1], draft, out, scratch,
                            (cudaStream_t)stream);
}
