// Exchange kernels of the tensor-parallel engine (see tp.cuh for the protocol).
#include <algorithm>

#include "common.cuh"
#include "ptx.cuh"
#include "tp.cuh"

namespace snl {
namespace {

// Allreduce of the bulk partials (prefill's row-parallel outputs, [m, hidden]): every rank
// reads every rank's partial over NVLink and adds them in rank order, so all ranks hold
// bit-identical sums. The partials were written by the previous kernel.
__global__ void __launch_bounds__(256) tp_allreduce_kernel(TpComm c, uint32_t site, uint64_t n, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ int ok_sh;
  const uint64_t epoch = tp_epoch(c, site);
  const uint64_t par = (epoch & 1) * c.bp_elems;
  if (threadIdx.x == 0) {
    tp_signal(c, kSlotBulk, epoch);  // every CTA: none depends on another being resident
    int ok = 1;
    for (int q = 0; q < c.size; q++)
      if (q != c.rank && !tp_wait_one(c, kSlotBulk, q, epoch)) ok = 0;
    ok_sh = ok;
  }
  __syncthreads();
  if (!ok_sh) return;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int q = 0; q < c.size; q++) v += ld_cv(c.bparts[q] + par + i);
    out[i] = v;
  }
}

// Gathers the LM-head shards: out[r][q * vl + j] = rank q's logits[r][j]. With rows == 0
// it only exchanges the flags (a step without logits still takes part in the site order).
__global__ void __launch_bounds__(256) tp_gather_kernel(TpComm c, uint32_t site, uint32_t rows, uint32_t vl,
                                                        float* __restrict__ full) {
  pdl_trigger();
  pdl_wait();
  __shared__ int ok_sh;
  const uint64_t epoch = tp_epoch(c, site);
  if (threadIdx.x == 0) {
    tp_signal(c, kSlotLogits, epoch);
    int ok = 1;
    for (int q = 0; q < c.size; q++)
      if (q != c.rank && !tp_wait_one(c, kSlotLogits, q, epoch)) ok = 0;
    ok_sh = ok;
  }
  __syncthreads();
  if (!ok_sh) return;
  const uint64_t per = (uint64_t)rows * vl, total = per * c.size;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t q = (uint32_t)(i / per);
    const uint64_t rem = i % per;
    const uint32_t r = (uint32_t)(rem / vl), j = (uint32_t)(rem % vl);
    full[(uint64_t)r * vl * c.size + (uint64_t)q * vl + j] = ld_cv(c.logits[q] + rem);
  }
}

}  // namespace

int launch_tp_allreduce(const TpComm& c, uint32_t site, uint64_t n, float* out, cudaStream_t s) {
  if (n > c.bp_elems) return fail(SNL_E_INVALID, "tp allreduce: too many elements");
  const uint32_t grid = (uint32_t)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count() * 4);
  SNL_PDL_LAUNCH("tp_allreduce", tp_allreduce_kernel, dim3(std::max(grid, 1u)), dim3(256), (size_t)0, s, c, site, n, out);
  return SNL_OK;
}

int launch_tp_gather_logits(const TpComm& c, uint32_t site, uint32_t rows, uint32_t vl, float* full, cudaStream_t s) {
  const uint64_t total = (uint64_t)rows * vl * c.size;
  const uint32_t grid = (uint32_t)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 4);
  SNL_PDL_LAUNCH("tp_gather", tp_gather_kernel, dim3(std::max(grid, 1u)), dim3(256), (size_t)0, s, c, site, rows, vl, full);
  return SNL_OK;
}

}  // namespace snl
