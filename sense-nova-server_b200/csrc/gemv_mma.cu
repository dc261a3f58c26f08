// Block-quantized GEMV on the tensor cores (decode and 2-row verify).
//
// y[t, n] = sum_k x[t, k] * q[n, k] * s[n, k/32] for t < M <= 4 token rows.
//
// The dot products run as mma.sync m16n8k16 (f16 inputs, f32 accumulation):
//   * A = 16 weight rows x 16 k. Q8_0 codes and Q4_0 nibbles are exact in fp16: a byte
//     permute builds 1024 + (code + 128) (or 1024 + nibble) in the mantissa of fp16 and
//     one packed subtract removes the offset.
//   * B = 16 k x 8 columns: column 2t holds x_hi of token t and column 2t+1 its x_lo,
//     where x = 16 * (x_hi + x_lo) with x_hi = fp16(x / 16), x_lo = fp16(x / 16 - x_hi).
//     The pair carries ~22 significant bits, so the products match an fp32 dot product
//     well inside the 1e-3 bar; the 1/16 pre-scale keeps |x| up to 10^6 in fp16 range.
//   * Each 32-element block is two MMAs; its f32 result is scaled by the block's scale
//     and added to an f32 accumulator in registers, so the per-block scale of the
//     reference layout (weights.rs:48-55) is applied exactly as in matmul.wgsl.
// k placement inside a block: thread (group g, lane-in-group t) loads bytes [8t, 8t+8)
// of its two rows (Q8: one 8-byte load per row; Q4: the 4-byte word t). Any bijection
// of k onto the MMA's k slots gives the same sum as long as A and B use the same one;
// here MMA 0 takes k in {8t..8t+3} and MMA 1 k in {8t+4..8t+7} (Q4 pairs (8t+i, 8t+i+4)).
//
// The x operand arrives packed ("x planes", [2M][K] halves, natural k order), written
// by the kernel that produced x, so a GEMV CTA starts streaming weights immediately.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "gemv_mma.cuh"
#include "mhc.cuh"
#include "ptx.cuh"

namespace snl {
namespace {

constexpr int kWarpsK = 4;  // warps of a CTA split K into 4 contiguous ranges
constexpr int kUnroll = 8;  // blocks (32 k) per iteration: 16 8-byte weight loads in flight per thread

__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// 4 int8 codes of w -> two half2 (codes 0,1) and (2,3), exact.
__device__ __forceinline__ void q8_half2(uint32_t w, uint32_t& h01, uint32_t& h23) {
  const uint32_t u = w ^ 0x80808080u;                   // code + 128 as unsigned bytes
  const uint32_t off = 0x64806480u;                     // half2(1152, 1152)
  h01 = hsub2_u32(__byte_perm(u, 0x64646464u, 0x4140), off);  // [b0, 0x64, b1, 0x64]
  h23 = hsub2_u32(__byte_perm(u, 0x64646464u, 0x4342), off);
}
__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b), *reinterpret_cast<__half2*>(&c));
  return *reinterpret_cast<uint32_t*>(&r);
}

// 8 nibbles of w (element i = nibble i, value nibble - 8) -> half2 pairs (i, i+4), i < 4,
// exact, in 9 instructions per word. A nibble at bits 0-3 of a half, or-ed into fp16 1024
// (0x6400), is 1024 + n: subtract 1032. A nibble left at bits 4-7 gives 1024 + 16 n:
// (1024 + 16 n) / 16 - 72 = n - 8 is one packed fma (both steps exact in fp16). Nibbles
// 2, 3, 6, 7 take the same two forms after one shift of the word by 8.
__device__ __forceinline__ void q4_half2(uint32_t w, uint32_t h[4]) {
  constexpr uint32_t kMagic = 0x64006400u;   // half2(1024, 1024)
  constexpr uint32_t kOff = 0x64086408u;     // half2(1032, 1032)
  constexpr uint32_t kSixteenth = 0x2C002C00u;  // half2(1/16, 1/16)
  constexpr uint32_t kNeg72 = 0xD480D480u;   // half2(-72, -72)
  const uint32_t w8 = w >> 8;
  h[0] = hsub2_u32((w & 0x000F000Fu) | kMagic, kOff);
  h[1] = hfma2_u32((w & 0x00F000F0u) | kMagic, kSixteenth, kNeg72);
  h[2] = hsub2_u32((w8 & 0x000F000Fu) | kMagic, kOff);
  h[3] = hfma2_u32((w8 & 0x00F000F0u) | kMagic, kSixteenth, kNeg72);
}

template <typename ST>
__device__ __forceinline__ float scale_at(const ST* s, uint64_t i) {
  if constexpr (sizeof(ST) == 4) return __ldg(reinterpret_cast<const float*>(s) + i);
  else return __half2float(__ldg(reinterpret_cast<const __half*>(s) + i));
}

// Streaming 8-byte weight load (read once per token: no L1 allocation).
__device__ __forceinline__ uint2 ld_w8(const uint8_t* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_w4(const uint8_t* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

template <int DT, int M, typename ST>
__global__ void __launch_bounds__(kWarpsK * 32) gemv_mma_kernel(GemvArgs a, const ST* __restrict__ ws) {
  static_assert(M >= 1 && M <= 4, "2M B columns must fit the MMA's 8");
  __shared__ float red[kWarpsK][M][16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t K = a.k, nb = K / 32;
  const uint32_t row0 = blockIdx.x * 16;
  const uint32_t rA = min(row0 + g, a.n - 1), rB = min(row0 + g + 8, a.n - 1);
  constexpr uint32_t BPB = DT == SNL_Q8_0 ? 32 : 16;  // weight bytes per block per row
  const uint8_t* wA = a.wq + (uint64_t)rA * nb * BPB;
  const uint8_t* wB = a.wq + (uint64_t)rB * nb * BPB;
  const ST* sA = ws + (uint64_t)rA * nb;
  const ST* sB = ws + (uint64_t)rB * nb;
  // This warp's K range, in blocks.
  const uint32_t per = (nb + kWarpsK - 1) / kWarpsK;
  const uint32_t b_begin = min(nb, warp * per), b_end = min(nb, b_begin + per);
  // x planes: thread loads plane g (< 2M) at k = 32 b + 8 t.
  const bool has_x = g < 2 * M;
  const __half* xp = a.xplanes + (uint64_t)(has_x ? g : 0) * a.plane_stride + 8 * t;

  float accA = 0.f, accB = 0.f;  // rows g and g+8 for token t (t < M)
  for (uint32_t b0 = b_begin; b0 < b_end; b0 += kUnroll) {
    uint32_t wa[kUnroll][2], wb[kUnroll][2];
    float sa[kUnroll], sb[kUnroll];
    uint4 xv[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      const uint32_t b = min(b0 + u, b_end - 1);  // tail: reload the last block, masked below
      if constexpr (DT == SNL_Q8_0) {
        const uint2 va = ld_w8(wA + (uint64_t)b * 32 + 8 * t), vb = ld_w8(wB + (uint64_t)b * 32 + 8 * t);
        wa[u][0] = va.x; wa[u][1] = va.y; wb[u][0] = vb.x; wb[u][1] = vb.y;
      } else {
        wa[u][0] = ld_w4(wA + (uint64_t)b * 16 + 4 * t);
        wb[u][0] = ld_w4(wB + (uint64_t)b * 16 + 4 * t);
      }
      sa[u] = scale_at(sA, b);
      sb[u] = scale_at(sB, b);
      xv[u] = has_x ? __ldg(reinterpret_cast<const uint4*>(xp + (uint64_t)b * 32)) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; u++) {
      if (b0 + u >= b_end) break;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      if constexpr (DT == SNL_Q8_0) {
        uint32_t A0[4], A1[4];
        q8_half2(wa[u][0], A0[0], A0[2]);
        q8_half2(wb[u][0], A0[1], A0[3]);
        q8_half2(wa[u][1], A1[0], A1[2]);
        q8_half2(wb[u][1], A1[1], A1[3]);
        mma16816(d, A0, xv[u].x, xv[u].y);
        mma16816(d, A1, xv[u].z, xv[u].w);
      } else {
        uint32_t ha[4], hb[4];
        q4_half2(wa[u][0], ha);
        q4_half2(wb[u][0], hb);
        // B pairs (8t+i, 8t+i+4) from the natural-order halves x[8t..8t+8).
        const uint32_t x01 = xv[u].x, x23 = xv[u].y, x45 = xv[u].z, x67 = xv[u].w;
        const uint32_t p04 = __byte_perm(x01, x45, 0x5410), p15 = __byte_perm(x01, x45, 0x7632);
        const uint32_t p26 = __byte_perm(x23, x67, 0x5410), p37 = __byte_perm(x23, x67, 0x7632);
        const uint32_t A0[4] = {ha[0], hb[0], ha[1], hb[1]};
        const uint32_t A1[4] = {ha[2], hb[2], ha[3], hb[3]};
        mma16816(d, A0, p04, p15);
        mma16816(d, A1, p26, p37);
      }
      // d0/d1: row g, columns 2t (hi) and 2t+1 (lo); d2/d3: row g+8.
      accA = fmaf(sa[u], d[0] + d[1], accA);
      accB = fmaf(sb[u], d[2] + d[3], accB);
    }
  }
  if (t < M) {
    red[warp][t][g] = accA;
    red[warp][t][g + 8] = accB;
  }
  __syncthreads();
  if (warp == 0) {
    // lanes 0..15: token 0 rows, 16..31: token 1 rows; tokens 2, 3 in a second pass.
#pragma unroll
    for (int pass = 0; pass < (M + 1) / 2; pass++) {
      const int tt = pass * 2 + lane / 16, r = lane % 16;
      const uint32_t row = row0 + r;
      const bool live = tt < M && row < a.n;
      float2 nx = make_float2(0.f, 0.f);
      if (live) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarpsK; w++) v += red[w][tt][r];
        nx = gemv_epilogue(a, tt, row, v * kXPlaneScale);
      }
      merge_partials(a, tt, row, live, nx, (uint64_t)tt * gridDim.x + blockIdx.x, r == 0 && tt < M);
    }
  }
}

template <int DT, int M, typename ST>
int launch_t(const GemvArgs& a, const void* ws, cudaStream_t s) {
  const unsigned grid = (a.n + 15) / 16;
  gemv_mma_kernel<DT, M, ST><<<grid, kWarpsK * 32, 0, s>>>(a, static_cast<const ST*>(ws));
  SNL_LAUNCH_CHECK("gemv_mma");
  return SNL_OK;
}

template <int DT, typename ST>
int launch_m(const GemvArgs& a, uint32_t m, const void* ws, cudaStream_t s) {
  switch (m) {
    case 1: return launch_t<DT, 1, ST>(a, ws, s);
    case 2: return launch_t<DT, 2, ST>(a, ws, s);
    case 3: return launch_t<DT, 3, ST>(a, ws, s);
    case 4: return launch_t<DT, 4, ST>(a, ws, s);
  }
  return fail(SNL_E_INVALID, "gemv_mma: 1..4 token rows");
}

// x [m, x_stride] f32 -> planes [2m][plane_stride] halves (hi, lo per token).
__global__ void xpack_kernel(const float* __restrict__ x, uint32_t k, uint32_t x_stride, uint32_t m,
                             __half* __restrict__ planes, uint32_t plane_stride) {
  pdl_trigger();
  pdl_wait();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t t = blockIdx.y;
  if (i >= k || t >= m) return;
  xplane_store(planes, plane_stride, t, i, x[(uint64_t)t * x_stride + i]);
}

}  // namespace

int launch_gemv_mma(int dtype, const GemvArgs& a, uint32_t m, const void* ws, int scale_f16, cudaStream_t s) {
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return fail(SNL_E_INVALID, "gemv_mma: dtype");
  if (a.k == 0 || a.k % 32) return fail(SNL_E_INVALID, "gemv_mma: k must be a multiple of 32");
  if (a.plane_stride % 8 || ((uintptr_t)a.xplanes % 16)) return fail(SNL_E_INVALID, "gemv_mma: planes must be 16-byte aligned");
  if (a.n == 0) return SNL_OK;
  if (dtype == SNL_Q8_0)
    return scale_f16 ? launch_m<SNL_Q8_0, __half>(a, m, ws, s) : launch_m<SNL_Q8_0, float>(a, m, ws, s);
  return scale_f16 ? launch_m<SNL_Q4_0, __half>(a, m, ws, s) : launch_m<SNL_Q4_0, float>(a, m, ws, s);
}

int launch_xpack(const float* x, uint32_t m, uint32_t k, uint32_t x_stride, __half* planes, uint32_t plane_stride,
                 cudaStream_t s) {
  if (m == 0 || k == 0) return SNL_OK;
  SNL_PDL_LAUNCH("xpack_kernel", xpack_kernel, dim3(dim3((k + 255) / 256, m)), dim3(256), (size_t)(0), s, x, k, x_stride, m, planes, plane_stride);
  return SNL_OK;
}

}  // namespace snl

extern "C" int snl_xpack(const float* x, uint32_t m, uint32_t k, uint32_t x_stride, void* planes, void* stream) {
  if (!x || !planes || m == 0 || m > 4) return snl::fail(SNL_E_INVALID, "snl_xpack: bad argument");
  if (k % 32 || x_stride < k) return snl::fail(SNL_E_INVALID, "snl_xpack: k must be a multiple of 32");
  return snl::launch_xpack(x, m, k, x_stride, static_cast<__half*>(planes), k, (cudaStream_t)stream);
}

extern "C" int snl_mat_xpack(int dtype, const snl_mat_p* p, uint32_t rows_m, const void* planes, const void* wq,
                             const float* ws, float* y, void* stream) {
  if (!p || !planes || !wq || !ws || !y) return snl::fail(SNL_E_INVALID, "snl_mat_xpack: null argument");
  if (rows_m == 0 || rows_m > 4) return snl::fail(SNL_E_INVALID, "snl_mat_xpack: 1..4 token rows");
  snl::GemvArgs a = snl::gemv_args_plain(*p, static_cast<const __half*>(planes), p->k, wq, y);
  return snl::launch_gemv_mma(dtype, a, rows_m, ws, 0, (cudaStream_t)stream);
}

// =====================================================================================
// Tile layout and the tile GEMV (the engine's decode path).
//
// The decode GEMV is issue-bound on the reference layout: every 16-row x 32-k tile
// costs ~60 warp instructions (two 8-byte loads per thread at row stride, an xor,
// address arithmetic). The engine therefore keeps a second copy of each matrix in a
// "tile layout" made for the MMA fragments:
//   * rows are grouped by 16 (padded with zero rows); within a group, block b (32 k)
//     is one 512-byte Q8_0 tile (256 bytes for Q4_0) and the tiles of a group follow
//     each other along k;
//   * in a Q8_0 tile, lane L = 4g + t owns bytes [16L, 16L + 16): bytes [8t, 8t + 8) of
//     the block of row g, then the same bytes of row g + 8, each code stored as
//     code + 128 (offset binary), so a warp reads 512 contiguous bytes with one 16-byte
//     load per thread and the fp16 conversion needs no xor;
//   * in a Q4_0 tile, lane L owns 8 bytes: word t of row g, then word t of row g + 8,
//     with nibble i of word t holding element 8t + 2(i % 4) + (i / 4) (nibbles i and
//     i + 4 form the pair (8t + 2j, 8t + 2j + 1) that matches the natural-order x halves);
//   * scales: per row group, blocks in fours: [group][b / 4][16 rows][4 blocks], as fp16
//     when every block scale of the matrix is an fp16 number (checked before the repack;
//     true of Q8_0/Q4_0 files whose scales came from fp16 blocks), else as f32, the file's
//     own values.
// The values are the file's, bit for bit; only their order changes.
// =====================================================================================

namespace snl {
namespace {

// pair_half != 0 (n = 2 * pair_half, pair_half % 8 == 0): group grp holds rows
// 8*grp .. 8*grp+7 in its first 8 rows and pair_half + 8*grp .. +7 in the last 8, so a
// [gate; up] matrix puts each gate row in the group of its up row (the SwiGLU epilogue).
__device__ __forceinline__ uint32_t tile_row(uint32_t grp, uint32_t r, uint32_t pair_half) {
  return pair_half ? (r < 8 ? 8 * grp + r : pair_half + 8 * grp + (r - 8)) : grp * 16 + r;
}

__global__ void repack_tiles_kernel(int dtype, uint32_t n, uint32_t k, const uint8_t* __restrict__ q,
                                    const float* __restrict__ s, uint8_t* __restrict__ tiles, void* __restrict__ ts,
                                    int ts_f16, uint32_t pair_half) {
  // one thread per (group, block, lane)
  const uint32_t nb = k / 32, groups = (n + 15) / 16;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)groups * nb * 32) return;
  const uint32_t lane = (uint32_t)(idx % 32), b = (uint32_t)((idx / 32) % nb), grp = (uint32_t)(idx / 32 / nb);
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t rA = tile_row(grp, g, pair_half), rB = tile_row(grp, g + 8, pair_half);
  const uint64_t tile = (uint64_t)grp * nb + b;
  if (dtype == SNL_Q8_0) {
    uint8_t* dst = tiles + tile * 512 + lane * 16;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      dst[e] = rA < n ? (uint8_t)(q[(uint64_t)rA * k + b * 32 + 8 * t + e] ^ 0x80u) : (uint8_t)0x80u;
      dst[8 + e] = rB < n ? (uint8_t)(q[(uint64_t)rB * k + b * 32 + 8 * t + e] ^ 0x80u) : (uint8_t)0x80u;
    }
  } else {
    uint32_t* dst = reinterpret_cast<uint32_t*>(tiles + tile * 256 + lane * 8);
    for (int r = 0; r < 2; r++) {
      const uint32_t row = r ? rB : rA;
      uint32_t word = 0x88888888u;  // padding rows: nibble 8 = value 0
      if (row < n) {
        const uint32_t src = reinterpret_cast<const uint32_t*>(q + (uint64_t)row * (k / 2))[b * 4 + t];
        word = 0;
        for (int i = 0; i < 8; i++) {
          const uint32_t e = 2 * (i % 4) + (i / 4);  // element 8t + e goes to nibble i
          word |= ((src >> (4 * e)) & 0xFu) << (4 * i);
        }
      }
      dst[r] = word;
    }
  }
  // scales: lanes 0..15 of each (group, block) write row `lane`'s scale.
  if (lane < 16) {
    const uint32_t row = tile_row(grp, lane, pair_half);
    const uint32_t nb4 = (nb + 3) / 4;
    const float v = row < n ? s[(uint64_t)row * nb + b] : 0.f;
    const uint64_t i = (((uint64_t)grp * nb4 + b / 4) * 16 + lane) * 4 + b % 4;
    if (ts_f16) static_cast<__half*>(ts)[i] = __float2half_rn(v);
    else static_cast<float*>(ts)[i] = v;
  }
}

// Q8 codes stored as code + 128: half2(code_a, code_b) with one permute and one subtract.
// Sets *inexact if any of the count scales is not an fp16 number.
__global__ void fp16_exact_kernel(const float* __restrict__ s, uint64_t count, int* __restrict__ inexact) {
  bool bad = false;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (uint64_t)gridDim.x * blockDim.x) {
    const float v = s[i];
    bad |= !(__half2float(__float2half_rn(v)) == v);
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(inexact, 1);
}

__device__ __forceinline__ float scale_f(float v) { return v; }
__device__ __forceinline__ float scale_f(__half v) { return __half2float(v); }

__device__ __forceinline__ uint32_t u8pair(uint32_t w, uint32_t sel) {
  return hsub2_u32(__byte_perm(w, 0x64646464u, sel), 0x64806480u);
}

// ---------------------------------------------------------------------------
// Persistent row-group tile GEMV (the default decode GEMV).
//
// A grid of up to kPgCtasPerSm CTAs per SM; CTA b owns the contiguous row groups
// [b*G/grid, (b+1)*G/grid). The warps of a CTA split every group's K range
// into equal runs of stages (kPgTiles tiles plus their scales, one contiguous bulk copy
// each), stream them through a per-warp ring of kStages stages, and meet once per group
// in shared memory, where warp 0 adds the warp partials in warp order and runs the
// epilogue (double-buffered, so the other warps go on streaming the next group).
// The first stages are issued before pdl_wait(): the weights are constant during a
// step, so their copies overlap the tail of the kernel before.
// ---------------------------------------------------------------------------
// Two shapes of CTA: matrices with many row groups use 8 warps with 2 stages each, 3
// CTAs per SM (registers capped for that); matrices with few groups (n <= 16 * 2 * SMs,
// the 4096-row projections) get one 16-warp CTA per group, 2 per SM, each warp one
// stage of its 1/16 of K, so more bytes are in flight per group.
constexpr int kPgTiles = 8;
constexpr int kPgCtasPerSm = 3;

template <int DT, int WARPS, int S, typename ST>
struct PgGeom {
  static constexpr uint32_t TB = DT == SNL_Q8_0 ? 512 : 256;
  static constexpr uint32_t kStageW = kPgTiles * TB;
  static constexpr uint32_t kStageS = kPgTiles / 4 * 64 * sizeof(ST);  // scales: 16 rows x 4 blocks per four tiles
  static constexpr uint32_t kStage = kStageW + kStageS;
  static constexpr uint32_t kWarpBytes = S * kStage;
  static constexpr uint32_t kSmem = WARPS * kWarpBytes + WARPS * S * 8;
};

// The epilogue of one finished row group, run by one warp: val(tt, r) is the dot of
// token tt, row 16*grp + r (lanes 16*j + r handle token 2*pass + j). Norm partials
// go to rpart slot tt * groups + grp (merge_partials).
template <int M, class V>
__device__ __forceinline__ void finish_body(const GemvArgs& a, uint32_t grp, uint32_t groups, int lane, V&& val) {
  if (a.mode == 2) {
    // SwiGLU (layers.wgsl `swiglu`): rows 0-7 of the group are gate rows 8*grp + r,
    // rows 8-15 the matching up rows (tiles repacked with pair_half).
#pragma unroll
    for (int pass = 0; pass < (M + 1) / 2; pass++) {
      const int tt = pass * 2 + lane / 16, r = lane % 16;
      const float v = tt < M ? val(tt, r) * kXPlaneScale : 0.f;
      const float up = __shfl_down_sync(0xffffffffu, v, 8);
      if (tt < M && r < 8) {
        const uint32_t i = grp * 8 + r;
        const float act = v / (1.0f + __expf(-v)) * up;
        if (a.y) a.y[(uint64_t)tt * a.y_stride + i] = act;
        xplane_store(a.act_planes, a.act_stride, tt, i, act);
      }
    }
    return;
  }
  if (a.tp.size > 1) {
    // Row-parallel projection: push this rank's partials of the group into every peer's
    // memory as tagged words, collect the peers' from this rank's memory, and merge the
    // sum of all ranks' partials in rank order (identical on every rank).
    const uint64_t epoch = tp_epoch(a.tp, a.tp_site);
    const uint32_t tag = (uint32_t)epoch;
    const uint64_t par = epoch & 1;
    const int N = a.tp.size, me = a.tp.rank;
    float own[(M + 1) / 2];
#pragma unroll
    for (int pass = 0; pass < (M + 1) / 2; pass++) {
      const int tt = pass * 2 + lane / 16, r = lane % 16;
      const uint32_t row = grp * 16 + r;
      own[pass] = 0.f;
      if (tt < M && row < a.n) {
        own[pass] = val(tt, r);
        const unsigned long long w = ll_word(tag, __float_as_uint(own[pass]));
        for (int q = 0; q < N; q++)
          if (q != me) st_relaxed_sys_u64(a.tp.ll[q] + ((par * kTpMax + me) * 4 + tt) * a.tp.gp_rows + row, w);
      }
    }
#pragma unroll
    for (int pass = 0; pass < (M + 1) / 2; pass++) {
      const int tt = pass * 2 + lane / 16, r = lane % 16;
      const uint32_t row = grp * 16 + r;
      const bool live = tt < M && row < a.n;
      float2 nx = make_float2(0.f, 0.f);
      if (live) {
        float v = 0.f;
        for (int q = 0; q < N; q++)
          v += q == me ? own[pass]
                       : __uint_as_float(ll_wait(a.tp, a.tp.ll[me] + ((par * kTpMax + q) * 4 + tt) * a.tp.gp_rows + row, tag));
        nx = gemv_epilogue(a, tt, row, v * kXPlaneScale);
      }
      merge_partials(a, tt, row, live, nx, (uint64_t)tt * groups + grp, r == 0 && tt < M);
    }
    return;
  }
#pragma unroll
  for (int pass = 0; pass < (M + 1) / 2; pass++) {
    const int tt = pass * 2 + lane / 16, r = lane % 16;
    const uint32_t row = grp * 16 + r;
    const bool live = tt < M && row < a.n;
    float2 nx = make_float2(0.f, 0.f);
    if (live) nx = gemv_epilogue(a, tt, row, val(tt, r) * kXPlaneScale);
    merge_partials(a, tt, row, live, nx, (uint64_t)tt * groups + grp, r == 0 && tt < M);
  }
}

// A finished row group. With a fused norm the M dot products are the two weighted
// streams of M/2 tokens, combined as c0 * stream 0 + c1 * stream 1 with the token's
// coefficients nrm[2 tt], nrm[2 tt + 1] (pre0 * rinv, pre1 * rinv) before the epilogue.
template <int M, class V>
__device__ __forceinline__ void group_finish(const GemvArgs& a, uint32_t grp, uint32_t groups, int lane, V&& val,
                                             const float* nrm) {
  if constexpr (M % 2 == 0) {
    if (a.fused_norm) {
      finish_body<M / 2>(a, grp, groups, lane, [&](int tt, int r) {
        return nrm[2 * tt] * val(2 * tt, r) + nrm[2 * tt + 1] * val(2 * tt + 1, r);
      });
      return;
    }
  }
  finish_body<M>(a, grp, groups, lane, val);
}

// Fused-norm prologue (one warp): the norm's router coefficients and 1 / rms of each of
// the T tokens from the producing GEMV's per-group partials, into nrm (see group_finish);
// block 0 also writes the coefficients for the later residual merge (layers.wgsl
// branch_norm + mhc_finish, the separate kernels' math).
template <int T>
__device__ __forceinline__ void fused_norm_prologue(const GemvArgs& a, int lane, float* nrm) {
  static_assert(kRpStride % 4 == 0 && kRpStride >= 11, "a part is whole float4s holding 11 sums");
#pragma unroll 1
  for (int tt = 0; tt < T; tt++) {
    float acc[11];
#pragma unroll
    for (int o = 0; o < 11; o++) acc[o] = 0.f;
    // Parts lane, lane + 32, ... in batches of 4 whose 12 vector loads are all in flight
    // before the first add; the adds keep the part order, so the sums are unchanged.
    const float4* rp4 = reinterpret_cast<const float4*>(a.nrpart + (uint64_t)tt * a.nparts * kRpStride);
    for (uint32_t i0 = lane; i0 < a.nparts; i0 += 32 * 4) {
      float4 v[4][3];
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const uint32_t i = i0 + 32 * b;
#pragma unroll
        for (int q = 0; q < 3; q++)
          v[b][q] = i < a.nparts ? rp4[(uint64_t)i * (kRpStride / 4) + q] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int b = 0; b < 4; b++) {
        if (i0 + 32 * b >= a.nparts) break;
        const float f[11] = {v[b][0].x, v[b][0].y, v[b][0].z, v[b][0].w, v[b][1].x, v[b][1].y,
                             v[b][1].z, v[b][1].w, v[b][2].x, v[b][2].y, v[b][2].z};
#pragma unroll
        for (int o = 0; o < 11; o++) acc[o] += f[o];
      }
    }
#pragma unroll
    for (int o = 0; o < 11; o++) acc[o] = warp_sum(acc[o]);
    if (lane == 0) {
      float pre0 = 1.f, pre1 = 0.f;
      if (a.nrouter) {
        float raw[9], bias[8], cb[8];
#pragma unroll
        for (int o = 0; o < 8; o++) {
          raw[o] = acc[o];
          bias[o] = a.nrouter[(uint64_t)16 * a.h + o];
        }
        raw[8] = acc[8] + acc[9];
        mhc_coef_b(raw, bias, 2 * a.h, a.niter, cb);
        pre0 = cb[0];
        pre1 = cb[1];
        if (blockIdx.x == 0) {
#pragma unroll
          for (int o = 0; o < 8; o++) a.ncoef[tt * 8 + o] = cb[o];
        }
      }
      const float ss = fmaf(pre0 * pre0, acc[8], fmaf(2.f * pre0 * pre1, acc[10], pre1 * pre1 * acc[9]));
      const float rinv = rsqrtf(ss / (float)a.h + a.neps);
      nrm[2 * tt] = pre0 * rinv;
      nrm[2 * tt + 1] = pre1 * rinv;
    }
  }
}

template <int DT, int M, int WARPS, int S, typename ST>
__global__ void __launch_bounds__(WARPS * 32, WARPS >= 16 ? 2 : 3) gemv_pg_kernel(GemvArgs a, const uint8_t* __restrict__ tiles,
                                                             const ST* __restrict__ ts, uint32_t groups, int* err) {
  using G = PgGeom<DT, WARPS, S, ST>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[2][WARPS][M][16];
  __shared__ float nrm[M];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t nb = a.k / 32, nb4 = (nb + 3) / 4;
  const uint32_t spg = (nb + kPgTiles - 1) / kPgTiles;
  const uint32_t per = (spg + WARPS - 1) / WARPS;
  const uint32_t st0 = min(spg, warp * per), nst = min(spg, st0 + per) - st0;
  const uint32_t g0 = (uint32_t)((uint64_t)blockIdx.x * groups / gridDim.x);
  const uint32_t g1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * groups / gridDim.x);
  const uint32_t njobs = (g1 - g0) * nst;
  uint8_t* ring = smem + warp * G::kWarpBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WARPS * G::kWarpBytes) + warp * S;

  if (lane == 0)
    for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
  fence_mbar_init();
  __syncwarp();
  const uint64_t pol = l2_policy_evict_first();
  auto issue = [&](uint32_t j) {
    if (lane != 0) return;
    const uint32_t grp = g0 + j / nst, sg = st0 + j % nst;
    const uint32_t nt = min((uint32_t)kPgTiles, nb - sg * kPgTiles);
    const uint32_t wbytes = nt * G::TB, sbytes = (nt + 3) / 4 * 64 * (uint32_t)sizeof(ST);
    uint8_t* st = ring + (j % S) * G::kStage;
    mbar_arrive_expect_tx(&bars[j % S], wbytes + sbytes);
    bulk_g2s(st, tiles + ((uint64_t)grp * nb + sg * kPgTiles) * G::TB, wbytes, &bars[j % S], pol);
    bulk_g2s(st + G::kStageW, ts + ((uint64_t)grp * nb4 + sg * (kPgTiles / 4)) * 64, sbytes, &bars[j % S], pol);
  };
  // The epilogue operands of this CTA's first group go to L2 early (its dot products hide
  // the fetch): a residual merge's router and norm weights (constant) before the wait, its
  // residual rows and merge coefficients (written by earlier kernels) right after it.
  const bool pf = a.mode == 1 && warp == WARPS - 1 && g0 < g1;
  const uint32_t prow = g0 * 16;  // 16 rows = one 64-byte line per array
  if (pf) {
    if (a.rnext && lane < 16)
      prefetch_l2(a.rnext + (uint64_t)(lane >> 1) * 2 * a.h + (lane & 1) * a.h + prow);
    if (a.nw && lane == 16) prefetch_l2(a.nw + prow);
  }
  for (uint32_t j = 0; j < min((uint32_t)S, njobs); j++) issue(j);
  pdl_wait();
  if (pf && lane < 2 * M) {
    const uint32_t tt = lane >> 1;
    prefetch_l2(a.resid + (uint64_t)tt * 2 * a.h + (lane & 1) * a.h + prow);
    if ((lane & 1) == 0 && a.coef) prefetch_l2(a.coef + tt * 8);
  }
  if constexpr (M % 2 == 0) {
    // Visible to the epilogue through the first group's __syncthreads.
    if (a.fused_norm && warp == 0) fused_norm_prologue<M / 2>(a, lane, nrm);
  }

  const bool has_x = g < 2 * M;
  const __half* xbase = a.xplanes + (uint64_t)(has_x ? g : 0) * a.plane_stride + 8 * t;
  bool ok = true;
  uint32_t j_fail = 0, j = 0;
  for (uint32_t gi = 0; gi < g1 - g0; gi++) {
    float accA = 0.f, accB = 0.f;
    for (uint32_t si = 0; si < nst; si++, j++) {
      if (!ok) continue;
      const uint32_t sg = st0 + si;
      const uint32_t nt = min((uint32_t)kPgTiles, nb - sg * kPgTiles);
      const bool full = nt == (uint32_t)kPgTiles;
      uint4 xv[kPgTiles];
      if (full) {
        // A full stage (every stage when k is a multiple of 256): one base address,
        // constant offsets, no per-tile bound checks.
        const uint4* xs = reinterpret_cast<const uint4*>(xbase + (uint64_t)sg * (kPgTiles * 32));
#pragma unroll
        for (int u = 0; u < kPgTiles; u++) xv[u] = has_x ? __ldg(xs + 4 * u) : make_uint4(0, 0, 0, 0);
      } else {
#pragma unroll
        for (int u = 0; u < kPgTiles; u++) {
          const uint32_t uu = min((uint32_t)u, nt - 1);
          xv[u] = has_x ? __ldg(reinterpret_cast<const uint4*>(xbase + ((uint64_t)sg * kPgTiles + uu) * 32))
                        : make_uint4(0, 0, 0, 0);
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bars[j % S], (j / S) & 1))) {
        ok = false;
        j_fail = j;
        continue;
      }
      const uint8_t* st = ring + (j % S) * G::kStage;
      const ST* sc = reinterpret_cast<const ST*>(st + G::kStageW);
      auto tile = [&](int u) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (DT == SNL_Q8_0) {
          const uint4 w = *reinterpret_cast<const uint4*>(st + u * G::TB + lane * 16);
          const uint32_t A0[4] = {u8pair(w.x, 0x4140), u8pair(w.z, 0x4140), u8pair(w.x, 0x4342), u8pair(w.z, 0x4342)};
          const uint32_t A1[4] = {u8pair(w.y, 0x4140), u8pair(w.w, 0x4140), u8pair(w.y, 0x4342), u8pair(w.w, 0x4342)};
          mma16816(d, A0, xv[u].x, xv[u].y);
          mma16816(d, A1, xv[u].z, xv[u].w);
        } else {
          const uint2 w = *reinterpret_cast<const uint2*>(st + u * G::TB + lane * 8);
          // Tile nibble order: nibbles (j, j + 4) of a word are elements (8t + 2j, 8t + 2j + 1).
          uint32_t hx[4], hy[4];
          q4_half2(w.x, hx);
          q4_half2(w.y, hy);
          const uint32_t A0[4] = {hx[0], hy[0], hx[1], hy[1]};
          const uint32_t A1[4] = {hx[2], hy[2], hx[3], hy[3]};
          mma16816(d, A0, xv[u].x, xv[u].y);
          mma16816(d, A1, xv[u].z, xv[u].w);
        }
        const float scA = scale_f(sc[(u / 4) * 64 + g * 4 + (u % 4)]);
        const float scB = scale_f(sc[(u / 4) * 64 + (g + 8) * 4 + (u % 4)]);
        accA = fmaf(scA, d[0] + d[1], accA);
        accB = fmaf(scB, d[2] + d[3], accB);
      };
      if (full) {
#pragma unroll
        for (int u = 0; u < kPgTiles; u++) tile(u);
      } else {
#pragma unroll
        for (int u = 0; u < kPgTiles; u++) {
          if ((uint32_t)u >= nt) break;
          tile(u);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (j + S < njobs) issue(j + S);
    }
    // All warps meet once per group; warp 0 sums the partials in warp order.
    const int buf = gi & 1;
    if (t < M) {
      red[buf][warp][t][g] = accA;
      red[buf][warp][t][g + 8] = accB;
    }
    __syncthreads();
    if (warp == 0)
      group_finish<M>(a, g0 + gi, groups, lane, [&](int tt, int r) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < WARPS; w++) v += red[buf][w][tt][r];
        return v;
      }, nrm);
  }
  if (!ok) {
    // A bounded wait gave up: flag it and let the copies still in flight land before
    // the CTA exits.
    if (lane == 0) report_timeout(err);
    const uint32_t last = min(njobs, j_fail + S);
    for (uint32_t k2 = j_fail; k2 < last; k2++) (void)mbar_wait_bounded(&bars[k2 % S], (k2 / S) & 1);
  }
}

// Grid of the persistent tile GEMV for `groups` row groups and `slots` resident CTAs. With
// more groups than slots, a full grid leaves some CTAs one group more than others, and
// the kernel's last phase runs on those alone, below the HBM rate. When the largest share
// is 4 groups or more, the grid is the smallest one that still gives every CTA at most
// ceil(groups / slots) groups (1536 groups over 444 slots: 384 CTAs of 4, not 204 of 4
// and 240 of 3): decode 278.8 -> 279.9 tok/s, same box A/B. With fewer groups per CTA the
// full grid's extra bytes in flight win (768 groups: 384 CTAs of 2 took 10.62 us against
// 10.15 us for 444 CTAs of 1 or 2). SNL_PG_FILL=1 fills every slot.
uint32_t pg_grid(uint32_t groups, uint32_t slots) {
  static const bool fill = getenv("SNL_PG_FILL") != nullptr;
  if (groups <= slots || fill) return std::min(groups, slots);
  const uint32_t q = (groups + slots - 1) / slots;
  if (q < 4) return slots;
  return (groups + q - 1) / q;
}

template <int DT, int M, int WARPS, int S, typename ST>
int launch_pg_cfg(const GemvArgs& a, const void* tiles, const ST* ts, uint32_t groups, int* err, cudaStream_t s) {
  using G = PgGeom<DT, WARPS, S, ST>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = gemv_pg_kernel<DT, M, WARPS, S, ST>;
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_pg: smem attribute");
    attr[dev] = true;
  }
  const uint32_t grid = pg_grid(groups, (uint32_t)sm_count() * kPgCtasPerSm);
  SNL_PDL_LAUNCH("gemv_pg", kern, dim3(grid), dim3(WARPS * 32), (size_t)G::kSmem, s, a,
                 static_cast<const uint8_t*>(tiles), ts, groups, err);
  return SNL_OK;
}

template <int DT, int M, typename ST>
int launch_pg_t(const GemvArgs& a, const void* tiles, const ST* ts, int* err, cudaStream_t s) {
  const uint32_t groups = (a.n + 15) / 16;
  const bool few = groups <= 2u * (uint32_t)sm_count();
  constexpr int kSA = DT == SNL_Q8_0 ? 2 : 3;  // stages per warp, 8-warp CTA
  if (few) return launch_pg_cfg<DT, M, 16, 1, ST>(a, tiles, ts, groups, err, s);
  return launch_pg_cfg<DT, M, 8, kSA, ST>(a, tiles, ts, groups, err, s);
}

}  // namespace

void tile_sizes(int dtype, uint32_t n, uint32_t k, size_t* tile_bytes, size_t* scale_floats) {
  const size_t groups = (n + 15) / 16, nb = k / 32, nb4 = (nb + 3) / 4;
  *tile_bytes = groups * nb * (dtype == SNL_Q8_0 ? 512 : 256);
  *scale_floats = groups * nb4 * 64;
}

int scales_fp16_exact(const float* s, uint64_t count, int* dflag, bool* exact, cudaStream_t st) {
  if (!dflag || !exact) return fail(SNL_E_INVALID, "scale check: no flag");
  cudaError_t e = cudaMemsetAsync(dflag, 0, sizeof(int), st);
  if (e != cudaSuccess) return cuda_fail(e, "scale check: memset");
  if (count) {
    const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, (uint64_t)sm_count() * 8);
    fp16_exact_kernel<<<(unsigned)blocks, 256, 0, st>>>(s, count, dflag);
    SNL_LAUNCH_CHECK("fp16_exact");
  }
  int h = 0;
  e = cudaMemcpyAsync(&h, dflag, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "scale check: flag");
  *exact = h == 0;
  return SNL_OK;
}

int launch_repack_tiles(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, void* tiles, void* ts,
                        int ts_f16, cudaStream_t st, uint32_t pair_half) {
  if (k % 32 || n == 0) return fail(SNL_E_INVALID, "repack: k must be a multiple of 32");
  if (pair_half && (n != 2 * pair_half || pair_half % 8)) return fail(SNL_E_INVALID, "repack: bad row pairing");
  size_t tb, sf;
  tile_sizes(dtype, n, k, &tb, &sf);
  // Scales of blocks past k in the last four stay zero.
  cudaError_t e = cudaMemsetAsync(ts, 0, sf * (ts_f16 ? sizeof(__half) : sizeof(float)), st);
  if (e != cudaSuccess) return cuda_fail(e, "repack: memset");
  const uint64_t threads = (uint64_t)((n + 15) / 16) * (k / 32) * 32;
  repack_tiles_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      dtype, n, k, static_cast<const uint8_t*>(q), s, static_cast<uint8_t*>(tiles), ts, ts_f16, pair_half);
  SNL_LAUNCH_CHECK("repack_tiles");
  return SNL_OK;
}

template <typename ST>
int launch_gemv_tile_t(int dtype, const GemvArgs& a, uint32_t m, const void* tiles, const ST* ts, cudaStream_t s) {
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  if (dtype == SNL_Q8_0) {
    switch (m) {
      case 1: return launch_pg_t<SNL_Q8_0, 1, ST>(a, tiles, ts, err, s);
      case 2: return launch_pg_t<SNL_Q8_0, 2, ST>(a, tiles, ts, err, s);
      case 3: return launch_pg_t<SNL_Q8_0, 3, ST>(a, tiles, ts, err, s);
      case 4: return launch_pg_t<SNL_Q8_0, 4, ST>(a, tiles, ts, err, s);
    }
  } else if (dtype == SNL_Q4_0) {
    switch (m) {
      case 1: return launch_pg_t<SNL_Q4_0, 1, ST>(a, tiles, ts, err, s);
      case 2: return launch_pg_t<SNL_Q4_0, 2, ST>(a, tiles, ts, err, s);
      case 3: return launch_pg_t<SNL_Q4_0, 3, ST>(a, tiles, ts, err, s);
      case 4: return launch_pg_t<SNL_Q4_0, 4, ST>(a, tiles, ts, err, s);
    }
  }
  return fail(SNL_E_INVALID, "gemv_tile: dtype / rows");
}

int launch_gemv_tile(int dtype, const GemvArgs& a, uint32_t m, const void* tiles, const void* ts, int ts_f16,
                     cudaStream_t s) {
  if (a.k == 0 || a.k % 32) return fail(SNL_E_INVALID, "gemv_tile: k must be a multiple of 32");
  if (a.plane_stride % 8 || ((uintptr_t)a.xplanes % 16)) return fail(SNL_E_INVALID, "gemv_tile: planes alignment");
  if (a.n == 0) return SNL_OK;
  if (a.mode == 2 && (!a.act_planes || a.n % 16)) return fail(SNL_E_INVALID, "gemv_tile: swiglu epilogue arguments");
  if (a.fused_norm && (m % 2 || a.mode == 1 || !a.nrpart)) return fail(SNL_E_INVALID, "gemv_tile: fused norm arguments");
  if (ts_f16) return launch_gemv_tile_t(dtype, a, m, tiles, static_cast<const __half*>(ts), s);
  return launch_gemv_tile_t(dtype, a, m, tiles, static_cast<const float*>(ts), s);
}

}  // namespace snl

extern "C" int snl_tile_sizes(int dtype, uint32_t n, uint32_t k, size_t* tile_bytes, size_t* scale_bytes) {
  if (!tile_bytes || !scale_bytes || (dtype != SNL_Q8_0 && dtype != SNL_Q4_0)) return snl::fail(SNL_E_INVALID, "snl_tile_sizes");
  size_t sf = 0;
  snl::tile_sizes(dtype, n, k, tile_bytes, &sf);
  *scale_bytes = sf * sizeof(float);
  return SNL_OK;
}
extern "C" int snl_tile_repack(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, void* tiles,
                               void* tile_scales, int* scales_f16, void* stream) {
  if (!q || !s || !tiles || !tile_scales || !scales_f16 || (dtype != SNL_Q8_0 && dtype != SNL_Q4_0))
    return snl::fail(SNL_E_INVALID, "snl_tile_repack: bad argument");
  if (k % 32) return snl::fail(SNL_E_INVALID, "snl_tile_repack: k must be a multiple of 32");
  int* dflag = nullptr;
  if (cudaMalloc(&dflag, sizeof(int)) != cudaSuccess) return snl::fail(SNL_E_OOM, "snl_tile_repack: flag");
  bool exact = false;
  int rc = snl::scales_fp16_exact(s, (uint64_t)n * (k / 32), dflag, &exact, (cudaStream_t)stream);
  cudaFree(dflag);
  if (rc) return rc;
  *scales_f16 = exact ? 1 : 0;
  return snl::launch_repack_tiles(dtype, n, k, q, s, tiles, tile_scales, *scales_f16, (cudaStream_t)stream);
}
extern "C" int snl_mat_tiles(int dtype, const snl_mat_p* p, uint32_t rows_m, const void* planes, const void* tiles,
                             const void* tile_scales, int scales_f16, float* y, void* stream) {
  if (!p || !planes || !tiles || !tile_scales || !y) return snl::fail(SNL_E_INVALID, "snl_mat_tiles: null argument");
  if (rows_m == 0 || rows_m > 4) return snl::fail(SNL_E_INVALID, "snl_mat_tiles: 1..4 token rows");
  snl::GemvArgs a = snl::gemv_args_plain(*p, static_cast<const __half*>(planes), p->k, tiles, y);
  return snl::launch_gemv_tile(dtype, a, rows_m, tiles, tile_scales, scales_f16, (cudaStream_t)stream);
}
