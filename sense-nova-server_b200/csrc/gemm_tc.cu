// Block-quantized GEMM for prefill on the 5th-generation tensor cores (tcgen05).
//
// Y[t, n] = sum_k X[t, k] * q[n, k] * s[n, k/32], t < m tokens (matmul.wgsl:204-318,
// `matmul` with load_slice/dequant8, for prefill chunks of up to 512 rows).
//
// CTA tile: 128 weight rows x 256 tokens (128 when 256-token tiles would not fill one
// wave), K in blocks of 64 (two quant blocks). The fp32 accumulator lives in tensor
// memory (128 lanes x one column per token). Precision: both operands are split into
// fp16 hi + lo parts and three products are accumulated (hi*hi + hi*lo + lo*hi), which
// keeps ~21 significant bits, well inside the 1e-3 bar; the dropped lo*lo term is
// below 2^-22 of the result.
//   * A (weights): 8 warps dequantize the file layout (weights.rs:48-55) into two fp16
//     tiles in the swizzled K-major layout of the MMA: v = code * scale * 256,
//     hi = fp16(v), lo = fp16(v - hi). Each thread keeps the raw codes of its half of a
//     K block three blocks ahead in registers.
//   * B (tokens) comes from "x planes" [2][m][k] fp16 (x/16 split into hi and lo),
//     written once per GEMM by tc_xpack_kernel and loaded by TMA with the same swizzle,
//     one K block ahead of its MMAs.
//   * A 9th warp issues the TMA loads and, on one thread, the 12 MMAs of a K block
//     (4 k-steps x 3 products, M=128 N=256 or 128, K=16, kind::f16), committed to the
//     stage's "empty" mbarrier. Dequantization and MMA issue meet only at per-stage
//     mbarriers, never at a CTA-wide barrier.
//   * Epilogue: the 8 dequant warps read the accumulator with tcgen05.ld (warp w: TMEM
//     lanes 32*(w%4).., the (w/4)-th half of the columns) and store y = acc / 16 (16 from
//     the x prescale, 1/256 from the weight prescale).
// Every mbarrier wait is bounded; a wait that gives up sets the device error word, the
// CTA stops issuing work, waits (bounded) for its MMAs, frees its tensor memory and
// returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace snl {
namespace {

constexpr uint32_t kTcM = 128;
// Tile geometry: NT tokens (256 or 128), K blocks of KB (32: one quant block, rows of 64
// bytes, 64-byte swizzle; 64: two quant blocks, 128-byte rows and swizzle), S stages,
// x tiles loaded AH blocks ahead of their MMAs (AH <= S - 1).
template <uint32_t NT, uint32_t KB, int S, uint32_t AH>
struct TcGeom {
  static_assert(KB == 32 || KB == 64, "K block");
  static_assert(AH + 1 <= (uint32_t)S, "lookahead");
  static constexpr uint32_t kRowBytes = KB * 2;
  static constexpr uint32_t kATile = kTcM * KB * 2;
  static constexpr uint32_t kBTile = NT * KB * 2;
  static constexpr uint32_t kStageBytes = 2 * kATile + 2 * kBTile;
  static constexpr uint32_t kSmem = S * kStageBytes + 1024;  // + alignment slack
  // Instruction descriptor, kind::f16: D f32, A and B f16, both K-major, N = NT, M = 128.
  static constexpr uint32_t kIdesc = (1u << 4) | ((NT >> 3) << 17) | ((kTcM >> 4) << 24);
};
constexpr float kAScale = 256.0f;
constexpr float kXPlaneScaleTc = 16.0f;  // x planes hold x / 16 (fp16 range for |x| up to ~1e6)

struct TcArgs {
  uint32_t n, k, m;
  const uint8_t* wq;
  const float* ws;
  float* y;
  uint32_t y_off, y_stride, n_off;
  int* err;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint32_t pack_hl(float a, float b, bool lo) {
  const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
  if (!lo) return (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
  const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
  return (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}

// The raw quants and scale one thread dequantizes per K block: row t/2 of the tile and
// half t%2 of the K block (KB/2 elements, inside one quant block).
struct RawA {
  uint4 w[2];  // Q8: KB/2 codes; Q4: KB/2 nibbles
  float sc;
};

__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

template <int DT, uint32_t KB>
__device__ __forceinline__ RawA load_a(const TcArgs& a, uint32_t n0, uint32_t kb, uint32_t nkb, uint32_t tid) {
  const uint32_t r = tid >> 1, h = tid & 1;
  const uint32_t row = n0 + r;
  const uint32_t e0 = kb * KB + h * (KB / 2);  // first element of this thread's half
  RawA raw{{make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)}, 0.f};
  if (row < a.n && kb < nkb && e0 < a.k) {
    raw.sc = __ldg(a.ws + (uint64_t)row * (a.k / 32) + e0 / 32) * kAScale;
    if constexpr (DT == SNL_Q8_0) {
      const uint8_t* src = a.wq + (uint64_t)row * a.k + e0;
      raw.w[0] = ld_stream16(src);
      if constexpr (KB == 64) raw.w[1] = ld_stream16(src + 16);
    } else {
      const uint8_t* src = a.wq + (uint64_t)row * (a.k / 2) + e0 / 2;
      if constexpr (KB == 64) {
        raw.w[0] = ld_stream16(src);
      } else {
        const uint2 w = ld_stream8(src);
        raw.w[0].x = w.x;
        raw.w[0].y = w.y;
      }
    }
  }
  return raw;
}

// Writes one thread's KB/2 dequantized values as hi and lo fp16 into the A tiles
// (swizzled rows: 16-byte chunk c of row r at chunk c ^ (r % 8) for 128-byte rows,
// c ^ ((r / 2) % 4) for 64-byte rows).
template <int DT, uint32_t KB>
__device__ __forceinline__ void store_a(const RawA& raw, uint8_t* ahi, uint8_t* alo, uint32_t tid) {
  constexpr uint32_t E = KB / 2, RB = KB * 2;
  const uint32_t r = tid >> 1, h = tid & 1;
  float v[E];
  const uint32_t wd[8] = {raw.w[0].x, raw.w[0].y, raw.w[0].z, raw.w[0].w,
                          raw.w[1].x, raw.w[1].y, raw.w[1].z, raw.w[1].w};
  if constexpr (DT == SNL_Q8_0) {
#pragma unroll
    for (uint32_t i = 0; i < E; i++) v[i] = (float)(int8_t)((wd[i / 4] >> (8 * (i % 4))) & 0xFFu) * raw.sc;
  } else {
#pragma unroll
    for (uint32_t i = 0; i < E; i++) v[i] = (float)((int)((wd[i / 8] >> (4 * (i % 8))) & 0xFu) - 8) * raw.sc;
  }
#pragma unroll
  for (uint32_t c = 0; c < E / 8; c++) {
    const uint32_t chunk = h * (E / 8) + c;
    const uint32_t sw = RB == 128 ? (r & 7) : ((r >> 1) & 3);
    const uint32_t off = r * RB + ((chunk ^ sw) << 4);
    uint4 hi, lo;
    hi.x = pack_hl(v[8 * c + 0], v[8 * c + 1], false);
    hi.y = pack_hl(v[8 * c + 2], v[8 * c + 3], false);
    hi.z = pack_hl(v[8 * c + 4], v[8 * c + 5], false);
    hi.w = pack_hl(v[8 * c + 6], v[8 * c + 7], false);
    lo.x = pack_hl(v[8 * c + 0], v[8 * c + 1], true);
    lo.y = pack_hl(v[8 * c + 2], v[8 * c + 3], true);
    lo.z = pack_hl(v[8 * c + 4], v[8 * c + 5], true);
    lo.w = pack_hl(v[8 * c + 6], v[8 * c + 7], true);
    *reinterpret_cast<uint4*>(ahi + off) = hi;
    *reinterpret_cast<uint4*>(alo + off) = lo;
  }
}

__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Warp roles: warps 0-7 dequantize A (thread t: row t/2, half t%2 of the K block) and
// run the epilogue; warp 8 (lane 0) issues the x-tile TMA loads and the MMAs. Per stage,
// a_full (8 arrivals, one per dequant warp) and b_full (TMA bytes) hand the stage to
// the MMA thread, and empty (tcgen05.commit) hands it back once its MMAs completed. No
// CTA-wide barrier runs inside the K loop.
constexpr uint32_t kTcDqWarps = 8;
constexpr uint32_t kTcThreads = (kTcDqWarps + 1) * 32;

template <int DT, uint32_t NT, uint32_t KB, int S, uint32_t AH>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, TcArgs a) {
  using G = TcGeom<NT, KB, S, AH>;
  constexpr uint32_t kTmemCols = NT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t a_full[S], b_full[S], empty_bar[S], done_bar;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int fail_sh;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t n0 = blockIdx.x * kTcM, t0 = blockIdx.y * NT;
  const uint32_t nkb = (a.k + KB - 1) / KB;

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&a_full[s], kTcDqWarps);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    fail_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;

  if (warp < kTcDqWarps) {
    // Dequantization: block kb into stage kb % S once the MMAs of block kb - S are done.
    RawA r0 = load_a<DT, KB>(a, n0, 0, nkb, tid), r1 = load_a<DT, KB>(a, n0, 1, nkb, tid),
         r2 = load_a<DT, KB>(a, n0, 2, nkb, tid);
    for (uint32_t kb = 0; kb < nkb; kb++) {
      const RawA r3 = load_a<DT, KB>(a, n0, kb + 3, nkb, tid);
      const int s = kb % S;
      const uint32_t use = kb / S;
      // Warp-uniform: a lane that gave up stops the whole warp (the __syncwarp below).
      const bool ok = __all_sync(0xffffffffu, kb < (uint32_t)S || mbar_wait_bounded(&empty_bar[s], (use - 1) & 1));
      if (!ok) fail_sh = 1;
      if (__shfl_sync(0xffffffffu, fail_sh, 0)) break;
      uint8_t* st = smem + s * G::kStageBytes;
      store_a<DT, KB>(r0, st, st + G::kATile, tid);
      r0 = r1;
      r1 = r2;
      r2 = r3;
      fence_proxy_async_smem();  // the dequantized tiles are read by the tensor cores (async proxy)
      __syncwarp();
      if (lane == 0) mbar_arrive_cta(&a_full[s]);
    }
  } else if (lane == 0) {
    // TMA and MMA issue.
    auto load_b = [&](uint32_t j) {
      uint8_t* sp = smem + (j % S) * G::kStageBytes + 2 * G::kATile;
      mbar_arrive_expect_tx(&b_full[j % S], 2 * G::kBTile);
      tma_load_3d(sp, &xmap, (int)(j * KB), (int)t0, 0, &b_full[j % S]);
      tma_load_3d(sp + G::kBTile, &xmap, (int)(j * KB), (int)t0, 1, &b_full[j % S]);
    };
    uint32_t issued = 0, consumed = 0;
    for (; issued < nkb && issued <= AH && issued < (uint32_t)S; issued++) load_b(issued);
    for (uint32_t kb = 0; kb < nkb && !fail_sh; kb++) {
      // x tile of block kb + AH once its stage's previous block's MMAs are done.
      const uint32_t j = kb + AH;
      if (j < nkb && j == issued) {
        if (j >= (uint32_t)S && !mbar_wait_bounded(&empty_bar[j % S], (j / S - 1) & 1)) {
          fail_sh = 1;
          break;
        }
        load_b(j);
        issued++;
      }
      const int s = kb % S;
      const uint32_t use = kb / S;
      if (!mbar_wait_bounded(&b_full[s], use & 1) || !mbar_wait_bounded(&a_full[s], use & 1)) {
        fail_sh = 1;
        break;
      }
      consumed = kb + 1;
      tc_fence_after();
      uint8_t* st = smem + s * G::kStageBytes;
      const uint32_t sa_hi = smem_u32(st), sa_lo = sa_hi + G::kATile;
      const uint32_t sb_hi = sa_hi + 2 * G::kATile, sb_lo = sb_hi + G::kBTile;
#pragma unroll
      for (uint32_t kk = 0; kk < KB / 16; kk++) {
        const uint32_t o = kk * 32;  // 16 fp16 along K inside the swizzled row
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_hi + o), sdesc<G::kRowBytes>(sb_hi + o), G::kIdesc, (kb | kk) != 0);
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_hi + o), sdesc<G::kRowBytes>(sb_lo + o), G::kIdesc, 1);
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_lo + o), sdesc<G::kRowBytes>(sb_hi + o), G::kIdesc, 1);
      }
      tc_commit(&empty_bar[s]);
    }
    tc_commit(&done_bar);  // arrives when every MMA issued above has completed
    if (fail_sh) {
      report_timeout(a.err);
      // Let the x tiles still in flight land before the CTA exits.
      for (uint32_t j = consumed; j < issued; j++) (void)mbar_wait_bounded(&b_full[j % S], (j / S) & 1);
    }
  }
  if (warp == kTcDqWarps) __syncwarp();  // lane 0 rejoins before the CTA barrier below
  // Epilogue (dequant warps): TMEM -> y once every MMA has completed. The condition is
  // warp-uniform (tcgen05.ld is a warp-collective instruction).
  if (warp < kTcDqWarps) {
    const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(&done_bar, 0));
    tc_fence_after();
    if (done && !__shfl_sync(0xffffffffu, fail_sh, 0)) {
      const uint32_t quarter = warp & 3, half = warp >> 2;
      const uint32_t row = n0 + quarter * 32 + lane;
      const float out_scale = kXPlaneScaleTc / kAScale;
#pragma unroll 1
      for (uint32_t c0 = half * (NT / 2); c0 < half * (NT / 2) + NT / 2; c0 += 32) {
        uint32_t r[32];
        const uint32_t taddr = tmem + ((quarter * 32) << 16) + c0;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
            "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
              "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
              "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
              "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < a.n) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const uint32_t t = t0 + c0 + j;
            if (t < a.m) a.y[a.y_off + (uint64_t)t * a.y_stride + a.n_off + row] = __uint_as_float(r[j]) * out_scale;
          }
        }
      }
    } else if (tid == 0 && !done) {
      report_timeout(a.err);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Weight planes: the A operand of the GEMM precomputed once per matrix, planes [2][n][k]
// fp16, plane 0 = hi and plane 1 = lo of code * scale * 256 (the values the dequant
// warps of gemm_tc_kernel write, bit for bit). Thread = 8 consecutive elements of a row.
__global__ void weight_planes_kernel(int dtype, uint32_t n, uint32_t k, const uint8_t* __restrict__ q,
                                     const float* __restrict__ s, __half* __restrict__ planes) {
  const uint64_t total = (uint64_t)n * (k / 8);
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t row = (uint32_t)(e / (k / 8)), c8 = (uint32_t)(e % (k / 8));
    const float sc = s[(uint64_t)row * (k / 32) + c8 / 4] * kAScale;
    float v[8];
    if (dtype == SNL_Q8_0) {
      const uint2 w = *reinterpret_cast<const uint2*>(q + (uint64_t)row * k + 8 * c8);
      const uint32_t wd[2] = {w.x, w.y};
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = (float)(int8_t)((wd[i / 4] >> (8 * (i % 4))) & 0xFFu) * sc;
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(q + (uint64_t)row * (k / 2) + 4 * c8);
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = (float)((int)((w >> (4 * i)) & 0xFu) - 8) * sc;
    }
    uint4 hi, lo;
    hi.x = pack_hl(v[0], v[1], false);
    hi.y = pack_hl(v[2], v[3], false);
    hi.z = pack_hl(v[4], v[5], false);
    hi.w = pack_hl(v[6], v[7], false);
    lo.x = pack_hl(v[0], v[1], true);
    lo.y = pack_hl(v[2], v[3], true);
    lo.z = pack_hl(v[4], v[5], true);
    lo.w = pack_hl(v[6], v[7], true);
    const uint64_t o = (uint64_t)row * k + 8 * c8;
    *reinterpret_cast<uint4*>(planes + o) = hi;
    *reinterpret_cast<uint4*>(planes + (uint64_t)n * k + o) = lo;
  }
}

// The GEMM with both operands loaded by TMA (weight planes and x planes): warp 0 lane 0
// issues the loads of each stage, warp 1 lane 0 its 12 MMAs; all 8 warps run the
// epilogue. Same tiles, K blocks and MMA order as gemm_tc_kernel, so the same results.
template <uint32_t NT, uint32_t KB, int S>
__global__ void __launch_bounds__(256, 1) gemm_tc_planes_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const __grid_constant__ CUtensorMap amap, TcArgs a) {
  using G = TcGeom<NT, KB, S, 1>;
  // TMEM is allocated in powers of two columns (a 192-token tile takes 256).
  constexpr uint32_t kTmemCols = NT <= 128 ? 128 : 256;
  static_assert(NT % 32 == 0 && NT <= 256, "token tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ uint64_t full_bar[S], empty_bar[S], done_bar;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int fail_sh;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Token tiles run along x, so the CTAs that share a weight tile are launched together
  // and the second read of its planes hits L2.
  const uint32_t n0 = blockIdx.y * kTcM, t0 = blockIdx.x * NT;
  const uint32_t nkb = (a.k + KB - 1) / KB;
  if (tid == 0) {
    for (int st = 0; st < S; st++) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], 1);
    }
    mbar_init(&done_bar, 1);
    fail_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_sh)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  if (warp == 0 && lane == 0) {
    // Loads: stage kb % S once the MMAs of block kb - S are done.
    uint32_t issued = 0;
    for (uint32_t kb = 0; kb < nkb && !fail_sh; kb++) {
      const int st = kb % S;
      if (kb >= (uint32_t)S && !mbar_wait_bounded(&empty_bar[st], (kb / S - 1) & 1)) {
        fail_sh = 1;
        break;
      }
      uint8_t* sp = smem + st * G::kStageBytes;
      mbar_arrive_expect_tx(&full_bar[st], 2 * G::kATile + 2 * G::kBTile);
      tma_load_3d(sp, &amap, (int)(kb * KB), (int)n0, 0, &full_bar[st]);
      tma_load_3d(sp + G::kATile, &amap, (int)(kb * KB), (int)n0, 1, &full_bar[st]);
      tma_load_3d(sp + 2 * G::kATile, &xmap, (int)(kb * KB), (int)t0, 0, &full_bar[st]);
      tma_load_3d(sp + 2 * G::kATile + G::kBTile, &xmap, (int)(kb * KB), (int)t0, 1, &full_bar[st]);
      issued = kb + 1;
    }
    if (fail_sh) {
      // Let the last stages' loads land (older ones were consumed before their stage
      // was reused) before the CTA exits.
      for (uint32_t j = issued > (uint32_t)S ? issued - S : 0; j < issued; j++)
        (void)mbar_wait_bounded(&full_bar[j % S], (j / S) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    for (uint32_t kb = 0; kb < nkb; kb++) {
      const int st = kb % S;
      if (fail_sh || !mbar_wait_bounded(&full_bar[st], (kb / S) & 1)) {
        fail_sh = 1;
        break;
      }
      tc_fence_after();
      const uint32_t sa_hi = smem_u32(smem + st * G::kStageBytes), sa_lo = sa_hi + G::kATile;
      const uint32_t sb_hi = sa_hi + 2 * G::kATile, sb_lo = sb_hi + G::kBTile;
#pragma unroll
      for (uint32_t kk = 0; kk < KB / 16; kk++) {
        const uint32_t o = kk * 32;
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_hi + o), sdesc<G::kRowBytes>(sb_hi + o), G::kIdesc, (kb | kk) != 0);
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_hi + o), sdesc<G::kRowBytes>(sb_lo + o), G::kIdesc, 1);
        tc_mma(tmem, sdesc<G::kRowBytes>(sa_lo + o), sdesc<G::kRowBytes>(sb_hi + o), G::kIdesc, 1);
      }
      tc_commit(&empty_bar[st]);
    }
    tc_commit(&done_bar);
    if (fail_sh) report_timeout(a.err);
  }
  __syncwarp();
  const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(&done_bar, 0));
  tc_fence_after();
  if (done && !__shfl_sync(0xffffffffu, fail_sh, 0)) {
    const uint32_t quarter = warp & 3, half = warp >> 2;
    const uint32_t row = n0 + quarter * 32 + lane;
    const float out_scale = kXPlaneScaleTc / kAScale;
#pragma unroll 1
    for (uint32_t c0 = half * (NT / 2); c0 < half * (NT / 2) + NT / 2; c0 += 32) {
      uint32_t r[32];
      const uint32_t taddr = tmem + ((quarter * 32) << 16) + c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
          "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
            "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
            "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
            "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row < a.n) {
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const uint32_t t = t0 + c0 + j;
          if (t < a.m) a.y[a.y_off + (uint64_t)t * a.y_stride + a.n_off + row] = __uint_as_float(r[j]) * out_scale;
        }
      }
    }
  } else if (tid == 0 && !done) {
    report_timeout(a.err);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// x [m][x_stride] fp32 (from x_off) -> planes [2][m][k] fp16: hi and lo of x / 16.
__global__ void tc_xpack_kernel(const float* __restrict__ x, uint32_t x_stride, uint32_t m, uint32_t k,
                                __half* __restrict__ planes) {
  // Row blockIdx.y, four consecutive elements per thread (x_stride and k multiples of 4).
  const uint32_t t = blockIdx.y, j = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (t >= m || j >= k) return;
  const float4 v = *reinterpret_cast<const float4*>(x + (uint64_t)t * x_stride + j);
  const float vs[4] = {v.x * (1.0f / kXPlaneScaleTc), v.y * (1.0f / kXPlaneScaleTc), v.z * (1.0f / kXPlaneScaleTc),
                       v.w * (1.0f / kXPlaneScaleTc)};
  __half hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    hi[e] = __float2half_rn(vs[e]);
    lo[e] = __float2half_rn(vs[e] - __half2float(hi[e]));
  }
  const uint64_t o = (uint64_t)t * k + j, total = (uint64_t)m * k;
  *reinterpret_cast<uint2*>(planes + o) = *reinterpret_cast<const uint2*>(hi);
  *reinterpret_cast<uint2*>(planes + total + o) = *reinterpret_cast<const uint2*>(lo);
}

PFN_cuTensorMapEncodeTiled encode_fn() {
  static PFN_cuTensorMapEncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(p);
  }();
  return fn;
}

// Per-device scratch for the x planes of one GEMM, grown on demand.
__half* planes_scratch(size_t halves) {
  static std::mutex mu;
  static __half* buf[64] = {nullptr};
  static size_t cap[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (cap[dev] < halves) {
    if (buf[dev]) cudaFree(buf[dev]);
    buf[dev] = nullptr;
    cap[dev] = 0;
    void* p = nullptr;
    if (cudaMalloc(&p, halves * sizeof(__half)) != cudaSuccess) return nullptr;
    buf[dev] = static_cast<__half*>(p);
    cap[dev] = halves;
  }
  return buf[dev];
}

}  // namespace

bool gemm_tc_enabled() {
  static const bool on = getenv("SNL_NO_TC_GEMM") == nullptr;
  return on;
}

int launch_weight_planes(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, __half* planes,
                         cudaStream_t st) {
  if ((dtype != SNL_Q8_0 && dtype != SNL_Q4_0) || k % 32 || n == 0) return fail(SNL_E_INVALID, "weight planes: shape");
  const uint64_t total = (uint64_t)n * (k / 8);
  weight_planes_kernel<<<(unsigned)std::min<uint64_t>((total + 255) / 256, (uint64_t)sm_count() * 16), 256, 0, st>>>(
      dtype, n, k, static_cast<const uint8_t*>(q), s, planes);
  SNL_LAUNCH_CHECK("weight_planes");
  return SNL_OK;
}

int launch_gemm_tc(int dtype, const snl_mat_p& p, uint32_t m, const float* x, const void* wq, const float* ws, float* y,
                   cudaStream_t s, const __half* wplanes) {
  if (dtype != SNL_Q8_0 && dtype != SNL_Q4_0) return fail(SNL_E_INVALID, "gemm_tc: dtype");
  if (p.k % 32 || p.k == 0 || m == 0) return fail(SNL_E_INVALID, "gemm_tc: k must be a positive multiple of 32");
  PFN_cuTensorMapEncodeTiled enc = encode_fn();
  if (!enc) return fail(SNL_E_CUDA, "gemm_tc: cuTensorMapEncodeTiled is unavailable");
  int* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  __half* planes = planes_scratch((size_t)2 * m * p.k);
  if (!planes) return fail(SNL_E_OOM, "gemm_tc: x planes scratch");
  const uint64_t total = (uint64_t)m * p.k;
  tc_xpack_kernel<<<dim3((p.k / 4 + 255) / 256, m), 256, 0, s>>>(x + p.x_off, p.x_stride, m, p.k, planes);
  SNL_LAUNCH_CHECK("gemm_tc xpack");

  // 256-token tiles (K blocks of 64, 2 stages, x one block ahead) unless the step has at
  // most 128 tokens or 256-token tiles would not fill one wave; then 128-token tiles
  // (3 stages). Measured on 512 x 12288 x 4096 (Q8_0): 189 us with 256-token tiles
  // against 277 us with 128-token tiles, whose dequantization per MMA doubles.
  const uint32_t row_tiles = (p.n + kTcM - 1) / kTcM;
  const bool narrow = m <= 128 || (uint64_t)row_tiles * ((m + 255) / 256) < (uint64_t)sm_count();
  const uint32_t nt = narrow ? 128 : 256;
  const uint32_t kbk = 64;
  CUtensorMap map;
  const cuuint64_t dims[3] = {p.k, m, 2};
  const cuuint64_t strides[2] = {(cuuint64_t)p.k * 2, (cuuint64_t)m * p.k * 2};
  const cuuint32_t box[3] = {kbk, nt, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, planes, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, kbk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return fail(SNL_E_CUDA, "gemm_tc: cuTensorMapEncodeTiled failed");

  TcArgs ta{p.n, p.k, m, static_cast<const uint8_t*>(wq), ws, y, p.y_off, p.y_stride, p.n_off, err};
  if (wplanes) {
    // A from the weight planes [2][n][k] fp16 and x from its planes, both by TMA in K
    // blocks of 32 (64-byte swizzle), 4 stages (6 for 128-token tiles). Measured on
    // 512 x 12288 x 4096: 156 us, against 183 us with K blocks of 64 in 2 stages.
    const uint32_t pk = 32;
    const CUtensorMapSwizzle psw = CU_TENSOR_MAP_SWIZZLE_64B;
    CUtensorMap amap, pxmap;
    const cuuint64_t adims[3] = {p.k, p.n, 2};
    const cuuint64_t astr[2] = {(cuuint64_t)p.k * 2, (cuuint64_t)p.n * p.k * 2};
    const cuuint32_t abox[3] = {pk, kTcM, 1};
    cr = enc(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(wplanes), adims, astr, abox, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, psw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(SNL_E_CUDA, "gemm_tc: weight-plane tensor map");
    // Token tile: 128 as above; else 256, or 192 when that takes fewer waves x tile width
    // (512 rows over 96-97 row tiles: 288 CTAs in 2 waves of 192-token tiles against 192
    // CTAs in 2 waves of 256-token tiles).
    uint32_t pnt = nt;
    if (!narrow) {
      const uint64_t sms = (uint64_t)sm_count();
      auto waves = [&](uint64_t t) { return ((uint64_t)row_tiles * ((m + t - 1) / t) + sms - 1) / sms; };
      if (waves(192) * 192 < waves(256) * 256) pnt = 192;
    }
    const cuuint32_t xbox[3] = {pk, pnt, 1};
    cr = enc(&pxmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, planes, dims, strides, xbox, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, psw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return fail(SNL_E_CUDA, "gemm_tc: x-plane tensor map");
    // Grid: token tiles along x (the CTAs sharing a weight tile run together; 2K prefill
    // 10070 -> 10380 tok/s and 512 x 12288 x 4096 149.5 -> 138.3 us, same box A/B).
    if (row_tiles > 65535u) return fail(SNL_E_UNSUPPORTED, "gemm_tc: more than 65535 row tiles");
    const dim3 pgrid((m + pnt - 1) / pnt, row_tiles);
    int pdev = 0;
    cudaGetDevice(&pdev);
    static bool pattr[3][64] = {};
    auto pgo = [&](auto kern, uint32_t smem, bool& done) -> int {
      if (!done) {
        SNL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        done = true;
      }
      kern<<<pgrid, 256, smem, s>>>(pxmap, amap, ta);
      return SNL_OK;
    };
    const int d = pdev >= 0 && pdev < 64 ? pdev : 0;
    const int rc = pnt == 128   ? pgo(gemm_tc_planes_kernel<128, 32, 6>, TcGeom<128, 32, 6, 1>::kSmem, pattr[1][d])
                   : pnt == 192 ? pgo(gemm_tc_planes_kernel<192, 32, 5>, TcGeom<192, 32, 5, 1>::kSmem, pattr[2][d])
                                : pgo(gemm_tc_planes_kernel<256, 32, 4>, TcGeom<256, 32, 4, 1>::kSmem, pattr[0][d]);
    if (rc) return rc;
    SNL_LAUNCH_CHECK("gemm_tc_planes");
    return SNL_OK;
  }
  const dim3 grid(row_tiles, (m + nt - 1) / nt);
  int dev = 0;
  cudaGetDevice(&dev);
  static bool attr[2][2][64] = {};
  auto go = [&](auto kern, uint32_t smem) -> int {
    bool& done = attr[dtype == SNL_Q8_0 ? 0 : 1][narrow ? 1 : 0][dev >= 0 && dev < 64 ? dev : 0];
    if (!done) {
      SNL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      done = true;
    }
    kern<<<grid, kTcThreads, smem, s>>>(map, ta);
    return SNL_OK;
  };
  int rc;
  if (dtype == SNL_Q8_0)
    rc = narrow ? go(gemm_tc_kernel<SNL_Q8_0, 128, 64, 3, 1>, TcGeom<128, 64, 3, 1>::kSmem)
                : go(gemm_tc_kernel<SNL_Q8_0, 256, 64, 2, 1>, TcGeom<256, 64, 2, 1>::kSmem);
  else
    rc = narrow ? go(gemm_tc_kernel<SNL_Q4_0, 128, 64, 3, 1>, TcGeom<128, 64, 3, 1>::kSmem)
                : go(gemm_tc_kernel<SNL_Q4_0, 256, 64, 2, 1>, TcGeom<256, 64, 2, 1>::kSmem);
  if (rc) return rc;
  SNL_LAUNCH_CHECK("gemm_tc");
  return SNL_OK;
}

}  // namespace snl
