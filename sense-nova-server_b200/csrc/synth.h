// Seeded synthetic weights and inputs, bit-identical on the host and the GPU.
//
// The benchmark configurations run on random-init weights (no checkpoints are
// available), so the GPU engine and the CPU checker must generate the same
// tensors from a seed. Everything here uses integer arithmetic, exact int->f32
// conversions and single correctly-rounded f32 multiplies, so a value does not
// depend on the compiler, the FMA contraction policy or the device.
//
// Value distributions (tensor-kind constants below):
//   * Q8_0 quants: uniform in [-127, 127]; scale = f16(|z| * 0.02 / 127).
//   * Q4_0 nibbles: uniform in [0, 15] (value = nibble - 8); scale = f16(|z| * 0.02 / 8).
//   * z is an Irwin-Hall(4) approximation of N(0, 1) (bounded at about 3.46 sigma).
// The block layout follows the reference's quantizers: Q8_0 = int8 per element plus
// one f32 scale per 32 elements (weights.rs:123-133); Q4_0 = nibble i of little-endian
// 32-bit word w holds element w*8+i, stored as n+8 (weights.rs:135-153).
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define SNL_HD __host__ __device__ __forceinline__
#else
#define SNL_HD static inline
#endif

// 1 / sqrt(4 * (65536^2 - 1) / 12): unit variance for the sum of four 16-bit uniforms.
#define SNL_GAUSS_K 0x1.bb67aep-16f
#define SNL_Q8_SCALE_K 0x1.4a429ap-13f  // 0.02 / 127
#define SNL_Q4_SCALE_K 0x1.47ae14p-9f   // 0.02 / 8

SNL_HD uint64_t snl_mix64(uint64_t z) {
  // splitmix64 finaliser (Steele, Lea & Flood 2014).
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Per-tensor key: one stream per (seed, tensor name hash, sub-stream).
SNL_HD uint64_t snl_key(uint64_t seed, uint64_t name_hash, uint64_t sub) {
  return snl_mix64(snl_mix64(seed ^ 0x5EEDull) ^ snl_mix64(name_hash + 0x100000001B3ull * (sub + 1)));
}

SNL_HD uint64_t snl_draw(uint64_t key, uint64_t i) { return snl_mix64(key + i * 0xD1B54A32D192ED03ull); }

SNL_HD float snl_mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}

SNL_HD float snl_add_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  return a + b;
#endif
}

// Approximately N(0, 1): four 16-bit uniforms summed exactly, centred, scaled once.
SNL_HD float snl_gauss(uint64_t h) {
  int32_t s = (int32_t)(h & 0xFFFF) + (int32_t)((h >> 16) & 0xFFFF) + (int32_t)((h >> 32) & 0xFFFF) +
              (int32_t)(h >> 48) - 131070;
  return snl_mul_rn((float)s, SNL_GAUSS_K);
}

// int8 uniform in [-127, 127] (multiply-shift range reduction of the high 32 bits).
SNL_HD int8_t snl_q8(uint64_t h) { return (int8_t)((int32_t)(((h >> 32) * 255ull) >> 32) - 127); }

// Nibble uniform in [0, 15].
SNL_HD uint32_t snl_nib(uint64_t h) { return (uint32_t)(h >> 60); }

SNL_HD uint32_t snl_f2u(float f) {
  union { float f; uint32_t u; } c;
  c.f = f;
  return c.u;
}
SNL_HD float snl_u2f(uint32_t u) {
  union { float f; uint32_t u; } c;
  c.u = u;
  return c.f;
}

// IEEE binary32 -> binary16, round to nearest even (integer implementation).
SNL_HD uint16_t snl_f32_to_f16(float f) {
  uint32_t x = snl_f2u(f);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mag = x & 0x7FFFFFFFu;
  if (mag >= 0x7F800000u) return (uint16_t)(sign | (mag > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (mag >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
  if (mag < 0x33000000u) return (uint16_t)sign;                // < 2^-25 rounds to 0
  int32_t e = (int32_t)(mag >> 23) - 127;
  uint32_t m = (mag & 0x7FFFFFu) | 0x800000u;
  if (e < -14) {  // subnormal result
    uint32_t shift = (uint32_t)(-14 - e) + 13;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = ((uint32_t)(e + 15) << 10) | ((m >> 13) & 0x3FFu);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(sign | q);
}

SNL_HD float snl_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = ((uint32_t)h >> 10) & 0x1F;
  uint32_t m = (uint32_t)h & 0x3FFu;
  if (e == 0) {
    if (m == 0) return snl_u2f(sign);
    // subnormal: normalise
    int32_t ee = -1;
    do { m <<= 1; ee++; } while ((m & 0x400u) == 0);
    m &= 0x3FFu;
    return snl_u2f(sign | ((uint32_t)(127 - 15 - ee) << 23) | (m << 13));
  }
  if (e == 31) return snl_u2f(sign | 0x7F800000u | (m << 13));
  return snl_u2f(sign | ((e - 15 + 127) << 23) | (m << 13));
}

SNL_HD float snl_f16_round(float f) { return snl_f16_to_f32(snl_f32_to_f16(f)); }

// Q8_0 scale and Q4_0 scale for one block, fp16-exact, stored as f32.
SNL_HD float snl_q8_scale(uint64_t h) {
  float z = snl_gauss(h);
  return snl_f16_round(snl_mul_rn(z < 0.f ? -z : z, SNL_Q8_SCALE_K));
}
SNL_HD float snl_q4_scale(uint64_t h) {
  float z = snl_gauss(h);
  return snl_f16_round(snl_mul_rn(z < 0.f ? -z : z, SNL_Q4_SCALE_K));
}

// Small f32 parameter: offset + mult * z (two correctly-rounded steps, never fused).
SNL_HD float snl_param(uint64_t h, float mult, float offset) {
  return snl_add_rn(snl_mul_rn(snl_gauss(h), mult), offset);
}

// 64-bit FNV-1a of a tensor name: the stream id for that tensor.
SNL_HD uint64_t snl_fnv1a(const char* s) {
  uint64_t h = 0xCBF29CE484222325ull;
  while (*s) {
    h ^= (uint8_t)*s++;
    h *= 0x100000001B3ull;
  }
  return h;
}
