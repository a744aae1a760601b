/*
 * TEST INFRASTRUCTURE ONLY: the MXFP4 block decode of the oracle restatement, in C.
 *
 * Restates megabench/tasks/quantization.py:40-51 (`unpack_mxfp4`) as the oracle uses it
 * (oracle/kimi_oracle.py:decode_mxfp4): code bytes [groups, 16] hold 32 E2M1 values, low nibble first;
 * value = E2M1_TABLE[nibble] * 2^(scale - 127) in FP32 (quantization.py:8-9 table; the reference's
 * torch.ldexp multiplies by an FP32 power of two); a scale byte of 255 makes the whole group NaN
 * (quantization.py:49-50). The result is written as FP32 or rounded to BF16 the way torch's
 * float -> bfloat16 conversion rounds (nearest even; NaN stays NaN), which is what `.to(torch.bfloat16)`
 * of the reference's FP32 decode gives. Bit-identical to the torch restatement (tests/test_oracle_golden.py
 * checks both on every scale byte, 0 and 255 included); it exists because the oracle's CPU step spends most
 * of its time in the torch decode, and the timed CPU baseline runs whole steps.
 *
 * Built by kimi_k3_goalbox_b200/build.py (gcc -O2 -fopenmp -shared), loaded by the oracle with ctypes.
 * Compiled without -ffast-math: subnormal products (scale bytes near 0) must be exact, as in torch.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float kE2M1[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0xffff; /* NaN (the payload torch's vector path gives) */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline void decode_group(const uint8_t* codes, uint8_t scale, float* v) {
  if (scale == 255) {
    for (int i = 0; i < 32; ++i) v[i] = NAN;
    return;
  }
  const float f = ldexpf(1.0f, (int)scale - 127);
  for (int j = 0; j < 16; ++j) {
    v[2 * j] = kE2M1[codes[j] & 15] * f;
    v[2 * j + 1] = kE2M1[codes[j] >> 4] * f;
  }
}

/* codes [groups][16] u8, scales [groups] u8 -> out [groups][32] FP32 */
void kk3o_decode_mxfp4_f32(const uint8_t* codes, const uint8_t* scales, long long groups, float* out) {
#pragma omp parallel for schedule(static)
  for (long long g = 0; g < groups; ++g) decode_group(codes + g * 16, scales[g], out + g * 32);
}

/* codes [groups][16] u8, scales [groups] u8 -> out [groups][32] BF16 bits */
void kk3o_decode_mxfp4_bf16(const uint8_t* codes, const uint8_t* scales, long long groups, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (long long g = 0; g < groups; ++g) {
    float v[32];
    decode_group(codes + g * 16, scales[g], v);
    for (int i = 0; i < 32; ++i) out[g * 32 + i] = f32_to_bf16_rne(v[i]);
  }
}
