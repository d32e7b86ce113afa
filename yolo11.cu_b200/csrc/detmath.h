// Bit-reproducible fp32 math shared by the CUDA post-processing kernels (decode, NMS, masks,
// letterbox) and any host code that must reproduce them exactly.
//
// Every operation is an explicitly rounded IEEE-754 binary32 op (no FMA contraction, no
// fast-math intrinsics), so nvcc device code and gcc/g++ host code (built with
// -ffp-contract=off) produce identical bits:
//   * DM_ADD/SUB/MUL/DIV: single correctly rounded ops (__fadd_rn & co. on the device);
//   * DM_FMA: one fused multiply-add with a single rounding (fmaf on both sides);
//   * dm_exp: e^x by Cody-Waite range reduction x = k*ln2 + r, |r| <= ln2/2 (ln2 split in a
//     high part with trailing zero bits and a low correction term, as in Cody & Waite,
//     "Software Manual for the Elementary Functions", 1980), a degree-7 Taylor polynomial
//     e^r = sum r^i/i! evaluated by Horner with fmaf (truncation error < 2^-26 relative on
//     |r| <= 0.3466), and an exact scaling by 2^k through the exponent bits.
//     Accuracy: within 2 ulp of e^x on [-87, 88]; underflows to 0 below -87.3, saturates
//     to +inf above 88.7.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define DM_HD __host__ __device__ __forceinline__
#else
#define DM_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define DM_ADD(a, b) __fadd_rn((a), (b))
#define DM_SUB(a, b) __fsub_rn((a), (b))
#define DM_MUL(a, b) __fmul_rn((a), (b))
#define DM_DIV(a, b) __fdiv_rn((a), (b))
#define DM_FMA(a, b, c) __fmaf_rn((a), (b), (c))
#else
#include <math.h>
#define DM_ADD(a, b) ((float)((float)(a) + (float)(b)))
#define DM_SUB(a, b) ((float)((float)(a) - (float)(b)))
#define DM_MUL(a, b) ((float)((float)(a) * (float)(b)))
#define DM_DIV(a, b) ((float)((float)(a) / (float)(b)))
#define DM_FMA(a, b, c) fmaf((a), (b), (c))
#endif

DM_HD float dm_bits2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float f; memcpy(&f, &u, 4); return f;
#endif
}
DM_HD uint32_t dm_f2bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}

DM_HD float dm_exp(float x) {
  if (!(x == x)) return x;                 // NaN
  if (x > 88.7f) return dm_bits2f(0x7f800000u);
  if (x < -87.3f) return 0.0f;
  const float inv_ln2 = 1.44269504088896341f;
  const float ln2_hi = 0.693145751953125f;        // 0x3F317200: low 12 bits zero
  const float ln2_lo = 1.42860682030941723e-6f;   // ln2 - ln2_hi
  float t = DM_MUL(x, inv_ln2);
  // round-half-away-from-zero to an integer without libm
  int k = (int)(t + (t >= 0.f ? 0.5f : -0.5f));
  float kf = (float)k;
  float r = DM_FMA(-kf, ln2_hi, x);              // exact: kf*ln2_hi has <= 24 bits
  r = DM_FMA(-kf, ln2_lo, r);
  // Taylor e^r = 1 + r + r^2/2! + ... + r^7/7!
  float p = 1.98412698412698413e-4f;               // 1/7!
  p = DM_FMA(p, r, 1.38888888888888889e-3f);       // 1/6!
  p = DM_FMA(p, r, 8.33333333333333333e-3f);       // 1/5!
  p = DM_FMA(p, r, 4.16666666666666667e-2f);       // 1/4!
  p = DM_FMA(p, r, 1.66666666666666667e-1f);       // 1/3!
  p = DM_FMA(p, r, 0.5f);                          // 1/2!
  p = DM_FMA(p, r, 1.0f);
  p = DM_FMA(p, r, 1.0f);
  // scale by 2^k in two steps so that 2^k never over/underflows on its own
  int k1 = k / 2, k2 = k - k1;
  float s1 = dm_bits2f((uint32_t)(k1 + 127) << 23);
  float s2 = dm_bits2f((uint32_t)(k2 + 127) << 23);
  return DM_MUL(DM_MUL(p, s1), s2);
}

// 1 / (1 + e^-x)
DM_HD float dm_sigmoid(float x) { return DM_DIV(1.0f, DM_ADD(1.0f, dm_exp(-x))); }

// fp16 bits -> fp32 (exact)
DM_HD float dm_h2f(uint16_t h) {
  uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ffu;
  if (e == 0) {
    if (m == 0) return dm_bits2f(s);
    float f = DM_MUL((float)m, 5.9604644775390625e-8f);   // m * 2^-24 (exact)
    return s ? -f : f;
  }
  if (e == 31) return dm_bits2f(s | 0x7f800000u | (m << 13));
  return dm_bits2f(s | ((e + 112) << 23) | (m << 13));
}

// fp32 -> fp16 bits, round to nearest even (matches __float2half_rn)
DM_HD uint16_t dm_f2h(float f) {
  uint32_t x = dm_f2bits(f);
  uint32_t s = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(s | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(s | 0x7c00u);          // rounds to >= 65520 -> inf
  if (ax < 0x38800000u) {                                          // subnormal / zero in fp16
    if (ax < 0x33000000u) return (uint16_t)s;                      // < 2^-25 -> 0
    uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126 - e;                                      // 14..24
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(s | q);
  }
  uint32_t q = ((ax >> 13) - (112u << 10)), rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(s | q);
}

// One DFL side: softmax over 16 bin logits, expectation sum(p_i * i) / sum(p_i), i = 0..15.
// Sequential accumulation order i = 0..15 (part of the bit-exact contract).
DM_HD float dm_dfl16(const float* l) {
  float mx = l[0];
  for (int i = 1; i < 16; i++) mx = l[i] > mx ? l[i] : mx;
  float sum = 0.f, e = 0.f;
  for (int i = 0; i < 16; i++) {
    float p = dm_exp(DM_SUB(l[i], mx));
    sum = DM_ADD(sum, p);
    e = DM_ADD(e, DM_MUL(p, (float)i));
  }
  return DM_DIV(e, sum);
}

// IoU > thr test of two xyxy boxes with the reference's formula
// (inter / (area_a + area_b - inter), union must be > 0).
DM_HD int dm_iou_gt(float ax1, float ay1, float ax2, float ay2, float aarea,
                    float bx1, float by1, float bx2, float by2, float thr) {
  float xx1 = ax1 > bx1 ? ax1 : bx1, yy1 = ay1 > by1 ? ay1 : by1;
  float xx2 = ax2 < bx2 ? ax2 : bx2, yy2 = ay2 < by2 ? ay2 : by2;
  float w = DM_SUB(xx2, xx1), h = DM_SUB(yy2, yy1);
  w = w > 0.f ? w : 0.f;
  h = h > 0.f ? h : 0.f;
  float inter = DM_MUL(w, h);
  if (inter == 0.f && thr >= 0.f) return 0;   // 0 / ua is 0, or ua > 0 fails: never > thr
  float barea = DM_MUL(DM_SUB(bx2, bx1), DM_SUB(by2, by1));
  float ua = DM_SUB(DM_ADD(aarea, barea), inter);
  return ua > 0.f && DM_DIV(inter, ua) > thr;
}

DM_HD float dm_area(float x1, float y1, float x2, float y2) {
  return DM_MUL(DM_SUB(x2, x1), DM_SUB(y2, y1));
}

// Logit threshold equivalent of sigmoid(x) >= conf is NOT used: the gate is the sigmoid
// itself (score = dm_sigmoid(best) >= conf), so host and device agree bit for bit.
