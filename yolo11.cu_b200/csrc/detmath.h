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
// v / 255 correctly rounded without a division: q = RN(v * RN(1/255)), then one Markstein
// correction step, q' = RN(q + RN(v - q * 255) * RN(1/255)) with both steps as single-rounding
// FMAs (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990).  Checked exhaustively against v / 255 for every
// binary32 v in [0, 256] (the letterbox's range: bilinear sums of bytes).
DM_HD float dm_div255(float v) {
  const float inv = 0.0039215688593685627f;   // RN(1/255) = 0x1.010102p-8
  const float q = DM_MUL(v, inv);
  const float r = DM_FMA(-q, 255.0f, v);
  return DM_FMA(r, inv, q);
}

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
// RN(a / b) > t for b > 0, 0 <= t < FLT_MAX, without a division: with t+ the next float
// above t and m = (t + t+) / 2 their midpoint, RN(q) > t holds exactly when q > m, or q == m
// and round-to-nearest-even takes m up to t+ (t+ has an even significand).  m has at most 25
// significant bits and b 24, so m * b is exact in binary64 and the test on a > m * b is exact.
DM_HD int dm_quot_gt(float a, float b, float t) {
  const float tp = dm_bits2f(dm_f2bits(t) + 1u);
  const double m = 0.5 * ((double)t + (double)tp);
  const double mb = m * (double)b;
  const double ad = (double)a;
  return ad > mb || (ad == mb && (dm_f2bits(tp) & 1u) == 0u);
}

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
  if (!(ua > 0.f)) return 0;
  if (!(thr >= 0.f) || !(thr < 3.0e38f)) return DM_DIV(inter, ua) > thr;
  return dm_quot_gt(inter, ua, thr);
}

DM_HD float dm_area(float x1, float y1, float x2, float y2) {
  return DM_MUL(DM_SUB(x2, x1), DM_SUB(y2, y1));
}

// Logit threshold equivalent of sigmoid(x) >= conf is NOT used: the gate is the sigmoid
// itself (score = dm_sigmoid(best) >= conf), so host and device agree bit for bit.

// ---------------- oriented boxes ----------------
#if defined(__CUDA_ARCH__)
#define DM_SQRT(a) __fsqrt_rn(a)
#else
#define DM_SQRT(a) sqrtf(a)
#endif

// sin and cos of x (|x| < 2^20): Cody-Waite reduction x = k*pi/2 + r, |r| <= pi/4 (pi/2 split
// into a 12-bit high part and a low correction), Taylor polynomials of sin r (to r^13) and
// cos r (to r^14) by Horner with fmaf (truncation < 2^-30 on |r| <= pi/4), then the quadrant
// k mod 4 selects and signs the pair.
DM_HD void dm_sincos(float x, float* s, float* c) {
  const float two_over_pi = 0.636619772367581343f;
  const float pio2_hi = 1.5703125f;                 // low 12 bits zero: k * hi is exact
  const float pio2_lo = 4.83826792333275079e-4f;    // pi/2 - pio2_hi
  float t = DM_MUL(x, two_over_pi);
  int k = (int)(t + (t >= 0.f ? 0.5f : -0.5f));
  float kf = (float)k;
  float r = DM_FMA(-kf, pio2_hi, x);
  r = DM_FMA(-kf, pio2_lo, r);
  float r2 = DM_MUL(r, r);
  float ps = 1.60590438368216146e-10f;               // 1/13!
  ps = DM_FMA(ps, r2, -2.50521083854417188e-8f);     // -1/11!
  ps = DM_FMA(ps, r2, 2.75573192239858907e-6f);      // 1/9!
  ps = DM_FMA(ps, r2, -1.98412698412698413e-4f);     // -1/7!
  ps = DM_FMA(ps, r2, 8.33333333333333333e-3f);      // 1/5!
  ps = DM_FMA(ps, r2, -1.66666666666666667e-1f);     // -1/3!
  float sr = DM_FMA(DM_MUL(ps, r2), r, r);
  float pc = -1.14707455977297247e-11f;              // -1/14!
  pc = DM_FMA(pc, r2, 2.08767569878680990e-9f);      // 1/12!
  pc = DM_FMA(pc, r2, -2.75573192239858907e-7f);     // -1/10!
  pc = DM_FMA(pc, r2, 2.48015873015873016e-5f);      // 1/8!
  pc = DM_FMA(pc, r2, -1.38888888888888889e-3f);     // -1/6!
  pc = DM_FMA(pc, r2, 4.16666666666666667e-2f);      // 1/4!
  pc = DM_FMA(pc, r2, -0.5f);                        // -1/2!
  float cr = DM_FMA(pc, r2, 1.0f);
  switch (k & 3) {
    case 0: *s = sr; *c = cr; break;
    case 1: *s = cr; *c = -sr; break;
    case 2: *s = -sr; *c = -cr; break;
    default: *s = -cr; *c = sr; break;
  }
}

// natural log of x > 0 (normal range): x = m * 2^e with m in [sqrt(1/2), sqrt(2)),
// log m = 2 atanh(s), s = (m - 1) / (m + 1), |s| < 0.1716, by the odd series to s^15
// (truncation < 2^-40); log x = e * ln2 (split hi / lo) + log m.  Returns -inf for 0 and NaN
// for negative or NaN input; denormals are scaled up first.
DM_HD float dm_log(float x) {
  if (!(x > 0.f)) return x == 0.f ? dm_bits2f(0xff800000u) : dm_bits2f(0x7fc00000u);
  if (x == dm_bits2f(0x7f800000u)) return x;
  int e = 0;
  if (x < 1.17549435e-38f) { x = DM_MUL(x, 16777216.f); e = -24; }   // 2^24
  uint32_t u = dm_f2bits(x);
  e += (int)((u >> 23) & 0xff) - 127;
  float m = dm_bits2f((u & 0x7fffffu) | 0x3f800000u);   // [1, 2)
  if (m > 1.41421356f) { m = DM_MUL(m, 0.5f); e += 1; }
  float s = DM_DIV(DM_SUB(m, 1.f), DM_ADD(m, 1.f));
  float s2 = DM_MUL(s, s);
  float p = 6.66666666666666667e-2f;                  // 1/15
  p = DM_FMA(p, s2, 7.69230769230769231e-2f);         // 1/13
  p = DM_FMA(p, s2, 9.09090909090909091e-2f);         // 1/11
  p = DM_FMA(p, s2, 1.11111111111111111e-1f);         // 1/9
  p = DM_FMA(p, s2, 1.42857142857142857e-1f);         // 1/7
  p = DM_FMA(p, s2, 2.0e-1f);                         // 1/5
  p = DM_FMA(p, s2, 3.33333333333333333e-1f);         // 1/3
  float lm = DM_MUL(2.f, DM_FMA(DM_MUL(p, s2), s, s));
  const float ln2_hi = 0.693145751953125f, ln2_lo = 1.42860682030941723e-6f;
  float ef = (float)e;
  return DM_FMA(ef, ln2_hi, DM_FMA(ef, ln2_lo, lm));
}

// Covariance (a, b, c) of the Gaussian of an oriented box (w, h, theta): a = w^2/12,
// b = h^2/12 rotated by theta (ultralytics _get_covariance_matrix).
DM_HD void dm_obb_cov(float w, float h, float th, float* cov) {
  float a = DM_DIV(DM_MUL(w, w), 12.f), b = DM_DIV(DM_MUL(h, h), 12.f);
  float s, c;
  dm_sincos(th, &s, &c);
  float c2 = DM_MUL(c, c), s2 = DM_MUL(s, s);
  cov[0] = DM_ADD(DM_MUL(a, c2), DM_MUL(b, s2));
  cov[1] = DM_ADD(DM_MUL(a, s2), DM_MUL(b, c2));
  cov[2] = DM_MUL(DM_MUL(DM_SUB(a, b), c), s);
}

// probiou of two oriented boxes from their centres and covariances (ultralytics
// batch_probiou: Bhattacharyya distance of the two Gaussians, clamped to [eps, 100], then
// 1 - sqrt(1 - exp(-bd) + eps); eps = 1e-7 in the same three places).
DM_HD float dm_probiou(float x1, float y1, const float* c1, float x2, float y2, const float* c2) {
  const float eps = 1e-7f;
  float dx = DM_SUB(x1, x2), dy = DM_SUB(y1, y2);
  float sa = DM_ADD(c1[0], c2[0]), sb = DM_ADD(c1[1], c2[1]), sc = DM_ADD(c1[2], c2[2]);
  float disc = DM_SUB(DM_MUL(sa, sb), DM_MUL(sc, sc));
  float den = DM_ADD(disc, eps);
  float t1 = DM_DIV(DM_MUL(0.25f, DM_ADD(DM_MUL(DM_MUL(sa, dy), dy), DM_MUL(DM_MUL(sb, dx), dx))), den);
  float t2 = DM_DIV(DM_MUL(0.5f, DM_MUL(DM_MUL(sc, -dx), dy)), den);
  float d1 = DM_SUB(DM_MUL(c1[0], c1[1]), DM_MUL(c1[2], c1[2]));
  float d2 = DM_SUB(DM_MUL(c2[0], c2[1]), DM_MUL(c2[2], c2[2]));
  d1 = d1 > 0.f ? d1 : 0.f;
  d2 = d2 > 0.f ? d2 : 0.f;
  float t3 = DM_MUL(0.5f, dm_log(DM_ADD(DM_DIV(disc, DM_ADD(DM_MUL(4.f, DM_SQRT(DM_MUL(d1, d2))), eps)), eps)));
  float bd = DM_ADD(DM_ADD(t1, t2), t3);
  bd = bd > eps ? bd : eps;
  bd = bd < 100.f ? bd : 100.f;
  return DM_SUB(1.f, DM_SQRT(DM_ADD(DM_SUB(1.f, dm_exp(-bd)), eps)));
}
