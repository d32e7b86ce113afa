/* ORACLE / TEST INFRASTRUCTURE — CPU restatement of the reference's pre/post-processing.
 *
 * Used only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker; never by the engine.  Plain C, single thread, straight loops in the order the
 * reference kernels define:
 *   oref_letterbox  engine/engine.cu:968-998 (k_preprocess) + 1704-1713 (host geometry)
 *   oref_decode_obb_level / oref_nms_obb  engine/engine.cu:908-960 (k_decode_obb) and
 *                   1160-1252 (probiou, k_nms_obb): first-max class, sigmoid score >= conf,
 *                   DFL sides, theta = (sigmoid(a) - 0.25) * pi, centre offset rotated by
 *                   theta; NMS in score order (ties: anchor asc), candidate j dropped when
 *                   any earlier candidate of its class (dropped or not) has probiou >= thr
 *                   with it (ultralytics fast-NMS), every candidate considered
 *   oref_preprocess_cls  engine/engine.cu:1000-1046 (k_preprocess_cls + clsGeom): shortest
 *                   edge to S (long edge S*long/short truncated), centre crop with
 *                   round-half-even offsets, per-axis triangle filter of support
 *                   max(src/resized, 1), weights normalised by their sums, RGB /255
 *   oref_decode     engine/engine.cu:848-906 (k_decode): first-max class over nc logits,
 *                   sigmoid score, gate score >= conf, DFL softmax expectation, xyxy*stride
 *   oref_nms        engine/engine.cu:1051-1123 (k_nms) without its 1024-candidate cap:
 *                   candidates sorted by score desc (ties: anchor index asc), greedy
 *                   same-class suppression with IoU = inter/(area_a+area_b-inter) > thr
 *   oref_masks      engine/engine.cu:1129-1158 (k_mask_assemble): logit = coef . proto
 *                   (fp32, c = 0..nm-1 in order), half-open crop at proto scale, logit > 0
 * Arithmetic goes through detmath.h (explicitly rounded binary32 ops, Cody-Waite exp), the
 * same formulas the CUDA kernels use, so results must match bit for bit.  Build with
 * -ffp-contract=off (oracle/Makefile).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#include "../yolo11.cu_b200/csrc/detmath.h"

/* fp16 NHWC view: element (y, x, c) of image n at base[((n*H + y)*W + x)*stride + c] */
typedef struct {
  const uint16_t* base; /* already offset by the view's channel offset */
  int H, W, stride;
} OView;

static const uint16_t* opix(const OView* v, int n, int y, int x) {
  return v->base + (((size_t)n * v->H + y) * v->W + x) * (size_t)v->stride;
}

void oref_letterbox_geom(int S, int sh, int sw, float* scale, int* nh, int* nw, int* top,
                         int* left) {
  float a = (float)S / (float)sh, b = (float)S / (float)sw;
  float s = a < b ? a : b;
  *scale = s;
  *nh = (int)roundf((float)sh * s);
  *nw = (int)roundf((float)sw * s);
  *top = (S - *nh) / 2;
  *left = (S - *nw) / 2;
}

/* bgr: sh x sw x 3 u8; out: S x S x 3 fp16 bits (RGB, /255, pad 114) */
void oref_letterbox(const uint8_t* bgr, int sh, int sw, int S, uint16_t* out) {
  float scale;
  int nh, nw, top, left;
  oref_letterbox_geom(S, sh, sw, &scale, &nh, &nw, &top, &left);
  for (int y = 0; y < S; y++)
    for (int x = 0; x < S; x++) {
      float r, g, b;
      if (y < top || y >= top + nh || x < left || x >= left + nw) {
        r = g = b = 114.f;
      } else {
        float fy = DM_SUB(DM_DIV(DM_ADD((float)(y - top), 0.5f), scale), 0.5f);
        float fx = DM_SUB(DM_DIV(DM_ADD((float)(x - left), 0.5f), scale), 0.5f);
        int y0 = (int)floorf(fy), x0 = (int)floorf(fx);
        float wy = DM_SUB(fy, (float)y0), wx = DM_SUB(fx, (float)x0);
        int y1 = y0 + 1 < sh - 1 ? y0 + 1 : sh - 1, x1 = x0 + 1 < sw - 1 ? x0 + 1 : sw - 1;
        if (y0 < 0) y0 = 0;
        if (x0 < 0) x0 = 0;
        const uint8_t* p00 = bgr + ((size_t)y0 * sw + x0) * 3;
        const uint8_t* p01 = bgr + ((size_t)y0 * sw + x1) * 3;
        const uint8_t* p10 = bgr + ((size_t)y1 * sw + x0) * 3;
        const uint8_t* p11 = bgr + ((size_t)y1 * sw + x1) * 3;
        float w00 = DM_MUL(DM_SUB(1.f, wy), DM_SUB(1.f, wx));
        float w01 = DM_MUL(DM_SUB(1.f, wy), wx);
        float w10 = DM_MUL(wy, DM_SUB(1.f, wx));
        float w11 = DM_MUL(wy, wx);
        float v[3];
        for (int c = 0; c < 3; c++) {
          float t = DM_MUL((float)p00[c], w00);
          t = DM_ADD(t, DM_MUL((float)p01[c], w01));
          t = DM_ADD(t, DM_MUL((float)p10[c], w10));
          v[c] = DM_ADD(t, DM_MUL((float)p11[c], w11));
        }
        b = v[0]; g = v[1]; r = v[2];
      }
      uint16_t* o = out + ((size_t)y * S + x) * 3;
      o[0] = dm_f2h(DM_DIV(r, 255.f));
      o[1] = dm_f2h(DM_DIV(g, 255.f));
      o[2] = dm_f2h(DM_DIV(b, 255.f));
    }
}

/* One level of one image.  Writes conf-passing anchors in anchor order as 7-float records
 * [x1 y1 x2 y2 score cls anchor] (anchor = abase + y*W + x).  Returns the count. */
int oref_decode_level(const uint16_t* box, int bstride, const uint16_t* cls, int cstride, int H,
                      int W, int img, int nc, int stride, float conf, int abase, float* out) {
  OView bv = {box, H, W, bstride}, cv = {cls, H, W, cstride};
  int n = 0;
  for (int y = 0; y < H; y++)
    for (int x = 0; x < W; x++) {
      const uint16_t* cp = opix(&cv, img, y, x);
      float best = -INFINITY;
      int bc = 0;
      for (int c = 0; c < nc; c++) {
        float f = dm_h2f(cp[c]);
        if (f > best) { best = f; bc = c; }
      }
      float score = dm_sigmoid(best);
      if (!(score >= conf)) continue;
      const uint16_t* bp = opix(&bv, img, y, x);
      float d[4];
      for (int s = 0; s < 4; s++) {
        float l[16];
        for (int i = 0; i < 16; i++) l[i] = dm_h2f(bp[s * 16 + i]);
        d[s] = dm_dfl16(l);
      }
      float cx = DM_ADD((float)x, 0.5f), cy = DM_ADD((float)y, 0.5f), st = (float)stride;
      float* o = out + (size_t)n * 7;
      o[0] = DM_MUL(DM_SUB(cx, d[0]), st);
      o[1] = DM_MUL(DM_SUB(cy, d[1]), st);
      o[2] = DM_MUL(DM_ADD(cx, d[2]), st);
      o[3] = DM_MUL(DM_ADD(cy, d[3]), st);
      o[4] = score;
      o[5] = (float)bc;
      o[6] = (float)(abase + y * W + x);
      n++;
    }
  return n;
}

/* out: n x 8 records (cx cy w h score cls theta anchor) in anchor order */
int oref_decode_obb_level(const uint16_t* box, int bstride, const uint16_t* cls, int cstride,
                          const uint16_t* ang, int astride, int H, int W, int img, int nc,
                          int stride, float conf, int abase, float* out) {
  OView bv = {box, H, W, bstride}, cv = {cls, H, W, cstride}, av = {ang, H, W, astride};
  int n = 0;
  for (int y = 0; y < H; y++)
    for (int x = 0; x < W; x++) {
      const uint16_t* cp = opix(&cv, img, y, x);
      float best = -INFINITY;
      int bc = 0;
      for (int c = 0; c < nc; c++) {
        float f = dm_h2f(cp[c]);
        if (f > best) { best = f; bc = c; }
      }
      float score = dm_sigmoid(best);
      if (!(score >= conf)) continue;
      const uint16_t* bp = opix(&bv, img, y, x);
      float d[4];
      for (int s = 0; s < 4; s++) {
        float l[16];
        for (int i = 0; i < 16; i++) l[i] = dm_h2f(bp[s * 16 + i]);
        d[s] = dm_dfl16(l);
      }
      float th = DM_MUL(DM_SUB(dm_sigmoid(dm_h2f(opix(&av, img, y, x)[0])), 0.25f), 3.14159265358979f);
      float sn, cs;
      dm_sincos(th, &sn, &cs);
      float xf = DM_MUL(DM_SUB(d[2], d[0]), 0.5f), yf = DM_MUL(DM_SUB(d[3], d[1]), 0.5f);
      float st = (float)stride;
      float* o = out + (size_t)n * 8;
      o[0] = DM_MUL(DM_SUB(DM_ADD(DM_ADD((float)x, 0.5f), DM_MUL(xf, cs)), DM_MUL(yf, sn)), st);
      o[1] = DM_MUL(DM_ADD(DM_ADD(DM_ADD((float)y, 0.5f), DM_MUL(xf, sn)), DM_MUL(yf, cs)), st);
      o[2] = DM_MUL(DM_ADD(d[0], d[2]), st);
      o[3] = DM_MUL(DM_ADD(d[1], d[3]), st);
      o[4] = score;
      o[5] = (float)bc;
      o[6] = th;
      o[7] = (float)(abase + y * W + x);
      n++;
    }
  return n;
}

static const float* g_obb_recs;
static int cmp_obb(const void* a, const void* b) {
  const float* ra = g_obb_recs + (size_t)(*(const int*)a) * 8;
  const float* rb = g_obb_recs + (size_t)(*(const int*)b) * 8;
  if (ra[4] != rb[4]) return ra[4] > rb[4] ? -1 : 1;
  return ra[7] < rb[7] ? -1 : ra[7] > rb[7];
}

/* recs: n x 8 (anchor order); out: up to max_out x 8 survivors in score order */
int oref_nms_obb(const float* recs, int n, float thr, int max_out, float* out) {
  int* order = (int*)malloc(sizeof(int) * (n > 0 ? n : 1));
  float* cov = (float*)malloc(sizeof(float) * 3 * (n > 0 ? n : 1));
  for (int i = 0; i < n; i++) order[i] = i;
  g_obb_recs = recs;
  qsort(order, n, sizeof(int), cmp_obb);
  for (int i = 0; i < n; i++) {
    const float* r = recs + (size_t)order[i] * 8;
    dm_obb_cov(r[2], r[3], r[6], cov + 3 * i);
  }
  int m = 0;
  for (int j = 0; j < n && m < max_out; j++) {
    const float* b = recs + (size_t)order[j] * 8;
    int dead = 0;
    for (int i = 0; i < j && !dead; i++) {
      const float* a = recs + (size_t)order[i] * 8;
      if (a[5] != b[5]) continue;
      if (dm_probiou(a[0], a[1], cov + 3 * i, b[0], b[1], cov + 3 * j) >= thr) dead = 1;
    }
    if (!dead) memcpy(out + (size_t)(m++) * 8, b, 8 * sizeof(float));
  }
  free(order);
  free(cov);
  return m;
}

static const float* g_sort_recs;
static int cmp_score_desc(const void* a, const void* b) {
  const float* ra = g_sort_recs + (size_t)(*(const int*)a) * 7;
  const float* rb = g_sort_recs + (size_t)(*(const int*)b) * 7;
  if (ra[4] != rb[4]) return ra[4] > rb[4] ? -1 : 1;
  return ra[6] < rb[6] ? -1 : (ra[6] > rb[6] ? 1 : 0);
}

/* recs: n 7-float records from oref_decode_level (any order).  Writes up to max_out
 * survivors as 7-float records (same layout) in output order; returns the count. */
int oref_nms(const float* recs, int n, float thr, int max_out, float* out) {
  int* order = (int*)malloc(sizeof(int) * (n > 0 ? n : 1));
  unsigned char* dead = (unsigned char*)calloc(n > 0 ? n : 1, 1);
  for (int i = 0; i < n; i++) order[i] = i;
  g_sort_recs = recs;
  qsort(order, n, sizeof(int), cmp_score_desc);
  int m = 0;
  for (int i = 0; i < n; i++) {
    const float* a = recs + (size_t)order[i] * 7;
    if (dead[order[i]]) continue;
    if (m < max_out) memcpy(out + (size_t)m * 7, a, 7 * sizeof(float));
    m++;
    float aarea = dm_area(a[0], a[1], a[2], a[3]);
    for (int j = i + 1; j < n; j++) {
      const float* b = recs + (size_t)order[j] * 7;
      if (dead[order[j]] || b[5] != a[5]) continue;
      if (dm_iou_gt(a[0], a[1], a[2], a[3], aarea, b[0], b[1], b[2], b[3], thr)) dead[order[j]] = 1;
    }
  }
  free(order);
  free(dead);
  return m < max_out ? m : max_out;
}

/* coef: nm fp16 coefficients of the survivor's anchor; proto view of image img;
 * det: x1 y1 x2 y2 in letterbox pixels; out: Ph*Pw bytes. */
void oref_mask(const uint16_t* coef, int nm, const uint16_t* proto, int pstride, int Ph, int Pw,
               int img, const float* det, float rx, float ry, uint8_t* out) {
  OView pv = {proto, Ph, Pw, pstride};
  float co[256];
  for (int c = 0; c < nm; c++) co[c] = dm_h2f(coef[c]);
  float bx1 = DM_MUL(det[0], rx), by1 = DM_MUL(det[1], ry);
  float bx2 = DM_MUL(det[2], rx), by2 = DM_MUL(det[3], ry);
  for (int py = 0; py < Ph; py++)
    for (int px = 0; px < Pw; px++) {
      uint8_t m = 0;
      if ((float)px >= bx1 && (float)px < bx2 && (float)py >= by1 && (float)py < by2) {
        const uint16_t* pp = opix(&pv, img, py, px);
        float acc = 0.f;
        for (int c = 0; c < nm; c++) acc = DM_FMA(co[c], dm_h2f(pp[c]), acc);
        m = acc > 0.f;
      }
      out[(size_t)py * Pw + px] = m;
    }
}

/* exposed for the math tests */
float oref_exp(float x) { return dm_exp(x); }
float oref_sigmoid(float x) { return dm_sigmoid(x); }
/* dm_quot_gt over arrays: out[i] = (RN(a[i] / b[i]) > t[i]) by the division-free test. */
void oref_quot_gt(const float* a, const float* b, const float* t, int n, int* out) {
  for (int i = 0; i < n; i++) out[i] = dm_quot_gt(a[i], b[i], t[i]);
}
/* Mismatches of dm_div255(v) against v / 255 over the binary32 bit patterns lo..hi (step). */
long oref_div255_check(unsigned lo, unsigned hi, unsigned step) {
  long bad = 0;
  for (unsigned long long u = lo; u <= hi; u += step) {
    const float v = dm_bits2f((unsigned)u);
    if (dm_f2bits(dm_div255(v)) != dm_f2bits(DM_DIV(v, 255.0f))) bad++;
  }
  return bad;
}
float oref_sin(float x) { float s, c; dm_sincos(x, &s, &c); return s; }
float oref_cos(float x) { float s, c; dm_sincos(x, &s, &c); return c; }
float oref_log(float x) { return dm_log(x); }
float oref_probiou(const float* a, const float* b) {   /* a, b: cx cy w h theta */
  float ca[3], cb[3];
  dm_obb_cov(a[2], a[3], a[4], ca);
  dm_obb_cov(b[2], b[3], b[4], cb);
  return dm_probiou(a[0], a[1], ca, b[0], b[1], cb);
}
static float cls_tri(int i, float centre, float sup) {
  float d = fabsf(DM_SUB(DM_ADD((float)i, 0.5f), centre));
  float w = DM_SUB(1.f, DM_DIV(d, sup));
  return w > 0.f ? w : 0.f;
}

/* out: S*S*3 fp16 (RGB), geom: {resized h, resized w, top, left} */
void oref_preprocess_cls(const uint8_t* src, int sh, int sw, int S, uint16_t* out, int* geom) {
  long rh, rw;
  if (sw <= sh) { rw = S; rh = (long)S * sh / sw; }
  else { rh = S; rw = (long)S * sw / sh; }
  int dy = (int)rh - S, dx = (int)rw - S;
  int top = dy / 2 + ((dy & 1) && ((dy / 2) & 1));
  int left = dx / 2 + ((dx & 1) && ((dx / 2) & 1));
  geom[0] = (int)rh; geom[1] = (int)rw; geom[2] = top; geom[3] = left;
  float scy = DM_DIV((float)sh, (float)rh), scx = DM_DIV((float)sw, (float)rw);
  float supy = scy > 1.f ? scy : 1.f, supx = scx > 1.f ? scx : 1.f;
  for (int y = 0; y < S; y++)
    for (int x = 0; x < S; x++) {
      float cy = DM_MUL(DM_ADD((float)(y + top), 0.5f), scy);
      float cx = DM_MUL(DM_ADD((float)(x + left), 0.5f), scx);
      int y0 = (int)DM_ADD(DM_SUB(cy, supy), 0.5f), y1 = (int)DM_ADD(DM_ADD(cy, supy), 0.5f);
      int x0 = (int)DM_ADD(DM_SUB(cx, supx), 0.5f), x1 = (int)DM_ADD(DM_ADD(cx, supx), 0.5f);
      if (y0 < 0) y0 = 0;
      if (x0 < 0) x0 = 0;
      if (y1 > sh) y1 = sh;
      if (x1 > sw) x1 = sw;
      float wys = 0.f, wxs = 0.f, b = 0.f, g = 0.f, r = 0.f;
      for (int i = y0; i < y1; i++) wys = DM_ADD(wys, cls_tri(i, cy, supy));
      for (int j = x0; j < x1; j++) wxs = DM_ADD(wxs, cls_tri(j, cx, supx));
      for (int i = y0; i < y1; i++) {
        float wy = cls_tri(i, cy, supy);
        for (int j = x0; j < x1; j++) {
          float w = DM_MUL(wy, cls_tri(j, cx, supx));
          const uint8_t* p = src + ((size_t)i * sw + j) * 3;
          b = DM_ADD(b, DM_MUL(w, (float)p[0]));
          g = DM_ADD(g, DM_MUL(w, (float)p[1]));
          r = DM_ADD(r, DM_MUL(w, (float)p[2]));
        }
      }
      float inv = DM_DIV(1.f, DM_MUL(DM_MUL(wys, wxs), 255.f));
      uint16_t* o = out + ((size_t)y * S + x) * 3;
      o[0] = dm_f2h(DM_MUL(r, inv));
      o[1] = dm_f2h(DM_MUL(g, inv));
      o[2] = dm_f2h(DM_MUL(b, inv));
    }
}

uint16_t oref_f2h(float x) { return dm_f2h(x); }
float oref_h2f(uint16_t h) { return dm_h2f(h); }
