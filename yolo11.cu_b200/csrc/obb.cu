// Oriented boxes (task "obb"): decode and rotated NMS.
//
//   decode_obb_kernel  one thread per anchor: first-max class over nc logits, sigmoid score
//                      gated at conf, DFL side distances, theta = (sigmoid(angle) - 0.25)*pi,
//                      centre = anchor + ((r - l)/2, (b - t)/2) rotated by theta, size
//                      (l + r, t + b), all times the stride (reference k_decode_obb,
//                      engine/engine.cu:908-960; ultralytics dist2rbox)
//   nms_obb_kernel     one 1024-thread block per image: candidates compacted in anchor order
//                      (every candidate is kept; the reference truncates at 2048), sorted by
//                      score (ties: anchor order) with a bitonic sort of 64-bit keys in the
//                      workspace, Gaussian covariances per candidate, then ultralytics
//                      fast-NMS: candidate j is dropped when any earlier candidate of its
//                      class, dropped or not, has probiou >= thr with it; so every j is
//                      independent and the pairs split across the block (reference k_nms_obb
//                      + probiou, engine/engine.cu:1160-1252).
// All float math is detmath.h's explicitly rounded arithmetic, so the C oracle
// (oracle/postproc_ref.c) reproduces candidates and survivors bit for bit.
#include "common.cuh"
#include "detmath.h"

namespace yk {

struct ObbLevel {
  DView box, cls, ang;
  int H, W, stride, abase;
};
struct ObbLevels {
  ObbLevel l[4];
  int n, A;
};

// per-image workspace: rec[A][8] f32 (cx cy w h score cls theta anchor), flag[A] i32,
// cand[A] i32 (compacted anchors), keys[P] u64 (P = pow2 >= A), cov[A][3] f32 and
// rcls[A] f32 (in rank order), dead[A] u8
struct ObbWs {
  size_t rec, flag, cand, keys, cov, rcls, dead, per_img;
  int A, P;
};
static inline ObbWs obb_ws(int A) {
  ObbWs L;
  L.A = A;
  L.P = 1;
  while (L.P < A) L.P <<= 1;
  size_t o = 0;
  auto al = [](size_t v) { return (v + 15) & ~(size_t)15; };
  L.rec = o;  o = al(o + (size_t)A * 32);
  L.flag = o; o = al(o + (size_t)A * 4);
  L.cand = o; o = al(o + (size_t)A * 4);
  L.keys = o; o = al(o + (size_t)L.P * 8);
  L.cov = o;  o = al(o + (size_t)A * 12);
  L.rcls = o; o = al(o + (size_t)A * 4);
  L.dead = o; o = al(o + (size_t)A);
  L.per_img = o;
  return L;
}

__global__ void __launch_bounds__(256) decode_obb_kernel(ObbLevels lv, int batch, int nc,
                                                         float conf, uint8_t* ws, ObbWs L) {
  pdl_wait();
  pdl_trigger();
  const long long ga = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (ga >= (long long)batch * lv.A) return;
  const int img = (int)(ga / lv.A), a = (int)(ga - (long long)img * lv.A);
  int li = 0;
  while (li + 1 < lv.n && a >= lv.l[li + 1].abase) li++;
  const ObbLevel& Lv = lv.l[li];
  const int rem = a - Lv.abase, y = rem / Lv.W, x = rem - y * Lv.W;
  uint8_t* wimg = ws + (size_t)img * L.per_img;
  int* flag = (int*)(wimg + L.flag);
  const __half* cp = Lv.cls.p + Lv.cls.pix(img, y, x);
  float best = -INFINITY;
  int bcls = 0;
  for (int c0 = 0; c0 < nc; c0 += 8) {
    const uint4 v = *(const uint4*)(cp + c0);
    const __half* h = (const __half*)&v;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float f = __half2float(h[i]);
      if (c0 + i < nc && f > best) { best = f; bcls = c0 + i; }   // first max wins
    }
  }
  const float score = dm_sigmoid(best);
  if (!(score >= conf)) { flag[a] = 0; return; }
  const __half* bp = Lv.box.p + Lv.box.pix(img, y, x);
  float d[4];
#pragma unroll
  for (int s = 0; s < 4; s++) {
    const uint4 v0 = *(const uint4*)(bp + s * 16), v1 = *(const uint4*)(bp + s * 16 + 8);
    const __half* h0 = (const __half*)&v0;
    const __half* h1 = (const __half*)&v1;
    float l[16];
#pragma unroll
    for (int i = 0; i < 8; i++) { l[i] = __half2float(h0[i]); l[i + 8] = __half2float(h1[i]); }
    d[s] = dm_dfl16(l);
  }
  const float th = DM_MUL(DM_SUB(dm_sigmoid(__half2float(Lv.ang.p[Lv.ang.pix(img, y, x)])), 0.25f),
                          3.14159265358979f);
  float sn, cs;
  dm_sincos(th, &sn, &cs);
  const float xf = DM_MUL(DM_SUB(d[2], d[0]), 0.5f), yf = DM_MUL(DM_SUB(d[3], d[1]), 0.5f);
  const float st = (float)Lv.stride;
  float* o = (float*)(wimg + L.rec) + (size_t)a * 8;
  o[0] = DM_MUL(DM_SUB(DM_ADD(DM_ADD((float)x, 0.5f), DM_MUL(xf, cs)), DM_MUL(yf, sn)), st);
  o[1] = DM_MUL(DM_ADD(DM_ADD(DM_ADD((float)y, 0.5f), DM_MUL(xf, sn)), DM_MUL(yf, cs)), st);
  o[2] = DM_MUL(DM_ADD(d[0], d[2]), st);
  o[3] = DM_MUL(DM_ADD(d[1], d[3]), st);
  o[4] = score;
  o[5] = (float)bcls;
  o[6] = th;
  o[7] = (float)a;
  flag[a] = 1;
}

constexpr int kObbThreads = 1024;

__global__ void __launch_bounds__(kObbThreads, 1)
nms_obb_kernel(float thr, int max_out, uint8_t* ws, ObbWs L, float* outdets, int* outcnt,
               int* rawcnt) {
  pdl_wait();
  pdl_trigger();
  __shared__ int wsum[32];
  __shared__ int s_n, s_m;
  const int tid = threadIdx.x;
  uint8_t* wimg = ws + (size_t)blockIdx.x * L.per_img;
  const float* rec = (const float*)(wimg + L.rec);
  const int* flag = (const int*)(wimg + L.flag);
  int* cand = (int*)(wimg + L.cand);
  unsigned long long* keys = (unsigned long long*)(wimg + L.keys);
  float* cov = (float*)(wimg + L.cov);
  float* rcls = (float*)(wimg + L.rcls);
  uint8_t* dead = wimg + L.dead;
  // 1. compaction in anchor order
  int base = 0;
  for (int a0 = 0; a0 < L.A; a0 += kObbThreads) {
    const int a = a0 + tid;
    const int f = a < L.A ? flag[a] : 0;
    int tot;
    const int pre = block_scan(f, wsum, &tot);
    if (f) cand[base + pre] = a;
    base += tot;
  }
  const int n = base;
  // 2. keys: descending score, then ascending anchor; padding sorts last
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = tid; i < P; i += kObbThreads) {
    unsigned long long k = ~0ull;
    if (i < n) {
      const int a = cand[i];
      const uint32_t sb = dm_f2bits(rec[(size_t)a * 8 + 4]);   // score > 0: bits ordered
      k = ((unsigned long long)(0xffffffffu - sb) << 32) | (uint32_t)a;
    }
    keys[i] = k;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < P; i += kObbThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = keys[i], b = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) { keys[i] = b; keys[ixj] = a; }
        }
      }
      __syncthreads();
    }
  // 3. covariances and classes in rank order
  for (int i = tid; i < n; i += kObbThreads) {
    const float* r = rec + (size_t)(uint32_t)keys[i] * 8;
    dm_obb_cov(r[2], r[3], r[6], cov + 3 * i);
    rcls[i] = r[5];
    dead[i] = 0;
  }
  __syncthreads();
  // 4. fast-NMS: j is dropped by any earlier same-class i with probiou >= thr
  for (int j = tid; j < n; j += kObbThreads) {
    const float* rj = rec + (size_t)(uint32_t)keys[j] * 8;
    const float cj = rcls[j];
    uint8_t dj = 0;
    for (int i = 0; i < j && !dj; i++) {
      if (rcls[i] != cj) continue;
      const float* ri = rec + (size_t)(uint32_t)keys[i] * 8;
      if (dm_probiou(ri[0], ri[1], cov + 3 * i, rj[0], rj[1], cov + 3 * j) >= thr) dj = 1;
    }
    dead[j] = dj;
  }
  __syncthreads();
  // 5. survivors in rank order, the first max_out
  int m = 0;
  for (int i0 = 0; i0 < n && m < max_out; i0 += kObbThreads) {
    const int i = i0 + tid;
    const int alive = i < n && !dead[i];
    int tot;
    const int pre = block_scan(alive, wsum, &tot);
    if (alive && m + pre < max_out) {
      const float* r = rec + (size_t)(uint32_t)keys[i] * 8;
      float* o = outdets + ((size_t)blockIdx.x * max_out + m + pre) * 7;
#pragma unroll
      for (int k = 0; k < 7; k++) o[k] = r[k];
    }
    m += tot;
  }
  if (tid == 0) {
    s_n = n;
    s_m = m < max_out ? m : max_out;
    outcnt[blockIdx.x] = s_m;
    rawcnt[blockIdx.x] = s_n;
  }
}

}  // namespace yk

using namespace yk;

extern "C" size_t yk_obb_workspace_bytes(int batch, int anchors) {
  return (size_t)batch * obb_ws(anchors).per_img;
}

extern "C" int yk_decode_obb(const YkLevel* levels, int nlevels, int batch, int nc, float conf,
                             void* ws, yk_stream_t st) {
  if (!levels || nlevels < 1 || nlevels > 4 || batch < 1 || nc < 1 || !ws) return YK_EINVAL;
  ObbLevels lv;
  int A = 0;
  for (int i = 0; i < nlevels; i++) {
    const YkLevel& l = levels[i];
    if (!view_vec8(&l.box) || !view_vec8(&l.cls) || !view_ok(&l.coef) || l.box.C != 64 ||
        l.cls.C < (nc + 7) / 8 * 8 || l.coef.C < 1 || l.box.H != l.cls.H || l.box.W != l.cls.W ||
        l.coef.H != l.box.H || l.coef.W != l.box.W || l.box.batch < batch ||
        l.cls.batch < batch || l.coef.batch < batch)
      return YK_EINVAL;
    lv.l[i] = {dview(l.box), dview(l.cls), dview(l.coef), l.box.H, l.box.W, l.stride, A};
    A += l.box.H * l.box.W;
  }
  lv.n = nlevels;
  lv.A = A;
  if (A >= (1 << 24)) return YK_EUNSUP;
  const long long total = (long long)batch * A;
  launch_k(decode_obb_kernel, (unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)st, lv,
           batch, nc, conf, (uint8_t*)ws, obb_ws(A));
  note_launch();
  return check_launch("decode_obb");
}

extern "C" int yk_nms_obb(int batch, int anchors, float iou, int max_out, void* ws,
                          float* outdets, int* outcnt, int* rawcnt, yk_stream_t st) {
  if (batch < 1 || anchors < 1 || max_out < 1 || !ws || !outdets || !outcnt || !rawcnt)
    return YK_EINVAL;
  launch_k(nms_obb_kernel, batch, kObbThreads, 0, (cudaStream_t)st, iou, max_out,
           (uint8_t*)ws, obb_ws(anchors), outdets, outcnt, rawcnt);
  note_launch();
  return check_launch("nms_obb");
}
