// Pre- and post-processing: letterbox, DFL decode, exact NMS, segment masks.
//
// Everything here computes with the explicitly rounded fp32 operations of detmath.h, so a
// host restatement built from the same formulas reproduces it bit for bit: candidate
// lists, survivor indices and boxes are deterministic and independent of thread timing
// (the reference appends candidates with atomicAdd and truncates NMS input at 1024 in that
// order, engine/engine.cu:890, 1064).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "detmath.h"

namespace yk {

// ---------------- letterbox (engine/engine.cu:968-998) ----------------
__global__ void letterbox_kernel(const uint8_t* __restrict__ src, int sh, int sw, __half* dst,
                                 int dh, int dw, int dstride, float scale, int top, int left,
                                 int nh, int nw) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= dh * dw) return;
  const int x = idx % dw, y = idx / dw;
  float r, g, b;
  if (y < top || y >= top + nh || x < left || x >= left + nw) {
    r = g = b = 114.f;
  } else {
    const float fy = DM_SUB(DM_DIV(DM_ADD((float)(y - top), 0.5f), scale), 0.5f);
    const float fx = DM_SUB(DM_DIV(DM_ADD((float)(x - left), 0.5f), scale), 0.5f);
    int y0 = (int)floorf(fy), x0 = (int)floorf(fx);
    const float wy = DM_SUB(fy, (float)y0), wx = DM_SUB(fx, (float)x0);
    const int y1 = min(y0 + 1, sh - 1), x1 = min(x0 + 1, sw - 1);
    y0 = max(y0, 0);
    x0 = max(x0, 0);
    const uint8_t* p00 = src + ((size_t)y0 * sw + x0) * 3;
    const uint8_t* p01 = src + ((size_t)y0 * sw + x1) * 3;
    const uint8_t* p10 = src + ((size_t)y1 * sw + x0) * 3;
    const uint8_t* p11 = src + ((size_t)y1 * sw + x1) * 3;
    const float w00 = DM_MUL(DM_SUB(1.f, wy), DM_SUB(1.f, wx));
    const float w01 = DM_MUL(DM_SUB(1.f, wy), wx);
    const float w10 = DM_MUL(wy, DM_SUB(1.f, wx));
    const float w11 = DM_MUL(wy, wx);
    float v[3];
#pragma unroll
    for (int c = 0; c < 3; c++) {
      float t = DM_MUL((float)p00[c], w00);
      t = DM_ADD(t, DM_MUL((float)p01[c], w01));
      t = DM_ADD(t, DM_MUL((float)p10[c], w10));
      v[c] = DM_ADD(t, DM_MUL((float)p11[c], w11));
    }
    b = v[0]; g = v[1]; r = v[2];
  }
  __half* o = dst + (size_t)idx * dstride;
  o[0] = __float2half_rn(DM_DIV(r, 255.f));   // RGB order
  o[1] = __float2half_rn(DM_DIV(g, 255.f));
  o[2] = __float2half_rn(DM_DIV(b, 255.f));
}

// ---------------- decode (engine/engine.cu:848-906) ----------------
struct DevLevel {
  DView box, cls;
  int H, W, stride, abase;
};
struct DevLevels {
  DevLevel l[4];
  int n, A;
};

// Per-image workspace layout (all 16-byte aligned): rec[A][6] f32, flag[A] i32,
// keys[P2] u64 (P2 = next pow2 of A; global fallback of the shared-memory sort),
// kept[A][5] f32, surv[A] i32.
struct WsLayout {
  size_t rec, flag, keys, kept, surv, per_img;
};
static inline size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }
static inline int pow2ge(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}
static inline WsLayout ws_layout(int A) {
  WsLayout L;
  size_t o = 0;
  L.rec = o;  o = al16(o + (size_t)A * 6 * 4);
  L.flag = o; o = al16(o + (size_t)A * 4);
  L.keys = o; o = al16(o + (size_t)pow2ge(A) * 8);
  L.kept = o; o = al16(o + (size_t)A * 5 * 4);
  L.surv = o; o = al16(o + (size_t)A * 4);
  L.per_img = o;
  return L;
}

__global__ void decode_kernel(DevLevels lv, int batch, int nc, float conf, uint8_t* ws,
                              WsLayout L) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)batch * lv.A) return;
  const int img = (int)(gid / lv.A), a = (int)(gid - (long long)img * lv.A);
  int li = 0;
  while (li + 1 < lv.n && a >= lv.l[li + 1].abase) li++;
  const DevLevel& L0 = lv.l[li];
  const int rem = a - L0.abase;
  const int y = rem / L0.W, x = rem - y * L0.W;
  uint8_t* wimg = ws + (size_t)img * L.per_img;
  int* flag = (int*)(wimg + L.flag);
  const __half* cp = L0.cls.p + L0.cls.pix(img, y, x);
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
  const __half* bp = L0.box.p + L0.box.pix(img, y, x);
  float d[4];
#pragma unroll
  for (int side = 0; side < 4; side++) {
    const uint4 v0 = *(const uint4*)(bp + side * 16), v1 = *(const uint4*)(bp + side * 16 + 8);
    const __half* h0 = (const __half*)&v0;
    const __half* h1 = (const __half*)&v1;
    float l[16];
#pragma unroll
    for (int i = 0; i < 8; i++) { l[i] = __half2float(h0[i]); l[i + 8] = __half2float(h1[i]); }
    d[side] = dm_dfl16(l);
  }
  const float cx = DM_ADD((float)x, 0.5f), cy = DM_ADD((float)y, 0.5f), st = (float)L0.stride;
  float* o = (float*)(wimg + L.rec) + (size_t)a * 6;
  o[0] = DM_MUL(DM_SUB(cx, d[0]), st);
  o[1] = DM_MUL(DM_SUB(cy, d[1]), st);
  o[2] = DM_MUL(DM_ADD(cx, d[2]), st);
  o[3] = DM_MUL(DM_ADD(cy, d[3]), st);
  o[4] = score;
  o[5] = (float)bcls;
  flag[a] = 1;
}

// ---------------- NMS (engine/engine.cu:1051-1123, exact + deterministic) ----------------
constexpr int kNmsThreads = 1024;
constexpr int kNmsSmemKeys = 16384;    // keys sorted in shared memory up to this count
constexpr int kMaxClasses = 1024;
constexpr int kKeptSmem = 48;          // kept boxes per class held in shared memory

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Block-wide exclusive scan of one int per thread; returns the prefix, *total = block sum.
__device__ int block_scan(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(~0u, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x >> 5) ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(~0u, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;   // inclusive
  }
  __syncthreads();
  const int pre = (warp ? wsum[warp - 1] : 0) + x - v;
  *total = wsum[(blockDim.x >> 5) - 1];
  __syncthreads();
  return pre;
}

__device__ void bitonic_sort(unsigned long long* keys, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const bool asc = (i & k) == 0;
          const unsigned long long a = keys[i], b = keys[ixj];
          if ((a > b) == asc) { keys[i] = b; keys[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
}

__global__ void __launch_bounds__(kNmsThreads, 1)
nms_kernel(int A, float iou, int max_out, uint8_t* ws, WsLayout L, float* outdets,
           int* outidx, int* outcnt, int* rawcnt) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ __align__(16) unsigned long long skeys[];
  __shared__ int wsum[32];
  __shared__ int segs[kMaxClasses + 1];
  __shared__ int s_total;
  __shared__ float kept_s[32][kKeptSmem][5];
  const int img = blockIdx.x, tid = threadIdx.x;
  uint8_t* wimg = ws + (size_t)img * L.per_img;
  const float* rec = (const float*)(wimg + L.rec);
  const int* flag = (const int*)(wimg + L.flag);
  float* kept = (float*)(wimg + L.kept);
  int* surv = (int*)(wimg + L.surv);

  // 1. count the candidates per warp (each warp owns a contiguous anchor range, ballots)
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int span = ((A + nwarps - 1) / nwarps + 31) & ~31;
  const int a_lo = warp * span, a_hi = min(A, a_lo + span);
  int cnt = 0;
  for (int a0 = a_lo; a0 < a_hi; a0 += 32) {
    const int a = a0 + lane;
    cnt += __popc(__ballot_sync(~0u, a < a_hi && flag[a]));
  }
  if (lane == 0) wsum[warp] = cnt;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < nwarps ? wsum[lane] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y2 = __shfl_up_sync(~0u, x, o);
      if (lane >= o) x += y2;
    }
    wsum[lane] = x - v;                       // exclusive prefix
    if (lane == 31) s_total = x;
  }
  __syncthreads();
  const int n = s_total;
  int P = 2;
  while (P < n) P <<= 1;
  unsigned long long* keys = P <= kNmsSmemKeys ? skeys : (unsigned long long*)(wimg + L.keys);

  // 2. keys in anchor order: class | ~score bits | anchor
  {
    int pos = wsum[warp];
    for (int a0 = a_lo; a0 < a_hi; a0 += 32) {
      const int a = a0 + lane;
      const bool f = a < a_hi && flag[a];
      const unsigned m = __ballot_sync(~0u, f);
      if (f) {
        const float* r = rec + (size_t)a * 6;
        const unsigned long long cls = (unsigned long long)(int)r[5];
        const unsigned long long sb = (~dm_f2bits(r[4])) & 0xffffffffull;
        keys[pos + __popc(m & lanemask_lt())] = (cls << 52) | (sb << 20) | (unsigned long long)a;
      }
      pos += __popc(m);
    }
  }
  __syncthreads();
  for (int i = n + tid; i < P; i += blockDim.x) keys[i] = ~0ull;
  __syncthreads();
  bitonic_sort(keys, P);

  // 3. class segments of the sorted list
  {
    int nseg_running = 0;
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
      const int i = i0 + tid;
      const int st = i < n && (i == 0 || (keys[i] >> 52) != (keys[i - 1] >> 52));
      int t;
      const int pos = nseg_running + block_scan(st, wsum, &t);
      if (st && pos < kMaxClasses) segs[pos] = i;
      nseg_running += t;
    }
    if (tid == 0) s_total = min(nseg_running, kMaxClasses);
    __syncthreads();
  }
  const int nseg = s_total;
  if (tid == 0) segs[nseg] = n;
  __syncthreads();

  // 4. greedy suppression per class, one warp per class, 32 candidates per step; the first
  // kKeptSmem kept boxes of the class live in shared memory, later ones in the workspace
  for (int sg = warp; sg < nseg; sg += blockDim.x >> 5) {
    const int s = segs[sg], e = segs[sg + 1];
    int nk = 0;
    for (int c0 = s; c0 < e; c0 += 32) {
      const int i = c0 + lane;
      const bool valid = i < e;
      float x1 = 0, y1 = 0, x2 = 0, y2 = 0, ar = 0;
      if (valid) {
        const float* r = rec + (size_t)(keys[i] & 0xfffffull) * 6;
        x1 = r[0]; y1 = r[1]; x2 = r[2]; y2 = r[3];
        ar = dm_area(x1, y1, x2, y2);
      }
      bool alive = valid;
      for (int t = 0; t < nk; t++) {
        if (!__any_sync(~0u, alive)) break;
        const float* kb = t < kKeptSmem ? kept_s[warp][t] : kept + (size_t)(s + t) * 5;
        if (alive && dm_iou_gt(kb[0], kb[1], kb[2], kb[3], kb[4], x1, y1, x2, y2, iou)) alive = false;
      }
      for (int l = 0; l < 32; l++) {
        const unsigned m = __ballot_sync(~0u, alive);
        const float bx1 = __shfl_sync(~0u, x1, l), by1 = __shfl_sync(~0u, y1, l);
        const float bx2 = __shfl_sync(~0u, x2, l), by2 = __shfl_sync(~0u, y2, l);
        const float bar = __shfl_sync(~0u, ar, l);
        if (((m >> l) & 1u) && lane > l && alive &&
            dm_iou_gt(bx1, by1, bx2, by2, bar, x1, y1, x2, y2, iou))
          alive = false;
      }
      const unsigned m = __ballot_sync(~0u, alive);
      if (alive) {
        const int t = nk + __popc(m & lanemask_lt());
        float* kb = t < kKeptSmem ? kept_s[warp][t] : kept + (size_t)(s + t) * 5;
        kb[0] = x1; kb[1] = y1; kb[2] = x2; kb[3] = y2; kb[4] = ar;
      }
      if (valid) surv[i] = alive ? 1 : 0;
      nk += __popc(m);
      __syncwarp();
    }
  }
  __syncthreads();

  // 5. survivors in (score desc, anchor asc) order, first max_out kept
  int ns = 0;
  for (int i = tid; i < n; i += blockDim.x) {
    const bool sv = surv[i] != 0;
    keys[i] = sv ? (keys[i] & ((1ull << 52) - 1)) : ~0ull;
    ns += sv;
  }
  int tot;
  block_scan(ns, wsum, &tot);
  const int nsurv = tot;
  bitonic_sort(keys, P);
  const int nout = min(nsurv, max_out);
  for (int i = tid; i < nout; i += blockDim.x) {
    const int a = (int)(keys[i] & 0xfffffull);
    const float* r = rec + (size_t)a * 6;
    float* o = outdets + ((size_t)img * max_out + i) * 6;
#pragma unroll
    for (int q = 0; q < 6; q++) o[q] = r[q];
    outidx[(size_t)img * max_out + i] = a;
  }
  if (tid == 0) {
    outcnt[img] = nout;
    rawcnt[img] = n;
  }
}

// ---------------- masks (engine/engine.cu:1129-1158) ----------------
struct DevCoefs {
  DView coef[4];
  int W[4], abase[4];
  int n;
};

__global__ void masks_kernel(DevCoefs cf, DView proto, int nm, float rx, float ry, int max_out,
                             const float* __restrict__ outdets, const int* __restrict__ outidx,
                             const int* __restrict__ outcnt, uint8_t* __restrict__ masks) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const int img = blockIdx.y, d = blockIdx.x;
  if (d >= outcnt[img]) return;
  __shared__ float co[64];
  const int a = outidx[(size_t)img * max_out + d];
  int li = 0;
  while (li + 1 < cf.n && a >= cf.abase[li + 1]) li++;
  const int rem = a - cf.abase[li];
  const int y = rem / cf.W[li], x = rem - y * cf.W[li];
  if ((int)threadIdx.x < nm)
    co[threadIdx.x] = __half2float(cf.coef[li].p[cf.coef[li].pix(img, y, x) + threadIdx.x]);
  __syncthreads();
  const float* det = outdets + ((size_t)img * max_out + d) * 6;
  const float bx1 = DM_MUL(det[0], rx), by1 = DM_MUL(det[1], ry);
  const float bx2 = DM_MUL(det[2], rx), by2 = DM_MUL(det[3], ry);
  const int Ph = proto.H, Pw = proto.W;
  uint8_t* out = masks + ((size_t)img * max_out + d) * Ph * Pw;
  for (int p = threadIdx.x; p < Ph * Pw; p += blockDim.x) {
    const int px = p % Pw, py = p / Pw;
    uint8_t m = 0;
    if ((float)px >= bx1 && (float)px < bx2 && (float)py >= by1 && (float)py < by2) {
      const __half* pp = proto.p + proto.pix(img, py, px);
      float acc = 0.f;
      for (int c = 0; c < nm; c += 8) {
        const uint4 v = *(const uint4*)(pp + c);
        const __half* h = (const __half*)&v;
#pragma unroll
        for (int j = 0; j < 8; j++) acc = DM_FMA(co[c + j], __half2float(h[j]), acc);
      }
      m = acc > 0.f;
    }
    out[p] = m;
  }
}

static int anchors_of(const YkLevel* lv, int n) {
  int A = 0;
  for (int i = 0; i < n; i++) A += lv[i].box.H * lv[i].box.W;
  return A;
}

}  // namespace yk

using namespace yk;

extern "C" {

int yk_letterbox(const uint8_t* bgr, int sh, int sw, const YkView* y, int slot,
                 float* scale_out, int* top_out, int* left_out, yk_stream_t st) {
  if (!bgr || sh < 1 || sw < 1 || !view_ok(y) || y->C != 3 || slot < 0 || slot >= y->batch)
    return YK_EINVAL;
  const float scale = std::min((float)y->H / sh, (float)y->W / sw);
  const int nh = (int)roundf(sh * scale), nw = (int)roundf(sw * scale);
  const int top = (y->H - nh) / 2, left = (y->W - nw) / 2;
  if (scale_out) *scale_out = scale;
  if (top_out) *top_out = top;
  if (left_out) *left_out = left;
  __half* dst = (__half*)y->ptr + y->coff + (size_t)slot * y->H * y->W * y->stride;
  const int npx = y->H * y->W;
  launch_k(letterbox_kernel, (npx + 255) / 256, 256, 0, (cudaStream_t)st, 
      bgr, sh, sw, dst, y->H, y->W, y->stride, scale, top, left, nh, nw);
  note_launch();
  return check_launch("letterbox");
}

size_t yk_post_workspace_bytes(int batch, int anchors) {
  return (size_t)batch * ws_layout(anchors).per_img;
}

int yk_decode(const YkLevel* levels, int nlevels, int batch, int nc, float conf,
              const YkPost* post, yk_stream_t st) {
  if (!levels || nlevels < 1 || nlevels > 4 || batch < 1 || nc < 1 || !post || !post->ws)
    return YK_EINVAL;
  DevLevels lv;
  int A = 0;
  for (int i = 0; i < nlevels; i++) {
    const YkLevel& l = levels[i];
    if (!view_vec8(&l.box) || !view_vec8(&l.cls) || l.box.C != 64 || l.cls.C < nc ||
        l.box.H != l.cls.H || l.box.W != l.cls.W || l.box.batch < batch || l.cls.batch < batch)
      return YK_EINVAL;
    lv.l[i] = {dview(l.box), dview(l.cls), l.box.H, l.box.W, l.stride, A};
    A += l.box.H * l.box.W;
  }
  lv.n = nlevels;
  lv.A = A;
  if (A >= (1 << 20)) return YK_EUNSUP;
  WsLayout L = ws_layout(A);
  if (post->ws_bytes < (size_t)batch * L.per_img) return YK_EINVAL;
  const long long total = (long long)batch * A;
  launch_k(decode_kernel, (unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)st, 
      lv, batch, nc, conf, (uint8_t*)post->ws, L);
  note_launch();
  return check_launch("decode");
}

int yk_nms(int batch, int anchors, float iou, int max_out, const YkPost* post, yk_stream_t st) {
  if (batch < 1 || anchors < 1 || anchors >= (1 << 20) || max_out < 1 || !post || !post->ws ||
      !post->outdets || !post->outidx || !post->outcnt || !post->rawcnt)
    return YK_EINVAL;
  WsLayout L = ws_layout(anchors);
  if (post->ws_bytes < (size_t)batch * L.per_img) return YK_EINVAL;
  const size_t smem = (size_t)std::min(pow2ge(std::max(anchors, 2)), kNmsSmemKeys) * 8;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(nms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kNmsSmemKeys * 8);
    attr = true;
  }
  launch_k(nms_kernel, batch, kNmsThreads, smem, (cudaStream_t)st, 
      anchors, iou, max_out, (uint8_t*)post->ws, L, post->outdets, post->outidx, post->outcnt,
      post->rawcnt);
  note_launch();
  return check_launch("nms");
}

int yk_masks(const YkLevel* levels, int nlevels, const YkView* proto, int in_h, int in_w,
             int max_out, const YkPost* post, uint8_t* masks, yk_stream_t st) {
  if (!levels || nlevels < 1 || nlevels > 4 || !view_vec8(proto) || proto->C > 64 || !post ||
      !masks || in_h < 1 || in_w < 1 || max_out < 1)
    return YK_EINVAL;
  DevCoefs cf;
  int A = 0;
  for (int i = 0; i < nlevels; i++) {
    if (!levels[i].coef.ptr || levels[i].coef.C != proto->C || !view_ok(&levels[i].coef))
      return YK_EINVAL;
    cf.coef[i] = dview(levels[i].coef);
    cf.W[i] = levels[i].coef.W;
    cf.abase[i] = A;
    A += levels[i].coef.H * levels[i].coef.W;
  }
  cf.n = nlevels;
  dim3 grid(max_out, proto->batch);
  launch_k(masks_kernel, grid, 256, 0, (cudaStream_t)st, 
      cf, dview(*proto), proto->C, (float)proto->W / in_w, (float)proto->H / in_h, max_out,
      post->outdets, post->outidx, post->outcnt, masks);
  note_launch();
  return check_launch("masks");
}


}  // extern "C"

// ---------------- decode + NMS without any allocation ----------------
// Some callers cannot allocate device memory: code running where cudaMalloc is off limits
// (a host with a fixed memory budget, a plugin whose host framework owns every allocation,
// a real-time loop that must never hit the allocator).  yk_decode_nms_static gives them the
// decode + NMS chain with its workspace in this fixed device array instead of a caller
// buffer.  Every GPU that loads the library holds it until the process exits.
namespace yk {
constexpr size_t kStaticPostBytes = (size_t)8 << 20;   // 8 MiB
static __device__ __align__(256) unsigned char g_static_post_ws[kStaticPostBytes];
}  // namespace yk

extern "C" int yk_decode_nms_static(const YkLevel* levels, int nlevels, int batch, int nc,
                                    float conf, float iou, int max_out, float* outdets,
                                    int* outidx, int* outcnt, int* rawcnt, yk_stream_t st) {
  using namespace yk;
  if (!levels || nlevels < 1 || nlevels > 4 || batch < 1) return YK_EINVAL;
  const int A = anchors_of(levels, nlevels);
  const size_t need = (size_t)batch * ws_layout(A).per_img;
  if (need > kStaticPostBytes) {
    snprintf(g_cuda_err, sizeof g_cuda_err,
             "yk_decode_nms_static: batch %d x %d anchors needs %zu bytes of scratch, more than "
             "the %zu-byte static array",
             batch, A, need, kStaticPostBytes);
    return YK_EINVAL;
  }
  // Host code cannot use g_static_post_ws directly (the name is a host-side stand-in, not a
  // device address): look up its address once per device, with that device current.
  static std::mutex mu;
  static void* addr[128] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return check_launch("static ws");
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_static_post_ws);
      if (e != cudaSuccess || !p) {
        snprintf(g_cuda_err, sizeof g_cuda_err, "yk_decode_nms_static: cudaGetSymbolAddress: %s",
                 cudaGetErrorString(e));
        return YK_ECUDA;
      }
      addr[dev] = p;
    }
    ws = addr[dev];
  }
  // No part of the scratch has to start at zero: decode writes every anchor's flag and the
  // NMS kernel writes each key / kept / survivor slot before reading it.
  YkPost post;
  post.ws = ws;
  post.ws_bytes = kStaticPostBytes;
  post.outdets = outdets;
  post.outidx = outidx;
  post.outcnt = outcnt;
  post.rawcnt = rawcnt;
  int r = yk_decode(levels, nlevels, batch, nc, conf, &post, st);
  if (r != YK_OK) return r;
  return yk_nms(batch, A, iou, max_out, &post, st);
}

