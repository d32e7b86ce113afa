// Bandwidth-bound kernels: first conv (Cin = 3), depthwise conv, SPPF max pools, nearest
// upsample, pixel shuffle, channel-slice copy and add, plus the yk_conv dispatcher.
// All activation accesses are 16-byte vectors of 8 channels where the view allows it
// (channel counts, offsets and strides are multiples of 8 in every exported graph).
#include <algorithm>
#include <atomic>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace yk {

static std::atomic<long long> g_launches{0};
static thread_local char g_cuda_err[256];

static bool dw_tiled_enabled() {
  static const bool on = [] {
    const char* e = getenv("YK_DW_ROWS");   // 1: the register-blocked row kernel instead
    return !(e && *e && *e != '0');
  }();
  return on;
}

bool bulk_store_enabled() {
  static const bool on = [] {
    const char* e = getenv("YK_NO_BULK_STORE");
    return !(e && *e && *e != '0');
  }();
  return on;
}

bool streams_enabled() {
  static const bool on = [] {
    const char* e = getenv("YK_NO_STREAMS");
    return !(e && *e && *e != '0');
  }();
  return on;
}

bool patch_enabled() {
  static const bool on = [] {
    const char* e = getenv("YK_NO_PATCH");
    return !(e && *e && *e != '0');
  }();
  return on;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("YK_NO_PDL");
    return !(e && *e && *e != '0');
  }();
  return on;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

cudaError_t ensure_smem_attr(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;   // (kernel, device) -> bytes set
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{kernel, dev}];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}
int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return YK_OK;
  snprintf(g_cuda_err, sizeof g_cuda_err, "%s: %s", what, cudaGetErrorString(e));
  return YK_ECUDA;
}

int conv_tc(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, cudaStream_t st);

static inline unsigned nblk(long long n, int tb) { return (unsigned)((n + tb - 1) / tb); }

// ---------------- first conv: Cin <= 4, dense, direct FMA ----------------
// Thread = one output pixel x 8 output channels; the block's 8-channel weight slice and bias
// live in shared memory.  Replaces k_conv0 (engine/engine.cu:487-532).
__global__ void conv_small_cin_kernel(DView x, DView y, const __half* __restrict__ w,
                                      const float* __restrict__ b, int Cin, int k, int s, int p,
                                      int act, long long npix) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ float wsm[];   // [8][k*k*Cin] then bias[8]
  const int KK = k * k * Cin;
  const int co0 = blockIdx.y * 8;
  for (int i = threadIdx.x; i < 8 * KK; i += blockDim.x) wsm[i] = __half2float(w[(size_t)co0 * KK + i]);
  if (threadIdx.x < 8) wsm[8 * KK + threadIdx.x] = b[co0 + threadIdx.x];
  __syncthreads();
  long long pix = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= npix) return;
  const int HW = y.H * y.W;
  const int img = (int)(pix / HW), rem = (int)(pix - (long long)img * HW);
  const int oy = rem / y.W, ox = rem - oy * y.W;
  float acc[8];
#pragma unroll
  for (int c = 0; c < 8; c++) acc[c] = wsm[8 * KK + c];
  for (int ky = 0; ky < k; ky++) {
    const int iy = oy * s - p + ky;
    if (iy < 0 || iy >= x.H) continue;
    for (int kx = 0; kx < k; kx++) {
      const int ix = ox * s - p + kx;
      if (ix < 0 || ix >= x.W) continue;
      const __half* xp = x.p + x.pix(img, iy, ix);
      for (int ci = 0; ci < Cin; ci++) {
        const float v = __half2float(xp[ci]);
        const int kidx = (ky * k + kx) * Cin + ci;
#pragma unroll
        for (int c = 0; c < 8; c++) acc[c] = fmaf(v, wsm[c * KK + kidx], acc[c]);
      }
    }
  }
  uint4 o;
  __half2* oh = (__half2*)&o;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    float a0 = acc[2 * q], a1 = acc[2 * q + 1];
    if (act == 1) { a0 = silu(a0); a1 = silu(a1); }
    oh[q] = __floats2half2_rn(a0, a1);
  }
  *(uint4*)(y.p + (size_t)pix * y.stride + co0) = o;
}

// First conv of every YOLO (k = 3, Cin = 3, stride s, pad p <= 2) on the warp-level tensor
// cores.  The layer is bound by its output writes (Cout channels per pixel from 27 taps).
// Persistent blocks walk output rows; each row's 3 input rows come into a double-buffered
// shared window by 16-byte cp.async (packed stride-3 rows; element loads otherwise), the
// borders staying zero.  Each warp builds the m16n8k16 A fragments of 16 output pixels
// straight from the window (K = 27 taps padded to 32), multiplies by the filter held in
// B-fragment registers for the whole kernel (NF = Cout / 8 fragments), and writes bias + SiLU
// through a padded [16][Cout] staging block as whole 16-byte channel groups per pixel.
// Replaces k_conv0 (engine/engine.cu:487-532).
template <int NF>
__global__ void __launch_bounds__(128) conv_stem_mma_kernel(DView x, DView y,
                                                            const __half* __restrict__ w,
                                                            const float* __restrict__ b, int s,
                                                            int p, int act, int pitch, int vec,
                                                            int rows) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  constexpr int Cout = NF * 8, kStgRow = Cout + 8;
  // [2 buffers][3 rows][pitch]: element (input column ix >= -p, channel c) of a row sits at
  // 8 + 3*ix + c; then the per-warp staging blocks
  extern __shared__ __align__(16) __half stem_sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __half* stg = stem_sm + 6 * pitch + warp * 16 * kStgRow;
  for (int i = tid; i < 6 * pitch / 8; i += 128) ((uint4*)stem_sm)[i] = make_uint4(0, 0, 0, 0);
  // this lane's K indices per k-step: 2t, 2t+1, 2t+8, 2t+9 (+16); tap-major (ky, kx, ci) order
  const int g = lane >> 2, t = lane & 3;
  int koff[2][4];
#pragma unroll
  for (int ks = 0; ks < 2; ks++)
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int k = 16 * ks + 2 * t + (j & 1) + (j >> 1) * 8;
      // taps 27..31 pad K to 32 with zero weights: their A element may be any finite window
      // value, so they read tap 26 and the gathers need no bounds select
      const int kc = k < 27 ? k : 26;
      const int tc = kc / 3, cc = kc - tc * 3, kyc = tc / 3, kxc = tc - kyc * 3;
      koff[ks][j] = kyc * pitch + 8 + (kxc - p) * 3 + cc;
    }
  uint32_t bf[2][NF][2];
  float bias2[NF][2];
#pragma unroll
  for (int f = 0; f < NF; f++) {
    const int n = 8 * f + g;
#pragma unroll
    for (int ks = 0; ks < 2; ks++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int k0 = 16 * ks + 2 * t + 8 * h;
        const float lo = k0 < 27 ? __half2float(w[n * 27 + k0]) : 0.f;
        const float hi = k0 + 1 < 27 ? __half2float(w[n * 27 + k0 + 1]) : 0.f;
        bf[ks][f][h] = pack_half2(lo, hi);
      }
    bias2[f][0] = b[8 * f + 2 * t];
    bias2[f][1] = b[8 * f + 2 * t + 1];
  }
  __syncthreads();   // zeroed window before the first fill
  auto stage = [&](int r, __half* buf) {
    const int img = r / y.H, oy = r - img * y.H;
    if (vec) {
      const int cpr = x.W * 3 / 8;
      for (int i = tid; i < 3 * cpr; i += 128) {
        const int ky = i / cpr, c = i - ky * cpr, iy = oy * s - p + ky;
        const bool ok = iy >= 0 && iy < x.H;
        const __half* src = ok ? x.p + ((size_t)img * x.H + iy) * x.W * 3 + c * 8 : x.p;
        cp_async16(smem_u32(buf + ky * pitch + 8 + c * 8), src, ok ? 16u : 0u);
      }
    } else {
      for (int i = tid; i < 3 * x.W * 3; i += 128) {
        const int ky = i / (x.W * 3), rem = i - ky * x.W * 3, col = rem / 3, ch = rem - col * 3;
        const int iy = oy * s - p + ky;
        buf[ky * pitch + 8 + rem] = (iy >= 0 && iy < x.H) ? x.p[x.pix(img, iy, col) + ch]
                                                          : __float2half(0.f);
      }
    }
  };
  int r = blockIdx.x;
  if (r < rows) stage(r, stem_sm);
  cp_async_commit();
  const int ntile = (y.W + 15) / 16;
  for (int it = 0; r < rows; r += gridDim.x, it++) {
    const __half* cur = stem_sm + (it & 1) * 3 * pitch;
    if (r + (int)gridDim.x < rows) stage(r + gridDim.x, stem_sm + ((it + 1) & 1) * 3 * pitch);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int img = r / y.H, oy = r - img * y.H;
    for (int mt = warp; mt < ntile; mt += 4) {
      const int ox0 = mt * 16;
      const int oxa = min(ox0 + g, y.W - 1), oxb = min(ox0 + g + 8, y.W - 1);
      const __half* pa = cur + oxa * s * 3;
      const __half* pb = cur + oxb * s * 3;
      float acc[NF][4];
#pragma unroll
      for (int f = 0; f < NF; f++) acc[f][0] = acc[f][1] = acc[f][2] = acc[f][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 2; ks++) {
        __half va[4], vb[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          va[j] = pa[koff[ks][j]];
          vb[j] = pb[koff[ks][j]];
        }
        uint32_t a[4];
        a[0] = (uint32_t)__half_as_ushort(va[0]) | ((uint32_t)__half_as_ushort(va[1]) << 16);
        a[1] = (uint32_t)__half_as_ushort(vb[0]) | ((uint32_t)__half_as_ushort(vb[1]) << 16);
        a[2] = (uint32_t)__half_as_ushort(va[2]) | ((uint32_t)__half_as_ushort(va[3]) << 16);
        a[3] = (uint32_t)__half_as_ushort(vb[2]) | ((uint32_t)__half_as_ushort(vb[3]) << 16);
#pragma unroll
        for (int f = 0; f < NF; f++) mma16816(acc[f], a, bf[ks][f][0], bf[ks][f][1]);
      }
#pragma unroll
      for (int f = 0; f < NF; f++) {
        const float2 bb = make_float2(bias2[f][0], bias2[f][1]);
        const __half2 h01 = bias_act2(make_float2(acc[f][0], acc[f][1]), bb, act);
        const __half2 h23 = bias_act2(make_float2(acc[f][2], acc[f][3]), bb, act);
        *(__half2*)(stg + g * kStgRow + 8 * f + 2 * t) = h01;
        *(__half2*)(stg + (g + 8) * kStgRow + 8 * f + 2 * t) = h23;
      }
      __syncwarp();
      __half* yrow = y.p + y.pix(img, oy, ox0);
      for (int q = lane; q < 16 * NF; q += 32) {
        const int px = q / NF, f = q - px * NF;
        if (ox0 + px < y.W)
          *(uint4*)(yrow + px * y.stride + 8 * f) = *(const uint4*)(stg + px * kStgRow + 8 * f);
      }
      __syncwarp();
    }
    __syncthreads();   // the buffer is refilled two rows later
  }
  cp_async_wait<0>();
}

// ---------------- im2col for thin inputs (stem) ----------------
// Thread = one output pixel: gathers its k*k*C taps (C <= 8) and writes the padded row as
// 16-byte stores.
__global__ void im2col_kernel(DView x, DView col, int k, int s, int p, long long npix) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const long long pix = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= npix) return;
  const int HW = col.H * col.W;
  const int img = (int)(pix / HW), rem = (int)(pix - (long long)img * HW);
  const int oy = rem / col.W, ox = rem - oy * col.W;
  __half* o = col.p + (size_t)pix * col.stride;
  __half buf[8];
  int n = 0, base = 0;
  const __half zero = __float2half(0.f);
  for (int ky = 0; ky < k; ky++) {
    const int iy = oy * s - p + ky;
    for (int kx = 0; kx < k; kx++) {
      const int ix = ox * s - p + kx;
      const bool ok = iy >= 0 && iy < x.H && ix >= 0 && ix < x.W;
      const __half* xp = x.p + x.pix(img, ok ? iy : 0, ok ? ix : 0);
      for (int c = 0; c < x.C; c++) {
        buf[n++] = ok ? xp[c] : zero;
        if (n == 8) { *(uint4*)(o + base) = *(uint4*)buf; base += 8; n = 0; }
      }
    }
  }
  while (base < col.C) {
    while (n < 8) buf[n++] = zero;
    *(uint4*)(o + base) = *(uint4*)buf;
    base += 8;
    n = 0;
  }
}

// ---------------- depthwise conv ----------------
// Thread = one output pixel x 8 channels, 16-byte activation loads.  The block first stages
// the OHWI [C][k][k][1] weights transposed to [k*k][C] in shared memory, so each tap's 8
// channel weights are one 16-byte shared load.  Replaces k_dwconv8 (engine/engine.cu:535-580,
// which repacks the weights on the host at load time), including its fused residual.
__global__ void dwconv_kernel(DView x, DView y, DView r, const __half* __restrict__ w,
                              const float* __restrict__ b, int k, int s, int p, int act,
                              long long total) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ __align__(16) __half wt[];   // [k*k][C]
  const int C = y.C, KK = k * k;
  for (int i = threadIdx.x; i < C * KK; i += blockDim.x) {
    const int c = i / KK, t = i - c * KK;
    wt[t * C + c] = w[i];
  }
  __syncthreads();
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int cg = C >> 3;
  if (idx >= total) return;
  const int g = (int)(idx % cg);
  const long long pix = idx / cg;
  const int c = g << 3;
  const int HW = y.H * y.W;
  const int img = (int)(pix / HW), rem = (int)(pix - (long long)img * HW);
  const int oy = rem / y.W, ox = rem - oy * y.W;
  float acc[8];
  {
    const float4 b0 = *(const float4*)(b + c), b1 = *(const float4*)(b + c + 4);
    acc[0] = b0.x; acc[1] = b0.y; acc[2] = b0.z; acc[3] = b0.w;
    acc[4] = b1.x; acc[5] = b1.y; acc[6] = b1.z; acc[7] = b1.w;
  }
  for (int ky = 0; ky < k; ky++) {
    const int iy = oy * s - p + ky;
    if (iy < 0 || iy >= x.H) continue;
    for (int kx = 0; kx < k; kx++) {
      const int ix = ox * s - p + kx;
      if (ix < 0 || ix >= x.W) continue;
      const uint4 xv = *(const uint4*)(x.p + x.pix(img, iy, ix) + c);
      const uint4 wv = *(const uint4*)(wt + (ky * k + kx) * C + c);
      const __half2* xh = (const __half2*)&xv;
      const __half2* wh = (const __half2*)&wv;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 fx = __half22float2(xh[q]), fw = __half22float2(wh[q]);
        acc[2 * q] = fmaf(fx.x, fw.x, acc[2 * q]);
        acc[2 * q + 1] = fmaf(fx.y, fw.y, acc[2 * q + 1]);
      }
    }
  }
  float rv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (r.p) {
    const uint4 v = *(const uint4*)(r.p + (size_t)pix * r.stride + c);
    const __half* h = (const __half*)&v;
#pragma unroll
    for (int q = 0; q < 8; q++) rv[q] = __half2float(h[q]);
  }
  uint4 o;
  __half2* oh = (__half2*)&o;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    float a0 = acc[2 * q], a1 = acc[2 * q + 1];
    if (act == 1) { a0 = silu(a0); a1 = silu(a1); }
    oh[q] = __floats2half2_rn(a0 + rv[2 * q], a1 + rv[2 * q + 1]);
  }
  *(uint4*)(y.p + (size_t)pix * y.stride + c) = o;
}

// 3x3 stride-1 depthwise conv on shared-memory tiles.  A tile is 64 channels x 8 output rows
// x 16 output columns; its 10 x 18 input window comes into shared memory by 16-byte cp.async
// (zero outside the image), so every input element is read from L2 about 1.4 times instead
// of once per tap.  Persistent blocks, each with a fixed channel tile (the grid is a multiple
// of the channel-tile count, so the [9][64] fp16 filter is staged once), double-buffer the
// windows: the next tile's loads are in flight while the current one is computed.  Thread =
// 8 channels x 2 output rows x 4 output columns, so each loaded input row feeds two output
// rows; mixed-precision FMAs (fp16 inputs, fp32 accumulators), taps accumulated in
// (ky, kx) order like the other depthwise
// kernels.
constexpr int kDwTY = 8, kDwTX = 16, kDwCh = 64, kDwThreads = 128;
constexpr int kDwIW = kDwTX + 2, kDwIH = kDwTY + 2;
constexpr int kDwWin = kDwIH * kDwIW * kDwCh;   // halves per window buffer
#ifndef YK_DW_MINB
#define YK_DW_MINB 4   // resident blocks per SM the register budget is sized for
#endif
__global__ void __launch_bounds__(kDwThreads, YK_DW_MINB) dwconv3t_kernel(DView x, DView y, DView r,
                                                                 const __half* __restrict__ w,
                                                                 const float* __restrict__ b,
                                                                 int act, int tiles_c,
                                                                 int tiles_x, int tiles_y,
                                                                 int ntiles) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ __align__(16) __half dw_smem[];   // [2][window] + fp32 [9][64] filter
  __half* wsm = dw_smem + 2 * kDwWin;
  const int tid = threadIdx.x;
  const int tc = blockIdx.x % tiles_c;                  // fixed: gridDim.x % tiles_c == 0
  const int c0 = tc * kDwCh;
  const int cvalid = min(kDwCh, y.C - c0);
  for (int i = tid; i < 9 * kDwCh; i += kDwThreads) {
    const int t = i / kDwCh, c = i - t * kDwCh;
    wsm[i] = c < cvalid ? w[(size_t)(c0 + c) * 9 + t] : __float2half(0.f);
  }
  const int per_img = tiles_y * tiles_x * tiles_c;
  // staging: thread tid copies channel chunk tid % 8 of window positions tid / 8 + 16 k (the
  // chunk is the same for all its copies, as 128 threads are a multiple of 8); addresses are
  // 32-bit offsets from the tile's image (the host checks an image fits in 2^31 elements)
  const int sch = tid & 7;
  const bool sch_ok = sch * 8 < cvalid;
  auto stage = [&](int t, __half* buf) {
    const int img = t / per_img;
    const int q = (t - img * per_img) / tiles_c;
    const int ty = q / tiles_x, tx = q - ty * tiles_x;
    const int oy0 = ty * kDwTY - 1, ox0 = tx * kDwTX - 1;
    const __half* ibase = x.p + (size_t)img * x.H * x.W * x.stride + c0 + sch * 8;
#pragma unroll 4
    for (int pos = tid >> 3; pos < kDwIH * kDwIW; pos += kDwThreads / 8) {
      const int rr = pos / kDwIW, cc = pos - rr * kDwIW;
      const int iy = oy0 + rr, ix = ox0 + cc;
      const bool ok = sch_ok && (unsigned)iy < (unsigned)x.H && (unsigned)ix < (unsigned)x.W;
      const __half* src = ok ? ibase + (iy * x.W + ix) * x.stride : x.p;
      cp_async16(smem_u32(buf + pos * kDwCh + sch * 8), src, ok ? 16u : 0u);
    }
  };
  const int cg = tid & 7, q16 = tid >> 3;                // q16: 4 row pairs x 4 column quads
  const int r0 = (q16 >> 2) * 2, xq = (q16 & 3) * 4;
  const int c = c0 + cg * 8;
  const bool cok = cg * 8 < cvalid;
  float2 bias[4] = {};
  if (cok) {
    const float4 b0 = *(const float4*)(b + c), b1 = *(const float4*)(b + c + 4);
    bias[0] = make_float2(b0.x, b0.y); bias[1] = make_float2(b0.z, b0.w);
    bias[2] = make_float2(b1.x, b1.y); bias[3] = make_float2(b1.z, b1.w);
  }
  int t = blockIdx.x;
  if (t < ntiles) stage(t, dw_smem);
  cp_async_commit();
  for (int it = 0; t < ntiles; t += gridDim.x, it++) {
    __half* cur = dw_smem + (it & 1) * kDwWin;
    if (t + (int)gridDim.x < ntiles) stage(t + gridDim.x, dw_smem + ((it + 1) & 1) * kDwWin);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int img = t / per_img;
    const int q = (t - img * per_img) / tiles_c;
    const int ty = q / tiles_x, tx = q - ty * tiles_x;
    const int oy = ty * kDwTY + r0, ox0 = tx * kDwTX + xq;
    if (cok && oy < y.H) {
      float acc[2][4][8];   // [output row][pixel][channel]; tap (0, 0) starts from the bias
      // input rows r0 .. r0+3 of the window; input row ir feeds output row h with ky = ir - h;
      // fp16 inputs and weights go straight into mixed-precision FMAs
#pragma unroll
      for (int ir = 0; ir < 4; ir++) {
        const __half* trow = cur + ((r0 + ir) * kDwIW + xq) * kDwCh + cg * 8;
        uint4 xr[6];
#pragma unroll
        for (int u = 0; u < 6; u++) xr[u] = *(const uint4*)(trow + u * kDwCh);
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int ky = ir - h;
          if (ky < 0 || ky > 2) continue;
#pragma unroll
          for (int kx = 0; kx < 3; kx++) {
            const uint4 wv = *(const uint4*)(wsm + (ky * 3 + kx) * kDwCh + cg * 8);
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
              const uint32_t xx[4] = {xr[j + kx].x, xr[j + kx].y, xr[j + kx].z, xr[j + kx].w};
#pragma unroll
              for (int e = 0; e < 4; e++) {
                if (ky == 0 && kx == 0)
                  fma2_f16f32_from(acc[h][j][2 * e], acc[h][j][2 * e + 1], xx[e], ww[e],
                                   bias[e].x, bias[e].y);
                else
                  fma2_f16f32(acc[h][j][2 * e], acc[h][j][2 * e + 1], xx[e], ww[e]);
              }
            }
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        if (oy + h >= y.H) break;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int ox = ox0 + j;
          if (ox >= y.W) break;
          const size_t pix = ((size_t)img * y.H + oy + h) * y.W + ox;
          float2 rv[4] = {};
          if (r.p) {
            const uint4 v = *(const uint4*)(r.p + pix * r.stride + c);
            const __half2* hr = (const __half2*)&v;
#pragma unroll
            for (int e = 0; e < 4; e++) rv[e] = __half22float2(hr[e]);
          }
          uint4 o;
          __half2* oh = (__half2*)&o;
#pragma unroll
          for (int e = 0; e < 4; e++) {
            float a0 = acc[h][j][2 * e], a1 = acc[h][j][2 * e + 1];
            if (act == 1) { a0 = silu_fast(a0); a1 = silu_fast(a1); }
            oh[e] = __floats2half2_rn(a0 + rv[e].x, a1 + rv[e].y);
          }
          *(uint4*)(y.p + pix * y.stride + c) = o;
        }
      }
    }
    __syncthreads();   // the buffer is refilled two tiles later
  }
  cp_async_wait<0>();
}

// 3x3 depthwise conv, register-blocked: thread = 8 channels x 4 consecutive output pixels
// of one row.  The block stages the filter transposed to [9][C] in shared memory and each
// filter row's 24 weights of a thread's channels are loaded to registers per row, each input column of
// the 3 x (3*S + 1 ... ) window is loaded once (16 bytes) and feeds every output it touches.
// Index arithmetic is 32-bit (I = unsigned) whenever the element count allows it.
template <int S, typename I>
__global__ void __launch_bounds__(256) dwconv3_kernel(DView x, DView y, DView r,
                                                      const __half* __restrict__ w,
                                                      const float* __restrict__ b, int act,
                                                      int batch) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  constexpr int PX = 4, NIN = (PX - 1) * S + 3;
  extern __shared__ __align__(16) __half dw_wsm[];   // weights transposed to [9][C]
  for (int i = threadIdx.x; i < y.C * 9; i += blockDim.x) {
    const int t = i / y.C, ch = i - t * y.C;
    dw_wsm[i] = w[ch * 9 + t];
  }
  __syncthreads();
  const int cg = y.C >> 3, nxb = (y.W + PX - 1) / PX;
  const I total = (I)batch * y.H * nxb * cg;
  for (I idx = (I)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (I)gridDim.x * blockDim.x) {
  const int g = (int)(idx % cg);
  I rr = idx / cg;
  const int xb = (int)(rr % nxb);
  rr /= nxb;
  const int oy = (int)(rr % y.H), img = (int)(rr / y.H);
  const int c = g << 3, ox0 = xb * PX;
  float acc[PX][8];
  {
    const float4 b0 = *(const float4*)(b + c), b1 = *(const float4*)(b + c + 4);
#pragma unroll
    for (int j = 0; j < PX; j++) {
      acc[j][0] = b0.x; acc[j][1] = b0.y; acc[j][2] = b0.z; acc[j][3] = b0.w;
      acc[j][4] = b1.x; acc[j][5] = b1.y; acc[j][6] = b1.z; acc[j][7] = b1.w;
    }
  }
  const int ix0 = ox0 * S - 1;
#pragma unroll
  for (int ky = 0; ky < 3; ky++) {
    const int iy = oy * S - 1 + ky;
    if (iy < 0 || iy >= x.H) continue;
    const __half* xrow = x.p + x.pix(img, iy, 0) + c;
    float wr[3][8];   // this filter row's weights for the thread's 8 channels
#pragma unroll
    for (int kx = 0; kx < 3; kx++) {
      const uint4 v = *(const uint4*)(dw_wsm + (ky * 3 + kx) * y.C + c);
      const __half2* hw = (const __half2*)&v;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __half22float2(hw[q]);
        wr[kx][2 * q] = f.x;
        wr[kx][2 * q + 1] = f.y;
      }
    }
    uint4 xin[NIN];   // issue the whole row of loads first: one latency per filter row
#pragma unroll
    for (int u = 0; u < NIN; u++) {
      const int ix = ix0 + u;
      xin[u] = (ix >= 0 && ix < x.W) ? *(const uint4*)(xrow + (size_t)ix * x.stride)
                                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < NIN; u++) {
      const __half2* xh = (const __half2*)&xin[u];
      float xf[8];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __half22float2(xh[q]);
        xf[2 * q] = f.x;
        xf[2 * q + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < PX; j++) {
        const int kx = u - j * S;   // compile-time after unrolling
        if (kx < 0 || kx > 2) continue;
#pragma unroll
        for (int q = 0; q < 8; q++) acc[j][q] = fmaf(xf[q], wr[kx][q], acc[j][q]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < PX; j++) {
    const int ox = ox0 + j;
    if (ox >= y.W) break;
    const size_t pix = ((size_t)img * y.H + oy) * y.W + ox;
    float rv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (r.p) {
      const uint4 v = *(const uint4*)(r.p + pix * r.stride + c);
      const __half2* h = (const __half2*)&v;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float2 f = __half22float2(h[q]);
        rv[2 * q] = f.x;
        rv[2 * q + 1] = f.y;
      }
    }
    uint4 o;
    __half2* oh = (__half2*)&o;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      float a0 = acc[j][2 * q], a1 = acc[j][2 * q + 1];
      if (act == 1) { a0 = silu(a0); a1 = silu(a1); }
      oh[q] = __floats2half2_rn(a0 + rv[2 * q], a1 + rv[2 * q + 1]);
    }
    *(uint4*)(y.p + pix * y.stride + c) = o;
  }
  }
}

// ---------------- SPPF max pools ----------------
__device__ __forceinline__ void hmax8(uint4& m, const uint4 v) {
  __half2* a = (__half2*)&m;
  const __half2* b = (const __half2*)&v;
#pragma unroll
  for (int i = 0; i < 4; i++) a[i] = __hmax2(a[i], b[i]);
}

// nr outputs: output j (j < nr) is the max over the (5+4j) x (5+4j) window clipped to the
// image, i.e. j+1 chained 5x5/s1/p2 pools (max pooling composes: pool5(pool5(x)) = pool9(x)
// with -inf padding).  Replaces k_maxpool5 (engine/engine.cu:672-695).
template <typename I>
__global__ void maxpool_kernel(DView x, DView y1, DView y2, DView y3, int nr, I total) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const I idx = (I)blockIdx.x * blockDim.x + threadIdx.x;
  const int cg = x.C >> 3;
  if (idx >= total) return;
  const int g = (int)(idx % cg);
  const I pix = idx / cg;
  const int c = g << 3;
  const int HW = x.H * x.W;
  const int img = (int)(pix / HW), rem = (int)(pix - (I)img * HW);
  const int y0 = rem / x.W, x0 = rem - y0 * x.W;
  const uint4 ninf = make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
  uint4 m1 = ninf, m2 = ninf, m3 = ninf;
  const int R = 2 + 2 * (nr - 1);
  for (int dy = -R; dy <= R; dy++) {
    const int iy = y0 + dy;
    if (iy < 0 || iy >= x.H) continue;
    const int ady = dy < 0 ? -dy : dy;
    for (int dx = -R; dx <= R; dx++) {
      const int ix = x0 + dx;
      if (ix < 0 || ix >= x.W) continue;
      const int adx = dx < 0 ? -dx : dx;
      const int d = ady > adx ? ady : adx;
      const uint4 v = *(const uint4*)(x.p + x.pix(img, iy, ix) + c);
      if (d <= 2) hmax8(m1, v);
      if (d <= 4) hmax8(m2, v);
      hmax8(m3, v);
    }
  }
  *(uint4*)(y1.p + (size_t)pix * y1.stride + c) = m1;
  if (nr > 1) *(uint4*)(y2.p + (size_t)pix * y2.stride + c) = m2;
  if (nr > 2) *(uint4*)(y3.p + (size_t)pix * y3.stride + c) = m3;
}

// SPPF chain y1 = pool5(x), y2 = pool5(y1), y3 = pool5(y2) for images small enough to keep
// a channel block's whole plane in shared memory (the P5 level: 20x20 at 640).  Block = one
// (image, CB-channel block): the plane comes in once, each 5x5 max is separable (max over
// 5 columns, then over 5 rows, borders clipped like -inf padding) and runs shared-memory to
// shared-memory, and the three results go out once each.  Max is exact in fp16, so this
// equals the direct 5x5 / 9x9 / 13x13 windows of maxpool_kernel.
template <int CB>
__global__ void __launch_bounds__(256) pool5x3_plane_kernel(DView x, DView y1, DView y2,
                                                            DView y3, int ncb) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ __align__(16) uint4 pl_sm[];   // two planes [H*W][CB/8] chunks
  constexpr int kG = CB / 8;
  const int img = blockIdx.x / ncb, c0 = (blockIdx.x - img * ncb) * CB;
  const int H = x.H, W = x.W, n = H * W * kG;
  uint4* A = pl_sm;
  uint4* Bp = pl_sm + n;
  for (int i0 = threadIdx.x; i0 < n; i0 += 256 * 8) {   // all loads in flight, then stores
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * 256, px = i / kG, g = i - px * kG;
      if (i < n) v[u] = *(const uint4*)(x.p + (size_t)(img * H * W + px) * x.stride + c0 + g * 8);
    }
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (i0 + u * 256 < n) A[i0 + u * 256] = v[u];
  }
  __syncthreads();
  const DView* outs[3] = {&y1, &y2, &y3};
  const int wk = W * kG;                 // 16-byte chunks per plane row
  if (wk <= 256) {
    // each thread keeps one (column, channel group) and walks rows rstep apart: no
    // per-element division, and neighbours along a row are chunk offsets of +-kG
    const int rstep = 256 / wk;
    const int col = threadIdx.x % wk, r0 = threadIdx.x / wk;
    const int xx = col / kG;
    const bool act = r0 < rstep;
#pragma unroll 1
    for (int pass = 0; pass < 3; pass++) {
      if (act)
        for (int yy = r0; yy < H; yy += rstep) {   // max over 5 columns: A -> B
          const int i = yy * wk + col;
          uint4 m = A[i];
#pragma unroll
          for (int dx = -2; dx <= 2; dx++)
            if (dx != 0 && xx + dx >= 0 && xx + dx < W) hmax8(m, A[i + dx * kG]);
          Bp[i] = m;
        }
      __syncthreads();
      const DView& yo = *outs[pass];
      __half* orow = yo.p + (size_t)img * H * W * yo.stride + c0 + (col - xx * kG) * 8;
      if (act)
        for (int yy = r0; yy < H; yy += rstep) {   // max over 5 rows: B -> A, and out
          const int i = yy * wk + col;
          uint4 m = Bp[i];
#pragma unroll
          for (int dy = -2; dy <= 2; dy++)
            if (dy != 0 && yy + dy >= 0 && yy + dy < H) hmax8(m, Bp[i + dy * wk]);
          A[i] = m;
          *(uint4*)(orow + (size_t)(yy * W + xx) * yo.stride) = m;
        }
      __syncthreads();
    }
    return;
  }
#pragma unroll 1
  for (int pass = 0; pass < 3; pass++) {
    for (int i = threadIdx.x; i < n; i += 256) {   // max over 5 columns: A -> B
      const int px = i / kG, g = i - px * kG;
      const int yy = px / W, xx = px - yy * W;
      uint4 m = A[i];
      for (int dx = -2; dx <= 2; dx++) {
        const int ix = xx + dx;
        if (dx != 0 && ix >= 0 && ix < W) hmax8(m, A[(yy * W + ix) * kG + g]);
      }
      Bp[i] = m;
    }
    __syncthreads();
    const DView& yo = *outs[pass];
    for (int i = threadIdx.x; i < n; i += 256) {   // max over 5 rows: B -> A, and out
      const int px = i / kG, g = i - px * kG;
      const int yy = px / W, xx = px - yy * W;
      uint4 m = Bp[i];
      for (int dy = -2; dy <= 2; dy++) {
        const int iy = yy + dy;
        if (dy != 0 && iy >= 0 && iy < H) hmax8(m, Bp[(iy * W + xx) * kG + g]);
      }
      A[i] = m;
      *(uint4*)(yo.p + (size_t)(img * H * W + px) * yo.stride + c0 + g * 8) = m;
    }
    __syncthreads();
  }
}

// ---------------- data movement ----------------
// mode 0: nearest 2x upsample (engine/engine.cu:697-708); mode 1: pixel shuffle r=2 from
// quadrant blocks (engine/engine.cu:713-725); mode 2: channel-slice copy (727-732).
// Thread = one output pixel x 8 channels.
// One block row per output image row (blockIdx.y strides over batch x H), threads over
// (x, 8-channel group): no 64-bit or per-thread image/row divisions.
__global__ void move8_kernel(DView x, DView y, int mode, int rows) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const int cg = y.C >> 3;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= y.W * cg) return;
  const int g = i % cg, ox = i / cg;
  const int c = g << 3;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int img = row / y.H, oy = row - img * y.H;
    const __half* src;
    if (mode == 0) src = x.p + x.pix(img, oy >> 1, ox >> 1) + c;
    else if (mode == 1) src = x.p + x.pix(img, oy >> 1, ox >> 1) + (((oy & 1) << 1) | (ox & 1)) * y.C + c;
    else src = x.p + x.pix(img, oy, ox) + c;
    *(uint4*)(y.p + y.pix(img, oy, ox) + c) = *(const uint4*)src;
  }
}

__global__ void copy_scalar_kernel(DView x, DView y, long long total) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int c = (int)(idx % y.C);
  const long long pix = idx / y.C;
  y.p[(size_t)pix * y.stride + c] = x.p[(size_t)pix * x.stride + c];
}

template <typename I>
__global__ void add8_kernel(DView a, DView b, DView y, I total) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const I idx = (I)blockIdx.x * blockDim.x + threadIdx.x;
  const int cg = y.C >> 3;
  if (idx >= total) return;
  const int c = (int)(idx % cg) << 3;
  const I pix = idx / cg;
  const uint4 va = *(const uint4*)(a.p + (size_t)pix * a.stride + c);
  const uint4 vb = *(const uint4*)(b.p + (size_t)pix * b.stride + c);
  const __half2* ha = (const __half2*)&va;
  const __half2* hb = (const __half2*)&vb;
  uint4 o;
  __half2* ho = (__half2*)&o;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float2 fa = __half22float2(ha[i]), fb = __half22float2(hb[i]);
    ho[i] = __floats2half2_rn(fa.x + fb.x, fa.y + fb.y);
  }
  *(uint4*)(y.p + (size_t)pix * y.stride + c) = o;
}

static bool same_shape(const YkView* a, const YkView* b) {
  return a->batch == b->batch && a->H == b->H && a->W == b->W && a->C == b->C;
}

}  // namespace yk

using namespace yk;

extern "C" {

long long yk_launch_count(void) { return g_launches.load(); }
const char* yk_last_cuda_error(void) { return g_cuda_err; }

int yk_test_inject(int withhold, unsigned long long wait_ns) {
  const unsigned long long w = wait_ns ? wait_ns : kWaitNs;
  const int h = withhold ? 1 : 0;
  if (cudaMemcpyToSymbol(g_wait_ns, &w, sizeof w) != cudaSuccess ||
      cudaMemcpyToSymbol(g_test_withhold, &h, sizeof h) != cudaSuccess)
    return check_launch("yk_test_inject");
  return YK_OK;
}

int yk_fetch_device_error(void) {
  int v = 0, z = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof v) != cudaSuccess) return YK_ECUDA;
  if (v) cudaMemcpyToSymbol(g_device_error, &z, sizeof z);
  return v;
}

int yk_conv(const YkView* x, const YkView* y, const YkView* res, const YkConv* p,
            yk_stream_t st_) {
  cudaStream_t st = (cudaStream_t)st_;
  if (!p || !view_ok(x) || !view_ok(y) || !p->weight || !p->bias) return YK_EINVAL;
  if (x->batch != y->batch || x->C != p->Cin || y->C != p->Cout || p->k < 1 || p->s < 1) return YK_EINVAL;
  const int Ho = (x->H + 2 * p->p - p->k) / p->s + 1, Wo = (x->W + 2 * p->p - p->k) / p->s + 1;
  if (Ho != y->H || Wo != y->W) return YK_EINVAL;
  if (res && (!view_vec8(res) || !same_shape(res, y))) return YK_EINVAL;
  if (!view_vec8(y) || ((uintptr_t)p->bias & 15) || ((uintptr_t)p->weight & 15)) return YK_EINVAL;
  const long long npix = (long long)y->batch * y->H * y->W;
  if (p->groups == 1 && p->Cin % 8 == 0) {
    if (!view_vec8(x)) return YK_EINVAL;
    return conv_tc(x, y, res, p, st);
  }
  if (p->groups == 1 && p->Cin == 3 && p->k == 3 && !res && p->Cout % 8 == 0 &&
      p->Cout <= 96 && x->stride >= 3 && x->C == 3) {
    // a window row holds input columns [-p, max(W, (Wo-1)*s + 3 - p)) after an 8-half lead
    const int cols = std::max(x->W + 2 * p->p, (y->W - 1) * p->s + 3);
    const int pitch = (8 + 3 * cols + 8 + 7) & ~7;
    const size_t smem = (size_t)6 * pitch * 2 + 4 * 16 * (p->Cout + 8) * 2;
    const long long rows = (long long)y->batch * y->H;
    if (rows >= (1LL << 31) || smem > 200 * 1024 || p->p > 2) return YK_EUNSUP;
    static int nsm = 0;
    if (!nsm) {
      int dev = 0;
      cudaGetDevice(&dev);
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
      if (nsm <= 0) nsm = 148;
    }
#ifndef YK_STEM_BPS
#define YK_STEM_BPS 5   // persistent blocks per SM (96 registers x 128 threads: five fit)
#endif
    const unsigned grid = (unsigned)std::min<long long>(rows, (long long)nsm * YK_STEM_BPS);
    const int vec = x->stride == 3 && (x->W * 3) % 8 == 0 &&
                    (((uintptr_t)x->ptr + (size_t)x->coff * 2) & 15) == 0;
    void (*kern)(DView, DView, const __half*, const float*, int, int, int, int, int, int) = nullptr;
    switch (p->Cout / 8) {
      case 2: kern = conv_stem_mma_kernel<2>; break;
      case 4: kern = conv_stem_mma_kernel<4>; break;
      case 6: kern = conv_stem_mma_kernel<6>; break;
      case 8: kern = conv_stem_mma_kernel<8>; break;
      case 10: kern = conv_stem_mma_kernel<10>; break;
      case 12: kern = conv_stem_mma_kernel<12>; break;
      default: break;
    }
    if (kern) {
      if (smem > 48 * 1024 && smem_attr(kern, (int)smem) != cudaSuccess)
        return check_launch("conv_stem attr");
      launch_k(kern, grid, 128, smem, (cudaStream_t)st, dview(*x), dview(*y),
               (const __half*)p->weight, p->bias, p->s, p->p, p->act, pitch, vec, (int)rows);
      note_launch();
      return check_launch("conv_stem");
    }
  }
  if (p->groups == 1 && p->Cin <= 4) {
    if (res || p->Cout % 8) return YK_EUNSUP;
    const int KK = p->k * p->k * p->Cin;
    dim3 grid(nblk(npix, 256), p->Cout / 8);
    launch_k(conv_small_cin_kernel, grid, 256, (8 * KK + 8) * sizeof(float), (cudaStream_t)st, 
        dview(*x), dview(*y), (const __half*)p->weight, p->bias, p->Cin, p->k, p->s, p->p,
        p->act, npix);
    note_launch();
    return check_launch("conv_small_cin");
  }
  if (p->groups == p->Cin && p->Cin == p->Cout && p->Cin % 8 == 0) {
    if (!view_vec8(x)) return YK_EINVAL;
    DView r = res ? dview(*res) : DView{nullptr, 0, 0, 0, 0};
    const long long total = npix * (p->Cout / 8);
    // tiled path: 32-bit offsets within one image (larger images take the direct kernel)
    if (p->k == 3 && p->p == 1 && p->s == 1 && dw_tiled_enabled() &&
        (long long)x->H * x->W * x->stride < (1LL << 31)) {
      const int tcn = (p->Cout + kDwCh - 1) / kDwCh, txn = (y->W + kDwTX - 1) / kDwTX;
      const int tyn = (y->H + kDwTY - 1) / kDwTY;
      const long long nt = (long long)y->batch * tyn * txn * tcn;
      if (nt >= (1LL << 31)) return YK_EUNSUP;
      static int nsm = 0;
      if (!nsm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
        if (nsm <= 0) nsm = 148;
      }
      // persistent grid, a multiple of the channel-tile count (each block keeps its filter)
      long long grid = std::min<long long>(nt, (long long)nsm * YK_DW_MINB);
      grid = std::max<long long>(tcn, grid / tcn * tcn);
      const size_t smem = (2 * (size_t)kDwWin + 9 * kDwCh) * sizeof(__half);
      if (smem_attr(dwconv3t_kernel, (int)smem) != cudaSuccess) return check_launch("dwconv3t attr");
      launch_k(dwconv3t_kernel, (unsigned)grid, kDwThreads, smem, (cudaStream_t)st, dview(*x),
               dview(*y), r, (const __half*)p->weight, p->bias, p->act, tcn, txn, tyn, (int)nt);
      note_launch();
      return check_launch("dwconv3t");
    }
    if (p->k == 3 && p->p == 1 && (p->s == 1 || p->s == 2)) {
      const long long t3 = (long long)y->batch * y->H * ((y->W + 3) / 4) * (p->Cout / 8);
      const unsigned nb = (unsigned)std::min<long long>(nblk(t3, 256), 148 * 8);  // grid-stride
      const size_t wsmem = (size_t)p->Cout * 9 * sizeof(__half);
      if (wsmem > 48 * 1024) return YK_EUNSUP;
      const __half* wp = (const __half*)p->weight;
      if (t3 < (1LL << 31)) {
        if (p->s == 1) launch_k(dwconv3_kernel<1, unsigned>, nb, 256, wsmem, (cudaStream_t)st, dview(*x), dview(*y), r, wp, p->bias, p->act, y->batch);
        else launch_k(dwconv3_kernel<2, unsigned>, nb, 256, wsmem, (cudaStream_t)st, dview(*x), dview(*y), r, wp, p->bias, p->act, y->batch);
      } else {
        if (p->s == 1) launch_k(dwconv3_kernel<1, long long>, nb, 256, wsmem, (cudaStream_t)st, dview(*x), dview(*y), r, wp, p->bias, p->act, y->batch);
        else launch_k(dwconv3_kernel<2, long long>, nb, 256, wsmem, (cudaStream_t)st, dview(*x), dview(*y), r, wp, p->bias, p->act, y->batch);
      }
      note_launch();
      return check_launch("dwconv3");
    }
    const size_t smem = (size_t)p->Cout * p->k * p->k * sizeof(__half);
    if (smem > 96 * 1024) return YK_EUNSUP;
    if (smem_attr(dwconv_kernel, 96 * 1024) != cudaSuccess) return check_launch("dwconv attr");
    launch_k(dwconv_kernel, nblk(total, 256), 256, smem, (cudaStream_t)st, dview(*x), dview(*y), r,
                                                    (const __half*)p->weight, p->bias, p->k,
                                                    p->s, p->p, p->act, total);
    note_launch();
    return check_launch("dwconv");
  }
  return YK_EUNSUP;
}

int yk_im2col(const YkView* x, const YkView* col, int k, int s, int p, yk_stream_t st) {
  if (!view_ok(x) || !view_vec8(col) || x->C > 8 || k < 1 || s < 1 || p < 0 ||
      x->batch != col->batch || col->C < k * k * x->C ||
      (x->H + 2 * p - k) / s + 1 != col->H || (x->W + 2 * p - k) / s + 1 != col->W)
    return YK_EINVAL;
  const long long npix = (long long)col->batch * col->H * col->W;
  launch_k(im2col_kernel, nblk(npix, 256), 256, 0, (cudaStream_t)st, dview(*x), dview(*col), k, s, p, npix);
  note_launch();
  return check_launch("im2col");
}

int yk_maxpool5(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_vec8(x) || !view_vec8(y) || !same_shape(x, y)) return YK_EINVAL;
  const long long total = (long long)x->batch * x->H * x->W * (x->C / 8);
  DView Y = dview(*y);
  if (total < (1LL << 31)) launch_k(maxpool_kernel<unsigned>, nblk(total, 256), 256, 0, (cudaStream_t)st, dview(*x), Y, Y, Y, 1, (unsigned)total);
  else launch_k(maxpool_kernel<long long>, nblk(total, 256), 256, 0, (cudaStream_t)st, dview(*x), Y, Y, Y, 1, total);
  note_launch();
  return check_launch("maxpool5");
}

int yk_maxpool5x3(const YkView* x, const YkView* y1, const YkView* y2, const YkView* y3,
                  yk_stream_t st) {
  if (!view_vec8(x) || !view_vec8(y1) || !view_vec8(y2) || !view_vec8(y3) ||
      !same_shape(x, y1) || !same_shape(x, y2) || !same_shape(x, y3))
    return YK_EINVAL;
  const long long total = (long long)x->batch * x->H * x->W * (x->C / 8);
  // whole planes in shared memory: two of H*W*CB halves within 200 KB
  const size_t plane = (size_t)x->H * x->W * 2;
  // 64-channel blocks only when 32-channel ones would not fill the GPU
  const bool many32 = (long long)x->batch * (x->C / 32) >= 148;
  const int cbk = (x->C % 32 == 0 && 2 * plane * 32 <= 200 * 1024 && (many32 || x->C % 64))
                      ? 32
                  : (x->C % 64 == 0 && 2 * plane * 64 <= 200 * 1024) ? 64
                  : (x->C % 32 == 0 && 2 * plane * 32 <= 200 * 1024) ? 32 : 0;
  // a handful of planes (small batches): 8-channel planes, 4x-8x more blocks
  const int cbp = cbk && (long long)x->batch * (x->C / 32) < 148 ? 8 : cbk;
  if (cbp && (long long)x->batch * (x->C / cbp) < (1LL << 31)) {
    const int ncb = x->C / cbp;
    const size_t smem = 2 * plane * cbp;
    auto kern = cbp == 64 ? pool5x3_plane_kernel<64>
                : cbp == 32 ? pool5x3_plane_kernel<32> : pool5x3_plane_kernel<8>;
    if (smem > 48 * 1024 && smem_attr(kern, (int)smem) != cudaSuccess)
      return check_launch("pool5x3 attr");
    launch_k(kern, (unsigned)(x->batch * ncb), 256, smem, (cudaStream_t)st, dview(*x),
             dview(*y1), dview(*y2), dview(*y3), ncb);
  } else if (total < (1LL << 31))
    launch_k(maxpool_kernel<unsigned>, nblk(total, 256), 256, 0, (cudaStream_t)st, 
        dview(*x), dview(*y1), dview(*y2), dview(*y3), 3, (unsigned)total);
  else
    launch_k(maxpool_kernel<long long>, nblk(total, 256), 256, 0, (cudaStream_t)st, 
        dview(*x), dview(*y1), dview(*y2), dview(*y3), 3, total);
  note_launch();
  return check_launch("maxpool5x3");
}

// Nearest 2x upsample: thread = one input pixel x 8 channels, one 16-byte load, four stores.
__global__ void upsample2_kernel(DView x, DView y, int rows) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const int cg = x.C >> 3;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= x.W * cg) return;
  const int c = (i % cg) << 3, ix = i / cg;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int img = row / x.H, iy = row - img * x.H;
    const uint4 v = *(const uint4*)(x.p + x.pix(img, iy, ix) + c);
    __half* o = y.p + y.pix(img, 2 * iy, 2 * ix) + c;
    const size_t rs = (size_t)y.W * y.stride;
    *(uint4*)o = v;
    *(uint4*)(o + y.stride) = v;
    *(uint4*)(o + rs) = v;
    *(uint4*)(o + rs + y.stride) = v;
  }
}

static int move8(const YkView* x, const YkView* y, int mode, yk_stream_t st) {
  const int rows = y->batch * y->H;
  dim3 grid(nblk((long long)y->W * (y->C / 8), 256), rows < 65535 ? rows : 65535);
  launch_k(move8_kernel, grid, 256, 0, (cudaStream_t)st, dview(*x), dview(*y), mode, rows);
  note_launch();
  return check_launch("move8");
}

int yk_upsample2(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_vec8(x) || !view_vec8(y) || x->batch != y->batch || x->C != y->C ||
      y->H != 2 * x->H || y->W != 2 * x->W)
    return YK_EINVAL;
  const int rows = x->batch * x->H;
  dim3 grid(nblk((long long)x->W * (x->C / 8), 256), rows < 65535 ? rows : 65535);
  launch_k(upsample2_kernel, grid, 256, 0, (cudaStream_t)st, dview(*x), dview(*y), rows);
  note_launch();
  return check_launch("upsample2");
}

int yk_ps2(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_vec8(x) || !view_vec8(y) || x->batch != y->batch || x->C != 4 * y->C ||
      y->H != 2 * x->H || y->W != 2 * x->W)
    return YK_EINVAL;
  return move8(x, y, 1, st);
}

int yk_copyc(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_ok(x) || !view_ok(y) || !same_shape(x, y)) return YK_EINVAL;
  if (view_vec8(x) && view_vec8(y)) return move8(x, y, 2, st);
  const long long total = (long long)y->batch * y->H * y->W * y->C;
  launch_k(copy_scalar_kernel, nblk(total, 256), 256, 0, (cudaStream_t)st, dview(*x), dview(*y), total);
  note_launch();
  return check_launch("copyc");
}

int yk_add(const YkView* a, const YkView* b, const YkView* y, yk_stream_t st) {
  if (!view_vec8(a) || !view_vec8(b) || !view_vec8(y) || !same_shape(a, b) || !same_shape(a, y))
    return YK_EINVAL;
  const long long total = (long long)y->batch * y->H * y->W * (y->C / 8);
  if (total < (1LL << 31))
    launch_k(add8_kernel<unsigned>, nblk(total, 256), 256, 0, (cudaStream_t)st, dview(*a), dview(*b), dview(*y), (unsigned)total);
  else
    launch_k(add8_kernel<long long>, nblk(total, 256), 256, 0, (cudaStream_t)st, dview(*a), dview(*b), dview(*y), total);
  note_launch();
  return check_launch("add");
}

}  // extern "C"
