// Classification head and preprocessing (task "classify").
//
//   gap_kernel          global average pool [B][H][W][C] -> [B][1][1][C], fp32 sums
//                       (reference k_gap, engine/engine.cu:735-744; one thread per image and
//                       8-channel group, 16-byte loads, pixels summed in order)
//   softmax_ch_kernel   channel softmax of [B][1][1][C] (reference k_softmax_ch,
//                       engine/engine.cu:746-785): one block per image, fp32 max and sum of
//                       exp(x - max), fp16 out; not in place
//   cls_resize_kernel   torchvision classify preprocessing of a BGR u8 frame into an input
//                       slot: shortest edge resized to S with the antialiased triangle filter
//                       (support widened by the scale on downscale), centre crop S x S, RGB,
//                       /255 (reference k_preprocess_cls + clsGeom, engine/engine.cu:1000-1046).
//                       Every float step is an explicitly rounded intrinsic, so the result
//                       is bit-identical to a C restatement compiled without contraction.
#include "common.cuh"

namespace yk {

__global__ void gap_kernel(DView x, DView y, int HW, int C8, int B) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * C8) return;
  const int img = idx / C8, c8 = idx - img * C8;
  const __half* src = x.p + (size_t)img * HW * x.stride + c8 * 8;
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int p = 0; p < HW; p++) {
    const uint4 v = *(const uint4*)(src + (size_t)p * x.stride);
    const __half2* h = (const __half2*)&v;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float2 f = __half22float2(h[e]);
      s[2 * e] += f.x;
      s[2 * e + 1] += f.y;
    }
  }
  uint4 o;
  __half2* oh = (__half2*)&o;
  const float n = (float)HW;
#pragma unroll
  for (int e = 0; e < 4; e++) oh[e] = __floats2half2_rn(s[2 * e] / n, s[2 * e + 1] / n);
  *(uint4*)(y.p + (size_t)img * y.stride + c8 * 8) = o;
}

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  for (int o = 16; o > 0; o >>= 1) {
    const float u = __shfl_xor_sync(~0u, v, o);
    v = is_max ? fmaxf(v, u) : v + u;
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < nw ? red[threadIdx.x] : (is_max ? -INFINITY : 0.f);
    for (int o = 16; o > 0; o >>= 1) {
      const float u = __shfl_xor_sync(~0u, t, o);
      t = is_max ? fmaxf(t, u) : t + u;
    }
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(256) softmax_ch_kernel(DView x, DView y, int C) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[33];
  const __half* src = x.p + (size_t)blockIdx.x * x.stride;
  __half* dst = y.p + (size_t)blockIdx.x * y.stride;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < C; c += blockDim.x) m = fmaxf(m, __half2float(src[c]));
  m = block_reduce(m, red, true);
  float s = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) s += expf(__half2float(src[c]) - m);
  s = block_reduce(s, red, false);
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    dst[c] = __float2half(expf(__half2float(src[c]) - m) / s);
}

// triangle-filter weight of source index i for an output centred at `centre` (support sup)
__device__ __forceinline__ float tri_w(int i, float centre, float sup) {
  const float d = fabsf(__fsub_rn(__fadd_rn((float)i, 0.5f), centre));
  return fmaxf(0.f, __fsub_rn(1.f, __fdiv_rn(d, sup)));
}

// one thread per output pixel of the S x S crop; (rh, rw) resized size, (top, left) crop
__global__ void cls_resize_kernel(const uint8_t* __restrict__ src, int sh, int sw,
                                  __half* __restrict__ dst, int S, int stride, int rh, int rw,
                                  int top, int left) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= S * S) return;
  const int oy = idx / S, ox = idx - oy * S;
  const float scy = __fdiv_rn((float)sh, (float)rh), scx = __fdiv_rn((float)sw, (float)rw);
  const float supy = fmaxf(scy, 1.f), supx = fmaxf(scx, 1.f);
  const float cy = __fmul_rn(__fadd_rn((float)(oy + top), 0.5f), scy);
  const float cx = __fmul_rn(__fadd_rn((float)(ox + left), 0.5f), scx);
  const int y0 = max(0, (int)__fadd_rn(__fsub_rn(cy, supy), 0.5f));
  const int y1 = min(sh, (int)__fadd_rn(__fadd_rn(cy, supy), 0.5f));
  const int x0 = max(0, (int)__fadd_rn(__fsub_rn(cx, supx), 0.5f));
  const int x1 = min(sw, (int)__fadd_rn(__fadd_rn(cx, supx), 0.5f));
  float wys = 0.f, wxs = 0.f;
  for (int i = y0; i < y1; i++) wys = __fadd_rn(wys, tri_w(i, cy, supy));
  for (int j = x0; j < x1; j++) wxs = __fadd_rn(wxs, tri_w(j, cx, supx));
  float b = 0.f, g = 0.f, r = 0.f;
  for (int i = y0; i < y1; i++) {
    const float wy = tri_w(i, cy, supy);
    const uint8_t* row = src + (size_t)i * sw * 3;
    for (int j = x0; j < x1; j++) {
      const float w = __fmul_rn(wy, tri_w(j, cx, supx));
      const uint8_t* p = row + (size_t)j * 3;
      b = __fadd_rn(b, __fmul_rn(w, (float)p[0]));
      g = __fadd_rn(g, __fmul_rn(w, (float)p[1]));
      r = __fadd_rn(r, __fmul_rn(w, (float)p[2]));
    }
  }
  const float inv = __fdiv_rn(1.f, __fmul_rn(__fmul_rn(wys, wxs), 255.f));
  __half* o = dst + (size_t)idx * stride;
  o[0] = __float2half_rn(__fmul_rn(r, inv));
  o[1] = __float2half_rn(__fmul_rn(g, inv));
  o[2] = __float2half_rn(__fmul_rn(b, inv));
}

}  // namespace yk

using namespace yk;

extern "C" int yk_gap(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_vec8(x) || !view_vec8(y) || x->batch != y->batch || y->H != 1 || y->W != 1 ||
      x->C != y->C || x->H < 1 || x->W < 1)
    return YK_EINVAL;
  const int C8 = x->C / 8, n = x->batch * C8;
  launch_k(gap_kernel, (n + 127) / 128, 128, 0, (cudaStream_t)st, dview(*x), dview(*y),
           x->H * x->W, C8, x->batch);
  note_launch();
  return check_launch("gap");
}

extern "C" int yk_softmax(const YkView* x, const YkView* y, yk_stream_t st) {
  if (!view_ok(x) || !view_ok(y) || x->batch != y->batch || x->H != 1 || x->W != 1 ||
      y->H != 1 || y->W != 1 || x->C != y->C || x->C < 1)
    return YK_EINVAL;
  launch_k(softmax_ch_kernel, x->batch, 256, 0, (cudaStream_t)st, dview(*x), dview(*y), x->C);
  note_launch();
  return check_launch("softmax");
}

extern "C" int yk_preprocess_cls(const uint8_t* bgr, int sh, int sw, const YkView* y, int slot,
                                 int* geom_out, yk_stream_t st) {
  if (!bgr || sh < 1 || sw < 1 || !view_ok(y) || y->C != 3 || y->H != y->W || slot < 0 ||
      slot >= y->batch)
    return YK_EINVAL;
  // torchvision Resize(S) of the shortest edge: the long edge is S * long / short truncated;
  // CenterCrop offsets round half to even (Python round)
  const long S = y->H;
  long rh, rw;
  if (sw <= sh) { rw = S; rh = S * sh / sw; }
  else { rh = S; rw = S * sw / sh; }
  auto half_even = [](long d) { return d / 2 + ((d & 1) && ((d / 2) & 1)); };
  const int top = (int)half_even(rh - S), left = (int)half_even(rw - S);
  if (geom_out) { geom_out[0] = (int)rh; geom_out[1] = (int)rw; geom_out[2] = top; geom_out[3] = left; }
  __half* dst = (__half*)y->ptr + y->coff + (size_t)slot * y->H * y->W * y->stride;
  const int npx = y->H * y->W;
  launch_k(cls_resize_kernel, (npx + 127) / 128, 128, 0, (cudaStream_t)st, bgr, sh, sw, dst,
           (int)S, y->stride, (int)rh, (int)rw, top, left);
  note_launch();
  return check_launch("preprocess_cls");
}
