// PSA attention, fused: out[n, h*hd + c] = sum_j softmax_j(q_n . k_j / sqrt(kd)) v_j[c]
// over the N = H*W tokens of one image, per head.  Replaces the reference's per-image,
// per-head chain QK^T GEMM -> row softmax -> V transpose -> PV GEMM with an fp16 N x N
// score matrix in HBM (engine/engine.cu:1363-1397, 583-608) and its scalar fallback
// (785-842): nothing N x N is materialised, every batch image runs in the same launch.
//
// Block = (128/KS queries, head, image), 128 threads.  K and V of the head are staged once
// in shared memory as fp16 (N*(kd+hd)*2 bytes: 77 KB at N=400, 196 KB at N=1024).  KS
// adjacent lanes share one query and walk interleaved key subsets (key j goes to lane
// j % KS), each with its own online (max-rescaled) softmax in fp32; the KS partial states
// are merged with warp shuffles.  KS is picked so the grid covers the SMs even at batch 1.
#include "common.cuh"

namespace yk {

template <int KD, int HD, int KS>
__global__ void __launch_bounds__(128) attn_kernel(DView qkv, DView y, int N) {
  extern __shared__ __align__(16) __half kv[];   // [N][KD] keys then [N][HD] values
  __half* ks = kv;
  __half* vs = kv + (size_t)N * KD;
  const int h = blockIdx.y, img = blockIdx.z;
  const int per = 2 * KD + HD;
  const __half* base = qkv.p + (size_t)img * N * qkv.stride + h * per;
  constexpr int KC = KD / 8, VC = HD / 8;
  for (int i = threadIdx.x; i < N * (KC + VC); i += blockDim.x) {
    const int j = i / (KC + VC), c = i - j * (KC + VC);
    const uint4 v = *(const uint4*)(base + (size_t)j * qkv.stride + KD + c * 8);  // k, v adjacent
    if (c < KC) *(uint4*)(ks + (size_t)j * KD + c * 8) = v;
    else *(uint4*)(vs + (size_t)j * HD + (c - KC) * 8) = v;
  }
  __syncthreads();
  const int sub = threadIdx.x % KS;
  const int n = blockIdx.x * (128 / KS) + threadIdx.x / KS;
  const bool valid = n < N;
  const float scale = rsqrtf((float)KD);
  float q[KD];
  {
    const __half* qp = base + (size_t)(valid ? n : 0) * qkv.stride;
#pragma unroll
    for (int c = 0; c < KC; c++) {
      const uint4 v = *(const uint4*)(qp + c * 8);
      const __half2* hv = (const __half2*)&v;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float2 f = __half22float2(hv[e]);
        q[c * 8 + 2 * e] = f.x * scale;
        q[c * 8 + 2 * e + 1] = f.y * scale;
      }
    }
  }
  float acc[HD];
#pragma unroll
  for (int c = 0; c < HD; c++) acc[c] = 0.f;
  float mrun = -INFINITY, lrun = 0.f;
  constexpr int CH = 16;   // keys per rescale step (per lane)
  for (int j0 = sub; j0 < N; j0 += CH * KS) {
    float s[CH];
    float cmax = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < CH; jj++) {
      const int j = j0 + jj * KS;
      float d = -INFINITY;
      if (j < N) {
        const __half2* kp = (const __half2*)(ks + (size_t)j * KD);
        d = 0.f;
#pragma unroll
        for (int e = 0; e < KD / 2; e++) {
          const float2 f = __half22float2(kp[e]);
          d = fmaf(q[2 * e], f.x, d);
          d = fmaf(q[2 * e + 1], f.y, d);
        }
      }
      s[jj] = d;
      cmax = fmaxf(cmax, d);
    }
    const float mnew = fmaxf(mrun, cmax);
    const float corr = __expf(mrun - mnew);
    lrun *= corr;
#pragma unroll
    for (int c = 0; c < HD; c++) acc[c] *= corr;
#pragma unroll
    for (int jj = 0; jj < CH; jj++) {
      const int j = j0 + jj * KS;
      if (j < N) {
        const float pj = __expf(s[jj] - mnew);
        lrun += pj;
        const __half2* vp = (const __half2*)(vs + (size_t)j * HD);
#pragma unroll
        for (int e = 0; e < HD / 2; e++) {
          const float2 f = __half22float2(vp[e]);
          acc[2 * e] = fmaf(pj, f.x, acc[2 * e]);
          acc[2 * e + 1] = fmaf(pj, f.y, acc[2 * e + 1]);
        }
      }
    }
    mrun = mnew;
  }
  // merge the KS partial softmax states of this query (lanes sharing n are adjacent)
#pragma unroll
  for (int o = 1; o < KS; o <<= 1) {
    const float m2 = __shfl_xor_sync(~0u, mrun, o);
    const float l2 = __shfl_xor_sync(~0u, lrun, o);
    const float mm = fmaxf(mrun, m2);
    const float c1 = mrun == -INFINITY ? 0.f : __expf(mrun - mm);
    const float c2 = m2 == -INFINITY ? 0.f : __expf(m2 - mm);
    lrun = lrun * c1 + l2 * c2;
#pragma unroll
    for (int c = 0; c < HD; c++) {
      const float a2 = __shfl_xor_sync(~0u, acc[c], o);
      acc[c] = acc[c] * c1 + a2 * c2;
    }
    mrun = mm;
  }
  if (!valid) return;
  const float inv = 1.f / lrun;
  __half* yp = y.p + ((size_t)img * N + n) * y.stride + h * HD;
  // lane `sub` writes the 16-byte chunks sub, sub+KS, ... of the HD outputs
#pragma unroll
  for (int c = 0; c < HD / 8; c++) {
    if (c % KS != sub) continue;
    uint4 o;
    __half2* oh = (__half2*)&o;
#pragma unroll
    for (int e = 0; e < 4; e++)
      oh[e] = __floats2half2_rn(acc[c * 8 + 2 * e] * inv, acc[c * 8 + 2 * e + 1] * inv);
    *(uint4*)(yp + c * 8) = o;
  }
}

template <int KS>
static int launch_attn(const YkView* qkv, const YkView* y, int heads, int N, size_t smem,
                       cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(attn_kernel<32, 64, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         227 * 1024);
    attr = true;
  }
  dim3 grid((N + 128 / KS - 1) / (128 / KS), heads, qkv->batch);
  attn_kernel<32, 64, KS><<<grid, 128, smem, st>>>(dview(*qkv), dview(*y), N);
  note_launch();
  return check_launch("attn");
}

}  // namespace yk

using namespace yk;

extern "C" int yk_attn(const YkView* qkv, const YkView* y, int heads, int kd, int hd,
                       yk_stream_t st) {
  if (!view_vec8(qkv) || !view_vec8(y) || heads < 1 || qkv->batch != y->batch ||
      qkv->H != y->H || qkv->W != y->W || qkv->C != heads * (2 * kd + hd) || y->C != heads * hd)
    return YK_EINVAL;
  if (kd != 32 || hd != 64) return YK_EUNSUP;
  const int N = qkv->H * qkv->W;
  const size_t smem = (size_t)N * (kd + hd) * sizeof(__half);
  if (smem > 227 * 1024) return YK_EUNSUP;
  // enough blocks to cover the SMs: split keys further when batch x heads is small
  const long long blocks1 = (long long)qkv->batch * heads * ((N + 127) / 128);
  if (blocks1 >= 4 * 148) return launch_attn<1>(qkv, y, heads, N, smem, (cudaStream_t)st);
  if (blocks1 * 4 >= 148) return launch_attn<4>(qkv, y, heads, N, smem, (cudaStream_t)st);
  return launch_attn<8>(qkv, y, heads, N, smem, (cudaStream_t)st);
}
