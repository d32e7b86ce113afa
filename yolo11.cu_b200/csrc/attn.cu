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
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
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
  if (smem_attr(attn_kernel<32, 64, KS>, 227 * 1024) != cudaSuccess)
    return check_launch("attn attr");
  dim3 grid((N + 128 / KS - 1) / (128 / KS), heads, qkv->batch);
  launch_k(attn_kernel<32, 64, KS>, grid, 128, smem, (cudaStream_t)st, dview(*qkv), dview(*y), N);
  note_launch();
  return check_launch("attn");
}


// ---------------- tensor-core path (kd = 32, hd = 64) ----------------
// Flash-style: a warp owns 16 queries; keys stream through shared memory in chunks of 192
// (copied by cp.async, zero past the last key; K rows padded to 40 halves, V rows to 72, so fragment loads are bank-conflict free).
// Per 16-key block: S = Q K^T with four m16n8k16 MMAs (fp32 accumulate), online softmax in
// registers (row max / sum shared by the 4 lanes of a row through shuffles), then the fp16
// probabilities are reused in place as the A operand of O += P V (eight MMAs, V fragments by
// ldmatrix.trans).  The FLOPs are ~0.2 % of the network, so the warp-level MMA is enough.

constexpr int kAttnChunk = 192, kKs = 40, kVs = 72;

__global__ void __launch_bounds__(128) attn_mma_kernel(DView qkv, DView y, int N, float scale) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  __shared__ __align__(16) __half Ks[kAttnChunk * kKs];
  __shared__ __align__(16) __half Vs[kAttnChunk * kVs];
  const int h = blockIdx.y, img = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __half* base = qkv.p + (size_t)img * N * qkv.stride + h * 128;   // per head: q32 k32 v64
  const int q0 = blockIdx.x * 64 + warp * 16;
  // Q fragments (2 K-steps of 16 over kd = 32), rows beyond N are zero
  uint32_t qa[2][4];
  {
    const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
    for (int ks = 0; ks < 2; ks++) {
      const int c = ks * 16 + 2 * t;
      qa[ks][0] = r0 < N ? *(const uint32_t*)(base + (size_t)r0 * qkv.stride + c) : 0u;
      qa[ks][1] = r1 < N ? *(const uint32_t*)(base + (size_t)r1 * qkv.stride + c) : 0u;
      qa[ks][2] = r0 < N ? *(const uint32_t*)(base + (size_t)r0 * qkv.stride + c + 8) : 0u;
      qa[ks][3] = r1 < N ? *(const uint32_t*)(base + (size_t)r1 * qkv.stride + c + 8) : 0u;
    }
  }
  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows g and g+8
  for (int c0 = 0; c0 < N; c0 += kAttnChunk) {
    const int cn = min(kAttnChunk, N - c0);
    __syncthreads();
    const int cn16 = (cn + 15) & ~15;   // rows past the last key are zero (P = 0 there)
    // 4 K + 8 V 16-byte chunks per key, all of the block's copies in flight at once
    for (int i = threadIdx.x; i < cn16 * 12; i += 128) {
      const int j = i / 12, cc = i - j * 12;
      const bool ok = j < cn;
      const __half* src = ok ? base + (size_t)(c0 + j) * qkv.stride + 32 + cc * 8 : base;
      const uint32_t dst = cc < 4 ? smem_u32(Ks + j * kKs + cc * 8)
                                  : smem_u32(Vs + j * kVs + (cc - 4) * 8);
      cp_async16(dst, src, ok ? 16u : 0u);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int kb = 0; kb < cn; kb += 16) {
      // S = Q K^T for 16 keys: two n-tiles of 8 keys
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; nt++) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
        const int key = kb + nt * 8 + g;
#pragma unroll
        for (int ks = 0; ks < 2; ks++) {
          const __half* kp = Ks + key * kKs + ks * 16 + 2 * t;
          mma16816(sc[nt], qa[ks], *(const uint32_t*)kp, *(const uint32_t*)(kp + 8));
        }
      }
      // scale, mask keys past the end, online softmax per row
      float mx0 = m0, mx1 = m1;
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const bool ok = kb + nt * 8 + 2 * t + e < cn;
          sc[nt][e] = ok ? sc[nt][e] * scale : -INFINITY;
          sc[nt][2 + e] = ok ? sc[nt][2 + e] * scale : -INFINITY;
          mx0 = fmaxf(mx0, sc[nt][e]);
          mx1 = fmaxf(mx1, sc[nt][2 + e]);
        }
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(~0u, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(~0u, mx1, off));
      }
      const float cor0 = __expf(m0 - mx0), cor1 = __expf(m1 - mx1);
      m0 = mx0;
      m1 = mx1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          sc[nt][e] = __expf(sc[nt][e] - mx0);
          sc[nt][2 + e] = __expf(sc[nt][2 + e] - mx1);
          ps0 += sc[nt][e];
          ps1 += sc[nt][2 + e];
        }
      l0 = l0 * cor0 + ps0;   // per-lane partial sums; the row total is reduced at the end
      l1 = l1 * cor1 + ps1;
#pragma unroll
      for (int n = 0; n < 8; n++) {
        o[n][0] *= cor0; o[n][1] *= cor0;
        o[n][2] *= cor1; o[n][3] *= cor1;
      }
      // O += P V: P (16 q x 16 keys) as the A operand, V via ldmatrix.trans
      uint32_t pa[4] = {pack_half2(sc[0][0], sc[0][1]), pack_half2(sc[0][2], sc[0][3]),
                        pack_half2(sc[1][0], sc[1][1]), pack_half2(sc[1][2], sc[1][3])};
#pragma unroll
      for (int np = 0; np < 4; np++) {   // pairs of 8-column n-tiles
        const __half* vp = Vs + (kb + (lane & 7) + ((lane >> 3) & 1) * 8) * kVs + np * 16 + (lane >> 4) * 8;
        uint32_t r0, r1, r2, r3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                     : "r"(smem_u32(vp)));
        mma16816(o[2 * np], pa, r0, r1);
        mma16816(o[2 * np + 1], pa, r2, r3);
      }
    }
  }
  l0 += __shfl_xor_sync(~0u, l0, 1);
  l0 += __shfl_xor_sync(~0u, l0, 2);
  l1 += __shfl_xor_sync(~0u, l1, 1);
  l1 += __shfl_xor_sync(~0u, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const int r0 = q0 + g, r1 = q0 + g + 8;
  __half* y0 = y.p + ((size_t)img * N + r0) * y.stride + h * 64;
  __half* y1 = y.p + ((size_t)img * N + r1) * y.stride + h * 64;
#pragma unroll
  for (int n = 0; n < 8; n++) {
    if (r0 < N) *(__half2*)(y0 + n * 8 + 2 * t) = __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
    if (r1 < N) *(__half2*)(y1 + n * 8 + 2 * t) = __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
  }
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
  if (!getenv("YK_ATTN_SIMT")) {
    dim3 grid((N + 63) / 64, heads, qkv->batch);
    launch_k(attn_mma_kernel, grid, 128, 0, (cudaStream_t)st, dview(*qkv), dview(*y), N,
                                                        rsqrtf((float)kd));
    note_launch();
    return check_launch("attn_mma");
  }
  const size_t smem = (size_t)N * (kd + hd) * sizeof(__half);
  if (smem > 227 * 1024) return YK_EUNSUP;
  // enough blocks to cover the SMs: split keys further when batch x heads is small
  const long long blocks1 = (long long)qkv->batch * heads * ((N + 127) / 128);
  if (blocks1 >= 4 * 148) return launch_attn<1>(qkv, y, heads, N, smem, (cudaStream_t)st);
  if (blocks1 * 4 >= 148) return launch_attn<4>(qkv, y, heads, N, smem, (cudaStream_t)st);
  return launch_attn<8>(qkv, y, heads, N, smem, (cudaStream_t)st);
}
