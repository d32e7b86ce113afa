// Implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[M = batch*Ho*Wo, N = Cout] = A[M, K = k*k*Cin] * W[N, K]^T,   fp16 in, fp32 in TMEM
//
// A is the im2col of an NHWC fp16 channel-slice view, never materialised: the K axis is the
// flat (ky, kx, ci) index with no per-tap padding (the reference's dense-K packing,
// engine/engine.cu:270-358), so Cin = 8/16 layers waste nothing.  W is the OHWI weight
// tensor, already [N][K] K-contiguous.
//
// CTA = 160 threads, one 128 x BN output tile:
//   warps 0-3  producers: gather 16-byte chunks of A (im2col with zero padding) and W with
//              cp.async into a STAGES-deep ring of 128-byte-swizzled K-major tiles
//              (BK = 64), then signal "full" on an mbarrier once their copies landed;
//              after the mainloop the same warps are the epilogue (warp w owns TMEM lanes
//              32w..32w+31 = output rows), reading the fp32 accumulator with tcgen05.ld and
//              applying bias, SiLU, residual and the fp16 channel-slice store.
//   warp 4     allocates TMEM (BN columns) and one lane issues tcgen05.mma (M=128, N=BN,
//              K=16, four per stage) and tcgen05.commit to release each stage and finally
//              signal the epilogue.
// Every mbarrier wait is bounded (common.cuh kWaitNs); on timeout the CTA records an error
// in the device error word, drains its copies, frees TMEM and returns.
#include "common.cuh"

namespace yk {

struct ConvArgs {
  const __half* x;  // view base (offset by coff)
  int H, W, xs;
  __half* y;
  int Ho, Wo, ys;
  const __half* res;  // nullable, offset by coff
  int rs;
  const __half* w;
  const float* bias;
  int Cin, Cout, k, s, p, act;
  int Ktot, M, nk, ntn;
};

constexpr int kProducers = 128;
constexpr int kThreads = 160;

template <int BN, int STAGES>
struct TcCfg {
  static constexpr int kABytes = 128 * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr size_t kSmem = (size_t)STAGES * kStage + 1024 + 256;
};

__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1) conv_tc_kernel(const ConvArgs a) {
  using Cfg = TcCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar_base = base + STAGES * Cfg::kStage;
  // barriers: full[0..S), empty[S..2S), accum[2S]; tmem slot after them
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  const uint32_t accum_bar = bar_base + 8u * (2 * STAGES);
  const uint32_t tslot = bar_base + 8u * (2 * STAGES + 1);
  uint32_t* tslot_ptr = (uint32_t*)(smem_raw + (tslot - raw));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nt = blockIdx.x % a.ntn;
  const int mt = blockIdx.x / a.ntn;
  const int m0 = mt * 128, n0 = nt * BN;

  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full_bar(s), kProducers);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accum_bar, 1);
    mbar_fence_init();
  }
  if (warp == 4) {
    tmem_alloc(tslot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *(volatile uint32_t*)tslot_ptr;

  if (warp < 4) {
    // ---------------- producers ----------------
    const int c = tid & 7, r0 = tid >> 3;
    const int HWo = a.Ho * a.Wo;
    int ybase[8], xbase[8];
    const __half* rowp[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      int m = m0 + r0 + 16 * i;
      bool ok = m < a.M;
      int mm = ok ? m : 0;
      int img = mm / HWo, rem = mm - img * HWo;
      int oy = rem / a.Wo, ox = rem - oy * a.Wo;
      ybase[i] = ok ? oy * a.s - a.p : -(1 << 28);   // invalid rows never pass the bounds test
      xbase[i] = ox * a.s - a.p;
      rowp[i] = a.x + (size_t)img * a.H * a.W * a.xs;
    }
    const uint32_t offA = sw_off(r0, c);
    bool ok_all = true;
    int kb = 0;
    for (; kb < a.nk; kb++) {
      const int s = kb % STAGES, u = kb / STAGES;
      if (u > 0 && !mbar_wait(empty_bar(s), (u - 1) & 1, 0x101)) { ok_all = false; break; }
      const uint32_t sA = base + s * Cfg::kStage, sB = sA + Cfg::kABytes;
      const int kk = kb * 64 + c * 8;
      const bool kval = kk < a.Ktot;
      const int tap = kval ? kk / a.Cin : 0;
      const int ci = kk - tap * a.Cin;
      const int ky = tap / a.k, kx = tap - ky * a.k;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int iy = ybase[i] + ky, ix = xbase[i] + kx;
        const bool ok = kval && (unsigned)iy < (unsigned)a.H && (unsigned)ix < (unsigned)a.W;
        const __half* src = ok ? rowp[i] + ((size_t)iy * a.W + ix) * a.xs + ci : a.x;
        cp_async16(sA + offA + (uint32_t)(i * 2048), src, ok ? 16u : 0u);
      }
#pragma unroll
      for (int j = 0; j < BN / 16; j++) {
        const int n = n0 + r0 + 16 * j;
        const bool ok = kval && n < a.Cout;
        const __half* src = ok ? a.w + (size_t)n * a.Ktot + kk : a.w;
        cp_async16(sB + sw_off(r0 + 16 * j, c), src, ok ? 16u : 0u);
      }
      cp_async_commit();
      // signal stage kb-2 once its copies have landed (two stages stay in flight)
      if (kb >= 2) {
        cp_async_wait<2>();
        fence_proxy_async();
        mbar_arrive(full_bar((kb - 2) % STAGES));
      }
    }
    cp_async_wait<0>();
    fence_proxy_async();
    if (ok_all) {
      for (int t = (kb >= 2 ? kb - 2 : 0); t < kb; t++) mbar_arrive(full_bar(t % STAGES));
    }

    // ---------------- epilogue ----------------
    const bool acc_ok = mbar_wait(accum_bar, 0, 0x103);
    tc_fence_after();
    const int row = warp * 32 + lane;
    const int m = m0 + row;
    const bool mok = m < a.M && acc_ok;
    __half* yrow = a.y + (size_t)(mok ? m : 0) * a.ys;
    const __half* rrow = a.res ? a.res + (size_t)(mok ? m : 0) * a.rs : nullptr;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    if (acc_ok) {
#pragma unroll 1
      for (int cc = 0; cc < BN / 16; cc++) {
        const int n = n0 + cc * 16;
        if (n >= a.Cout) break;  // uniform across the warp
        uint32_t r[16];
        tmem_ld16(trow + cc * 16, r);
        tmem_ld_wait();
        if (!mok) continue;
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int nn = n + 8 * h;
          if (nn >= a.Cout) break;
          const float4 b0 = __ldg((const float4*)(a.bias + nn));
          const float4 b1 = __ldg((const float4*)(a.bias + nn + 4));
          float v[8] = {__uint_as_float(r[8 * h + 0]) + b0.x, __uint_as_float(r[8 * h + 1]) + b0.y,
                        __uint_as_float(r[8 * h + 2]) + b0.z, __uint_as_float(r[8 * h + 3]) + b0.w,
                        __uint_as_float(r[8 * h + 4]) + b1.x, __uint_as_float(r[8 * h + 5]) + b1.y,
                        __uint_as_float(r[8 * h + 6]) + b1.z, __uint_as_float(r[8 * h + 7]) + b1.w};
          if (a.act == 1) {
#pragma unroll
            for (int q = 0; q < 8; q++) v[q] = silu(v[q]);
          }
          if (rrow) {
            uint4 rv = *(const uint4*)(rrow + nn);
            const __half2* rh = (const __half2*)&rv;
#pragma unroll
            for (int q = 0; q < 4; q++) {
              float2 f = __half22float2(rh[q]);
              v[2 * q] += f.x;
              v[2 * q + 1] += f.y;
            }
          }
          uint4 o;
          __half2* oh = (__half2*)&o;
#pragma unroll
          for (int q = 0; q < 4; q++) oh[q] = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
          *(uint4*)(yrow + nn) = o;
        }
      }
    }
    tc_fence_before();
  } else if (lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_f16_m128(BN);
    bool ok = true;
    for (int kb = 0; kb < a.nk; kb++) {
      const int s = kb % STAGES;
      if (!mbar_wait(full_bar(s), (kb / STAGES) & 1, 0x102)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sA = base + s * Cfg::kStage, sB = sA + Cfg::kABytes;
#pragma unroll
      for (int kk = 0; kk < 4; kk++)
        tc_mma_f16(tmem, sw128_desc(sA + kk * 32), sw128_desc(sB + kk * 32), idesc,
                   (kb | kk) != 0);
      tc_commit(empty_bar(s));
    }
    if (ok) tc_commit(accum_bar);
  }
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int BN, int STAGES>
static int launch_tc(const ConvArgs& a, cudaStream_t st) {
  using Cfg = TcCfg<BN, STAGES>;
  static bool attr_set = false;   // per process; the attribute is per function, all devices
  if (!attr_set) {
    if (cudaFuncSetAttribute(conv_tc_kernel<BN, STAGES>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Cfg::kSmem) != cudaSuccess)
      return check_launch("conv_tc attr");
    attr_set = true;
  }
  const long long mtiles = (a.M + 127) / 128;
  const long long blocks = mtiles * a.ntn;
  if (blocks > 0x7fffffffLL) return YK_EUNSUP;
  conv_tc_kernel<BN, STAGES><<<(unsigned)blocks, kThreads, Cfg::kSmem, st>>>(a);
  note_launch();
  return check_launch("conv_tc");
}

// Heuristic N tile: widest tile that does not waste half of it, shrunk when the grid would
// leave most of the 148 SMs idle.
int pick_tile(int M, int Cout) {
  int bn = Cout <= 32 ? 32 : Cout <= 64 ? 64 : Cout <= 128 ? 128 : (Cout % 256 == 0 ? 256 : 128);
  long long mt = (M + 127) / 128;
  while (bn > 64 && mt * ((Cout + bn - 1) / bn) < 148) bn >>= 1;
  return bn;
}

int conv_tc(const YkView* x, const YkView* y, const YkView* res, const YkConv* p,
            cudaStream_t st) {
  ConvArgs a;
  DView X = dview(*x), Y = dview(*y);
  a.x = X.p; a.H = x->H; a.W = x->W; a.xs = x->stride;
  a.y = Y.p; a.Ho = y->H; a.Wo = y->W; a.ys = y->stride;
  a.res = res ? dview(*res).p : nullptr;
  a.rs = res ? res->stride : 0;
  a.w = (const __half*)p->weight; a.bias = p->bias;
  a.Cin = p->Cin; a.Cout = p->Cout; a.k = p->k; a.s = p->s; a.p = p->p; a.act = p->act;
  a.Ktot = p->k * p->k * p->Cin;
  long long M = (long long)y->batch * y->H * y->W;
  if (M > 0x7fffffffLL) return YK_EUNSUP;
  a.M = (int)M;
  a.nk = (a.Ktot + 63) / 64;
  int bn = p->tile ? p->tile : pick_tile(a.M, a.Cout);
  a.ntn = (a.Cout + bn - 1) / bn;
  switch (bn) {
    case 32: return launch_tc<32, 5>(a, st);
    case 64: return launch_tc<64, 4>(a, st);
    case 128: return launch_tc<128, 4>(a, st);
    case 256: return launch_tc<256, 4>(a, st);
    default: return YK_EINVAL;
  }
}

}  // namespace yk
