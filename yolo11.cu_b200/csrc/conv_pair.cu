// Convolution on SM pairs: tcgen05.mma with cta_group::2 (algo 6).
//
// The transposed tiles of conv_tc.cu (M = 128 output channels, N = 256 pixels per CTA) move
// (128 + 256) x 64 fp16 operand rows from L2 into shared memory per 4.2 MFLOP; on the large
// 1x1 and stride-2 convs that is about 13 TB/s of L2 -> SMEM traffic at ~800 TF/s, and the
// loads, not the tensor pipe, set the pace.  Here two CTAs of a cluster share one MMA of
// M = 256 channels x N = 256 pixels: each CTA stages its own 128 weight rows and HALF of the
// pixel rows (128), and the pair's leader issues the MMA over both shared memories.  Per
// CTA that is 256 rows per 8.4 MFLOP, a third fewer bytes per FLOP, and each CTA's TMEM
// still holds two 128 x 256 fp32 accumulators, so epilogues overlap the next tile.
//
// Roles (672 threads per CTA, one CTA per SM, clusters of two):
//   warp 0     lane 0: TMA producer.  Both CTAs load their halves with the .cta_group::2
//              form of the tensor copy, completing bytes on the LEADER's full barrier (the
//              leader arms it with both halves' bytes).  Each CTA's loads fill only its own memory.
//   warp 20    both CTAs: TMEM allocation (cta_group::2).  Leader lane 0: issues the MMAs,
//              releases each stage group in both CTAs and hands finished accumulators to
//              both CTAs' epilogues by tcgen05.commit to each CTA's barrier (two commits).
//   warps 4-19 epilogue in each CTA, two groups taking alternate tiles: the CTA's 128
//              channels x 256 pixels, as the transposed epilogue of conv_tc.cu; one lane per
//              warp then arrives on the leader's accumulator-free barrier (remote for the
//              second CTA).
// Waits are bounded as everywhere else; both CTAs always reach the final cluster barrier.
#include "common.cuh"

namespace yk {

constexpr int kPairThreads = 672;
constexpr int kPairMma = 20;

template <int STAGES, int G>
struct PairCfg {
  static constexpr int kHalf = 128 * 128;                  // 128 rows x 64 fp16 channels
  static constexpr int kStage = 2 * kHalf;                 // weight half + pixel half
  static constexpr int kNacc = 2;                          // 2 x 256 TMEM columns
  static constexpr int kStg = 16 * 32 * 32 * 2;            // per-warp [32 px][32 ch] staging
  static constexpr int kBars = 256;
  static constexpr size_t kSmem = (size_t)STAGES * kStage + 1024 + kBars + kStg;
  static_assert(kSmem <= 232448, "smem budget");
  static_assert(STAGES % G == 0 && STAGES / G >= 2, "stage groups");
};

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// tensor copies of one CTA of the pair: data into this CTA, bytes on the barrier at
// `bar` (a shared::cluster address, the leader's barrier)
__device__ __forceinline__ void tma_pair_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_pair_im2col(uint32_t dst, const CUtensorMap* map,
                                                uint32_t bar, int c, int w, int h, int n,
                                                uint16_t kx, uint16_t ky) {
  asm volatile(
      "cp.async.bulk.tensor.4d.im2col.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(kx), "h"(ky)
      : "memory");
}
__device__ __forceinline__ void tc_mma_pair(uint32_t dtmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on the barrier at `bar` (shared::cluster) once this thread's pair MMAs finish
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

template <int STAGES, int G>
__global__ void __launch_bounds__(kPairThreads, 1)
conv_pair_kernel(const ConvArgs a, const __grid_constant__ CUtensorMap tmW,
                 const __grid_constant__ CUtensorMap tmX) {
  using Cfg = PairCfg<STAGES, G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar_base = base + STAGES * Cfg::kStage;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + 2 + b); };
  const uint32_t tslot = bar_base + 8u * (2 * STAGES + 4);
  static_assert(8 * (2 * STAGES + 4) + 16 <= Cfg::kBars, "barrier area");
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  volatile int* abort_flag = (volatile int*)(smem_raw + (tslot - raw) + 8);
  __half* stg_s = (__half*)(smem_raw + (bar_base - raw) + Cfg::kBars);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full_bar(s), 1);
      if (s < STAGES / G) mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < Cfg::kNacc; b++) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 16);   // 8 epilogue warps in each CTA
    }
    *abort_flag = 0;
    mbar_fence_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
  }
  // global memory and TMEM (a co-resident predecessor may still hold it) only after the
  // previous kernel has completed
  pdl_wait();
  pdl_trigger();
  if (warp == kPairMma) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncwarp();
  cluster_barrier();   // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;
  const int HWo = a.Ho * a.Wo;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const int batch = a.M / HWo;
      uint32_t g = 0;
      for (int t = pair; t < a.ntiles && !*abort_flag; t += npairs) {
        const int tm = t / a.ntn, tn = t - tm * a.ntn;
        const int m0 = tm * 256 + (int)rank * 128, c0 = tn * 256 + (int)rank * 128;
        int i0 = batch, h0 = 0, w0 = 0;   // im2col origin of this CTA's 128 pixels
        if (a.tmaA == 2 && m0 < a.M) {
          i0 = m0 / HWo;
          const int rem = m0 - i0 * HWo, oy = rem / a.Wo;
          h0 = oy * a.s - a.p;
          w0 = (rem - oy * a.Wo) * a.s - a.p;
        }
        bool ok = true;
        for (int kb = 0; kb < a.nk; kb++, g++) {
          const int s = g % STAGES;
          const uint32_t u = g / STAGES;
          if (u > 0 && s % G == 0 && !mbar_wait(empty_bar(s / G), (u - 1) & 1, 0x601)) {
            ok = false;
            break;
          }
          const uint32_t sW = base + s * Cfg::kStage, sP = sW + Cfg::kHalf;
          const uint32_t fb = cluster_map(full_bar(s), 0);
          if (rank == 0) mbar_expect_tx(full_bar(s), 2 * Cfg::kStage);
          if (a.tmaA == 2) {
            const int tap = kb / a.ncb, cbi = kb - tap * a.ncb;
            const int ky = tap / a.k, kx = tap - ky * a.k;
            tma_pair_2d(sW, &tmW, fb, tap * a.Cin + cbi * 64, c0);
            tma_pair_im2col(sP, &tmX, fb, cbi * 64, w0, h0, i0, (uint16_t)kx, (uint16_t)ky);
          } else {
            tma_pair_2d(sW, &tmW, fb, kb * 64, c0);
            tma_pair_2d(sP, &tmX, fb, kb * 64, m0);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp >= 4 && warp < kPairMma) {
    // ---------------- epilogue: this CTA's 128 channels x the tile's 256 pixels ----------------
    // group grp takes alternate tiles; its two warps per TMEM sub-partition take alternate
    // 32-pixel chunks
    const int sp = warp & 3, grp = (warp - 4) >> 3, half = ((warp - 4) >> 2) & 1;
    __half* stg = stg_s + (warp - 4) * 32 * 32;
    const uint32_t tempty_leader0 = cluster_map(tempty_bar(0), 0);
    uint32_t li = 0;
    for (int t = pair; t < a.ntiles; t += npairs, li++) {
      if ((int)(li & 1) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (!mbar_wait(tfull_bar(acc), use & 1, 0x603)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int tm = t / a.ntn, tn = t - tm * a.ntn;
      const int m0 = tm * 256;
      const int n0 = tn * 256 + (int)rank * 128;
      const int ch = n0 + sp * 32 + lane;
      const float bc = ch < a.Cout ? a.bias[ch] : 0.f;
      const uint32_t tcol = tmem + ((uint32_t)(sp * 32) << 16) + acc * 256;
      const bool any_ch = n0 + sp * 32 < a.Cout;   // uniform
#pragma unroll 1
      for (int pc = half; pc < 8 && any_ch; pc += 2) {
        uint32_t r[32];
        tmem_ld16p(tcol + pc * 32, r);
        tmem_ld16p(tcol + pc * 32 + 16, r + 16);
        tmem_ld_wait();
        // lanes 2j and 2j+1 (channels c, c+1) swap halves so that each writes one 32-bit
        // (pixel, channel pair): even lanes pixel k, odd lanes pixel k+1, one full 128-byte
        // shared-memory wavefront per store instead of two half-used ones
        const bool odd = lane & 1;
        uint32_t* stg32 = (uint32_t*)stg;
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const __half2 h = bias_act2(make_float2(__uint_as_float(r[k]), __uint_as_float(r[k + 1])),
                                      make_float2(bc, bc), a.act);
          const uint32_t own = *(const uint32_t*)&h;
          const uint32_t other = __shfl_xor_sync(~0u, own, 1);
          // even: (own.lo, other.lo) = pixel k, channels c, c+1; odd: (other.hi, own.hi)
          const uint32_t v = odd ? __byte_perm(other, own, 0x7632) : __byte_perm(own, other, 0x5410);
          stg32[((k + odd) * 32 + (lane & ~1)) >> 1] = v;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int q = lane + 32 * i, px = q >> 2, cc = q & 3;
          const int m = m0 + pc * 32 + px, c8 = n0 + sp * 32 + cc * 8;
          if (m < a.M && c8 < a.Cout) {
            uint4 o = *(const uint4*)(stg + px * 32 + cc * 8);
            if (a.res) {
              const uint4 rv = *(const uint4*)(a.res + (size_t)m * a.rs + c8);
              __half2* oh = (__half2*)&o;
              const __half2* rh = (const __half2*)&rv;
#pragma unroll
              for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(oh[e]), g2 = __half22float2(rh[e]);
                oh[e] = __floats2half2_rn(f.x + g2.x, f.y + g2.y);
              }
            }
            *(uint4*)(a.y + (size_t)m * a.ys + c8) = o;
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + 8u * acc);
    }
  } else if (warp == kPairMma && rank == 0 && lane == 0) {
    // ---------------- MMA issuer (leader CTA) ----------------
    constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
    uint32_t g = 0, li = 0;
    for (int t = pair; t < a.ntiles && !*abort_flag; t += npairs, li++) {
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (use > 0 && !mbar_wait(tempty_bar(acc), (use - 1) & 1, 0x604)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + acc * 256;
      bool ok = true;
      for (int kb = 0; kb < a.nk; kb++, g++) {
        const int s = g % STAGES;
        if (!mbar_wait(full_bar(s), (g / STAGES) & 1, 0x602)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sW = base + s * Cfg::kStage, sP = sW + Cfg::kHalf;
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          // M = channels (this CTA's 128 weight rows), N = the tile's 256 pixels
          tc_mma_pair(d, swz_desc<128>(sW + kk * 32), swz_desc<128>(sP + kk * 32), idesc,
                      (kb | kk) != 0);
        if (s % G == G - 1) {
          tc_commit_pair(empty_bar(s / G));
          tc_commit_pair(cluster_map(empty_bar(s / G), 1));
        }
      }
      if (!ok) { *abort_flag = 1; break; }
      tc_commit_pair(tfull_bar(acc));
      tc_commit_pair(cluster_map(tfull_bar(acc), 1));
    }
  }
  tc_fence_before();
  __syncwarp();
  cluster_barrier();   // no remote arrivals or MMAs into the other CTA remain
  if (warp == kPairMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

template <int STAGES, int G>
static int launch_pair(const ConvArgs& a, cudaStream_t st) {
  using Cfg = PairCfg<STAGES, G>;
  if (smem_attr(conv_pair_kernel<STAGES, G>, (int)Cfg::kSmem) != cudaSuccess) return check_launch("conv_pair attr");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return YK_EUNSUP;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed =
      g_pdl_override >= 0 ? g_pdl_override : pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  // persistent: as many pairs as can be resident at once (SM pairs of one TPC)
  static int max_clusters[64] = {};
  if (!max_clusters[dev]) {
    cfg.gridDim = dim3(2);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (void*)conv_pair_kernel<STAGES, G>, &cfg) !=
            cudaSuccess || n < 1)
      return check_launch("conv_pair occupancy");
    max_clusters[dev] = n;
  }
  const int pairs = a.ntiles < max_clusters[dev] ? a.ntiles : max_clusters[dev];
  cfg.gridDim = dim3(2 * pairs);
  CUtensorMap tmW, tmX;
  if (!encode_2d(&tmW, a.w, (uint64_t)a.Ktot, (uint64_t)a.Cout, (uint64_t)a.Ktot * 2, 128, 64))
    return YK_EUNSUP;
  if (a.tmaA == 1 &&
      !encode_2d(&tmX, a.x, (uint64_t)a.Cin, (uint64_t)a.M, (uint64_t)a.xs * 2, 128, 64))
    return YK_EUNSUP;
  if (a.tmaA == 2 && !encode_im2col(&tmX, a, 64)) return YK_EUNSUP;
  cudaLaunchKernelEx(&cfg, conv_pair_kernel<STAGES, G>, a, tmW, tmX);
  note_launch();
  return check_launch("conv_pair");
}

// Tiles of 256 output channels x 256 pixels on a CTA pair; A operand by TMA (2-D for 1x1
// stride-1, im2col otherwise), 64-channel blocks (Cin >= 64, 16-byte aligned view).
int conv_pair(const ConvArgs& a0, cudaStream_t st) {
  ConvArgs a = a0;
  if (!a.tmaA) return YK_EUNSUP;
  a.ntn = (a.Cout + 255) / 256;
  const long long nt = ((long long)(a.M + 255) / 256) * a.ntn;
  if (nt > 0x7fffffffLL) return YK_EUNSUP;
  a.ntiles = (int)nt;
  return launch_pair<6, 2>(a, st);
}

}  // namespace yk
