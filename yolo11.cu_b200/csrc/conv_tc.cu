// Implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[M = batch*Ho*Wo, N = Cout] = A[M, K = k*k*Cin] * W[N, K]^T,   fp16 in, fp32 in TMEM
//
// A is the im2col of an NHWC fp16 channel-slice view, never materialised: the K axis is the
// flat (ky, kx, ci) index with no per-tap padding (the reference's dense-K packing,
// engine/engine.cu:270-358), so Cin = 8/16 layers waste nothing.  W is the OHWI weight
// tensor, already [N][K] K-contiguous.
//
// Persistent, warp-specialised CTA (448 threads, one per SM); a CTA tile is MT stacked
// 128-row sub-tiles x BN columns, taken round-robin:
//   warps 0-3  producers, into a STAGES-deep ring of 128-byte-swizzled K-major tiles (BK=64):
//              W tiles come by TMA (2-D tensor map over [Cout][K], zero fill past the edges,
//              no cluster sharing); A tiles with Cin >= 64 come by TMA too (2-D for 1x1
//              stride-1 convs, the TMA im2col mode for k x k / stride s, where one stage is
//              one 64-channel block of one filter tap); thinner A tiles are gathered in 16-byte
//              cp.async chunks whose completion arrives on the stage's mbarrier in hardware
//              (cp.async.mbarrier.arrive.noinc), so producers never stall on their own loads.
//   warp 12    allocates TMEM and one lane issues tcgen05.mma (M=128, N=BN, K=16; warp 13
//              issues for half of the stacked sub-tiles of plain tiles): per stage
//              four K steps x MT independent sub-tile accumulators (independent chains keep
//              the tensor pipe busy when BN is small), then tcgen05.commit releases the stage;
//              a finished tile's accumulators are handed to the epilogue.
//   warps 4-11 epilogue, two groups of four warps taking alternate tiles (warp w reads TMEM
//              lanes 32(w%4)..): tcgen05.ld of the accumulator, bias (cached in shared
//              memory), SiLU, residual, fp16 store into the output channel slice; then free the
//              accumulator.  A ring of 2-4 TMEM accumulators lets the epilogues of earlier
//              tiles overlap the mainloop of later ones.
// Every mbarrier wait is bounded (common.cuh kWaitNs): on timeout the CTA records an error
// in the device error word, raises an abort flag that every role polls, drains its copies,
// frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

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
  int Ktot, M, nk, ntn, ntiles;
  int tmaA;          // A tiles: 0 cp.async gather, 1 TMA 2-D (1x1 s1 p0), 2 TMA im2col
  int ncb;           // TMA modes: CB-channel blocks per filter tap
  int bulk_store;    // plain tiles: epilogue rows leave by bulk tensor stores (tmY)
};

constexpr int kProducers = 128;
constexpr int kEpiGroup = 128;      // one epilogue group = 4 warps = all 128 sub-tile rows
constexpr int kBiasSmem = 1024;     // bias floats cached in shared memory
constexpr int kThreads = 416;      // halo-patch kernel: 13 warps
constexpr int kTcThreads = 448;    // implicit GEMM: 14 warps (warp 13 = second MMA issuer)
constexpr int kMmaWarp = 12;

template <int BN, int STAGES, int MT, int CB, bool T = false>
struct TcCfg {
  static constexpr int kTPS = 64 / CB;                      // K blocks (CB wide) per stage
  static constexpr int kABytes = 128 * 128;                 // one 128-row sub-tile
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStage = MT * kABytes + kBBytes;
  static constexpr int kAccCols = BN < 32 ? 32 : BN;         // one sub-tile accumulator
  static constexpr int kTileCols = MT * kAccCols;
  static constexpr int kNacc = 512 / kTileCols >= 4 ? 4 : 512 / kTileCols;  // TMEM ring
  static constexpr int kTmemCols = kNacc * kTileCols;        // <= 512, power of two
  // transposed tiles: per epilogue warp a [32 pixels][32 channels] fp16 staging block
  // per epilogue warp a 2 KB staging block ([32 px][32 ch] transposed, or [32 rows][32 ch]
  // for the bulk row stores), 512-byte aligned
  static constexpr int kStg = 8 * 32 * 32 * 2 + 512;
  static constexpr size_t kSmem = (size_t)STAGES * kStage + 1024 + 256 + kBiasSmem * 4 + kStg;
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert((size_t)STAGES * kStage + 1024 + 256 + kBiasSmem * 4 + kStg <= 232448,
                "smem budget");
};

__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
// im2col-mode TMA load (NHWC, 4-D): 128 output pixels starting at input coordinate (w, h, n)
// for filter tap (kx, ky), 64 channels from channel c; the tensor map carries the padding
// box and the conv stride.
__device__ __forceinline__ void tma_load_im2col(uint32_t dst, const CUtensorMap* map,
                                                uint32_t bar, int c, int w, int h, int n,
                                                uint16_t kx, uint16_t ky) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(kx), "h"(ky)
      : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory, completing its bytes on the mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

template <int BN, int STAGES, int MT, int CB, int G, bool T>
__global__ void __launch_bounds__(kTcThreads, 1)
conv_tc_kernel(const ConvArgs a, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmY) {
  using Cfg = TcCfg<BN, STAGES, MT, CB, T>;
  static_assert(!T || ((BN == 128 || BN == 256) && CB == 64),
                "transposed tiles: 128 or 256 channels, 64-channel blocks");
  // 256 transposed channels: two M = 128 MMAs per K step share the pixel operand (half the
  // operand bytes per FLOP of 128-channel tiles); one accumulator fills TMEM, and the two
  // epilogue groups drain its channel halves together
  constexpr bool kT2 = T && BN == 256;
  // 512 transposed pixels (MT = 4): two N = 256 MMAs per K step share the weight operand;
  // one accumulator fills TMEM, the two epilogue groups drain its pixel halves together
  constexpr bool kT4 = T && MT == 4;
  static_assert(!(kT2 && kT4), "one split at a time");
  constexpr bool kSplit = kT2 || kT4;
  // Plain tiles with stacked sub-tiles have two MMA issuers (warps 12 and 13), each owning half
  // of the sub-tiles: a single thread issues a narrow MMA only every ~50-80 cycles, below the
  // tensor pipe's rate, and each issuer's commits stall only itself.
  constexpr int kNMma = (!T && MT >= 2) ? 2 : 1;
  static_assert(STAGES % G == 0 && STAGES / G >= 2, "stage groups");
  constexpr int kTM = 128 * MT;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bar_base = base + STAGES * Cfg::kStage;
  // barriers: full[S], empty[S], tfull[NACC], tempty[NACC]; the TMEM slot, the abort flag;
  // then the bias cache
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * STAGES + Cfg::kNacc + b); };
  const uint32_t tslot = bar_base + 8u * (2 * STAGES + 2 * Cfg::kNacc);
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  volatile int* abort_flag = (volatile int*)(smem_raw + (tslot - raw) + 8);
  float* bias_s = (float*)(smem_raw + (base - raw) + STAGES * Cfg::kStage + 256);
  const uint32_t stg_base =
      (smem_u32(bias_s + kBiasSmem) + 511u) & ~511u;   // per-warp 2 KB staging blocks
  __half* stg_s = (__half*)(smem_raw + (stg_base - raw));

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full_bar(s), a.tmaA ? 1 : kProducers + 1);
      if (s < STAGES / G) mbar_init(empty_bar(s), kNMma);
    }
    for (int b = 0; b < Cfg::kNacc; b++) {
      mbar_init(tfull_bar(b), kNMma);
      mbar_init(tempty_bar(b), kSplit ? 2 * kEpiGroup : kEpiGroup);
    }
    *abort_flag = 0;
    mbar_fence_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
    if (a.tmaA) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmA) : "memory");
  }
  // everything above overlaps the previous kernel; activations, the output and TMEM (which a
  // co-resident predecessor may still hold) are touched only after it has completed
  pdl_wait();
  pdl_trigger();
  if (warp == kMmaWarp) {
    tmem_alloc(tslot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;
  const long long t_role = clock64();

  if (warp < 4) {
    // ---------------- producers ----------------
    const int c = tid & 7, r0 = tid >> 3;
    const int HWo = a.Ho * a.Wo;
    const uint32_t offA = sw_off(r0, c);
    const int batch = a.M / HWo;
    uint32_t g = 0;   // global stage counter across tiles
    const bool gather = !a.tmaA;
    // test hook (yk_test_inject): withhold block 0's first stage (no expect-tx, no loads),
    // so its MMA warp's bounded wait runs out and the abort path unwinds the CTA
    const bool withhold = !gather && blockIdx.x == 0 && *(volatile int*)&g_test_withhold;
    for (int t = blockIdx.x; t < a.ntiles && !*abort_flag && (gather || tid == 0); t += gridDim.x) {
      const int m0 = (t / a.ntn) * kTM, n0 = (t % a.ntn) * BN;
      int w0[MT], h0[MT], i0[MT];      // im2col start of each sub-tile (input coords of its pixel 0)
      if (a.tmaA == 2) {
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          const int m = m0 + mt * 128;
          if (m < a.M) {
            i0[mt] = m / HWo;
            const int rem = m - i0[mt] * HWo, oy = rem / a.Wo;
            h0[mt] = oy * a.s - a.p;
            w0[mt] = (rem - oy * a.Wo) * a.s - a.p;
          } else {
            i0[mt] = batch; h0[mt] = 0; w0[mt] = 0;   // past the last image: reads zeros
          }
        }
      }
      // gather: per row, the pixel offset of its image and the packed (y, x) window origin
      int rowpix[8 * MT], yx[8 * MT];
      if (gather) {
#pragma unroll
        for (int i = 0; i < 8 * MT; i++) {
          const int m = m0 + r0 + 16 * i;
          const bool ok = m < a.M;
          const int mm = ok ? m : 0;
          const int img = mm / HWo, rem = mm - img * HWo;
          const int oy = rem / a.Wo, ox = rem - oy * a.Wo;
          rowpix[i] = img * a.H * a.W;
          const int yb = ok ? oy * a.s - a.p : -30000;   // invalid rows fail the bounds test
          yx[i] = (yb << 16) | ((ox * a.s - a.p) & 0xffff);
        }
      }
      for (int kb = 0; kb < a.nk; kb++, g++) {
        const int s = g % STAGES;
        const uint32_t u = g / STAGES;
        // stages are released G at a time (one tcgen05.commit per group)
        if (u > 0 && s % G == 0 && !mbar_wait(empty_bar(s / G), (u - 1) & 1, 0x101)) {
          *abort_flag = 1;
          break;
        }
        const uint32_t sA = base + s * Cfg::kStage, sB = sA + MT * Cfg::kABytes;
        if (tid == 0 && !(withhold && g == 0)) {
          mbar_expect_tx(full_bar(s), Cfg::kBBytes + (gather ? 0 : MT * Cfg::kABytes));
          // stage kb holds K blocks q = kb*TPS + j (j < TPS), each CB channels of one tap;
          // blocks past the end read weights out of range (zeros), so they add nothing
          constexpr uint32_t kABlk = 128 * CB * 2, kBBlk = BN * CB * 2;
#pragma unroll
          for (int j = 0; j < Cfg::kTPS; j++) {
            const int q = kb * Cfg::kTPS + j;
            if (a.tmaA == 2) {
              const int tap = q / a.ncb, cbi = q - tap * a.ncb;
              const int tapc = tap < a.k * a.k ? tap : a.k * a.k - 1;
              const int ky = tapc / a.k, kx = tapc - ky * a.k;
              tma_load_2d(sB + j * kBBlk, &tmB, full_bar(s), tap * a.Cin + cbi * CB, n0);
#pragma unroll
              for (int mt = 0; mt < MT; mt++)
                tma_load_im2col(sA + (mt * Cfg::kTPS + j) * kABlk, &tmA, full_bar(s), cbi * CB,
                                w0[mt], h0[mt], i0[mt], (uint16_t)kx, (uint16_t)ky);
            } else {
              tma_load_2d(sB + j * kBBlk, &tmB, full_bar(s), q * CB, n0);
              if (!gather)
#pragma unroll
                for (int mt = 0; mt < MT; mt++)
                  tma_load_2d(sA + (mt * Cfg::kTPS + j) * kABlk, &tmA, full_bar(s), q * CB,
                              m0 + mt * 128);
            }
          }
        }
        if (!gather) continue;
        const int kk = kb * 64 + c * 8;
        const bool kval = kk < a.Ktot;
        const int tap = kval ? kk / a.Cin : 0;
        const int ci = kk - tap * a.Cin;
        const int ky = tap / a.k, kx = tap - ky * a.k;
#pragma unroll
        for (int i = 0; i < 8 * MT; i++) {
          const int iy = (yx[i] >> 16) + ky, ix = (int)(short)(yx[i] & 0xffff) + kx;
          const bool ok = kval && (unsigned)iy < (unsigned)a.H && (unsigned)ix < (unsigned)a.W;
          const __half* src = ok ? a.x + (size_t)(rowpix[i] + iy * a.W + ix) * a.xs + ci : a.x;
          cp_async16(sA + offA + (uint32_t)(i * 2048), src, ok ? 16u : 0u);
        }
        cp_async_arrive_noinc(full_bar(s));   // arrives when this thread's copies land
      }
    }
    cp_async_wait<0>();
    if (tid == 0) YK_PROF_ADD(10, clock64() - t_role);
  } else if (warp < kMmaWarp && T) {
    // ---------------- epilogue, transposed tiles ----------------
    // TMEM lane = output channel n0 + 32*sp + lane, column = pixel m0 + col.  Per 32-pixel
    // chunk: bias + SiLU per lane, fp16 into the warp's [pixel][channel] staging block, then
    // 16-byte rows of 8 channels (residual added) stored pixel by pixel.
    const int sp = warp & 3, grp = (warp - 4) >> 2;
    __half* stg = stg_s + (warp - 4) * 32 * 32;
    uint32_t li = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, li++) {
      if (!kSplit && (int)(li & 1) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (!mbar_wait(tfull_bar(acc), use & 1, 0x103)) { *abort_flag = 1; break; }
      tc_fence_after();
#ifdef YK_TC_DIAG_NOEPI   // diagnostic builds only: drain the accumulator without reading it
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
      continue;
#endif
      const int m0 = (t / a.ntn) * kTM + (kT4 ? 256 * grp : 0);
      const int n0 = (t % a.ntn) * BN + (kT2 ? 128 * grp : 0);
      const int ch = n0 + sp * 32 + lane;
      const float bc = ch < a.Cout ? a.bias[ch] : 0.f;
      const uint32_t tcol = tmem + ((uint32_t)(sp * 32) << 16) + acc * Cfg::kTileCols +
                            (kSplit ? 256 * grp : 0);
      const bool any_ch = n0 + sp * 32 < a.Cout;   // uniform
#pragma unroll 1
      for (int pc = 0; pc < (kT4 ? 256 : kTM) / 32 && any_ch; pc++) {
        uint32_t r[32];
        tmem_ld16p(tcol + pc * 32, r);
        tmem_ld16p(tcol + pc * 32 + 16, r + 16);
        tmem_ld_wait();
        // lanes 2j and 2j+1 (channels c, c+1) swap halves so that each writes one 32-bit
        // (pixel, channel pair): even lanes pixel k, odd lanes pixel k+1, one full 128-byte
        // shared-memory wavefront per store instead of two half-used ones
        const bool odd = lane & 1;
        uint32_t* stg32 = (uint32_t*)stg;
        if (a.bulk_store) {   // the previous chunk's store has read the staging block
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
        }
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
        if (a.bulk_store) {   // no residual: the block leaves by one bulk tensor store
          fence_proxy_async();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmY, smem_u32(stg), n0 + sp * 32, m0 + pc * 32);
            bulk_commit();
          }
          continue;
        }
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
      mbar_arrive(tempty_bar(acc));
    }
    if (a.bulk_store && lane == 0) bulk_wait0();
    if (lane == 0) YK_PROF_ADD(9, clock64() - t_role);
  } else if (warp < kMmaWarp) {
    // ---------------- epilogue ----------------
    const int sp = warp & 3;              // TMEM sub-partition this warp may read
    const int grp = (warp - 4) >> 2;      // epilogue group: takes every other tile
    const int row = sp * 32 + lane;
    const bool bias_cached = a.Cout <= kBiasSmem;
    if (bias_cached)
      for (int i = tid - 128; i < a.Cout; i += 256) bias_s[i] = a.bias[i];
    asm volatile("bar.sync 1, 256;" ::: "memory");   // epilogue warps only
    const float* bias = bias_cached ? bias_s : a.bias;
    uint32_t li = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, li++) {
      if ((int)(li & 1) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (!mbar_wait(tfull_bar(acc), use & 1, 0x103)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int m0 = (t / a.ntn) * kTM, n0 = (t % a.ntn) * BN;
#pragma unroll 1
      for (int mt = 0; mt < MT; mt++) {
        const int m = m0 + mt * 128 + row;
        const bool mok = m < a.M;
        __half* yrow = a.y + (size_t)(mok ? m : 0) * a.ys;
        const __half* rrow = a.res ? a.res + (size_t)(mok ? m : 0) * a.rs : nullptr;
        const uint32_t trow = tmem + ((uint32_t)(sp * 32) << 16) + acc * Cfg::kTileCols +
                              mt * Cfg::kAccCols;
        if (a.bulk_store)
          epi_rows_tma<BN>(trow, n0, a.Cout, m0 + mt * 128 + sp * 32, mok ? rrow : nullptr,
                           bias, a.act, stg_base + (warp - 4) * 2048, &tmY, lane);
        else
          epi_row<BN>(trow, n0, a.Cout, mok, yrow, rrow, bias, a.act);
      }
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));
    }
    if (lane == 0) bulk_wait0();
    if (lane == 0) YK_PROF_ADD(9, clock64() - t_role);
  } else if (lane == 0 && warp - kMmaWarp < kNMma) {
    // ---------------- MMA issuers (warp 12, and 13 for stacked plain tiles) ----------------
    constexpr uint32_t idesc = idesc_f16_m128(BN);
    constexpr int kMtPer = MT / kNMma;
    const int mt0 = (warp - kMmaWarp) * kMtPer;
    uint32_t g = 0, li = 0;
    for (int t = blockIdx.x; t < a.ntiles && !*abort_flag; t += gridDim.x, li++) {
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (use > 0 && !mbar_wait(tempty_bar(acc), (use - 1) & 1, 0x104)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + acc * Cfg::kTileCols;
      bool ok = true;
      for (int kb = 0; kb < a.nk; kb++, g++) {
        const int s = g % STAGES;
        if (!mbar_wait(full_bar(s), (g / STAGES) & 1, 0x102)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sA = base + s * Cfg::kStage, sB = sA + MT * Cfg::kABytes;
        constexpr uint32_t kABlk = 128 * CB * 2, kBBlk = BN * CB * 2;
        if constexpr (T) {
          // transposed: A = 128 weight rows (output channels), B = all MT*128 pixel rows
          constexpr uint32_t idt = idesc_f16_m128(kT4 ? 256 : MT * 128);
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            tc_mma_f16(d, swz_desc<128>(sB + kk * 32), swz_desc<128>(sA + kk * 32), idt,
                       (kb | kk) != 0);
            if constexpr (kT2)   // channels 128-255: weight rows 128-255, columns 256-511
              tc_mma_f16(d + 256, swz_desc<128>(sB + 128 * 128 + kk * 32),
                         swz_desc<128>(sA + kk * 32), idt, (kb | kk) != 0);
            if constexpr (kT4)   // pixels 256-511: pixel rows 256-511, columns 256-511
              tc_mma_f16(d + 256, swz_desc<128>(sB + kk * 32),
                         swz_desc<128>(sA + 2 * Cfg::kABytes + kk * 32), idt, (kb | kk) != 0);
          }
        } else if constexpr (CB == 8) {
          // 16-byte blocks, no swizzle: one K=16 step spans blocks 2i and 2i+1 (LBO apart)
#pragma unroll
          for (int i = 0; i < Cfg::kTPS / 2; i++)
#pragma unroll
            for (int q = 0; q < kMtPer; q++) {
              const int mt = mt0 + q;
              tc_mma_f16(d + mt * Cfg::kAccCols,
                         nosw_desc(sA + (mt * Cfg::kTPS + 2 * i) * kABlk, kABlk, 128),
                         nosw_desc(sB + 2 * i * kBBlk, kBBlk, 128), idesc, (kb | i) != 0);
            }
        } else {
#pragma unroll
          for (int j = 0; j < Cfg::kTPS; j++)
#pragma unroll
            for (int kk = 0; kk < CB / 16; kk++)
#pragma unroll
              for (int q = 0; q < kMtPer; q++) {
                const int mt = mt0 + q;
                tc_mma_f16(d + mt * Cfg::kAccCols,
                           swz_desc<CB * 2>(sA + (mt * Cfg::kTPS + j) * kABlk + kk * 32),
                           swz_desc<CB * 2>(sB + j * kBBlk + kk * 32), idesc, (kb | j | kk) != 0);
              }
        }
        if (s % G == G - 1) tc_commit(empty_bar(s / G));
      }
      if (!ok) { *abort_flag = 1; break; }
      tc_commit(tfull_bar(acc));
    }
    if (warp == kMmaWarp) {
      YK_PROF_ADD(8, clock64() - t_role);
      YK_PROF_ADD(11, 1);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

static int g_num_sms[64] = {};

static CUtensorMapSwizzle swizzle_of(int cb) {
  return cb == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : cb == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
         : cb == 16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
}

// 2-D fp16 tensor map with a 64-element (128-byte) inner box and the 128-byte swizzle that
// matches the UMMA K-major layout; out-of-range elements read as zero.
static bool encode_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_bytes, uint32_t box_outer, int cb, bool swizzle = true) {
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
              cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return false;
      encode = (PFN_cuTensorMapEncodeTiled)fn;
    }
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)cb, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                swizzle ? swizzle_of(cb) : CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// im2col tensor map over the NHWC input view: dims {C, W, H, N}, the padding bounding box
// [-p, W-1+p-(k-1)] per spatial dim, conv stride as the traversal stride, 64 channels x 128
// output pixels per load, 128-byte swizzle; outside the image reads as zero.
static bool encode_im2col(CUtensorMap* m, const ConvArgs& a, int cb) {
  static PFN_cuTensorMapEncodeIm2col encode = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &fn, cudaEnableDefault, &q) !=
              cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return false;
      encode = (PFN_cuTensorMapEncodeIm2col)fn;
    }
  }
  const uint64_t batch = (uint64_t)a.M / ((uint64_t)a.Ho * a.Wo);
  const cuuint64_t dims[4] = {(cuuint64_t)a.Cin, (cuuint64_t)a.W, (cuuint64_t)a.H, batch};
  const cuuint64_t strides[3] = {(cuuint64_t)a.xs * 2, (cuuint64_t)a.W * a.xs * 2,
                                 (cuuint64_t)a.H * a.W * a.xs * 2};
  const int lower[2] = {-a.p, -a.p};
  const int upper[2] = {a.p - (a.k - 1), a.p - (a.k - 1)};
  const cuuint32_t estr[4] = {1, (cuuint32_t)a.s, (cuuint32_t)a.s, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(a.x), dims, strides,
                lower, upper, (cuuint32_t)cb, 128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                swizzle_of(cb), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int STAGES, int MT, int G, int CB = 64, bool T = false>
static int launch_tc(const ConvArgs& a, cudaStream_t st) {
  using Cfg = TcCfg<BN, STAGES, MT, CB, T>;
  if (smem_attr(conv_tc_kernel<BN, STAGES, MT, CB, G, T>, (int)Cfg::kSmem) != cudaSuccess)
    return check_launch("conv_tc attr");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return YK_EUNSUP;
  if (!g_num_sms[dev]) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.ntiles < g_num_sms[dev] ? a.ntiles : g_num_sms[dev];
  CUtensorMap tmB, tmA;
  memset(&tmA, 0, sizeof tmA);
  if (!encode_2d(&tmB, a.w, (uint64_t)a.Ktot, (uint64_t)a.Cout, (uint64_t)a.Ktot * 2, BN, CB))
    return YK_EUNSUP;
  if (a.tmaA == 1 &&
      !encode_2d(&tmA, a.x, (uint64_t)a.Cin, (uint64_t)a.M, (uint64_t)a.xs * 2, 128, CB))
    return YK_EUNSUP;
  if (a.tmaA == 2 && !encode_im2col(&tmA, a, CB))
    return YK_EUNSUP;
  CUtensorMap tmY;
  memset(&tmY, 0, sizeof tmY);
  ConvArgs b = a;
  // output [M][Cout] view with row stride ys: 32 channels x 32 rows per store (plain tiles:
  // 64-byte swizzle; transposed tiles without a residual: the unswizzled [32 px][32 ch]
  // staging block)
  b.bulk_store = (!T || !a.res) && ((uintptr_t)a.y & 15) == 0 && a.ys % 8 == 0 &&
                 bulk_store_enabled() &&
                 encode_2d(&tmY, a.y, (uint64_t)a.Cout, (uint64_t)a.M, (uint64_t)a.ys * 2, 32, 32,
                           !T);
  launch_k(conv_tc_kernel<BN, STAGES, MT, CB, G, T>, grid, kTcThreads, Cfg::kSmem,
           (cudaStream_t)st, b, tmB, tmA, tmY);
  note_launch();
  return check_launch("conv_tc");
}

// Heuristic N tile: widest tile that does not waste half of it, shrunk when the tile count
// would leave most of the 148 SMs idle.
int pick_tile(int M, int Cout) {
  int bn = Cout <= 32 ? 32 : Cout <= 64 ? 64 : Cout <= 128 ? 128 : (Cout % 256 == 0 ? 256 : 128);
  long long mt = (M + 127) / 128;
  while (bn > 64 && mt * ((Cout + bn - 1) / bn) < 148) bn >>= 1;
  return bn;
}

// Heuristic M sub-tiles per CTA tile: narrow N tiles stack 2-4 sub-tiles so independent
// accumulation chains keep the tensor pipe busy, as long as the grid still fills the SMs.
int pick_msub(int M, int Cout, int bn) {
  int ms = bn <= 32 ? 4 : bn <= 64 ? 2 : 1;
  const long long nt = (Cout + bn - 1) / bn;
  while (ms > 1 && ((M + 128LL * ms - 1) / (128LL * ms)) * nt < 2 * 148) ms >>= 1;
  return ms;
}

#ifdef YK_CONV_PROF
extern "C" void yk_conv_prof(unsigned long long* out, int reset) {
  cudaMemcpyFromSymbol(out, g_prof, sizeof(unsigned long long) * 16);
  if (reset) {
    unsigned long long z[16] = {};
    cudaMemcpyToSymbol(g_prof, z, sizeof z);
  }
}
#endif

int conv_patch(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, int bn,
               int ms, bool trans, cudaStream_t st);

int conv_kxn(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, int bn,
             int ms, cudaStream_t st);

int conv_pair(const ConvArgs& a, cudaStream_t st);

int conv_tc(const YkView* x, const YkView* y, const YkView* res, const YkConv* p,
            cudaStream_t st) {
  if (p->algo == 5) {
    const int bn = p->tile ? p->tile : p->Cout <= 32 ? 32 : 64;
    const int ms = p->msub ? p->msub : 1;
    return conv_kxn(x, y, res, p, bn, ms, st);
  }
  if (p->algo == 2 || p->algo == 4) {
    const bool trans = p->algo == 4;
    const int bn = p->tile ? p->tile
                   : p->Cout <= 64 ? 64 : (p->Cout <= 128 || trans) ? 128 : 256;
    const int ms = p->msub ? p->msub : trans ? 2 : 1;
    return conv_patch(x, y, res, p, bn, ms, trans, st);
  }
  if (p->algo < 0 || p->algo > 6) return YK_EINVAL;
  ConvArgs a;
  DView X = dview(*x), Y = dview(*y);
  a.x = X.p; a.H = x->H; a.W = x->W; a.xs = x->stride;
  a.y = Y.p; a.Ho = y->H; a.Wo = y->W; a.ys = y->stride;
  a.res = res ? dview(*res).p : nullptr;
  a.rs = res ? res->stride : 0;
  a.w = (const __half*)p->weight; a.bias = p->bias;
  a.Cin = p->Cin; a.Cout = p->Cout; a.k = p->k; a.s = p->s; a.p = p->p; a.act = p->act;
  a.Ktot = p->k * p->k * p->Cin;
  const long long M = (long long)y->batch * y->H * y->W;
  if (M > 0x7fffffffLL || (long long)x->batch * x->H * x->W > 0x7fffffffLL) return YK_EUNSUP;
  if (x->H > 30000 || x->W > 30000) return YK_EUNSUP;   // packed 16-bit window origins
  a.M = (int)M;
  a.nk = (a.Ktot + 63) / 64;
  const int bn = p->algo == 3 ? (p->tile == 256 ? 256 : 128)
                 : p->tile ? p->tile : pick_tile(a.M, a.Cout);
  if (bn != 32 && bn != 64 && bn != 128 && bn != 256) return YK_EINVAL;
  int ms = p->msub ? p->msub : p->algo == 3 ? 2 : pick_msub(a.M, a.Cout, bn);
  if (bn == 256 && p->algo != 3) ms = 1;
  if (bn == 128 && ms > 2 && p->algo != 3) ms = 2;
  if (ms != 1 && ms != 2 && ms != 4) return YK_EINVAL;
  a.ntn = (a.Cout + bn - 1) / bn;
  const long long nt = ((M + 128LL * ms - 1) / (128LL * ms)) * a.ntn;
  if (nt > 0x7fffffffLL) return YK_EUNSUP;
  a.ntiles = (int)nt;
  // A by TMA when the view allows it: CB = 64-channel blocks (128-byte rows) for Cin >= 64,
  // 32 / 16 / 8-channel blocks (64 / 32-byte swizzled rows, 16-byte unswizzled core matrices)
  // for Cin = 32 / 16 / 8
  // (1x1 convs with other Cin below 64: the widest block padding Cin by at most a third,
  // e.g. 48 -> 64;
  // the A tensor map's channel extent stays Cin, so the padding channels load as zeros and
  // whatever weights the B box reads for them add nothing)
  int cb = p->Cin >= 64 ? 64
           : ((p->Cin == 32 || p->Cin == 16 || p->Cin == 8) && bn <= 64) ? p->Cin : 0;
  if (!cb && p->Cin % 8 == 0 && p->k == 1 && p->s == 1 && p->p == 0)   // tiled 2-D maps only
    for (int c : {64, 32, 16, 8})
      if ((c == 64 || bn <= 64) && (p->Cin + c - 1) / c * c * 3 <= p->Cin * 4) { cb = c; break; }
  const bool tma_ok = cb && ((uintptr_t)a.x & 15) == 0 && (a.xs % 8) == 0;
  a.tmaA = 0;
  a.ncb = cb ? (p->Cin + cb - 1) / cb : 0;
  if (tma_ok && p->k == 1 && p->s == 1 && p->p == 0) a.tmaA = 1;
  else if (tma_ok && p->p < 128 && p->k - 1 - p->p < 128 && p->s <= 8) a.tmaA = 2;
  if (a.tmaA) {
    const int tps = 64 / cb;                      // K blocks per stage
    a.nk = (p->k * p->k * a.ncb + tps - 1) / tps;
  }
  // (STAGES, G): a tcgen05.commit costs about as much issue time as ten MMAs, so stages are
  // released in groups of G with at least 16 MMAs per commit where shared memory allows
  if (p->algo == 6) {   // CTA pairs: 256 output channels x 256 pixels
    if (cb != 64 || !a.tmaA) return YK_EINVAL;
    return conv_pair(a, st);
  }
  if (p->algo == 3) {   // transposed tiles: 128 output channels x 128*ms pixels
    if (cb != 64) return YK_EINVAL;
    if (bn == 256) return ms == 2 ? launch_tc<256, 3, 2, 1, 64, true>(a, st) : YK_EINVAL;
    if (ms == 4) return launch_tc<128, 2, 4, 1, 64, true>(a, st);
    if (ms == 1) return launch_tc<128, 6, 1, 3, 64, true>(a, st);
    if (ms == 2) return launch_tc<128, 4, 2, 2, 64, true>(a, st);
    return YK_EINVAL;
  }
  if (a.tmaA && cb < 64) {
    switch (bn * 1000 + ms * 100 + cb) {
      case 32116: return launch_tc<32, 8, 1, 4, 16>(a, st);
      case 32216: return launch_tc<32, 4, 2, 2, 16>(a, st);
      case 32416: return launch_tc<32, 3, 4, 1, 16>(a, st);
      case 64116: return launch_tc<64, 8, 1, 4, 16>(a, st);
      case 64216: return launch_tc<64, 4, 2, 2, 16>(a, st);
      case 64416: return launch_tc<64, 2, 4, 1, 16>(a, st);
      case 32132: return launch_tc<32, 8, 1, 4, 32>(a, st);
      case 32232: return launch_tc<32, 4, 2, 2, 32>(a, st);
      case 32432: return launch_tc<32, 3, 4, 1, 32>(a, st);
      case 64132: return launch_tc<64, 8, 1, 4, 32>(a, st);
      case 64232: return launch_tc<64, 4, 2, 2, 32>(a, st);
      case 64432: return launch_tc<64, 2, 4, 1, 32>(a, st);
      case 32108: return launch_tc<32, 8, 1, 4, 8>(a, st);
      case 32208: return launch_tc<32, 4, 2, 2, 8>(a, st);
      case 32408: return launch_tc<32, 3, 4, 1, 8>(a, st);
      case 64108: return launch_tc<64, 8, 1, 4, 8>(a, st);
      case 64208: return launch_tc<64, 4, 2, 2, 8>(a, st);
      case 64408: return launch_tc<64, 2, 4, 1, 8>(a, st);
      default: return YK_EINVAL;
    }
  }
  switch (bn * 10 + ms) {
    case 321: return launch_tc<32, 8, 1, 4>(a, st);
    case 322: return launch_tc<32, 4, 2, 2>(a, st);
    case 324: return launch_tc<32, 3, 4, 1>(a, st);
    case 641: return launch_tc<64, 8, 1, 4>(a, st);
    case 642: return launch_tc<64, 4, 2, 2>(a, st);
    case 644: return launch_tc<64, 2, 4, 1>(a, st);
    case 1281: return launch_tc<128, 6, 1, 3>(a, st);
    case 1282: return launch_tc<128, 4, 2, 2>(a, st);
    case 2561: return launch_tc<256, 4, 1, 2>(a, st);
    default: return YK_EINVAL;
  }
}

}  // namespace yk
