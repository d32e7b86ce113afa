// 3x3 stride-1 convolution on tcgen05 with halo patches and the horizontal filter taps
// folded into the MMA's N side.
//
// Each tcgen05.mma costs the issuing thread tens of cycles whatever its size, so a conv with
// few output channels (N = Cout per MMA) cannot keep the tensor pipe busy with one MMA per
// filter tap.  Here the three horizontal taps (kx) become extra output columns instead:
//
//   D'[r][3c + kx] = sum over (ky, ci) of  window[r + 16*ky][ci] * W[c][ky][kx][ci]
//   out[i][c]      = D'[i][3c] + D'[i+1][3c+1] + D'[i+2][3c+2]
//
// where r / i index the positions of the halo patch (rows of 16, the first 14 real outputs,
// as in conv_patch.cu).  One MMA is M = 128 positions x N = 3*BN x K = 16, so a 64-channel
// 3x3 conv needs 12 MMAs of N = 192 per 128 positions instead of 36 of N = 64, with the
// same multiply-adds.  The epilogue adds the three kx partial sums: rows i+1 and i+2 are the
// next TMEM lanes, one and two lanes down in the same warp (a patch row is 16 lanes).
//
// Weights come straight from the OHWI tensor by a 4-D tensor map {ci, kx, ky, c}: the box
// {CB, 3, 1, BN} for one ky lands as rows (c, kx) = 3c + kx of CB channels, exactly the
// K-major B operand.  Per 64- (or 32-) channel block of Cin the CTA loads one input window
// (as conv_patch.cu) and three weight stages (ky = 0, 1, 2); one tcgen05.commit releases all
// four.  Roles, TMEM ring, bounded waits: as conv_tc.cu.
#include "common.cuh"

namespace yk {

// 21 warps: 0 producer, 4-19 epilogue, 20 MMA.  The epilogue has 16 warps (the kx sums):
// with four TMEM accumulators (when four tiles fit in 512 columns) each accumulator has its
// own four warps and four tiles drain at once; with two, each is drained by eight warps
// taking alternate 16-channel blocks.  Residual rows are
// copied to shared memory (cp.async) before the accumulator wait, hiding their latency
// behind the MMAs.
constexpr int kKxMma = 20;
constexpr int kKxThreads = 32 * (kKxMma + 1);

template <int BN, int MT, int CB, int WR = 0>
struct KxnCfg {
  static constexpr int kRows = 8 * MT + 2;
  static constexpr int kRB = CB * 2;
  static constexpr int kWinTx = kRows * kPatchCols * kRB;
  static constexpr int kWin = (kWinTx + 1023) & ~1023;
  static constexpr int kB = 3 * BN * kRB;                         // one ky: rows (c, kx)
  static constexpr int kSub = 3 * BN;                             // accumulator columns
  static constexpr int kTileCols = MT * kSub;
  // TMEM accumulator ring: four when they fit (so four tiles drain at once), else two
  static constexpr int kNacc = 4 * kTileCols <= 512 ? 4 : 2;
  // epilogue warps per sub-partition and tile: 16 epilogue warps = kNacc groups of 4 * kH,
  // the kH warps of one sub-partition taking alternate 16-channel blocks
  static constexpr int kH = 4 / kNacc;
  // window ring: as deep as 216 KB allows (up to 6), so small tiles keep several TMA loads
  // in flight; each slot holds a window and its three weight stages, or, with WR > 0 (the
  // CTA's filter slice is WR channel blocks, loaded once and kept), the 3 * WR weight stages
  // exist once and the slots hold windows only
  static constexpr int kResSlot = MT * (BN / (16 * kH)) * 2 * 16;   // residual bytes per thread
  static constexpr int kRes = 512 * kResSlot;                      // all epilogue threads
  static constexpr int kWSTfit =
      WR ? (216 * 1024 - kRes - 3 * WR * kB) / kWin : (216 * 1024 - kRes) / (kWin + 3 * kB);
  static constexpr int kWST = kWSTfit > 6 ? 6 : kWSTfit < 2 ? 2 : kWSTfit;
  static constexpr int kBST = WR ? 3 * WR : 3 * kWST;
  static constexpr int kTmemCols = kNacc * kTileCols <= 256 ? 256 : 512;
  static constexpr int kBars = 512;
  static constexpr size_t kSmem =
      (size_t)kWST * kWin + (size_t)kBST * kB + 1024 + kBars + kBiasSmem * 4 + kRes;
  // TMA epilogue: per epilogue warp and (sub-tile, channel block) one staging box of
  // 2 rows x kPatchUse positions x 16 channels (residual in, then the output in place)
  static constexpr int kEpiBox = 2 * 14 * 16 * 2;      // bytes one box moves
  static constexpr int kEpiStride = 1024;              // boxes on 128-byte boundaries
  static_assert(kRes >= 16 * MT * (BN / (16 * kH)) * kEpiStride, "TMA epilogue staging");
  static_assert(kNacc * kTileCols <= 512, "TMEM budget");
  // resident weights need a window ring of two slots besides them
  static constexpr bool kFits = kSmem <= 232448 && (WR == 0 || kWSTfit >= 2);
  static_assert(3 * BN <= 256 && BN % 16 == 0, "N = 3 * BN");
};

template <int BN, int MT, int CB, int WR>
__global__ void __launch_bounds__(kKxThreads, 1)
conv_kxn_kernel(const PatchArgs a, const __grid_constant__ CUtensorMap tmW,
                const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY,
                const __grid_constant__ CUtensorMap tmR) {
  using Cfg = KxnCfg<BN, MT, CB, WR>;
  static_assert(Cfg::kFits, "smem budget");
  constexpr int kRB = Cfg::kRB, WST = Cfg::kWST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t wbase = base, bbase = base + WST * Cfg::kWin;
  const uint32_t bar_base = bbase + Cfg::kBST * Cfg::kB;
  // barriers: wfull[WST], wempty[WST], bfull[BST], tfull[NACC], tempty[NACC]
  auto wfull = [&](int s) { return bar_base + 8u * s; };
  auto wempty = [&](int s) { return bar_base + 8u * (WST + s); };
  auto bfull = [&](int s) { return bar_base + 8u * (2 * WST + s); };
  auto tfull = [&](int b) { return bar_base + 8u * (2 * WST + Cfg::kBST + b); };
  auto tempty = [&](int b) { return bar_base + 8u * (2 * WST + Cfg::kBST + Cfg::kNacc + b); };
  const uint32_t tslot = bar_base + 8u * (2 * WST + Cfg::kBST + 2 * Cfg::kNacc);
  static_assert(8 * (2 * WST + Cfg::kBST + 2 * Cfg::kNacc) + 16 + 8 * 16 <= Cfg::kBars, "barrier area");
  auto rbar = [&](int e) { return tslot + 16u + 8u * e; };   // epilogue warp e's residual boxes
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  volatile int* abort_flag = (volatile int*)(smem_raw + (tslot - raw) + 8);
  float* bias_s = (float*)(smem_raw + (bar_base - raw) + Cfg::kBars);
  const uint32_t res_base = bar_base + Cfg::kBars + kBiasSmem * 4;   // residual staging

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < WST; s++) { mbar_init(wfull(s), 1); mbar_init(wempty(s), 1); }
    for (int s = 0; s < Cfg::kBST; s++) mbar_init(bfull(s), 1);
    for (int b = 0; b < Cfg::kNacc; b++) { mbar_init(tfull(b), 1); mbar_init(tempty(b), Cfg::kH * kEpiGroup); }
    for (int e = 0; e < 16; e++) mbar_init(rbar(e), 1);
    *abort_flag = 0;
    mbar_fence_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmW) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
    if (a.tma_epi) {
      asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmY) : "memory");
      if (a.res) asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmR) : "memory");
    }
  }
  pdl_wait();
  pdl_trigger();
  if (warp == kKxMma) {
    tmem_alloc(tslot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot_ptr;
  const int per_img = a.nty * a.ntx;
  // resident weights (WR = a.ncb channel blocks; the grid is a multiple of a.ntn, so every
  // tile of this CTA has the same output channels): stage 3 * cb + ky, loaded with the
  // first tile's blocks and kept
  constexpr bool wres = WR > 0;

  if (warp == 0) {
    // ---------------- producer (one thread, all loads by TMA) ----------------
    if (tid == 0) {
      uint32_t gw = 0;
      for (int t = blockIdx.x; t < a.ntiles && !*abort_flag; t += gridDim.x) {
        const int mtile = t / a.ntn, n0 = (t - mtile * a.ntn) * BN;
        const int img = mtile / per_img, r = mtile - img * per_img;
        const int ty = r / a.ntx, tx = r - ty * a.ntx;
        bool ok = true;
        for (int cb = 0; cb < a.ncb; cb++, gw++) {
          const int ws = gw % WST;
          const uint32_t uw = gw / WST;
          // one commit releases the window and its three weight stages together
          if (uw > 0 && !mbar_wait(wempty(ws), (uw - 1) & 1, 0x301)) { ok = false; break; }
          mbar_expect_tx(wfull(ws), Cfg::kWinTx);
          tma_load_4d(wbase + ws * Cfg::kWin, &tmX, wfull(ws), cb * CB, tx * kPatchUse - 1,
                      ty * 8 * MT - 1, img);
          for (int ky = 0; ky < 3 && !(wres && gw >= (uint32_t)WR); ky++) {
            const int bs = (wres ? cb : ws) * 3 + ky;
            mbar_expect_tx(bfull(bs), Cfg::kB);
            tma_load_4d(bbase + bs * Cfg::kB, &tmW, bfull(bs), cb * CB, 0, ky, n0);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
    }
  } else if (warp >= 4 && warp < kKxMma) {
    // ---------------- epilogue ----------------
    const int sp = warp & 3;
    constexpr int kH = Cfg::kH;
    const int grp = (warp - 4) / (4 * kH);    // the accumulator (tile index mod kNacc) it drains
    const int half = ((warp - 4) >> 2) % kH;  // which alternate 16-channel blocks
    const int row = sp * 32 + lane;
    const int pr = row >> 4, pc = row & 15;
    const bool bias_cached = a.Cout <= kBiasSmem;
    if (bias_cached)
      for (int i = tid - 128; i < a.Cout; i += 512) bias_s[i] = a.bias[i];
    asm volatile("bar.sync 1, 512;" ::: "memory");
    const float* bias = bias_cached ? bias_s : a.bias;
    const int e = warp - 4;                                  // epilogue warp index
    const uint32_t ebuf = res_base + (uint32_t)(e * MT * (BN / (16 * kH)) * Cfg::kEpiStride);
    uint32_t li = 0, ruse = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, li++) {
      if ((int)(li % Cfg::kNacc) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      const int mtile = t / a.ntn, n0 = (t - mtile * a.ntn) * BN;
      const int img = mtile / per_img, r = mtile - img * per_img;
      const int ty = r / a.ntx, tx = r - ty * a.ntx;
      const int x = tx * kPatchUse + pc;
      constexpr int kNcb = BN / (16 * kH);
      const int y_box = ty * 8 * MT + 2 * sp;        // first image row of this warp's box
      if (a.tma_epi) {
        // residual boxes before the accumulator wait, so their latency hides behind the
        // MMAs; the staging boxes are free once this warp's earlier stores have read them
        if (lane == 0) {
          bulk_wait_read0();
          if (a.res) {
            int nbox = 0;
            for (int cb = 0; cb < kNcb; cb++) nbox += n0 + 16 * half + 16 * kH * cb < a.Cout;
            mbar_expect_tx(rbar(e), (uint32_t)(MT * nbox * Cfg::kEpiBox));
#pragma unroll
            for (int mt = 0; mt < MT; mt++)
#pragma unroll
              for (int cb = 0; cb < kNcb; cb++) {
                const int c0 = 16 * half + 16 * kH * cb;
                if (n0 + c0 < a.Cout)
                  tma_load_4d(ebuf + (uint32_t)((mt * kNcb + cb) * Cfg::kEpiStride), &tmR, rbar(e),
                              n0 + c0, tx * kPatchUse, y_box + mt * 8, img);
              }
          }
        }
        __syncwarp();
      } else if (a.res) {
        // residual rows by cp.async: [mt][channel block][8-channel half]
        const uint32_t rslot = res_base + (uint32_t)(tid - 128) * Cfg::kResSlot;
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          const int y = ty * 8 * MT + mt * 8 + pr;
          const bool mok = pc < kPatchUse && x < a.W && y < a.H;
          const __half* rrow = a.res + (mok ? ((size_t)img * a.H + y) * a.W + x : 0) * a.rs;
#pragma unroll
          for (int cb = 0; cb < kNcb; cb++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const int nn = n0 + 16 * half + 16 * kH * cb + 8 * h;
              const bool ok = mok && nn < a.Cout;
              cp_async16(rslot + (uint32_t)(((mt * kNcb + cb) * 2 + h) * 16),
                         ok ? (const void*)(rrow + nn) : (const void*)a.res, ok ? 16u : 0u);
            }
        }
        cp_async_commit();
      }
      if (!mbar_wait(tfull(acc), use & 1, 0x303)) { *abort_flag = 1; break; }
      tc_fence_after();
#ifdef YK_KXN_DIAG_NOEPI   // diagnostic builds only: drain the accumulator without reading it
      if (a.tma_epi && a.res) { mbar_wait(rbar(e), ruse & 1, 0x307); ruse++; }
      tc_fence_before();
      mbar_arrive(tempty(acc));
      continue;
#endif
      if (a.tma_epi && a.res) {
        if (!mbar_wait(rbar(e), ruse & 1, 0x307)) { *abort_flag = 1; break; }
        ruse++;
      } else if (a.res) {
        cp_async_wait<0>();
      }
#pragma unroll 1
      for (int mt = 0; mt < MT; mt++) {
        const int y = ty * 8 * MT + mt * 8 + pr;
        const bool mok = pc < kPatchUse && x < a.W && y < a.H;
        const size_t m = mok ? ((size_t)img * a.H + y) * a.W + x : 0;
        __half* yrow = a.y + m * a.ys;
        const bool has_res = a.res != nullptr;
        const uint32_t trow = tmem + ((uint32_t)(sp * 32) << 16) + acc * Cfg::kTileCols +
                              mt * Cfg::kSub;
#pragma unroll
        for (int cb = 0; cb < kNcb; cb++) {   // 16 channels = 48 columns
          const int c0 = 16 * half + 16 * kH * cb;
          if (n0 + c0 >= a.Cout) break;           // uniform
          uint32_t rg[48];
          __syncwarp();   // the loads below are warp-collective; stores before may diverge
          tmem_ld16p(trow + 3 * c0, rg);
          tmem_ld16p(trow + 3 * c0 + 16, rg + 16);
          tmem_ld16p(trow + 3 * c0 + 32, rg + 32);
          tmem_ld_wait();
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const float p1 = __shfl_down_sync(~0u, __uint_as_float(rg[3 * j + 1]), 1);
            const float p2 = __shfl_down_sync(~0u, __uint_as_float(rg[3 * j + 2]), 2);
            v[j] = (__uint_as_float(rg[3 * j]) + p1) + p2;
          }
          // box position of this lane (2 rows x kPatchUse positions x 16 channels, 32 bytes
          // per position); the halo lanes (pc >= kPatchUse) have none
          const uint32_t box = ebuf + (uint32_t)((mt * kNcb + cb) * Cfg::kEpiStride);
          const uint32_t bpos = box + (uint32_t)(((lane >> 4) * kPatchUse + pc) * 32);
          if (a.tma_epi ? pc < kPatchUse : mok) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
              const int nn = n0 + c0 + 8 * h;
              uint4 o = make_uint4(0u, 0u, 0u, 0u);
              __half2* oh = (__half2*)&o;
              if (nn < a.Cout) {
                const float4 b0 = *(const float4*)(bias + nn);
                const float4 b1 = *(const float4*)(bias + nn + 4);
                const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                                      make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
                if (!has_res) {
#pragma unroll
                  for (int q = 0; q < 4; q++)
                    oh[q] = bias_act2(make_float2(v[8 * h + 2 * q], v[8 * h + 2 * q + 1]), bb[q],
                                      a.act);
                } else {
                  const uint32_t raddr =
                      a.tma_epi ? bpos + 16u * h
                                : res_base + (uint32_t)(tid - 128) * Cfg::kResSlot +
                                      (uint32_t)(((mt * kNcb + cb) * 2 + h) * 16);
                  uint4 rv;
                  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                               : "=r"(rv.x), "=r"(rv.y), "=r"(rv.z), "=r"(rv.w)
                               : "r"(raddr));
                  const __half2* rh = (const __half2*)&rv;
#pragma unroll
                  for (int q = 0; q < 4; q++) {
                    float v0 = v[8 * h + 2 * q] + bb[q].x, v1 = v[8 * h + 2 * q + 1] + bb[q].y;
                    if (a.act == 1) { v0 = silu_fast(v0); v1 = silu_fast(v1); }
                    const float2 f = __half22float2(rh[q]);
                    oh[q] = __floats2half2_rn(v0 + f.x, v1 + f.y);
                  }
                }
              } else if (!a.tma_epi) {
                break;
              }
              if (a.tma_epi)
                asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(bpos + 16u * h),
                             "r"(o.x), "r"(o.y), "r"(o.z), "r"(o.w)
                             : "memory");
              else
                *(uint4*)(yrow + nn) = o;
            }
          }
          if (a.tma_epi) {   // the box leaves by one bulk tensor store (clipped at the edges)
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_4d(&tmY, box, n0 + c0, tx * kPatchUse, y_box + mt * 8, img);
              bulk_commit();
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty(acc));
    }
    if (a.tma_epi && lane == 0) bulk_wait0();   // every store has completed before exit
  } else if (warp == kKxMma && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_f16_m128(3 * BN);
    uint32_t gw = 0, li = 0;
    // resident weight stages complete once (with the first tile) and stay valid: their
    // barriers are not polled again (three polls and fences per tile cost the 32-channel
    // 160x160 conv 15 %)
    bool wready = false;
    for (int t = blockIdx.x; t < a.ntiles && !*abort_flag; t += gridDim.x, li++) {
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (use > 0 && !mbar_wait(tempty(acc), (use - 1) & 1, 0x304)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + acc * Cfg::kTileCols;
      bool ok = true;
      for (int cb = 0; cb < a.ncb && ok; cb++, gw++) {
        const int ws = gw % WST;
        const uint32_t par = (gw / WST) & 1;
        if (!mbar_wait(wfull(ws), par, 0x305)) { ok = false; break; }
        tc_fence_after();
        const uint32_t win = wbase + ws * Cfg::kWin;
#pragma unroll
        for (int ky = 0; ky < 3; ky++) {
          const int bs = (wres ? cb : ws) * 3 + ky;
          if (!(wres && wready)) {
            if (!mbar_wait(bfull(bs), wres ? 0u : par, 0x306)) { ok = false; break; }
            tc_fence_after();
          }
          const uint32_t sb = bbase + bs * Cfg::kB;
#pragma unroll
          for (int kk = 0; kk < CB / 16; kk++)
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
              // A: the window shifted by ky patch rows (the swizzle follows the absolute
              // shared-memory address, so whole-row shifts need no descriptor base offset)
              const uint32_t sa = win + (uint32_t)((mt * 8 + ky) * kPatchCols * kRB + kk * 32);
#ifndef YK_KXN_DIAG_NOMMA   // diagnostic builds only: skip the MMAs, keep the pipeline
              tc_mma_f16(d + mt * Cfg::kSub, swz_desc<kRB>(sa), swz_desc<kRB>(sb + kk * 32),
                         idesc, (cb | ky | kk) != 0);
#endif
            }
        }
        if (ok) tc_commit(wempty(ws));
      }
      if (!ok) { *abort_flag = 1; break; }
      tc_commit(tfull(acc));
      wready = true;
    }
  }
  __syncthreads();
  if (warp == kKxMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// 4-D tiled map over the OHWI weights {ci, kx, ky, c}: box {CB, 3, 1, BN} = one ky's rows
// (c, kx), swizzled like the activations.
static bool encode_kxn_w(CUtensorMap* m, const __half* w, int Cin, int Cout, int bn, int cb) {
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
  const cuuint64_t dims[4] = {(cuuint64_t)Cin, 3, 3, (cuuint64_t)Cout};
  const cuuint64_t strides[3] = {(cuuint64_t)Cin * 2, (cuuint64_t)3 * Cin * 2,
                                 (cuuint64_t)9 * Cin * 2};
  const cuuint32_t box[4] = {(cuuint32_t)cb, 3, 1, (cuuint32_t)bn};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(w), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(cb),
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map {c, x, y, image} over an output / residual view (c = the view's channels, element
// stride `stride`): box {16 channels, kPatchUse positions, 2 rows, 1} = one epilogue warp's
// share of a tile, no swizzle.
static bool encode_epi_box(CUtensorMap* m, const __half* p, int C, int W, int H, int N,
                           int stride) {
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
  const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N};
  const cuuint64_t strides[3] = {(cuuint64_t)stride * 2, (cuuint64_t)W * stride * 2,
                                 (cuuint64_t)H * W * stride * 2};
  const cuuint32_t box[4] = {16, (cuuint32_t)kPatchUse, 2, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(p), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int MT, int CB, int WR = 0>
static int launch_kxn(const PatchArgs& a, const YkView* x, cudaStream_t st) {
  if constexpr (WR == 0) {
    // the CTA's whole filter slice stays in shared memory when it fits beside two windows
    if (a.ncb == 1 && KxnCfg<BN, MT, CB, 1>::kFits) return launch_kxn<BN, MT, CB, 1>(a, x, st);
    if (a.ncb == 2 && KxnCfg<BN, MT, CB, 2>::kFits) return launch_kxn<BN, MT, CB, 2>(a, x, st);
  }
  using Cfg = KxnCfg<BN, MT, CB, WR>;
  if (smem_attr(conv_kxn_kernel<BN, MT, CB, WR>, (int)Cfg::kSmem) != cudaSuccess) return check_launch("conv_kxn attr");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return YK_EUNSUP;
  if (!g_num_sms[dev]) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  int grid = a.ntiles < g_num_sms[dev] ? a.ntiles : g_num_sms[dev];
  if (WR) grid -= grid % a.ntn;   // fixed output channels per CTA (ntiles is a multiple of ntn)
  CUtensorMap tmW, tmX, tmY = {}, tmR = {};
  if (!encode_kxn_w(&tmW, a.w, a.Cin, a.Cout, BN, CB)) return YK_EUNSUP;
  if (!encode_patch_x(&tmX, a.x, a.Cin, a.W, a.H, x->batch, x->stride, Cfg::kRows, CB))
    return YK_EUNSUP;
  PatchArgs b = a;
  if (b.tma_epi &&
      !(encode_epi_box(&tmY, b.y, b.Cout, b.W, b.H, x->batch, b.ys) &&
        (!b.res || encode_epi_box(&tmR, b.res, b.Cout, b.W, b.H, x->batch, b.rs))))
    b.tma_epi = 0;
  launch_k(conv_kxn_kernel<BN, MT, CB, WR>, grid, kKxThreads, Cfg::kSmem, st, b, tmW, tmX, tmY, tmR);
  note_launch();
  return check_launch("conv_kxn");
}

// 3x3 stride-1 pad-1 conv with kx folded into N; Cin % 8 == 0 (64-, 32- or 16-channel
// blocks, swizzle matched to the block, the last block zero-filled past Cin), 16-byte
// aligned view.
// bn (output channels per tile) in {32, 64}, ms (stacked 8x16 sub-tiles) in {1, 2} (bn 32).
int conv_kxn(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, int bn,
             int ms, cudaStream_t st) {
  // channel block: the widest of 64 / 32 / 16 that pads Cin by at most a third (the tensor
  // maps' channel extent stays Cin, so the padding channels load as zeros from both the
  // activations and the weights and add nothing): 48 -> one 64-block, 80 -> three 32-blocks
  int cbw = 0;
  if (p->Cin % 8 == 0) {
    for (int c : {64, 32, 16})
      if ((p->Cin + c - 1) / c * c * 3 <= p->Cin * 4) { cbw = c; break; }
    if (!cbw) cbw = 16;   // thin inputs (8 channels): one zero-filled 16-channel block
  }
  if (p->k != 3 || p->s != 1 || p->p != 1 || p->groups != 1 || !cbw ||
      ((uintptr_t)x->ptr & 15) || x->stride % 8 || (x->coff % 8) ||
      ((uintptr_t)p->weight & 15))
    return YK_EUNSUP;
  if (y->H != x->H || y->W != x->W) return YK_EINVAL;
  PatchArgs a{};
  DView X = dview(*x), Y = dview(*y);
  a.x = X.p; a.H = x->H; a.W = x->W;
  a.y = Y.p; a.ys = y->stride;
  a.res = res ? dview(*res).p : nullptr;
  a.rs = res ? res->stride : 0;
  a.w = (const __half*)p->weight; a.bias = p->bias;
  a.Cin = p->Cin; a.Cout = p->Cout; a.act = p->act;
  a.ncb = (p->Cin + cbw - 1) / cbw;
  a.nty = (x->H + 8 * ms - 1) / (8 * ms);
  a.ntx = (x->W + kPatchUse - 1) / kPatchUse;
  a.ntn = (p->Cout + bn - 1) / bn;
  const long long nt = (long long)y->batch * a.nty * a.ntx * a.ntn;
  if (nt > 0x7fffffffLL) return YK_EUNSUP;
  a.ntiles = (int)nt;
  // outputs (and residual) by 4-D TMA boxes when the views are 16-byte rows
  static const bool direct = [] {
    const char* e = getenv("YK_KXN_DIRECT_EPI");
    return e && *e && *e != '0';
  }();
  a.tma_epi = !direct && ((uintptr_t)a.y & 15) == 0 && a.ys % 8 == 0 &&
              (!a.res || (((uintptr_t)a.res & 15) == 0 && a.rs % 8 == 0));
  switch (bn * 1000 + ms * 100 + cbw) {
    case 32132: return launch_kxn<32, 1, 32>(a, x, st);
    case 32232: return launch_kxn<32, 2, 32>(a, x, st);
    case 64132: return launch_kxn<64, 1, 32>(a, x, st);
    case 32164: return launch_kxn<32, 1, 64>(a, x, st);
    case 32264: return launch_kxn<32, 2, 64>(a, x, st);
    case 64164: return launch_kxn<64, 1, 64>(a, x, st);
    case 32116: return launch_kxn<32, 1, 16>(a, x, st);
    case 32216: return launch_kxn<32, 2, 16>(a, x, st);
    case 64116: return launch_kxn<64, 1, 16>(a, x, st);
    default: return YK_EINVAL;
  }
}

}  // namespace yk
