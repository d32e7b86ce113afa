// 3x3 stride-1 convolution on tcgen05 with halo patches: each input element crosses from L2
// into shared memory about 1.3-1.4 times instead of 9 times.  Channel blocks (CB) are 64
// channels (128-byte rows, 128-byte swizzle) or, for the transposed tiles of inputs whose
// channel count is a multiple of 32 only, 32 channels (64-byte rows, 64-byte swizzle); the
// text below says 64.
//
// The CTA tile is MT sub-tiles of 8 x 16 output positions (one 128-row UMMA operand each),
// stacked vertically, of which the first 14 columns are real outputs (the last two of each
// row are computed and dropped).  One 4-D TMA box {64 channels, 16 columns, 8*MT + 2 rows,
// 1 image}, starting one row and one column before the tile (the image border reads as
// zero), brings the tile's whole input window for a 64-channel block into shared memory,
// 128-byte swizzled rows of 64 channels, one row per input position.  Because the window's
// row pitch (16 positions) equals the output patch's, the A operand of filter tap (ky, kx)
// is the window itself shifted by ky*16 + kx positions: nine UMMA descriptors over one
// load, no im2col.  Weights ([Cout][ky][kx][Cin], K-major per tap) stream through a ring of
// per-tap stages as in conv_tc.cu.  Roles, TMEM ring, bounded waits and the epilogue follow
// conv_tc.cu; the epilogue maps accumulator row r to patch (r / 16, r % 16).
#include "common.cuh"

namespace yk {

struct PatchArgs {
  const __half* x;  // unused on the device (the tensor map carries it); kept for checks
  int H, W;
  __half* y;
  int ys;
  const __half* res;
  int rs;
  const __half* w;  // [Cout][3][3][Cin]
  const float* bias;
  int Cin, Cout, act;
  int ncb;          // 64-channel blocks of Cin
  int nty, ntx;     // patch tiles per image (rows of 8*MT, columns of 14)
  int ntn, ntiles;
  int tma_epi;      // kx-folded kernel: residual in / output out by 4-D TMA boxes (0 = direct)
};

constexpr int kPatchCols = 16;     // positions per patch row (row pitch)
constexpr int kPatchUse = 14;      // real output columns per patch row

template <int BN, int MT, int BST, int WST, bool T = false, int CB = 64>
struct PatchCfg {
  static constexpr int kRows = 8 * MT + 2;                        // window rows
  static constexpr int kRB = CB * 2;                              // bytes per position row
  static constexpr int kWinTx = kRows * kPatchCols * kRB;         // bytes one TMA box brings
  // The junk columns of the last window row read 2 positions past the box: inside the next
  // buffer (the next window or the weight ring), so no padding is needed.
  static constexpr int kWin = (kWinTx + 1023) & ~1023;
  static constexpr int kB = BN * kRB;                             // one tap's weights, CB ch
  static constexpr int kAccCols = BN;
  // transposed tiles: one accumulator of 128*MT columns (positions) x BN lanes (channels)
  static constexpr int kTileCols = T ? 128 * MT : MT * BN;
  static constexpr int kNacc = 512 / kTileCols >= 4 ? 4 : 2;
  static constexpr int kTmemCols = kNacc * kTileCols;
  // transposed: per epilogue warp a [32 positions][32 or 16 channels] fp16 staging block and
  // no bias cache (each lane holds its channel's bias); otherwise the bias cache
  static constexpr int kStg = T ? 8 * 32 * (BN == 128 ? 32 : 16) * 2 : kBiasSmem * 4;
  static constexpr int kBars = 512;   // mbarriers, TMEM slot, abort flag
  static_assert(8 * (2 * WST + 2 * BST + 2 * kNacc) + 16 <= kBars, "barrier area");
  static constexpr size_t kSmem = (size_t)WST * kWin + (size_t)BST * kB + 1024 + kBars + kStg;
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert((size_t)WST * kWin + (size_t)BST * kB + 1024 + kBars + kStg <= 232448,
                "smem budget");
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c, int x, int y, int n) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c), "r"(x), "r"(y), "r"(n)
      : "memory");
}
// 4-D tiled bulk store shared -> global (coordinates: channel, x, y, image; the store clips
// elements past the tensor map's extents).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c, int x,
                                             int y, int n) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          (uint64_t)map),
      "r"(src), "r"(c), "r"(x), "r"(y), "r"(n)
      : "memory");
}

template <int BN, int MT, int BST, int WST, int G, bool T, int CB>
__global__ void __launch_bounds__(kThreads, 1)
conv_patch_kernel(const PatchArgs a, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmX) {
  using Cfg = PatchCfg<BN, MT, BST, WST, T, CB>;
  constexpr int kRB = Cfg::kRB;
  static_assert(CB == 64 || CB == 32, "64- or 32-channel blocks");
  static_assert(!T || BN == 64 || BN == 128, "transposed tiles: 64 or 128 channels");
  static_assert(BST % G == 0 && BST / G >= 2, "weight stage groups");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t wbase = base, bbase = base + WST * Cfg::kWin;
  const uint32_t bar_base = bbase + BST * Cfg::kB;
  // barriers: wfull[WST], wempty[WST], bfull[BST], bempty[BST], tfull[NACC], tempty[NACC]
  auto wfull = [&](int s) { return bar_base + 8u * s; };
  auto wempty = [&](int s) { return bar_base + 8u * (WST + s); };
  auto bfull = [&](int s) { return bar_base + 8u * (2 * WST + s); };
  auto bempty = [&](int s) { return bar_base + 8u * (2 * WST + BST + s); };
  auto tfull = [&](int b) { return bar_base + 8u * (2 * WST + 2 * BST + b); };
  auto tempty = [&](int b) { return bar_base + 8u * (2 * WST + 2 * BST + Cfg::kNacc + b); };
  const uint32_t tslot = bar_base + 8u * (2 * WST + 2 * BST + 2 * Cfg::kNacc);
  volatile uint32_t* tslot_ptr = (volatile uint32_t*)(smem_raw + (tslot - raw));
  volatile int* abort_flag = (volatile int*)(smem_raw + (tslot - raw) + 8);
  float* bias_s = (float*)(smem_raw + (bar_base - raw) + Cfg::kBars);   // plain tiles
  __half* stg_s = (__half*)(smem_raw + (bar_base - raw) + Cfg::kBars);   // transposed tiles
  // G == 9: the weight stages of a window are its 9 taps in slots 9*ws .. 9*ws+8, released
  // with the window by one commit (the ring holds BST = 9*WST stages)
  constexpr bool kFused = G == 9;
  static_assert(!kFused || BST == 9 * WST, "fused weight stages");

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < WST; s++) { mbar_init(wfull(s), 1); mbar_init(wempty(s), 1); }
    for (int s = 0; s < BST; s++) {
      mbar_init(bfull(s), 1);
      if (s < BST / G) mbar_init(bempty(s), 1);
    }
    for (int b = 0; b < Cfg::kNacc; b++) { mbar_init(tfull(b), 1); mbar_init(tempty(b), kEpiGroup); }
    *abort_flag = 0;
    mbar_fence_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmB) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&tmX) : "memory");
  }
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
  const int per_img = a.nty * a.ntx;
  const long long t_role = clock64();

  if (warp == 0) {
    // ---------------- producer (one thread, all loads by TMA) ----------------
    if (tid == 0) {
      uint32_t gw = 0, gb = 0;
      for (int t = blockIdx.x; t < a.ntiles && !*abort_flag; t += gridDim.x) {
        const int mtile = t / a.ntn, n0 = (t - mtile * a.ntn) * BN;
        const int img = mtile / per_img, r = mtile - img * per_img;
        const int ty = r / a.ntx, tx = r - ty * a.ntx;
        bool ok = true;
        for (int cb = 0; cb < a.ncb && ok; cb++, gw++) {
          const int ws = gw % WST;
          const uint32_t uw = gw / WST;
          if (uw > 0 && !mbar_wait(wempty(ws), (uw - 1) & 1, 0x201)) { ok = false; break; }
          mbar_expect_tx(wfull(ws), Cfg::kWinTx);
          tma_load_4d(wbase + ws * Cfg::kWin, &tmX, wfull(ws), cb * CB, tx * kPatchUse - 1,
                      ty * 8 * MT - 1, img);
          for (int tap = 0; tap < 9; tap++, gb++) {
            const int bs = kFused ? ws * 9 + tap : gb % BST;
            const uint32_t ub = gb / BST;
            // weight stages are released G at a time (one tcgen05.commit per group)
            if (!kFused && ub > 0 && bs % G == 0 &&
                !mbar_wait(bempty(bs / G), (ub - 1) & 1, 0x202)) {
              ok = false;
              break;
            }
            mbar_expect_tx(bfull(bs), Cfg::kB);
            tma_load_2d(bbase + bs * Cfg::kB, &tmB, bfull(bs), tap * a.Cin + cb * CB, n0);
          }
        }
        if (!ok) { *abort_flag = 1; break; }
      }
      YK_PROF_ADD(10, clock64() - t_role);
    }
  } else if (warp >= 4 && warp < kMmaWarp && T) {
    // ---------------- epilogue, transposed tiles ----------------
    // TMEM column = window position (sub-tile position + 128*mt), lane = output channel: for
    // 128 channels lane = channel, for 64 channels (M = 64 MMA) channel c sits in lane
    // 32*(c/16) + c%16, so each warp owns 16 channels in its lanes 0-15.  Per 32 positions
    // (two patch rows): bias + SiLU per lane, fp16 into the warp's [position][channel]
    // staging block, then 16-byte rows of 8 channels stored for the real output pixels.
    constexpr int kCw = BN == 128 ? 32 : 16;    // channels per warp
    const int sp = warp & 3, grp = (warp - 4) >> 2;
    __half* stg = stg_s + (warp - 4) * 32 * kCw;   // kStg = 8 warps x 32 x kCw halves
    const bool lane_ok = lane < kCw;
    uint32_t li = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, li++) {
      if ((int)(li & 1) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (!mbar_wait(tfull(acc), use & 1, 0x203)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int mtile = t / a.ntn, n0 = (t - mtile * a.ntn) * BN;
      const int img = mtile / per_img, r = mtile - img * per_img;
      const int ty = r / a.ntx, tx = r - ty * a.ntx;
      const int cw0 = n0 + sp * kCw;                 // first channel of this warp
      const int ch = cw0 + lane;
      const float bc = lane_ok && ch < a.Cout ? a.bias[ch] : 0.f;
      const uint32_t tcol = tmem + ((uint32_t)(sp * 32) << 16) + acc * Cfg::kTileCols;
      const bool any_ch = cw0 < a.Cout;              // uniform
#pragma unroll 1
      for (int pc = 0; pc < MT * 4 && any_ch; pc++) {   // 32 positions per chunk
        uint32_t rg[32];
        tmem_ld16p(tcol + pc * 32, rg);
        tmem_ld16p(tcol + pc * 32 + 16, rg + 16);
        tmem_ld_wait();
        if (lane_ok) {
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const __half2 h = bias_act2(
                make_float2(__uint_as_float(rg[k]), __uint_as_float(rg[k + 1])),
                make_float2(bc, bc), a.act);
            stg[k * kCw + lane] = __low2half(h);
            stg[(k + 1) * kCw + lane] = __high2half(h);
          }
        }
        __syncwarp();
        constexpr int kChunks = 32 * kCw / 8;          // 16-byte pieces in the block
#pragma unroll
        for (int i = 0; i < kChunks / 32; i++) {
          const int q = lane + 32 * i, pos = q / (kCw / 8), cc = q % (kCw / 8);
          const int gpos = pc * 32 + pos;               // position within the tile
          const int mt = gpos >> 7, pr = (gpos & 127) >> 4, pcol = gpos & 15;
          const int y = ty * 8 * MT + mt * 8 + pr, x = tx * kPatchUse + pcol;
          const int c8 = cw0 + cc * 8;
          if (pcol < kPatchUse && x < a.W && y < a.H && c8 < a.Cout) {
            const size_t m = ((size_t)img * a.H + y) * a.W + x;
            uint4 o = *(const uint4*)(stg + pos * kCw + cc * 8);
            if (a.res) {
              const uint4 rv = *(const uint4*)(a.res + m * a.rs + c8);
              __half2* oh = (__half2*)&o;
              const __half2* rh = (const __half2*)&rv;
#pragma unroll
              for (int e = 0; e < 4; e++) {
                const float2 f = __half22float2(oh[e]), g2 = __half22float2(rh[e]);
                oh[e] = __floats2half2_rn(f.x + g2.x, f.y + g2.y);
              }
            }
            *(uint4*)(a.y + m * a.ys + c8) = o;
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(tempty(acc));
    }
    if (lane == 0) YK_PROF_ADD(9, clock64() - t_role);
  } else if (warp >= 4 && warp < kMmaWarp) {
    // ---------------- epilogue ----------------
    const int sp = warp & 3;
    const int grp = (warp - 4) >> 2;
    const int row = sp * 32 + lane;
    const int pr = row >> 4, pc = row & 15;
    const bool bias_cached = a.Cout <= kBiasSmem;
    if (bias_cached)
      for (int i = tid - 128; i < a.Cout; i += 256) bias_s[i] = a.bias[i];
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float* bias = bias_cached ? bias_s : a.bias;
    uint32_t li = 0;
    for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x, li++) {
      if ((int)(li & 1) != grp) continue;
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (!mbar_wait(tfull(acc), use & 1, 0x203)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int mtile = t / a.ntn, n0 = (t - mtile * a.ntn) * BN;
      const int img = mtile / per_img, r = mtile - img * per_img;
      const int ty = r / a.ntx, tx = r - ty * a.ntx;
      const int x = tx * kPatchUse + pc;
#pragma unroll 1
      for (int mt = 0; mt < MT; mt++) {
        const int y = ty * 8 * MT + mt * 8 + pr;
        const bool mok = pc < kPatchUse && x < a.W && y < a.H;
        const size_t m = mok ? ((size_t)img * a.H + y) * a.W + x : 0;
        __half* yrow = a.y + m * a.ys;
        const __half* rrow = a.res ? a.res + m * a.rs : nullptr;
        const uint32_t trow = tmem + ((uint32_t)(sp * 32) << 16) + acc * Cfg::kTileCols +
                              mt * Cfg::kAccCols;
        epi_row<BN>(trow, n0, a.Cout, mok, yrow, rrow, bias, a.act);
      }
      tc_fence_before();
      mbar_arrive(tempty(acc));
    }
  } else if (warp == kMmaWarp && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = idesc_f16_m128(BN);
    uint32_t gw = 0, gb = 0, li = 0;
    for (int t = blockIdx.x; t < a.ntiles && !*abort_flag; t += gridDim.x, li++) {
      const int acc = li % Cfg::kNacc;
      const uint32_t use = li / Cfg::kNacc;
      if (use > 0 && !mbar_wait(tempty(acc), (use - 1) & 1, 0x204)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t d = tmem + acc * Cfg::kTileCols;
      bool ok = true;
      for (int cb = 0; cb < a.ncb && ok; cb++, gw++) {
        const int ws = gw % WST;
        if (!mbar_wait(wfull(ws), (gw / WST) & 1, 0x205)) { ok = false; break; }
        tc_fence_after();
        const uint32_t win = wbase + ws * Cfg::kWin;
        for (int tap = 0; tap < 9; tap++, gb++) {
          const int bs = kFused ? ws * 9 + tap : gb % BST;
          const uint32_t bpar = kFused ? (gw / WST) & 1 : (gb / BST) & 1;
          if (!mbar_wait(bfull(bs), bpar, 0x206)) { ok = false; break; }
          tc_fence_after();
          const int ky = tap / 3, kx = tap - ky * 3;
          const uint32_t sb = bbase + bs * Cfg::kB;
          if constexpr (T) {
            // transposed: A = BN weight rows (channels), B = 128*MT window positions from
            // the tap's shift (sub-tiles are 128 positions apart, so one operand covers all)
            constexpr uint32_t idt = (1u << 4) | ((uint32_t)((128 * MT) >> 3) << 17) |
                                     ((uint32_t)(BN >> 4) << 24);
#pragma unroll
            for (int kk = 0; kk < CB / 16; kk++) {
              const uint32_t sa = win + (uint32_t)((ky * kPatchCols + kx) * kRB + kk * 32);
              tc_mma_f16(d, swz_desc<kRB>(sb + kk * 32), swz_desc<kRB>(sa), idt,
                         (cb | tap | kk) != 0);
            }
          } else
#pragma unroll
          for (int kk = 0; kk < CB / 16; kk++)
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
              // the swizzle follows the absolute shared-memory address, so a start shifted
              // by whole rows needs no base offset in the descriptor
              const uint32_t sa =
                  win + (uint32_t)(((mt * 8 + ky) * kPatchCols + kx) * kRB + kk * 32);
              tc_mma_f16(d + mt * Cfg::kAccCols, swz_desc<kRB>(sa), swz_desc<kRB>(sb + kk * 32),
                         idesc, (cb | tap | kk) != 0);
            }
          if (!kFused && bs % G == G - 1) tc_commit(bempty(bs / G));
        }
        if (ok) tc_commit(wempty(ws));
      }
      if (!ok) { *abort_flag = 1; break; }
      tc_commit(tfull(acc));
    }
    YK_PROF_ADD(8, clock64() - t_role);
    YK_PROF_ADD(11, 1);
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// 4-D tiled map over the NHWC input view {C, W, H, N}: box {64, 16, rows, 1}, 128-byte
// swizzle; coordinates outside the image (the 1-pixel border) read as zero.
static bool encode_patch_x(CUtensorMap* m, const __half* x, int C, int W, int H, int N,
                           int xs, int rows, int cb) {
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
  const cuuint64_t strides[3] = {(cuuint64_t)xs * 2, (cuuint64_t)W * xs * 2,
                                 (cuuint64_t)H * W * xs * 2};
  const cuuint32_t box[4] = {(cuuint32_t)cb, (cuuint32_t)kPatchCols, (cuuint32_t)rows, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(x), dims, strides,
                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_of(cb),
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int MT, int BST, int WST, int G, bool T = false, int CB = 64>
static int launch_patch(const PatchArgs& a, const YkView* x, cudaStream_t st) {
  using Cfg = PatchCfg<BN, MT, BST, WST, T, CB>;
  if (smem_attr(conv_patch_kernel<BN, MT, BST, WST, G, T, CB>, (int)Cfg::kSmem) != cudaSuccess) return check_launch("conv_patch attr");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return YK_EUNSUP;
  if (!g_num_sms[dev]) cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.ntiles < g_num_sms[dev] ? a.ntiles : g_num_sms[dev];
  CUtensorMap tmB, tmX;
  if (!encode_2d(&tmB, a.w, (uint64_t)9 * a.Cin, (uint64_t)a.Cout, (uint64_t)9 * a.Cin * 2, BN, CB))
    return YK_EUNSUP;
  if (!encode_patch_x(&tmX, a.x, a.Cin, a.W, a.H, x->batch, x->stride, Cfg::kRows, CB))
    return YK_EUNSUP;
  launch_k(conv_patch_kernel<BN, MT, BST, WST, G, T, CB>, grid, kThreads, Cfg::kSmem, st, a, tmB, tmX);
  note_launch();
  return check_launch("conv_patch");
}

// Halo-patch 3x3 stride-1 pad-1 conv; Cin a multiple of 64, 16-byte aligned view.
// bn in {64, 128, 256}, ms (stacked 8x16 sub-tiles) in {1, 2}.
int conv_patch(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, int bn,
               int ms, bool trans, cudaStream_t st) {
  // 64-channel blocks when Cin allows them; 32-channel blocks (transposed tiles) otherwise
  const int cbw = p->Cin % 64 == 0 ? 64 : p->Cin % 32 == 0 ? 32 : 0;
  if (p->k != 3 || p->s != 1 || p->p != 1 || p->groups != 1 || !cbw ||
      ((uintptr_t)x->ptr & 15) || x->stride % 8 || (x->coff % 8))
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
  a.ncb = p->Cin / cbw;
  a.nty = (x->H + 8 * ms - 1) / (8 * ms);
  a.ntx = (x->W + kPatchUse - 1) / kPatchUse;
  a.ntn = (p->Cout + bn - 1) / bn;
  const long long nt = (long long)y->batch * a.nty * a.ntx * a.ntn;
  if (nt > 0x7fffffffLL) return YK_EUNSUP;
  a.ntiles = (int)nt;
  if (trans && cbw == 32) {
    switch (bn * 10 + ms) {
      case 641: return launch_patch<64, 1, 18, 2, 9, true, 32>(a, x, st);
      case 642: return launch_patch<64, 2, 18, 2, 9, true, 32>(a, x, st);
      case 1281: return launch_patch<128, 1, 6, 3, 3, true, 32>(a, x, st);
      case 1282: return launch_patch<128, 2, 6, 2, 3, true, 32>(a, x, st);
      default: return YK_EINVAL;
    }
  }
  if (trans) {
    switch (bn * 10 + ms) {
      case 641: return launch_patch<64, 1, 18, 2, 9, true>(a, x, st);
      case 642: return launch_patch<64, 2, 18, 2, 9, true>(a, x, st);
      case 1281: return launch_patch<128, 1, 6, 3, 3, true>(a, x, st);
      case 1282: return launch_patch<128, 2, 6, 2, 3, true>(a, x, st);
      default: return YK_EINVAL;
    }
  }
  if (cbw == 32) {
    switch (bn * 10 + ms) {
      case 321: return launch_patch<32, 1, 18, 2, 9, false, 32>(a, x, st);
      case 322: return launch_patch<32, 2, 18, 2, 9, false, 32>(a, x, st);
      case 641: return launch_patch<64, 1, 18, 2, 9, false, 32>(a, x, st);
      case 642: return launch_patch<64, 2, 18, 2, 9, false, 32>(a, x, st);
      default: return YK_EINVAL;
    }
  }
  switch (bn * 10 + ms) {
    case 321: return launch_patch<32, 1, 18, 2, 9>(a, x, st);
    case 322: return launch_patch<32, 2, 18, 2, 9>(a, x, st);
    case 641: return launch_patch<64, 1, 6, 3, 3>(a, x, st);
    case 642: return launch_patch<64, 2, 6, 2, 3>(a, x, st);
    case 1281: return launch_patch<128, 1, 6, 3, 3>(a, x, st);
    case 1282: return launch_patch<128, 2, 6, 2, 3>(a, x, st);
    case 2561: return launch_patch<256, 1, 4, 3, 2>(a, x, st);
    default: return YK_EINVAL;
  }
}

}  // namespace yk
