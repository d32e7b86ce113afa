// Pre- and post-processing: letterbox, DFL decode, exact NMS, segment masks.
//
// Everything here computes with the explicitly rounded fp32 operations of detmath.h, so a
// host restatement built from the same formulas reproduces it bit for bit: candidate
// lists, survivor indices and boxes are deterministic and independent of thread timing
// (the reference appends candidates with atomicAdd and truncates NMS input at 1024 in that
// order, engine/engine.cu:890, 1064).
#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "detmath.h"

namespace yk {

// ---------------- letterbox (engine/engine.cu:968-998) ----------------
// One launch letterboxes a batch of equal-size frames: grid (row blocks, frames), `rows`
// output rows per block (1 for a single frame, up to 4 for a batch, so the grid fills the
// GPU).  The block first copies the two source rows each of its output rows samples into
// shared memory with 16-byte cp.async copies (rows outside the image band are skipped), then
// every thread computes whole output pixels, consecutive lanes on consecutive pixels, so the
// shared-memory byte reads of a warp fall on neighbouring bytes and its fp16 stores on one
// contiguous span.  The arithmetic is the reference's formula in explicitly rounded fp32
// (src = (dst - off + 0.5) / scale - 0.5, bilinear weights, /255, pad 114); /255 is
// dm_div255 (bit-identical to the division), so the C oracle reproduces every value.
constexpr int kLbMaxRows = 4;

__device__ __forceinline__ int lb_src_row(int y, int top, float scale, int sh, int which) {
  const float fy = DM_SUB(DM_DIV(DM_ADD((float)(y - top), 0.5f), scale), 0.5f);
  const int y0 = (int)floorf(fy);
  return which ? min(y0 + 1, sh - 1) : max(y0, 0);
}

// A byte as a float, exactly: 2^23 + b has b in its low mantissa bits, and the subtraction
// of 2^23 is exact.
__device__ __forceinline__ float lb_u8f(uint32_t b) {
  return __fsub_rn(__uint_as_float(0x4B000000u | b), 8388608.f);
}

__global__ void __launch_bounds__(256) letterbox_kernel(
    const uint8_t* __restrict__ src, size_t src_frame, int sh, int sw, __half* dst,
    size_t dst_frame, int dh, int dw, int dstride, float scale, int top, int left, int nh,
    int nw, int rows, int pitch) {
  extern __shared__ __align__(16) uint8_t lb_rows[];   // [2 * rows][pitch]
  pdl_wait();     // the destination may still be read by the previous graph's kernels
  pdl_trigger();
  const uint8_t* img = src + (size_t)blockIdx.y * src_frame;
  __half* out = dst + (size_t)blockIdx.y * dst_frame;
  const int y_beg = blockIdx.x * rows, nrow = min(rows, dh - y_beg);
  const int rb = sw * 3;
  // stage: slot 2r / 2r + 1 hold the upper / lower source row of output row y_beg + r; a
  // slot starts at the 16-byte boundary at or below its row, `shift` bytes before it
  for (int slot = threadIdx.y; slot < 2 * nrow; slot += blockDim.y) {
    const int y = y_beg + (slot >> 1);
    if (y < top || y >= top + nh) continue;
    const uint8_t* row = img + (size_t)lb_src_row(y, top, scale, sh, slot & 1) * rb;
    const uintptr_t a0 = (uintptr_t)row & ~(uintptr_t)15, end = (uintptr_t)row + rb;
    uint8_t* s = lb_rows + slot * pitch;
    const int nvec = (int)((end - a0) >> 4);           // whole 16-byte words inside the row
    // asynchronous copies, all of the block's words in flight at once (the head word may
    // start before the row: the aligned word holding the row's first byte lies inside the
    // same allocation, and the bytes before the row are never read from shared memory)
    for (int i = threadIdx.x; i < nvec; i += blockDim.x)
      cp_async16(smem_u32(s + i * 16), (const void*)(a0 + ((uintptr_t)i << 4)), 16u);
    // bytes past the last whole word (all of a row shorter than one word), never before it
    const uintptr_t t0 = max(a0 + ((uintptr_t)nvec << 4), (uintptr_t)row);
    for (uintptr_t p = t0 + threadIdx.x; p < end; p += blockDim.x)
      s[p - a0] = __ldg((const uint8_t*)p);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  const __half pad = __float2half_rn(dm_div255(114.f));
  const int tid = threadIdx.y * blockDim.x + threadIdx.x, nthr = blockDim.x * blockDim.y;
  // per-row terms (the vertical weight and the staged source rows), computed once
  float wyr[kLbMaxRows], wy1r[kLbMaxRows];
  const uint8_t* s0r[kLbMaxRows];
  const uint8_t* s1r[kLbMaxRows];
  bool inr[kLbMaxRows];
#pragma unroll
  for (int r = 0; r < kLbMaxRows; r++) {
    const int y = y_beg + r;
    inr[r] = r < nrow && y >= top && y < top + nh;
    float wy = 0.f;
    int sh0 = 0, sh1 = 0;
    if (inr[r]) {
      const float fy = DM_SUB(DM_DIV(DM_ADD((float)(y - top), 0.5f), scale), 0.5f);
      wy = DM_SUB(fy, floorf(fy));
      sh0 = (int)((uintptr_t)(img + (size_t)lb_src_row(y, top, scale, sh, 0) * rb) & 15);
      sh1 = (int)((uintptr_t)(img + (size_t)lb_src_row(y, top, scale, sh, 1) * rb) & 15);
    }
    wyr[r] = wy;
    wy1r[r] = DM_SUB(1.f, wy);
    s0r[r] = lb_rows + (2 * r) * pitch + sh0;
    s1r[r] = lb_rows + (2 * r + 1) * pitch + sh1;
  }
  // Column-major walk: the horizontal terms of a column (a division, a floor and two
  // float/int conversions) are computed once and serve every row of the block, and source
  // bytes become floats by an exact integer-or / subtract on the ALU and FMA pipes instead
  // of the conversion unit, which bounded the row-major version.
  for (int x = tid; x < dw; x += nthr) {
    const bool col_in = x >= left && x < left + nw;
    float wx = 0.f, wx1 = 1.f;
    int x0 = 0, x1 = 0;
    if (col_in) {
      const float fx = DM_SUB(DM_DIV(DM_ADD((float)(x - left), 0.5f), scale), 0.5f);
      x0 = (int)floorf(fx);
      wx = DM_SUB(fx, (float)x0);
      x1 = min(x0 + 1, sw - 1) * 3;
      x0 = max(x0, 0) * 3;
      wx1 = DM_SUB(1.f, wx);
    }
#pragma unroll
    for (int r = 0; r < kLbMaxRows; r++) {
      if (r >= nrow) break;
      __half o0 = pad, o1 = pad, o2 = pad;
      if (inr[r] && col_in) {
        // tap weights: upper-left, upper-right, lower-left, lower-right
        const float wul = DM_MUL(wy1r[r], wx1), wur = DM_MUL(wy1r[r], wx);
        const float wll = DM_MUL(wyr[r], wx1), wlr = DM_MUL(wyr[r], wx);
        const uint8_t* up = s0r[r];
        const uint8_t* lo = s1r[r];
        float v[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
          float acc = DM_MUL(lb_u8f(up[x0 + c]), wul);
          acc = DM_ADD(acc, DM_MUL(lb_u8f(up[x1 + c]), wur));
          acc = DM_ADD(acc, DM_MUL(lb_u8f(lo[x0 + c]), wll));
          v[c] = DM_ADD(acc, DM_MUL(lb_u8f(lo[x1 + c]), wlr));
        }
        // BGR in, RGB out
        o0 = __float2half_rn(dm_div255(v[2]));
        o1 = __float2half_rn(dm_div255(v[1]));
        o2 = __float2half_rn(dm_div255(v[0]));
      }
      __half* o = out + ((size_t)(y_beg + r) * dw + x) * dstride;
      o[0] = o0;
      o[1] = o1;
      o[2] = o2;
    }
  }
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

// Per-image workspace layout (all 16-byte aligned): rec[A][6] f32 and flag[A] i32 from
// decode; then the NMS candidate arrays, used in place of shared memory when an image has
// more candidates than shared memory holds: anchor[A] u32, box[A] float4, skey[A] u32,
// cls[A] u32, ord[3][A] u32, surv[A] u8; kept[A][5] f32 (kept boxes past the shared cache).
struct WsLayout {
  size_t rec, flag, anch, box, skey, cls, ord, surv, kept, bmask, per_img;
  int A, bmask_words;
};
constexpr int kBitMax = 512;   // classes of kBitMin+1..kBitMax candidates: bit-mask suppression
// Below that the greedy loop is cheaper: real detections suppress heavily, and its cost
// follows the kept boxes, while the masks cost every pair (yolo11n, 268 candidates in four
// classes, 16 kept: 24 us of masks and scan against a few us of greedy).
constexpr int kBitMin = 128;
// With a cluster of 4 or more CTAs per image the rows are built by 128+ warps, so smaller
// classes pay for masks too.
#ifndef YK_NMS_BITMIN_CLUSTER
#define YK_NMS_BITMIN_CLUSTER 32
#endif
constexpr int kBitMinCluster = YK_NMS_BITMIN_CLUSTER;
static inline size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }
static inline WsLayout ws_layout(int A) {
  WsLayout L;
  size_t o = 0;
  L.A = A;
  L.rec = o;  o = al16(o + (size_t)A * 6 * 4);
  L.flag = o; o = al16(o + (size_t)A * 4);
  L.anch = o; o = al16(o + (size_t)A * 4);
  L.box = o;  o = al16(o + (size_t)A * 16);
  L.skey = o; o = al16(o + (size_t)A * 4);
  L.cls = o;  o = al16(o + (size_t)A * 4);
  L.ord = o;  o = al16(o + (size_t)A * 12);
  L.surv = o; o = al16(o + (size_t)A);
  L.kept = o; o = al16(o + (size_t)A * 5 * 4);
  // bit masks of the mid-size classes: up to 16 words per candidate, at most 128 KB
  L.bmask_words = (int)std::min<size_t>((size_t)A * 16, 32768);
  L.bmask = o; o = al16(o + (size_t)L.bmask_words * 4);
  L.per_img = o;
  return L;
}

// Anchor -> (level, y, x) and its element offsets in the level's views.
struct AnchorLoc {
  int li, y, x;
};
__device__ __forceinline__ AnchorLoc locate(const DevLevels& lv, int a) {
  int li = 0;
  while (li + 1 < lv.n && a >= lv.l[li + 1].abase) li++;
  const int rem = a - lv.l[li].abase;
  const int y = rem / lv.l[li].W;
  return {li, y, rem - y * lv.l[li].W};
}

// One 4-lane group per anchor.  Class scores: the lanes take interleaved 16-byte chunks of
// the logits and reduce (max, then the lowest class index: the reference's first-max-wins
// scan).  For a candidate, lane k runs the DFL expectation of box side k, so all four lanes
// share the 64 exponentials.
__global__ void __launch_bounds__(256) decode_kernel(DevLevels lv, int batch, int nc, float conf,
                                                     uint8_t* ws, WsLayout L) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  const long long ga = (long long)blockIdx.x * (blockDim.x >> 2) + (threadIdx.x >> 2);
  if (ga >= (long long)batch * lv.A) return;   // whole 4-lane groups leave together
  const int sub = threadIdx.x & 3, g0 = threadIdx.x & 28;
  const unsigned gm = 0xfu << g0;
  const int img = (int)(ga / lv.A), a = (int)(ga - (long long)img * lv.A);
  const AnchorLoc p = locate(lv, a);
  const DevLevel& L0 = lv.l[p.li];
  uint8_t* wimg = ws + (size_t)img * L.per_img;
  const __half* cp = L0.cls.p + L0.cls.pix(img, p.y, p.x);
  float best = -INFINITY;
  int bcls = 0;
  // the first 128 classes: every 16-byte load of the lane is issued before the first
  // compare, so an anchor costs one memory latency, not one per word
  constexpr int kPre = 4;
  uint4 cv[kPre];
#pragma unroll
  for (int k = 0; k < kPre; k++)
    if (sub * 8 + 32 * k < nc) cv[k] = *(const uint4*)(cp + sub * 8 + 32 * k);
#pragma unroll
  for (int k = 0; k < kPre; k++) {
    const int c0 = sub * 8 + 32 * k;
    if (c0 >= nc) break;
    const __half* h = (const __half*)&cv[k];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float f = __half2float(h[i]);
      if (c0 + i < nc && f > best) { best = f; bcls = c0 + i; }   // first max wins
    }
  }
  for (int c0 = sub * 8 + 32 * kPre; c0 < nc; c0 += 32) {
    const uint4 v = *(const uint4*)(cp + c0);
    const __half* h = (const __half*)&v;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float f = __half2float(h[i]);
      if (c0 + i < nc && f > best) { best = f; bcls = c0 + i; }
    }
  }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    const float ob = __shfl_xor_sync(gm, best, o);
    const int oc = __shfl_xor_sync(gm, bcls, o);
    if (ob > best || (ob == best && oc < bcls)) { best = ob; bcls = oc; }
  }
  int* flag = (int*)(wimg + L.flag);
  const float score = dm_sigmoid(best);
  if (!(score >= conf)) {
    if (sub == 0) flag[a] = 0;
    return;
  }
  const __half* bp = L0.box.p + L0.box.pix(img, p.y, p.x) + sub * 16;
  const uint4 v0 = *(const uint4*)bp, v1 = *(const uint4*)(bp + 8);
  const __half* h0 = (const __half*)&v0;
  const __half* h1 = (const __half*)&v1;
  float l[16];
#pragma unroll
  for (int i = 0; i < 8; i++) { l[i] = __half2float(h0[i]); l[i + 8] = __half2float(h1[i]); }
  const float d = dm_dfl16(l);
  const float d0 = __shfl_sync(gm, d, g0), d1 = __shfl_sync(gm, d, g0 + 1);
  const float d2 = __shfl_sync(gm, d, g0 + 2), d3 = __shfl_sync(gm, d, g0 + 3);
  if (sub != 0) return;
  const float cx = DM_ADD((float)p.x, 0.5f), cy = DM_ADD((float)p.y, 0.5f), st = (float)L0.stride;
  float* o = (float*)(wimg + L.rec) + (size_t)a * 6;
  o[0] = DM_MUL(DM_SUB(cx, d0), st);
  o[1] = DM_MUL(DM_SUB(cy, d1), st);
  o[2] = DM_MUL(DM_ADD(cx, d2), st);
  o[3] = DM_MUL(DM_ADD(cy, d3), st);
  o[4] = score;
  o[5] = (float)bcls;
  flag[a] = 1;
}

// ---------------- NMS (engine/engine.cu:1051-1123, exact + deterministic) ----------------
// Order of work, one 1024-thread block per image:
//   1. compaction of the decode flags into the candidate list (anchor order);
//   2. a stable sort by score (descending; anchor order breaks ties) and, from that, a stable
//      sort by class: a rank sort for small lists, LSD radix passes (8-bit digits, only the
//      bytes that vary) otherwise;
//   3. greedy suppression per class, one warp per class, 32 candidates per step;
//   4. survivors in score order, the first max_out written out.
// Up to kNmsSmemCand candidates live in shared memory, more in the workspace.
// An image may own a cluster of `csize` CTAs (distributed shared memory): with the
// candidates in shared memory every CTA runs steps 1-2 on its own copy (the same work, the
// same result), otherwise CTA 0 alone sorts in the workspace; step 3 is shared out, the bit-mask rows
// over all warps of the cluster and the classes round-robin over the CTAs (class s to CTA
// s mod csize), the survivor flags going to CTA 0, which alone runs step 4.  A batch that
// leaves SMs idle (batch 1: one SM of 148) thus spreads its pair tests over up to 8 SMs.
constexpr int kNmsThreads = 1024;
// Diagnostic builds (-DYK_NMS_PROF) record %globaltimer at each phase boundary of image 0.
#ifdef YK_NMS_PROF
__device__ unsigned long long g_nms_prof[8];
#define NMS_MARK(i) do { if (blockIdx.x == 0 && threadIdx.x == 0) g_nms_prof[i] = globaltimer(); } while (0)
extern "C" int yk_nms_prof(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_nms_prof, sizeof g_nms_prof) == cudaSuccess ? 0 : -1;
}
#else
#define NMS_MARK(i) ((void)0)
#endif
constexpr int kNmsSmemCand = 4096;
constexpr int kRankSortMax = 512;
constexpr int kMaxClasses = 1024;
constexpr int kKeptSmem = 32;          // kept boxes per class held in shared memory
constexpr int kHistStride = 33;        // per-warp digit counters, [digit][warp] padded
constexpr size_t kNmsDynSmem = (size_t)kNmsSmemCand * (16 + 4 + 4 + 12 + 1) + 256 * kHistStride * 4;

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

// Lanes of the warp (among those in `valid`) whose 8-bit digit equals this lane's: the
// intersection over the 8 bits of the ballot of lanes agreeing on that bit.
__device__ __forceinline__ unsigned digit_peers(unsigned d, unsigned valid) {
  unsigned m = valid;
#pragma unroll
  for (int b = 0; b < 8; b++) {
    const unsigned bb = __ballot_sync(~0u, (d >> b) & 1u);
    m &= ((d >> b) & 1u) ? bb : ~bb;
  }
  return m;
}

// One stable LSD radix pass (8-bit digit of karr[item] at `shift`) from src to dst.  Warp w
// owns a contiguous slice of src; within a warp, lanes of one 32-item step that share a
// digit are ranked by lane (digit_peers), so the (digit, warp, position) order is the input
// order.
// Needs exactly 1024 threads (the scan gives each thread 8 of the 256 x 32 counters).
__device__ void radix_pass(const uint32_t* src, uint32_t* dst, int n, const uint32_t* karr,
                           int shift, uint32_t* hist, int* wsum) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 256 * kHistStride; i += kNmsThreads) hist[i] = 0;
  __syncthreads();
  const int chunk = (((n + 31) >> 5) + 31) & ~31;
  const int lo = warp * chunk, hi = min(n, lo + chunk);
  for (int j = lo; j < hi; j += 32) {
    const int it = j + lane;
    const bool v = it < hi;
    const unsigned vm = __ballot_sync(~0u, v);
    const unsigned d = v ? (karr[src[it]] >> shift) & 255u : 0u;
    const unsigned peers = digit_peers(d, vm);
    if (v && lane == __ffs(peers) - 1) hist[d * kHistStride + warp] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {
    const int d = tid >> 2, w0 = (tid & 3) * 8;
    uint32_t loc[8];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) { loc[k] = hist[d * kHistStride + w0 + k]; sum += (int)loc[k]; }
    int tot;
    int pre = block_scan(sum, wsum, &tot);
#pragma unroll
    for (int k = 0; k < 8; k++) { hist[d * kHistStride + w0 + k] = (uint32_t)pre; pre += (int)loc[k]; }
  }
  __syncthreads();
  for (int j = lo; j < hi; j += 32) {
    const int it = j + lane;
    const bool v = it < hi;
    const unsigned vm = __ballot_sync(~0u, v);
    const uint32_t item = v ? src[it] : 0u;
    const unsigned d = v ? (karr[item] >> shift) & 255u : 0u;
    const unsigned peers = digit_peers(d, vm);
    unsigned base = 0;
    if (v) {
      base = hist[d * kHistStride + warp];
      dst[base + __popc(peers & lanemask_lt())] = item;
    }
    __syncwarp();
    if (v && lane == __ffs(peers) - 1) hist[d * kHistStride + warp] = base + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
}

__device__ __forceinline__ unsigned warp_or(unsigned v) {
  return __reduce_or_sync(~0u, v);
}
__device__ __forceinline__ unsigned warp_and(unsigned v) {
  return __reduce_and_sync(~0u, v);
}

__global__ void __launch_bounds__(kNmsThreads, 1)
nms_kernel(float iou, int max_out, uint8_t* ws, WsLayout L, float* outdets, int* outidx,
           int* outcnt, int* rawcnt, int csize) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t nsm[];
  __shared__ int wsum[32];
  __shared__ int segs[kMaxClasses + 1];
  __shared__ int msegoff[kMaxClasses + 1];
  __shared__ int s_total;
  __shared__ unsigned s_bits[4];        // OR / AND of the score keys, OR / AND of the classes
  __shared__ float kept_s[32][kKeptSmem][5];
  __shared__ int s_ordc;                // workspace sort: which ord buffer holds the class order
  const int rank = csize > 1 ? (int)cluster_rank() : 0;
  const int img = blockIdx.x / csize, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int A = L.A;
  NMS_MARK(0);
  uint8_t* wimg = ws + (size_t)img * L.per_img;
  const float* rec = (const float*)(wimg + L.rec);
  const int* flag = (const int*)(wimg + L.flag);
  uint32_t* canch = (uint32_t*)(wimg + L.anch);
  float* kept = (float*)(wimg + L.kept);
  if (tid == 0) { s_bits[0] = 0u; s_bits[1] = ~0u; s_bits[2] = 0u; s_bits[3] = ~0u; }

  // 1. count: thread t owns anchors [t*per, t*per + per), per a multiple of 4 (int4 loads)
  const int per = ((A + kNmsThreads - 1) / kNmsThreads + 3) & ~3;
  const int a0 = tid * per;
  int cnt = 0;
  for (int q = 0; q < per; q += 4) {
    const int a = a0 + q;
    if (a < A) {
      const int4 f = *(const int4*)(flag + a);
      cnt += (f.x != 0) + (a + 1 < A && f.y != 0) + (a + 2 < A && f.z != 0) + (a + 3 < A && f.w != 0);
    }
  }
  int n;
  int pos = block_scan(cnt, wsum, &n);
  const bool in_smem = n <= kNmsSmemCand;
  const int cap = in_smem ? kNmsSmemCand : A;
  uint8_t* cb = in_smem ? nsm : wimg + L.box;
  // shared layout: box | skey | cls | ord0..2 | hist | surv ; workspace: the same arrays
  float4* box = (float4*)cb;
  uint32_t* skey = in_smem ? (uint32_t*)(nsm + (size_t)cap * 16) : (uint32_t*)(wimg + L.skey);
  uint32_t* ccls = in_smem ? (uint32_t*)(nsm + (size_t)cap * 20) : (uint32_t*)(wimg + L.cls);
  uint32_t* ord = in_smem ? (uint32_t*)(nsm + (size_t)cap * 24) : (uint32_t*)(wimg + L.ord);
  uint32_t* hist = (uint32_t*)(nsm + (size_t)kNmsSmemCand * 36);
  uint8_t* surv = in_smem ? nsm + (size_t)kNmsSmemCand * 36 + 256 * kHistStride * 4
                          : wimg + L.surv;
  uint32_t* ord0 = ord;
  uint32_t* ord1 = ord + cap;
  uint32_t* ord2 = ord + 2 * cap;

  // workspace mode: CTA 0 alone gathers and sorts (the arrays are the cluster's)
  const bool active = in_smem || rank == 0;
  const uint32_t* ordS = ord1;
  const uint32_t* ordC = ord2;
  if (active) {
  // 1b. gather the candidates in anchor order
  unsigned kor = 0, kand = ~0u, cor = 0, cand_ = ~0u;
  for (int q0 = 0; q0 < per; q0 += 32) {
    unsigned fm = 0;   // bit q: anchor a0 + q0 + q is a candidate
#pragma unroll
    for (int q = 0; q < 32; q += 4) {
      const int a = a0 + q0 + q;
      if (q0 + q < per && a < A) {
        const int4 f = *(const int4*)(flag + a);
        fm |= (unsigned)(f.x != 0) << q | (unsigned)(a + 1 < A && f.y != 0) << (q + 1) |
              (unsigned)(a + 2 < A && f.z != 0) << (q + 2) |
              (unsigned)(a + 3 < A && f.w != 0) << (q + 3);
      }
    }
    while (fm) {
      const int q = __ffs(fm) - 1;
      fm &= fm - 1;
      const int a = a0 + q0 + q;
      const float* r = rec + (size_t)a * 6;
      const uint32_t sk = ~dm_f2bits(r[4]);
      const uint32_t c = (uint32_t)(int)r[5];
      box[pos] = make_float4(r[0], r[1], r[2], r[3]);
      skey[pos] = sk;
      ccls[pos] = c;
      if (rank == 0) canch[pos] = (uint32_t)a;
      ord0[pos] = (uint32_t)pos;
      surv[pos] = 0;
      kor |= sk; kand &= sk; cor |= c; cand_ &= c;
      pos++;
    }
  }
  kor = warp_or(kor); kand = warp_and(kand); cor = warp_or(cor); cand_ = warp_and(cand_);
  if (lane == 0) {
    atomicOr(&s_bits[0], kor); atomicAnd(&s_bits[1], kand);
    atomicOr(&s_bits[2], cor); atomicAnd(&s_bits[3], cand_);
  }
  __syncthreads();
  NMS_MARK(1);

  // 2. score order (ordS) and class order (ordC), both stable on the anchor order
  if (n <= kRankSortMax) {
    // bitonic sort of the unique 64-bit keys (score key, index) and (class, score key,
    // index) in the radix histogram area, unused on this path: threads 0-511 sort the first,
    // 512-1023 the second, one compare-exchange each per stage; padding keys sort last
    unsigned long long* kS = (unsigned long long*)hist;
    unsigned long long* kC = kS + kRankSortMax;
    int P = 2;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += kNmsThreads) {
      if (i < n) {
        const unsigned long long ks = ((unsigned long long)skey[i] << 20) | (unsigned)i;
        kS[i] = ks;
        kC[i] = ((unsigned long long)ccls[i] << 52) | ks;
      } else {
        kS[i] = kC[i] = ~0ull;
      }
    }
    __syncthreads();
    // element p of each array lives in thread p's register; partner distances j >= 32 go
    // through shared memory (one barrier per stage), j < 32 by warp shuffles
    unsigned long long* arr = tid < kRankSortMax ? kS : kC;
    const int p = tid & (kRankSortMax - 1);
    const bool live = p < P;
    unsigned long long key = live ? arr[p] : ~0ull;
    for (int k = 2; k <= P; k <<= 1) {
      for (int j = k >> 1; j >= 32; j >>= 1) {
        __syncthreads();
        if (live) arr[p] = key;
        __syncthreads();
        if (live) {
          const unsigned long long o = arr[p ^ j];
          const bool lower = (p & j) == 0, up = (p & k) == 0;
          key = (lower == up) ? (key < o ? key : o) : (key > o ? key : o);
        }
      }
      for (int j = min(k >> 1, 16); j > 0; j >>= 1) {
        const unsigned long long o = __shfl_xor_sync(~0u, key, j);
        const bool lower = (p & j) == 0, up = (p & k) == 0;
        key = (lower == up) ? (key < o ? key : o) : (key > o ? key : o);
      }
    }
    __syncthreads();
    if (live) arr[p] = key;
    __syncthreads();
    for (int i = tid; i < n; i += kNmsThreads) {
      ord1[i] = (uint32_t)(kS[i] & 0xFFFFFu);
      ord2[i] = (uint32_t)(kC[i] & 0xFFFFFu);
    }
    __syncthreads();
    ordS = ord1;
    ordC = ord2;
  } else {
    uint32_t* bufs[3] = {ord0, ord1, ord2};
    int cur = 0;
    const unsigned kvar = s_bits[0] ^ s_bits[1], cvar = s_bits[2] ^ s_bits[3];
    for (int sh = 0; sh < 32; sh += 8) {
      if (!((kvar >> sh) & 255u)) continue;
      radix_pass(bufs[cur], bufs[cur ^ 1], n, skey, sh, hist, wsum);
      cur ^= 1;
    }
    const int sidx = cur, o1 = sidx == 0 ? 1 : 0, o2 = 2;
    // class passes never overwrite the score order: they run over the other two buffers
    int ccur = sidx;
    int nxt = o1;
    for (int sh = 0; sh < 16; sh += 8) {
      if (!((cvar >> sh) & 255u)) continue;
      radix_pass(bufs[ccur], bufs[nxt], n, ccls, sh, hist, wsum);
      ccur = nxt;
      nxt = nxt == o1 ? o2 : o1;
    }
    ordS = bufs[sidx];
    ordC = bufs[ccur];
  }

  NMS_MARK(2);
  // 3. class segments of the class order
  {
    int nseg_running = 0;
    for (int i0 = 0; i0 < n; i0 += kNmsThreads) {
      const int i = i0 + tid;
      const int st = i < n && (i == 0 || ccls[ordC[i]] != ccls[ordC[i - 1]]);
      int t;
      const int p = nseg_running + block_scan(st, wsum, &t);
      if (st && p < kMaxClasses) segs[p] = i;
      nseg_running += t;
    }
    if (tid == 0) {
      s_total = min(nseg_running, kMaxClasses);
      s_ordc = (int)((ordC - ord) / cap);
    }
    __syncthreads();
  }
  }   // active
  if (csize > 1) {
    cluster_barrier();   // every CTA is past its sort: shared memory may be written remotely
    if (!active) {       // workspace mode: CTA 0's class segments and class order
      if (tid == 0) {
        s_total = (int)ld_cluster_u32(cluster_map(smem_u32(&s_total), 0));
        s_ordc = (int)ld_cluster_u32(cluster_map(smem_u32(&s_ordc), 0));
      }
      __syncthreads();
      for (int i = tid; i < s_total; i += kNmsThreads)
        segs[i] = (int)ld_cluster_u32(cluster_map(smem_u32(&segs[i]), 0));
      ordC = ord + (size_t)s_ordc * cap;
      __syncthreads();
    }
  }
  const int nseg = s_total;
  if (tid == 0) segs[nseg] = n;
  __syncthreads();
  NMS_MARK(3);

  // 4. per-class suppression in score order.  Classes of kBitMin+1..kBitMax candidates
  // (kBitMinCluster+1.. with 4 or more CTAs per image) whose bit masks fit, with all
  // candidates in shared memory, use bit masks: every warp of the cluster builds them (bit j
  // of row i: dm_iou_gt(i, j) for a later j, the same test as the greedy path), then one
  // warp per class walks the rows: a row not yet removed is kept and removes its mask.  The
  // other classes run the greedy loop, one warp per class.  Both are exact greedy NMS, and both
  // stop a class at max_out kept boxes: its later survivors could never reach the output.
  int* moff = msegoff;                 // per class: first mask word, or -1 (greedy)
  // Up to kRankSortMax candidates the radix histogram area is unused: the masks live there
  // (8448 words >= 512 x 16), else in the workspace.  Offsets by a block scan over the
  // classes; a class takes the bit-mask path if it is mid-size and its words still fit.
  const bool mask_smem = n <= kRankSortMax;
  uint32_t* bmask = mask_smem ? hist : (uint32_t*)(wimg + L.bmask);
  const int mask_cap = mask_smem ? 256 * kHistStride : L.bmask_words;
  {
    int need = 0;
    if (tid < nseg) {
      const int m = segs[tid + 1] - segs[tid], words = (m + 31) >> 5;
      // (only with the candidates in shared memory: from the workspace, the pair tests'
      // loads cost more than the greedy loop saves)
      if (in_smem && m > (csize >= 4 ? kBitMinCluster : kBitMin) && m <= kBitMax) need = m * words;
    }
    int total;
    const int off = block_scan(need, wsum, &total);
    if (tid < nseg) moff[tid] = need && off + need <= mask_cap ? off : -1;
    if (tid == 0) moff[nseg] = min(total, mask_cap);
    __syncthreads();
  NMS_MARK(4);
  }
  // a class's bit-mask rows go to the CTA that scans them (class s: CTA s mod csize)
  auto put_row = [&](uint32_t* rows, size_t idx, uint32_t v, int owner) {
    if (csize > 1 && mask_smem) st_cluster_u32(cluster_map(smem_u32(rows + idx), (uint32_t)owner), v);
    else rows[idx] = v;
  };
  {
    // one warp per row of a bit-mask class: lane k tests the pair (i, j = 32 w + k) and a
    // ballot gives word w of row i (bit k: candidate j is suppressed by candidate i);
    // words below the diagonal are zero.  The rows are shared out over every warp of the
    // cluster.
    // Work units are (four rows, one word): four independent chains of loads and tests per
    // warp, and enough units that a single class spreads over every warp of the cluster.
    // Units are dealt round-robin over the cluster's warps across all classes.
    const int gwarp = rank * (kNmsThreads >> 5) + warp, nwarps = csize * (kNmsThreads >> 5);
    int ubase = 0;
    for (int sg = 0; sg < nseg; sg++) {
      if (moff[sg] < 0) continue;                         // uniform across the cluster
      const int s = segs[sg], m = segs[sg + 1] - s, words = (m + 31) >> 5;
      const int owner = sg % csize, units = ((m + 3) >> 2) * words;
      uint32_t* rows = bmask + moff[sg];
      for (int un = (gwarp - ubase % nwarps + nwarps) % nwarps; un < units; un += nwarps) {
        const int i0 = (un / words) * 4, w = un - (un / words) * words;
        if (w < (i0 >> 5)) {                              // left of the diagonal: zero
          if (lane < 4 && i0 + lane < m) put_row(rows, (size_t)(i0 + lane) * words + w, 0u, owner);
          continue;
        }
        float4 bi[4];
        float ai[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          bi[u] = box[ordC[s + min(i0 + u, m - 1)]];
          ai[u] = dm_area(bi[u].x, bi[u].y, bi[u].z, bi[u].w);
        }
        const int j = w * 32 + lane;
        const float4 bj = box[ordC[s + min(j, m - 1)]];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const int i = i0 + u;
          const bool sup = i < m && j > i && j < m &&
                           dm_iou_gt(bi[u].x, bi[u].y, bi[u].z, bi[u].w, ai[u], bj.x, bj.y,
                                     bj.z, bj.w, iou);
          const unsigned bits = __ballot_sync(~0u, sup);
          if (lane == 0 && i < m) put_row(rows, (size_t)i * words + w, bits, owner);
        }
      }
      ubase += units;
    }
  }
  if (csize > 1) cluster_barrier();   // the rows are complete in their owners' memory
  else __syncthreads();
  NMS_MARK(5);
  // survivor flags live in CTA 0 (shared memory) or the workspace
  const bool surv_remote = csize > 1 && in_smem;
  const uint32_t surv0 = surv_remote ? cluster_map(smem_u32(surv), 0) : 0u;
  auto put_surv = [&](uint32_t ci, uint32_t v) {
    if (surv_remote) st_cluster_u8(surv0 + ci, v);
    else surv[ci] = (uint8_t)v;
  };
  for (int sg = rank + csize * warp; sg < nseg; sg += csize * (kNmsThreads >> 5)) {
    const int s = segs[sg], e = segs[sg + 1];
    if (moff[sg] >= 0) {
      const int m = e - s, words = (m + 31) >> 5;
      const uint32_t* rows = bmask + moff[sg];
      uint32_t removed = 0;                 // lane w holds word w of the removed set
      int nk = 0;
      for (int i0 = 0; i0 < m; i0 += 32) {  // 32 rows: their own bits share word wq
        const int wq = i0 >> 5;
        const uint32_t valid = m - i0 >= 32 ? ~0u : (1u << (m - i0)) - 1u;
        uint32_t cand = ~__shfl_sync(~0u, removed, wq) & valid;   // rows not yet removed
        if (__popc(cand) <= 8) {
          // few rows left (the usual case: detections suppress heavily): take the first,
          // drop what it removes (its diagonal word, held by lane u), repeat
          const uint32_t diag = i0 + lane < m ? rows[(size_t)(i0 + lane) * words + wq] : 0u;
          uint32_t keep = 0;
          int k = nk;
          while (cand && k < max_out) {
            const int u = __ffs(cand) - 1;
            keep |= 1u << u;
            k++;
            cand &= ~(1u << u) & ~__shfl_sync(~0u, diag, u);
          }
          if (lane < words)                 // every lane adds its word of the kept rows
            for (uint32_t km = keep; km; km &= km - 1)
              removed |= rows[(size_t)(i0 + __ffs(km) - 1) * words + lane];
          if (i0 + lane < m) put_surv(ordC[s + i0 + lane], (keep >> lane) & 1u);
          nk = k;
          continue;
        }
        // many rows left: 16 rows at a time, every lane loading its word of each row and
        // the lane holding word wq deciding the 16 rows in order from its words alone
        for (int h = i0; h < i0 + 32 && h < m; h += 16) {
          const int sh = h & 31;
          uint32_t r16[16];
#pragma unroll
          for (int u = 0; u < 16; u++)
            r16[u] = h + u < m && lane < words ? rows[(size_t)(h + u) * words + lane] : 0u;
          uint32_t keep = 0;
          if (lane == wq) {
            uint32_t rem = removed;
            int k = nk;
#pragma unroll
            for (int u = 0; u < 16; u++)
              if (h + u < m && !((rem >> (sh + u)) & 1u) && k < max_out) {
                keep |= 1u << u;
                rem |= r16[u];
                k++;
              }
          }
          keep = __shfl_sync(~0u, keep, wq);
#pragma unroll
          for (int u = 0; u < 16; u++)      // every lane removes the kept rows' words
            if ((keep >> u) & 1u) removed |= r16[u];
          if (lane < 16 && h + lane < m) put_surv(ordC[s + h + lane], (keep >> lane) & 1u);
          nk += __popc(keep);
        }
      }
      continue;
    }
    int nk = 0;
    for (int c0 = s; c0 < e; c0 += 32) {
      if (nk >= max_out) {                  // the rest of the class cannot reach the output
        for (int q = c0 + lane; q < e; q += 32) put_surv(ordC[q], 0u);
        break;
      }
      const int i = c0 + lane;
      const bool valid = i < e;
      const uint32_t ci = valid ? ordC[i] : 0u;
      float x1 = 0, y1 = 0, x2 = 0, y2 = 0, ar = 0;
      if (valid) {
        const float4 b = box[ci];
        x1 = b.x; y1 = b.y; x2 = b.z; y2 = b.w;
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
        if (!(m >> l)) break;
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
      if (valid) put_surv(ci, alive ? 1u : 0u);
      nk += __popc(m);
      __syncwarp();
    }
  }
  if (csize > 1) cluster_barrier();   // every survivor flag is in CTA 0
  else __syncthreads();
  if (rank != 0) return;
  NMS_MARK(6);

  // 5. survivors in score order, the first max_out kept
  int base = 0;
  for (int i0 = 0; i0 < n && base < max_out; i0 += kNmsThreads) {
    const int i = i0 + tid;
    const uint32_t ci = i < n ? ordS[i] : 0u;
    const bool sv = i < n && surv[ci];
    int tot;
    const int p = base + block_scan(sv ? 1 : 0, wsum, &tot);
    if (sv && p < max_out) {
      const int a = (int)canch[ci];
      const float* r = rec + (size_t)a * 6;
      float* o = outdets + ((size_t)img * max_out + p) * 6;
#pragma unroll
      for (int q = 0; q < 6; q++) o[q] = r[q];
      outidx[(size_t)img * max_out + p] = a;
    }
    base += tot;
  }
  if (tid == 0) {
    outcnt[img] = min(base, max_out);
    rawcnt[img] = n;
  }
  NMS_MARK(7);
}

// ---------------- masks (engine/engine.cu:1129-1158) ----------------
struct DevCoefs {
  DView coef[4];
  int W[4], abase[4];
  int n;
};

// Masks by pixel tiles (nm == NM): one block per (image, 256-pixel tile of the proto plane).
// Each thread holds its pixel's NM proto values in registers, so the proto is read once per
// image instead of once per survivor; survivors go through in chunks whose coefficients and
// crop boxes are staged in shared memory.  Per (pixel, survivor) the arithmetic is
// masks_kernel's (crop test, then the dot product in channel order), so results are equal.
constexpr int kMaskTile = 256, kMaskChunk = 128;
template <int NM>
__global__ void __launch_bounds__(kMaskTile) masks_tile_kernel(
    DevCoefs cf, DView proto, float rx, float ry, int max_out, const float* __restrict__ outdets,
    const int* __restrict__ outidx, const int* __restrict__ outcnt, uint8_t* __restrict__ masks) {
  pdl_wait();     // inputs come from the previous kernel
  pdl_trigger();
  __shared__ float co[kMaskChunk][NM + 1];
  __shared__ float4 bx[kMaskChunk];
  const int img = blockIdx.y, n = outcnt[img];
  if (n == 0) return;
  const int Ph = proto.H, Pw = proto.W, p = blockIdx.x * kMaskTile + threadIdx.x;
  const bool live = p < Ph * Pw;
  const int px = live ? p % Pw : 0, py = live ? p / Pw : 0;
  float pv[NM];
  {
    const __half* pp = proto.p + proto.pix(img, py, px);
#pragma unroll
    for (int c = 0; c < NM; c += 8) {
      const uint4 v = live ? *(const uint4*)(pp + c) : make_uint4(0u, 0u, 0u, 0u);
      const __half* h = (const __half*)&v;
#pragma unroll
      for (int j = 0; j < 8; j++) pv[c + j] = __half2float(h[j]);
    }
  }
  const float fx = (float)px, fy = (float)py;
  for (int d0 = 0; d0 < n; d0 += kMaskChunk) {
    const int nd = min(kMaskChunk, n - d0);
    __syncthreads();   // the previous chunk is done with the staging
    for (int i = threadIdx.x; i < nd * (NM / 8); i += kMaskTile) {
      const int dd = i / (NM / 8), c8 = (i - dd * (NM / 8)) * 8;
      const int a = outidx[(size_t)img * max_out + d0 + dd];
      int li = 0;
      while (li + 1 < cf.n && a >= cf.abase[li + 1]) li++;
      const int rem = a - cf.abase[li];
      const int y = rem / cf.W[li], x = rem - y * cf.W[li];
      const uint4 v = *(const uint4*)(cf.coef[li].p + cf.coef[li].pix(img, y, x) + c8);
      const __half* h = (const __half*)&v;
#pragma unroll
      for (int j = 0; j < 8; j++) co[dd][c8 + j] = __half2float(h[j]);
    }
    for (int dd = threadIdx.x; dd < nd; dd += kMaskTile) {
      const float* det = outdets + ((size_t)img * max_out + d0 + dd) * 6;
      bx[dd] = make_float4(DM_MUL(det[0], rx), DM_MUL(det[1], ry), DM_MUL(det[2], rx),
                           DM_MUL(det[3], ry));
    }
    __syncthreads();
    if (!live) continue;
    uint8_t* out = masks + ((size_t)img * max_out + d0) * Ph * Pw + p;
    for (int dd = 0; dd < nd; dd++) {
      const float4 b = bx[dd];
      uint8_t m = 0;
      if (fx >= b.x && fx < b.z && fy >= b.y && fy < b.w) {
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < NM; c++) acc = DM_FMA(co[dd][c], pv[c], acc);
        m = acc > 0.f;
      }
      out[(size_t)dd * Ph * Pw] = m;
    }
  }
}

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

int yk_letterbox_batch(const uint8_t* bgr, size_t frame_stride, int n, int sh, int sw,
                       const YkView* y, int slot0, float* scale_out, int* top_out,
                       int* left_out, yk_stream_t st) {
  if (!bgr || n < 1 || sh < 1 || sw < 1 || !view_ok(y) || y->C != 3 || slot0 < 0 ||
      slot0 + n > y->batch || (n > 1 && frame_stride < (size_t)sh * sw * 3))
    return YK_EINVAL;
  // geometry as yolo_preprocess computes it (engine/engine.cu:1704-1713)
  const float scale = std::min((float)y->H / sh, (float)y->W / sw);
  const int nh = (int)roundf(sh * scale), nw = (int)roundf(sw * scale);
  const int top = (y->H - nh) / 2, left = (y->W - nw) / 2;
  if (scale_out) *scale_out = scale;
  if (top_out) *top_out = top;
  if (left_out) *left_out = left;
  const size_t dframe = (size_t)y->H * y->W * y->stride;
  __half* dst = (__half*)y->ptr + y->coff + (size_t)slot0 * dframe;
  // rows per block: about eight blocks per SM, at most kLbMaxRows rows each
  const int rows = std::max(1, std::min(kLbMaxRows, (int)((long long)y->H * n / (148 * 8))));
  const int pitch = (sw * 3 + 16 + 15) & ~15;          // a row plus its alignment shift
  const size_t smem = (size_t)2 * rows * pitch;
  if (smem > 200 * 1024) return YK_EUNSUP;             // source rows wider than ~34k pixels
  if (smem > 48 * 1024 && smem_attr(letterbox_kernel, (int)smem) != cudaSuccess)
    return check_launch("letterbox attr");
  const dim3 grid((y->H + rows - 1) / rows, n), block(64, 4);
  launch_k(letterbox_kernel, grid, block, smem, (cudaStream_t)st, bgr, frame_stride, sh, sw,
           dst, dframe, y->H, y->W, y->stride, scale, top, left, nh, nw, rows, pitch);
  note_launch();
  return check_launch("letterbox");
}

int yk_letterbox(const uint8_t* bgr, int sh, int sw, const YkView* y, int slot,
                 float* scale_out, int* top_out, int* left_out, yk_stream_t st) {
  return yk_letterbox_batch(bgr, 0, 1, sh, sw, y, slot, scale_out, top_out, left_out, st);
}

size_t yk_post_workspace_bytes(int batch, int anchors) {
  return (size_t)batch * ws_layout(anchors).per_img;
}

int yk_decode(const YkLevel* levels, int nlevels, int batch, int nc, float conf,
              const YkPost* post, yk_stream_t st) {
  if (!levels || nlevels < 1 || nlevels > 4 || batch < 1 || nc < 1 || !post || !post->ws)
    return YK_EINVAL;
  if (nc > kMaxClasses) return YK_EUNSUP;
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
  launch_k(decode_kernel, (unsigned)((total + 63) / 64), 256, 0, (cudaStream_t)st,
      lv, batch, nc, conf, (uint8_t*)post->ws, L);
  note_launch();
  return check_launch("decode");
}

// CTAs per image: the largest power of two up to 8 that keeps batch x size within the SMs,
// capped by what the device can co-schedule (cudaOccupancyMaxActiveClusters, once per
// device); yk_test_nms_cluster forces a size (0: this rule).
static std::atomic<int> g_nms_cluster_force{0};
static int nms_cluster(int batch) {
  static std::mutex mu;
  static int fit[128], sms[128];   // per device: largest size that schedules (0: not probed)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 1;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!fit[dev]) {
      cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
      fit[dev] = 1;
      for (int c = 8; c > 1; c >>= 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c);
        cfg.blockDim = dim3(kNmsThreads);
        cfg.dynamicSmemBytes = kNmsDynSmem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)c;
        at[0].val.clusterDim.y = at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, nms_kernel, &cfg) == cudaSuccess && n >= 1) {
          fit[dev] = c;
          break;
        }
        cudaGetLastError();   // an unsupported size is not an error of the next launch
      }
    }
  }
  const int force = g_nms_cluster_force.load();
  int c = 1;
  if (force > 0) c = force;
  else
    while (c < 8 && (long long)batch * c * 2 <= sms[dev]) c <<= 1;
  return c < fit[dev] ? c : fit[dev];
}

extern "C" int yk_test_nms_cluster(int size) {
  if (size != 0 && size != 1 && size != 2 && size != 4 && size != 8) return YK_EINVAL;
  g_nms_cluster_force.store(size);
  return YK_OK;
}

int yk_nms(int batch, int anchors, float iou, int max_out, const YkPost* post, yk_stream_t st) {
  if (batch < 1 || anchors < 1 || anchors >= (1 << 20) || max_out < 1 || !post || !post->ws ||
      !post->outdets || !post->outidx || !post->outcnt || !post->rawcnt)
    return YK_EINVAL;
  WsLayout L = ws_layout(anchors);
  if (post->ws_bytes < (size_t)batch * L.per_img) return YK_EINVAL;
  if (smem_attr(nms_kernel, (int)kNmsDynSmem) != cudaSuccess) return check_launch("nms attr");
  const int cs = nms_cluster(batch);
  launch_kc(nms_kernel, batch * cs, kNmsThreads, kNmsDynSmem, cs, (cudaStream_t)st, iou,
            max_out, (uint8_t*)post->ws, L, post->outdets, post->outidx, post->outcnt,
            post->rawcnt, cs);
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
  bool tiles = proto->C == 32;
  for (int i = 0; i < nlevels; i++) tiles = tiles && view_vec8(&levels[i].coef);
  if (tiles) {   // pixel tiles, proto in registers (the 32-coefficient heads)
    const dim3 grid((proto->H * proto->W + kMaskTile - 1) / kMaskTile, proto->batch);
    launch_k(masks_tile_kernel<32>, grid, kMaskTile, 0, (cudaStream_t)st, cf, dview(*proto),
             (float)proto->W / in_w, (float)proto->H / in_h, max_out, post->outdets,
             post->outidx, post->outcnt, masks);
    note_launch();
    return check_launch("masks");
  }
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
  if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("static ws");
  if (dev < 0 || dev >= 128) {
    snprintf(g_cuda_err, sizeof g_cuda_err,
             "yk_decode_nms_static: device ordinal %d outside the 128 this entry point tracks", dev);
    return YK_EUNSUP;
  }
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

