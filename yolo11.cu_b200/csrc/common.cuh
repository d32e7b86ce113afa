// Shared device/host helpers of the B200 engine: view addressing, error reporting, the
// device error word of bounded waits, and the PTX wrappers (mbarrier, cp.async, tcgen05).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <utility>

#include "../../include/yk.h"

namespace yk {

// A view with its base pointer already offset by coff (device-side form).
struct DView {
  __half* p;        // &buf[coff]
  int H, W, stride, C;
  __device__ __forceinline__ size_t pix(int n, int y, int x) const {
    return ((size_t)(n * (size_t)H + y) * W + x) * stride;
  }
};

static inline DView dview(const YkView& v) {
  DView d;
  d.p = (__half*)v.ptr + v.coff;
  d.H = v.H; d.W = v.W; d.stride = v.stride; d.C = v.C;
  return d;
}

// Host-side validation shared by the launchers.
static inline bool view_ok(const YkView* v) {
  return v && v->ptr && v->batch > 0 && v->H > 0 && v->W > 0 && v->C > 0 && v->coff >= 0 &&
         v->coff + v->C <= v->stride;
}
static inline bool view_vec8(const YkView* v) {
  return view_ok(v) && v->C % 8 == 0 && v->coff % 8 == 0 && v->stride % 8 == 0 &&
         ((uintptr_t)v->ptr & 15) == 0;
}

void note_launch();                        // bumps the launch counter

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the current device.
// The attribute belongs to the device's context, so it is set once per (kernel, device);
// the record is guarded by a mutex so handles on several host threads may launch at once.
cudaError_t ensure_smem_attr(const void* kernel, int bytes);
template <class K>
static inline cudaError_t smem_attr(K* kernel, int bytes) {
  return ensure_smem_attr((const void*)kernel, bytes);
}
int check_launch(const char* what);        // cudaGetLastError -> YK_OK / YK_ECUDA
__device__ int g_device_error = 0;         // set by bounded waits that give up (one TU)

// Bounded-wait budget: a wait that has not completed after this many nanoseconds of
// %globaltimer gives up, sets g_device_error and lets the kernel unwind.
constexpr unsigned long long kWaitNs = 2000000000ull;
// The budget the kernels use (kWaitNs unless a test shortened it with yk_test_inject), and
// the test-only withheld arrival: when set, block 0 of the tensor-core conv kernel's TMA
// path skips its first stage load, so the MMA warp's wait on that stage runs out.
__device__ unsigned long long g_wait_ns = kWaitNs;
__device__ int g_test_withhold = 0;

// ---------------- programmatic dependent launch ----------------
// Every kernel is launched with programmatic stream serialisation, so the next kernel in
// the stream (or graph) may be scheduled while this one still runs and do its set-up
// (barrier init, tensor-map prefetch) in the shadow of our tail.  The contract each kernel
// keeps: pdl_wait() before its first access to memory that an earlier kernel writes or
// reads (it returns once the previous grid has completed and flushed), then pdl_trigger()
// to let the following kernel start its own set-up.  With the wait placed before the
// trigger, at most one kernel waits behind the running one.  YK_NO_PDL=1 launches plainly.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
bool pdl_enabled();
bool patch_enabled();         // halo-patch 3x3 convs offered to the autotuner (YK_NO_PATCH=1: no)
bool streams_enabled();      // multi-stream graph capture candidate (YK_NO_STREAMS=1: no)
bool bulk_store_enabled();   // epilogue bulk tensor stores (YK_NO_BULK_STORE=1: per-row stores)
// Per host thread: -1 follows pdl_enabled(), 0 / 1 force plain / programmatic launches (the
// engine captures its graphs both ways and keeps the faster).
static thread_local int g_pdl_override = -1;

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                   size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed =
      g_pdl_override >= 0 ? g_pdl_override : pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_k with thread-block clusters of `cluster` CTAs along x (1: a plain launch)
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_kc(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, int cluster, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed =
      g_pdl_override >= 0 ? g_pdl_override : pdl_enabled() ? 1 : 0;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = (unsigned)cluster;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---- thread-block cluster primitives (distributed shared memory) ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster: shared-memory writes (local or remote) and global
// writes before it are visible to every thread of the cluster after it.
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local, uint32_t rank) {
  uint32_t o;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(o) : "r"(local), "r"(rank));
  return o;
}
__device__ __forceinline__ void st_cluster_u8(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u8 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------- mbarrier ----------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Returns false (and sets the device error word to `code`) if the phase did not complete
// within g_wait_ns (kWaitNs by default).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int code) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  const unsigned long long lim = *(volatile unsigned long long*)&g_wait_ns;
  while (!mbar_try(bar, parity)) {
    if (globaltimer() - t0 > lim) {
      atomicCAS(&g_device_error, 0, code);
      return false;
    }
  }
  return true;
}
#ifdef YK_CONV_PROF
// Role timing of the tensor-core kernels (diagnostic builds only): cycles spent in each wait,
// summed over lane 0 of every waiting warp, indexed by the low 4 bits of the wait's code.
__device__ unsigned long long g_prof[16];
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int code) {
  const long long t0 = clock64();
  const bool r = mbar_wait_bounded(bar, parity, code);
  if ((threadIdx.x & 31) == 0) atomicAdd(&g_prof[code & 15], (unsigned long long)(clock64() - t0));
  return r;
}
#define YK_PROF_ADD(i, v) atomicAdd(&g_prof[i], (unsigned long long)(v))
#else
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int code) {
  return mbar_wait_bounded(bar, parity, code);
}
#define YK_PROF_ADD(i, v) ((void)0)
#endif

// ---------------- cp.async ----------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------- tcgen05 ----------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t dtmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (count 1) on an mbarrier once all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns: thread t gets lane (base + t), columns c..c+15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16p(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Warp-level tensor-core MMA m16n8k16, fp16 inputs, fp32 accumulators (d += a * b).
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *(uint32_t*)&h;
}

// Packed fp32 pair FMA (one instruction for two lanes, each rounded like fmaf).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("{\n\t.reg .b64 pa, pb, pc;\n\t"
      "mov.b64 pa, {%1, %2};\n\tmov.b64 pb, {%3, %4};\n\tmov.b64 pc, {%5, %6};\n\t"
      "fma.rn.f32x2 %0, pa, pb, pc;\n\t}"
      : "=l"(d)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}

// Two mixed-precision FMAs on the halves of packed fp16 pairs: c0 += x.lo * w.lo and
// c1 += x.hi * w.hi with fp32 accumulators (fp16 products are exact in fp32, so this rounds
// like fmaf on converted inputs, without the conversions).
__device__ __forceinline__ void fma2_f16f32(float& c0, float& c1, uint32_t x2, uint32_t w2) {
  asm("{\n\t.reg .f16 xl, xh, wl, wh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\tmov.b32 {wl, wh}, %3;\n\t"
      "fma.rn.f32.f16 %0, xl, wl, %0;\n\tfma.rn.f32.f16 %1, xh, wh, %1;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "r"(x2), "r"(w2));
}

// As fma2_f16f32, starting from (b0, b1) instead of the accumulators.
__device__ __forceinline__ void fma2_f16f32_from(float& c0, float& c1, uint32_t x2, uint32_t w2,
                                                 float b0, float b1) {
  asm("{\n\t.reg .f16 xl, xh, wl, wh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\tmov.b32 {wl, wh}, %3;\n\t"
      "fma.rn.f32.f16 %0, xl, wl, %4;\n\tfma.rn.f32.f16 %1, xh, wh, %5;\n\t}"
      : "=f"(c0), "=f"(c1)
      : "r"(x2), "r"(w2), "f"(b0), "f"(b1));
}

// SiLU with one special-function op: v * sigmoid(v), sigmoid(v) = 0.5 + 0.5 * tanh(v / 2)
// (the hardware tanh approximation, relative error about 2^-11, below fp16 output rounding).
__device__ __forceinline__ float silu_fast(float v) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * v));
  return v * fmaf(0.5f, t, 0.5f);
}

// Bias + optional SiLU of a pair of fp32 accumulators with packed pair arithmetic, rounded to
// a half2: v = acc + bias; act: v * (0.5 + 0.5 * tanh(v / 2)).
__device__ __forceinline__ __half2 bias_act2(float2 acc, float2 bias, int act) {
  float2 v = ffma2(acc, make_float2(1.f, 1.f), bias);
  if (act == 1) {
    const float2 h = ffma2(v, make_float2(0.5f, 0.5f), make_float2(0.f, 0.f));
    float2 t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t.x) : "f"(h.x));
    asm("tanh.approx.f32 %0, %1;" : "=f"(t.y) : "f"(h.y));
    const float2 sg = ffma2(t, make_float2(0.5f, 0.5f), make_float2(0.5f, 0.5f));
    v = ffma2(v, sg, make_float2(0.f, 0.f));
  }
  return __floats2half2_rn(v.x, v.y);
}

// ---------------- bulk tensor stores (shared -> global) ----------------
__device__ __forceinline__ void tma_store_2d(const void* map, uint32_t src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          (uint64_t)map),
      "r"(src), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Epilogue of one warp's 32 accumulator rows (one row per lane: TMEM lane, output row
// row0 + lane) of a BN-column tile, through a [32 rows][32 channels] staging block in
// shared memory (64-byte rows, 64-byte swizzle; 2 KB, 512-byte aligned) and one bulk tensor
// store per 32 channels: the global writes leave as whole rows of channels instead of a
// 16-byte piece per row and instruction.  Rows past the tensor map (the M tail) and channels
// past Cout are clipped by the store.  rrow: this lane's residual row or null.
template <int BN>
__device__ __forceinline__ void epi_rows_tma(uint32_t trow, int n0, int Cout, int row0,
                                             const __half* rrow, const float* bias, int act,
                                             uint32_t stg, const void* ymap, int lane) {
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    if (n0 + c0 >= Cout) break;   // uniform across the warp
    uint32_t r[32];
    tmem_ld16p(trow + c0, r);
    if (BN > 16 && n0 + c0 + 16 < Cout) tmem_ld16p(trow + c0 + 16, r + 16);
    tmem_ld_wait();
    if (lane == 0) bulk_wait_read0();   // the previous store has read the staging block
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 4; h++) {
      const int nn = n0 + c0 + 8 * h;
      if (8 * h >= BN || nn >= Cout) break;
      const float4 b0 = *(const float4*)(bias + nn);
      const float4 b1 = *(const float4*)(bias + nn + 4);
      const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
      uint4 o;
      __half2* oh = (__half2*)&o;
      if (!rrow) {
#pragma unroll
        for (int q = 0; q < 4; q++)
          oh[q] = bias_act2(make_float2(__uint_as_float(r[8 * h + 2 * q]),
                                        __uint_as_float(r[8 * h + 2 * q + 1])), bb[q], act);
      } else {
        const uint4 rv = *(const uint4*)(rrow + nn);
        const __half2* rh = (const __half2*)&rv;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float v0 = __uint_as_float(r[8 * h + 2 * q]) + bb[q].x;
          float v1 = __uint_as_float(r[8 * h + 2 * q + 1]) + bb[q].y;
          if (act == 1) { v0 = silu_fast(v0); v1 = silu_fast(v1); }
          const float2 f = __half22float2(rh[q]);
          oh[q] = __floats2half2_rn(v0 + f.x, v1 + f.y);
        }
      }
      // 64-byte swizzle: 16-byte chunk h of row `lane` at chunk h ^ ((lane >> 1) & 3)
      const uint32_t dst = stg + lane * 64 + ((h ^ ((lane >> 1) & 3)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(o.x), "r"(o.y),
                   "r"(o.z), "r"(o.w)
                   : "memory");
    }
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(ymap, stg, n0 + c0, row0);
      bulk_commit();
    }
  }
}

// Epilogue of one accumulator row (this thread's TMEM lane) of a BN-column tile: output
// channels n0 .. n0+BN-1 (those < Cout) get bias, SiLU (act == 1), the residual row, and are
// stored as fp16 into yrow.  TMEM columns come in batches of up to 64 with one wait each.
template <int BN>
__device__ __forceinline__ void epi_row(uint32_t trow, int n0, int Cout, bool mok, __half* yrow,
                                        const __half* rrow, const float* bias, int act) {
  constexpr int kBatch = BN < 64 ? BN : 64;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += kBatch) {
    if (n0 + c0 >= Cout) break;   // uniform across the warp
    uint32_t r[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch / 16; j++)
      if (n0 + c0 + 16 * j < Cout) tmem_ld16p(trow + c0 + 16 * j, r + 16 * j);
    tmem_ld_wait();
    if (!mok) continue;
#pragma unroll
    for (int h = 0; h < kBatch / 8; h++) {
      const int nn = n0 + c0 + 8 * h;
      if (nn >= Cout) break;
      const float4 b0 = *(const float4*)(bias + nn);
      const float4 b1 = *(const float4*)(bias + nn + 4);
      const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
      uint4 o;
      __half2* oh = (__half2*)&o;
      if (!rrow) {
#pragma unroll
        for (int q = 0; q < 4; q++)
          oh[q] = bias_act2(make_float2(__uint_as_float(r[8 * h + 2 * q]),
                                        __uint_as_float(r[8 * h + 2 * q + 1])), bb[q], act);
      } else {
        // residual: act(acc + bias) + res in fp32, one rounding
        const uint4 rv = *(const uint4*)(rrow + nn);
        const __half2* rh = (const __half2*)&rv;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float v0 = __uint_as_float(r[8 * h + 2 * q]) + bb[q].x;
          float v1 = __uint_as_float(r[8 * h + 2 * q + 1]) + bb[q].y;
          if (act == 1) { v0 = silu_fast(v0); v1 = silu_fast(v1); }
          const float2 f = __half22float2(rh[q]);
          oh[q] = __floats2half2_rn(v0 + f.x, v1 + f.y);
        }
      }
      *(uint4*)(yrow + nn) = o;
    }
  }
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle layout
// (8-row x 128-byte atoms, 1024-byte aligned; SBO = 1024 B between 8-row groups).
// Same for a K-major operand whose rows are cb_bytes = 128 / 64 / 32 wide (swizzle span equal
// to the row): atoms of 8 rows, SBO = 8 * cb_bytes.
template <int CB_BYTES>
__device__ __forceinline__ uint64_t swz_desc(uint32_t saddr) {
  constexpr uint64_t layout = CB_BYTES == 128 ? 2 : CB_BYTES == 64 ? 4 : 6;
  constexpr uint64_t sbo = (8 * CB_BYTES) >> 4;
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (sbo << 32) | (1ull << 46) |
         (layout << 61);
}
// K-major operand without swizzle: 8-row x 16-byte core matrices, SBO between core matrices
// along M/N, LBO between the two core matrices of one K=16 step.
__device__ __forceinline__ uint64_t nosw_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) |
         ((uint64_t)(sbo >> 4) << 32) | (1ull << 46);
}
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor: fp16 A/B, fp32 D, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16_m128(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

}  // namespace yk
