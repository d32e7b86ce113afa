// Kernel-level C ABI of the B200 engine (libyolob200.so).
//
// One launcher per hot-path kernel family.  Every launcher is asynchronous on the given
// stream, takes plain pointers and view descriptors (no C++ or torch types), validates its
// arguments on the host and returns 0 on success or a negative YK_E* code (nothing is
// launched on error).  The engine's executor calls these for every op of a model graph; the
// parity tests call them one op at a time through ctypes.
//
// Tensors are NHWC fp16 "views" over a buffer of shape [batch][H][W][stride]:
// element (n, y, x, c) lives at ptr[((n*H + y)*W + x)*stride + coff + c].  This is the
// reference's (buffer, channel offset, C) view (engine/engine.cu:1254-1259) with the batch
// made explicit.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* yk_stream_t;   // == cudaStream_t

#define YK_OK 0
#define YK_EINVAL (-1)      // bad shape / alignment / argument
#define YK_ECUDA (-2)       // CUDA launch error (see yk_last_cuda_error)
#define YK_ETIMEOUT (-3)    // a kernel's bounded wait gave up (device error word set)
#define YK_EUNSUP (-4)      // shape outside what the kernels implement

typedef struct {
  void* ptr;          // fp16 buffer base (NOT offset by coff)
  int batch, H, W;    // logical shape of the view
  int stride;         // channels per pixel of the underlying buffer
  int coff;           // first channel of the view
  int C;              // channels in the view
} YkView;

typedef struct {
  const void* weight;   // fp16 OHWI [Cout][k][k][Cin/groups]
  const float* bias;    // fp32 [Cout]
  int k, s, p;          // square kernel, stride, padding
  int groups;           // 1 (dense) or == Cin == Cout (depthwise)
  int act;              // 0 identity, 1 SiLU
  int Cin, Cout;
  int tile;             // tensor-core N tile (0 = heuristic, else 32/64/128/256)
  int msub;             // stacked 128-row sub-tiles per CTA tile (0 = heuristic, 1/2/4)
  int algo;             // 0 heuristic, 1 implicit GEMM (TMA im2col / gather), 2 halo patches
                        // (3x3 stride 1 pad 1, Cin % 64 == 0; tile 64/128/256, msub 1/2),
                        // 3 implicit GEMM with transposed tiles (128 output channels x
                        // 128*msub pixels per MMA; Cin >= 64; msub 1/2; tile 256: two
                        // 128-channel MMAs share the pixel operand, msub 2 only; msub 4:
                        // two 256-pixel MMAs share the weight operand),
                        // 4 halo patches with transposed tiles (as 2 but Cin % 32 == 0;
                        // tile = output channels per MMA, 64 or 128; msub 1/2),
                        // 5 halo patches with the 3 horizontal taps folded into the MMA's N
                        // (3x3 stride 1 pad 1, Cin % 32 == 0; tile 32/64 output channels,
                        // N = 3*tile; msub 1/2 for tile 32, 1 for 64),
                        // 6 CTA pairs: one M = 256 MMA over two SMs' shared memory, 256
                        // output channels x 256 pixels per pair (Cin >= 64; tile, msub
                        // ignored)
} YkConv;

// Convolution with bias, activation, optional residual (y = act(conv(x)+b) + res) written
// into y's channel slice.  Dense convs with Cin % 8 == 0 run on the tcgen05 implicit-GEMM
// kernel; Cin == 3 (first conv) and depthwise convs run on dedicated direct kernels.
// Replaces the CONV dispatch of runOp (engine/engine.cu:1263-1336).
int yk_conv(const YkView* x, const YkView* y, const YkView* res, const YkConv* p, yk_stream_t st);

// im2col of a thin input (x->C <= 8) for a k x k / stride s / pad p conv: row (n, oy, ox) of
// col gets the k*k*x->C taps in (ky, kx, c) order, zero past the image and past k*k*C
// (col->C >= k*k*x->C, a multiple of 8).  With it the first conv (Cin = 3, k*k*C = 27 -> 32)
// runs as a 1x1 tensor-core GEMM.  Replaces the reference's direct k_conv0 (engine/engine.cu:487-532).
int yk_im2col(const YkView* x, const YkView* col, int k, int s, int p, yk_stream_t st);

// 5x5 stride-1 pad-2 max pool (SPPF), engine/engine.cu:672-695.
int yk_maxpool5(const YkView* x, const YkView* y, yk_stream_t st);
// The SPPF chain y1 = pool5(x), y2 = pool5(y1), y3 = pool5(y2) in one pass over x.
int yk_maxpool5x3(const YkView* x, const YkView* y1, const YkView* y2, const YkView* y3, yk_stream_t st);
// Nearest 2x upsample, engine/engine.cu:697-708.
int yk_upsample2(const YkView* x, const YkView* y, yk_stream_t st);
// Pixel shuffle r=2 from quadrant channel blocks, engine/engine.cu:713-725.
int yk_ps2(const YkView* x, const YkView* y, yk_stream_t st);
// Channel-slice copy, engine/engine.cu:727-732.
int yk_copyc(const YkView* x, const YkView* y, yk_stream_t st);
// y = a + b, engine/engine.cu:663-670.
int yk_add(const YkView* a, const YkView* b, const YkView* y, yk_stream_t st);
// PSA attention: per image and head, out = softmax(q k^T / sqrt(kd)) v over the H*W tokens;
// qkv channel layout per head [q kd | k kd | v hd].  Replaces engine/engine.cu:1363-1404.
int yk_attn(const YkView* qkv, const YkView* y, int heads, int kd, int hd, yk_stream_t st);

// Letterbox one BGR u8 HWC frame (device memory, sh x sw) into batch slot `slot` of the
// S x S x 3 input view y (RGB, /255, pad 114, bilinear as cv2 INTER_LINEAR's formula).
// Geometry (scale, top, left) is computed on the host as in engine/engine.cu:1704-1713
// and returned through the optional out pointers.  Kernel: engine/engine.cu:968-998.
int yk_letterbox(const uint8_t* bgr, int sh, int sw, const YkView* y, int slot,
                 float* scale_out, int* top_out, int* left_out, yk_stream_t st);
// The same for n equal-size frames in one launch: frame i (BGR u8 HWC, sh x sw, device
// memory) starts at bgr + i * frame_stride bytes and fills slot slot0 + i.  All frames
// share one geometry, returned as by yk_letterbox.  Replaces one k_preprocess launch per
// frame (engine/engine.cu:1704-1713, serve.cpp's per-frame yolo_preprocess loop).
// Source rows up to about 34,000 pixels wide (YK_EUNSUP beyond).
int yk_letterbox_batch(const uint8_t* bgr, size_t frame_stride, int n, int sh, int sw,
                       const YkView* y, int slot0, float* scale_out, int* top_out,
                       int* left_out, yk_stream_t st);

// Classification head (task "classify").  Global average pool of x [B][H][W][C] into
// y [B][1][1][C], fp32 sums (engine/engine.cu:735-744, k_gap); C % 8 == 0, 16-byte views.
int yk_gap(const YkView* x, const YkView* y, yk_stream_t st);
// Channel softmax of x [B][1][1][C] into y (not in place), fp32 max / exp sum
// (engine/engine.cu:746-785, k_softmax_ch).
int yk_softmax(const YkView* x, const YkView* y, yk_stream_t st);
// Classify preprocessing of one BGR u8 HWC frame (device memory, sh x sw) into batch slot
// `slot` of the S x S x 3 input view y: shortest edge resized to S with the antialiased
// triangle filter, centre crop, RGB, /255 (torchvision Resize + CenterCrop + ToTensor;
// engine/engine.cu:1000-1046, k_preprocess_cls + clsGeom).  geom_out (optional, 4 ints)
// receives the resized height, width and the crop's top, left.
int yk_preprocess_cls(const uint8_t* bgr, int sh, int sw, const YkView* y, int slot,
                      int* geom_out, yk_stream_t st);

// Detection head levels for decode / NMS / masks.
typedef struct {
  YkView box;     // 64 channels: 4 sides x 16 DFL bins
  YkView cls;     // >= nc channels (multiple of 8; pad logits ignored)
  YkView coef;    // segment: nm mask coefficients; ptr == NULL for detect
  int stride;     // 8, 16, 32
} YkLevel;

// Oriented boxes (task "obb").  Workspace bytes for batch x anchors.
size_t yk_obb_workspace_bytes(int batch, int anchors);
// Decode of every anchor: levels[i].coef is the ANGLE view (channel 0 real); cls views hold
// nc logits zero-padded to a multiple of 8.  Records cx, cy, w, h (letterbox px), score,
// cls, theta (engine/engine.cu:908-960, k_decode_obb).
int yk_decode_obb(const YkLevel* levels, int nlevels, int batch, int nc, float conf, void* ws,
                  yk_stream_t st);
// Rotated NMS over ALL candidates (the reference keeps the first 2048): score order (ties by
// anchor), same-class probiou >= iou drops the later box, dropped boxes still suppress
// (ultralytics fast-NMS; engine/engine.cu:1160-1252).  outdets [batch][max_out][7] as the
// decode records, outcnt / rawcnt per image (survivors / candidates).
int yk_nms_obb(int batch, int anchors, float iou, int max_out, void* ws, float* outdets,
               int* outcnt, int* rawcnt, yk_stream_t st);

// Device workspace of the post-processing chain, sized by yk_post_workspace_bytes.
typedef struct {
  void* ws;          // device scratch
  size_t ws_bytes;
  float* outdets;    // device [batch][max_out][6]: x1 y1 x2 y2 score cls (letterbox px)
  int* outidx;       // device [batch][max_out]: anchor index of each survivor
  int* outcnt;       // device [batch]: survivors
  int* rawcnt;       // device [batch]: conf-passing candidates before NMS
} YkPost;

size_t yk_post_workspace_bytes(int batch, int anchors);
// Decode (engine/engine.cu:848-906): per anchor best class over nc, score = sigmoid,
// keep if score >= conf, DFL box.  Candidates keep anchor order (no atomics).
int yk_decode(const YkLevel* levels, int nlevels, int batch, int nc, float conf,
              const YkPost* post, yk_stream_t st);
// NMS (engine/engine.cu:1051-1123, made exact and deterministic): every candidate is
// considered (no 1024 cap); order = score desc, anchor index asc; same-class IoU > iou
// suppresses; at most max_out survivors per image.
int yk_nms(int batch, int anchors, float iou, int max_out, const YkPost* post, yk_stream_t st);
// Masks for NMS survivors (engine/engine.cu:1129-1158): logit = coef . proto, crop to the
// box scaled to proto resolution (half-open), mask = logit > 0.  masks: [batch][max_out][Ph][Pw].
int yk_masks(const YkLevel* levels, int nlevels, const YkView* proto, int in_h, int in_w,
             int max_out, const YkPost* post, uint8_t* masks, yk_stream_t st);

// Decode + NMS with no allocation at all (no counterpart in the reference).  For callers
// that cannot call cudaMalloc — code under a fixed device-memory budget, plugins whose host
// framework owns all allocations, loops that must never enter the allocator — the scratch
// lives in one static 8 MiB device array inside the library instead of a YkPost workspace.
// Same arguments and results as yk_decode + yk_nms; outputs as in YkPost ([batch][max_out][6],
// [batch][max_out], [batch], [batch]).  Limit: batch * per-image scratch <= 8 MiB (about
// 9 images of 8400 anchors at 640, 3 images at 1024); larger requests return YK_EINVAL with
// the reason in yk_last_cuda_error.  The first call on each device looks up the array's
// device address (cudaGetSymbolAddress), so make that first call before any stream capture.
// All calls on a device share the one array and it keeps the last call's contents: calls
// whose kernels overlap on the GPU (other streams, other threads) race and corrupt each other.
// The looked-up address is kept for the life of the process: resetting a device
// (cudaDeviceReset) while the library stays loaded is not supported by this entry point.
int yk_decode_nms_static(const YkLevel* levels, int nlevels, int batch, int nc, float conf,
                         float iou, int max_out, float* outdets, int* outidx, int* outcnt,
                         int* rawcnt, yk_stream_t st);

// Device error word (bounded-wait timeouts) of the current device; cleared by the call.
int yk_fetch_device_error(void);
// Test hook for the bounded-wait failure path (no counterpart in the reference, which has no
// bounded waits): wait_ns sets the wait budget of every kernel on the current device (0 =
// the default 2 s); withhold = 1 makes block 0 of the next tensor-core conv launches on the
// TMA path skip its first stage load, so that block's MMA wait runs out, the device error
// word is set and the kernel unwinds (no trap, no hang: the wait is bounded).  Synchronous;
// call yk_test_inject(0, 0) to restore normal operation.
int yk_test_inject(int withhold, unsigned long long wait_ns);
// Test hook: CTAs per image of the NMS launch (thread-block cluster size 1, 2, 4 or 8; 0
// restores the default, the largest power of two up to 8 with batch x size <= the SM count).
// Results do not depend on it; tests compare every size bit for bit.
int yk_test_nms_cluster(int size);
const char* yk_last_cuda_error(void);
// Number of kernels this library launched since load (all devices) — a host-side counter.
long long yk_launch_count(void);

#ifdef __cplusplus
}
#endif
