// Engine C ABI of the B200 engine (libyolob200.so): a drop-in for the reference's
// engine/yolo.h (same symbols, same structs, same argument meaning), plus additive
// extensions marked EXT.  Each entry cites the reference declaration it replaces.
//
// Differences from the reference, all in the direction of safety:
//   * errors never exit(): yolo_create returns NULL (see yolo_last_error), the void calls
//     record the error for yolo_last_error and do nothing;
//   * NMS considers every candidate (the reference truncates at 1024) and orders ties by
//     anchor index, so results are deterministic;
//   * CUDA graphs are captured lazily per batch size on first use (the reference captures
//     B = 1..max_batch inside yolo_create); yolo_exec_ms(B) captures and calibrates B on demand.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// engine/yolo.h:7-8
typedef struct { float x1, y1, x2, y2, score; int cls; } YoloDet;
typedef struct { float x, y, w, h, angle, score; int cls; } YoloObbDet;

// engine/yolo.h:10-11 — load a model directory on the current device; buffers for up to
// max_batch frames.  NULL on failure.
void* yolo_create(const char* model_dir, int max_batch);
// engine/yolo.h:12-16 — 0 detect, 1 obb, 2 classify, 3 segment.
int yolo_task(void* h);
// engine/yolo.h:17-18 — calibrated GPU latency (ms) of one batch-B graph launch.
float yolo_exec_ms(void* h, int B);
// engine/yolo.h:19
cudaStream_t yolo_stream(void* h);
// engine/yolo.h:20-23 — letterbox a device BGR u8 HWC frame into batch slot `slot`
// (async on the engine stream; the frame must stay valid until the stream passes it).
void yolo_preprocess(void* h, const unsigned char* dev_bgr, int height, int width, int slot);
// engine/yolo.h:24-25 — run the batch-B graph (net + decode + NMS [+ masks] + D2H) and sync.
void yolo_run(void* h, int B);
// engine/yolo.h:26-28
void yolo_run_async(void* h, int B);
void yolo_sync(void* h);
// engine/yolo.h:29-30 — detections of a slot in original-image coordinates; returns count.
int yolo_get(void* h, int slot, YoloDet* out, int cap);
// engine/yolo.h:31-33 — classify models: resize the shortest edge to S (antialiased
// triangle filter), centre crop, RGB /255 into slot `slot` (async on the engine stream).
void yolo_preprocess_cls(void* h, const unsigned char* dev_bgr, int height, int width, int slot);
// engine/yolo.h:34-35 — top-k class ids and probabilities of a slot after yolo_run, descending
// (ties in class order); 0 for non-classify handles.  Returns the entries written.
int yolo_get_cls(void* h, int slot, int* ids, float* probs, int k);
// engine/yolo.h:36-38
void yolo_slot_geom(void* h, int slot, float* scale, int* top, int* left);
// engine/yolo.h:39-41 — oriented boxes of a slot (obb handles): centre / size in original
// image coordinates, angle in radians, no clipping; 0 for other handles (and yolo_get
// returns 0 on obb handles).
int yolo_get_obb(void* h, int slot, YoloObbDet* out, int cap);
// engine/yolo.h:42-43 — proto resolution (0/0 for detect models).
void yolo_mask_dim(void* h, int* ph, int* pw);
// engine/yolo.h:44-49 — binary {0,1} mask (ph*pw bytes) of detection `det`; 0 or -1.
int yolo_get_mask(void* h, int slot, int det, unsigned char* out);

// ---- EXT (no counterpart in the reference header) ----
typedef struct {
  int device;          // CUDA device ordinal (-1 = current)
  float conf;          // score gate (reference: 0.25)
  float iou;           // NMS IoU threshold (reference: 0.45)
  int max_det;         // survivors per image (reference: 300)
  int autotune;        // 1 = time tensor-core tile variants per conv at create
  int fuse;            // 1 = fold CONV + ADD into the conv epilogue (reference fuseAdds)
} YoloOptions;
void yolo_default_options(YoloOptions* o);
void* yolo_create_ex(const char* model_dir, int max_batch, const YoloOptions* opts);
void yolo_destroy(void* h);
// Message of the most recent failed call on this thread: every call that can fail clears it
// on entry, so after a void call an empty string means success.
const char* yolo_last_error(void);
// JPEG front end (the reference server's nvJPEG decode, server/serve.cpp:84-102, as a
// library call): decode host JPEG bytes on the GPU and preprocess them into slot `slot`
// (letterbox, or the classify resize + crop on classify handles).  Returns when done (the
// bytes may be freed); 0, or -1 (not a JPEG / decode failure; see yolo_last_error).
int yolo_preprocess_jpeg(void* h, const unsigned char* jpeg, size_t nbytes, int slot);
// One-graph pipeline (the reference CLI's `pipeline` graph, engine/engine.cu:1992-2004:
// H2D + preprocess + forward captured together, generalised to a batch and to the API).
// Bind `count` (<= max_batch) equal-size BGR u8 HWC frames, frame i at
// frames + i * height * width * 3, as input array `id` (0..3).  host = 1: page-locked host
// memory, copied to the device inside the graph; host = 0: device memory of the handle's
// GPU.  The memory must stay valid while the binding is used; rebinding an id drops its
// graphs.  0, or -1 (see yolo_last_error).
int yolo_bind_frames(void* h, int id, const unsigned char* frames, int height, int width,
                     int count, int host);
// Replay binding id's pipeline graph for its first B frames into slots 0..B-1: [H2D] +
// preprocessing of all B frames (one letterbox launch) + net + decode + NMS (+ masks) + the
// D2H of the results.  The _async form returns after the launch (yolo_sync, then yolo_get);
// the frames are read when the graph runs.  0, or -1.
int yolo_run_frames_async(void* h, int id, int B);
int yolo_run_frames(void* h, int id, int B);
// Calibrated GPU time (ms) of one launch of binding id's batch-B pipeline graph.
float yolo_frames_exec_ms(void* h, int id, int B);
// Kernel nodes in the graph yolo_run (id = -1) or yolo_run_frames (id >= 0) replays for
// batch B; 0 before that graph has been captured, -1 on bad arguments.
int yolo_graph_kernels(void* h, int id, int B);
// Device time (ms) of the tensor-core convolutions of one batch-B forward, captured alone as
// one graph in the planned order and replayed; *nconv (optional) receives their count.
float yolo_conv_exec_ms(void* h, int B, int* nconv);
// Detections of slots 0..B-1 of binding id's most recent completed run, from the binding's
// own pinned result block (each binding's graphs copy their results there, and yolo_get
// reads the block of the most recently launched run).  A caller with two bindings can
// therefore launch the next batch before reading this one: results of binding id stay
// valid until binding id runs again.  Wait for the run first (yolo_sync, or an event on
// yolo_stream after the launch).  Detect / segment handles; returns the total or -1.
int yolo_get_frames(void* h, int id, int B, YoloDet* out, int cap, int* counts);
// Detections of slots 0..B-1 in one call: slot s's go to out + s * cap (at most cap each),
// its count to counts[s].  Returns the total, or -1 (bad arguments / obb handle).
int yolo_get_batch(void* h, int B, YoloDet* out, int cap, int* counts);
// Number of conf-passing candidates of a slot before NMS (reference h_rawcnt tripwire).
int yolo_raw_count(void* h, int slot);
// Run one op of the UNFUSED graph for B images (dump mode, engine/engine.cu:1843-1888);
// returns 0, 1 if the op has no output view (decode/masks), <0 on error.
int yolo_run_op(void* h, int op_index, int B);
int yolo_num_ops(void* h);
// Device pointer / geometry of a graph tensor view (for dump / resync / tests).
int yolo_tensor_view(void* h, int tensor, void** ptr, int* H, int* W, int* stride, int* coff, int* C);
// Copy a graph tensor view of images 0..B-1 to / from contiguous host fp16 [B][H][W][C]
// (dump mode, resync, tests).  Synchronous; 0 or -1.
int yolo_read_tensor(void* h, int tensor, int B, void* host);
int yolo_write_tensor(void* h, int tensor, int B, const void* host);
// Per-op device timings over `iters` runs of the fused op list (CLI `profile`); fills up to
// cap entries of ms[] in op order and returns the number of ops.
int yolo_profile(void* h, int B, int iters, float* ms, int cap);
// Kind name of fused op i ("CONV", ...) and its tensor-core tile (0 if none).
const char* yolo_op_desc(void* h, int op_index, int* tile);
// Shape of fused op i: info[0..9] = Cin, Cout, k, s, groups, output H, output W, algo, msub,
// has residual.  0, or -1 for a bad index.
int yolo_op_shape(void* h, int op_index, int* info);

#ifdef __cplusplus
}
#endif
