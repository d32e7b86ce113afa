// Engine runtime: model-directory loader, op planner (residual / pool-chain fusion),
// executor over the yk_* kernel ABI, per-batch CUDA graphs, and the yolo.h C ABI.
//
// Reference counterparts: loadGraph (engine/engine.cu:88-248), runOp (1261-1453),
// forward (1455-1481), fuseAdds (1484-1501), autotune (1504-1533), the yolo_* API
// (1653-1794).  Differences: every failure is an error return (never exit), device memory
// is owned per handle and released by yolo_destroy, NMS output is exact (no 1024 cap),
// and graphs are captured per batch size on first use.
#include <cuda_runtime.h>
#include <nvjpeg.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/yk.h"
#include "../../include/yolo.h"

namespace {

thread_local std::string g_err;

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

#define CKE(x)                                                                          \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    if (e_ != cudaSuccess)                                                              \
      throw Error(std::string(#x) + ": " + cudaGetErrorString(e_));                     \
  } while (0)
#define CKY(x)                                                                          \
  do {                                                                                  \
    int r_ = (x);                                                                       \
    if (r_ != YK_OK)                                                                    \
      throw Error(std::string(#x) + " failed (" + std::to_string(r_) + ") " +          \
                  yk_last_cuda_error());                                                \
  } while (0)

enum Kind { CONV, ADD, MAXPOOL5, UPSAMPLE2, COPYC, ATTN, DECODE, GAP, SOFTMAX, DECODEOBB, PS2,
            DECODESEG, MASKS, POOLX3 };
const char* kKindNames[] = {"CONV", "ADD", "MAXPOOL5", "UPSAMPLE2", "COPYC", "ATTN", "DECODE",
                            "GAP", "SOFTMAX", "DECODEOBB", "PS2", "DECODESEG", "MASKS", "POOLX3"};

struct Buf { int H, W, C; void* p = nullptr; };
struct Ten { int buf, coff, C; };
struct Op {
  Kind kind;
  int a = -1, b = -1, out = -1;   // tensors (CONV: a in, out; ADD: a, b, out; DECODE*: a box, b cls, out coef)
  int k = 0, s = 0, p = 0, g = 0, act = 0, Cin = 0, Cout = 0;
  long woff = 0, boff = 0;
  int heads = 0, kd = 0, hd = 0, stride = 0;
  int res = -1;                   // fused residual tensor
  int y2 = -1, y3 = -1;           // POOLX3 outputs 2 and 3
  int tile = 0;                   // tensor-core N tile chosen by the planner / autotuner
  int msub = 0;                   // tensor-core stacked M sub-tiles (0 = heuristic)
  int algo = 0;                   // tensor-core conv algorithm (YkConv::algo)
  const void* wpad = nullptr;     // stem conv as GEMM over an im2col buffer: padded weights
  void* col = nullptr;            // its im2col buffer [maxB][Ho][Wo][kpad]
  int kpad = 0;
};

struct SlotGeom { float scale = 1.f; int top = 0, left = 0; };

std::vector<char> read_file(const std::string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) throw Error("cannot open " + path);
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  std::vector<char> v(n);
  size_t rd = n ? fread(v.data(), 1, n, f) : 0;
  fclose(f);
  if ((long)rd != n) throw Error("short read " + path);
  return v;
}

struct Engine {
  YoloOptions opt;
  int device = 0, maxB = 1;
  std::string task = "detect";
  int nc = 80, S = 0;
  std::vector<Buf> bufs;
  std::vector<Ten> tens;
  std::vector<Op> raw, ops;       // unfused (dump order) and planned (fused) op lists
  void* dweights = nullptr;
  void* dstem = nullptr;          // stem convs: zero-padded [Cout][kpad] weights
  std::vector<void*> dcols;       // stem convs: im2col buffers
  float* dbias = nullptr;
  size_t nweights = 0, nbias = 0;
  // head
  struct Level { int box, cls, coef, stride; };
  std::vector<Level> levels;
  int protoTen = -1, A = 0;
  int probsTen = -1;              // classify: SOFTMAX output ([1,1,nc] standalone buffer)
  __half* h_probs = nullptr;      // classify: pinned [maxB][nc] fp16 probabilities
  // post-processing state
  YkPost post{};
  uint8_t* dmasks = nullptr;
  // results in one block, device and pinned host alike, so one copy per run fetches them:
  // rawcnt[maxB] | outcnt[maxB] | (16-byte aligned) outdets[maxB][max_det][rec]
  void* dres = nullptr;
  void* hres = nullptr;
  void* hres_dst = nullptr;       // D2H target of run_post: hres, or a binding's own block
  size_t res_bytes = 0;
  size_t res_hdr = 0;
  float* h_out = nullptr;
  int* h_cnt = nullptr;
  int* h_raw = nullptr;
  cudaStream_t st = nullptr;
  // graphs by key: the batch size B for the plain forward (input already in the slots), or
  // frames_key(id, B) for the whole pipeline over frame binding `id`
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, float> exec_ms;
  std::map<int, int> graph_kernels;   // kernel nodes of each kept graph
  // Frame bindings: a fixed array of equal-size BGR u8 frames the pipeline graph reads.
  // Host (page-locked) frames are copied into `stage` inside the graph.
  struct Binding {
    const uint8_t* frames = nullptr;
    int h = 0, w = 0, count = 0;
    bool host = false;
    void* stage = nullptr;
    size_t stage_bytes = 0;
    void* hres = nullptr;         // pinned result block of this binding's graphs
    SlotGeom geom;                // letterbox geometry of its frames (all equal-size)
  };
  static constexpr int kBindings = 4;
  Binding binds[kBindings];
  static int frames_key(int id, int B) { return ((id + 1) << 20) | B; }
  nvjpegHandle_t jpeg = nullptr;   // JPEG front end (created on first use)
  nvjpegJpegState_t jstate = nullptr;
  std::vector<void*> jbuf;         // per slot: the decoded BGR frame
  std::vector<size_t> jcap;
  std::vector<cudaStream_t> side;  // extra streams of the multi-stream graph capture
  std::vector<cudaEvent_t> opev;   // one event per planned op (capture-time ordering)
  std::vector<SlotGeom> slots;
  // point the result getters (yolo_get & co.) at a pinned result block
  void use_results(void* block) {
    h_raw = (int*)block;
    h_cnt = (int*)block + maxB;
    h_out = (float*)((char*)block + res_hdr);
  }
  bool seg() const { return task == "segment"; }
  bool cls() const { return task == "classify"; }
  bool obb() const { return task == "obb"; }
  int rec() const { return obb() ? 7 : 6; }   // floats per survivor record

  ~Engine() { release(); }

  void release() {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    graphs.clear();
    for (Binding& b : binds) {
      if (b.stage) cudaFree(b.stage);
      if (b.hres) cudaFreeHost(b.hres);
      b = Binding{};
    }
    for (cudaStream_t s : side) cudaStreamDestroy(s);
    side.clear();
    for (void* b : jbuf)
      if (b) cudaFree(b);
    jbuf.clear();
    jcap.clear();
    if (jstate) nvjpegJpegStateDestroy(jstate);
    if (jpeg) nvjpegDestroy(jpeg);
    jstate = nullptr;
    jpeg = nullptr;
    for (cudaEvent_t e : opev) cudaEventDestroy(e);
    opev.clear();
    for (auto& b : bufs)
      if (b.p) cudaFree(b.p), b.p = nullptr;
    if (dweights) cudaFree(dweights);
    if (dstem) cudaFree(dstem);
    for (void* c : dcols) cudaFree(c);
    dcols.clear();
    if (dbias) cudaFree(dbias);
    if (post.ws) cudaFree(post.ws);
    if (dres) cudaFree(dres);
    if (post.outidx) cudaFree(post.outidx);
    if (dmasks) cudaFree(dmasks);
    if (hres) cudaFreeHost(hres);
    dres = hres = nullptr;
    if (h_probs) cudaFreeHost(h_probs);
    h_probs = nullptr;
    if (st) cudaStreamDestroy(st);
    dweights = nullptr; dstem = nullptr; dbias = nullptr; post = YkPost{}; dmasks = nullptr;
    h_out = nullptr; h_cnt = nullptr; h_raw = nullptr; st = nullptr;
    if (prev >= 0) cudaSetDevice(prev);
  }

  YkView view(int t, int B) const {
    const Ten& tv = tens.at(t);
    const Buf& b = bufs.at(tv.buf);
    YkView v;
    v.ptr = b.p; v.batch = B; v.H = b.H; v.W = b.W; v.stride = b.C; v.coff = tv.coff; v.C = tv.C;
    return v;
  }

  void parse(const std::string& dir);
  void validate(const std::string& dir);
  void allocate(const std::string& dir);
  void plan();
  void autotune();
  std::string tuning_key() const;
  bool load_tuning(const char* path);
  void save_tuning(const char* path) const;
  void run_op(const Op& op, int B);
  void run_post(int B);
  void forward(int B);
  void forward_streams(int B);
  void load_frames(int id, int B);
  cudaGraphExec_t graph_for(int B, int bind = -1);
  float conv_graph_ms(int B);
  bool tc_conv(const Op& op) const {
    return op.kind == CONV && op.g == 1 && (op.Cin % 8 == 0 || op.wpad);
  }
};

void Engine::parse(const std::string& dir) {
  FILE* f = fopen((dir + "/model.graph").c_str(), "r");
  if (!f) throw Error("no model.graph in " + dir);
  std::unique_ptr<FILE, int (*)(FILE*)> guard(f, fclose);
  char magic[64], tag[32], taskbuf[32];
  int ver = 0;
  if (fscanf(f, "%63s %d", magic, &ver) != 2 || strcmp(magic, "YOLO11GRAPH"))
    throw Error("bad graph magic");
  int hsz = 0;
  if (ver >= 2) {
    if (fscanf(f, "%31s %31s %d %d", tag, taskbuf, &nc, &hsz) != 4 || strcmp(tag, "TASK"))
      throw Error("bad TASK header");
    task = taskbuf;
  }
  int nb, nt, no;
  if (fscanf(f, "%d %d %d", &nb, &nt, &no) != 3 || nb < 1 || nt < 1 || no < 1 || nb > 100000 ||
      nt > 100000 || no > 100000)
    throw Error("bad graph counts");
  bufs.resize(nb);
  tens.resize(nt);
  for (auto& b : bufs)
    if (fscanf(f, "%31s %d %d %d", tag, &b.H, &b.W, &b.C) != 4 || strcmp(tag, "B") || b.H < 1 ||
        b.W < 1 || b.C < 1)
      throw Error("bad buffer line");
  for (auto& t : tens)
    if (fscanf(f, "%31s %d %d %d", tag, &t.buf, &t.coff, &t.C) != 4 || strcmp(tag, "T") ||
        t.buf < 0 || t.buf >= nb || t.coff < 0 || t.C < 1 || t.coff + t.C > bufs[t.buf].C)
      throw Error("bad tensor line");
  auto rd = [&](int n, int* v) {
    for (int i = 0; i < n; i++)
      if (fscanf(f, "%d", &v[i]) != 1) throw Error("truncated op line");
  };
  for (int i = 0; i < no; i++) {
    if (fscanf(f, "%31s", tag) != 1) throw Error("truncated graph");
    Op op;
    int v[10];
    if (!strcmp(tag, "CONV")) {
      op.kind = CONV;
      rd(9, v);
      op.a = v[0]; op.out = v[1]; op.k = v[2]; op.s = v[3]; op.p = v[4]; op.g = v[5];
      op.act = v[6]; op.Cin = v[7]; op.Cout = v[8];
      if (fscanf(f, "%ld %ld", &op.woff, &op.boff) != 2) throw Error("truncated CONV");
    } else if (!strcmp(tag, "ADD")) {
      op.kind = ADD; rd(3, v); op.a = v[0]; op.b = v[1]; op.out = v[2];
    } else if (!strcmp(tag, "MAXPOOL5") || !strcmp(tag, "UPSAMPLE2") || !strcmp(tag, "COPYC") ||
               !strcmp(tag, "PS2") || !strcmp(tag, "GAP") || !strcmp(tag, "SOFTMAX")) {
      op.kind = !strcmp(tag, "MAXPOOL5") ? MAXPOOL5 : !strcmp(tag, "UPSAMPLE2") ? UPSAMPLE2
              : !strcmp(tag, "COPYC") ? COPYC : !strcmp(tag, "PS2") ? PS2
              : !strcmp(tag, "GAP") ? GAP : SOFTMAX;
      rd(2, v); op.a = v[0]; op.out = v[1];
    } else if (!strcmp(tag, "ATTN")) {
      op.kind = ATTN; rd(5, v);
      op.a = v[0]; op.out = v[1]; op.heads = v[2]; op.kd = v[3]; op.hd = v[4];
    } else if (!strcmp(tag, "DECODE")) {
      op.kind = DECODE; rd(3, v); op.a = v[0]; op.b = v[1]; op.stride = v[2];
    } else if (!strcmp(tag, "DECODESEG") || !strcmp(tag, "DECODEOBB")) {
      op.kind = !strcmp(tag, "DECODESEG") ? DECODESEG : DECODEOBB;
      rd(4, v); op.a = v[0]; op.b = v[1]; op.out = v[2]; op.stride = v[3];
    } else if (!strcmp(tag, "MASKS")) {
      op.kind = MASKS; rd(1, v); op.a = v[0];
    } else {
      throw Error(std::string("bad op ") + tag);
    }
    for (int t : {op.a, op.b, op.out})
      if (t >= nt) throw Error("op references a missing tensor");
    raw.push_back(op);
  }
  const Buf& ib = bufs[tens[0].buf];
  if (hsz && (hsz != ib.H || hsz != ib.W)) throw Error("imgsz header mismatch");
  S = ib.H;
}

void Engine::validate(const std::string& dir) {
  if (task != "detect" && task != "segment" && task != "classify" && task != "obb")
    throw Error("task '" + task + "' is not supported by this engine");
  const Ten& t0 = tens[0];
  if (t0.coff != 0 || t0.C != 3 || bufs[t0.buf].C != 3 || bufs[t0.buf].H != bufs[t0.buf].W)
    throw Error("tensor 0 must be a standalone S x S x 3 input");
  A = 0;
  for (const Op& op : raw) {
    switch (op.kind) {
      case CONV: {
        const Ten &x = tens[op.a], &y = tens[op.out];
        const Buf &bx = bufs[x.buf], &by = bufs[y.buf];
        if (x.C != op.Cin || y.C != op.Cout || op.k < 1 || op.s < 1)
          throw Error("CONV channel mismatch");
        if ((bx.H + 2 * op.p - op.k) / op.s + 1 != by.H || (bx.W + 2 * op.p - op.k) / op.s + 1 != by.W)
          throw Error("CONV spatial mismatch");
        const bool dw = op.g > 1;
        if (dw && (op.g != op.Cin || op.Cin != op.Cout)) throw Error("unsupported grouped CONV");
        if (op.woff < 0 || op.boff < 0 || op.woff % 8 || op.boff % 4) throw Error("bad weight offset");
        break;
      }
      case GAP: case SOFTMAX: {
        const Ten &x = tens[op.a], &y = tens[op.out];
        const Buf &bx = bufs[x.buf], &by = bufs[y.buf];
        if (!cls()) throw Error(std::string(kKindNames[op.kind]) + " needs task=classify");
        if (x.C != y.C || by.H != 1 || by.W != 1 || (op.kind == SOFTMAX && (bx.H != 1 || bx.W != 1)))
          throw Error(std::string(kKindNames[op.kind]) + " shape mismatch");
        if (op.kind == SOFTMAX) probsTen = op.out;
        break;
      }
      case DECODEOBB: {   // a = box view, b = cls view, out = angle view (channel 0 real)
        if (!obb()) throw Error("DECODEOBB needs task=obb");
        const Ten &c = tens[op.b], &an = tens[op.out];
        if (c.C % 8 || c.C < nc || an.C % 8 || an.C < 1)
          throw Error("DECODEOBB needs 8-aligned cls / angle views covering nc");
        if (tens[op.a].C != 64) throw Error("DECODEOBB box view must have 64 channels");
        levels.push_back({op.a, op.b, op.out, op.stride});
        const Buf& bb = bufs[tens[op.a].buf];
        A += bb.H * bb.W;
        break;
      }
      case DECODE: case DECODESEG: {
        const Ten& c = tens[op.b];
        if (c.C % 8 || c.C < nc) throw Error("DECODE needs an 8-aligned cls view covering nc");
        if (tens[op.a].C != 64) throw Error("DECODE box view must have 64 channels");
        if ((op.kind == DECODESEG) != seg()) throw Error("DECODESEG needs task=segment");
        levels.push_back({op.a, op.b, op.kind == DECODESEG ? op.out : -1, op.stride});
        const Buf& bb = bufs[tens[op.a].buf];
        A += bb.H * bb.W;
        break;
      }
      case MASKS: protoTen = op.a; break;
      default: break;
    }
  }
  if (cls()) {
    // the D2H copy reads [B][nc] contiguous: a standalone full-width [1,1,nc] buffer
    if (probsTen < 0) throw Error("classify graph without SOFTMAX");
    const Ten& t = tens[probsTen];
    const Buf& b = bufs[t.buf];
    if (t.coff || t.C != b.C || b.H != 1 || b.W != 1 || t.C != nc)
      throw Error("probs tensor must be a standalone [1,1,nc] buffer");
    if (!levels.empty()) throw Error("classify graph with DECODE ops");
  } else if (levels.empty() || levels.size() > 4) {
    throw Error("graph needs 1..4 DECODE levels");
  }
  auto fsize = [&](const char* name) -> long {
    FILE* f = fopen((dir + "/" + name).c_str(), "rb");
    if (!f) throw Error(std::string("cannot open ") + dir + "/" + name);
    fseek(f, 0, SEEK_END);
    long n = ftell(f);
    fclose(f);
    return n;
  };
  const long nw = fsize("weights.f16") / 2, nbb = fsize("bias.f32") / 4;
  for (const Op& op : raw)
    if (op.kind == CONV) {
      const long wcount = (long)op.Cout * op.k * op.k * (op.Cin / std::max(op.g, 1));
      if (op.woff + wcount > nw || op.boff + op.Cout > nbb)
        throw Error("weights.f16 / bias.f32 too small for the graph");
    }
  if (seg()) {
    if (protoTen < 0) throw Error("segment graph without MASKS op");
    const int nm = tens[protoTen].C;
    if (nm % 8 || nm > 64) throw Error("unsupported mask coefficient count");
    for (auto& l : levels)
      if (tens[l.coef].C != nm) throw Error("coef view width != proto channels");
  }
}

void Engine::allocate(const std::string& dir) {
  CKE(cudaSetDevice(device));
  CKE(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  // Dense 3x3 convs on the 3-channel input (the stem) with Cout <= 96 run on the direct
  // warp-MMA stem kernel (yk_conv).  Other convs on the 3-channel input run as a tensor-core
  // GEMM over an im2col buffer: each output pixel's k*k*3 taps padded to a multiple of 8
  // (27 -> 32), one contiguous row per pixel, so the GEMM's A operand streams by 2-D TMA
  // (YK_STEM_GEMM=1 forces this path for every stem).
  static const bool force_gemm = [] {
    const char* e = getenv("YK_STEM_GEMM");
    return e && *e && *e != '0';
  }();
  auto is_stem = [&](const Op& op) {
    const bool direct = op.k == 3 && op.Cout % 8 == 0 && op.Cout <= 96 && !force_gemm;
    return op.kind == CONV && op.g == 1 && op.Cin == 3 && op.k * op.k * 3 <= 64 && !direct;
  };
  bool stem = false;
  for (const Op& op : raw) stem = stem || is_stem(op);
  for (auto& b : bufs) {
    const size_t bytes = (size_t)maxB * b.H * b.W * b.C * 2;
    CKE(cudaMalloc(&b.p, bytes));
    CKE(cudaMemset(b.p, 0, bytes));
  }
  auto wf = read_file(dir + "/weights.f16");
  auto bf = read_file(dir + "/bias.f32");
  nweights = wf.size() / 2;
  nbias = bf.size() / 4;
  for (const Op& op : raw)
    if (op.kind == CONV) {
      const size_t wcount = (size_t)op.Cout * op.k * op.k * (op.Cin / std::max(op.g, 1));
      if (op.woff + wcount > nweights || op.boff + (size_t)op.Cout > nbias)
        throw Error("weights.f16 / bias.f32 too small for the graph");
    }
  if (stem) {
    const uint16_t* w16 = (const uint16_t*)wf.data();
    std::vector<uint16_t> pad;
    std::vector<size_t> offs;
    for (const Op& op : raw)
      if (is_stem(op)) {
        const int kk = op.k * op.k * 3, kp = (kk + 7) / 8 * 8;
        offs.push_back(pad.size());
        for (int o = 0; o < op.Cout; o++)
          for (int i = 0; i < kp; i++) pad.push_back(i < kk ? w16[op.woff + (size_t)o * kk + i] : 0);
      }
    CKE(cudaMalloc(&dstem, pad.size() * 2));
    CKE(cudaMemcpy(dstem, pad.data(), pad.size() * 2, cudaMemcpyHostToDevice));
    size_t i = 0;
    for (Op& op : raw)
      if (is_stem(op)) {
        op.wpad = (const uint16_t*)dstem + offs[i++];
        op.kpad = (op.k * op.k * 3 + 7) / 8 * 8;
        const Buf& yb = bufs[tens[op.out].buf];
        void* col = nullptr;
        CKE(cudaMalloc(&col, (size_t)maxB * yb.H * yb.W * op.kpad * 2));
        dcols.push_back(col);
        op.col = col;
      }
  }
  CKE(cudaMalloc(&dweights, std::max<size_t>(wf.size(), 16)));
  CKE(cudaMemcpy(dweights, wf.data(), wf.size(), cudaMemcpyHostToDevice));
  CKE(cudaMalloc(&dbias, std::max<size_t>(bf.size(), 16)));
  CKE(cudaMemcpy(dbias, bf.data(), bf.size(), cudaMemcpyHostToDevice));
  post.ws_bytes = obb() ? yk_obb_workspace_bytes(maxB, A) : yk_post_workspace_bytes(maxB, A);
  CKE(cudaMalloc(&post.ws, post.ws_bytes));
  res_hdr = ((size_t)2 * maxB * sizeof(int) + 15) & ~(size_t)15;
  res_bytes = res_hdr + (size_t)maxB * opt.max_det * rec() * sizeof(float);
  CKE(cudaMalloc(&dres, res_bytes));
  CKE(cudaMemset(dres, 0, res_bytes));
  post.rawcnt = (int*)dres;
  post.outcnt = (int*)dres + maxB;
  post.outdets = (float*)((char*)dres + res_hdr);
  CKE(cudaMalloc(&post.outidx, (size_t)maxB * opt.max_det * sizeof(int)));
  if (seg()) {
    const Buf& pb = bufs[tens[protoTen].buf];
    CKE(cudaMalloc(&dmasks, (size_t)maxB * opt.max_det * pb.H * pb.W));
  }
  CKE(cudaMallocHost(&hres, res_bytes));
  hres_dst = hres;
  h_raw = (int*)hres;
  h_cnt = (int*)hres + maxB;
  h_out = (float*)((char*)hres + res_hdr);
  if (cls()) {
    CKE(cudaMallocHost(&h_probs, (size_t)maxB * nc * sizeof(__half)));
    memset(h_probs, 0, (size_t)maxB * nc * sizeof(__half));   // defined before the first run
  }
  memset(h_cnt, 0, maxB * sizeof(int));
  memset(h_raw, 0, maxB * sizeof(int));
  slots.assign(maxB, SlotGeom{});
  CKE(cudaDeviceSynchronize());   // weights / memsets complete before the non-blocking stream runs
}

// Planner: the reference's fuseAdds (a CONV directly followed by an ADD that consumes its
// output becomes a residual epilogue) plus folding SPPF's three chained MAXPOOL5 ops into
// one pass.  The unfused list stays available for per-op dumps.
void Engine::plan() {
  ops.clear();
  // the exporter may give one buffer slice several tensor ids
  auto same_view = [&](int a, int b) {
    return a == b || (a >= 0 && b >= 0 && tens[a].buf == tens[b].buf &&
                      tens[a].coff == tens[b].coff && tens[a].C == tens[b].C);
  };
  for (size_t i = 0; i < raw.size(); i++) {
    Op op = raw[i];
    if (opt.fuse && op.kind == CONV && i + 1 < raw.size()) {
      const Op& nx = raw[i + 1];
      if (nx.kind == ADD && (same_view(nx.a, op.out) || same_view(nx.b, op.out))) {
        op.res = same_view(nx.a, op.out) ? nx.b : nx.a;
        op.out = nx.out;
        i++;
      }
    } else if (opt.fuse && op.kind == MAXPOOL5 && i + 2 < raw.size() &&
               raw[i + 1].kind == MAXPOOL5 && raw[i + 2].kind == MAXPOOL5 &&
               same_view(raw[i + 1].a, op.out) && same_view(raw[i + 2].a, raw[i + 1].out)) {
      op.kind = POOLX3;
      op.y2 = raw[i + 1].out;
      op.y3 = raw[i + 2].out;
      i += 2;
    }
    if (op.kind == DECODE || op.kind == DECODESEG || op.kind == DECODEOBB || op.kind == MASKS) continue;
    ops.push_back(op);
  }
}

void Engine::run_op(const Op& op, int B) {
  switch (op.kind) {
    case CONV: {
      YkConv p;
      p.weight = (const uint16_t*)dweights + op.woff;
      p.bias = dbias + op.boff;
      p.k = op.k; p.s = op.s; p.p = op.p; p.groups = op.g; p.act = op.act;
      p.Cin = op.Cin; p.Cout = op.Cout; p.tile = op.tile; p.msub = op.msub; p.algo = op.algo;
      YkView x = view(op.a, B), y = view(op.out, B);
      if (op.wpad) {            // stem: im2col into the padded buffer, then a 1x1 GEMM
        YkView col;
        col.ptr = op.col; col.batch = B; col.H = y.H; col.W = y.W;
        col.stride = op.kpad; col.coff = 0; col.C = op.kpad;
        CKY(yk_im2col(&x, &col, op.k, op.s, op.p, (yk_stream_t)st));
        x = col;
        p.weight = op.wpad;
        p.Cin = op.kpad;
        p.k = 1; p.s = 1; p.p = 0;
      }
      YkView r;
      if (op.res >= 0) r = view(op.res, B);
      CKY(yk_conv(&x, &y, op.res >= 0 ? &r : nullptr, &p, (yk_stream_t)st));
      break;
    }
    case ADD: {
      YkView a = view(op.a, B), b = view(op.b, B), y = view(op.out, B);
      CKY(yk_add(&a, &b, &y, (yk_stream_t)st));
      break;
    }
    case MAXPOOL5: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_maxpool5(&x, &y, (yk_stream_t)st));
      break;
    }
    case POOLX3: {
      YkView x = view(op.a, B), y1 = view(op.out, B), y2 = view(op.y2, B), y3 = view(op.y3, B);
      CKY(yk_maxpool5x3(&x, &y1, &y2, &y3, (yk_stream_t)st));
      break;
    }
    case UPSAMPLE2: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_upsample2(&x, &y, (yk_stream_t)st));
      break;
    }
    case PS2: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_ps2(&x, &y, (yk_stream_t)st));
      break;
    }
    case COPYC: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_copyc(&x, &y, (yk_stream_t)st));
      break;
    }
    case ATTN: {
      YkView q = view(op.a, B), y = view(op.out, B);
      CKY(yk_attn(&q, &y, op.heads, op.kd, op.hd, (yk_stream_t)st));
      break;
    }
    case GAP: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_gap(&x, &y, (yk_stream_t)st));
      break;
    }
    case SOFTMAX: {
      YkView x = view(op.a, B), y = view(op.out, B);
      CKY(yk_softmax(&x, &y, (yk_stream_t)st));
      break;
    }
    default:
      break;   // DECODE / DECODESEG / MASKS run in run_post
  }
}

void Engine::run_post(int B) {
  if (cls()) {   // no decode / NMS: the probabilities go to the host
    CKE(cudaMemcpyAsync(h_probs, bufs[tens[probsTen].buf].p, (size_t)B * nc * sizeof(__half),
                        cudaMemcpyDeviceToHost, st));
    return;
  }
  std::vector<YkLevel> lv(levels.size());
  for (size_t i = 0; i < levels.size(); i++) {
    lv[i].box = view(levels[i].box, B);
    lv[i].cls = view(levels[i].cls, B);
    if (levels[i].coef >= 0) lv[i].coef = view(levels[i].coef, B);
    else memset(&lv[i].coef, 0, sizeof(YkView));
    lv[i].stride = levels[i].stride;
  }
  if (obb()) {
    CKY(yk_decode_obb(lv.data(), (int)lv.size(), B, nc, opt.conf, post.ws, (yk_stream_t)st));
    CKY(yk_nms_obb(B, A, opt.iou, opt.max_det, post.ws, post.outdets, post.outcnt, post.rawcnt,
                   (yk_stream_t)st));
  } else {
    CKY(yk_decode(lv.data(), (int)lv.size(), B, nc, opt.conf, &post, (yk_stream_t)st));
    CKY(yk_nms(B, A, opt.iou, opt.max_det, &post, (yk_stream_t)st));
  }
  if (seg()) {
    YkView pr = view(protoTen, B);
    CKY(yk_masks(lv.data(), (int)lv.size(), &pr, S, S, opt.max_det, &post, dmasks,
                 (yk_stream_t)st));
  }
  // counts of all slots and the first B images' records: one copy
  CKE(cudaMemcpyAsync(hres_dst, dres, res_hdr + (size_t)B * opt.max_det * rec() * sizeof(float),
                      cudaMemcpyDeviceToHost, st));
}

void Engine::forward(int B) {
  for (const Op& op : ops) run_op(op, B);
  run_post(B);
}

// The same forward spread over several streams inside one capture, so the graph has the
// op DAG instead of a chain: independent branches (the detection head's per-level box and
// class chains, neck paths) run concurrently, which pays when each kernel fills only part
// of the GPU (batch 1).  Op k depends on every earlier op whose written channel range
// overlaps one it reads or writes, or that reads a range it writes (read-after-write,
// write-after-write, write-after-read on buffer channel ranges).  Ops join the stream whose
// last op they depend on, else a fresh stream (up to 8); cross-stream dependencies are
// event waits.  The post-processing runs on the main stream after all streams join.
void Engine::forward_streams(int B) {
  constexpr int kMaxStreams = 8;
  const int n = (int)ops.size();
  while ((int)side.size() < kMaxStreams - 1) {
    cudaStream_t s;
    CKE(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    side.push_back(s);
  }
  while ((int)opev.size() < n + 1) {
    cudaEvent_t e;
    CKE(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    opev.push_back(e);
  }
  struct Reg { int buf, c0, c1; };
  auto reg = [&](int t) { const Ten& v = tens[t]; return Reg{v.buf, v.coff, v.coff + v.C}; };
  auto overlap = [](const Reg& a, const Reg& b) { return a.buf == b.buf && a.c0 < b.c1 && b.c0 < a.c1; };
  std::vector<std::vector<Reg>> rd(n), wr(n);
  for (int k = 0; k < n; k++) {
    const Op& o = ops[k];
    if (o.a >= 0) rd[k].push_back(reg(o.a));
    if (o.kind == ADD && o.b >= 0) rd[k].push_back(reg(o.b));
    if (o.res >= 0) rd[k].push_back(reg(o.res));
    if (o.out >= 0) wr[k].push_back(reg(o.out));
    if (o.y2 >= 0) wr[k].push_back(reg(o.y2));
    if (o.y3 >= 0) wr[k].push_back(reg(o.y3));
  }
  auto any = [&](const std::vector<Reg>& x, const std::vector<Reg>& y) {
    for (const Reg& a : x)
      for (const Reg& b : y)
        if (overlap(a, b)) return true;
    return false;
  };
  std::vector<cudaStream_t> strm(kMaxStreams);
  strm[0] = st;
  for (int i = 1; i < kMaxStreams; i++) strm[i] = side[i - 1];
  std::vector<int> tail(kMaxStreams, -1), on(n, 0);
  int used = 1;
  // fork: every stream starts after what the main stream holds so far
  CKE(cudaEventRecord(opev[n], st));
  for (int i = 1; i < kMaxStreams; i++) CKE(cudaStreamWaitEvent(strm[i], opev[n], 0));
  const cudaStream_t main_st = st;
  try {
    for (int k = 0; k < n; k++) {
      std::vector<int> deps;
      for (int j = 0; j < k; j++)
        if (any(wr[j], rd[k]) || any(wr[j], wr[k]) || any(rd[j], wr[k])) deps.push_back(j);
      int s = -1;
      for (int i = 0; i < used; i++)      // continue the chain of the latest dependency
        if (tail[i] >= 0 && std::find(deps.begin(), deps.end(), tail[i]) != deps.end() &&
            (s < 0 || tail[i] > tail[s]))
          s = i;
      if (s < 0) {
        if (used < kMaxStreams) s = used++;
        else {
          s = 0;
          for (int i = 1; i < used; i++)
            if (tail[i] < tail[s]) s = i;
        }
      }
      std::vector<int> latest(kMaxStreams, -1);   // latest dependency on each other stream
      for (int j : deps)
        if (on[j] != s) latest[on[j]] = std::max(latest[on[j]], j);
      for (int i = 0; i < kMaxStreams; i++)
        if (latest[i] >= 0) CKE(cudaStreamWaitEvent(strm[s], opev[latest[i]], 0));
      st = strm[s];
      run_op(ops[k], B);
      st = main_st;
      CKE(cudaEventRecord(opev[k], strm[s]));
      on[k] = s;
      tail[s] = k;
    }
  } catch (...) {
    st = main_st;
    throw;
  }
  // join every stream back into the main one, then decode / NMS / D2H there
  for (int i = 1; i < kMaxStreams; i++) {
    CKE(cudaEventRecord(opev[n], strm[i]));
    CKE(cudaStreamWaitEvent(st, opev[n], 0));
  }
  run_post(B);
}

// Startup autotune (reference engine/engine.cu:1504-1533): time every tensor-core tile width
// that fits the layer at the full batch and keep the fastest.
void Engine::autotune() {
  cudaEvent_t e0, e1;
  CKE(cudaEventCreate(&e0));
  CKE(cudaEventCreate(&e1));
  // {algo, tile, msub}: implicit GEMM; implicit GEMM with transposed tiles (Cin >= 64);
  // halo patches with transposed tiles (3x3 stride-1 convs, Cin % 32 == 0); kx-folded halo
  // patches; CTA pairs (Cin >= 64, input view on 16-byte rows for its TMA loads)
  static const int combos[][3] = {{1, 32, 1}, {1, 32, 2}, {1, 32, 4}, {1, 64, 1}, {1, 64, 2},
                                  {1, 64, 4}, {1, 128, 1}, {1, 128, 2}, {1, 256, 1},
                                  {3, 128, 1}, {3, 128, 2}, {3, 256, 2},
                                  {4, 64, 1}, {4, 64, 2}, {4, 128, 1}, {4, 128, 2},
                                  {5, 32, 1}, {5, 32, 2}, {5, 64, 1}, {6, 256, 2}};
  for (Op& op : ops) {
    if (op.kind != CONV || op.g != 1 || (op.Cin % 8 && !op.wpad)) continue;
    const bool patch_ok = !op.wpad && op.k == 3 && op.s == 1 && op.p == 1 && op.Cin % 32 == 0 &&
                          patch_enabled();
    // the kx-folded kernel also takes 16-channel blocks (the 48-channel bottlenecks) and
    // zero-filled ones (8-channel inputs)
    const bool kxn_ok = !op.wpad && op.k == 3 && op.s == 1 && op.p == 1 && op.Cin % 8 == 0 &&
                        patch_enabled();
    const bool trans_ok = !op.wpad && op.Cin >= 64;
    const YkView xin = view(op.a, maxB);
    const bool pair_ok = trans_ok && xin.coff % 8 == 0 && xin.stride % 8 == 0;
    int best_t = 0, best_m = 0, best_a = 1;
    float tbest = 1e30f;
    for (const auto& cm : combos) {
      const int tile = cm[1];
      if (cm[0] == 4 && (!patch_ok || (tile == 128 && op.Cout <= 64))) continue;
      if (cm[0] == 5 && (!kxn_ok || (tile == 64 && op.Cout <= 32))) continue;
      if (cm[0] == 3 && (!trans_ok || (tile == 256 && op.Cout <= 128))) continue;
      if (cm[0] == 6 && (!pair_ok || op.Cout <= 128)) continue;
      if (cm[0] == 1 && tile > 32 && tile / 2 >= op.Cout) continue;   // half the tile wasted
      // (narrow plain / patch tiles only pay for thin outputs; the kx-folded kernel's
      // 32-channel tiles also win on wider ones: 96 -> 96 at 128x128 78 us vs 98 us)
      if (tile == 32 && op.Cout > 64 && cm[0] != 5) continue;
      op.algo = cm[0];
      op.tile = tile;
      op.msub = cm[2];
      run_op(op, maxB);
      CKE(cudaEventRecord(e0, st));
      for (int r = 0; r < 5; r++) run_op(op, maxB);
      CKE(cudaEventRecord(e1, st));
      CKE(cudaEventSynchronize(e1));
      float ms = 0;
      CKE(cudaEventElapsedTime(&ms, e0, e1));
      if (ms < tbest) { tbest = ms; best_t = tile; best_m = cm[2]; best_a = cm[0]; }
    }
    op.algo = best_a;
    op.tile = best_t;
    op.msub = best_m;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  // the tuning runs overwrote activations; every forward recomputes them
}

std::string Engine::tuning_key() const {
  cudaDeviceProp pr;
  cudaGetDeviceProperties(&pr, device);
  std::string k = "v3|" + std::string(pr.name) + "|B" + std::to_string(maxB);
  for (const Op& op : ops)
    if (op.kind == CONV)
      k += "|" + std::to_string(op.Cin) + "," + std::to_string(op.Cout) + "," +
           std::to_string(op.k) + "," + std::to_string(op.s) + "," +
           std::to_string(bufs[tens[op.out].buf].H);
  return k;
}

bool Engine::load_tuning(const char* path) {
  FILE* f = fopen(path, "r");
  if (!f) return false;
  std::unique_ptr<FILE, int (*)(FILE*)> g(f, fclose);
  std::string key = tuning_key();
  std::vector<char> line(key.size() + 16);
  if (!fgets(line.data(), (int)line.size(), f)) return false;
  std::string got(line.data());
  while (!got.empty() && (got.back() == '\n' || got.back() == '\r')) got.pop_back();
  if (got != key) return false;
  struct Tuned { int algo, tile, msub; };
  std::vector<Tuned> tiles;
  int al, t, m;
  while (fscanf(f, "%d %d %d", &al, &t, &m) == 3) tiles.push_back({al, t, m});
  size_t i = 0;
  for (const Op& op : ops)
    if (op.kind == CONV) i++;
  if (tiles.size() != i) return false;
  i = 0;
  for (Op& op : ops)
    if (op.kind == CONV) {
      op.algo = tiles[i].algo; op.tile = tiles[i].tile; op.msub = tiles[i].msub;
      i++;
    }
  return true;
}

void Engine::save_tuning(const char* path) const {
  FILE* f = fopen(path, "w");
  if (!f) return;
  fprintf(f, "%s\n", tuning_key().c_str());
  for (const Op& op : ops)
    if (op.kind == CONV) fprintf(f, "%d %d %d\n", op.algo, op.tile, op.msub);
  fclose(f);
}

// Pipeline prologue of frame binding `id`: the H2D copy of B host frames (one copy of the
// contiguous array) and the preprocessing of all B slots.  Detect / segment / obb models
// letterbox every frame in one launch; classify models run their resize + crop per frame.
void Engine::load_frames(int id, int B) {
  const Binding& b = binds[id];
  const size_t fb = (size_t)b.h * b.w * 3;
  const uint8_t* src = b.frames;
  if (b.host) {
    CKE(cudaMemcpyAsync(b.stage, b.frames, fb * B, cudaMemcpyHostToDevice, st));
    src = (const uint8_t*)b.stage;
  }
  YkView in = view(0, maxB);
  if (cls()) {
    for (int i = 0; i < B; i++)
      CKY(yk_preprocess_cls(src + fb * i, b.h, b.w, &in, i, nullptr, (yk_stream_t)st));
  } else {
    CKY(yk_letterbox_batch(src, fb, B, b.h, b.w, &in, 0, nullptr, nullptr, nullptr,
                           (yk_stream_t)st));
  }
}

int count_kernel_nodes(cudaGraph_t g) {
  size_t n = 0;
  if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess) return -1;
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return -1;
  int k = 0;
  for (size_t i = 0; i < n; i++) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
  }
  return k;
}

// Device time of the tensor-core convs of one batch-B forward as they run inside a graph:
// the planned op list's tcgen05 convs (the stem GEMM with its im2col) captured alone, in
// order, on one stream, with programmatic dependent launch when enabled, and replayed
// (3 warm-up + 10 timed launches, the better of two rounds).  The convs read what the last
// forward left in their input buffers, so shapes and data are those of the real forward.
float Engine::conv_graph_ms(int B) {
  cudaGraph_t g;
  g_pdl_override = pdl_enabled() ? 1 : 0;
  CKE(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  try {
    for (const Op& op : ops)
      if (tc_conv(op)) run_op(op, B);
  } catch (...) {
    g_pdl_override = -1;
    cudaGraph_t dummy;
    cudaStreamEndCapture(st, &dummy);
    if (dummy) cudaGraphDestroy(dummy);
    throw;
  }
  g_pdl_override = -1;
  CKE(cudaStreamEndCapture(st, &g));
  cudaGraphExec_t ge;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  CKE(e);
  cudaEvent_t e0, e1;
  CKE(cudaEventCreate(&e0));
  CKE(cudaEventCreate(&e1));
  float best = 1e30f;
  for (int round = 0; round < 2; round++) {
    for (int i = 0; i < 3; i++) CKE(cudaGraphLaunch(ge, st));
    CKE(cudaEventRecord(e0, st));
    for (int i = 0; i < 10; i++) CKE(cudaGraphLaunch(ge, st));
    CKE(cudaEventRecord(e1, st));
    CKE(cudaEventSynchronize(e1));
    float ms = 0;
    CKE(cudaEventElapsedTime(&ms, e0, e1));
    best = std::min(best, ms / 10.f);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(ge);
  return best;
}

cudaGraphExec_t Engine::graph_for(int B, int bind) {
  const int key = bind >= 0 ? frames_key(bind, B) : B;
  auto it = graphs.find(key);
  if (it != graphs.end()) return it->second;
  // Capture the forward once with programmatic dependent launch between the kernels and,
  // when that is enabled, once without; keep the faster.  Overlapping each kernel's set-up
  // with its predecessor's tail pays at small batches, where every kernel is a few
  // microseconds; at large batches the early-resident waiting CTAs can cost a little.
  int kernels = 0, best_kernels = 0;
  auto capture = [&](int pdl, bool multi = false) {
    cudaGraph_t g;
    g_pdl_override = pdl;
    CKE(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    hres_dst = bind >= 0 && binds[bind].hres ? binds[bind].hres : hres;
    try {
      if (bind >= 0) load_frames(bind, B);
      if (multi) forward_streams(B);
      else forward(B);
    } catch (...) {
      hres_dst = hres;
      g_pdl_override = -1;
      cudaGraph_t dummy;
      cudaStreamEndCapture(st, &dummy);
      if (dummy) cudaGraphDestroy(dummy);
      throw;
    }
    g_pdl_override = -1;
    hres_dst = hres;
    CKE(cudaStreamEndCapture(st, &g));
    kernels = count_kernel_nodes(g);
    cudaGraphExec_t ge;
    const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    CKE(e);
    return ge;
  };
  cudaEvent_t e0, e1;
  CKE(cudaEventCreate(&e0));
  CKE(cudaEventCreate(&e1));
  // calibration as the reference does it: 3 warm + 10 timed launches
  auto time10 = [&](cudaGraphExec_t ge) {
    for (int i = 0; i < 3; i++) CKE(cudaGraphLaunch(ge, st));
    CKE(cudaEventRecord(e0, st));
    for (int i = 0; i < 10; i++) CKE(cudaGraphLaunch(ge, st));
    CKE(cudaEventRecord(e1, st));
    CKE(cudaEventSynchronize(e1));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    return ms / 10.f;
  };
  cudaGraphExec_t best = capture(0);
  best_kernels = kernels;
  float best_ms = time10(best);
  if (pdl_enabled()) {
    cudaGraphExec_t alt = nullptr;
    try {
      alt = capture(1);
      float alt_ms = time10(alt), plain_ms = time10(best);
      alt_ms = std::min(alt_ms, time10(alt));
      best_ms = std::min(best_ms, plain_ms);
      if (alt_ms < best_ms) {
        std::swap(alt, best);
        best_ms = alt_ms;
        best_kernels = kernels;
      }
    } catch (...) {
      if (alt) cudaGraphExecDestroy(alt);
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      cudaGraphExecDestroy(best);
      throw;
    }
    cudaGraphExecDestroy(alt);
  }
  if (streams_enabled()) {   // the op DAG over several streams; kept only if faster
    // (YK_STREAMS=force keeps it regardless: tests use it to check the DAG capture)
    const char* fs = getenv("YK_STREAMS");
    const bool force = fs && !strcmp(fs, "force");
    cudaGraphExec_t alt = nullptr;
    try {
      alt = capture(pdl_enabled() ? 1 : 0, true);
      float alt_ms = std::min(time10(alt), time10(alt)), cur_ms = time10(best);
      best_ms = std::min(best_ms, cur_ms);
      if (force || alt_ms < best_ms) {
        std::swap(alt, best);
        best_ms = alt_ms;
        best_kernels = kernels;
      }
    } catch (...) {
      if (alt) cudaGraphExecDestroy(alt);
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      cudaGraphExecDestroy(best);
      throw;
    }
    cudaGraphExecDestroy(alt);
  }
  graphs[key] = best;
  exec_ms[key] = best_ms;
  graph_kernels[key] = best_kernels;
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return best;
}

Engine* as_engine(void* h) { return (Engine*)h; }

struct DeviceScope {   // makes the handle's device current for the duration of a call
  int prev = -1;
  explicit DeviceScope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

template <class F>
auto guarded(F&& f, decltype(f()) fail) -> decltype(f()) {
  g_err.clear();   // the last error describes the most recent call on this thread
  try {
    return f();
  } catch (const std::exception& e) {
    g_err = e.what();
    return fail;
  }
}

}  // namespace

extern "C" {

const char* yolo_last_error(void) { return g_err.c_str(); }

void yolo_default_options(YoloOptions* o) {
  o->device = -1;
  o->conf = 0.25f;
  o->iou = 0.45f;
  o->max_det = 300;
  o->autotune = 1;
  o->fuse = 1;
}

void* yolo_create_ex(const char* model_dir, int max_batch, const YoloOptions* opts) {
  return guarded([&]() -> void* {
    if (!model_dir || max_batch < 1) throw Error("yolo_create: bad arguments");
    std::unique_ptr<Engine> e(new Engine());
    if (opts) e->opt = *opts; else yolo_default_options(&e->opt);
    if (e->opt.max_det < 1 || e->opt.max_det > 100000) throw Error("bad max_det");
    e->maxB = max_batch;
    e->parse(model_dir);      // host-only checks first: bad directories fail without a GPU
    e->validate(model_dir);
    int dev = e->opt.device;
    if (dev < 0) CKE(cudaGetDevice(&dev));
    e->device = dev;
    DeviceScope ds(dev);
    e->allocate(model_dir);
    e->plan();
    if (e->opt.autotune) {
      // optional tuning cache (env YOLO_TUNE_CACHE=path): tiles keyed by device name, batch
      // and the conv list; a miss tunes and rewrites the file
      const char* cache = getenv("YOLO_TUNE_CACHE");
      if (!(cache && e->load_tuning(cache))) {
        e->autotune();
        if (cache) e->save_tuning(cache);
      }
    }
    CKE(cudaStreamSynchronize(e->st));
    int derr = yk_fetch_device_error();
    if (derr) throw Error("device error word set during create: " + std::to_string(derr));
    return e.release();
  }, nullptr);
}

void* yolo_create(const char* model_dir, int max_batch) {
  YoloOptions o;
  yolo_default_options(&o);
  return yolo_create_ex(model_dir, max_batch, &o);
}

void yolo_destroy(void* h) { delete as_engine(h); }

int yolo_task(void* h) {
  if (!h) return 0;
  return as_engine(h)->seg() ? 3 : as_engine(h)->cls() ? 2 : as_engine(h)->obb() ? 1 : 0;
}

float yolo_exec_ms(void* h, int B) {
  return guarded([&]() -> float {
    Engine* e = as_engine(h);
    if (!e || B < 1 || B > e->maxB) throw Error("yolo_exec_ms: bad batch");
    DeviceScope ds(e->device);
    e->graph_for(B);
    return e->exec_ms[B];
  }, -1.f);
}

cudaStream_t yolo_stream(void* h) { return h ? as_engine(h)->st : nullptr; }

void yolo_preprocess(void* h, const unsigned char* dev_bgr, int height, int width, int slot) {
  guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || slot < 0 || slot >= e->maxB) throw Error("yolo_preprocess: bad slot");
    DeviceScope ds(e->device);
    YkView in = e->view(0, e->maxB);
    SlotGeom& g = e->slots[slot];
    CKY(yk_letterbox(dev_bgr, height, width, &in, slot, &g.scale, &g.top, &g.left,
                     (yk_stream_t)e->st));
    return 0;
  }, -1);
}

// JPEG front end (the reference server's decodeOne, server/serve.cpp:84-102): nvJPEG
// decodes the host bytes to a device BGR frame (per-slot buffer), then the task's own
// preprocessing (letterbox, or the classify resize + crop) fills the slot.  Synchronises the
// engine stream before returning, so the bytes may be freed at once.
int yolo_preprocess_jpeg(void* h, const unsigned char* bytes, size_t nbytes, int slot) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || slot < 0 || slot >= e->maxB || !bytes) throw Error("yolo_preprocess_jpeg: bad arguments");
    if (nbytes < 4 || bytes[0] != 0xFF || bytes[1] != 0xD8) throw Error("yolo_preprocess_jpeg: not a JPEG");
    DeviceScope ds(e->device);
    auto ckj = [](nvjpegStatus_t r, const char* what) {
      if (r != NVJPEG_STATUS_SUCCESS) throw Error(std::string(what) + " failed (nvjpeg " + std::to_string((int)r) + ")");
    };
    if (!e->jpeg) {
      ckj(nvjpegCreateSimple(&e->jpeg), "nvjpegCreateSimple");
      ckj(nvjpegJpegStateCreate(e->jpeg, &e->jstate), "nvjpegJpegStateCreate");
      e->jbuf.assign(e->maxB, nullptr);
      e->jcap.assign(e->maxB, 0);
    }
    int ncomp = 0, ws[NVJPEG_MAX_COMPONENT] = {}, hs[NVJPEG_MAX_COMPONENT] = {};
    nvjpegChromaSubsampling_t sub;
    ckj(nvjpegGetImageInfo(e->jpeg, bytes, nbytes, &ncomp, &sub, ws, hs), "nvjpegGetImageInfo");
    const int w = ws[0], hgt = hs[0];
    if (w < 1 || hgt < 1) throw Error("yolo_preprocess_jpeg: empty image");
    const size_t need = (size_t)w * hgt * 3;
    if (e->jcap[slot] < need) {
      CKE(cudaStreamSynchronize(e->st));      // the old buffer may still be in use
      if (e->jbuf[slot]) CKE(cudaFree(e->jbuf[slot]));
      e->jbuf[slot] = nullptr;
      e->jcap[slot] = 0;
      CKE(cudaMalloc(&e->jbuf[slot], need));
      e->jcap[slot] = need;
    }
    nvjpegImage_t out{};
    out.channel[0] = (unsigned char*)e->jbuf[slot];
    out.pitch[0] = (size_t)w * 3;
    ckj(nvjpegDecode(e->jpeg, e->jstate, bytes, nbytes, NVJPEG_OUTPUT_BGRI, &out, e->st),
        "nvjpegDecode");
    YkView in = e->view(0, e->maxB);
    const uint8_t* src = (const uint8_t*)e->jbuf[slot];
    if (e->cls()) {
      CKY(yk_preprocess_cls(src, hgt, w, &in, slot, nullptr, (yk_stream_t)e->st));
    } else {
      SlotGeom& g = e->slots[slot];
      CKY(yk_letterbox(src, hgt, w, &in, slot, &g.scale, &g.top, &g.left, (yk_stream_t)e->st));
    }
    CKE(cudaStreamSynchronize(e->st));
    return 0;
  }, -1);
}

void yolo_preprocess_cls(void* h, const unsigned char* dev_bgr, int height, int width, int slot) {
  guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || slot < 0 || slot >= e->maxB) throw Error("yolo_preprocess_cls: bad slot");
    DeviceScope ds(e->device);
    YkView in = e->view(0, e->maxB);
    CKY(yk_preprocess_cls(dev_bgr, height, width, &in, slot, nullptr, (yk_stream_t)e->st));
    return 0;
  }, -1);
}

// Top-k of a slot's probabilities: descending, ties in class order (a value enters ahead of
// the entries it strictly exceeds), as engine/engine.cu:1593-1605.
int yolo_get_cls(void* h, int slot, int* ids, float* probs, int k) {
  Engine* e = as_engine(h);
  if (!e || !e->cls() || slot < 0 || slot >= e->maxB || k < 1 || !ids || !probs) return 0;
  k = std::min(k, e->nc);
  const __half* p = e->h_probs + (size_t)slot * e->nc;
  for (int i = 0; i < k; i++) { ids[i] = -1; probs[i] = -1.f; }
  for (int c = 0; c < e->nc; c++) {
    const float v = __half2float(p[c]);
    for (int i = 0; i < k; i++)
      if (v > probs[i]) {
        for (int j = k - 1; j > i; j--) { probs[j] = probs[j - 1]; ids[j] = ids[j - 1]; }
        probs[i] = v;
        ids[i] = c;
        break;
      }
  }
  return k;
}

// Oriented boxes of a slot in original-image coordinates: centre and size mapped back
// through the letterbox, angle unchanged, no clipping (engine/engine.cu:1783-1794).
int yolo_get_obb(void* h, int slot, YoloObbDet* out, int cap) {
  Engine* e = as_engine(h);
  if (!e || !e->obb() || slot < 0 || slot >= e->maxB || (!out && cap > 0)) return 0;
  const SlotGeom& g = e->slots[slot];
  const int n = std::min(e->h_cnt[slot], cap);
  for (int i = 0; i < n; i++) {
    const float* d = e->h_out + ((size_t)slot * e->opt.max_det + i) * 7;
    out[i].x = (d[0] - g.left) / g.scale;
    out[i].y = (d[1] - g.top) / g.scale;
    out[i].w = d[2] / g.scale;
    out[i].h = d[3] / g.scale;
    out[i].angle = d[6];
    out[i].score = d[4];
    out[i].cls = (int)d[5];
  }
  return n;
}

void yolo_run_async(void* h, int B) {
  guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || B < 1 || B > e->maxB) throw Error("yolo_run: bad batch");
    DeviceScope ds(e->device);
    CKE(cudaGraphLaunch(e->graph_for(B), e->st));
    e->use_results(e->hres);
    return 0;
  }, -1);
}

void yolo_sync(void* h) {
  guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e) throw Error("yolo_sync: null handle");
    CKE(cudaStreamSynchronize(e->st));
    int derr = yk_fetch_device_error();
    if (derr) throw Error("device error word set: " + std::to_string(derr));
    return 0;
  }, -1);
}

void yolo_run(void* h, int B) {
  yolo_run_async(h, B);
  yolo_sync(h);
}

int yolo_bind_frames(void* h, int id, const unsigned char* frames, int height, int width,
                     int count, int host) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || id < 0 || id >= Engine::kBindings || !frames || height < 1 || width < 1 ||
        count < 1 || count > e->maxB)
      throw Error("yolo_bind_frames: bad arguments");
    DeviceScope ds(e->device);
    cudaPointerAttributes pa;
    CKE(cudaPointerGetAttributes(&pa, frames));
    if (host && pa.type != cudaMemoryTypeHost)
      throw Error("yolo_bind_frames: host frames must be page-locked (cudaMallocHost / cudaHostRegister)");
    if (!host && !((pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) &&
                   pa.device == e->device))
      throw Error("yolo_bind_frames: frames are not device memory of the handle's GPU");
    CKE(cudaStreamSynchronize(e->st));        // no graph of this binding is in flight
    for (auto it = e->graphs.begin(); it != e->graphs.end();) {
      if ((it->first >> 20) == id + 1) {
        cudaGraphExecDestroy(it->second);
        e->exec_ms.erase(it->first);
        it = e->graphs.erase(it);
      } else {
        ++it;
      }
    }
    Engine::Binding& b = e->binds[id];
    const size_t need = host ? (size_t)height * width * 3 * count : 0;
    if (b.stage_bytes < need) {
      if (b.stage) CKE(cudaFree(b.stage));
      b.stage = nullptr;
      b.stage_bytes = 0;
      CKE(cudaMalloc(&b.stage, need));
      b.stage_bytes = need;
    }
    if (!b.hres) {
      CKE(cudaMallocHost(&b.hres, e->res_bytes));
      memset(b.hres, 0, e->res_bytes);
    }
    b.frames = frames;
    b.h = height;
    b.w = width;
    b.count = count;
    b.host = host != 0;
    return 0;
  }, -1);
}

int yolo_run_frames_async(void* h, int id, int B) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || id < 0 || id >= Engine::kBindings || !e->binds[id].frames || B < 1 ||
        B > e->binds[id].count)
      throw Error("yolo_run_frames: bad binding or batch");
    DeviceScope ds(e->device);
    const Engine::Binding& b = e->binds[id];
    SlotGeom g;
    if (!e->cls()) {   // the letterbox geometry (engine/engine.cu:1704-1713)
      const Buf& ib = e->bufs[e->tens[0].buf];
      g.scale = std::min((float)ib.H / b.h, (float)ib.W / b.w);
      const int nh = (int)roundf(b.h * g.scale), nw = (int)roundf(b.w * g.scale);
      g.top = (ib.H - nh) / 2;
      g.left = (ib.W - nw) / 2;
    }
    CKE(cudaGraphLaunch(e->graph_for(B, id), e->st));
    Engine::Binding& bb = e->binds[id];
    bb.geom = g;
    for (int i = 0; i < B; i++) e->slots[i] = g;
    // yolo_get & co. read the most recently launched run's results: this binding's block
    e->use_results(bb.hres);
    return 0;
  }, -1);
}

int yolo_run_frames(void* h, int id, int B) {
  if (yolo_run_frames_async(h, id, B) != 0) return -1;
  yolo_sync(h);
  return yolo_last_error()[0] ? -1 : 0;
}

float yolo_frames_exec_ms(void* h, int id, int B) {
  return guarded([&]() -> float {
    Engine* e = as_engine(h);
    if (!e || id < 0 || id >= Engine::kBindings || !e->binds[id].frames || B < 1 ||
        B > e->binds[id].count)
      throw Error("yolo_frames_exec_ms: bad binding or batch");
    DeviceScope ds(e->device);
    e->graph_for(B, id);
    return e->exec_ms[Engine::frames_key(id, B)];
  }, -1.f);
}

int yolo_graph_kernels(void* h, int id, int B) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || id < -1 || id >= Engine::kBindings || B < 1 || B > e->maxB)
      throw Error("yolo_graph_kernels: bad arguments");
    const int key = id >= 0 ? Engine::frames_key(id, B) : B;
    auto it = e->graph_kernels.find(key);
    return it == e->graph_kernels.end() ? 0 : it->second;
  }, -1);
}

float yolo_conv_exec_ms(void* h, int B, int* nconv) {
  return guarded([&]() -> float {
    Engine* e = as_engine(h);
    if (!e || B < 1 || B > e->maxB) throw Error("yolo_conv_exec_ms: bad batch");
    DeviceScope ds(e->device);
    if (nconv) {
      *nconv = 0;
      for (const Op& op : e->ops) *nconv += e->tc_conv(op);
    }
    return e->conv_graph_ms(B);
  }, -1.f);
}

int yolo_get_frames(void* h, int id, int B, YoloDet* out, int cap, int* counts) {
  Engine* e = as_engine(h);
  if (!e || e->obb() || e->cls() || id < 0 || id >= Engine::kBindings || !e->binds[id].hres ||
      B < 1 || B > e->binds[id].count || cap < 0 || (!out && cap > 0) || !counts)
    return -1;
  const Engine::Binding& b = e->binds[id];
  const int* cnt = (const int*)b.hres + e->maxB;
  const float* recs = (const float*)((const char*)b.hres + e->res_hdr);
  int total = 0;
  for (int s = 0; s < B; s++) {
    const int n = std::min(cnt[s], cap);
    for (int i = 0; i < n; i++) {
      const float* d = recs + ((size_t)s * e->opt.max_det + i) * 6;
      YoloDet& o = out[(size_t)s * cap + i];
      o.x1 = (d[0] - b.geom.left) / b.geom.scale;
      o.y1 = (d[1] - b.geom.top) / b.geom.scale;
      o.x2 = (d[2] - b.geom.left) / b.geom.scale;
      o.y2 = (d[3] - b.geom.top) / b.geom.scale;
      o.score = d[4];
      o.cls = (int)d[5];
    }
    counts[s] = n;
    total += n;
  }
  return total;
}

int yolo_get_batch(void* h, int B, YoloDet* out, int cap, int* counts) {
  Engine* e = as_engine(h);
  if (!e || e->obb() || B < 1 || B > e->maxB || cap < 0 || (!out && cap > 0) || !counts)
    return -1;
  int total = 0;
  for (int s = 0; s < B; s++) {
    counts[s] = yolo_get(h, s, out ? out + (size_t)s * cap : nullptr, cap);
    total += counts[s];
  }
  return total;
}

int yolo_get(void* h, int slot, YoloDet* out, int cap) {
  Engine* e = as_engine(h);
  if (!e || e->obb() || slot < 0 || slot >= e->maxB || (!out && cap > 0)) return 0;
  const SlotGeom& g = e->slots[slot];
  const int n = std::min(e->h_cnt[slot], cap);
  for (int i = 0; i < n; i++) {
    const float* d = e->h_out + ((size_t)slot * e->opt.max_det + i) * 6;
    out[i].x1 = (d[0] - g.left) / g.scale;
    out[i].y1 = (d[1] - g.top) / g.scale;
    out[i].x2 = (d[2] - g.left) / g.scale;
    out[i].y2 = (d[3] - g.top) / g.scale;
    out[i].score = d[4];
    out[i].cls = (int)d[5];
  }
  return n;
}

int yolo_raw_count(void* h, int slot) {
  Engine* e = as_engine(h);
  if (!e || slot < 0 || slot >= e->maxB) return -1;
  return e->h_raw[slot];
}

void yolo_slot_geom(void* h, int slot, float* scale, int* top, int* left) {
  Engine* e = as_engine(h);
  if (!e || slot < 0 || slot >= e->maxB) return;
  const SlotGeom& g = e->slots[slot];
  if (scale) *scale = g.scale;
  if (top) *top = g.top;
  if (left) *left = g.left;
}

void yolo_mask_dim(void* h, int* ph, int* pw) {
  Engine* e = as_engine(h);
  int H = 0, W = 0;
  if (e && e->seg()) {
    const Buf& b = e->bufs[e->tens[e->protoTen].buf];
    H = b.H; W = b.W;
  }
  if (ph) *ph = H;
  if (pw) *pw = W;
}

int yolo_get_mask(void* h, int slot, int det, unsigned char* out) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || !e->seg() || slot < 0 || slot >= e->maxB || det < 0 || det >= e->h_cnt[slot] || !out)
      return -1;
    DeviceScope ds(e->device);
    const Buf& b = e->bufs[e->tens[e->protoTen].buf];
    const size_t sz = (size_t)b.H * b.W;
    CKE(cudaMemcpy(out, e->dmasks + ((size_t)slot * e->opt.max_det + det) * sz, sz,
                   cudaMemcpyDeviceToHost));
    return 0;
  }, -1);
}

int yolo_num_ops(void* h) { return h ? (int)as_engine(h)->raw.size() : -1; }

int yolo_run_op(void* h, int op_index, int B) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || op_index < 0 || op_index >= (int)e->raw.size() || B < 1 || B > e->maxB)
      throw Error("yolo_run_op: bad arguments");
    DeviceScope ds(e->device);
    const Op& op = e->raw[op_index];
    if (op.kind == DECODE || op.kind == DECODESEG || op.kind == DECODEOBB || op.kind == MASKS) {
      // the whole post chain runs once, at the last head op of the graph
      bool last = true;
      for (size_t j = op_index + 1; j < e->raw.size(); j++)
        if (e->raw[j].kind == DECODE || e->raw[j].kind == DECODESEG ||
            e->raw[j].kind == DECODEOBB || e->raw[j].kind == MASKS)
          last = false;
      if (last) {
        e->run_post(B);
        e->use_results(e->hres);
      }
      CKE(cudaStreamSynchronize(e->st));
      return 1;
    }
    Op o = op;
    if (o.kind == CONV && o.g == 1 && o.Cin % 8 == 0) {
      for (const Op& f : e->ops)   // reuse the tuned tile of the matching planned conv
        if (f.kind == CONV && f.woff == o.woff) { o.tile = f.tile; o.msub = f.msub; o.algo = f.algo; }
    }
    e->run_op(o, B);
    CKE(cudaStreamSynchronize(e->st));
    int derr = yk_fetch_device_error();
    if (derr) throw Error("device error word set: " + std::to_string(derr));
    return 0;
  }, -2);
}

int yolo_tensor_view(void* h, int tensor, void** ptr, int* H, int* W, int* stride, int* coff,
                     int* C) {
  Engine* e = as_engine(h);
  if (!e || tensor < 0 || tensor >= (int)e->tens.size()) return -1;
  YkView v = e->view(tensor, e->maxB);
  if (ptr) *ptr = v.ptr;
  if (H) *H = v.H;
  if (W) *W = v.W;
  if (stride) *stride = v.stride;
  if (coff) *coff = v.coff;
  if (C) *C = v.C;
  return 0;
}

static int copy_tensor(void* h, int tensor, int B, void* host, bool to_host) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || tensor < 0 || tensor >= (int)e->tens.size() || B < 1 || B > e->maxB || !host)
      throw Error("yolo_read/write_tensor: bad arguments");
    DeviceScope ds(e->device);
    CKE(cudaStreamSynchronize(e->st));
    YkView v = e->view(tensor, B);
    char* dev = (char*)v.ptr + (size_t)v.coff * 2;
    const size_t rows = (size_t)B * v.H * v.W;
    // on the engine stream (non-blocking w.r.t. the legacy stream), then wait for it: a
    // plain cudaMemcpy from pageable memory may return before the data reaches the device
    if (to_host)
      CKE(cudaMemcpy2DAsync(host, (size_t)v.C * 2, dev, (size_t)v.stride * 2, (size_t)v.C * 2,
                            rows, cudaMemcpyDeviceToHost, e->st));
    else
      CKE(cudaMemcpy2DAsync(dev, (size_t)v.stride * 2, host, (size_t)v.C * 2, (size_t)v.C * 2,
                            rows, cudaMemcpyHostToDevice, e->st));
    CKE(cudaStreamSynchronize(e->st));
    return 0;
  }, -1);
}

int yolo_read_tensor(void* h, int tensor, int B, void* host) {
  return copy_tensor(h, tensor, B, host, true);
}
int yolo_write_tensor(void* h, int tensor, int B, const void* host) {
  return copy_tensor(h, tensor, B, (void*)host, false);
}

const char* yolo_op_desc(void* h, int op_index, int* tile) {
  Engine* e = as_engine(h);
  if (!e || op_index < 0 || op_index >= (int)e->ops.size()) return nullptr;
  if (tile) *tile = e->ops[op_index].tile;
  return kKindNames[e->ops[op_index].kind];
}

int yolo_op_shape(void* h, int op_index, int* info) {
  Engine* e = as_engine(h);
  if (!e || !info || op_index < 0 || op_index >= (int)e->ops.size()) return -1;
  const Op& o = e->ops[op_index];
  const Buf& b = e->bufs[e->tens[o.out >= 0 ? o.out : o.a].buf];
  const int v[10] = {o.Cin, o.Cout, o.k, o.s, o.g, b.H, b.W, o.algo, o.msub, o.res >= 0};
  for (int i = 0; i < 10; i++) info[i] = v[i];
  return 0;
}

int yolo_profile(void* h, int B, int iters, float* ms, int cap) {
  return guarded([&]() -> int {
    Engine* e = as_engine(h);
    if (!e || B < 1 || B > e->maxB || iters < 1) throw Error("yolo_profile: bad arguments");
    DeviceScope ds(e->device);
    const int n = (int)e->ops.size();
    std::vector<cudaEvent_t> ev(n + 2);
    for (auto& x : ev) CKE(cudaEventCreate(&x));
    std::vector<double> acc(n + 1, 0.0);
    for (int w = 0; w < 3; w++) e->forward(B);
    for (int it = 0; it < iters; it++) {
      CKE(cudaEventRecord(ev[0], e->st));
      for (int k = 0; k < n; k++) {
        e->run_op(e->ops[k], B);
        CKE(cudaEventRecord(ev[k + 1], e->st));
      }
      e->run_post(B);
      CKE(cudaEventRecord(ev[n + 1], e->st));
      CKE(cudaEventSynchronize(ev[n + 1]));
      for (int k = 0; k <= n; k++) {
        float t = 0;
        cudaEventElapsedTime(&t, ev[k], ev[k + 1]);
        acc[k] += t;
      }
    }
    for (auto& x : ev) cudaEventDestroy(x);
    for (int k = 0; k <= n && k < cap; k++) ms[k] = (float)(acc[k] / iters);
    return n + 1;   // the last entry is the decode + NMS (+ masks) tail
  }, -1);
}

}  // extern "C"
