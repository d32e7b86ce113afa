// yolocuda — command-line front end of the B200 engine, built on the yolo.h C ABI only.
// Same modes and arguments as the reference CLI (engine/engine.cu:1638-1651, 1796-2096):
//   yolocuda <detect|pipeline|bench|profile|dump> [model-dir] [iters] [--image path.jpg]
//            [--batch N] [--save-masks]
// Additions: `pipeline` and `bench` report p50/p99 besides the mean; --iou / --conf.
// `pipeline` replays one CUDA graph per iteration (H2D of the raw frames + letterbox of the
// batch + net + decode + NMS + D2H, yolo_bind_frames / yolo_run_frames).  --image decodes a
// JPEG on the GPU (nvJPEG, yolo_preprocess_jpeg); the reference decodes any format with
// stb_image on the host (engine/engine.cu:1630-1636, 1891-1897).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/yolo.h"

static std::vector<char> slurp(const std::string& p) {
  std::vector<char> v;
  FILE* f = fopen(p.c_str(), "rb");
  if (!f) return v;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  v.resize(n);
  if (n && fread(v.data(), 1, n, f) != (size_t)n) v.clear();
  fclose(f);
  return v;
}

#define CK(x)                                                                              \
  do {                                                                                     \
    cudaError_t e_ = (x);                                                                  \
    if (e_ != cudaSuccess) {                                                               \
      fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
      return 1;                                                                            \
    }                                                                                      \
  } while (0)

static void usage() {
  printf("yolocuda - B200 (sm_100a) inference engine for YOLOv8 / YOLO11\n\n"
         "usage: yolocuda <mode> [model-dir] [iters] [--image path.jpg] [--batch N] [--save-masks]\n"
         "                [--iou X] [--conf X]\n\n"
         "modes:\n"
         "  detect    one inference on the directory's input.f16 (or --image, a JPEG decoded on\n"
         "            the GPU), print detections (segment: --save-masks; obb: oriented boxes;\n"
         "            classify: top-5 with names.txt)\n"
         "  bench     net + post-processing CUDA-graph latency (mean / p50 / p99)\n"
         "  pipeline  end to end: H2D of the raw frame + preprocessing (letterbox, or the\n"
         "            classify resize + crop) + net + post-processing\n"
         "  profile   per-op device time of the planned op list\n"
         "  dump      per-op outputs (gpu/opNNN.bin) with reference resync for compare.py\n");
}

// fp32 payload of a C-order .npy file with a v1/v2 header; empty on mismatch
static std::vector<float> read_npy_f32(const std::string& path, size_t count) {
  std::vector<float> out;
  auto raw = slurp(path);
  if (raw.size() < 10 || memcmp(raw.data(), "\x93NUMPY", 6)) return out;
  size_t hlen, off;
  if (raw[6] == 1) { hlen = (uint8_t)raw[8] | ((uint8_t)raw[9] << 8); off = 10; }
  else { hlen = (uint8_t)raw[8] | ((uint8_t)raw[9] << 8) | ((size_t)(uint8_t)raw[10] << 16); off = 12; }
  std::string hdr(raw.data() + off, hlen);
  if (hdr.find("<f4") == std::string::npos || hdr.find("True") != std::string::npos) return out;
  if (raw.size() != off + hlen + count * 4) return out;
  out.resize(count);
  memcpy(out.data(), raw.data() + off + hlen, count * 4);
  return out;
}

static double pct(std::vector<double> v, double p) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  size_t i = (size_t)std::min<double>(v.size() - 1, p * (v.size() - 1) + 0.5);
  return v[i];
}

static int load_input(void* h, const std::string& dir, int batch) {
  auto in = slurp(dir + "/input.f16");
  void* p; int H, W, s, c, C;
  yolo_tensor_view(h, 0, &p, &H, &W, &s, &c, &C);
  if (in.size() != (size_t)H * W * 3 * 2) {
    fprintf(stderr, "input.f16 missing or wrong size\n");
    return 1;
  }
  for (int b = 0; b < batch; b++)
    CK(cudaMemcpy((char*)p + (size_t)b * in.size(), in.data(), in.size(), cudaMemcpyHostToDevice));
  CK(cudaDeviceSynchronize());
  return 0;
}

static void print_dets(void* h, int slot, bool orig) {
  std::vector<YoloDet> d(100000);
  int n = yolo_get(h, slot, d.data(), (int)d.size());
  float sc; int top, left;
  yolo_slot_geom(h, slot, &sc, &top, &left);
  printf("kept=%d (candidates %d)%s\n", n, yolo_raw_count(h, slot),
         orig ? "  (boxes in original image coords)" : "");
  for (int i = 0; i < n; i++)
    printf("cls=%2d score=%.4f box=(%.1f, %.1f, %.1f, %.1f)\n", d[i].cls, d[i].score, d[i].x1,
           d[i].y1, d[i].x2, d[i].y2);
}

// classify models: top-5 of slot 0 with names from <dir>/names.txt (index if absent), and
// the top-1 of every slot for the batch self-consistency check
static void print_cls(void* h, const std::string& dir, int batch) {
  std::vector<std::string> names;
  if (FILE* f = fopen((dir + "/names.txt").c_str(), "r")) {
    char line[256];
    while (fgets(line, sizeof line, f)) {
      std::string n = line;
      while (!n.empty() && (n.back() == '\n' || n.back() == '\r')) n.pop_back();
      names.push_back(n);
    }
    fclose(f);
  }
  int ids[5];
  float probs[5];
  if (batch > 1) {
    printf("batch=%d per-image top1:", batch);
    int c0 = -1;
    bool same = true;
    for (int b = 0; b < batch; b++) {
      yolo_get_cls(h, b, ids, probs, 1);
      printf(" %d", ids[0]);
      if (b == 0) c0 = ids[0];
      same &= ids[0] == c0;
    }
    printf("  %s\n", same ? "(consistent)" : "(MISMATCH!)");
  }
  const int n = yolo_get_cls(h, 0, ids, probs, 5);
  printf("top5:\n");
  for (int i = 0; i < n; i++)
    printf("%4d %-24s %.4f\n", ids[i],
           ids[i] >= 0 && ids[i] < (int)names.size() ? names[ids[i]].c_str() : "", probs[i]);
}

int main(int argc, char** argv) {
  std::string mode = argc > 1 ? argv[1] : "detect";
  std::string dir = "build/yolo11n";
  int iters = -1, batch = 1;
  bool save_masks = false;
  std::string image;
  YoloOptions opt;
  yolo_default_options(&opt);
  for (int i = 2; i < argc; i++) {
    std::string a = argv[i];
    if (a == "--batch" && i + 1 < argc) batch = atoi(argv[++i]);
    else if (a == "--image" && i + 1 < argc) image = argv[++i];
    else if (a == "--iou" && i + 1 < argc) opt.iou = (float)atof(argv[++i]);
    else if (a == "--conf" && i + 1 < argc) opt.conf = (float)atof(argv[++i]);
    else if (a == "--save-masks") save_masks = true;
    else if (a == "-h" || a == "--help") { usage(); return 0; }
    else if (a[0] >= '0' && a[0] <= '9') iters = atoi(a.c_str());
    else dir = a;
  }
  if (mode != "detect" && mode != "bench" && mode != "pipeline" && mode != "profile" &&
      mode != "dump") {
    usage();
    return mode == "-h" || mode == "--help" || mode == "help" ? 0 : 1;
  }
  if (getenv("NOFUSE") || mode == "dump") opt.fuse = 0;
  if (getenv("NOTUNE") || mode == "dump") opt.autotune = 0;
  void* h = yolo_create_ex(dir.c_str(), batch, &opt);
  if (!h) {
    fprintf(stderr, "yolo_create failed: %s\n", yolo_last_error());
    return 1;
  }
  if (load_input(h, dir, batch)) return 1;
  if (!image.empty() && mode == "detect") {   // any JPEG: nvJPEG decode + preprocessing per slot
    auto bytes = slurp(image);
    if (bytes.empty()) { fprintf(stderr, "cannot read image %s\n", image.c_str()); return 1; }
    for (int b = 0; b < batch; b++)
      if (yolo_preprocess_jpeg(h, (const unsigned char*)bytes.data(), bytes.size(), b) != 0) {
        fprintf(stderr, "image %s: %s\n", image.c_str(), yolo_last_error());
        return 1;
      }
  }

  if (mode == "dump") {
    if (system(("mkdir -p " + dir + "/gpu").c_str()) != 0) return 1;
    const int n = yolo_num_ops(h);
    for (int k = 0; k < n; k++) {
      int r = yolo_run_op(h, k, batch);
      if (r < 0) { fprintf(stderr, "op %d: %s\n", k, yolo_last_error()); return 1; }
      if (r == 1) continue;
      // output view of op k: read the op's tensor through the graph file order
      int t = -1;
      {
        // yolo_run_op does not expose the op; re-parse cheaply from model.graph
        static std::vector<int> outs;
        if (outs.empty()) {
          FILE* f = fopen((dir + "/model.graph").c_str(), "r");
          char tag[64]; int ver, nb, nt, no;
          if (fscanf(f, "%63s %d", tag, &ver) != 2) return 1;
          if (ver >= 2) { char t2[64]; int a, b; if (fscanf(f, "%63s %63s %d %d", tag, t2, &a, &b) != 4) return 1; }
          if (fscanf(f, "%d %d %d", &nb, &nt, &no) != 3) return 1;
          char line[512];
          if (!fgets(line, sizeof line, f)) return 1;
          for (int i = 0; i < nb + nt; i++) if (!fgets(line, sizeof line, f)) return 1;
          for (int i = 0; i < no; i++) {
            if (!fgets(line, sizeof line, f)) return 1;
            char kind[32]; int v0 = -1, v1 = -1, v2 = -1;
            sscanf(line, "%31s %d %d %d", kind, &v0, &v1, &v2);
            outs.push_back(!strcmp(kind, "ADD") ? v2 : v1);
          }
          fclose(f);
        }
        t = outs[k];
      }
      void* p; int H, W, s, c, C;
      yolo_tensor_view(h, t, &p, &H, &W, &s, &c, &C);
      std::vector<__half> host((size_t)H * W * C);
      CK(cudaMemcpy2D(host.data(), C * 2, (char*)p + (size_t)c * 2, (size_t)s * 2, C * 2,
                      (size_t)H * W, cudaMemcpyDeviceToHost));
      char path[512];
      snprintf(path, sizeof path, "%s/gpu/op%03d.bin", dir.c_str(), k);
      FILE* f = fopen(path, "wb");
      fwrite(host.data(), 2, host.size(), f);
      fclose(f);
      // resync with the reference output so each op sees exact inputs (isolated kernel check)
      snprintf(path, sizeof path, "%s/ref/op%03d.npy", dir.c_str(), k);
      auto rf = read_npy_f32(path, host.size());
      if (!rf.empty()) {
        for (size_t i = 0; i < host.size(); i++) host[i] = __float2half(rf[i]);
        CK(cudaMemcpy2D((char*)p + (size_t)c * 2, (size_t)s * 2, host.data(), C * 2, C * 2,
                        (size_t)H * W, cudaMemcpyHostToDevice));
        CK(cudaDeviceSynchronize());
      }
    }
    printf("dumped %d ops\n", n);
  } else if (mode == "detect") {
    yolo_run(h, batch);
    if (*yolo_last_error()) { fprintf(stderr, "run: %s\n", yolo_last_error()); return 1; }
    if (yolo_task(h) == 2) {
      print_cls(h, dir, batch);
      yolo_destroy(h);
      return 0;
    }
    if (yolo_task(h) == 1) {   // oriented boxes, original image coordinates
      std::vector<YoloObbDet> d(10000);
      const int n = yolo_get_obb(h, 0, d.data(), (int)d.size());
      printf("kept=%d (candidates %d)\n", n, yolo_raw_count(h, 0));
      for (int i = 0; i < n; i++)
        printf("cls=%2d score=%.4f obb=(%.1f, %.1f, %.1f, %.1f, %.3f rad)\n", d[i].cls, d[i].score,
               d[i].x, d[i].y, d[i].w, d[i].h, d[i].angle);
      yolo_destroy(h);
      return 0;
    }
    if (batch > 1) {
      printf("batch=%d per-image kept:", batch);
      std::vector<YoloDet> d(100000);
      int n0 = yolo_get(h, 0, d.data(), (int)d.size());
      bool same = true;
      for (int b = 0; b < batch; b++) {
        int nb = yolo_get(h, b, d.data(), (int)d.size());
        printf(" %d", nb);
        same &= nb == n0;
      }
      printf("  %s\n", same ? "(consistent)" : "(MISMATCH!)");
    }
    print_dets(h, 0, !image.empty());
    int ph, pw;
    yolo_mask_dim(h, &ph, &pw);
    if (save_masks && ph) {
      std::vector<YoloDet> d(100000);
      int n = yolo_get(h, 0, d.data(), (int)d.size());
      std::vector<unsigned char> m((size_t)n * ph * pw);
      for (int i = 0; i < n; i++) yolo_get_mask(h, 0, i, m.data() + (size_t)i * ph * pw);
      if (system(("mkdir -p " + dir + "/gpu").c_str()) != 0) return 1;
      FILE* f = fopen((dir + "/gpu/masks.u8").c_str(), "wb");
      fwrite(m.data(), 1, m.size(), f);
      fclose(f);
      f = fopen((dir + "/gpu/dets.f32").c_str(), "wb");
      for (int i = 0; i < n; i++) {
        float r[6] = {d[i].x1, d[i].y1, d[i].x2, d[i].y2, d[i].score, (float)d[i].cls};
        fwrite(r, 4, 6, f);
      }
      fclose(f);
      printf("wrote %s/gpu/masks.u8 (%d x %dx%d) + dets.f32\n", dir.c_str(), n, ph, pw);
    }
  } else if (mode == "pipeline" || mode == "bench") {
    const int it = iters > 0 ? iters : 300;
    unsigned char* himg = nullptr;
    if (mode == "pipeline") {   // the exporter's raw frame, pinned, bound as the graph's input
      int sh = 0, sw = 0;
      FILE* fd = fopen((dir + "/bus_raw.txt").c_str(), "r");
      if (!fd || fscanf(fd, "%d %d", &sh, &sw) != 2) { fprintf(stderr, "no bus_raw.txt\n"); return 1; }
      fclose(fd);
      auto raw = slurp(dir + "/bus_raw.u8");
      if (raw.size() != (size_t)sh * sw * 3) { fprintf(stderr, "bad bus_raw.u8\n"); return 1; }
      CK(cudaMallocHost(&himg, raw.size() * batch));
      for (int b = 0; b < batch; b++) memcpy(himg + b * raw.size(), raw.data(), raw.size());
      if (yolo_bind_frames(h, 0, himg, sh, sw, batch, 1) != 0) {
        fprintf(stderr, "bind: %s\n", yolo_last_error());
        return 1;
      }
    }
    const float graph_ms = himg ? yolo_frames_exec_ms(h, 0, batch) : yolo_exec_ms(h, batch);
    std::vector<YoloDet> d((size_t)300 * batch);
    std::vector<int> counts(batch);
    std::vector<double> lat;
    for (int i = 0; i < 20 + it; i++) {
      auto t0 = std::chrono::steady_clock::now();
      if (himg) {
        if (yolo_run_frames(h, 0, batch) != 0) { fprintf(stderr, "run: %s\n", yolo_last_error()); return 1; }
      } else {
        yolo_run(h, batch);
      }
      if (yolo_task(h) != 1 && yolo_task(h) != 2) yolo_get_batch(h, batch, d.data(), 300, counts.data());
      auto t1 = std::chrono::steady_clock::now();
      if (i >= 20) lat.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
    }
    if (*yolo_last_error()) { fprintf(stderr, "run: %s\n", yolo_last_error()); return 1; }
    double mean = 0;
    for (double v : lat) mean += v;
    mean /= lat.size();
    printf("%s (B=%d): mean %.3f ms  p50 %.3f ms  p99 %.3f ms  (%.1f frames/s at p50); "
           "graph exec %.3f ms\n",
           mode == "pipeline"
               ? (yolo_task(h) == 2 ? "end-to-end pipeline graph (H2D + preprocess + net + probs D2H)"
                                    : "end-to-end pipeline graph (H2D + letterbox + net + decode + NMS + D2H)")
               : (yolo_task(h) == 2 ? "cuda graph (net + softmax + probs D2H)"
                                    : "cuda graph (net + decode + NMS)"),
           batch, mean, pct(lat, 0.5), pct(lat, 0.99), 1000.0 * batch / pct(lat, 0.5), graph_ms);
    if (mode == "pipeline" && yolo_task(h) != 2) print_dets(h, 0, true);
    if (himg) cudaFreeHost(himg);
  } else if (mode == "profile") {
    std::vector<float> ms(4096);
    int n = yolo_profile(h, batch, 50, ms.data(), (int)ms.size());
    if (n < 0) { fprintf(stderr, "profile: %s\n", yolo_last_error()); return 1; }
    std::vector<int> order(n);
    double tot = 0;
    for (int i = 0; i < n; i++) { order[i] = i; tot += ms[i]; }
    std::sort(order.begin(), order.end(), [&](int a, int b) { return ms[a] > ms[b]; });
    printf("total %.3f ms/iter (B=%d) - top ops:\n", tot, batch);
    const int top = getenv("YOLO_PROFILE_ALL") ? n : 25;
    for (int i = 0; i < top && i < n; i++) {
      int k = order[i], tile = 0;
      const char* kind = k == n - 1 ? "POST" : yolo_op_desc(h, k, &tile);
      int si[10] = {0};
      char shape[96] = "";
      if (k < n - 1 && !strcmp(kind, "CONV") && yolo_op_shape(h, k, si) == 0)
        snprintf(shape, sizeof shape, "  %d->%d k%ds%d g%d %dx%d algo%d ms%d%s", si[0], si[1],
                 si[2], si[3], si[4], si[5], si[6], si[7], si[8], si[9] ? " +res" : "");
      printf("op%03d %-9s tile=%-3d %8.1f us (%4.1f%%)%s\n", k, kind, tile, ms[k] * 1000.0,
             100.0 * ms[k] / tot, shape);
    }
  }
  yolo_destroy(h);
  return 0;
}
