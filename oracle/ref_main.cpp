// TEST INFRASTRUCTURE ONLY — the CPU baseline / reference arm.
//
// Runs yalm's own decode path on a .yalm file the way run_completion does (src/main.cpp:121-211):
// the model on the CPU or moved to a device as setup_cuda does (src/main.cpp:57-86), one warm-up
// forward at position 0 (main.cpp:148), prompt tokens one forward each (HYDRATE except the last,
// main.cpp:171-177), then greedy decode steps with argmax (sampler.cpp:27-38).  Prompt ids come
// from argv so no tokenizer is involved.  Prints one JSON line with per-phase wall times
// (steady_clock) and the greedy ids.
//
//   ref_decode <file.yalm> <context> <n_decode> <threads> [-d cpu|cuda|cuda-coop] <id0> <id1> ...
#include "model.h"

#include <chrono>
#include <cfloat>
#include <cstdio>
#include <cstdlib>
#include <omp.h>
#include <string>
#include <vector>

extern "C" void* ref_open(const char* path, int context);

static double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

extern "C" void ref_forward(void* hp, int token, int pos, int mode, float* logits_out);
extern "C" void ref_config(void* hp, int* out12, float* out3);
extern "C" int ref_to_device(void* hp, const char* device);

int main(int argc, char** argv) {
  if (argc < 6) {
    std::fprintf(stderr, "usage: %s <file.yalm> <context> <n_decode> <threads> <prompt ids...>\n", argv[0]);
    return 2;
  }
  const char* path = argv[1];
  int context = std::atoi(argv[2]);
  int n_decode = std::atoi(argv[3]);
  int threads = std::atoi(argv[4]);
  if (threads > 0) omp_set_num_threads(threads);
  std::string device = "cpu";
  int first_id = 5;
  if (argc > 6 && std::string(argv[5]) == "-d") {
    device = argv[6];
    first_id = 7;
  }
  std::vector<int> prompt;
  for (int i = first_id; i < argc; ++i) prompt.push_back(std::atoi(argv[i]));
  if (prompt.empty()) {
    std::fprintf(stderr, "ref_decode: no prompt ids\n");
    return 2;
  }

  double t0 = now_s();
  void* h = ref_open(path, context);
  if (!h) {
    std::fprintf(stderr, "ref_decode: cannot open %s\n", path);
    return 1;
  }
  int cfg[12];
  float cfgf[3];
  ref_config(h, cfg, cfgf);
  int vocab = cfg[6];
  std::vector<float> logits(vocab);
  if (ref_to_device(h, device.c_str()) != 0) {
    std::fprintf(stderr, "ref_decode: unknown device %s\n", device.c_str());
    return 2;
  }
  ref_forward(h, 0, 0, 1, logits.data());  // run_completion's warm-up forward (main.cpp:148)
  double t1 = now_s();
  for (size_t p = 0; p < prompt.size(); ++p) {
    int mode = (p + 1 == prompt.size()) ? 1 : 0;
    ref_forward(h, prompt[p], (int)p, mode, logits.data());
  }
  double t2 = now_s();
  std::vector<int> out;
  std::vector<double> step_s;
  int pos = (int)prompt.size();
  for (int i = 0; i < n_decode; ++i) {
    int best = 0;
    float mx = -FLT_MAX;
    for (int v = 0; v < vocab; ++v) {
      if (logits[v] > mx) {
        mx = logits[v];
        best = v;
      }
    }
    out.push_back(best);
    double a = now_s();
    ref_forward(h, best, pos++, 1, logits.data());
    step_s.push_back(now_s() - a);
  }
  double t3 = now_s();
  std::printf("{\"device\": \"%s\", \"load_s\": %.6f, \"prefill_s\": %.6f, \"decode_s\": %.6f, \"n_prompt\": %zu, "
              "\"n_decode\": %d, \"threads\": %d, \"step_s\": [",
              device.c_str(), t1 - t0, t2 - t1, t3 - t2, prompt.size(), n_decode, omp_get_max_threads());
  for (size_t i = 0; i < step_s.size(); ++i) std::printf("%s%.6f", i ? ", " : "", step_s[i]);
  std::printf("], \"tokens\": [");
  for (size_t i = 0; i < out.size(); ++i) std::printf("%s%d", i ? ", " : "", out[i]);
  std::printf("]}\n");
  return 0;
}
