// dropin_forward.cpp — LittleLLM's own model runner on its CPU backend and on
// its CUDA backend, same model file, same tokens; prints the largest logit
// difference of every step.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile links this against the
// reference's sources (ModelWeights::load, LlamaRunner::forward,
// src/model/{weights,llama}.cpp) twice: once with the in-scope CUDA operators
// from littlellm_b200 (the drop-in build) and once with the reference's own
// CUDA operators, so the two CUDA backends can be compared with each other
// and with the fp32 CPU path.
//
// usage: dropin_forward MODEL.kllm IDS_CSV DECODE_STEPS MAX_SEQ
// output, one line per step:  step <s> max_abs_diff <d> max_abs_cpu <m> argmax_cpu <i> argmax_cuda <j>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <sstream>
#include <string>
#include <vector>

#include "kllm/base/tensor.h"
#include "kllm/model/llama.h"
#include "kllm/model/weights.h"

namespace {

std::vector<int> parse_ids(const std::string& csv) {
  std::vector<int> ids;
  std::stringstream ss(csv);
  std::string item;
  while (std::getline(ss, item, ',')) {
    if (!item.empty()) ids.push_back(std::stoi(item));
  }
  return ids;
}

int argmax(const std::vector<float>& v) {
  return static_cast<int>(std::max_element(v.begin(), v.end()) - v.begin());
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 5) {
    std::fprintf(stderr, "usage: %s MODEL.kllm IDS_CSV DECODE_STEPS MAX_SEQ\n", argv[0]);
    return 2;
  }
  try {
    const std::string path = argv[1];
    std::vector<int> ids = parse_ids(argv[2]);
    const int steps = std::atoi(argv[3]);
    const int max_seq = std::atoi(argv[4]);
    kllm::LlamaRunner cpu(kllm::ModelWeights::load(path, kllm::DeviceType::CPU), kllm::DeviceType::CPU, max_seq);
    kllm::LlamaRunner gpu(kllm::ModelWeights::load(path, kllm::DeviceType::CUDA), kllm::DeviceType::CUDA, max_seq);
    int past = 0;
    std::vector<int> input = ids;
    for (int s = 0; s <= steps; ++s) {
      const std::vector<float> a = cpu.forward(input, past).to_float_vector();
      const std::vector<float> b = gpu.forward(input, past).to_float_vector();
      if (a.size() != b.size()) {
        std::fprintf(stderr, "logit sizes differ: %zu vs %zu\n", a.size(), b.size());
        return 1;
      }
      float diff = 0.0f, mag = 0.0f;
      for (std::size_t i = 0; i < a.size(); ++i) {
        diff = std::max(diff, std::fabs(a[i] - b[i]));
        mag = std::max(mag, std::fabs(a[i]));
      }
      const int next = argmax(a);
      std::printf("step %d max_abs_diff %.6g max_abs_cpu %.6g argmax_cpu %d argmax_cuda %d\n", s, diff, mag, next,
                  argmax(b));
      past += static_cast<int>(input.size());
      input = {next};  // both runners continue with the CPU's greedy token
    }
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
}
