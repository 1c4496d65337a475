// ref_load.cpp — times the reference's own weight loader onto the GPU.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile (target dropin) against
// the reference's sources with its CUDA backend. Runs ModelWeights::load(path,
// CUDA) (src/model/weights.cpp:47-163: host reads, host INT8 dequant +
// float_to_half, blocking uploads), synchronises, prints the wall time, then
// one checksum line per tensor of the loaded device bytes:
//   load_seconds <s>
//   <name> <sum64> <xor64>
// where sum64 / xor64 are the wrapping sum / xor of the tensor's bytes read
// as little-endian uint64 words (zero-padded to 8 bytes).
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "kllm/base/tensor.h"
#include "kllm/model/weights.h"

int main(int argc, char** argv) {
  if (argc != 3) {
    std::fprintf(stderr, "usage: %s MODEL.kllm NAMES.txt\n", argv[0]);
    return 2;
  }
  try {
    const auto t0 = std::chrono::steady_clock::now();
    kllm::ModelWeights w = kllm::ModelWeights::load(argv[1], kllm::DeviceType::CUDA);
    if (cudaDeviceSynchronize() != cudaSuccess) throw std::runtime_error("cudaDeviceSynchronize failed");
    const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    std::printf("load_seconds %.6f\n", secs);
    std::ifstream names(argv[2]);
    std::string name;
    while (std::getline(names, name)) {
      const kllm::Tensor* t = w.find(name);
      if (t == nullptr) throw std::runtime_error("missing tensor " + name);
      std::vector<unsigned char> host((t->nbytes() + 7) / 8 * 8, 0);
      t->copy_to_host(host.data(), t->nbytes());
      std::uint64_t sum = 0, x = 0;
      for (std::size_t i = 0; i < host.size(); i += 8) {
        std::uint64_t v;
        std::memcpy(&v, host.data() + i, 8);
        sum += v;
        x ^= v;
      }
      std::printf("%s %llu %llu\n", name.c_str(), (unsigned long long)sum, (unsigned long long)x);
    }
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
}
