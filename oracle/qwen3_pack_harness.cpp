// Drives the reference's own ternary packer, addPacked() of qwen3/convert.cpp:39-74, on raw
// buffers: the reference file is compiled into this translation unit (its main() renamed), so
// the call reaches its anonymous-namespace function unchanged. TEST INFRASTRUCTURE ONLY.
//
//   qwen3_pack <codes.u32 [n][k/16]> <scales.f16 [n][k/128]> <biases.f16 [n][k/128]> <n> <k> <out dir>
// writes <out dir>/weights.bin (t.w then t.s, as addPacked lays them out) and manifest.txt;
// exits 1 with the reference's message when a group is not ternary (bias != -scale).
#define main qwen3_convert_main
#include REF_QWEN3_CONVERT
#undef main

#include <fstream>
#include <iterator>

static std::vector<char> slurp(const char *path) {
  std::ifstream f(path, std::ios::binary);
  return std::vector<char>(std::istreambuf_iterator<char>(f), {});
}

int main(int argc, char **argv) {
  if (argc != 7) {
    fprintf(stderr, "usage: qwen3_pack codes scales biases n k outdir\n");
    return 2;
  }
  const int64_t n = atoll(argv[4]), k = atoll(argv[5]);
  std::vector<char> w = slurp(argv[1]), s = slurp(argv[2]), b = slurp(argv[3]);
  if (static_cast<int64_t>(w.size()) != n * k / 16 * 4 || static_cast<int64_t>(s.size()) != n * k / 128 * 2 ||
      s.size() != b.size()) {
    fprintf(stderr, "qwen3_pack: input sizes do not match n=%lld k=%lld\n", (long long)n, (long long)k);
    return 2;
  }
  tensors["t.weight"] = Tensor{"U32", {n, k / 16}, w.data()};
  tensors["t.scales"] = Tensor{"F16", {n, k / 128}, s.data()};
  tensors["t.biases"] = Tensor{"F16", {n, k / 128}, b.data()};
  std::string dir = argv[6];
  weights = fopen((dir + "/weights.bin").c_str(), "wb");
  manifest = fopen((dir + "/manifest.txt").c_str(), "w");
  if (!weights || !manifest) return 2;
  try {
    addPacked("t", {"t"}, k);
  } catch (const std::exception &e) {
    fprintf(stderr, "qwen3_pack: %s\n", e.what());
    return 1;
  }
  fclose(weights);
  fclose(manifest);
  return 0;
}
