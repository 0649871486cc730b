// gen_std_random.cpp — prints the exact input values the reference's tests
// draw, so the golden fixtures can reproduce them:
//   mt19937 <seed> <count> <lo> <hi> : std::mt19937(seed) with
//       std::uniform_real_distribution<float>(lo, hi), as in
//       tests/compute/test_wmma.cu:33-39 and tests/test_end2end.cpp:32-53;
//   rand <count> : static_cast<float>(rand()) / RAND_MAX with glibc's
//       unseeded rand(), as in tests/test_baselines.cpp:248-249.
// Output: one IEEE-754 float bit pattern per line, hexadecimal.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>

static void emit(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  std::printf("%08x\n", b);
}

int main(int argc, char** argv) {
  if (argc >= 6 && std::string(argv[1]) == "mt19937") {
    std::mt19937 gen(static_cast<unsigned>(std::strtoul(argv[2], nullptr, 10)));
    const long n = std::strtol(argv[3], nullptr, 10);
    std::uniform_real_distribution<float> dist(std::strtof(argv[4], nullptr), std::strtof(argv[5], nullptr));
    for (long i = 0; i < n; ++i) emit(dist(gen));
    return 0;
  }
  if (argc >= 3 && std::string(argv[1]) == "rand") {
    const long n = std::strtol(argv[2], nullptr, 10);
    for (long i = 0; i < n; ++i) emit(static_cast<float>(rand()) / RAND_MAX);
    return 0;
  }
  std::fprintf(stderr, "usage: %s mt19937 seed count lo hi | rand count\n", argv[0]);
  return 2;
}
