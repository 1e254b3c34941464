// Builds the reference program from its own source, in place (oracle/Makefile passes -I to
// the reference tree; nothing is copied).  TEST INFRASTRUCTURE ONLY.
//   ref_harness rng SEED COUNT       first COUNT draws of the reference's nrand() (src/sffft.cu:308-310)
//   ref_harness run [sffft args...]  the unmodified reference benchmark main (src/sffft.cu:430-515)
#define main sffft_reference_main
#include "sffft.cu"
#undef main
#include <cstdlib>
#include <cstring>

int main(int argc, char** argv) {
  if (argc >= 4 && !std::strcmp(argv[1], "rng")) {
    unsigned long long seed = std::strtoull(argv[2], nullptr, 10);
    if (seed) rng = seed;
    const int n = std::atoi(argv[3]);
    for (int i = 0; i < n; i++) std::printf("%.17g\n", nrand());
    return 0;
  }
  if (argc >= 2 && !std::strcmp(argv[1], "run")) {
    argv[1] = argv[0];
    return sffft_reference_main(argc - 1, argv + 1);
  }
  std::fprintf(stderr, "usage: ref_harness rng SEED COUNT | run [sffft args]\n");
  return 1;
}
