// sffft: calibration / benchmark CLI over the C ABI (include/sffft.h).
//
// Drop-in for the reference program's command line and output (sfFFT src/sffft.cu:423-515):
//   sffft [B H [L]] [--max-error REL_L2] [--io fp32|bf16|any] [--seed N] [--input-scale S]
//         [--allocator device|managed|mapped|hybrid] [--kernel legacy|cached|auto] [--memory-info]
// Same argument rules and exit codes (0 ok, 1 invalid arguments, 2 no candidate met --max-error), the
// same "# ..." header lines and RESULT / SELECT / NO_MATCH / MEMORY rows, the same calibration inputs
// (seeded generator) and error definition (relative L2 against the cuFFT fp32 pipeline over every output
// element; cuFFT itself against an fp64 direct convolution of three sampled sequences).  L may also be
// 16384 when requested explicitly; the all-lengths sweep stays 128..8192.
#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "../../include/sffft.h"
#include "cli_rng.h"

namespace {

#define CK(x)                                                                                       \
  do {                                                                                              \
    cudaError_t e_ = (x);                                                                           \
    if (e_ != cudaSuccess) {                                                                        \
      std::printf("CUDA error %s at %s:%d: %s\n", #x, __FILE__, __LINE__, cudaGetErrorString(e_)); \
      std::exit(1);                                                                                 \
    }                                                                                               \
  } while (0)
#define SK(x)                                                                                            \
  do {                                                                                                   \
    int s_ = (x);                                                                                        \
    if (s_ != SFFFT_OK) {                                                                                \
      std::printf("sffft error %s at %s:%d: %s\n", #x, __FILE__, __LINE__, sffft_status_string(s_));     \
      std::exit(1);                                                                                      \
    }                                                                                                    \
  } while (0)

enum class Alloc { Device, Managed, Mapped, Hybrid };
const char* alloc_name(Alloc a) {
  return a == Alloc::Device ? "device" : a == Alloc::Managed ? "managed" : a == Alloc::Mapped ? "mapped" : "hybrid";
}
using Clock = std::chrono::steady_clock;
double since_ms(Clock::time_point t) { return std::chrono::duration<double, std::milli>(Clock::now() - t).count(); }

// Owned buffers under one of the four allocation modes; counts bytes, copies and time for MEMORY rows.
struct Buffers {
  struct Block { void* dev; void* host; size_t bytes; Alloc kind; };
  Alloc mode;
  bool can_prefetch;
  std::vector<Block> blocks;
  size_t owned = 0, uploaded = 0, downloaded = 0;
  double alloc_ms = 0, copy_ms = 0;
  Buffers(Alloc m, bool pf) : mode(m), can_prefetch(pf) {}
  Buffers(const Buffers&) = delete;
  template <class T>
  T* get(size_t bytes, bool host_visible_io = true) {
    const Alloc kind = mode == Alloc::Hybrid ? (host_visible_io ? Alloc::Mapped : Alloc::Device) : mode;
    const auto t0 = Clock::now();
    void *dev = nullptr, *host = nullptr;
    if (kind == Alloc::Mapped) {
      CK(cudaHostAlloc(&host, bytes, cudaHostAllocMapped));
      CK(cudaHostGetDevicePointer(&dev, host, 0));
    } else if (kind == Alloc::Managed) {
      CK(cudaMallocManaged(&dev, bytes));
      host = dev;
    } else {
      CK(cudaMalloc(&dev, bytes));
    }
    blocks.push_back({dev, host, bytes, kind});
    owned += bytes;
    alloc_ms += since_ms(t0);
    return static_cast<T*>(dev);
  }
  template <class T>
  T* host_view(const T* dev) const {
    for (const auto& b : blocks)
      if (b.dev == dev) return static_cast<T*>(b.host);
    return nullptr;
  }
  void prefetch(const void* p, size_t bytes, bool to_gpu) {
    if (mode != Alloc::Managed || !can_prefetch) return;
#if CUDART_VERSION >= 13000
    cudaMemLocation loc{};
    loc.type = to_gpu ? cudaMemLocationTypeDevice : cudaMemLocationTypeHost;
    loc.id = 0;
    CK(cudaMemPrefetchAsync(p, bytes, loc, 0));
#else
    CK(cudaMemPrefetchAsync(p, bytes, to_gpu ? 0 : cudaCpuDeviceId));
#endif
  }
  void to_gpu() {
    for (const auto& b : blocks) prefetch(b.dev, b.bytes, true);
  }
  template <class T>
  void upload(T* dev, const T* src, size_t n) {
    T* h = host_view(dev);
    if (h == src) return;
    const auto t0 = Clock::now();
    if (h) std::memcpy(h, src, n * sizeof(T));
    else {
      CK(cudaMemcpy(dev, src, n * sizeof(T), cudaMemcpyHostToDevice));
      uploaded += n * sizeof(T);
    }
    copy_ms += since_ms(t0);
  }
  template <class T>
  const T* read(const T* dev, size_t n, std::vector<T>& shadow) {
    if (T* h = host_view(dev)) {
      prefetch(dev, n * sizeof(T), false);
      CK(cudaDeviceSynchronize());
      return h;
    }
    shadow.resize(n);
    const auto t0 = Clock::now();
    CK(cudaMemcpy(shadow.data(), dev, n * sizeof(T), cudaMemcpyDeviceToHost));
    downloaded += n * sizeof(T);
    copy_ms += since_ms(t0);
    return shadow.data();
  }
  ~Buffers() {
    for (const auto& b : blocks) {
      if (b.kind == Alloc::Mapped) cudaFreeHost(b.host);
      else cudaFree(b.dev);
    }
  }
};

uint16_t to_bf16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  x += 0x7FFFu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}
float from_bf16_bits(uint16_t b) {
  const uint32_t x = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

struct Cand {
  std::string method, io, config;
  double ms, rel_err;
};

struct Run {
  int L, N, B, H, iters;
  size_t BH;
  int kernel_mode;   // 0 legacy, 1 cached, 2 both
  Buffers mem;
  std::vector<float> hu_shadow, hk, yref_shadow;
  float* hu = nullptr;
  const float* yref = nullptr;
  float *du, *dy, *dyref, *dk;
  uint16_t *dub, *dyb;
  float* dKf;
  sffft_baseline_t bl = nullptr;
  cudaEvent_t e0, e1;
  double setup_ms = 0;
  std::vector<Cand> cands;

  template <class F>
  float timeit(F f) {
    for (int i = 0; i < 3; i++) f();
    CK(cudaDeviceSynchronize());
    CK(cudaEventRecord(e0));
    for (int i = 0; i < iters; i++) f();
    CK(cudaEventRecord(e1));
    CK(cudaEventSynchronize(e1));
    float ms;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    CK(cudaGetLastError());
    return ms / iters;
  }

  Run(int L_, int B_, int H_, double scale, Alloc mode, bool can_prefetch, int kmode, sffft_cli::Rng& rng)
      : L(L_), N(2 * L_), B(B_), H(H_), BH((size_t)B_ * H_), kernel_mode(kmode), mem(mode, can_prefetch) {
    const auto t0 = Clock::now();
    iters = std::min(200, std::max(10, 20000 / L));
    du = mem.get<float>(BH * L * 4);
    dy = mem.get<float>(BH * L * 4);
    dyref = mem.get<float>(BH * L * 4);
    dub = mem.get<uint16_t>(BH * L * 2, false);
    dyb = mem.get<uint16_t>(BH * L * 2);
    dk = mem.get<float>((size_t)H * L * 4);
    dKf = mem.get<float>((size_t)H * N * 8, false);
    hu = mem.host_view(du);
    if (!hu) {
      hu_shadow.resize(BH * L);
      hu = hu_shadow.data();
    }
    hk.resize((size_t)H * L);
    sffft_cli::generate(rng, BH, H, L, scale, hu, hk.data());
    std::vector<uint16_t> ub(BH * L);
    for (size_t i = 0; i < ub.size(); i++) ub[i] = to_bf16_bits(hu[i]);
    mem.upload(du, hu, BH * L);
    mem.upload(dk, hk.data(), (size_t)H * L);
    mem.upload(dub, ub.data(), BH * L);
    mem.to_gpu();
    SK(sffft_baseline_create(&bl, L, B, H, dk, 0));
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaDeviceSynchronize());
    setup_ms = since_ms(t0);
  }
  ~Run() {
    if (bl) sffft_baseline_destroy(bl);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }

  void baseline() {
    const float t_full = timeit([&] { SK(sffft_baseline_run(bl, du, dyref, 1, nullptr)); });
    const float t_core = timeit([&] { SK(sffft_baseline_run(bl, du, nullptr, 0, nullptr)); });
    SK(sffft_baseline_run(bl, du, dyref, 1, nullptr));
    CK(cudaDeviceSynchronize());
    yref = mem.read(dyref, BH * L, yref_shadow);
    double num = 0, den = 0;
    for (size_t s : {(size_t)0, BH / 2, BH - 1}) {
      const int h = (int)(s % H);
      for (int n = 0; n < L; n++) {
        double acc = 0;
        for (int m = 0; m <= n; m++) acc += (double)hu[s * L + m] * (double)hk[(size_t)h * L + n - m];
        const double d = yref[s * L + n] - acc;
        num += d * d;
        den += acc * acc;
      }
    }
    const double err = sffft_relative_l2(num, den);
    std::printf("RESULT,%d,cufft_pipeline_fp32,-,%.5f,%.3e\n", L, t_full, err);
    std::printf("RESULT,%d,cufft_core_fp32,-,%.5f,%.3e\n", L, t_core, err);
  }

  void fused(const char* name, int acc, int kmode) {
    sffft_plan_t p32, p16;
    SK(sffft_plan_create(&p32, L, SFFFT_IO_FP32, acc, name, kmode, 0));
    SK(sffft_plan_create(&p16, L, SFFFT_IO_BF16, acc, name, kmode, 0));
    sffft_plan_info_t info;
    SK(sffft_plan_info(p32, &info));
    SK(sffft_filter_spectrum(p32, dk, SFFFT_IO_FP32, H, dKf, nullptr));
    const float t32 = timeit([&] { SK(sffft_conv(p32, du, dKf, dy, B, H, nullptr)); });
    const float t16 = timeit([&] { SK(sffft_conv(p16, dub, dKf, dyb, B, H, nullptr)); });
    SK(sffft_conv(p32, du, dKf, dy, B, H, nullptr));
    SK(sffft_plan_check(p32));
    std::vector<float> ysh;
    const float* y = mem.read(dy, BH * L, ysh);
    SK(sffft_conv(p16, dub, dKf, dyb, B, H, nullptr));
    SK(sffft_plan_check(p16));
    std::vector<uint16_t> ybsh;
    const uint16_t* yb = mem.read(dyb, BH * L, ybsh);
    double n1 = 0, n2 = 0, d = 0;
    for (size_t i = 0; i < BH * L; i++) {
      const double r = yref[i], a = y[i] - r, b = (double)from_bf16_bits(yb[i]) - r;
      n1 += a * a;
      n2 += b * b;
      d += r * r;
    }
    std::string plan = name;
    plan = plan.substr(0, plan.find('/'));
    char config[128];
    std::snprintf(config, sizeof(config), "%s/w%d/occ%d/smem%d/kernel_%s", plan.c_str(), info.warps, info.occupancy,
                  info.smem_bytes, kmode == SFFFT_KERNEL_CACHED ? "cached" : "legacy");
    const char* m32 = acc == SFFFT_ACC_FP32 ? "fused_fp32io" : "fused_fp16acc_fp32io";
    const char* m16 = acc == SFFFT_ACC_FP32 ? "fused_bf16io" : "fused_fp16acc_bf16io";
    const double e32 = sffft_relative_l2(n1, d), e16 = sffft_relative_l2(n2, d);
    cands.push_back({m32, "fp32", config, t32, e32});
    cands.push_back({m16, "bf16", config, t16, e16});
    std::printf("RESULT,%d,%s,%s,%.5f,%.3e\n", L, m32, config, t32, e32);
    std::printf("RESULT,%d,%s,%s,%.5f,%.3e\n", L, m16, config, t16, e16);
    std::fflush(stdout);
    sffft_plan_destroy(p32);
    sffft_plan_destroy(p16);
  }

  void variants(const char* name) {
    if (kernel_mode != 1) {
      fused(name, SFFFT_ACC_FP32, SFFFT_KERNEL_LEGACY);
      fused(name, SFFFT_ACC_FP16, SFFFT_KERNEL_LEGACY);
    }
    if (kernel_mode != 0) {
      fused(name, SFFFT_ACC_FP32, SFFFT_KERNEL_CACHED);
      fused(name, SFFFT_ACC_FP16, SFFFT_KERNEL_CACHED);
    }
  }

  bool select(double max_error, const char* io) {
    std::vector<sffft_candidate_t> c;
    for (const auto& x : cands) c.push_back({x.method.c_str(), x.io.c_str(), x.config.c_str(), x.ms, x.rel_err});
    const int i = sffft_select_candidate(c.data(), (int)c.size(), max_error, io);
    if (i < 0) {
      std::printf("NO_MATCH,%d,%s,%.9e\n", L, io, max_error);
      return false;
    }
    const Cand& b = cands[i];
    std::printf("SELECT,%d,%s,%s,%.5f,%.9e,%.9e,%s\n", L, b.method.c_str(), b.config.c_str(), b.ms, b.rel_err, max_error,
                b.io.c_str());
    return true;
  }

  void report_memory() {
    std::printf("MEMORY,%d,%s,%zu,%zu,%.3f,%zu,%zu,%.3f,%.3f\n", L, alloc_name(mem.mode), mem.owned,
                (hu_shadow.size() + yref_shadow.size()) * sizeof(float), mem.alloc_ms, mem.uploaded, mem.downloaded,
                mem.copy_ms, setup_ms);
  }
};

void usage() {
  std::printf(
      "Usage: sffft [B H [L]] [--max-error REL_L2] [--io fp32|bf16|any] [--seed N] [--input-scale SCALE]"
      " [--allocator device|managed|mapped|hybrid] [--kernel legacy|cached|auto] [--memory-info]\n"
      "B, H: batch and channels (default 8 and 768).  L: 0 runs every length 128..8192; otherwise a power of two\n"
      "from 128 to 16384.  Without --max-error every candidate is timed and its error reported; with it, the fastest\n"
      "fused candidate within the budget (relative L2 against the cuFFT fp32 pipeline) is selected per length and\n"
      "the program exits 2 when a length has none.  Invalid arguments exit 1.\n");
}

}  // namespace

int main(int argc, char** argv) {
  int B = 8, H = 768, only = 0, positional = 0, failed = 0, kernel_mode = 0;
  double max_error = -1, input_scale = 1;
  const char* io = "fp32";
  Alloc alloc = Alloc::Device;
  bool memory_info = false;
  sffft_cli::Rng rng;
  for (int i = 1; i < argc; i++) {
    const char* a = argv[i];
    char* end = nullptr;
    errno = 0;
    if (!std::strcmp(a, "--help") || !std::strcmp(a, "-h")) {
      usage();
      return 0;
    }
    if (!std::strcmp(a, "--memory-info")) {
      memory_info = true;
      continue;
    }
    if (!std::strcmp(a, "--allocator")) {
      if (++i == argc) { usage(); return 1; }
      const char* v = argv[i];
      if (!std::strcmp(v, "device")) alloc = Alloc::Device;
      else if (!std::strcmp(v, "managed")) alloc = Alloc::Managed;
      else if (!std::strcmp(v, "mapped")) alloc = Alloc::Mapped;
      else if (!std::strcmp(v, "hybrid")) alloc = Alloc::Hybrid;
      else { std::fprintf(stderr, "--allocator takes device, managed, mapped or hybrid\n"); return 1; }
    } else if (!std::strcmp(a, "--kernel")) {
      if (++i == argc) { usage(); return 1; }
      const char* v = argv[i];
      if (!std::strcmp(v, "legacy")) kernel_mode = 0;
      else if (!std::strcmp(v, "cached")) kernel_mode = 1;
      else if (!std::strcmp(v, "auto")) kernel_mode = 2;
      else { std::fprintf(stderr, "--kernel takes legacy, cached or auto\n"); return 1; }
    } else if (!std::strcmp(a, "--max-error")) {
      if (++i == argc) { usage(); return 1; }
      max_error = std::strtod(argv[i], &end);
      if (errno || end == argv[i] || *end || !std::isfinite(max_error) || max_error <= 0) {
        std::fprintf(stderr, "--max-error needs a positive finite number\n");
        return 1;
      }
    } else if (!std::strcmp(a, "--input-scale")) {
      if (++i == argc) { usage(); return 1; }
      input_scale = std::strtod(argv[i], &end);
      if (errno || end == argv[i] || *end || !std::isfinite(input_scale) || input_scale <= 0 ||
          input_scale > std::numeric_limits<float>::max()) {
        std::fprintf(stderr, "--input-scale needs a positive finite number within fp32 range\n");
        return 1;
      }
    } else if (!std::strcmp(a, "--io")) {
      if (++i == argc) { usage(); return 1; }
      io = argv[i];
      if (std::strcmp(io, "fp32") && std::strcmp(io, "bf16") && std::strcmp(io, "any")) {
        std::fprintf(stderr, "--io takes fp32, bf16 or any\n");
        return 1;
      }
    } else if (!std::strcmp(a, "--seed")) {
      if (++i == argc) { usage(); return 1; }
      rng.s = std::strtoull(argv[i], &end, 10);
      if (errno || end == argv[i] || *end || argv[i][0] == '-' || !rng.s) {
        std::fprintf(stderr, "--seed needs a nonzero unsigned integer\n");
        return 1;
      }
    } else {
      const long v = std::strtol(a, &end, 10);
      if (errno || end == a || *end || v < 0 || v > INT_MAX || positional == 3) {
        std::fprintf(stderr, "Invalid argument: %s\n", a);
        usage();
        return 1;
      }
      if (positional == 0) B = (int)v;
      else if (positional == 1) H = (int)v;
      else only = (int)v;
      positional++;
    }
  }
  if (B < 1 || H < 1 || (long long)B * H > INT_MAX ||
      (only && (only < 128 || only > 16384 || (only & (only - 1))))) {
    std::fprintf(stderr, "B and H must be positive with B*H <= INT_MAX; L must be 0 or a power of two in 128..16384\n");
    return 1;
  }
  if (alloc == Alloc::Mapped || alloc == Alloc::Hybrid) CK(cudaSetDeviceFlags(cudaDeviceMapHost));
  cudaDeviceProp p;
  CK(cudaGetDeviceProperties(&p, 0));
  int managed = 0, concurrent = 0, pageable = 0, host_tables = 0;
  CK(cudaDeviceGetAttribute(&managed, cudaDevAttrManagedMemory, 0));
  CK(cudaDeviceGetAttribute(&concurrent, cudaDevAttrConcurrentManagedAccess, 0));
  CK(cudaDeviceGetAttribute(&pageable, cudaDevAttrPageableMemoryAccess, 0));
  CK(cudaDeviceGetAttribute(&host_tables, cudaDevAttrPageableMemoryAccessUsesHostPageTables, 0));
  std::printf("# MEMORY_CAPS,mapped=%d,managed=%d,concurrent_managed=%d,pageable=%d,host_page_tables=%d,integrated=%d\n",
              p.canMapHostMemory, managed, concurrent, pageable, host_tables, p.integrated);
  if (memory_info) return 0;
  if (((alloc == Alloc::Mapped || alloc == Alloc::Hybrid) && !p.canMapHostMemory) || (alloc == Alloc::Managed && !managed)) {
    std::fprintf(stderr, "Requested allocator is unsupported on this device\n");
    return 1;
  }
  std::printf("# %s sm_%d%d %d SMs, smem/block %zu, L2 %d MB, B=%d H=%d\n", p.name, p.major, p.minor,
              p.multiProcessorCount, p.sharedMemPerBlockOptin, p.l2CacheSize >> 20, B, H);
  std::printf("# calibration seed=%llu, input_scale=%.9e, max_error=%.9e, io=%s,allocator=%s,kernel=%s\n", rng.s,
              input_scale, max_error, io, alloc_name(alloc),
              kernel_mode == 0 ? "legacy" : kernel_mode == 1 ? "cached" : "auto");
  std::printf("# RESULT,L,method,config,ms,rel_err\n");
  std::printf("# MEMORY,L,allocator,owned_bytes,persistent_host_shadow_bytes,allocation_ms,upload_bytes,download_bytes,copy_ms,setup_ms\n");
  if (max_error > 0) std::printf("# SELECT,L,method,config,ms,rel_err,max_error,io\n");

  const int ncat = sffft_catalog_count();
  for (int L = 128; L <= 16384; L *= 2) {
    if (only ? only != L : L > 8192) continue;
    Run run(L, B, H, input_scale, alloc, concurrent != 0, kernel_mode, rng);
    run.baseline();
    char name[96];
    for (int i = 0; i < ncat; i++) {
      int cl = 0;
      SK(sffft_catalog_entry(i, &cl, name, sizeof(name)));
      if (cl == L) run.variants(name);
    }
    if (max_error > 0 && !run.select(max_error, io)) failed++;
    run.report_memory();
  }
  return failed ? 2 : 0;
}
