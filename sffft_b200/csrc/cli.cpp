// sffft: calibration / benchmark CLI over the C ABI (include/sffft.h).
//
// Command-line contract of the reference program (sfFFT src/sffft.cu:423-515), kept so that its scripts and
// tests/precision_smoke.sh drive this binary unchanged:
//   sffft [B H [L]] [--max-error REL_L2] [--io fp32|bf16|any] [--seed N] [--input-scale S]
//         [--allocator device|managed|mapped|hybrid] [--kernel legacy|cached|auto] [--memory-info]
// exit codes 0 (ok), 1 (invalid arguments), 2 (a length had no candidate within --max-error); the "# ..."
// header lines and the RESULT / SELECT / NO_MATCH / MEMORY rows; the seeded calibration inputs; errors as the
// relative L2 against the cuFFT fp32 pipeline over every output (cuFFT itself against an fp64 direct
// convolution of three sampled sequences); timing as the mean of clamp(20000 / L, 10, 200) back-to-back calls
// after three warm-ups.  L may also be 16384 when requested; the all-lengths sweep stays 128..8192.
//
// Structure (this program's own): a declarative option table; an Arena that places every buffer by its
// role under the allocation mode and keeps the MEMORY row's accounts; a Calibration per length that owns the
// inputs, the cuFFT reference output and the candidate list and prints its rows.
#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <limits>
#include <string>
#include <vector>

#include "../../include/sffft.h"
#include "cli_rng.h"

namespace {

[[noreturn]] void die(const char* what, const char* detail) {
  std::printf("error: %s: %s\n", what, detail);
  std::exit(1);
}
void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(what, cudaGetErrorString(e));
}
void sffft_ok(int s, const char* what) {
  if (s != SFFFT_OK) die(what, sffft_status_string(s));
}

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t) { return std::chrono::duration<double, std::milli>(Clock::now() - t).count(); }

// ------------------------------------------------------------------------------------------------
// Options
// ------------------------------------------------------------------------------------------------
enum class Mode { Device, Managed, Mapped, Hybrid };
const char* mode_name(Mode m) {
  switch (m) {
    case Mode::Device: return "device";
    case Mode::Managed: return "managed";
    case Mode::Mapped: return "mapped";
    default: return "hybrid";
  }
}
const char* kernel_name(int k) { return k == 0 ? "legacy" : k == 1 ? "cached" : "auto"; }

struct Options {
  int B = 8, H = 768, L = 0;   // L = 0: every length 128..8192
  double max_error = -1, input_scale = 1;
  const char* io = "fp32";
  Mode mode = Mode::Device;
  int kernels = 0;             // 0 legacy, 1 cached, 2 both
  bool memory_info = false;
  unsigned long long seed = sffft_cli::Rng().s;
};

bool parse_double(const char* s, double* out) {
  char* end = nullptr;
  errno = 0;
  *out = std::strtod(s, &end);
  return !errno && end != s && !*end;
}

bool pick(const char* v, const std::vector<const char*>& names, int* idx) {
  for (size_t i = 0; i < names.size(); i++)
    if (!std::strcmp(v, names[i])) { *idx = (int)i; return true; }
  return false;
}

void usage() {
  std::printf(
      "Usage: sffft [B H [L]] [--max-error REL_L2] [--io fp32|bf16|any] [--seed N] [--input-scale SCALE]"
      " [--allocator device|managed|mapped|hybrid] [--kernel legacy|cached|auto] [--memory-info]\n"
      "B, H: batch and channels (default 8 and 768).  L: 0 runs every length 128..8192; otherwise a power of two\n"
      "from 128 to 16384.  Without --max-error every candidate is timed and its error reported; with it, the fastest\n"
      "fused candidate within the budget (relative L2 against the cuFFT fp32 pipeline) is selected per length and\n"
      "the program exits 2 when a length has none.  Invalid arguments exit 1.\n");
}

// Returns -1 to continue, or the exit code.
int parse(int argc, char** argv, Options& o) {
  struct Flag {
    const char* name;
    const char* complaint;                       // printed when the value is rejected
    std::function<bool(const char*)> apply;      // null: a switch without a value
  };
  const std::vector<Flag> flags = {
      {"--max-error", "--max-error needs a positive finite number",
       [&](const char* v) { return parse_double(v, &o.max_error) && std::isfinite(o.max_error) && o.max_error > 0; }},
      {"--input-scale", "--input-scale needs a positive finite number within fp32 range",
       [&](const char* v) {
         return parse_double(v, &o.input_scale) && std::isfinite(o.input_scale) && o.input_scale > 0 &&
                o.input_scale <= std::numeric_limits<float>::max();
       }},
      {"--io", "--io takes fp32, bf16 or any",
       [&](const char* v) {
         int i;
         if (!pick(v, {"fp32", "bf16", "any"}, &i)) return false;
         o.io = i == 0 ? "fp32" : i == 1 ? "bf16" : "any";
         return true;
       }},
      {"--seed", "--seed needs a nonzero unsigned integer",
       [&](const char* v) {
         char* end = nullptr;
         errno = 0;
         o.seed = std::strtoull(v, &end, 10);
         return !errno && end != v && !*end && v[0] != '-' && o.seed != 0;
       }},
      {"--allocator", "--allocator takes device, managed, mapped or hybrid",
       [&](const char* v) {
         int i;
         if (!pick(v, {"device", "managed", "mapped", "hybrid"}, &i)) return false;
         o.mode = (Mode)i;
         return true;
       }},
      {"--kernel", "--kernel takes legacy, cached or auto",
       [&](const char* v) { return pick(v, {"legacy", "cached", "auto"}, &o.kernels); }},
      {"--memory-info", nullptr, nullptr},
  };
  int positional = 0;
  for (int i = 1; i < argc; i++) {
    const char* a = argv[i];
    if (!std::strcmp(a, "--help") || !std::strcmp(a, "-h")) {
      usage();
      return 0;
    }
    const Flag* f = nullptr;
    for (const Flag& c : flags)
      if (!std::strcmp(a, c.name)) f = &c;
    if (f && !f->apply) {
      o.memory_info = true;
      continue;
    }
    if (f) {
      if (i + 1 == argc) {
        usage();
        return 1;
      }
      if (!f->apply(argv[++i])) {
        std::fprintf(stderr, "%s\n", f->complaint);
        return 1;
      }
      continue;
    }
    char* end = nullptr;
    errno = 0;
    const long v = std::strtol(a, &end, 10);
    if (errno || end == a || *end || v < 0 || v > INT_MAX || positional == 3) {
      std::fprintf(stderr, "Invalid argument: %s\n", a);
      usage();
      return 1;
    }
    int* slot[3] = {&o.B, &o.H, &o.L};
    *slot[positional++] = (int)v;
  }
  if (o.B < 1 || o.H < 1 || (long long)o.B * o.H > INT_MAX ||
      (o.L && (o.L < 128 || o.L > 16384 || (o.L & (o.L - 1))))) {
    std::fprintf(stderr, "B and H must be positive with B*H <= INT_MAX; L must be 0 or a power of two in 128..16384\n");
    return 1;
  }
  return -1;
}

// ------------------------------------------------------------------------------------------------
// Arena: buffers placed by role under the allocation mode, with the MEMORY row's accounts
// ------------------------------------------------------------------------------------------------
// Roles: the calibration input u, the outputs and the cuFFT reference are "host facing" (the host writes or
// reads them); the bf16 input copy, the filter and the spectrum are "device only".  The hybrid mode maps the
// host-facing ones and keeps the others in device memory; the other modes place every buffer the same way.
// Host access goes through the host view of a mapped / managed buffer (no copy) or through an explicit copy
// of a device buffer (counted: uploads, downloads, and the host shadow that a copied-in input keeps).
class Arena {
 public:
  struct Accounts {
    size_t owned = 0, shadow = 0, uploaded = 0, downloaded = 0;
    double alloc_ms = 0, copy_ms = 0;
  };

  Arena(Mode m, bool prefetch_ok) : mode_(m), prefetch_ok_(prefetch_ok) {}
  Arena(const Arena&) = delete;
  ~Arena() {
    for (const Buf& b : bufs_) {
      if (b.placement == Mode::Mapped) cudaFreeHost(b.host);
      else cudaFree(b.dev);
    }
  }

  void* make(size_t bytes, bool host_facing) {
    const Mode where = mode_ == Mode::Hybrid ? (host_facing ? Mode::Mapped : Mode::Device) : mode_;
    const auto t0 = Clock::now();
    Buf b{nullptr, nullptr, bytes, where};
    if (where == Mode::Mapped) {
      cuda_ok(cudaHostAlloc(&b.host, bytes, cudaHostAllocMapped), "cudaHostAlloc");
      cuda_ok(cudaHostGetDevicePointer(&b.dev, b.host, 0), "cudaHostGetDevicePointer");
    } else if (where == Mode::Managed) {
      cuda_ok(cudaMallocManaged(&b.dev, bytes), "cudaMallocManaged");
      b.host = b.dev;
    } else {
      cuda_ok(cudaMalloc(&b.dev, bytes), "cudaMalloc");
    }
    acc_.alloc_ms += ms_since(t0);
    acc_.owned += bytes;
    bufs_.push_back(b);
    return b.dev;
  }

  // Host address of a buffer the host can touch directly, or null for device memory.
  void* host_of(const void* dev) const {
    for (const Buf& b : bufs_)
      if (b.dev == dev) return b.host;
    return nullptr;
  }

  // Places host data into a buffer: in place for host-visible buffers, else one counted copy.
  void fill(void* dev, const void* src, size_t bytes) {
    void* h = host_of(dev);
    if (h == src) return;
    const auto t0 = Clock::now();
    if (h) {
      std::memcpy(h, src, bytes);
    } else {
      cuda_ok(cudaMemcpy(dev, src, bytes, cudaMemcpyHostToDevice), "upload");
      acc_.uploaded += bytes;
    }
    acc_.copy_ms += ms_since(t0);
  }

  // Host-readable view of a device result: the buffer itself, or a counted copy into `scratch`.
  template <class T>
  const T* view(const T* dev, size_t n, std::vector<T>& scratch) {
    if (void* h = host_of(dev)) {
      migrate(dev, n * sizeof(T), false);
      cuda_ok(cudaDeviceSynchronize(), "synchronize");
      return static_cast<const T*>(h);
    }
    scratch.resize(n);
    const auto t0 = Clock::now();
    cuda_ok(cudaMemcpy(scratch.data(), dev, n * sizeof(T), cudaMemcpyDeviceToHost), "download");
    acc_.downloaded += n * sizeof(T);
    acc_.copy_ms += ms_since(t0);
    return scratch.data();
  }

  // Managed memory: move every buffer to the GPU before the timed calls.
  void to_device() {
    for (const Buf& b : bufs_) migrate(b.dev, b.bytes, true);
  }

  void note_shadow(size_t bytes) { acc_.shadow += bytes; }
  Mode mode() const { return mode_; }
  const Accounts& accounts() const { return acc_; }

 private:
  struct Buf {
    void *dev, *host;
    size_t bytes;
    Mode placement;
  };
  void migrate(const void* p, size_t bytes, bool to_gpu) {
    if (mode_ != Mode::Managed || !prefetch_ok_) return;
#if CUDART_VERSION >= 13000
    cudaMemLocation loc{};
    loc.type = to_gpu ? cudaMemLocationTypeDevice : cudaMemLocationTypeHost;
    loc.id = 0;
    cuda_ok(cudaMemPrefetchAsync(p, bytes, loc, 0), "prefetch");
#else
    cuda_ok(cudaMemPrefetchAsync(p, bytes, to_gpu ? 0 : cudaCpuDeviceId), "prefetch");
#endif
  }
  Mode mode_;
  bool prefetch_ok_;
  std::vector<Buf> bufs_;
  Accounts acc_;
};

// ------------------------------------------------------------------------------------------------
// Timing: three warm-up calls, then the mean of `iters` back-to-back calls between two events.
// ------------------------------------------------------------------------------------------------
class EventTimer {
 public:
  explicit EventTimer(int iters) : iters_(iters) {
    cuda_ok(cudaEventCreate(&a_), "event");
    cuda_ok(cudaEventCreate(&b_), "event");
  }
  ~EventTimer() {
    cudaEventDestroy(a_);
    cudaEventDestroy(b_);
  }
  double mean_ms(const std::function<void()>& call) {
    for (int i = 0; i < 3; i++) call();
    cuda_ok(cudaDeviceSynchronize(), "warm-up");
    cuda_ok(cudaEventRecord(a_), "event");
    for (int i = 0; i < iters_; i++) call();
    cuda_ok(cudaEventRecord(b_), "event");
    cuda_ok(cudaEventSynchronize(b_), "event");
    float ms = 0;
    cuda_ok(cudaEventElapsedTime(&ms, a_, b_), "event");
    cuda_ok(cudaGetLastError(), "timed calls");
    return ms / iters_;
  }

 private:
  int iters_;
  cudaEvent_t a_, b_;
};

uint16_t bf16_round(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0u;
  return (uint16_t)((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}
double bf16_value(uint16_t b) {
  const uint32_t x = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// ------------------------------------------------------------------------------------------------
// Calibration of one length
// ------------------------------------------------------------------------------------------------
struct Candidate {
  std::string method, io, config;
  double ms, rel_err;
};

class Calibration {
 public:
  Calibration(const Options& o, int L, bool prefetch_ok, sffft_cli::Rng& rng)
      : L_(L), B_(o.B), H_(o.H), n_((size_t)o.B * o.H * L), arena_(o.mode, prefetch_ok),
        timer_(std::min(200, std::max(10, 20000 / L))) {
    const auto t0 = Clock::now();
    u_ = static_cast<float*>(arena_.make(n_ * 4, true));
    y_ = static_cast<float*>(arena_.make(n_ * 4, true));
    yref_ = static_cast<float*>(arena_.make(n_ * 4, true));
    ub_ = static_cast<uint16_t*>(arena_.make(n_ * 2, false));
    yb_ = static_cast<uint16_t*>(arena_.make(n_ * 2, true));
    k_ = static_cast<float*>(arena_.make((size_t)H_ * L * 4, true));
    Kf_ = arena_.make((size_t)H_ * 2 * L * 8, false);
    // the generator writes u straight into a host-visible input, else into a host copy that stays alive
    float* hu = static_cast<float*>(arena_.host_of(u_));
    if (!hu) {
      hu_.resize(n_);
      hu = hu_.data();
    }
    hk_.resize((size_t)H_ * L);
    sffft_cli::generate(rng, (size_t)B_ * H_, H_, L, o.input_scale, hu, hk_.data());
    host_u_ = hu;
    std::vector<uint16_t> b16(n_);
    for (size_t i = 0; i < n_; i++) b16[i] = bf16_round(hu[i]);
    arena_.fill(u_, hu, n_ * 4);
    arena_.fill(k_, hk_.data(), hk_.size() * 4);
    arena_.fill(ub_, b16.data(), n_ * 2);
    arena_.to_device();
    sffft_ok(sffft_baseline_create(&cufft_, L, B_, H_, k_, 0), "cuFFT pipeline");
    cuda_ok(cudaDeviceSynchronize(), "set-up");
    setup_ms_ = ms_since(t0);
  }
  ~Calibration() {
    if (cufft_) sffft_baseline_destroy(cufft_);
  }

  // cuFFT pipeline rows; its output becomes the reference of every fused candidate.
  void cufft_rows() {
    const double full = timer_.mean_ms([&] { sffft_ok(sffft_baseline_run(cufft_, u_, yref_, 1, nullptr), "cuFFT"); });
    const double core = timer_.mean_ms([&] { sffft_ok(sffft_baseline_run(cufft_, u_, nullptr, 0, nullptr), "cuFFT"); });
    sffft_ok(sffft_baseline_run(cufft_, u_, yref_, 1, nullptr), "cuFFT");
    cuda_ok(cudaDeviceSynchronize(), "cuFFT");
    ref_ = arena_.view(yref_, n_, ref_copy_);
    // fp64 direct convolution of the first, middle and last sequence (channel = sequence % H)
    const size_t BH = (size_t)B_ * H_;
    double err = 0, norm = 0;
    for (size_t s : {(size_t)0, BH / 2, BH - 1}) {
      const float* us = host_u_ + s * L_;
      const float* ks = hk_.data() + (s % H_) * L_;
      for (int n = 0; n < L_; n++) {
        double v = 0;
        for (int m = 0; m <= n; m++) v += (double)us[m] * (double)ks[n - m];
        const double d = ref_[s * L_ + n] - v;
        err += d * d;
        norm += v * v;
      }
    }
    const double rel = sffft_relative_l2(err, norm);
    std::printf("RESULT,%d,cufft_pipeline_fp32,-,%.5f,%.3e\n", L_, full, rel);
    std::printf("RESULT,%d,cufft_core_fp32,-,%.5f,%.3e\n", L_, core, rel);
  }

  // Both I/O types of one catalog plan with one accumulation and one DFT-matrix mode.
  void fused_rows(const char* plan_name, int acc, int kmode) {
    struct Side {
      int io;
      const void* in;
      void* out;
      const char* method;
      const char* io_name;
    };
    const Side sides[2] = {
        {SFFFT_IO_FP32, u_, y_, acc == SFFFT_ACC_FP32 ? "fused_fp32io" : "fused_fp16acc_fp32io", "fp32"},
        {SFFFT_IO_BF16, ub_, yb_, acc == SFFFT_ACC_FP32 ? "fused_bf16io" : "fused_fp16acc_bf16io", "bf16"}};
    std::string config;
    double ms[2], err[2];
    for (int i = 0; i < 2; i++) {
      const Side& sd = sides[i];
      sffft_plan_t plan;
      sffft_ok(sffft_plan_create(&plan, L_, sd.io, acc, plan_name, kmode, 0), "plan");
      if (i == 0) {
        sffft_plan_info_t info;
        sffft_ok(sffft_plan_info(plan, &info), "plan info");
        const std::string radices = std::string(plan_name).substr(0, std::string(plan_name).find('/'));
        char buf[128];
        std::snprintf(buf, sizeof(buf), "%s/w%d/occ%d/smem%d/kernel_%s", radices.c_str(), info.warps, info.occupancy,
                      info.smem_bytes, kmode == SFFFT_KERNEL_CACHED ? "cached" : "legacy");
        config = buf;
        sffft_ok(sffft_filter_spectrum(plan, k_, SFFFT_IO_FP32, H_, Kf_, nullptr), "spectrum");
      }
      ms[i] = timer_.mean_ms([&] { sffft_ok(sffft_conv(plan, sd.in, Kf_, sd.out, B_, H_, nullptr), "conv"); });
      sffft_ok(sffft_conv(plan, sd.in, Kf_, sd.out, B_, H_, nullptr), "conv");
      sffft_ok(sffft_plan_check(plan), "device status");
      double e = 0, norm = 0;
      if (sd.io == SFFFT_IO_FP32) {
        std::vector<float> copy;
        const float* y = arena_.view(static_cast<const float*>(sd.out), n_, copy);
        for (size_t j = 0; j < n_; j++) {
          const double d = y[j] - ref_[j];
          e += d * d;
          norm += (double)ref_[j] * ref_[j];
        }
      } else {
        std::vector<uint16_t> copy;
        const uint16_t* y = arena_.view(static_cast<const uint16_t*>(sd.out), n_, copy);
        for (size_t j = 0; j < n_; j++) {
          const double d = bf16_value(y[j]) - ref_[j];
          e += d * d;
          norm += (double)ref_[j] * ref_[j];
        }
      }
      err[i] = sffft_relative_l2(e, norm);
      sffft_plan_destroy(plan);
    }
    for (int i = 0; i < 2; i++) {
      cands_.push_back({sides[i].method, sides[i].io_name, config, ms[i], err[i]});
      std::printf("RESULT,%d,%s,%s,%.5f,%.3e\n", L_, sides[i].method, config.c_str(), ms[i], err[i]);
    }
    std::fflush(stdout);
  }

  // Every catalog plan of this length, in the DFT-matrix modes asked for, both accumulations.
  void all_candidates(int kernels) {
    const int modes[2] = {SFFFT_KERNEL_LEGACY, SFFFT_KERNEL_CACHED};
    char name[96];
    for (int i = 0; i < sffft_catalog_count(); i++) {
      int len = 0;
      sffft_ok(sffft_catalog_entry(i, &len, name, sizeof(name)), "catalog");
      if (len != L_) continue;
      for (int km : modes) {
        if ((kernels == 0 && km != SFFFT_KERNEL_LEGACY) || (kernels == 1 && km != SFFFT_KERNEL_CACHED)) continue;
        fused_rows(name, SFFFT_ACC_FP32, km);
        fused_rows(name, SFFFT_ACC_FP16, km);
      }
    }
  }

  // SELECT or NO_MATCH row; false when nothing met the budget.
  bool select_row(double max_error, const char* io) const {
    std::vector<sffft_candidate_t> c;
    for (const Candidate& x : cands_) c.push_back({x.method.c_str(), x.io.c_str(), x.config.c_str(), x.ms, x.rel_err});
    const int pick = sffft_select_candidate(c.data(), (int)c.size(), max_error, io);
    if (pick < 0) {
      std::printf("NO_MATCH,%d,%s,%.9e\n", L_, io, max_error);
      return false;
    }
    const Candidate& w = cands_[pick];
    std::printf("SELECT,%d,%s,%s,%.5f,%.9e,%.9e,%s\n", L_, w.method.c_str(), w.config.c_str(), w.ms, w.rel_err,
                max_error, w.io.c_str());
    return true;
  }

  void memory_row() {
    const Arena::Accounts& a = arena_.accounts();
    const size_t shadows = (hu_.size() + ref_copy_.size()) * sizeof(float);
    std::printf("MEMORY,%d,%s,%zu,%zu,%.3f,%zu,%zu,%.3f,%.3f\n", L_, mode_name(arena_.mode()), a.owned, shadows,
                a.alloc_ms, a.uploaded, a.downloaded, a.copy_ms, setup_ms_);
  }

 private:
  int L_, B_, H_;
  size_t n_;
  Arena arena_;
  EventTimer timer_;
  float *u_, *y_, *yref_, *k_;
  uint16_t *ub_, *yb_;
  void* Kf_;
  const float* host_u_ = nullptr;
  const float* ref_ = nullptr;
  std::vector<float> hu_, hk_, ref_copy_;
  sffft_baseline_t cufft_ = nullptr;
  std::vector<Candidate> cands_;
  double setup_ms_ = 0;
};

}  // namespace

int main(int argc, char** argv) {
  Options o;
  const int rc = parse(argc, argv, o);
  if (rc >= 0) return rc;

  if (o.mode == Mode::Mapped || o.mode == Mode::Hybrid) cuda_ok(cudaSetDeviceFlags(cudaDeviceMapHost), "device flags");
  cudaDeviceProp p;
  cuda_ok(cudaGetDeviceProperties(&p, 0), "device properties");
  auto attr = [](cudaDeviceAttr a) {
    int v = 0;
    cuda_ok(cudaDeviceGetAttribute(&v, a, 0), "device attribute");
    return v;
  };
  const int managed = attr(cudaDevAttrManagedMemory), concurrent = attr(cudaDevAttrConcurrentManagedAccess);
  const int pageable = attr(cudaDevAttrPageableMemoryAccess);
  const int host_tables = attr(cudaDevAttrPageableMemoryAccessUsesHostPageTables);
  std::printf("# MEMORY_CAPS,mapped=%d,managed=%d,concurrent_managed=%d,pageable=%d,host_page_tables=%d,integrated=%d\n",
              p.canMapHostMemory, managed, concurrent, pageable, host_tables, p.integrated);
  if (o.memory_info) return 0;
  const bool needs_map = o.mode == Mode::Mapped || o.mode == Mode::Hybrid;
  if ((needs_map && !p.canMapHostMemory) || (o.mode == Mode::Managed && !managed)) {
    std::fprintf(stderr, "Requested allocator is unsupported on this device\n");
    return 1;
  }
  std::printf("# %s sm_%d%d %d SMs, smem/block %zu, L2 %d MB, B=%d H=%d\n", p.name, p.major, p.minor,
              p.multiProcessorCount, p.sharedMemPerBlockOptin, p.l2CacheSize >> 20, o.B, o.H);
  std::printf("# calibration seed=%llu, input_scale=%.9e, max_error=%.9e, io=%s,allocator=%s,kernel=%s\n", o.seed,
              o.input_scale, o.max_error, o.io, mode_name(o.mode), kernel_name(o.kernels));
  std::printf("# RESULT,L,method,config,ms,rel_err\n");
  std::printf("# MEMORY,L,allocator,owned_bytes,persistent_host_shadow_bytes,allocation_ms,upload_bytes,download_bytes,"
              "copy_ms,setup_ms\n");
  if (o.max_error > 0) std::printf("# SELECT,L,method,config,ms,rel_err,max_error,io\n");

  // one generator stream across the lengths, as the reference draws them
  sffft_cli::Rng rng;
  rng.s = o.seed;
  int misses = 0;
  for (int L = 128; L <= 16384; L *= 2) {
    if (o.L ? o.L != L : L > 8192) continue;
    Calibration cal(o, L, concurrent != 0, rng);
    cal.cufft_rows();
    cal.all_candidates(o.kernels);
    if (o.max_error > 0 && !cal.select_row(o.max_error, o.io)) misses++;
    cal.memory_row();
  }
  return misses ? 2 : 0;
}
