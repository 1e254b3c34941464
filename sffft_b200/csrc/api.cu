// C ABI of the library (declared in include/sffft.h).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <limits>
#include <string>
#include <vector>

#include "../../include/sffft.h"
#include "calibration.h"
#include "fused_conv.cuh"
#include "registry.h"
#include "spectrum.h"

namespace sffft {
cudaError_t launch_rfft(const void* x, bool x_bf16, int rows, float2* X, float2* W, const int* R, int S, int sms,
                        cudaStream_t stream);
cudaError_t launch_irfft(const float2* X, int rows, float* x, float2* W, const int* R, int S, int sms,
                         cudaStream_t stream);
struct Baseline;
int baseline_create(Baseline** out, int L, int B, int H, const float* k_dev, int device);
int baseline_run(Baseline* b, const float* u, float* y, int full, cudaStream_t st);
void baseline_destroy(Baseline* b);
int umma_probe(int a_kind, int a_slice, int b_pitch, int b_slice, int n, int acc16, const uint16_t* A_host,
               const uint16_t* B_host, uint32_t* D_host);
int wait_timeout_probe(int limit_us);
}  // namespace sffft

using namespace sffft;

struct sffft_plan {
  const ConvEntry* e;    // the fused kernel's plan (the block plan of a composite plan)
  int blocks, L;         // composite plans: L = blocks * e->L (blocks = 1: the plan itself)
  int kio;               // I/O type of the fused kernel launches
  const BlockEntry* be;  // composite plans: the partitioned-convolution kernels of the block plan
  void* work;            // composite plans: workspace attached by sffft_plan_set_workspace (caller-owned)
  size_t work_bytes;
  int io, acc, kernel_mode, device, occupancy, smem_launch, sms;
  int smem_small[2];     // launch shared memory of the 1- and 2-slot variants (0: not compiled for this plan)
  uint4* btab;   // cached DFT-matrix image (device), null in legacy mode
  int* status;   // device status word
};
struct sffft_baseline {
  Baseline* b;
};

static thread_local int g_last_cuda = 0;
#ifdef SFFFT_TRACE
static unsigned long long* g_trace = nullptr;
extern "C" void sffft_debug_set_trace(void* buf) { g_trace = (unsigned long long*)buf; }
#endif
static int cuda_fail(cudaError_t e) {
  g_last_cuda = (int)e;
  return SFFFT_ERR_CUDA;
}

static const BlockEntry* block_entry(const char* name) {
  static const std::vector<const BlockEntry*> all = [] {
    std::vector<const BlockEntry*> v;
    const BlockEntry* p;
    int n = block_entries_2stage(&p);
    for (int i = 0; i < n; i++) v.push_back(p + i);
    n = block_entries_3stage(&p);
    for (int i = 0; i < n; i++) v.push_back(p + i);
    return v;
  }();
  for (const BlockEntry* b : all)
    if (std::strcmp(b->name, name) == 0) return b;
  return nullptr;
}

static const std::vector<const ConvEntry*>& catalog() {
  static std::vector<const ConvEntry*> all = [] {
    std::vector<const ConvEntry*> v;
    const ConvEntry* p;
    int n = entries_small(&p);
    for (int i = 0; i < n; i++) v.push_back(p + i);
    n = entries_mid(&p);
    for (int i = 0; i < n; i++) v.push_back(p + i);
    n = entries_large(&p);
    for (int i = 0; i < n; i++) v.push_back(p + i);
    return v;
  }();
  return all;
}

// Built-in B200 default per length: the calibrated plan of calibration.h (measured on one B200 by
// `python -m sffft_b200.calibrate`, chosen by make_calibration.py); the CLI's empirical selector can override it
// from its own measurements.
// Composite plans: lengths above the largest single-kernel plan run as partitioned convolutions of up to
// kMaxBlocks blocks (a forward transform per input block, a spectrum sum and an inverse transform per output
// block; the sums read blocks * (blocks + 1) / 2 block spectra).
constexpr int kMaxBlockL = 16384, kMaxBlocks = 16;

static const char* default_for(int L) {
  for (const CalibratedPlan& c : kCalibratedPlans)
    if (c.L == L) return c.name;
  return nullptr;
}

static int copy_name(const char* s, char* out, int cap) {
  if (!out || cap <= 0) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((int)std::strlen(s) >= cap) return SFFFT_ERR_INVALID_ARGUMENT;
  std::strcpy(out, s);
  return SFFFT_OK;
}

extern "C" {

const char* sffft_status_string(int s) {
  switch (s) {
    case SFFFT_OK: return "ok";
    case SFFFT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SFFFT_ERR_UNSUPPORTED: return "unsupported length, plan or data type";
    case SFFFT_ERR_CUDA: return "CUDA runtime error";
    case SFFFT_ERR_DEVICE: return "device is not an sm_100 GPU with enough shared memory for the plan";
    case SFFFT_ERR_TIMEOUT: return "device barrier wait timed out";
    case SFFFT_ERR_NO_MATCH: return "no candidate meets the error budget";
    case SFFFT_ERR_ALLOC: return "device allocation failed";
    case SFFFT_ERR_SCRATCH_LIMIT: return "problem exceeds the fixed scratch of the allocation-free entry point";
    case SFFFT_ERR_WORKSPACE: return "composite plan needs a workspace of sffft_conv_workspace_bytes";
    default: return "unknown status";
  }
}

int sffft_last_cuda_error(void) { return g_last_cuda; }

int sffft_catalog_count(void) { return (int)catalog().size(); }

int sffft_catalog_entry(int index, int* L, char* name, int cap) {
  if (index < 0 || index >= (int)catalog().size()) return SFFFT_ERR_INVALID_ARGUMENT;
  if (L) *L = catalog()[index]->L;
  return name ? copy_name(catalog()[index]->name, name, cap) : SFFFT_OK;
}

int sffft_default_config(int L, char* name, int cap) {
  const char* d = default_for(L);
  if (!d) return SFFFT_ERR_UNSUPPORTED;
  return copy_name(d, name, cap);
}

int sffft_plan_create(sffft_plan_t* out, int L, int io, int acc, const char* config, int kernel_mode, int device) {
  if (!out) return SFFFT_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if ((io != SFFFT_IO_FP32 && io != SFFFT_IO_BF16) || (acc != SFFFT_ACC_FP32 && acc != SFFFT_ACC_FP16) ||
      (kernel_mode != SFFFT_KERNEL_LEGACY && kernel_mode != SFFFT_KERNEL_CACHED) || device < 0)
    return SFFFT_ERR_INVALID_ARGUMENT;
  // A composite plan "<P>x[<block plan>]" runs lengths L = P * Lb as partitioned convolutions on the block plan;
  // lengths above the largest catalog plan get one by default.
  int blocks = 1;
  std::string want;
  if (config && *config) {
    want = config;
    const size_t lb = want.find("x["), n = want.size();
    if (lb != std::string::npos && lb > 0 && n > lb + 3 && want[n - 1] == ']' &&
        want.find_first_not_of("0123456789") == lb) {
      blocks = std::atoi(want.substr(0, lb).c_str());
      want = want.substr(lb + 2, n - lb - 3);
      if (blocks < 2 || blocks > kMaxBlocks || (blocks & (blocks - 1))) return SFFFT_ERR_UNSUPPORTED;
    }
  } else if (default_for(L)) {
    want = default_for(L);
  } else if (L > kMaxBlockL && L % kMaxBlockL == 0) {
    blocks = L / kMaxBlockL;
    want = default_for(kMaxBlockL);
    if (blocks > kMaxBlocks || (blocks & (blocks - 1))) return SFFFT_ERR_UNSUPPORTED;
  } else {
    return SFFFT_ERR_UNSUPPORTED;
  }
  const ConvEntry* e = nullptr;
  for (const ConvEntry* c : catalog())
    if (want == c->name) e = c;
  if (!e || (long long)e->L * blocks != L) return SFFFT_ERR_UNSUPPORTED;
  const BlockEntry* be = blocks > 1 ? block_entry(e->name) : nullptr;
  if (blocks > 1 && !be) return SFFFT_ERR_UNSUPPORTED;   // block plan without partitioned-convolution kernels

  int ndev = 0;
  cudaError_t ce = cudaGetDeviceCount(&ndev);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (device >= ndev) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((ce = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(ce);
  cudaDeviceProp prop;
  if ((ce = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return cuda_fail(ce);
  const int kio = io;
  const int need = e->smem_bytes[kio];
  if (prop.major != 10 || prop.minor != 0 || (int)prop.sharedMemPerBlockOptin < need) return SFFFT_ERR_DEVICE;

  // The kernel is persistent with one CTA per SM (the grid never exceeds the SM count).  Requesting
  // more than half of an SM's shared memory keeps the block scheduler from placing two CTAs on one SM.
  int smem_launch = need;
  const int half = (int)prop.sharedMemPerMultiprocessor / 2 + 1024;
  if (smem_launch < half) smem_launch = half;
  if (smem_launch > (int)prop.sharedMemPerBlockOptin) smem_launch = (int)prop.sharedMemPerBlockOptin;
  const void* fn = e->func[kio][acc];
  if ((ce = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_launch)) != cudaSuccess)
    return cuda_fail(ce);
  for (int m = 0; be && m < 2; m++)   // the forward and inverse kernels have the block plan's shared memory
    if ((ce = cudaFuncSetAttribute(be->func[m][kio][acc], cudaFuncAttributeMaxDynamicSharedMemorySize, smem_launch)) !=
        cudaSuccess)
      return cuda_fail(ce);
  // the small-launch variants (fewer, wider teams) run launches with at most one or two groups per SM
  int smem_small[2] = {0, 0};
  for (int v = 0; v < 2; v++) {
    if (!e->func_small[v][kio][acc]) continue;
    int sm_v = e->smem_small[v][kio] < half ? half : e->smem_small[v][kio];
    if (sm_v > (int)prop.sharedMemPerBlockOptin) sm_v = (int)prop.sharedMemPerBlockOptin;
    if ((ce = cudaFuncSetAttribute(e->func_small[v][kio][acc], cudaFuncAttributeMaxDynamicSharedMemorySize, sm_v)) !=
        cudaSuccess)
      return cuda_fail(ce);
    smem_small[v] = sm_v;
  }
  const int occ = 1;

  sffft_plan* p = new sffft_plan();
  p->e = e; p->blocks = blocks; p->L = L; p->kio = kio;
  p->io = io; p->acc = acc; p->kernel_mode = kernel_mode; p->device = device;
  p->occupancy = occ; p->smem_launch = smem_launch; p->sms = prop.multiProcessorCount;
  p->smem_small[0] = smem_small[0]; p->smem_small[1] = smem_small[1];
  p->btab = nullptr; p->status = nullptr; p->be = be; p->work = nullptr; p->work_bytes = 0;
  if ((ce = cudaMalloc(&p->status, sizeof(int))) != cudaSuccess || (ce = cudaMemset(p->status, 0, sizeof(int))) != cudaSuccess) {
    cudaFree(p->status);
    delete p;
    return cuda_fail(ce);
  }
  if (kernel_mode == SFFFT_KERNEL_CACHED) {
    std::vector<uint8_t> img(e->bmat_bytes[kio], 0);
    e->build_bmat[kio](img.data());
    if ((ce = cudaMalloc(&p->btab, e->bmat_bytes[kio])) != cudaSuccess ||
        (ce = cudaMemcpy(p->btab, img.data(), e->bmat_bytes[kio], cudaMemcpyHostToDevice)) != cudaSuccess) {
      cudaFree(p->btab); cudaFree(p->status);
      delete p;
      return cuda_fail(ce);
    }
  }
  *out = p;
  return SFFFT_OK;
}

int sffft_plan_destroy(sffft_plan_t p) {
  if (!p) return SFFFT_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  cudaFree(p->btab);
  cudaFree(p->status);
  cudaSetDevice(prev);
  delete p;
  return SFFFT_OK;
}

int sffft_plan_info(sffft_plan_t p, sffft_plan_info_t* info) {
  if (!p || !info) return SFFFT_ERR_INVALID_ARGUMENT;
  const ConvEntry* e = p->e;
  std::memset(info, 0, sizeof(*info));
  info->L = p->L; info->N = 2 * p->L; info->blocks = p->blocks; info->stages = e->R2 > 1 ? 3 : 2;
  info->R0 = e->R0; info->R1 = e->R1; info->R2 = e->R2; info->pairs_per_cta = e->G;
  info->warps = e->W; info->threads = e->threads; info->smem_bytes = e->smem_bytes[p->kio];
  info->tmem_cols = e->tmem_cols[p->kio];
  info->occupancy = p->occupancy; info->io = p->io; info->acc = p->acc; info->kernel_mode = p->kernel_mode;
  info->device = p->device;
  if (p->blocks > 1) std::snprintf(info->config, sizeof(info->config), "%dx[%s]", p->blocks, e->name);
  else std::strncpy(info->config, e->name, sizeof(info->config) - 1);
  return SFFFT_OK;
}

static int use_device(int device) {
  int cur = -1;
  cudaError_t ce = cudaGetDevice(&cur);
  if (ce != cudaSuccess) return cuda_fail(ce);
  if (cur != device && (ce = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(ce);
  return SFFFT_OK;
}

int sffft_filter_spectrum(sffft_plan_t p, const void* k, int k_dtype, int H, void* Kf, void* stream) {
  return sffft_filter_spectrum_ex(p, k, k_dtype, SFFFT_FILTER_CAUSAL, H, Kf, stream);
}

int sffft_filter_spectrum_ex(sffft_plan_t p, const void* k, int k_dtype, int layout, int H, void* Kf, void* stream) {
  if (!p || !k || !Kf || H < 1 || (k_dtype != SFFFT_IO_FP32 && k_dtype != SFFFT_IO_BF16)) return SFFFT_ERR_INVALID_ARGUMENT;
  if (layout != SFFFT_FILTER_CAUSAL && layout != SFFFT_FILTER_TWO_SIDED && layout != SFFFT_FILTER_CIRCULAR)
    return SFFFT_ERR_INVALID_ARGUMENT;
  if (((uintptr_t)Kf & 15) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  int rc = use_device(p->device);
  if (rc) return rc;
  const int R[3] = {p->e->R0, p->e->R1, p->e->R2}, S = p->e->R2 > 1 ? 3 : 2;
  const bool bf = k_dtype == SFFFT_IO_BF16;
  if (p->blocks == 1) {
    const cudaError_t ce = launch_spectrum((float2*)Kf, k, bf, layout, H, R, S, (cudaStream_t)stream, false, -1, 0);
    return ce == cudaSuccess ? SFFFT_OK : cuda_fail(ce);
  }
  // composite: spectrum of filter segment d at Kf + d * H * Nb, [blocks][H][Nb]: kw_d[n] = k[d Lb + n] and
  // kw_d[Lb + m] = k[(d - 1) Lb + m] for n, m < Lb (zero for d = 0), rows of k having the full length L
  if (layout != SFFFT_FILTER_CAUSAL) return SFFFT_ERR_UNSUPPORTED;
  const int Lb = p->e->L;
  for (int d = 0; d < p->blocks; d++) {
    float2* dst = (float2*)Kf + (size_t)d * H * p->e->N;
    const cudaError_t ce = launch_spectrum(dst, k, bf, kLayoutSegment, H, R, S, (cudaStream_t)stream, false, p->L,
                                           (long long)(d - 1) * Lb);
    if (ce != cudaSuccess) return cuda_fail(ce);
  }
  return SFFFT_OK;
}

int sffft_fft_workspace_bytes(sffft_plan_t p, int B, size_t* bytes) {
  if (!p || !bytes || B < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  *bytes = (size_t)B * 2 * p->L * sizeof(float2);
  return SFFFT_OK;
}

// Digits of the standalone FFT of length 2L: the plan's radices, the last one times the block count.
static int fft_radices(sffft_plan_t p, int R[3]) {
  const int S = p->e->R2 > 1 ? 3 : 2;
  R[0] = p->e->R0; R[1] = p->e->R1; R[2] = p->e->R2;
  R[S - 1] *= p->blocks;
  return S;
}

int sffft_rfft(sffft_plan_t p, const void* x, int x_dtype, int B, void* X, void* work, void* stream) {
  if (!p || !x || !X || !work || B < 1 || (x_dtype != SFFFT_IO_FP32 && x_dtype != SFFFT_IO_BF16))
    return SFFFT_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)X | (uintptr_t)work) & 7) != 0 || ((uintptr_t)x & (x_dtype == SFFFT_IO_BF16 ? 1 : 3)) != 0)
    return SFFFT_ERR_INVALID_ARGUMENT;
  int rc = use_device(p->device);
  if (rc) return rc;
  int R[3];
  const int S = fft_radices(p, R);
  const cudaError_t ce = launch_rfft(x, x_dtype == SFFFT_IO_BF16, B, (float2*)X, (float2*)work, R, S, p->sms,
                                     (cudaStream_t)stream);
  return ce == cudaSuccess ? SFFFT_OK : cuda_fail(ce);
}

int sffft_irfft(sffft_plan_t p, const void* X, int B, float* x, void* work, void* stream) {
  if (!p || !X || !x || !work || B < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)X | (uintptr_t)work) & 7) != 0 || ((uintptr_t)x & 3) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  int rc = use_device(p->device);
  if (rc) return rc;
  int R[3];
  const int S = fft_radices(p, R);
  const cudaError_t ce = launch_irfft((const float2*)X, B, x, (float2*)work, R, S, p->sms, (cudaStream_t)stream);
  return ce == cudaSuccess ? SFFFT_OK : cuda_fail(ce);
}

static int conv_launch(sffft_plan_t p, const void* u, const void* Kf, void* y, int B, int H, cudaStream_t stream,
                       unsigned long long wait_ns, int skip_arrive, int mode = 0, const BlockArgs* blk = nullptr);

// Workspace of a composite plan's convolution of a B x H batch: the pair spectra of all input blocks
// ([H * blocks][ceil(B/2)][N] complex fp32, *zbytes) and then the row energies ([B][H] fp32); 0 for a
// single-pass plan.
static size_t conv_ws_bytes(sffft_plan_t p, int B, int H, size_t* zbytes) {
  *zbytes = 0;
  if (p->blocks == 1) return 0;
  *zbytes = (size_t)((B + 1) / 2) * (size_t)H * (size_t)p->blocks * (size_t)p->e->N * sizeof(float2);
  return *zbytes + ((size_t)B * H * sizeof(float) + 255) / 256 * 256;
}

int sffft_conv_workspace_bytes(sffft_plan_t p, int B, int H, size_t* bytes) {
  if (!p || !bytes || B < 1 || H < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  size_t z;
  *bytes = conv_ws_bytes(p, B, H, &z);
  return SFFFT_OK;
}

int sffft_plan_set_workspace(sffft_plan_t p, void* work, size_t bytes) {
  if (!p || (work && ((uintptr_t)work & 255) != 0)) return SFFFT_ERR_INVALID_ARGUMENT;
  p->work = work;
  p->work_bytes = work ? bytes : 0;
  return SFFFT_OK;
}

int sffft_conv(sffft_plan_t p, const void* u, const void* Kf, void* y, int B, int H, void* stream) {
  if (!p) return SFFFT_ERR_INVALID_ARGUMENT;
  return sffft_conv_ws(p, u, Kf, y, B, H, p->work, p->work_bytes, stream);
}

int sffft_conv_ws(sffft_plan_t p, const void* u, const void* Kf, void* y, int B, int H, void* work, size_t work_bytes,
                  void* stream) {
  if (!p || !u || !Kf || !y || B < 1 || H < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)u | (uintptr_t)y | (uintptr_t)Kf) & 15) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  if (p->blocks == 1) return conv_launch(p, u, Kf, y, B, H, (cudaStream_t)stream, 0, 0);

  // composite plan: partitioned convolution over the [B][H * P][Lb] view of u and y (stages.h)
  const int P = p->blocks, Lb = p->e->L;
  if ((long long)H * P > std::numeric_limits<int>::max() / 2 || (long long)B * H * P > std::numeric_limits<int>::max())
    return SFFFT_ERR_INVALID_ARGUMENT;
  size_t zbytes;
  const size_t need = conv_ws_bytes(p, B, H, &zbytes);
  if (!work || work_bytes < need) return SFFFT_ERR_WORKSPACE;
  if (((uintptr_t)work & 255) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  int rc = use_device(p->device);
  if (rc) return rc;
  const cudaStream_t st = (cudaStream_t)stream;
  BlockArgs blk;
  blk.Z = (float*)work;
  blk.En = (const float*)((char*)work + zbytes);
  blk.lgP = 0;
  while ((1 << blk.lgP) < P) blk.lgP++;
  blk.Hb = H;
  const cudaError_t ce = launch_row_energy(u, p->io == SFFFT_IO_BF16, (long long)B * H, p->L, Lb,
                                           (float*)((char*)work + zbytes), st);
  if (ce != cudaSuccess) return cuda_fail(ce);
  rc = conv_launch(p, u, nullptr, nullptr, B, H * P, st, 0, 0, 1, &blk);
  if (rc) return rc;
  const cudaError_t cs = launch_spectrum_sum(blk.Z, (const float*)Kf, H, (B + 1) / 2, p->e->N, P, p->sms, st);
  if (cs != cudaSuccess) return cuda_fail(cs);
  return conv_launch(p, nullptr, Kf, y, B, H * P, st, 0, 0, 2, &blk);
}

static int conv_launch(sffft_plan_t p, const void* u, const void* Kf, void* y, int B, int H, cudaStream_t stream,
                       unsigned long long wait_ns, int skip_arrive, int mode, const BlockArgs* blk) {
  const ConvEntry* e = p->e;
  const long long pairs = (long long)((B + 1) / 2) * H;
  const long long groups = (pairs + e->G - 1) / e->G;
  if ((long long)B * H > std::numeric_limits<int>::max() || groups > std::numeric_limits<int>::max())
    return SFFFT_ERR_INVALID_ARGUMENT;
  const int grid = (int)(groups < p->sms ? groups : p->sms);
  int rc = use_device(p->device);
  if (rc) return rc;
  ConvParams prm;
  prm.u = u; prm.Kf = (const float*)Kf; prm.btab = p->btab; prm.y = y; prm.status = p->status; prm.B = B; prm.H = H;
  prm.ngroups = (int)groups;
  prm.wait_ns = wait_ns;
  prm.debug_skip_arrive = skip_arrive;
  prm.blk = blk ? *blk : BlockArgs{nullptr, nullptr, 0, 0};
#ifdef SFFFT_TRACE
  prm.trace = g_trace;
#endif
  cudaError_t ce;
  if (mode > 0) {
    ce = p->be->launch[mode - 1][p->kio][p->acc](prm, grid, p->smem_launch, stream);
  } else {
    // one or two groups per SM: the variant with as many (wider) teams as there are groups shortens each
    // group's chain; otherwise the plan's own 4-slot kernel
    const long long per_cta = (groups + p->sms - 1) / p->sms;
    const int v = per_cta <= 1 ? 0 : (per_cta <= 2 ? 1 : -1);
    ce = (v >= 0 && p->smem_small[v]) ? e->launch_small[v][p->kio][p->acc](prm, grid, p->smem_small[v], stream)
                                      : e->launch[p->kio][p->acc](prm, grid, p->smem_launch, stream);
  }
  return ce == cudaSuccess ? SFFFT_OK : cuda_fail(ce);
}

int sffft_plan_check(sffft_plan_t p) {
  if (!p) return SFFFT_ERR_INVALID_ARGUMENT;
  int rc = use_device(p->device);
  if (rc) return rc;
  cudaError_t ce = cudaDeviceSynchronize();
  if (ce != cudaSuccess) return cuda_fail(ce);
  int st = 0;
  if ((ce = cudaMemcpy(&st, p->status, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess) return cuda_fail(ce);
  if (st && (ce = cudaMemset(p->status, 0, sizeof(int))) != cudaSuccess) return cuda_fail(ce);
  return st;
}

double sffft_relative_l2(double se, double sr) {
  if (sr > 0) return std::sqrt(se / sr);
  return se == 0 ? 0 : std::numeric_limits<double>::infinity();
}

int sffft_select_candidate(const sffft_candidate_t* c, int n, double max_error, const char* io) {
  if (!io || !std::isfinite(max_error) || max_error <= 0) return -1;
  if (std::strcmp(io, "fp32") && std::strcmp(io, "bf16") && std::strcmp(io, "any")) return -1;
  if (n > 0 && !c) return -1;
  int best = -1;
  for (int i = 0; i < n; i++) {
    if (std::strcmp(io, "any") && (!c[i].io || std::strcmp(io, c[i].io))) continue;
    if (!std::isfinite(c[i].ms) || c[i].ms <= 0 || !std::isfinite(c[i].rel_err) || c[i].rel_err < 0 ||
        c[i].rel_err > max_error)
      continue;
    if (best < 0 || c[i].ms < c[best].ms || (c[i].ms == c[best].ms && c[i].rel_err < c[best].rel_err)) best = i;
  }
  return best;
}

int sffft_shard_range(int H, int shards, int shard, int* h0, int* h1) {
  if (H < 1 || shards < 1 || shard < 0 || shard >= shards || !h0 || !h1) return SFFFT_ERR_INVALID_ARGUMENT;
  const int base = H / shards, extra = H % shards;
  *h0 = shard * base + (shard < extra ? shard : extra);
  *h1 = *h0 + base + (shard < extra ? 1 : 0);
  return SFFFT_OK;
}

int sffft_baseline_create(sffft_baseline_t* out, int L, int B, int H, const float* k_dev, int device) {
  if (!out) return SFFFT_ERR_INVALID_ARGUMENT;
  Baseline* b = nullptr;
  const int rc = baseline_create(&b, L, B, H, k_dev, device);
  if (rc) return rc;
  *out = new sffft_baseline{b};
  return SFFFT_OK;
}

int sffft_baseline_run(sffft_baseline_t bl, const float* u, float* y, int full, void* stream) {
  if (!bl || !u || (full && !y)) return SFFFT_ERR_INVALID_ARGUMENT;
  return baseline_run(bl->b, u, y, full, (cudaStream_t)stream);
}

int sffft_baseline_destroy(sffft_baseline_t bl) {
  if (!bl) return SFFFT_ERR_INVALID_ARGUMENT;
  baseline_destroy(bl->b);
  delete bl;
  return SFFFT_OK;
}

int sffft_debug_umma_probe(int a_kind, int a_slice, int b_pitch, int b_slice, int n, int acc16, const unsigned short* A,
                           const unsigned short* B, unsigned int* D) {
  if (!A || !B || !D) return SFFFT_ERR_INVALID_ARGUMENT;
  return umma_probe(a_kind, a_slice, b_pitch, b_slice, n, acc16, A, B, D);
}

int sffft_debug_wait_timeout(int limit_us) { return wait_timeout_probe(limit_us); }

int sffft_debug_conv_timeout(sffft_plan_t p, const void* u, const void* Kf, void* y, int B, int H, int limit_us,
                             void* stream) {
  if (!p || !u || !Kf || !y || B < 1 || H < 1 || p->blocks != 1 || limit_us < 1 || limit_us > 1000000)
    return SFFFT_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)u | (uintptr_t)y | (uintptr_t)Kf) & 15) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  return conv_launch(p, u, Kf, y, B, H, (cudaStream_t)stream, 1000ull * (unsigned long long)limit_us, 1);
}

}  // extern "C"
