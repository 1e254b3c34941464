// Allocation-free convolution entry point.
//
// The regular path needs device memory that the caller (or the library) allocates: the filter spectrum
// Kf that sffft_filter_spectrum writes, and the plan's status word and DFT-matrix table that
// sffft_plan_create allocates.  Some callers cannot allocate at all once they are running -- for example
// an inference-engine plugin whose execute step must not allocate, or a process whose device memory is
// entirely reserved by another allocator.  sffft_conv_noalloc serves them: the caller passes only u, the
// filter k and y, and the spectrum plus the status word live in one fixed-size array defined below,
// which every GPU that loads the library holds until the process exits.
//
// The array is shared by every call on a device and keeps the last call's contents, so calls that
// overlap on the GPU (different streams, host threads or processes sharing a context) race on it.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "../../include/sffft.h"
#include "fused_conv.cuh"
#include "registry.h"
#include "spectrum.h"

namespace {

using namespace sffft;

// Largest filter spectrum the fixed scratch holds: H * 2L complex fp32 values (16 MiB, e.g. H = 1024
// channels at L = 1024, or H = 128 at L = 8192).
constexpr size_t kSpectrumBytes = 16u << 20;
constexpr size_t kStatusBytes = 256;   // status word, padded so the spectrum starts 256-byte aligned

static __device__ __align__(256) unsigned char g_noalloc_scratch[kStatusBytes + kSpectrumBytes];

constexpr int kMaxDevices = 64;
constexpr int kMaxEntries = 64;

struct DeviceState {
  unsigned char* scratch = nullptr;        // device address of g_noalloc_scratch on this device
  int sms = 0, smem_per_sm = 0, smem_optin = 0;
  bool attr_set[kMaxEntries][2][2] = {};   // shared-memory attribute set for (entry, io, acc)
};
DeviceState g_dev[kMaxDevices];
std::mutex g_mutex;

const ConvEntry* find_entry(const char* name, int* index) {
  const ConvEntry* p;
  int base = 0;
  int (*parts[3])(const ConvEntry**) = {entries_small, entries_mid, entries_large};
  for (auto part : parts) {
    const int n = part(&p);
    for (int i = 0; i < n; i++)
      if (std::strcmp(p[i].name, name) == 0) {
        *index = base + i;
        return p + i;
      }
    base += n;
  }
  return nullptr;
}

}  // namespace

extern "C" int sffft_conv_noalloc(int L, int io, int acc, const void* u, const void* k, int k_dtype, void* y, int B,
                                  int H, void* stream, int sync) {
  if (!u || !k || !y || B < 1 || H < 1) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((io != SFFFT_IO_FP32 && io != SFFFT_IO_BF16) || (acc != SFFFT_ACC_FP32 && acc != SFFFT_ACC_FP16) ||
      (k_dtype != SFFFT_IO_FP32 && k_dtype != SFFFT_IO_BF16))
    return SFFFT_ERR_INVALID_ARGUMENT;
  if ((((uintptr_t)u | (uintptr_t)y) & 15) != 0) return SFFFT_ERR_INVALID_ARGUMENT;
  char name[96];
  if (sffft_default_config(L, name, sizeof(name)) != SFFFT_OK) return SFFFT_ERR_UNSUPPORTED;
  int index = -1;
  const ConvEntry* e = find_entry(name, &index);
  if (!e || index >= kMaxEntries) return SFFFT_ERR_UNSUPPORTED;
  const long long pairs = (long long)((B + 1) / 2) * H;
  const long long groups = (pairs + e->G - 1) / e->G;
  if ((long long)B * H > 0x7fffffffLL || groups > 0x7fffffffLL) return SFFFT_ERR_INVALID_ARGUMENT;
  if ((size_t)H * (size_t)e->N * 8 > kSpectrumBytes) return SFFFT_ERR_SCRATCH_LIMIT;

  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SFFFT_ERR_CUDA;
  DeviceState& ds = g_dev[dev];
  {
    // one-time set-up per device (and per kernel variant), with that device current
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds.scratch) {
      // the device check comes first: on another GPU the library has no kernel image, so the symbol lookup
      // below would fail with a CUDA error instead of SFFFT_ERR_DEVICE
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return SFFFT_ERR_CUDA;
      if (prop.major != 10 || prop.minor != 0) return SFFFT_ERR_DEVICE;
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
        cudaGetLastError();   // leave no pending error behind for the caller's next CUDA call
        return SFFFT_ERR_CUDA;
      }
      ds.sms = prop.multiProcessorCount;
      ds.smem_per_sm = (int)prop.sharedMemPerMultiprocessor;
      ds.smem_optin = (int)prop.sharedMemPerBlockOptin;
      ds.scratch = static_cast<unsigned char*>(ptr);
    }
  }
  const int need = e->smem_bytes[io];
  if (need > ds.smem_optin) return SFFFT_ERR_DEVICE;
  int smem_launch = need;
  const int half = ds.smem_per_sm / 2 + 1024;   // one CTA per SM, as for plans
  if (smem_launch < half) smem_launch = half;
  if (smem_launch > ds.smem_optin) smem_launch = ds.smem_optin;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds.attr_set[index][io][acc]) {
      if (cudaFuncSetAttribute(e->func[io][acc], cudaFuncAttributeMaxDynamicSharedMemorySize, smem_launch) != cudaSuccess)
        return SFFFT_ERR_CUDA;
      ds.attr_set[index][io][acc] = true;
    }
  }

  cudaStream_t st = (cudaStream_t)stream;
  int* status = reinterpret_cast<int*>(ds.scratch);
  float2* Kf = reinterpret_cast<float2*>(ds.scratch + kStatusBytes);
  if (cudaMemsetAsync(status, 0, sizeof(int), st) != cudaSuccess) return SFFFT_ERR_CUDA;
  const int R[3] = {e->R0, e->R1, e->R2};
  if (launch_spectrum(Kf, k, k_dtype == SFFFT_IO_BF16, SFFFT_FILTER_CAUSAL, H, R, e->R2 > 1 ? 3 : 2, st, false, -1, 0) != cudaSuccess) return SFFFT_ERR_CUDA;
  ConvParams prm;
  std::memset(&prm, 0, sizeof(prm));
  prm.u = u; prm.Kf = reinterpret_cast<const float*>(Kf); prm.btab = nullptr;   // DFT matrices built in-kernel
  prm.y = y; prm.status = status; prm.B = B; prm.H = H; prm.ngroups = (int)groups;
  const int grid = (int)(groups < ds.sms ? groups : ds.sms);
  if (e->launch[io][acc](prm, grid, smem_launch, st) != cudaSuccess) return SFFFT_ERR_CUDA;
  if (sync) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return SFFFT_ERR_CUDA;
    int word = 0;
    if (cudaMemcpy(&word, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return SFFFT_ERR_CUDA;
    if (word) return word;
  }
  return SFFFT_OK;
}
