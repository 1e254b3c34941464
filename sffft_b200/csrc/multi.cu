// Channel-sharded convolution over several devices (no reference counterpart: the reference runs on device 0
// only, sfFFT src/sffft.cu:490).
//
// Sequences are independent, so shard g of G owns the contiguous channel range [h0, h1) of
// sffft_shard_range(H, G, g) together with its spectrum rows; nothing is exchanged between devices.
//   sffft_conv_multi       device-resident shards: plan g's device holds u_g, y_g [B][h1 - h0][L] and
//                          Kf_g [h1 - h0][N]; one sffft_conv per device on that device's stream.
//   sffft_conv_host_multi  one [B][H][L] batch in (pinned) host memory: device g uploads its channel slice
//                          (one pitched copy per chunk: B rows of (h1 - h0) * L contiguous values), convolves
//                          it and downloads its slice of y through a host pipe of its own, so the devices'
//                          copies and kernels run concurrently; the call returns when every device is done.
#include <cuda_runtime.h>

#include <new>
#include <vector>

#include "../../include/sffft.h"

int sffft_pipe_create_slice(sffft_pipe_t* pipe, sffft_plan_t plan, int B, int H, int hp, int chunks);

namespace {

int shard_of(int H, int G, int g, int* h0, int* h1) { return sffft_shard_range(H, G, g, h0, h1); }

int device_of(sffft_plan_t p, int* dev, int* L, int* io) {
  sffft_plan_info_t info;
  const int rc = sffft_plan_info(p, &info);
  if (rc) return rc;
  *dev = info.device;
  *L = info.L;
  *io = info.io;
  return SFFFT_OK;
}

}  // namespace

struct sffft_multi {
  int G, B, H, L, sio;
  std::vector<sffft_plan_t> plans;
  std::vector<int> h0, h1, dev;
  std::vector<sffft_pipe_t> pipes;
  std::vector<cudaStream_t> streams;   // per shard: the stream its pipe is ordered on
};

extern "C" int sffft_conv_multi(const sffft_plan_t* plans, int G, const void* const* u, const void* const* Kf,
                                void* const* y, int B, int H, void* const* streams) {
  if (!plans || G < 1 || !u || !Kf || !y || B < 1 || H < G) return SFFFT_ERR_INVALID_ARGUMENT;
  int L0 = -1, io0 = -1;
  for (int g = 0; g < G; g++) {
    int dev, L, io;
    if (!plans[g]) return SFFFT_ERR_INVALID_ARGUMENT;
    const int rc = device_of(plans[g], &dev, &L, &io);
    if (rc) return rc;
    if (g > 0 && (L != L0 || io != io0)) return SFFFT_ERR_INVALID_ARGUMENT;
    L0 = L;
    io0 = io;
  }
  for (int g = 0; g < G; g++) {
    int h0, h1;
    int rc = shard_of(H, G, g, &h0, &h1);
    if (!rc) rc = sffft_conv(plans[g], u[g], Kf[g], y[g], B, h1 - h0, streams ? streams[g] : nullptr);
    if (rc) return rc;
  }
  return SFFFT_OK;
}

extern "C" int sffft_multi_pipe_create(sffft_multi_t* out, const sffft_plan_t* plans, int G, int B, int H,
                                       int chunks) {
  if (!out || !plans || G < 1 || B < 1 || H < G || chunks < 0) return SFFFT_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  sffft_multi* m = new (std::nothrow) sffft_multi();
  if (!m) return SFFFT_ERR_ALLOC;
  m->G = G;
  m->B = B;
  m->H = H;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) {
    delete m;
    return SFFFT_ERR_CUDA;
  }
  int rc = SFFFT_OK;
  for (int g = 0; g < G && rc == SFFFT_OK; g++) {
    int dev = 0, L = 0, io = 0, h0 = 0, h1 = 0;
    if (!plans[g]) rc = SFFFT_ERR_INVALID_ARGUMENT;
    if (!rc) rc = device_of(plans[g], &dev, &L, &io);
    if (!rc && g > 0 && (L != m->L || (io == SFFFT_IO_BF16 ? 2 : 4) != m->sio)) rc = SFFFT_ERR_INVALID_ARGUMENT;
    if (!rc) rc = shard_of(H, G, g, &h0, &h1);
    sffft_pipe_t pipe = nullptr;
    if (!rc) rc = sffft_pipe_create_slice(&pipe, plans[g], B, h1 - h0, H, chunks);
    cudaStream_t st = nullptr;
    if (!rc && (cudaSetDevice(dev) != cudaSuccess || cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess))
      rc = SFFFT_ERR_CUDA;
    if (rc) {
      if (pipe) sffft_pipe_destroy(pipe);
      break;
    }
    m->L = L;
    m->sio = io == SFFFT_IO_BF16 ? 2 : 4;
    m->plans.push_back(plans[g]);
    m->h0.push_back(h0);
    m->h1.push_back(h1);
    m->dev.push_back(dev);
    m->pipes.push_back(pipe);
    m->streams.push_back(st);
  }
  cudaSetDevice(prev);
  if (rc) {
    sffft_multi_pipe_destroy(m);
    return rc;
  }
  *out = m;
  return SFFFT_OK;
}

extern "C" int sffft_conv_host_multi(sffft_multi_t m, const void* u_host, const void* const* Kf, void* y_host) {
  if (!m || !u_host || !Kf || !y_host) return SFFFT_ERR_INVALID_ARGUMENT;
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return SFFFT_ERR_CUDA;
  // queue every device's chunks first (the calls return once queued), then wait for all of them
  int rc = SFFFT_OK;
  const size_t col = (size_t)m->L * m->sio;   // bytes of one channel row
  for (int g = 0; g < m->G && rc == SFFFT_OK; g++) {
    if (!Kf[g]) { rc = SFFFT_ERR_INVALID_ARGUMENT; break; }
    rc = sffft_conv_host(m->pipes[g], (const char*)u_host + (size_t)m->h0[g] * col, Kf[g],
                         (char*)y_host + (size_t)m->h0[g] * col, m->streams[g]);
  }
  for (int g = 0; g < m->G; g++) {
    if (cudaSetDevice(m->dev[g]) != cudaSuccess || cudaStreamSynchronize(m->streams[g]) != cudaSuccess) {
      if (!rc) rc = SFFFT_ERR_CUDA;
      continue;
    }
    const int st = sffft_plan_check(m->plans[g]);   // device-side status of the shard's kernels
    if (!rc) rc = st;
  }
  cudaSetDevice(prev);
  return rc;
}

extern "C" int sffft_multi_pipe_destroy(sffft_multi_t m) {
  if (!m) return SFFFT_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaGetDevice(&prev);
  for (size_t g = 0; g < m->pipes.size(); g++) {
    sffft_pipe_destroy(m->pipes[g]);
    cudaSetDevice(m->dev[g]);
    if (m->streams[g]) cudaStreamDestroy(m->streams[g]);
  }
  cudaSetDevice(prev);
  delete m;
  return SFFFT_OK;
}
