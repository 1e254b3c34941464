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
//                          Each device has a host thread of its own (started with the multi-device pipe), which
//                          issues that device's copies and kernels and waits for them, so no device waits for
//                          the host to finish issuing another device's work.
#include <cuda_runtime.h>

#include <condition_variable>
#include <mutex>
#include <new>
#include <thread>
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
  // one worker thread per shard; a call publishes its arguments, bumps `gen` and waits until `pending` is 0
  std::vector<std::thread> workers;
  std::mutex mu;
  std::condition_variable go, done;
  unsigned gen = 0;
  int pending = 0;
  bool quit = false;
  const void* u_host = nullptr;
  const void* const* Kf = nullptr;
  void* y_host = nullptr;
  std::vector<int> rc;                 // per shard: the status of the current call
};

namespace {

// Shard g's part of one sffft_conv_host_multi call, on its worker thread: issue the shard's chunks on its device,
// wait for them and read the device-side status.
int run_shard(sffft_multi* m, int g) {
  if (!m->Kf[g]) return SFFFT_ERR_INVALID_ARGUMENT;
  if (cudaSetDevice(m->dev[g]) != cudaSuccess) return SFFFT_ERR_CUDA;
  const size_t col = (size_t)m->L * m->sio;   // bytes of one channel row
  int rc = sffft_conv_host(m->pipes[g], (const char*)m->u_host + (size_t)m->h0[g] * col, m->Kf[g],
                           (char*)m->y_host + (size_t)m->h0[g] * col, m->streams[g]);
  if (cudaStreamSynchronize(m->streams[g]) != cudaSuccess && !rc) rc = SFFFT_ERR_CUDA;
  const int st = sffft_plan_check(m->plans[g]);   // device-side status of the shard's kernels
  return rc ? rc : st;
}

void worker(sffft_multi* m, int g) {
  unsigned seen = 0;
  while (true) {
    {
      std::unique_lock<std::mutex> lk(m->mu);
      m->go.wait(lk, [&] { return m->quit || m->gen != seen; });
      if (m->quit) return;
      seen = m->gen;
    }
    const int rc = run_shard(m, g);
    std::lock_guard<std::mutex> lk(m->mu);
    m->rc[g] = rc;
    if (--m->pending == 0) m->done.notify_all();
  }
}

}  // namespace

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
  m->rc.assign(G, SFFFT_OK);
  try {
    for (int g = 0; g < G; g++) m->workers.emplace_back(worker, m, g);
  } catch (...) {
    sffft_multi_pipe_destroy(m);
    return SFFFT_ERR_ALLOC;
  }
  *out = m;
  return SFFFT_OK;
}

extern "C" int sffft_conv_host_multi(sffft_multi_t m, const void* u_host, const void* const* Kf, void* y_host) {
  if (!m || !u_host || !Kf || !y_host) return SFFFT_ERR_INVALID_ARGUMENT;
  // every shard's worker issues and waits for its own device's work; the first error (in shard order) is returned
  std::unique_lock<std::mutex> lk(m->mu);
  m->u_host = u_host;
  m->Kf = Kf;
  m->y_host = y_host;
  m->pending = m->G;
  m->gen++;
  m->go.notify_all();
  m->done.wait(lk, [&] { return m->pending == 0; });
  for (int g = 0; g < m->G; g++)
    if (m->rc[g]) return m->rc[g];
  return SFFFT_OK;
}

extern "C" int sffft_multi_pipe_destroy(sffft_multi_t m) {
  if (!m) return SFFFT_ERR_INVALID_ARGUMENT;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    m->quit = true;
  }
  m->go.notify_all();
  for (std::thread& t : m->workers) t.join();
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
