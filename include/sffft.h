/* sffft — B200 (sm_100a) fused causal long convolution, C ABI.
 *
 *   y[b,h,n] = sum_{m<=n} u[b,h,m] * k[h,n-m],   0 <= n < L
 *
 * Drop-in for the operator surface of sfFFT (github.com/solidsf-inc/sfFFT, src/sffft.cu and
 * src/selection.h).  All device buffers are caller-owned; calls are asynchronous on the given CUDA
 * stream (cudaStream_t passed as void*, NULL = default stream); every call returns an int status
 * (SFFFT_OK = 0) and never exits the process.  Plans are immutable after creation and may be shared
 * by host threads.  There is no CPU fallback: without a B200-class device, plan creation fails.
 *
 * Layouts (identical to the reference):
 *   u, y : [B][H][L] contiguous, fp32 or bf16 (plan io), 16-byte aligned
 *   k    : [H][L] contiguous real filter, fp32 or bf16 (k_dtype)
 *   Kf   : [H][N] complex fp32 (float pairs), N = 2L, unnormalised DFT of the zero-padded filter in the
 *          plan's digit order: position p = k0*R1*R2 + k1*R2 + k2 holds frequency k0 + R0*k1 + R0*R1*k2
 *          (the layout permuteK writes, src/sffft.cu:283-288)
 */
#ifndef SFFFT_H_
#define SFFFT_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SFFFT_OK 0
#define SFFFT_ERR_INVALID_ARGUMENT 1
#define SFFFT_ERR_UNSUPPORTED 2
#define SFFFT_ERR_CUDA 3
#define SFFFT_ERR_DEVICE 4
#define SFFFT_ERR_TIMEOUT 5
#define SFFFT_ERR_NO_MATCH 6
#define SFFFT_ERR_ALLOC 7
#define SFFFT_ERR_SCRATCH_LIMIT 8 /* problem too large for sffft_conv_noalloc's fixed scratch */
#define SFFFT_ERR_WORKSPACE 9     /* composite plan called without a large enough workspace */

#define SFFFT_IO_FP32 0
#define SFFFT_IO_BF16 1
#define SFFFT_ACC_FP32 0
#define SFFFT_ACC_FP16 1
#define SFFFT_KERNEL_LEGACY 0 /* DFT matrices computed inside every CTA (reference --kernel legacy) */
#define SFFFT_KERNEL_CACHED 1 /* DFT matrices copied from a precomputed table (reference --kernel cached) */

typedef struct sffft_plan* sffft_plan_t;

typedef struct {
  int L, N, stages, R0, R1, R2;
  int pairs_per_cta;   /* G: pairs of batch elements (same channel) per CTA */
  int warps, threads, smem_bytes, tmem_cols, occupancy;
  int io, acc, kernel_mode, device;
  int blocks;          /* 1, or the block count of a composite plan (L = blocks * block length) */
  char config[96];     /* catalog name, e.g. "64x32/w4", or "2x[32x32x32/w8]" for a composite plan */
} sffft_plan_info_t;

/* Creates a plan for length L (power of two).  config: catalog name ("64x32/w4") for L = 128..16384, or
 * NULL / "" for the built-in B200 default for L.  Replaces the compile-time choice of fftconv<Plan<R0,R1,R2>,
 * W,TIO,TAcc,CACHED> plus its cudaFuncSetAttribute / occupancy setup (src/sffft.cu:243-245, 385-388).
 * Composite plans (no reference counterpart; the reference stops at L = 8192 and lists multi-pass plans
 * as missing, README.md:175): config "<P>x[<catalog name>]" runs L = P * Lb (P = 2..16) as a partitioned
 * convolution on the catalog plan of length Lb (a forward transform per input block, then per output block
 * the sum of block spectra times filter-segment spectra and one inverse transform; block plans: the default
 * plan of each length up to 16384, and 16x16/w4), and the default for L = 32768 .. 262144 is
 * "<L/16384>x[<default for 16384>]".  For a composite plan Kf holds the P filter-segment spectra
 * [P][H][2 Lb] (the same H * 2L complex values), filter layouts other than causal are unsupported, and the
 * convolution needs a caller-owned workspace (sffft_conv_workspace_bytes): passed to sffft_conv_ws, or
 * attached to the plan for sffft_conv with sffft_plan_set_workspace. */
int sffft_plan_create(sffft_plan_t* plan, int L, int io, int acc, const char* config, int kernel_mode, int device);
int sffft_plan_destroy(sffft_plan_t plan);
int sffft_plan_info(sffft_plan_t plan, sffft_plan_info_t* info);

/* Filter spectrum in the plan's digit order, once per channel (untimed prep).  k_dtype: SFFFT_IO_FP32 or
 * SFFFT_IO_BF16.  Replaces host zero-padding + cufftExecC2C + permuteK (src/sffft.cu:342-344, 365,
 * 283-288, 384). */
int sffft_filter_spectrum(sffft_plan_t plan, const void* k, int k_dtype, int H, void* Kf, void* stream);

/* Filter layouts: which convolution sffft_conv computes, for n in [0, L), with the spectrum of k. */
#define SFFFT_FILTER_CAUSAL 0    /* k [H][L]:    y[n] = sum_{m<=n} u[m] k[n-m]           (the reference's) */
#define SFFFT_FILTER_TWO_SIDED 1 /* k [H][2L-1]: y[n] = sum_{m<L} u[m] k[L-1+n-m]        (non-causal) */
#define SFFFT_FILTER_CIRCULAR 2  /* k [H][L]:    y[n] = sum_{m<L} u[m] k[(n-m) mod L]    (period L) */

/* sffft_filter_spectrum for a filter in the given layout (SFFFT_FILTER_*); the fused convolution is the
 * same kernel for all three.  The reference exposes only the causal form; non-causal and circular
 * convolution are listed as not yet exposed (README.md:174). */
int sffft_filter_spectrum_ex(sffft_plan_t plan, const void* k, int k_dtype, int layout, int H, void* Kf,
                             void* stream);

/* Standalone real FFTs of length N = 2L (the plan's N) over B rows, on the same digit decomposition as
 * the filter-spectrum prep (fp32 CUDA cores, exact twiddles); no reference counterpart (README.md:174
 * lists standalone forward and inverse FFTs as not yet exposed).
 *   sffft_rfft:  x [B][N] real (x_dtype SFFFT_IO_FP32 or SFFFT_IO_BF16) -> X [B][N/2+1] complex fp32,
 *                X[f] = sum_n x[n] exp(-2 pi i f n / N)              (numpy.fft.rfft)
 *   sffft_irfft: X [B][N/2+1] complex fp32 -> x [B][N] fp32,
 *                x[n] = (1/N) sum_f Xfull[f] exp(+2 pi i f n / N)    (numpy.fft.irfft; the imaginary
 *                parts of X[0] and X[N/2] are ignored)
 * work: caller-owned device buffer of sffft_fft_workspace_bytes(plan, B) bytes, 8-byte aligned. */
int sffft_fft_workspace_bytes(sffft_plan_t plan, int B, size_t* bytes);
int sffft_rfft(sffft_plan_t plan, const void* x, int x_dtype, int B, void* X, void* work, void* stream);
int sffft_irfft(sffft_plan_t plan, const void* X, int B, float* x, void* work, void* stream);

/* The fused convolution: one kernel launch per call (four for a composite plan, which needs a workspace: see
 * sffft_conv_ws).  Replaces the launch fftconv<P,W,TIO,TAcc,CACHED><<<B*H, 32*W, smem>>>(u, Kf, tw, dft, y, B, H)
 * (src/sffft.cu:243-280, 389-390); the unused twiddle table and the DFT table are owned by the plan.  The kernel
 * is a programmatic dependent of the stream's previous kernel: its prologue may overlap that kernel's end, and it
 * reads u and Kf only after that kernel has completed. */
int sffft_conv(sffft_plan_t plan, const void* u, const void* Kf, void* y, int B, int H, void* stream);

/* Workspace of a composite plan's convolution of a B x H batch, in bytes: the forward spectra of every
 * input block (ceil(B/2) * H * L * 16 bytes) and the row energies; 0 for single-pass plans. */
int sffft_conv_workspace_bytes(sffft_plan_t plan, int B, int H, size_t* bytes);
/* sffft_conv with a caller-owned device workspace (256-byte aligned, at least sffft_conv_workspace_bytes;
 * NULL for single-pass plans).  A composite call is four launches in stream order (row energies, forward
 * transforms, spectrum sums, inverse transforms); the workspace must not be shared by calls that can overlap.
 * Returns SFFFT_ERR_WORKSPACE when a composite plan gets no workspace or too small a one. */
int sffft_conv_ws(sffft_plan_t plan, const void* u, const void* Kf, void* y, int B, int H, void* work,
                  size_t work_bytes, void* stream);
/* Attaches a caller-owned workspace (256-byte aligned; NULL detaches) that sffft_conv uses for composite
 * plans, which otherwise return SFFFT_ERR_WORKSPACE.  The plan does not free it. */
int sffft_plan_set_workspace(sffft_plan_t plan, void* work, size_t bytes);

/* Waits for the plan's device and returns (and clears) the device-side status word: SFFFT_OK, or
 * SFFFT_ERR_TIMEOUT when a kernel barrier wait gave up.  No reference counterpart (the reference has no
 * device-side error reporting; its CUDA errors surface through cudaGetLastError, src/sffft.cu:324). */
int sffft_plan_check(sffft_plan_t plan);

/* Plan catalog (the candidates of the reference's RUN rows, src/sffft.cu:506-513, plus L = 16384). */
int sffft_catalog_count(void);
int sffft_catalog_entry(int index, int* L, char* name, int name_cap);
int sffft_default_config(int L, char* name, int name_cap);

/* Empirical selector with the semantics of select_candidate / relative_l2 (src/selection.h:13-29):
 * returns the index of the fastest candidate with finite ms > 0 and finite 0 <= rel_err <= max_error
 * whose io matches (or io == "any"); ties go to the lower error; -1 when nothing qualifies or the budget
 * or io is invalid. */
typedef struct {
  const char* method;
  const char* io;
  const char* config;
  double ms, rel_err;
} sffft_candidate_t;
int sffft_select_candidate(const sffft_candidate_t* candidates, int count, double max_error, const char* io);
double sffft_relative_l2(double squared_error, double squared_reference);

/* Channel sharding across devices: shard g of G owns channels [h0, h1) (contiguous, sizes differ by at
 * most one).  No reference counterpart (the reference is single-GPU, src/sffft.cu:490). */
int sffft_shard_range(int H, int shards, int shard, int* h0, int* h1);

const char* sffft_status_string(int status);
int sffft_last_cuda_error(void);

/* cuFFT baseline pipeline on the same device (src/sffft.cu:289-305, 365-371): spectrum from the
 * fp32 filter k_dev [H][L]; run(full=1) = pad -> R2C -> multiply -> C2R -> slice, run(full=0) = core
 * only (reuses the padded input of the previous full run). */
typedef struct sffft_baseline* sffft_baseline_t;
int sffft_baseline_create(sffft_baseline_t* bl, int L, int B, int H, const float* k_dev, int device);
int sffft_baseline_run(sffft_baseline_t bl, const float* u, float* y, int full, void* stream);
int sffft_baseline_destroy(sffft_baseline_t bl);

/* Debug: one tcgen05.mma through the fused kernel's layout writers and descriptors (no reference
 * counterpart).  a_kind: 0 = MN-major 128-B swizzle, 32/64/128 = K-major row pitch; A: 128x16 halves,
 * B: n x 16 halves (B[n][k]), D: 128 x n raw TMEM words. */
int sffft_debug_umma_probe(int a_kind, int a_slice, int b_pitch, int b_slice, int n, int acc16,
                           const unsigned short* A, const unsigned short* B, unsigned int* D);

/* Allocation-free convolution, for callers that cannot allocate device memory while they run (an
 * inference-engine plugin whose execute step must not allocate, a process whose device memory is all
 * reserved by another allocator).  No counterpart in the reference.  The caller passes u [B][H][L], the
 * real filter k [H][L] (k_dtype fp32 or bf16) and y; the filter spectrum and a status word live in a fixed
 * array inside the library (16 MiB of spectrum, i.e. H * 2L * 8 bytes <= 16 MiB, plus 256 bytes), which
 * every GPU that loads the library holds until the process exits.  Larger problems return
 * SFFFT_ERR_SCRATCH_LIMIT without launching anything.  Uses the built-in plan for L with DFT matrices built
 * in-kernel; results equal sffft_filter_spectrum + sffft_conv on a "legacy" plan.  The first call on a
 * device sets up that device (looks up the array's device address, sets kernel attributes); make it
 * before any stream capture.  All calls on a device share the array, so calls whose work overlaps on the
 * GPU race.  sync != 0 waits for the stream and returns the kernel's device-side status; with sync == 0 the
 * call returns once the work is queued and a device-side error of that call (a barrier timeout) is not
 * reported, since the next call on the device clears the status word before it launches. */
int sffft_conv_noalloc(int L, int io, int acc, const void* u, const void* k, int k_dtype, void* y, int B, int H,
                       void* stream, int sync);

/* Host-buffer pipeline (no reference counterpart: the reference keeps u and y on the device and times the
 * kernel alone).  sffft_pipe_create sizes device staging for a B x H batch cut into about `chunks` chunks
 * (0 = 4) of whole batch-row pairs (contiguous, one copy each way), or of pairs and channel ranges when B/2
 * is smaller than `chunks`, and creates one stream per stage (upload, convolution, download) with three
 * staging slots; sffft_conv_host then computes y_host = causal_conv(u_host, k) for host buffers u_host,
 * y_host [B][H][L] (the plan's I/O type; pinned for overlap) and the device spectrum Kf [H][N]: chunk i goes
 * through slot i % 3, so uploads, kernels and downloads of different chunks overlap.  Ordered after earlier work on `stream`; later work on
 * `stream` waits for it.  Calls on one pipe must not overlap. */
typedef struct sffft_pipe* sffft_pipe_t;
int sffft_pipe_create(sffft_pipe_t* pipe, sffft_plan_t plan, int B, int H, int chunks);
int sffft_conv_host(sffft_pipe_t pipe, const void* u_host, const void* Kf, void* y_host, void* stream);
int sffft_pipe_destroy(sffft_pipe_t pipe);

/* Channel-sharded convolution over several devices.  No reference counterpart: the reference runs on device 0
 * only (src/sffft.cu:490).  Shard g of G owns channels [h0, h1) = sffft_shard_range(H, G, g) and runs on the
 * device of plans[g] (plans share L and the I/O type; one device may hold several shards).
 *   sffft_conv_multi: device-resident shards, asynchronous: u[g], y[g] are [B][h1 - h0][L] and Kf[g] is
 *     [h1 - h0][N] on plans[g]'s device; one sffft_conv per shard on streams[g] (NULL: default streams).
 *   sffft_multi_pipe_create / sffft_conv_host_multi: one [B][H][L] batch in host memory (pinned for overlap);
 *     every device uploads its channel slice, convolves it with its spectrum rows Kf[g] ([h1 - h0][N] on that
 *     device) and downloads its slice of y_host, all devices concurrently, each through a host pipe of its own
 *     (as sffft_pipe_create with `chunks`) driven by a host thread of its own (started by
 *     sffft_multi_pipe_create, joined by sffft_multi_pipe_destroy); the call returns when every device has
 *     finished, with the first error or device-side status (SFFFT_ERR_TIMEOUT) of any shard.  Composite plans
 *     in sffft_conv_multi use the workspace attached to each plan (sffft_plan_set_workspace); the pipes
 *     allocate their own. */
int sffft_conv_multi(const sffft_plan_t* plans, int G, const void* const* u, const void* const* Kf, void* const* y,
                     int B, int H, void* const* streams);
typedef struct sffft_multi* sffft_multi_t;
int sffft_multi_pipe_create(sffft_multi_t* multi, const sffft_plan_t* plans, int G, int B, int H, int chunks);
int sffft_conv_host_multi(sffft_multi_t multi, const void* u_host, const void* const* Kf, void* y_host);
int sffft_multi_pipe_destroy(sffft_multi_t multi);

/* Debug: a kernel waits on a barrier that nothing arrives at, using the same bounded wait as the fused
 * kernel; returns SFFFT_ERR_TIMEOUT after about limit_us microseconds (1..1e6) with the context intact.
 * No reference counterpart (the reference has no device-side timeouts). */
int sffft_debug_wait_timeout(int limit_us);

/* Debug: sffft_conv with every barrier wait of the fused kernel limited to limit_us microseconds (1..1e6) and
 * one arrival withheld (the first warp of the team that converts the first group skips its arrival on the
 * "operand ready" barrier), so the stage-0 MMAs are never issued and the bounded waits run out: the kernel's
 * roles see the abort flag, wait for their MMAs in flight, free TMEM and return; sffft_plan_check then reports
 * SFFFT_ERR_TIMEOUT and the context stays usable.  Exercises the fused kernel's failure path without a fault.
 * No reference counterpart (the reference fails fast on host errors only, src/sffft.cu:22-23). */
int sffft_debug_conv_timeout(sffft_plan_t plan, const void* u, const void* Kf, void* y, int B, int H, int limit_us,
                             void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SFFFT_H_ */
