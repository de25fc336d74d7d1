/*
 * mtorch_cuda.h — C ABI of the B200 (sm_100a) kernel library behind mtorch's `cuda` device.
 *
 * Every entry point takes plain device pointers, sizes, strides (in ELEMENTS) and a
 * `cudaStream_t` passed as `void*` (NULL = legacy default stream).  No C++ or torch types cross
 * this boundary; the library never allocates device memory on its own behalf: scratch space is
 * passed in by the caller as a workspace whose size is reported by a `*_workspace_size` query.
 * Each function returns MT_OK (0) or an `mt_status` code; `mt_cuda_last_error_string()` gives a
 * human-readable reason for the last failure on the calling thread.
 *
 * The functions replace, one for one, the portable CPU op functions of the reference core
 * (cpp/mtorch/core/tensor.h); the citation above each declaration names the function whose
 * result the device path reproduces.  The CPython layer (the reference's
 * cpp/mtorch/python/module.cpp, or this repository's mtorch_b200 package) keeps argument
 * parsing, broadcasting rules, dtype promotion and error translation; these kernels receive
 * already-validated descriptors.
 */
#ifndef MTORCH_CUDA_H_
#define MTORCH_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status, dtypes -------------------------------------------------------------------- */
typedef enum {
  MT_OK = 0,
  MT_ERR_INVALID = 1,     /* bad argument (shape, stride, alignment, null pointer)          */
  MT_ERR_UNSUPPORTED = 2, /* valid request the device path does not implement: caller raises */
  MT_ERR_LAUNCH = 3,      /* CUDA launch / runtime error                                     */
  MT_ERR_TIMEOUT = 4,     /* a bounded device-side wait expired (kernel returned early)      */
  MT_ERR_WORKSPACE = 5    /* workspace missing or smaller than the *_workspace_size query    */
} mt_status;

/* Element types.  The reference's ScalarType (tensor.h:13-20) has no bfloat16; the device path
 * adds it (MT_BF16) as a storage/compute type for the Stable-Diffusion configurations. */
typedef enum { MT_F32 = 0, MT_BF16 = 1, MT_F16 = 2, MT_F64 = 3, MT_I32 = 4, MT_I64 = 5, MT_BOOL = 6 } mt_dtype;

/* Maximum tensor rank handled by the strided elementwise kernels. */
#define MT_MAX_DIMS 8

const char* mt_cuda_last_error_string(void);
/* Number of visible devices (0 when there is no driver / GPU). */
int mt_cuda_device_count(void);
/* Replaces the reference's device check `require_cpu_device` (tensor.cpp:231-239): makes
 * `device` current on the calling thread and verifies it is an sm_100 part. */
int mt_cuda_set_device(int device);
int mt_cuda_synchronize(void* stream);
/* Device-side error word written by bounded waits inside kernels (MT_ERR_TIMEOUT); `clear`
 * resets it.  Returns MT_OK when no kernel reported a problem. */
int mt_cuda_device_status(int clear);
/* Failure-detection self test (no counterpart in the reference, which has no device): launches
 * one kernel whose bounded mbarrier wait can never complete; after `budget_cycles` SM clocks it
 * gives up, records MT_ERR_TIMEOUT in the device status word and returns, so that the next
 * mt_cuda_device_status reports the timeout while the context stays usable. */
int mt_cuda_selftest_wait_timeout(long long budget_cycles, void* stream);
/* Number of kernels this library has launched in the process (all devices); instrumentation for
 * benchmarks (no counterpart in the reference, which has no device). */
uint64_t mt_cuda_launch_count(void);

/* ---- memory movement: replaces `to` (tensor.cpp:8479-8505) and `contiguous` (tensor.cpp:8210) */
/* kind: 0 = host->device, 1 = device->host, 2 = device->device. */
int mt_cuda_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream);
int mt_cuda_memset(void* dst, int value, size_t bytes, void* stream);

/* ---- device runtime: storage, streams, events, graphs, NCCL ------------------------------ */
/* The reference keeps tensor bytes in a host `Storage` (cpp/mtorch/core/tensor.h:60-63, a
 * shared `std::vector<uint8_t>`) allocated by `Storage(size_t)`; the device counterpart is this
 * caching allocator.  mt_cuda_malloc serves a block on the CURRENT device (mt_cuda_set_device)
 * from the device's free list or cudaMalloc; mt_cuda_free returns it to the free list.  Blocks
 * are reused in stream order: issue all of a device's work on one stream (mt_cuda_library_stream)
 * or synchronise before freeing a block another stream still reads.  While a graph capture is
 * open on a device (mt_cuda_graph_begin), allocations come from a pool private to that graph
 * that lives until mt_cuda_graph_destroy.  On out-of-memory the cached blocks are released and
 * the allocation retried once. */
int mt_cuda_malloc(void** ptr, size_t bytes);
int mt_cuda_free(void* ptr);
/* Bytes handed out and bytes held in free lists on `device`. */
int mt_cuda_memory_stats(int device, size_t* in_use, size_t* cached);
/* Releases the current device's cached free blocks (synchronises the device). */
int mt_cuda_empty_cache(void);
/* Page-locked host memory for asynchronous host<->device copies. */
int mt_cuda_host_alloc(void** ptr, size_t bytes);
int mt_cuda_host_free(void* ptr);
/* Streams: mt_cuda_library_stream returns the device's own non-blocking stream (created on
 * first request, lives until exit) on which the host layer issues all of that device's work. */
int mt_cuda_stream_create(void** stream);
int mt_cuda_stream_destroy(void* stream);
int mt_cuda_library_stream(int device, void** stream);
/* Timing events (cudaEvent_t as void*). */
int mt_cuda_event_create(void** event);
int mt_cuda_event_destroy(void* event);
int mt_cuda_event_record(void* event, void* stream);
int mt_cuda_event_synchronize(void* event);
int mt_cuda_event_elapsed_ms(void* start, void* end, float* ms);
/* CUDA-graph capture of the work issued on `stream` (thread-local capture mode) between begin
 * and end; end instantiates it and returns an opaque graph handle for launch / destroy.  The
 * graph's private allocation pool is released by destroy (blocks still held by the caller are
 * released when they are freed). */
int mt_cuda_graph_begin(void* stream);
int mt_cuda_graph_end(void* stream, void** graph);
int mt_cuda_graph_launch(void* graph, void* stream);
int mt_cuda_graph_destroy(void* graph);
/* NCCL over NVLink for the batch-sharded job (no counterpart in the single-process reference):
 * libnccl.so.2 is loaded on first use.  The unique id (128 bytes) is made on one rank and
 * handed to the others by the host layer; all_gather concatenates `bytes_per_rank` bytes from
 * every rank in rank order into `recv`. */
int mt_nccl_available(void);
int mt_nccl_unique_id(void* id, size_t bytes);
int mt_nccl_comm_init(void** comm, const void* id, size_t bytes, int world, int rank);
int mt_nccl_all_gather(const void* send, void* recv, size_t bytes_per_rank, void* comm, void* stream);
int mt_nccl_comm_destroy(void* comm);
/* Strided copy with dtype conversion (f32/bf16/f16/f64 <-> each other):
 * dst[i0..] = cast(src[i0..]) over `ndim` dims of `sizes`, each side with its own strides. */
int mt_cuda_copy_strided(void* dst, int dst_dtype, const int64_t* dst_strides, const void* src, int src_dtype,
                         const int64_t* src_strides, const int64_t* sizes, int ndim, void* stream);
/* Device counterpart of mtorch's uniform_ for contiguous tensors (module.cpp:335-365 with
 * next_random_u64 / next_uniform_open at module.cpp:76-88): element i receives the (i+1)-th draw
 * of SplitMix64 after `state`, so results are bit-identical to the host generator.  The caller
 * advances its host state by `n` draws afterwards. */
int mt_cuda_fill_uniform(void* dst, int dtype, int64_t n, uint64_t state, double from, double to, void* stream);
int mt_cuda_fill(void* dst, int dtype, int64_t n, double value, void* stream);

/* ---- elementwise ------------------------------------------------------------------------- */
typedef enum { MT_UNARY_SILU = 0, MT_UNARY_GELU = 1, MT_UNARY_GELU_TANH = 2, MT_UNARY_NEG = 3,
               MT_UNARY_EXP = 4, MT_UNARY_SIGMOID = 5, MT_UNARY_RELU = 6,
               MT_UNARY_QUICK_GELU = 7 } mt_unary_op;
/* Replaces `silu` (tensor.cpp:16480-16600) and `gelu` (tensor.cpp:17207-17290); QUICK_GELU is
 * CLIP's x * sigmoid(1.702 x) (the reference composes it, tests/compat/benchmarking.py:7714).  Contiguous,
 * n elements; x and y may alias; dtypes may differ (compute in fp32). */
int mt_cuda_unary(int op, void* y, int y_dtype, const void* x, int x_dtype, int64_t n, void* stream);

typedef enum { MT_BIN_ADD = 0, MT_BIN_SUB = 1, MT_BIN_MUL = 2, MT_BIN_DIV = 3 } mt_binary_op;
/* Replaces `binary_tensor_tensor` (tensor.cpp:18965-19104): y = a OP b over the broadcast shape
 * `sizes` (ndim <= MT_MAX_DIMS); each operand gives its strides for that shape (0 on broadcast
 * dims).  `b` may be NULL, in which case `scalar` is the right operand (binary_tensor_scalar,
 * tensor.cpp:19106).  Output is written with `y_strides`. */
int mt_cuda_binary(int op, void* y, int y_dtype, const int64_t* y_strides, const void* a, int a_dtype,
                   const int64_t* a_strides, const void* b, int b_dtype, const int64_t* b_strides, double scalar,
                   const int64_t* sizes, int ndim, void* stream);
/* Fused a*x + b*y + c*z (y, z may be NULL) over contiguous n elements, fp32 math: the DDIM latent
 * update of the reference's scheduler scenario (tests/compat/benchmarking.py:6148-6168). */
int mt_cuda_axpby(void* out, int out_dtype, const void* x, int x_dtype, double a, const void* y, int y_dtype,
                  double b, const void* z, int z_dtype, double c, int64_t n, void* stream);
/* One DDIM update of n latents, fp32 math, as the reference's scheduler step
 * (tests/compat/benchmarking.py:6148-6168): x0 = (x - sqrt(1-a_t) eps) / sqrt(a_t), clamped to
 * [-1, 1] when clip != 0; eps' = (x - sqrt(a_t) x0) / sqrt(1-a_t);
 * out = sqrt(a_prev) x0 + sqrt(1-a_prev) eps'.  out may alias x. */
int mt_cuda_ddim_step(void* out, const void* x, const void* eps, int dtype, int eps_dtype, int64_t n, double alpha_t,
                      double alpha_prev, int clip, void* stream);

/* The same DDIM update with the timestep read from device memory, so that one captured CUDA graph
 * serves every step of the loop, and with classifier-free guidance folded in
 * (tests/compat/benchmarking.py:5847-5850 for the guidance, 6148-6168 for the step):
 *   t = *timestep (clamped to [0, num_train_steps)), t_prev = max(t - interval, 0),
 *   a_t = alphas_cumprod[t], a_prev = alphas_cumprod[t_prev] (fp64 table on the device);
 *   cfg != 0: eps holds 2n values [uncond; text] and the noise used is
 *   uncond + (text - uncond) * guidance_scale (fp32, in that order); cfg == 0: eps holds n values.
 * The result is written to out[c*n + i] for c < out_copies (1 or 2): with 2 the next step's
 * batch-doubled model input [x; x] is produced in the same pass.  out may alias x. */
int mt_cuda_ddim_step_indexed(void* out, int64_t out_copies, const void* x, const void* eps, int dtype, int eps_dtype,
                              int64_t n, const double* alphas_cumprod, int64_t num_train_steps,
                              const int64_t* timestep, int64_t interval, int cfg, double guidance_scale, int clip,
                              void* stream);
/* Sinusoidal timestep embedding [n, dim] of the reference's scenario
 * (tests/compat/benchmarking.py:6011-6036): freq_j = exp((-ln(max_period) * j) / (dim/2)),
 * arg = t * freq_j, row = [cos | sin] (flip_sin_to_cos != 0, SD's layout) or [sin | cos]; fp32
 * math.  Row r reads timesteps[r * t_stride] (f32, f64, f16, bf16 or i64; stride 0 broadcasts one
 * device scalar).  dim must be even. */
int mt_cuda_timestep_embedding(void* out, int out_dtype, const void* timesteps, int t_dtype, int64_t t_stride,
                               int64_t n, int64_t dim, double max_period, int flip_sin_to_cos, void* stream);

/* Replaces `embedding` (tensor.cpp:31748-31800) for a contiguous [rows, dim] table and n int64 ids:
 * out[r, :] = weight[ids[r], :], negative ids counted from the end.  With `add` (a second table
 * [add_rows, dim] and its ids, e.g. CLIP's position embedding) the two rows are summed in fp32 and
 * rounded once.  An out-of-range id writes a zero row and increments *invalid_count (device int,
 * may be NULL): the caller raises the reference's IndexError when it is non-zero. */
int mt_cuda_embedding(void* out, int out_dtype, const void* weight, int w_dtype, int64_t rows, int64_t dim,
                      const int64_t* ids, int64_t n, const void* add, int add_dtype, int64_t add_rows,
                      const int64_t* add_ids, int* invalid_count, void* stream);

/* ---- normalisation / softmax ------------------------------------------------------------- */
/* Replaces `softmax` (tensor.cpp:15145-15213, fp32 kernel 7508-7742) along the innermost,
 * contiguous dimension: rows x cols, row pitch `ld` (elements). */
int mt_cuda_softmax(void* y, int y_dtype, const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ld,
                    int log_output, void* stream);
/* Replaces `layer_norm` (tensor.cpp:17386-17714) over the last `cols` elements of each row
 * (weight/bias optional, length cols). */
int mt_cuda_layer_norm(void* y, int y_dtype, const void* x, int x_dtype, const void* weight, const void* bias,
                       int wb_dtype, int64_t rows, int64_t cols, double eps, void* stream);
/* Replaces `group_norm` (tensor.cpp:18643-18963).  Input is [N, C, HW] with element strides
 * (sn, sc, shw) — NCHW contiguous is (C*HW, HW, 1), channels-last is (HW*C, 1, C); output uses
 * its own strides.  `fuse_silu` applies x*sigmoid(x) after the affine (the SD ResNet pattern
 * GroupNorm -> SiLU).  Workspace: mt_cuda_group_norm_workspace_size(). */
size_t mt_cuda_group_norm_workspace_size(int64_t N, int64_t C, int64_t HW, int64_t groups);
int mt_cuda_group_norm(void* y, int y_dtype, const int64_t* y_strides, const void* x, int x_dtype,
                       const int64_t* x_strides, const void* weight, const void* bias, int wb_dtype, int64_t N,
                       int64_t C, int64_t HW, int64_t groups, double eps, int fuse_silu, void* workspace,
                       size_t workspace_bytes, void* stream);
/* Group norm of the channel concatenation [x1 | x2] without forming it (the SD up-block skip
 * connection, `cat(dim=1)` tensor.cpp:32141 followed by `group_norm`): the result equals
 * mt_cuda_group_norm on the concatenated [N, C, HW] input.  bf16 only; x1 ([N, C1, HW]) and x2
 * ([N, C - C1, HW]) dense channels-last with C1 and C - C1 multiples of 8, y dense channels-last
 * [N, C, HW]; other layouts return MT_ERR_UNSUPPORTED (concatenate and call mt_cuda_group_norm).
 * Workspace: mt_cuda_group_norm_workspace_size(N, C, HW, groups). */
int mt_cuda_group_norm_cat(void* y, int y_dtype, const int64_t* y_strides, const void* x1, const int64_t* x1_strides,
                           int64_t C1, const void* x2, const int64_t* x2_strides, int x_dtype, const void* weight,
                           const void* bias, int wb_dtype, int64_t N, int64_t C, int64_t HW, int64_t groups, double eps,
                           int fuse_silu, void* workspace, size_t workspace_bytes, void* stream);

/* Group norm for callers that cannot hand the library a workspace — for example code running
 * inside a host callback, a custom allocator hook, or an embedding runtime that owns every
 * device allocation and forbids cudaMalloc / cudaFree on its threads.  Same arguments and result
 * as mt_cuda_group_norm minus the workspace; the statistics scratch lives in a fixed array
 * inside this library (MT_GROUP_NORM_STATIC_SCRATCH_BYTES per GPU, held until process exit).
 * Requests needing more scratch than that (about N * ceil(HW/64) * groups > 500000 for
 * channels-last input, 16 bytes each) are rejected with MT_ERR_INVALID.  The first call on each device looks up
 * the array's device address and should therefore come before any stream capture.  All calls
 * share the one array: calls that may overlap on the GPU (different streams, or different host
 * threads) race and must be serialised by the caller.  No counterpart in the reference. */
#define MT_GROUP_NORM_STATIC_SCRATCH_BYTES (8u << 20)
int mt_cuda_group_norm_noalloc(void* y, int y_dtype, const int64_t* y_strides, const void* x, int x_dtype,
                               const int64_t* x_strides, const void* weight, const void* bias, int wb_dtype, int64_t N,
                               int64_t C, int64_t HW, int64_t groups, double eps, int fuse_silu, void* stream);

/* ---- dense contractions on tcgen05 / TMEM ---------------------------------------------- */
typedef enum {
  MT_EPI_NONE = 0,
  MT_EPI_GELU = 1,  /* y = gelu(acc + bias)                                                       */
  MT_EPI_SILU = 2,  /* y = silu(acc + bias)                                                       */
  MT_EPI_GEGLU = 3, /* B columns come in (64 value, 64 gate) groups: y[:, j] = v_j * gelu(g_j), N/2 */
  MT_EPI_QUICK_GELU = 4 /* y = z * sigmoid(1.702 z), z = acc + bias (CLIP's MLP activation)           */
} mt_epilogue;

/*
 * D[b] = alpha * op(A[b]) @ op(B[b]) + beta * C[b] + bias  (then activation, then + residual)
 *
 * Replaces `matmul` (tensor.cpp:24896-25064), `bmm` (25066-25182), `addmm` (25184-25366),
 * `baddbmm` (25557-25694) and `linear` (31401-31694).  A is M x K, B is K x N (logical).
 *   a_trans = 0: A stored row-major [M, K] with row pitch lda;  1: stored [K, M] (pitch lda).
 *   b_trans = 0: B stored row-major [K, N] (pitch ldb, the matmul case);
 *             1: stored [N, K] (pitch ldb, the linear-weight case, y = x @ W^T).
 * Batched operands step by stride_* elements per batch (0 broadcasts).  bias is length N
 * (bias_batch_stride 0) or [batch, N] (stride N).  residual (optional) is [M, N] per batch with
 * pitch ldr.  dtype: MT_BF16/MT_F16 run kind::f16 with fp32 accumulation; MT_F32 runs three
 * tf32 tensor-core products (hi*hi + hi*lo + lo*hi, "3xTF32") for ~fp32 accuracy.
 * Workspace: mt_cuda_gemm_workspace_size(desc).
 */
typedef struct {
  int64_t M, N, K, batch;
  int dtype;      /* input dtype of A and B                                                 */
  int out_dtype;  /* dtype of D (and C / residual)                                          */
  const void* A; int64_t lda, stride_a; int a_trans;
  const void* B; int64_t ldb, stride_b; int b_trans;
  void* D; int64_t ldd, stride_d;
  const void* C; int64_t ldc, stride_c; /* used when beta != 0                             */
  const void* bias; int bias_dtype; int64_t bias_batch_stride;
  const void* residual; int64_t ldr, stride_r;
  float alpha, beta;
  int epilogue;   /* mt_epilogue */
  /* MT_F32 only, optional: precomputed low parts (x - tf32_truncate(x)) of A ([M, Kp] per batch)
   * and B ([N, Kp] per batch), Kp = K rounded up to a multiple of 4, e.g. cached for a constant
   * weight.  NULL = computed into the workspace on every call. */
  const void* A_lo; const void* B_lo;
} mt_gemm_desc;
size_t mt_cuda_gemm_workspace_size(const mt_gemm_desc* desc);
int mt_cuda_gemm(const mt_gemm_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/*
 * 2-D convolution.  Replaces `conv2d` (tensor.cpp:26490-27528; portable loop 27359-27400).
 * x is [N, C, H, W] given by element strides (NCHW or channels-last), weight is [K, C, R, S]
 * (torch layout, contiguous) or pre-packed, output [N, K, P, Q] with its own strides.  bias:
 * length K, or [N, K] when bias_batch_stride == K (per-sample bias: the SD ResNet time-embedding
 * add).  residual (optional) has the output's shape and `res_strides`.  groups > 1 is
 * MT_ERR_UNSUPPORTED.  Stride-1 convolutions with C % 64 == 0 (bf16/f16) or C % 32 == 0 (fp32)
 * run as implicit GEMM (4-D TMA boxes over channels-last activations, zero padding from TMA
 * out-of-bounds fill); others go through an explicit im2col gather + the same GEMM.
 */
typedef struct {
  int64_t N, C, H, W, K, R, S, P, Q;
  int stride_h, stride_w, pad_h, pad_w, dil_h, dil_w, groups;
  int dtype, out_dtype;
  const void* x; int64_t x_strides[4];
  const void* w;
  /* w_packed = 1: `w` is already [K, R, S, Cp] contiguous (Cp = mt_cuda_conv2d_packed_channels)
   * from mt_cuda_conv2d_pack_weight and, for MT_F32, `w_lo` its tf32 low part (or NULL). */
  int w_packed; const void* w_lo;
  const void* bias; int bias_dtype; int64_t bias_batch_stride;
  const void* residual; int64_t res_strides[4];
  void* y; int64_t y_strides[4];
  int epilogue;
} mt_conv2d_desc;
size_t mt_cuda_conv2d_workspace_size(const mt_conv2d_desc* desc);
int mt_cuda_conv2d(const mt_conv2d_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
/* Convolution of the channel concatenation [x | x2] without forming it (`cat(dim=1)`
 * tensor.cpp:32141 followed by `conv2d`; the SD up-block's 1x1 shortcut): desc->x / x_strides
 * describe the first source with C1 channels, desc->C is the total, x2 / x2_strides the second
 * source (element strides n, c, h, w).  16-bit implicit-GEMM convolutions only, both sources
 * dense channels-last and 16-byte aligned, C1 and C - C1 multiples of 64 (bf16/f16); otherwise
 * MT_ERR_UNSUPPORTED.  Workspace: mt_cuda_conv2d_cat_workspace_size. */
size_t mt_cuda_conv2d_cat_workspace_size(const mt_conv2d_desc* desc, const void* x2, const int64_t* x2_strides,
                                         int64_t C1);
int mt_cuda_conv2d_cat(const mt_conv2d_desc* desc, const void* x2, const int64_t* x2_strides, int64_t C1,
                       void* workspace, size_t workspace_bytes, void* stream);
/* Repacks a torch-layout weight [K, C, R, S] into [K, R, S, Cp] (Cp = C rounded up to a 16-byte
 * multiple) and, for MT_F32 with w_lo != NULL, writes the tf32 low part beside it.  Used once
 * per weight version by the module layer. */
int64_t mt_cuda_conv2d_packed_channels(int64_t C, int64_t R, int64_t S, int dtype);
int mt_cuda_conv2d_pack_weight(void* w_packed, void* w_lo, const void* w, int dtype, int64_t K, int64_t C,
                               int64_t R, int64_t S, void* stream);

/*
 * 3x3 convolution (stride 1, padding 1, dilation 1) of the nearest-2x upsample of x, without
 * forming the upsampled tensor.  Replaces the up-block pair `interpolate(scale_factor=2,
 * mode="nearest")` (tensor.cpp:10897) + `conv2d` (tensor.cpp:26490-27528) of the SD UNet
 * (scenario benchmarking.py:5981-6000).  The descriptor is the convolution's own: x [N, C, H, W]
 * at the SOURCE resolution, weight [K, C, 3, 3], R = S = 3, pad 1, stride 1, P = 2H, Q = 2W,
 * output [N, K, 2H, 2W] channels-last with 16-byte aligned rows.  Each output parity (2i+a, 2j+b)
 * is a 2x2 convolution of the source with taps summed from the 3x3 taps, so the work is 16/36
 * of the upsample-then-convolve FLOPs.  Needs C to fill whole 128-byte chunks (C % 64 == 0 for
 * bf16/f16, C % 32 == 0 for fp32); other cases return MT_ERR_UNSUPPORTED (the caller upsamples
 * and convolves instead).  w_packed = 1: `w` holds mt_cuda_conv2d_up2x_packed_elems elements
 * from mt_cuda_conv2d_up2x_pack_weight ([4 parities][K][2][2][Cp]), w_lo its tf32 low parts
 * (MT_F32) or NULL.
 */
size_t mt_cuda_conv2d_up2x_workspace_size(const mt_conv2d_desc* desc);
int mt_cuda_conv2d_up2x(const mt_conv2d_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
int64_t mt_cuda_conv2d_up2x_packed_elems(int64_t K, int64_t C, int dtype);
int mt_cuda_conv2d_up2x_pack_weight(void* w_packed, void* w_lo, const void* w, int dtype, int64_t K, int64_t C,
                                    void* stream);

/*
 * Fused attention O = softmax(Q K^T * scale + mask) V.  Replaces
 * `scaled_dot_product_attention` (tensor.cpp:30930-31324; portable loop 31158-31207).
 * Q [B, H, Sq, D], K [B, Hkv, Sk, D], V [B, Hkv, Sk, Dv], O [B, H, Sq, Dv], each with element
 * strides (b, h, s, d); H % Hkv == 0 (grouped-query attention, enable_gqa).  mask_kind 0 = none,
 * 1 = bool (nonzero keeps, uint8 storage), 2 = additive float in `mask_dtype`; the mask is indexed
 * with `mask_strides` over (b, h, q, k), zeros for broadcast dims.  causal masks key > query.
 * bf16/f16 run a flash-style tcgen05 kernel (fp32 online softmax) where the shape allows; f32
 * and the remaining cases run an fp32 SIMT flash kernel.  Workspace: mt_cuda_sdpa_workspace_size.
 */
typedef struct {
  int64_t B, H, Hkv, Sq, Sk, D, Dv;
  int dtype;
  const void* q; int64_t q_strides[4];
  const void* k; int64_t k_strides[4];
  const void* v; int64_t v_strides[4];
  void* o; int64_t o_strides[4];
  const void* mask; int mask_kind; int mask_dtype; int64_t mask_strides[4];
  int causal;
  double scale;
} mt_sdpa_desc;
size_t mt_cuda_sdpa_workspace_size(const mt_sdpa_desc* desc);
int mt_cuda_sdpa(const mt_sdpa_desc* desc, void* workspace, size_t workspace_bytes, void* stream);
/* Which kernel mt_cuda_sdpa runs for `desc` (no counterpart in the reference, whose SDPA has one
 * CPU path): the tcgen05 kernel with the output kept in TMEM (head dims 33-48, more than 128
 * queries, no mask or causal), the general tcgen05 kernel (16-bit types, head dims that are
 * multiples of 8 up to 160, padded to 32/48/64/80/128/160; bool or f32/bf16/f16 additive masks,
 * causal, positive scale), the short-key tcgen05 kernel (at most 128 keys, head dims up to 128,
 * no mask or causal: K and V loaded once per CTA for several query tiles), or the fp32 SIMT
 * kernel (fp32, other head dims, scales or strides).  Returns 0 for an invalid descriptor. */
#define MT_SDPA_PATH_TC_LAZY 1
#define MT_SDPA_PATH_TC 2
#define MT_SDPA_PATH_SIMT 3
#define MT_SDPA_PATH_TC_SHORT 4
int mt_cuda_sdpa_path(const mt_sdpa_desc* desc);

/* ---- host random generator: the reference's RandomState (module.cpp:47-183) ------------- */
/* SplitMix64 + Marsaglia-polar normal with the odd-count "spare" rule, bit-identical to
 * mtorch.manual_seed / randn / normal_ / uniform_ on contiguous float tensors.  The state is a
 * caller-owned struct so Python can keep mtorch's single global generator. */
typedef struct {
  uint64_t state;
  int32_t has_spare;
  double spare;
} mt_rng_state;
void mt_rng_seed(mt_rng_state* rng, uint64_t seed);
/* dtype MT_F32 or MT_F64 host buffer, n contiguous elements, value = mean + std * N(0,1). */
void mt_rng_fill_normal(mt_rng_state* rng, void* dst, int dtype, int64_t n, double mean, double std);
void mt_rng_fill_uniform(mt_rng_state* rng, void* dst, int dtype, int64_t n, double from, double to);

#ifdef __cplusplus
}
#endif
#endif /* MTORCH_CUDA_H_ */
