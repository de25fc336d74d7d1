// The extern "C" boundary (include/mtorch_cuda.h): argument checks, error strings, device
// management, TMA tensor-map encoding, and the host random generator.
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cudaTypedefs.h>

#include "runtime.h"

namespace mt {

static thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MT_OK;
  return fail(MT_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

static std::atomic<uint64_t> g_launches{0};

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cuda_check(cudaGetLastError(), what);
}

struct DevProps {
  int sms = 0;
  int major = 0, minor = 0;
};
static DevProps g_props[64];
static std::once_flag g_props_once[64];

static const DevProps& props() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  std::call_once(g_props_once[dev], [dev] {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) {
      g_props[dev].sms = p.multiProcessorCount;
      g_props[dev].major = p.major;
      g_props[dev].minor = p.minor;
    }
  });
  return g_props[dev];
}
int num_sms() { return props().sms > 0 ? props().sms : 148; }

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tensor_map(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle, const uint32_t* elem_strides) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(MT_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  CUtensorMapDataType t;
  switch (dtype) {
    case MT_F32: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case MT_BF16: t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case MT_F16: t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    default: return fail(MT_ERR_UNSUPPORTED, "tensor map: dtype %d", dtype);
  }
  if ((uintptr_t)base % 16 != 0) return fail(MT_ERR_INVALID, "tensor map: base address not 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0) return fail(MT_ERR_INVALID, "tensor map: stride not a multiple of 16 bytes");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  if (elem_strides)
    for (int i = 0; i < rank; ++i) {
      if (elem_strides[i] < 1 || elem_strides[i] > 8) return fail(MT_ERR_INVALID, "tensor map: element stride out of range");
      estr[i] = elem_strides[i];
    }
  const CUtensorMapSwizzle sw = swizzle == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = g_encode(map, t, (cuuint32_t)rank, const_cast<void*>(base), (const cuuint64_t*)dims,
                        (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MT_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MT_OK;
}

}  // namespace mt

using namespace mt;

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

const char* mt_cuda_last_error_string(void) { return t_last_error.c_str(); }

int mt_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int mt_cuda_set_device(int device) {
  int rc = cuda_check(cudaSetDevice(device), "cudaSetDevice");
  if (rc) return rc;
  const DevProps& p = props();
  if (p.major != 10)
    return fail(MT_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device, p.major,
                p.minor);
  return MT_OK;
}

int mt_cuda_synchronize(void* stream) {
  if (stream) return cuda_check(cudaStreamSynchronize(S(stream)), "cudaStreamSynchronize");
  return cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
}

int mt_cuda_device_status(int clear) {
  const int vals[3] = {read_status_gemm(clear), read_status_attention(clear), read_status_norm(clear)};
  for (int v : vals) {
    if (v < 0) return fail(MT_ERR_LAUNCH, "could not read the device status word");
    if (v) return fail(v & 0xff, "a device-side wait expired (site %d)", v >> 8);
  }
  return MT_OK;
}

int mt_cuda_selftest_wait_timeout(long long budget_cycles, void* stream) {
  return run_wait_timeout_selftest(budget_cycles, S(stream));
}

uint64_t mt_cuda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int mt_cuda_memcpy(void* dst, const void* src, size_t bytes, int kind, void* stream) {
  if (bytes == 0) return MT_OK;
  if (!dst || !src) return fail(MT_ERR_INVALID, "memcpy: null pointer");
  cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  return cuda_check(cudaMemcpyAsync(dst, src, bytes, k, S(stream)), "cudaMemcpyAsync");
}

int mt_cuda_memset(void* dst, int value, size_t bytes, void* stream) {
  if (bytes == 0) return MT_OK;
  return cuda_check(cudaMemsetAsync(dst, value, bytes, S(stream)), "cudaMemsetAsync");
}

int mt_cuda_copy_strided(void* dst, int dst_dtype, const int64_t* dst_strides, const void* src, int src_dtype,
                         const int64_t* src_strides, const int64_t* sizes, int ndim, void* stream) {
  if (ndim > 0 && (!dst_strides || !src_strides || !sizes)) return fail(MT_ERR_INVALID, "copy_strided: null argument");
  return launch_copy_strided(dst, dst_dtype, dst_strides, src, src_dtype, src_strides, sizes, ndim, S(stream));
}

int mt_cuda_fill_uniform(void* dst, int dtype, int64_t n, uint64_t state, double from, double to, void* stream) {
  return launch_fill_uniform(dst, dtype, n, state, from, to, S(stream));
}
int mt_cuda_fill(void* dst, int dtype, int64_t n, double value, void* stream) {
  return launch_fill(dst, dtype, n, value, S(stream));
}

int mt_cuda_unary(int op, void* y, int y_dtype, const void* x, int x_dtype, int64_t n, void* stream) {
  if (op < MT_UNARY_SILU || op > MT_UNARY_QUICK_GELU) return fail(MT_ERR_UNSUPPORTED, "unary: op %d", op);
  return launch_unary(op, y, y_dtype, x, x_dtype, n, S(stream));
}

int mt_cuda_binary(int op, void* y, int y_dtype, const int64_t* y_strides, const void* a, int a_dtype,
                   const int64_t* a_strides, const void* b, int b_dtype, const int64_t* b_strides, double scalar,
                   const int64_t* sizes, int ndim, void* stream) {
  if (op < MT_BIN_ADD || op > MT_BIN_DIV) return fail(MT_ERR_UNSUPPORTED, "binary: op %d", op);
  return launch_binary(op, y, y_dtype, y_strides, a, a_dtype, a_strides, b, b_dtype, b_strides, scalar, sizes, ndim,
                       S(stream));
}

int mt_cuda_axpby(void* out, int out_dtype, const void* x, int x_dtype, double a, const void* y, int y_dtype, double b,
                  const void* z, int z_dtype, double c, int64_t n, void* stream) {
  return launch_axpby(out, out_dtype, x, x_dtype, a, y, y_dtype, b, z, z_dtype, c, n, S(stream));
}

int mt_cuda_ddim_step(void* out, const void* x, const void* eps, int dtype, int eps_dtype, int64_t n, double alpha_t,
                      double alpha_prev, int clip, void* stream) {
  if (!(alpha_t > 0.0 && alpha_t < 1.0) || !(alpha_prev > 0.0 && alpha_prev <= 1.0))
    return fail(MT_ERR_INVALID, "ddim_step: alphas must lie in (0, 1)");
  return launch_ddim_step(out, x, eps, dtype, eps_dtype, n, alpha_t, alpha_prev, clip, S(stream));
}

int mt_cuda_ddim_step_indexed(void* out, int64_t out_copies, const void* x, const void* eps, int dtype, int eps_dtype,
                              int64_t n, const double* alphas_cumprod, int64_t num_train_steps,
                              const int64_t* timestep, int64_t interval, int cfg, double guidance_scale, int clip,
                              void* stream) {
  if (!out || !x || !eps || !alphas_cumprod || !timestep) return fail(MT_ERR_INVALID, "ddim_step_indexed: null pointer");
  if (out_copies < 1 || out_copies > 2) return fail(MT_ERR_INVALID, "ddim_step_indexed: out_copies must be 1 or 2");
  if (num_train_steps < 1 || interval < 0) return fail(MT_ERR_INVALID, "ddim_step_indexed: bad schedule");
  if (dtype != MT_F32 && dtype != MT_BF16 && dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "ddim_step_indexed: dtype %d", dtype);
  return launch_ddim_indexed(out, out_copies, x, eps, dtype, eps_dtype, n, alphas_cumprod, num_train_steps, timestep,
                             interval, cfg ? 1 : 0, guidance_scale, clip, S(stream));
}

int mt_cuda_timestep_embedding(void* out, int out_dtype, const void* timesteps, int t_dtype, int64_t t_stride,
                               int64_t n, int64_t dim, double max_period, int flip_sin_to_cos, void* stream) {
  if (!out || !timesteps) return fail(MT_ERR_INVALID, "timestep_embedding: null pointer");
  if (dim % 2 != 0) return fail(MT_ERR_UNSUPPORTED, "timestep_embedding: odd dim %lld", (long long)dim);
  if (!(max_period > 1.0)) return fail(MT_ERR_INVALID, "timestep_embedding: max_period must exceed 1");
  if (t_dtype != MT_F32 && t_dtype != MT_I64 && t_dtype != MT_F64 && t_dtype != MT_BF16 && t_dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "timestep_embedding: timestep dtype %d", t_dtype);
  if (out_dtype != MT_F32 && out_dtype != MT_BF16 && out_dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "timestep_embedding: dtype %d", out_dtype);
  return launch_timestep_embedding(out, out_dtype, timesteps, t_dtype, t_stride, n, dim, max_period, flip_sin_to_cos,
                                   S(stream));
}

int mt_cuda_embedding(void* out, int out_dtype, const void* weight, int w_dtype, int64_t rows, int64_t dim,
                      const int64_t* ids, int64_t n, const void* add, int add_dtype, int64_t add_rows,
                      const int64_t* add_ids, int* invalid_count, void* stream) {
  if (n > 0 && dim > 0 && (!out || !weight || !ids)) return fail(MT_ERR_INVALID, "embedding: null pointer");
  if (add && !add_ids) return fail(MT_ERR_INVALID, "embedding: add table without ids");
  if (rows < 0 || dim < 0) return fail(MT_ERR_INVALID, "embedding: negative size");
  auto ok = [](int d) { return d == MT_F32 || d == MT_BF16 || d == MT_F16 || d == MT_F64; };
  if (!ok(out_dtype) || !ok(w_dtype) || (add && !ok(add_dtype))) return fail(MT_ERR_UNSUPPORTED, "embedding: dtype");
  return launch_embedding(out, out_dtype, weight, w_dtype, rows, dim, ids, n, add, add_dtype, add_rows, add_ids,
                          invalid_count, S(stream));
}

int mt_cuda_softmax(void* y, int y_dtype, const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ld,
                    int log_output, void* stream) {
  return launch_softmax(y, y_dtype, x, x_dtype, rows, cols, ld, log_output, S(stream));
}

int mt_cuda_layer_norm(void* y, int y_dtype, const void* x, int x_dtype, const void* weight, const void* bias,
                       int wb_dtype, int64_t rows, int64_t cols, double eps, void* stream) {
  return launch_layer_norm(y, y_dtype, x, x_dtype, weight, bias, wb_dtype, rows, cols, eps, S(stream));
}

size_t mt_cuda_group_norm_workspace_size(int64_t N, int64_t C, int64_t HW, int64_t groups) {
  return group_norm_workspace(N, C, HW, groups);
}

int mt_cuda_group_norm(void* y, int y_dtype, const int64_t* y_strides, const void* x, int x_dtype,
                       const int64_t* x_strides, const void* weight, const void* bias, int wb_dtype, int64_t N,
                       int64_t C, int64_t HW, int64_t groups, double eps, int fuse_silu, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return launch_group_norm(y, y_dtype, y_strides, x, x_dtype, x_strides, weight, bias, wb_dtype, N, C, HW, groups,
                           eps, fuse_silu, workspace, workspace_bytes, S(stream));
}

int mt_cuda_group_norm_cat(void* y, int y_dtype, const int64_t* y_strides, const void* x1, const int64_t* x1_strides,
                           int64_t C1, const void* x2, const int64_t* x2_strides, int x_dtype, const void* weight,
                           const void* bias, int wb_dtype, int64_t N, int64_t C, int64_t HW, int64_t groups, double eps,
                           int fuse_silu, void* workspace, size_t workspace_bytes, void* stream) {
  return launch_group_norm_cat(y, y_dtype, y_strides, x1, x1_strides, C1, x2, x2_strides, x_dtype, weight, bias,
                               wb_dtype, N, C, HW, groups, eps, fuse_silu, workspace, workspace_bytes, S(stream));
}

size_t mt_cuda_gemm_workspace_size(const mt_gemm_desc* desc) { return desc ? gemm_workspace(*desc) : 0; }
int mt_cuda_gemm(const mt_gemm_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return fail(MT_ERR_INVALID, "gemm: null descriptor");
  return run_gemm(*desc, workspace, workspace_bytes, S(stream));
}

size_t mt_cuda_conv2d_workspace_size(const mt_conv2d_desc* desc) { return desc ? conv_workspace(*desc) : 0; }
int mt_cuda_conv2d(const mt_conv2d_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return fail(MT_ERR_INVALID, "conv2d: null descriptor");
  return run_conv2d(*desc, workspace, workspace_bytes, S(stream));
}
size_t mt_cuda_conv2d_cat_workspace_size(const mt_conv2d_desc* desc, const void* x2, const int64_t* x2_strides,
                                         int64_t C1) {
  return desc ? conv_cat_workspace(*desc, x2, x2_strides, C1) : 0;
}
int mt_cuda_conv2d_cat(const mt_conv2d_desc* desc, const void* x2, const int64_t* x2_strides, int64_t C1,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return fail(MT_ERR_INVALID, "conv2d_cat: null descriptor");
  return run_conv2d_cat(*desc, x2, x2_strides, C1, workspace, workspace_bytes, S(stream));
}
int64_t mt_cuda_conv2d_packed_channels(int64_t C, int64_t R, int64_t S_, int dtype) {
  return conv_packed_channels(C, R, S_, dtype);
}
int mt_cuda_conv2d_pack_weight(void* w_packed, void* w_lo, const void* w, int dtype, int64_t K, int64_t C, int64_t R,
                               int64_t S_, void* stream) {
  const int64_t Cp = conv_packed_channels(C, R, S_, dtype);
  return launch_conv_pack_weight(w_packed, (float*)w_lo, w, dtype, K, C, R, S_, Cp, S(stream));
}

size_t mt_cuda_conv2d_up2x_workspace_size(const mt_conv2d_desc* desc) { return desc ? conv_up2x_workspace(*desc) : 0; }
int mt_cuda_conv2d_up2x(const mt_conv2d_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return fail(MT_ERR_INVALID, "conv2d_up2x: null descriptor");
  return run_conv2d_up2x(*desc, workspace, workspace_bytes, S(stream));
}
int64_t mt_cuda_conv2d_up2x_packed_elems(int64_t K, int64_t C, int dtype) { return conv_up2x_packed_elems(K, C, dtype); }
int mt_cuda_conv2d_up2x_pack_weight(void* w_packed, void* w_lo, const void* w, int dtype, int64_t K, int64_t C,
                                    void* stream) {
  if (!w_packed && !w_lo) return fail(MT_ERR_INVALID, "conv2d_up2x pack: no output");
  return launch_conv_up2x_pack_weight(w_packed, (float*)w_lo, w, dtype, K, C, conv_packed_channels(C, 2, 2, dtype),
                                      S(stream));
}

int mt_cuda_sdpa_path(const mt_sdpa_desc* desc) {
  if (!desc || validate_sdpa_desc(*desc) != MT_OK) return 0;
  return sdpa_tc_path(*desc);
}

size_t mt_cuda_sdpa_workspace_size(const mt_sdpa_desc* desc) { return desc ? sdpa_workspace(*desc) : 0; }
int mt_cuda_sdpa(const mt_sdpa_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return fail(MT_ERR_INVALID, "sdpa: null descriptor");
  return run_sdpa(*desc, workspace, workspace_bytes, S(stream));
}

// ---- host generator: SplitMix64 + Marsaglia polar, as the reference's RandomState ----------
static uint64_t rng_next(mt_rng_state* r) {
  r->state += 0x9E3779B97F4A7C15ULL;
  uint64_t v = r->state;
  v = (v ^ (v >> 30U)) * 0xBF58476D1CE4E5B9ULL;
  v = (v ^ (v >> 27U)) * 0x94D049BB133111EBULL;
  return v ^ (v >> 31U);
}
static double rng_uniform_open(mt_rng_state* r) {
  const double k = 1.0 / 9007199254740992.0;
  const double v = (double)(rng_next(r) >> 11U) * k;
  return v <= 0.0 ? k : v;
}
static void rng_pair(mt_rng_state* r, double* a, double* b) {
  double u, v, s;
  do {
    u = 2.0 * rng_uniform_open(r) - 1.0;
    v = 2.0 * rng_uniform_open(r) - 1.0;
    s = u * u + v * v;
  } while (s >= 1.0 || s <= 0.0);
  const double m = std::sqrt(-2.0 * std::log(s) / s);
  *a = u * m;
  *b = v * m;
}

void mt_rng_seed(mt_rng_state* rng, uint64_t seed) {
  rng->state = seed;
  rng->has_spare = 0;
  rng->spare = 0.0;
}

static inline void put(void* dst, int dtype, int64_t i, double v) {
  if (dtype == MT_F64) static_cast<double*>(dst)[i] = v;
  else static_cast<float*>(dst)[i] = (float)v;
}

void mt_rng_fill_normal(mt_rng_state* rng, void* dst, int dtype, int64_t n, double mean, double std) {
  int64_t i = 0;
  if (n <= 0) return;
  if (rng->has_spare) {
    put(dst, dtype, i++, mean + std * rng->spare);
    rng->has_spare = 0;
  }
  while (i + 1 < n) {
    double a, b;
    rng_pair(rng, &a, &b);
    put(dst, dtype, i++, mean + std * a);
    put(dst, dtype, i++, mean + std * b);
  }
  if (i < n) {
    double a, b;
    rng_pair(rng, &a, &b);
    put(dst, dtype, i++, mean + std * a);
    rng->spare = b;
    rng->has_spare = 1;
  }
}

void mt_rng_fill_uniform(mt_rng_state* rng, void* dst, int dtype, int64_t n, double from, double to) {
  const double scale = to - from;
  for (int64_t i = 0; i < n; ++i) put(dst, dtype, i, from + scale * rng_uniform_open(rng));
}

}  // extern "C"
