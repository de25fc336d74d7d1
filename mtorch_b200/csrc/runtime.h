// Internal host-side runtime of the kernel library: error reporting, device properties,
// TMA tensor-map encoding and the launcher declarations shared between translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace mt {

// Records a printf-style message as the calling thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
int cuda_check(cudaError_t e, const char* what);
int check_launch(const char* what);

inline int dtype_size(int dtype) {
  switch (dtype) {
    case MT_F32: return 4;
    case MT_BF16: return 2;
    case MT_F16: return 2;
    case MT_F64: return 8;
    case MT_I32: return 4;
    case MT_I64: return 8;
    case MT_BOOL: return 1;
    default: return 0;
  }
}

int num_sms();  // SM count of the current device (148 on B200)

// TMA tensor map over a dense tensor: dims innermost first; strides in BYTES for dims
// 1..rank-1; box in elements.  swizzle: 0 none, 128 = 128-byte.  elem_strides (optional): the
// traversal stride of each dimension; a box then holds ceil(box[i] / elem_strides[i]) elements
// along dimension i, taken every elem_strides[i]-th element from the start coordinate.
int make_tensor_map(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int swizzle,
                    const uint32_t* elem_strides = nullptr);

// elementwise.cu
int launch_copy_strided(void* dst, int dd, const int64_t* dst_st, const void* src, int sd, const int64_t* src_st,
                        const int64_t* sizes, int ndim, cudaStream_t st);
int launch_fill_uniform(void* dst, int dtype, int64_t n, uint64_t state, double from, double to, cudaStream_t st);
int launch_fill(void* dst, int dtype, int64_t n, double value, cudaStream_t st);
int launch_fill_strided_nan(void* dst, int dtype, const int64_t* strides, const int64_t* sizes, cudaStream_t st);
int launch_unary(int op, void* y, int yd, const void* x, int xd, int64_t n, cudaStream_t st);
int launch_binary(int op, void* y, int yd, const int64_t* ys, const void* a, int ad, const int64_t* as,
                  const void* b, int bd, const int64_t* bs, double scalar, const int64_t* sizes, int ndim,
                  cudaStream_t st);
int launch_axpby(void* out, int od, const void* x, int xd, double a, const void* y, int yd, double b, const void* z,
                 int zd, double c, int64_t n, cudaStream_t st);
int launch_ddim_step(void* out, const void* x, const void* eps, int dtype, int eps_dtype, int64_t n, double a_t,
                     double a_prev, int clip, cudaStream_t st);
int launch_ddim_indexed(void* out, int64_t copies, const void* x, const void* eps, int dtype, int eps_dtype,
                        int64_t n, const double* ac, int64_t len, const int64_t* tstep, int64_t interval, int cfg,
                        double g, int clip, cudaStream_t st);
int launch_timestep_embedding(void* out, int od, const void* t, int td, int64_t t_stride, int64_t n, int64_t dim,
                              double max_period, int flip, cudaStream_t st);
int launch_embedding(void* out, int od, const void* w, int wd, int64_t rows, int64_t dim, const int64_t* ids,
                     int64_t n, const void* add, int ad, int64_t add_rows, const int64_t* add_ids, int* invalid,
                     cudaStream_t st);
int launch_pack2d(void* out, float* lo, const void* in, int dtype, int64_t batch, int64_t rows, int64_t cols,
                  int64_t sr, int64_t sc, int64_t sb, int64_t out_pitch, cudaStream_t st);
int launch_conv_pack_weight(void* out, float* lo, const void* w, int dtype, int64_t K, int64_t C, int64_t R,
                            int64_t S, int64_t Cp, cudaStream_t st);
int launch_conv_up2x_pack_weight(void* out, float* lo, const void* w, int dtype, int64_t K, int64_t C, int64_t Cp,
                                 cudaStream_t st);
int launch_im2col(void* col, float* lo, const void* x, int dtype, const mt_conv2d_desc& d, int64_t Cp, int64_t Kp,
                  cudaStream_t st);

// norm.cu
int launch_softmax(void* y, int yd, const void* x, int xd, int64_t rows, int64_t cols, int64_t ld, int log_output,
                   cudaStream_t st);
int launch_layer_norm(void* y, int yd, const void* x, int xd, const void* w, const void* b, int wbd, int64_t rows,
                      int64_t cols, double eps, cudaStream_t st);
size_t group_norm_workspace(int64_t N, int64_t C, int64_t HW, int64_t G);
int launch_group_norm(void* y, int yd, const int64_t* ys, const void* x, int xd, const int64_t* xs, const void* w,
                      const void* b, int wbd, int64_t N, int64_t C, int64_t HW, int64_t G, double eps, int silu,
                      void* ws, size_t ws_bytes, cudaStream_t st);

// gemm.cu
int launch_group_norm_cat(void* y, int yd, const int64_t* ys, const void* x1, const int64_t* xs1, int64_t C1,
                          const void* x2, const int64_t* xs2, int xd, const void* w, const void* b, int wbd, int64_t N,
                          int64_t C, int64_t HW, int64_t G, double eps, int silu, void* ws, size_t ws_bytes,
                          cudaStream_t st);
size_t gemm_workspace(const mt_gemm_desc& d);
int run_gemm(const mt_gemm_desc& d, void* ws, size_t ws_bytes, cudaStream_t st);
size_t conv_workspace(const mt_conv2d_desc& d);
int run_conv2d(const mt_conv2d_desc& d, void* ws, size_t ws_bytes, cudaStream_t st);
size_t conv_cat_workspace(const mt_conv2d_desc& d, const void* x2, const int64_t* x2_strides, int64_t c1);
int run_conv2d_cat(const mt_conv2d_desc& d, const void* x2, const int64_t* x2_strides, int64_t c1, void* ws,
                   size_t ws_bytes, cudaStream_t st);
int64_t conv_up2x_packed_elems(int64_t K, int64_t C, int dtype);
size_t conv_up2x_workspace(const mt_conv2d_desc& d);
int run_conv2d_up2x(const mt_conv2d_desc& d, void* ws, size_t ws_bytes, cudaStream_t st);
int64_t conv_packed_channels(int64_t C, int64_t R, int64_t S, int dtype);

// attention.cu
size_t sdpa_workspace(const mt_sdpa_desc& d);
int run_sdpa(const mt_sdpa_desc& d, void* ws, size_t ws_bytes, cudaStream_t st);
int validate_sdpa_desc(const mt_sdpa_desc& d);
int sdpa_tc_path(const mt_sdpa_desc& d);

// Per-translation-unit device status readers (see g_device_error).
int read_status_gemm(int clear);
int run_wait_timeout_selftest(long long budget_cycles, cudaStream_t st);
int read_status_attention(int clear);
int read_status_norm(int clear);
#define MT_STATUS_READER(name)                                                   \
  int name(int clear) {                                                          \
    int v = 0;                                                                   \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) {  \
      cudaGetLastError();                                                        \
      return -1;                                                                 \
    }                                                                            \
    if (clear && v) {                                                            \
      int z = 0;                                                                 \
      cudaMemcpyToSymbol(g_device_error, &z, sizeof(int));                       \
    }                                                                            \
    return v;                                                                    \
  }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace mt
