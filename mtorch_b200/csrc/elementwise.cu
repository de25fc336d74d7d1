// Memory-bound kernels: strided copy / cast, fills (incl. the SplitMix64 uniform stream),
// unary activations, broadcast binary ops, the fused DDIM axpby, and the operand packing
// kernels used by the tensor-core paths (transpose + tf32 split, conv im2col, weight repack).
#include "runtime.h"

namespace mt {

struct StridedND {
  int ndim;
  int64_t sizes[MT_MAX_DIMS];
  int64_t s0[MT_MAX_DIMS];
  int64_t s1[MT_MAX_DIMS];
  int64_t s2[MT_MAX_DIMS];
};

__device__ __forceinline__ void nd_offsets(const StridedND& nd, int64_t linear, int64_t& o0, int64_t& o1,
                                           int64_t& o2) {
  o0 = o1 = o2 = 0;
  for (int d = nd.ndim - 1; d >= 0; --d) {
    const int64_t sz = nd.sizes[d];
    const int64_t c = linear % sz;
    linear /= sz;
    o0 += c * nd.s0[d];
    o1 += c * nd.s1[d];
    o2 += c * nd.s2[d];
  }
}

static int grid_for(int64_t n, int threads) {
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

#define MT_GRID_STRIDE(i, n) \
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (n); i += (int64_t)gridDim.x * blockDim.x)

// ---------------------------------------------------------------------------------------------
__global__ void copy_strided_kernel(void* dst, int dd, const void* src, int sd, StridedND nd, int64_t n) {
  MT_GRID_STRIDE(i, n) {
    int64_t od, os, unused;
    nd_offsets(nd, i, od, os, unused);
    if (dd == MT_F64 || sd == MT_F64)
      store_from_f64(dst, od, dd, load_as_f64(src, os, sd));
    else
      store_from_f32(dst, od, dd, load_as_f32(src, os, sd));
  }
}

// Same-type strided copy of integer / bool elements (bit patterns moved, no conversion).
template <typename T>
__global__ void copy_strided_raw_kernel(T* dst, const T* src, StridedND nd, int64_t n) {
  MT_GRID_STRIDE(i, n) {
    int64_t od, os, unused;
    nd_offsets(nd, i, od, os, unused);
    dst[od] = src[os];
  }
}

// Same-dtype strided copy in 16-byte units (offsets of `nd` are in 16-byte units).
__global__ void copy_rows16_kernel(uint4* dst, const uint4* src, StridedND nd, int64_t n16) {
  const int64_t inner = nd.sizes[nd.ndim - 1];
  MT_GRID_STRIDE(i, n16) {
    const int64_t row = i / inner, v = i - row * inner;
    int64_t od = 0, os = 0, r = row;
    for (int d = nd.ndim - 2; d >= 0; --d) {
      const int64_t c = r % nd.sizes[d];
      r /= nd.sizes[d];
      od += c * nd.s0[d];
      os += c * nd.s1[d];
    }
    dst[od + v] = src[os + v];
  }
}

// Contiguous same-dtype 16-byte copies.
__global__ void copy_vec16_kernel(uint4* dst, const uint4* src, int64_t n16) {
  MT_GRID_STRIDE(i, n16) dst[i] = src[i];
}

template <typename TD, typename TS>
__global__ void cast_contig_kernel(TD* dst, const TS* src, int64_t n) {
  MT_GRID_STRIDE(i, n) dst[i] = from_f32<TD>(to_f32<TS>(src[i]));
}

static bool is_contig(const int64_t* st, const int64_t* sizes, int ndim) {
  int64_t expect = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    if (sizes[d] != 1 && st[d] != expect) return false;
    expect *= sizes[d];
  }
  return true;
}

// ---------------------------------------------------------------------------------------------
// SplitMix64 stream: the k-th draw after `state` is mix(state + k * golden).  Matches
// next_random_u64 / next_uniform_open of the reference generator (module.cpp:76-88); the double
// arithmetic uses explicit round-to-nearest intrinsics so that no FMA contraction changes the last
// bit relative to the host code.
__device__ __forceinline__ uint64_t splitmix_draw(uint64_t state, uint64_t k) {
  uint64_t v = state + k * 0x9E3779B97F4A7C15ULL;
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
  return v ^ (v >> 31);
}
__global__ void fill_uniform_kernel(void* dst, int dtype, int64_t n, uint64_t state, double from, double scale) {
  const double kScale = 1.0 / 9007199254740992.0;
  MT_GRID_STRIDE(i, n) {
    double u = __dmul_rn((double)(splitmix_draw(state, (uint64_t)i + 1) >> 11), kScale);
    if (u <= 0.0) u = kScale;
    const double v = __dadd_rn(from, __dmul_rn(scale, u));
    store_from_f64(dst, i, dtype, v);
  }
}
__global__ void fill_kernel(void* dst, int dtype, int64_t n, double value) {
  MT_GRID_STRIDE(i, n) store_from_f64(dst, i, dtype, value);
}

__global__ void fill_strided_kernel(void* dst, int dtype, StridedND nd, int64_t n, double value) {
  MT_GRID_STRIDE(i, n) {
    int64_t o, u1, u2;
    nd_offsets(nd, i, o, u1, u2);
    store_from_f64(dst, o, dtype, value);
  }
}

// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float apply_unary(int op, float x) {
  switch (op) {
    case MT_UNARY_SILU: return silu_f(x);
    case MT_UNARY_GELU: return gelu_f(x);
    case MT_UNARY_GELU_TANH: return gelu_tanh_f(x);
    case MT_UNARY_NEG: return -x;
    case MT_UNARY_EXP: return expf(x);
    case MT_UNARY_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case MT_UNARY_RELU: return x > 0.f ? x : 0.f;
    case MT_UNARY_QUICK_GELU: return x * (1.0f / (1.0f + expf(-__fmul_rn(x, 1.702f))));
    default: return x;
  }
}
__global__ void unary_f32_kernel(int op, float* y, const float* x, int64_t n) {
  MT_GRID_STRIDE(i, n) y[i] = apply_unary(op, x[i]);
}
// bf16 -> bf16, 8 elements per thread.
__global__ void unary_bf16x8_kernel(int op, uint4* y, const uint4* x, int64_t n8) {
  MT_GRID_STRIDE(i, n8) {
    uint4 v = x[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      h[j] = __floats2bfloat162_rn(apply_unary(op, f.x), apply_unary(op, f.y));
    }
    y[i] = v;
  }
}
__global__ void unary_generic_kernel(int op, void* y, int yd, const void* x, int xd, int64_t n) {
  MT_GRID_STRIDE(i, n) store_from_f32(y, i, yd, apply_unary(op, load_as_f32(x, i, xd)));
}

// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T apply_binary(int op, T a, T b) {
  switch (op) {
    case MT_BIN_ADD: return a + b;
    case MT_BIN_SUB: return a - b;
    case MT_BIN_MUL: return a * b;
    case MT_BIN_DIV: return a / b;
    default: return a;
  }
}
// Generic broadcast: fp32 math (fp64 when any operand is f64).
__global__ void binary_strided_kernel(int op, void* y, int yd, const void* a, int ad, const void* b, int bd,
                                      double scalar, StridedND nd, int64_t n) {
  const bool wide = (yd == MT_F64 || ad == MT_F64 || (b && bd == MT_F64));
  MT_GRID_STRIDE(i, n) {
    int64_t oy, oa, ob;
    nd_offsets(nd, i, oy, oa, ob);
    if (wide) {
      const double bv = b ? load_as_f64(b, ob, bd) : scalar;
      store_from_f64(y, oy, yd, apply_binary<double>(op, load_as_f64(a, oa, ad), bv));
    } else {
      const float bv = b ? load_as_f32(b, ob, bd) : (float)scalar;
      store_from_f32(y, oy, yd, apply_binary<float>(op, load_as_f32(a, oa, ad), bv));
    }
  }
}
// Same-shape contiguous fp32 / bf16 fast paths (vectorised).
__global__ void binary_f32x4_kernel(int op, float4* y, const float4* a, const float4* b, int64_t n4) {
  MT_GRID_STRIDE(i, n4) {
    float4 va = a[i], vb = b[i];
    y[i] = make_float4(apply_binary<float>(op, va.x, vb.x), apply_binary<float>(op, va.y, vb.y),
                       apply_binary<float>(op, va.z, vb.z), apply_binary<float>(op, va.w, vb.w));
  }
}
__global__ void binary_bf16x8_kernel(int op, uint4* y, const uint4* a, const uint4* b, int64_t n8) {
  MT_GRID_STRIDE(i, n8) {
    uint4 va = a[i], vb = b[i], vy;
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&va);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&vb);
    __nv_bfloat162* hy = reinterpret_cast<__nv_bfloat162*>(&vy);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 fa = __bfloat1622float2(ha[j]), fb = __bfloat1622float2(hb[j]);
      hy[j] = __floats2bfloat162_rn(apply_binary<float>(op, fa.x, fb.x), apply_binary<float>(op, fa.y, fb.y));
    }
    y[i] = vy;
  }
}

__global__ void axpby_kernel(void* out, int od, const void* x, int xd, float a, const void* y, int yd, float b,
                             const void* z, int zd, float c, int64_t n) {
  MT_GRID_STRIDE(i, n) {
    float v = a * load_as_f32(x, i, xd);
    if (y) v += b * load_as_f32(y, i, yd);
    if (z) v += c * load_as_f32(z, i, zd);
    store_from_f32(out, i, od, v);
  }
}

// ---------------------------------------------------------------------------------------------
// Operand packing for the tensor-core paths.  out[b][r][c] = in[b*sb + r*sr + c*sc], written
// row-major [batch, rows, out_pitch] through a 32x32 shared-memory tile so that both the read
// (along whichever input axis is unit-stride) and the write are coalesced.  For fp32, `lo`
// (optional) receives x - tf32_hi(x) (the low half of the 3xTF32 split); `out` (optional)
// receives x itself.
template <typename T>
__global__ void pack2d_kernel(T* out, float* lo, const T* in, int64_t rows, int64_t cols, int64_t sr, int64_t sc,
                              int64_t sb, int64_t out_pitch) {
  __shared__ float tile[32][33];
  const int64_t b = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const T* src = in + b * sb;
  const bool read_along_rows = (sr == 1 && sc != 1);
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int i = threadIdx.x;
    int64_t r, c;
    if (read_along_rows) { r = r0 + i; c = c0 + j; } else { r = r0 + j; c = c0 + i; }
    float v = 0.f;
    if (r < rows && c < cols) v = to_f32<T>(src[r * sr + c * sc]);
    if (read_along_rows) tile[i][j] = v; else tile[j][i] = v;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int64_t r = r0 + j, c = c0 + threadIdx.x;
    if (r < rows && c < cols) {
      const float v = tile[j][threadIdx.x];
      const int64_t o = b * rows * out_pitch + r * out_pitch + c;
      if (out) out[o] = from_f32<T>(v);
      if (lo) lo[o] = tf32_lo(v);
    }
  }
}

// Conv weight [K, C, R, S] -> [K, R, S, Cp] (zero-filled channels C..Cp), optional tf32 low part.
template <typename T>
__global__ void conv_pack_weight_kernel(T* out, float* lo, const T* w, int64_t K, int64_t C, int64_t R, int64_t S,
                                        int64_t Cp) {
  const int64_t n = K * R * S * Cp;
  MT_GRID_STRIDE(i, n) {
    const int64_t c = i % Cp;
    int64_t t = i / Cp;
    const int64_t s = t % S; t /= S;
    const int64_t r = t % R;
    const int64_t k = t / R;
    const float v = c < C ? to_f32<T>(w[((k * C + c) * R + r) * S + s]) : 0.f;
    if (out) out[i] = from_f32<T>(v);
    if (lo) lo[i] = tf32_lo(v);
  }
}

// Weights of a 3x3 convolution applied to a nearest-2x upsampled input, regrouped per output
// parity.  Output row 2i+a reads upsampled rows 2i+a-1 .. 2i+a+1, i.e. source rows
// a = 0: {i-1: tap 0, i: taps 1+2},  a = 1: {i: taps 0+1, i+1: tap 2}  (columns likewise), so each
// parity (a, b) is a 2x2 convolution of the source whose taps are sums of the 3x3 taps.
// out: [4 = 2a+b][K][2][2][Cp] (sums formed in fp32, then rounded once); lo: tf32 low parts.
template <typename T>
__global__ void conv_up2x_pack_weight_kernel(T* out, float* lo, const T* w, int64_t K, int64_t C, int64_t Cp) {
  const int64_t n = 4 * K * 4 * Cp;
  MT_GRID_STRIDE(i, n) {
    const int64_t c = i % Cp;
    int64_t t = i / Cp;
    const int v = (int)(t % 2); t /= 2;
    const int u = (int)(t % 2); t /= 2;
    const int64_t k = t % K;
    const int par = (int)(t / K);
    const int a = par >> 1, b = par & 1;
    // 3x3 taps [r0, r1] feeding 2x2 tap u (rows) for parity a; likewise columns
    const int r0 = a == 0 ? (u == 0 ? 0 : 1) : (u == 0 ? 0 : 2);
    const int r1 = a == 0 ? (u == 0 ? 0 : 2) : (u == 0 ? 1 : 2);
    const int s0 = b == 0 ? (v == 0 ? 0 : 1) : (v == 0 ? 0 : 2);
    const int s1 = b == 0 ? (v == 0 ? 0 : 2) : (v == 0 ? 1 : 2);
    float acc = 0.f;
    if (c < C)
      for (int r = r0; r <= r1; ++r)
        for (int s = s0; s <= s1; ++s) acc += to_f32<T>(w[((k * C + c) * 3 + r) * 3 + s]);
    if (out) out[i] = from_f32<T>(acc);
    if (lo) lo[i] = tf32_lo(acc);
  }
}

int launch_conv_up2x_pack_weight(void* out, float* lo, const void* w, int dtype, int64_t K, int64_t C, int64_t Cp,
                                 cudaStream_t st) {
  const int64_t n = 16 * K * Cp;
  switch (dtype) {
    case MT_F32:
      conv_up2x_pack_weight_kernel<float><<<grid_for(n, 256), 256, 0, st>>>((float*)out, lo, (const float*)w, K, C, Cp);
      break;
    case MT_BF16:
      conv_up2x_pack_weight_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, st>>>(
          (__nv_bfloat16*)out, nullptr, (const __nv_bfloat16*)w, K, C, Cp);
      break;
    case MT_F16:
      conv_up2x_pack_weight_kernel<__half><<<grid_for(n, 256), 256, 0, st>>>((__half*)out, nullptr, (const __half*)w,
                                                                              K, C, Cp);
      break;
    default: return fail(MT_ERR_UNSUPPORTED, "conv up2x weight pack: dtype");
  }
  return check_launch("conv_up2x_pack_weight");
}

// im2col for the general convolution path: col[(n*P+p)*Q+q][(r*S+s)*Cp + c] (zero padded in
// space and channels); x addressed through its own (n, c, h, w) strides.
template <typename T>
__global__ void im2col_kernel(T* col, float* lo, const T* x, int64_t N, int64_t C, int64_t H, int64_t W, int64_t P,
                              int64_t Q, int R, int S, int sh, int sw, int ph, int pw, int dh, int dw, int64_t xs0,
                              int64_t xs1, int64_t xs2, int64_t xs3, int64_t Cp, int64_t Kp) {
  const int64_t n_total = N * P * Q * Kp;
  MT_GRID_STRIDE(i, n_total) {
    const int64_t kk = i % Kp;
    const int64_t m = i / Kp;
    float v = 0.f;
    if (kk < (int64_t)R * S * Cp) {
      const int64_t c = kk % Cp;
      const int64_t rs = kk / Cp;
      const int r = (int)(rs / S), s = (int)(rs % S);
      const int64_t q = m % Q;
      const int64_t p = (m / Q) % P;
      const int64_t nn = m / (P * Q);
      const int64_t h = p * sh - ph + (int64_t)r * dh;
      const int64_t w = q * sw - pw + (int64_t)s * dw;
      if (c < C && h >= 0 && h < H && w >= 0 && w < W) v = to_f32<T>(x[nn * xs0 + c * xs1 + h * xs2 + w * xs3]);
    }
    if (col) col[i] = from_f32<T>(v);
    if (lo) lo[i] = tf32_lo(v);
  }
}

// ---------------------------------------------------------------------------------------------
// Host launchers.
int launch_copy_strided(void* dst, int dd, const int64_t* dst_st, const void* src, int sd, const int64_t* src_st,
                        const int64_t* sizes, int ndim, cudaStream_t st) {
  if (ndim < 0 || ndim > MT_MAX_DIMS) return fail(MT_ERR_INVALID, "copy_strided: ndim out of range");
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) n *= sizes[d];
  if (n == 0) return MT_OK;
  if (dtype_size(dd) == 0 || dtype_size(sd) == 0) return fail(MT_ERR_UNSUPPORTED, "copy_strided: dtype");
  const bool raw = dd > MT_F64 || sd > MT_F64;  // integer / bool: same-type copies only, no casts
  if (raw && dd != sd) return fail(MT_ERR_UNSUPPORTED, "copy_strided: integer dtype casts");
  const bool dc = is_contig(dst_st, sizes, ndim), sc = is_contig(src_st, sizes, ndim);
  if (dc && sc) {
    if (dd == sd) {
      const int64_t bytes = n * dtype_size(dd);
      if (bytes % 16 == 0 && ((uintptr_t)dst % 16 == 0) && ((uintptr_t)src % 16 == 0)) {
        copy_vec16_kernel<<<grid_for(bytes / 16, 256), 256, 0, st>>>((uint4*)dst, (const uint4*)src, bytes / 16);
        return check_launch("copy_vec16");
      }
      return cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st), "copy");
    }
    if (dd == MT_BF16 && sd == MT_F32) {
      cast_contig_kernel<__nv_bfloat16, float>
          <<<grid_for(n, 256), 256, 0, st>>>((__nv_bfloat16*)dst, (const float*)src, n);
      return check_launch("cast");
    }
    if (dd == MT_F32 && sd == MT_BF16) {
      cast_contig_kernel<float, __nv_bfloat16>
          <<<grid_for(n, 256), 256, 0, st>>>((float*)dst, (const __nv_bfloat16*)src, n);
      return check_launch("cast");
    }
  }
  // Normalise: drop size-1 dims, order by destination stride (largest first) and merge dims
  // that are contiguous in both operands.  A channel-concat into a channels-last tensor, or a
  // nearest-upsample view, becomes [rows, inner] with a unit-stride inner run on both sides.
  StridedND nd{};
  int m = 0;
  for (int d = 0; d < ndim; ++d) {
    if (sizes[d] == 1) continue;
    nd.sizes[m] = sizes[d];
    nd.s0[m] = dst_st[d];
    nd.s1[m] = src_st[d];
    ++m;
  }
  for (int i = 1; i < m; ++i)  // insertion sort, descending |dst stride|
    for (int j = i; j > 0 && llabs(nd.s0[j]) > llabs(nd.s0[j - 1]); --j) {
      std::swap(nd.sizes[j], nd.sizes[j - 1]);
      std::swap(nd.s0[j], nd.s0[j - 1]);
      std::swap(nd.s1[j], nd.s1[j - 1]);
    }
  int k = 0;
  for (int i = 1; i < m; ++i) {
    if (nd.s0[k] == nd.s0[i] * nd.sizes[i] && nd.s1[k] == nd.s1[i] * nd.sizes[i]) {
      nd.sizes[k] *= nd.sizes[i];
      nd.s0[k] = nd.s0[i];
      nd.s1[k] = nd.s1[i];
    } else {
      ++k;
      nd.sizes[k] = nd.sizes[i];
      nd.s0[k] = nd.s0[i];
      nd.s1[k] = nd.s1[i];
    }
  }
  nd.ndim = m ? k + 1 : 0;
  if (nd.ndim == 0) {  // a single element
    nd.ndim = 1;
    nd.sizes[0] = 1;
    nd.s0[0] = nd.s1[0] = 1;
  }
  const int es = dtype_size(dd);
  const int last = nd.ndim - 1;
  if (dd == sd && nd.s0[last] == 1 && nd.s1[last] == 1 && (nd.sizes[last] * es) % 16 == 0 &&
      (uintptr_t)dst % 16 == 0 && (uintptr_t)src % 16 == 0) {
    bool ok = true;
    for (int d = 0; d < last; ++d) ok = ok && (nd.s0[d] * es) % 16 == 0 && (nd.s1[d] * es) % 16 == 0;
    if (ok) {
      // rows of 16-byte vectors: the outer dims are addressed in units of 16 bytes
      StridedND rows{};
      rows.ndim = nd.ndim;
      for (int d = 0; d < last; ++d) {
        rows.sizes[d] = nd.sizes[d];
        rows.s0[d] = nd.s0[d] * es / 16;
        rows.s1[d] = nd.s1[d] * es / 16;
      }
      rows.sizes[last] = nd.sizes[last] * es / 16;
      rows.s0[last] = rows.s1[last] = 1;
      const int64_t n16 = n * es / 16;
      copy_rows16_kernel<<<grid_for(n16, 256), 256, 0, st>>>((uint4*)dst, (const uint4*)src, rows, n16);
      return check_launch("copy_rows16");
    }
  }
  if (raw) {
    switch (es) {
      case 1: copy_strided_raw_kernel<<<grid_for(n, 256), 256, 0, st>>>((uint8_t*)dst, (const uint8_t*)src, nd, n); break;
      case 4: copy_strided_raw_kernel<<<grid_for(n, 256), 256, 0, st>>>((uint32_t*)dst, (const uint32_t*)src, nd, n); break;
      case 8: copy_strided_raw_kernel<<<grid_for(n, 256), 256, 0, st>>>((uint64_t*)dst, (const uint64_t*)src, nd, n); break;
      default: return fail(MT_ERR_UNSUPPORTED, "copy_strided: element size %d", es);
    }
    return check_launch("copy_strided_raw");
  }
  copy_strided_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, dd, src, sd, nd, n);
  return check_launch("copy_strided");
}

int launch_fill_uniform(void* dst, int dtype, int64_t n, uint64_t state, double from, double to, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  fill_uniform_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, dtype, n, state, from, to - from);
  return check_launch("fill_uniform");
}
int launch_fill(void* dst, int dtype, int64_t n, double value, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  fill_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, dtype, n, value);
  return check_launch("fill");
}

int launch_fill_strided_nan(void* dst, int dtype, const int64_t* strides, const int64_t* sizes, cudaStream_t st) {
  StridedND nd{};
  nd.ndim = 4;
  int64_t n = 1;
  for (int d = 0; d < 4; ++d) {
    nd.sizes[d] = sizes[d];
    nd.s0[d] = strides[d];
    n *= sizes[d];
  }
  if (n == 0) return MT_OK;
  fill_strided_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, dtype, nd, n, __builtin_nan(""));
  return check_launch("fill_strided");
}

int launch_unary(int op, void* y, int yd, const void* x, int xd, int64_t n, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  if (yd == MT_BF16 && xd == MT_BF16 && n % 8 == 0 && (uintptr_t)y % 16 == 0 && (uintptr_t)x % 16 == 0) {
    unary_bf16x8_kernel<<<grid_for(n / 8, 256), 256, 0, st>>>(op, (uint4*)y, (const uint4*)x, n / 8);
  } else if (yd == MT_F32 && xd == MT_F32) {
    unary_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(op, (float*)y, (const float*)x, n);
  } else {
    unary_generic_kernel<<<grid_for(n, 256), 256, 0, st>>>(op, y, yd, x, xd, n);
  }
  return check_launch("unary");
}

int launch_binary(int op, void* y, int yd, const int64_t* ys, const void* a, int ad, const int64_t* as,
                  const void* b, int bd, const int64_t* bs, double scalar, const int64_t* sizes, int ndim,
                  cudaStream_t st) {
  if (ndim < 0 || ndim > MT_MAX_DIMS) return fail(MT_ERR_INVALID, "binary: ndim out of range");
  int64_t n = 1;
  for (int d = 0; d < ndim; ++d) n *= sizes[d];
  if (n == 0) return MT_OK;
  if (b && yd == ad && ad == bd && is_contig(ys, sizes, ndim) && is_contig(as, sizes, ndim) &&
      is_contig(bs, sizes, ndim) && (uintptr_t)y % 16 == 0 && (uintptr_t)a % 16 == 0 && (uintptr_t)b % 16 == 0) {
    if (yd == MT_F32 && n % 4 == 0) {
      binary_f32x4_kernel<<<grid_for(n / 4, 256), 256, 0, st>>>(op, (float4*)y, (const float4*)a, (const float4*)b,
                                                                 n / 4);
      return check_launch("binary_f32x4");
    }
    if (yd == MT_BF16 && n % 8 == 0) {
      binary_bf16x8_kernel<<<grid_for(n / 8, 256), 256, 0, st>>>(op, (uint4*)y, (const uint4*)a, (const uint4*)b,
                                                                  n / 8);
      return check_launch("binary_bf16x8");
    }
  }
  StridedND nd{};
  nd.ndim = ndim;
  for (int d = 0; d < ndim; ++d) {
    nd.sizes[d] = sizes[d];
    nd.s0[d] = ys[d];
    nd.s1[d] = as[d];
    nd.s2[d] = b ? bs[d] : 0;
  }
  binary_strided_kernel<<<grid_for(n, 256), 256, 0, st>>>(op, y, yd, a, ad, b, bd, scalar, nd, n);
  return check_launch("binary");
}

int launch_axpby(void* out, int od, const void* x, int xd, double a, const void* y, int yd, double b, const void* z,
                 int zd, double c, int64_t n, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  axpby_kernel<<<grid_for(n, 256), 256, 0, st>>>(out, od, x, xd, (float)a, y, yd, (float)b, z, zd, (float)c, n);
  return check_launch("axpby");
}

// One DDIM update in fp32 (sa = sqrt(a_t), sb = sqrt(1 - a_t), sap / sbp the same for a_prev).
__device__ __forceinline__ float ddim_update(float xv, float ev, float sa, float sb, float sap, float sbp, int clip) {
  float x0 = (xv - sb * ev) / sa;
  if (clip) x0 = fminf(fmaxf(x0, -1.0f), 1.0f);
  const float e2 = (xv - sa * x0) / sb;
  return sap * x0 + sbp * e2;
}

__global__ void ddim_step_kernel(void* out, const void* x, const void* eps, int dtype, int eps_dtype, int64_t n,
                                 float sa, float sb, float sap, float sbp, int clip) {
  MT_GRID_STRIDE(i, n) {
    const float xv = load_as_f32(x, i, dtype), ev = load_as_f32(eps, i, eps_dtype);
    store_from_f32(out, i, dtype, ddim_update(xv, ev, sa, sb, sap, sbp, clip));
  }
}

// DDIM update whose timestep is read from device memory (so one captured graph serves every step)
// with optional classifier-free guidance folded in: eps holds [uncond; text] (2n values) and the
// guided noise is uncond + (text - uncond) * g, evaluated in that order with no FMA contraction
// (tests/compat/benchmarking.py:5847-5850).  The result goes to out[c*n + i] for c < copies, so the
// next step's doubled model input is written in the same pass.
__global__ void ddim_indexed_kernel(void* out, int64_t copies, const void* x, const void* eps, int dtype,
                                    int eps_dtype, int64_t n, const double* ac, int64_t len, const int64_t* tstep,
                                    int64_t interval, int cfg, float g, int clip) {
  int64_t t = *tstep;
  t = t < 0 ? 0 : (t >= len ? len - 1 : t);
  const int64_t tp = t - interval > 0 ? t - interval : 0;
  const double a_t = ac[t], a_p = ac[tp];
  const float sa = (float)sqrt(a_t), sb = (float)sqrt(1.0 - a_t), sap = (float)sqrt(a_p),
              sbp = (float)sqrt(1.0 - a_p);
  MT_GRID_STRIDE(i, n) {
    const float xv = load_as_f32(x, i, dtype);
    float ev = load_as_f32(eps, i, eps_dtype);
    if (cfg) ev = __fadd_rn(ev, __fmul_rn(__fsub_rn(load_as_f32(eps, n + i, eps_dtype), ev), g));
    const float v = ddim_update(xv, ev, sa, sb, sap, sbp, clip);
    for (int64_t c = 0; c < copies; ++c) store_from_f32(out, c * n + i, dtype, v);
  }
}

int launch_ddim_indexed(void* out, int64_t copies, const void* x, const void* eps, int dtype, int eps_dtype,
                        int64_t n, const double* ac, int64_t len, const int64_t* tstep, int64_t interval, int cfg,
                        double g, int clip, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  ddim_indexed_kernel<<<grid_for(n, 256), 256, 0, st>>>(out, copies, x, eps, dtype, eps_dtype, n, ac, len, tstep,
                                                        interval, cfg, (float)g, clip);
  return check_launch("ddim_step_indexed");
}

// Sinusoidal timestep embedding in fp32, as the reference's scenario builds it
// (tests/compat/benchmarking.py:6016-6021, 6035-6036): freq_j = exp((-ln(max_period) * j) / half),
// arg = t * freq_j, row = [cos(arg) | sin(arg)] (flip != 0) or [sin | cos]; accurate expf / cosf /
// sinf (the library is built without fast-math), so large arguments (t up to 999) keep full range
// reduction.  Timestep k of row r is t[r * t_stride] (stride 0 broadcasts one device scalar).
__global__ void timestep_embedding_kernel(void* out, int od, const void* t, int td, int64_t t_stride, int64_t n,
                                          int64_t half, float neg_log_period, int flip) {
  MT_GRID_STRIDE(i, n * 2 * half) {
    const int64_t r = i / (2 * half), c = i - r * 2 * half;
    const int64_t j = c < half ? c : c - half;
    const float tv = td == MT_I64 ? (float)static_cast<const int64_t*>(t)[r * t_stride]
                                  : load_as_f32(t, r * t_stride, td);
    const float freq = expf(__fdiv_rn(__fmul_rn(neg_log_period, (float)j), (float)half));
    const float arg = __fmul_rn(tv, freq);
    const bool first = c < half;
    store_from_f32(out, i, od, (first == (flip != 0)) ? cosf(arg) : sinf(arg));
  }
}

int launch_timestep_embedding(void* out, int od, const void* t, int td, int64_t t_stride, int64_t n, int64_t dim,
                              double max_period, int flip, cudaStream_t st) {
  if (n <= 0 || dim <= 0) return MT_OK;
  timestep_embedding_kernel<<<grid_for(n * dim, 256), 256, 0, st>>>(out, od, t, td, t_stride, n, dim / 2,
                                                                    -logf((float)max_period), flip);
  return check_launch("timestep_embedding");
}

int launch_ddim_step(void* out, const void* x, const void* eps, int dtype, int eps_dtype, int64_t n, double a_t,
                     double a_prev, int clip, cudaStream_t st) {
  if (n <= 0) return MT_OK;
  ddim_step_kernel<<<grid_for(n, 256), 256, 0, st>>>(out, x, eps, dtype, eps_dtype, n, (float)sqrt(a_t),
                                                     (float)sqrt(1.0 - a_t), (float)sqrt(a_prev),
                                                     (float)sqrt(1.0 - a_prev), clip);
  return check_launch("ddim_step");
}

// Embedding row gather (tensor.cpp:31748-31800): out[r, :] = weight[ids[r], :] (+ add[add_ids[r], :]),
// negative ids counted from the end as the reference's normalized_dim_index does.  An id outside
// [-rows, rows) writes a zero row and increments *invalid (when given) so the caller can raise the
// reference's IndexError.  Each warp copies one row; the optional add is done in fp32 and rounded
// once to the output type (for 16-bit tables this equals the reference's separate add).
__device__ __forceinline__ int64_t embed_row(const int64_t* ids, int64_t r, int64_t rows, int* invalid, bool* ok) {
  int64_t id = ids[r];
  if (id < 0) id += rows;
  *ok = id >= 0 && id < rows;
  if (!*ok && invalid && (threadIdx.x & 31) == 0) atomicAdd(invalid, 1);
  return *ok ? id : 0;
}

__global__ void embedding_kernel(void* out, int od, const void* w, int wd, int64_t rows, int64_t dim,
                                 const int64_t* ids, int64_t n, const void* add, int ad, int64_t add_rows,
                                 const int64_t* add_ids, int* invalid) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < n; r += warps) {
    bool ok, ok2 = true;
    const int64_t id = embed_row(ids, r, rows, invalid, &ok);
    const int64_t id2 = add ? embed_row(add_ids, r, add_rows, invalid, &ok2) : 0;
    for (int64_t c = lane; c < dim; c += 32) {
      float v = 0.f;
      if (ok && ok2) {
        v = load_as_f32(w, id * dim + c, wd);
        if (add) v += load_as_f32(add, id2 * dim + c, ad);
      }
      store_from_f32(out, r * dim + c, od, v);
    }
  }
}

int launch_embedding(void* out, int od, const void* w, int wd, int64_t rows, int64_t dim, const int64_t* ids,
                     int64_t n, const void* add, int ad, int64_t add_rows, const int64_t* add_ids, int* invalid,
                     cudaStream_t st) {
  if (n <= 0 || dim <= 0) return MT_OK;
  const int64_t blocks = (n + 7) / 8;
  embedding_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(out, od, w, wd, rows, dim, ids, n, add,
                                                                              ad, add_rows, add_ids, invalid);
  return check_launch("embedding");
}

int launch_pack2d(void* out, float* lo, const void* in, int dtype, int64_t batch, int64_t rows, int64_t cols,
                  int64_t sr, int64_t sc, int64_t sb, int64_t out_pitch, cudaStream_t st) {
  if (rows == 0 || cols == 0 || batch == 0) return MT_OK;
  if (batch > 65535 || (rows + 31) / 32 > 65535) return fail(MT_ERR_UNSUPPORTED, "pack2d: grid too large");
  dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch), block(32, 8);
  switch (dtype) {
    case MT_F32:
      pack2d_kernel<float><<<grid, block, 0, st>>>((float*)out, lo, (const float*)in, rows, cols, sr, sc, sb, out_pitch);
      break;
    case MT_BF16:
      pack2d_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((__nv_bfloat16*)out, nullptr, (const __nv_bfloat16*)in,
                                                            rows, cols, sr, sc, sb, out_pitch);
      break;
    case MT_F16:
      pack2d_kernel<__half><<<grid, block, 0, st>>>((__half*)out, nullptr, (const __half*)in, rows, cols, sr, sc, sb,
                                                     out_pitch);
      break;
    default: return fail(MT_ERR_UNSUPPORTED, "pack2d: dtype");
  }
  return check_launch("pack2d");
}

int launch_conv_pack_weight(void* out, float* lo, const void* w, int dtype, int64_t K, int64_t C, int64_t R,
                            int64_t S, int64_t Cp, cudaStream_t st) {
  const int64_t n = K * R * S * Cp;
  if (n == 0) return MT_OK;
  switch (dtype) {
    case MT_F32:
      conv_pack_weight_kernel<float><<<grid_for(n, 256), 256, 0, st>>>((float*)out, lo, (const float*)w, K, C, R, S, Cp);
      break;
    case MT_BF16:
      conv_pack_weight_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, st>>>(
          (__nv_bfloat16*)out, nullptr, (const __nv_bfloat16*)w, K, C, R, S, Cp);
      break;
    case MT_F16:
      conv_pack_weight_kernel<__half><<<grid_for(n, 256), 256, 0, st>>>((__half*)out, nullptr, (const __half*)w, K,
                                                                         C, R, S, Cp);
      break;
    default: return fail(MT_ERR_UNSUPPORTED, "conv weight pack: dtype");
  }
  return check_launch("conv_pack_weight");
}

int launch_im2col(void* col, float* lo, const void* x, int dtype, const mt_conv2d_desc& d, int64_t Cp, int64_t Kp,
                  cudaStream_t st) {
  const int64_t n = d.N * d.P * d.Q * Kp;
  if (n == 0) return MT_OK;
#define MT_IM2COL(T)                                                                                            \
  im2col_kernel<T><<<grid_for(n, 256), 256, 0, st>>>((T*)col, lo, (const T*)x, d.N, d.C, d.H, d.W, d.P, d.Q,    \
                                                      (int)d.R, (int)d.S, d.stride_h, d.stride_w, d.pad_h, d.pad_w, \
                                                      d.dil_h, d.dil_w, d.x_strides[0], d.x_strides[1],         \
                                                      d.x_strides[2], d.x_strides[3], Cp, Kp)
  switch (dtype) {
    case MT_F32: MT_IM2COL(float); break;
    case MT_BF16: MT_IM2COL(__nv_bfloat16); break;
    case MT_F16: MT_IM2COL(__half); break;
    default: return fail(MT_ERR_UNSUPPORTED, "im2col: dtype");
  }
#undef MT_IM2COL
  return check_launch("im2col");
}

}  // namespace mt
