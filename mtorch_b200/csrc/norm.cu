// Row softmax, layer norm and group norm (+ fused SiLU).  HBM-bound; fp32 arithmetic with
// fp64 combination of group-norm partial sums.
#include <mutex>

#include "runtime.h"

namespace mt {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t = fmaxf(t, red[i]);
  return t;
}

// ---------------------------------------------------------------------------------------------
// Softmax over contiguous rows.  Rows of up to NT*PER elements stay in registers (one read,
// one write); longer rows take three passes.
template <int NT, int PER>
__global__ void __launch_bounds__(NT) softmax_kernel(void* y, int yd, const void* x, int xd, int64_t cols, int64_t ld,
                                                     int log_output) {
  __shared__ float red[NT / 32];
  const int64_t base = (int64_t)blockIdx.x * ld;
  const bool cached = cols <= (int64_t)NT * PER;
  float vals[PER];
  float m = -INFINITY;
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      vals[i] = c < cols ? load_as_f32(x, base + c, xd) : -INFINITY;
      m = fmaxf(m, vals[i]);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) m = fmaxf(m, load_as_f32(x, base + c, xd));
  }
  m = block_max<NT>(m, red);
  float s = 0.f;
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      if (c < cols) s += expf(vals[i] - m);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) s += expf(load_as_f32(x, base + c, xd) - m);
  }
  s = block_sum<NT>(s, red);
  const float inv = 1.0f / s, ls = logf(s);
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      if (c < cols) store_from_f32(y, base + c, yd, log_output ? vals[i] - m - ls : expf(vals[i] - m) * inv);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) {
      const float v = load_as_f32(x, base + c, xd);
      store_from_f32(y, base + c, yd, log_output ? v - m - ls : expf(v - m) * inv);
    }
  }
}

int launch_softmax(void* y, int yd, const void* x, int xd, int64_t rows, int64_t cols, int64_t ld, int log_output,
                   cudaStream_t st) {
  if (rows == 0 || cols == 0) return MT_OK;
  if (rows > 0x7fffffffLL) return fail(MT_ERR_UNSUPPORTED, "softmax: too many rows");
  if (cols <= 1024)
    softmax_kernel<128, 8><<<(unsigned)rows, 128, 0, st>>>(y, yd, x, xd, cols, ld, log_output);
  else
    softmax_kernel<256, 16><<<(unsigned)rows, 256, 0, st>>>(y, yd, x, xd, cols, ld, log_output);
  return check_launch("softmax");
}

// ---------------------------------------------------------------------------------------------
// LayerNorm over the last `cols` elements (two-pass mean / variance in registers).
template <int NT, int PER>
__global__ void __launch_bounds__(NT) layer_norm_kernel(void* y, int yd, const void* x, int xd, const void* w,
                                                        const void* b, int wbd, int64_t cols, float eps) {
  __shared__ float red[NT / 32];
  const int64_t base = (int64_t)blockIdx.x * cols;
  const bool cached = cols <= (int64_t)NT * PER;
  float vals[PER];
  float s = 0.f;
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      vals[i] = c < cols ? load_as_f32(x, base + c, xd) : 0.f;
      s += vals[i];
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) s += load_as_f32(x, base + c, xd);
  }
  const float mean = block_sum<NT>(s, red) / (float)cols;
  float q = 0.f;
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      if (c < cols) q += (vals[i] - mean) * (vals[i] - mean);
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) {
      const float d = load_as_f32(x, base + c, xd) - mean;
      q += d * d;
    }
  }
  const float var = block_sum<NT>(q, red) / (float)cols;
  const float inv = rsqrtf(var + eps);
  if (cached) {
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * NT;
      if (c < cols) {
        float v = (vals[i] - mean) * inv;
        if (w) v *= load_as_f32(w, c, wbd);
        if (b) v += load_as_f32(b, c, wbd);
        store_from_f32(y, base + c, yd, v);
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < cols; c += NT) {
      float v = (load_as_f32(x, base + c, xd) - mean) * inv;
      if (w) v *= load_as_f32(w, c, wbd);
      if (b) v += load_as_f32(b, c, wbd);
      store_from_f32(y, base + c, yd, v);
    }
  }
}

// Eight consecutive affine parameters starting at c0 (a multiple of 8) as floats: one 16-byte load
// for bf16, two for fp32 when the array is 16-byte aligned, else element by element.
__device__ __forceinline__ void load8_f32(const void* p, int dtype, int c0, float (&o)[8]) {
  const bool al = (reinterpret_cast<uintptr_t>(p) & 15) == 0;
  if (dtype == MT_BF16 && al) {
    const uint4 u = reinterpret_cast<const uint4*>(p)[c0 / 8];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      o[2 * j] = f.x;
      o[2 * j + 1] = f.y;
    }
  } else if (dtype == MT_F32 && al) {
    const float4 a = reinterpret_cast<const float4*>(p)[c0 / 4], b = reinterpret_cast<const float4*>(p)[c0 / 4 + 1];
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = load_as_f32(p, c0 + j, dtype);
  }
}

// bf16 rows of cols = 8*k elements, LPR lanes per row (16 or 32; 32 / LPR rows per warp), VPL
// 16-byte vectors per lane with VPL = ceil(cols / 8 / LPR), so few lanes idle (320 columns: 16
// lanes x 3 vectors).  Rows held in registers, two-pass mean / variance reduced within the row's
// lane group, affine parameters loaded 8 at a time, 16-byte stores.
template <int VPL, int LPR>
__global__ void __launch_bounds__(256) layer_norm_bf16_sub_kernel(__nv_bfloat16* y, const __nv_bfloat16* x,
                                                                  const void* w, const void* b, int wbd, int64_t rows,
                                                                  int cols, float eps) {
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const int64_t row = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * RPW + sub;
  const bool live = row < rows;
  const int nv = cols / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x + (live ? row : 0) * cols);
  float v[VPL][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int vi = l + LPR * k;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (live && vi < nv) u = src[vi];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[k][2 * j] = f.x;
      v[k][2 * j + 1] = f.y;
      s += f.x + f.y;
    }
  }
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / (float)cols;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < VPL; ++k)
    if (l + LPR * k < nv)
#pragma unroll
      for (int j = 0; j < 8; ++j) q += (v[k][j] - mean) * (v[k][j] - mean);
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float inv = rsqrtf(q / (float)cols + eps);
  if (!live) return;
  uint4* dst = reinterpret_cast<uint4*>(y + row * cols);
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int vi = l + LPR * k;
    if (vi >= nv) continue;
    float gw[8], gb[8];
    if (w) {
      load8_f32(w, wbd, vi * 8, gw);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) gw[j] = 1.f;
    }
    if (b) {
      load8_f32(b, wbd, vi * 8, gb);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) gb[j] = 0.f;
    }
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2((v[k][2 * j] - mean) * inv * gw[2 * j] + gb[2 * j],
                         (v[k][2 * j + 1] - mean) * inv * gw[2 * j + 1] + gb[2 * j + 1]);
    dst[vi] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Persistent variant of layer_norm_bf16_sub_kernel for rows of 5 * LPR vectors: a grid of three
// CTAs per SM walks row groups (8 warps x 32 / LPR rows) with a stride of the grid, keeps the
// next group's loads in flight while it reduces and stores the current one, and reads gamma /
// beta (as fp32) from shared memory filled once per CTA.  The per-row arithmetic is the same
// sequence as layer_norm_bf16_sub_kernel's.
template <int VPL, int LPR>
__global__ void __launch_bounds__(256, 3) layer_norm_bf16_persist_kernel(__nv_bfloat16* y, const __nv_bfloat16* x,
                                                                      const void* w, const void* b, int wbd,
                                                                      int64_t rows, int cols, float eps) {
  extern __shared__ float ln_wb[];  // [2][cols]
  constexpr int RPW = 32 / LPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, l = lane % LPR;
  const int nv = cols / 8;
  for (int c = threadIdx.x; c < cols; c += 256) {
    ln_wb[c] = w ? load_as_f32(w, c, wbd) : 1.f;
    ln_wb[cols + c] = b ? load_as_f32(b, c, wbd) : 0.f;
  }
  __syncthreads();
  const int64_t groups = (rows + 8 * RPW - 1) / (8 * RPW);
  auto load = [&](int64_t g, uint4 (&u)[VPL]) {
    const int64_t row = (g * 8 + (threadIdx.x >> 5)) * RPW + sub;
    const uint4* src = reinterpret_cast<const uint4*>(x + row * cols);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int vi = l + LPR * k;
      u[k] = (g < groups && row < rows && vi < nv) ? __ldcs(src + vi) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  uint4 cur[VPL], nxt[VPL];
  int64_t g = blockIdx.x;
  load(g, cur);
  for (; g < groups; g += gridDim.x) {
    load(g + gridDim.x, nxt);
    const int64_t row = (g * 8 + (threadIdx.x >> 5)) * RPW + sub;
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        s += f.x + f.y;
      }
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)cols;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < VPL; ++k)
      if (l + LPR * k < nv) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[k]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          q += (f.x - mean) * (f.x - mean);
          q += (f.y - mean) * (f.y - mean);
        }
      }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = rsqrtf(q / (float)cols + eps);
    if (row < rows) {
      uint4* dst = reinterpret_cast<uint4*>(y + row * cols);
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int vi = l + LPR * k;
        if (vi >= nv) continue;
        const float4* wv = reinterpret_cast<const float4*>(ln_wb + vi * 8);
        const float4* bv = reinterpret_cast<const float4*>(ln_wb + cols + vi * 8);
        const float4 w0 = wv[0], w1 = wv[1], b0 = bv[0], b1 = bv[1];
        const float gw[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const float gb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&cur[k]);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          o[j] = pack_bf16x2((f.x - mean) * inv * gw[2 * j] + gb[2 * j],
                             (f.y - mean) * inv * gw[2 * j + 1] + gb[2 * j + 1]);
        }
        __stcs(dst + vi, make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
#pragma unroll
    for (int k = 0; k < VPL; ++k) cur[k] = nxt[k];
  }
}

int launch_layer_norm(void* y, int yd, const void* x, int xd, const void* w, const void* b, int wbd, int64_t rows,
                      int64_t cols, double eps, cudaStream_t st) {
  if (rows == 0 || cols == 0) return MT_OK;
  if (rows > 0x7fffffffLL) return fail(MT_ERR_UNSUPPORTED, "layer_norm: too many rows");
  if (xd == MT_BF16 && yd == MT_BF16 && cols % 8 == 0 && cols <= 8 * 32 * 8 && (uintptr_t)x % 16 == 0 &&
      (uintptr_t)y % 16 == 0 && rows / 8 < 0x7fffffffLL) {
    const int nv = (int)(cols / 8);
    const unsigned g32 = (unsigned)((rows + 7) / 8), g16 = (unsigned)((rows + 15) / 16);
    auto* yy = (__nv_bfloat16*)y;
    auto* xx = (const __nv_bfloat16*)x;
    // rows of 5 * LPR vectors (the UNet's 320 / 640 / 1280 columns): 5 vectors per lane, no idle
    // lanes (320 columns x 262144 rows: 75 us against 85 us for 3 vectors on 16 lanes); MT_LN_V5=0
    // restores the general mapping
    static const bool v5 = [] {
      const char* e = getenv("MT_LN_V5");
      return !(e && e[0] == '0');
    }();
    // persistent grid-stride variant of the same mapping (MT_LN_PERSIST=0 turns it off)
    static const bool persist = [] {
      const char* e = getenv("MT_LN_PERSIST");
      return !(e && e[0] == '0');
    }();
    if (v5 && persist && nv % 5 == 0 && (nv / 5 == 8 || nv / 5 == 16 || nv / 5 == 32)) {
      const int lpr = nv / 5, rpc = 8 * (32 / lpr);
      const int64_t groups = (rows + rpc - 1) / rpc;
      const size_t sh = 2 * (size_t)cols * sizeof(float);
      const unsigned grid = (unsigned)std::min<int64_t>(groups, (int64_t)num_sms() * 3);  // 3 resident per SM
      if (lpr == 8)
        layer_norm_bf16_persist_kernel<5, 8><<<grid, 256, sh, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      else if (lpr == 16)
        layer_norm_bf16_persist_kernel<5, 16><<<grid, 256, sh, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      else
        layer_norm_bf16_persist_kernel<5, 32><<<grid, 256, sh, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      return check_launch("layer_norm_bf16_persist");
    }
    if (v5 && nv % 5 == 0 && (nv / 5 == 8 || nv / 5 == 16 || nv / 5 == 32)) {
      const unsigned g8 = (unsigned)((rows + 31) / 32);
      if (nv / 5 == 8)
        layer_norm_bf16_sub_kernel<5, 8><<<g8, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      else if (nv / 5 == 16)
        layer_norm_bf16_sub_kernel<5, 16><<<g16, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      else
        layer_norm_bf16_sub_kernel<5, 32><<<g32, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
      return check_launch("layer_norm_bf16_warp");
    }
    if (nv <= 16)
      layer_norm_bf16_sub_kernel<1, 16><<<g16, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else if (nv <= 32)
      layer_norm_bf16_sub_kernel<2, 16><<<g16, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else if (nv <= 48)
      layer_norm_bf16_sub_kernel<3, 16><<<g16, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else if (nv <= 96)
      layer_norm_bf16_sub_kernel<3, 32><<<g32, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else if (nv <= 128)
      layer_norm_bf16_sub_kernel<4, 32><<<g32, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else if (nv <= 160)
      layer_norm_bf16_sub_kernel<5, 32><<<g32, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    else
      layer_norm_bf16_sub_kernel<8, 32><<<g32, 256, 0, st>>>(yy, xx, w, b, wbd, rows, (int)cols, (float)eps);
    return check_launch("layer_norm_bf16_warp");
  }
  if (cols <= 512)
    layer_norm_kernel<64, 8><<<(unsigned)rows, 64, 0, st>>>(y, yd, x, xd, w, b, wbd, cols, (float)eps);
  else
    layer_norm_kernel<128, 16><<<(unsigned)rows, 128, 0, st>>>(y, yd, x, xd, w, b, wbd, cols, (float)eps);
  return check_launch("layer_norm");
}

// ---------------------------------------------------------------------------------------------
// GroupNorm: (1) per-(image, chunk) partial sums per group, (2) per-(image, group) mean / rstd
// combined in double in a fixed order, (3) normalise + affine (+ SiLU).  The chunking depends
// only on the per-image problem, never on N, so an image's result is the same whatever the batch
// size or its position in the batch.
//
// Channels-last input ([N, HW, C] with C contiguous): a CTA walks a chunk of 64 pixels; each
// (pixel lane, channel) slot is owned by one thread; per-group sums are formed in shared memory.
// NCHW input ([N, C, HW] with HW contiguous): a CTA reduces a 4096-element slice of one group.
constexpr int kGnThreads = 256;
constexpr int kGnMaxChunks = 1024;

__global__ void __launch_bounds__(kGnThreads) gn_partial_cl_kernel(const void* x, int xd, int64_t sn, int64_t spix,
                                                                   int64_t C, int64_t HW, int64_t G, int chunks,
                                                                   double* part) {
  extern __shared__ float gn_sh[];  // [2][slots]
  const int n = blockIdx.y, chunk = blockIdx.x;
  const int64_t per = (HW + chunks - 1) / chunks;
  const int64_t p0 = chunk * per, p1 = min(HW, p0 + per);
  const int64_t lanes = C >= kGnThreads ? 1 : kGnThreads / C;
  const int64_t slots = lanes * C;
  for (int64_t t = threadIdx.x; t < slots; t += kGnThreads) {
    const int64_t lane = t / C, c = t % C;
    float s = 0.f, q = 0.f;
    for (int64_t p = p0 + lane; p < p1; p += lanes) {
      const float v = load_as_f32(x, n * sn + p * spix + c, xd);
      s += v;
      q += v * v;
    }
    gn_sh[t] = s;
    gn_sh[slots + t] = q;
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < C; c += kGnThreads) {
    float s = 0.f, q = 0.f;
    for (int64_t l = 0; l < lanes; ++l) {
      s += gn_sh[l * C + c];
      q += gn_sh[slots + l * C + c];
    }
    gn_sh[c] = s;
    gn_sh[slots + c] = q;
  }
  __syncthreads();
  const int64_t Cg = C / G;
  for (int64_t g = threadIdx.x; g < G; g += kGnThreads) {
    double s = 0.0, q = 0.0;
    for (int64_t c = g * Cg; c < (g + 1) * Cg; ++c) {
      s += gn_sh[c];
      q += gn_sh[slots + c];
    }
    double* o = part + (((int64_t)n * chunks + chunk) * G + g) * 2;
    o[0] = s;
    o[1] = q;
  }
}

// Channels-last bf16 partial sums, 8 channels (16 bytes) per load: V = C/8 vectors per pixel,
// thread t owns vector t % V of pixel lane t / V; one (lane, channel) slot per thread and
// channel in shared memory keeps the reduction order fixed.
//
// TWO: the input is the channel concatenation of x (C1 channels per pixel, image stride sn) and
// x2 (C - C1 channels, image stride sn2), read in place.
template <bool TWO = false, int U = 4>
__global__ void __launch_bounds__(kGnThreads, 5) gn_partial_cl_bf16x8_kernel(const __nv_bfloat16* x, int64_t sn,
                                                                          int64_t C, int64_t HW, int64_t G,
                                                                          int chunks, double* part,
                                                                          const __nv_bfloat16* x2 = nullptr,
                                                                          int64_t sn2 = 0, int64_t C1 = 0) {
  extern __shared__ float gn_sh[];  // [2][lanes * C]
  const int n = blockIdx.y, chunk = blockIdx.x;
  const int64_t per = (HW + chunks - 1) / chunks;
  const int64_t p0 = chunk * per, p1 = min(HW, p0 + per);
  const int64_t V = C / 8;
  const int64_t lanes = V >= kGnThreads ? 1 : kGnThreads / V;
  const int64_t slots = lanes * C;
  const __nv_bfloat16* xb = x + (int64_t)n * sn;
  for (int64_t t = threadIdx.x; t < lanes * V; t += kGnThreads) {
    const int64_t lane = t / V, v = t % V;
    float s[8], q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = q[j] = 0.f;
    // four pixels' 16-byte loads in flight per thread (those past the chunk read as zero)
    const __nv_bfloat16* xv = xb + v * 8;
    int64_t pitch = C;
    if (TWO) {
      if (v * 8 < C1) {
        pitch = C1;
      } else {
        xv = x2 + (int64_t)n * sn2 + (v * 8 - C1);
        pitch = C - C1;
      }
    }
    for (int p = (int)(p0 + lane); p < p1; p += U * (int)lanes) {
      uint4 u[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int pp = p + k * (int)lanes;
        u[k] = pp < p1 ? *reinterpret_cast<const uint4*>(xv + (int64_t)pp * pitch) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[k]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          s[2 * j] += f.x;
          q[2 * j] = __fmaf_rn(f.x, f.x, q[2 * j]);
          s[2 * j + 1] += f.y;
          q[2 * j + 1] = __fmaf_rn(f.y, f.y, q[2 * j + 1]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      gn_sh[lane * C + v * 8 + j] = s[j];
      gn_sh[slots + lane * C + v * 8 + j] = q[j];
    }
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < C; c += kGnThreads) {
    float s = 0.f, q = 0.f;
    for (int64_t l = 0; l < lanes; ++l) {
      s += gn_sh[l * C + c];
      q += gn_sh[slots + l * C + c];
    }
    gn_sh[c] = s;
    gn_sh[slots + c] = q;
  }
  __syncthreads();
  const int64_t Cg = C / G;
  for (int64_t g = threadIdx.x; g < G; g += kGnThreads) {
    double s = 0.0, q = 0.0;
    for (int64_t c = g * Cg; c < (g + 1) * Cg; ++c) {
      s += gn_sh[c];
      q += gn_sh[slots + c];
    }
    double* o = part + (((int64_t)n * chunks + chunk) * G + g) * 2;
    o[0] = s;
    o[1] = q;
  }
}

// Persistent variant of gn_partial_cl_bf16x8_kernel for C <= 2048 (one (lane, vector) slot per
// thread): a grid of four CTAs per SM deals the (image, chunk) items round-robin, and while a
// CTA reduces one item's slots it already has the next item's first U loads in flight.  Every
// slot sums the same pixels in the same order as gn_partial_cl_bf16x8_kernel (batch k of U
// pixels, zeros past the chunk), and the channel / group sums are the same loops, so the
// partials are bitwise equal to it.
template <bool TWO = false, int U = 4>
__global__ void __launch_bounds__(kGnThreads, 4) gn_partial_cl_bf16x8_persist_kernel(
    const __nv_bfloat16* x, int64_t sn, int64_t C, int64_t HW, int64_t G, int chunks, int items, double* part,
    const __nv_bfloat16* x2 = nullptr, int64_t sn2 = 0, int64_t C1 = 0) {
  extern __shared__ float gn_sh[];  // [2][lanes * C]
  const int64_t per = (HW + chunks - 1) / chunks;
  const int V = (int)(C / 8);
  const int lanes = V >= kGnThreads ? 1 : kGnThreads / V;
  const int64_t slots = (int64_t)lanes * C;
  const int t = threadIdx.x;
  const bool act = t < lanes * V;
  const int lane = t / V, v = t % V;
  // this thread's channel vector: its source, pitch between pixels and image stride
  const __nv_bfloat16* src = x + v * 8;
  int64_t pitch = C, istride = sn;
  if (TWO) {
    if (v * 8 < C1) {
      pitch = C1;
    } else {
      src = x2 + (v * 8 - C1);
      pitch = C - C1;
      istride = sn2;
    }
  }
  uint4 u[U];
  auto load_batch = [&](int item, int p) {
    const int n = item / chunks, chunk = item % chunks;
    const int64_t p1 = min(HW, chunk * per + per);
    const __nv_bfloat16* xv = src + (int64_t)n * istride;
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int pp = p + k * lanes;
      u[k] = pp < p1 ? *reinterpret_cast<const uint4*>(xv + (int64_t)pp * pitch) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  int item = blockIdx.x;
  if (act && item < items) load_batch(item, (int)((item % chunks) * per) + lane);
  for (; item < items; item += gridDim.x) {
    const int n = item / chunks, chunk = item % chunks;
    const int64_t p0 = chunk * per, p1 = min(HW, p0 + per);
    if (act) {
      float s[8], q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = q[j] = 0.f;
      for (int p = (int)(p0 + lane);;) {
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[k]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            s[2 * j] += f.x;
            q[2 * j] = __fmaf_rn(f.x, f.x, q[2 * j]);
            s[2 * j + 1] += f.y;
            q[2 * j + 1] = __fmaf_rn(f.y, f.y, q[2 * j + 1]);
          }
        }
        p += U * lanes;
        if (p >= p1) break;
        load_batch(item, p);
      }
      // the next item's first batch goes out before this item's reduction
      const int nxt = item + gridDim.x;
      if (nxt < items) load_batch(nxt, (int)((nxt % chunks) * per) + lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        gn_sh[lane * C + v * 8 + j] = s[j];
        gn_sh[slots + lane * C + v * 8 + j] = q[j];
      }
    }
    __syncthreads();
    for (int64_t c = t; c < C; c += kGnThreads) {
      float s = 0.f, q = 0.f;
      for (int64_t l = 0; l < lanes; ++l) {
        s += gn_sh[l * C + c];
        q += gn_sh[slots + l * C + c];
      }
      gn_sh[c] = s;
      gn_sh[slots + c] = q;
    }
    __syncthreads();
    const int64_t Cg = C / G;
    for (int64_t g = t; g < G; g += kGnThreads) {
      double s = 0.0, q = 0.0;
      for (int64_t c = g * Cg; c < (g + 1) * Cg; ++c) {
        s += gn_sh[c];
        q += gn_sh[slots + c];
      }
      double* o = part + (((int64_t)n * chunks + chunk) * G + g) * 2;
      o[0] = s;
      o[1] = q;
    }
    __syncthreads();
  }
}

// Per-(image, channel) affine of the normalisation: y = x * a + b with a = rstd * gamma and
// b = beta - mean * a, so the apply pass needs no division or group lookup.
__global__ void gn_table_kernel(const float* stats, const void* w, const void* b, int wbd, int64_t N, int64_t C,
                                int64_t G, float2* tab) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= N * C) return;
  const int64_t n = i / C, c = i % C;
  const float* st = stats + (n * G + c / (C / G)) * 2;
  float a = st[1], sh = -st[0] * st[1];
  if (w) {
    const float gm = load_as_f32(w, c, wbd);
    a *= gm;
    sh *= gm;
  }
  if (b) sh += load_as_f32(b, c, wbd);
  tab[i] = make_float2(a, sh);
}

// SiLU for results rounded to bf16: x * sigmoid(x) = h + h * tanh(h) with h = x / 2, one MUFU
// operation (tanh.approx, relative error ~2^-11, below bf16's 2^-8 rounding) instead of two.
__device__ __forceinline__ float silu_bf16out(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return __fmaf_rn(h, t, h);
}

// (a, b) of channel c for y = x * a + b: a = rstd * gamma, b = beta - mean * rstd * gamma, each
// product and sum rounded on its own (no contraction), so every kernel gets the same bits.
__device__ __forceinline__ float2 gn_affine(float rstd, float mf, const void* w, const void* b, int wbd, int64_t c) {
  float a = rstd, sh = __fmul_rn(-mf, rstd);
  if (w) {
    const float gm = load_as_f32(w, c, wbd);
    a = __fmul_rn(a, gm);
    sh = __fmul_rn(sh, gm);
  }
  if (b) sh = __fadd_rn(sh, load_as_f32(b, c, wbd));
  return make_float2(a, sh);
}

__device__ __forceinline__ float2 gn_affine_v(float rstd, float mf, bool has_w, float gm, bool has_b, float be) {
  float a = rstd, sh = __fmul_rn(-mf, rstd);
  if (has_w) {
    a = __fmul_rn(a, gm);
    sh = __fmul_rn(sh, gm);
  }
  if (has_b) sh = __fadd_rn(sh, be);
  return make_float2(a, sh);
}

// Finalize + affine table in one pass: one warp per (image, group).  Lane l sums chunks l, l+32,
// ... in double, then a fixed xor-shuffle tree combines the lanes, so the result depends only on
// the per-image chunking (not on N) and is the same on every run.  The warp then writes the
// (a, b) pairs of the group's channels: y = x * a + b.
__global__ void gn_finalize_table_kernel(const double* part, const void* w, const void* b, int wbd, int64_t N,
                                         int64_t C, int64_t G, int chunks, double count, double eps, float2* tab) {
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= N * G) return;
  const int64_t n = i / G, g = i % G;
  double s = 0, q = 0;
  for (int c = lane; c < chunks; c += 32) {
    const double* p = part + ((n * chunks + c) * G + g) * 2;
    s += p[0];
    q += p[1];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  const double mean = s / count;
  double var = q / count - mean * mean;
  if (var < 0) var = 0;
  const float rstd = (float)(1.0 / sqrt(var + eps)), mf = (float)mean;
  const int64_t Cg = C / G;
  for (int64_t c = g * Cg + lane; c < (g + 1) * Cg; c += 32) {
    tab[n * C + c] = gn_affine(rstd, mf, w, b, wbd, c);
  }
}

// Apply with one grid row per image and a grid stride that is a multiple of C/8: every thread
// always meets the same 8 channels, so it holds their (a, b) pairs in registers and each 16 bytes
// of x cost one load and one store.  32-bit indexing inside the image (HW * C / 8 < 2^31).
// TWO: x is the concatenation of x (C1 = 8 * c1_8 channels per pixel) and x2 (C - C1 channels),
// both dense channels-last; the thread's fixed channel vector decides which source it reads.
template <bool TWO = false>
__global__ void __launch_bounds__(256) gn_apply_img_bf16x8_kernel(__nv_bfloat16* y, const __nv_bfloat16* x,
                                                                  const float2* tab, int per_img8, int C8, int silu,
                                                                  const __nv_bfloat16* x2 = nullptr, int c1_8 = 0) {
  const int64_t n = blockIdx.y;
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
  const int stride = gridDim.x * blockDim.x;
  const int c8 = i0 % C8;
  // source vector of element vector i: pixel i / C8 at channel vector c8 of its source; the stride
  // is a multiple of C8, so the pixel advances by stride / C8 per iteration
  const uint4* xi;
  int src_c8 = C8, src_off = c8;
  if (TWO) {
    const int c2_8 = C8 - c1_8;
    if (c8 < c1_8) {
      xi = reinterpret_cast<const uint4*>(x) + n * (int64_t)per_img8 / C8 * c1_8;
      src_c8 = c1_8;
    } else {
      xi = reinterpret_cast<const uint4*>(x2) + n * (int64_t)per_img8 / C8 * c2_8;
      src_c8 = c2_8;
      src_off = c8 - c1_8;
    }
  } else {
    xi = reinterpret_cast<const uint4*>(x) + n * per_img8;
  }
  uint4* yi = reinterpret_cast<uint4*>(y) + n * per_img8;
  const float4* t = reinterpret_cast<const float4*>(tab + n * C8 * 8) + c8 * 4;
  float4 ab[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) ab[j] = t[j];  // (a0, b0, a1, b1) for channel pairs 2j, 2j+1
  const int pix_step = stride / C8;
  int pix = i0 / C8;
  // four 16-byte loads in flight per thread (issued before any of their stores)
  constexpr int U = 4;
  for (int64_t i = i0; i < per_img8; i += (int64_t)U * stride, pix += U * pix_step) {
    uint4 v[U];
#pragma unroll
    for (int k = 0; k < U; ++k)
      if (i + (int64_t)k * stride < per_img8)
        v[k] = TWO ? xi[(int64_t)(pix + k * pix_step) * src_c8 + src_off] : xi[i + (int64_t)k * stride];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      if (i + (int64_t)k * stride >= per_img8) break;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        float r0 = __fmaf_rn(f.x, ab[j].x, ab[j].y), r1 = __fmaf_rn(f.y, ab[j].z, ab[j].w);
        if (silu) {
          r0 = silu_bf16out(r0);
          r1 = silu_bf16out(r1);
        }
        h[j] = __floats2bfloat162_rn(r0, r1);
      }
      yi[i + (int64_t)k * stride] = v[k];
    }
  }
}

__global__ void gn_apply_cl_bf16x8_tab_kernel(__nv_bfloat16* y, const __nv_bfloat16* x, const float2* tab, int64_t HW,
                                              int64_t C, int64_t total8, int silu) {
  const int64_t C8 = C / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c8 = i % C8;
    const int64_t n = i / (HW * C8);
    uint4 v = reinterpret_cast<const uint4*>(x)[i];
    const float4* t = reinterpret_cast<const float4*>(tab + n * C + c8 * 8);
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 ab = t[j];  // (a0, b0, a1, b1)
      float2 f = __bfloat1622float2(h[j]);
      float r0 = f.x * ab.x + ab.y, r1 = f.y * ab.z + ab.w;
      if (silu) {
        r0 = silu_bf16out(r0);
        r1 = silu_bf16out(r1);
      }
      h[j] = __floats2bfloat162_rn(r0, r1);
    }
    reinterpret_cast<uint4*>(y)[i] = v;
  }
}

__global__ void __launch_bounds__(kGnThreads) gn_partial_nchw_kernel(const void* x, int xd, int64_t sn, int64_t sc,
                                                                     int64_t C, int64_t HW, int64_t G, int chunks,
                                                                     double* part) {
  __shared__ double red[2][kGnThreads / 32];
  const int64_t ng = blockIdx.y;  // n * G + g
  const int64_t n = ng / G, g = ng % G;
  const int64_t Cg = C / G;
  const int64_t len = Cg * HW;
  const int64_t per = (len + chunks - 1) / chunks;
  const int64_t e0 = blockIdx.x * per, e1 = min(len, e0 + per);
  float s = 0.f, q = 0.f;
  for (int64_t e = e0 + threadIdx.x; e < e1; e += kGnThreads) {
    const int64_t c = g * Cg + e / HW, p = e % HW;
    const float v = load_as_f32(x, n * sn + c * sc + p, xd);
    s += v;
    q += v * v;
  }
  double ds = warp_sum_d((double)s), dq = warp_sum_d((double)q);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][w] = ds;
    red[1][w] = dq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0, tq = 0;
    for (int i = 0; i < kGnThreads / 32; ++i) {
      ts += red[0][i];
      tq += red[1][i];
    }
    double* o = part + ((n * chunks + blockIdx.x) * G + g) * 2;
    o[0] = ts;
    o[1] = tq;
  }
}

__global__ void gn_finalize_kernel(const double* part, float* stats, int64_t N, int64_t G, int chunks, double count,
                                   double eps) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= N * G) return;
  const int64_t n = i / G, g = i % G;
  double s = 0, q = 0;
  for (int c = 0; c < chunks; ++c) {
    const double* p = part + ((n * chunks + c) * G + g) * 2;
    s += p[0];
    q += p[1];
  }
  const double mean = s / count;
  double var = q / count - mean * mean;
  if (var < 0) var = 0;
  stats[i * 2] = (float)mean;
  stats[i * 2 + 1] = (float)(1.0 / sqrt(var + eps));
}

// Channels-last bf16 apply: 8 channels per thread (16-byte loads / stores).
__global__ void gn_apply_cl_bf16x8_kernel(__nv_bfloat16* y, const __nv_bfloat16* x, const float* stats,
                                          const void* w, const void* b, int wbd, int64_t N, int64_t HW, int64_t C,
                                          int64_t G, int silu) {
  const int64_t C8 = C / 8, Cg = C / G;
  const int64_t total = N * HW * C8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t c0 = (i % C8) * 8;
    const int64_t n = i / (HW * C8);
    uint4 v = reinterpret_cast<const uint4*>(x)[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      float o[2] = {f.x, f.y};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t c = c0 + 2 * j + k;
        const float* stt = stats + (n * G + c / Cg) * 2;
        float r = (o[k] - stt[0]) * stt[1];
        if (w) r *= load_as_f32(w, c, wbd);
        if (b) r += load_as_f32(b, c, wbd);
        if (silu) r = silu_f(r);
        o[k] = r;
      }
      h[j] = __floats2bfloat162_rn(o[0], o[1]);
    }
    reinterpret_cast<uint4*>(y)[i] = v;
  }
}

// Generic apply: logical [N, C, HW] with separate x / y strides.
__global__ void gn_apply_generic_kernel(void* y, int yd, int64_t ys0, int64_t ys1, int64_t ys2, const void* x, int xd,
                                        int64_t xs0, int64_t xs1, int64_t xs2, const float* stats, const void* w,
                                        const void* b, int wbd, int64_t N, int64_t C, int64_t HW, int64_t G, int silu,
                                        int channels_inner) {
  const int64_t total = N * C * HW, Cg = C / G;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t n, c, p;
    if (channels_inner) {
      c = i % C; p = (i / C) % HW; n = i / (C * HW);
    } else {
      p = i % HW; c = (i / HW) % C; n = i / (C * HW);
    }
    const float* stt = stats + (n * G + c / Cg) * 2;
    float v = (load_as_f32(x, n * xs0 + c * xs1 + p * xs2, xd) - stt[0]) * stt[1];
    if (w) v *= load_as_f32(w, c, wbd);
    if (b) v += load_as_f32(b, c, wbd);
    if (silu) v = silu_f(v);
    store_from_f32(y, n * ys0 + c * ys1 + p * ys2, yd, v);
  }
}

// Bytes of input per image group of the channels-last bf16 path: MT_GN_L2_GROUP_MB > 0 processes
// the batch in groups of that size so that the apply pass re-reads x from L2.  Off by default:
// measured at 320 channels x 64x64 x 64 images it took 265 us against 124 us for the whole batch
// at once (three dependent launches per group, and groups too small to fill the GPU).
static int64_t gn_l2_group_bytes() {
  static const int64_t v = [] {
    const char* e = getenv("MT_GN_L2_GROUP_MB");
    return (int64_t)(e ? atof(e) * (1 << 20) : 0.0);
  }();
  return v;
}

// Pixels per statistics chunk of the vectorised channels-last path: 40960 / C (128 at 320
// channels, 32 at 1280; between 16 and 128), or MT_GN_PX.  A function of C only, so the
// reduction order never depends on the batch.
static int64_t gn_chunk_px(int64_t C) {
  static const int64_t px_env = [] {
    const char* e = getenv("MT_GN_PX");
    return (int64_t)(e ? atoi(e) : 0);
  }();
  return px_env > 0 ? px_env : std::max<int64_t>(16, std::min<int64_t>(128, 40960 / C));
}

static int gn_chunks(int64_t C, int64_t HW, int64_t G, bool cl) {
  int64_t chunks = cl ? (HW + 63) / 64 : (C / G * HW + 4095) / 4096;
  if (chunks < 1) chunks = 1;
  if (chunks > kGnMaxChunks) chunks = kGnMaxChunks;
  return (int)chunks;
}

static size_t gn_part_bytes(int64_t N, int64_t G) {
  return align_up((size_t)N * kGnMaxChunks * G * 2 * sizeof(double), 256);
}
static size_t gn_stats_bytes(int64_t N, int64_t G) { return align_up((size_t)N * G * 2 * sizeof(float), 256); }

size_t group_norm_workspace(int64_t N, int64_t C, int64_t HW, int64_t G) {
  return gn_part_bytes(N, G) + gn_stats_bytes(N, G) + (size_t)N * C * sizeof(float2);
}

// ---------------------------------------------------------------------------------------------
// Single-read GroupNorm (channels-last bf16, dense): one cooperative persistent launch.  A work
// item is (image n, chunk k) of gn_chunk_px(C) pixels, at most kGnFusedBytes of activations: the
// CTA copies the chunk into shared memory with one bulk copy per source (cp.async.bulk, the
// pixels of a chunk are contiguous in a dense channels-last image), forms its per-group partial
// sums, publishes them and counts itself in the image's arrival counter, waits (bounded) until all
// chunks of the image have arrived, combines the image's partials in a fixed order into the
// (a, b) affine of its channels, normalises the chunk in shared memory and writes it back with a
// bulk copy.  HBM sees one read and one write of the activation.
//
// Items are dealt round-robin (item = blockIdx.x + i * gridDim.x), the chunks of an image are
// consecutive items, and the grid holds at least `chunks` CTAs, all resident (cooperative launch):
// no CTA ever holds two chunks of one image, and the CTAs holding the chunks of the lowest image
// still waited on are all past their earlier items, so every wait completes.
//
// The arithmetic is exactly that of the three-launch path (gn_partial_cl_bf16x8_kernel,
// gn_finalize_table_kernel, gn_apply_img_bf16x8_kernel): the same chunk boundaries, slots of
// 256 / (C / 8) pixel lanes summed in float in pixel order, double group sums, one warp per group
// combining the chunks with the same xor tree, the same affine and FMA apply.  So the choice
// between the two paths — this one while every chunk of the batch fits on the GPU at once, which
// depends on the batch size — never changes a bit of the result.
constexpr int kGnFusedBytes = 80 * 1024;
constexpr int kGnFusedThreads = 256;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

struct GnFusedParams {
  const __nv_bfloat16* x;   // first source: C1 channels per pixel, image stride sn (elements)
  const __nv_bfloat16* x2;  // second source (C - C1 channels, image stride sn2) or null
  __nv_bfloat16* y;         // dense [N, HW, C]
  int64_t sn, sn2;
  int C, C1, HW, G, px, chunks, items;
  const void* w;
  const void* b;
  int wbd;
  double eps;
  int silu;
  double* part;       // [N][chunks][G][2]
  unsigned* arrived;  // [N], zero at launch
};

__global__ void __launch_bounds__(kGnFusedThreads) gn_fused_cl_bf16x8_kernel(const GnFusedParams p) {
  extern __shared__ __align__(128) uint8_t gnf_raw[];
  uint8_t* data = gnf_raw;  // chunk: [px][C1] then [px][C2], bf16
  const int C = p.C, C1 = p.C1, C2 = C - C1, V = C / 8, G = p.G, Cg = C / G;
  const int lanes = V >= kGnThreads ? 1 : kGnThreads / V;  // the slot layout of the partial kernel
  float* red = reinterpret_cast<float*>(gnf_raw + kGnFusedBytes);  // [2][lanes * C]
  float* ab = red;                                                  // reused: [C][2] affine
  double* gstat = reinterpret_cast<double*>(red + 2 * lanes * C);   // [G][2] mean, rstd
  float* gb = reinterpret_cast<float*>(gstat + 2 * G);              // [2][C] gamma, beta
  uint64_t* bar = reinterpret_cast<uint64_t*>(gb + 2 * C);
  __shared__ int s_abort;  // a bounded wait gave up: stop
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    s_abort = 0;
  }
  __syncthreads();
  const double count = (double)Cg * (double)p.HW;
  uint32_t phase = 0;
  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int n = item / p.chunks, k = item % p.chunks;
    const int p0 = k * p.px, np = min(p.px, p.HW - p0);
    const uint32_t bytes1 = (uint32_t)np * C1 * 2, bytes2 = (uint32_t)np * C2 * 2;
    const __nv_bfloat16* src1 = p.x + (int64_t)n * p.sn + (int64_t)p0 * C1;
    const __nv_bfloat16* src2 = p.x2 ? p.x2 + (int64_t)n * p.sn2 + (int64_t)p0 * C2 : nullptr;
    uint8_t* d2 = data + bytes1;
    if (tid == 0) {
      mbar_arrive_expect_tx(bar, bytes1 + bytes2);
      bulk_g2s(data, src1, bytes1, bar);
      if (bytes2) bulk_g2s(d2, src2, bytes2, bar);
    }
    if (item == (int)blockIdx.x)  // affine parameters, fetched while the chunk is in flight
      for (int c = tid; c < C; c += kGnFusedThreads) {
        gb[c] = p.w ? load_as_f32(p.w, c, p.wbd) : 1.f;
        gb[C + c] = p.b ? load_as_f32(p.b, c, p.wbd) : 0.f;
      }
    int ok = mbar_wait(bar, phase, 40, &s_abort) ? 1 : 0;
    phase ^= 1;
    // partial sums: thread t owns channel vector t % V of pixel lane t / V (fixed order)
    for (int t = tid; t < lanes * V; t += kGnFusedThreads) {
      const int lane = t / V, v = t % V;
      float s8[8], q8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) s8[j] = q8[j] = 0.f;
      const bool first = v * 8 < C1;
      const uint8_t* base = first ? data + v * 16 : d2 + (v * 8 - C1) * 2;
      const int pitch = (first ? C1 : C2) * 2;
#pragma unroll 4
      for (int px = lane; px < np; px += lanes) {
        const uint4 u = *reinterpret_cast<const uint4*>(base + px * pitch);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          s8[2 * j] += f.x;
          q8[2 * j] = __fmaf_rn(f.x, f.x, q8[2 * j]);
          s8[2 * j + 1] += f.y;
          q8[2 * j + 1] = __fmaf_rn(f.y, f.y, q8[2 * j + 1]);
        }
      }
      float4* rs = reinterpret_cast<float4*>(red + lane * C + v * 8);
      float4* rq = reinterpret_cast<float4*>(red + lanes * C + lane * C + v * 8);
      rs[0] = make_float4(s8[0], s8[1], s8[2], s8[3]);
      rs[1] = make_float4(s8[4], s8[5], s8[6], s8[7]);
      rq[0] = make_float4(q8[0], q8[1], q8[2], q8[3]);
      rq[1] = make_float4(q8[4], q8[5], q8[6], q8[7]);
    }
    __syncthreads();
    for (int c = tid; c < C; c += kGnFusedThreads) {
      float s = 0.f, q = 0.f;
      for (int l = 0; l < lanes; ++l) {
        s += red[l * C + c];
        q += red[lanes * C + l * C + c];
      }
      red[c] = s;
      red[lanes * C + c] = q;
    }
    __syncthreads();
    double* part_n = p.part + (int64_t)n * p.chunks * G * 2;
    for (int g = tid; g < G; g += kGnFusedThreads) {
      double s = 0.0, q = 0.0;
      for (int c = g * Cg; c < (g + 1) * Cg; ++c) {
        s += red[c];
        q += red[lanes * C + c];
      }
      __stcg(part_n + ((int64_t)k * G + g) * 2, s);
      __stcg(part_n + ((int64_t)k * G + g) * 2 + 1, q);
    }
    __syncthreads();
    // publish, then wait for every chunk of image n (bounded)
    if (tid == 0) {
      __threadfence();
      atomicAdd(&p.arrived[n], 1u);
      const long long start = clock64();
      while (true) {
        unsigned a;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(a) : "l"(&p.arrived[n]) : "memory");
        if (a >= (unsigned)p.chunks) break;
        if (s_abort || clock64() - start > kWaitBudgetCycles) {
          report_device_error(41);
          s_abort = 1;
          break;
        }
        __nanosleep(64);
      }
      __threadfence();
    }
    __syncthreads();
    ok = ok && !s_abort;
    // group statistics of image n: one warp per group, lane l sums chunks l, l + 32, ... and a
    // fixed xor tree combines the lanes (the same order as gn_finalize_table_kernel)
    {
      const int wid = tid >> 5, lane = tid & 31;
      constexpr int W = kGnFusedThreads / 32, GPW = 4;  // a warp's groups g0 + W * i, loads in flight together
      for (int g0 = wid; g0 < G; g0 += W * GPW) {
        double s[GPW], q[GPW];
#pragma unroll
        for (int i = 0; i < GPW; ++i) s[i] = q[i] = 0.0;
        for (int c = lane; c < p.chunks; c += 32) {
#pragma unroll
          for (int i = 0; i < GPW; ++i) {
            const int g = g0 + W * i;
            if (g < G) {
              const double2 v = __ldcg(reinterpret_cast<const double2*>(part_n + ((int64_t)c * G + g) * 2));
              s[i] += v.x;
              q[i] += v.y;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            s[i] += __shfl_xor_sync(0xffffffffu, s[i], o);
            q[i] += __shfl_xor_sync(0xffffffffu, q[i], o);
          }
          const int g = g0 + W * i;
          if (lane == 0 && g < G) {
            const double mean = s[i] / count;
            double var = q[i] / count - mean * mean;
            if (var < 0) var = 0;
            gstat[2 * g] = mean;
            gstat[2 * g + 1] = 1.0 / sqrt(var + p.eps);
          }
        }
      }
    }
    __syncthreads();
    for (int c = tid; c < C; c += kGnFusedThreads) {
      const int g = c / Cg;
      const float rstd = (float)gstat[2 * g + 1], mf = (float)gstat[2 * g];
      const float2 t = gn_affine_v(rstd, mf, p.w != nullptr, gb[c], p.b != nullptr, gb[C + c]);
      ab[2 * c] = t.x;
      ab[2 * c + 1] = t.y;
    }
    __syncthreads();
    // normalise: thread (lane, v) keeps the (a, b) pairs of its 8 channels in registers and walks
    // pixels lane, lane + lanes, ... (conflict-free 16-byte shared-memory accesses); one source is
    // normalised in place and stored with a bulk copy, two sources go straight to global memory
    for (int t = tid; t < lanes * V; t += kGnFusedThreads) {
      const int lane = t / V, v = t % V;
      float a8[8], b8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        a8[j] = ab[2 * (v * 8 + j)];
        b8[j] = ab[2 * (v * 8 + j) + 1];
      }
      const bool first = v * 8 < C1;
      uint8_t* base = first ? data + v * 16 : d2 + (v * 8 - C1) * 2;
      const int pitch = (first ? C1 : C2) * 2;
      uint4* dst = reinterpret_cast<uint4*>(p.y + ((int64_t)n * p.HW + p0) * C) + v;
#pragma unroll 4
      for (int px = lane; px < np; px += lanes) {
        uint4 u = *reinterpret_cast<const uint4*>(base + px * pitch);
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          float r0 = __fmaf_rn(f.x, a8[2 * j], b8[2 * j]), r1 = __fmaf_rn(f.y, a8[2 * j + 1], b8[2 * j + 1]);
          if (p.silu) {
            r0 = silu_bf16out(r0);
            r1 = silu_bf16out(r1);
          }
          h[j] = __floats2bfloat162_rn(r0, r1);
        }
        if (!p.x2)
          *reinterpret_cast<uint4*>(base + px * pitch) = u;
        else if (ok)
          dst[(int64_t)px * V] = u;
      }
    }
    if (!p.x2) {
      fence_async_smem();
      __syncthreads();
      if (tid == 0 && ok) {
        bulk_s2g(p.y + ((int64_t)n * p.HW + p0) * C, data, bytes1);
        bulk_commit();
      }
    }
    // the next item's copy overwrites `data` and `red`: the store must have read them, and the
    // generic-proxy accesses above are ordered before that asynchronous write
    fence_async_smem();
    if (tid == 0) bulk_wait_read0();
    __syncthreads();
    if (!ok) break;
  }
  if (tid == 0) bulk_wait0();
}

MT_STATUS_READER(read_status_norm)


// Shared memory of the fused kernel for C channels and G groups.
static size_t gn_fused_smem(int64_t C, int64_t G) {
  const int64_t V = C / 8;
  const int64_t lanes = V >= kGnThreads ? 1 : kGnThreads / V;
  return kGnFusedBytes + align_up((size_t)2 * lanes * C * sizeof(float), 16) + (size_t)G * 2 * sizeof(double) +
         (size_t)2 * C * sizeof(float) + 16;
}

// Launches the fused path when it applies: returns 1 (launched, *rc the status) or 0 (not taken:
// the chunk exceeds kGnFusedBytes, the CTAs that fit on the GPU at once are fewer than an image's
// chunks, or MT_GN_FUSED=0).  The decision depends on (C, HW, G) and the device only.
static int gn_fused_try(__nv_bfloat16* y, const __nv_bfloat16* x, int64_t sn, const __nv_bfloat16* x2, int64_t sn2,
                        int64_t C1, const void* w, const void* b, int wbd, int64_t N, int64_t C, int64_t HW, int64_t G,
                        double eps, int silu, double* part, unsigned* arrived, cudaStream_t st, int* rc) {
  static const bool off = [] {
    const char* e = getenv("MT_GN_FUSED");
    return e && e[0] == '0';
  }();
  if (off) return 0;
  // the three-launch path's chunking: ceil(HW / gn_chunk_px(C)) chunks of ceil(HW / chunks) pixels
  const int64_t chunks = (HW + gn_chunk_px(C) - 1) / gn_chunk_px(C);
  const int64_t px = (HW + chunks - 1) / chunks;
  if (px * C * 2 > kGnFusedBytes || chunks > kGnMaxChunks || HW > (1 << 30)) return 0;
  const size_t smem = gn_fused_smem(C, G);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    if (cudaFuncSetAttribute(gn_fused_cl_bf16x8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    attr_set[dev & 63] = true;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gn_fused_cl_bf16x8_kernel, kGnFusedThreads, smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (occ < 1) return 0;
  // one item per CTA: taken while the whole batch fits on the GPU at once and fills at least
  // every SM (the three-launch path is faster for more items, which need several rounds, and for
  // fewer, where its finer-grained launches use more of the GPU)
  const int64_t resident = (int64_t)occ * num_sms();
  if (resident < N * chunks || N * chunks < num_sms()) return 0;
  GnFusedParams p{};
  p.x = x;
  p.x2 = x2;
  p.y = y;
  p.sn = sn;
  p.sn2 = sn2;
  p.C = (int)C;
  p.C1 = x2 ? (int)C1 : (int)C;
  p.HW = (int)HW;
  p.G = (int)G;
  p.px = (int)px;
  p.chunks = (int)chunks;
  p.items = (int)(N * chunks);
  p.w = w;
  p.b = b;
  p.wbd = wbd;
  p.eps = eps;
  p.silu = silu;
  p.part = part;
  p.arrived = arrived;
  *rc = cuda_check(cudaMemsetAsync(arrived, 0, (size_t)N * sizeof(unsigned), st), "group_norm counters");
  if (*rc) return 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)std::min<int64_t>(resident, p.items));
  cfg.blockDim = dim3(kGnFusedThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gn_fused_cl_bf16x8_kernel, p);
  *rc = e == cudaSuccess ? check_launch("group_norm fused") : cuda_check(e, "group_norm fused launch");
  return 1;
}

// The channels-last bf16 path (dense [N, HW, C] in and out, C % 8 == 0): per-image partial sums,
// finalize into a per-(image, channel) affine table, apply.  With gn_l2_group_bytes() > 0 the
// images are processed in groups (statistics, table and apply of one group back to back).  The
// per-image work does not depend on the grouping, so results are identical for every batch size.  x2 != nullptr: the input is the channel concatenation [x (C1 channels) | x2 (C - C1)].
static int gn_fast_cl(__nv_bfloat16* y, const __nv_bfloat16* x, int64_t sn, const __nv_bfloat16* x2, int64_t sn2,
                      int64_t C1, const void* w, const void* b, int wbd, int64_t N, int64_t C, int64_t HW, int64_t G,
                      double eps, int silu, double* part, float2* tab, int chunks, cudaStream_t st) {
  {
    // the per-image arrival counters of the fused kernel live in the affine-table region
    int rc = MT_OK;
    if (gn_fused_try(y, x, sn, x2, sn2, C1, w, b, wbd, N, C, HW, G, eps, silu, part,
                     reinterpret_cast<unsigned*>(tab), st, &rc))
      return rc;
  }
  const int64_t img_bytes = HW * C * 2;
  const int64_t group_bytes = gn_l2_group_bytes();
  const int64_t per = group_bytes > 0 ? std::max<int64_t>(1, group_bytes / img_bytes) : N;
  const int64_t ngroups = (N + per - 1) / per;
  const int64_t nc_max = (N + ngroups - 1) / ngroups;  // balanced groups
  const int64_t V = C / 8;
  const int64_t slots = (V >= kGnThreads ? 1 : kGnThreads / V) * C;
  if (2 * slots * sizeof(float) > 48 * 1024) return fail(MT_ERR_UNSUPPORTED, "group_norm: too many channels");
  const int per_img8 = (int)(HW * C / 8);
  const int C8 = (int)(C / 8);
  // blocks per image: a multiple of C8 / gcd(C8, 256), so that the stride is a multiple of C8
  int g = C8, r = 256;
  while (r) {
    const int t = g % r;
    g = r;
    r = t;
  }
  const int unit = C8 / g;
  for (int64_t n0 = 0; n0 < N; n0 += nc_max) {
    const int64_t nc = std::min<int64_t>(nc_max, N - n0);
    double* part_g = part + n0 * chunks * G * 2;
    float2* tab_g = tab + n0 * C;
    const __nv_bfloat16* xg = x + n0 * sn;
    const __nv_bfloat16* x2g = x2 ? x2 + n0 * sn2 : nullptr;
    const size_t sh = 2 * slots * sizeof(float);
    static const bool u8 = [] {
      const char* e = getenv("MT_GN_UNROLL");
      return e && atoi(e) == 8;
    }();
    const dim3 grid(chunks, (unsigned)nc);
    static const bool persist = [] {
      const char* e = getenv("MT_GN_PERSIST");
      return !(e && e[0] == '0');
    }();
    const int64_t items = chunks * nc;
    if (persist && V <= kGnThreads && items < (1LL << 31)) {
      const unsigned pg = (unsigned)std::min<int64_t>(items, (int64_t)num_sms() * 4);  // 4 resident per SM
      if (x2)
        gn_partial_cl_bf16x8_persist_kernel<true, 4><<<pg, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks, (int)items,
                                                                                 part_g, x2g, sn2, C1);
      else
        gn_partial_cl_bf16x8_persist_kernel<false, 4><<<pg, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks,
                                                                                  (int)items, part_g);
    } else if (x2 && u8)
      gn_partial_cl_bf16x8_kernel<true, 8><<<grid, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks, part_g, x2g, sn2, C1);
    else if (x2)
      gn_partial_cl_bf16x8_kernel<true, 4><<<grid, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks, part_g, x2g, sn2, C1);
    else if (u8)
      gn_partial_cl_bf16x8_kernel<false, 8><<<grid, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks, part_g);
    else
      gn_partial_cl_bf16x8_kernel<false, 4><<<grid, kGnThreads, sh, st>>>(xg, sn, C, HW, G, chunks, part_g);
    int rc = check_launch("group_norm partial");
    if (rc) return rc;
    gn_finalize_table_kernel<<<(unsigned)((nc * G * 32 + 255) / 256), 256, 0, st>>>(
        part_g, w, b, wbd, nc, C, G, chunks, (double)(C / G) * (double)HW, eps, tab_g);
    rc = check_launch("group_norm finalize");
    if (rc) return rc;
    int bx = (int)std::max<int64_t>(1, std::min<int64_t>((per_img8 + 255) / 256, (int64_t)num_sms() * 16 / nc + 1));
    bx = (bx + unit - 1) / unit * unit;
    if (x2)
      gn_apply_img_bf16x8_kernel<true><<<dim3((unsigned)bx, (unsigned)nc), 256, 0, st>>>(
          y + n0 * HW * C, xg, tab_g, per_img8, C8, silu, x2g, (int)(C1 / 8));
    else
      gn_apply_img_bf16x8_kernel<false><<<dim3((unsigned)bx, (unsigned)nc), 256, 0, st>>>(y + n0 * HW * C, xg, tab_g,
                                                                                        per_img8, C8, silu);
    rc = check_launch("group_norm apply");
    if (rc) return rc;
  }
  return MT_OK;
}

int launch_group_norm(void* y, int yd, const int64_t* ys, const void* x, int xd, const int64_t* xs, const void* w,
                      const void* b, int wbd, int64_t N, int64_t C, int64_t HW, int64_t G, double eps, int silu,
                      void* ws, size_t ws_bytes, cudaStream_t st) {
  if (G <= 0 || C % G != 0)
    return fail(MT_ERR_INVALID, "group_norm: channels %lld not divisible by groups %lld", (long long)C, (long long)G);
  if (N == 0 || C == 0 || HW == 0) return MT_OK;
  if (!ws || ws_bytes < group_norm_workspace(N, C, HW, G)) return fail(MT_ERR_WORKSPACE, "group_norm: workspace");
  const bool cl = (xs[1] == 1 && xs[2] == C) && HW > 1;
  const bool nchw = (xs[2] == 1 && xs[1] == HW) || (HW == 1 && xs[1] == 1);
  if (!cl && !nchw) return fail(MT_ERR_UNSUPPORTED, "group_norm: input must be NCHW-contiguous or channels-last");
  if (N > 65535 || (!cl && N * G > 65535)) return fail(MT_ERR_UNSUPPORTED, "group_norm: batch too large");
  double* part = (double*)ws;
  float* stats = (float*)((char*)ws + gn_part_bytes(N, G));
  float2* tab = (float2*)((char*)ws + gn_part_bytes(N, G) + gn_stats_bytes(N, G));
  const bool vec_in = cl && xd == MT_BF16 && C % 8 == 0 && (uintptr_t)x % 16 == 0 && (xs[0] * 2) % 16 == 0;
  // the vectorised channels-last path walks chunks of 40960 / C pixels (128 at 320 channels, 32 at
  // 1280; between 16 and 128): long enough CTAs for narrow images, enough CTAs for wide ones
  const int64_t gn_px = gn_chunk_px(C);
  const int chunks = vec_in ? (int)std::min<int64_t>(kGnMaxChunks, (HW + gn_px - 1) / gn_px) : gn_chunks(C, HW, G, cl);
  const bool ycl = (ys[1] == 1 && ys[2] == C && ys[0] == HW * C);
  const bool fast = vec_in && ycl && xs[0] == HW * C && yd == MT_BF16 && (uintptr_t)y % 16 == 0 &&
                    HW * C / 8 < (1LL << 31);
  if (fast)
    return gn_fast_cl((__nv_bfloat16*)y, (const __nv_bfloat16*)x, xs[0], nullptr, 0, 0, w, b, wbd, N, C, HW, G, eps,
                      silu, part, tab, chunks, st);
  if (vec_in) {
    const int64_t V = C / 8;
    const int64_t slots = (V >= kGnThreads ? 1 : kGnThreads / V) * C;
    if (2 * slots * sizeof(float) > 48 * 1024) return fail(MT_ERR_UNSUPPORTED, "group_norm: too many channels");
    gn_partial_cl_bf16x8_kernel<<<dim3(chunks, (unsigned)N), kGnThreads, 2 * slots * sizeof(float), st>>>(
        (const __nv_bfloat16*)x, xs[0], C, HW, G, chunks, part);
  } else if (cl) {
    const int64_t slots = C >= kGnThreads ? C : (kGnThreads / C) * C;
    if (2 * slots * sizeof(float) > 48 * 1024) return fail(MT_ERR_UNSUPPORTED, "group_norm: too many channels");
    gn_partial_cl_kernel<<<dim3(chunks, (unsigned)N), kGnThreads, 2 * slots * sizeof(float), st>>>(
        x, xd, xs[0], xs[2], C, HW, G, chunks, part);
  } else {
    gn_partial_nchw_kernel<<<dim3(chunks, (unsigned)(N * G)), kGnThreads, 0, st>>>(x, xd, xs[0], xs[1], C, HW, G,
                                                                                  chunks, part);
  }
  int rc = check_launch("group_norm partial");
  if (rc) return rc;
  const int64_t total = N * C * HW;
  gn_finalize_kernel<<<(unsigned)((N * G + 127) / 128), 128, 0, st>>>(part, stats, N, G, chunks,
                                                                      (double)(C / G) * (double)HW, eps);
  rc = check_launch("group_norm finalize");
  if (rc) return rc;
  if (vec_in && ycl && xs[0] == HW * C && yd == MT_BF16 && (uintptr_t)y % 16 == 0) {
    gn_table_kernel<<<(unsigned)((N * C + 255) / 256), 256, 0, st>>>(stats, w, b, wbd, N, C, G, tab);
    rc = check_launch("group_norm table");
    if (rc) return rc;
    const int64_t blocks = std::min<int64_t>((total / 8 + 255) / 256, (int64_t)num_sms() * 32);
    gn_apply_cl_bf16x8_tab_kernel<<<(unsigned)blocks, 256, 0, st>>>((__nv_bfloat16*)y, (const __nv_bfloat16*)x, tab,
                                                                    HW, C, total / 8, silu);
  } else {
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
    gn_apply_generic_kernel<<<(unsigned)blocks, 256, 0, st>>>(y, yd, ys[0], ys[1], ys[2], x, xd, xs[0], xs[1], xs[2],
                                                             stats, w, b, wbd, N, C, HW, G, silu, cl ? 1 : 0);
  }
  return check_launch("group_norm apply");
}

// Group norm of the channel concatenation [x1 | x2] (the up-block skip connection) without forming
// it: bf16 dense channels-last sources of C1 and C - C1 channels (multiples of 8), bf16 dense
// channels-last output of C channels.  Same statistics and chunking as launch_group_norm's
// channels-last path on the concatenated tensor.
int launch_group_norm_cat(void* y, int yd, const int64_t* ys, const void* x1, const int64_t* xs1, int64_t C1,
                          const void* x2, const int64_t* xs2, int xd, const void* w, const void* b, int wbd, int64_t N,
                          int64_t C, int64_t HW, int64_t G, double eps, int silu, void* ws, size_t ws_bytes,
                          cudaStream_t st) {
  if (G <= 0 || C % G != 0)
    return fail(MT_ERR_INVALID, "group_norm_cat: channels %lld not divisible by groups %lld", (long long)C,
                (long long)G);
  if (!x1 || !x2 || !y || !xs1 || !xs2 || !ys) return fail(MT_ERR_INVALID, "group_norm_cat: null argument");
  const int64_t C2 = C - C1;
  if (C1 <= 0 || C2 <= 0 || C1 % 8 || C2 % 8)
    return fail(MT_ERR_UNSUPPORTED, "group_norm_cat: source channel counts must be positive multiples of 8");
  if (xd != MT_BF16 || yd != MT_BF16) return fail(MT_ERR_UNSUPPORTED, "group_norm_cat: bf16 only");
  if (N == 0 || HW == 0) return MT_OK;
  if (N > 65535) return fail(MT_ERR_UNSUPPORTED, "group_norm_cat: batch too large");
  auto dense_cl = [&](const int64_t* s, int64_t c) { return s[1] == 1 && s[2] == c && s[0] == HW * c; };
  if (!dense_cl(xs1, C1) || !dense_cl(xs2, C2) || !dense_cl(ys, C) || (uintptr_t)x1 % 16 || (uintptr_t)x2 % 16 ||
      (uintptr_t)y % 16 || HW * C / 8 >= (1LL << 31))
    return fail(MT_ERR_UNSUPPORTED, "group_norm_cat: dense 16-byte aligned channels-last tensors only");
  if (!ws || ws_bytes < group_norm_workspace(N, C, HW, G)) return fail(MT_ERR_WORKSPACE, "group_norm_cat: workspace");
  double* part = (double*)ws;
  float2* tab = (float2*)((char*)ws + gn_part_bytes(N, G) + gn_stats_bytes(N, G));
  const int64_t gn_px = gn_chunk_px(C);
  const int chunks = (int)std::min<int64_t>(kGnMaxChunks, (HW + gn_px - 1) / gn_px);
  return gn_fast_cl((__nv_bfloat16*)y, (const __nv_bfloat16*)x1, xs1[0], (const __nv_bfloat16*)x2, xs2[0], C1, w, b,
                    wbd, N, C, HW, G, eps, silu, part, tab, chunks, st);
}

// ---------------------------------------------------------------------------------------------
// Group norm without a caller workspace: the partial sums and per-group statistics live in a
// fixed array of this translation unit, so the call performs no device allocation at all.
// Every byte of the scratch that is read is first written in the same call (partial kernel ->
// finalize -> apply), so nothing has to be cleared between calls.

static __device__ __align__(256) unsigned char g_gn_static_scratch[MT_GROUP_NORM_STATIC_SCRATCH_BYTES];

static void* g_gn_scratch_addr[64];
static cudaError_t g_gn_scratch_err[64];
static std::once_flag g_gn_scratch_once[64];

// Device address of the scratch array on the current device.  In host code the array's name is
// only a host-side stand-in; the address must come from cudaGetSymbolAddress, once per device,
// with that device current.
static int gn_static_scratch(void** out) {
  int dev = 0;
  int rc = cuda_check(cudaGetDevice(&dev), "group_norm_noalloc: cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= 64) return fail(MT_ERR_UNSUPPORTED, "group_norm_noalloc: device index %d", dev);
  std::call_once(g_gn_scratch_once[dev], [dev] {
    void* p = nullptr;
    g_gn_scratch_err[dev] = cudaGetSymbolAddress(&p, g_gn_static_scratch);
    g_gn_scratch_addr[dev] = p;
  });
  if (g_gn_scratch_err[dev] != cudaSuccess)
    return fail(MT_ERR_LAUNCH, "group_norm_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(g_gn_scratch_err[dev]));
  *out = g_gn_scratch_addr[dev];
  return MT_OK;
}

static int launch_group_norm_noalloc(void* y, int yd, const int64_t* ys, const void* x, int xd, const int64_t* xs,
                                     const void* w, const void* b, int wbd, int64_t N, int64_t C, int64_t HW,
                                     int64_t G, double eps, int silu, cudaStream_t st) {
  if (!ys || !xs) return fail(MT_ERR_INVALID, "group_norm_noalloc: null strides");
  if (G <= 0 || C % G != 0)
    return fail(MT_ERR_INVALID, "group_norm: channels %lld not divisible by groups %lld", (long long)C, (long long)G);
  if (N == 0 || C == 0 || HW == 0) return MT_OK;
  const bool cl = (xs[1] == 1 && xs[2] == C) && HW > 1;
  const bool nchw = (xs[2] == 1 && xs[1] == HW) || (HW == 1 && xs[1] == 1);
  if (!cl && !nchw) return fail(MT_ERR_UNSUPPORTED, "group_norm: input must be NCHW-contiguous or channels-last");
  if (N > 65535 || (!cl && N * G > 65535)) return fail(MT_ERR_UNSUPPORTED, "group_norm: batch too large");
  const int chunks = gn_chunks(C, HW, G, cl);
  const size_t part_bytes = align_up((size_t)N * chunks * G * 2 * sizeof(double), 256);
  const size_t need = part_bytes + (size_t)N * G * 2 * sizeof(float);
  if (need > MT_GROUP_NORM_STATIC_SCRATCH_BYTES)
    return fail(MT_ERR_INVALID,
                "group_norm_noalloc: this shape needs %zu bytes of scratch, more than the fixed %u bytes; "
                "use mt_cuda_group_norm with a workspace",
                need, (unsigned)MT_GROUP_NORM_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  int rc = gn_static_scratch(&scratch);
  if (rc) return rc;
  double* part = static_cast<double*>(scratch);
  float* stats = reinterpret_cast<float*>(static_cast<char*>(scratch) + part_bytes);
  if (cl) {
    const int64_t slots = C >= kGnThreads ? C : (kGnThreads / C) * C;
    if (2 * slots * sizeof(float) > 48 * 1024) return fail(MT_ERR_UNSUPPORTED, "group_norm: too many channels");
    gn_partial_cl_kernel<<<dim3(chunks, (unsigned)N), kGnThreads, 2 * slots * sizeof(float), st>>>(
        x, xd, xs[0], xs[2], C, HW, G, chunks, part);
  } else {
    gn_partial_nchw_kernel<<<dim3(chunks, (unsigned)(N * G)), kGnThreads, 0, st>>>(x, xd, xs[0], xs[1], C, HW, G,
                                                                                  chunks, part);
  }
  rc = check_launch("group_norm_noalloc partial");
  if (rc) return rc;
  gn_finalize_kernel<<<(unsigned)((N * G + 127) / 128), 128, 0, st>>>(part, stats, N, G, chunks,
                                                                      (double)(C / G) * (double)HW, eps);
  rc = check_launch("group_norm_noalloc finalize");
  if (rc) return rc;
  const bool ycl = (ys[1] == 1 && ys[2] == C && ys[0] == HW * C);
  const int64_t total = N * C * HW;
  if (cl && ycl && xs[0] == HW * C && xd == MT_BF16 && yd == MT_BF16 && C % 8 == 0 && (uintptr_t)x % 16 == 0 &&
      (uintptr_t)y % 16 == 0) {
    const int64_t blocks = std::min<int64_t>((total / 8 + 255) / 256, (int64_t)num_sms() * 16);
    gn_apply_cl_bf16x8_kernel<<<(unsigned)blocks, 256, 0, st>>>((__nv_bfloat16*)y, (const __nv_bfloat16*)x, stats, w,
                                                                b, wbd, N, HW, C, G, silu);
  } else {
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
    gn_apply_generic_kernel<<<(unsigned)blocks, 256, 0, st>>>(y, yd, ys[0], ys[1], ys[2], x, xd, xs[0], xs[1], xs[2],
                                                             stats, w, b, wbd, N, C, HW, G, silu, cl ? 1 : 0);
  }
  return check_launch("group_norm_noalloc apply");
}

}  // namespace mt

extern "C" int mt_cuda_group_norm_noalloc(void* y, int y_dtype, const int64_t* y_strides, const void* x, int x_dtype,
                                          const int64_t* x_strides, const void* weight, const void* bias, int wb_dtype,
                                          int64_t N, int64_t C, int64_t HW, int64_t groups, double eps, int fuse_silu,
                                          void* stream) {
  return mt::launch_group_norm_noalloc(y, y_dtype, y_strides, x, x_dtype, x_strides, weight, bias, wb_dtype, N, C, HW,
                                       groups, eps, fuse_silu, reinterpret_cast<cudaStream_t>(stream));
}
