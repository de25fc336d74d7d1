// Fused scaled-dot-product attention, fp32 SIMT flash kernel + dispatch.
//
// sdpa_simt_kernel: flash-style (online softmax; scores never leave the SM) fp32 kernel for every
// dtype, mask kind, causal flag and head dim <= 256.  It is the fp32 path (rtol 1e-4 against the
// reference's double-precision loop) and the general fallback; the bf16 / f16 tensor-core kernel
// lives in attention_sm100.cu.
#include <algorithm>

#include "runtime.h"

namespace mt {

constexpr int kAttBq = 64;
constexpr int kAttBk = 64;
constexpr int kAttThreads = 256;

struct SdpaParams {
  int64_t B, H, Hkv, Sq, Sk, D, Dv;
  int dtype;
  const void* q; int64_t qs[4];
  const void* k; int64_t ks[4];
  const void* v; int64_t vs[4];
  void* o; int64_t os[4];
  const void* mask; int mask_kind, mask_dtype; int64_t ms[4];
  int causal;
  float scale;
  int Dp, Dvp;  // padded to multiples of 16
};

__device__ __forceinline__ float mask_value(const SdpaParams& p, int64_t b, int64_t h, int64_t qi, int64_t ki) {
  const int64_t off = b * p.ms[0] + h * p.ms[1] + qi * p.ms[2] + ki * p.ms[3];
  if (p.mask_kind == 1) return static_cast<const uint8_t*>(p.mask)[off] ? 0.f : -INFINITY;
  return load_as_f32(p.mask, off, p.mask_dtype);
}

// Thread (ty, tx) in a 16 x 16 grid owns score rows ty*4..+3 and columns tx*4..+3 of the 64 x 64
// tile, and output rows ty*4..+3, columns tx + 16*j.
__global__ void __launch_bounds__(kAttThreads) sdpa_simt_kernel(SdpaParams p) {
  extern __shared__ float att_sh[];
  const int Dp = p.Dp, Dvp = p.Dvp;
  float* Qs = att_sh;                  // [Bq][Dp]
  float* Ks = Qs + kAttBq * Dp;        // [Bk][Dp+1]
  float* Vs = Ks + kAttBk * (Dp + 1);  // [Bk][Dvp]
  float* Ps = Vs + kAttBk * Dvp;       // [Bq][Bk+1]
  const int64_t bh = blockIdx.y;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t hk = h / (p.H / p.Hkv);
  const int64_t q0 = (int64_t)blockIdx.x * kAttBq;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;

  for (int i = tid; i < kAttBq * Dp; i += kAttThreads) {
    const int r = i / Dp, d = i % Dp;
    const int64_t qi = q0 + r;
    float val = 0.f;
    if (qi < p.Sq && d < p.D) val = load_as_f32(p.q, b * p.qs[0] + h * p.qs[1] + qi * p.qs[2] + d * p.qs[3], p.dtype);
    Qs[i] = val * p.scale;
  }
  constexpr int MAXJ = 16;  // Dvp <= 256
  const int nj = Dvp / 16;
  float acc[4][MAXJ];
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) acc[i][j] = 0.f;
  }
  int64_t k_end = p.Sk;
  if (p.causal && !p.mask) k_end = std::min<int64_t>(p.Sk, q0 + kAttBq);
  for (int64_t k0 = 0; k0 < k_end; k0 += kAttBk) {
    __syncthreads();
    for (int i = tid; i < kAttBk * Dp; i += kAttThreads) {
      const int r = i / Dp, d = i % Dp;
      const int64_t ki = k0 + r;
      float val = 0.f;
      if (ki < p.Sk && d < p.D)
        val = load_as_f32(p.k, b * p.ks[0] + hk * p.ks[1] + ki * p.ks[2] + d * p.ks[3], p.dtype);
      Ks[r * (Dp + 1) + d] = val;
    }
    for (int i = tid; i < kAttBk * Dvp; i += kAttThreads) {
      const int r = i / Dvp, d = i % Dvp;
      const int64_t ki = k0 + r;
      float val = 0.f;
      if (ki < p.Sk && d < p.Dv)
        val = load_as_f32(p.v, b * p.vs[0] + hk * p.vs[1] + ki * p.vs[2] + d * p.vs[3], p.dtype);
      Vs[i] = val;
    }
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    for (int d = 0; d < p.D; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = Qs[(ty * 4 + i) * Dp + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = Ks[(tx * 4 + j) * (Dp + 1) + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t qi = q0 + ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t ki = k0 + tx * 4 + j;
        if (ki >= p.Sk) {
          s[i][j] = -INFINITY;
          continue;
        }
        if (p.causal && ki > qi) s[i][j] = -INFINITY;
        if (p.mask && qi < p.Sq) s[i][j] += mask_value(p, b, h, qi, ki);
      }
    }
    // online softmax: row max / sum across the 16 threads sharing a row (lanes tx = 0..15)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float mx = fmaxf(fmaxf(s[i][0], s[i][1]), fmaxf(s[i][2], s[i][3]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[i], mx);
      // all keys masked so far: keep the exponent arguments finite (a row that stays fully
      // masked ends as 0/0 = NaN, as in the reference).
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float corr = expf(m_run[i] - m_use);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float e = expf(s[i][j] - m_use);
        s[i][j] = e;
        sum += e;
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_run[i] = l_run[i] * corr + sum;
      m_run[i] = m_new;
#pragma unroll
      for (int j = 0; j < MAXJ; ++j) acc[i][j] *= corr;
#pragma unroll
      for (int j = 0; j < 4; ++j) Ps[(ty * 4 + i) * (kAttBk + 1) + tx * 4 + j] = s[i][j];
    }
    __syncthreads();
    for (int kk = 0; kk < kAttBk; ++kk) {
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = Ps[(ty * 4 + i) * (kAttBk + 1) + kk];
#pragma unroll
      for (int j = 0; j < MAXJ; ++j) {
        if (j < nj) {
          const float vv = Vs[kk * Dvp + tx + 16 * j];
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i][j] = fmaf(pv[i], vv, acc[i][j]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t qi = q0 + ty * 4 + i;
    if (qi >= p.Sq) continue;
    const float inv = 1.0f / l_run[i];
#pragma unroll
    for (int j = 0; j < MAXJ; ++j) {
      const int d = tx + 16 * j;
      if (j < nj && d < p.Dv)
        store_from_f32(p.o, b * p.os[0] + h * p.os[1] + qi * p.os[2] + d * p.os[3], p.dtype, acc[i][j] * inv);
    }
  }
}

static int run_sdpa_simt(const SdpaParams& p, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)kAttBq * p.Dp + (size_t)kAttBk * (p.Dp + 1) + (size_t)kAttBk * p.Dvp +
                                       (size_t)kAttBq * (kAttBk + 1));
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(sdpa_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
                        "sdpa smem attribute");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  if (p.B * p.H > 65535) return fail(MT_ERR_UNSUPPORTED, "sdpa: batch*heads > 65535");
  dim3 grid((unsigned)((p.Sq + kAttBq - 1) / kAttBq), (unsigned)(p.B * p.H));
  sdpa_simt_kernel<<<grid, kAttThreads, smem, st>>>(p);
  return check_launch("sdpa_simt");
}

// attention_sm100.cu
int run_sdpa_tc(const mt_sdpa_desc& d, void* ws, size_t ws_bytes, cudaStream_t st, bool* handled);
size_t sdpa_tc_workspace(const mt_sdpa_desc& d);

int validate_sdpa_desc(const mt_sdpa_desc& d) {
  if (d.B < 0 || d.H <= 0 || d.Hkv <= 0 || d.Sq < 0 || d.Sk < 0 || d.D <= 0 || d.Dv <= 0)
    return fail(MT_ERR_INVALID, "sdpa: bad sizes");
  if (d.H % d.Hkv != 0)
    return fail(MT_ERR_INVALID, "sdpa: heads %lld not a multiple of kv heads %lld", (long long)d.H, (long long)d.Hkv);
  if (d.D > 256 || d.Dv > 256) return fail(MT_ERR_UNSUPPORTED, "sdpa: head dim > 256");
  if (d.dtype != MT_F32 && d.dtype != MT_BF16 && d.dtype != MT_F16) return fail(MT_ERR_UNSUPPORTED, "sdpa: dtype");
  if (d.mask_kind < 0 || d.mask_kind > 2) return fail(MT_ERR_INVALID, "sdpa: mask kind");
  if (d.B > 0 && d.Sq > 0 && (!d.q || !d.k || !d.v || !d.o)) return fail(MT_ERR_INVALID, "sdpa: null operand");
  return MT_OK;
}

size_t sdpa_workspace(const mt_sdpa_desc& d) {
  if (validate_sdpa_desc(d) != MT_OK) return 0;
  return sdpa_tc_workspace(d);
}

int run_sdpa(const mt_sdpa_desc& d, void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = validate_sdpa_desc(d);
  if (rc) return rc;
  if (d.B == 0 || d.Sq == 0) return MT_OK;
  if (d.Sk == 0) {
    // softmax over an empty key set: the reference produces NaN rows (0/0).
    int64_t sizes[4] = {d.B, d.H, d.Sq, d.Dv};
    return launch_fill_strided_nan(d.o, d.dtype, d.o_strides, sizes, st);
  }
  bool handled = false;
  rc = run_sdpa_tc(d, ws, ws_bytes, st, &handled);
  if (rc || handled) return rc;
  SdpaParams p{};
  p.B = d.B; p.H = d.H; p.Hkv = d.Hkv; p.Sq = d.Sq; p.Sk = d.Sk; p.D = d.D; p.Dv = d.Dv;
  p.dtype = d.dtype;
  p.q = d.q; p.k = d.k; p.v = d.v; p.o = d.o;
  for (int i = 0; i < 4; ++i) {
    p.qs[i] = d.q_strides[i]; p.ks[i] = d.k_strides[i]; p.vs[i] = d.v_strides[i]; p.os[i] = d.o_strides[i];
    p.ms[i] = d.mask_strides[i];
  }
  p.mask = d.mask_kind ? d.mask : nullptr;
  p.mask_kind = d.mask_kind;
  p.mask_dtype = d.mask_dtype;
  p.causal = d.causal;
  p.scale = (float)d.scale;
  p.Dp = (int)((d.D + 15) / 16 * 16);
  p.Dvp = (int)((d.Dv + 15) / 16 * 16);
  return run_sdpa_simt(p, st);
}

}  // namespace mt
