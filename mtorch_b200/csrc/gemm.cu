// Dense contractions on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// One persistent, warp-specialised kernel serves matmul / bmm / addmm / baddbmm / linear and
// conv2d (as implicit GEMM):
//   warp 0      TMA producer: K-major 128-byte-swizzled tiles of A (128 rows x 128 B) and B
//               (BN rows x 128 B) into a STAGES-deep shared-memory ring (mbarrier full/empty);
//   warp 1      MMA issuer: one thread issues tcgen05.mma (kind::f16 for bf16/f16, three
//               kind::tf32 products for fp32) into one of two TMEM accumulators (2 x BN columns);
//   warps 2..9  epilogue: tcgen05.ld the accumulator (two warps per 32-lane TMEM quarter),
//               apply alpha / beta*C / bias / activation / residual and store; the TMEM buffer
//               is then released, so the next tile's MMAs overlap this tile's stores.
// Convolution: the A tile of output pixels (tn x th x tw = 128) at filter tap (r, s) and channel
// chunk c is ONE 4-D TMA box over the channels-last activation at coordinates
// (c, q0 + s*dil - pad, p0 + r*dil - pad, n0); TMA's out-of-bounds zero fill is the padding.
// No cluster multicast: every CTA loads its own tiles.
#include <algorithm>

#include "runtime.h"

namespace mt {

MT_STATUS_READER(read_status_gemm)

constexpr int kBM = 128;
constexpr int kGemmThreads = 320;  // 2 producer/MMA warps + 8 epilogue warps

struct TileParams {
  int num_m_tiles, num_n_tiles, batch;
  int k_iters;
  int a_batched, b_batched;
  // implicit convolution
  int tw, th, tn, tiles_q, tiles_p;
  int c_chunks, R, S, pad_h, pad_w, dil_h, dil_w, stride_h, stride_w;
  int bk;  // elements per 128-byte K chunk
  int a_stages;  // B-resident variant: A-only stages behind the resident B tile
  int m_pairs;   // CTA-pair variant: row-tile pairs, ceil(num_m_tiles / 2)
  // split K (implicit convolutions): tile t >= base tiles computes K iterations
  // [s * k_per, (s + 1) * k_per) of tile t % base, s = t / base, and writes raw fp32 partial sums
  // (EpiParams::part); a reduction kernel adds the splits in order and applies the epilogue
  int k_splits, k_per;
  // implicit convolution over the channel concatenation of two sources (16-bit only): channel
  // chunks [0, c_split) come from tmA, the rest from the second source's map, passed in the tmAlo
  // slot (unused by 16-bit kernels); 0 = one source
  int c_split;
};

struct EpiParams {
  int mode;   // 0 gemm (b, m), 1 conv via im2col (m -> n, p, q), 2 implicit conv (tile coordinates)
  int64_t M;  // rows (mode 0/1) or images (mode 2)
  int64_t N;  // GEMM columns (before GEGLU halving)
  int64_t P, Q;
  void* D; int out_dtype; int64_t d_s0, d_s1, d_s2;
  const void* C; int64_t c_s0, c_s1, c_s2; float beta;
  const void* res; int64_t r_s0, r_s1, r_s2;
  const void* bias; int bias_dtype; int64_t bias_bstride;
  float alpha; int act;
  int vec_ok;  // 16-byte aligned rows of D / C / residual
  int bias_vec;  // bias rows 16-byte aligned and bf16 / fp32: vector loads
  float* part;   // split K: [k_splits][M rows][N] fp32 partial sums (rows in (n, p, q) order)
  int64_t part_stride;
  // TMA-store epilogue of a plain GEMM: the residual is read through a tensor map (32 x 32 boxes,
  // 64-byte swizzle, passed in the tmAlo slot) into the output staging buffers, a tile ahead
  int res_tma;
};

// 256-bit global accesses (sm_100): one instruction covers a whole 32-byte sector, so a warp whose
// threads each own a row writes full sectors instead of two half-sector writes per sector.
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void ld_global_v8(const void* p, uint32_t (&w)[8]) {
  asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}

// GELU for the 16-bit GEMM epilogues, on the FMA pipe only (no reciprocal / exp): the normal CDF
// Phi(x) = 1/2 + x * R(x^2 / 4.5^2) on |x| <= 4.5 (x clamped beyond: Phi(4.5) = 1 - 3.4e-6),
// R a degree-9 polynomial fitted offline (iterated reweighted least squares) for minimum absolute
// error against 0.5 * erf(x / sqrt 2);
// |GELU error| <= 5.1e-5 absolute over the real line, ~1/150 of a bf16 ulp at 1.  Evaluated on
// pairs with the packed fma.rn.f32x2.  fp32 GEMMs keep gelu_f (erf by A&S 7.1.26, 1.5e-7).
__device__ __forceinline__ uint64_t ep_f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint64_t ep_fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ void gelu_poly_pair(float& x0, float& x1) {
  constexpr float kC[10] = {3.989246786e-01f, -1.345018744e+00f, 4.056245804e+00f, -9.488839149e+00f,
                            1.710670662e+01f, -2.320115280e+01f, 2.260896301e+01f, -1.475468349e+01f,
                            5.718395233e+00f, -9.884314537e-01f};
  const float c0 = fminf(fmaxf(x0, -4.5f), 4.5f), c1 = fminf(fmaxf(x1, -4.5f), 4.5f);
  const float s0 = c0 * (1.0f / 4.5f), s1 = c1 * (1.0f / 4.5f);
  const uint64_t t = ep_f2(s0 * s0, s1 * s1);
  uint64_t r = ep_f2(kC[9], kC[9]);
#pragma unroll
  for (int k = 8; k >= 0; --k) r = ep_fma2(r, t, ep_f2(kC[k], kC[k]));
  const uint64_t phi = ep_fma2(ep_f2(c0, c1), r, ep_f2(0.5f, 0.5f));
  float p0, p1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(p0), "=f"(p1) : "l"(phi));
  x0 *= p0;
  x1 *= p1;
}
// x = x * Phi(g) for 32 (value, gate) pairs, or x = GELU(x) when g == x.
template <bool TF32>
__device__ __forceinline__ void epi_gelu32(float (&v)[32], const float (&g)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    if (TF32) {
      v[j] = v[j] * gelu_f(g[j]);
      v[j + 1] = v[j + 1] * gelu_f(g[j + 1]);
    } else {
      float a = g[j], b = g[j + 1];
      gelu_poly_pair(a, b);
      v[j] *= a;
      v[j + 1] *= b;
    }
  }
}

// 32 consecutive values of one row: load (accumulate scale*x into v) / store, runtime dtype.
__device__ __forceinline__ void row_load_add(const void* p, int dtype, int64_t off, int nvalid, bool vec, float scale,
                                             float (&v)[32]) {
  if (vec && nvalid >= 32) {
    if (dtype == MT_BF16 && (reinterpret_cast<uintptr_t>(static_cast<const __nv_bfloat16*>(p) + off) & 31) == 0) {
      const uint8_t* q = reinterpret_cast<const uint8_t*>(static_cast<const __nv_bfloat16*>(p) + off);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t w[8];
        ld_global_v8(q + 32 * i, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          v[i * 16 + 2 * j] += scale * f.x;
          v[i * 16 + 2 * j + 1] += scale * f.y;
        }
      }
      return;
    }
    if (dtype == MT_BF16) {
      const uint4* q = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + off);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 u = q[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(h[j]);
          v[i * 8 + 2 * j] += scale * f.x;
          v[i * 8 + 2 * j + 1] += scale * f.y;
        }
      }
      return;
    }
    if (dtype == MT_F32) {
      const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 f = q[i];
        v[4 * i] += scale * f.x;
        v[4 * i + 1] += scale * f.y;
        v[4 * i + 2] += scale * f.z;
        v[4 * i + 3] += scale * f.w;
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nvalid) v[j] += scale * load_as_f32(p, off + j, dtype);
}

__device__ __forceinline__ void row_store(void* p, int dtype, int64_t off, int nvalid, bool vec, const float (&v)[32]) {
  if (vec && nvalid >= 32) {
    if ((dtype == MT_BF16 || dtype == MT_F16) && (reinterpret_cast<uintptr_t>(static_cast<uint16_t*>(p) + off) & 31) == 0) {
      uint8_t* q = reinterpret_cast<uint8_t*>(static_cast<uint16_t*>(p) + off);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          w[j] = dtype == MT_BF16 ? pack_bf16x2(v[16 * i + 2 * j], v[16 * i + 2 * j + 1])
                                  : pack_f16x2(v[16 * i + 2 * j], v[16 * i + 2 * j + 1]);
        st_global_v8(q + 32 * i, w);
      }
      return;
    }
    if (dtype == MT_BF16) {
      uint4* q = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p) + off);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        q[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                          pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
      return;
    }
    if (dtype == MT_F16) {
      uint4* q = reinterpret_cast<uint4*>(static_cast<__half*>(p) + off);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        q[i] = make_uint4(pack_f16x2(v[8 * i], v[8 * i + 1]), pack_f16x2(v[8 * i + 2], v[8 * i + 3]),
                          pack_f16x2(v[8 * i + 4], v[8 * i + 5]), pack_f16x2(v[8 * i + 6], v[8 * i + 7]));
      return;
    }
    if (dtype == MT_F32) {
      float4* q = reinterpret_cast<float4*>(static_cast<float*>(p) + off);
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nvalid) store_from_f32(p, off + j, dtype, v[j]);
}

__device__ __forceinline__ void decode_tile(const TileParams& tp, int t, int& b, int& mt, int& nt) {
  nt = t % tp.num_n_tiles;
  const int rest = t / tp.num_n_tiles;
  mt = rest % tp.num_m_tiles;
  b = rest / tp.num_m_tiles;
}

// Shared memory of the B-resident variant's operand region (B tile + A stages).
constexpr int kResBytes = 200 * 1024;
// TMA-store epilogue: each epilogue warp stages its 32 x 32 output chunks in private 2 KB
// shared-memory buffers (64-byte swizzle), one per chunk the warp owns in a tile (at least two),
// and stores each with one bulk tensor store.  With a residual, the residual chunk is first
// TMA-loaded into the same buffer (prefetched a tile ahead), added, and overwritten by the output.
// Only the residual instance (TST == 2, streaming column tiles of 128 / 160 / 256) has more than two
// buffers per warp: the others keep the room for their operand ring.
__host__ __device__ constexpr int store_bufs(int bn, bool rt) {
  return rt && (bn / 32 + 1) / 2 > 2 ? (bn / 32 + 1) / 2 : 2;
}
__host__ __device__ constexpr int store_bytes(int bn, bool rt) { return 8 * store_bufs(bn, rt) * 2048; }
// barriers of the GEMM kernel: ring (<= 8 + 8), TMEM (2 + 2), resident B, TMEM slot + abort flag,
// residual buffers (8 warps x <= 5)
constexpr int kGemmBarBytes = 512;

__device__ __forceinline__ void gemm_fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Stage 32 output values of this lane's row (bf16 / f16) into the warp's 32 x 64-byte buffer with
// the 64-byte swizzle the store's tensor map uses (16-byte chunk k of row r at k ^ ((r >> 1) & 3)),
// which keeps the warp's shared-memory writes free of bank conflicts.
__device__ __forceinline__ void stage_row32(uint8_t* buf, int lane, int dtype, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = dtype == MT_BF16 ? pack_bf16x2(v[8 * k + 2 * j], v[8 * k + 2 * j + 1])
                              : pack_f16x2(v[8 * k + 2 * j], v[8 * k + 2 * j + 1]);
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
constexpr int kMaxResStages = 8;

template <int BN, bool TF32, bool PAIR = false, int TST = 0>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * 128;
  static constexpr int B_BYTES = BN * 128;
  // CTA pair: each CTA stages half of the B columns
  static constexpr int B_STAGE_BYTES = PAIR ? B_BYTES / 2 : B_BYTES;
  static constexpr int OPS = TF32 ? 2 : 1;
  static constexpr int STAGE_BYTES = (A_BYTES + B_STAGE_BYTES) * OPS;
  static constexpr int ST_BUFS = store_bufs(BN, TST == 2);
  static constexpr int ST_BYTES = TST ? store_bytes(BN, TST == 2) : 0;
  // TST: the staging buffers come on top of the usual ring where the 227 KB limit allows
  // (320-wide tiles: 56 KB stages, four of them fill the 227 KB limit)
  static constexpr int STAGES_RAW = TST ? (226 * 1024 - ST_BYTES) / STAGE_BYTES
                                        : (BN > 256 ? 224 * 1024 : 200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : (STAGES_RAW < 2 ? 2 : STAGES_RAW);
  // tiles wider than 256 columns (a single MMA's and a TMA box's limit) use two halves: two B
  // loads and two N = BN / 2 MMAs per K step, and one TMEM accumulator instead of two
  static constexpr bool SPLIT_N = BN > 256;
  static constexpr int NBUF = 2 * BN <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = (2 * BN <= 32)    ? 32
                                   : (2 * BN <= 64)  ? 64
                                   : (2 * BN <= 128) ? 128
                                   : (2 * BN <= 256) ? 256
                                                     : 512;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + ST_BYTES + 1024 /*align*/ + kGemmBarBytes;
  // B-resident variant: [B tile, all K chunks][A stages] within kResBytes, barriers after it.
  static constexpr int RES_SMEM_BYTES = kResBytes + 1024 + kGemmBarBytes;
  static_assert(SMEM_BYTES <= 227 * 1024 && RES_SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};

// BRES (B resident): every tile of this CTA has the same column tile (the grid is a multiple of
// the number of column tiles), so the whole [BN x K] B tile is loaded into shared memory once and
// only A streams through the stage ring; for the short-K projections this removes the re-reads
// of B from L2 that otherwise cost more than the A traffic.
//
// PAIR (CTA pairs, cluster of 2): the pair computes a 256 x BN tile with tcgen05 cta_group::2 MMAs
// issued by the even CTA; each CTA loads its own 128 rows of A and BN/2 rows of B (its half of
// the columns), so every SM streams half as many B bytes per MMA as a single-CTA tile of the same
// width.  Each CTA's TMEM holds its 128 rows of D and its epilogue stores them.
//
// TST (TMA-store epilogue, plain GEMMs with 16-bit output): output chunks go through per-warp
// shared-memory buffers and bulk tensor stores (tmD) instead of per-row global stores.
template <int BN, bool TF32, bool CONV, bool BRES, bool PAIR = false, int TST = 0>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmAlo, const __grid_constant__ CUtensorMap tmBlo,
                      const __grid_constant__ CUtensorMap tmD, const TileParams tp, const EpiParams ep,
                      const uint32_t idesc) {
  using Cfg = GemmCfg<BN, TF32, PAIR, TST>;
  static_assert(!TST || (!TF32 && !CONV && !PAIR), "TMA-store epilogue: plain 16-bit GEMMs");
  static_assert(TST != 2 || (!BRES && BN <= 256), "residual through the store buffers: streaming tiles");
  static_assert(!BRES || (!TF32 && !CONV), "B-resident variant: 16-bit GEMMs only");
  static_assert(!PAIR || (!TF32 && !BRES), "CTA-pair variant: 16-bit streaming GEMMs only");
  static_assert(!Cfg::SPLIT_N || (!TF32 && !BRES && !PAIR), "320-wide tiles: 16-bit streaming GEMMs only");
  const int STAGES = BRES ? tp.a_stages : Cfg::STAGES;
  // stage s: A at stage_base + s * STAGE_BYTES; B (not BRES) right after it
  constexpr int STAGE_BYTES = BRES ? Cfg::A_BYTES : Cfg::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sbres = smem;  // BRES: k_iters chunks of B_BYTES
  uint8_t* stage_base = BRES ? smem + tp.k_iters * Cfg::B_BYTES : smem;
  // TST staging: after the ring, or (BRES) the last store_bytes(BN, false) of the resident region (the host
  // sizes the B tile + A stages to leave it free)
  uint8_t* sstore = BRES ? smem + kResBytes - Cfg::ST_BYTES : smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t* full =
      reinterpret_cast<uint64_t*>(smem + (BRES ? kResBytes : Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::ST_BYTES));
  uint64_t* empty = full + (BRES ? kMaxResStages : Cfg::STAGES);
  uint64_t* tfull = empty + (BRES ? kMaxResStages : Cfg::STAGES);
  uint64_t* tempty = tfull + 2;
  uint64_t* b_full = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(b_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* rbar = reinterpret_cast<uint64_t*>(tmem_slot + 2);  // TST residual: [8 warps][ST_BUFS]
  static_assert((2 * 8 + 2 + 2 + 1 + 1 + 8 * Cfg::ST_BUFS) * 8 <= kGemmBarBytes, "GEMM barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PAIR ? 512 : 256);  // pair: both CTAs' epilogue threads
    }
    mbar_init(b_full, 1);
    if (TST == 2)
      for (int i = 0; i < 8 * Cfg::ST_BUFS; ++i) mbar_init(&rbar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (TF32 || (CONV && tp.c_split > 0) || TST == 2) {
      tma_prefetch_desc(&tmAlo);
      tma_prefetch_desc(&tmBlo);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // PAIR: tiles are row-tile pairs; CTA `crank` of the pair takes row tile 2 * pair + crank.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0;
  const int base_tiles = (PAIR ? tp.m_pairs : tp.num_m_tiles) * tp.num_n_tiles * tp.batch;
  const int splits = tp.k_splits > 1 ? tp.k_splits : 1;
  const int total_tiles = base_tiles * splits;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  // K iterations [kb, ke) of tile t (all of them without split K)
  auto k_range = [&](int t, int& kb, int& ke) {
    if (splits > 1) {
      kb = (t / base_tiles) * tp.k_per;
      ke = min(tp.k_iters, kb + tp.k_per);
    } else {
      kb = 0;
      ke = tp.k_iters;
    }
  };
  auto decode = [&](int t, int& b, int& mt, int& nt) {
    t %= base_tiles;
    nt = t % tp.num_n_tiles;
    const int rest = t / tp.num_n_tiles;
    const int mcount = PAIR ? tp.m_pairs : tp.num_m_tiles;
    mt = rest % mcount;
    b = rest / mcount;
    if (PAIR) mt = 2 * mt + (int)crank;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      if (BRES && blockIdx.x < total_tiles) {
        int b, mt, nt;
        decode_tile(tp, blockIdx.x, b, mt, nt);
        mbar_arrive_expect_tx(b_full, tp.k_iters * Cfg::B_BYTES);
        for (int kk = 0; kk < tp.k_iters; ++kk)
          tma_load_3d(sbres + kk * Cfg::B_BYTES, &tmB, b_full, kk * tp.bk, nt * BN, 0);
      }
      for (int t = tile0; t < total_tiles && !*abort_flag; t += tstep) {
        int b, mt, nt;
        decode(t, b, mt, nt);
        const int n0 = nt * BN + (int)crank * (BN / 2);  // PAIR: this CTA's half of the columns
        int q0 = 0, p0 = 0, i0 = 0;
        if (CONV) {
          q0 = (mt % tp.tiles_q) * tp.tw;
          p0 = ((mt / tp.tiles_q) % tp.tiles_p) * tp.th;
          i0 = (mt / (tp.tiles_q * tp.tiles_p)) * tp.tn;
        }
        int kb, ke;
        k_range(t, kb, ke);
        for (int kk = kb; kk < ke; ++kk) {
          if (!mbar_wait(&empty[stage], phase ^ 1, 1, abort_flag)) break;
          // PAIR: the even CTA's barrier counts both CTAs' bytes
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], PAIR ? 2 * STAGE_BYTES : STAGE_BYTES);
          uint8_t* sa = stage_base + stage * STAGE_BYTES;
          uint8_t* sb = sa + Cfg::A_BYTES;
          uint8_t* salo = sb + Cfg::B_BYTES;
          uint8_t* sblo = salo + Cfg::A_BYTES;
          if (CONV) {
            const int rs = kk / tp.c_chunks, cc = kk - rs * tp.c_chunks;
            const int r = rs / tp.S, s = rs - r * tp.S;
            const int cx = cc * tp.bk, wx = q0 * tp.stride_w + s * tp.dil_w - tp.pad_w,
                      hy = p0 * tp.stride_h + r * tp.dil_h - tp.pad_h;
            if (PAIR) {
              const uint32_t fb = mapa_rank(&full[stage], 0);
              tma_load_4d_pair(sa, &tmA, fb, cx, wx, hy, i0);
              tma_load_3d_pair(sb, &tmB, fb, kk * tp.bk, n0, 0);
            } else if (!TF32 && tp.c_split > 0 && cc >= tp.c_split) {
              // second source of a channel concatenation: its own channel coordinate
              tma_load_4d(sa, &tmAlo, &full[stage], (cc - tp.c_split) * tp.bk, wx, hy, i0);
              tma_load_3d(sb, &tmB, &full[stage], kk * tp.bk, n0, 0);
              if (Cfg::SPLIT_N) tma_load_3d(sb + Cfg::B_BYTES / 2, &tmB, &full[stage], kk * tp.bk, n0 + BN / 2, 0);
            } else {
              tma_load_4d(sa, &tmA, &full[stage], cx, wx, hy, i0);
              tma_load_3d(sb, &tmB, &full[stage], kk * tp.bk, n0, 0);
              if (Cfg::SPLIT_N) tma_load_3d(sb + Cfg::B_BYTES / 2, &tmB, &full[stage], kk * tp.bk, n0 + BN / 2, 0);
            }
            if (TF32) {
              tma_load_4d(salo, &tmAlo, &full[stage], cx, wx, hy, i0);
              tma_load_3d(sblo, &tmBlo, &full[stage], kk * tp.bk, n0, 0);
            }
          } else {
            const int ab = tp.a_batched ? b : 0, bb = tp.b_batched ? b : 0;
            if (PAIR) {
              const uint32_t fb = mapa_rank(&full[stage], 0);
              tma_load_3d_pair(sa, &tmA, fb, kk * tp.bk, mt * kBM, ab);
              tma_load_3d_pair(sb, &tmB, fb, kk * tp.bk, n0, bb);
            } else {
              tma_load_3d(sa, &tmA, &full[stage], kk * tp.bk, mt * kBM, ab);
              if (!BRES) tma_load_3d(sb, &tmB, &full[stage], kk * tp.bk, n0, bb);
              if (Cfg::SPLIT_N) tma_load_3d(sb + Cfg::B_BYTES / 2, &tmB, &full[stage], kk * tp.bk, n0 + BN / 2, bb);
            }
            if (TF32) {
              tma_load_3d(salo, &tmAlo, &full[stage], kk * tp.bk, mt * kBM, ab);
              tma_load_3d(sblo, &tmBlo, &full[stage], kk * tp.bk, n0, bb);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (PAIR: the even CTA only) ----------------
    if (lane == 0 && crank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      if (BRES && blockIdx.x < total_tiles && !mbar_wait(b_full, 0, 4, abort_flag)) local = -1;
      for (int t = tile0; local >= 0 && t < total_tiles && !*abort_flag; t += tstep, ++local) {
        const int buf = Cfg::NBUF == 2 ? (local & 1) : 0;
        const uint32_t tph = Cfg::NBUF == 2 ? ((local >> 1) & 1) : (local & 1);
        if (!mbar_wait(&tempty[buf], tph ^ 1, 2, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        int kb, ke;
        k_range(t, kb, ke);
        for (int kk = kb; kk < ke; ++kk) {
          if (!mbar_wait(&full[stage], phase, 3, abort_flag)) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_base + stage * STAGE_BYTES);
          const uint32_t b_addr = BRES ? smem_u32(sbres + kk * Cfg::B_BYTES) : a_addr + Cfg::A_BYTES;
          const uint32_t alo_addr = b_addr + Cfg::B_BYTES;
          const uint32_t blo_addr = alo_addr + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sdesc_sw128(a_addr + k * 32), bd = sdesc_sw128(b_addr + k * 32);
            const uint32_t acc = (kk > kb || k > 0) ? 1u : 0u;
            if (PAIR) {
              umma_f16_pair(d_tmem, ad, bd, idesc, acc);
            } else if (TF32) {
              umma_tf32(d_tmem, ad, bd, idesc, acc);
              umma_tf32(d_tmem, ad, sdesc_sw128(blo_addr + k * 32), idesc, 1u);
              umma_tf32(d_tmem, sdesc_sw128(alo_addr + k * 32), bd, idesc, 1u);
            } else if (Cfg::SPLIT_N) {
              umma_f16(d_tmem, ad, bd, idesc, acc);
              umma_f16(d_tmem + BN / 2, ad, sdesc_sw128(b_addr + Cfg::B_BYTES / 2 + k * 32), idesc, acc);
            } else {
              umma_f16(d_tmem, ad, bd, idesc, acc);
            }
          }
          if (PAIR)
            umma_commit_pair_both(&empty[stage]);
          else
            umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (PAIR)
          umma_commit_pair_both(&tfull[buf]);
        else
          umma_commit(&tfull[buf]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    // Two warps per TMEM lane quarter: warps 2..5 take the even 32-column chunks of the tile,
    // warps 6..9 the odd ones.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const bool geglu = ep.act == MT_EPI_GEGLU;
    const int64_t n_out = geglu ? ep.N / 2 : ep.N;
    int local = 0;
    int sbuf = 0;  // TST: which of this warp's two staging buffers is next
    // TST + residual map: buffer i of this warp holds chunk i (tile columns half*32 + 64 i) of the
    // tile being stored and, once that store has read it, the residual chunk i of the warp's next
    // tile.  `rpend` / `rpar`: per buffer, a residual load in flight / the parity it completes.
    constexpr bool rtma = TST == 2;
    const int nch = (BN - half * 32 + 63) / 64;
    uint64_t* rbar_w = rbar + (warp - 2) * Cfg::ST_BUFS;
    uint8_t* sbw = sstore + (warp - 2) * Cfg::ST_BUFS * 2048;
    uint32_t rpend = 0, rpar = 0;
    // whether chunk i of tile tt exists (columns below N, this warp's rows below M)
    auto res_chunk = [&](int tt, int i, int& x, int& y, int& z) -> bool {
      int b2, mt2, nt2;
      decode(tt, b2, mt2, nt2);
      x = nt2 * BN + half * 32 + 64 * i;
      y = mt2 * kBM + quarter * 32;
      z = b2;
      return x < n_out && y < ep.M;
    };
    // every lane keeps the bookkeeping; lane 0 issues the load
    auto res_issue = [&](int tt, int i) {
      int x, y, z;
      if (tt < total_tiles && res_chunk(tt, i, x, y, z)) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&rbar_w[i], 2048);
          tma_load_3d(sbw + i * 2048, &tmAlo, &rbar_w[i], x, y, z);
        }
        rpend |= 1u << i;
      }
    };
    if (rtma)
      for (int i = 0; i < nch; ++i) res_issue(tile0, i);
    // TST: the warp's 32 output rows x 32 columns via shared memory and one bulk tensor store
    auto store_chunk = [&](const float (&v)[32], int64_t col0, int mt, int b) {
      uint8_t* sb = sstore + ((warp - 2) * 2 + sbuf) * 2048;
      if (lane == 0) bulk_wait_read1();  // the store that last read this buffer has read it
      __syncwarp();
      stage_row32(sb, lane, ep.out_dtype, v);
      gemm_fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&tmD, sb, (int)col0, mt * kBM + (warp & 3) * 32, b);
        bulk_commit();
      }
      sbuf ^= 1;
    };
    for (int t = tile0; t < total_tiles; t += tstep, ++local) {
      const int buf = Cfg::NBUF == 2 ? (local & 1) : 0;
      const uint32_t tph = Cfg::NBUF == 2 ? ((local >> 1) & 1) : (local & 1);
      if (!mbar_wait(&tfull[buf], tph, 4, abort_flag)) break;
      tc_fence_after();
      int b, mt, nt;
      decode(t, b, mt, nt);
      // Map this thread's accumulator row to output coordinates (i0, i1, i2).
      int64_t i0 = 0, i1 = 0, i2 = 0;
      bool valid;
      if (ep.mode == 0) {
        i0 = b;
        i1 = (int64_t)mt * kBM + row;
        valid = i1 < ep.M;
      } else if (ep.mode == 1) {
        const int64_t m = (int64_t)mt * kBM + row;
        valid = m < ep.M;
        i0 = m / (ep.P * ep.Q);
        const int64_t rem = m - i0 * ep.P * ep.Q;
        i1 = rem / ep.Q;
        i2 = rem - i1 * ep.Q;
      } else {
        const int q0 = (mt % tp.tiles_q) * tp.tw;
        const int p0 = ((mt / tp.tiles_q) % tp.tiles_p) * tp.th;
        const int n0 = (mt / (tp.tiles_q * tp.tiles_p)) * tp.tn;
        const int tn_i = row / (tp.th * tp.tw), th_i = (row / tp.tw) % tp.th, tw_i = row % tp.tw;
        i0 = n0 + tn_i;
        i1 = p0 + th_i;
        i2 = q0 + tw_i;
        valid = i0 < ep.M && i1 < ep.P && i2 < ep.Q;
      }
      const int64_t offD = i0 * ep.d_s0 + i1 * ep.d_s1 + i2 * ep.d_s2;
      const int64_t offC = i0 * ep.c_s0 + i1 * ep.c_s1 + i2 * ep.c_s2;
      const int64_t offR = i0 * ep.r_s0 + i1 * ep.r_s1 + i2 * ep.r_s2;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN;
      const bool vec = ep.vec_ok != 0;
      if (splits > 1) {
        // split K: the raw fp32 partial sums of this K range, row (n, p, q) of split t / base
        float* part = ep.part + (int64_t)(t / base_tiles) * ep.part_stride;
        const int64_t m_lin = (i0 * ep.P + i1) * ep.Q + i2;
#pragma unroll 1
        for (int c0 = half * 32; c0 < BN; c0 += 64) {
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_ld_wait();
          const int64_t col0 = (int64_t)nt * BN + c0;
          const int64_t remain = ep.N - col0;
          const int nvalid = remain < 32 ? (int)remain : 32;
          if (valid && nvalid > 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            row_store(part, MT_F32, m_lin * ep.N + col0, nvalid, true, v);
          }
        }
      } else if (rtma) {
        // plain GEMM, TMA-store epilogue, residual from the prefetched buffers (mode 0, no GEGLU)
        const int tnext = t + tstep;
        uint32_t issued = 0;  // buffers already refilled for tnext
#pragma unroll 1
        for (int i = 0; i < nch; ++i) {
          const int c0 = half * 32 + 64 * i;
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_ld_wait();
          const int64_t col0 = (int64_t)nt * BN + c0;
          if (col0 >= n_out) break;  // chunks past N: none after this one either
          const int nvalid = n_out - col0 < 32 ? (int)(n_out - col0) : 32;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = ep.alpha * __uint_as_float(r[j]);
          if (ep.bias)
            row_load_add(ep.bias, ep.bias_dtype, i0 * ep.bias_bstride + col0, nvalid, ep.bias_vec != 0, 1.f, v);
          if (ep.C && valid) row_load_add(ep.C, ep.out_dtype, offC + col0, nvalid, vec, ep.beta, v);
          if (ep.act == MT_EPI_GELU) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) gelu_poly_pair(v[j], v[j + 1]);
          } else if (ep.act == MT_EPI_SILU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
          } else if (ep.act == MT_EPI_QUICK_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = v[j] * (1.0f / (1.0f + expf(-__fmul_rn(v[j], 1.702f))));
          }
          uint8_t* sb = sbw + i * 2048;
          if ((rpend >> i) & 1) {
            const bool got = mbar_wait(&rbar_w[i], (rpar >> i) & 1, 19, abort_flag);
            if (!__all_sync(0xffffffffu, got)) break;
            rpend &= ~(1u << i);
            rpar ^= 1u << i;
            // this lane's row: 16-byte chunk k at k ^ ((lane >> 1) & 3) (64-byte swizzle)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 u = *reinterpret_cast<const uint4*>(sb + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16));
              const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float2 f;
                if (ep.out_dtype == MT_BF16) {
                  f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
                } else {
                  f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
                }
                v[8 * k + 2 * j] += f.x;
                v[8 * k + 2 * j + 1] += f.y;
              }
            }
            __syncwarp();  // every lane has read the residual before the buffer is overwritten
          }
          stage_row32(sb, lane, ep.out_dtype, v);
          gemm_fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmD, sb, (int)col0, mt * kBM + quarter * 32, b);
            bulk_commit();
            if (i > 0) bulk_wait_read1();  // the store of chunk i - 1 has read its buffer
          }
          if (i > 0) {  // refill buffer i - 1 with the residual of tnext
            res_issue(tnext, i - 1);
            issued |= 1u << (i - 1);
          }
        }
        if (lane == 0) bulk_wait_read0();
        for (int i = 0; i < nch; ++i)
          if (!((issued >> i) & 1) && !((rpend >> i) & 1)) res_issue(tnext, i);
        __syncwarp();
        if (*abort_flag) break;
      } else if (!geglu) {
#pragma unroll 1
        for (int c0 = half * 32; c0 < BN; c0 += 64) {
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_ld_wait();
          const int64_t col0 = (int64_t)nt * BN + c0;
          const int64_t remain = n_out - col0;
          const int nvalid = remain < 32 ? (int)remain : 32;
          // TST: every lane of the warp takes part in the store (rows past M are clipped by TMA)
          if ((valid || TST) && nvalid > 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = ep.alpha * __uint_as_float(r[j]);
            if (ep.bias)
              row_load_add(ep.bias, ep.bias_dtype, i0 * ep.bias_bstride + col0, nvalid, ep.bias_vec != 0, 1.f, v);
            if (ep.C && valid) row_load_add(ep.C, ep.out_dtype, offC + col0, nvalid, vec, ep.beta, v);
            if (ep.act == MT_EPI_GELU) {
              if (TF32) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = gelu_f(v[j]);
              } else {
#pragma unroll
                for (int j = 0; j < 32; j += 2) gelu_poly_pair(v[j], v[j + 1]);
              }
            } else if (ep.act == MT_EPI_SILU) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
            } else if (ep.act == MT_EPI_QUICK_GELU) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = v[j] * (1.0f / (1.0f + expf(-__fmul_rn(v[j], 1.702f))));
            }
            if (ep.res && valid) row_load_add(ep.res, ep.out_dtype, offR + col0, nvalid, vec, 1.f, v);
            if (TST)
              store_chunk(v, col0, mt, b);
            else
              row_store(ep.D, ep.out_dtype, offD + col0, nvalid, vec, v);
          }
        }
      } else {
        // (value, gate) 64-column groups: tile columns [g*128, g*128+64) are values, the next
        // 64 their gates; output column = nt*BN/2 + g*64 + j.
#pragma unroll 1
        for (int g = 0; g < BN / 128; ++g) {
          {
            const int h = half * 32;
            uint32_t rv[32], rg[32];
            tmem_ld32(taddr + g * 128 + h, rv);
            tmem_ld32(taddr + g * 128 + 64 + h, rg);
            tmem_ld_wait();
            const int64_t gcol_v = (int64_t)nt * BN + g * 128 + h;
            const int64_t col0 = (int64_t)nt * (BN / 2) + g * 64 + h;
            const int64_t remain = n_out - col0;
            const int nvalid = remain < 32 ? (int)remain : 32;
            if ((valid || TST) && nvalid > 0) {
              float v[32], gt[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                v[j] = ep.alpha * __uint_as_float(rv[j]);
                gt[j] = ep.alpha * __uint_as_float(rg[j]);
              }
              if (ep.bias) {
                row_load_add(ep.bias, ep.bias_dtype, i0 * ep.bias_bstride + gcol_v, nvalid, ep.bias_vec != 0, 1.f, v);
                row_load_add(ep.bias, ep.bias_dtype, i0 * ep.bias_bstride + gcol_v + 64, nvalid, ep.bias_vec != 0, 1.f,
                             gt);
              }
              epi_gelu32<TF32>(v, gt);
              if (ep.res && valid) row_load_add(ep.res, ep.out_dtype, offR + col0, nvalid, vec, 1.f, v);
              if (TST)
                store_chunk(v, col0, mt, b);
              else
                row_store(ep.D, ep.out_dtype, offD + col0, nvalid, vec, v);
            }
          }
        }
      }
      tc_fence_before();
      if (PAIR)
        mbar_arrive_cluster(mapa_rank(&tempty[buf], 0));
      else
        mbar_arrive(&tempty[buf]);
    }
    if (TST && lane == 0) bulk_wait_all();  // this warp's stores are done before the CTA exits
    if (rtma && lane == 0) {
      // after an abort: let residual loads still in flight land (bounded) before the CTA exits
      for (int i = 0; i < nch; ++i) {
        if (!((rpend >> i) & 1)) continue;
        const long long start = clock64();
        while (!mbar_try_wait(&rbar_w[i], (rpar >> i) & 1) && clock64() - start < kWaitBudgetCycles) {
        }
      }
    }
  }
  __syncthreads();
  if (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------------------------
// Split-K reduction of an implicit convolution: out[n, p, q, c] = epilogue(sum_s part[s][m][c])
// with m = (n * P + p) * Q + q, the splits added in order 0..S-1 (fixed, so results do not depend
// on the batch), then the GEMM epilogue's order: alpha, bias (per column or per image), activation,
// residual.  One thread per 8 consecutive columns.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* part, int splits, int64_t stride,
                                                            int64_t rows, int64_t N, const EpiParams ep) {
  const int64_t n8 = N / 8;
  const int64_t total = rows * n8;
  const int64_t PQ = ep.P * ep.Q;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / n8, c = (i - m * n8) * 8;
    float v[8];
    {
      const float4* q = reinterpret_cast<const float4*>(part + m * N + c);
      const float4 a = q[0], b = q[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    for (int s = 1; s < splits; ++s) {
      const float4* q = reinterpret_cast<const float4*>(part + s * stride + m * N + c);
      const float4 a = q[0], b = q[1];
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    const int64_t n = m / PQ, rem = m - n * PQ, pp = rem / ep.Q, qq = rem - pp * ep.Q;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= ep.alpha;
    if (ep.bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += load_as_f32(ep.bias, n * ep.bias_bstride + c + j, ep.bias_dtype);
    }
    if (ep.act == MT_EPI_GELU) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = gelu_f(v[j]);
    } else if (ep.act == MT_EPI_SILU) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = silu_f(v[j]);
    }
    if (ep.res) {
      const int64_t offR = n * ep.r_s0 + pp * ep.r_s1 + qq * ep.r_s2 + c;
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += load_as_f32(ep.res, offR + j, ep.out_dtype);
    }
    const int64_t offD = n * ep.d_s0 + pp * ep.d_s1 + qq * ep.d_s2 + c;
    if (ep.vec_ok && (ep.out_dtype == MT_BF16 || ep.out_dtype == MT_F16)) {
      uint4 w;
      uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        wp[j] = ep.out_dtype == MT_BF16 ? pack_bf16x2(v[2 * j], v[2 * j + 1]) : pack_f16x2(v[2 * j], v[2 * j + 1]);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(ep.D) + offD) = w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) store_from_f32(ep.D, offD + j, ep.out_dtype, v[j]);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Host side.

struct GemmLaunch {
  CUtensorMap a, b, alo, blo;
  TileParams tp;
  EpiParams ep;
  int kind;  // MT_BF16 / MT_F16 / MT_F32 (tf32 x3)
  int bn;
  bool conv;
  // B operand as mapped (K-major), kept so the CTA-pair variant can re-map it with half-width boxes
  const void* b_ptr; int64_t b_K, b_rows, b_batch, b_pitch, b_bstride;
  // TMA-store epilogue: output map (32 x 32 boxes, 64-byte swizzle) when `tst`
  CUtensorMap d;
  bool tst;
};

static int map_kmajor(CUtensorMap* m, int dtype, const void* base, int64_t K, int64_t rows, int64_t batch,
                      int64_t pitch, int64_t bstride, int box_rows);

template <int BN, bool TF32, bool CONV, bool BRES = false, bool PAIR = false, int TST = 0>
static int launch_variant(const GemmLaunch& L, cudaStream_t st) {
  using Cfg = GemmCfg<BN, TF32, PAIR, TST>;
  constexpr int smem = BRES ? Cfg::RES_SMEM_BYTES : Cfg::SMEM_BYTES;
  auto kern = gemm_sm100_kernel<BN, TF32, CONV, BRES, PAIR, TST>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                        "gemm smem attribute");
    if (rc) return rc;
    attr_set[dev & 63] = true;
  }
  const int64_t tiles =
      (int64_t)L.tp.num_m_tiles * L.tp.num_n_tiles * L.tp.batch * std::max(1, L.tp.k_splits);
  if (tiles > 0x7fffffffLL) return fail(MT_ERR_UNSUPPORTED, "gemm: too many tiles");
  int grid = (int)std::min<int64_t>(tiles, num_sms());
  if (BRES) grid = num_sms() / L.tp.num_n_tiles * L.tp.num_n_tiles;  // one column tile per CTA
  const int fmt = L.kind == MT_BF16 ? 1 : L.kind == MT_F16 ? 0 : 2;
  if (PAIR) {
    // clusters of two CTAs, one pair per two SMs; the MMA spans 256 rows
    const int64_t pairs = (int64_t)L.tp.m_pairs * L.tp.num_n_tiles * L.tp.batch;
    GemmLaunch P = L;
    int rc = map_kmajor(&P.b, L.kind, L.b_ptr, L.b_K, L.b_rows, L.b_batch, L.b_pitch, L.b_bstride, BN / 2);
    if (rc) return rc;
    const uint32_t idesc = make_idesc(fmt, 2 * kBM, BN);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(pairs, num_sms() / 2)));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P.a, P.b, P.alo, P.b, P.a, P.tp, P.ep, idesc);
    if (e != cudaSuccess) return fail(MT_ERR_LAUNCH, "gemm_sm100 (CTA pairs): %s", cudaGetErrorString(e));
    return check_launch("gemm_sm100_pair");
  }
  const uint32_t idesc = make_idesc(fmt, kBM, Cfg::SPLIT_N ? BN / 2 : BN);
  kern<<<grid, kGemmThreads, smem, st>>>(L.a, L.b, L.alo, L.blo, TST ? L.d : L.a, L.tp, L.ep, idesc);
  return check_launch("gemm_sm100");
}

// Whether the B-resident variant pays: 16-bit, unbatched, the [BN x K] B tile leaves room for at
// least 3 A stages, a grid that is a multiple of the column-tile count loses at most 4% of the SMs,
// and every CTA gets at least 8 tiles to amortise its B load.  A_stages is set as a side effect.
static bool use_bres(GemmLaunch& L) {
  static const bool off = getenv("MT_GEMM_NO_BRES") != nullptr;
  if (off || L.kind == MT_F32 || L.conv || L.tp.batch != 1 || L.bn > 256) return false;
  const int b_bytes = L.bn * 128 * L.tp.k_iters;
  const int stages = std::min(kMaxResStages, (kResBytes - (L.tst ? store_bytes(L.bn, false) : 0) - b_bytes) / (kBM * 128));
  if (stages < 3) return false;
  const int sms = num_sms(), nn = L.tp.num_n_tiles;
  if (nn > sms) return false;
  const int grid = sms / nn * nn;
  if ((sms - grid) * 25 > sms) return false;
  if ((int64_t)L.tp.num_m_tiles * nn < 8LL * grid) return false;
  L.tp.a_stages = stages;
  return true;
}

// Whether the CTA-pair variant is used: 16-bit, column tiles of 128 / 160 / 256 (half-width B
// boxes of whole 8-row swizzle atoms), at least two row tiles.  MT_GEMM_PAIR=1 turns it on.
static bool use_pair(GemmLaunch& L) {
  static const bool off = [] {
    const char* e = getenv("MT_GEMM_PAIR");
    return !(e && e[0] == '1');
  }();
  if (off || L.kind == MT_F32 || !L.b_ptr || L.tp.c_split > 0 || L.tp.k_splits > 1) return false;
  if (L.bn != 128 && L.bn != 160 && L.bn != 256) return false;
  if (L.tp.num_m_tiles < 2) return false;
  L.tp.m_pairs = (L.tp.num_m_tiles + 1) / 2;
  return true;
}

static int dispatch(GemmLaunch& L, cudaStream_t st) {
  if (L.kind == MT_F32) {
    if (L.conv) return launch_variant<128, true, true>(L, st);
    if (L.bn == 64) return launch_variant<64, true, false>(L, st);
    return launch_variant<128, true, false>(L, st);
  }
  if (use_pair(L)) {
    if (L.conv) {
      switch (L.bn) {
        case 128: return launch_variant<128, false, true, false, true>(L, st);
        case 160: return launch_variant<160, false, true, false, true>(L, st);
        default: return launch_variant<256, false, true, false, true>(L, st);
      }
    }
    if (!use_bres(L)) {
      switch (L.bn) {
        case 128: return launch_variant<128, false, false, false, true>(L, st);
        case 160: return launch_variant<160, false, false, false, true>(L, st);
        default: return launch_variant<256, false, false, false, true>(L, st);
      }
    }
  }
  if (L.conv) {
    switch (L.bn) {
      case 64: return launch_variant<64, false, true>(L, st);
      case 128: return launch_variant<128, false, true>(L, st);
      case 160: return launch_variant<160, false, true>(L, st);
      case 320: return launch_variant<320, false, true>(L, st);
      default: return launch_variant<256, false, true>(L, st);
    }
  }
  if (L.tst) {
    // the residual instance gives up a stage of the operand ring for its staging buffers: it pays
    // for short reductions (measured: K = 640 gains 15 %, K = 1280 loses 3 %)
    if (L.ep.res_tma && (L.bn == 128 || L.bn == 160 || L.bn == 256) && L.tp.k_iters <= 10 && !use_bres(L)) {
      switch (L.bn) {
        case 128: return launch_variant<128, false, false, false, false, 2>(L, st);
        case 160: return launch_variant<160, false, false, false, false, 2>(L, st);
        default: return launch_variant<256, false, false, false, false, 2>(L, st);
      }
    }
    L.ep.res_tma = 0;
    if (use_bres(L)) {
      switch (L.bn) {
        case 64: return launch_variant<64, false, false, true, false, true>(L, st);
        case 128: return launch_variant<128, false, false, true, false, true>(L, st);
        case 160: return launch_variant<160, false, false, true, false, true>(L, st);
        default: return launch_variant<256, false, false, true, false, true>(L, st);
      }
    }
    switch (L.bn) {
      case 64: return launch_variant<64, false, false, false, false, true>(L, st);
      case 128: return launch_variant<128, false, false, false, false, true>(L, st);
      case 160: return launch_variant<160, false, false, false, false, true>(L, st);
      case 320: return launch_variant<320, false, false, false, false, true>(L, st);
      default: return launch_variant<256, false, false, false, false, true>(L, st);
    }
  }
  if (use_bres(L)) {
    switch (L.bn) {
      case 64: return launch_variant<64, false, false, true>(L, st);
      case 128: return launch_variant<128, false, false, true>(L, st);
      case 160: return launch_variant<160, false, false, true>(L, st);
      default: return launch_variant<256, false, false, true>(L, st);
    }
  }
  switch (L.bn) {
    case 64: return launch_variant<64, false, false>(L, st);
    case 128: return launch_variant<128, false, false>(L, st);
    case 160: return launch_variant<160, false, false>(L, st);
    case 320: return launch_variant<320, false, false>(L, st);
    default: return launch_variant<256, false, false>(L, st);
  }
}

// Column-tile width (GEGLU needs a multiple of 128).  fp32 (two operand pairs per stage) and
// implicit conv with fp32 use 128.
static int pick_bn(int64_t N, int kind, bool geglu, bool conv) {
  if (kind == MT_F32) return (N <= 64 && !geglu && !conv) ? 64 : 128;
  // Tuning knob: MT_GEMM_BN=<64|128|160|256> forces the column tile of bf16/f16 GEMMs.
  static const int forced = [] {
    const char* e = getenv("MT_GEMM_BN");
    const int v = e ? atoi(e) : 0;
    return (v == 64 || v == 128 || v == 160 || v == 256 || v == 320) ? v : 0;
  }();
  if (forced == 320 && geglu) return 256;  // GEGLU tiles pair 64-column value / gate groups
  if (forced && !(geglu && forced % 128)) return forced;
  if (geglu) return N % 256 == 0 ? 256 : 128;
  if (N <= 64) return 64;
  // Wider tiles move fewer operand bytes per MMA cycle, and the mainloop is bound by the L2 ->
  // shared-memory delivery rate (about 55-75 bytes per clock per SM measured at every width), so
  // the tile-level efficiency grows with the width: measured 0.28 / 0.50 / 0.66 / 0.88 of the bf16
  // peak for 64 / 128 / 160 / 256 columns.  Pick the width minimising padded columns / efficiency.
  const int cands[4] = {256, 160, 128, 64};
  const double eff[4] = {0.88, 0.66, 0.50, 0.28};
  int best = 256;
  double best_cost = 1e300;
  for (int i = 0; i < 4; ++i) {
    const double cost = (double)((N + cands[i] - 1) / cands[i] * cands[i]) / eff[i];
    if (cost < best_cost) {
      best_cost = cost;
      best = cands[i];
    }
  }
  return best;
}

// Small problems (fewer tiles than SMs — the deep UNet levels at a few samples per GPU) use a
// narrower column tile to spread over more SMs.  Each output element is still accumulated over
// K in the same order, so results do not depend on the choice (batch invariance is kept).
static int narrow_bn(int bn, int64_t N, int64_t m_tiles, bool geglu) {
  const int64_t sms = num_sms();
  auto tiles = [&](int c) { return m_tiles * ((N + c - 1) / c); };
  const int cands[2] = {128, 64};
  for (int c : cands) {
    if (tiles(bn) >= sms) break;
    if (c >= bn || (geglu && c % 128 != 0)) continue;
    if (tiles(c) > tiles(bn)) bn = c;
  }
  return bn;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int bias_vec_ok(const void* bias, int dtype, int64_t bstride) {
  if (!bias || (dtype != MT_BF16 && dtype != MT_F32)) return 0;
  return aligned16(bias) && (bstride * dtype_size(dtype)) % 16 == 0;
}

// 3-D K-major map: dims {K, rows, batch}, 128-byte-wide box of `box_rows` rows.
static int map_kmajor(CUtensorMap* m, int dtype, const void* base, int64_t K, int64_t rows, int64_t batch,
                      int64_t pitch, int64_t bstride, int box_rows) {
  const int es = dtype_size(dtype);
  uint64_t dims[3] = {(uint64_t)K, (uint64_t)rows, (uint64_t)std::max<int64_t>(batch, 1)};
  uint64_t strides[2] = {(uint64_t)(pitch * es), (uint64_t)((batch > 1 ? bstride : rows * pitch) * es)};
  uint32_t box[3] = {(uint32_t)(128 / es), (uint32_t)box_rows, 1};
  return make_tensor_map(m, dtype, 3, base, dims, strides, box, 128);
}

struct WsCursor {
  char* base;
  size_t off;
  void* take(size_t bytes) {
    off = align_up(off, 256);
    void* p = base ? base + off : nullptr;
    off += bytes;
    return p;
  }
};

// Operand plan for a GEMM; with `run == false` it only measures the workspace.
struct GemmPlan {
  const void* A; int64_t lda, sa; bool a_batched;
  const void* B; int64_t ldb, sb; bool b_batched;
  const void* Alo; const void* Blo;
  int64_t Kp;
};

static int plan_gemm(const mt_gemm_desc& d, WsCursor& ws, GemmPlan& p, cudaStream_t st, bool run) {
  const int es = dtype_size(d.dtype);
  const int64_t align_elems = 16 / es;
  p.Kp = (d.K + align_elems - 1) / align_elems * align_elems;
  const bool tf32 = d.dtype == MT_F32;
  // A: want [M, K] K-major with a 16-byte aligned pitch.
  const bool a_ok = !d.a_trans && aligned16(d.A) && (d.lda * es) % 16 == 0 &&
                    (d.batch == 1 || d.stride_a == 0 || (d.stride_a * es) % 16 == 0);
  p.a_batched = d.batch > 1 && d.stride_a != 0;
  const int64_t a_b = p.a_batched ? d.batch : 1;
  const int64_t asr = d.a_trans ? 1 : d.lda, asc = d.a_trans ? d.lda : 1;
  if (a_ok) {
    p.A = d.A; p.lda = d.lda; p.sa = d.stride_a;
  } else {
    void* dst = ws.take((size_t)a_b * d.M * p.Kp * es);
    p.A = dst; p.lda = p.Kp; p.sa = d.M * p.Kp;
    if (run) {
      int rc = launch_pack2d(dst, nullptr, d.A, d.dtype, a_b, d.M, d.K, asr, asc, d.stride_a, p.Kp, st);
      if (rc) return rc;
    }
  }
  p.Alo = nullptr;
  if (tf32) {
    if (d.A_lo) {
      p.Alo = d.A_lo;
    } else {
      void* lo = ws.take((size_t)a_b * d.M * p.Kp * 4);
      p.Alo = lo;
      if (run) {
        int rc = launch_pack2d(nullptr, (float*)lo, d.A, d.dtype, a_b, d.M, d.K, asr, asc, d.stride_a, p.Kp, st);
        if (rc) return rc;
      }
    }
  }
  // B: want [N, K] K-major.
  const bool b_ok = d.b_trans && aligned16(d.B) && (d.ldb * es) % 16 == 0 &&
                    (d.batch == 1 || d.stride_b == 0 || (d.stride_b * es) % 16 == 0);
  p.b_batched = d.batch > 1 && d.stride_b != 0;
  const int64_t b_b = p.b_batched ? d.batch : 1;
  const int64_t bsr = d.b_trans ? d.ldb : 1, bsc = d.b_trans ? 1 : d.ldb;
  if (b_ok) {
    p.B = d.B; p.ldb = d.ldb; p.sb = d.stride_b;
  } else {
    void* dst = ws.take((size_t)b_b * d.N * p.Kp * es);
    p.B = dst; p.ldb = p.Kp; p.sb = d.N * p.Kp;
    if (run) {
      int rc = launch_pack2d(dst, nullptr, d.B, d.dtype, b_b, d.N, d.K, bsr, bsc, d.stride_b, p.Kp, st);
      if (rc) return rc;
    }
  }
  p.Blo = nullptr;
  if (tf32) {
    if (d.B_lo) {
      p.Blo = d.B_lo;
    } else {
      void* lo = ws.take((size_t)b_b * d.N * p.Kp * 4);
      p.Blo = lo;
      if (run) {
        int rc = launch_pack2d(nullptr, (float*)lo, d.B, d.dtype, b_b, d.N, d.K, bsr, bsc, d.stride_b, p.Kp, st);
        if (rc) return rc;
      }
    }
  }
  return MT_OK;
}

static int validate_gemm(const mt_gemm_desc& d) {
  if (d.M < 0 || d.N < 0 || d.K < 0 || d.batch < 1) return fail(MT_ERR_INVALID, "gemm: negative size");
  if (d.dtype != MT_F32 && d.dtype != MT_BF16 && d.dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "gemm: input dtype %d", d.dtype);
  if (d.out_dtype != MT_F32 && d.out_dtype != MT_BF16 && d.out_dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "gemm: output dtype %d", d.out_dtype);
  if (d.epilogue < MT_EPI_NONE || d.epilogue > MT_EPI_QUICK_GELU) return fail(MT_ERR_UNSUPPORTED, "gemm: epilogue");
  if (d.epilogue == MT_EPI_GEGLU && d.N % 128 != 0)
    return fail(MT_ERR_INVALID, "gemm: GEGLU needs N %% 128 == 0 (interleaved 64-column groups)");
  if (d.M > 0 && d.N > 0 && d.K == 0) return fail(MT_ERR_UNSUPPORTED, "gemm: K == 0 (caller fills)");
  if (d.M > 0 && d.N > 0 && (!d.A || !d.B || !d.D)) return fail(MT_ERR_INVALID, "gemm: null operand");
  if (d.M > INT32_MAX || d.N > INT32_MAX || d.K > INT32_MAX) return fail(MT_ERR_UNSUPPORTED, "gemm: size");
  return MT_OK;
}

size_t gemm_workspace(const mt_gemm_desc& d) {
  if (validate_gemm(d) != MT_OK) return 0;
  WsCursor ws{nullptr, 0};
  GemmPlan p;
  plan_gemm(d, ws, p, nullptr, false);
  return ws.off;
}

int run_gemm(const mt_gemm_desc& d, void* wsp, size_t ws_bytes, cudaStream_t st) {
  int rc = validate_gemm(d);
  if (rc) return rc;
  if (d.M == 0 || d.N == 0) return MT_OK;
  const size_t need = gemm_workspace(d);
  if (need > 0 && (!wsp || ws_bytes < need)) return fail(MT_ERR_WORKSPACE, "gemm: workspace of %zu bytes required", need);
  WsCursor ws{(char*)wsp, 0};
  GemmPlan p;
  rc = plan_gemm(d, ws, p, st, true);
  if (rc) return rc;

  GemmLaunch L{};
  L.kind = d.dtype;
  L.conv = false;
  const bool geglu = d.epilogue == MT_EPI_GEGLU;
  L.bn = pick_bn(d.N, d.dtype, geglu, false);
  if (d.dtype != MT_F32) L.bn = narrow_bn(L.bn, d.N, (int64_t)((d.M + kBM - 1) / kBM) * d.batch, geglu);
  const int64_t a_b = p.a_batched ? d.batch : 1, b_b = p.b_batched ? d.batch : 1;
  rc = map_kmajor(&L.a, d.dtype, p.A, d.K, d.M, a_b, p.lda, p.sa, kBM);
  if (!rc) rc = map_kmajor(&L.b, d.dtype, p.B, d.K, d.N, b_b, p.ldb, p.sb, L.bn > 256 ? L.bn / 2 : L.bn);
  L.b_ptr = p.B; L.b_K = d.K; L.b_rows = d.N; L.b_batch = b_b; L.b_pitch = p.ldb; L.b_bstride = p.sb;
  if (!rc && d.dtype == MT_F32) {
    rc = map_kmajor(&L.alo, MT_F32, p.Alo, d.K, d.M, a_b, p.Kp, d.M * p.Kp, kBM);
    if (!rc) rc = map_kmajor(&L.blo, MT_F32, p.Blo, d.K, d.N, b_b, p.Kp, d.N * p.Kp, L.bn);
  } else {
    L.alo = L.a;
    L.blo = L.b;
  }
  if (rc) return rc;
  TileParams& tp = L.tp;
  tp.num_m_tiles = (int)((d.M + kBM - 1) / kBM);
  tp.num_n_tiles = (int)((d.N + L.bn - 1) / L.bn);
  tp.batch = (int)d.batch;
  tp.bk = 128 / dtype_size(d.dtype);
  tp.k_iters = (int)((d.K + tp.bk - 1) / tp.bk);
  tp.a_batched = p.a_batched;
  tp.b_batched = p.b_batched;
  EpiParams& ep = L.ep;
  ep.mode = 0;
  ep.M = d.M;
  ep.N = d.N;
  ep.D = d.D; ep.out_dtype = d.out_dtype; ep.d_s0 = d.stride_d; ep.d_s1 = d.ldd; ep.d_s2 = 0;
  ep.C = (d.beta != 0.f) ? d.C : nullptr; ep.c_s0 = d.stride_c; ep.c_s1 = d.ldc; ep.c_s2 = 0; ep.beta = d.beta;
  ep.res = d.residual; ep.r_s0 = d.stride_r; ep.r_s1 = d.ldr; ep.r_s2 = 0;
  ep.bias = d.bias; ep.bias_dtype = d.bias_dtype; ep.bias_bstride = d.bias_batch_stride;
  ep.alpha = d.alpha; ep.act = d.epilogue;
  const int oes = dtype_size(d.out_dtype);
  bool vec = aligned16(d.D) && (d.ldd * oes) % 16 == 0 && (d.batch == 1 || (d.stride_d * oes) % 16 == 0);
  if (ep.C) vec = vec && aligned16(d.C) && (d.ldc * oes) % 16 == 0 && (d.batch == 1 || (d.stride_c * oes) % 16 == 0);
  if (ep.res)
    vec = vec && aligned16(d.residual) && (d.ldr * oes) % 16 == 0 && (d.batch == 1 || (d.stride_r * oes) % 16 == 0);
  ep.vec_ok = vec;
  ep.bias_vec = bias_vec_ok(d.bias, d.bias_dtype, d.bias_batch_stride);
  // TMA-store epilogue for 16-bit outputs with 16-byte aligned rows (MT_GEMM_TSTORE=0 turns it off)
  static const bool tst_off = [] {
    const char* e = getenv("MT_GEMM_TSTORE");
    return e && e[0] == '0';
  }();
  L.tst = false;
  if (!tst_off && d.dtype != MT_F32 && (d.out_dtype == MT_BF16 || d.out_dtype == MT_F16) && vec &&
      d.M <= INT32_MAX && d.N <= INT32_MAX) {
    const int64_t n_out = geglu ? d.N / 2 : d.N;
    uint64_t dims[3] = {(uint64_t)n_out, (uint64_t)d.M, (uint64_t)d.batch};
    uint64_t strides[2] = {(uint64_t)(d.ldd * oes), (uint64_t)((d.batch > 1 ? d.stride_d : d.M * d.ldd) * oes)};
    uint32_t box[3] = {32, 32, 1};
    L.tst = make_tensor_map(&L.d, d.out_dtype, 3, d.D, dims, strides, box, 64) == MT_OK;
    // the residual through the same box geometry (MT_GEMM_RES_TMA=0 turns it off)
    static const bool rt_off = [] {
      const char* e = getenv("MT_GEMM_RES_TMA");
      return e && e[0] == '0';
    }();
    if (L.tst && !rt_off && ep.res && !geglu && (d.batch == 1 || d.stride_r != 0)) {
      uint64_t rstrides[2] = {(uint64_t)(d.ldr * oes), (uint64_t)((d.batch > 1 ? d.stride_r : d.M * d.ldr) * oes)};
      ep.res_tma = make_tensor_map(&L.alo, d.out_dtype, 3, d.residual, dims, rstrides, box, 64) == MT_OK;
    }
  }
  return dispatch(L, st);
}

// ---------------------------------------------------------------------------------------------
// Convolution.

// Implicit GEMM needs whole 128-byte channel chunks; strides 1 and 2 (the tensor map walks the
// input with that element stride, so a stride-2 box spans twice the output tile's extent).
static bool conv_implicit_ok(const mt_conv2d_desc& d) {
  const int bk = 128 / dtype_size(d.dtype);
  return d.stride_h >= 1 && d.stride_h <= 2 && d.stride_w >= 1 && d.stride_w <= 2 && d.C % bk == 0 &&
         d.groups == 1;
}

int64_t conv_packed_channels(int64_t C, int64_t R, int64_t S, int dtype) {
  const int es = dtype_size(dtype);
  if (es == 0) return C;
  const int64_t a = 16 / es;
  return (C + a - 1) / a * a;
}

static bool is_channels_last(const int64_t* s, int64_t C, int64_t H, int64_t W) {
  return s[1] == 1 && s[3] == C && s[2] == W * C && s[0] == H * W * C;
}

// `cat` (optional): the input is the channel concatenation of d.x (cat->c1 channels, strides
// d.x_strides) and cat->x2 (d.C - c1 channels); only the implicit 16-bit path takes it.
struct ConvCat {
  const void* x2;
  int64_t x2_strides[4];
  int64_t c1;
};

// K splits of an implicit 16-bit convolution: a function of the per-image output size and the
// reduction length only (never of the batch), so a sample's result is the same at every batch size.
// Small images (the UNet's 16x16 and 8x8 levels) have few output rows per image; splitting K keeps
// the GPU busy at small batches and evens out the last wave at large ones.  MT_CONV_SPLITK=0 turns
// it off.
static int conv_k_splits(const mt_conv2d_desc& d, int64_t k_iters) {
  static const bool off = [] {
    const char* e = getenv("MT_CONV_SPLITK");
    return e && e[0] == '0';
  }();
  if (off || d.K % 8 != 0) return 1;
  if (d.dtype == MT_F32) {
    // 3xTF32: the tensor core's fp32 accumulation is biased (measured: relative error growing
    // linearly with K, 1.6e-4 at K = 23040 even for exactly representable tf32 inputs), so the
    // reduction is cut into chunks of about 1024 elements (32 iterations of 32) whose sums are
    // added in IEEE fp32 by the split reduction: relative error ~sqrt(K * 1024) / K of the
    // unchunked figure (measured 8.6e-5 -> see the fp32 conv tests).
    const int64_t s = std::min<int64_t>(16, (k_iters + 31) / 32);
    return s >= 2 ? (int)s : 1;
  }
  if (k_iters < 64) return 1;
  const int64_t pq = d.P * d.Q;
  if (pq <= 64) return 4;
  if (pq <= 256) return 2;
  return 1;
}

static int plan_conv(const mt_conv2d_desc& d, WsCursor& ws, bool run, cudaStream_t st, GemmLaunch* L,
                     const ConvCat* cat = nullptr, bool allow_split = false) {
  const int es = dtype_size(d.dtype);
  const bool tf32 = d.dtype == MT_F32;
  const bool implicit = conv_implicit_ok(d);
  if (cat && (tf32 || !implicit)) return fail(MT_ERR_UNSUPPORTED, "conv2d_cat: implicit 16-bit convolutions only");
  const int64_t Cp = conv_packed_channels(d.C, d.R, d.S, d.dtype);
  const int64_t Kg = d.R * d.S * Cp;  // GEMM K (16-byte aligned pitch)
  // Weights -> [K, R, S, Cp].
  const void* wp = d.w;
  const void* wlo = d.w_lo;
  if (!d.w_packed) {
    void* dst = ws.take((size_t)d.K * Kg * es);
    void* lo = tf32 ? ws.take((size_t)d.K * Kg * 4) : nullptr;
    wp = dst;
    wlo = lo;
    if (run) {
      int rc = launch_conv_pack_weight(dst, (float*)lo, d.w, d.dtype, d.K, d.C, d.R, d.S, Cp, st);
      if (rc) return rc;
    }
  } else if (tf32 && !d.w_lo) {
    void* lo = ws.take((size_t)d.K * Kg * 4);
    wlo = lo;
    if (run) {
      int rc = launch_pack2d(nullptr, (float*)lo, d.w, MT_F32, 1, d.K, Kg, Kg, 1, 0, Kg, st);
      if (rc) return rc;
    }
  }
  // The epilogue needs a unit channel stride; any (n, p, q) strides whose rows stay 16-byte
  // aligned are written in place (dense channels-last, a channel slice, a parity sub-grid).
  const int64_t oes_ = dtype_size(d.out_dtype);
  const bool y_cl = d.y_strides[1] == 1 && aligned16(d.y) && (d.y_strides[0] * oes_) % 16 == 0 &&
                    (d.y_strides[2] * oes_) % 16 == 0 && (d.y_strides[3] * oes_) % 16 == 0 &&
                    d.y_strides[3] >= d.K;
  void* yout = d.y;
  int64_t ys[4] = {d.y_strides[0], d.y_strides[1], d.y_strides[2], d.y_strides[3]};
  if (!y_cl) {
    yout = ws.take((size_t)d.N * d.P * d.Q * d.K * dtype_size(d.out_dtype));
    ys[0] = d.P * d.Q * d.K; ys[1] = 1; ys[2] = d.Q * d.K; ys[3] = d.K;
  }
  const void* res = d.residual;
  int64_t rs[4] = {d.res_strides[0], d.res_strides[1], d.res_strides[2], d.res_strides[3]};
  if (res && !is_channels_last(rs, d.K, d.P, d.Q)) {
    void* dst = ws.take((size_t)d.N * d.P * d.Q * d.K * dtype_size(d.out_dtype));
    int64_t cl[4] = {d.P * d.Q * d.K, 1, d.Q * d.K, d.K};
    int64_t sizes[4] = {d.N, d.K, d.P, d.Q};
    if (run) {
      int rc = launch_copy_strided(dst, d.out_dtype, cl, d.residual, d.out_dtype, d.res_strides, sizes, 4, st);
      if (rc) return rc;
    }
    res = dst;
    for (int i = 0; i < 4; ++i) rs[i] = cl[i];
  }
  // Activation operand.
  const void* a = nullptr;
  const void* alo = nullptr;
  int64_t M = 0;
  if (implicit && cat) {
    a = d.x;
  } else if (implicit) {
    const bool x_cl = is_channels_last(d.x_strides, d.C, d.H, d.W) && aligned16(d.x);
    a = d.x;
    if (!x_cl) {
      void* dst = ws.take((size_t)d.N * d.H * d.W * d.C * es);
      a = dst;
      if (run) {
        int64_t cl[4] = {d.H * d.W * d.C, 1, d.W * d.C, d.C};
        int64_t sizes[4] = {d.N, d.C, d.H, d.W};
        int rc = launch_copy_strided(dst, d.dtype, cl, d.x, d.dtype, d.x_strides, sizes, 4, st);
        if (rc) return rc;
      }
    }
    if (tf32) {
      void* lo = ws.take((size_t)d.N * d.H * d.W * d.C * 4);
      alo = lo;
      if (run) {
        int rc = launch_pack2d(nullptr, (float*)lo, a, MT_F32, 1, d.N * d.H * d.W, d.C, d.C, 1, 0, d.C, st);
        if (rc) return rc;
      }
    }
  } else {
    M = d.N * d.P * d.Q;
    void* col = ws.take((size_t)M * Kg * es);
    void* lo = tf32 ? ws.take((size_t)M * Kg * 4) : nullptr;
    a = col;
    alo = lo;
    if (run) {
      int rc = launch_im2col(col, (float*)lo, d.x, d.dtype, d, Cp, Kg, st);
      if (rc) return rc;
    }
  }
  // split-K partial sums (decided from the per-image shape; see conv_k_splits)
  float* part = nullptr;
  int splits = 1;
  if (allow_split && implicit) {
    splits = conv_k_splits(d, d.R * d.S * (d.C / (128 / es)));
    if (splits > 1) part = (float*)ws.take((size_t)splits * d.N * d.P * d.Q * d.K * sizeof(float));
  }
  if (!run) return MT_OK;

  L->kind = d.dtype;
  L->conv = implicit;
  L->bn = pick_bn(d.K, d.dtype, false, implicit);
  TileParams& tp = L->tp;
  tp.bk = 128 / es;
  tp.batch = 1;
  tp.a_batched = tp.b_batched = 0;
  int rc;
  if (implicit) {
    auto pow2_ge = [](int64_t v) {
      int64_t p = 1;
      while (p < v) p <<= 1;
      return p;
    };
    const int64_t tw = std::min<int64_t>(128, pow2_ge(d.Q));
    const int64_t th = std::min<int64_t>(128 / tw, pow2_ge(d.P));
    const int64_t tn = 128 / (tw * th);
    tp.tw = (int)tw; tp.th = (int)th; tp.tn = (int)tn;
    tp.tiles_q = (int)((d.Q + tw - 1) / tw);
    tp.tiles_p = (int)((d.P + th - 1) / th);
    const int64_t tiles_n = (d.N + tn - 1) / tn;
    tp.num_m_tiles = (int)(tiles_n * tp.tiles_q * tp.tiles_p);
    tp.c_chunks = (int)(d.C / tp.bk);
    tp.R = (int)d.R; tp.S = (int)d.S;
    tp.pad_h = d.pad_h; tp.pad_w = d.pad_w; tp.dil_h = d.dil_h; tp.dil_w = d.dil_w;
    tp.stride_h = d.stride_h; tp.stride_w = d.stride_w;
    tp.k_iters = (int)(d.R * d.S * tp.c_chunks);
    uint64_t dims[4] = {(uint64_t)d.C, (uint64_t)d.W, (uint64_t)d.H, (uint64_t)d.N};
    uint64_t strides[3] = {(uint64_t)(d.C * es), (uint64_t)(d.W * d.C * es), (uint64_t)(d.H * d.W * d.C * es)};
    // tw, th <= 128, so a stride-2 box (2 tw x 2 th input pixels) stays within TMA's 256 limit
    uint32_t box[4] = {(uint32_t)tp.bk, (uint32_t)(tw * d.stride_w), (uint32_t)(th * d.stride_h), (uint32_t)tn};
    const uint32_t estr[4] = {1, (uint32_t)d.stride_w, (uint32_t)d.stride_h, 1};
    tp.c_split = 0;
    if (cat) {
      // two 4-D maps over the two channels-last sources, chunk c of the concatenation from the
      // first when c < c1 / bk
      const int64_t c2 = d.C - cat->c1;
      uint64_t dims1[4] = {(uint64_t)cat->c1, (uint64_t)d.W, (uint64_t)d.H, (uint64_t)d.N};
      uint64_t str1[3] = {(uint64_t)(d.x_strides[3] * es), (uint64_t)(d.x_strides[2] * es),
                          (uint64_t)(d.x_strides[0] * es)};
      uint64_t dims2[4] = {(uint64_t)c2, (uint64_t)d.W, (uint64_t)d.H, (uint64_t)d.N};
      uint64_t str2[3] = {(uint64_t)(cat->x2_strides[3] * es), (uint64_t)(cat->x2_strides[2] * es),
                          (uint64_t)(cat->x2_strides[0] * es)};
      rc = make_tensor_map(&L->a, d.dtype, 4, d.x, dims1, str1, box, 128, estr);
      if (!rc) rc = make_tensor_map(&L->alo, d.dtype, 4, cat->x2, dims2, str2, box, 128, estr);
      tp.c_split = (int)(cat->c1 / tp.bk);
    } else {
      rc = make_tensor_map(&L->a, d.dtype, 4, a, dims, strides, box, 128, estr);
    }
    if (!rc && tf32) rc = make_tensor_map(&L->alo, MT_F32, 4, alo, dims, strides, box, 128, estr);
  } else {
    tp.num_m_tiles = (int)((M + kBM - 1) / kBM);
    tp.k_iters = (int)((Kg + tp.bk - 1) / tp.bk);
    rc = map_kmajor(&L->a, d.dtype, a, Kg, M, 1, Kg, 0, kBM);
    if (!rc && tf32) rc = map_kmajor(&L->alo, MT_F32, alo, Kg, M, 1, Kg, 0, kBM);
  }
  tp.k_splits = 1;
  tp.k_per = tp.k_iters;
  if (splits > 1) {
    tp.k_splits = splits;
    tp.k_per = (tp.k_iters + splits - 1) / splits;
  } else if (!tf32) {
    L->bn = narrow_bn(L->bn, d.K, tp.num_m_tiles, false);
  }
  // 320-wide tiles (one TMEM accumulator, two N = 160 MMAs per K step) for 3x3 convolutions with
  // output channels in multiples of 320: 0.77-0.90 of the bf16 peak against 0.57-0.72 for the 160 /
  // 256-wide tiles at the UNet's 64x64 and 32x32 levels, and faster at 16x16; not at 8x8, where the
  // split-K tiles are short and the accumulator's drain is not hidden, nor with fewer tiles than
  // SMs (measured; same box).  MT_GEMM_BN forces a width; MT_GEMM_NO_BN320 keeps the old choice.
  static const bool bn320_off = getenv("MT_GEMM_NO_BN320") != nullptr || getenv("MT_GEMM_BN") != nullptr;
  if (!bn320_off && !tf32 && implicit && d.K % 320 == 0 && d.R * d.S > 1 && d.P * d.Q >= 256 &&
      (int64_t)tp.num_m_tiles * (d.K / 320) >= num_sms())
    L->bn = 320;
  tp.num_n_tiles = (int)((d.K + L->bn - 1) / L->bn);
  // (320-wide tiles load B in two 160-row boxes)
  if (!rc) rc = map_kmajor(&L->b, d.dtype, wp, Kg, d.K, 1, Kg, 0, L->bn > 256 ? L->bn / 2 : L->bn);
  L->b_ptr = wp; L->b_K = Kg; L->b_rows = d.K; L->b_batch = 1; L->b_pitch = Kg; L->b_bstride = 0;
  if (!rc && tf32) rc = map_kmajor(&L->blo, MT_F32, wlo, Kg, d.K, 1, Kg, 0, L->bn);
  if (rc) return rc;
  if (!tf32) {
    if (!(cat && implicit)) L->alo = L->a;
    L->blo = L->b;
  }

  EpiParams& ep = L->ep;
  ep.mode = implicit ? 2 : 1;
  ep.M = implicit ? d.N : M;
  ep.N = d.K;
  ep.P = d.P; ep.Q = d.Q;
  ep.D = yout; ep.out_dtype = d.out_dtype; ep.d_s0 = ys[0]; ep.d_s1 = ys[2]; ep.d_s2 = ys[3];
  ep.C = nullptr; ep.beta = 0.f;
  ep.res = res; ep.r_s0 = rs[0]; ep.r_s1 = rs[2]; ep.r_s2 = rs[3];
  ep.bias = d.bias; ep.bias_dtype = d.bias_dtype; ep.bias_bstride = d.bias_batch_stride;
  ep.alpha = 1.f; ep.act = d.epilogue;
  const int oes = dtype_size(d.out_dtype);
  ep.vec_ok = aligned16(yout) && (d.K * oes) % 16 == 0 && (!res || aligned16(res));
  ep.bias_vec = bias_vec_ok(d.bias, d.bias_dtype, d.bias_batch_stride);
  ep.part = part;
  ep.part_stride = d.N * d.P * d.Q * d.K;
  return MT_OK;
}

// The reduction that completes a split-K convolution (no-op otherwise).
static int finish_split(const GemmLaunch& L, cudaStream_t st) {
  if (L.tp.k_splits <= 1) return MT_OK;
  const EpiParams& ep = L.ep;
  const int64_t rows = ep.M * ep.P * ep.Q;
  const int64_t total = rows * (ep.N / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  splitk_reduce_kernel<<<blocks, 256, 0, st>>>(ep.part, L.tp.k_splits, ep.part_stride, rows, ep.N, ep);
  return check_launch("splitk_reduce");
}

static int validate_conv(const mt_conv2d_desc& d) {
  if (d.N < 0 || d.C <= 0 || d.H <= 0 || d.W <= 0 || d.K <= 0 || d.R <= 0 || d.S <= 0)
    return fail(MT_ERR_INVALID, "conv2d: bad sizes");
  if (d.stride_h <= 0 || d.stride_w <= 0 || d.dil_h <= 0 || d.dil_w <= 0 || d.pad_h < 0 || d.pad_w < 0)
    return fail(MT_ERR_INVALID, "conv2d: bad stride / dilation / padding");
  if (d.groups < 1 || d.C % d.groups || d.K % d.groups)
    return fail(MT_ERR_INVALID, "conv2d: channels %lld / %lld not divisible by groups %d", (long long)d.C,
                (long long)d.K, d.groups);
  if (d.groups > 1 && d.w_packed)
    return fail(MT_ERR_UNSUPPORTED, "conv2d: grouped convolutions take the unpacked [K, C/groups, R, S] weight");
  if (d.dtype != MT_F32 && d.dtype != MT_BF16 && d.dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "conv2d: dtype %d", d.dtype);
  if (d.out_dtype != MT_F32 && d.out_dtype != MT_BF16 && d.out_dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "conv2d: output dtype %d", d.out_dtype);
  const int64_t P = (d.H + 2 * d.pad_h - d.dil_h * (d.R - 1) - 1) / d.stride_h + 1;
  const int64_t Q = (d.W + 2 * d.pad_w - d.dil_w * (d.S - 1) - 1) / d.stride_w + 1;
  if (P != d.P || Q != d.Q) return fail(MT_ERR_INVALID, "conv2d: output size mismatch");
  if (d.epilogue == MT_EPI_GEGLU) return fail(MT_ERR_UNSUPPORTED, "conv2d: GEGLU epilogue");
  if (d.N > 0 && (!d.x || !d.w || !d.y)) return fail(MT_ERR_INVALID, "conv2d: null operand");
  return MT_OK;
}

// Group g of a grouped convolution (groups > 1, `conv2d` tensor.cpp:26498-26543): input
// channels [g*C/G, (g+1)*C/G), weight rows and output channels [g*K/G, (g+1)*K/G), as a plain
// convolution on views of the same buffers (the weight in its unpacked [K, C/G, R, S] layout).
static mt_conv2d_desc conv_group_desc(const mt_conv2d_desc& d, int g) {
  mt_conv2d_desc e = d;
  const int64_t cg = d.C / d.groups, kg = d.K / d.groups;
  const int es = dtype_size(d.dtype), oes = dtype_size(d.out_dtype);
  e.groups = 1;
  e.C = cg;
  e.K = kg;
  e.x = static_cast<const char*>(d.x) + (int64_t)g * cg * d.x_strides[1] * es;
  e.w = static_cast<const char*>(d.w) + (int64_t)g * kg * cg * d.R * d.S * es;
  e.w_lo = nullptr;
  if (d.bias) e.bias = static_cast<const char*>(d.bias) + (int64_t)g * kg * dtype_size(d.bias_dtype);
  if (d.residual) e.residual = static_cast<const char*>(d.residual) + (int64_t)g * kg * d.res_strides[1] * oes;
  e.y = static_cast<char*>(d.y) + (int64_t)g * kg * d.y_strides[1] * oes;
  return e;
}

size_t conv_workspace(const mt_conv2d_desc& d) {
  if (validate_conv(d) != MT_OK) return 0;
  if (d.groups > 1) return conv_workspace(conv_group_desc(d, 0));  // the same for every group
  WsCursor ws{nullptr, 0};
  plan_conv(d, ws, false, nullptr, nullptr, nullptr, true);
  return ws.off;
}

int run_conv2d(const mt_conv2d_desc& d, void* wsp, size_t ws_bytes, cudaStream_t st) {
  int rc = validate_conv(d);
  if (rc) return rc;
  if (d.N == 0 || d.P <= 0 || d.Q <= 0) return MT_OK;
  if (d.groups > 1) {
    // one plain convolution per group, stream-ordered on the same workspace
    for (int g = 0; g < d.groups; ++g) {
      rc = run_conv2d(conv_group_desc(d, g), wsp, ws_bytes, st);
      if (rc) return rc;
    }
    return MT_OK;
  }
  const size_t need = conv_workspace(d);
  if (need > 0 && (!wsp || ws_bytes < need))
    return fail(MT_ERR_WORKSPACE, "conv2d: workspace of %zu bytes required", need);
  WsCursor ws{(char*)wsp, 0};
  GemmLaunch L{};
  rc = plan_conv(d, ws, true, st, &L, nullptr, true);
  if (rc) return rc;
  rc = dispatch(L, st);
  if (!rc) rc = finish_split(L, st);
  if (rc) return rc;
  if (L.ep.D != d.y) {
    int64_t cl[4] = {d.P * d.Q * d.K, 1, d.Q * d.K, d.K};
    int64_t sizes[4] = {d.N, d.K, d.P, d.Q};
    rc = launch_copy_strided(d.y, d.out_dtype, d.y_strides, L.ep.D, d.out_dtype, cl, sizes, 4, st);
  }
  return rc;
}

size_t conv_cat_workspace(const mt_conv2d_desc& d, const void* x2, const int64_t* x2_strides, int64_t c1) {
  if (validate_conv(d) != MT_OK || !x2_strides) return 0;
  ConvCat cat{};
  cat.x2 = x2;
  for (int i = 0; i < 4; ++i) cat.x2_strides[i] = x2_strides[i];
  cat.c1 = c1;
  WsCursor ws{nullptr, 0};
  plan_conv(d, ws, false, nullptr, nullptr, &cat, true);
  return ws.off;
}

// Convolution of the channel concatenation [x1 | x2] (the up-block skip connection) without
// forming it: d.x / d.x_strides describe x1 with c1 channels, d.C is the total channel count.
int run_conv2d_cat(const mt_conv2d_desc& d, const void* x2, const int64_t* x2_strides, int64_t c1, void* wsp,
                   size_t ws_bytes, cudaStream_t st) {
  int rc = validate_conv(d);
  if (rc) return rc;
  if (!x2 || !x2_strides) return fail(MT_ERR_INVALID, "conv2d_cat: null second source");
  if (d.dtype != MT_BF16 && d.dtype != MT_F16) return fail(MT_ERR_UNSUPPORTED, "conv2d_cat: 16-bit inputs only");
  const int64_t bk = 128 / dtype_size(d.dtype);
  const int64_t c2 = d.C - c1;
  if (c1 <= 0 || c2 <= 0 || c1 % bk || c2 % bk)
    return fail(MT_ERR_UNSUPPORTED, "conv2d_cat: source channel counts must be multiples of %lld", (long long)bk);
  if (!conv_implicit_ok(d)) return fail(MT_ERR_UNSUPPORTED, "conv2d_cat: shape needs the im2col path");
  if (!is_channels_last(d.x_strides, c1, d.H, d.W) || !is_channels_last(x2_strides, c2, d.H, d.W) ||
      !aligned16(d.x) || !aligned16(x2))
    return fail(MT_ERR_UNSUPPORTED, "conv2d_cat: sources must be dense channels-last and 16-byte aligned");
  if (d.N == 0 || d.P <= 0 || d.Q <= 0) return MT_OK;
  const size_t need = conv_cat_workspace(d, x2, x2_strides, c1);
  if (need > 0 && (!wsp || ws_bytes < need))
    return fail(MT_ERR_WORKSPACE, "conv2d_cat: workspace of %zu bytes required", need);
  ConvCat cat{};
  cat.x2 = x2;
  for (int i = 0; i < 4; ++i) cat.x2_strides[i] = x2_strides[i];
  cat.c1 = c1;
  WsCursor ws{(char*)wsp, 0};
  GemmLaunch L{};
  rc = plan_conv(d, ws, true, st, &L, &cat, true);
  if (rc) return rc;
  rc = dispatch(L, st);
  if (!rc) rc = finish_split(L, st);
  if (rc) return rc;
  if (L.ep.D != d.y) {
    int64_t cl[4] = {d.P * d.Q * d.K, 1, d.Q * d.K, d.K};
    int64_t sizes[4] = {d.N, d.K, d.P, d.Q};
    rc = launch_copy_strided(d.y, d.out_dtype, d.y_strides, L.ep.D, d.out_dtype, cl, sizes, 4, st);
  }
  return rc;
}

// ---------------------------------------------------------------------------------------------
// 3x3 convolution (pad 1, stride 1) of a nearest-2x upsampled input without materialising it:
// four 2x2 implicit-GEMM convolutions of the source, one per output parity (a, b), with taps
// pre-summed per parity (launch_conv_up2x_pack_weight).  Parity (a, b) output (i, j) lands at
// (2i + a, 2j + b) and reads source rows i - 1 + a .. i + a (columns likewise): top / left padding
// 1 - a / 1 - b with P = H, Q = W.

int64_t conv_up2x_packed_elems(int64_t K, int64_t C, int dtype) {
  return 16 * K * conv_packed_channels(C, 2, 2, dtype);
}

static int validate_conv_up2x(const mt_conv2d_desc& d) {
  if (d.N < 0 || d.C <= 0 || d.H <= 0 || d.W <= 0 || d.K <= 0) return fail(MT_ERR_INVALID, "conv2d_up2x: bad sizes");
  if (d.R != 3 || d.S != 3 || d.stride_h != 1 || d.stride_w != 1 || d.pad_h != 1 || d.pad_w != 1 || d.dil_h != 1 ||
      d.dil_w != 1 || d.groups != 1)
    return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: only 3x3, stride 1, padding 1, dilation 1, groups 1");
  if (d.P != 2 * d.H || d.Q != 2 * d.W) return fail(MT_ERR_INVALID, "conv2d_up2x: output must be [2H, 2W]");
  if (d.dtype != MT_F32 && d.dtype != MT_BF16 && d.dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: dtype %d", d.dtype);
  if (d.out_dtype != MT_F32 && d.out_dtype != MT_BF16 && d.out_dtype != MT_F16)
    return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: output dtype %d", d.out_dtype);
  if (d.epilogue == MT_EPI_GEGLU) return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: GEGLU epilogue");
  mt_conv2d_desc e = d;
  e.R = e.S = 2;
  if (!conv_implicit_ok(e)) return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: channels must fill whole 128-byte chunks");
  const int oes = dtype_size(d.out_dtype);
  if (d.y_strides[1] != 1 || (2 * d.y_strides[2] * oes) % 16 || (2 * d.y_strides[3] * oes) % 16 ||
      (d.y_strides[0] * oes) % 16 || (reinterpret_cast<uintptr_t>(d.y) % 16))
    return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: output must be channels-last with 16-byte aligned rows");
  if (d.residual && (d.res_strides[1] != 1 || (2 * d.res_strides[2] * oes) % 16 || (2 * d.res_strides[3] * oes) % 16 ||
                     (d.res_strides[0] * oes) % 16 || (reinterpret_cast<uintptr_t>(d.residual) % 16)))
    return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: residual must be channels-last with 16-byte aligned rows");
  if (d.N > 0 && (!d.x || !d.w || !d.y)) return fail(MT_ERR_INVALID, "conv2d_up2x: null operand");
  return MT_OK;
}

// The per-parity descriptor: 2x2 taps over the source, packed weights of that parity.
static mt_conv2d_desc up2x_parity_desc(const mt_conv2d_desc& d, int par, const void* wp, const float* wlo) {
  const int a = par >> 1, b = par & 1;
  const int oes = dtype_size(d.out_dtype);
  const int64_t Cp = conv_packed_channels(d.C, 2, 2, d.dtype);
  const int64_t per = d.K * 4 * Cp;
  mt_conv2d_desc e = d;
  e.R = e.S = 2;
  e.P = d.H;
  e.Q = d.W;
  e.pad_h = 1 - a;
  e.pad_w = 1 - b;
  e.w = static_cast<const char*>(wp) + (size_t)par * per * dtype_size(d.dtype);
  e.w_packed = 1;
  e.w_lo = wlo ? wlo + (size_t)par * per : nullptr;
  e.y = static_cast<char*>(d.y) + (a * d.y_strides[2] + b * d.y_strides[3]) * oes;
  e.y_strides[2] = 2 * d.y_strides[2];
  e.y_strides[3] = 2 * d.y_strides[3];
  if (d.residual) {
    e.residual = static_cast<const char*>(d.residual) + (a * d.res_strides[2] + b * d.res_strides[3]) * oes;
    e.res_strides[2] = 2 * d.res_strides[2];
    e.res_strides[3] = 2 * d.res_strides[3];
  }
  return e;
}

size_t conv_up2x_workspace(const mt_conv2d_desc& d) {
  if (validate_conv_up2x(d) != MT_OK) return 0;
  const bool tf32 = d.dtype == MT_F32;
  const size_t elems = (size_t)conv_up2x_packed_elems(d.K, d.C, d.dtype);
  size_t pack = 0;
  if (!d.w_packed) pack += align_up(elems * dtype_size(d.dtype), 256);
  if (tf32 && (!d.w_packed || !d.w_lo)) pack += align_up(elems * 4, 256);
  // the four parity plans reuse one region after the packed weights (stream-ordered launches);
  // with packed low parts present a plan needs no per-call weight split
  mt_conv2d_desc e = up2x_parity_desc(d, 0, d.w, tf32 ? reinterpret_cast<const float*>(d.w) : nullptr);
  WsCursor ws{nullptr, 0};
  plan_conv(e, ws, false, nullptr, nullptr, nullptr, true);
  return pack + 256 + ws.off;
}

int run_conv2d_up2x(const mt_conv2d_desc& d, void* wsp, size_t ws_bytes, cudaStream_t st) {
  int rc = validate_conv_up2x(d);
  if (rc) return rc;
  if (d.N == 0) return MT_OK;
  const size_t need = conv_up2x_workspace(d);
  if (need > 0 && (!wsp || ws_bytes < need))
    return fail(MT_ERR_WORKSPACE, "conv2d_up2x: workspace of %zu bytes required", need);
  const bool tf32 = d.dtype == MT_F32;
  const int64_t Cp = conv_packed_channels(d.C, 2, 2, d.dtype);
  const int64_t elems = conv_up2x_packed_elems(d.K, d.C, d.dtype);
  WsCursor ws{(char*)wsp, 0};
  const void* wp = d.w;
  const float* wlo = static_cast<const float*>(d.w_lo);
  if (!d.w_packed) {
    void* dst = ws.take((size_t)elems * dtype_size(d.dtype));
    float* lo = tf32 ? (float*)ws.take((size_t)elems * 4) : nullptr;
    rc = launch_conv_up2x_pack_weight(dst, lo, d.w, d.dtype, d.K, d.C, Cp, st);
    if (rc) return rc;
    wp = dst;
    wlo = lo;
  } else if (tf32 && !wlo) {
    float* lo = (float*)ws.take((size_t)elems * 4);
    rc = launch_pack2d(nullptr, lo, d.w, MT_F32, 1, 4 * d.K, 4 * Cp, 4 * Cp, 1, 0, 4 * Cp, st);
    if (rc) return rc;
    wlo = lo;
  }
  const size_t base = align_up(ws.off, 256);
  for (int par = 0; par < 4; ++par) {
    const mt_conv2d_desc e = up2x_parity_desc(d, par, wp, wlo);
    WsCursor wsp2{(char*)wsp, base};
    GemmLaunch L{};
    rc = plan_conv(e, wsp2, true, st, &L, nullptr, true);
    if (rc) return rc;
    if (L.ep.D != e.y) return fail(MT_ERR_UNSUPPORTED, "conv2d_up2x: output layout");
    rc = dispatch(L, st);
    if (!rc) rc = finish_split(L, st);
    if (rc) return rc;
  }
  return MT_OK;
}

// ---------------------------------------------------------------------------------------------
// Failure-detection self test: one thread waits, through the same bounded mbar_wait every kernel
// of this library uses, on an mbarrier that nothing ever arrives on.  The wait gives up after
// `budget_cycles`, records MT_ERR_TIMEOUT (site kSiteSelftest) in this unit's device status word
// and the kernel returns; the context stays usable.
constexpr int kSiteSelftest = 99;

__global__ void wait_timeout_selftest_kernel(long long budget_cycles) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, kSiteSelftest, &abort_flag, budget_cycles);
}

int run_wait_timeout_selftest(long long budget_cycles, cudaStream_t st) {
  if (budget_cycles < 0 || budget_cycles > kWaitBudgetCycles)
    return fail(MT_ERR_INVALID, "wait self test: budget %lld cycles outside [0, %lld]", budget_cycles,
                kWaitBudgetCycles);
  wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(budget_cycles);
  return check_launch("wait_timeout_selftest_kernel");
}

}  // namespace mt
