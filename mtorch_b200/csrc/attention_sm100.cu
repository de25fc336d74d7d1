// Flash attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16 / f16, sm_100a.
//
// One CTA = NQ tiles of 128 query rows (NQ = 2 for head dims <= 128) of one (batch, head); KV
// tiles of 128 keys stream through a TMA ring and are shared by the NQ query tiles.
// Roles (64 + 128*NQ threads):
//   warp 0      TMA producer: the Q tiles once, then (K_j, V_j) per stage.  Operands are read
//               straight from the caller's strided [B, H, S, D] views (e.g. head slices of a
//               fused QKV projection) with 5-D tensor maps {8, S, D/8, H, B}: a box lands in
//               shared memory as [D/8 chunk][row][8 elems] — the UMMA no-swizzle core-matrix
//               layout — and the head-dim padding to a multiple of 16 is TMA's zero fill.
//   warp 1      MMA issuer: S_x = Q_x K_j^T into TMEM (fp32) for each query tile x, then
//               O_x = P_x V_j (P from shared memory, V as an MN-major operand) into TMEM.
//   warps 2..   one softmax warpgroup per query tile (one query row per thread = its TMEM lane):
//               online softmax in base 2 on S (pass 1: row max of the raw scores; pass 2:
//               p = 2^(s*scale*log2e - m) with packed f32x2 FMAs, row sums, bf16/f16 P to shared
//               memory), then O += O_j with the running rescale in registers; finally O / l.
// While one warpgroup exponentiates its scores the tensor core computes the other tile's
// scores, so the two query tiles interleave.  Masks / causal requests run the SIMT kernel (the
// UNet does not use them).  All waits are bounded (timeout -> device error word, return).
#include "runtime.h"

namespace mt {

MT_STATUS_READER(read_status_attention)

constexpr int kFaBM = 128;  // query rows per tile
constexpr int kFaBN = 128;  // keys per KV tile
constexpr int kFaMaxStages = 4;

struct FaParams {
  int Sq, Sk, H, Hkv, B;
  float scale_log2;  // softmax scale * log2(e)
  void* o;
  int64_t os[4];
  int Dv;
  int out_dtype;
  int stages;    // KV stages (K and V tiles together); the lazy kernel: K stages
  int stages_v;  // lazy kernel: V stages
  int causal;    // fa_sm100_kernel: key j of query i is masked when j > i (top-left aligned)
  // fa_sm100_kernel: attention mask, 0 none / 1 bool (uint8, nonzero keeps) / 2 additive in
  // mask_dtype, indexed with element strides ms over (b, h, query, key)
  const void* mask;
  int mask_kind, mask_dtype;
  int64_t ms[4];
  int pairs;  // fa_short_sm100_kernel: pairs of 128-query tiles per CTA
};

// log2-domain additive term of the mask for (query row, key) at element offset `off`: 0 / -inf
// for a bool mask, value * log2(e) for an additive one.
__device__ __forceinline__ float fa_mask_add(const FaParams& p, int64_t off) {
  if (p.mask_kind == 1) return static_cast<const uint8_t*>(p.mask)[off] ? 0.f : -INFINITY;
  return load_as_f32(p.mask, off, p.mask_dtype) * 1.4426950408889634f;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// three-input maximum (sm_100 max.f32 with three sources)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// maximum of 64 scores as a tree of independent three-input maxima (no serial chain)
__device__ __forceinline__ float max64(const uint32_t (&r)[64]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmax3(__uint_as_float(r[i]), __uint_as_float(r[8 + i]), __uint_as_float(r[16 + i]));
#pragma unroll
  for (int k = 24; k < 56; k += 16)  // columns 24..55
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m[i] = fmax3(m[i], __uint_as_float(r[k + i]), __uint_as_float(r[k + 8 + i]));
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], __uint_as_float(r[56 + i]));  // columns 56..63
  return fmaxf(fmax3(m[0], m[1], m[2]), fmax3(fmax3(m[3], m[4], m[5]), m[6], m[7]));
}

__device__ __forceinline__ uint64_t f2_bits(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
// (a0, a1) * (b0, b1) + (c0, c1) in one instruction
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Shared-memory descriptor, no swizzle: lbo / sbo in bytes.
__device__ __forceinline__ uint64_t sdesc_none(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;  // layout type 0 = SWIZZLE_NONE
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16_raw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

template <int DP, int DVP, int NQ, bool F16, bool MASK = false>
__global__ void __launch_bounds__(64 + 128 * NQ, 1)
    fa_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  constexpr int Q_BYTES = kFaBM * DP * 2;
  constexpr int K_BYTES = kFaBN * DP * 2;
  constexpr int V_BYTES = kFaBN * DVP * 2;
  constexpr int P_BYTES = kFaBM * kFaBN * 2;
  constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  constexpr uint32_t kLbo = kFaBM * 16;  // next 8-element K chunk (128 rows * 16 B); BM == BN
  constexpr uint32_t kSbo = 128;        // next 8 rows
  constexpr int FMT = F16 ? 0 : 1;
  constexpr uint32_t idesc_s = make_idesc(FMT, kFaBM, kFaBN);
  constexpr uint32_t idesc_o = make_idesc(FMT, kFaBM, DVP) | (1u << 16);  // B (V) MN-major
  static_assert(NQ == 1 || 2 * 128 + 2 * DVP <= 512, "TMEM budget");

  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // [NQ][Q]
  uint8_t* sP = sQ + NQ * Q_BYTES;      // [NQ][P]
  uint8_t* sKV = sP + NQ * P_BYTES;     // [stages][K, V]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + p.stages * STAGE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kFaMaxStages;
  uint64_t* s_full = kv_empty + kFaMaxStages;  // [2] score slots
  uint64_t* s_empty = s_full + 2;              // [2]
  uint64_t* p_full = s_empty + 2;              // [NQ]
  uint64_t* o_full = p_full + 2;               // [NQ]
  uint64_t* o_empty = o_full + 2;              // [NQ]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages = p.stages;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int qbase = blockIdx.x * (kFaBM * NQ);
  const int n_tiles = (p.Sk + kFaBN - 1) / kFaBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // score slot i at columns [128 i, 128 i + 128); O of query tile x after the score slots
  const uint32_t t_o0 = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, NQ * Q_BYTES);
      for (int x = 0; x < NQ; ++x) tma_load_5d(sQ + x * Q_BYTES, &tmQ, q_full, 0, qbase + x * kFaBM, 0, h, b);
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; j < n_tiles; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1, 11, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[stage], STAGE_BYTES);
        uint8_t* sk = sKV + stage * STAGE_BYTES;
        tma_load_5d(sk, &tmK, &kv_full[stage], 0, j * kFaBN, 0, hk, b);
        tma_load_5d(sk + K_BYTES, &tmV, &kv_full[stage], 0, j * kFaBN, 0, hk, b);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, 12, abort_flag);
      int stage = 0, prev_stage = 0;
      uint32_t phase = 0;
      // O_x = P_x V_{jj} for every query tile; releases the KV stage of tile jj.
      auto issue_pv = [&](int jj) -> bool {
        const uint32_t v_addr = smem_u32(sKV + prev_stage * STAGE_BYTES + K_BYTES);
        for (int x = 0; x < NQ; ++x) {
          if (!mbar_wait(&p_full[x], jj & 1, 15, abort_flag)) return false;
          if (!mbar_wait(&o_empty[x], (jj & 1) ^ 1, 16, abort_flag)) return false;
          tc_fence_after();
          const uint32_t pa = p_addr + x * P_BYTES;
          // V (MN-major): next 8 keys = 128 B (LBO), next 8 value dims = BN * 16 B (SBO)
#pragma unroll
          for (int kk = 0; kk < kFaBN / 16; ++kk)
            umma_f16(t_o0 + x * DVP, sdesc_none(pa + kk * 2 * kLbo, kLbo, kSbo),
                     sdesc_none(v_addr + kk * 256, 128, kFaBN * 16), idesc_o, kk > 0 ? 1u : 0u);
          umma_commit(&o_full[x]);
        }
        umma_commit(&kv_empty[prev_stage]);
        return true;
      };
      for (int j = 0; ok && j <= n_tiles; ++j) {
        // With a single KV stage the next tile's K/V can only arrive after PV of this one.
        if (j > 0 && stages == 1 && !issue_pv(j - 1)) break;
        if (j < n_tiles) {
          if (!mbar_wait(&kv_full[stage], phase, 13, abort_flag)) break;
          const uint32_t k_addr = smem_u32(sKV + stage * STAGE_BYTES);
          bool sok = true;
          for (int x = 0; x < NQ; ++x) {
            // NQ == 2: slot x is reused every KV tile; NQ == 1: the two slots alternate
            const int slot = NQ == 2 ? x : (j & 1);
            const uint32_t par = NQ == 2 ? ((j & 1) ^ 1) : (((j >> 1) & 1) ^ 1);
            if (!mbar_wait(&s_empty[slot], par, 14, abort_flag)) {
              sok = false;
              break;
            }
            tc_fence_after();
            const uint32_t qa = q_addr + x * Q_BYTES;
#pragma unroll
            for (int kk = 0; kk < DP / 16; ++kk)
              umma_f16(tmem + slot * 128, sdesc_none(qa + kk * 2 * kLbo, kLbo, kSbo),
                       sdesc_none(k_addr + kk * 2 * kLbo, kLbo, kSbo), idesc_s, kk > 0 ? 1u : 0u);
            umma_commit(&s_full[slot]);
          }
          if (!sok) break;
        }
        if (j > 0 && stages > 1 && !issue_pv(j - 1)) break;
        if (j < n_tiles) {
          prev_stage = stage;
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else {
    // ---------------- softmax / output warpgroups ----------------
    const int x = (warp - 2) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* sPx = sP + x * P_BYTES;
    const uint32_t t_o = t_o0 + x * DVP + lane_off;
    float o_acc[DVP];
#pragma unroll
    for (int i = 0; i < DVP; ++i) o_acc[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    const float sl = p.scale_log2;
    const uint64_t sl2 = f2_bits(sl, sl);
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int slot = NQ == 2 ? x : (j & 1);
      const uint32_t par = NQ == 2 ? (j & 1) : ((j >> 1) & 1);
      if (!mbar_wait(&s_full[slot], par, 17, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t ts = tmem + slot * 128 + lane_off;
      // keys of this tile the row may see; causal rows see keys 0..qi (tile 0 always holds key 0,
      // so the running max is finite after the first tile)
      int kvalid = min(kFaBN, p.Sk - j * kFaBN);
      if (p.causal) kvalid = max(0, min(kvalid, qbase + x * kFaBM + row - j * kFaBN + 1));
      const bool full = kvalid == kFaBN;
      // masked rows: element offset of (b, h, query, first key of the tile); rows past Sq read
      // no mask
      const int qrow = qbase + x * kFaBM + row;
      const bool masked = MASK && qrow < p.Sq;
      const int64_t moff = masked ? (int64_t)b * p.ms[0] + (int64_t)h * p.ms[1] + (int64_t)qrow * p.ms[2] +
                                        (int64_t)j * kFaBN * p.ms[3]
                                  : 0;
      // TMEM reads are issued 64 columns at a time before one tcgen05.wait::ld, so the load
      // latency is paid twice per pass rather than once per 16 columns.
      // pass 1: row max of the raw scores (the scale is positive); masked rows: of the scaled
      // scores plus the mask in the log2 domain
      float mx = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < kFaBN; c0 += 64) {
        uint32_t r[64];
        tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (masked) {
#pragma unroll 4
          for (int i = 0; i < 64; ++i)
            if (c0 + i < kvalid)
              mx = fmaxf(mx, __uint_as_float(r[i]) * sl + fa_mask_add(p, moff + (int64_t)(c0 + i) * p.ms[3]));
        } else if (full) {
          mx = fmaxf(mx, max64(r));
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (c0 + i < kvalid) mx = fmaxf(mx, __uint_as_float(r[i]));
        }
      }
      // a masked row whose keys so far are all masked keeps m = -inf; exponents then use 0
      const float m_new = masked ? fmaxf(m_run, mx) : fmaxf(m_run, mx * sl);
      const float m_use = (masked && m_new == -INFINITY) ? 0.f : m_new;
      const float corr = ex2(m_run - m_use);  // 0 on the first tile (m_run = -inf)
      const uint64_t negm2 = f2_bits(-m_use, -m_use);
      // pass 2: p = 2^(s * sl - m), packed row sums, P (bf16/f16) to shared memory
      uint64_t sum2 = f2_bits(0.f, 0.f);
#pragma unroll 1
      for (int c0 = 0; c0 < kFaBN; c0 += 64) {
        uint32_t r[64];
        tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 16 keys -> two 16-byte P chunks
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int k = q * 16 + i;
            const uint64_t arg = ffma2(f2_bits(__uint_as_float(r[k]), __uint_as_float(r[k + 1])), sl2, negm2);
            float a0, a1;
            f2_unpack(arg, a0, a1);
            if (masked) {
              if (c0 + k < kvalid) a0 += fa_mask_add(p, moff + (int64_t)(c0 + k) * p.ms[3]);
              if (c0 + k + 1 < kvalid) a1 += fa_mask_add(p, moff + (int64_t)(c0 + k + 1) * p.ms[3]);
            }
            float e0 = ex2(a0), e1 = ex2(a1);
            if (!full) {
              if (c0 + k >= kvalid) e0 = 0.f;
              if (c0 + k + 1 >= kvalid) e1 = 0.f;
            }
            sum2 = fadd2(sum2, f2_bits(e0, e1));
            pk[i / 2] = F16 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
          }
          // keys c..c+7 -> chunk c/8, keys c+8..c+15 -> chunk c/8+1; this row at +row*16
          const int c = c0 + q * 16;
          uint4* d0 = reinterpret_cast<uint4*>(sPx + (c / 8) * (kFaBM * 16) + row * 16);
          uint4* d1 = reinterpret_cast<uint4*>(sPx + (c / 8 + 1) * (kFaBM * 16) + row * 16);
          *d0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *d1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[slot]);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[x]);
      float s0, s1;
      f2_unpack(sum2, s0, s1);
      l_run = l_run * corr + (s0 + s1);
      m_run = m_new;
      // accumulate O_j (scaled by the same running max) once the PV MMA is done
      if (!mbar_wait(&o_full[x], j & 1, 18, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < DVP; c0 += 32) {
        if (c0 + 32 <= DVP) {
          uint32_t r[32];
          tmem_ld32(t_o + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_acc[c0 + i] = fmaf(o_acc[c0 + i], corr, __uint_as_float(r[i]));
        } else {
          uint32_t r[16];
          tmem_ld16_raw(t_o + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o_acc[c0 + i] = fmaf(o_acc[c0 + i], corr, __uint_as_float(r[i]));
        }
      }
      tc_fence_before();
      mbar_arrive(&o_empty[x]);
    }
    const int qi = qbase + x * kFaBM + row;
    if (ok && qi < p.Sq) {
      const float inv = 1.0f / l_run;
      char* base = static_cast<char*>(p.o);
      const int64_t off = (int64_t)b * p.os[0] + (int64_t)h * p.os[1] + (int64_t)qi * p.os[2];
      if (p.os[3] == 1 && (p.Dv % 8) == 0 && ((reinterpret_cast<uintptr_t>(base) + off * 2) % 16) == 0) {
        uint4* dst = reinterpret_cast<uint4*>(base + off * 2);
#pragma unroll
        for (int c = 0; c < DVP; c += 8) {
          if (c < p.Dv) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = F16 ? pack_f16x2(o_acc[c + 2 * i] * inv, o_acc[c + 2 * i + 1] * inv)
                         : pack_bf16x2(o_acc[c + 2 * i] * inv, o_acc[c + 2 * i + 1] * inv);
            dst[c / 8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < DVP; ++c)
          if (c < p.Dv) store_from_f32(p.o, off + (int64_t)c * p.os[3], p.out_dtype, o_acc[c] * inv);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Variant for small head dims (D <= 64) with the output kept in TMEM across KV tiles.
//
// Same roles and two query tiles per CTA, but the PV products accumulate into O in TMEM and the
// running max is only raised when a row's new maximum exceeds the one in use by more than 2^8
// ("lazy rescale"): p = 2^(s*scale*log2e - m_used) then stays <= 256, exact enough in bf16 / fp32.
// For head dims of at most DVP - 8 the row sum comes from the tensor core (a column of ones in the
// padding of V accumulates it into O), so the softmax warps only evaluate, round and store p.
// A rescale (rare after the first tile) waits for the previous PV, multiplies the row of O in
// TMEM and continues.  P is double-buffered in shared memory, so a softmax warpgroup never waits
// for its previous PV product — only for the S tile it consumes.
constexpr float kLazyThreshold = 8.0f;  // log2 of the largest p allowed before rescaling

template <int DP, int DVP, bool F16, bool SUMCOL, int PB>
__global__ void __launch_bounds__(320, 1)
    fa_lazy_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  constexpr int NQ = 2;
  constexpr int Q_BYTES = kFaBM * DP * 2;
  constexpr int K_BYTES = kFaBN * DP * 2;
  constexpr int V_BYTES = kFaBN * DVP * 2;
  // SUMCOL: the last 8-column chunk of each V stage is not loaded; its first column holds ones, so
  // the PV product also accumulates the row sum of P into column DVP - 8 of O.
  constexpr int V_TX = SUMCOL ? V_BYTES - kFaBN * 16 : V_BYTES;
  constexpr int P_BYTES = kFaBM * kFaBN * 2;
  constexpr uint32_t kLbo = kFaBM * 16;
  constexpr uint32_t kSbo = 128;
  constexpr int FMT = F16 ? 0 : 1;
  constexpr uint32_t idesc_s = make_idesc(FMT, kFaBM, kFaBN);
  constexpr uint32_t idesc_o = make_idesc(FMT, kFaBM, DVP) | (1u << 16);
  static_assert(2 * 128 + 2 * DVP <= 512, "TMEM budget");
  // PB P buffers per query tile (2 where shared memory allows): buffer and use number of tile j
  static_assert(PB == 1 || PB == 2, "P buffers");
  auto pbuf = [](int x, int j) { return x * PB + (PB == 2 ? (j & 1) : 0); };
  auto puse = [](int j) { return PB == 2 ? (j >> 1) : j; };

  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // [2][Q]
  uint8_t* sP = sQ + NQ * Q_BYTES;       // [2 tiles][PB buffers][P]
  // K and V in separate rings: a K tile is released once both QK^T products have read it, a V
  // tile only after both PV products, so loading K ahead never waits for the softmax.
  const int stages_k = p.stages, stages_v = p.stages_v;
  uint8_t* sK = sP + NQ * PB * P_BYTES;  // [stages_k][K]
  uint8_t* sV = sK + stages_k * K_BYTES;  // [stages_v][V]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + stages_v * V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + kFaMaxStages;
  uint64_t* v_full = k_empty + kFaMaxStages;
  uint64_t* v_empty = v_full + kFaMaxStages;
  uint64_t* s_full = v_empty + kFaMaxStages;  // [2]
  uint64_t* s_empty = s_full + 2;              // [2]
  // p_full / p_free are per P buffer: a softmax warpgroup may finish tile j+1 before the MMA warp
  // consumes tile j, so one barrier per tile could complete two phases ahead of its waiter.
  uint64_t* p_full = s_empty + 2;              // [2 tiles][2 buffers]
  uint64_t* p_free = p_full + 4;               // [2 tiles][2 buffers]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_free + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int qbase = blockIdx.x * (kFaBM * NQ);
  const int n_tiles = (p.Sk + kFaBN - 1) / kFaBN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kFaMaxStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (SUMCOL) {
    for (int i = threadIdx.x; i < stages_v * kFaBN; i += blockDim.x) {
      uint4* d = reinterpret_cast<uint4*>(sV + (i / kFaBN) * V_BYTES + (DVP / 8 - 1) * kFaBN * 16) + (i % kFaBN);
      *d = make_uint4(F16 ? 0x3C00u : 0x3F80u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o0 = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, NQ * Q_BYTES);
      for (int x = 0; x < NQ; ++x) tma_load_5d(sQ + x * Q_BYTES, &tmQ, q_full, 0, qbase + x * kFaBM, 0, h, b);
      // order: K(0), then K(j+1) before V(j) — the next QK^T needs its K before this PV needs V
      int ks = 0, vs = 0;
      uint32_t kph = 0, vph = 0;
      bool ok = true;
      for (int j = -1; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles) {
          if (!mbar_wait(&k_empty[ks], kph ^ 1, 21, abort_flag)) break;
          mbar_arrive_expect_tx(&k_full[ks], K_BYTES);
          tma_load_5d(sK + ks * K_BYTES, &tmK, &k_full[ks], 0, (j + 1) * kFaBN, 0, hk, b);
          if (++ks == stages_k) {
            ks = 0;
            kph ^= 1;
          }
        }
        if (j >= 0) {
          if (!mbar_wait(&v_empty[vs], vph ^ 1, 20, abort_flag)) break;
          mbar_arrive_expect_tx(&v_full[vs], V_TX);
          tma_load_5d(sV + vs * V_BYTES, &tmV, &v_full[vs], 0, j * kFaBN, 0, hk, b);
          if (++vs == stages_v) {
            vs = 0;
            vph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, 22, abort_flag);
      int ks = 0, vs = 0;
      uint32_t kph = 0, vph = 0;
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j < n_tiles) {
          if (!mbar_wait(&k_full[ks], kph, 23, abort_flag)) break;
          const uint32_t k_addr = smem_u32(sK + ks * K_BYTES);
          bool sok = true;
          for (int x = 0; x < NQ && sok; ++x) {
            if (!mbar_wait(&s_empty[x], (j & 1) ^ 1, 24, abort_flag)) {
              sok = false;
              break;
            }
            tc_fence_after();
            const uint32_t qa = q_addr + x * Q_BYTES;
#pragma unroll
            for (int kk = 0; kk < DP / 16; ++kk)
              umma_f16(tmem + x * 128, sdesc_none(qa + kk * 2 * kLbo, kLbo, kSbo),
                       sdesc_none(k_addr + kk * 2 * kLbo, kLbo, kSbo), idesc_s, kk > 0 ? 1u : 0u);
            umma_commit(&s_full[x]);
          }
          if (!sok) break;
          umma_commit(&k_empty[ks]);
          if (++ks == stages_k) {
            ks = 0;
            kph ^= 1;
          }
        }
        if (j > 0) {
          const int jj = j - 1;
          if (!mbar_wait(&v_full[vs], vph, 30, abort_flag)) break;
          const uint32_t v_addr = smem_u32(sV + vs * V_BYTES);
          bool pok = true;
          for (int x = 0; x < NQ; ++x) {
            if (!mbar_wait(&p_full[pbuf(x, jj)], puse(jj) & 1, 25, abort_flag)) {
              pok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pa = p_addr + pbuf(x, jj) * P_BYTES;
#pragma unroll
            for (int kk = 0; kk < kFaBN / 16; ++kk)
              umma_f16(t_o0 + x * DVP, sdesc_none(pa + kk * 2 * kLbo, kLbo, kSbo),
                       sdesc_none(v_addr + kk * 256, 128, kFaBN * 16), idesc_o, (jj > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&p_free[pbuf(x, jj)]);
          }
          if (!pok) break;
          umma_commit(&v_empty[vs]);
          if (++vs == stages_v) {
            vs = 0;
            vph ^= 1;
          }
        }
      }
    }
  } else {
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_o = t_o0 + x * DVP + lane_off;
    const uint32_t ts = tmem + x * 128 + lane_off;
    float m_used = -INFINITY, l_run = 0.f;
    const float sl = p.scale_log2;
    const uint64_t sl2 = f2_bits(sl, sl);
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!mbar_wait(&s_full[x], j & 1, 26, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int kvalid = min(kFaBN, p.Sk - j * kFaBN);
      const bool full = kvalid == kFaBN;
      float mx = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < kFaBN; c0 += 64) {
        uint32_t r[64];
        tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (full) {
          mx = fmaxf(mx, max64(r));
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (c0 + i < kvalid) mx = fmaxf(mx, __uint_as_float(r[i]));
        }
      }
      const float mt = mx * sl;
      if (j == 0) {
        m_used = mt;
      } else {
        const bool need = mt > m_used + kLazyThreshold;
        if (__any_sync(0xffffffffu, need)) {
          // O holds the sum over the previous tiles: wait for the last PV, then rescale in TMEM
          const float m_new = need ? mt : m_used;
          const float corr = ex2(m_used - m_new);
          // PV_{j-1} released P buffer (j-1)&1 (its use number (j-1)>>1); commits complete in issue
          // order, so this also covers every earlier PV.  Phases of p_free are consumed in order,
          // which keeps the parity test unambiguous.
          if (!mbar_wait(&p_free[pbuf(x, j - 1)], puse(j - 1) & 1, 27, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c0 = 0; c0 < DVP; c0 += 16) {
            uint32_t r[16];
            tmem_ld16_raw(t_o + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * corr);
            tmem_st16(t_o + c0, r);
          }
          tmem_st_wait();
          l_run *= corr;
          m_used = m_new;
        }
      }
      // the P buffer this tile writes was read by the PV two tiles back
      if (!mbar_wait(&p_free[pbuf(x, j)], (puse(j) & 1) ^ 1, 28, abort_flag)) {
        ok = false;
        break;
      }
      uint8_t* sPx = sP + pbuf(x, j) * P_BYTES;
      const uint64_t negm2 = f2_bits(-m_used, -m_used);
      uint64_t sum2 = f2_bits(0.f, 0.f);
#pragma unroll 1
      for (int c0 = 0; c0 < kFaBN; c0 += 64) {
        uint32_t r[64];
        tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        tmem_ld_wait();
        if (c0 == kFaBN - 64) {  // the last read of S: the next QK^T may overwrite it
          tc_fence_before();
          mbar_arrive(&s_empty[x]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int k = q * 16 + i;
            const uint64_t arg = ffma2(f2_bits(__uint_as_float(r[k]), __uint_as_float(r[k + 1])), sl2, negm2);
            float a0, a1;
            f2_unpack(arg, a0, a1);
            float e0 = ex2(a0), e1 = ex2(a1);
            if (!full) {
              if (c0 + k >= kvalid) e0 = 0.f;
              if (c0 + k + 1 >= kvalid) e1 = 0.f;
            }
            if (!SUMCOL) sum2 = fadd2(sum2, f2_bits(e0, e1));
            pk[i / 2] = F16 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
          }
          const int c = c0 + q * 16;
          uint4* d0 = reinterpret_cast<uint4*>(sPx + (c / 8) * (kFaBM * 16) + row * 16);
          uint4* d1 = reinterpret_cast<uint4*>(sPx + (c / 8 + 1) * (kFaBM * 16) + row * 16);
          *d0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *d1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[pbuf(x, j)]);
      float s0, s1;
      f2_unpack(sum2, s0, s1);
      l_run += s0 + s1;
    }
    // final: O (all PV products accumulated) / l
    if (ok && mbar_wait(&p_free[pbuf(x, n_tiles - 1)], puse(n_tiles - 1) & 1, 29, abort_flag)) {
      tc_fence_after();
      float o[DVP];
#pragma unroll
      for (int c0 = 0; c0 < DVP; c0 += 16) {
        uint32_t r[16];
        tmem_ld16_raw(t_o + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) o[c0 + i] = __uint_as_float(r[i]);
      }
      const int qi = qbase + x * kFaBM + row;
      if (qi < p.Sq) {
        const float inv = 1.0f / (SUMCOL ? o[DVP - 8] : l_run);
        char* base = static_cast<char*>(p.o);
        const int64_t off = (int64_t)b * p.os[0] + (int64_t)h * p.os[1] + (int64_t)qi * p.os[2];
        if (p.os[3] == 1 && (p.Dv % 8) == 0 && ((reinterpret_cast<uintptr_t>(base) + off * 2) % 16) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(base + off * 2);
#pragma unroll
          for (int c = 0; c < DVP; c += 8) {
            if (c < p.Dv) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                w[i] = F16 ? pack_f16x2(o[c + 2 * i] * inv, o[c + 2 * i + 1] * inv)
                           : pack_bf16x2(o[c + 2 * i] * inv, o[c + 2 * i + 1] * inv);
              dst[c / 8] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < DVP; ++c)
            if (c < p.Dv) store_from_f32(p.o, off + (int64_t)c * p.os[3], p.out_dtype, o[c] * inv);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------------
// Attention over at most one key tile (Sk <= 128: the UNet's cross-attention to 77 context tokens).
//
// With one key tile a CTA of the general kernels spends most of its life on fixed costs (TMEM
// allocation, barrier set-up, the first Q load, the output store) for a few hundred cycles of
// work.  Here a CTA loads K and V once and walks `p.pairs` consecutive pairs of 128-query tiles of
// one (b, h): warp 0 streams Q (one buffer per warpgroup), warp 1 issues S = Q K^T and O = P V,
// warpgroup x (warps 2-5, 6-9) takes query tile x of every pair: softmax of its S row (the whole
// row is in TMEM, so the maximum is exact and no rescale exists), P to shared memory, then O / l to
// global.  While a warpgroup finishes pair i, the MMA warp already computes S for the other
// warpgroup and, once S is released and the next Q has landed, for pair i + 1.
template <int DP, int DVP, bool F16, bool SUMCOL, int SN>
__global__ void __launch_bounds__(320, (2 * SN + 2 * DVP <= 256) ? 2 : 1)
    fa_short_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const FaParams p) {
  constexpr int Q_BYTES = kFaBM * DP * 2;
  constexpr int K_BYTES = kFaBN * DP * 2;
  constexpr int V_BYTES = kFaBN * DVP * 2;
  constexpr int V_TX = SUMCOL ? V_BYTES - kFaBN * 16 : V_BYTES;
  constexpr int P_BYTES = kFaBM * SN * 2;
  constexpr uint32_t kLbo = kFaBM * 16;
  constexpr uint32_t kSbo = 128;
  constexpr int FMT = F16 ? 0 : 1;
  // SN score columns (keys rounded up to 16: 80 for the 77 context tokens, else 128): with
  // 2 SN + 2 DVP <= 256 TMEM columns (SN 80, head dims up to 48) two CTAs share an SM
  static_assert(SN % 16 == 0 && SN <= kFaBN, "score width");
  constexpr int TCOLS = (2 * SN + 2 * DVP <= 256) ? 256 : 512;
  constexpr uint32_t idesc_s = make_idesc(FMT, kFaBM, SN);
  constexpr uint32_t idesc_o = make_idesc(FMT, kFaBM, DVP) | (1u << 16);
  static_assert(2 * SN + 2 * DVP <= 512, "TMEM budget");

  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;             // [2][Q]
  uint8_t* sP = sQ + 2 * Q_BYTES;  // [2][P]
  uint8_t* sK = sP + 2 * P_BYTES;
  uint8_t* sV = sK + K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + V_BYTES);
  uint64_t* kv_full = bars;        // K and V loaded
  uint64_t* q_full = bars + 1;     // [2]
  uint64_t* q_empty = q_full + 2;  // [2]
  uint64_t* s_full = q_empty + 2;  // [2]
  uint64_t* s_empty = s_full + 2;  // [2]
  uint64_t* p_full = s_empty + 2;  // [2]
  uint64_t* o_full = p_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int hk = h / (p.H / p.Hkv);
  const int pair0 = blockIdx.x * p.pairs;
  const int total_pairs = (p.Sq + 2 * kFaBM - 1) / (2 * kFaBM);
  const int npairs = min(p.pairs, total_pairs - pair0);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (SUMCOL) {  // the unloaded last 8-column chunk of V: a column of ones (row sums of P)
    for (int i = threadIdx.x; i < kFaBN; i += blockDim.x) {
      uint4* d = reinterpret_cast<uint4*>(sV + (DVP / 8 - 1) * kFaBN * 16) + i;
      *d = make_uint4(F16 ? 0x3C00u : 0x3F80u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o0 = tmem + 2 * SN;  // S slots at [0, SN) and [SN, 2 SN), then O of each tile

  if (warp == 0) {
    if (lane == 0 && npairs > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(kv_full, K_BYTES + V_TX);
      tma_load_5d(sK, &tmK, kv_full, 0, 0, 0, hk, b);
      tma_load_5d(sV, &tmV, kv_full, 0, 0, 0, hk, b);
      for (int i = 0; i < npairs; ++i)
        for (int x = 0; x < 2; ++x) {
          if (!mbar_wait(&q_empty[x], (i & 1) ^ 1, 41, abort_flag)) i = npairs;
          if (i >= npairs) break;
          mbar_arrive_expect_tx(&q_full[x], Q_BYTES);
          tma_load_5d(sQ + x * Q_BYTES, &tmQ, &q_full[x], 0, ((pair0 + i) * 2 + x) * kFaBM, 0, h, b);
        }
    }
  } else if (warp == 1) {
    if (lane == 0 && npairs > 0) {
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, 42, abort_flag);
      for (int i = 0; ok && i < npairs; ++i) {
        for (int x = 0; x < 2 && ok; ++x) {
          ok = mbar_wait(&q_full[x], i & 1, 43, abort_flag) && mbar_wait(&s_empty[x], (i & 1) ^ 1, 44, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t qa = q_addr + x * Q_BYTES;
#pragma unroll
          for (int kk = 0; kk < DP / 16; ++kk)
            umma_f16(tmem + x * SN, sdesc_none(qa + kk * 2 * kLbo, kLbo, kSbo),
                     sdesc_none(k_addr + kk * 2 * kLbo, kLbo, kSbo), idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[x]);
          umma_commit(&q_empty[x]);
        }
        for (int x = 0; x < 2 && ok; ++x) {
          // P of pair i is written only after the warpgroup has read O of pair i - 1, so the
          // product below never overwrites an O still being read
          ok = mbar_wait(&p_full[x], i & 1, 45, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t pa = p_addr + x * P_BYTES;
#pragma unroll
          for (int kk = 0; kk < SN / 16; ++kk)
            umma_f16(t_o0 + x * DVP, sdesc_none(pa + kk * 2 * kLbo, kLbo, kSbo),
                     sdesc_none(v_addr + kk * 256, 128, kFaBN * 16), idesc_o, kk > 0 ? 1u : 0u);
          umma_commit(&o_full[x]);
        }
      }
    }
  } else {
    const int x = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_o = t_o0 + x * DVP + lane_off;
    const uint32_t ts = tmem + x * SN + lane_off;
    const float sl = p.scale_log2;
    const uint64_t sl2 = f2_bits(sl, sl);
    const int kvalid = p.Sk;  // <= kFaBN
    const bool full = kvalid == kFaBN;
    uint8_t* sPx = sP + x * P_BYTES;
    for (int i = 0; i < npairs; ++i) {
      if (!mbar_wait(&s_full[x], i & 1, 46, abort_flag)) break;
      tc_fence_after();
      float mx = -INFINITY;
      if (SN == kFaBN) {
#pragma unroll 1
        for (int c0 = 0; c0 < kFaBN; c0 += 64) {
          uint32_t r[64];
          tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_ld_wait();
          if (full) {
            mx = fmaxf(mx, max64(r));
          } else {
#pragma unroll
            for (int k = 0; k < 64; ++k)
              if (c0 + k < kvalid) mx = fmaxf(mx, __uint_as_float(r[k]));
          }
        }
      } else {
        // the whole SN-column row in one round of loads (16-column pieces)
        uint32_t r[SN];
#pragma unroll
        for (int c0 = 0; c0 < SN; c0 += 16) tmem_ld16_raw(ts + c0, *reinterpret_cast<uint32_t(*)[16]>(&r[c0]));
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < SN; ++k)
          if (k < kvalid) mx = fmaxf(mx, __uint_as_float(r[k]));
      }
      const uint64_t negm2 = f2_bits(-mx * sl, -mx * sl);
      uint64_t sum2 = f2_bits(0.f, 0.f);
      constexpr int CW = SN == kFaBN ? 64 : SN;  // columns per round of TMEM loads
#pragma unroll 1
      for (int c0 = 0; c0 < SN; c0 += CW) {
        uint32_t r[CW];
        if (CW == 64) {
          tmem_ld32(ts + c0, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(ts + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32 % CW]));
        } else {
#pragma unroll
          for (int cc = 0; cc < CW; cc += 16) tmem_ld16_raw(ts + c0 + cc, *reinterpret_cast<uint32_t(*)[16]>(&r[cc]));
        }
        tmem_ld_wait();
        if (c0 == SN - CW) {  // the last read of S: the next QK^T may overwrite it
          tc_fence_before();
          mbar_arrive(&s_empty[x]);
        }
#pragma unroll
        for (int q = 0; q < CW / 16; ++q) {
          uint32_t pk[8];
          const int c = c0 + q * 16;
          if (c >= kvalid) {  // 16 keys past the end: P is zero, no exponentials (uniform branch)
            uint4* d0 = reinterpret_cast<uint4*>(sPx + (c / 8) * (kFaBM * 16) + row * 16);
            uint4* d1 = reinterpret_cast<uint4*>(sPx + (c / 8 + 1) * (kFaBM * 16) + row * 16);
            *d0 = make_uint4(0u, 0u, 0u, 0u);
            *d1 = make_uint4(0u, 0u, 0u, 0u);
            continue;
          }
#pragma unroll
          for (int k2 = 0; k2 < 16; k2 += 2) {
            const int k = q * 16 + k2;
            const uint64_t arg = ffma2(f2_bits(__uint_as_float(r[k]), __uint_as_float(r[k + 1])), sl2, negm2);
            float a0, a1;
            f2_unpack(arg, a0, a1);
            float e0 = ex2(a0), e1 = ex2(a1);
            if (!full) {
              if (c0 + k >= kvalid) e0 = 0.f;
              if (c0 + k + 1 >= kvalid) e1 = 0.f;
            }
            if (!SUMCOL) sum2 = fadd2(sum2, f2_bits(e0, e1));
            pk[k2 / 2] = F16 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
          }
          uint4* d0 = reinterpret_cast<uint4*>(sPx + (c / 8) * (kFaBM * 16) + row * 16);
          uint4* d1 = reinterpret_cast<uint4*>(sPx + (c / 8 + 1) * (kFaBM * 16) + row * 16);
          *d0 = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *d1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
      if (!mbar_wait(&o_full[x], i & 1, 47, abort_flag)) break;
      tc_fence_after();
      float o[DVP];
#pragma unroll
      for (int c0 = 0; c0 < DVP; c0 += 16) {
        uint32_t r[16];
        tmem_ld16_raw(t_o + c0, r);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; ++k) o[c0 + k] = __uint_as_float(r[k]);
      }
      float s0, s1;
      f2_unpack(sum2, s0, s1);
      const int qi = ((pair0 + i) * 2 + x) * kFaBM + row;
      if (qi < p.Sq) {
        const float inv = 1.0f / (SUMCOL ? o[DVP - 8] : s0 + s1);
        char* base = static_cast<char*>(p.o);
        const int64_t off = (int64_t)b * p.os[0] + (int64_t)h * p.os[1] + (int64_t)qi * p.os[2];
        if (p.os[3] == 1 && (p.Dv % 8) == 0 && ((reinterpret_cast<uintptr_t>(base) + off * 2) % 16) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(base + off * 2);
#pragma unroll
          for (int c = 0; c < DVP; c += 8) {
            if (c < p.Dv) {
              uint32_t w[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                w[k] = F16 ? pack_f16x2(o[c + 2 * k] * inv, o[c + 2 * k + 1] * inv)
                           : pack_bf16x2(o[c + 2 * k] * inv, o[c + 2 * k + 1] * inv);
              dst[c / 8] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        } else {
#pragma unroll
          for (int c = 0; c < DVP; ++c)
            if (c < p.Dv) store_from_f32(p.o, off + (int64_t)c * p.os[3], p.out_dtype, o[c] * inv);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side.

template <int DP, int DVP, int NQ>
struct FaCfg {
  static constexpr int FIXED = NQ * (kFaBM * DP * 2 + kFaBM * kFaBN * 2);
  static constexpr int STAGE = kFaBN * (DP + DVP) * 2;
  static constexpr int SMEM_MAX = 224 * 1024;
  static constexpr int STAGES_RAW = (SMEM_MAX - 2048 - FIXED) / STAGE;
  static constexpr int STAGES = STAGES_RAW > kFaMaxStages ? kFaMaxStages : STAGES_RAW;
  static constexpr int smem_bytes(int stages) { return FIXED + stages * STAGE + 2048; }
};

// 5-D map {8, S, D/8, heads, batch} over a strided [B, Hx, S, D] view (element strides st).
static int fa_map(CUtensorMap* m, int dtype, const void* base, int64_t B, int64_t Hx, int64_t S, int64_t D,
                  const int64_t* st, int box_chunks) {
  if (st[3] != 1) return fail(MT_ERR_UNSUPPORTED, "flash attention: head dim must be unit-stride");
  uint64_t dims[5] = {8, (uint64_t)S, (uint64_t)(D / 8), (uint64_t)Hx, (uint64_t)B};
  uint64_t strides[4] = {(uint64_t)st[2] * 2, 16, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  if (Hx == 1) strides[2] = 16;  // single head: any legal stride
  if (B == 1) strides[3] = 16;   // single batch entry: any legal stride
  uint32_t box[5] = {8, 128, (uint32_t)box_chunks, 1, 1};
  return make_tensor_map(m, dtype, 5, base, dims, strides, box, 0);
}

template <int DP, int DVP, int NQ, bool F16, bool MASK = false>
static int fa_launch(const mt_sdpa_desc& d, cudaStream_t st) {
  using Cfg = FaCfg<DP, DVP, NQ>;
  const int stages = Cfg::STAGES;
  if (stages < 1) return fail(MT_ERR_UNSUPPORTED, "flash attention: head dim too large for shared memory");
  const int smem = Cfg::smem_bytes(stages) + 1024;
  auto kern = fa_sm100_kernel<DP, DVP, NQ, F16, MASK>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                        "flash attention smem attribute");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  CUtensorMap mq, mk, mv;
  int rc = fa_map(&mq, d.dtype, d.q, d.B, d.H, d.Sq, d.D, d.q_strides, DP / 8);
  if (!rc) rc = fa_map(&mk, d.dtype, d.k, d.B, d.Hkv, d.Sk, d.D, d.k_strides, DP / 8);
  if (!rc) rc = fa_map(&mv, d.dtype, d.v, d.B, d.Hkv, d.Sk, d.Dv, d.v_strides, DVP / 8);
  if (rc) return rc;
  FaParams p{};
  p.Sq = (int)d.Sq; p.Sk = (int)d.Sk; p.H = (int)d.H; p.Hkv = (int)d.Hkv; p.B = (int)d.B;
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.o = d.o;
  for (int i = 0; i < 4; ++i) p.os[i] = d.o_strides[i];
  p.Dv = (int)d.Dv;
  p.out_dtype = d.dtype;
  p.stages = stages;
  p.causal = d.causal ? 1 : 0;
  p.mask = d.mask_kind ? d.mask : nullptr;
  p.mask_kind = d.mask_kind;
  p.mask_dtype = d.mask_dtype;
  for (int i = 0; i < 4; ++i) p.ms[i] = d.mask_strides[i];
  dim3 grid((unsigned)((d.Sq + kFaBM * NQ - 1) / (kFaBM * NQ)), (unsigned)(d.B * d.H));
  kern<<<grid, 64 + 128 * NQ, smem, st>>>(mq, mk, mv, p);
  return check_launch("flash_attention_sm100");
}

// Launch of the lazy-rescale variant with PB P buffers per query tile; returns false (not
// launched) when two KV stages do not fit.
template <int DP, int DVP, bool F16, bool SUMCOL, int PB>
static int fa_lazy_launch(const mt_sdpa_desc& d, cudaStream_t st, bool* launched) {
  constexpr int FIXED = 2 * (kFaBM * DP * 2 + PB * kFaBM * kFaBN * 2);
  constexpr int K_BYTES = kFaBN * DP * 2, V_BYTES = kFaBN * DVP * 2;
  constexpr int SMEM_MAX = 224 * 1024;
  const int stages_v = 2;
  int stages_k = (SMEM_MAX - 2048 - FIXED - stages_v * V_BYTES) / K_BYTES;
  if (stages_k > kFaMaxStages) stages_k = kFaMaxStages;
  *launched = false;
  if (stages_k < 2) return MT_OK;
  const int smem = FIXED + stages_k * K_BYTES + stages_v * V_BYTES + 2048 + 1024;
  auto kern = fa_lazy_sm100_kernel<DP, DVP, F16, SUMCOL, PB>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                        "flash attention smem attribute");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  CUtensorMap mq, mk, mv;
  int rc = fa_map(&mq, d.dtype, d.q, d.B, d.H, d.Sq, d.D, d.q_strides, DP / 8);
  if (!rc) rc = fa_map(&mk, d.dtype, d.k, d.B, d.Hkv, d.Sk, d.D, d.k_strides, DP / 8);
  if (!rc) rc = fa_map(&mv, d.dtype, d.v, d.B, d.Hkv, d.Sk, d.Dv, d.v_strides, SUMCOL ? DVP / 8 - 1 : DVP / 8);
  if (rc) return rc;
  FaParams p{};
  p.Sq = (int)d.Sq; p.Sk = (int)d.Sk; p.H = (int)d.H; p.Hkv = (int)d.Hkv; p.B = (int)d.B;
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.o = d.o;
  for (int i = 0; i < 4; ++i) p.os[i] = d.o_strides[i];
  p.Dv = (int)d.Dv;
  p.out_dtype = d.dtype;
  p.stages = stages_k;
  p.stages_v = stages_v;
  dim3 grid((unsigned)((d.Sq + 2 * kFaBM - 1) / (2 * kFaBM)), (unsigned)(d.B * d.H));
  kern<<<grid, 320, smem, st>>>(mq, mk, mv, p);
  *launched = true;
  return check_launch("flash_attention_lazy_sm100");
}

// Launch of the short-KV kernel (Sk <= 128): CTAs of `pairs` 256-query pairs of one (b, h), about
// four CTAs per SM in total so that the last wave is short.
template <int DP, int DVP, bool F16, bool SUMCOL, int SN>
static int fa_short_launch_sn(const mt_sdpa_desc& d, cudaStream_t st);

template <int DP, int DVP, bool F16, bool SUMCOL>
static int fa_short_launch(const mt_sdpa_desc& d, cudaStream_t st) {
  // 80 score columns (two CTAs per SM where TMEM allows) for up to 80 keys, else 128
  if constexpr (2 * 80 + 2 * DVP <= 256) {
    static const bool wide = getenv("MT_FA_SHORT_WIDE") != nullptr;
    if (d.Sk <= 80 && !wide) return fa_short_launch_sn<DP, DVP, F16, SUMCOL, 80>(d, st);
  }
  return fa_short_launch_sn<DP, DVP, F16, SUMCOL, kFaBN>(d, st);
}

template <int DP, int DVP, bool F16, bool SUMCOL, int SN>
static int fa_short_launch_sn(const mt_sdpa_desc& d, cudaStream_t st) {
  constexpr int SMEM = 2 * kFaBM * DP * 2 + 2 * kFaBM * SN * 2 + kFaBN * (DP + DVP) * 2 + 1024 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  constexpr int OCC = (2 * SN + 2 * DVP <= 256) ? 2 : 1;  // CTAs per SM
  auto kern = fa_short_sm100_kernel<DP, DVP, F16, SUMCOL, SN>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM),
                        "short attention smem attribute");
    if (rc) return rc;
    attr[dev & 63] = true;
  }
  CUtensorMap mq, mk, mv;
  int rc = fa_map(&mq, d.dtype, d.q, d.B, d.H, d.Sq, d.D, d.q_strides, DP / 8);
  if (!rc) rc = fa_map(&mk, d.dtype, d.k, d.B, d.Hkv, d.Sk, d.D, d.k_strides, DP / 8);
  if (!rc) rc = fa_map(&mv, d.dtype, d.v, d.B, d.Hkv, d.Sk, d.Dv, d.v_strides, SUMCOL ? DVP / 8 - 1 : DVP / 8);
  if (rc) return rc;
  FaParams p{};
  p.Sq = (int)d.Sq; p.Sk = (int)d.Sk; p.H = (int)d.H; p.Hkv = (int)d.Hkv; p.B = (int)d.B;
  p.scale_log2 = (float)(d.scale * 1.4426950408889634);
  p.o = d.o;
  for (int i = 0; i < 4; ++i) p.os[i] = d.o_strides[i];
  p.Dv = (int)d.Dv;
  p.out_dtype = d.dtype;
  const int64_t pairs_bh = (d.Sq + 2 * kFaBM - 1) / (2 * kFaBM);
  const int64_t bh = d.B * d.H;
  const int64_t cpb =
      std::min<int64_t>(pairs_bh, std::max<int64_t>(1, (4 * OCC * (int64_t)num_sms() + bh - 1) / bh));
  p.pairs = (int)((pairs_bh + cpb - 1) / cpb);
  dim3 grid((unsigned)((pairs_bh + p.pairs - 1) / p.pairs), (unsigned)bh);
  kern<<<grid, 320, SMEM, st>>>(mq, mk, mv, p);
  return check_launch("flash_attention_short_sm100");
}

size_t sdpa_tc_workspace(const mt_sdpa_desc&) { return 0; }

static bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Padded head dim of the tcgen05 kernels for head dim D (a multiple of 8): the smallest
// instantiated width >= D (TMA zero-fills the padding columns); 0 when none fits.
static int64_t tc_head_pad(int64_t D) {
  if (D % 8 != 0) return 0;
  for (int64_t w : {32, 48, 64, 80, 128, 160})
    if (D <= w) return w;
  return 0;
}

// Which kernel run_sdpa_tc launches for `d`: MT_SDPA_PATH_TC_LAZY, MT_SDPA_PATH_TC, or
// MT_SDPA_PATH_SIMT when the tcgen05 kernels do not take it.
int sdpa_tc_path(const mt_sdpa_desc& d) {
  if (d.dtype != MT_BF16 && d.dtype != MT_F16) return MT_SDPA_PATH_SIMT;
  if (d.mask_kind != 0 && (!d.mask || (d.mask_kind == 2 && d.mask_dtype != MT_F32 && d.mask_dtype != MT_BF16 &&
                                       d.mask_dtype != MT_F16)))
    return MT_SDPA_PATH_SIMT;
  if (d.D != d.Dv) return MT_SDPA_PATH_SIMT;
  if (!(d.scale > 0)) return MT_SDPA_PATH_SIMT;  // the tcgen05 kernels take the row max of unscaled scores
  const int64_t Dp = tc_head_pad(d.D);
  if (Dp == 0) return MT_SDPA_PATH_SIMT;
  if (d.Sq > INT32_MAX || d.Sk > INT32_MAX || d.B * d.H > 65535) return MT_SDPA_PATH_SIMT;
  if (!aligned16p(d.q) || !aligned16p(d.k) || !aligned16p(d.v)) return MT_SDPA_PATH_SIMT;
  for (int i = 0; i < 3; ++i)
    if ((d.q_strides[i] * 2) % 16 || (d.k_strides[i] * 2) % 16 || (d.v_strides[i] * 2) % 16)
      return MT_SDPA_PATH_SIMT;
  if (d.q_strides[3] != 1 || d.k_strides[3] != 1 || d.v_strides[3] != 1) return MT_SDPA_PATH_SIMT;
  const bool two = d.Sq > kFaBM;
  static const bool no_short = getenv("MT_FA_NO_SHORT") != nullptr;
  if (d.Sk <= kFaBN && Dp <= 128 && !d.causal && d.mask_kind == 0 && !no_short) return MT_SDPA_PATH_TC_SHORT;
  // the lazy variant (O in TMEM) for padded head dims up to 80 (MT_FA_LAZY_MAX lowers the limit)
  static const int lazy_max = [] {
    const char* e = getenv("MT_FA_LAZY_MAX");
    return e ? atoi(e) : 80;
  }();
  if (two && Dp <= lazy_max && Dp <= 80 && d.scale > 0 && !d.causal && d.mask_kind == 0 && !getenv("MT_FA_NO_LAZY"))
    return MT_SDPA_PATH_TC_LAZY;
  return MT_SDPA_PATH_TC;
}

template <bool F16>
static int fa_short_dispatch(const mt_sdpa_desc& d, int64_t Dp, cudaStream_t st) {
  const bool sumcol = d.Dv <= Dp - 8;
  switch (Dp) {
    case 32: return sumcol ? fa_short_launch<32, 32, F16, true>(d, st) : fa_short_launch<32, 32, F16, false>(d, st);
    case 48: return sumcol ? fa_short_launch<48, 48, F16, true>(d, st) : fa_short_launch<48, 48, F16, false>(d, st);
    case 64: return sumcol ? fa_short_launch<64, 64, F16, true>(d, st) : fa_short_launch<64, 64, F16, false>(d, st);
    case 80: return sumcol ? fa_short_launch<80, 80, F16, true>(d, st) : fa_short_launch<80, 80, F16, false>(d, st);
    case 128:
      return sumcol ? fa_short_launch<128, 128, F16, true>(d, st) : fa_short_launch<128, 128, F16, false>(d, st);
    default: return fail(MT_ERR_UNSUPPORTED, "sdpa: no short-KV kernel for padded head dim %lld", (long long)Dp);
  }
}

template <bool F16>
static int fa_dispatch(const mt_sdpa_desc& d, int64_t Dp, bool lazy, cudaStream_t st) {
  // two query tiles per CTA when there are enough queries to fill them
  const bool two = d.Sq > kFaBM;
  if (lazy) {
    bool launched = false;
    // double-buffered P up to head dim 48; one P buffer per query tile beyond (shared memory)
    int rc = MT_OK;
    switch (Dp) {
      case 32: rc = d.Dv <= 24 ? fa_lazy_launch<32, 32, F16, true, 2>(d, st, &launched)
                               : fa_lazy_launch<32, 32, F16, false, 2>(d, st, &launched); break;
      case 48: rc = d.Dv <= 40 ? fa_lazy_launch<48, 48, F16, true, 2>(d, st, &launched)
                               : fa_lazy_launch<48, 48, F16, false, 2>(d, st, &launched); break;
      case 64: rc = d.Dv <= 56 ? fa_lazy_launch<64, 64, F16, true, 1>(d, st, &launched)
                               : fa_lazy_launch<64, 64, F16, false, 1>(d, st, &launched); break;
      default: rc = d.Dv <= 72 ? fa_lazy_launch<80, 80, F16, true, 1>(d, st, &launched)
                               : fa_lazy_launch<80, 80, F16, false, 1>(d, st, &launched); break;
    }
    if (rc || launched) return rc;
  }
  if (d.mask_kind != 0) {
    // masked calls: one query tile per CTA, the mask read per score in the softmax
    switch (Dp) {
      case 32: return fa_launch<32, 32, 1, F16, true>(d, st);
      case 48: return fa_launch<48, 48, 1, F16, true>(d, st);
      case 64: return fa_launch<64, 64, 1, F16, true>(d, st);
      case 80: return fa_launch<80, 80, 1, F16, true>(d, st);
      case 128: return fa_launch<128, 128, 1, F16, true>(d, st);
      case 160: return fa_launch<160, 160, 1, F16, true>(d, st);
      default: return fail(MT_ERR_UNSUPPORTED, "sdpa: no tcgen05 kernel for padded head dim %lld", (long long)Dp);
    }
  }
  switch (Dp) {
    case 32: return two ? fa_launch<32, 32, 2, F16>(d, st) : fa_launch<32, 32, 1, F16>(d, st);
    case 48: return two ? fa_launch<48, 48, 2, F16>(d, st) : fa_launch<48, 48, 1, F16>(d, st);
    case 64: return two ? fa_launch<64, 64, 2, F16>(d, st) : fa_launch<64, 64, 1, F16>(d, st);
    case 80: return two ? fa_launch<80, 80, 2, F16>(d, st) : fa_launch<80, 80, 1, F16>(d, st);
    case 128: return two ? fa_launch<128, 128, 2, F16>(d, st) : fa_launch<128, 128, 1, F16>(d, st);
    case 160: return fa_launch<160, 160, 1, F16>(d, st);
    default: return fail(MT_ERR_UNSUPPORTED, "sdpa: no tcgen05 kernel for padded head dim %lld", (long long)Dp);
  }
}

int run_sdpa_tc(const mt_sdpa_desc& d, void*, size_t, cudaStream_t st, bool* handled) {
  const int path = sdpa_tc_path(d);
  *handled = path != MT_SDPA_PATH_SIMT;
  if (!*handled) return MT_OK;
  const int64_t Dp = tc_head_pad(d.D);
  if (path == MT_SDPA_PATH_TC_SHORT)
    return d.dtype == MT_F16 ? fa_short_dispatch<true>(d, Dp, st) : fa_short_dispatch<false>(d, Dp, st);
  const bool lazy = path == MT_SDPA_PATH_TC_LAZY;
  return d.dtype == MT_F16 ? fa_dispatch<true>(d, Dp, lazy, st) : fa_dispatch<false>(d, Dp, lazy, st);
}

}  // namespace mt
