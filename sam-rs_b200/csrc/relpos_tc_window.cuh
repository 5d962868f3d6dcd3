// relpos_tc_window.cuh - tcgen05 kernel for SAM's windowed layers: 14x14 windows (196 tokens),
// head_dim 64 or 80, f16/bf16 I/O, f32 accumulation and softmax.
//
// Math as the global kernel (src/kernels.rs:131-225; windows from src/sam1/encoder.rs:118-121,132-145):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+13] + q_r . Tw[j-kw+13],  r = 14 i + j, k = 14 kh + kw.
//
// These layers are HBM-bound (~98 FLOP/B at hd 80), so the kernel is built to stream: a persistent grid
// (one CTA per SM) walks over units = (window, head) pairs, with the loads of unit u+1 in flight while
// unit u is computed (2-stage ring of Q | V | K). Per unit the 196 query rows are two 128-row MMA tiles
// (rows >= 196 are zero-filled by TMA and never stored) and all 196 keys fit one N = 208 key tile, so
// the softmax is a plain two-pass row softmax: no online rescaling.
//
// Loads: q and v through 3-D TMA tensor maps [bh][196][hd] (OOB rows -> 0). kt ([bh][hd][196]) has a
// 392-byte row pitch, which TMA cannot tile (strides must be multiples of 16 B), so 128 loader threads
// move it with 8-byte cp.async straight into the canonical no-swizzle MN-major UMMA layout (8 keys x 8
// dims per 128-byte core matrix); padded keys 196..207 stay zero.
// Bias: one prologue MMA per tile gives [RH | RW] = Q [Th(27) | Tw(27)]^T (N = 64) in TMEM; each thread
// selects its 14 + 14 values with a lane-dependent 4-stage shift (by i for rh, by j for rw).
//
// Warps: 0 TMA producer, 1 MMA issuer, 2 TMEM allocator, 4-7 kt loaders, 8-11 / 12-15 softmax + epilogue
// of query tile 0 / 1 (thread = query row = TMEM lane).
// TMEM (512 columns): tile t owns [256t, 256t+208): S_t (f32, 208 keys), then P_t (16-bit, cols 0..103)
// written over the consumed S; O_t accumulates in cols [128, 128+hd) once the softmax has consumed S_t;
// the prologue's [RH | RW] uses cols [0, 64).
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tcw {

constexpr int kThreads = 512;
constexpr int kSide = 14, kN = 196, kNP = 208, kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct Layout {
  static constexpr int HC = HD / 16;
  static constexpr int kQChunk = 128 * 32;          // [128 rows x 32 B] SW32
  static constexpr int kQTile = HC * kQChunk;
  static constexpr int kQBytes = 2 * kQTile;
  static constexpr int kVChunk = kNP * 32;          // [208 keys x 32 B] SW32
  static constexpr int kVBytes = HC * kVChunk;
  static constexpr int kKSbo = (HD / 8) * 128;       // stride between 8-key core columns
  static constexpr int kKBytes = (kNP / 8) * kKSbo;
  static constexpr int kStage = kQBytes + kVBytes + kKBytes;
  static constexpr int OFF_Q = 0, OFF_V = kQBytes, OFF_K = kQBytes + kVBytes;
  static constexpr int kTabChunk = 64 * 32;         // [Th 32 rows | Tw 32 rows] x 32 B
  static constexpr int kTabBytes = HC * kTabChunk;
  static constexpr int OFF_TAB = kStages * kStage;
  static constexpr int OFF_BAR = OFF_TAB + kTabBytes;
  static constexpr int kSmemBytes = OFF_BAR + 256 + 1024;
  static_assert(kStage % 1024 == 0 && kVChunk % 256 == 0 && OFF_K % 128 == 0, "alignment");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Bars {
  uint64_t q_full[kStages], v_full[kStages], k_full[kStages], stage_free[kStages];
  uint64_t tab_full, final_mma;
  uint64_t rhw_full[2], bias_done[2], s_full[2], p_full[2], o_full[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Byte offset of (key n, dim d) in the no-swizzle MN-major K tile.
template <int HD>
__device__ __forceinline__ uint32_t k_off(int n, int d) {
  return (uint32_t)((n >> 3) * Layout<HD>::kKSbo + (d >> 3) * 128 + (d & 7) * 16 + (n & 7) * 2);
}

// a[m] <- a[m + 2^B] where bit B of `sh` is set, for m < LEN.
template <int B, int LEN>
__device__ __forceinline__ void wshift(uint32_t (&a)[32], int sh) {
  const uint32_t take = (sh >> B) & 1;
#pragma unroll
  for (int m = 0; m < LEN; ++m) a[m] = sm100::select_u32(take, a[m + (1 << B)], a[m]);
}

// out[k] = a[sh + 13 - k] * log2(e) for k = 0..13, sh in [0, 15].
__device__ __forceinline__ void select14(uint32_t (&a)[32], int sh, float (&out)[14]) {
  wshift<3, 21>(a, sh);
  wshift<2, 17>(a, sh);
  wshift<1, 15>(a, sh);
  wshift<0, 14>(a, sh);
#pragma unroll
  for (int k = 0; k < 14; ++k) out[k] = __uint_as_float(a[13 - k]) * kLog2e;
}

// Pass 1 over one 32-key chunk: running max of S*c + rh[kh] + rw[kw] over valid keys.
template <int CH>
__device__ __forceinline__ float chunk_max(uint32_t tS, float c, const float (&rh)[14], const float (&rw)[14], float m) {
  using namespace sm100;
  uint32_t sv[32];
  tmem_ld32(tS + 32 * CH, sv);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int key = 32 * CH + e;
    if (key < kN) m = fmaxf(m, fmaf(__uint_as_float(sv[e]), c, rh[key / kSide]) + rw[key % kSide]);
  }
  return m;
}

// Pass 2 over one 32-key chunk: p = 2^(S*c + rh + rw - m), row sum, 16-bit P into TMEM columns 16*CH...
template <int CH, bool BF16>
__device__ __forceinline__ float chunk_exp(uint32_t tS, float c, const float (&rh)[14], const float (&rwm)[14],
                                           float sum) {
  using namespace sm100;
  uint32_t sv[32];
  tmem_ld32(tS + 32 * CH, sv);
  tmem_wait_ld();
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const int k0 = 32 * CH + e, k1 = k0 + 1;
    const float p0 = k0 < kN ? ex2(fmaf(__uint_as_float(sv[e]), c, rh[k0 / kSide]) + rwm[k0 % kSide]) : 0.f;
    const float p1 = k1 < kN ? ex2(fmaf(__uint_as_float(sv[e + 1]), c, rh[k1 / kSide]) + rwm[k1 % kSide]) : 0.f;
    sum += p0 + p1;
    pk[e >> 1] = pack2(p0, p1, BF16);
  }
  tmem_st16(tS + 16 * CH, pk);
  return sum;
}

// Keys 192..207 (last 16 columns; 192..195 valid).
__device__ __forceinline__ float tail_max(uint32_t tS, float c, const float (&rh)[14], const float (&rw)[14], float m) {
  using namespace sm100;
  uint32_t sv[16];
  tmem_ld16(tS + 192, sv);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int key = 192 + e;
    m = fmaxf(m, fmaf(__uint_as_float(sv[e]), c, rh[key / kSide]) + rw[key % kSide]);
  }
  return m;
}

template <bool BF16>
__device__ __forceinline__ float tail_exp(uint32_t tS, float c, const float (&rh)[14], const float (&rwm)[14],
                                          float sum) {
  using namespace sm100;
  uint32_t sv[16];
  tmem_ld16(tS + 192, sv);
  tmem_wait_ld();
  uint32_t pk[8];
#pragma unroll
  for (int e = 0; e < 16; e += 2) {
    const int k0 = 192 + e, k1 = k0 + 1;
    const float p0 = k0 < kN ? ex2(fmaf(__uint_as_float(sv[e]), c, rh[k0 / kSide]) + rwm[k0 % kSide]) : 0.f;
    const float p1 = k1 < kN ? ex2(fmaf(__uint_as_float(sv[e + 1]), c, rh[k1 / kSide]) + rwm[k1 % kSide]) : 0.f;
    sum += p0 + p1;
    pk[e >> 1] = pack2(p0, p1, BF16);
  }
  tmem_st8(tS + 96, pk);
  return sum;
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_window(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmT, const T* __restrict__ kt, T* __restrict__ out,
                       long bh_total, float scale) {
  using L = Layout<HD>;
  using namespace sm100;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  if (device_faulted()) return;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long first = blockIdx.x;
  const int n_units = first < bh_total ? (int)((bh_total - first + gridDim.x - 1) / gridDim.x) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->k_full[s], 128);
      mbar_init(&bars->stage_free[s], 1);
    }
    mbar_init(&bars->tab_full, 1);
    mbar_init(&bars->final_mma, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->rhw_full[t], 1);
      mbar_init(&bars->bias_done[t], 128);
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 128);
      mbar_init(&bars->o_full[t], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (q, v, table)
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmT);
      mbar_arrive_expect_tx(&bars->tab_full, L::kTabBytes);
      for (int c = 0; c < L::HC; ++c) {
        tma_load_2d(smem + L::OFF_TAB + c * L::kTabChunk, &tmT, &bars->tab_full, c * 16, 0);                // Th
        tma_load_2d(smem + L::OFF_TAB + c * L::kTabChunk + 32 * 32, &tmT, &bars->tab_full, c * 16, 2 * kSide - 1);  // Tw
      }
      int issued = 0;
      for (int ui = 0; ui < n_units; ++ui) {
        const int s = ui & 1;
        const int u = (int)(first + (long)ui * gridDim.x);
        if (ui >= kStages && !mbar_wait(&bars->stage_free[s], ((ui >> 1) - 1) & 1, abort_flag)) break;
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(&bars->q_full[s], L::kQBytes);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < L::HC; ++c)
            tma_load_3d(st + L::OFF_Q + t * L::kQTile + c * L::kQChunk, &tmQ, &bars->q_full[s], c * 16, 128 * t, u);
        mbar_arrive_expect_tx(&bars->v_full[s], L::kVBytes);
        for (int c = 0; c < L::HC; ++c)
          tma_load_3d(st + L::OFF_V + c * L::kVChunk, &tmV, &bars->v_full[s], c * 16, 0, u);
        issued = ui + 1;
      }
      if (*abort_flag) {
        for (int ui = issued > kStages ? issued - kStages : 0; ui < issued; ++ui) {
          mbar_drain(&bars->q_full[ui & 1], (ui >> 1) & 1);
          mbar_drain(&bars->v_full[ui & 1], (ui >> 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idRHW = idesc_f16(kBf16, 128, 64, false, false);
      constexpr uint32_t idS = idesc_f16(kBf16, 128, kNP, false, true);
      constexpr uint32_t idPV = idesc_f16(kBf16, 128, HD, false, true);
      const uint32_t sb = smem_u32(smem);
      auto descQ = [&](int s, int t, int c) {
        return smem_desc(sb + s * L::kStage + L::OFF_Q + t * L::kQTile + c * L::kQChunk, 16, 256, kLayoutSw32);
      };
      auto descTab = [&](int c) { return smem_desc(sb + L::OFF_TAB + c * L::kTabChunk, 16, 256, kLayoutSw32); };
      auto descK = [&](int s, int c) {
        return smem_desc(sb + s * L::kStage + L::OFF_K + c * 256, 128, L::kKSbo, kLayoutNone);
      };
      auto descV = [&](int s, int k) {
        return smem_desc(sb + s * L::kStage + L::OFF_V + k * 512, L::kVChunk, 256, kLayoutSw32);
      };
      bool okk = mbar_wait(&bars->tab_full, 0, abort_flag);
      for (int ui = 0; ui < n_units && okk; ++ui) {
        const int s = ui & 1;
        const uint32_t ph = (ui >> 1) & 1;
        okk = mbar_wait(&bars->q_full[s], ph, abort_flag);
        if (!okk) break;
        tc_fence_after();
        for (int t = 0; t < 2; ++t) {
          for (int c = 0; c < L::HC; ++c) mma_ss(tmem + 256 * t, descQ(s, t, c), descTab(c), idRHW, c > 0);
          mma_commit(&bars->rhw_full[t]);
        }
        okk = mbar_wait(&bars->k_full[s], ph, abort_flag);
        for (int t = 0; t < 2 && okk; ++t) {
          okk = mbar_wait(&bars->bias_done[t], ui & 1, abort_flag);
          if (!okk) break;
          tc_fence_after();
          for (int c = 0; c < L::HC; ++c) mma_ss(tmem + 256 * t, descQ(s, t, c), descK(s, c), idS, c > 0);
          mma_commit(&bars->s_full[t]);
        }
        if (okk) okk = mbar_wait(&bars->v_full[s], ph, abort_flag);
        for (int t = 0; t < 2 && okk; ++t) {
          okk = mbar_wait(&bars->p_full[t], ui & 1, abort_flag);
          if (!okk) break;
          tc_fence_after();
          for (int k = 0; k < kNP / 16; ++k)
            mma_ts(tmem + 256 * t + 128, tmem + 256 * t + 8 * k, descV(s, k), idPV, k > 0 ? 1u : 0u);
          mma_commit(&bars->o_full[t]);
        }
        if (okk) mma_commit(&bars->stage_free[s]);
      }
      mma_commit(&bars->final_mma);
      mbar_drain(&bars->final_mma, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------------ kt loaders (cp.async relayout)
    const int tl = threadIdx.x - 128;
    for (int s = 0; s < kStages; ++s) {  // padded keys 196..207 stay zero for the whole kernel
      uint8_t* kb = smem + s * L::kStage + L::OFF_K;
      for (int idx = tl; idx < HD * 3; idx += 128) {
        const int d = idx / 3, n = kN + 4 * (idx % 3);
        *reinterpret_cast<uint2*>(kb + k_off<HD>(n, d)) = make_uint2(0u, 0u);
      }
    }
    for (int ui = 0; ui < n_units; ++ui) {
      const int s = ui & 1;
      const long u = first + (long)ui * gridDim.x;
      if (ui >= kStages && !mbar_wait(&bars->stage_free[s], ((ui >> 1) - 1) & 1, abort_flag)) break;
      uint8_t* kb = smem + s * L::kStage + L::OFF_K;
      const T* src = kt + u * (long)HD * kN;
      for (int idx = tl; idx < HD * (kN / 4); idx += 128) {
        const int d = idx / (kN / 4), n = 4 * (idx % (kN / 4));
        cp_async_8(kb + k_off<HD>(n, d), src + d * kN + n);
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&bars->k_full[s]);
    }
    cp_async_wait_all();
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 8) >> 2;
    const int wq = warp & 3;
    const int rt = 128 * t + 32 * wq + lane;  // query row within the window
    const int i = rt / kSide, j = rt % kSide;
    const uint32_t tS = tmem + ((uint32_t)(32 * wq) << 16) + 256 * t;
    const uint32_t tO = tS + 128;
    const float c = scale * kLog2e;
    for (int ui = 0; ui < n_units; ++ui) {
      const long u = first + (long)ui * gridDim.x;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->rhw_full[t], ui & 1, abort_flag))) break;
      tc_fence_after();
      float rh[14], rw[14];
      {
        uint32_t a[32];
        tmem_ld32(tS, a);
        tmem_wait_ld();
        select14(a, i, rh);
        tmem_ld32(tS + 32, a);
        tmem_wait_ld();
        select14(a, j, rw);
      }
      tc_fence_before();
      mbar_arrive(&bars->bias_done[t]);
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[t], ui & 1, abort_flag))) break;
      tc_fence_after();
      float m = -INFINITY;
      m = chunk_max<0>(tS, c, rh, rw, m);
      m = chunk_max<1>(tS, c, rh, rw, m);
      m = chunk_max<2>(tS, c, rh, rw, m);
      m = chunk_max<3>(tS, c, rh, rw, m);
      m = chunk_max<4>(tS, c, rh, rw, m);
      m = chunk_max<5>(tS, c, rh, rw, m);
      m = tail_max(tS, c, rh, rw, m);
#pragma unroll
      for (int k = 0; k < 14; ++k) rw[k] -= m;
      float sum = 0.f;
      sum = chunk_exp<0, kBf16>(tS, c, rh, rw, sum);
      sum = chunk_exp<1, kBf16>(tS, c, rh, rw, sum);
      sum = chunk_exp<2, kBf16>(tS, c, rh, rw, sum);
      sum = chunk_exp<3, kBf16>(tS, c, rh, rw, sum);
      sum = chunk_exp<4, kBf16>(tS, c, rh, rw, sum);
      sum = chunk_exp<5, kBf16>(tS, c, rh, rw, sum);
      sum = tail_exp<kBf16>(tS, c, rh, rw, sum);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->o_full[t], ui & 1, abort_flag))) break;
      tc_fence_after();
      const float inv = 1.f / sum;
      T* orow = out + (u * kN + rt) * HD;
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
        uint32_t ov[16];
        tmem_ld16(tO + c0, ov);
        tmem_wait_ld();
        uint32_t pw[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          pw[e] = pack2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv, kBf16);
        if (rt < kN) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
          dst[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
          dst[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
        }
      }
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tcw
}  // namespace samrs
