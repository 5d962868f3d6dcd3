// relpos_tc.cuh - tcgen05 (sm_100a tensor-core) kernel of the rel-pos attention path for SAM's global
// layers (64x64 tokens, head_dim 64 or 80, f16/bf16 I/O, f32 accumulation and softmax).
//
// Math (src/kernels.rs:131-225 restated, src/sam1/encoder.rs:73-85):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+63] + q_r . Tw[j-kw+63],   out_r = sum_k softmax_k(x) v_k
// with r = 64 i + j and k = 64 kh + kw.
//
// One CTA = one head (bh) x 256 query rows (two 128-row tiles Q0, Q1 = grid rows I0..I0+3), looping
// over 32 key tiles of 128 keys (= grid rows kh = 2t, 2t+1). 12 warps:
//   warp 0      TMA producer: Q0, Q1 and the two table slices once, then K/V tiles through a 2-stage ring
//   warp 1      MMA issuer (one thread): prologue bias MMAs, then S_q = Q_q K^T and O_q += P_q V per tile
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax of Q0 (thread = query row = TMEM lane), warps 8-11 softmax of Q1
// Rel-pos bias, computed in-tile: the prologue MMAs give RW = Q Tw^T (128 cols) and RH = Q Th[I0..I0+79]^T
// (80 cols) in TMEM. Each thread keeps its 64 rw values (log2 units) in registers (a lane-dependent
// barrel shift selects the window j..j+63) and parks its 64 rh values in shared memory; a key tile then
// needs rw[kw] for every key and just two rh values (one per 64-key half).
// The softmax is online in the log2 domain with conditional rescaling (O is rescaled only when the row
// max grows by more than 8); P is written back as 16-bit into the S columns of TMEM and fed to the PV MMA
// as the A operand straight from TMEM. No score ever reaches HBM.
//
// TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 [256,256+HD), O1 [256+HD, 256+2HD); prologue:
// RW_q in S_q, RH_q at [256+80q, 256+80q+80).
// Shared memory (1 KB aligned): Q0 | Q1 | K ring | V ring | RH park (tables alias it in the prologue) | barriers.
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "relpos_tc_window.cuh"
#include "sm100.cuh"

namespace samrs {

enum class TcShape { kNone, kGlobal, kWindow };

namespace tcg {

constexpr int kThreads = 384;
// Registers: launched at 168 per thread; warpgroup 0 (producer, MMA, allocator) gives back to 56 and the
// two softmax warpgroups take 224: 128 x 56 + 256 x 224 = 64512 = 384 x 168.
constexpr uint32_t kRegsLow = 96, kRegsHigh = 200;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kThreads * 168, "register split exceeds the launch allotment");
constexpr int kBQ = 128, kBK = 128, kSide = 64, kN = 4096, kNT = kN / kBK, kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;  // log2 units

template <int HD>
struct Layout {
  static constexpr int HC = HD / 16;                  // 16-element (32 B) chunks of a row
  static constexpr int kChunkBytes = 128 * 32;        // one [128 rows x 32 B] SW32 chunk
  static constexpr int kQBytes = HC * kChunkBytes;    // a 128-row tile of q / v / table
  static constexpr int kKAtom = HD * 128;             // one [HD rows x 64 keys] SW128 box
  static constexpr int kKBytes = 2 * kKAtom;
  static constexpr int kVBytes = kQBytes;
  static constexpr int kRhBytes = 64 * 256 * 4;       // rh park: [kh][256 rows] f32
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * kQBytes;
  static constexpr int OFF_V = OFF_K + kStages * kKBytes;
  static constexpr int OFF_RH = OFF_V + kStages * kVBytes;
  static constexpr int OFF_TH = OFF_RH;               // prologue only (aliases the rh park)
  static constexpr int OFF_TW = OFF_RH + kQBytes;
  static constexpr int OFF_BAR = OFF_RH + kRhBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int kSmemBytes = OFF_BAR + kBarBytes + 1024;  // + alignment slack
  static_assert(2 * kQBytes <= kRhBytes, "tables must fit in the rh park");
  static_assert(kKAtom % 1024 == 0 && OFF_K % 1024 == 0 && OFF_V % 1024 == 0, "SW128 atoms need 1 KB alignment");
};

struct Bars {
  uint64_t q_full, pro_done, final_mma;
  uint64_t k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t bias_done[2], s_full[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort_flag;
};

// One stage of the lane-dependent shift: a[m] <- a[m + 2^B] where bit B of the lane is set.
template <int B, int LEN>
__device__ __forceinline__ void shift_stage(uint32_t (&a)[48], int lane) {
  const uint32_t take = (lane >> B) & 1;
#pragma unroll
  for (int m = 0; m < LEN; ++m) a[m] = sm100::select_u32(take, a[m + (1 << B)], a[m]);
}

// rw output block C of one softmax thread: rwc[kw] for kw = 16C..16C+15 (log2 units). tW addresses
// this lane's row at column jb = 32*(warp&1); the thread's window starts at jb + lane + 48 - 16C.
template <int C>
__device__ __forceinline__ void rw_block(uint32_t tW, int lane, float (&rwc)[64]) {
  using namespace sm100;
  uint32_t a[48];
#pragma unroll
  for (int blk = 0; blk < 3; ++blk) {
    uint32_t v[16];
    tmem_ld16(tW + 48 - 16 * C + 16 * blk, v);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; ++e) a[16 * blk + e] = v[e];
  }
  shift_stage<4, 31>(a, lane);
  shift_stage<3, 23>(a, lane);
  shift_stage<2, 19>(a, lane);
  shift_stage<1, 17>(a, lane);
  shift_stage<0, 16>(a, lane);
  // a[e] = RW[r][j + 48 - 16C + e] = rw[kw] with kw = 15 + 16C - e
#pragma unroll
  for (int e = 0; e < 16; ++e) rwc[16 * C + 15 - e] = __uint_as_float(a[e]) * kLog2e;
}

// rh_park[kh][prow] = RH[OFF + 63 - kh] (log2 units) for kh = 0..63.
template <int OFF>
__device__ __forceinline__ void park_rh(const float (&a)[96], float* rh_park, int prow) {
#pragma unroll
  for (int kh = 0; kh < 64; ++kh) rh_park[kh * 256 + prow] = a[OFF + 63 - kh] * kLog2e;
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_global(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                       T* __restrict__ out, float scale) {
  using L = Layout<HD>;
  using namespace sm100;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  float* rh_park = reinterpret_cast<float*>(smem + L::OFF_RH);
  volatile int* abort_flag = &bars->abort_flag;

  if (device_faulted()) return;  // an earlier CTA reported a fault: do no more work
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long bh = blockIdx.x / (kN / 256);
  const int ct = blockIdx.x % (kN / 256);
  const int row0 = ct * 256;  // first query row of the CTA
  const int I0 = ct * 4;      // its first grid row

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->pro_done, 1);
    mbar_init(&bars->final_mma, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&bars->bias_done[q], 128);
      mbar_init(&bars->s_full[q], 1);
      mbar_init(&bars->p_full[q], 128);
      mbar_init(&bars->o_done[q], 1);
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
  if (warp < 4) {
    regs_dec<kRegsLow>();
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmT);
      mbar_arrive_expect_tx(&bars->q_full, 4 * L::kQBytes);
      for (int q = 0; q < 2; ++q)
        for (int c = 0; c < L::HC; ++c)
          tma_load_2d(smem + L::OFF_Q + q * L::kQBytes + c * L::kChunkBytes, &tmQ, &bars->q_full, c * 16,
                      (int)(bh * kN + row0 + q * kBQ));
      for (int c = 0; c < L::HC; ++c) {
        tma_load_2d(smem + L::OFF_TH + c * L::kChunkBytes, &tmT, &bars->q_full, c * 16, I0);        // Th[I0..]
        tma_load_2d(smem + L::OFF_TW + c * L::kChunkBytes, &tmT, &bars->q_full, c * 16, 2 * kSide - 1);  // Tw
      }
      int issued = 0;
      for (int j = 0; j < kNT; ++j) {
        const int st = j % kStages;
        if (j >= kStages && !mbar_wait(&bars->kv_empty[st], ((j / kStages) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars->k_full[st], L::kKBytes);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(smem + L::OFF_K + st * L::kKBytes + a * L::kKAtom, &tmK, &bars->k_full[st], j * kBK + a * 64,
                      (int)(bh * HD));
        mbar_arrive_expect_tx(&bars->v_full[st], L::kVBytes);
        for (int c = 0; c < L::HC; ++c)
          tma_load_2d(smem + L::OFF_V + st * L::kVBytes + c * L::kChunkBytes, &tmV, &bars->v_full[st], c * 16,
                      (int)(bh * kN + j * kBK));
        issued = j + 1;
      }
      if (*abort_flag) {
        // drain this CTA's own copies still in flight before the CTA can exit
        for (int j = issued > kStages ? issued - kStages : 0; j < issued; ++j) {
          const int st = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          mbar_drain(&bars->k_full[st], ph);
          mbar_drain(&bars->v_full[st], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(kBf16, 128, 128, false, true);    // S = Q K^T, K MN-major
      constexpr uint32_t idRW = idesc_f16(kBf16, 128, 128, false, false);  // RW = Q Tw^T
      constexpr uint32_t idRH = idesc_f16(kBf16, 128, 80, false, false);   // RH = Q Th^T
      constexpr uint32_t idPV = idesc_f16(kBf16, 128, HD, false, true);    // O += P V, V MN-major
      const uint32_t sbase = smem_u32(smem);
      auto descQ = [&](int q, int c) {
        return smem_desc(sbase + L::OFF_Q + q * L::kQBytes + c * L::kChunkBytes, 16, 256, kLayoutSw32);
      };
      auto descTab = [&](int off, int c) { return smem_desc(sbase + off + c * L::kChunkBytes, 16, 256, kLayoutSw32); };
      auto descK = [&](int st, int c) {
        return smem_desc(sbase + L::OFF_K + st * L::kKBytes + c * 2048, L::kKAtom, 1024, kLayoutSw128);
      };
      auto descV = [&](int st, int s) {
        return smem_desc(sbase + L::OFF_V + st * L::kVBytes + s * 512, L::kChunkBytes, 256, kLayoutSw32);
      };
      bool okk = mbar_wait(&bars->q_full, 0, abort_flag);
      if (okk) {
        tc_fence_after();
        for (int q = 0; q < 2; ++q) {
          for (int c = 0; c < L::HC; ++c) mma_ss(tmem + q * 128, descQ(q, c), descTab(L::OFF_TW, c), idRW, c > 0);
          for (int c = 0; c < L::HC; ++c)
            mma_ss(tmem + 256 + q * 80, descQ(q, c), descTab(L::OFF_TH, c), idRH, c > 0);
        }
        mma_commit(&bars->pro_done);
        okk = mbar_wait(&bars->bias_done[0], 0, abort_flag) && mbar_wait(&bars->bias_done[1], 0, abort_flag) &&
              mbar_wait(&bars->k_full[0], 0, abort_flag);
      }
      if (okk) {
        tc_fence_after();
        for (int q = 0; q < 2; ++q) {
          for (int c = 0; c < L::HC; ++c) mma_ss(tmem + q * 128, descQ(q, c), descK(0, c), idS, c > 0);
          mma_commit(&bars->s_full[q]);
        }
        for (int j = 0; j < kNT && okk; ++j) {
          const int st = j % kStages;
          const uint32_t ph = (j / kStages) & 1;
          for (int q = 0; q < 2 && okk; ++q) {
            okk = mbar_wait(&bars->p_full[q], j & 1, abort_flag);
            if (okk && q == 0) okk = mbar_wait(&bars->v_full[st], ph, abort_flag);
            if (!okk) break;
            tc_fence_after();
            for (int s = 0; s < kBK / 16; ++s)
              mma_ts(tmem + 256 + q * HD, tmem + q * 128 + s * 8, descV(st, s), idPV, (j > 0 || s > 0) ? 1u : 0u);
            if (j == kNT - 1) mma_commit(&bars->o_done[q]);
            if (j + 1 < kNT) {
              const int st1 = (j + 1) % kStages;
              if (q == 0) {
                okk = mbar_wait(&bars->k_full[st1], ((j + 1) / kStages) & 1, abort_flag);
                if (!okk) break;
                tc_fence_after();
              }
              for (int c = 0; c < L::HC; ++c) mma_ss(tmem + q * 128, descQ(q, c), descK(st1, c), idS, c > 0);
              mma_commit(&bars->s_full[q]);
            }
          }
          if (okk) mma_commit(&bars->kv_empty[st]);
        }
      }
      // every MMA issued by this thread has completed before the CTA tears down TMEM
      mma_commit(&bars->final_mma);
      mbar_drain(&bars->final_mma, 0);
    }
  }
  } else {
    regs_inc<kRegsHigh>();
  {
    // ------------------------------------------------------------------ softmax warpgroups
    const int q = (warp - 4) >> 2;        // query tile
    const int wq = warp & 3;              // TMEM lane quarter
    const int r = wq * 32 + lane;         // row within the tile
    const int prow = q * 128 + r;         // row within the CTA (rh park column)
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + q * 128;
    const uint32_t tO = tmem + lane_off + 256 + q * HD;
    const uint32_t tRH = tmem + lane_off + 256 + q * 80;
    const float c_log2 = scale * kLog2e;
    float rwc[64];
    bool okk = __all_sync(0xffffffffu, mbar_wait(&bars->pro_done, 0, abort_flag));
    if (okk) {
      tc_fence_after();
      // rw: this row's window RW[r][j .. j+63] reversed, j = 32*(wq&1) + lane. Output block c
      // (kw = 16c..16c+15) reads columns jb + lane + 48 - 16c + e' (e' = 0..15): load the 48 columns
      // from jb + 48 - 16c and shift them down by `lane` with a 5-stage select network.
      {
        const uint32_t tW = tS + 32 * (wq & 1);
        rw_block<0>(tW, lane, rwc);
        rw_block<1>(tW, lane, rwc);
        rw_block<2>(tW, lane, rwc);
        rw_block<3>(tW, lane, rwc);
      }
      // rh: RH_q[r][c] = q_r . Th[I0 + c] (both tiles share the Th slice from grid row I0). Row r of tile
      // q sits on grid row i = I0 + 2q + r/64, so rh[kh] = q_r . Th[i - kh + 63] = RH_q[r][off + 63 - kh]
      // with off = 2q + r/64 (warp-uniform).
      {
        float a[96];
#pragma unroll
        for (int blk = 0; blk < 3; ++blk) {
          uint32_t v[32];
          tmem_ld32(tRH + 32 * blk, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) a[32 * blk + e] = __uint_as_float(v[e]);
        }
        switch (2 * q + (wq >> 1)) {
          case 0:
            park_rh<0>(a, rh_park, prow);
            break;
          case 1:
            park_rh<1>(a, rh_park, prow);
            break;
          case 2:
            park_rh<2>(a, rh_park, prow);
            break;
          default:
            park_rh<3>(a, rh_park, prow);
            break;
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->bias_done[q]);
    }
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < kNT && okk; ++j) {
      okk = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[q], j & 1, abort_flag));
      if (!okk) break;
      tc_fence_after();
      const float rh0 = rh_park[(2 * j) * 256 + prow];
      const float rh1 = rh_park[(2 * j + 1) * 256 + prow];
      // pass 1: row max of S*c + rw (+ rh per 64-key half), 32 columns at a time
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t sv[32];
        tmem_ld32(tS + 32 * ch, sv);
        tmem_wait_ld();
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          m0 = fmaxf(m0, fmaf(__uint_as_float(sv[e]), c_log2, rwc[(ch & 1) * 32 + e]));
          m1 = fmaxf(m1, fmaf(__uint_as_float(sv[e + 1]), c_log2, rwc[(ch & 1) * 32 + e + 1]));
        }
        if (ch < 2)
          mx0 = fmaxf(mx0, fmaxf(m0, m1));
        else
          mx1 = fmaxf(mx1, fmaxf(m0, m1));
      }
      const float m_tile = fmaxf(mx0 + rh0, mx1 + rh1);
      const float m_new = fmaxf(m_run, m_tile);
      const bool need = (j == 0) || (m_new > m_run + kRescaleThreshold);
      float alpha = 1.f;
      if (need) {
        alpha = ex2(m_run - m_new);
        m_run = m_new;
      }
      // pass 2: p = 2^(S*c + rw + rh - m), row sum, 16-bit P written over the consumed S columns
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const float bias = (ch < 2 ? rh0 : rh1) - m_run;
        uint32_t sv[32];
        tmem_ld32(tS + 32 * ch, sv);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(sv[e]), c_log2, rwc[(ch & 1) * 32 + e] + bias));
          const float p1 = ex2(fmaf(__uint_as_float(sv[e + 1]), c_log2, rwc[(ch & 1) * 32 + e + 1] + bias));
          sum0 += p0;
          sum1 += p1;
          pk[e >> 1] = pack2(p0, p1, kBf16);
        }
        tmem_st16(tS + 16 * ch, pk);
      }
      l_run = l_run * alpha + (sum0 + sum1);
      // O rescale: PV_q(j-1) has completed (it was issued before S_q(j), whose commit we waited on).
      if (__any_sync(0xffffffffu, need && j > 0)) {
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 16) {
          uint32_t ov[16];
          tmem_ld16(tO + c0, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st16(tO + c0, ov);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[q]);
    }
    // epilogue: O / l -> out
    if (okk) okk = __all_sync(0xffffffffu, mbar_wait(&bars->o_done[q], 0, abort_flag));
    if (okk) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      T* orow = out + (bh * kN + row0 + q * kBQ + r) * HD;
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
        uint32_t ov[16];
        tmem_ld16(tO + c0, ov);
        tmem_wait_ld();
        uint32_t pw[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
          pw[e] = pack2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv, kBf16);
        uint4* dst = reinterpret_cast<uint4*>(orow + c0);
        dst[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        dst[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
      }
    }
  }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] 16-bit tensor, box [box_rows, box_cols].
inline int make_map(CUtensorMap* map, bool bf16, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                    uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

// 3-D map over a row-major [d2, d1, d0] 16-bit tensor, box [1, box1, box0].
inline int make_map3(CUtensorMap* map, bool bf16, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                     uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return 2;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

}  // namespace tcg

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline TcShape tc_select(int h, int w, int hd, const void* q, const void* kt, const void* v, const void* table,
                         const void* out) {
  if (!(aligned16(q) && aligned16(kt) && aligned16(v) && aligned16(table) && aligned16(out))) return TcShape::kNone;
  if (h == 64 && w == 64 && (hd == 64 || hd == 80)) return TcShape::kGlobal;
  if (h == 14 && w == 14 && (hd == 64 || hd == 80)) return TcShape::kWindow;
  return TcShape::kNone;
}

template <typename T, int HD>
int tc_launch_global(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                     float scale, cudaStream_t st) {
  using namespace tcg;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (bh * kN > 0x7fffffffLL || bh * (kN / 256) > 0x7fffffffLL) return 4;
  CUtensorMap mq, mk, mv, mt;
  int rc = make_map(&mq, bf16, q, HD, (uint64_t)bh * kN, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&mk, bf16, kt, kN, (uint64_t)bh * HD, 64, HD, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&mv, bf16, v, HD, (uint64_t)bh * kN, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&mt, bf16, table, HD, 4 * kSide - 2, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  auto kern = relpos_attn_global<T, HD>;
  const int smem = Layout<HD>::kSmemBytes;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 5;
  kern<<<(unsigned)(bh * (kN / 256)), kThreads, smem, st>>>(mq, mk, mv, mt, static_cast<T*>(out), scale);
  return 0;
}

template <typename T, int HD>
int tc_launch_window(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                     float scale, cudaStream_t st, int num_sms) {
  using namespace tcg;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (bh > 0x7fffffffLL) return 4;
  CUtensorMap mq, mv;
  int rc = make_map3(&mq, bf16, q, HD, tcw::kN, (uint64_t)bh, 16, tcw::Layout<HD>::kQRows, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map3(&mv, bf16, v, HD, tcw::kN, (uint64_t)bh, 16, tcw::kNP, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  auto kern = tcw::relpos_attn_window<T, HD>;
  const int smem = tcw::Layout<HD>::kSmemBytes;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 5;
  const int grid = (int)(bh < num_sms ? bh : num_sms);
  kern<<<grid, tcw::kThreads, smem, st>>>(mq, mv, static_cast<const T*>(table), static_cast<const T*>(kt),
                                         static_cast<T*>(out), (long)bh, scale);
  return 0;
}

template <typename T>
int tc_launch(TcShape shape, const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
              int h, int w, int hd, float scale, cudaStream_t st, int num_sms) {
  (void)h;
  (void)w;
  if (shape == TcShape::kGlobal)
    return hd == 80 ? tc_launch_global<T, 80>(q, kt, v, table, out, bh, scale, st)
                    : tc_launch_global<T, 64>(q, kt, v, table, out, bh, scale, st);
  if (shape == TcShape::kWindow)
    return hd == 80 ? tc_launch_window<T, 80>(q, kt, v, table, out, bh, scale, st, num_sms)
                    : tc_launch_window<T, 64>(q, kt, v, table, out, bh, scale, st, num_sms);
  return 1;
}

inline const char* tc_error_string(int rc) {
  switch (rc) {
    case 1:
      return "no tensor-core kernel for this shape";
    case 2:
      return "cuTensorMapEncodeTiled is not available from the driver";
    case 3:
      return "cuTensorMapEncodeTiled rejected a tensor map";
    case 4:
      return "batch too large for 32-bit TMA coordinates";
    case 5:
      return "cannot set the kernel's shared memory size";
    default:
      return "unknown tensor-core launch error";
  }
}

}  // namespace samrs
