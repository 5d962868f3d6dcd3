// relpos_tc_global.cuh - tcgen05 (sm_100a tensor-core) kernel for SAM's global layers (64x64 tokens,
// head_dim 64 or 80, f16/bf16 I/O, f32 accumulation and softmax).
//
// Math (src/kernels.rs:131-225 restated, src/sam1/encoder.rs:73-85):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+63] + q_r . Tw[j-kw+63],   out_r = sum_k softmax_k(x) v_k
// with r = 64 i + j and k = 64 kh + kw.
//
// One CTA = one head (bh) x 256 query rows (two 128-row tiles Q0, Q1 = grid rows I0..I0+3), looping
// over 32 key tiles of 128 keys (grid rows kh = 2t, 2t+1); both query tiles share every K/V tile.
// 20 warps:
//   warp 0       TMA producer: Q0, Q1 and the two table slices once, then K and V tiles (2-stage rings)
//   warp 1       MMA issuer (the warp runs the loop, lane 0 issues): prologue bias MMAs, then per tile and
//                query tile, in order, O_q += P_q(t) [V(t) | 1] and S_q(t+1) = Q_q K(t+1)^T. In-order issue
//                lets S_q(t+1) overwrite P_q(t) (both live in the S_q columns) without a round trip through
//                a barrier.
//   warp 2       TMEM allocator (512 columns)
//   warps 4-11   softmax of Q0, warps 12-19 softmax of Q1: two warps per TMEM lane quarter, one per
//                16-lane half. With the 16x256b access shape four threads share a row pair (rows r and
//                r+8 of the half), each holding key pairs 8m + 2(t%4), +1: 64 scores per thread and
//                tile, row maxima combined with two shuffles. Four softmax warps per SM sub-partition keep
//                the exp unit busy while the other query tile waits on its MMAs.
//
// Rel-pos bias, computed in-tile: the prologue MMAs give RW = Q Tw^T (128 cols) and RH = Q Th[I0..I0+79]^T
// (80 cols) in TMEM. Each query row owns 64 words of shared memory (the park), used twice: first the two
// warps of a lane quarter write each row's window RW[r][j .. j+63] there reversed (= rw[kw], log2 units)
// and every thread reads the 16 values of its key pairs for its two rows into registers; then the row's
// 64 rh values are parked there for the key tiles (two per tile and row, one per 64-key half).
// The softmax is online in the log2 domain; P is written back as 16-bit pairs into the S columns of TMEM
// and fed to the P.V MMA as the A operand straight from TMEM. The V stages carry a block of ones, so the
// MMA also accumulates the row sums of P as rounded. Exact mode (f16): two passes per tile, O rescaled only
// when the row max grows by more than 8. Speculative mode (bf16): one pass per tile after the first,
// against a predicted max; a CTA that overflows leaves a NaN marker and is recomputed by the fixup mode
// (exact, marked CTAs only) launched right after. No score ever reaches HBM.
//
// TMEM columns: S0/P0 [0,128), S1/P1 [128,256), O0 and its row sums [256, 256+HD+16), O1 after it;
// prologue: RW_q in S_q, RH_q at [256+80q, 256+80q+80).
// Shared memory (1 KB aligned): Q0 | Q1 | K ring | V ring (each stage: v, then ones) | RH park (tables
// alias it in the prologue) | barriers.
#pragma once
#include <cuda.h>

#include <stddef.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tcg {

constexpr int kThreads = 640;
constexpr int kLaunchRegs = 96;  // 65536 / 640 rounded down to the allocation granularity
// Registers: warpgroup 0 (producer, issuer, allocator) gives back to 64 and the four softmax warpgroups
// take 104: 128 x 64 + 512 x 104 = 61440 = 640 x 96.
constexpr uint32_t kRegsLow = 64, kRegsHigh = 104;
static_assert(128 * kRegsLow + 512 * kRegsHigh <= kThreads * kLaunchRegs, "register split exceeds the launch allotment");
constexpr int kBQ = 128, kBK = 128, kSide = 64, kN = 4096, kNT = kN / kBK, kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.f;  // log2 units
// bf16: single-pass tiles against one reference per row fixed at tile 0 (see the softmax). The reference
// is capped kSpecCap above the row's max over tile 0 (P of the dominant keys >= 2^-96, well inside bf16's
// normal range), and a CTA with a row whose largest P exceeded 2^kSpecLimit (seen as a row sum of 2^112 or
// more) or with a non-finite output is recomputed exactly by a second launch.
constexpr float kSpecCap = 96.f, kSpecLimit = 112.f;
constexpr float kSpecSumLimit = 0x1p112f;  // 2^kSpecLimit
// Kernel modes: the exact two-pass softmax (f16); the speculative pass (bf16), which marks a CTA that needs
// the exact pass by a NaN in the first element of its output block; the exact pass of the marked blocks
// only (bf16, launched right after the speculative one with at most one CTA per SM, each scanning its share
// of the markers).
constexpr int kModeExact = 0, kModeSpec = 1, kModeFixup = 2;

template <int HD>
struct Layout {
  static constexpr int HC = HD / 16;                  // 16-element (32 B) chunks of a row
  static constexpr int kChunkBytes = 128 * 32;        // one [128 rows x 32 B] SW32 chunk
  static constexpr int kQBytes = HC * kChunkBytes;    // a 128-row tile of q / v / table
  static constexpr int kKAtom = HD * 128;             // one [HD rows x 64 keys] SW128 box
  static constexpr int kKBytes = 2 * kKAtom;
  static constexpr int kVBytes = kQBytes;             // bytes of v loaded per stage
  // A V stage holds the HC chunks of v and then a chunk of ones: the P.V MMA runs with N = HD + 16, so
  // that O's last 16 columns accumulate the row sums of the 16-bit P exactly as the product uses them.
  static constexpr int kVStage = (HC + 1) * kChunkBytes;
  static constexpr int kOCols = HD + 16;
  static constexpr int kRhBytes = 256 * 64 * 4;       // park: [256 rows][64] f32 (rw staging, then rh)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * kQBytes;
  static constexpr int OFF_V = OFF_K + kStages * kKBytes;
  static constexpr int OFF_RH = OFF_V + kStages * kVStage;
  static constexpr int OFF_TH = OFF_RH;               // prologue only (aliases the rh park)
  static constexpr int OFF_TW = OFF_RH + kQBytes;
  static constexpr int OFF_BAR = OFF_RH + kRhBytes;
  static constexpr int kBarBytes = 256;
  static constexpr int OFF_RHMAX = OFF_BAR + kBarBytes;  // [2][256 rows] f32: the largest rh of each row
  static constexpr int kSmemBytes = OFF_RHMAX + 2 * 256 * 4 + 1024;  // + alignment slack
  static_assert(2 * kQBytes <= kRhBytes, "tables must fit in the rh park");
  static_assert(kKAtom % 1024 == 0 && OFF_K % 1024 == 0 && OFF_V % 1024 == 0, "SW128 atoms need 1 KB alignment");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Bars {
  uint64_t q_full, pro_done, final_mma;
  uint64_t k_full[kStages], v_full[kStages], k_empty[kStages], v_empty[kStages];
  uint64_t bias_done[2], s_full[2], p_full[2], o_done[2];
  uint64_t epi_done;
  uint64_t p_half[2];  // P of the first 64 keys written (one arrival per softmax warp)
  uint64_t stg[8];     // per lane quarter (4q + wq), one arrival per warp: rw staged (phase 0), read (1)
  uint32_t tmem_base;
  int abort_flag;
  int rerun;  // speculative pass: a softmax thread asks for the exact pass
};
static_assert(sizeof(Bars) <= 256, "barrier block");

// rw staging, one lane per query row (32x32b): row r = 32wq + lane of the quarter has grid column
// j = jb + lane (jb = 32(wq & 1)), and rw[kw] = RW[r][j + 63 - kw]. The warp of 16-lane half hh loads the
// window columns jb + 48hh .. jb + 48hh + 47 and writes each value whose kw lies in 0..63 to
// row[kw ^ sw] (sw = 8 (r & 3): the 16x256b readers of eight consecutive rows then hit distinct banks).
__device__ __forceinline__ void stage_rw(uint32_t tW, int lane, int hh, float* row, int sw) {
  using namespace sm100;
  const int c0 = 48 * hh;
  uint32_t v[32], u[16];
  tmem_ld32(tW + c0, v);
  tmem_ld16(tW + c0 + 32, u);
  tmem_wait_ld_regs(v);
  tmem_wait_ld_regs(u);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int kw = lane + 63 - (c0 + i);
    if (kw >= 0 && kw < 64) row[kw ^ sw] = __uint_as_float(v[i]) * kLog2e;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int kw = lane + 63 - (c0 + 32 + i);
    if (kw >= 0 && kw < 64) row[kw ^ sw] = __uint_as_float(u[i]) * kLog2e;
  }
}

// rh park of one row (32x32b, lane = row): row[kh ^ rl] = RH[OFF + 63 - kh] (log2 units) for the kh
// whose column OFF + 63 - kh lies in COL0 .. COL0 + N - 1 (held in v); mx tracks their maximum. rl = the
// row's low five bits, so the per-tile reads of eight consecutive rows hit distinct banks.
template <int OFF, int COL0, int N>
__device__ __forceinline__ void park_rh(const uint32_t* v, float* row, int rl, float& mx) {
#pragma unroll
  for (int cc = 0; cc < N; ++cc) {
    const int kh = OFF + 63 - (COL0 + cc);
    if (kh >= 0 && kh < 64) {
      const float x = __uint_as_float(v[cc]) * kLog2e;
      row[kh ^ rl] = x;
      mx = fmaxf(mx, x);
    }
  }
}
// The 64 rh of the row, split between the two warps of the quarter (hh 0: columns 0..31, hh 1: 32..79,
// of which only OFF + 63 and below hold a kh); the warp's partial maximum goes to rhmax[hh][prow].
template <int OFF>
__device__ __forceinline__ void park_rh_half(uint32_t tRH, int hh, float* row, int rl, float* rhmax, int prow) {
  using namespace sm100;
  float mx = -INFINITY;
  if (hh == 0) {
    uint32_t v[32];
    tmem_ld32(tRH, v);
    tmem_wait_ld_regs(v);
    park_rh<OFF, 0, 32>(v, row, rl, mx);
  } else {
    uint32_t v[32];
    tmem_ld32(tRH + 32, v);
    tmem_wait_ld_regs(v);
    park_rh<OFF, 32, 32>(v, row, rl, mx);
    uint32_t u[16];
    tmem_ld16(tRH + 64, u);
    tmem_wait_ld_regs(u);
    park_rh<OFF, 64, 16>(u, row, rl, mx);
  }
  rhmax[hh * 256 + prow] = mx;
}

// Key block g = 0..15 of a tile holds keys 8g..8g+7 (64-key half g/8, rw index g%8); this thread's keys
// in it are the pair 8g + 2c, +1 for rows A and B. A chunk = blocks G0, G0+1, loaded with 16x256b.x2:
// v[4i], v[4i+1] row A and v[4i+2], v[4i+3] row B of block G0+i.

// Pass 1: running maxima of S*c + rw for rows A and B.
template <int G0>
__device__ __forceinline__ void chunk_max(const uint32_t (&v)[8], float2 c2, const float2 (&rwA)[8],
                                          const float2 (&rwB)[8], float& mA, float& mB) {
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int m = (G0 + i) & 7;
    const float2 xa = sm100::fma2(make_float2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), c2, rwA[m]);
    const float2 xb =
        sm100::fma2(make_float2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), c2, rwB[m]);
    mA = sm100::max3(mA, xa.x, xa.y);
    mB = sm100::max3(mB, xb.x, xb.y);
  }
}

// Pass 2: p = 2^(S*c + rw + (rh - m)) for both rows as 16-bit pairs in the 16x128b store order (pw[2i]
// row A, pw[2i+1] row B: P column 4(G0+i) + c = keys 8(G0+i) + 2c, +1). Staged (exponents, then the ex2,
// then packing) so the ex2 issue back to back. The row sums come from the P.V MMA (ones block of V).
template <int G0, bool BF16>
__device__ __forceinline__ void chunk_exp(const uint32_t (&v)[8], float2 c2, const float2 (&rwA)[8],
                                          const float2 (&rwB)[8], float2 bA, float2 bB, uint32_t (&pw)[4]) {
  float x[8];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int m = (G0 + i) & 7;
    const float2 xa = sm100::fma2(make_float2(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), c2,
                                  sm100::add2(rwA[m], bA));
    const float2 xb = sm100::fma2(make_float2(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])), c2,
                                  sm100::add2(rwB[m], bB));
    x[4 * i] = xa.x;
    x[4 * i + 1] = xa.y;
    x[4 * i + 2] = xb.x;
    x[4 * i + 3] = xb.y;
  }
  // all on the exp unit (with the single pass it has room: moving a pair in four to the FMA pipe's
  // polynomial measured slower)
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = sm100::ex2(x[i]);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    pw[2 * i] = sm100::pack2(x[4 * i], x[4 * i + 1], BF16);
    pw[2 * i + 1] = sm100::pack2(x[4 * i + 2], x[4 * i + 3], BF16);
  }
}

template <typename T, int HD, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_global(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                       T* __restrict__ out, float scale, unsigned long long* recompute_slot, long n_blocks) {
  using L = Layout<HD>;
  using namespace sm100;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  static_assert(MODE == kModeExact || kBf16, "the speculative pass and its fixup are bf16 only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  float* rh_park = reinterpret_cast<float*>(smem + L::OFF_RH);
  float* rhmax_park = reinterpret_cast<float*>(smem + L::OFF_RHMAX);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // One output block (one head x 256 query rows): the speculative and exact launches run one per CTA, the
  // fixup launch runs the marked ones of its share (below).
  auto run_block = [&](const long blk) {
  const long bh = blk / (kN / 256);
  const int ct = (int)(blk % (kN / 256));
  const int row0 = ct * 256;  // first query row of the CTA
  const int I0 = ct * 4;      // its first grid row
  T* const marker = out + (bh * kN + row0) * HD;  // first element of the CTA's output block
  // The whole CTA leaves here or none of it does (thread 0 decides; the barriers, TMEM and the warp roles
  // below need every warp): after an earlier CTA reported a fault.
  if (__syncthreads_or(threadIdx.x == 0 && device_faulted())) return;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->pro_done, 1);
    mbar_init(&bars->final_mma, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int q = 0; q < 2; ++q) {
      mbar_init(&bars->bias_done[q], 8);  // one arrival per softmax warp of the query tile
      mbar_init(&bars->s_full[q], 1);
      mbar_init(&bars->p_full[q], 8);
      mbar_init(&bars->o_done[q], 1);
      mbar_init(&bars->p_half[q], 8);
    }
    mbar_init(&bars->epi_done, 16);  // one arrival per softmax warp
    for (int i = 0; i < 8; ++i) mbar_init(&bars->stg[i], 2);
    bars->abort_flag = 0;
    bars->rerun = 0;
    fence_mbar_init();
    // Q0, Q1 and the two table slices, issued before the TMEM allocation and the CTA barrier (thread 0 is
    // the producer's lane 0)
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    mbar_arrive_expect_tx(&bars->q_full, 4 * L::kQBytes);
    for (int q = 0; q < 2; ++q)
      for (int c = 0; c < L::HC; ++c)
        tma_load_2d(smem + L::OFF_Q + q * L::kQBytes + c * L::kChunkBytes, &tmQ, &bars->q_full, c * 16,
                    (int)(bh * kN + row0 + q * kBQ));
    for (int c = 0; c < L::HC; ++c) {
      tma_load_2d(smem + L::OFF_TH + c * L::kChunkBytes, &tmT, &bars->q_full, c * 16, I0);             // Th[I0..]
      tma_load_2d(smem + L::OFF_TW + c * L::kChunkBytes, &tmT, &bars->q_full, c * 16, 2 * kSide - 1);  // Tw
    }
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, 512);
    // the fixup launch allocates again for its CTA's next block, so it keeps the permit
    if constexpr (MODE != kModeFixup) tmem_relinquish();
  }
  {
    // the ones block of every V stage (the TMA loads never write it); read by the MMA (async proxy)
    const uint32_t one2 = kBf16 ? 0x3F803F80u : 0x3C003C00u;
    for (int idx = threadIdx.x; idx < kStages * L::kChunkBytes / 16; idx += kThreads) {
      const int st = idx / (L::kChunkBytes / 16), o = idx % (L::kChunkBytes / 16);
      reinterpret_cast<uint4*>(smem + L::OFF_V + st * L::kVStage + L::HC * L::kChunkBytes)[o] =
          make_uint4(one2, one2, one2, one2);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  if (warp < 4) {
    // (the fixup launch runs several blocks per CTA and keeps the launch's even split: its blocks are rare)
    if constexpr (MODE != kModeFixup) regs_dec<kRegsLow>();
    if (warp == 0) {
      // ---------------------------------------------------------------- TMA producer
      // (Q and the tables went out with the barrier set-up) K and V of every key tile
      int issued_k = 0, issued_v = 0;
      if (lane == 0) {
        // test hook: CTA 0 never loads this key tile (-1: none), so the MMA issuer's wait for it runs out
        const int withhold = blk == 0 ? *reinterpret_cast<volatile int*>(&g_withhold_key_tile) : -1;
        for (int j = 0; j < kNT; ++j) {
          const int jj = j, st = jj % kStages;
          const uint32_t prev = ((jj / kStages) - 1) & 1;
          if (jj >= kStages && !mbar_wait(&bars->k_empty[st], prev, abort_flag)) break;
          if (j != withhold) {
            mbar_arrive_expect_tx(&bars->k_full[st], L::kKBytes);
            for (int a = 0; a < 2; ++a)
              tma_load_2d(smem + L::OFF_K + st * L::kKBytes + a * L::kKAtom, &tmK, &bars->k_full[st],
                          j * kBK + a * 64, (int)(bh * HD));
          }
          issued_k = jj + 1;
          if (jj >= kStages && !mbar_wait(&bars->v_empty[st], prev, abort_flag)) break;
          mbar_arrive_expect_tx(&bars->v_full[st], L::kVBytes);
          for (int c = 0; c < L::HC; ++c)
            tma_load_2d(smem + L::OFF_V + st * L::kVStage + c * L::kChunkBytes, &tmV, &bars->v_full[st], c * 16,
                        (int)(bh * kN + j * kBK));
          issued_v = jj + 1;
        }
      }
      if (lane == 0 && *abort_flag) {
        // drain this CTA's own copies still in flight before the CTA can exit
        for (int jj = issued_k > kStages ? issued_k - kStages : 0; jj < issued_k; ++jj)
          mbar_drain(&bars->k_full[jj % kStages], (jj / kStages) & 1);
        for (int jj = issued_v > kStages ? issued_v - kStages : 0; jj < issued_v; ++jj)
          mbar_drain(&bars->v_full[jj % kStages], (jj / kStages) & 1);
      }
    } else if (warp == 1) {
      // ---------------------------------------------------------------- MMA issuer
      // The whole warp runs the issue loop (waits, descriptors); lane 0, elected inside each MMA and commit,
      // issues them.
      constexpr uint32_t idS = idesc_f16(kBf16, 128, 128, false, true);    // S = Q K^T, K MN-major
      constexpr uint32_t idRW = idesc_f16(kBf16, 128, 128, false, false);  // RW = Q Tw^T
      constexpr uint32_t idRH = idesc_f16(kBf16, 128, 80, false, false);   // RH = Q Th^T
      constexpr uint32_t idPV = idesc_f16(kBf16, 128, L::kOCols, false, true);  // O += P [V | 1], MN-major
      const uint32_t sb = smem_u32(smem);
      const uint64_t dQ = smem_desc(sb + L::OFF_Q, 16, 256, kLayoutSw32);
      const uint64_t dTh = smem_desc(sb + L::OFF_TH, 16, 256, kLayoutSw32);
      const uint64_t dTw = smem_desc(sb + L::OFF_TW, 16, 256, kLayoutSw32);
      const uint64_t dK = smem_desc(sb + L::OFF_K, L::kKAtom, 1024, kLayoutSw128);
      const uint64_t dV = smem_desc(sb + L::OFF_V, L::kChunkBytes, 256, kLayoutSw32);
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      // S_q from K stage st into the S_q columns
      auto issue_s = [&](int q, int st) {
        const uint64_t dKs = desc_add(dK, st * L::kKBytes);
#pragma unroll
        for (int c = 0; c < L::HC; ++c)
          mma_ss_w(tmem + q * 128, desc_add(dQ, q * L::kQBytes + c * L::kChunkBytes), desc_add(dKs, c * 2048), idS,
                   c > 0);
      };
      bool okk = wait(&bars->q_full, 0);
      if (okk) {
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 2; ++q) {
#pragma unroll
          for (int c = 0; c < L::HC; ++c)
            mma_ss_w(tmem + q * 128, desc_add(dQ, q * L::kQBytes + c * L::kChunkBytes),
                     desc_add(dTw, c * L::kChunkBytes), idRW, c > 0);
#pragma unroll
          for (int c = 0; c < L::HC; ++c)
            mma_ss_w(tmem + 256 + q * 80, desc_add(dQ, q * L::kQBytes + c * L::kChunkBytes),
                     desc_add(dTh, c * L::kChunkBytes), idRH, c > 0);
        }
        mma_commit_w(&bars->pro_done);
        okk = wait(&bars->k_full[0], 0);
      }
      {
        // S_q(0) overwrites RW_q: once query tile q's warps have read it (their bias_done)
        for (int q = 0; q < 2 && okk; ++q) {
          okk = wait(&bars->bias_done[q], 0);
          if (!okk) break;
          tc_fence_after();
          issue_s(q, 0);
          mma_commit_w(&bars->s_full[q]);
        }
        if (okk) mma_commit_w(&bars->k_empty[0]);
        for (int j = 0; j < kNT && okk; ++j) {
          const int st = j % kStages, st1 = (j + 1) % kStages;
          const uint64_t dVs = desc_add(dV, st * L::kVStage);
          const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            // the operands of this tile and of the next S (loaded long before; checked while the softmax
            // still runs), then the softmax's P: PV_q(j) and S_q(j+1) issue back to back
            if (q == 0) okk = wait(&bars->v_full[st], (j / kStages) & 1);
            if (okk && q == 0 && j + 1 < kNT) okk = wait(&bars->k_full[st1], ((j + 1) / kStages) & 1);
            int s0 = 0;
            {
              // the first half of P.V as soon as the softmax has written P of keys 0..63
              if (okk) okk = wait(&bars->p_half[q], j & 1);
              if (!okk) break;
              tc_fence_after();
#pragma unroll
              for (int s = 0; s < kBK / 32; ++s)
                mma_ts_w(tmem + 256 + q * L::kOCols, tmem + q * 128 + s * 8, desc_add(dVs, s * 512), idPV,
                         s > 0 ? 1u : acc0);
              s0 = kBK / 32;
            }
            if (okk) okk = wait(&bars->p_full[q], j & 1);
            if (!okk) break;
            tc_fence_after();
#pragma unroll
            for (int s = 0; s < kBK / 16; ++s)
              if (s >= s0)
                mma_ts_w(tmem + 256 + q * L::kOCols, tmem + q * 128 + s * 8, desc_add(dVs, s * 512), idPV,
                         s > 0 ? 1u : acc0);
            if (j + 1 < kNT) {
              // issued after PV_q(j), which reads P_q(j) from the same columns: in-order execution
              issue_s(q, st1);
              mma_commit_w(&bars->s_full[q]);
            } else {
              mma_commit_w(&bars->o_done[q]);
            }
          }
          if (!okk) break;
          mma_commit_w(&bars->v_empty[st]);
          if (j + 1 < kNT) mma_commit_w(&bars->k_empty[st1]);
        }
        // every MMA issued by this warp has completed before the CTA tears down TMEM
        mma_commit_w(&bars->final_mma);
        mbar_drain(&bars->final_mma, 0);
      }
    }
  } else {
    if constexpr (MODE != kModeFixup) regs_inc<kRegsHigh>();
    // ------------------------------------------------------------------ softmax warps
    const int sw = warp - 4;
    const int q = sw >> 3;                // query tile
    const int hh = (sw >> 2) & 1;         // 16-lane half of the lane quarter
    const int wq = warp & 3;              // TMEM lane quarter
    const int c = lane & 3;               // key-pair column within each 8-key block
    const int lb = 32 * wq + 16 * hh;     // first TMEM lane (tile row) of this warp
    const int rA = lb + (lane >> 2);      // this thread's rows rA and rA + 8 within the tile
    const int prowA = q * 128 + rA, prowB = prowA + 8;
    const uint32_t tS = tmem + ((uint32_t)lb << 16) + q * 128;
    const uint32_t tO = tmem + ((uint32_t)lb << 16) + 256 + q * L::kOCols;
    const float c_log2 = scale * kLog2e;
    const float2 c2 = make_float2(c_log2, c_log2);
    float2 rwA[8], rwB[8];
    bool okk = __all_sync(0xffffffffu, mbar_wait(&bars->pro_done, 0, abort_flag));
    if (okk) {
      tc_fence_after();
      const uint32_t tQuarter = tmem + ((uint32_t)(32 * wq) << 16);
      // The quarter's 32 rows (32x32b view: lane = row); the park aliases the tables, which only the
      // prologue MMAs read (they completed before pro_done).
      const int qi = 4 * q + wq;
      const int srow = q * 128 + 32 * wq + lane;
      float* const park_row = rh_park + srow * 64;
      // rw: each row's window staged in its park row, then each thread reads its key pairs of rows A, B
      stage_rw(tQuarter + q * 128 + 32 * (wq & 1), lane, hh, park_row, 8 * (srow & 3));
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->stg[qi]);
      okk = __all_sync(0xffffffffu, mbar_wait(&bars->stg[qi], 0, abort_flag));
      {
        const float* ra = rh_park + prowA * 64;
        const float* rb = rh_park + prowB * 64;
        const int sw = 8 * (prowA & 3);  // the same for prowB = prowA + 8
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          rwA[m] = *reinterpret_cast<const float2*>(ra + ((8 * m + 2 * c) ^ sw));
          rwB[m] = *reinterpret_cast<const float2*>(rb + ((8 * m + 2 * c) ^ sw));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->stg[qi]);
      okk = okk && __all_sync(0xffffffffu, mbar_wait(&bars->stg[qi], 1, abort_flag));
      // rh: RH_q[r][c'] = q_r . Th[I0 + c']. Row r of tile q sits on grid row i = I0 + 2q + r/64, so
      // rh[kh] = q_r . Th[i - kh + 63] = RH_q[r][off + 63 - kh] with off = 2q + r/64 (warp-uniform).
      {
        const uint32_t tRH = tQuarter + 256 + q * 80;
        const int rl = srow & 31;
        switch (2 * q + (wq >> 1)) {
          case 0:
            park_rh_half<0>(tRH, hh, park_row, rl, rhmax_park, srow);
            break;
          case 1:
            park_rh_half<1>(tRH, hh, park_row, rl, rhmax_park, srow);
            break;
          case 2:
            park_rh_half<2>(tRH, hh, park_row, rl, rhmax_park, srow);
            break;
          default:
            park_rh_half<3>(tRH, hh, park_row, rl, rhmax_park, srow);
            break;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->bias_done[q]);
    }
    // pass 2 over the tile with reference maxima (mrA, mrB): p = 2^(S*c + rw + rh - m); P of chunk k (16-bit
    // pairs, columns 8k..8k+7) lands on scores of chunk k/2 <= k, already read. The load of chunk k+1 is in
    // flight meanwhile. Once P of keys 0..63 is written the warp arrives on p_half (the first half of P.V
    // may start).
    float mrA = -INFINITY, mrB = -INFINITY;
    // this thread's rows of the rh park (row-swizzled by the low five row bits)
    const float* const rhA_row = rh_park + prowA * 64;
    const float* const rhB_row = rh_park + prowB * 64;
    const int rlA = prowA & 31, rlB = prowB & 31;
    auto pass2 = [&](float rhA0, float rhA1, float rhB0, float rhB1) {
      const float2 bA0 = make_float2(rhA0 - mrA, rhA0 - mrA), bA1 = make_float2(rhA1 - mrA, rhA1 - mrA);
      const float2 bB0 = make_float2(rhB0 - mrB, rhB0 - mrB), bB1 = make_float2(rhB1 - mrB, rhB1 - mrB);
      uint32_t v0[8], v1[8], pw[4];
      tmem_ld_16x256b_x2(tS + 0, v0);
      tmem_wait_ld_regs(v0);
      static_for<0, 8>([&](auto kk) {
        constexpr int k = decltype(kk)::value;  // chunk k = blocks 2k, 2k+1
        uint32_t(&cur)[8] = (k & 1) ? v1 : v0;
        uint32_t(&nxt)[8] = (k & 1) ? v0 : v1;
        if constexpr (k + 1 < 8) tmem_ld_16x256b_x2(tS + 16 * (k + 1), nxt);
        if constexpr (k < 4)
          chunk_exp<2 * k, kBf16>(cur, c2, rwA, rwB, bA0, bB0, pw);
        else
          chunk_exp<2 * k, kBf16>(cur, c2, rwA, rwB, bA1, bB1, pw);
        tmem_st_16x128b_x2(tS + 8 * k, pw);
        if constexpr (k == 3) {
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_half[q]);
        }
        if constexpr (k + 1 < 8) tmem_wait_ld_regs(nxt);
      });
    };
    // O and row-sum rescale by (alA, alB) where the reference was raised: PV_q(j-1) has completed (it was
    // issued before S_q(j), whose commit was waited on), and PV_q(j) starts only once P of the tile's first
    // 64 keys is written, after this.
    auto rescale_o = [&](int j, bool needA, bool needB, float alA, float alB) {
      if (__any_sync(0xffffffffu, (needA || needB) && j > 0)) {
#pragma unroll
        for (int c0 = 0; c0 < L::kOCols; c0 += 16) {
          uint32_t ov[8];
          tmem_ld_16x256b_x2(tO + c0, ov);
          tmem_wait_ld_regs(ov);
          ov[0] = __float_as_uint(__uint_as_float(ov[0]) * alA);
          ov[1] = __float_as_uint(__uint_as_float(ov[1]) * alA);
          ov[4] = __float_as_uint(__uint_as_float(ov[4]) * alA);
          ov[5] = __float_as_uint(__uint_as_float(ov[5]) * alA);
          ov[2] = __float_as_uint(__uint_as_float(ov[2]) * alB);
          ov[3] = __float_as_uint(__uint_as_float(ov[3]) * alB);
          ov[6] = __float_as_uint(__uint_as_float(ov[6]) * alB);
          ov[7] = __float_as_uint(__uint_as_float(ov[7]) * alB);
          tmem_st_16x256b_x2(tO + c0, ov);
        }
      }
    };
    // Exact tile: pass 1 gives the row maxima t of S*c + rw + rh (rh per 64-key half) across the row's four
    // threads, then pass 2 against the raised reference.
    auto exact_tile = [&](int j, float rhA0, float rhA1, float rhB0, float rhB1, float& alA, float& alB,
                          bool& needA, bool& needB, float& tA, float& tB) {
      {
        uint32_t v0[8], v1[8];
        float mA[2] = {-INFINITY, -INFINITY}, mB[2] = {-INFINITY, -INFINITY};
        static_for<0, 4>([&](auto kk) {
          constexpr int k = decltype(kk)::value;  // chunks 2k and 2k+1 = blocks 4k .. 4k+3
          tmem_ld_16x256b_x2(tS + 32 * k, v0);
          tmem_ld_16x256b_x2(tS + 32 * k + 16, v1);
          tmem_wait_ld_regs(v0);
          tmem_wait_ld_regs(v1);
          chunk_max<4 * k>(v0, c2, rwA, rwB, mA[k >> 1], mB[k >> 1]);
          chunk_max<4 * k + 2>(v1, c2, rwA, rwB, mA[k >> 1], mB[k >> 1]);
        });
        tA = fmaxf(mA[0] + rhA0, mA[1] + rhA1);
        tB = fmaxf(mB[0] + rhB0, mB[1] + rhB1);
        tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 1));
        tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 1));
        tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 2));
        tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 2));
      }
      needA = (j == 0) || (tA > mrA + kRescaleThreshold);
      needB = (j == 0) || (tB > mrB + kRescaleThreshold);
      if (needA) {
        const float mn = fmaxf(mrA, tA);
        alA = ex2(mrA - mn);
        mrA = mn;
      }
      if (needB) {
        const float mn = fmaxf(mrB, tB);
        alB = ex2(mrB - mn);
        mrB = mn;
      }
      rescale_o(j, needA, needB, alA, alB);
      pass2(rhA0, rhA1, rhB0, rhB1);
    };
    // End of a tile: one P-ready arrival per warp once every lane's P stores are done.
    auto finish_tile = [&]() {
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[q]);
    };
    // Epilogue of a pass: O / l -> out once PV_q of the last tile has completed; false if an output is not
    // finite.
    auto epilogue = [&](int pass) {
      bool finite = true;
      if (okk) okk = __all_sync(0xffffffffu, mbar_wait(&bars->o_done[q], pass & 1, abort_flag));
      if (okk) {
        tc_fence_after();
        // every column of the ones block holds the row sum
        uint32_t lv[8];
        tmem_ld_16x256b_x2(tO + HD, lv);
        tmem_wait_ld_regs(lv);
        const float invA = 1.f / __uint_as_float(lv[0]), invB = 1.f / __uint_as_float(lv[2]);
        // the row sum is at least the row's largest P: a sum of 2^kSpecLimit or more (or a NaN) means an
        // exponent above kSpecLimit somewhere in the row
        finite &= __uint_as_float(lv[0]) < kSpecSumLimit && __uint_as_float(lv[2]) < kSpecSumLimit;
        T* oA = out + (bh * kN + row0 + prowA) * HD + 2 * c;
        T* oB = oA + 8 * HD;
#pragma unroll
        for (int c0 = 0; c0 < HD; c0 += 16) {
          uint32_t ov[8];
          tmem_ld_16x256b_x2(tO + c0, ov);
          tmem_wait_ld_regs(ov);
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            y[e] = __uint_as_float(ov[e]) * ((e & 2) ? invB : invA);
            finite &= fabsf(y[e]) < INFINITY;  // false for inf and NaN
          }
          *reinterpret_cast<uint32_t*>(oA + c0) = pack2(y[0], y[1], kBf16);
          *reinterpret_cast<uint32_t*>(oA + c0 + 8) = pack2(y[4], y[5], kBf16);
          *reinterpret_cast<uint32_t*>(oB + c0) = pack2(y[2], y[3], kBf16);
          *reinterpret_cast<uint32_t*>(oB + c0 + 8) = pack2(y[6], y[7], kBf16);
        }
      }
      return finite;
    };
    // The exact two-pass softmax over all key tiles (f16, and the marked CTAs of the bf16 fixup launch).
    auto exact_pass = [&](int pass) {
      mrA = -INFINITY;
      mrB = -INFINITY;
      for (int j = 0; j < kNT && okk; ++j) {
        okk = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[q], j & 1, abort_flag));
        if (!okk) break;
        tc_fence_after();
        const float rhA0 = rhA_row[(2 * j) ^ rlA], rhA1 = rhA_row[(2 * j + 1) ^ rlA];
        const float rhB0 = rhB_row[(2 * j) ^ rlB], rhB1 = rhB_row[(2 * j + 1) ^ rlB];
        bool needA, needB;
        float alA = 1.f, alB = 1.f, tA, tB;
        exact_tile(j, rhA0, rhA1, rhB0, rhB1, alA, alB, needA, needB, tA, tB);
        finish_tile();
      }
      epilogue(pass);
    };
    if constexpr (MODE != kModeSpec) {
      exact_pass(0);
    } else {
      // Speculative pass (bf16): one pass per tile against one reference per row, set at tile 0 from its
      // row max pass: base = max over tile 0 of S*c + rw (the score without the per-key-row rh term;
      // tile 0 covers every key column, so every rw), rhmax = the largest rh over all 64 key rows, and the
      // reference = min(base + rhmax, t + kSpecCap) with t tile 0's max of the full score. base + rhmax
      // bounds every later score unless S*c + rw grows beyond tile 0's, so later exponents stay near or
      // below 0; the cap keeps the dominant keys' P above 2^-96. Any reference gives the same softmax (O
      // and its row sums from the ones block scale together) and bf16 P and the f32 sums hold 2^-126 ..
      // 2^127: the epilogue checks each row sum (at least the row's largest P) against 2^kSpecLimit and
      // each output for finiteness, and a CTA that fails either leaves the NaN marker for the fixup launch.
      // No O rescale is ever needed.
      float rhmaxA, rhmaxB;
      for (int j = 0; j < kNT && okk; ++j) {
        okk = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[q], j & 1, abort_flag));
        if (!okk) break;
        tc_fence_after();
        const float rhA0 = rhA_row[(2 * j) ^ rlA], rhA1 = rhA_row[(2 * j + 1) ^ rlA];
        const float rhB0 = rhB_row[(2 * j) ^ rlB], rhB1 = rhB_row[(2 * j + 1) ^ rlB];
        if (j == 0) {
          rhmaxA = fmaxf(rhmax_park[prowA], rhmax_park[256 + prowA]);
          rhmaxB = fmaxf(rhmax_park[prowB], rhmax_park[256 + prowB]);
          uint32_t v0[8], v1[8];
          float mA[2] = {-INFINITY, -INFINITY}, mB[2] = {-INFINITY, -INFINITY};
          static_for<0, 4>([&](auto kk) {
            constexpr int k = decltype(kk)::value;
            tmem_ld_16x256b_x2(tS + 32 * k, v0);
            tmem_ld_16x256b_x2(tS + 32 * k + 16, v1);
            tmem_wait_ld_regs(v0);
            tmem_wait_ld_regs(v1);
            chunk_max<4 * k>(v0, c2, rwA, rwB, mA[k >> 1], mB[k >> 1]);
            chunk_max<4 * k + 2>(v1, c2, rwA, rwB, mA[k >> 1], mB[k >> 1]);
          });
          float tA = fmaxf(mA[0] + rhA0, mA[1] + rhA1), tB = fmaxf(mB[0] + rhB0, mB[1] + rhB1);
          float bA = fmaxf(mA[0], mA[1]), bB = fmaxf(mB[0], mB[1]);
          tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 1));
          tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 1));
          bA = fmaxf(bA, __shfl_xor_sync(0xffffffffu, bA, 1));
          bB = fmaxf(bB, __shfl_xor_sync(0xffffffffu, bB, 1));
          tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 2));
          tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 2));
          bA = fmaxf(bA, __shfl_xor_sync(0xffffffffu, bA, 2));
          bB = fmaxf(bB, __shfl_xor_sync(0xffffffffu, bB, 2));
          mrA = fminf(bA + rhmaxA, tA + kSpecCap);
          mrB = fminf(bB + rhmaxB, tB + kSpecCap);
        }
        pass2(rhA0, rhA1, rhB0, rhB1);
        finish_tile();
      }
      const bool unsafe = !epilogue(0);
      // The marker goes in after its element's own output (written by this very thread of warp 4 in its
      // epilogue) and after every warp's flag.
      if (__any_sync(0xffffffffu, unsafe) && lane == 0) bars->rerun = 1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->epi_done);
      if (warp == 4 && __all_sync(0xffffffffu, mbar_wait(&bars->epi_done, 0, abort_flag)) && lane == 0 &&
          *reinterpret_cast<volatile int*>(&bars->rerun) != 0)
        *marker = from_f<T>(__int_as_float(0x7fc00000));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if constexpr (MODE == kModeFixup) {
    // the barriers are initialised again for the CTA's next block
    __syncthreads();
    if (threadIdx.x == 0) {
      uint64_t* b = reinterpret_cast<uint64_t*>(bars);
      for (int i = 0; i < (int)(offsetof(Bars, tmem_base) / sizeof(uint64_t)); ++i) mbar_inval(b + i);
    }
    __syncthreads();
  }
  };

  if constexpr (MODE == kModeFixup) {
    // The fixup launch: a grid of at most one CTA per SM; CTA b owns the blocks b, b + grid, b + 2 grid, ...
    // Its threads read those blocks' markers at once (640 at a time), and the CTA runs the exact pass of
    // the marked ones only. With nothing marked a launch is one pass of marker reads per CTA.
    __shared__ int fx_count;
    __shared__ int fx_list[kThreads];
    for (long k0 = 0; blockIdx.x + k0 * (long)gridDim.x < n_blocks; k0 += kThreads) {
      if (threadIdx.x == 0) fx_count = 0;
      __syncthreads();
      const long cand = blockIdx.x + (k0 + threadIdx.x) * (long)gridDim.x;
      if (cand < n_blocks && !device_faulted()) {
        const T* m = out + ((cand / (kN / 256)) * kN + (cand % (kN / 256)) * 256) * HD;
        const float v = to_f(*reinterpret_cast<const volatile T*>(m));
        if (v != v) {
          fx_list[atomicAdd(&fx_count, 1)] = threadIdx.x;
          atomicAdd(&g_recomputed, 1ull);
          if (recompute_slot) atomicAdd(recompute_slot, 1ull);  // the host's per-layer measurement
        }
      }
      __syncthreads();
      const int n = fx_count;
      for (int i = 0; i < n; ++i) run_block(blockIdx.x + (k0 + fx_list[i]) * (long)gridDim.x);
      __syncthreads();
    }
  } else {
    (void)n_blocks;
    run_block(blockIdx.x);
  }
}

}  // namespace tcg
}  // namespace samrs
