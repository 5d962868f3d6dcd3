// relpos_tc_window.cuh - tcgen05 kernel for SAM's windowed layers: 14x14 windows (196 tokens),
// head_dim 64 or 80, f16/bf16 I/O, f32 accumulation and softmax.
//
// Math as the global kernel (src/kernels.rs:131-225; windows from src/sam1/encoder.rs:118-121,132-145):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+13] + q_r . Tw[j-kw+13],  r = 14 i + j, k = 14 kh + kw.
//
// These layers are HBM-bound (~98 FLOP/B at hd 80), so the kernel streams: a persistent grid (one CTA
// per SM) walks over units = (window, head) pairs with the loads of later units in flight. Per unit the
// 196 query rows are two 128-row MMA tiles and all keys fit one key tile, so each row's softmax sees all
// its keys at once: f16 takes the exact row max in a first pass over S; bf16 takes a single pass with the
// reference from the row's first 32 keys (row_exp_online).
//
// One N = 256 MMA per tile yields scores and bias projections together: the B operand holds the 196
// keys followed by the 27 rows of rel_pos_h and the 27 rows of rel_pos_w (196 + 54 = 250 <= 256), so
// S_t = Q_t [K | Th | Tw]^T gives q.k in columns 0..195, RH = q.Th in 196..222 and RW = q.Tw in 223..249.
// Each thread then selects its 14 + 14 bias values with a lane-dependent 4-stage shift (by its grid row
// i for rh, by its grid column j for rw).
//
// Loads: q and v through 3-D TMA tensor maps [bh][196][hd] (OOB rows -> 0). kt ([bh][hd][196]) has a
// 392-byte row pitch, which TMA cannot tile (strides must be multiples of 16 B), so 64 loader threads
// move it with 8-byte cp.async straight into the canonical no-swizzle MN-major UMMA layout (8 keys x 8
// dims per 128-byte core matrix). The table rows are written into both K buffers once, at start-up.
// Rings: Q+K (2 stages, released when a unit's S MMAs complete) and a single V stage (reloaded once both
// tiles' PV MMAs completed; the load has the next unit's softmax to land). Output rows are staged in
// shared memory and written back by one bulk store per warp.
//
// Warps: 0 / 1 MMA issuers of query tile 1 / 0 (one warp each, so the two tiles' S -> softmax -> PV ->
// epilogue chains never wait on each other; tile 1 starts half a step after tile 0, except in the bf16
// hd-80 kernel, whose tiles run in step), 2-3 kt loaders (thread 0 also issues the q TMA loads, the last
// thread the v TMA loads; warp 2 allocates TMEM), 4-7 / 8-11 softmax + epilogue of query tile 0 / 1
// (thread = query row = TMEM lane); warp 11 covers rows 224..255 only, which are all padding, so it only
// keeps the barrier counts.
// TMEM (512 columns): tile t owns [256t, 256t+256): S_t; then P_t (16-bit pairs, cols 0..103) written
// over the consumed scores; O_t and its row sums accumulate in cols [128, 128+hd+16) once the softmax
// has consumed S_t (the P.V MMA multiplies by [V | ones]).
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tcw {

constexpr int kThreads = 384;
constexpr int kLoaders = 64;  // threads of warps 2-3
// Registers: launched at 168 per thread (384 x 168 = 64512); warpgroup 0 (producer, MMA, loaders) gives
// back to 96, the two softmax warpgroups take 200: 128 x 96 + 256 x 200 = 63488.
constexpr uint32_t kRegsLow = 96, kRegsHigh = 200;
static_assert(128 * kRegsLow + 256 * kRegsHigh <= kThreads * 168, "register split exceeds the launch allotment");
constexpr int kSide = 14, kN = 196, kNP = 208, kNB = 256, kStages = 2;
constexpr int kTabRows = 2 * kSide - 1;           // 27 rows each of rel_pos_h and rel_pos_w
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct Layout {
  static constexpr int HC = HD / 16;
  // q: one [200 rows x 32 B] SW32 chunk per 16 dims (rows 196..199 zero-filled by TMA). Tile 1's MMA
  // reads rows 128..255, i.e. past the chunk end into the next chunk / the K buffer: finite data whose
  // S, P and O rows are discarded (every MMA output row depends on its own A row only).
  static constexpr int kQRows = 200;
  static constexpr int kQChunk = kQRows * 32;
  static constexpr int kQBytes = HC * kQChunk;
  static constexpr int kVChunk = kNP * 32;          // [208 keys x 32 B] SW32
  static constexpr int kVBytes = HC * kVChunk;      // bytes of v loaded per unit
  // The V stage holds the HC chunks of v and then a chunk of ones: the P.V MMA runs with N = HD + 16, so
  // that O's last 16 columns accumulate the row sums of the 16-bit P exactly as the product uses them.
  static constexpr int kVStageBytes = (HC + 1) * kVChunk;
  static constexpr int kOCols = HD + 16;
  // B operand of the S MMA, N = 256: keys, then table rows. Stride between 8-column core columns: HD/8
  // core matrices of 128 B plus 16 B, so consecutive columns fall in different banks for the 8-byte
  // cp.async writes (2 wavefronts per warp, the minimum for 256 B).
  static constexpr int kKSbo = (HD / 8) * 128 + 16;
  static constexpr int kKBytes = (kNB / 8) * kKSbo;
  static constexpr int kQKStage = (kQBytes + kKBytes + 255) / 256 * 256;
  static constexpr int kVStage = (kVStageBytes + 255) / 256 * 256;
  static constexpr int OFF_Q = 0, OFF_K = kQBytes;  // within a QK stage
  static constexpr int OFF_V = kStages * kQKStage;  // one V stage: loaded during the unit's softmax
  // output staging: the 128 rows of each tile (row-major, as in `out`), written back by bulk stores
  static constexpr int kStgTile = 128 * HD * 2;
  static constexpr int OFF_STG = OFF_V + kVStage;
  static constexpr int OFF_BAR = OFF_STG + 2 * kStgTile;
  static constexpr int kSmemBytes = OFF_BAR + 256 + 1024;
  static_assert(kQChunk % 256 == 0 && kVChunk % 256 == 0 && OFF_K % 128 == 0 && kQKStage % 256 == 0, "alignment");
  static_assert((256 - kQRows) * 32 <= kKBytes, "tile-1 over-read stays inside the stage");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Bars {
  uint64_t q_full[kStages], k_full[kStages], qk_free[kStages], v_full, v_free;
  uint64_t final_mma[2];
  uint64_t s_full[2], p_full[2], o_full[2], t_free[2];
  uint32_t tmem_base;
  int abort_flag;
};

// Byte offset of (column n, dim d) in the no-swizzle MN-major B tile.
template <int HD>
__device__ __forceinline__ uint32_t k_off(int n, int d) {
  return (uint32_t)((n >> 3) * Layout<HD>::kKSbo + (d >> 3) * 128 + (d & 7) * 16 + (n & 7) * 2);
}

// a[m] <- a[m + 2^B] where bit B of `sh` is set, for m < LEN (one 3-input logic op per element).
template <int B, int LEN>
__device__ __forceinline__ void wshift(uint32_t (&a)[32], int sh) {
  const uint32_t mask = 0u - ((uint32_t)(sh >> B) & 1u);
#pragma unroll
  for (int m = 0; m < LEN; ++m) a[m] = (a[m] & ~mask) | (a[m + (1 << B)] & mask);
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

// Bias pairs for key pairs (k, k+1), k even. Since 14 is even, such a pair never straddles a window
// row: it shares kh, and kw, kw+1 are both in the row. rhp[kh] = (rh[kh], rh[kh]), rwp[m] = (rw[2m], rw[2m+1]).
struct Bias {
  float2 rhp[14];
  float2 rwp[7];
};

// Pass 1 over the 32 keys of chunk CH held in `sv`: 8 independent running maxima of S*c + rh + rw.
template <int CH>
__device__ __forceinline__ void chunk_max(const uint32_t (&sv)[32], float2 c2, const Bias& b, float (&m)[8]) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const int k0 = 32 * CH + e;
    if (k0 < kN) {  // k0 even and kN even: k0 + 1 < kN too
      const float2 s2 = make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
      const float2 x = sm100::add2(sm100::fma2(s2, c2, b.rhp[k0 / kSide]), b.rwp[(k0 % kSide) >> 1]);
      m[(e >> 1) & 7] = sm100::max3(m[(e >> 1) & 7], x.x, x.y);
    }
  }
}

// Pass 2 over chunk CH (keys 32*CH + e, e < NE): p = 2^(S*c + rh + (rw - m)) as 16-bit pairs into pk
// (keys >= 196 get p = 0). The row sums come from the P.V MMA (ones block of V).
template <int CH, int NE, bool BF16>
__device__ __forceinline__ void chunk_exp(const uint32_t (&sv)[32], float2 c2, const Bias& b, uint32_t (&pk)[16]) {
  // Staged: all exponents, then the exponentials (one pair in eight on the FMA pipe), then packing.
  constexpr int NV = (32 * CH + NE <= kN) ? NE : (kN - 32 * CH);  // keys of the chunk below kN (even)
  float x[32];
#pragma unroll
  for (int e = 0; e < NV; e += 2) {
    const int k0 = 32 * CH + e;
    const float2 s2 = make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
    const float2 t = sm100::add2(sm100::fma2(s2, c2, b.rhp[k0 / kSide]), b.rwp[(k0 % kSide) >> 1]);
    x[e] = t.x;
    x[e + 1] = t.y;
  }
#pragma unroll
  for (int e = 0; e < NV; e += 2) {
    if ((e & 14) == 14) {
      const float2 p = sm100::ex2_poly2(make_float2(x[e], x[e + 1]));
      x[e] = p.x;
      x[e + 1] = p.y;
    } else {
      x[e] = sm100::ex2(x[e]);
      x[e + 1] = sm100::ex2(x[e + 1]);
    }
  }
#pragma unroll
  for (int e = 0; e < NE; e += 2) pk[e >> 1] = e < NV ? sm100::pack2(x[e], x[e + 1], BF16) : 0u;
}

// Row max over the 196 keys: two chunks per wait, the next two loads in flight while a pair is reduced.
__device__ __forceinline__ float row_max(uint32_t tS, float2 c2, const Bias& b) {
  using namespace sm100;
  uint32_t a[32], bb[32], a2[32], bb2[32];
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = -INFINITY;
  tmem_ld32(tS + 0, a);
  tmem_ld32(tS + 32, bb);
  tmem_wait_ld_regs(a);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 64, a2);
  tmem_ld32(tS + 96, bb2);
  chunk_max<0>(a, c2, b, m);
  chunk_max<1>(bb, c2, b, m);
  tmem_wait_ld_regs(a2);
  tmem_wait_ld_regs(bb2);
  tmem_ld32(tS + 128, a);
  tmem_ld32(tS + 160, bb);
  chunk_max<2>(a2, c2, b, m);
  chunk_max<3>(bb2, c2, b, m);
  tmem_wait_ld_regs(a);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 192, a2);  // columns 192..223: keys 192..195
  chunk_max<4>(a, c2, b, m);
  chunk_max<5>(bb, c2, b, m);
  tmem_wait_ld_regs(a2);
  chunk_max<6>(a2, c2, b, m);
  return max3(max3(m[0], m[1], m[2]), max3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// p = 2^(x - m) for all keys (the bias pairs already hold rw - m), P written as 16-bit pairs over the
// consumed S columns 0..103. The load of chunk k+1 is in flight while chunk k is exponentiated.
template <bool BF16>
__device__ __forceinline__ void row_exp(uint32_t tS, float2 c2, const Bias& b) {
  using namespace sm100;
  uint32_t a[32], bb[32], pk[16];
  tmem_ld32(tS + 0, a);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 32, bb);
  chunk_exp<0, 32, BF16>(a, c2, b, pk);
  tmem_st16(tS + 0, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 64, a);
  chunk_exp<1, 32, BF16>(bb, c2, b, pk);
  tmem_st16(tS + 16, pk);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 96, bb);
  chunk_exp<2, 32, BF16>(a, c2, b, pk);
  tmem_st16(tS + 32, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 128, a);
  chunk_exp<3, 32, BF16>(bb, c2, b, pk);
  tmem_st16(tS + 48, pk);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 160, bb);
  chunk_exp<4, 32, BF16>(a, c2, b, pk);
  tmem_st16(tS + 64, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 192, a);
  chunk_exp<5, 32, BF16>(bb, c2, b, pk);
  tmem_st16(tS + 80, pk);
  tmem_wait_ld_regs(a);
  chunk_exp<6, 16, BF16>(a, c2, b, pk);  // keys 192..207 (196.. get p = 0)
  uint32_t p8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) p8[e] = pk[e];
  tmem_st8(tS + 96, p8);
}

// Exponents x = S*c + rh + rw of the keys of chunk CH below kN (b.rwp may already hold rw minus a
// reference) into x; returns their max.
template <int CH>
__device__ __forceinline__ float chunk_x(const uint32_t (&sv)[32], float2 c2, const Bias& b, float (&x)[32]) {
  constexpr int NV = (32 * CH + 32 <= kN) ? 32 : (kN - 32 * CH);
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int e = 0; e < NV; e += 2) {
    const int k0 = 32 * CH + e;
    const float2 s2 = make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
    const float2 t = sm100::add2(sm100::fma2(s2, c2, b.rhp[k0 / kSide]), b.rwp[(k0 % kSide) >> 1]);
    x[e] = t.x;
    x[e + 1] = t.y;
    mx[(e >> 1) & 3] = sm100::max3(mx[(e >> 1) & 3], t.x, t.y);
  }
  return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
}

// 2^x of the chunk's keys below kN packed as 16-bit pairs; keys >= kN get p = 0. With POLY, one key pair in
// eight goes to the FMA-pipe polynomial: at hd 80 that measured 0.389 ms against 0.405 (one in four), 0.406
// (one in sixteen) and 0.413 (none) per bh-12800 layer; at hd 64 none measured best (0.178 against 0.181 with
// one in eight, bh 6400).
template <int CH, int NE, bool BF16, bool POLY>
__device__ __forceinline__ void chunk_pack(float (&x)[32], uint32_t (&pk)[16]) {
  constexpr int NV = (32 * CH + NE <= kN) ? NE : (kN - 32 * CH);
#pragma unroll
  for (int e = 0; e < NV; e += 2) {
    if (POLY && (e & 14) == 14) {
      const float2 p = sm100::ex2_poly2(make_float2(x[e], x[e + 1]));
      x[e] = p.x;
      x[e + 1] = p.y;
    } else {
      x[e] = sm100::ex2(x[e]);
      x[e + 1] = sm100::ex2(x[e + 1]);
    }
  }
#pragma unroll
  for (int e = 0; e < NE; e += 2) pk[e >> 1] = e < NV ? sm100::pack2(x[e], x[e + 1], BF16) : 0u;
}

// A later chunk's exponents exceed the row's reference by more than the single pass allows: the reference
// of every row with such a chunk moves up by d (the chunk's max), so the P already written (columns
// 0 .. 16 * nprev) are scaled by 2^-d here, and the caller takes d off the chunk's exponents and off the bias
// pairs of the chunks still to come. The other rows of the warp pass d = 0 (scale by 1). Rare: the overflow
// guard of the single pass.
template <bool BF16>
__device__ __forceinline__ void scale_written_p(uint32_t tS, int nprev, float d) {
  using namespace sm100;
  const float f = ex2(-d);
  tmem_wait_st();  // this thread's P stores are complete before they are read back
  for (int cc = 0; cc < nprev; ++cc) {
    uint32_t p[16];
    tmem_ld16(tS + 16 * cc, p);
    tmem_wait_ld_regs(p);
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float lo, hi;
      if (BF16) {
        lo = __uint_as_float(p[e] << 16);
        hi = __uint_as_float(p[e] & 0xFFFF0000u);
      } else {
        const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&p[e]));
        lo = v2.x;
        hi = v2.y;
      }
      p[e] = pack2(lo * f, hi * f, BF16);
    }
    tmem_st16(tS + 16 * cc, p);
  }
}
// The same, as a call: at hd 64 the softmax loop measured 18 % faster with the rare path out of line
// (0.183 vs 0.211 ms at bh 6400), at hd 80 6 % slower than inline (0.430 vs 0.409 ms at bh 12800).
template <bool BF16>
__device__ __noinline__ void scale_written_p_call(uint32_t tS, int nprev, float d) {
  scale_written_p<BF16>(tS, nprev, d);
}

// Single-pass P for bf16: the reference is the max of the row's first 32 exponents (at or below the row's
// true max, so the row's largest P is >= 1 and nothing that matters underflows). Later keys' P may exceed 1:
// bf16 P and the f32 row sums and O hold up to 2^127, and a chunk whose max exceeds the reference by more
// than kOnlineLimit raises the reference first (scale_written_p), so every P stays <= 2^64. The row sums
// come from the P.V MMA (ones block of V), from the same rounded P, so any reference gives the same softmax.
constexpr float kOnlineLimit = 64.f;

template <int CH, int NE, bool BF16, int HD, bool OOL>
__device__ __forceinline__ void online_chunk(const uint32_t (&sv)[32], uint32_t tS, float2 c2, Bias& b,
                                             uint32_t (&pk)[16]) {
  float x[32];
  const float mc = chunk_x<CH>(sv, c2, b, x);
  if (__any_sync(0xffffffffu, mc > kOnlineLimit)) {
    const float d = mc > kOnlineLimit ? mc : 0.f;
    if constexpr (OOL)
      scale_written_p_call<BF16>(tS, CH, d);
    else
      scale_written_p<BF16>(tS, CH, d);
#pragma unroll
    for (int k = 0; k < 7; ++k) b.rwp[k] = make_float2(b.rwp[k].x - d, b.rwp[k].y - d);
#pragma unroll
    for (int e = 0; e < 32; ++e) x[e] -= d;
  }
  chunk_pack<CH, NE, BF16, HD != 64>(x, pk);
}

template <bool BF16, int HD, bool OOL>
__device__ __forceinline__ void row_exp_online(uint32_t tS, float2 c2, Bias& b) {
  using namespace sm100;
  uint32_t a[32], bb[32], pk[16];
  tmem_ld32(tS + 0, a);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 32, bb);
  {
    float x[32];
    const float m = chunk_x<0>(a, c2, b, x);
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float2 t = add2(make_float2(x[e], x[e + 1]), make_float2(-m, -m));
      x[e] = t.x;
      x[e + 1] = t.y;
    }
#pragma unroll
    for (int k = 0; k < 7; ++k) b.rwp[k] = add2(b.rwp[k], make_float2(-m, -m));
    chunk_pack<0, 32, BF16, HD != 64>(x, pk);
  }
  tmem_st16(tS + 0, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 64, a);
  online_chunk<1, 32, BF16, HD, OOL>(bb, tS, c2, b, pk);
  tmem_st16(tS + 16, pk);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 96, bb);
  online_chunk<2, 32, BF16, HD, OOL>(a, tS, c2, b, pk);
  tmem_st16(tS + 32, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 128, a);
  online_chunk<3, 32, BF16, HD, OOL>(bb, tS, c2, b, pk);
  tmem_st16(tS + 48, pk);
  tmem_wait_ld_regs(a);
  tmem_ld32(tS + 160, bb);
  online_chunk<4, 32, BF16, HD, OOL>(a, tS, c2, b, pk);
  tmem_st16(tS + 64, pk);
  tmem_wait_ld_regs(bb);
  tmem_ld32(tS + 192, a);
  online_chunk<5, 32, BF16, HD, OOL>(bb, tS, c2, b, pk);
  tmem_st16(tS + 80, pk);
  tmem_wait_ld_regs(a);
  online_chunk<6, 16, BF16, HD, OOL>(a, tS, c2, b, pk);  // keys 192..207 (196.. get p = 0)
  uint32_t p8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) p8[e] = pk[e];
  tmem_st8(tS + 96, p8);
}

// Bias of this thread's row from the S columns 192..255: rh from RH (cols 196..222) shifted by the grid
// row i, rw from RW (cols 223..249) shifted by the grid column j.
__device__ __forceinline__ void read_bias(uint32_t tS, int i, int j, Bias& b) {
  using namespace sm100;
  uint32_t v0[32], v1[32];
  tmem_ld32(tS + 192, v0);
  tmem_ld32(tS + 224, v1);
  tmem_wait_ld_regs(v0);
  tmem_wait_ld_regs(v1);
  uint32_t a[32];
  float rh[14], rw[14];
#pragma unroll
  for (int m = 0; m < 32; ++m) a[m] = m + 4 < 32 ? v0[m + 4] : v1[m + 4 - 32];  // column 196 + m
  select14(a, i, rh);
#pragma unroll
  for (int m = 0; m < 32; ++m) a[m] = m == 0 ? v0[31] : v1[m - 1];  // column 223 + m
  select14(a, j, rw);
#pragma unroll
  for (int k = 0; k < 14; ++k) b.rhp[k] = make_float2(rh[k], rh[k]);
#pragma unroll
  for (int k = 0; k < 7; ++k) b.rwp[k] = make_float2(rw[2 * k], rw[2 * k + 1]);
}

template <typename T, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_window(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmV,
                       const T* __restrict__ table, const T* __restrict__ kt, T* __restrict__ out, long bh_total,
                       float scale) {
  using L = Layout<HD>;
  using namespace sm100;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  // After an earlier CTA reported a fault the whole CTA leaves, together (thread 0 decides: the barriers,
  // TMEM and the warp roles below need every warp).
  if (__syncthreads_or(threadIdx.x == 0 && device_faulted())) return;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long first = blockIdx.x;
  const int n_units = first < bh_total ? (int)((bh_total - first + gridDim.x - 1) / gridDim.x) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->k_full[s], kLoaders - 1);  // the last loader thread issues the v loads instead
      mbar_init(&bars->qk_free[s], 2);            // one commit per tile issuer
    }
    mbar_init(&bars->v_full, 1);
    mbar_init(&bars->v_free, 2);
    mbar_init(&bars->final_mma[0], 1);
    mbar_init(&bars->final_mma[1], 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 4);  // one arrival per softmax warp of the tile
      mbar_init(&bars->o_full[t], 1);
      mbar_init(&bars->t_free[t], 4);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  {
    // the ones block of the V stage (the TMA loads never write it); read by the MMA (async proxy)
    const uint32_t one2 = kBf16 ? 0x3F803F80u : 0x3C003C00u;
    for (int idx = threadIdx.x; idx < L::kVChunk / 16; idx += kThreads)
      reinterpret_cast<uint4*>(smem + L::OFF_V + L::HC * L::kVChunk)[idx] = make_uint4(one2, one2, one2, one2);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp < 4) {
    regs_dec<kRegsLow>();
    if (warp < 2) {
      // ---------------------------------------------------------------- MMA issuer of tile t
      // The whole warp runs the issue loop; lane 0, elected inside each MMA and commit, issues them.
      const int t = 1 - warp;
      constexpr uint32_t idS = idesc_f16(kBf16, 128, kNB, false, true);
      constexpr uint32_t idPV = idesc_f16(kBf16, 128, L::kOCols, false, true);  // O += P [V | 1]
      const uint32_t sb = smem_u32(smem);
      const uint64_t dQ = smem_desc(sb + L::OFF_Q + t * 128 * 32, 16, 256, kLayoutSw32);
      const uint64_t dK = smem_desc(sb + L::OFF_K, 128, L::kKSbo, kLayoutNone);
      const uint64_t dV = smem_desc(sb + L::OFF_V, L::kVChunk, 256, kLayoutSw32);
      const uint32_t tT = tmem + 256 * t;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      bool okk = true;
      for (int ui = 0; ui < n_units && okk; ++ui) {
        const int s = ui & 1;
        const uint32_t ph = (ui >> 1) & 1;
        // S_t(u) overwrites the tile's columns: the softmax warps must have read O_t(u-1). Tile 1's first S
        // waits for tile 0's first softmax, which sets the two tiles half a step apart: one tile's softmax on
        // the exp unit then overlaps the other's MMAs and epilogue instead of competing with its softmax. The
        // bf16 hd-80 kernel (one-pass softmax) runs the tiles in step instead: there the half-step lag left
        // tile 0 waiting for the single V stage, which tile 1's P.V of the previous unit still holds (0.407
        // vs 0.419 ms at bh 12800, faster in each of six interleaved rounds; hd 64 and f16 keep the lag:
        // 0.180 vs 0.197 ms at hd 64).
        constexpr bool kInStep = kBf16 && HD == 80;
        okk = wait(&bars->q_full[s], ph) && wait(&bars->k_full[s], ph) &&
              (ui == 0 ? (t == 0 || kInStep || wait(&bars->p_full[0], 0)) : wait(&bars->t_free[t], (ui - 1) & 1));
        if (!okk) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < L::HC; ++c)
          mma_ss_w(tT, desc_add(dQ, s * L::kQKStage + c * L::kQChunk), desc_add(dK, s * L::kQKStage + c * 256), idS,
                   c > 0);
        mma_commit_w(&bars->s_full[t]);
        mma_commit_w(&bars->qk_free[s]);  // this tile's reads of the unit's Q and K are done once S_t completes
        okk = wait(&bars->v_full, ui & 1) && wait(&bars->p_full[t], ui & 1);
        if (!okk) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kNP / 16; ++k)
          mma_ts_w(tT + 128, tT + 8 * k, desc_add(dV, k * 512), idPV, k > 0 ? 1u : 0u);
        mma_commit_w(&bars->o_full[t]);
        mma_commit_w(&bars->v_free);
      }
      mma_commit_w(&bars->final_mma[t]);
      mbar_drain(&bars->final_mma[t], 0);
    } else {
      // ---------------------------------------------------------------- kt loaders (cp.async relayout)
      const int tl = threadIdx.x - 64;
      // Table rows into both B buffers once: columns 196..222 = rel_pos_h, 223..249 = rel_pos_w,
      // 250..255 = 0.
      for (int s = 0; s < kStages; ++s) {
        uint8_t* kb = smem + s * L::kQKStage + L::OFF_K;
        for (int idx = tl; idx < (kNB - kN) * HD; idx += kLoaders) {
          const int r = idx / HD, d = idx - r * HD;
          const T v = r < 2 * kTabRows ? table[r * HD + d] : from_f<T>(0.f);
          *reinterpret_cast<T*>(kb + k_off<HD>(kN + r, d)) = v;
        }
      }
      // Thread tl owns the 8-byte key chunk c = tl (keys 4c..4c+3) of every dim row d: the source walks
      // down kt by one 392-byte row per d, the destination by 16 bytes ((d/8)*128 + (d%8)*16 = 16 d).
      const int c = tl;
      const uint32_t dst0 = (uint32_t)((c >> 1) * L::kKSbo + (c & 1) * 8);
      if (tl == kLoaders - 1) {
        // v loads: the single V stage is reloaded once both tiles' PV MMAs of the previous unit completed
        tma_prefetch_desc(&tmV);
        int issued_v = 0;
        for (int ui = 0; ui < n_units; ++ui) {
          const long u = first + (long)ui * gridDim.x;
          if (ui > 0 && !mbar_wait(&bars->v_free, (ui - 1) & 1, abort_flag)) break;
          mbar_arrive_expect_tx(&bars->v_full, L::kVBytes);
          for (int cv = 0; cv < L::HC; ++cv)
            tma_load_3d(smem + L::OFF_V + cv * L::kVChunk, &tmV, &bars->v_full, cv * 16, 0, (int)u);
          issued_v = ui + 1;
        }
        if (*abort_flag && issued_v > 0) mbar_drain(&bars->v_full, (issued_v - 1) & 1);
      } else {
        // Thread 0 also issues the unit's q TMA load (same stage as its K).
        if (tl == 0) tma_prefetch_desc(&tmQ);
        int issued_q = 0;
        for (int ui = 0; ui < n_units; ++ui) {
          const int s = ui & 1;
          const long u = first + (long)ui * gridDim.x;
          const uint32_t prev = ((ui >> 1) - 1) & 1;
          if (ui >= kStages && !mbar_wait(&bars->qk_free[s], prev, abort_flag)) break;
          if (tl == 0) {
            mbar_arrive_expect_tx(&bars->q_full[s], L::kQBytes);
            for (int cq = 0; cq < L::HC; ++cq)
              tma_load_3d(smem + s * L::kQKStage + L::OFF_Q + cq * L::kQChunk, &tmQ, &bars->q_full[s], cq * 16, 0,
                          (int)u);
            issued_q = ui + 1;
          }
          if (c < kN / 4) {
            uint8_t* dst = smem + s * L::kQKStage + L::OFF_K + dst0;
            const T* src = kt + u * (long)HD * kN + 4 * c;
#pragma unroll 8
            for (int d = 0; d < HD; ++d) cp_async_8(dst + 16 * d, src + d * kN);
          }
          cp_async_wait_all();
          fence_proxy_async_smem();
          mbar_arrive(&bars->k_full[s]);
        }
        cp_async_wait_all();
        if (tl == 0 && *abort_flag) {
          // drain this CTA's own TMA copies still in flight before the CTA can exit
          for (int ui = issued_q > kStages ? issued_q - kStages : 0; ui < issued_q; ++ui)
            mbar_drain(&bars->q_full[ui & 1], (ui >> 1) & 1);
        }
      }
    }
  } else {
    regs_inc<kRegsHigh>();
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int rt = 128 * t + 32 * wq + lane;  // query row within the window
    const bool live = 128 * t + 32 * wq < kN;  // warp holds at least one real row (warp-uniform)
    const int i = rt / kSide, j = rt % kSide;
    const uint32_t tS = tmem + ((uint32_t)(32 * wq) << 16) + 256 * t;
    const uint32_t tO = tS + 128;
    const float c = scale * kLog2e;
    for (int ui = 0; ui < n_units; ++ui) {
      const long u = first + (long)ui * gridDim.x;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[t], ui & 1, abort_flag))) break;
      tc_fence_after();
      if (live) {
        Bias b;
        read_bias(tS, i, j, b);
        const float2 c2 = make_float2(c, c);
        if constexpr (kBf16) {
          row_exp_online<kBf16, HD, HD == 64>(tS, c2, b);
        } else {
          // f16 P holds only 2^-14 .. 2^15: the exact max first
          const float m = row_max(tS, c2, b);
#pragma unroll
          for (int k = 0; k < 7; ++k) b.rwp[k] = make_float2(b.rwp[k].x - m, b.rwp[k].y - m);
          row_exp<kBf16>(tS, c2, b);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[t]);
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->o_full[t], ui & 1, abort_flag))) break;
      tc_fence_after();
      // Epilogue: O/l into registers (l = any column of the ones block), the tile's TMEM columns handed
      // back at once (the next unit's S MMA may overwrite them), then the row's 16-byte stores.
      uint32_t pw[HD / 16][8];
      if (live) {
        uint32_t ov[HD / 16 + 1][16];
#pragma unroll
        for (int c0 = 0; c0 <= HD / 16; ++c0) tmem_ld16(tO + 16 * c0, ov[c0]);
#pragma unroll
        for (int c0 = 0; c0 <= HD / 16; ++c0) tmem_wait_ld_regs(ov[c0]);
        const float inv = 1.f / __uint_as_float(ov[HD / 16][0]);
#pragma unroll
        for (int c0 = 0; c0 < HD / 16; ++c0)
#pragma unroll
          for (int e = 0; e < 8; ++e)
            pw[c0][e] = pack2(__uint_as_float(ov[c0][2 * e]) * inv, __uint_as_float(ov[c0][2 * e + 1]) * inv, kBf16);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->t_free[t]);  // O_t read and S_t columns free for the next unit's S MMA
      // Rows -> this warp's 32-row block of the staging buffer (its previous bulk store has read it), then
      // one bulk store of the block's real rows, which are contiguous in `out`.
      const int nrows = kN - (128 * t + 32 * wq) < 32 ? kN - (128 * t + 32 * wq) : 32;
      if (live) {
        if (lane == 0) bulk_wait_read();
        __syncwarp();
        uint8_t* stg_row = smem + L::OFF_STG + t * L::kStgTile + (32 * wq + lane) * (HD * 2);
        if (lane < nrows) {
#pragma unroll
          for (int c0 = 0; c0 < HD / 16; ++c0) {
            reinterpret_cast<uint4*>(stg_row)[2 * c0] = make_uint4(pw[c0][0], pw[c0][1], pw[c0][2], pw[c0][3]);
            reinterpret_cast<uint4*>(stg_row)[2 * c0 + 1] = make_uint4(pw[c0][4], pw[c0][5], pw[c0][6], pw[c0][7]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          bulk_store(out + (u * kN + 128 * t + 32 * wq) * HD, smem + L::OFF_STG + t * L::kStgTile + 32 * wq * (HD * 2),
                     (uint32_t)(nrows * HD * 2));
          bulk_commit();
        }
      }
    }
  }
  if (warp >= 4 && lane == 0) bulk_wait();  // this warp's output stores have completed
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tcw
}  // namespace samrs
