// relpos_tc_f32.cuh - tcgen05 kernel for f32 I/O (SAM's 64x64 global and 14x14 windowed layers, head_dim 64
// or 80). The two contractions run on the tensor cores as kind::tf32 MMAs with every f32 operand split in
// two TF32 terms, x = hi + lo (hi: x with its 13 low mantissa bits cleared; lo: x - hi, cleared the same
// way), and every product taken as lo.hi + hi.lo + hi.hi ("3xTF32"). The dropped lo.lo term and the
// truncation of lo leave a relative error near 2^-20 per product term; the bias projections, softmax and
// normalisation are f32 on the CUDA cores.
//
// Math (src/kernels.rs:131-225, the f32 body of `attention_relpos_cpu`, as the f16/bf16 kernels):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+h-1] + q_r . Tw[j-kw+w-1],  r = w i + j, k = w kh + kw
//   out_r  = sum_k softmax_k(x[r, .]) v_k
//
// CTA = one head x 128 query rows; key tiles of 64 keys (a 64x64 layer: tile t = grid row kh = t, 64 tiles;
// a 14x14 window: 4 tiles, keys 196..255 masked). kind::tf32 takes its shared-memory operand K-major only
// (an MN-major B operand reads as zeros on sm_100a), so kt ([hd][keys]) and v ([keys][hd]) are transposed
// on the way in. Warps (16, 512 threads):
//   0      MMA issuer: S_t = Q K_t^T (A = q from TMEM, B = k K-major, N = 64) and O += P_t V_t (A = P from
//          TMEM, B = v^T K-major), three TF32 products each, each issued as soon as its inputs are ready.
//          v^T's hi term carries 16 extra rows of ones, so that the P.V MMAs with it (N = hd + 16) also
//          accumulate the row sums l = P.1 beside O: O and l then carry the tensor core's accumulation alike.
//   1      TMEM allocator (512 columns)
//   4-11   row threads, two per query row: warp w serves TMEM lane quarter w % 4 and key half (w - 4) / 4
//          of every tile. The q row from HBM, q split into TMEM, the row's bias projections in f32 on the
//          CUDA cores against the table staged in shared memory by one bulk copy (each half takes its
//          share); per tile 32 scores each, the row maximum exchanged between the two halves through shared
//          memory (an mbarrier per lane-quarter pair), a lazily rescaled running maximum (O is rescaled only
//          when a row's maximum grows by more than 2^8), P split into TMEM; at the end O / l to HBM.
//   12-13  k splitters, 14-15 v splitters: per key tile, 4x4 blocks (4 rows of 4 consecutive keys or dims)
//          by 16-byte loads from HBM / L2 (the query tiles of a head share the tiles), issued one tile
//          ahead, transposed in registers, split, and stored as 16-byte granules (4 K-values of one row) of
//          the canonical no-swizzle K-major layout. Row groups of 8 are 144 B apart (SBO), not 128, so that
//          the 8 lanes of a store phase (rows 4 apart) hit 8 different bank groups. 2-slot rings for k
//          (a slot frees when its S MMAs complete) and v (when its P.V MMAs complete).
// TMEM columns: S_t / P_t hi (2 buffers of 64), P_t lo (2 x 64), O and l (hd + 16), q hi and q lo (hd each).
// Every wait is bounded (sm100::mbar_wait, or the MMA issuer's own bounded polling); no multicast.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tcf {

constexpr int kThreads = 512;
// Registers: launched at 128 per thread (512 x 128 = 65536); warpgroup 0 (MMA issuer, allocator) gives back
// to 56, the row threads and the splitters take 152: 128 x 56 + 384 x 152 = 65536.
constexpr uint32_t kRegsLow = 56, kRegsHigh = 152;
static_assert(128 * kRegsLow + 384 * kRegsHigh <= kThreads * 128, "register split exceeds the launch allotment");
constexpr int kKT = 64;  // keys per tile
constexpr int kSbo = 144;  // bytes between 8-row groups of a K block (128 + 16: conflict-free stores)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 8.f;  // rescale O once a row maximum grows by more than this (log2 units)
constexpr uint32_t kTfMask = 0xFFFFE000u;

// Bytes of one term of a K-major operand tile with `rows` rows (a multiple of 8) and `kvals` K-values.
__host__ __device__ constexpr int term_bytes(int rows, int kvals) { return (kvals / 4) * (rows / 8) * kSbo; }

template <int H, int W, int HD>
struct Geo {
  static constexpr bool kGlobal = (H == 64 && W == 64);
  static constexpr int kN = H * W;
  static constexpr int kTiles = (kN + kKT - 1) / kKT;
  static constexpr int kQTiles = (kN + 127) / 128;
  static constexpr int kVRows = HD + 16;  // v^T hi rows: dims, then ones
  // k: rows = 64 keys, K = HD dims; v^T: rows = dims, K = 64 keys (K block = 4 values)
  static constexpr int kKLbo = (kKT / 8) * kSbo, kVhiLbo = (kVRows / 8) * kSbo, kVloLbo = (HD / 8) * kSbo;
  static constexpr int kKTerm = term_bytes(kKT, HD), kVhiTerm = term_bytes(kVRows, kKT), kVloTerm = term_bytes(HD, kKT);
  static constexpr int kKSlot = 2 * kKTerm, kVSlot = kVhiTerm + kVloTerm;
  static constexpr int OFF_K = 0, OFF_V = 2 * kKSlot;
  // prologue only, over the k / v slots: the table (2h-1 + 2w-1 rows of HD), then the rows' rw scratch
  static constexpr int kTabBytes = (2 * H - 1 + 2 * W - 1) * HD * 4;
  static constexpr int OFF_RWTMP = (kTabBytes + 127) / 128 * 128;
  // the rows' bias projections in log2 units: rh [kh][128 rows]; windows also rw [kw][128 rows]
  static constexpr int OFF_RH = OFF_V + 2 * kVSlot;
  static constexpr int OFF_RW = OFF_RH + H * 128 * 4;
  static constexpr int OFF_RED = OFF_RW + (kGlobal ? 0 : W * 128 * 4);  // row-max exchange [2][2][128]
  static constexpr int OFF_BARS = OFF_RED + 2 * 2 * 128 * 4;
  static constexpr int kSmemBytes = OFF_BARS + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(OFF_RWTMP + (kGlobal ? W * 128 * 4 : 0) <= OFF_RH, "the table and the rw scratch must fit the slots");
  static_assert(kKSlot % 128 == 0 && kVhiTerm % 16 == 0 && kTabBytes % 16 == 0, "alignment");
  // TMEM columns
  static constexpr int T_S = 0, T_PLO = 128, T_O = 256, T_L = T_O + HD;
  static constexpr int T_QHI = T_O + (kVRows + 31) / 32 * 32, T_QLO = T_QHI + HD;
  static_assert(T_QLO + HD <= 512, "TMEM budget");
  // column split of O (+ l) and of q between the two halves: [0, 48) and [48, end)
  static constexpr int kColSplit = 48;
};

// Byte offset of the granule (row n, K block kb) in a term with K blocks `lbo` bytes apart.
__device__ __forceinline__ int granule(int n, int kb, int lbo) { return kb * lbo + (n >> 3) * kSbo + (n & 7) * 16; }

struct Bars {
  uint64_t k_ready[2], k_empty[2], v_ready[2], v_empty[2];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t pair[4][2];  // row-max exchange of lane quarter q, tile parity
  uint64_t q_ready, tab_full, tab_free, rows_done, final_mma;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & kTfMask;
  lo = __float_as_uint(x - __uint_as_float(hi)) & kTfMask;
}

// q . t for a table row in shared memory (all lanes read the same row: a broadcast)
template <int HD>
__device__ __forceinline__ float dot_row(const float (&q)[HD], const float* t) {
  const float4* t4 = reinterpret_cast<const float4*>(t);
  float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < HD / 4; ++c) {
    const float4 v = t4[c];
    a[c & 3] = fmaf(q[4 * c], v.x, a[c & 3]);
    a[c & 3] = fmaf(q[4 * c + 1], v.y, a[c & 3]);
    a[c & 3] = fmaf(q[4 * c + 2], v.z, a[c & 3]);
    a[c & 3] = fmaf(q[4 * c + 3], v.w, a[c & 3]);
  }
  return (a[0] + a[1]) + (a[2] + a[3]);
}

// q . t0 and q . t1 for two table rows in shared memory, interleaved (two independent FMA chains each).
template <int HD>
__device__ __forceinline__ float2 dot_rows2(const float (&q)[HD], const float* t0, const float* t1) {
  const float4* a4 = reinterpret_cast<const float4*>(t0);
  const float4* b4 = reinterpret_cast<const float4*>(t1);
  float a[2] = {0.f, 0.f}, b[2] = {0.f, 0.f};
#pragma unroll
  for (int c = 0; c < HD / 4; ++c) {
    const float4 u = a4[c], v = b4[c];
    a[c & 1] = fmaf(q[4 * c], u.x, a[c & 1]);
    b[c & 1] = fmaf(q[4 * c], v.x, b[c & 1]);
    a[c & 1] = fmaf(q[4 * c + 1], u.y, a[c & 1]);
    b[c & 1] = fmaf(q[4 * c + 1], v.y, b[c & 1]);
    a[c & 1] = fmaf(q[4 * c + 2], u.z, a[c & 1]);
    b[c & 1] = fmaf(q[4 * c + 2], v.z, b[c & 1]);
    a[c & 1] = fmaf(q[4 * c + 3], u.w, a[c & 1]);
    b[c & 1] = fmaf(q[4 * c + 3], v.w, b[c & 1]);
  }
  return make_float2(a[0] + a[1], b[0] + b[1]);
}

// Splitter of one operand (64 threads). A block = 4 source rows x 4 consecutive values: k: 4 dims x 4 keys
// of kt [hd][n]; v: 4 keys x 4 dims of v [n][hd]. Transposed, each block gives 4 granules (4 K-values of one
// operand row): k rows are keys (K = dims), v^T rows are dims (K = keys).
template <int H, int W, int HD, bool kK>
struct Splitter {
  using G = Geo<H, W, HD>;
  static constexpr int kBlocks = (kKT / 4) * (HD / 4) / 64;  // per thread and tile
  float4 x[kBlocks][4];

  // block b: key group kg (4 keys), dim group dg (4 dims); k blocks run over keys fastest, v over dims
  __device__ __forceinline__ void coords(int b, int& kg, int& dg) const {
    if constexpr (kK) {
      kg = b % (kKT / 4);
      dg = b / (kKT / 4);
    } else {
      dg = b % (HD / 4);
      kg = b / (HD / 4);
    }
  }

  __device__ __forceinline__ void load(const float* __restrict__ src, int tid, int t) {
#pragma unroll
    for (int i = 0; i < kBlocks; ++i) {
      int kg, dg;
      coords(tid + 64 * i, kg, dg);
      const int key = kKT * t + 4 * kg;  // G::kN is a multiple of 4: a block is all in or all out
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float* p = kK ? src + (long)(4 * dg + c) * G::kN + key : src + (long)(key + c) * HD + 4 * dg;
        x[i][c] = key < G::kN ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }

  __device__ __forceinline__ void store(uint8_t* hi, uint8_t* lo, int tid) const {
#pragma unroll
    for (int i = 0; i < kBlocks; ++i) {
      int kg, dg;
      coords(tid + 64 * i, kg, dg);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // operand row: key 4 kg + e (k) or dim 4 dg + e (v^T); its 4 K-values: x[i][0..3].e
        const float v0 = e == 0 ? x[i][0].x : e == 1 ? x[i][0].y : e == 2 ? x[i][0].z : x[i][0].w;
        const float v1 = e == 0 ? x[i][1].x : e == 1 ? x[i][1].y : e == 2 ? x[i][1].z : x[i][1].w;
        const float v2 = e == 0 ? x[i][2].x : e == 1 ? x[i][2].y : e == 2 ? x[i][2].z : x[i][2].w;
        const float v3 = e == 0 ? x[i][3].x : e == 1 ? x[i][3].y : e == 2 ? x[i][3].z : x[i][3].w;
        uint4 h, l;
        split_tf32(v0, h.x, l.x);
        split_tf32(v1, h.y, l.y);
        split_tf32(v2, h.z, l.z);
        split_tf32(v3, h.w, l.w);
        if constexpr (kK) {
          const int off = granule(4 * kg + e, dg, G::kKLbo);
          *reinterpret_cast<uint4*>(hi + off) = h;
          *reinterpret_cast<uint4*>(lo + off) = l;
        } else {
          *reinterpret_cast<uint4*>(hi + granule(4 * dg + e, kg, G::kVhiLbo)) = h;
          *reinterpret_cast<uint4*>(lo + granule(4 * dg + e, kg, G::kVloLbo)) = l;
        }
      }
    }
  }
};

template <int H, int W, int HD>
__global__ void __launch_bounds__(kThreads, 1)
    relpos_attn_f32(const float* __restrict__ qg, const float* __restrict__ ktg, const float* __restrict__ vg,
                    const float* __restrict__ table, float* __restrict__ out, float scale) {
  using namespace sm100;
  using G = Geo<H, W, HD>;
  extern __shared__ uint8_t smem_raw[];
  if (__syncthreads_or(threadIdx.x == 0 && device_faulted())) return;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + G::OFF_BARS);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % G::kQTiles;
  const int bh = blockIdx.x / G::kQTiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_ready[s], 64);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_ready[s], 64);
      mbar_init(&bars->v_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 256);
      mbar_init(&bars->pv_done[s], 1);
      for (int q = 0; q < 4; ++q) mbar_init(&bars->pair[q][s], 64);
    }
    mbar_init(&bars->q_ready, 256);
    mbar_init(&bars->tab_full, 1);
    mbar_init(&bars->tab_free, 256);
    mbar_init(&bars->rows_done, 256);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    // the whole table over the (still unused) k / v slots
    mbar_arrive_expect_tx(&bars->tab_full, G::kTabBytes);
    bulk_load(smem + G::OFF_K, table, G::kTabBytes, &bars->tab_full);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  if (warp < 4)
    regs_dec<kRegsLow>();
  else
    regs_inc<kRegsHigh>();

  if (warp == 0) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idS = idesc_tf32(128, kKT, false);
    constexpr uint32_t idPV = idesc_tf32(128, HD, false);
    constexpr uint32_t idPVL = idesc_tf32(128, G::kVRows, false);  // with the ones rows: O and l
    const uint32_t sb = smem_u32(smem);
    // K-major, no swizzle: 8-row groups kSbo apart (SBO), 4-value K blocks LBO apart; a K step of 8 spans two
    // K blocks
    const uint64_t dK = smem_desc(sb + G::OFF_K, G::kKLbo, kSbo, kLayoutNone);
    const uint64_t dVhi = smem_desc(sb + G::OFF_V, G::kVhiLbo, kSbo, kLayoutNone);
    const uint64_t dVlo = smem_desc(sb + G::OFF_V + G::kVhiTerm, G::kVloLbo, kSbo, kLayoutNone);
    // lane 0 polls, the warp follows (warp-uniform decisions)
    auto ready = [&](uint64_t* bar, uint32_t parity) {
      return __shfl_sync(0xffffffffu, lane == 0 ? (int)mbar_try_wait(bar, parity) : 0, 0) != 0;
    };
    auto issue_s = [&](int t) {
      const int s = t & 1;
#pragma unroll
      for (int pr = 0; pr < 3; ++pr) {  // q lo . k hi, q hi . k lo, q hi . k hi
#pragma unroll
        for (int ks = 0; ks < HD / 8; ++ks)
          mma_ts_tf32_w(tmem + G::T_S + kKT * s, tmem + (pr == 0 ? G::T_QLO : G::T_QHI) + 8 * ks,
                        desc_add(dK, s * G::kKSlot + (pr == 1 ? G::kKTerm : 0) + ks * 2 * G::kKLbo), idS,
                        (pr > 0 || ks > 0) ? 1u : 0u);
      }
      mma_commit_w(&bars->s_full[s]);
      mma_commit_w(&bars->k_empty[s]);  // the k slot may be rewritten once these MMAs completed
    };
    auto issue_pv = [&](int u) {
      const int s = u & 1;
#pragma unroll
      for (int pr = 0; pr < 3; ++pr) {  // p lo . v hi (+ l), p hi . v lo, p hi . v hi (+ l)
#pragma unroll
        for (int ks = 0; ks < kKT / 8; ++ks) {
          const uint32_t a = tmem + (pr == 0 ? G::T_PLO : G::T_S) + kKT * s + 8 * ks;
          if (pr == 1)
            mma_ts_tf32_w(tmem + G::T_O, a, desc_add(dVlo, s * G::kVSlot + ks * 2 * G::kVloLbo), idPV, 1u);
          else
            mma_ts_tf32_w(tmem + G::T_O, a, desc_add(dVhi, s * G::kVSlot + ks * 2 * G::kVhiLbo), idPVL,
                          (u > 0 || pr > 0 || ks > 0) ? 1u : 0u);
        }
      }
      mma_commit_w(&bars->pv_done[s]);
      mma_commit_w(&bars->v_empty[s]);  // the v slot may be rewritten once these MMAs completed
    };
    bool okk = __all_sync(0xffffffffu, mbar_wait(&bars->q_ready, 0, abort_flag));
    tc_fence_after();
    // S(t) writes the S / P-hi buffer of tile t - 2, so it needs PV(t - 2) issued (in-order execution of the
    // MMAs does the rest); otherwise S and P.V go as soon as their inputs are ready.
    int ns = 0, np = 0;
    long long t0 = clock64();
    const long long limit = wait_limit();
    for (uint32_t it = 0; okk && np < G::kTiles; ++it) {
      if (np < ns && ready(&bars->p_full[np & 1], (np >> 1) & 1) && ready(&bars->v_ready[np & 1], (np >> 1) & 1)) {
        tc_fence_after();
        issue_pv(np++);
        t0 = clock64();
      } else if (ns < G::kTiles && ns <= np + 1 && ready(&bars->k_ready[ns & 1], (ns >> 1) & 1)) {
        tc_fence_after();
        issue_s(ns++);
        t0 = clock64();
      } else if ((it & 255u) == 0) {
        const bool bad = *abort_flag || device_faulted();
        if (bad || clock64() - t0 > limit) {
          if (!bad && lane == 0) report(kStatusWaitTimeout);
          *abort_flag = 1;
          okk = false;
        }
      }
    }
    // every MMA issued by this warp has completed before the CTA tears down TMEM
    mma_commit_w(&bars->final_mma);
    mbar_drain(&bars->final_mma, 0);
  } else if (warp >= 12) {
    // ------------------------------------------------------------------ k / v splitters
    const bool is_k = warp < 14;
    const int tid = threadIdx.x - (is_k ? 384 : 448);
    auto run = [&](auto& sp, const float* src, int off, int slot, uint64_t* rdy, uint64_t* emp) {
      sp.load(src, tid, 0);
      // the slots hold the table and the rw scratch until the row threads are done with them
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->tab_free, 0, abort_flag))) return;
      if (!is_k) {
        // the ones rows of the v^T hi term (rows HD .. HD+15 of every K block, both slots), written once
        for (int g = tid; g < 2 * 16 * 16; g += 64)
          *reinterpret_cast<uint4*>(smem + off + (g >> 8) * slot + granule(HD + (g & 15), (g >> 4) & 15, G::kVhiLbo)) =
              make_uint4(0x3f800000u, 0x3f800000u, 0x3f800000u, 0x3f800000u);
      }
      for (int t = 0; t < G::kTiles; ++t) {
        const int s = t & 1;
        if (t >= 2 && !__all_sync(0xffffffffu, mbar_wait(&emp[s], ((t >> 1) - 1) & 1, abort_flag))) break;
        uint8_t* hi = smem + off + s * slot;
        sp.store(hi, hi + (is_k ? G::kKTerm : G::kVhiTerm), tid);
        fence_proxy_async_smem();  // the MMAs (async proxy) read what these threads wrote
        mbar_arrive(&rdy[s]);
        if (t + 1 < G::kTiles) sp.load(src, tid, t + 1);
      }
    };
    if (is_k) {
      Splitter<H, W, HD, true> sp;
      run(sp, ktg + (long)bh * HD * G::kN, G::OFF_K, G::kKSlot, bars->k_ready, bars->k_empty);
    } else {
      Splitter<H, W, HD, false> sp;
      run(sp, vg + (long)bh * G::kN * HD, G::OFF_V, G::kVSlot, bars->v_ready, bars->v_empty);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ row threads
    const int rq = warp & 3, hf = (warp - 4) >> 2;  // lane quarter, key half
    const int r = 32 * rq + lane;                   // TMEM lane = query row within the tile
    const int row = qt * 128 + r;
    const bool valid = row < G::kN;
    const uint32_t tl = tmem + ((uint32_t)(32 * rq) << 16);
    const long row_off = ((long)bh * G::kN + (valid ? row : 0)) * HD;
    float* srh = reinterpret_cast<float*>(smem + G::OFF_RH);
    float* srw = reinterpret_cast<float*>(smem + G::OFF_RW);
    float* srwtmp = reinterpret_cast<float*>(smem + G::OFF_K + G::OFF_RWTMP);
    float* sred = reinterpret_cast<float*>(smem + G::OFF_RED);
    const float* stab = reinterpret_cast<const float*>(smem + G::OFF_K);
    // the bias in registers: 64x64 layers rw of this half's 32 keys; windows all of rh and rw
    float rwr[G::kGlobal ? 32 : 1], rh2[G::kGlobal ? 1 : H], rw2[G::kGlobal ? 1 : W];
    bool okk;
    {
      float q[HD];
      const float4* q4 = reinterpret_cast<const float4*>(qg + row_off);
#pragma unroll
      for (int c = 0; c < HD / 4; ++c) {
        const float4 v = valid ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        q[4 * c] = v.x;
        q[4 * c + 1] = v.y;
        q[4 * c + 2] = v.z;
        q[4 * c + 3] = v.w;
      }
      // q hi / lo into TMEM (A operand of the S MMAs): half hf writes columns [48 hf, ...)
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
        if ((c0 < G::kColSplit) == (hf == 0)) {
          uint32_t h[16], l[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) split_tf32(q[c0 + c], h[c], l[c]);
          tmem_st16(tl + G::T_QHI + c0, h);
          tmem_st16(tl + G::T_QLO + c0, l);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->q_ready);
      // Bias projections. Row (i, j) needs Th[i - kh + h - 1] (table rows i .. i + h - 1) and
      // Tw[j - kw + w - 1] (rows j .. j + w - 1). A warp walks the union of its rows' ranges one table row at
      // a time, so that all lanes read the same row (a broadcast), and each lane keeps the rows in its range.
      const int i = valid ? row / W : 0, j = valid ? row - (row / W) * W : 0;
      constexpr int kBig = 1 << 20;
      const int i_lo = __reduce_min_sync(0xffffffffu, valid ? i : kBig);
      const int i_hi = __reduce_max_sync(0xffffffffu, valid ? i : -1);
      const int j_lo = __reduce_min_sync(0xffffffffu, valid ? j : kBig);
      const int j_hi = __reduce_max_sync(0xffffffffu, valid ? j : -1);
      okk = __all_sync(0xffffffffu, mbar_wait(&bars->tab_full, 0, abort_flag));
      if constexpr (G::kGlobal) {
        // rh: half hf takes kh in [32 hf, 32 hf + 32), table rows i + 63 - kh (the warp's rows share i)
        for (int mrow = i + 32 - 32 * hf; okk && mrow <= i + 63 - 32 * hf; mrow += 2) {  // 32 rows, in pairs
          const float2 d = dot_rows2<HD>(q, stab + mrow * HD, stab + (mrow + 1) * HD);
          srh[(i + 63 - mrow) * 128 + r] = d.x * kLog2e;
          srh[(i + 62 - mrow) * 128 + r] = d.y * kLog2e;
        }
        // rw of this half's keys kw in [32 hf, 32 hf + 32) (table rows j + 32 - 32 hf .. j + 63 - 32 hf) into
        // the row's own scratch
        // (63 rows in pairs: the last pair's second row, one past the range, is computed and not kept)
        for (int mrow = j_lo + 32 - 32 * hf; okk && mrow <= j_hi + 63 - 32 * hf; mrow += 2) {
          const float2 d = dot_rows2<HD>(q, stab + (2 * H - 1 + mrow) * HD, stab + (2 * H + mrow) * HD);
          const int kw = j + 63 - mrow;
          if (kw >= 32 * hf && kw < 32 * hf + 32) srwtmp[kw * 128 + r] = d.x * kLog2e;
          if (kw - 1 >= 32 * hf && kw - 1 < 32 * hf + 32) srwtmp[(kw - 1) * 128 + r] = d.y * kLog2e;
        }
      } else {
        // windows: half 0 computes rh, half 1 rw; both read all of them back into registers below
        if (!valid) {
          for (int k = 0; k < (hf ? W : H); ++k) (hf ? srw : srh)[k * 128 + r] = 0.f;
        }
        if (hf == 0) {
          for (int mrow = i_lo; okk && mrow <= i_hi + H - 1; ++mrow) {
            const float d = dot_row<HD>(q, stab + mrow * HD) * kLog2e;
            const int kh = i + H - 1 - mrow;
            if (valid && kh >= 0 && kh < H) srh[kh * 128 + r] = d;
          }
        } else {
          for (int mrow = j_lo; okk && mrow <= j_hi + W - 1; ++mrow) {
            const float d = dot_row<HD>(q, stab + (2 * H - 1 + mrow) * HD) * kLog2e;
            const int kw = j + W - 1 - mrow;
            if (valid && kw >= 0 && kw < W) srw[kw * 128 + r] = d;
          }
        }
      }
    }
    if constexpr (G::kGlobal) {
#pragma unroll
      for (int c = 0; c < 32; ++c) rwr[c] = srwtmp[(32 * hf + c) * 128 + r];
    }
    mbar_arrive(&bars->tab_free);  // this thread is done with the table and its scratch
    // all rows' rh (and, for windows, rw) are in shared memory
    mbar_arrive(&bars->rows_done);
    okk = __all_sync(0xffffffffu, okk && mbar_wait(&bars->rows_done, 0, abort_flag));
    if constexpr (!G::kGlobal) {
#pragma unroll
      for (int k = 0; k < H; ++k) rh2[k] = srh[k * 128 + r];
#pragma unroll
      for (int k = 0; k < W; ++k) rw2[k] = srw[k * 128 + r];
    }
    const float sc = scale * kLog2e;
    float m = -INFINITY;

    // One key tile: this half's 32 scores + bias (log2 units), the row maximum shared with the other half,
    // P = 2^(x - m) split into TMEM.
    auto tile = [&](int t, auto&& bias) {
      const int b = t & 1;
      if (!(okk = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[b], (t >> 1) & 1, abort_flag)))) return;
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(tl + G::T_S + kKT * b + 32 * hf, sv);
      tmem_wait_ld_regs(sv);
      float x[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) x[c] = bias(c, __uint_as_float(sv[c]) * sc);
      float mt = x[0];
#pragma unroll
      for (int c = 1; c < 32; ++c) mt = fmaxf(mt, x[c]);
      sred[(b * 2 + hf) * 128 + r] = mt;
      mbar_arrive(&bars->pair[rq][b]);
      if (!(okk = __all_sync(0xffffffffu, mbar_wait(&bars->pair[rq][b], (t >> 1) & 1, abort_flag)))) return;
      mt = fmaxf(mt, sred[(b * 2 + (hf ^ 1)) * 128 + r]);
      if (t == 0) {
        m = mt;
      } else {
        const bool need = mt > m + kLazy;
        if (__any_sync(0xffffffffu, need)) {
          // O holds the products of tiles < t: rescale this half's columns of O (and l) to the new maximum
          // once PV(t-1) is done. Both halves of a row take the same decision (same mt, same m).
          if (!(okk = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag))))
            return;
          tc_fence_after();
          const float f = need ? ex2(m - mt) : 1.f;
          if (need) m = mt;
#pragma unroll
          for (int c0 = 0; c0 < G::kVRows; c0 += 16) {
            if ((c0 < G::kColSplit) == (hf == 0)) {
              uint32_t o[16];
              tmem_ld16(tl + G::T_O + c0, o);
              tmem_wait_ld_regs(o);
#pragma unroll
              for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
              tmem_st16(tl + G::T_O + c0, o);
            }
          }
          tmem_wait_st();
        }
      }
      // ex2.approx: relative error near 2^-22, far inside the f32 bar
#pragma unroll
      for (int c0 = 0; c0 < 32; c0 += 16) {
        uint32_t h[16], lo[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) split_tf32(ex2(x[c0 + c] - m), h[c], lo[c]);
        tmem_st16(tl + G::T_S + kKT * b + 32 * hf + c0, h);
        tmem_st16(tl + G::T_PLO + kKT * b + 32 * hf + c0, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[b]);
    };

    if constexpr (G::kGlobal) {
      for (int t = 0; t < G::kTiles && okk; ++t) {
        const float rh = srh[t * 128 + r];
        tile(t, [&](int c, float s) { return s + rh + rwr[c]; });
      }
    } else {
      static_for<0, G::kTiles>([&](auto tt) {
        constexpr int t = decltype(tt)::value;
        if (okk)
          tile(t, [&](int c, float s) {
            // keys kKT t + 32 hf + c; hf is not compile-time, so both halves' keys are formed and selected
            const int k0 = kKT * t + c, k1 = kKT * t + 32 + c;
            const float b0 = k0 < G::kN ? rh2[k0 / W] + rw2[k0 % W] : -INFINITY;
            const float b1 = k1 < G::kN ? rh2[k1 / W] + rw2[k1 % W] : -INFINITY;
            return s + (hf ? b1 : b0);
          });
      });
    }

    if (okk && __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[(G::kTiles - 1) & 1], ((G::kTiles - 1) >> 1) & 1,
                                                 abort_flag))) {
      tc_fence_after();
      uint32_t lv[16];
      tmem_ld16(tl + G::T_L, lv);
      tmem_wait_ld_regs(lv);
      const float inv = 1.f / __uint_as_float(lv[0]);
      float4* o4 = reinterpret_cast<float4*>(out + row_off);
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
        if ((c0 < G::kColSplit) == (hf == 0)) {
          uint32_t o[16];
          tmem_ld16(tl + G::T_O + c0, o);
          tmem_wait_ld_regs(o);
          if (valid) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              o4[c0 / 4 + c] = make_float4(__uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv,
                                           __uint_as_float(o[4 * c + 2]) * inv, __uint_as_float(o[4 * c + 3]) * inv);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tcf
}  // namespace samrs
