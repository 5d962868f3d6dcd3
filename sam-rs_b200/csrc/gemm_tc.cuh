// gemm_tc.cuh - tcgen05 (sm_100a) GEMM with fused epilogues for the projections around the attention:
//   C[M, N] = A[M, K] . W[N, K]^T  (A: activations, W: a Linear weight as stored, [out, in]; both K-major)
// followed, in the same kernel, by one of the epilogues of the reference's encoder block
// (src/sam1/encoder.rs:73-85, 115-129):
//   kEpiBias          out = C + bias                         (Linear + bias)
//   kEpiBiasResidual  out = res + C + bias                   (proj / lin2 + `bias_residual`, kernels/sam.cu:129-135)
//   kEpiBiasGelu      out = gelu_erf(C + bias)               (lin1 + `bias_gelu`, kernels/sam.cu:136-143)
//   kEpiQkvWindow     q / kt / v = split(C + bias) written straight into the windowed attention layout
//                     (the qkv projection + `qkv_split`, kernels/sam.cu:108-128, on the real tokens of a
//                     window-partitioned grid, src/sam1/encoder.rs:132-140; the pad tokens are written by
//                     qkv_pad_fill_kernel, see window_io.cuh)
//
// Structure: persistent grid over output tiles, rows of A fastest-varying tiles sharing them back to back
// (the A tile stays in L2 across the N tiles of its row). By default a tile is 256 x 256 and belongs to a
// CTA pair (a cluster of two CTAs on two SMs, one cta_group::2 MMA of M = 256): each CTA loads its 128 rows of
// A and its 128 rows of W, so a pair reads W once per 256 rows instead of once per 128, and each SM stages
// 32 KB per k-step instead of 48 KB (6 stages in flight instead of 4). Where no 2-CTA cluster can be resident
// the same kernel runs one CTA per 128 x 256 tile. Warps:
//   warp 0   TMA producer: A [128 x 64] and W [128 x 64] (pair) or [256 x 64] boxes, 128-byte swizzle. A pair's
//            loads all complete on the leader's (rank 0's) full barrier.
//   warp 1   MMA issuer, leader only (the warp runs the loop, lane 0 issues): 4 x tcgen05.mma K=16 per stage,
//            N = 256, M = 256 (pair) or 128; commits go to the barriers of both CTAs of a pair.
//   warp 2   TMEM allocator (512 columns: two 256-column accumulators, so the epilogue of one tile overlaps
//            the main loop of the next; a pair allocates with cta_group::2 in both CTAs)
//   warps 4+ epilogue (epi_warps: 16 in the pair kernel and for the GELU, else 8): warps per TMEM lane quarter
//            each take a slice of the tile's columns; thread = output row (TMEM lane), 16-column groups read
//            with tcgen05.ld, the epilogue applied in f32, 16-byte stores of the row's columns. A pair's
//            epilogue warps hand the accumulator back on the leader's acc_empty barrier.
// No multicast anywhere; every wait on an mbarrier is bounded (sm100::mbar_wait).
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tgemm {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB: this CTA's 128 rows of A per stage
// Stage layout. One CTA: A [128 x 64] and W [256 x 64] (48 KB), 4 stages. CTA pair (cta_group::2, a 256 x 256
// tile per pair): each CTA holds its 128 rows of A and its 128 rows of W (32 KB), 6 stages.
__host__ __device__ constexpr int b_rows(bool pair) { return pair ? kBN / 2 : kBN; }
__host__ __device__ constexpr int stage_bytes(bool pair) { return kABytes + b_rows(pair) * kBK * 2; }
__host__ __device__ constexpr int stages(bool pair) { return pair ? 6 : 4; }
__host__ __device__ constexpr int smem_bytes(bool pair) { return stages(pair) * stage_bytes(pair) + 256 + 1024; }
__host__ __device__ constexpr int tile_m(bool pair) { return pair ? 2 * kBM : kBM; }
constexpr int kMaxStages = 6;
static_assert(smem_bytes(false) <= 232448 && smem_bytes(true) <= 232448, "shared memory budget");

enum Epi : int { kEpiBias = 0, kEpiBiasResidual = 1, kEpiBiasGelu = 2, kEpiQkvWindow = 3 };

// Epilogue warps per CTA: 16 (four per TMEM lane quarter) for the erf GELU, whose per-tile epilogue at
// K = 768 issues more instructions than the tile's main loop and needs the extra warps to hide latency, and
// for every epilogue of the CTA-pair kernel, whose main loop per tile is shorter (ViT-H qkv 1.34 -> 1.24 ms,
// lin2 1.46 -> 1.41 ms with 16 instead of 8); 8 for the others in the single-CTA kernel.
__host__ __device__ constexpr int epi_warps(int epi, bool pair = false) {
  return (epi == kEpiBiasGelu || pair) ? 16 : 8;
}
__host__ __device__ constexpr int threads_for(int epi, bool pair = false) { return 128 + 32 * epi_warps(epi, pair); }

// Window geometry of the qkv epilogue: token m = (image, y, x) of an H x W grid cut into ws x ws windows
// (ws = 0: the whole grid is one window), windows row-major per image over the grid padded up to multiples
// of ws; q, kt, v planes back to back in `out`, bh = window * nh + head.
struct QkvGeom {
  int h, w, ws_h, ws_w, nwh, nww, nh, hd;
  long plane;  // elements per q / kt / v plane
  int pairs;   // w even and the window width even (or one window): consecutive token pairs share a window row
};

struct Params {
  int M, N, K;
  int group;  // M blocks whose tiles of one N block run side by side (1: the tiles of an M block run together)
  int band_rows;  // rows of A that one group should cover (0: group = 1); the launch sets `group` from it
  const void* bias;  // [N]
  const void* res;   // [M, N] (kEpiBiasResidual)
  void* out;         // [M, N], or the packed q | kt | v planes (kEpiQkvWindow)
  QkvGeom g;
};

struct Bars {
  uint64_t full[kMaxStages], empty[kMaxStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t final_mma;
  uint32_t tmem_base;
  int abort_flag;
  int skip;  // CTA pair: rank 0's decision to leave at entry (a fault reported earlier), read by both CTAs
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float (&f)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  const uint4 a = q[0], b = q[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 f2 = __half22float2(h2);
      f[2 * i] = f2.x;
      f[2 * i + 1] = f2.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float (&f)[16]) {
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = sm100::pack2(f[2 * i], f[2 * i + 1], kBf16);
  uint4* q = reinterpret_cast<uint4*>(p);
  q[0] = make_uint4(w[0], w[1], w[2], w[3]);
  q[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// Exact (erf) GELU, as the reference's bias_gelu: 0.5 x (1 + erf(x / sqrt 2)).
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

// The epilogue of 16 columns n0 .. n0 + 15 of row m (v: the f32 accumulators). The per-row window position
// of the qkv epilogue (bh base and token index within the window) is computed once per tile row.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4 (&q)[2], float (&f)[16]) {
  const uint32_t w[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = f2.x;
      f[2 * i + 1] = f2.y;
    }
  }
}

template <typename T, int EPI>
__device__ __forceinline__ void epilogue16(const Params& p, bool row_ok, int m, int n0, float (&v)[16], long win_base,
                                           int n_in, int npw, const uint4 (&res)[2]) {
  if (EPI != kEpiQkvWindow && !row_ok) return;
  float b[16];
  load16(static_cast<const T*>(p.bias) + n0, b);
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] += b[j];
  if constexpr (EPI == kEpiBias) {
    store16(static_cast<T*>(p.out) + (long)m * p.N + n0, v);
  } else if constexpr (EPI == kEpiBiasResidual) {
    float r[16];
    unpack16<T>(res, r);  // loaded before the tile's accumulator was ready
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] += r[j];
    store16(static_cast<T*>(p.out) + (long)m * p.N + n0, v);
  } else if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = gelu_erf(v[j]);
    store16(static_cast<T*>(p.out) + (long)m * p.N + n0, v);
  } else {
    // column n0 -> (q / k / v, head, first dim); 16-column groups never straddle a head (hd % 16 == 0)
    const int c = p.g.nh * p.g.hd;
    const int which = n0 / c, cc = n0 - which * c;
    const int head = cc / p.g.hd, d0 = cc - head * p.g.hd;
    const long bh = win_base + head;
    T* base = static_cast<T*>(p.out) + which * p.g.plane;
    if (which == 1 && p.g.pairs) {
      // kt [bh][hd][n]: a token's 16 dims are npw elements apart. Lanes 2p and 2p+1 hold tokens x and x+1 of
      // one grid row (x even; the rows of a lane pair are consecutive tokens), which share a window row when
      // the window side is even, so they trade halves and each stores 8 dims of the token pair as 4-byte
      // words: the even lane dims 0..7, the odd lane dims 8..15, both at the even lane's token.
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const int lane = threadIdx.x & 31;
      const bool odd = lane & 1;
      uint32_t own[8], oth[4];
#pragma unroll
      for (int j = 0; j < 8; ++j) own[j] = sm100::pack2(v[2 * j], v[2 * j + 1], kBf16);  // dims 2j, 2j+1
#pragma unroll
      for (int j = 0; j < 4; ++j) oth[j] = __shfl_xor_sync(0xffffffffu, odd ? own[j] : own[4 + j], 1);
      T* dst = base + (bh * p.g.hd + d0 + (odd ? 8 : 0)) * (long)npw + (n_in - (odd ? 1 : 0));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // dim (odd ? 8 : 0) + j of the even token (lo) and the odd token (hi)
        const uint32_t mine = odd ? own[4 + (j >> 1)] : own[j >> 1], theirs = oth[j >> 1];
        const uint32_t ev = odd ? theirs : mine, od = odd ? mine : theirs;
        const uint32_t w = (j & 1) ? ((ev >> 16) | (od & 0xFFFF0000u)) : ((ev & 0xFFFFu) | (od << 16));
        if (row_ok) *reinterpret_cast<uint32_t*>(dst + (long)j * npw) = w;
      }
    } else if (!row_ok) {
      return;
    } else if (which == 1) {
      T* dst = base + (bh * p.g.hd + d0) * (long)npw + n_in;
#pragma unroll
      for (int j = 0; j < 16; ++j) dst[(long)j * npw] = from_f<T>(v[j]);
    } else {
      store16(base + (bh * npw + n_in) * (long)p.g.hd + d0, v);
    }
  }
}

// Tile t -> (M block, N block). Groups of p.group M blocks: within a group the N block varies slowest, so
// the group's M blocks of one N block are computed at the same time (the qkv epilogue's band of window rows:
// each k^T row of a window is then written whole within one wave), and with p.group = 1 the N blocks of one
// M block run back to back (its A tile stays in L2).
__device__ __forceinline__ void tile_coords(const Params& p, int m_blocks, int n_blocks, int t, int& m0, int& n0,
                                            int bm = kBM) {
  const int gsize = p.group * n_blocks;
  const int grp = t / gsize, r = t - grp * gsize;
  const int gm = m_blocks - grp * p.group < p.group ? m_blocks - grp * p.group : p.group;  // M blocks in the group
  const int nb = r / gm, mb = grp * p.group + (r - nb * gm);
  m0 = mb * bm;
  n0 = nb * kBN;
}

template <typename T, int EPI, bool kPair>
__global__ void __launch_bounds__(threads_for(EPI, kPair), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using namespace sm100;
  constexpr int kEpiWarps = epi_warps(EPI, kPair);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int kStages = stages(kPair), kStageBytes = stage_bytes(kPair), kTM = tile_m(kPair);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kStages * kStageBytes);
  volatile int* abort_flag = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA pair: rank 0 (the leader) issues the pair's MMAs and owns the full and acc_empty barriers; both CTAs
  // load their halves of A and W, and run the epilogue of their 128 rows.
  const uint32_t rank = kPair ? cluster_rank() : 0;
  const bool leader = rank == 0;
  const int unit = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // the pair (or CTA) index
  const int n_units = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  if constexpr (!kPair) {
    if (__syncthreads_or(threadIdx.x == 0 && device_faulted())) return;
  }
  const int m_blocks = (p.M + kTM - 1) / kTM, n_blocks = (p.N + kBN - 1) / kBN;
  const int tiles = m_blocks * n_blocks;
  const int nk = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], kPair ? 2 * kEpiWarps : kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    bars->skip = kPair && leader ? (int)device_faulted() : 0;
    fence_mbar_init();
  }
  if constexpr (kPair) {
    // Both CTAs leave together after an earlier CTA reported a fault (rank 0 decides; the second cluster
    // barrier keeps rank 0's shared memory alive until rank 1 has read the decision).
    cluster_sync();
    const int skip = ld_cluster_s32(cluster_addr(&bars->skip, 0));
    cluster_sync();
    if (skip) return;
    if (warp == 2) {
      tmem_alloc_pair(&bars->tmem_base, 512);
      tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs before any load or MMA
    tc_fence_after();
  } else {
    if (warp == 2) {
      tmem_alloc(&bars->tmem_base, 512);
      tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int it = 0;
      bool okk = true;
      for (int tile = unit; tile < tiles && okk; tile += n_units) {
        int m0, n0;
        tile_coords(p, m_blocks, n_blocks, tile, m0, n0, kTM);
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !mbar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, abort_flag)) {
            okk = false;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          if constexpr (kPair) {
            // both halves' bytes complete on the leader's barrier
            const uint32_t full = cluster_addr(&bars->full[s], 0);
            if (leader) mbar_arrive_expect_tx(&bars->full[s], 2 * kStageBytes);
            tma_load_2d_pair(st, &tmA, full, kb * kBK, m0 + kBM * (int)rank);
            tma_load_2d_pair(st + kABytes, &tmB, full, kb * kBK, n0 + (kBN / 2) * (int)rank);
          } else {
            mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
            tma_load_2d(st, &tmA, &bars->full[s], kb * kBK, m0);
            tma_load_2d(st + kABytes, &tmB, &bars->full[s], kb * kBK, n0);
          }
        }
      }
      if (*abort_flag && leader) {
        // drain the copies still in flight before the CTA can exit (a pair's copies all count on the leader)
        for (int j = it > kStages ? it - kStages : 0; j < it; ++j) mbar_drain(&bars->full[j % kStages], (j / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (leader) {
      constexpr uint32_t idesc = idesc_f16(kBf16, kTM, kBN, false, false);
      const uint32_t sb = smem_u32(smem);
      // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart; K steps of 16 advance 32 B
      const uint64_t dA = smem_desc(sb, 16, 1024, kLayoutSw128);
      const uint64_t dB = smem_desc(sb + kABytes, 16, 1024, kLayoutSw128);
      auto wait = [&](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag)); };
      // commit to a barrier of this CTA, and for a pair to the same barrier of the other CTA as well
      auto commit = [&](uint64_t* bar) {
        if constexpr (kPair) {
          mma_commit_pair_w(cluster_addr(bar, 0));
          mma_commit_pair_w(cluster_addr(bar, 1));
        } else {
          mma_commit_w(bar);
        }
      };
      int it = 0, ti = 0;
      bool okk = true;
      for (int tile = unit; tile < tiles && okk; tile += n_units, ++ti) {
        const int ab = ti & 1;
        // the epilogue (of both CTAs) has read this accumulator's previous tile
        if (ti >= 2 && !(okk = wait(&bars->acc_empty[ab], ((ti >> 1) - 1) & 1))) break;
        tc_fence_after();
        const uint32_t tacc = tmem + ab * kBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % kStages;
          if (!(okk = wait(&bars->full[s], (it / kStages) & 1))) break;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t a = desc_add(dA, s * kStageBytes + 32 * k), bd = desc_add(dB, s * kStageBytes + 32 * k);
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            if constexpr (kPair)
              mma_ss_pair_w(tacc, a, bd, idesc, acc);
            else
              mma_ss_w(tacc, a, bd, idesc, acc);
          }
          commit(&bars->empty[s]);  // the stage may be refilled once these MMAs completed
        }
        if (!okk) break;
        commit(&bars->acc_full[ab]);
      }
      // every MMA issued by this warp has completed before the CTA (pair) tears down TMEM
      commit(&bars->final_mma);
    }
    mbar_drain(&bars->final_mma, 0);
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int wq = warp & 3;            // TMEM lane quarter
    const int half = (warp - 4) >> 2;  // column slice of the tile (kEpiWarps / 4 slices)
    constexpr int kGroups = kBN / 16 / (kEpiWarps / 4);
    int ti = 0;
    for (int tile = unit; tile < tiles; tile += n_units, ++ti) {
      const int ab = ti & 1;
      int m0, n0;
      tile_coords(p, m_blocks, n_blocks, tile, m0, n0, kTM);
      const int m = m0 + kBM * (int)rank + 32 * wq + lane;
      const bool row_ok = m < p.M;
      // the residual's columns of this thread, loaded while the tile's main loop still runs
      constexpr int kRes = EPI == kEpiBiasResidual ? kGroups : 1;
      uint4 res[kRes][2];
      if constexpr (EPI == kEpiBiasResidual) {
#pragma unroll
        for (int grp = 0; grp < kGroups; ++grp) {
          const int n = n0 + 16 * (kGroups * half + grp);
          if (row_ok && n < p.N) {
            const uint4* q = reinterpret_cast<const uint4*>(static_cast<const T*>(p.res) + (long)m * p.N + n);
            res[grp][0] = q[0];
            res[grp][1] = q[1];
          } else {
            res[grp][0] = res[grp][1] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->acc_full[ab], (ti >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      long win_base = 0;
      int n_in = 0, npw = 0;
      if constexpr (EPI == kEpiQkvWindow) {
        const QkvGeom& g = p.g;
        const int hw = g.h * g.w;
        const int img = m / hw, r = m - img * hw, y = r / g.w, x = r - y * g.w;
        const int wy = y / g.ws_h, wx = x / g.ws_w;
        win_base = ((long)img * g.nwh * g.nww + wy * g.nww + wx) * g.nh;
        n_in = (y - wy * g.ws_h) * g.ws_w + (x - wx * g.ws_w);
        npw = g.ws_h * g.ws_w;
      }
      const uint32_t tacc = tmem + ((uint32_t)(32 * wq) << 16) + ab * kBN + 16 * kGroups * half;
      uint32_t va[16], vb[16];
      tmem_ld16(tacc, va);
      static_for<0, kGroups>([&](auto gg) {
        constexpr int grp = decltype(gg)::value;
        uint32_t(&cur)[16] = (grp & 1) ? vb : va;
        uint32_t(&nxt)[16] = (grp & 1) ? va : vb;
        tmem_wait_ld_regs(cur);
        if constexpr (grp + 1 < kGroups) {
          tmem_ld16(tacc + 16 * (grp + 1), nxt);
        } else {
          // every column of this accumulator is in registers: hand it back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (kPair)
              mbar_arrive_cluster(cluster_addr(&bars->acc_empty[ab], 0));
            else
              mbar_arrive(&bars->acc_empty[ab]);
          }
        }
        const int n = n0 + 16 * (kGroups * half + grp);
        if (n < p.N) {  // warp-uniform (the qkv epilogue's lane pairs exchange values: every lane takes part)
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(cur[j]);
          epilogue16<T, EPI>(p, row_ok, m, n, v, win_base, n_in, npw, res[EPI == kEpiBiasResidual ? grp : 0]);
        }
      });
    }
  }
  tc_fence_before();
  if constexpr (kPair) {
    // neither CTA leaves while the pair's MMAs, copies or arrivals may still touch the other's memory
    cluster_sync();
    if (warp == 2) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, 512);
    }
  } else {
    __syncthreads();
    if (warp == 2) {
      tc_fence_after();
      tmem_dealloc(tmem, 512);
    }
  }
}

}  // namespace tgemm
}  // namespace samrs
