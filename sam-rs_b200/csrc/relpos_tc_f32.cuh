// relpos_tc_f32.cuh - tcgen05 kernel for f32 I/O (SAM's 64x64 global and 14x14 windowed layers, head_dim 64
// or 80). The two contractions run on the tensor cores as kind::tf32 MMAs with every f32 operand split in
// two TF32 terms, x = hi + lo (hi: x with its 13 low mantissa bits cleared; lo: x - hi, cleared the same
// way), and every product taken as lo.hi + hi.lo + hi.hi ("3xTF32"). The dropped lo.lo term and the
// truncation of lo leave a relative error near 2^-20 per product term; softmax, bias and normalisation are
// f32 on the CUDA cores.
//
// Math (src/kernels.rs:131-225, the f32 body of `attention_relpos_cpu`, as the f16/bf16 kernels):
//   x[r,k] = scale * q_r . k_k + q_r . Th[i-kh+h-1] + q_r . Tw[j-kw+w-1],  r = w i + j, k = w kh + kw
//   out_r  = sum_k softmax_k(x[r, .]) v_k
//
// CTA = one head x 128 query rows; key tiles of 64 keys (a 64x64 layer: tile t = grid row kh = t, 64 tiles;
// a 14x14 window: 4 tiles, keys 196..255 masked). kind::tf32 takes its shared-memory operand K-major only
// (an MN-major B operand reads as zeros on sm_100a), so both kt ([hd][keys]) and v ([keys][hd]) are
// transposed on the way in. Warps:
//   0      MMA issuer: S_t = Q K_t^T (A = q from TMEM, B = k K-major), then O += P_{t-1} V_{t-1}
//          (A = P from TMEM, B = v^T K-major); three TF32 products each
//   1      TMEM allocator (512 columns)
//   4-7    row threads (thread = query row = TMEM lane): the q row from HBM, its bias projections in f32 on
//          the CUDA cores (q.Th, q.Tw), q split into TMEM; per tile the softmax with a lazily rescaled
//          running maximum (O is rescaled only when a row's maximum grows by more than 2^8) and P split into
//          TMEM; at the end O / l to HBM
//   8-11   splitters: per key tile, coalesced loads of kt and v (L2-resident: the 32 query tiles of a head
//          share them), split, and 16-byte stores of hi and lo into the canonical no-swizzle K-major
//          layout (core matrix = 8 rows x 4 K-values): 16-byte granule g = kblock * rows + row, so the
//          lanes of a warp store consecutive granules. 2-stage ring.
// TMEM columns: S_t / P_t hi (2 buffers of 64), P_t lo (2 x 64), O (hd), q hi and q lo (hd each).
// Every wait is bounded (sm100::mbar_wait).
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace samrs {
namespace tcf {

constexpr int kThreads = 384;
constexpr int kKT = 64;  // keys per tile
constexpr int kStages = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 8.f;  // rescale O once a row maximum grows by more than this (log2 units)
constexpr uint32_t kTfMask = 0xFFFFE000u;

template <int H, int W, int HD>
struct Geo {
  static constexpr bool kGlobal = (H == 64 && W == 64);
  static constexpr int kN = H * W;
  static constexpr int kTiles = (kN + kKT - 1) / kKT;
  static constexpr int kQTiles = (kN + 127) / 128;
  static constexpr int kTileBytes = kKT * HD * 4;  // one term (hi or lo) of a k or v tile
  // a stage: k hi | k lo | v hi | v lo. k: rows = 64 keys, K = HD dims; v^T: rows = HD dims, K = 64 keys
  static constexpr int OFF_KHI = 0, OFF_KLO = kTileBytes, OFF_VHI = 2 * kTileBytes, OFF_VLO = 3 * kTileBytes;
  static constexpr int kStage = 4 * kTileBytes;
  // 64x64 layers: the row's bias projections, [kh][128 rows] and [kw/4][128 rows][4] f32 (log2 units)
  static constexpr int OFF_RH = kStages * kStage;
  static constexpr int kRBytes = kGlobal ? H * 128 * 4 : 0;
  static constexpr int OFF_RW = OFF_RH + kRBytes;
  static constexpr int OFF_BARS = OFF_RW + kRBytes;
  static constexpr int kSmemBytes = OFF_BARS + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kTileBytes % 128 == 0, "core matrices need 128-byte alignment");
  // TMEM columns
  static constexpr int T_S = 0, T_PLO = 128, T_O = 256;
  static constexpr int T_QHI = T_O + (HD + 31) / 32 * 32, T_QLO = T_QHI + HD;
  static_assert(T_QLO + HD <= 512, "TMEM budget");
};

struct Bars {
  uint64_t kv_ready[kStages], kv_empty[kStages];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t q_ready, final_mma;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & kTfMask;
  lo = __float_as_uint(x - __uint_as_float(hi)) & kTfMask;
}

template <int HD>
__device__ __forceinline__ float dot_row(const float (&q)[HD], const float* __restrict__ t) {
  const float4* t4 = reinterpret_cast<const float4*>(t);
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int c = 0; c < HD / 4; ++c) {
    const float4 v = __ldg(t4 + c);
    a0 = fmaf(q[4 * c], v.x, a0);
    a1 = fmaf(q[4 * c + 1], v.y, a1);
    a0 = fmaf(q[4 * c + 2], v.z, a0);
    a1 = fmaf(q[4 * c + 3], v.w, a1);
  }
  return a0 + a1;
}

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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_ready[s], 128);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], 128);
      mbar_init(&bars->pv_done[b], 1);
    }
    mbar_init(&bars->q_ready, 128);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idS = idesc_tf32(128, kKT, false);
    constexpr uint32_t idPV = idesc_tf32(128, HD, false);
    const uint32_t sb = smem_u32(smem);
    // K-major, no swizzle: 8-row groups 128 B apart (SBO), 4-value K blocks rows * 16 B apart (LBO); a K step
    // of 8 spans two K blocks
    const uint64_t dK = smem_desc(sb, kKT * 16, 128, kLayoutNone);
    const uint64_t dV = smem_desc(sb + G::OFF_VHI, HD * 16, 128, kLayoutNone);
    auto wait = [&](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag)); };
    bool okk = wait(&bars->q_ready, 0);
    tc_fence_after();
    for (int t = 0; okk && t <= G::kTiles; ++t) {
      if (t < G::kTiles) {
        const int s = t & 1, b = t & 1;
        if (!(okk = wait(&bars->kv_ready[s], (t >> 1) & 1))) break;
        tc_fence_after();
#pragma unroll
        for (int pr = 0; pr < 3; ++pr) {  // q lo . k hi, q hi . k lo, q hi . k hi
#pragma unroll
          for (int ks = 0; ks < HD / 8; ++ks)
            mma_ts_tf32_w(tmem + G::T_S + kKT * b, tmem + (pr == 0 ? G::T_QLO : G::T_QHI) + 8 * ks,
                          desc_add(dK, s * G::kStage + (pr == 1 ? G::OFF_KLO : 0) + ks * (2 * kKT * 16)), idS,
                          (pr > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit_w(&bars->s_full[b]);
      }
      if (t >= 1) {
        const int u = t - 1, s = u & 1, b = u & 1;
        if (!(okk = wait(&bars->p_full[b], (u >> 1) & 1))) break;
        tc_fence_after();
#pragma unroll
        for (int pr = 0; pr < 3; ++pr) {  // p lo . v hi, p hi . v lo, p hi . v hi
#pragma unroll
          for (int ks = 0; ks < kKT / 8; ++ks)
            mma_ts_tf32_w(tmem + G::T_O, tmem + (pr == 0 ? G::T_PLO : G::T_S) + kKT * b + 8 * ks,
                          desc_add(dV, s * G::kStage + (pr == 1 ? G::kTileBytes : 0) + ks * (2 * HD * 16)), idPV,
                          (u > 0 || pr > 0 || ks > 0) ? 1u : 0u);
        }
        mma_commit_w(&bars->pv_done[b]);
        mma_commit_w(&bars->kv_empty[s]);  // the stage may be rewritten once these MMAs completed
      }
    }
    // every MMA issued by this warp has completed before the CTA tears down TMEM
    mma_commit_w(&bars->final_mma);
    mbar_drain(&bars->final_mma, 0);
  } else if (warp >= 8) {
    // ------------------------------------------------------------------ splitters
    const int tid = threadIdx.x - 256;
    const float* ktb = ktg + (long)bh * HD * G::kN;
    const float* vb = vg + (long)bh * G::kN * HD;
    for (int t = 0; t < G::kTiles; ++t) {
      const int s = t & 1;
      if (t >= kStages && !__all_sync(0xffffffffu, mbar_wait(&bars->kv_empty[s], ((t >> 1) - 1) & 1, abort_flag)))
        break;
      uint8_t* st = smem + s * G::kStage;
      const int key0 = kKT * t;
      // k: granule idx = dim block * 64 + key (row = key, K block = 4 dims)
      {
        float x[HD / 8][4];
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          const int idx = tid + 128 * i, key = key0 + (idx & (kKT - 1)), d0 = 4 * (idx / kKT);
#pragma unroll
          for (int c = 0; c < 4; ++c) x[i][c] = key < G::kN ? __ldg(ktb + (long)(d0 + c) * G::kN + key) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          const int idx = tid + 128 * i;
          uint4 h, l;
          split_tf32(x[i][0], h.x, l.x);
          split_tf32(x[i][1], h.y, l.y);
          split_tf32(x[i][2], h.z, l.z);
          split_tf32(x[i][3], h.w, l.w);
          reinterpret_cast<uint4*>(st + G::OFF_KHI)[idx] = h;
          reinterpret_cast<uint4*>(st + G::OFF_KLO)[idx] = l;
        }
      }
      // v^T: granule idx = key block * HD + dim (row = dim, K block = 4 keys)
      {
        float x[HD / 8][4];
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          const int idx = tid + 128 * i, kb = idx / HD, d = idx - kb * HD;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int key = key0 + 4 * kb + c;
            x[i][c] = key < G::kN ? __ldg(vb + (long)key * HD + d) : 0.f;
          }
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          const int idx = tid + 128 * i;
          uint4 h, l;
          split_tf32(x[i][0], h.x, l.x);
          split_tf32(x[i][1], h.y, l.y);
          split_tf32(x[i][2], h.z, l.z);
          split_tf32(x[i][3], h.w, l.w);
          reinterpret_cast<uint4*>(st + G::OFF_VHI)[idx] = h;
          reinterpret_cast<uint4*>(st + G::OFF_VLO)[idx] = l;
        }
      }
      fence_proxy_async_smem();  // the MMAs (async proxy) read what these threads wrote
      mbar_arrive(&bars->kv_ready[s]);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ row threads
    const int r = threadIdx.x - 128;  // TMEM lane
    const int row = qt * 128 + r;
    const bool valid = row < G::kN;
    const uint32_t tl = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    const long row_off = ((long)bh * G::kN + (valid ? row : 0)) * HD;
    float* srh = reinterpret_cast<float*>(smem + G::OFF_RH);
    float* srw = reinterpret_cast<float*>(smem + G::OFF_RW);
    float rh2[G::kGlobal ? 1 : H], rw2[G::kGlobal ? 1 : W];  // windowed layers: the bias in registers
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
      const int i = valid ? row / W : 0, j = valid ? row - (row / W) * W : 0;
      const float* th = table + (long)(i + H - 1) * HD;              // Th[i - kh + h - 1] = th - kh * HD
      const float* tw = table + (long)(2 * H - 1 + j + W - 1) * HD;  // Tw[j - kw + w - 1] = tw - kw * HD
      if constexpr (G::kGlobal) {
        for (int kh = 0; kh < H; ++kh) srh[kh * 128 + r] = dot_row<HD>(q, th - kh * HD) * kLog2e;
        for (int kw = 0; kw < W; kw += 4) {
          float4 v;
          v.x = dot_row<HD>(q, tw - kw * HD) * kLog2e;
          v.y = dot_row<HD>(q, tw - (kw + 1) * HD) * kLog2e;
          v.z = dot_row<HD>(q, tw - (kw + 2) * HD) * kLog2e;
          v.w = dot_row<HD>(q, tw - (kw + 3) * HD) * kLog2e;
          reinterpret_cast<float4*>(srw)[(kw / 4) * 128 + r] = v;
        }
      } else {
#pragma unroll
        for (int kh = 0; kh < H; ++kh) rh2[kh] = valid ? dot_row<HD>(q, th - kh * HD) * kLog2e : 0.f;
#pragma unroll
        for (int kw = 0; kw < W; ++kw) rw2[kw] = valid ? dot_row<HD>(q, tw - kw * HD) * kLog2e : 0.f;
      }
      // q hi / lo into TMEM (A operand of the S MMAs)
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
        uint32_t h[16], l[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) split_tf32(q[c0 + c], h[c], l[c]);
        tmem_st16(tl + G::T_QHI + c0, h);
        tmem_st16(tl + G::T_QLO + c0, l);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->q_ready);
    }
    const float sc = scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool okk = true;

    // One key tile: x = scores + bias (log2 units), the running maximum, P = 2^(x - m) split into TMEM.
    auto tile = [&](int t, auto&& bias) {
      const int b = t & 1;
      if (!(okk = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[b], (t >> 1) & 1, abort_flag)))) return;
      tc_fence_after();
      uint32_t s0[32], s1[32];
      tmem_ld32(tl + G::T_S + kKT * b, s0);
      tmem_ld32(tl + G::T_S + kKT * b + 32, s1);
      tmem_wait_ld_regs(s0);
      tmem_wait_ld_regs(s1);
      float x[kKT];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] = bias(c, __uint_as_float(s0[c]) * sc);
        x[32 + c] = bias(32 + c, __uint_as_float(s1[c]) * sc);
      }
      float mt = x[0];
#pragma unroll
      for (int c = 1; c < kKT; ++c) mt = fmaxf(mt, x[c]);
      if (t == 0) {
        m = mt;
      } else {
        const bool need = mt > m + kLazy;
        if (__any_sync(0xffffffffu, need)) {
          // O holds the products of tiles < t: rescale it (and l) to the new maximum once PV(t-1) is done
          if (!(okk = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort_flag))))
            return;
          tc_fence_after();
          const float f = need ? exp2f(m - mt) : 1.f;
          if (need) m = mt;
          l *= f;
#pragma unroll
          for (int c0 = 0; c0 < HD; c0 += 16) {
            uint32_t o[16];
            tmem_ld16(tl + G::T_O + c0, o);
            tmem_wait_ld_regs(o);
#pragma unroll
            for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
            tmem_st16(tl + G::T_O + c0, o);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int c0 = 0; c0 < kKT; c0 += 16) {
        uint32_t h[16], lo[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float p = exp2f(x[c0 + c] - m);
          l += p;
          split_tf32(p, h[c], lo[c]);
        }
        tmem_st16(tl + G::T_S + kKT * b + c0, h);
        tmem_st16(tl + G::T_PLO + kKT * b + c0, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[b]);
    };

    if constexpr (G::kGlobal) {
      for (int t = 0; t < G::kTiles && okk; ++t) {
        const float rh = srh[t * 128 + r];
        const float4* rw4 = reinterpret_cast<const float4*>(srw) + r;
        tile(t, [&](int c, float s) {
          const float4 w4 = rw4[(c / 4) * 128];
          const float w = (c & 3) == 0 ? w4.x : (c & 3) == 1 ? w4.y : (c & 3) == 2 ? w4.z : w4.w;
          return s + rh + w;
        });
      }
    } else {
      static_for<0, G::kTiles>([&](auto tt) {
        constexpr int t = decltype(tt)::value;
        if (okk)
          tile(t, [&](int c, float s) {
            const int k = kKT * t + c;  // compile-time after unrolling
            return k < G::kN ? s + rh2[k / W] + rw2[k % W] : -INFINITY;
          });
      });
    }

    if (okk && __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[(G::kTiles - 1) & 1], ((G::kTiles - 1) >> 1) & 1,
                                                 abort_flag))) {
      tc_fence_after();
      const float inv = 1.f / l;
      float4* o4 = reinterpret_cast<float4*>(out + row_off);
#pragma unroll
      for (int c0 = 0; c0 < HD; c0 += 16) {
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
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tcf
}  // namespace samrs
