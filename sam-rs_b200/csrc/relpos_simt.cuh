// relpos_simt.cuh - CUDA-core kernels of the rel-pos attention path.
//
//  * relpos_attn_simt: fused flash-style attention with the decomposed rel-pos bias, any (h, w, hd<=128),
//    any dtype. It is the f32 path (f32 FMA arithmetic, expf) and the path for shapes the tensor-core
//    kernels do not cover. Math: src/kernels.rs:131-225 (cpu::TiledAttention), i.e.
//        x[r,k] = scale * q_r . kt[:,k] + q_r . Th[i-kh+h-1] + q_r . Tw[j-kw+w-1],  out_r = softmax_k(x) . v
//    computed with an online softmax over 64-key tiles, so no score row is ever stored.
//  * relpos_softmax_rows: the materialising probs-only op (src/kernels.rs:12-43 / 62-105,
//    kernels/sam.cu:44-106): one CTA per score row, two passes over the row (max/sum, then write).
//  * qkv_split: bias add + head split + K transpose (src/kernels.rs:234-263, kernels/sam.cu:108-128).
#pragma once
#include "common.cuh"

namespace samrs {

constexpr int kSimtBQ = 64;   // query rows per CTA
constexpr int kSimtBK = 64;   // keys per tile
constexpr int kSimtThreads = 256;
constexpr int kSimtMaxHd = 128;
constexpr int kPsStride = kSimtBK + 1;

// Dynamic shared memory (floats) of relpos_attn_simt.
__host__ __device__ inline size_t simt_smem_floats(int h, int w, int hd) {
  return (size_t)3 * kSimtBQ * hd + (size_t)kSimtBQ * kPsStride + (size_t)kSimtBQ * (h + w);
}

// grid.x = bh * ceil(n / 64); 256 threads. Thread (ty, tx) = (tid / 16, tid % 16) owns score rows
// ty*4..ty*4+3 x key columns tx*4..tx*4+3 of each tile, and output rows ty*4.. x columns tx + 16c.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) relpos_attn_simt(const T* __restrict__ q, const T* __restrict__ kt,
                                                                 const T* __restrict__ v,
                                                                 const T* __restrict__ table, T* __restrict__ out,
                                                                 int h, int w, int hd, float scale) {
  extern __shared__ float4 smem_f4[];
  float* smem = reinterpret_cast<float*>(smem_f4);
  const int n = h * w;
  const int qtiles = (n + kSimtBQ - 1) / kSimtBQ;
  const long bh = blockIdx.x / qtiles;
  const int r0 = (blockIdx.x % qtiles) * kSimtBQ;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

  float* Qs = smem;                          // [hd][64]  (transposed)
  float* Ks = Qs + kSimtBQ * hd;             // [hd][64]
  float* Vs = Ks + kSimtBK * hd;             // [64][hd]
  float* Ps = Vs + kSimtBK * hd;             // [64][65]
  float* rh_s = Ps + kSimtBQ * kPsStride;    // [64][h]
  float* rw_s = rh_s + kSimtBQ * h;          // [64][w]

  const T* qb = q + (bh * n) * hd;
  const T* ktb = kt + bh * (long)hd * n;
  const T* vb = v + (bh * n) * hd;

  // Q tile, transposed into Qs[d][r]; rows beyond n are zero.
  for (int idx = tid; idx < kSimtBQ * hd; idx += kSimtThreads) {
    const int r = idx % kSimtBQ, d = idx / kSimtBQ;
    const int row = r0 + r;
    Qs[d * kSimtBQ + r] = row < n ? to_f(qb[(long)row * hd + d]) : 0.f;
  }
  __syncthreads();
  // Rel-pos bias vectors of every row of the tile: rh_s[r][kh] = q_r . Th[i-kh+h-1], rw_s[r][kw] = q_r . Tw[j-kw+w-1].
  {
    const T* th = table;
    const T* tw = table + (long)(2 * h - 1) * hd;
    for (int idx = tid; idx < kSimtBQ * (h + w); idx += kSimtThreads) {
      const int r = idx % kSimtBQ, c = idx / kSimtBQ;
      const int row = r0 + r;
      const int i = row / w, j = row % w;
      const bool is_h = c < h;
      float acc = 0.f;
      if (row < n) {
        const T* trow = is_h ? th + (long)(i - c + h - 1) * hd : tw + (long)(j - (c - h) + w - 1) * hd;
        for (int d = 0; d < hd; ++d) acc = fmaf(Qs[d * kSimtBQ + r], to_f(trow[d]), acc);
      }
      if (is_h)
        rh_s[r * h + c] = acc;
      else
        rw_s[r * w + (c - h)] = acc;
    }
  }

  const int hdc = (hd + 15) / 16;  // output columns per thread (<= 8)
  float o[4][8];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 8; ++c) o[a][c] = 0.f;
  float m_run[4], l_run[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m_run[a] = -INFINITY;
    l_run[a] = 0.f;
  }

  for (int k0 = 0; k0 < n; k0 += kSimtBK) {
    __syncthreads();  // previous tile's Ks/Vs/Ps fully consumed (and rh/rw written on the first pass)
    for (int idx = tid; idx < kSimtBK * hd; idx += kSimtThreads) {
      const int k = idx % kSimtBK, d = idx / kSimtBK;
      Ks[d * kSimtBK + k] = (k0 + k) < n ? to_f(ktb[(long)d * n + k0 + k]) : 0.f;
    }
    for (int idx = tid; idx < kSimtBK * hd; idx += kSimtThreads) {
      const int k = idx / hd, d = idx % hd;
      Vs[k * hd + d] = (k0 + k) < n ? to_f(vb[(long)(k0 + k) * hd + d]) : 0.f;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) s[a][b] = 0.f;
    for (int d = 0; d < hd; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(&Qs[d * kSimtBQ + ty * 4]);
      const float4 kb = *reinterpret_cast<const float4*>(&Ks[d * kSimtBK + tx * 4]);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
      const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) s[a][b] = fmaf(qv[a], kv[b], s[a][b]);
    }
    // bias + scale, masked keys -> -inf
    int khs[4], kws[4];
    bool valid[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int key = k0 + tx * 4 + b;
      valid[b] = key < n;
      khs[b] = key / w;
      kws[b] = key - khs[b] * w;
    }
    float alpha[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int r = ty * 4 + a;
      float mt = -INFINITY;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float x = -INFINITY;
        if (valid[b]) x = s[a][b] * scale + rh_s[r * h + khs[b]] + rw_s[r * w + kws[b]];
        s[a][b] = x;
        mt = fmaxf(mt, x);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_run[a], mt);
      alpha[a] = expf(m_run[a] - m_new);  // exp(-inf) = 0 on the first tile
      m_run[a] = m_new;
      float ls = 0.f;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float p = expf(s[a][b] - m_new);
        ls += p;
        Ps[r * kPsStride + tx * 4 + b] = p;
      }
      l_run[a] = l_run[a] * alpha[a] + ls;
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 8; ++c) o[a][c] *= alpha[a];
    const int kmax = min(kSimtBK, n - k0);
    for (int k = 0; k < kmax; ++k) {
      float pv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) pv[a] = Ps[(ty * 4 + a) * kPsStride + k];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < hdc) {
          const int d = tx + 16 * c;
          const float vv = d < hd ? Vs[k * hd + d] : 0.f;
#pragma unroll
          for (int a = 0; a < 4; ++a) o[a][c] = fmaf(pv[a], vv, o[a][c]);
        }
      }
    }
  }
  // Row sums are split over the 16 lanes of a row.
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    float l = l_run[a];
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    const float inv = 1.f / l;
    const int row = r0 + ty * 4 + a;
    if (row < n) {
      T* orow = out + (bh * n + row) * hd;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int d = tx + 16 * c;
        if (c < hdc && d < hd) orow[d] = from_f<T>(o[a][c] * inv);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------
// Probs-only rel-pos softmax: one CTA of 256 threads per score row.
// ------------------------------------------------------------------------------------------------
constexpr int kSoftmaxThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kSoftmaxThreads) relpos_softmax_rows(const T* __restrict__ s,
                                                                       const T* __restrict__ q,
                                                                       const T* __restrict__ table,
                                                                       T* __restrict__ out, int h, int w, int hd,
                                                                       float scale) {
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* qs = sm;        // [hd]
  float* rh = qs + hd;   // [h]
  float* rw = rh + h;    // [w]
  __shared__ float red_m[kSoftmaxThreads / 32], red_l[kSoftmaxThreads / 32];
  const int n = h * w;
  const long row = blockIdx.x;
  const int rem = (int)(row % n), i = rem / w, j = rem % w;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int d = tid; d < hd; d += kSoftmaxThreads) qs[d] = to_f(q[row * hd + d]);
  __syncthreads();
  // one warp per bias dot product
  for (int c = warp; c < h + w; c += kSoftmaxThreads / 32) {
    const bool is_h = c < h;
    const T* tr = is_h ? table + (long)(i - c + h - 1) * hd : table + (long)(2 * h - 1 + j - (c - h) + w - 1) * hd;
    float a = 0.f;
    for (int d = lane; d < hd; d += 32) a = fmaf(qs[d], to_f(tr[d]), a);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
    if (lane == 0) (is_h ? rh[c] : rw[c - h]) = a;
  }
  __syncthreads();
  const T* sr = s + row * n;
  // pass 1: per-thread running (max, sum), then a block merge
  float m = -INFINITY, l = 0.f;
  for (int k = tid; k < n; k += kSoftmaxThreads) {
    const int kh = k / w, kw = k - kh * w;
    const float x = to_f(sr[k]) * scale + rh[kh] + rw[kw];
    if (x > m) {
      l = l * expf(m - x) + 1.f;
      m = x;
    } else {
      l += expf(x - m);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
    const float mm = fmaxf(m, m2);
    l = (m == -INFINITY ? 0.f : l * expf(m - mm)) + (m2 == -INFINITY ? 0.f : l2 * expf(m2 - mm));
    m = mm;
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_l[warp] = l;
  }
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int wi = 0; wi < kSoftmaxThreads / 32; ++wi) M = fmaxf(M, red_m[wi]);
  float L = 0.f;
#pragma unroll
  for (int wi = 0; wi < kSoftmaxThreads / 32; ++wi)
    if (red_m[wi] != -INFINITY) L += red_l[wi] * expf(red_m[wi] - M);
  const float inv = 1.f / L;
  T* orow = out + row * n;
  for (int k = tid; k < n; k += kSoftmaxThreads) {
    const int kh = k / w, kw = k - kh * w;
    const float x = to_f(sr[k]) * scale + rh[kh] + rw[kw];
    orow[k] = from_f<T>(expf(x - M) * inv);
  }
}

// ------------------------------------------------------------------------------------------------
// qkv split. Each CTA takes one window and one head (blockIdx.x = win * nh + head) and a chunk of
// 32 tokens (blockIdx.y); the K block is transposed through shared memory so that both the reads of
// y and the writes of q, kt and v are coalesced.
// ------------------------------------------------------------------------------------------------
constexpr int kSplitTok = 32;

template <typename T>
__global__ void __launch_bounds__(256) qkv_split_kernel(const T* __restrict__ y, const T* __restrict__ bias,
                                                        T* __restrict__ outp, long tokens, int n, int nh, int hd) {
  extern __shared__ float4 smem_f4[];
  float* kbuf = reinterpret_cast<float*>(smem_f4);  // [kSplitTok][hd + 1]
  const long bhx = blockIdx.x;
  const long win = bhx / nh;
  const int head = (int)(bhx % nh);
  const int tok0 = blockIdx.y * kSplitTok;
  if (tok0 >= n) return;
  const int ntok = min(kSplitTok, n - tok0);
  const long c = (long)nh * hd;
  const long plane = tokens * c;
  T* qo = outp;
  T* ko = outp + plane;
  T* vo = outp + 2 * plane;
  const int tid = threadIdx.x;
  const int hdp = hd + 1;
  for (int idx = tid; idx < ntok * hd; idx += 256) {
    const int t = idx / hd, d = idx % hd;
    const long tokg = win * n + tok0 + t;
    const T* yrow = y + tokg * 3 * c;
    const long cq = (long)head * hd + d;
    qo[(bhx * n + tok0 + t) * hd + d] = from_f<T>(to_f(yrow[cq]) + to_f(bias[cq]));
    vo[(bhx * n + tok0 + t) * hd + d] = from_f<T>(to_f(yrow[2 * c + cq]) + to_f(bias[2 * c + cq]));
    kbuf[t * hdp + d] = to_f(yrow[c + cq]) + to_f(bias[c + cq]);
  }
  __syncthreads();
  for (int idx = tid; idx < ntok * hd; idx += 256) {
    const int d = idx / ntok, t = idx % ntok;
    ko[(bhx * hd + d) * n + tok0 + t] = from_f<T>(kbuf[t * hdp + d]);
  }
}

}  // namespace samrs
