// window_io.cuh - the attention path's neighbours on the token grid: the QKV head split fused with the
// window partition, and the head merge fused with the window unpartition.
//
// Reference order (src/sam1/encoder.rs:115-145, 73-85): x [B, H, W, C] is zero-padded to multiples of the
// window size and cut into windows (window_partition, :132-140), the qkv projection runs on every padded
// token, qkv_split (src/kernels.rs:870-894) adds the bias and splits heads, attention runs per
// (window, head), the heads are merged back to [windows * ws*ws, C] (:82), the output projection runs on
// every padded token and window_unpartition crops the pads (:142-145).
//
// Here the projections run on the H x W real tokens only. A pad token's qkv in the reference is
// 0 * W + bias = bias, so the split writes the bias there; the projection is per token, so running it
// after the merge on the real tokens gives the same rows as running it before the crop.
//
//   qkv_split_window: y [B*H*W, 3C] (projection without bias) + bias [3C] ->
//                     q [BH, n, hd] | kt [BH, hd, n] | v [BH, n, hd],  BH = B * nWh * nWw * nh, n = wh * ww,
//                     bh = window * nh + head, windows row-major per image (window_partition's order).
//   window_merge:     attn [BH, n, hd] -> out [B*H*W, C], C = nh * hd (pads dropped).
// ws = 0 means one window of H x W (the global layers), with no padding.
#pragma once
#include "common.cuh"

namespace samrs {

struct WinGeom {
  int h, w;        // real token grid
  int wh, ww;      // window size (rows, columns)
  int nwh, nww;    // windows per image along rows / columns
  int nh, hd;      // heads, head dim
  __host__ __device__ int n() const { return wh * ww; }
  __host__ __device__ int c() const { return nh * hd; }
};

// Row of the real token (image, gy, gx) in [B*H*W, ...], or -1 for a pad position.
__device__ __forceinline__ long win_token_row(const WinGeom& g, long image, int win_r, int win_c, int tok) {
  const int gy = win_r * g.wh + tok / g.ww, gx = win_c * g.ww + tok % g.ww;
  if (gy >= g.h || gx >= g.w) return -1;
  return (image * g.h + gy) * (long)g.w + gx;
}

// Tokens per CTA of the split: a whole window when it has at most 256 tokens (and its K block fits in
// 96 KB of shared memory), else chunks of 64 tokens (fewer when hd is large; a multiple of 4).
__host__ __device__ inline int win_chunk(int n, int hd) {
  int cap = (96 * 1024) / ((hd + 1) * 4);
  cap = cap < 256 ? cap : 256;
  if (n <= cap) return n;
  cap = (cap < 64 ? cap : 64) & ~3;
  return cap < 4 ? 4 : cap;
}

// VEC elements of T moved as one access (16 bytes when VEC * sizeof(T) == 16).
template <int BYTES>
struct VecBytes;
template <>
struct VecBytes<16> {
  using type = uint4;
};
template <>
struct VecBytes<8> {
  using type = uint2;
};
template <>
struct VecBytes<4> {
  using type = uint32_t;
};
template <>
struct VecBytes<2> {
  using type = unsigned short;
};
template <typename T, int VEC>
struct VecOf {
  using type = typename VecBytes<(int)sizeof(T) * VEC>::type;
};
template <typename T, int VEC>
union Pack {
  typename VecOf<T, VEC>::type v;
  T e[VEC];
};

// blockIdx.x = unit = ((image * nwh + win_r) * nww + win_c) * nh + head; blockIdx.y = token chunk.
// q and v rows go out as VEC-element vectors; K goes through shared memory and out transposed, KT tokens
// per store, so both the reads of y and the writes of kt are coalesced.
template <typename T, int VEC, int KT>
__global__ void __launch_bounds__(256) qkv_split_window_kernel(const T* __restrict__ y, const T* __restrict__ bias,
                                                               T* __restrict__ outp, long units, WinGeom g) {
  extern __shared__ float4 smem_f4[];
  float* kbuf = reinterpret_cast<float*>(smem_f4);  // [chunk][hd + 1]
  const long unit = blockIdx.x;
  const int n = g.n(), hd = g.hd;
  const long c = g.c();
  const int head = (int)(unit % g.nh);
  const long win = unit / g.nh;
  const int win_c = (int)(win % g.nww), win_r = (int)((win / g.nww) % g.nwh);
  const long image = win / ((long)g.nww * g.nwh);
  const int chunk = win_chunk(n, hd);
  const int tok0 = blockIdx.y * chunk;
  if (tok0 >= n) return;
  const int ntok = min(chunk, n - tok0);
  const long plane = units * (long)n * hd;  // elements of each of q, kt, v
  T* qo = outp;
  T* ko = outp + plane;
  T* vo = outp + 2 * plane;
  const int hdp = hd + 1;
  const int nv = hd / VEC;
  for (int idx = threadIdx.x; idx < ntok * nv; idx += blockDim.x) {
    const int t = idx / nv, d = (idx % nv) * VEC;
    const long row = win_token_row(g, image, win_r, win_c, tok0 + t);
    const long cq = (long)head * hd + d;
    using V = typename VecOf<T, VEC>::type;
    Pack<T, VEC> bq, bk, bv, yq, yk, yv;
    bq.v = *reinterpret_cast<const V*>(bias + cq);
    bk.v = *reinterpret_cast<const V*>(bias + c + cq);
    bv.v = *reinterpret_cast<const V*>(bias + 2 * c + cq);
    if (row >= 0) {  // a real token: y + bias; a pad token: bias alone (its x is 0 in the reference)
      const T* yr = y + row * 3 * c;
      yq.v = *reinterpret_cast<const V*>(yr + cq);
      yk.v = *reinterpret_cast<const V*>(yr + c + cq);
      yv.v = *reinterpret_cast<const V*>(yr + 2 * c + cq);
    }
    Pack<T, VEC> oq, ov;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float fq = row >= 0 ? to_f(yq.e[e]) + to_f(bq.e[e]) : to_f(bq.e[e]);
      const float fk = row >= 0 ? to_f(yk.e[e]) + to_f(bk.e[e]) : to_f(bk.e[e]);
      const float fv = row >= 0 ? to_f(yv.e[e]) + to_f(bv.e[e]) : to_f(bv.e[e]);
      oq.e[e] = from_f<T>(fq);
      ov.e[e] = from_f<T>(fv);
      kbuf[t * hdp + d + e] = to_f(from_f<T>(fk));
    }
    const long o = (unit * n + tok0 + t) * (long)hd + d;
    *reinterpret_cast<V*>(qo + o) = oq.v;
    *reinterpret_cast<V*>(vo + o) = ov.v;
  }
  __syncthreads();
  // kt rows: KT consecutive tokens of one dim per store (n and the chunk are multiples of KT)
  const int ng = ntok / KT;
  for (int idx = threadIdx.x; idx < ng * hd; idx += blockDim.x) {
    const int d = idx / ng, t = (idx % ng) * KT;
    Pack<T, KT> pk;
#pragma unroll
    for (int e = 0; e < KT; ++e) pk.e[e] = from_f<T>(kbuf[(t + e) * hdp + d]);
    *reinterpret_cast<typename VecOf<T, KT>::type*>(ko + (unit * hd + d) * (long)n + tok0 + t) = pk.v;
  }
}

// One thread per VEC-element chunk of an output row (a chunk never straddles two heads: hd % VEC == 0).
// I is the index type: 32-bit when the chunk count allows (cheaper divisions), else 64-bit.
template <typename T, int VEC, typename I>
__global__ void __launch_bounds__(256) window_merge_kernel(const T* __restrict__ attn, T* __restrict__ out,
                                                           long images, WinGeom g) {
  using V = typename VecOf<T, VEC>::type;
  const I c = (I)g.c(), n = (I)g.n(), hd = (I)g.hd, w = (I)g.w, h = (I)g.h;
  const I cv = c / VEC;
  const I total = (I)images * h * w * cv;
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (I)gridDim.x * blockDim.x) {
    const I tokrow = i / cv;
    const I ch = (i - tokrow * cv) * VEC;
    const I head = ch / hd, d = ch - head * hd;
    const I rest = tokrow / w;
    const I gx = tokrow - rest * w;
    const I image = rest / h;
    const I gy = rest - image * h;
    const I wy = gy / (I)g.wh, wx = gx / (I)g.ww;
    const I win = (image * (I)g.nwh + wy) * (I)g.nww + wx;
    const I tok = (gy - wy * (I)g.wh) * (I)g.ww + (gx - wx * (I)g.ww);
    const I src = ((win * (I)g.nh + head) * n + tok) * hd + d;
    *reinterpret_cast<V*>(out + (size_t)tokrow * c + ch) = *reinterpret_cast<const V*>(attn + src);
  }
}

}  // namespace samrs

namespace samrs {

// Pad tokens of the window-partitioned grid: the reference zero-pads the normalised tokens before the qkv
// projection (src/sam1/encoder.rs:132-140), so a pad token's q / k / v is the projection's bias alone.
// Writes bias into q, kt and v at every (window, pad token, head) of the layout above. Only the windows of
// the last window row / column hold pads; one CTA per (such window, head): q and v by 16-byte chunks of a
// pad token's hd values (hd % 8 == 0), kt by one warp per dim row with the lanes over the row's tokens.
template <typename T>
__global__ void __launch_bounds__(128) qkv_pad_fill_kernel(const T* __restrict__ bias, T* __restrict__ out,
                                                           long images, WinGeom g) {
  const bool pad_rows = g.h % g.wh != 0, pad_cols = g.w % g.ww != 0;
  // edge windows of an image: the last window row (if its rows pad), then the last window column (if its
  // columns pad) without the corner already counted
  const int n_bottom = pad_rows ? g.nww : 0;
  const int n_edge = n_bottom + (pad_cols ? g.nwh - (pad_rows ? 1 : 0) : 0);
  const int c = g.c(), n = g.n(), hd8 = g.hd / 8;
  const long plane = images * g.nwh * g.nww * (long)g.nh * n * g.hd;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (long unit = blockIdx.x; unit < images * n_edge * g.nh; unit += gridDim.x) {
    const int head = (int)(unit % g.nh);
    const long we = unit / g.nh;
    const long img = we / n_edge;
    const int e = (int)(we - img * n_edge);
    const int wy = e < n_bottom ? g.nwh - 1 : e - n_bottom;
    const int wx = e < n_bottom ? e : g.nww - 1;
    const long bh = ((img * g.nwh + wy) * g.nww + wx) * g.nh + head;
    const int y0 = wy * g.wh, x0 = wx * g.ww;
    // q and v
    for (int idx = threadIdx.x; idx < n * hd8; idx += blockDim.x) {
      const int n_in = idx / hd8, ch = idx - n_in * hd8;
      if (y0 + n_in / g.ww < g.h && x0 + n_in % g.ww < g.w) continue;
      const int col = head * g.hd + 8 * ch;
      const long off = (bh * n + n_in) * g.hd + 8 * ch;
      *reinterpret_cast<uint4*>(out + off) = *reinterpret_cast<const uint4*>(bias + col);
      *reinterpret_cast<uint4*>(out + 2 * plane + off) = *reinterpret_cast<const uint4*>(bias + 2 * c + col);
    }
    // kt
    for (int d = warp; d < g.hd; d += nwarps) {
      const T b = bias[c + head * g.hd + d];
      T* row = out + plane + (bh * g.hd + d) * n;
      for (int n_in = lane; n_in < n; n_in += 32)
        if (y0 + n_in / g.ww >= g.h || x0 + n_in % g.ww >= g.w) row[n_in] = b;
    }
  }
}

}  // namespace samrs
