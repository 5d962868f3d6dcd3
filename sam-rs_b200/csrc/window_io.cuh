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

constexpr int kWinTok = 32;  // tokens per CTA of the split

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

// blockIdx.x = unit = ((image * nwh + win_r) * nww + win_c) * nh + head; blockIdx.y = 32-token chunk.
// q and v rows go out as VEC-element vectors; K goes through shared memory and out transposed, so both
// the reads of y and the writes of kt are coalesced.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) qkv_split_window_kernel(const T* __restrict__ y, const T* __restrict__ bias,
                                                               T* __restrict__ outp, long units, WinGeom g) {
  extern __shared__ float4 smem_f4[];
  float* kbuf = reinterpret_cast<float*>(smem_f4);  // [kWinTok][hd + 1]
  const long unit = blockIdx.x;
  const int n = g.n(), hd = g.hd;
  const long c = g.c();
  const int head = (int)(unit % g.nh);
  const long win = unit / g.nh;
  const int win_c = (int)(win % g.nww), win_r = (int)((win / g.nww) % g.nwh);
  const long image = win / ((long)g.nww * g.nwh);
  const int tok0 = blockIdx.y * kWinTok;
  if (tok0 >= n) return;
  const int ntok = min(kWinTok, n - tok0);
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
  for (int idx = threadIdx.x; idx < ntok * hd; idx += blockDim.x) {
    const int d = idx / ntok, t = idx % ntok;
    ko[(unit * hd + d) * (long)n + tok0 + t] = from_f<T>(kbuf[t * hdp + d]);
  }
}

// One thread per VEC-element chunk of an output row (a chunk never straddles two heads: hd % VEC == 0).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) window_merge_kernel(const T* __restrict__ attn, T* __restrict__ out,
                                                           long images, WinGeom g) {
  using V = typename VecOf<T, VEC>::type;
  const int c = g.c(), n = g.n();
  const int cv = c / VEC;
  const long total = images * g.h * (long)g.w * cv;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long tokrow = i / cv;
    const int ch = (int)(i % cv) * VEC;
    const int head = ch / g.hd, d = ch % g.hd;
    const int gx = (int)(tokrow % g.w);
    const long rest = tokrow / g.w;
    const int gy = (int)(rest % g.h);
    const long image = rest / g.h;
    const long win = (image * g.nwh + gy / g.wh) * g.nww + gx / g.ww;
    const int tok = (gy % g.wh) * g.ww + gx % g.ww;
    const long src = ((win * g.nh + head) * n + tok) * (long)g.hd + d;
    *reinterpret_cast<V*>(out + tokrow * c + ch) = *reinterpret_cast<const V*>(attn + src);
  }
}

}  // namespace samrs
