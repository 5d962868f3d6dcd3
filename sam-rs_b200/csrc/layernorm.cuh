// layernorm.cuh - LayerNorm over the channels of each token row, the norm1 / norm2 of the reference's
// encoder blocks (candle_nn::LayerNorm, eps 1e-6: src/sam1/encoder.rs:100-102, 121, 127):
//   out = (x - mean) / sqrt(var + eps) * weight + bias, mean and (biased) variance over the row in f32.
// One warp per row; each lane holds its 8-element slices of the row in registers (16-byte loads), so the
// row is read once: mean, then the centred sum of squares, then the output. HBM-bound byte work.
#pragma once
#include "common.cuh"

namespace samrs {

constexpr int kLnMaxChunks = 8;  // rows of up to 8 * 256 = 2048 channels on the vector path

template <typename T>
__device__ __forceinline__ void ln_unpack8(uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    T lo, hi;
    *reinterpret_cast<uint16_t*>(&lo) = (uint16_t)(w[i] & 0xFFFFu);
    *reinterpret_cast<uint16_t*>(&hi) = (uint16_t)(w[i] >> 16);
    f[2 * i] = to_f(lo);
    f[2 * i + 1] = to_f(hi);
  }
}

template <typename T>
__device__ __forceinline__ uint4 ln_pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const T lo = from_f<T>(f[2 * i]), hi = from_f<T>(f[2 * i + 1]);
    w[i] = (uint32_t)*reinterpret_cast<const uint16_t*>(&lo) | ((uint32_t)*reinterpret_cast<const uint16_t*>(&hi) << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Vector path: 16-bit T, c % 8 == 0, c <= 256 * NCH, 16-byte aligned rows.
template <typename T, int NCH>
__global__ void __launch_bounds__(256) layer_norm_vec_kernel(const T* __restrict__ x, const T* __restrict__ wt,
                                                            const T* __restrict__ bs, T* __restrict__ out, long rows,
                                                            int c, float eps) {
  const int lane = threadIdx.x & 31;
  const long warps = (long)gridDim.x * (blockDim.x >> 5);
  for (long row = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const T* xr = x + row * c;
    float v[NCH][8];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int col = 8 * (lane + 32 * k);
      if (col < c) {
        ln_unpack8<T>(*reinterpret_cast<const uint4*>(xr + col), v[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[k][e];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / c;
    float q = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int col = 8 * (lane + 32 * k);
      if (col < c) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = v[k][e] - mean;
          q += d * d;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = rsqrtf(q / c + eps);
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int col = 8 * (lane + 32 * k);
      if (col < c) {
        float w8[8], b8[8], y[8];
        ln_unpack8<T>(*reinterpret_cast<const uint4*>(wt + col), w8);
        ln_unpack8<T>(*reinterpret_cast<const uint4*>(bs + col), b8);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = (v[k][e] - mean) * inv * w8[e] + b8[e];
        *reinterpret_cast<uint4*>(out + row * c + col) = ln_pack8<T>(y);
      }
    }
  }
}

// Any dtype and width: one warp per row, three strided passes over the row in global memory.
template <typename T>
__global__ void __launch_bounds__(256) layer_norm_any_kernel(const T* __restrict__ x, const T* __restrict__ wt,
                                                            const T* __restrict__ bs, T* __restrict__ out, long rows,
                                                            int c, float eps) {
  const int lane = threadIdx.x & 31;
  const long warps = (long)gridDim.x * (blockDim.x >> 5);
  for (long row = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const T* xr = x + row * c;
    float s = 0.f;
    for (int i = lane; i < c; i += 32) s += to_f(xr[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / c;
    float q = 0.f;
    for (int i = lane; i < c; i += 32) {
      const float d = to_f(xr[i]) - mean;
      q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = rsqrtf(q / c + eps);
    for (int i = lane; i < c; i += 32)
      out[row * c + i] = from_f<T>((to_f(xr[i]) - mean) * inv * to_f(wt[i]) + to_f(bs[i]));
  }
}

}  // namespace samrs
