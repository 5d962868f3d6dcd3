// window_tma.cuh - the window partition and unpartition around the windowed layers as TMA tile moves
// (the TMA versions of window_io.cuh's qkv_split_window and window_merge, used where the shapes allow).
//
// The token grid is a 4-D tensor [B, H, W, channels] and one window of one head is a box of
// [wh, ww, hd] in it: a tensor-map load of that box at (x = wx * ww, y = wy * wh) reads the window's real
// tokens, and the hardware fills the positions past H or W with zeros. That is the reference's zero pad
// (window_partition, src/sam1/encoder.rs:132-140) without a pad copy. A tensor-map store of the same box
// writes the real tokens and drops the rest, which is window_unpartition's crop (:142-145).
//
//   qkv_split_window_tma: one CTA per (window, head, part); part 0 q, 1 k, 2 v. It loads the part's box of
//     y [B, H, W, 3C] (the projection without bias) with one TMA load, adds the bias (a pad token becomes the
//     bias alone, as the reference's 0 * W + b), transposes k, and writes the contiguous q / kt / v block
//     of the (window, head) with one bulk store (src/kernels.rs:870-894 with kernels/sam.cu:111-128's
//     layout: bh = window * nh + head).
//   window_merge_tma: one CTA per (window, head, band of rows): one bulk load of the band's rows of the
//     [n, hd] attention block, one tensor-map store of them into out [B, H, W, C] at the head's channels
//     (src/sam1/encoder.rs:82, :142-145).
//
// Both are HBM-bound byte moves: y's real tokens are read once and q / kt / v (pads included) written once;
// the attention rows are read once and the real tokens written once.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "relpos_tc.cuh"
#include "sm100.cuh"
#include "window_io.cuh"

namespace samrs {
namespace wtma {
using namespace sm100;

constexpr int kSplitThreads = 128;

struct alignas(8) SplitBars {
  uint64_t full;
  int abort_flag;
};

// 16 bytes of T and their element count
template <typename T>
struct Pack16 {
  static constexpr int kN = 16 / (int)sizeof(T);
  using type = Pack<T, kN>;
};

// 16 bytes of T: a + b elementwise in f32, rounded back to T (the reference's from_f(to_f(y) + to_f(b)))
template <typename T>
__device__ __forceinline__ uint4 add_bias16(uint4 a, uint4 b) {
  typename Pack16<T>::type pa, pb, po;
  pa.v = a;
  pb.v = b;
#pragma unroll
  for (int e = 0; e < Pack16<T>::kN; ++e) po.e[e] = from_f<T>(to_f(pa.e[e]) + to_f(pb.e[e]));
  return po.v;
}

// smem: the loaded box [wh][ww][hd] (token-major, the q / v order). q and v get their bias in place and go
// out by one bulk store; k is transposed on its way out by coalesced stores of token pairs. One buffer per
// CTA keeps seven CTAs (loads) in flight per SM at the ViT shapes.
template <typename T>
__global__ void __launch_bounds__(kSplitThreads) qkv_split_window_tma(const __grid_constant__ CUtensorMap tmY,
                                                                       const T* __restrict__ bias, T* __restrict__ out,
                                                                       long units, WinGeom g) {
  extern __shared__ uint8_t smem_raw[];
  T* tile = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int n = g.n(), hd = g.hd, c = g.c();
  __shared__ SplitBars bars;
  const long unit = blockIdx.x;
  const int part = (int)(unit % 3);
  const long bh = unit / 3;  // window * nh + head
  const int head = (int)(bh % g.nh);
  const long win = bh / g.nh;
  const int wx = (int)(win % g.nww), wy = (int)((win / g.nww) % g.nwh);
  const long img = win / ((long)g.nww * g.nwh);
  if (__syncthreads_or(threadIdx.x == 0 && device_faulted())) return;
  const uint32_t bytes = (uint32_t)((long)n * hd * sizeof(T));
  if (threadIdx.x == 0) {
    mbar_init(&bars.full, 1);
    bars.abort_flag = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(&bars.full, bytes);
    tma_load_4d(tile, &tmY, &bars.full, part * c + head * hd, wx * g.ww, wy * g.wh, (int)img);
  }
  __syncthreads();
  const bool ok = mbar_wait(&bars.full, 0, &bars.abort_flag);
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) mbar_drain(&bars.full, 0);  // this CTA's load must land before the CTA exits
    return;
  }
  const T* b = bias + part * c + head * hd;
  constexpr int kV = Pack16<T>::kN;  // elements per 16 bytes
  const int hv = hd / kV;
  if (part != 1) {
    // q, v: in[t][d] += b[d], in place
    for (int i = threadIdx.x; i < n * hv; i += kSplitThreads) {
      const int d = (i % hv) * kV;
      uint4* p = reinterpret_cast<uint4*>(tile) + i;
      *p = add_bias16<T>(*p, *reinterpret_cast<const uint4*>(b + d));
    }
  } else {
    // kt: out[d][t] = in[t][d] + b[d], straight to global memory: a thread takes tokens t, t+1 and kV dims
    // and stores kV token pairs; a warp's threads hold consecutive pairs, so each of its stores is one
    // contiguous 32 x 2-element run of a kt row
    const int np = n / 2;
    T* kt = out + units / 3 * (long)n * hd + bh * (long)n * hd;
    for (int i = threadIdx.x; i < np * hv; i += kSplitThreads) {
      const int t = (i % np) * 2, d = (i / np) * kV;
      const uint4 bb = *reinterpret_cast<const uint4*>(b + d);
      typename Pack16<T>::type p0, p1;
      p0.v = add_bias16<T>(*reinterpret_cast<const uint4*>(tile + (long)t * hd + d), bb);
      p1.v = add_bias16<T>(*reinterpret_cast<const uint4*>(tile + (long)(t + 1) * hd + d), bb);
#pragma unroll
      for (int e = 0; e < kV; ++e) {
        Pack<T, 2> pr;  // tokens t, t+1 of dim d+e: adjacent in the kt row (t and n even: aligned)
        pr.e[0] = p0.e[e];
        pr.e[1] = p1.e[e];
        *reinterpret_cast<typename VecOf<T, 2>::type*>(kt + (long)(d + e) * n + t) = pr.v;
      }
    }
    return;  // nothing left in shared memory to write out
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) {
    const long plane = units / 3 * (long)n * hd;  // elements of each of q, kt, v
    bulk_store(out + part * plane + bh * (long)n * hd, tile, bytes);
    bulk_commit();
    bulk_wait_read();  // shared memory has been read out before the CTA exits
  }
}

// One warp per (window, head, band of wh / bands rows); lane 0 moves the band: its rows are contiguous in
// the attention block (tokens are row-major within the window). Two bands per window halve each CTA's
// shared memory and double the moves in flight per SM.
template <typename T>
__global__ void __launch_bounds__(32) window_merge_tma(const __grid_constant__ CUtensorMap tmO,
                                                        const T* __restrict__ attn, WinGeom g, int bands) {
  extern __shared__ uint8_t smem_raw[];
  T* tile = reinterpret_cast<T*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  __shared__ SplitBars bars;
  if (threadIdx.x != 0) return;
  if (device_faulted()) return;
  const long bh = blockIdx.x / bands;
  const int band = (int)(blockIdx.x % bands);
  const int n = g.n(), hd = g.hd, rows = g.wh / bands;
  const int head = (int)(bh % g.nh);
  const long win = bh / g.nh;
  const int wx = (int)(win % g.nww), wy = (int)((win / g.nww) % g.nwh);
  const long img = win / ((long)g.nww * g.nwh);
  const int y0 = wy * g.wh + band * rows;
  if (y0 >= g.h) return;  // a band of pad rows only: nothing to write (and no store starts past the tensor)
  const uint32_t bytes = (uint32_t)((long)rows * g.ww * hd * sizeof(T));
  mbar_init(&bars.full, 1);
  bars.abort_flag = 0;
  fence_mbar_init();
  mbar_arrive_expect_tx(&bars.full, bytes);
  bulk_load(tile, attn + (bh * n + (long)band * rows * g.ww) * hd, bytes, &bars.full);
  if (!mbar_wait(&bars.full, 0, &bars.abort_flag)) {
    mbar_drain(&bars.full, 0);
    return;
  }
  fence_proxy_async_smem();
  tma_store_4d(&tmO, tile, head * hd, wx * g.ww, y0, (int)img);
  bulk_commit();
  bulk_wait_read();  // shared memory has been read out before the CTA exits
}

// ------------------------------------------------------------------------------------------ host
// 4-D map over a [d3, d2, d1, d0] row-major tensor of T (d0 innermost), box [b3=1, b2, b1, b0], no swizzle,
// out-of-bounds elements zero-filled on loads (and not written on stores).
template <typename T>
inline int make_map4(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                     uint32_t b0, uint32_t b1, uint32_t b2) {
  tcg::EncodeTiledFn fn = tcg::encode_fn();
  if (!fn) return 2;
  const CUtensorMapDataType dt = sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {d0 * sizeof(T), d0 * d1 * sizeof(T), d0 * d1 * d2 * sizeof(T)};
  cuuint32_t box[4] = {b0, b1, b2, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

// Whether a (window, head) block can move as one box: windowed layout (ws > 0), 16-byte rows of hd elements,
// box sides <= 256, the block and its output within the shared-memory budget, 16-byte aligned buffers and
// an even token count (kt goes out by token pairs).
template <typename T>
inline bool tma_window_ok(const WinGeom& g, bool windowed, int smem_tiles, const void* a, const void* b,
                          const void* c) {
  const long block = (long)g.n() * g.hd * sizeof(T);
  return windowed && (g.hd * sizeof(T)) % 16 == 0 && g.hd <= 256 && g.ww <= 256 && g.wh <= 256 &&
         g.n() % 2 == 0 && block % 16 == 0 && smem_tiles * block + 128 <= 200 * 1024 && aligned16(a) &&
         aligned16(b) && aligned16(c);
}

template <typename T>
inline int launch_split_window_tma(const void* y, const void* bias, void* out, int64_t images, const WinGeom& g,
                                   cudaStream_t st) {
  const int64_t units = images * g.nwh * g.nww * g.nh * 3;
  if (units > 0x7fffffffLL || images > 0x7fffffffLL) return 4;
  CUtensorMap my;
  const int rc = make_map4<T>(&my, y, (uint64_t)3 * g.c(), (uint64_t)g.w, (uint64_t)g.h, (uint64_t)images,
                              (uint32_t)g.hd, (uint32_t)g.ww, (uint32_t)g.wh);
  if (rc) return rc;
  const int smem = (int)((long)g.n() * g.hd * sizeof(T)) + 128;
  auto kern = qkv_split_window_tma<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 5;
  kern<<<(unsigned)units, kSplitThreads, smem, st>>>(my, static_cast<const T*>(bias), static_cast<T*>(out),
                                                      (long)units, g);
  return 0;
}

template <typename T>
inline int launch_merge_tma(const void* attn, void* out, int64_t images, const WinGeom& g, cudaStream_t st) {
  const int64_t units = images * g.nwh * g.nww * g.nh;
  if (units > 0x7fffffffLL || images > 0x7fffffffLL) return 4;
  // two bands of rows per window when the half block still moves as whole 16-byte units
  const int bands = (g.wh % 2 == 0 && ((long)(g.wh / 2) * g.ww * g.hd * sizeof(T)) % 16 == 0) ? 2 : 1;
  if (units * bands > 0x7fffffffLL) return 4;
  CUtensorMap mo;
  const int rc = make_map4<T>(&mo, out, (uint64_t)g.c(), (uint64_t)g.w, (uint64_t)g.h, (uint64_t)images,
                              (uint32_t)g.hd, (uint32_t)g.ww, (uint32_t)(g.wh / bands));
  if (rc) return rc;
  const int smem = (int)((long)(g.wh / bands) * g.ww * g.hd * sizeof(T)) + 128;
  auto kern = window_merge_tma<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 5;
  kern<<<(unsigned)(units * bands), 32, smem, st>>>(mo, static_cast<const T*>(attn), g, bands);
  return 0;
}

}  // namespace wtma
}  // namespace samrs
