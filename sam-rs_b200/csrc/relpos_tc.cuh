// relpos_tc.cuh - host side of the tcgen05 kernels: tensor maps, shape selection and launches. The
// kernels are in relpos_tc_global.cuh (64x64 global layers) and relpos_tc_window.cuh (14x14 windows).
#pragma once
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "global_policy.h"
#include "relpos_tc_f32.cuh"
#include "relpos_tc_global.cuh"
#include "relpos_tc_window.cuh"
#include "sm100.cuh"

namespace samrs {

enum class TcShape { kNone, kGlobal, kWindow };

namespace tcg {

// ------------------------------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &qr) ==
            cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] 16-bit tensor, box [box_rows, box_cols].
inline int make_map(CUtensorMap* map, bool bf16, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                    uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return 2;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

// 3-D map over a row-major [d2, d1, d0] 16-bit tensor, box [1, box1, box0].
inline int make_map3(CUtensorMap* map, bool bf16, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                     uint32_t box0, uint32_t box1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return 2;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * 2, d0 * d1 * 2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

}  // namespace tcg

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The warp-role register split (setmaxnreg) draws on the registers the CTA is launched with; a kernel built
// with fewer than the split needs would block in setmaxnreg.inc. Checked once per kernel before its launch.
template <typename K>
inline bool regs_cover_split(K kern, int threads, int split_regs) {
  cudaFuncAttributes fa;
  return cudaFuncGetAttributes(&fa, kern) == cudaSuccess && fa.numRegs * threads >= split_regs;
}

inline TcShape tc_select(int h, int w, int hd, const void* q, const void* kt, const void* v, const void* table,
                         const void* out) {
  if (!(aligned16(q) && aligned16(kt) && aligned16(v) && aligned16(table) && aligned16(out))) return TcShape::kNone;
  if (h == 64 && w == 64 && (hd == 64 || hd == 80)) return TcShape::kGlobal;
  if (h == 14 && w == 14 && (hd == 64 || hd == 80)) return TcShape::kWindow;
  return TcShape::kNone;
}

template <typename T, int HD>
int tc_launch_global(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                     float scale, cudaStream_t st, int num_sms) {
  using namespace tcg;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (bh * kN > 0x7fffffffLL || bh * (kN / 256) > 0x7fffffffLL) return 4;
  CUtensorMap mq, mk, mv, mt;
  int rc = make_map(&mq, bf16, q, HD, (uint64_t)bh * kN, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&mk, bf16, kt, kN, (uint64_t)bh * HD, 64, HD, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_map(&mv, bf16, v, HD, (uint64_t)bh * kN, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map(&mt, bf16, table, HD, 4 * kSide - 2, 16, 128, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  // f16: the exact kernel. bf16: the speculative kernel, then the fixup launch, which recomputes exactly
  // the blocks the first one marked (one CTA per SM scans the markers); or, for a layer whose measured recompute
  // share made the speculative pass the slower choice (global_policy.h), the exact kernel alone.
  auto exact = relpos_attn_global<T, HD, kModeExact>;
  auto first = relpos_attn_global<T, HD, bf16 ? kModeSpec : kModeExact>;
  auto fixup = relpos_attn_global<T, HD, bf16 ? kModeFixup : kModeExact>;
  const int split = 128 * kRegsLow + 512 * kRegsHigh;
  static const bool regs_ok = regs_cover_split(exact, kThreads, split) && regs_cover_split(first, kThreads, split) &&
                              regs_cover_split(fixup, kThreads, split);
  if (!regs_ok) return 6;
  const int smem = Layout<HD>::kSmemBytes;
  if (cudaFuncSetAttribute(exact, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(first, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
      cudaFuncSetAttribute(fixup, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 5;
  const unsigned grid = (unsigned)(bh * (kN / 256));
  GlobalPolicy::Choice ch;
  ch.exact = !bf16;
  int dev = -1;
  if (bf16 && cudaGetDevice(&dev) == cudaSuccess) ch = global_policy().choose(dev, table, grid, st);
  const long n_blocks = (long)grid;
  if (ch.exact) {
    exact<<<grid, kThreads, smem, st>>>(mq, mk, mv, mt, static_cast<T*>(out), scale, nullptr, n_blocks);
    return 0;
  }
  first<<<grid, kThreads, smem, st>>>(mq, mk, mv, mt, static_cast<T*>(out), scale, nullptr, n_blocks);
  // the fixup: at most one CTA per SM, each reading its share of the markers and recomputing the marked blocks
  const unsigned fixup_grid = bf16 && num_sms > 0 && grid > (unsigned)num_sms ? (unsigned)num_sms : grid;
  fixup<<<fixup_grid, kThreads, smem, st>>>(mq, mk, mv, mt, static_cast<T*>(out), scale, ch.slot, n_blocks);
  global_policy().after_launch(dev, ch, st);
  return 0;
}

template <typename T, int HD>
int tc_launch_window(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                     float scale, cudaStream_t st, int num_sms) {
  using namespace tcg;
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  if (bh > 0x7fffffffLL) return 4;
  CUtensorMap mq, mv;
  int rc = make_map3(&mq, bf16, q, HD, tcw::kN, (uint64_t)bh, 16, tcw::Layout<HD>::kQRows, CU_TENSOR_MAP_SWIZZLE_32B);
  if (!rc) rc = make_map3(&mv, bf16, v, HD, tcw::kN, (uint64_t)bh, 16, tcw::kNP, CU_TENSOR_MAP_SWIZZLE_32B);
  if (rc) return rc;
  auto kern = tcw::relpos_attn_window<T, HD>;
  static const bool regs_ok = regs_cover_split(kern, tcw::kThreads, 128 * tcw::kRegsLow + 256 * tcw::kRegsHigh);
  if (!regs_ok) return 6;
  const int smem = tcw::Layout<HD>::kSmemBytes;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 5;
  const int grid = (int)(bh < num_sms ? bh : num_sms);
  kern<<<grid, tcw::kThreads, smem, st>>>(mq, mv, static_cast<const T*>(table), static_cast<const T*>(kt),
                                         static_cast<T*>(out), (long)bh, scale);
  return 0;
}

// f32 I/O: the 3xTF32 kernel (relpos_tc_f32.cuh), one CTA per head and 128 query rows.
template <int H, int W, int HD>
int tc_launch_f32(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                  float scale, cudaStream_t st) {
  using G = tcf::Geo<H, W, HD>;
  if (bh * G::kQTiles > 0x7fffffffLL) return 4;
  auto kern = tcf::relpos_attn_f32<H, W, HD>;
  static const bool regs_ok = regs_cover_split(kern, tcf::kThreads, 128 * tcf::kRegsLow + 384 * tcf::kRegsHigh);
  if (!regs_ok) return 6;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes) != cudaSuccess) return 5;
  kern<<<(unsigned)(bh * G::kQTiles), tcf::kThreads, G::kSmemBytes, st>>>(
      static_cast<const float*>(q), static_cast<const float*>(kt), static_cast<const float*>(v),
      static_cast<const float*>(table), static_cast<float*>(out), scale);
  return 0;
}

inline int tc_launch_f32(TcShape shape, const void* q, const void* kt, const void* v, const void* table, void* out,
                         int64_t bh, int hd, float scale, cudaStream_t st) {
  if (shape == TcShape::kGlobal)
    return hd == 80 ? tc_launch_f32<64, 64, 80>(q, kt, v, table, out, bh, scale, st)
                    : tc_launch_f32<64, 64, 64>(q, kt, v, table, out, bh, scale, st);
  if (shape == TcShape::kWindow)
    return hd == 80 ? tc_launch_f32<14, 14, 80>(q, kt, v, table, out, bh, scale, st)
                    : tc_launch_f32<14, 14, 64>(q, kt, v, table, out, bh, scale, st);
  return 1;
}

template <typename T>
int tc_launch(TcShape shape, const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
              int h, int w, int hd, float scale, cudaStream_t st, int num_sms) {
  (void)h;
  (void)w;
  if (shape == TcShape::kGlobal)
    return hd == 80 ? tc_launch_global<T, 80>(q, kt, v, table, out, bh, scale, st, num_sms)
                    : tc_launch_global<T, 64>(q, kt, v, table, out, bh, scale, st, num_sms);
  if (shape == TcShape::kWindow)
    return hd == 80 ? tc_launch_window<T, 80>(q, kt, v, table, out, bh, scale, st, num_sms)
                    : tc_launch_window<T, 64>(q, kt, v, table, out, bh, scale, st, num_sms);
  return 1;
}

inline const char* tc_error_string(int rc) {
  switch (rc) {
    case 1:
      return "no tensor-core kernel for this shape";
    case 2:
      return "cuTensorMapEncodeTiled is not available from the driver";
    case 3:
      return "cuTensorMapEncodeTiled rejected a tensor map";
    case 4:
      return "batch too large for 32-bit TMA coordinates";
    case 5:
      return "cannot set the kernel's shared memory size";
    case 6:
      return "tensor-core kernel built with fewer registers than its warp-role split needs";
    default:
      return "unknown tensor-core launch error";
  }
}

}  // namespace samrs
