// samrs_abi.cu - the C ABI declared in include/samrs_b200.h: argument checks, dtype dispatch and
// kernel selection. The entry points mirror the reference's candle ops (src/kernels.rs): they take
// caller-owned device buffers, enqueue on the caller's stream, allocate nothing and never synchronise.
#include <cuda_runtime.h>
#include <stdarg.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "../../include/samrs_b200.h"
#include "common.cuh"
#include "relpos_simt.cuh"
#include "gemm_tc.cuh"
#include "layernorm.cuh"
#include "relpos_tc.cuh"
#include "window_io.cuh"
#include "window_tma.cuh"

namespace {

using namespace samrs;

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_last_error[0] = '\0';
  return SAMRS_OK;
}

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

size_t elem_size(int dtype) { return dtype == SAMRS_F32 ? 4 : 2; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Per-device cache of "is this an sm_100 device", the opt-in shared memory limit and the SM count,
// filled once per device (std::call_once: entry points may run on several host threads at once).
struct DevInfo {
  int is_sm100 = 0;
  int max_smem_optin = 0;
  int num_sms = 0;
};
constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];
// Host-side record of a nonzero device status word: set when samrs_device_status reads a nonzero word
// without clearing it, reset when it clears the word. While it is set every entry point of that device
// returns SAMRS_ERR_DEVICE instead of launching.
std::atomic<unsigned int> g_fault_seen[kMaxDevices];

int device_info(DevInfo** out, int* dev_out = nullptr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SAMRS_ERR_NODEVICE, "no CUDA device is current");
  DevInfo& d = g_dev[dev];
  std::call_once(g_dev_once[dev], [&d, dev]() {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    d.is_sm100 = (major == 10 && minor == 0);
  });
  if (!d.is_sm100) return fail(SAMRS_ERR_NODEVICE, "this library is built for sm_100a (B200) only");
  const unsigned int seen = g_fault_seen[dev].load(std::memory_order_relaxed);
  if (seen)
    return fail(SAMRS_ERR_DEVICE,
                "device status word is %u (a kernel reported a fault; kernels are no-ops until "
                "samrs_device_status(stream, 1) clears it)",
                seen);
  *out = &d;
  if (dev_out) *dev_out = dev;
  return SAMRS_OK;
}

int check_common(int64_t bh, int h, int w, int hd, int dtype, const char* what) {
  if (dtype != SAMRS_F32 && dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_INVALID, "%s: unsupported dtype code %d (0 f32, 1 f16, 2 bf16)", what, dtype);
  if (bh < 0) return fail(SAMRS_ERR_INVALID, "%s: negative batch-heads %lld", what, (long long)bh);
  if (h < 1 || w < 1 || h > 128 || w > 128)
    return fail(SAMRS_ERR_UNSUPPORTED, "%s: grid %dx%d outside 1..128", what, h, w);
  if (hd < 1 || hd > kSimtMaxHd) return fail(SAMRS_ERR_UNSUPPORTED, "%s: head_dim %d outside 1..128", what, hd);
  return SAMRS_OK;
}

template <typename T>
int launch_simt(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh, int h,
                int w, int hd, float scale, cudaStream_t st, const DevInfo& dev) {
  const int n = h * w;
  const int64_t qtiles = (n + kSimtBQ - 1) / kSimtBQ;
  const int64_t blocks = bh * qtiles;
  if (blocks > 0x7fffffffLL) return fail(SAMRS_ERR_UNSUPPORTED, "relpos_attn: %lld CTAs exceed the grid limit", (long long)blocks);
  const size_t smem = simt_smem_floats(h, w, hd) * sizeof(float);
  if ((int)smem > dev.max_smem_optin)
    return fail(SAMRS_ERR_UNSUPPORTED, "relpos_attn: %zu B of shared memory needed, %d available", smem,
                dev.max_smem_optin);
  auto kern = relpos_attn_simt<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return fail(SAMRS_ERR_LAUNCH, "relpos_attn: cannot set shared memory size %zu", smem);
  kern<<<(unsigned)blocks, kSimtThreads, smem, st>>>(static_cast<const T*>(q), static_cast<const T*>(kt),
                                                     static_cast<const T*>(v), static_cast<const T*>(table),
                                                     static_cast<T*>(out), h, w, hd, scale);
  return launch_status("relpos_attn_simt");
}

template <typename T>
int launch_softmax(const void* s, const void* q, const void* table, void* out, int64_t rows, int h, int w, int hd,
                   float scale, cudaStream_t st) {
  if (rows > 0x7fffffffLL) return fail(SAMRS_ERR_UNSUPPORTED, "relpos_softmax: too many rows");
  const size_t smem = (size_t)(hd + h + w) * sizeof(float);
  relpos_softmax_rows<T><<<(unsigned)rows, kSoftmaxThreads, smem, st>>>(
      static_cast<const T*>(s), static_cast<const T*>(q), static_cast<const T*>(table), static_cast<T*>(out), h, w, hd,
      scale);
  return launch_status("relpos_softmax_rows");
}

template <typename T>
int launch_split(const void* y, const void* bias, void* out, int64_t tokens, int n, int nh, int hd, cudaStream_t st) {
  const int64_t windows = tokens / n;
  const int64_t gx = windows * nh;
  const int gy = (n + kSplitTok - 1) / kSplitTok;
  if (gx > 0x7fffffffLL || gy > 65535) return fail(SAMRS_ERR_UNSUPPORTED, "qkv_split: grid too large");
  const size_t smem = (size_t)kSplitTok * (hd + 1) * sizeof(float);
  qkv_split_kernel<T><<<dim3((unsigned)gx, gy), 256, smem, st>>>(static_cast<const T*>(y),
                                                                 static_cast<const T*>(bias), static_cast<T*>(out),
                                                                 tokens, n, nh, hd);
  return launch_status("qkv_split");
}

bool aligned16_all(const void* a, const void* b, const void* c) {
  return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15u) == 0;
}

// Window geometry of a (images, h, w, ws) call; ws = 0: one window of h x w.
int win_geom(const char* what, int64_t images, int h, int w, int ws, int nh, int hd, WinGeom* g) {
  if (images < 0 || h < 1 || w < 1 || ws < 0 || nh < 1 || hd < 1 || hd > 1024 || h > 65535 || w > 65535 ||
      ws > 65535)
    return fail(SAMRS_ERR_INVALID, "%s: bad geometry images=%lld h=%d w=%d ws=%d nh=%d hd=%d", what, (long long)images,
                h, w, ws, nh, hd);
  g->h = h;
  g->w = w;
  g->wh = ws ? ws : h;
  g->ww = ws ? ws : w;
  g->nwh = (h + g->wh - 1) / g->wh;
  g->nww = (w + g->ww - 1) / g->ww;
  g->nh = nh;
  g->hd = hd;
  if ((int64_t)g->wh * g->ww > (1 << 24)) return fail(SAMRS_ERR_UNSUPPORTED, "%s: window too large", what);
  return ok();
}

template <typename T>
int launch_split_window(const void* y, const void* bias, void* out, int64_t images, const WinGeom& g, cudaStream_t st) {
  const int64_t units = images * g.nwh * g.nww * g.nh;
  const int chunk = win_chunk(g.n(), g.hd);
  const int gy = (g.n() + chunk - 1) / chunk;
  if (units > 0x7fffffffLL || gy > 65535) return fail(SAMRS_ERR_UNSUPPORTED, "qkv_split_window: grid too large");
  const size_t smem = (size_t)chunk * (g.hd + 1) * sizeof(float);
  constexpr int kVec = 16 / (int)sizeof(T);
  constexpr int kKt = sizeof(T) == 2 ? 4 : 2;  // kt tokens per 8-byte store
  const dim3 grid((unsigned)units, gy);
  const auto* yp = static_cast<const T*>(y);
  const auto* bp = static_cast<const T*>(bias);
  auto* op = static_cast<T*>(out);
  auto kvec = qkv_split_window_kernel<T, kVec, kKt>;
  auto kone = qkv_split_window_kernel<T, 1, 1>;
  const bool vec = (g.hd * (int)sizeof(T)) % 16 == 0 && aligned16_all(y, bias, out) && g.n() % kKt == 0 &&
                   chunk % kKt == 0;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(vec ? kvec : kone, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem) != cudaSuccess)
    return fail(SAMRS_ERR_UNSUPPORTED, "qkv_split_window: cannot set %zu bytes of shared memory", smem);
  if (vec)
    kvec<<<grid, 256, smem, st>>>(yp, bp, op, (long)units, g);
  else
    kone<<<grid, 256, smem, st>>>(yp, bp, op, (long)units, g);
  return launch_status("qkv_split_window");
}

// The windowed layers' split and merge as TMA tile moves (window_tma.cuh) where a (window, head) block moves
// as one box; the vectorised / scalar kernels of window_io.cuh otherwise (global layers, odd head dims,
// unaligned buffers). Both give the same bits.
template <typename T>
int split_window_any(const void* y, const void* bias, void* out, int64_t images, const WinGeom& g, bool windowed,
                     cudaStream_t st) {
  if (wtma::tma_window_ok<T>(g, windowed, 1, y, bias, out) &&
      wtma::launch_split_window_tma<T>(y, bias, out, images, g, st) == 0)
    return launch_status("qkv_split_window");
  return launch_split_window<T>(y, bias, out, images, g, st);
}

template <typename T>
int launch_merge(const void* attn, void* out, int64_t images, const WinGeom& g, int num_sms, cudaStream_t st);

template <typename T>
int merge_any(const void* attn, void* out, int64_t images, const WinGeom& g, bool windowed, int num_sms,
              cudaStream_t st) {
  if (wtma::tma_window_ok<T>(g, windowed, 1, attn, out, out) && wtma::launch_merge_tma<T>(attn, out, images, g, st) == 0)
    return launch_status("window_merge");
  return launch_merge<T>(attn, out, images, g, num_sms, st);
}

template <typename T>
int launch_merge(const void* attn, void* out, int64_t images, const WinGeom& g, int num_sms, cudaStream_t st) {
  constexpr int kVec = 16 / (int)sizeof(T);
  const bool vec = (g.hd * (int)sizeof(T)) % 16 == 0 && aligned16_all(attn, out, out);
  const int64_t chunks = images * g.h * (int64_t)g.w * g.c() / (vec ? kVec : 1);
  const int64_t blocks = std::min<int64_t>((chunks + 255) / 256, (int64_t)num_sms * 16);
  // 32-bit indices when every source and destination element index fits
  const int64_t elems = std::max<int64_t>(images * g.h * (int64_t)g.w * g.c(),
                                          images * g.nwh * (int64_t)g.nww * g.nh * g.n() * g.hd);
  const bool narrow = elems < (int64_t)0x7fffffff;
  const auto* ap = static_cast<const T*>(attn);
  auto* op = static_cast<T*>(out);
  if (vec && narrow)
    window_merge_kernel<T, kVec, uint32_t><<<(unsigned)blocks, 256, 0, st>>>(ap, op, (long)images, g);
  else if (vec)
    window_merge_kernel<T, kVec, uint64_t><<<(unsigned)blocks, 256, 0, st>>>(ap, op, (long)images, g);
  else if (narrow)
    window_merge_kernel<T, 1, uint32_t><<<(unsigned)blocks, 256, 0, st>>>(ap, op, (long)images, g);
  else
    window_merge_kernel<T, 1, uint64_t><<<(unsigned)blocks, 256, 0, st>>>(ap, op, (long)images, g);
  return launch_status("window_merge");
}

// ---------------------------------------------------------------------------------------- GEMM
// A CTA pair (cluster of 2, one cta_group::2 MMA) per 256 x 256 tile; one CTA per 128 x 256 tile where
// no 2-CTA cluster can be resident (a device partition that does not offer clusters).
template <typename T, int EPI, bool kPair>
int launch_gemm_as(const void* a, const void* w, tgemm::Params p, cudaStream_t st, int num_sms, int clusters) {
  constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int tm = tgemm::tile_m(kPair), smem = tgemm::smem_bytes(kPair);
  p.group = p.band_rows > 0 ? std::max(1, std::min(16, (p.band_rows + tm - 1) / tm)) : 1;
  CUtensorMap ma, mb;
  int rc = tcg::make_map(&ma, bf16, a, (uint64_t)p.K, (uint64_t)p.M, tgemm::kBK, tgemm::kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = tcg::make_map(&mb, bf16, w, (uint64_t)p.K, (uint64_t)p.N, tgemm::kBK, tgemm::b_rows(kPair),
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return fail(SAMRS_ERR_LAUNCH, "linear: %s", tc_error_string(rc));
  auto kern = tgemm::gemm_kernel<T, EPI, kPair>;
  const long tiles = (long)((p.M + tm - 1) / tm) * ((p.N + tgemm::kBN - 1) / tgemm::kBN);
  if (!kPair) {
    const int grid = (int)(tiles < num_sms ? tiles : num_sms);
    kern<<<grid, tgemm::threads_for(EPI, false), smem, st>>>(ma, mb, p);
    return launch_status("linear");
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(tgemm::threads_for(EPI, true));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // a persistent grid: as many pairs as are resident at once, at most one per tile
  cfg.gridDim = dim3(2 * (unsigned)(tiles < clusters ? tiles : clusters));
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, p);
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "linear (CTA pairs): launch failed: %s", cudaGetErrorString(e));
  return launch_status("linear (CTA pairs)");
}

// 2-CTA clusters of this kernel that can be resident at once on the current device (0: none), once per
// device and kernel. SAMRS_GEMM_SINGLE_CTA=1 in the environment forces the single-CTA kernel (0 clusters),
// which is how the tests compare the two.
template <typename T, int EPI>
int pair_clusters(int dev, int num_sms) {
  static std::once_flag once[kMaxDevices];
  static int clusters[kMaxDevices];
  std::call_once(once[dev], [&]() {
    auto kern = tgemm::gemm_kernel<T, EPI, true>;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tgemm::smem_bytes(true)) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * (unsigned)(num_sms / 2));
      cfg.blockDim = dim3(tgemm::threads_for(EPI, true));
      cfg.dynamicSmemBytes = tgemm::smem_bytes(true);
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    const char* force_single = getenv("SAMRS_GEMM_SINGLE_CTA");
    if (force_single && force_single[0] == '1') n = 0;
    cudaFuncSetAttribute(tgemm::gemm_kernel<T, EPI, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         tgemm::smem_bytes(false));
    cudaGetLastError();  // a refused query leaves no sticky error behind
    clusters[dev] = n;
  });
  return clusters[dev];
}

template <typename T, int EPI>
int launch_gemm(const void* a, const void* w, const tgemm::Params& p, cudaStream_t st, int num_sms) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int clusters = pair_clusters<T, EPI>(dev, num_sms);
  return clusters > 0 ? launch_gemm_as<T, EPI, true>(a, w, p, st, num_sms, clusters)
                      : launch_gemm_as<T, EPI, false>(a, w, p, st, num_sms, 0);
}

template <typename T>
int launch_gemm_epi(int epi, const void* a, const void* w, const tgemm::Params& p, cudaStream_t st, int num_sms) {
  switch (epi) {
    case tgemm::kEpiBias:
      return launch_gemm<T, tgemm::kEpiBias>(a, w, p, st, num_sms);
    case tgemm::kEpiBiasResidual:
      return launch_gemm<T, tgemm::kEpiBiasResidual>(a, w, p, st, num_sms);
    case tgemm::kEpiBiasGelu:
      return launch_gemm<T, tgemm::kEpiBiasGelu>(a, w, p, st, num_sms);
    default:
      return launch_gemm<T, tgemm::kEpiQkvWindow>(a, w, p, st, num_sms);
  }
}

// Shape and pointer checks shared by the GEMM entry points (16-bit I/O, TMA-compatible strides).
int check_gemm(const char* what, int64_t m, int n, int k, int dtype, const void* a, const void* w, const void* bias,
               const void* out) {
  if (dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_UNSUPPORTED, "%s: the tensor-core GEMM takes f16 or bf16 (dtype %d)", what, dtype);
  if (m < 0 || m > 0x7fffffffLL || n < 1 || k < 1)
    return fail(SAMRS_ERR_INVALID, "%s: bad shape m=%lld n=%d k=%d", what, (long long)m, n, k);
  if (k % 8 != 0 || n % 16 != 0)
    return fail(SAMRS_ERR_UNSUPPORTED, "%s: needs k %% 8 == 0 and n %% 16 == 0 (k=%d n=%d)", what, k, n);
  if (m > 0 && (!a || !w || !bias || !out)) return fail(SAMRS_ERR_INVALID, "%s: null pointer", what);
  if (m > 0 && !aligned16_all(a, w, bias)) return fail(SAMRS_ERR_INVALID, "%s: pointers must be 16-byte aligned", what);
  if (m > 0 && !aligned16_all(out, out, out)) return fail(SAMRS_ERR_INVALID, "%s: pointers must be 16-byte aligned", what);
  return SAMRS_OK;
}

// ---------------------------------------------------------------------------------------- LayerNorm
template <typename T>
int launch_layer_norm(const void* x, const void* wt, const void* b, void* out, int64_t rows, int c, float eps,
                      cudaStream_t st, int num_sms) {
  const long blocks = std::min<int64_t>((rows + 7) / 8, (int64_t)num_sms * 16);
  const auto* xp = static_cast<const T*>(x);
  const auto* wp = static_cast<const T*>(wt);
  const auto* bp = static_cast<const T*>(b);
  auto* op = static_cast<T*>(out);
  const bool vec = sizeof(T) == 2 && c % 8 == 0 && c <= 256 * kLnMaxChunks && aligned16_all(x, wt, b) &&
                   aligned16_all(out, out, out);
  if (vec) {
    const int nch = (c + 255) / 256;
    if (nch <= 3)
      layer_norm_vec_kernel<T, 3><<<(unsigned)blocks, 256, 0, st>>>(xp, wp, bp, op, rows, c, eps);
    else if (nch <= 4)
      layer_norm_vec_kernel<T, 4><<<(unsigned)blocks, 256, 0, st>>>(xp, wp, bp, op, rows, c, eps);
    else if (nch <= 5)
      layer_norm_vec_kernel<T, 5><<<(unsigned)blocks, 256, 0, st>>>(xp, wp, bp, op, rows, c, eps);
    else
      layer_norm_vec_kernel<T, kLnMaxChunks><<<(unsigned)blocks, 256, 0, st>>>(xp, wp, bp, op, rows, c, eps);
  } else {
    layer_norm_any_kernel<T><<<(unsigned)blocks, 256, 0, st>>>(xp, wp, bp, op, rows, c, eps);
  }
  return launch_status("layer_norm");
}

// Test hook of the windowed kernel's exp2 polynomial (sm100::ex2_poly2): y_poly = the polynomial, y_lib =
// CUDA's exp2f, for the same x (pairs (2i, 2i+1), as the kernel evaluates them).
__global__ void selftest_ex2_kernel(const float* __restrict__ x, float* __restrict__ y_poly, float* __restrict__ y_lib,
                                    int64_t n) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; 2 * p < n; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = 2 * p;
    const bool two = i + 1 < n;
    const float2 xv = make_float2(x[i], two ? x[i + 1] : 0.f);
    const float2 yv = sm100::ex2_poly2(xv);
    y_poly[i] = yv.x;
    y_lib[i] = exp2f(xv.x);
    if (two) {
      y_poly[i + 1] = yv.y;
      y_lib[i + 1] = exp2f(xv.y);
    }
  }
}

}  // namespace

extern "C" {

const char* samrs_last_error(void) { return g_last_error; }

int samrs_abi_version(void) { return SAMRS_ABI_VERSION; }

int samrs_relpos_attn_fwd_ex(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                             int h, int w, int hd, float scale, int dtype, int impl, void* stream) {
  int rc = check_common(bh, h, w, hd, dtype, "relpos_attn");
  if (rc) return rc;
  if (impl != SAMRS_IMPL_AUTO && impl != SAMRS_IMPL_SIMT && impl != SAMRS_IMPL_TC)
    return fail(SAMRS_ERR_INVALID, "relpos_attn: unknown impl %d", impl);
  if (bh == 0) return ok();
  if (!q || !kt || !v || !table || !out) return fail(SAMRS_ERR_INVALID, "relpos_attn: null pointer");
  const size_t es = elem_size(dtype);
  if (!aligned(q, es) || !aligned(kt, es) || !aligned(v, es) || !aligned(table, es) || !aligned(out, es))
    return fail(SAMRS_ERR_INVALID, "relpos_attn: pointers must be aligned to the element size");
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (impl != SAMRS_IMPL_SIMT) {
    const TcShape shape = tc_select(h, w, hd, q, kt, v, table, out);
    if (shape != TcShape::kNone) {
      if (dtype == SAMRS_F32)
        rc = tc_launch_f32(shape, q, kt, v, table, out, bh, hd, scale, st);
      else
        rc = dtype == SAMRS_BF16
                 ? tc_launch<__nv_bfloat16>(shape, q, kt, v, table, out, bh, h, w, hd, scale, st, dev->num_sms)
                 : tc_launch<__half>(shape, q, kt, v, table, out, bh, h, w, hd, scale, st, dev->num_sms);
      if (rc == 0) return launch_status("relpos_attn_tc");
      return fail(SAMRS_ERR_LAUNCH, "relpos_attn_tc: %s", tc_error_string(rc));
    }
  }
  if (impl == SAMRS_IMPL_TC)
    return fail(SAMRS_ERR_UNSUPPORTED,
                "relpos_attn: no tensor-core kernel for dtype %d, grid %dx%d, head_dim %d (or misaligned buffers)", dtype,
                h, w, hd);
  switch (dtype) {
    case SAMRS_F32:
      return launch_simt<float>(q, kt, v, table, out, bh, h, w, hd, scale, st, *dev);
    case SAMRS_F16:
      return launch_simt<__half>(q, kt, v, table, out, bh, h, w, hd, scale, st, *dev);
    default:
      return launch_simt<__nv_bfloat16>(q, kt, v, table, out, bh, h, w, hd, scale, st, *dev);
  }
}

int samrs_relpos_attn_fwd(const void* q, const void* kt, const void* v, const void* table, void* out, int64_t bh,
                          int h, int w, int hd, float scale, int dtype, void* stream) {
  return samrs_relpos_attn_fwd_ex(q, kt, v, table, out, bh, h, w, hd, scale, dtype, SAMRS_IMPL_AUTO, stream);
}

int samrs_relpos_softmax_fwd(const void* s, const void* q, const void* table, void* out, int64_t rows, int h, int w,
                             int hd, float scale, int dtype, void* stream) {
  int rc = check_common(rows, h, w, hd, dtype, "relpos_softmax");
  if (rc) return rc;
  if ((int64_t)h * w > 16384) return fail(SAMRS_ERR_UNSUPPORTED, "relpos_softmax: row of %d exceeds 16384", h * w);
  if (rows % ((int64_t)h * w) != 0)
    return fail(SAMRS_ERR_INVALID, "relpos_softmax: rows (%lld) must be a multiple of h*w (%d)", (long long)rows, h * w);
  if (rows == 0) return ok();
  if (!s || !q || !table || !out) return fail(SAMRS_ERR_INVALID, "relpos_softmax: null pointer");
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SAMRS_F32:
      return launch_softmax<float>(s, q, table, out, rows, h, w, hd, scale, st);
    case SAMRS_F16:
      return launch_softmax<__half>(s, q, table, out, rows, h, w, hd, scale, st);
    default:
      return launch_softmax<__nv_bfloat16>(s, q, table, out, rows, h, w, hd, scale, st);
  }
}

int samrs_qkv_split_fwd(const void* y, const void* bias, void* out, int64_t tokens, int n, int nh, int hd, int dtype,
                        void* stream) {
  if (dtype != SAMRS_F32 && dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_INVALID, "qkv_split: unsupported dtype code %d", dtype);
  if (tokens < 0 || n < 1 || nh < 1 || hd < 1 || hd > 1024)
    return fail(SAMRS_ERR_INVALID, "qkv_split: bad geometry tokens=%lld n=%d nh=%d hd=%d", (long long)tokens, n, nh,
                hd);
  if (tokens % n != 0) return fail(SAMRS_ERR_INVALID, "qkv_split: tokens (%lld) not a multiple of n (%d)", (long long)tokens, n);
  if (tokens == 0) return ok();
  if (!y || !bias || !out) return fail(SAMRS_ERR_INVALID, "qkv_split: null pointer");
  DevInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SAMRS_F32:
      return launch_split<float>(y, bias, out, tokens, n, nh, hd, st);
    case SAMRS_F16:
      return launch_split<__half>(y, bias, out, tokens, n, nh, hd, st);
    default:
      return launch_split<__nv_bfloat16>(y, bias, out, tokens, n, nh, hd, st);
  }
}

int samrs_qkv_split_window_fwd(const void* y, const void* bias, void* out, int64_t images, int h, int w, int ws, int nh,
                               int hd, int dtype, void* stream) {
  if (dtype != SAMRS_F32 && dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_INVALID, "qkv_split_window: unsupported dtype code %d", dtype);
  WinGeom g;
  int rc = win_geom("qkv_split_window", images, h, w, ws, nh, hd, &g);
  if (rc) return rc;
  if (images == 0) return ok();
  if (!y || !bias || !out) return fail(SAMRS_ERR_INVALID, "qkv_split_window: null pointer");
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SAMRS_F32:
      return split_window_any<float>(y, bias, out, images, g, ws > 0, st);
    case SAMRS_F16:
      return split_window_any<__half>(y, bias, out, images, g, ws > 0, st);
    default:
      return split_window_any<__nv_bfloat16>(y, bias, out, images, g, ws > 0, st);
  }
}

int samrs_window_merge_fwd(const void* attn, void* out, int64_t images, int h, int w, int ws, int nh, int hd, int dtype,
                           void* stream) {
  if (dtype != SAMRS_F32 && dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_INVALID, "window_merge: unsupported dtype code %d", dtype);
  WinGeom g;
  int rc = win_geom("window_merge", images, h, w, ws, nh, hd, &g);
  if (rc) return rc;
  if (images == 0) return ok();
  if (!attn || !out) return fail(SAMRS_ERR_INVALID, "window_merge: null pointer");
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SAMRS_F32:
      return merge_any<float>(attn, out, images, g, ws > 0, dev->num_sms, st);
    case SAMRS_F16:
      return merge_any<__half>(attn, out, images, g, ws > 0, dev->num_sms, st);
    default:
      return merge_any<__nv_bfloat16>(attn, out, images, g, ws > 0, dev->num_sms, st);
  }
}

int samrs_linear_fwd(const void* a, const void* w, const void* bias, const void* res, void* out, int64_t m, int n, int k,
                     int epilogue, int dtype, void* stream) {
  if (epilogue != SAMRS_EPI_BIAS && epilogue != SAMRS_EPI_BIAS_RESIDUAL && epilogue != SAMRS_EPI_BIAS_GELU)
    return fail(SAMRS_ERR_INVALID, "linear: unknown epilogue %d", epilogue);
  int rc = check_gemm("linear", m, n, k, dtype, a, w, bias, out);
  if (rc) return rc;
  if (epilogue == SAMRS_EPI_BIAS_RESIDUAL && m > 0 && (!res || !aligned16_all(res, res, res)))
    return fail(SAMRS_ERR_INVALID, "linear: the residual must be a 16-byte aligned [m, n] buffer");
  if (m == 0) return ok();
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  tgemm::Params p{};
  p.M = (int)m;
  p.N = n;
  p.K = k;
  p.group = 1;
  p.bias = bias;
  p.res = res;
  p.out = out;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == SAMRS_BF16 ? launch_gemm_epi<__nv_bfloat16>(epilogue, a, w, p, st, dev->num_sms)
                             : launch_gemm_epi<__half>(epilogue, a, w, p, st, dev->num_sms);
}

int samrs_qkv_linear_window_fwd(const void* x, const void* w, const void* bias, void* out, int64_t images, int h,
                                int w_grid, int ws, int nh, int hd, int dtype, void* stream) {
  WinGeom g;
  int rc = win_geom("qkv_linear_window", images, h, w_grid, ws, nh, hd, &g);
  if (rc) return rc;
  if (hd % 16 != 0)
    return fail(SAMRS_ERR_UNSUPPORTED, "qkv_linear_window: head_dim %d is not a multiple of 16", hd);
  const int64_t m = images * (int64_t)h * w_grid;
  const int c = nh * hd;
  rc = check_gemm("qkv_linear_window", m, 3 * c, c, dtype, x, w, bias, out);
  if (rc) return rc;
  if (images == 0) return ok();
  const int64_t bh = images * g.nwh * (int64_t)g.nww * nh;
  if (bh * g.n() > 0x7fffffffLL || bh * g.n() * (int64_t)hd > ((int64_t)1 << 40))
    return fail(SAMRS_ERR_UNSUPPORTED, "qkv_linear_window: batch too large");
  DevInfo* dev = nullptr;
  rc = device_info(&dev);
  if (rc) return rc;
  tgemm::Params p{};
  p.M = (int)m;
  p.N = 3 * c;
  p.K = c;
  // the M blocks of one band of window rows (ws grid rows of every image column) run side by side
  p.band_rows = ws ? (int)std::min<int64_t>((int64_t)g.wh * w_grid, 1 << 20) : 0;
  p.bias = bias;
  p.out = out;
  const int pairs = w_grid % 2 == 0 && g.ww % 2 == 0;  // ws = 0: g.ww = w_grid
  p.g = tgemm::QkvGeom{h, w_grid, g.wh, g.ww, g.nwh, g.nww, nh, hd, (long)(bh * g.n() * hd), pairs};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = dtype == SAMRS_BF16 ? launch_gemm<__nv_bfloat16, tgemm::kEpiQkvWindow>(x, w, p, st, dev->num_sms)
                           : launch_gemm<__half, tgemm::kEpiQkvWindow>(x, w, p, st, dev->num_sms);
  if (rc) return rc;
  // the pad tokens of the padded grid (none for ws = 0 or a grid that the windows tile exactly)
  const int64_t pads = images * ((int64_t)g.nwh * g.wh * g.nww * g.ww - (int64_t)h * w_grid);
  if (pads > 0) {
    const int64_t units = images * (g.nwh + g.nww) * (int64_t)nh;  // at least the edge windows x heads
    const unsigned blocks = (unsigned)std::min<int64_t>(units, (int64_t)dev->num_sms * 16);
    if (dtype == SAMRS_BF16)
      qkv_pad_fill_kernel<__nv_bfloat16><<<blocks, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(bias),
                                                                 static_cast<__nv_bfloat16*>(out), (long)images, g);
    else
      qkv_pad_fill_kernel<__half><<<blocks, 128, 0, st>>>(static_cast<const __half*>(bias), static_cast<__half*>(out),
                                                          (long)images, g);
    return launch_status("qkv_pad_fill");
  }
  return ok();
}

int samrs_layer_norm_fwd(const void* x, const void* weight, const void* bias, void* out, int64_t rows, int c, float eps,
                         int dtype, void* stream) {
  if (dtype != SAMRS_F32 && dtype != SAMRS_F16 && dtype != SAMRS_BF16)
    return fail(SAMRS_ERR_INVALID, "layer_norm: unsupported dtype code %d", dtype);
  if (rows < 0 || c < 1) return fail(SAMRS_ERR_INVALID, "layer_norm: bad shape rows=%lld c=%d", (long long)rows, c);
  if (!(eps >= 0.f)) return fail(SAMRS_ERR_INVALID, "layer_norm: eps must be >= 0");
  if (rows == 0) return ok();
  if (!x || !weight || !bias || !out) return fail(SAMRS_ERR_INVALID, "layer_norm: null pointer");
  const size_t es = elem_size(dtype);
  if (!aligned(x, es) || !aligned(weight, es) || !aligned(bias, es) || !aligned(out, es))
    return fail(SAMRS_ERR_INVALID, "layer_norm: pointers must be aligned to the element size");
  DevInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SAMRS_F32:
      return launch_layer_norm<float>(x, weight, bias, out, rows, c, eps, st, dev->num_sms);
    case SAMRS_F16:
      return launch_layer_norm<__half>(x, weight, bias, out, rows, c, eps, st, dev->num_sms);
    default:
      return launch_layer_norm<__nv_bfloat16>(x, weight, bias, out, rows, c, eps, st, dev->num_sms);
  }
}

int samrs_test_hooks(int64_t wait_limit_cycles, int withhold_key_tile) {
  if (wait_limit_cycles < 0) return fail(SAMRS_ERR_INVALID, "test_hooks: negative wait limit");
  const long long lim = (long long)wait_limit_cycles;
  cudaError_t e = cudaMemcpyToSymbol(samrs::g_wait_limit, &lim, sizeof(lim));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(samrs::g_withhold_key_tile, &withhold_key_tile, sizeof(int));
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "test_hooks: %s", cudaGetErrorString(e));
  return ok();
}

int samrs_device_status(void* stream, int clear) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(SAMRS_ERR_NODEVICE, "no CUDA device is current");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "device_status: stream sync failed: %s", cudaGetErrorString(e));
  unsigned int word = 0;
  e = cudaMemcpyFromSymbol(&word, samrs::g_status, sizeof(word));
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "device_status: read failed: %s", cudaGetErrorString(e));
  if (clear && word) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(samrs::g_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "device_status: clear failed: %s", cudaGetErrorString(e));
  }
  g_fault_seen[dev].store(clear ? 0u : word, std::memory_order_relaxed);
  return (int)word;
}

int samrs_recompute_count(void* stream, int64_t* count, int clear) {
  if (!count) return fail(SAMRS_ERR_INVALID, "recompute_count: null output pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "recompute_count: stream sync failed: %s", cudaGetErrorString(e));
  unsigned long long v = 0;
  e = cudaMemcpyFromSymbol(&v, samrs::g_recomputed, sizeof(v));
  if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "recompute_count: read failed: %s", cudaGetErrorString(e));
  if (clear) {
    const unsigned long long zero = 0;
    e = cudaMemcpyToSymbol(samrs::g_recomputed, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(SAMRS_ERR_LAUNCH, "recompute_count: clear failed: %s", cudaGetErrorString(e));
  }
  *count = (int64_t)v;
  return ok();
}

int samrs_global_policy(const void* table, double* share, int* exact, int reset) {
  if (!share || !exact) return fail(SAMRS_ERR_INVALID, "global_policy: null output pointer");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(SAMRS_ERR_NODEVICE, "no CUDA device is current");
  if (reset) global_policy().reset(dev);
  global_policy().state(dev, table, share, exact);
  return ok();
}

int samrs_selftest_ex2(const void* x, void* y_poly, void* y_lib, int64_t n, void* stream) {
  if (n < 0 || n > ((int64_t)1 << 30)) return fail(SAMRS_ERR_INVALID, "selftest_ex2: n = %lld", (long long)n);
  if (n == 0) return ok();
  if (!x || !y_poly || !y_lib) return fail(SAMRS_ERR_INVALID, "selftest_ex2: null pointer");
  DevInfo* dev = nullptr;
  int rc = device_info(&dev);
  if (rc) return rc;
  const int64_t pairs = (n + 1) / 2;
  const unsigned blocks = (unsigned)std::min<int64_t>((pairs + 255) / 256, (int64_t)dev->num_sms * 8);
  selftest_ex2_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(x), static_cast<float*>(y_poly), static_cast<float*>(y_lib), n);
  return launch_status("selftest_ex2");
}

}  // extern "C"
