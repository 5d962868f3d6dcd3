/*
 * relpos_oracle.c - CPU restatement of sam-rs's own CPU implementation of the SAM encoder's
 * decomposed-rel-pos attention. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py load it as the checker / the timed CPU reference. The product
 * library (sam-rs_b200/) never links or calls it.
 *
 * Reference: apiplant/sam-rs 0.1.1 (Rust). What each function restates:
 *   oracle_attention_relpos_f32   src/kernels.rs:131-225, `cpu::TiledAttention::cpu_fwd`, the exact
 *                                 f32 branch (packs == None): 32-row query tiles (TILE, :116), one task
 *                                 per (head, tile) (:157), QK^T GEMM (:183-185), scalar rel-bias dots
 *                                 (:190-196), scalar biased softmax with exp (:197-214), PV GEMM
 *                                 (:218-220). The f32 GEMMs are the `gemm` 0.19.0 crate in the
 *                                 reference (Cargo.lock:979-980, not vendored); here they are an
 *                                 AVX-512 FMA register-blocked GEMM of our own (same math, a
 *                                 different summation order, ~1e-7 relative).
 *   oracle_attention_relpos_bf16  src/kernels.rs:139-179 with src/cpu_gemm.rs: the default CPU mode on
 *                                 AVX-512-BF16 hosts (`enabled()`, cpu_gemm.rs:14-32): K and V packed
 *                                 once per head into bf16 panels of NR=32 columns (`PackedB`, :47-96,
 *                                 RNE conversion :38-45), `vdpbf16ps` microkernel with MR=8 (:128-178),
 *                                 `rel_bias` (:288-303), AVX-512 `softmax_row` (:224-270) with a
 *                                 degree-6 polynomial 2^x (`exp_ps`, :272-286; the coefficients are the
 *                                 Taylor terms ln2^k/k!, computed here from ln 2).
 *   oracle_relpos_softmax_f32     src/kernels.rs:62-105, `cpu::RelposSoftmax::cpu_fwd` (probs only).
 *   oracle_qkv_split_f32          src/kernels.rs:234-263, `cpu::QkvSplit::cpu_fwd`.
 *
 * Parity status: the reference cannot be built in this environment (no Rust toolchain) and ships no
 * golden vectors for this path, so this restatement is cross-checked against an independent float64
 * restatement of the reference's tensor-op fallback (src/kernels.rs:20-42), committed as fixtures
 * under tests/golden/ - parity against outputs of the reference binary itself is unpinned.
 *
 * Build: see oracle/build_oracle.py (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>
#include <immintrin.h>

#define TILE 32 /* src/kernels.rs:116 */

/* ------------------------------------------------------------------------------------------ */
/* f32 GEMM  C[m,n] = A[m,k] . B[k,n]  (row-major, leading dimensions given)                  */
/* ------------------------------------------------------------------------------------------ */

static void gemm_f32_scalar(int m, int n, int k, const float* A, long lda, const float* B, long ldb, float* C,
                            long ldc) {
  for (int r = 0; r < m; ++r) {
    float* c = C + r * ldc;
    for (int j = 0; j < n; ++j) c[j] = 0.f;
    for (int p = 0; p < k; ++p) {
      const float a = A[r * lda + p];
      const float* b = B + p * ldb;
      for (int j = 0; j < n; ++j) c[j] = fmaf(a, b[j], c[j]);
    }
  }
}

#define MR 8
#define NR 32

__attribute__((target("avx512f,fma"))) static inline void gemm_tile_avx512(int mr, int nr, int k, const float* A,
                                                                          long lda, const float* B, long ldb,
                                                                          float* C, long ldc) {
  __m512 acc[MR][2];
  for (int r = 0; r < MR; ++r) acc[r][0] = acc[r][1] = _mm512_setzero_ps();
  const __mmask16 m0 = nr >= 16 ? (__mmask16)0xffff : (__mmask16)((1u << nr) - 1);
  const __mmask16 m1 = nr >= 32 ? (__mmask16)0xffff : (nr <= 16 ? 0 : (__mmask16)((1u << (nr - 16)) - 1));
  for (int p = 0; p < k; ++p) {
    const __m512 b0 = _mm512_maskz_loadu_ps(m0, B + p * ldb);
    const __m512 b1 = _mm512_maskz_loadu_ps(m1, B + p * ldb + 16);
    for (int r = 0; r < MR; ++r) {
      if (r < mr) {
        const __m512 a = _mm512_set1_ps(A[r * lda + p]);
        acc[r][0] = _mm512_fmadd_ps(a, b0, acc[r][0]);
        acc[r][1] = _mm512_fmadd_ps(a, b1, acc[r][1]);
      }
    }
  }
  for (int r = 0; r < mr; ++r) {
    _mm512_mask_storeu_ps(C + r * ldc, m0, acc[r][0]);
    _mm512_mask_storeu_ps(C + r * ldc + 16, m1, acc[r][1]);
  }
}

__attribute__((target("avx512f,fma"))) static void gemm_f32_avx512(int m, int n, int k, const float* A, long lda,
                                                                  const float* B, long ldb, float* C, long ldc) {
  for (int r0 = 0; r0 < m; r0 += MR) {
    const int mr = m - r0 < MR ? m - r0 : MR;
    for (int c0 = 0; c0 < n; c0 += NR) {
      const int nr = n - c0 < NR ? n - c0 : NR;
      if (mr == MR)
        gemm_tile_avx512(MR, nr, k, A + r0 * lda, lda, B + c0, ldb, C + r0 * ldc + c0, ldc);
      else
        gemm_tile_avx512(mr, nr, k, A + r0 * lda, lda, B + c0, ldb, C + r0 * ldc + c0, ldc);
    }
  }
}

static int have_avx512f(void) { return __builtin_cpu_supports("avx512f"); }
static int have_avx512bf16(void) {
  return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bf16");
}

static void gemm_f32(int m, int n, int k, const float* A, long lda, const float* B, long ldb, float* C, long ldc) {
  if (have_avx512f())
    gemm_f32_avx512(m, n, k, A, lda, B, ldb, C, ldc);
  else
    gemm_f32_scalar(m, n, k, A, lda, B, ldb, C, ldc);
}

/* Sequential left-to-right f32 dot product, as `iter().zip().map(a*b).sum()` in the reference. */
static inline float dot_seq(const float* a, const float* b, int n) {
  float s = 0.f;
  for (int d = 0; d < n; ++d) s += a[d] * b[d];
  return s;
}

/* rh[kh] = q . Th[i+h-1-kh], rw[kw] = q . Tw[j+w-1-kw]  (src/kernels.rs:190-196) */
static void rel_bias_scalar(const float* qr, const float* th, const float* tw, int h, int w, int hd, int i, int j,
                            float* rh, float* rw) {
  for (int kh = 0; kh < h; ++kh) rh[kh] = dot_seq(th + (long)(i + h - 1 - kh) * hd, qr, hd);
  for (int kw = 0; kw < w; ++kw) rw[kw] = dot_seq(tw + (long)(j + w - 1 - kw) * hd, qr, hd);
}

/* Biased softmax of one score row in place (src/kernels.rs:197-214). */
static void softmax_row_exact(float* s, const float* rh, const float* rw, int h, int w, float scale) {
  float mx = -INFINITY;
  for (int kh = 0; kh < h; ++kh)
    for (int kw = 0; kw < w; ++kw) {
      float* x = &s[kh * w + kw];
      float t = *x * scale;
      t = t + rh[kh];
      t = t + rw[kw];
      *x = t;
      mx = fmaxf(mx, t);
    }
  const int n = h * w;
  float sum = 0.f;
  for (int k = 0; k < n; ++k) {
    s[k] = expf(s[k] - mx);
    sum += s[k];
  }
  const float inv = 1.0f / sum;
  for (int k = 0; k < n; ++k) s[k] *= inv;
}

static int check_geom(long bh, int h, int w, int hd) {
  return bh < 0 || h < 1 || w < 1 || hd < 1 || h > 4096 || w > 4096 || hd > 4096;
}

/* Exact f32 fused attention: out[bh, n, hd]. Returns 0 on success. */
int oracle_attention_relpos_f32(const float* q, const float* kt, const float* v, const float* table, float* out,
                                long bh, int h, int w, int hd, float scale, int threads) {
  if (check_geom(bh, h, w, hd)) return -1;
  const int n = h * w;
  const int tiles = (n + TILE - 1) / TILE;
  const float* th = table;
  const float* tw = table + (long)(2 * h - 1) * hd;
  const long tasks = bh * tiles;
  if (threads < 1) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
  {
    float* sc = (float*)malloc(sizeof(float) * TILE * n);
    float* rh = (float*)malloc(sizeof(float) * h);
    float* rw = (float*)malloc(sizeof(float) * w);
#pragma omp for schedule(dynamic, 1)
    for (long task = 0; task < tasks; ++task) {
      const long b = task / tiles;
      const int t = (int)(task % tiles);
      const int r0 = t * TILE;
      const int rows = n - r0 < TILE ? n - r0 : TILE;
      const float* qb = q + (b * n + r0) * hd;
      const float* ktb = kt + b * (long)hd * n;
      const float* vb = v + b * (long)n * hd;
      float* o = out + (b * n + r0) * hd;
      gemm_f32(rows, n, hd, qb, hd, ktb, n, sc, n); /* scores = q_tile @ kt */
      for (int r = 0; r < rows; ++r) {
        const int row = r0 + r;
        rel_bias_scalar(qb + (long)r * hd, th, tw, h, w, hd, row / w, row % w, rh, rw);
        softmax_row_exact(sc + (long)r * n, rh, rw, h, w, scale);
      }
      gemm_f32(rows, hd, n, sc, n, vb, hd, o, hd); /* out_tile = probs @ v */
    }
    free(sc);
    free(rh);
    free(rw);
  }
  return 0;
}

/* Probabilities only: out[rows, n] (src/kernels.rs:62-105). */
int oracle_relpos_softmax_f32(const float* s, const float* q, const float* table, float* out, long rows, int h,
                              int w, int hd, float scale, int threads) {
  if (check_geom(rows, h, w, hd)) return -1;
  const int n = h * w;
  const float* th = table;
  const float* tw = table + (long)(2 * h - 1) * hd;
  if (threads < 1) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
  {
    float* rh = (float*)malloc(sizeof(float) * h);
    float* rw = (float*)malloc(sizeof(float) * w);
#pragma omp for schedule(static)
    for (long row = 0; row < rows; ++row) {
      const int rem = (int)(row % n);
      rel_bias_scalar(q + row * hd, th, tw, h, w, hd, rem / w, rem % w, rh, rw);
      float* o = out + row * n;
      memcpy(o, s + row * n, sizeof(float) * n);
      softmax_row_exact(o, rh, rw, h, w, scale);
    }
    free(rh);
    free(rw);
  }
  return 0;
}

/* qkv split: y [tokens, 3*nh*hd] + bias -> out [3, tokens*nh*hd] (q, kt, v). */
int oracle_qkv_split_f32(const float* y, const float* bias, float* out, long tokens, int n, int nh, int hd) {
  if (tokens < 0 || n < 1 || nh < 1 || hd < 1 || tokens % n) return -1;
  const long c = (long)nh * hd;
  const long plane = tokens * c;
  for (long t = 0; t < tokens; ++t) {
    const long win = t / n, tok = t % n;
    for (int which = 0; which < 3; ++which)
      for (int head = 0; head < nh; ++head) {
        const long bhx = win * nh + head;
        for (int d = 0; d < hd; ++d) {
          const long col = which * c + (long)head * hd + d;
          const long dst = which == 1 ? (bhx * hd + d) * n + tok : (bhx * n + tok) * hd + d;
          out[which * plane + dst] = y[t * 3 * c + col] + bias[col];
        }
      }
  }
  return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* bf16 path (default CPU mode of the reference on AVX-512 BF16 hosts)                        */
/* ------------------------------------------------------------------------------------------ */

#define BNR 32 /* cpu_gemm.rs:34 */
#define BMR 8  /* cpu_gemm.rs:35 */

/* Round-to-nearest-even f32 -> bf16 bits, NaN kept quiet (cpu_gemm.rs:38-45). */
static inline uint16_t bf16_bits(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  if (x != x) return (uint16_t)((b >> 16) | 0x40);
  return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

typedef struct {
  int k, n, kp;
  uint32_t* data; /* panels * kp * BNR pairs (k even in the low half) */
} packed_b;

/* PackedB::from_slice: row-major [k, n] f32 -> bf16 panels of BNR columns (cpu_gemm.rs:62-80). */
static void packed_b_init(packed_b* pb, const float* wmat, int k, int n) {
  pb->k = k;
  pb->n = n;
  pb->kp = (k + 1) / 2;
  const int panels = (n + BNR - 1) / BNR;
  pb->data = (uint32_t*)calloc((size_t)panels * pb->kp * BNR, sizeof(uint32_t));
  for (int p = 0; p < panels; ++p)
    for (int qq = 0; qq < pb->kp; ++qq)
      for (int c = 0; c < BNR; ++c) {
        const int col = p * BNR + c;
        if (col >= n) continue;
        const uint32_t lo = bf16_bits(wmat[(long)2 * qq * n + col]);
        const uint32_t hi = 2 * qq + 1 < k ? bf16_bits(wmat[(long)(2 * qq + 1) * n + col]) : 0u;
        pb->data[((long)p * pb->kp + qq) * BNR + c] = lo | (hi << 16);
      }
}

static void packed_b_free(packed_b* pb) { free(pb->data); }

/* c[rows, n] = a[rows, k] @ B for one block of rows (cpu_gemm.rs:128-178). `ab` is scratch of
 * roundup(rows, BMR) * kpad u16. */
__attribute__((target("avx512f,avx512bf16,avx512bw,avx512vl"))) static void packed_block(const packed_b* b,
                                                                                        const float* a, int rows,
                                                                                        float* c, uint16_t* ab) {
  const int k = b->k, n = b->n, kp = b->kp;
  const int kpad = kp * 2;
  const int padded = (rows + BMR - 1) / BMR * BMR;
  memset(ab, 0, sizeof(uint16_t) * (size_t)padded * kpad);
  for (int r = 0; r < rows; ++r) {
    const float* src = a + (long)r * k;
    uint16_t* dst = ab + (long)r * kpad;
    int i = 0;
    for (; i + 16 <= k; i += 16) {
      const __m256bh hv = _mm512_cvtneps_pbh(_mm512_loadu_ps(src + i));
      _mm256_storeu_si256((__m256i*)(dst + i), (__m256i)hv);
    }
    for (; i < k; ++i) dst[i] = bf16_bits(src[i]);
  }
  const int panels = (n + BNR - 1) / BNR;
  float tmp[BMR * BNR];
  for (int p = 0; p < panels; ++p) {
    const uint32_t* bp = b->data + (long)p * kp * BNR;
    const int cols = n - p * BNR < BNR ? n - p * BNR : BNR;
    for (int r0 = 0; r0 < padded; r0 += BMR) {
      const uint16_t* ap = ab + (long)r0 * kpad;
      __m512 acc[BMR][2];
      for (int r = 0; r < BMR; ++r) acc[r][0] = acc[r][1] = _mm512_setzero_ps();
      for (int qq = 0; qq < kp; ++qq) {
        const __m512bh b0 = (__m512bh)_mm512_loadu_si512((const void*)(bp + (long)qq * BNR));
        const __m512bh b1 = (__m512bh)_mm512_loadu_si512((const void*)(bp + (long)qq * BNR + 16));
        for (int r = 0; r < BMR; ++r) {
          uint32_t pair;
          memcpy(&pair, ap + (long)r * kpad + 2 * qq, 4);
          const __m512bh av = (__m512bh)_mm512_set1_epi32((int)pair);
          acc[r][0] = _mm512_dpbf16_ps(acc[r][0], av, b0);
          acc[r][1] = _mm512_dpbf16_ps(acc[r][1], av, b1);
        }
      }
      const int live = rows - r0 < BMR ? rows - r0 : BMR;
      for (int r = 0; r < live; ++r) {
        _mm512_storeu_ps(tmp + r * BNR, acc[r][0]);
        _mm512_storeu_ps(tmp + r * BNR + 16, acc[r][1]);
        memcpy(c + (long)(r0 + r) * n + p * BNR, tmp + r * BNR, sizeof(float) * cols);
      }
    }
  }
}

/* 2^x on the FMA units: round-to-nearest split x = n + f, f in [-1/2, 1/2], degree-6 Taylor
 * polynomial of 2^f (coefficients ln2^k / k!), scaled by 2^n (cpu_gemm.rs:272-286). */
__attribute__((target("avx512f"))) static inline __m512 exp_ps_poly(__m512 x, const float* coef) {
  const __m512 t = _mm512_max_ps(_mm512_mul_ps(x, _mm512_set1_ps(1.4426950408889634f)), _mm512_set1_ps(-126.0f));
  const __m512 nn = _mm512_roundscale_ps(t, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  const __m512 r = _mm512_sub_ps(t, nn);
  __m512 p = _mm512_set1_ps(coef[6]);
  for (int i = 5; i >= 0; --i) p = _mm512_fmadd_ps(p, r, _mm512_set1_ps(coef[i]));
  return _mm512_scalef_ps(p, nn);
}

/* In-place biased softmax of one row, AVX-512 (cpu_gemm.rs:224-270). */
__attribute__((target("avx512f"))) static void softmax_row_avx512(float* s, const float* rh, const float* rw, int h,
                                                                 int w, float scale, const float* coef) {
  const int n = h * w;
  const __m512 vscale = _mm512_set1_ps(scale);
  __m512 vmax = _mm512_set1_ps(-INFINITY);
  for (int kh = 0; kh < h; ++kh) {
    const __m512 add = _mm512_set1_ps(rh[kh]);
    for (int kw = 0; kw < w; kw += 16) {
      const __mmask16 m = w - kw >= 16 ? (__mmask16)0xffff : (__mmask16)((1u << (w - kw)) - 1);
      float* p = s + kh * w + kw;
      const __m512 x = _mm512_maskz_loadu_ps(m, p);
      const __m512 bb = _mm512_maskz_loadu_ps(m, rw + kw);
      const __m512 vv = _mm512_add_ps(_mm512_fmadd_ps(x, vscale, add), bb);
      _mm512_mask_storeu_ps(p, m, vv);
      vmax = _mm512_mask_max_ps(vmax, m, vmax, vv);
    }
  }
  const __m512 vm = _mm512_set1_ps(_mm512_reduce_max_ps(vmax));
  __m512 vsum = _mm512_setzero_ps();
  for (int i = 0; i < n; i += 16) {
    const __mmask16 m = n - i >= 16 ? (__mmask16)0xffff : (__mmask16)((1u << (n - i)) - 1);
    float* p = s + i;
    const __m512 e = exp_ps_poly(_mm512_sub_ps(_mm512_maskz_loadu_ps(m, p), vm), coef);
    _mm512_mask_storeu_ps(p, m, e);
    vsum = _mm512_mask_add_ps(vsum, m, vsum, e);
  }
  const __m512 inv = _mm512_set1_ps(1.0f / _mm512_reduce_add_ps(vsum));
  for (int i = 0; i < n; i += 16) {
    const __mmask16 m = n - i >= 16 ? (__mmask16)0xffff : (__mmask16)((1u << (n - i)) - 1);
    float* p = s + i;
    _mm512_mask_storeu_ps(p, m, _mm512_mul_ps(_mm512_maskz_loadu_ps(m, p), inv));
  }
}

int oracle_cpu_has_bf16(void) { return have_avx512bf16(); }

/* bf16 fused attention (bf16 GEMMs, f32 accumulation and softmax). -2 if the CPU lacks AVX-512 BF16. */
int oracle_attention_relpos_bf16(const float* q, const float* kt, const float* v, const float* table, float* out,
                                 long bh, int h, int w, int hd, float scale, int threads) {
  if (check_geom(bh, h, w, hd)) return -1;
  if (!have_avx512bf16()) return -2;
  const int n = h * w;
  const int tiles = (n + TILE - 1) / TILE;
  const float* th = table;
  const float* tw = table + (long)(2 * h - 1) * hd;
  float coef[7];
  {
    const double ln2 = 0.69314718055994530942;
    double t = 1.0;
    for (int i = 0; i <= 6; ++i) {
      coef[i] = (float)t;
      t = t * ln2 / (double)(i + 1);
    }
  }
  if (threads < 1) threads = omp_get_max_threads();
  packed_b* kp = (packed_b*)malloc(sizeof(packed_b) * (bh > 0 ? bh : 1));
  packed_b* vp = (packed_b*)malloc(sizeof(packed_b) * (bh > 0 ? bh : 1));
#pragma omp parallel for num_threads(threads) schedule(static)
  for (long b = 0; b < bh; ++b) {
    packed_b_init(&kp[b], kt + b * (long)hd * n, hd, n);
    packed_b_init(&vp[b], v + b * (long)n * hd, n, hd);
  }
  const long tasks = bh * tiles;
#pragma omp parallel num_threads(threads)
  {
    float* sc = (float*)malloc(sizeof(float) * TILE * n);
    float* rh = (float*)malloc(sizeof(float) * h);
    float* rw = (float*)malloc(sizeof(float) * w);
    const int kmax = (hd > n ? hd : n) + 2;
    uint16_t* ab = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(TILE + BMR) * kmax);
#pragma omp for schedule(dynamic, 1)
    for (long task = 0; task < tasks; ++task) {
      const long b = task / tiles;
      const int t = (int)(task % tiles);
      const int r0 = t * TILE;
      const int rows = n - r0 < TILE ? n - r0 : TILE;
      const float* qb = q + (b * n + r0) * hd;
      float* o = out + (b * n + r0) * hd;
      packed_block(&kp[b], qb, rows, sc, ab);
      for (int r = 0; r < rows; ++r) {
        const int row = r0 + r;
        rel_bias_scalar(qb + (long)r * hd, th, tw, h, w, hd, row / w, row % w, rh, rw);
        softmax_row_avx512(sc + (long)r * n, rh, rw, h, w, scale, coef);
      }
      packed_block(&vp[b], sc, rows, o, ab);
    }
    free(sc);
    free(rh);
    free(rw);
    free(ab);
  }
  for (long b = 0; b < bh; ++b) {
    packed_b_free(&kp[b]);
    packed_b_free(&vp[b]);
  }
  free(kp);
  free(vp);
  return 0;
}

int oracle_max_threads(void) { return omp_get_max_threads(); }
