/*
 * samrs_b200.h - C ABI of the B200 (sm_100a) decomposed-rel-pos attention library.
 *
 * The entry points replace the device side of the candle custom ops that sam-rs uses for the
 * attention of its SAM ViT image encoder (reference: apiplant/sam-rs 0.1.1):
 *
 *   samrs_relpos_attn_fwd    <- src/kernels.rs:896-906  `attention_relpos_cpu(q, kt, v, table, h, w, scale)`
 *                               (the fused op; on CUDA the reference instead runs
 *                               src/sam1/encoder.rs:81 `bmm(relpos_softmax(bmm(q, kt)), v)`)
 *   samrs_relpos_softmax_fwd <- src/kernels.rs:12-43   `relpos_softmax(scores, q, table, h, w, scale)`
 *                               and its CUDA launcher src/kernels.rs:1108-1149 (kernels/sam.cu:44-106)
 *   samrs_qkv_split_fwd      <- src/kernels.rs:870-894 `qkv_split(y, bias, n, nh, hd)`
 *                               and its CUDA launcher src/kernels.rs:1196-1227 (kernels/sam.cu:108-128)
 *   samrs_qkv_split_window_fwd <- src/sam1/encoder.rs:132-140 `window_partition` (zero pad) followed
 *                               by the qkv projection's bias and `qkv_split` (src/kernels.rs:870-894)
 *   samrs_window_merge_fwd   <- src/sam1/encoder.rs:82 (heads back to [windows * n, C]) followed by
 *                               `window_unpartition` (src/sam1/encoder.rs:142-145, crop)
 *
 * Conventions shared by every entry point
 *  - All tensors are dense, contiguous, row-major device buffers owned by the caller
 *    (candle allocates them with `dev.alloc`, src/kernels.rs:1124). Nothing here allocates
 *    device memory, synchronises the stream or keeps per-call host state.
 *  - `dtype`: SAMRS_F32 / SAMRS_F16 / SAMRS_BF16, the same three candle dtypes the reference
 *    dispatches on (src/kernels.rs:1086-1095). All tensors of one call share the dtype.
 *  - `stream`: a `cudaStream_t` (cudarc's stream handle in candle); NULL = legacy default stream.
 *    Work is enqueued asynchronously on it.
 *  - Return value: SAMRS_OK (0) or a negative error code; `samrs_last_error()` then returns a
 *    message for the calling thread (the reference's `bail!` text, src/kernels.rs:1092,1097-1102).
 *  - Layouts (bh = window * nh + head, exactly as `qkv_split` produces them, src/kernels.rs:880-882):
 *        q     [bh, h*w, hd]
 *        kt    [bh, hd, h*w]       (K already transposed)
 *        v     [bh, h*w, hd]
 *        table [(2h-1) + (2w-1), hd]   rel_pos_h rows then rel_pos_w rows (src/sam1/encoder.rs:56-69)
 *        out   [bh, h*w, hd]
 */
#ifndef SAMRS_B200_H
#define SAMRS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAMRS_ABI_VERSION 1

#if defined(__GNUC__)
#define SAMRS_API __attribute__((visibility("default")))
#else
#define SAMRS_API
#endif

/* dtype codes */
#define SAMRS_F32 0
#define SAMRS_F16 1
#define SAMRS_BF16 2

/* return codes */
#define SAMRS_OK 0
#define SAMRS_ERR_INVALID (-1)     /* bad shape, dtype, null or misaligned pointer        */
#define SAMRS_ERR_UNSUPPORTED (-2) /* shape outside every kernel's range                   */
#define SAMRS_ERR_LAUNCH (-3)      /* CUDA launch / attribute error                         */
#define SAMRS_ERR_DEVICE (-4)      /* a kernel reported a fault in the device status word   */
#define SAMRS_ERR_NODEVICE (-5)    /* no sm_100 device is current                           */

/* epilogues of samrs_linear_fwd */
#define SAMRS_EPI_BIAS 0          /* out = a.w^T + bias                       */
#define SAMRS_EPI_BIAS_RESIDUAL 1 /* out = res + a.w^T + bias                 */
#define SAMRS_EPI_BIAS_GELU 2     /* out = gelu_erf(a.w^T + bias)             */

/* implementation selector for samrs_relpos_attn_fwd_ex */
#define SAMRS_IMPL_AUTO 0  /* tensor-core kernels where the shape allows, SIMT kernel otherwise */
#define SAMRS_IMPL_SIMT 1  /* CUDA-core fused flash kernel (any shape, any dtype)               */
#define SAMRS_IMPL_TC 2    /* tcgen05 kernels only; SAMRS_ERR_UNSUPPORTED if the shape does not fit */

/*
 * Fused attention with decomposed relative-position bias, one pass, no N x N tensor in memory:
 *   out[b, r, :] = sum_k softmax_k( scale * q[b,r,:].kt[b,:,k] + q[b,r,:].Th[i-kh+h-1] + q[b,r,:].Tw[j-kw+w-1] ) v[b,k,:]
 *   with r = i*w + j, k = kh*w + kw, Th = table[0 : 2h-1], Tw = table[2h-1 : 2h-1+2w-1].
 * Replaces src/kernels.rs:896-906 (`attention_relpos_cpu`, whose f32 CPU body is
 * src/kernels.rs:131-225 `cpu::TiledAttention`). Limits: 1 <= h, w <= 128, 1 <= hd <= 128,
 * bh >= 0 (bh == 0 is a no-op). Pointers must be aligned to the element size. 64x64 and 14x14 layers
 * with hd 64 or 80 run on the tensor cores in every dtype (f32 as three TF32 products per contraction,
 * about 2^-20 relative error per product) when q, kt, v, table and out are 16-byte aligned; other shapes
 * run on the SIMT kernel.
 * bf16 64x64 layers run as two launches on `stream`: a single-pass kernel that marks an output block
 * (one head x 256 rows) it cannot vouch for by a NaN in the block's first element, then an exact pass of
 * the marked blocks; `out` is final only after both, i.e. in stream order (samrs_recompute_count tells
 * how many blocks took the second pass).
 */
SAMRS_API int samrs_relpos_attn_fwd(const void* q, const void* kt, const void* v, const void* table, void* out,
                          int64_t bh, int h, int w, int hd, float scale, int dtype, void* stream);

/* Same as samrs_relpos_attn_fwd with an explicit implementation choice (SAMRS_IMPL_*). */
SAMRS_API int samrs_relpos_attn_fwd_ex(const void* q, const void* kt, const void* v, const void* table, void* out,
                             int64_t bh, int h, int w, int hd, float scale, int dtype, int impl, void* stream);

/*
 * Materialising rel-pos softmax (the reference's `relpos_softmax`, src/kernels.rs:12-43, CUDA
 * kernel kernels/sam.cu:44-106):
 *   out[row, kh*w+kw] = softmax( scale*s[row, k] + q[row,:].Th[i-kh+h-1] + q[row,:].Tw[j-kw+w-1] )
 *   s, out: [rows, h*w]; q: [rows, hd]; row % (h*w) = i*w + j. rows = bh*h*w.
 * Limits: as samrs_relpos_attn_fwd, plus h*w <= 16384.
 */
SAMRS_API int samrs_relpos_softmax_fwd(const void* s, const void* q, const void* table, void* out, int64_t rows,
                             int h, int w, int hd, float scale, int dtype, void* stream);

/*
 * QKV head split (the reference's `qkv_split`, src/kernels.rs:870-894, kernels/sam.cu:108-128):
 *   y [tokens, 3*nh*hd] (+ bias [3*nh*hd]) -> out = [q | kt | v], each tokens*nh*hd elements,
 *   q, v: [bh, n, hd], kt: [bh, hd, n], bh = (tokens / n) * nh. tokens must be a multiple of n.
 */
SAMRS_API int samrs_qkv_split_fwd(const void* y, const void* bias, void* out, int64_t tokens, int n, int nh, int hd,
                        int dtype, void* stream);

/*
 * QKV head split fused with the window partition (the neighbours of the attention on the token grid):
 *   y [images*h*w, 3*nh*hd] (the qkv projection of the REAL tokens, without bias) + bias [3*nh*hd]
 *   -> out = [q | kt | v], q, v: [bh, n, hd], kt: [bh, hd, n], bh = window * nh + head,
 *   n = ws*ws, windows row-major per image over the grid zero-padded up to multiples of ws
 *   (window_partition's order). A pad token's q/k/v is the bias alone: in the reference its input is
 *   zero, so its projection is 0 * W + bias. ws = 0: one window of h x w (the global layers; no pad),
 *   which is `qkv_split` on the token grid.
 */
SAMRS_API int samrs_qkv_split_window_fwd(const void* y, const void* bias, void* out, int64_t images, int h, int w,
                                         int ws, int nh, int hd, int dtype, void* stream);

/*
 * Head merge fused with the window unpartition: attn [bh, n, hd] (layout as above) -> out [images*h*w,
 * nh*hd], the real tokens only (the pads are cropped). The output projection, a per-token GEMM, then
 * runs on the real tokens, which gives the same rows as the reference's projection before the crop.
 */
SAMRS_API int samrs_window_merge_fwd(const void* attn, void* out, int64_t images, int h, int w, int ws, int nh, int hd,
                                     int dtype, void* stream);

/*
 * Linear layer with a fused epilogue on the tensor cores (tcgen05, f16 / bf16 I/O, f32 accumulation):
 *   out[m, n] = epilogue( sum_k a[m, k] w[n, k] + bias[n] )
 * w is the weight as stored in the checkpoint ([out, in]); the reference transposes it once into its
 * `Linear` (src/cpu_gemm.rs:205-222, src/sam1/encoder.rs:61-63, 103-107) and multiplies with candle.
 * Replaces, per epilogue:
 *   SAMRS_EPI_BIAS           a Linear followed by a broadcast bias add
 *   SAMRS_EPI_BIAS_RESIDUAL  src/kernels.rs:1040-1049 `bias_residual(res, Linear(x), bias)` (proj, mlp.lin2;
 *                            CUDA kernel kernels/sam.cu:129-135), res [m, n]
 *   SAMRS_EPI_BIAS_GELU      src/kernels.rs:1051-1061 `bias_gelu(Linear(x), bias)` (mlp.lin1; kernels/sam.cu:136-143,
 *                            exact erf GELU)
 * res is read only by SAMRS_EPI_BIAS_RESIDUAL (may be NULL otherwise; it may alias out).
 * Limits: f16 / bf16, k % 8 == 0, n % 16 == 0, 16-byte aligned buffers, m < 2^31.
 */
SAMRS_API int samrs_linear_fwd(const void* a, const void* w, const void* bias, const void* res, void* out, int64_t m,
                               int n, int k, int epilogue, int dtype, void* stream);

/*
 * The qkv projection of an attention block fused with the window partition and the head split:
 *   x [images*h*w, C] (the block's normalised real tokens), w [3C, C], bias [3C], C = nh * hd ->
 *   out = [q | kt | v] exactly as samrs_qkv_split_window_fwd lays it out (q, v: [bh, n, hd], kt: [bh, hd, n],
 *   bh = window * nh + head, n = ws*ws, windows of the grid zero-padded to multiples of ws; ws = 0: one window
 *   of h x w). The GEMM's epilogue adds the bias and stores each token's q / k / v straight into its window's
 *   rows; a pad token gets the bias alone (its reference input is zero). Replaces src/sam1/encoder.rs:132-140
 *   (window_partition) + :79 (qkv Linear) + src/kernels.rs:870-894 (`qkv_split`, kernels/sam.cu:108-128).
 * Limits: f16 / bf16, hd % 16 == 0, 16-byte aligned buffers.
 */
SAMRS_API int samrs_qkv_linear_window_fwd(const void* x, const void* w, const void* bias, void* out, int64_t images,
                                          int h, int w_grid, int ws, int nh, int hd, int dtype, void* stream);

/*
 * LayerNorm over the last dimension (the blocks' norm1 / norm2, candle_nn::LayerNorm with eps 1e-6,
 * src/sam1/encoder.rs:100-102, 121, 127): out = (x - mean) / sqrt(var + eps) * weight + bias per row of c,
 * statistics in f32. x, out: [rows, c]; weight, bias: [c].
 */
SAMRS_API int samrs_layer_norm_fwd(const void* x, const void* weight, const void* bias, void* out, int64_t rows,
                                   int c, float eps, int dtype, void* stream);

/* Message describing the last error returned on the calling thread ("" if none). */
SAMRS_API const char* samrs_last_error(void);

/* SAMRS_ABI_VERSION of the loaded library. */
SAMRS_API int samrs_abi_version(void);

/*
 * Device status word. Kernels never trap: a bounded wait that runs out, or an index check that
 * fails, records a code here and the kernel returns early. samrs_device_status synchronises
 * `stream`, returns the word of the current device (0 = healthy) and clears it when `clear` != 0.
 * Codes: 1 = mbarrier/TMA wait timed out, 2 = MMA wait timed out, 3 = bad launch geometry.
 * While the word is nonzero every tensor-core kernel of the device returns at entry without writing
 * its output: the outputs of the call that reported and of every later call are undefined until the
 * word is cleared. Once samrs_device_status has read a nonzero word without clearing it, every other
 * entry point on that device returns SAMRS_ERR_DEVICE (no launch) until a call with `clear` != 0.
 * Callers poll it where they synchronise anyway (sam-rs: `Sam::sync`, src/model.rs:121-124).
 * No counterpart in the reference (its kernels cannot wait on anything).
 */
SAMRS_API int samrs_device_status(void* stream, int clear);

/*
 * Test hooks of the failure path: every bounded wait of the kernels gives up after `wait_limit_cycles`
 * SM clock cycles instead of ~1 s (0 restores the default), and CTA 0 of the global-layer kernel never
 * loads key tile `withhold_key_tile` (-1: none). With both set, that CTA's wait for the tile runs out, the
 * kernel records code 1 in the device status word and every CTA returns (nothing faults or hangs); a test
 * then sees the status, clears it, restores the hooks and checks the next call. Synchronous. Test
 * infrastructure with no counterpart in the reference.
 */
SAMRS_API int samrs_test_hooks(int64_t wait_limit_cycles, int withhold_key_tile);

/*
 * Number of bf16 global-layer CTAs (one head x 256 query rows) that were recomputed by the exact second
 * pass since the last clear (the single-pass bf16 kernel hands a CTA to it when a row's softmax weights
 * left the range it keeps them in). Synchronises `stream`; `clear` != 0 resets the count.
 * A diagnostic with no counterpart in the reference.
 */
SAMRS_API int samrs_recompute_count(void* stream, int64_t* count, int clear);

/*
 * The per-layer choice for bf16 global layers on the current device. A layer is keyed by the address of its
 * rel-pos table. The speculative pass plus the fixup launch is kept while the measured share of CTAs that
 * the fixup recomputes stays at or below 0.15. Above that, the layer runs the exact two-pass kernel alone
 * for its next 32 calls, and is then measured again. The speculative pass costs 0.87x the exact kernel, and
 * each recomputed CTA costs an exact CTA on top of it.
 * A measurement is read back without waiting: it takes effect from the first call after its own call has
 * completed on the device.
 * Writes the layer's last measured share (-1 if never measured) to `share`, and to `exact` whether its next
 * call launches the exact kernel. `reset` != 0 first forgets every layer's history, so each layer's next call
 * measures again. Does not synchronise (a measurement still in flight is simply not read yet).
 * No counterpart in the reference (its kernels have no speculative pass).
 */
SAMRS_API int samrs_global_policy(const void* table, double* share, int* exact, int reset);

/*
 * Self-test hook of the library's own exp2 polynomial (the FMA-pipe exponential the windowed kernel uses
 * for one key pair in eight): y_poly[i] = the polynomial at x[i], y_lib[i] = CUDA's exp2f(x[i]); device
 * f32 buffers of n elements. Test infrastructure; no counterpart in the reference.
 */
SAMRS_API int samrs_selftest_ex2(const void* x, void* y_poly, void* y_lib, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SAMRS_B200_H */
