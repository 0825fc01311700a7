/* dc_b200.h -- C ABI of the B200 (sm_100a) backend for demucs-cuda's htdemucs_6s hot path.
 *
 * Part 1 is the drop-in boundary: every function of the reference kernel interface
 * worker-cuda/src/backend.h (lines 23-144), same names, argument meaning, types and
 * layouts, so the reference's unchanged C model code (ops.c, tensor.c, weights.c, stft.c,
 * htdemucs.c, layers.c, transformer.c, apply.c) links against libdc_b200.so in place of
 * backend_cuda.cu + gemm.cu + norm.cu + attn.cu + fft.cu.  Each declaration cites the
 * reference line it replaces.  As in the reference, every pointer is device memory, every
 * call is asynchronous on the backend's stream, and an invalid call or CUDA failure is
 * fatal (message on stderr, exit(1)) unless the host selected DCB_ERRORS_RETURN with
 * dcb_set_error_mode(), in which case the call records the error for dcb_last_error().
 *
 * Part 2 (dkx_*) are added fused entry points the model layer uses instead of the
 * im2col/col2im/split-heads/softmax sequences (no counterpart function in backend.h; the
 * reference composes each from the Part-1 calls cited beside it).
 *
 * Part 3 (dcb_*) is the runtime and model engine: stream/error control, an htdemucs_6s
 * model loaded from the reference's safetensors + JSON files, its forward pass (the
 * equivalent of dc_htdemucs_forward, htdemucs.c:136-280) and the segment scheduler
 * (dc_apply_model, apply.c:179-306).
 */
#ifndef DC_B200_H
#define DC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== Part 1: backend.h */

/* GEMM operand element: IEEE fp16 bit pattern (backend.h:20). */
typedef uint16_t dc_half;
/* float -> fp16, round to nearest even (backend.h:23, backend_cuda.cu dk_pack_half). */
dc_half dk_pack_half(float v, int weight);

#define DK_MAX_DIM 8

/* runtime (backend.h:28-40) */
int dk_init(int device, char *name, size_t name_cap);             /* backend.h:28 */
const char *dk_backend_name(void);                                /* backend.h:29 */
void dk_sync(void);                                               /* backend.h:30 */
void *dk_raw_malloc(size_t bytes);                                /* backend.h:31, NULL on OOM */
void dk_raw_free(void *p);                                        /* backend.h:32 */
void dk_memcpy_h2d(void *dst, const void *src, size_t bytes);     /* backend.h:33 */
void dk_memcpy_d2h(void *dst, const void *src, size_t bytes);     /* backend.h:34 */
void dk_memcpy_d2d(void *dst, const void *src, size_t bytes);     /* backend.h:35 */
void dk_memset0(void *dst, size_t bytes);                         /* backend.h:36 */
int dk_mem_info(size_t *free_bytes, size_t *total_bytes);         /* backend.h:37 */
void dk_range_push(const char *name);                             /* backend.h:39 */
void dk_range_pop(void);                                          /* backend.h:40 */

/* strided elementwise (backend.h:43-70); same struct layout as backend.h:43-48 */
typedef struct {
  int ndim;
  int64_t shape[DK_MAX_DIM];
  int64_t a_strides[DK_MAX_DIM]; /* source strides for copy */
  int64_t b_strides[DK_MAX_DIM]; /* destination strides for copy */
} DkStrided;

/* dst[idx . b_strides] (+)= src[idx . a_strides] (backend.h:51) */
void dk_strided_copy(const DkStrided *p, const float *src, float *dst, int accumulate);
typedef enum { DK_ADD = 0, DK_SUB, DK_MUL, DK_DIV, DK_MAX } DkBinOp;   /* backend.h:53 */
/* y contiguous over shape, a/b through their strides (backend.h:55) */
void dk_binary(DkBinOp op, const DkStrided *p, const float *a, const float *b, float *y);
typedef enum { DK_UN_AFFINE = 0, DK_UN_GELU, DK_UN_RELU, DK_UN_SIGMOID } DkUnOp; /* backend.h:57 */
void dk_unary(DkUnOp op, const float *x, float *y, int64_t n, float alpha, float beta); /* :59 */
void dk_fill(float *y, int64_t n, float v);                                              /* :60 */
void dk_glu(const float *x, float *y, int64_t outer, int64_t half, int64_t inner);       /* :62 */
void dk_channel_bias(float *y, const float *bias, int64_t outer, int64_t C, int64_t inner); /* :64 */
void dk_scale_add(float *y, const float *x, const float *scale, int64_t outer, int64_t C,
                  int64_t inner);                                                        /* :66 */
void dk_reflect_pad(const float *x, float *y, int64_t rows, int64_t L, int64_t left,
                    int64_t right);                                                      /* :69 */

/* normalisation (backend.h:72-89) */
void dk_row_stats(const float *x, int64_t rows, int64_t L, float *mean, float *var);    /* :74 */
void dk_groupnorm_apply(const float *x, float *y, const float *mean, const float *var,
                        const float *w, const float *b, int64_t B, int64_t C, int64_t S,
                        int64_t G, float eps, int act);                                  /* :77 */
void dk_norm_apply_last(const float *x, float *y, const float *mean, const float *var,
                        const float *w, const float *b, int64_t rows, int64_t L, int64_t C,
                        float eps);                                                      /* :81 */
void dk_affine_rows(const float *x, float *y, const float *mean, const float *var,
                    int64_t rows, int64_t L, float eps, int denorm);                     /* :85 */
void dk_layernorm(const float *x, float *y, const float *w, const float *b, int64_t rows,
                  int64_t C, float eps);                                                 /* :88 */

/* GEMM operand preparation (backend.h:91-115) */
void dk_to_half_rows(const float *x, dc_half *y, int64_t rows, int64_t C, int64_t Cp);  /* :93 */
void dk_transpose_to_half(const float *x, dc_half *y, int64_t batch, int64_t C, int64_t P,
                          int64_t Cp);                                                   /* :95 */
typedef struct {          /* backend.h:98-106, same field order */
  int C, H, W;
  int KH, KW;
  int SH, SW;
  int PH, PW;
  int DH, DW;
  int Ho, Wo;
  int64_t Kp;
} DkConvGeom;
void dk_im2col_half(const float *x, dc_half *col, const DkConvGeom *g, int64_t n0, int64_t nb,
                    int64_t p0, int64_t np);                                             /* :110 */
void dk_col2im_tr(const float *cols, float *y, const float *bias, int64_t nb, int O,
                  const DkConvGeom *g);                                                  /* :114 */

/* C[b] = alpha A[b] B[b]^T + beta C[b]; A [M][lda], B [N][ldb] fp16, C [M][ldc] fp32;
 * K, lda, ldb multiples of 8; stride 0 = shared operand (backend.h:117-122).
 * tcgen05/TMEM tensor-core path for sm_100a; any legal call is accepted (unaligned or
 * odd-strided calls take a CUDA-core path of the same kernel family). */
void dk_gemm_half(int64_t M, int64_t N, int64_t K, float alpha, const dc_half *A, int64_t lda,
                  int64_t strideA, const dc_half *B, int64_t ldb, int64_t strideB, float beta,
                  float *C, int64_t ldc, int64_t strideC, int64_t batch);

/* attention helpers (backend.h:124-131) */
void dk_softmax_to_half(const float *s, int64_t lds, dc_half *p, int64_t ldp, int64_t rows,
                        int64_t L, float scale);                                         /* :127 */
void dk_split_heads_half(const float *x, dc_half *y, int64_t B, int64_t T, int H, int hd,
                         int hdp, int64_t Tp, int transpose);                            /* :130 */

/* spectral (backend.h:133-144) */
void dk_stft(const float *sig, float *out, int64_t R, int64_t L, int n_fft, int hop,
             int frame0, int nframes, int nbins, const float *window);                  /* :136 */
void dk_istft_frames(const float *spec, float *frames, int64_t R, int nbins, int nframes,
                     int pad_frames, int n_fft, const float *window);                   /* :140 */
void dk_ola(const float *frames, float *out, int64_t R, int nframes, int n_fft, int hop,
            const float *window, int64_t start, int64_t length);                        /* :143 */

/* Allocation-free variant of dk_row_stats.  No counterpart in the reference: it exists for
 * callers that cannot let the library allocate device memory -- a real-time audio thread
 * that must never block (cudaMalloc/cudaFree can synchronise the whole device) or a host
 * that gives all device memory to its own pool.  Same results as dk_row_stats; the chunk
 * partials live in a fixed 1 MiB device array that every GPU loading the library keeps
 * until exit, so rows * ceil(L / 8192) must not exceed 43690.  A larger call is an error
 * like any other: fatal in the default error mode (message, exit(1)); with
 * DCB_ERRORS_RETURN it is recorded for dcb_last_error() and the call returns -1 before any
 * launch.  Calls no cudaMalloc/cudaFree.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current and caches it; the cache
 * does not survive cudaDeviceReset.  All calls share the one array: calls that overlap on
 * the GPU (different streams, or different host threads) race and must be serialised by
 * the caller.  Returns 0, or -1 if this call recorded an error (an error left pending by
 * an earlier call does not make it fail). */
int dk_row_stats_noalloc(const float *x, int64_t rows, int64_t L, float *mean, float *var);

/* ======================================================== Part 2: fused entry points */

/* Activation applied in a GEMM epilogue. */
enum { DKX_ACT_NONE = 0, DKX_ACT_GELU = 1, DKX_ACT_GLU = 2 };

/* Implicit-GEMM convolution, the fused replacement of conv_core's
 * dk_im2col_half + dk_gemm_half + dk_channel_bias (ops.c:31-77) with an optional GELU
 * (layers.c:120) or channel GLU (layers.c:134, 174) applied before the store.
 * x [N][C][H][W] fp32, weight [O][kp] fp16 in the loader's layout (k = (kh*KW+kw)*C + c,
 * weights.c:298-311), bias [O] fp32 or NULL, y [N][Oy][Ho][Wo] fp32 with Oy = O, or O/2
 * for GLU.  No im2col buffer: the tensor-core kernel gathers the patch tile from x. */
void dkx_conv2d(const float *x, int N, const DkConvGeom *g, const dc_half *weight, int O,
                const float *bias, int act, float *y);

/* Transposed convolution along one axis with kernel 2*stride (HTDemucs decoders), the fused
 * replacement of conv_tr_core's dk_transpose_to_half + dk_gemm_half + dk_col2im_tr
 * (ops.c:143-177) plus the decoder crop (layers.c:201-211) and GELU (layers.c:212-216).
 * x [N][C][H][W]; weight in the loader's conv_tr layout [O*KH*KW][kp]; the stride axis is
 * H when KW == 1 (2-D, freq) or W when KH == 1 (1-D, time).  Output y [N][O][Ho][Wo] keeps
 * full-output rows/cols [crop, crop + out_len) of the stride axis. */
void dkx_conv_tr(const float *x, int N, int C, int H, int W, const dc_half *weight, int O,
                 int KH, int KW, int stride, const float *bias, int crop, int out_len,
                 int gelu, float *y);

/* y[R][out] = x[R][in] . W^T + bias (dc_linear, ops.c:234-257) with x given as fp32
 * (rounded to fp16 on load, as dk_to_half_rows does). */
void dkx_linear(const float *x, int64_t R, int in, const dc_half *weight, int64_t kp, int out,
                const float *bias, float *y);

/* softmax(q k^T / sqrt(hd)) v per head (dc_attention, ops.c:390-443) as one flash kernel:
 * q [B][Tq][H*hd], k/v [B][Tk][H*hd] fp32 -> y [B][Tq][H*hd] fp32; no score matrix in
 * memory. */
void dkx_attention(const float *q, const float *k, const float *v, int B, int Tq, int Tk,
                   int H, int hd, float *y);

/* ============================================================ Part 3: runtime / engine */

enum { DCB_ERRORS_FATAL = 0, DCB_ERRORS_RETURN = 1 };
/* Fatal (default, the reference's dc_die behaviour) or record-and-return. */
void dcb_set_error_mode(int mode);
/* Last recorded error message ("" if none); clears it when clear != 0. */
const char *dcb_last_error(int clear);
/* Use an external stream (a cudaStream_t, e.g. a framework's current stream) for every
 * later call; NULL selects the legacy default stream.  dcb_use_own_stream() returns to the
 * backend's own non-blocking stream (the default, as backend_cuda.cu:41 creates one). */
void dcb_set_stream(void *stream);
void dcb_use_own_stream(void);
void *dcb_get_stream(void);
/* Backend options: "simt" (1 = CUDA-core kernels instead of tcgen05, for A/B checks),
 * "graphs" (1 = replay captured CUDA graphs for repeated forwards), "generic_epilogue"
 * (1 = channels-last convs use their generic epilogue instead of the specialised ones, for
 * A/B checks), "stream_istft" (0 = the two-pass inverse STFT instead of the fused
 * streaming one, for A/B checks), "streams" (1, the default = the time branch's layers on
 * a second stream beside the frequency branch's, and consecutive dcb_apply batches on two
 * alternating streams; 0 = one stream), "dconv_rows" (1, the default = both DConv layers of
 * the first frequency level in one kernel, one CTA per row; 0 = the per-layer path),
 * "wait_limit_ms" (limit of every bounded device-side
 * wait, default 2000; tests shorten it), "test_withhold_arrive" (1 = the next tensor-core
 * GEMM CTA does not release its first operand stage, so a bounded wait expires and sets
 * the device fault word: the failure-detection test).  Returns the old value. */
int dcb_set_option(const char *name, int value);
/* Number of this library's kernels launched so far (monotonic). */
uint64_t dcb_kernel_launches(void);
/* Device-side fault word: bounded waits that expire set a bit here (0 = healthy). */
uint32_t dcb_device_fault(int clear);
/* Kernel-class trace: bit c of mask enables class c (0 implicit-GEMM conv, 1 stride-phase
 * transposed conv, 2 transformer linear, 3 flash attention, 4 dk_gemm_half, 5 STFT /
 * inverse STFT and their layout passes, 6 DConv GroupNorm statistics and CUDA-core tail,
 * 7 transformer LayerNorm / GroupNorm; 5-7 carry bytes only).  Every
 * launch of an enabled class is bracketed by CUDA events on the backend stream and tagged
 * with its algorithmic FLOPs and bytes; dcb_trace_stop synchronises and returns per-class
 * totals (milliseconds, FLOPs, bytes, launches) for classes < ncls. */
void dcb_trace_start(uint32_t mask);
int dcb_trace_stop(double *ms, double *flops, double *bytes, int *launches, int ncls);
/* After dcb_trace_stop: write every traced launch (class, ms, FLOPs, bytes, M, N, K) as CSV. */
int dcb_trace_dump(const char *path);

typedef struct DcbModel DcbModel;
/* Load weights (safetensors, F32/F16/BF16, MLX layout) + model JSON (defaults =
 * htdemucs_6s), pack every GEMM operand once on the device.  NULL on error. */
DcbModel *dcb_model_load(const char *safetensors_path, const char *config_json_path);
void dcb_model_free(DcbModel *m);
int dcb_model_info(const DcbModel *m, int *n_sources, int *audio_channels, int *valid_length,
                   int *samplerate, float *segment);
/* The same model's layout from the safetensors header alone (no tensor data is read): the
 * device block is allocated and zeroed for the caller to fill, e.g. by an NCCL broadcast of
 * another rank's dcb_model_weight_block.  NULL on error. */
DcbModel *dcb_model_load_layout(const char *safetensors_path, const char *config_json_path);
/* Pre-packed on-disk image of a loaded model: the config, the safetensors header and the
 * device block exactly as packed (fp16 GEMM operands with GLU-interleaved rows, the TMA K
 * order, transposed-conv phase matrices, fp64 DConv statistic constants), with a checksum.
 * dcb_model_load_packed rebuilds the layout from the stored header and uploads the block
 * as stored: no fp32 tensor data is read or converted.  0 / NULL on error. */
int dcb_model_save_packed(const DcbModel *m, const char *path);
DcbModel *dcb_model_load_packed(const char *path);
/* Device bytes of the packed weight block (the NCCL broadcast payload) and its pointer. */
size_t dcb_model_weight_bytes(const DcbModel *m);
void *dcb_model_weight_block(DcbModel *m);

/* Stage callback: name (test_compare.c keys), device pointer, ndim, shape. */
typedef void (*DcbStageFn)(const char *name, const float *data, int ndim, const int *shape,
                           void *user);
/* Forward of mix [B][C][T] (device) into stems [B][S][C][Tout] (device); returns Tout, or
 * -1 on error.  fn may be NULL. */
int dcb_forward(DcbModel *m, const float *mix, int B, int T, float *out, DcbStageFn fn,
                void *user);

/* Teacher-forced single stages (mirror test_compare.c:139-216), all device tensors:
 * encoder layer idx of the freq (branch 0) or time (branch 1) path, decoder layer idx, and
 * the cross transformer (in place on x and xt).  Shapes follow the reference tensors. */
int dcb_stage_encoder(DcbModel *m, int branch, int idx, const float *x, int B, int C, int H,
                      int W, float *y, int *out_shape);
int dcb_stage_decoder(DcbModel *m, int branch, int idx, const float *x, const float *skip,
                      int B, int C, int H, int W, int length, float *y, int *out_shape);
int dcb_stage_transformer(DcbModel *m, float *x, float *xt, int B, int C, int Fr, int T1,
                          int T2);

/* Segment scheduler (dc_apply_model, apply.c:179-306) over a whole track. */
typedef struct {
  int shifts;
  int split;
  float overlap;
  float transition_power;
  int batch_size;
  unsigned seed;
  int use_seed;
  /* segment subset for data-parallel sharding: this caller runs only block shard_index of
   * shard_count contiguous blocks of the segment forwards (all shift passes, in output
   * order) and accumulates their weighted stems; the weight sums cover every segment, so
   * summing the shard outputs over all shards gives the full result.  shard_count 0/1 =
   * everything. */
  int shard_index;
  int shard_count;
} DcbApplyOpts;
void dcb_apply_defaults(DcbApplyOpts *o);
/* mix [B][C][T] (device) -> out [B][S][C][T] (device). Returns 0 or -1.  With
 * shard_count > 1, out holds this shard's share (zero outside its window), so the shards'
 * outputs sum to the full result. */
int dcb_apply(DcbModel *m, const float *mix, int B, int T, float *out, const DcbApplyOpts *o);
/* dcb_apply on HOST buffers: mix_h [B][C][T] and out_h [B][S][C][T] in host memory (page-
 * locked memory lets the copies overlap the compute; pageable memory works, serialised).
 * Each segment batch's input span is copied in just before the batch, and each stretch of
 * the output that no later batch touches is copied back while the next batches compute,
 * on two copy streams (one per direction); returns when out_h holds the stems.  Whole track only (shard_count
 * <= 1); the device buffers are kept by the model and reused.  Returns 0 or -1. */
int dcb_apply_host(DcbModel *m, const float *mix_h, int B, int T, float *out_h,
                   const DcbApplyOpts *o);
/* Data-parallel form of dcb_apply.  The segments of all shift passes, ordered by output
 * position, are split into shard_count contiguous blocks; a shard's share of the output is
 * non-zero only on its window [lo, hi) along time (about 1 / shard_count of the track plus
 * the overlaps).  dcb_apply_window (host only) gives the window; dcb_apply_shard writes the
 * share over the window only: win [B*S*C rows][ld], column j = time lo + j for
 * j < hi - lo (ld >= hi - lo; later columns untouched).  dcb_merge_windows is the root's
 * overlap-add after gathering the n shards' windows (window i at wins + i * win_stride,
 * rows of stride ld): out [rows][T] = their sum, zero where no window covers (n <= 64). */
int dcb_apply_window(int samplerate, float segment, int valid_length, int T,
                     const DcbApplyOpts *o, int64_t *lo, int64_t *hi);
int dcb_apply_shard(DcbModel *m, const float *mix, int B, int T, float *win, int64_t ld,
                    const DcbApplyOpts *o);
int dcb_merge_windows(float *out, int64_t rows, int64_t T, const float *wins, int64_t ld,
                      int64_t win_stride, const int64_t *lo, const int64_t *hi, int n);
/* Host-only pieces of the scheduler (no GPU needed):
 * dcb_py_randint: n draws of CPython's random.Random(seed).randint(lo, hi), the shift
 *   generator of apply.c:5-107;
 * dcb_segment_plan: the segment offsets of a track (apply.c:223-237) and, per offset, the
 *   index of the forward call that runs it on this shard (full segments batched up to
 *   batch_size, tails alone; -1 = another shard's segment).  Returns the offset count (the
 *   arrays are filled only if it is <= cap). */
int dcb_py_randint(uint64_t seed, int lo, int hi, int n, int *out);
int dcb_segment_plan(int samplerate, float segment, int length, const DcbApplyOpts *o,
                     int *offsets, int *call_of, int cap);
/* Number of forward passes dcb_apply would run for a track of T samples. */
int dcb_apply_plan(DcbModel *m, int T, const DcbApplyOpts *o, int *n_forwards, int *n_batched);

#ifdef __cplusplus
}
#endif

#endif /* DC_B200_H */
