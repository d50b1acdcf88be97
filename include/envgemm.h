/* envgemm.h -- C ABI of libenvgemm.so, the B200 (sm_100a) dense-linear engine for Envision.
 *
 * Envision (hshatti/Invision) runs every Linear of its FLUX.2 / Z-Image transformers and Qwen3
 * encoder, and every im2col convolution of its VAE, through one CPU GEMM.  This library replaces
 * that path with hand-written tcgen05/TMA kernels.  The Pascal host binds it at run time with
 * LoadLibrary/GetProcAddress (the reference's rule for optional libraries, README.md:102-104, and
 * the OpenBLAS binding block in src/quicknncpu.pas:3951-3996); every entry point therefore uses
 * plain C types, the cdecl convention (= Pascal `winapi` on x86-64 Linux) and returns a status.
 *
 * Conventions shared by every entry point (paths below are Envision source files):
 *   - Row-major throughout.  X fp32 [M, K]; W bf16 [N, K] (PyTorch Linear / safetensors order);
 *     Y fp32 [M, N].  alpha = 1 and beta = 0 for linears; Y is overwritten, never accumulated
 *     (quicknncpu.pas:1807-1828), except ENVG_EPI_GATED_RESIDUAL which reads Y as the residual.
 *   - The activation X is rounded fp32 -> bf16 with round-to-nearest-even on the device and
 *     multiplied with fp32 accumulation.  (The reference widens W to fp32 and runs an fp32 GEMM,
 *     quicknncpu.pas:1830-1847; the difference is bounded by the tests at max|d|/max|ref| <= 1e-2
 *     and sum|d|/sum|ref| <= 2e-3.)  An fp32 weight that is not made of bf16 numbers, and both
 *     operands of envg_sgemm, are split into bf16 hi/lo parts instead (bf16x3, see
 *     envg_weight_upload), which matches the fp32 GEMM to about 1e-5.
 *   - M == 0 is a no-op returning ENVG_OK.  dst must not alias x.
 *   - Errors never throw: a negative ENVG_ERR_* code is returned and envg_last_error() gives a
 *     thread-local message.  The Pascal shim turns a non-zero code into assert(false, msg), which
 *     is how the reference reports bad arguments (e.g. quicknn_kernels.pas:484-486).
 *   - Calls made from one host thread are serialised on the library's stream for the current
 *     device.  Host-pointer calls are synchronous (the Pascal caller reads dst right after the
 *     call); ENVG_DEVICE_PTRS calls are stream-ordered and return before completion when
 *     ENVG_ASYNC is also set (envg_sync() waits).
 */
#ifndef ENVGEMM_H
#define ENVGEMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------------------------- */
#define ENVG_OK 0
#define ENVG_ERR_ARG (-1)         /* bad shape, null pointer, unsupported combination          */
#define ENVG_ERR_OOM (-2)         /* device or pinned-host allocation failed                    */
#define ENVG_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed                          */
#define ENVG_ERR_NCCL (-4)        /* reserved for the multi-GPU gather                           */
#define ENVG_ERR_TIMEOUT (-5)     /* a bounded device-side wait gave up (see ENVG_WAIT_CAP)     */
#define ENVG_ERR_STATE (-6)       /* library not initialised / handle freed / wrong device      */
#define ENVG_ERR_UNSUPPORTED (-7) /* valid request this build does not implement                */

/* ---- weight layouts (envg_weight_upload.layout_flags) -------------------------------------- */
#define ENVG_LAYOUT_PLAIN 0   /* W [N, K]                                                     */
#define ENVG_LAYOUT_GATE_UP 1 /* W [N, K], rows [0, N/2) = gate, [N/2, N) = up (the fused     */
                              /* FLUX linear_in / Qwen3 gate+up tensor, quicknn_transformers.pas */
                              /* :595-597); re-laid out once at upload for ENVG_EPI_SILU_GATE   */
#define ENVG_LAYOUT_ROUND_BF16 4 /* OR-ed in: round an fp32 / fp16 weight to bf16 (RNE) even when */
                                 /* its values are not all bf16 numbers (see envg_weight_upload)  */

/* ---- epilogues (envg_linear.epilogue, envg_conv2d.epilogue) -------------------------------- */
#define ENVG_EPI_NONE 0           /* Y = X.W^T (+ bias if bias != NULL)                         */
#define ENVG_EPI_BIAS 1           /* Y = X.W^T + bias           (QNNLinear, quicknncpu.pas:1807) */
#define ENVG_EPI_SILU_GATE 2      /* Y[:, j] = silu(g_j) * u_j, g/u the gate/up halves          */
                                  /*   (QNNSiluMul, quicknncpu.pas:2404-2419); Y is [M, N/2]      */
#define ENVG_EPI_GATED_RESIDUAL 3 /* Y = Y + gate (.) (X.W^T + bias)  (QNNGatedAdd, :853-859)     */
#define ENVG_EPI_SILU 4           /* conv only: Y = silu(conv + bias)                            */

/* ---- call flags ----------------------------------------------------------------------------- */
#define ENVG_HOST_PTRS 0    /* x, dst, bias, gate are host pointers (pinned or pageable)       */
#define ENVG_DEVICE_PTRS 1  /* x, dst, bias, gate are device pointers on the current device   */
#define ENVG_ASYNC 2        /* with ENVG_DEVICE_PTRS: do not wait for completion               */
#define ENVG_KEEP_SHARDED 4 /* envg_linear_nsplit(_batch): the shard's columns stay on this     */
                            /* rank (y_local only; no transfer), for column-local consumers     */

/* Opaque device-resident weight (bf16 in HBM, laid out for the kernels). */
typedef struct envg_weight_s* envg_weight;

typedef struct envg_stats {
  uint64_t calls;            /* linear + conv + sgemm calls since init                     */
  uint64_t kernel_launches;  /* kernels launched by the library                            */
  double flops;              /* 2*M*N*K summed over calls                                  */
  double h2d_bytes;          /* host->device bytes copied by host-pointer calls            */
  double d2h_bytes;          /* device->host bytes                                         */
  uint64_t weight_bytes;     /* device bytes held by live weight handles                   */
  uint64_t workspace_bytes;  /* device scratch currently held by the library               */
  int32_t device;            /* current CUDA device                                        */
  int32_t last_status;       /* last non-zero status (0 if none)                           */
} envg_stats;

/* Select the device used by this host thread and create its stream and workspace.
 * ndev must be 1 in this build (one process per GPU; multi-GPU runs shard W across processes,
 * see envg_weight_upload_shard).  dev_ids may be NULL (device 0).  Replaces the library
 * detection in quicknncpu.pas:3951-3996 (`isUsingBlas`).  Fails with ENVG_ERR_CUDA when no
 * sm_100 device is present, so the caller keeps its CPU path. */
int envg_init(int ndev, const int* dev_ids);

/* Release the workspace and stream of the current device.  Weight handles must be freed first. */
int envg_shutdown(void);

/* Upload a weight once into HBM (replaces the per-call widening of QNNLinearNoBias_BF16,
 * quicknncpu.pas:1830-1847, and the per-step mmap re-reads of quicknn_transformers.pas:1581-1602).
 * Exactly one of w_bf16 (raw bf16 bits, the safetensors dtype BF16) or w_f32 is non-NULL; both
 * are host pointers to W[N, K] row-major.  After return the host memory may be unmapped
 * (safetensor.pas mmap views).
 * An fp32 weight whose values are all bf16 numbers (a widened bf16 checkpoint, the reference's
 * usual case, safetensor.pas:584-647) is stored as bf16, exactly.  Any other fp32 weight keeps
 * its precision as a bf16x3 split: each value v becomes hi = bf16_rn(v) and lo = bf16_rn(v - hi),
 * and the linear multiplies x_hi w_hi + x_hi w_lo + x_lo w_hi on the tensor cores, which matches
 * the reference's fp32 GEMM (QNNLinearNoBias, quicknncpu.pas:1822-1828) to about 1e-5 relative.
 * Such a weight holds 6 bytes per value and costs three times the tensor-core work; with
 * ENVG_LAYOUT_ROUND_BF16 in layout_flags it is rounded to bf16 (RNE) instead, like activations. */
int envg_weight_upload(const uint16_t* w_bf16, const float* w_f32, int64_t N, int64_t K,
                       int layout_flags, envg_weight* out);

/* Upload only the output-column shard [n0, n1) of W[N, K] (the N-split used when several
 * processes share one linear, one GPU each).  For ENVG_LAYOUT_GATE_UP the shard is taken in
 * gate/up pairs: rows [n0, n1) of the gate half and the same rows of the up half, so the SiLU
 * gate stays shard-local.  The handle then behaves like a W of n1 - n0 (x2 for GATE_UP) rows. */
int envg_weight_upload_shard(const uint16_t* w_bf16, const float* w_f32, int64_t N, int64_t K,
                             int64_t n0, int64_t n1, int layout_flags, envg_weight* out);

/* Upload a convolution weight W[out_ch, in_ch, kH, kW] (the layout QNNConv2d reads,
 * quicknncpu.pas:1958-2132) for envg_conv2d.  w_f32 is rounded to bf16 (RNE). */
int envg_conv_weight_upload(const uint16_t* w_bf16, const float* w_f32, int out_ch, int in_ch,
                            int kH, int kW, envg_weight* out);

int envg_weight_free(envg_weight w);

/* ---- weights straight from a .safetensors file ---------------------------------------------
 * Replace TSafeTensorFile.open (safetensor.pas:466-513) + getTensorDataMemBlock /
 * getTensorDataMemBlockBF16 (safetensor.pas:584-683), which map the file and then widen each
 * BF16/F16 weight to fp32 on the host for every linear.  Here the tensor's bytes are read from
 * the mapped file and go to HBM once, as bf16. */
#define ENVG_DTYPE_OTHER 0 /* any safetensors dtype other than the three below                   */
#define ENVG_DTYPE_BF16 1
#define ENVG_DTYPE_F16 2
#define ENVG_DTYPE_F32 3

typedef struct envg_tensor_info {
  int dtype;          /* ENVG_DTYPE_*                                                          */
  int ndim;           /* number of dimensions (<= 8)                                           */
  int64_t shape[8];   /* row-major shape; unused entries 0                                      */
  int64_t offset;     /* absolute byte offset of the tensor's data in the file                 */
  int64_t nbytes;     /* data_offsets[1] - data_offsets[0]                                      */
  char dtype_name[16];/* the dtype string as written in the header ("BF16", "F8_E4M3", ...)    */
} envg_tensor_info;

/* Header query; reads only the file's header and needs no GPU or envg_init.  Mirrors
 * TSafeTensorFile.find (safetensor.pas:525-531): ENVG_ERR_ARG when the tensor is absent or the
 * header is malformed (message in envg_last_error). */
int envg_safetensors_tensor_info(const char* path, const char* name, envg_tensor_info* out);

/* Reads tensor `name` widened to fp32 into host memory dst[count] (count = the element count).
 * BF16 -> fp32 is `bits << 16` (BF16ToSingle, quicknn_common.pas:1991-2008); F16 -> fp32 is the
 * exact IEEE widening (FP16ToSingle); F32 is copied.  For biases, norms and modulation vectors,
 * which stay on the host side of the boundary.  Needs no GPU. */
int envg_safetensors_read_f32(const char* path, const char* name, float* dst, int64_t count);

/* Uploads tensor `name` as a device weight.  2-D tensors [N, K] become a linear weight with
 * `layout_flags` (shard rows [n0, n1) as envg_weight_upload_shard; n0 = n1 = 0 means all rows);
 * 4-D tensors [out_ch, in_ch, kH, kW] become a convolution weight (n0 = n1 = 0 required).
 * BF16 bits are kept; F16 and F32 are stored as envg_weight_upload stores an fp32 weight (bf16
 * when every value is a bf16 number, else bf16x3 hi/lo parts, or RNE bf16 with
 * ENVG_LAYOUT_ROUND_BF16); convolution weights are rounded to bf16 (RNE). */
int envg_weight_upload_safetensors(const char* path, const char* name, int layout_flags, int64_t n0,
                                   int64_t n1, envg_weight* out);

/* Y = epilogue(X . W^T).  Mirrors QNNLinear(dst, x, W, B, seqLen, inDIM, outDIM)
 * (quicknn_kernels.pas:897-911 -> quicknncpu.pas:1807-1820) with M = seqLen, K = inDIM,
 * N = outDIM, and QNNLINEAR_BF16_OR_F32 / QNNLinearNoBias (quicknn_kernels.pas:2093-2103,
 * :913-927) with bias = NULL.  N is the number of W rows held by the handle; for
 * ENVG_EPI_SILU_GATE dst has N/2 columns.  bias: fp32 [N] or NULL.  gate: fp32 [N] for
 * ENVG_EPI_GATED_RESIDUAL, else NULL. */
int envg_linear(float* dst, const float* x, envg_weight W, const float* bias, int64_t M,
                int64_t K, int64_t N, int epilogue, const float* gate, int flags);

/* One linear of a batch (arguments as envg_linear). */
typedef struct envg_linear_desc {
  float* dst;
  const float* x;
  envg_weight W;
  const float* bias;
  int64_t M, K, N;
  int epilogue;
  const float* gate;
} envg_linear_desc;

/* Several linears in one call, in order.  Equivalent to n envg_linear calls.
 * ENVG_DEVICE_PTRS (ENVG_ASYNC optional): each distinct input x is rounded to bf16 once (the FLUX
 * Q/K/V and Qwen3 q/k/v projections read the same normalised input,
 * quicknn_transformers.pas:1402-1414, quicknn_qwen3.pas:712-714), and the rounding of the next
 * input runs on a second stream while the current GEMM runs.  An input that is the output of an
 * earlier linear of the batch waits for it.
 * ENVG_HOST_PTRS (synchronous): every linear is computed as envg_linear computes it from host
 * pointers, but the linears' copies in and out and their GEMMs overlap one another, so the call
 * costs about the larger of its total host->device and device->host bytes over PCIe rather than
 * the sum of each linear's.  A linear whose output overlaps another's output, or an input of a
 * later one, makes the call run them one after another. */
int envg_linear_batch(const envg_linear_desc* descs, int n, int flags);

/* One rank's part of an N-split linear, with the all-gather fused into the GEMM epilogue.  The
 * weight handle holds this rank's output-column shard (envg_weight_upload_shard); its outputs go
 * to columns [col0, col0 + shard width) of Y (row stride ldy) on EVERY rank:
 *   y_multicast != NULL: one multimem store per value to an NVLink multicast address (NVSwitch
 *                        NVLS) bound to all ranks' copies of Y;
 *   otherwise:           peer stores to each of y_peers[0 .. npeers) (every rank's copy of Y
 *                        mapped into this process, this rank's included; npeers <= 8).
 * y_local is this rank's copy (read for ENVG_EPI_GATED_RESIDUAL).  The transfer overlaps the
 * remaining tiles, replacing the separate all-gather + reorder of the N-split.  Device pointers
 * only; the caller synchronises the ranks (e.g. a symmetric-memory barrier) before Y is read.
 * With ENVG_KEEP_SHARDED in flags (or npeers == 0 and y_multicast == NULL) the shard's columns
 * are written to y_local only: the output stays column-sharded across the ranks, for a consumer
 * that reads only its own columns (per-head attention after head-aligned Q/K/V shards, the
 * per-pair SiLU gate after gate/up shards; quicknn_transformers.pas:1402-1405 -> :1174-1183).
 * New with this library (the reference runs on one CPU). */
int envg_linear_nsplit(float* y_local, float* const* y_peers, int npeers, float* y_multicast, int64_t ldy,
                       int64_t col0, const float* x, envg_weight W, const float* bias, int64_t M,
                       int64_t K, int64_t N, int epilogue, const float* gate, int flags);

/* Several N-split shards in one call, as envg_linear_batch runs several linears: each distinct
 * input is rounded to bf16 once, on a second stream, overlapped with the previous GEMM.  Each
 * descriptor is envg_linear_nsplit's arguments: lin.dst = this rank's copy of Y (row stride ldy),
 * lin.N = the shard's rows of W.  A descriptor with npeers == 0 and y_multicast == NULL (or every
 * descriptor, with ENVG_KEEP_SHARDED in flags) keeps its shard on this rank.  A linear that reads
 * another's gathered Y belongs in a later call, after the ranks' barrier. */
typedef struct envg_nsplit_desc {
  envg_linear_desc lin;
  float* const* y_peers;  /* every rank's copy of Y (this rank's included), or NULL */
  int npeers;
  float* y_multicast;     /* NVLS multicast address of Y, or NULL */
  int64_t ldy;
  int64_t col0;           /* first column of this shard in Y */
} envg_nsplit_desc;

int envg_linear_nsplit_batch(const envg_nsplit_desc* descs, int n, int flags);

/* dst[batch, out_ch, outH, outW] = conv(src[batch, in_ch, H, W], W) + bias, NCHW, as
 * QNNConv2d (quicknn_kernels.pas:984-1010 -> quicknncpu.pas:1958-2132); outH/outW follow
 * QNNConv2DShape (quicknn_kernels.pas:984-988).  epilogue: ENVG_EPI_NONE/BIAS or ENVG_EPI_SILU. */
int envg_conv2d(float* dst, const float* src, envg_weight W, const float* bias, int in_ch,
                int out_ch, int H, int W_, int kH, int kW, int stride, int pad, int batch,
                int epilogue, int flags);

/* dst = GroupNorm(src) (then SiLU when act_silu != 0), NCHW fp32 [batch, channels, H, W]; as
 * QNNGroupNorm (quicknncpu.pas:2259-2313: population variance, eps 1e-6, per-channel gamma /
 * beta) followed by QNNSiluInplace (:2372-2386).  gamma/beta may be NULL (1 / 0).  channels %
 * num_groups == 0.  dst may equal src.  gamma/beta follow the flags' pointer kind. */
int envg_group_norm(float* dst, const float* src, const float* gamma, const float* beta, int batch,
                    int channels, int H, int W, int num_groups, int act_silu, int flags);

/* One VAE ResBlock (TVAEResBlock.forward, quicknn_vae.pas:164-187):
 *   dst = skip(src) + conv2(SiLU(GN2(conv1(SiLU(GN1(src)))))),
 * skip = identity when skip == NULL (in_ch == out_ch), else the 1x1 conv `skip` + skip_bias.
 * Each GroupNorm + SiLU is folded into the NCHW -> NHWC bf16 cast that feeds the next 3x3 conv,
 * and the final add is the second conv's store (a TMA reduce-add into dst).  Vectors are host
 * pointers with ENVG_HOST_PTRS and device pointers with ENVG_DEVICE_PTRS, like src and dst. */
typedef struct envg_resblock {
  int in_ch, out_ch;
  const float* norm1_gamma;  /* [in_ch]  */
  const float* norm1_beta;   /* [in_ch]  */
  envg_weight conv1;         /* 3x3, in_ch -> out_ch, padding 1 */
  const float* conv1_bias;   /* [out_ch] */
  const float* norm2_gamma;  /* [out_ch] */
  const float* norm2_beta;   /* [out_ch] */
  envg_weight conv2;         /* 3x3, out_ch -> out_ch, padding 1 */
  const float* conv2_bias;   /* [out_ch] */
  envg_weight skip;          /* 1x1, in_ch -> out_ch, or NULL when in_ch == out_ch */
  const float* skip_bias;    /* [out_ch] or NULL */
} envg_resblock;

int envg_vae_resblock(float* dst, const float* src, const envg_resblock* rb, int batch, int H,
                      int W, int num_groups, int flags);

/* Multi-head attention, per head h (kv head h / (heads / kv_heads)):
 *   dst[:, h*hd : (h+1)*hd] = softmax(scale * Q_h K_kv^T + mask) V_kv
 * Q [seq_q, ldq], K and V [seq_k, ldk / ldv], dst [seq_q, ldo] fp32 row-major, head h at column
 * h * head_dim (the reference's [seq, hidden] layout).  Replaces the per-head cblas_gemm +
 * QNNSoftmaxRows + cblas_gemm of TTransformerFlux.multiHeadForward / jointAttentionForward
 * (quicknn_transformers.pas:1150-1270) and of the Qwen3 attention (quicknn_qwen3.pas:726-768,
 * GQA), and QNNFlashAttention(dst, Q, K, V, heads, seq_q, seq_k, head_dim, scale)
 * (quicknncpu.pas:2763-2860).  causal != 0 hides key c from query r when c > r + (seq_k -
 * seq_q) (QNNMatTriangularFill for seq_q == seq_k); key_mask (int32 [seq_k], may be NULL) hides
 * keys whose entry is 0.  Q, K and V are rounded to bf16 (RNE); both matrix products accumulate
 * in fp32; softmax is fp32.  head_dim must be 128 in this build. */
int envg_attention(float* dst, const float* Q, const float* K, const float* V, int seq_q, int seq_k,
                   int heads, int kv_heads, int head_dim, int64_t ldq, int64_t ldk, int64_t ldv,
                   int64_t ldo, float scale, int causal, const int32_t* key_mask, int flags);

/* The modulated linear of the FLUX blocks: QNNAdaLN (quicknn_kernels.pas:315 ->
 * quicknncpu.pas:3042-3060; call sites quicknn_transformers.pas:1400,1410,1440,1449,1500) followed
 * by QNNLinear, with the normalisation fused into the activation cast:
 *   xn[r][k] = (1 + scale[k]) * (x[r][k] - mean_r) / sqrt(var_r + 1e-6) + shift[k]
 *   dst = epilogue(xn . W^T)
 * mean_r / var_r are the row mean and population variance (QNNMean :679, QNNVariance :687); 1e-6
 * is EPSILON (quicknn_common.pas:51), which QNNAdaLN's body uses.  shift, scale: fp32 [K]; other
 * arguments and flags as envg_linear. */
int envg_linear_adaln(float* dst, const float* x, const float* shift, const float* scale, envg_weight W,
                      const float* bias, int64_t M, int64_t K, int64_t N, int epilogue, const float* gate,
                      int flags);

/* The normalised linear of the Qwen3 layer: QNNRMSNormRows (quicknncpu.pas:2159-2198; call sites
 * quicknn_qwen3.pas:802 input_layernorm and :817 post_attention_layernorm, whose outputs feed the
 * q/k/v and gate/up projections) followed by QNNLinear, with the normalisation fused into the
 * activation cast:
 *   xn[r][k] = x[r][k] * weight[k] / sqrt(sum_k x[r][k]^2 / K + 1e-6)   (weight NULL: x * inv)
 *   dst = epilogue(xn . W^T)
 * 1e-6 is EPSILON (quicknn_common.pas:51).  weight: fp32 [K] or NULL; other arguments and flags as
 * envg_linear. */
int envg_linear_rmsnorm(float* dst, const float* x, const float* weight, envg_weight W, const float* bias,
                        int64_t M, int64_t K, int64_t N, int epilogue, const float* gate, int flags);

/* Allocation-free linear for skinny M.  This entry point has no counterpart in the reference.
 *
 * envg_linear grows a device workspace on demand (cudaMalloc, and cudaFree of the smaller
 * buffer, which waits for all work on the device).  Some callers cannot allow that: a host
 * application whose own allocator has reserved the device memory and forbids other libraries to
 * allocate, or a caller that shares the GPU with streams it must not stall mid-step.  This
 * variant allocates nothing.  Its scratch (the bf16 copy of x, the split-K partial sums and
 * their counters) is one file-scope __device__ array of ENVG_NOALLOC_SCRATCH_BYTES (4 MiB), which
 * every GPU that loads the library holds until the process exits.
 *
 *  - Same arguments and epilogues as envg_linear, but x, dst, bias and gate must be device
 *    pointers: flags must contain ENVG_DEVICE_PTRS (ENVG_ASYNC optional).
 *  - Limits: 0 <= M <= 64 (M = 0 is a no-op) and M * Kp * 2 <= 2 MiB (Kp = K rounded up to 8,
 *    times 3 for a bf16x3 weight), i.e. K <= 16384 at M = 64; larger requests return
 *    ENVG_ERR_ARG with the limit in envg_last_error().  dst must not alias x.
 *  - envg_init prepares everything this entry point uses: it loads the code of every kernel it
 *    launches (which, with lazy module loading, would otherwise happen at the first launch and
 *    can map device memory), reserves their local memory, and looks up the array's device
 *    address (cudaGetSymbolAddress).  So the first call allocates no more than later ones.
 *  - Every call shares the one array, which keeps the last call's contents; the counters are
 *    cleared on every call.  Calls whose kernels overlap on the GPU (different streams without
 *    ordering) race on the array and must be serialised by the caller. */
#define ENVG_NOALLOC_SCRATCH_BYTES (4u << 20)
int envg_linear_noalloc(float* dst, const float* x, envg_weight W, const float* bias, int64_t M,
                        int64_t K, int64_t N, int epilogue, const float* gate, int flags);

/* cblas_sgemm-compatible fp32 GEMM on host pointers: the signature of the function-pointer
 * slot TQNNSingleOPS.cblas_sgemm (quicknncpu.pas:102-109; enums quicknn_common.pas:54-58:
 * RowMajor = 101, NoTrans = 111, Trans = 112).  Re-pointing that slot to this entry moves
 * every cblas_gemm call (attention products included) to the GPU without model edits.  Both
 * fp32 operands are split into bf16x3 parts on the device (see envg_weight_upload), so the
 * tensor-core product matches an fp32 GEMM to about 1e-5 relative; C = alpha*A.op(B) + beta*C.
 * RowMajor, NN/NT/TN only (as qgemm, quicknncpu.pas:1476). */
int envg_sgemm(int order, int transA, int transB, int64_t M, int64_t N, int64_t K, float alpha,
               const float* A, int64_t lda, const float* B, int64_t ldb, float beta, float* C,
               int64_t ldc);

/* Make the library launch on a caller-owned stream (a cudaStream_t passed as void*), or back on
 * its own non-blocking stream with NULL.  The legacy default stream is cudaStreamLegacy
 * ((void*)1), not NULL.  Lets a PyTorch or CUDA-graph caller order the kernels itself. */
int envg_set_stream(void* stream);

/* Wait for all work queued by this thread's calls. */
int envg_sync(void);

/* Thread-local text of the last error ("" if none). */
const char* envg_last_error(void);

int envg_get_stats(envg_stats* out);

/* Bound (nanoseconds) for every device-side spin wait; 0 restores the default (2 s, or the
 * ENVG_WAIT_CAP environment variable in ms).  A wait that runs out makes the call return
 * ENVG_ERR_TIMEOUT instead of hanging the GPU. */
int envg_set_wait_cap_ns(uint64_t ns);

/* Self-test of the bounded-wait path: launches one CTA that waits on an mbarrier nothing
 * arrives at, with cap_ns as the bound.  Returns ENVG_ERR_TIMEOUT when the bound works.  Used
 * by the fault-handling tests; faults nothing. */
int envg_selftest_wait_timeout(uint64_t cap_ns);

/* Per-kernel timing, measured with CUDA events recorded around each launch on the stream the
 * kernel runs on (used by the benchmark for the roofline figures; off by default). */
typedef struct envg_kernel_stat {
  char name[32];      /* kernel family, e.g. "k1_gemm", "k2_skinny", "k_cast_rows"           */
  uint64_t launches;
  double ms;          /* summed device time of those launches                                 */
  double flops;       /* algorithmic 2*M*N*K summed over the launches                         */
  double bytes;       /* algorithmic HBM bytes summed over the launches (operands read once,  */
                      /* outputs written once)                                                */
} envg_kernel_stat;

/* enable = 1: reset the counters and start recording; 0: stop recording. */
int envg_profile(int enable);

/* Synchronise, resolve pending events and copy up to max records; *count = records written. */
int envg_profile_read(envg_kernel_stat* out, int max, int* count);

/* Build/version string, e.g. "envgemm 0.1 sm_100a". */
const char* envg_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ENVGEMM_H */
