/*
 * spk.h - C ABI of libspk.so, the B200 (sm_100a) kernels for the spiking
 * hot path of flofiz/SpikingTransformer.
 *
 * Conventions (all entry points):
 *   - Every pointer is a device pointer unless stated otherwise; the library
 *     allocates nothing.  Buffers are owned by the caller.
 *   - Tensors are dense, row-major, in the reference's t-major fold: a tensor
 *     "[T][R][F]" holds timestep t of row r, feature f at ((t*R)+r)*F+f.
 *   - Neuron scalars (beta, v_th, v_reset, k, scale) are DEVICE pointers to
 *     one fp32 value, as in the reference kernels (Lif.py:121-123,145-147), so
 *     learnable values need no host synchronisation.
 *   - `stream` is a cudaStream_t; work is enqueued there, nothing synchronises.
 *   - Return value: 0 on success, otherwise an SPK_ERR_* code; the message of
 *     the last failure on the calling thread is spk_last_error().
 *
 * Reference interfaces replaced (file:line in flofiz/SpikingTransformer):
 *   spk_lif_fwd            lif_forward_kernel launch in LIFLayer.forward,
 *                          Triton_Layers/Lif.py:17-43 (kernel Lif.py:118-165)
 *   spk_lif_bwd            lif_backward_kernel launch + grad_beta sum in
 *                          LIFLayer.backward, Lif.py:46-102 (kernel Lif.py:181-282)
 *   spk_linear_ln_lif_fwd  nn.Linear -> nn.LayerNorm -> LIF triples:
 *                          SSA.py:218-228 (q/k/v), SSA.py:247-249 (out_proj),
 *                          SpikingMLP.py:31-36 (expand, compress), plus the
 *                          residual adds Encoder.py:19,22 / Decoder.py:18-25
 *   spk_linear_fwd         Seq2Seq.py:117 output_layer (nn.Linear)
 *   spk_linear_dgrad,      input and weight gradients of the Linear layers
 *   spk_linear_wgrad       (autograd of nn.Linear at SSA.py:218-249,
 *                          SpikingMLP.py:31-36 in train_spikeformer.py:545-561)
 *   spk_ssa_fwd            attention core of SSAMultiHeadAttention.forward,
 *                          SSA.py:230-245 (xnor_attention :145-165, log-PE
 *                          :177-201, mask, scale, @V, lifs) and of
 *                          SSAMultiHeadAttention_.forward SSA.py:77-87
 *   spk_ssa_fwd_heads      the same without a mask, on head-split operands
 *                          (the layout of SSA.py:226-228 after split_heads);
 *                          the training forward of the unmasked core
 *   spk_embed_pe_lif_fwd   TokenEmbedding + PositionalEncoding + lifPE,
 *                          Seq2Seq.py:11-36, :109-114
 *   spk_linear_affine_lif_fwd  conv (as a GEMM) -> eval BatchNorm -> LIF of
 *                          CNNBackbone, ImageEncoder.py:8-102
 *   spk_im2col             the convolutions' patch gather (PixelUnshuffle +
 *                          Conv2d, Conv1d), ImageEncoder.py:8-102
 *   spk_patch_im2col       patch gather of the 16x16 patch-embedding image
 *                          encoder (no reference counterpart; the OCR
 *                          benchmark's ImageEncoder)
 *   spk_synth_text_lines   on-device synthetic text-line batch (stands in for
 *                          the rendered lines of wiki_text_images3.py:173-236
 *                          and the DataLoader of train_spikeformer.py)
 *   spk_attn_masked_train_fwd / _bwd
 *                          the decoder's masked self-attention core in
 *                          training, SSA.py:234-242 and its autograd
 *   spk_ce_over_t          the training loss and token accuracy,
 *                          train_spikeformer.py:309-323 (step_loss with
 *                          CrossEntropyLoss(ignore_index, label_smoothing),
 *                          :269) and :84-93 (compute_token_accuracy of the
 *                          T-averaged logits, :556-559)
 */
#ifndef SPK_H_
#define SPK_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SPK_OK 0
#define SPK_ERR_INVALID 1     /* bad argument (null pointer, bad enum)       */
#define SPK_ERR_SHAPE 2       /* unsupported or inconsistent sizes            */
#define SPK_ERR_ALIGN 3       /* pointer alignment requirement not met        */
#define SPK_ERR_LAUNCH 4      /* kernel launch failed                          */
#define SPK_ERR_TIMEOUT 5     /* a device-side wait gave up (bounded spin)    */
#define SPK_ERR_UNSUPPORTED 6 /* device is not sm_100 / feature unavailable   */
#define SPK_ERR_CUDA 7        /* other CUDA runtime error                      */

/* element type codes */
#define SPK_F32 0
#define SPK_F16 1
#define SPK_BF16 2
#define SPK_U8 3
#define SPK_FP8 4 /* fp8 e4m3 (spikes only: 1.0 = 0x38, 0.0 = 0x00)          */
#define SPK_BIT 5 /* packed bits (spikes only): a [T][N] spike tensor is     */
                  /* T rows of ceil(N/8) bytes, neuron n at bit n%8 of byte  */
                  /* n/8; bits past N in a row's last byte are 0            */

/* LIF surrogate gradients */
#define SPK_SURROGATE_SUPERSPIKE 0 /* 1/(1+k|v-th|)^2, Lif.py:280-282        */
#define SPK_SURROGATE_ARCTAN 1     /* (a/2)/(1+(pi/2*a*(v-th))^2)            */

int spk_version(void);
const char* spk_status_string(int status);
const char* spk_last_error(void);
/* Reads (synchronising `stream`) and clears the device-side error flags set
 * by bounded waits in the tensor-core kernels; SPK_ERR_TIMEOUT if any was set. */
int spk_device_error_check(void* stream);
/* Self-test of the bounded device-side waits (no counterpart in the
 * reference): one block waits on an mbarrier that nothing arrives at, through
 * the wait loop the tensor-core kernels use but with a limit of limit_ns
 * (at most 1 s) instead of 2 s; the wait gives up, sets the device error flag
 * and the kernel returns, so the next spk_device_error_check reports
 * SPK_ERR_TIMEOUT (and clears the flag). */
int spk_test_bounded_wait(int64_t limit_ns, void* stream);

/*
 * LIF forward scan over T steps (Lif.py:118-165):
 *   v_0 = 0;  v = beta*v + in_gain*x[t];  s[t] = (v > v_th);  v = s[t] ? v_reset : v
 *   v_final = v after the last step.
 * x: [T][N] of x_dtype (F32/F16/BF16), spikes: [T][N] of spike_dtype
 * (F32/BF16/U8/FP8, values 0 or 1, or BIT: packed, ceil(N/8) bytes per
 * step), v_final: [N] fp32 (may be NULL).
 * in_gain == 1 reproduces the reference exactly (two roundings per step).
 */
int spk_lif_fwd(const void* x, int x_dtype, void* spikes, int spike_dtype, float* v_final,
                const float* beta, const float* v_th, const float* v_reset, float in_gain,
                int64_t T, int64_t N, void* stream);

/*
 * LIF backward (Lif.py:221-276) with the membrane history held in registers.
 * g_spikes: [T][N] fp32; g_vfinal: [N] fp32 or NULL; x: [T][N] x_dtype;
 * spikes: [T][N] spike_dtype (from spk_lif_fwd, any of its spike dtypes
 * including packed bits).  grad_x: [T][N] x_dtype.
 * grad_beta: one fp32 (device), the sum over all neurons (Lif.py:95);
 * may be NULL.  `surrogate_k` is k (SuperSpike) or alpha (arctan).
 * workspace: fp32 scratch of spk_lif_bwd_workspace_bytes(T, N) bytes
 * (per-block partial sums of grad_beta, reduced in a fixed order).
 * T <= 64.
 */
int64_t spk_lif_bwd_workspace_bytes(int64_t T, int64_t N);
int spk_lif_bwd(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype,
                const void* spikes, int spike_dtype, const float* beta, const float* v_th,
                const float* v_reset, float in_gain, int surrogate, float surrogate_k,
                void* grad_x, float* grad_beta, void* workspace, int64_t workspace_bytes,
                int64_t T, int64_t N, void* stream);

/*
 * spk_lif_bwd without a workspace argument; it allocates nothing.
 * No counterpart in the reference (its LIFLayer.backward allocates through
 * torch); this entry point exists for callers that cannot allocate device
 * memory: code running while a custom allocator owns the whole device heap,
 * plugin hosts with a memory budget fixed up front, or plain C / FFI callers
 * with no device allocator of their own.
 * Arguments and results are those of spk_lif_bwd, bit-identical to it.  The
 * grad_beta partial sums go to a file-scope 16 KiB device array (4096 floats,
 * the most any call's grid needs, so no N is too large; a call that would
 * need more is rejected with SPK_ERR_SHAPE; T > 64 is rejected as in
 * spk_lif_bwd).  The first call on a device, with that device current, looks
 * up the array's address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  The address stays cached for the life of the
 * process: after cudaDeviceReset on a device the module may load elsewhere,
 * so do not call this entry point on that device again.  All calls on a
 * device share the array: calls whose
 * kernels overlap on the GPU (unordered streams) race and must be serialised
 * by the caller.  No cudaMalloc, cudaFree or allocating library routine is
 * called.
 */
int spk_lif_bwd_noalloc(const float* g_spikes, const float* g_vfinal, const void* x, int x_dtype,
                        const void* spikes, int spike_dtype, const float* beta, const float* v_th,
                        const float* v_reset, float in_gain, int surrogate, float surrogate_k,
                        void* grad_x, float* grad_beta, int64_t T, int64_t N, void* stream);

/*
 * LayerNorm -> LIF for training, forward (replaces nn.LayerNorm followed by
 * the LIF module in the autograd path: SSA.py:218-228, :247-249,
 * SpikingMLP.py:31-36, LIFLayer.forward Lif.py:10-43).
 *   y = LN(pre + pre_bias) * ln_gamma + ln_beta over the D features of each
 *   of the T*R rows; LIF over t: v = lif_beta v + in_gain y, s = v > lif_vth,
 *   reset.  pre_bias ([D] fp32 or NULL) is the preceding Linear's bias, so
 *   that Linear can run without one.
 * pre: [T][R][D] (f32/f16/bf16); spikes: [T][R][D] in spike_dtype;
 * pre_ld: row stride of pre in elements (0 or D: contiguous; wider: pre is a
 * column slice of a wider GEMM output, D % 128 == 0 only).
 * With head_dim > 0 the spikes are written head-major instead,
 * [T*B][D/head_dim][seq_len][head_dim] with R = B * seq_len (the layout of
 * SSA.py's per-head Q, K, V, :221-233), for D % 128 == 0 only.
 * stats: [T*R] (mean, rstd) float pairs for the backward.  ln_gamma /
 * ln_beta may be NULL (1 / 0).  T <= 4; D a multiple of 32 up to 512, or of
 * 128 up to 2048.
 */
int spk_ln_lif_fwd(const void* pre, int pre_dtype, const float* pre_bias, const float* ln_gamma,
                   const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                   const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t D,
                   int64_t pre_ld, int64_t head_dim, int64_t seq_len, void* spikes, int spike_dtype,
                   float* stats, void* stream);

/*
 * spk_ln_lif_fwd with the residual connection of a transformer layer fused in
 * (Encoder.py:19-22, Decoder.py:18-24: x = x + LIF(LN(Linear(...)))):
 *   out[t*R + r][d] = residual[t*R + r][d] + spike,
 * fp32 row-major [T*R][D], and, when out_bf16 is not null, the same values in
 * bf16 (spike counts are small integers, exact in both; the bf16 copy is what
 * the next layer's GEMMs read).  stats as in spk_ln_lif_fwd.  D must be 384,
 * 768 or 1536 and every pointer 16-byte aligned; SPK_ERR_UNSUPPORTED
 * otherwise (the caller then adds the spikes of spk_ln_lif_fwd itself).  The
 * backward is spk_ln_lif_bwd with g_spikes = dL/dout (dL/dresidual = dL/dout).
 */
int spk_ln_lif_fwd_residual(const void* pre, int pre_dtype, const float* pre_bias, const float* ln_gamma,
                            const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                            const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t D,
                            int64_t pre_ld, const float* residual, float* out, void* out_bf16, float* stats,
                            void* stream);

/*
 * Backward of spk_ln_lif_fwd (LIFLayer.backward Lif.py:46-102 composed with
 * the LayerNorm backward): recomputes x^ and the membrane from pre and stats,
 * BPTT with the surrogate, then
 *   g_pre = rstd (g - mean(g) - x^ mean(g x^)),  g = ln_gamma dL/dy,
 *   g_gamma = sum dL/dy x^, g_beta_ln = sum dL/dy, g_bias = sum g_pre,
 *   g_lif_beta = sum g_v v_prev
 * (sums over all rows, reduced in a fixed order).  g_spikes: f32/f16/bf16;
 * g_pre has pre's dtype; pre_bias is the forward's; g_gamma / g_beta_ln /
 * g_bias / g_lif_beta may be NULL.  pre_ld / head_dim / seq_len: the
 * forward's; g_pre has pre's row stride, and g_spikes is read head-major when
 * head_dim > 0.
 * workspace: spk_ln_lif_bwd_workspace_bytes(T, R, D) bytes.
 */
int64_t spk_ln_lif_bwd_workspace_bytes(int64_t T, int64_t R, int64_t D);
int spk_ln_lif_bwd(const void* g_spikes, int gs_dtype, const void* pre, int pre_dtype,
                   const float* pre_bias, const float* stats, const float* ln_gamma,
                   const float* ln_beta, const float* lif_beta, const float* lif_vth,
                   const float* lif_vreset, float in_gain, int surrogate, float surrogate_k, int64_t T,
                   int64_t R, int64_t D, int64_t pre_ld, int64_t head_dim, int64_t seq_len, void* g_pre,
                   float* g_gamma, float* g_beta_ln, float* g_bias, float* g_lif_beta, void* workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * Fused Linear -> LayerNorm -> LIF (tcgen05, bf16 operands, fp32 accumulate).
 *   pre = A W^T + bias;  y = LN(pre) * ln_gamma + ln_beta  (over the N features,
 *   eps = ln_eps);  LIF over T on y;  spikes (0/1) written as bf16 or fp32.
 * t_broadcast == 0: A is [T][R][K] (t-major fold), spikes [T][R][N].
 * t_broadcast != 0: A is [R][K]; the LIF sees the same y at every step (input
 *                   repeated over T); spikes [T][R][N].
 * W: [N][K] bf16 (nn.Linear layout).  bias/ln_gamma/ln_beta: [N] fp32 or NULL
 * (0 / 1 / 0).  residual: [T][R][N] bf16 or NULL; if given, spikes are added
 * into it in place (the residual stream of Encoder/Decoder layers).  spikes
 * may be NULL when residual is given.  ln_out: [T][R][N] fp32 (or [R][N] for
 * t_broadcast) copy of y, or NULL.  Requires K % 8 == 0, N % 32 == 0,
 * N <= 4096 (rows wider than 384 are split over a CTA cluster), T <= 128.
 */
int spk_linear_ln_lif_fwd(const void* A, const void* W, const float* bias, const float* ln_gamma,
                          const float* ln_beta, float ln_eps, const float* lif_beta, const float* lif_vth,
                          const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t K, int64_t N,
                          int t_broadcast, void* spikes, int spike_dtype, void* residual, float* ln_out,
                          void* stream);

/*
 * Fused Linear -> per-feature affine -> LIF: the convolutions of the CNN
 * image encoder (as GEMMs over spk_im2col patches) with their eval-mode
 * BatchNorm and LIF (ImageEncoder.py:8-102: conv + bn + lif in
 * FusedInvertedBottleneck :19-28, ReduceConvBlock :34-44, RPE2D :50-61 and
 * CNNBackbone :75-100).
 *   y = (A W^T + bias) * scale + shift  (per feature; no row statistics);
 *   LIF over T on y; spikes (0/1) as bf16 or fp32; with residual, the spikes
 *   are also added into it in place (the identity of the bottleneck, the
 *   x + rpe sum).  For eval-mode BatchNorm, scale = weight / sqrt(var + eps)
 *   and shift = bias_bn - mean * scale.
 * A, W, t_broadcast, spikes, residual and the size limits are those of
 * spk_linear_ln_lif_fwd; scale / shift: [N] fp32 or NULL (1 / 0).
 */
int spk_linear_affine_lif_fwd(const void* A, const void* W, const float* bias, const float* scale,
                              const float* shift, const float* lif_beta, const float* lif_vth,
                              const float* lif_vreset, float in_gain, int64_t T, int64_t R, int64_t K, int64_t N,
                              int t_broadcast, void* spikes, int spike_dtype, void* residual, void* stream);

/*
 * Patch gather for a convolution with stride (stride_h, stride_w) and zero
 * padding (pad_h, pad_w): x [N][H][W][C] channels-last (F32 or BF16) ->
 * out [N*Ho*Wo][Kc] bf16, Ho = (H + 2 pad_h - kh) / stride_h + 1 (Wo alike),
 * row (n, ho, wo), column (i*kw + j)*C + c for tap (i, j).  BF16 input:
 * Kc = kh*kw*C.  F32 input: Kc = 2*kh*kw*C, the bf16 rounding of each value
 * in the first half and of its remainder in the second (against [W | W] the
 * product is the fp32 convolution to ~2^-17 relative).  Used for the CNN
 * image encoder's convolutions (ImageEncoder.py:8-102); PixelUnshuffle(p)
 * followed by a 3x3 / padding-1 convolution is one 3p x 3p / stride-p /
 * padding-p gather of the image.
 */
int spk_im2col(const void* x, int x_dtype, int64_t N, int64_t H, int64_t W, int64_t C, int64_t kh, int64_t kw,
               int64_t stride_h, int64_t stride_w, int64_t pad_h, int64_t pad_w, void* out, void* stream);

/*
 * Gradients of a bias-free Linear y[M][N] = x[M][K] W[N][K]^T for the
 * training path (autograd of nn.Linear in SSA.py:218-249 and
 * SpikingMLP.py:31-36 under the reference's autocast, train_spikeformer.py:545):
 *   spk_linear_dgrad:  dX[M][K] = G[M][N] W[N][K]        (fp32 out)
 *   spk_linear_wgrad:  dW[N][K] = G[M][N]^T X[M][K]      (fp32 out)
 * G, W, X bf16, row-major as torch holds them: the tcgen05 operands read W
 * (dgrad) and G, X (wgrad) contiguous along their output dimension, so no
 * transposed copy is made.  The weight gradient splits the sum over the M
 * rows across CTAs into fp32 partial sums in `workspace`
 * (spk_linear_wgrad_workspace_bytes(M, N, K) bytes, possibly 0), reduced in a
 * fixed order.  N and K multiples of 8; pointers 16-byte aligned.
 */
int spk_linear_dgrad(const void* G, const void* W, float* dX, int64_t M, int64_t N, int64_t K, void* stream);
int64_t spk_linear_wgrad_workspace_bytes(int64_t M, int64_t N, int64_t K);
int spk_linear_wgrad(const void* G, const void* X, float* dW, void* workspace, int64_t workspace_bytes, int64_t M,
                     int64_t N, int64_t K, void* stream);

/* out[M][N] (fp32) = A[M][K] W[N][K]^T + bias (bias may be NULL); bf16 A, W. */
int spk_linear_fwd(const void* A, const void* W, const float* bias, float* out, int64_t M, int64_t K, int64_t N,
                   void* stream);

/*
 * Spiking attention core + output LIF.
 * q: [T][B][Nq][H*dh], k, v: [T][B][Nk][H*dh], bf16 spikes (0/1).
 * variant 1 (XNOR, SSA.py:145-165,235-242):
 *   S[i,j] = dh - (|q_i| + |k_j| - 2 q_i.k_j) + R(|i-j|),
 *   R(d) = max(0, ceil(log2((max(Nq,Nk)-1)/(d+1))))
 * variant 0 (plain, SSA.py:81-84): S = q_i.k_j.
 * S is multiplied by the mask, O = S V (exact integer), a = scale * O, then a
 * LIF over T (lif_* parameters) gives out [T][B][Nq][H*dh] (bf16 or fp32).
 * mask_mode 0: none; 1: causal (key index <= query index); 2: dense uint8,
 * nonzero = keep, element (t,b,h,i,j) at t*mask_stride_t + b*mask_stride_b +
 * h*mask_stride_h + i*mask_stride_q + j (strides in elements, 0 broadcasts).
 * scale: device fp32 scalar (the learnable SSA.scale, or 0.125 for plain).
 * attn_out: [T][B][H][Nq][dh] fp32 copy of a (the LIF input), or NULL.
 * Requires dh % 8 == 0, 8 <= dh <= 64, Nq, Nk <= 8192.
 */
int spk_ssa_fwd(const void* q, const void* k, const void* v, int variant, int mask_mode, const uint8_t* mask,
                int64_t mask_stride_t, int64_t mask_stride_b, int64_t mask_stride_h, int64_t mask_stride_q,
                const float* scale, const float* lif_beta, const float* lif_vth, const float* lif_vreset,
                float in_gain, int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, void* out,
                int out_dtype, float* attn_out, void* stream);

/*
 * The unmasked core of spk_ssa_fwd (score-free kernel, Nq, Nk <= 256) on
 * head-split operands: q [T*B][H][Nq][dh], k, v [T*B][H][Nk][dh] bf16 spikes
 * (0/1), given as views with element strides strides[9] = {q: t*b, head,
 * position; k: the same; v: the same} (unit stride along dh; every stride a
 * positive multiple of 8 elements).  out, scale and the LIF parameters as
 * in spk_ssa_fwd (out token-major [T][B][Nq][H*dh]); attn_out (the LIF input
 * a = scale * O, or NULL) is token-major too: [T][B][Nq][H*dh] fp32.
 */
int spk_ssa_fwd_heads(const void* q, const void* k, const void* v, const int64_t* strides, int variant,
                      const float* scale, const float* lif_beta, const float* lif_vth, const float* lif_vreset,
                      float in_gain, int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, void* out,
                      int out_dtype, float* attn_out, void* stream);

/*
 * tokens: [B][N] int64; emb: [V][D] fp32; pe: [>=N][D] fp32 (row n for
 * position n).  x = emb[tok]*emb_scale + pe[n] (fp32, two roundings); LIF over
 * T with input x at every step; out [T][B][N][D] bf16 or fp32.
 * bad_token: device int set to 1 if a token is outside [0, V) (that token
 * then reads row 0); the caller zeroes it beforehand.
 */
int spk_embed_pe_lif_fwd(const int64_t* tokens, const float* emb, float emb_scale, const float* pe,
                         const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                         int64_t T, int64_t B, int64_t N, int64_t D, int64_t V, void* out, int out_dtype,
                         int* bad_token, void* stream);

/*
 * img: [B][C][H][W] fp32 -> out: [B*(H/p)*(W/p)][2*C*p*p] bf16; row
 * (b, ph, pw) in row-major patch order, columns [0, K) the bf16 rounding of
 * pixel (c, i, j) at k = (c*p + i)*p + j, columns [K, 2K) the bf16 rounding
 * of the remainder.  Against W' = [W | W] this reproduces Conv2d(C, D, p,
 * stride p) in fp32 to ~2^-17 relative.
 */
int spk_patch_im2col(const float* img, int64_t B, int64_t C, int64_t H, int64_t W, int64_t patch, void* out,
                     void* stream);

/*
 * img: [B][1][H][W] fp32 <- U(0, 0.2) background with 5-40 black (0.0)
 * rectangles of side 8-20 px per image; tokens (optional, else NULL):
 * [B][L] int64 uniform in [0, V).  Every value is a function of (seed,
 * image, draw) through a counter-based hash (SplitMix64), so batches are
 * reproducible on any GPU and on the CPU.  H, W >= 20.
 */
int spk_synth_text_lines(float* img, int64_t B, int64_t H, int64_t W, uint64_t seed, int64_t* tokens, int64_t L,
                         int64_t V, void* stream);

/*
 * logits: [T][rows][V] (dtype SPK_F32 or SPK_BF16); targets: [rows] int64.
 * out[0] = mean over t of CrossEntropyLoss(ignore_index, label_smoothing) of
 * step t (mean over non-ignored rows), out[1] = token accuracy of the argmax
 * of the T-averaged logits over non-ignored rows, out[2] = 1 / max(1, number
 * of non-ignored rows).  grad (optional, else NULL; logits' dtype and shape)
 * <- dloss/dlogits divided by out[2]'s reciprocal, i.e. the caller multiplies
 * grad by out[2].  workspace: spk_ce_over_t_workspace_bytes(rows) bytes.
 * bad_target: device int set to 1 if a non-ignored target is outside [0, V).
 */
int64_t spk_ce_over_t_workspace_bytes(int64_t rows);
int spk_ce_over_t(const void* logits, int dtype, const int64_t* targets, int64_t T, int64_t rows, int64_t V,
                  int64_t ignore_index, float label_smoothing, float* out, void* grad, void* workspace,
                  int64_t workspace_bytes, int* bad_target, void* stream);

/*
 * Memory-bound passes of the training-path XNOR attention core, the autograd
 * regrouping of SSAMultiHeadAttention's unmasked attention (SSA.py:145-165,
 * :177-201, :235-240; the reference differentiates the dense score matrix
 * instead).  With B = TB*H heads and M = 2 K^T V - 1 (1^T V)^T,
 * w = (dh - |k|)^T V, the forward is m = Q M + R V + 1 w^T; the products run
 * as library GEMMs with fp32 accumulation.  dh % 4 == 0, fp32 buffers
 * 16-byte aligned.
 *
 * combine: out[tb][n][h][:] = (qm[b][n][:] + rv[n][b][:] + w[b][:]) * scale[0]
 *   with b = tb*H + h; qm [B][Nq][dh], rv [Nq][B][dh], w [B][dh] fp32; out
 *   token-major [TB][Nq][H][dh] fp32.
 */
int spk_xnor_train_combine(const float* qm, const float* rv, const float* w, const float* scale, float* out,
                           int64_t TB, int64_t H, int64_t Nq, int64_t dh, void* stream);

/*
 * Row chunks of spk_xnor_train_grad_prep's partial sums (16 rows each).
 */
int64_t spk_xnor_train_prep_chunks(int64_t Nq);

/*
 * grad_prep: from the token-major gradient g [TB][Nq][H][dh] fp32 and the
 * forward's out, gs = g * scale[0] split into bf16 hi = bf16(gs) and
 * lo = bf16(gs - hi):
 *   g_heads [B][Nq][2 dh] bf16 (hi | lo along the last dimension),
 *   g_rows  [Nq][2][B][dh] bf16 (hi block, lo block),
 *   gcol_part [C][B][dh] fp32 (sums of gs over each chunk of 16 rows),
 *   gscale_part [C][B*dh/4] fp32 (partial sums of g * out),
 * C = spk_xnor_train_prep_chunks(Nq).
 */
int spk_xnor_train_grad_prep(const float* g, const float* out, const float* scale, void* g_heads, void* g_rows,
                             float* gcol_part, float* gscale_part, int64_t TB, int64_t H, int64_t Nq, int64_t dh,
                             void* stream);

/*
 * grad_finish: dv[b][j][:] = ke[b][j][:] + rg[j][b][:] + u[b][:] and
 * dk = dk32, both written in out_dtype (SPK_F32 / SPK_F16 / SPK_BF16),
 * head-major [B][Nk][dh]; ke, dk32 [B][Nk][dh], rg [Nk][B][dh], u [B][dh]
 * fp32.
 */
int spk_xnor_train_grad_finish(const float* ke, const float* rg, const float* u, const float* dk32, void* dk,
                               void* dv, int out_dtype, int64_t TB, int64_t H, int64_t Nk, int64_t dh, void* stream);

/*
 * n_major: out[n][b][:] = in[b][n][:] for B x N rows of row_bytes bytes
 * (a multiple of 16; in and out 16-byte aligned).  Makes the n-major
 * [Nk][B][dh] operand of the shared log-distance product R V (SSA.py:235-240)
 * from the head-major V [B][Nk][dh].
 */
int spk_xnor_train_n_major(const void* in, void* out, int64_t B, int64_t N, int64_t row_bytes, void* stream);

/*
 * combine followed by the attention's output LIF (SSA.py:242, the LIF
 * module of Lif.py:288-441 over the T-major fold, T <= 4, TB % T == 0):
 * a_out <- the combined pre-activation (as spk_xnor_train_combine's out),
 * spikes <- LIF(a_out) in spike_dtype (SPK_F32 / SPK_F16 / SPK_BF16), both
 * token-major [TB][Nq][H][dh].  The LIF arithmetic is spk_lif_fwd's.
 */
int spk_xnor_train_combine_lif(const float* qm, const float* rv, const float* w, const float* scale,
                               const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                               float* a_out, void* spikes, int spike_dtype, int64_t T, int64_t TB, int64_t H,
                               int64_t Nq, int64_t dh, void* stream);

/*
 * grad_prep after the output LIF's backward: g_spikes (dL/dspikes,
 * token-major, gs_dtype) and the pre-activation a give dL/da by BPTT with
 * the surrogate (spk_lif_bwd's arithmetic), then the outputs of
 * spk_xnor_train_grad_prep, except that gscale_part (and gbeta_part, the
 * partial sums of the LIF beta gradient, or NULL) are [C][TB/T*H*dh/4].
 */
int spk_xnor_train_grad_prep_lif(const void* g_spikes, int gs_dtype, const float* a, const float* scale,
                                 const float* lif_beta, const float* lif_vth, const float* lif_vreset, float in_gain,
                                 int surrogate, float surrogate_k, void* g_heads, void* g_rows, float* gcol_part,
                                 float* gscale_part, float* gbeta_part, int64_t T, int64_t TB, int64_t H, int64_t Nq,
                                 int64_t dh, void* stream);

/*
 * Masked spiking attention core for training, short sequences (Nq, Nk <= 64,
 * dh <= 64): the decoder's masked self-attention (SSA.py:234-242 with
 * xnor_attention :145-165 and the log-distance bias :177-201; plain form
 * SSA.py:81-84), which the reference differentiates with torch's autograd
 * through the dense score matrix.  One CTA per (t*b, head) keeps S in shared
 * memory.
 *   fwd:  a = scale * ((S * M) V), token-major a [T*B][Nq][H*dh] fp32
 *   bwd:  from g = dL/da (same layout, fp32): dq, dk, dv (the layout and
 *         dtype of q, k, v) and per-unit partial sums of dL/dscale,
 *         dscale_part [T*B*H] fp32 (summed by the caller).
 * q, k, v: dtype SPK_F32 / SPK_F16 / SPK_BF16 spikes, element (tb, h, n, d)
 * at tb*strides[0] + h*strides[1] + n*strides[2] + d for q (strides[3..5]
 * for k, strides[6..8] for v; `strides` is a host array of 9).  mask: NULL or
 * uint8 (t, b, h, i, j) at t*mask_stride_t + b*mask_stride_b + h*mask_stride_h
 * + i*mask_stride_q + j, nonzero = keep.  variant 1 XNOR, 0 plain; scale a
 * device fp32 scalar.
 */
int spk_attn_masked_train_fwd(const void* q, const void* k, const void* v, int dtype, const int64_t* strides,
                              const uint8_t* mask, int64_t mask_stride_t, int64_t mask_stride_b,
                              int64_t mask_stride_h, int64_t mask_stride_q, int variant, const float* scale,
                              int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, float* a,
                              void* stream);
int spk_attn_masked_train_bwd(const void* q, const void* k, const void* v, int dtype, const int64_t* strides,
                              const uint8_t* mask, int64_t mask_stride_t, int64_t mask_stride_b,
                              int64_t mask_stride_h, int64_t mask_stride_q, int variant, const float* scale,
                              int64_t T, int64_t B, int64_t H, int64_t Nq, int64_t Nk, int64_t dh, const float* g,
                              void* dq, void* dk, void* dv, float* dscale_part, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPK_H_ */
