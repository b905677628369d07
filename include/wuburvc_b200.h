/* wuburvc_b200.h — C ABI of the B200 (sm_100a) generator training library.
 *
 * Plain C types only: pointers, sizes, ints and floats.  Two groups of entry points:
 *
 *  1. Convolution primitives on device buffers (channels-last [B][T][C] bf16 activations).
 *     They replace the per-op kernels of the reference's CUDA trainer:
 *       k_conv1d        src/wubu_rvc_cuda.cu:36-53      -> wubu_b200_conv1d
 *       tk_conv1d_bwd   src/wubu_train_cuda.cu:67-105   -> wubu_b200_conv1d (flipped weights, dgrad)
 *                                                          + wubu_b200_conv1d_wgrad
 *       k_convt1d       src/wubu_rvc_cuda.cu:55-78      -> wubu_b200_convT
 *       tk_convt1d_bwd  src/wubu_train_cuda.cu:107-135  -> wubu_b200_convT_dgrad + wubu_b200_convT_wgrad
 *     and the spectral loss gradient of the host trainer:
 *       wubu_stft_loss_grad  src/wubu_train.c:318-446    -> wubu_b200_stft_loss_grad
 *
 *  2. The generator training step (wubu_b200_gen_*): forward, backward and the fused AdamW
 *     update over one flat parameter buffer, replacing wubu_train_forward_cuda /
 *     wubu_train_backward_cuda / wubu_train_step_cuda (src/wubu_train.h:92-104).
 *
 * Return codes: 0 = OK, negative = error (see WUBU_B200_ERR_*).  Nothing here allocates on
 * behalf of the caller except where stated; every call is synchronous unless it says so.
 */
#ifndef WUBURVC_B200_H
#define WUBURVC_B200_H

#ifdef __cplusplus
extern "C" {
#endif

#define WUBU_B200_OK 0
#define WUBU_B200_ERR_ARG (-1)
#define WUBU_B200_ERR_CUDA (-2)
#define WUBU_B200_ERR_SHAPE (-3)
#define WUBU_B200_ERR_TIMEOUT (-4) /* a kernel's bounded wait expired; the context stays usable */
#define WUBU_B200_ERR_COMM (-5)
#define WUBU_B200_ERR_NOMEM (-6)
#define WUBU_B200_ERR_RANGE (-7) /* a forward GEMM operand reached 65504, the limit of its fp16 split */

/* ---------------------------------------------------------------------------------------
 * 1. convolution primitives (device pointers, `stream` = cudaStream_t or NULL)
 * ------------------------------------------------------------------------------------- */

/* Conv1d, stride 1: out[b,t,o] = bias[o] + sum_{tap,i} x[b, t-pad+dil*tap, i] * w[tap,o,i]
 *   x_hi/x_lo [B][T][C_in], w_hi/w_lo [k][C_out][C_in], out [B][T_out][C_out] f32,
 *   T_out = T + 2*pad - dil*(k-1).
 *   split=1: fp32-accurate forward.  Each operand is an fp16 pair, value = hi + lo / 2048
 *            (hi = fp16(x), lo = fp16((x - hi) * 2048)); |x| must stay below 65504.  The product
 *            is hi*hi + (hi*lo + lo*hi) / 2048.
 *   split=0: x_hi and w_hi are bf16, the lo pointers are ignored (one bf16 product).
 *   Replaces k_conv1d (src/wubu_rvc_cuda.cu:36-53) and conv1d_fwd (src/wubu_train.c:461-486). */
int wubu_b200_conv1d(const void* x_hi, const void* x_lo, const void* w_hi, const void* w_lo,
                     const float* bias, float* out, int B, int C_in, int T, int C_out, int k, int dil,
                     int pad, int split, void* stream);

/* Conv1d weight gradient dw[o][i][tap] = sum_{b,t} dy[b,t,o] * x[b, t-pad+dil*tap, i]
 *   dy [B][T_out][C_out] bf16, x [B][T][C_in] bf16, dw f32.
 *   Replaces the dw part of tk_conv1d_bwd (src/wubu_train_cuda.cu:67-105), conv1d_bwd
 *   (src/wubu_train.c:490-527). */
int wubu_b200_conv1d_wgrad(const void* dy, const void* x, float* dw, int B, int C_in, int T, int C_out,
                           int k, int dil, int pad, void* stream);

/* Same result as wubu_b200_conv1d_wgrad, but allocates nothing.  No counterpart in the reference.
 *   For callers that cannot call cudaMalloc: a host whose device memory is owned entirely by its
 *   own allocator, or a host that forbids allocation in its processing callback (cudaMalloc /
 *   cudaFree take the driver's locks and cudaFree may synchronise the whole device).  The split-K
 *   scratch is a fixed file-scope __device__ array of 16 MiB (4 Mi floats) that every GPU loading
 *   the library keeps until exit; problems whose C_out*k*C_in partial tile exceeds it (or k > 256)
 *   are rejected with WUBU_B200_ERR_SHAPE, larger ones run with fewer splits.  The first call on a
 *   device resolves the array's device address (make it before any stream capture).  All calls
 *   share the array: calls that overlap on the GPU race.  The call returns once its stream has
 *   finished the work (it reads back the kernels' error word). */
int wubu_b200_conv1d_wgrad_noalloc(const void* dy, const void* x, float* dw, int B, int C_in, int T, int C_out,
                                   int k, int dil, int pad, void* stream);

/* ConvTranspose1d (polyphase): out[b, i*s-pad+tap, o] += x[b,i,c] * W[c][o][tap]
 *   x [B][T_in][C_in]; wp [k][C_out][C_in] = W taps in phase order (operand pairs as for
 *   wubu_b200_conv1d: fp16 hi + lo/2048 when split=1, bf16 hi alone when split=0)
 *   (phase r = 0..s-1, taps r, r+s, r+2s, ...), transposed; out [B][T_in*s][C_out] f32.
 *   Requires k - 2*pad == s.  Replaces k_convt1d (src/wubu_rvc_cuda.cu:55-78), convt1d_fwd
 *   (src/wubu_train.c:533-562). */
int wubu_b200_convT(const void* x_hi, const void* x_lo, const void* wp_hi, const void* wp_lo,
                    const float* bias, float* out, int B, int C_in, int T_in, int C_out, int k,
                    int stride, int pad, int split, void* stream);

/* ConvTranspose1d input gradient dx[b,i,c] = sum_{tap,o} dy[b, i*s-pad+tap, o] * W[c][o][tap]
 *   dy [B][T_in*s][C_out] bf16, wd [k][C_in][C_out] bf16, dx [B][T_in][C_in] f32.
 *   Replaces the din part of tk_convt1d_bwd (src/wubu_train_cuda.cu:107-135). */
int wubu_b200_convT_dgrad(const void* dy, const void* wd, float* dx, int B, int C_in, int T_in,
                          int C_out, int k, int stride, int pad, void* stream);

/* ConvTranspose1d weight gradient dw[c][o][tap] = sum_{b,i} x[b,i,c] * dy[b, i*s-pad+tap, o]
 *   Replaces the dw part of tk_convt1d_bwd (src/wubu_train_cuda.cu:107-135). */
int wubu_b200_convT_wgrad(const void* x, const void* dy, float* dw, int B, int C_in, int T_in,
                          int C_out, int k, int stride, int pad, void* stream);

/* Multi-scale STFT spectral loss (linear + log magnitude, windows 512/256/128, hop w/4) and its
 * gradient with respect to the first signal, for B signal pairs of n samples (device fp32
 * buffers [B][n]): loss[b] and grad[b][n].  n_scales <= 0 means 3.  Same loss and gradient as
 * wubu_stft_loss_grad (src/wubu_train.c:318-446, called by wubu_train_step at :1156-1178), which
 * it replaces for batches on the device; deterministic. */
int wubu_b200_stft_loss_grad(const float* a, const float* b, int B, int n, int n_scales, float* grad,
                             float* loss, void* stream);
/* The same on host buffers (copied to and from the current device; synchronous), the form a host
 * trainer such as the reference's wubu_train_step(_cuda) (src/wubu_train.c:1151-1176) calls. */
int wubu_b200_stft_loss_grad_host(const float* a, const float* b, int B, int n, int n_scales, float* grad,
                                  float* loss);

/* Bounded waits.  Every wait of the library's tensor-core kernels on a pipeline barrier gives up
 * after a limit (default 2 s, far above any legitimate wait); the kernel then records an error,
 * lets its own copies and MMAs in flight finish (each drain again bounded), frees its TMEM and
 * returns, and the call reports WUBU_B200_ERR_TIMEOUT with the context still usable.  No
 * counterpart in the reference (its kernels have no barrier waits).
 * set_wait_limit_ns sets the limit (ns) for the launch plans built afterwards (contexts created,
 * primitive calls made); 0 restores the default.  wait_selftest makes one warp wait on a barrier
 * that nothing arrives on, for limit_ns (0 < limit_ns <= 10 s): it returns WUBU_B200_ERR_TIMEOUT
 * when the wait ran out as designed. */
int wubu_b200_set_wait_limit_ns(unsigned long long ns);
int wubu_b200_wait_selftest(unsigned long long limit_ns, void* stream);

/* ---------------------------------------------------------------------------------------
 * 2. generator training step
 * ------------------------------------------------------------------------------------- */

/* Generator topology.  Mirrors the reference model config (WuBuRVCModel upsample_rates /
 * upsample_kernel_sizes / resblock_k / resblock_dil, src/wubu_rvc_parity.h:206-217) and the
 * upstream GeneratorNSF constructor (knowledge/rvc_original/infer/module/models.py:403-475). */
typedef struct WubuB200GenConfig {
  int sample_rate;            /* 40000 / 32000 / 48000 */
  int n_ups;                  /* must be 4 */
  int upsample_rates[4];      /* e.g. 10,10,2,2 */
  int upsample_kernels[4];    /* e.g. 16,16,4,4 */
  int initial_channel;        /* 512 */
  int in_channels;            /* 192 (z channels) */
  int gin_channels;           /* 256 speaker-embedding channels, 0 = no cond(g) */
  int n_kernels;              /* 3 resblock stacks per stage */
  int resblock_kernels[3];    /* 3, 7, 11 */
  int n_dilations;            /* 3 conv pairs per stack */
  int resblock_dilations[3][3];
  int harmonic_num;           /* 8 -> 9 source harmonics */
  float sine_amp;             /* 0.1 */
  float noise_std;            /* 0.003 */
  int activation;             /* 0 = LeakyReLU, 1 = Snake(alpha per channel) */
  float lrelu_slope;          /* 0.1 */
  float final_slope;          /* slope of the activation before conv_post (0.1 in the reference) */
  int weight_norm;            /* 1: ups / resblock weights trained as (g, v) */
  int nsf;                    /* 1: harmonic source + noise convs */
} WubuB200GenConfig;

/* Arithmetic of the backward GEMMs (WubuB200TrainOptions.precision).  The forward GEMMs take fp16
 * hi + scaled-lo operand pairs (three products, fp32-accurate) in both modes.
 *   BF16: input- and weight-gradient GEMMs on single bf16 operands with fp32 accumulation.
 *   FP32: every backward GEMM operand is a bf16 hi + bf16 lo pair (x = hi + lo to ~2^-17) and three
 *         products are taken (hi*hi + hi*lo + lo*hi): the fp32-accurate mode of the reference's fp32
 *         conv loops (src/wubu_train.c:461-601), at about three times the backward's tensor work. */
enum { WUBU_B200_PRECISION_BF16 = 0, WUBU_B200_PRECISION_FP32 = 1 };

typedef struct WubuB200TrainOptions {
  int batch;                  /* items per step on this GPU */
  int frames;                 /* frames per item */
  int device;                 /* CUDA device ordinal */
  float lr, beta1, beta2, eps, weight_decay;  /* AdamW, src/wubu_train.c:57-73 */
  unsigned long long seed;    /* source-noise generator seed */
  int precision;              /* WUBU_B200_PRECISION_BF16 (0, default) or _FP32 */
} WubuB200TrainOptions;

typedef struct WubuB200Gen WubuB200Gen; /* opaque */

/* Parameter table (host only, needs no GPU).  The flat fp32 buffer holds every trainable
 * tensor at a 64-float aligned offset; names follow the reference registry
 * (src/wubu_train.c:131-210: dec.conv_pre.weight, dec.ups.L.*, dec.resblocks.R.convsX.P.*,
 * dec.conv_post.weight) plus the GeneratorNSF extras (dec.cond.*, dec.noise_convs.L.*,
 * dec.m_source.l_linear.*, weight_g/weight_v pairs, Snake alphas). */
int wubu_b200_gen_param_count(const WubuB200GenConfig* cfg);
long long wubu_b200_gen_param_total(const WubuB200GenConfig* cfg);
int wubu_b200_gen_param_info(const WubuB200GenConfig* cfg, int index, char* name, int name_cap, int* shape3,
                             long long* offset, long long* numel);
/* Data-parallel gradient buckets (host only, no GPU needed): writes the end offset (floats, in the
 * flat gradient buffer) of each all-reduce bucket into ends[0..n) and returns n (5: stages 3, 2, 1, 0
 * in backward-completion order, then conv_pre / cond / source), or a negative error code.  Bucket b
 * spans [ends[b-1], ends[b]) (ends[-1] = 0) and may be empty. */
int wubu_b200_gen_bucket_plan(const WubuB200GenConfig* cfg, long long* ends, int cap);

/* Deterministic init: conv weights / v ~ N(0, 0.01), g = ||v|| per dim-0 row, biases 0,
 * Snake alpha 1, l_linear weight U(-1/3, 1/3). */
int wubu_b200_gen_init_params(const WubuB200GenConfig* cfg, unsigned long long seed, float* host_flat);

/* Model lifecycle: allocates every device buffer and builds every launch plan once. */
WubuB200Gen* wubu_b200_gen_create(const WubuB200GenConfig* cfg, const WubuB200TrainOptions* opt);
void wubu_b200_gen_destroy(WubuB200Gen* gen);
int wubu_b200_gen_set_params(WubuB200Gen* gen, const float* host_flat);
int wubu_b200_gen_get_params(WubuB200Gen* gen, float* host_flat);
/* Optimiser state for checkpoint / resume: the AdamW first and second moments as flat buffers in the
 * same reference layout as get_params, the step count and the source-noise stream.  Replaces the
 * host WuBuAdamW state (src/wubu_train.c:43-52) kept between wubu_adamw_step calls.  set_params
 * restarts the optimiser, so restore with set_params first, then set_opt_state. */
int wubu_b200_gen_get_opt_state(WubuB200Gen* gen, float* m_flat, float* v_flat, long long* step,
                                unsigned long long* noise_stream);
int wubu_b200_gen_set_opt_state(WubuB200Gen* gen, const float* m_flat, const float* v_flat, long long step,
                                unsigned long long noise_stream);
int wubu_b200_gen_get_grads(WubuB200Gen* gen, float* host_flat);
int wubu_b200_gen_samples(const WubuB200Gen* gen); /* output samples per item */

/* Step inputs, host pointers (copied in), all fp32:
 *   z    [B][in_channels][F]     latent (reference layout: channels x frames)
 *   f0   [B][F]                  Hz, 0 = unvoiced (may be NULL when nsf == 0)
 *   g    [B][gin_channels]       speaker embedding (may be NULL when gin == 0)
 *   noise[B][T][harmonic_num+1]  standard-normal source noise, or NULL -> device generator
 *                                (counter-based, keyed by opt.seed and noise_stream)
 *   dldy [B][T]                  upstream gradient dL/d(audio); may be NULL for forward-only
 *                                use (the previous upload's stays; zeros before the first)  */
#define WUBU_B200_INPUTS_RESIDENT 1 /* use the inputs already on the device (last upload) */
int wubu_b200_gen_upload(WubuB200Gen* gen, const float* z, const float* f0, const float* g, const float* noise,
                         const float* dldy);
int wubu_b200_gen_forward(WubuB200Gen* gen, unsigned long long noise_stream, float* audio_out);
/* Forward-only (inference) mode.  on = 1: the forward stops writing the tensors that only the
 * backward reads (the activations' bf16 copies, Snake pre-activations, z's bf16 copy and the
 * input-gradient weight layout); the waveform is bit-identical to the training forward's.
 * on = 2: in addition every forward GEMM takes single fp16 operands (one product per K step instead
 * of the fp16 pair's three; forward rel-L2 about 4e-4 against fp64, inside the 2e-3 forward gate);
 * after a range error the context returns to the exact pairs.  on = 0: training.  While on != 0,
 * backward, AdamW and the training steps return WUBU_B200_ERR_ARG.  The reference's CUDA inference
 * (wubu_generator_nsf_cuda, src/wubu_rvc_cuda.cu:280) runs in mode 1 (2 with
 * WUBU_B200_INFERENCE=fast in the environment). */
int wubu_b200_gen_set_forward_only(WubuB200Gen* gen, int on);
int wubu_b200_gen_backward(WubuB200Gen* gen);
int wubu_b200_gen_adamw(WubuB200Gen* gen);
/* One full step (upload unless RESIDENT, forward, backward, gradient all-reduce when a
 * communicator is attached, AdamW).  audio_out (host, may be NULL) receives the forward output.
 * The step is captured once into a CUDA graph and replayed.
 *
 * Forward GEMM operands are fp16 hi + fp16 lo/2048 pairs (fp32-accurate) while every operand stays
 * below 65504.  When one reaches it, the step's update is skipped on the device (on every rank under
 * data parallelism), the context switches for good to bf16 hi + bf16 lo pairs (range-safe, ~2^-17
 * relative) and train_step / forward recompute the step, so the caller sees no error.  The
 * asynchronous step cannot: wubu_b200_gen_sync then returns WUBU_B200_ERR_RANGE once (the steps
 * enqueued since the overflow left the parameters unchanged) and later steps use the bf16 pairs. */
int wubu_b200_gen_train_step(WubuB200Gen* gen, const float* z, const float* f0, const float* g, const float* noise,
                             const float* dldy, float* audio_out, unsigned long long noise_stream, int flags);
/* Enqueue one resident-input step without synchronising (for device-side timing). */
int wubu_b200_gen_train_step_async(WubuB200Gen* gen, unsigned long long noise_stream);
/* The model's CUDA stream (cudaStream_t) for timing with events. */
void* wubu_b200_gen_stream(WubuB200Gen* gen);
/* Host synchronisation + device error word check. */
int wubu_b200_gen_sync(WubuB200Gen* gen);

/* Kernel launches in one captured step (the graph's kernel nodes); -1 before the first step. */
int wubu_b200_gen_graph_kernels(WubuB200Gen* gen);

/* Times `iters` back-to-back launches of one convolution of the step with CUDA events on the
 * model stream.  which: 0 = forward conv1 of the first dilation pair of the largest-k stack of
 * stage `stage` (fp16 operand pairs), 1 = its input-gradient conv, 2 = its weight gradient, 3 = the
 * pair's forward conv2 (residual epilogue), 4 = conv2's input-gradient conv, 5 = the stage's
 * ConvTranspose forward, 6 = its input gradient, 7 = its weight gradient, 8 = conv_pre's forward
 * (stage ignored), 9 = conv2's weight gradient.  Under fp32 precision a weight gradient times its
 * first launch (one of three).  Returns the mean launch time (ms) and the algorithmic FLOPs of one
 * launch (2*MACs of the convolution, not counting split terms). */
int wubu_b200_gen_kernel_bench(WubuB200Gen* gen, int which, int stage, int iters, float* ms_per_launch,
                               double* flops_per_launch);

/* Data parallelism: one process per GPU.  Rank 0 creates the 128-byte NCCL unique id and the
 * caller ships it to the other ranks; every rank then attaches it.  Gradients are summed
 * over ranks in buckets on a communication stream while the backward runs, then scaled 1/world. */
int wubu_b200_nccl_unique_id(void* out128);
int wubu_b200_gen_attach_comm(WubuB200Gen* gen, int rank, int world, const void* id128);
/* A step's collectives must finish within `ms` (default 60000) of the call that waits for them
 * (train_step, sync, ...).  Past it, or on an NCCL error, the communicator is aborted (ending the
 * collectives that wait on a lost peer), the call returns WUBU_B200_ERR_COMM and the context runs no
 * further step.  Needs an attached communicator. */
int wubu_b200_gen_set_comm_timeout_ms(WubuB200Gen* gen, int ms);

/* ---------------------------------------------------------------------------------------------
 * 3. The GAN discriminators of RVC training (wubu_b200_disc_*): MultiPeriodDiscriminator =
 *    DiscriminatorS + one DiscriminatorP per period (knowledge/rvc_original/infer/module/
 *    models.py:928-1094), weight-normed, with discriminator_loss / generator_loss / feature_loss
 *    (train/losses.py:4-40) and torch.optim.AdamW, in the step order of train/train.py:500-525:
 *      wubu_b200_disc_step      forward on (real, generated detached), discriminator loss, every
 *                               parameter gradient, AdamW
 *      wubu_b200_disc_gen_loss  forward through the (updated) discriminators, generator_loss +
 *                               feature_loss (real feature maps detached) and dL/dy_hat, which the
 *                               generator takes as its dldy
 *    fp32 throughout.  periods = NULL or n_periods = 0: [2, 3, 5, 7, 11, 17] (V2 passes
 *    {2, 3, 5, 7, 11, 17, 23, 37}).  Parameters: one flat fp32 buffer in upstream's state_dict
 *    order, per convolution bias [C_out], weight_g [C_out], weight_v [C_out][C_in/groups][k].
 * ------------------------------------------------------------------------------------------- */
typedef struct WubuB200Disc WubuB200Disc;
#define WUBU_B200_DISC_DEVICE 1    /* y, y_hat (and dldy_hat) are device pointers; no host sync */
#define WUBU_B200_DISC_NO_UPDATE 2 /* wubu_b200_disc_step: gradients only, no AdamW step */
int wubu_b200_disc_param_count(const int* periods, int n_periods);       /* tensors */
long long wubu_b200_disc_param_total(const int* periods, int n_periods); /* floats */
int wubu_b200_disc_param_info(const int* periods, int n_periods, int index, char* name, int name_cap, int* shape3,
                              long long* offset);
/* B items of T samples per call; stream = NULL: the context makes its own. */
WubuB200Disc* wubu_b200_disc_create(int B, int T, const int* periods, int n_periods, void* stream);
void wubu_b200_disc_destroy(WubuB200Disc* d);
long long wubu_b200_disc_n_params(const WubuB200Disc* d);
int wubu_b200_disc_set_params(WubuB200Disc* d, const float* host_flat);
int wubu_b200_disc_get_params(WubuB200Disc* d, float* host_flat);
int wubu_b200_disc_get_grads(WubuB200Disc* d, float* host_flat);
/* torch.optim.AdamW hyper-parameters; default lr 1e-4, betas (0.8, 0.99), eps 1e-9 (the RVC
 * training configs), weight decay 0.01 (torch's default). */
int wubu_b200_disc_set_adamw(WubuB200Disc* d, float lr, float b1, float b2, float eps, float wd);
/* y, y_hat: [B][T] fp32.  loss_d (host, may be NULL with WUBU_B200_DISC_DEVICE: then the call
 * returns without synchronising) receives discriminator_loss. */
int wubu_b200_disc_step(WubuB200Disc* d, const float* y, const float* y_hat, int flags, float* loss_d);
/* dldy_hat [B][T] receives d(generator_loss + feature_loss)/d y_hat; losses2 (host, may be NULL
 * as above) receives {generator_loss, feature_loss}. */
int wubu_b200_disc_gen_loss(WubuB200Disc* d, const float* y, const float* y_hat, float* dldy_hat, int flags,
                            float* losses2);
void* wubu_b200_disc_stream(WubuB200Disc* d);
int wubu_b200_disc_sync(WubuB200Disc* d);
int wubu_b200_disc_launches(const WubuB200Disc* d); /* kernels the last step / gen_loss call launched */
/* Data parallelism (torch DDP's semantics): after attaching, wubu_b200_disc_step all-reduces the
 * gradient over NCCL on the context's stream and divides it by world before AdamW, so every rank
 * holds the mean gradient over all ranks' items and takes the same step.  id128 from
 * wubu_b200_nccl_unique_id on one rank, shipped to the others.  Host waits of an attached context
 * are bounded by the comm timeout (default 60 s): past it, or on an NCCL error, the communicator is
 * aborted and the call returns WUBU_B200_ERR_COMM (the context takes no further step). */
int wubu_b200_disc_attach_comm(WubuB200Disc* d, int rank, int world, const void* id128);
int wubu_b200_disc_set_comm_timeout_ms(WubuB200Disc* d, int ms);

#ifdef __cplusplus
}
#endif

#endif /* WUBURVC_B200_H */
