/* wubu_train_b200.c — the reference's CUDA entry points on libwuburvc_b200.so.
 *
 * Drop-in replacement of src/wubu_train_cuda.cu (wubu_train_{forward,backward,step}_cuda and
 * wubu_train_cache_{alloc,free}_cuda, declared at src/wubu_train.h:92-104) and of the CUDA
 * generator wubu_generator_nsf_cuda (src/wubu_rvc_real.h:95, src/wubu_rvc_cuda.cu:280), built
 * against the reference's own headers and linked with its host objects (wubu_rvc_find_tensor,
 * wubu_adamw_step, wubu_train_registry_find / _zero_grads).
 *
 * Semantics kept from the reference:
 *   - weights live on the host: every training forward reads them from the model (RVCTensor data
 *     found by name, model->hifi_upsample_denorm[L] for the upsampling weights), as
 *     src/wubu_train_cuda.cu does, so a model trained here is synthesis-ready and edits between
 *     calls are seen;
 *   - the backward OVERWRITES reg->params[i].grad for every registry entry (the caller zeroes
 *     first, src/wubu_train_cuda.cu:854) and returns 0 or -1;
 *   - the step is forward -> MSE (+ the spectral term, WUBU_SPECTRAL_WEIGHT, default 1) ->
 *     backward -> the host AdamW of the caller's WuBuAdamW (wubu_adamw_step, the same call the
 *     reference makes at src/wubu_train_cuda.cu:861), sets model->last_loss / last_epoch, and
 *     returns 1 if the loss is below 0.1, 0 otherwise, -1 on error;
 *   - -1 and a message on stderr for every failure, NULL arguments included.
 * WUBU_B200_PRECISION=fp32 in the environment runs the library's fp32 mode (the reference's entry
 * points have no dtype argument).
 * The spectral gradient runs on the GPU (wubu_b200_stft_loss_grad_host, the same loss and gradient
 * as the reference's wubu_stft_loss_grad).  One generator context per TrainCacheCuda (the step keeps
 * its own, re-created when the frame count changes).  Not thread-safe, like the reference, except
 * wubu_generator_nsf_cuda, which serialises its callers.
 */
#include "wubu_train.h"
#include "wubu_rvc_real.h"
#include "wuburvc_b200.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

struct TrainCacheCuda {
  WubuB200Gen *gen;
  WubuB200GenConfig cfg;
  int frames;
  long long total;   /* floats in the flat parameter buffer */
  float *flat;       /* host staging of the flat parameter / gradient buffer */
  float *audio;      /* the last forward's output */
  float *zeros;      /* zero source noise (inference without noise injection) */
  int n_out;
  int have_forward;
  int precision;                   /* WUBU_B200_PRECISION_* of the context */
  int forward_only;                /* inference mode of the context (wubu_generator_nsf_cuda): 0 none,
                                    * 1 exact, 2 fast (single fp16 operands) */
  const WuBuRVCModel *model;       /* inference cache: the model whose weights are on the device ... */
  unsigned long long fingerprint;  /* ... and a fingerprint of them */
};

static int fail(const char *what) {
  fprintf(stderr, "wubu_train_b200: %s\n", what);
  return -1;
}

/* ---- model -> generator config and flat parameters ------------------------------------------ */

/* Generator topology of a reference model.  full = 0: the decoder the reference trainer trains
 * (src/wubu_train_cuda.cu:8-10: no cond, sine source or noise convs, LeakyReLU 0.1 everywhere);
 * full = 1: the whole GeneratorNSF of the reference's inference (src/wubu_rvc_real.c:1302-1900). */
static int model_config(const WuBuRVCModel *m, int full, int with_g, int use_snake, WubuB200GenConfig *c) {
  memset(c, 0, sizeof(*c));
  const RVCTensor *pre = wubu_rvc_find_tensor((WuBuRVCModel *)m, "dec.conv_pre.weight");
  if (!pre || !pre->data || pre->n_dims < 3) return fail("model has no dec.conv_pre.weight");
  c->initial_channel = pre->dims[0];
  c->in_channels = pre->dims[1];
  c->sample_rate = m->sample_rate > 0 ? m->sample_rate : 40000;
  c->n_ups = 4;
  if (m->n_upsample_layers > 0 && m->n_upsample_layers != 4) return fail("only 4 upsampling layers are supported");
  static const int def_k[4] = {16, 16, 4, 4};
  for (int L = 0; L < 4; L++) {
    const int cin = c->initial_channel >> L, cout = c->initial_channel >> (L + 1);
    c->upsample_rates[L] = m->upsample_rates[L] > 0 ? m->upsample_rates[L] : 10;
    /* kernel size from the de-normalised weight itself, as the reference's inference takes it from
     * the weight shape (src/wubu_rvc_real.c:1357-1371) */
    int k = m->hifi_upsample_denorm_len[L] > 0 ? m->hifi_upsample_denorm_len[L] / (cin * cout) : 0;
    if (k <= 0) k = m->upsample_kernel_sizes[L] > 0 ? m->upsample_kernel_sizes[L] : def_k[L];
    c->upsample_kernels[L] = k;
  }
  const int ns = m->n_mrf_stacks > 0 ? m->n_mrf_stacks : 3, np = m->n_resblock_pairs > 0 ? m->n_resblock_pairs : 3;
  if (ns != 3 || np != 3) return fail("only 3 resblock stacks of 3 conv pairs are supported");
  c->n_kernels = 3;
  c->n_dilations = 3;
  static const int def_rk[3] = {3, 7, 11};
  for (int j = 0; j < 3; j++) {
    c->resblock_kernels[j] = m->resblock_k[j] > 0 ? m->resblock_k[j] : def_rk[j];
    for (int p = 0; p < 3; p++)
      c->resblock_dilations[j][p] = m->resblock_dil[j][p] > 0 ? m->resblock_dil[j][p] : 1 + 2 * p;
  }
  c->lrelu_slope = 0.1f;
  c->final_slope = 0.1f; /* src/wubu_train.c:913; the inference's final lrelu_c(.., 0.1f) */
  c->weight_norm = 0;    /* the model holds de-normalised weights (src/wubu_train.c:131-210) */
  c->sine_amp = 0.1f;
  c->noise_std = 0.003f;
  if (full) {
    const RVCTensor *cond = wubu_rvc_find_tensor((WuBuRVCModel *)m, "dec.cond.weight");
    c->gin_channels = (with_g && cond && cond->data) ? cond->dims[1] : 0;
    const RVCTensor *lw = wubu_rvc_find_tensor((WuBuRVCModel *)m, "dec.m_source.l_linear.weight");
    if (!lw || !lw->data) return fail("model has no dec.m_source.l_linear.weight");
    c->nsf = 1;
    c->harmonic_num = (lw->n_dims >= 2 ? lw->dims[1] : 1) - 1;
    c->activation = use_snake ? 1 : 0;
  }
  return 0;
}

/* the model's array for one of the library's parameter names, or NULL */
static const float *model_array(const WuBuRVCModel *m, const char *name, long long n) {
  int L;
  char tail[16];
  if (sscanf(name, "dec.ups.%d.%15s", &L, tail) == 2 && strcmp(tail, "weight") == 0 && L >= 0 && L < 4)
    return m->hifi_upsample_denorm[L] && m->hifi_upsample_denorm_len[L] == n ? m->hifi_upsample_denorm[L] : NULL;
  const RVCTensor *t = wubu_rvc_find_tensor((WuBuRVCModel *)m, name);
  if (!t || !t->data) return NULL;
  long long tn = 1;
  for (int d = 0; d < t->n_dims; d++) tn *= t->dims[d];
  return tn == n ? t->data : NULL;
}

/* Gathers the model's weights into c->flat in the library's parameter order (copy = 1), or only
 * checks that they exist (copy = 0).  Biases and Snake alphas the model does not carry are 0 and 1
 * (the reference treats a missing bias as none and runs Snake with alpha 1); a missing weight is an
 * error.  *fp receives a fingerprint of the weights (their addresses and three sampled values each),
 * which tells the inference path whether the device copy is still current. */
static int gather_params(TrainCacheCuda *c, const WuBuRVCModel *m, int copy, unsigned long long *fp) {
  char name[160];
  int shape[3];
  long long off, n;
  unsigned long long h = 1469598103934665603ull;
  const int np = wubu_b200_gen_param_count(&c->cfg);
  if (np <= 0) return fail("invalid generator config");
  for (int i = 0; i < np; i++) {
    if (wubu_b200_gen_param_info(&c->cfg, i, name, sizeof name, shape, &off, &n) < 0) return fail("param table");
    const float *src = model_array(m, name, n);
    const size_t len = strlen(name);
    if (src) {
      if (copy) memcpy(c->flat + off, src, (size_t)n * sizeof(float));
      unsigned int bits[3];
      const float probe[3] = {src[0], src[n / 2], src[n - 1]};
      memcpy(bits, probe, sizeof bits);
      h = (h ^ (unsigned long long)(size_t)src) * 1099511628211ull;
      for (int b = 0; b < 3; b++) h = (h ^ bits[b]) * 1099511628211ull;
    } else if (len > 5 && strcmp(name + len - 5, ".bias") == 0) {
      if (copy) memset(c->flat + off, 0, (size_t)n * sizeof(float));
    } else if (len > 6 && strcmp(name + len - 6, ".alpha") == 0) {
      if (copy)
        for (long long j = 0; j < n; j++) c->flat[off + j] = 1.0f;
    } else {
      fprintf(stderr, "wubu_train_b200: model has no tensor %s of %lld floats\n", name, n);
      return -1;
    }
  }
  /* the library's conv_post has no bias (upstream GeneratorNSF, models.py:467); a model carrying a
   * non-zero one cannot be represented */
  const RVCTensor *pb = wubu_rvc_find_tensor((WuBuRVCModel *)m, "dec.conv_post.bias");
  if (pb && pb->data && pb->dims[0] > 0 && pb->data[0] != 0.0f) return fail("a non-zero dec.conv_post.bias is not supported");
  if (fp) *fp = h;
  return 0;
}

/* (re)creates the cache's generator for this config and frame count */
/* The reference's entry points carry no arithmetic type: WUBU_B200_PRECISION=fp32 selects the
 * library's fp32 mode (bf16 hi + lo backward operands), anything else the default bf16 mode. */
static int shim_precision(void) {
  const char *p = getenv("WUBU_B200_PRECISION");
  return (p && strcmp(p, "fp32") == 0) ? WUBU_B200_PRECISION_FP32 : WUBU_B200_PRECISION_BF16;
}

static int ensure_gen(TrainCacheCuda *c, const WubuB200GenConfig *cfg, int frames) {
  const int precision = shim_precision();
  if (c->gen && c->frames == frames && c->precision == precision && memcmp(&c->cfg, cfg, sizeof *cfg) == 0)
    return 0;
  wubu_b200_gen_destroy(c->gen);
  free(c->flat);
  free(c->audio);
  free(c->zeros);
  c->gen = NULL;
  c->flat = c->audio = c->zeros = NULL;
  c->frames = 0;
  c->have_forward = 0;
  c->forward_only = 0;
  c->model = NULL;
  WubuB200TrainOptions o;
  memset(&o, 0, sizeof o);
  o.batch = 1;
  o.frames = frames;
  o.lr = 1e-3f; /* unused: the step runs the caller's host AdamW */
  o.beta1 = 0.9f;
  o.beta2 = 0.999f;
  o.eps = 1e-8f;
  o.precision = precision;
  c->gen = wubu_b200_gen_create(cfg, &o);
  if (!c->gen) return fail("wubu_b200_gen_create failed (no sm_100 GPU, unsupported shape or out of memory)");
  c->cfg = *cfg;
  c->total = wubu_b200_gen_param_total(cfg);
  const int T = wubu_b200_gen_samples(c->gen);
  c->flat = (float *)malloc((size_t)(c->total > 0 ? c->total : 1) * sizeof(float));
  c->audio = (float *)malloc((size_t)(T > 0 ? T : 1) * sizeof(float));
  if (c->total <= 0 || T <= 0 || !c->flat || !c->audio) {
    wubu_b200_gen_destroy(c->gen);
    c->gen = NULL;
    return fail("out of host memory");
  }
  c->n_out = T;
  c->frames = frames;
  c->precision = precision;
  return 0;
}

/* ---- the reference's training entry points ----------------------------------------------------- */

TrainCacheCuda *wubu_train_cache_alloc_cuda(void) { return (TrainCacheCuda *)calloc(1, sizeof(TrainCacheCuda)); }

void wubu_train_cache_free_cuda(TrainCacheCuda *c) {
  if (!c) return;
  wubu_b200_gen_destroy(c->gen);
  free(c->flat);
  free(c->audio);
  free(c->zeros);
  free(c);
}

int wubu_train_forward_cuda(WuBuRVCModel *model, const float *mel_in, int n_frames, float *audio, int max_samples,
                            TrainCacheCuda *cache) {
  if (!model || !mel_in || !audio || !cache || n_frames < 1) return fail("forward: bad argument");
  cache->have_forward = 0;
  WubuB200GenConfig cfg;
  if (model_config(model, 0, 0, 0, &cfg) != 0 || ensure_gen(cache, &cfg, n_frames) != 0) return -1;
  if (cache->n_out > max_samples) return fail("forward: max_samples is smaller than the output");
  if (gather_params(cache, model, 1, NULL) != 0) return -1;
  if (wubu_b200_gen_set_params(cache->gen, cache->flat) != 0) return fail("forward: weight upload failed");
  if (wubu_b200_gen_upload(cache->gen, mel_in, NULL, NULL, NULL, NULL) != 0) return fail("forward: input upload failed");
  if (wubu_b200_gen_forward(cache->gen, 0, cache->audio) != 0) return fail("forward failed");
  memcpy(audio, cache->audio, (size_t)cache->n_out * sizeof(float));
  cache->have_forward = 1;
  return cache->n_out;
}

int wubu_train_backward_cuda(WuBuRVCModel *model, TrainCacheCuda *cache, const float *mel_in, const float *d_audio,
                             WuBuTrainRegistry *reg) {
  if (!model || !cache || !mel_in || !d_audio || !reg) return fail("backward: bad argument");
  if (!cache->gen || !cache->have_forward) return fail("backward: no forward in this cache");
  if (wubu_b200_gen_upload(cache->gen, mel_in, NULL, NULL, NULL, d_audio) != 0) return fail("backward: upload failed");
  if (wubu_b200_gen_backward(cache->gen) != 0) return fail("backward failed");
  if (wubu_b200_gen_get_grads(cache->gen, cache->flat) != 0) return fail("backward: gradient download failed");
  char name[160];
  int shape[3];
  long long off, n;
  const int np = wubu_b200_gen_param_count(&cache->cfg);
  int matched = 0;
  for (int i = 0; i < np; i++) {
    if (wubu_b200_gen_param_info(&cache->cfg, i, name, sizeof name, shape, &off, &n) < 0) return fail("param table");
    const int r = wubu_train_registry_find(reg, name);
    if (r < 0) continue;
    if (!reg->params[r].grad || reg->params[r].n != n) return fail("backward: registry entry of another size");
    memcpy(reg->params[r].grad, cache->flat + off, (size_t)n * sizeof(float));
    matched++;
  }
  /* a (zero) conv_post bias in the registry: its gradient is the sum of dL/d(pre-tanh) */
  const int rb = wubu_train_registry_find(reg, "dec.conv_post.bias");
  if (rb >= 0 && reg->params[rb].grad && reg->params[rb].n == 1) {
    double s = 0.0;
    for (int t = 0; t < cache->n_out; t++) s += (double)d_audio[t] * (1.0 - (double)cache->audio[t] * cache->audio[t]);
    reg->params[rb].grad[0] = (float)s;
    matched++;
  }
  if (matched != reg->count) return fail("backward: the registry has entries the generator does not train");
  return 0;
}

int wubu_train_step_cuda(WuBuRVCModel *model, WuBuTrainRegistry *reg, WuBuAdamW *opt, const float *mel_in,
                         int n_frames, const float *wav, int n_samples, float *loss_out, int epoch) {
  /* one context for the process's steps (a context holds every device buffer and launch plan; the
   * reference re-allocates per step, src/wubu_train_cuda.cu:804-809) */
  static TrainCacheCuda *ctx;
  if (!model || !reg || !opt || !mel_in || !wav || n_frames < 1 || n_samples < 1) return fail("step: bad argument");
  if (!ctx && !(ctx = wubu_train_cache_alloc_cuda())) return fail("out of host memory");
  const int max_samples = n_frames * 480;
  float *audio = (float *)malloc((size_t)max_samples * sizeof(float));
  if (!audio) return fail("out of host memory");
  const int n_out = wubu_train_forward_cuda(model, mel_in, n_frames, audio, max_samples, ctx);
  if (n_out <= 0) {
    free(audio);
    return -1;
  }
  const int n = n_out < n_samples ? n_out : n_samples;
  /* MSE as the reference step forms it (src/wubu_train_cuda.cu:812-815) */
  float mse = 0.0f;
  for (int i = 0; i < n; i++) {
    const float e = audio[i] - wav[i];
    mse += e * e;
  }
  mse /= (float)n;
  /* the spectral term (src/wubu_train_cuda.cu:817-843), its gradient taken on the GPU */
  float weight = 1.0f;
  const char *sw = getenv("WUBU_SPECTRAL_WEIGHT");
  if (sw) weight = (float)atof(sw);
  float spec = 0.0f, *ds = NULL;
  if (weight > 0.0f && n > 128) {
    ds = (float *)malloc((size_t)n * sizeof(float));
    if (!ds) {
      free(audio);
      return fail("out of host memory");
    }
    if (wubu_b200_stft_loss_grad_host(audio, wav, 1, n, 3, ds, &spec) != 0) {
      free(ds);
      free(audio);
      return fail("step: spectral loss failed");
    }
    float g2 = 0.0f;
    for (int i = 0; i < n; i++) g2 += ds[i] * ds[i];
    g2 = sqrtf(g2 / (float)n);
    if (g2 > 1e-9f && mse > 1e-12f) {
      const float scale = weight * 0.5f * (2.0f / (float)n) * sqrtf(mse) / g2;
      for (int i = 0; i < n; i++) ds[i] *= scale;
    } else {
      for (int i = 0; i < n; i++) ds[i] = 0.0f;
    }
  }
  const float total = mse + spec;
  if (loss_out) *loss_out = total;
  model->last_loss = total;
  model->last_epoch = epoch;
  float *d = (float *)malloc((size_t)n_out * sizeof(float));
  if (!d) {
    free(ds);
    free(audio);
    return fail("out of host memory");
  }
  for (int i = 0; i < n; i++) d[i] = 2.0f * (audio[i] - wav[i]) / (float)n + (ds ? ds[i] : 0.0f);
  for (int i = n; i < n_out; i++) d[i] = 0.0f;
  wubu_train_registry_zero_grads(reg);
  const int rc = wubu_train_backward_cuda(model, ctx, mel_in, d, reg);
  free(d);
  free(ds);
  free(audio);
  if (rc != 0) return -1;
  /* AdamW on the host with the caller's optimiser state (src/wubu_train_cuda.cu:860-861) */
  for (int i = 0; i < reg->count; i++) wubu_adamw_step(opt, i, reg->params[i].data, reg->params[i].grad);
  return total < 0.1f ? 1 : 0;
}

/* ---- the reference's CUDA generator (inference) -------------------------------------------------- */

/* z [inter_channels][nF] (channel-major, as the reference passes it), nsff0 [nF] Hz (0 = unvoiced),
 * g [gin] speaker embedding (may be NULL: no cond), out_audio [max_samples].  inject_noise = 0 runs
 * the source without noise (deterministic); otherwise Gaussian source noise from the library's
 * generator (the reference draws it from the host rand()).  use_snake: Snake with alpha 1 in place
 * of LeakyReLU (src/wubu_rvc_real.c:676-685).  Returns the number of samples or -1.  One cached
 * context, as the reference keeps one weight cache (src/wubu_rvc_cuda.cu:228-276); the weights are
 * uploaded again when the model or a sample of its weights (three values per tensor) changes, so a
 * caller that edits single weights in place between calls must pass a fresh model. */
int wubu_generator_nsf_cuda(WuBuRVCModel *model, const float *z, int nF, int inter_channels, const float *nsff0,
                            const float *g, float *out_audio, int max_samples, int inject_noise, int use_snake) {
  static TrainCacheCuda *ctx;
  static unsigned long long calls;
  static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
  if (!model || !z || !nsff0 || !out_audio || nF < 1) return fail("generator: bad argument");
  pthread_mutex_lock(&mu);
  int rc = -1;
  WubuB200GenConfig cfg;
  unsigned long long fp = 0;
  const float *noise = NULL;
  if (!ctx && !(ctx = wubu_train_cache_alloc_cuda())) goto out;
  if (model_config(model, 1, g != NULL, use_snake, &cfg) != 0) goto out;
  if (cfg.in_channels != inter_channels) {
    fail("generator: inter_channels differs from dec.conv_pre.weight");
    goto out;
  }
  if (ensure_gen(ctx, &cfg, nF) != 0) goto out;
  {  /* inference: nothing the backward would read is written; WUBU_B200_INFERENCE=fast selects
      * single fp16 GEMM operands */
    const char *env = getenv("WUBU_B200_INFERENCE");
    const int mode = (env && strcmp(env, "fast") == 0) ? 2 : 1;
    if (ctx->forward_only != mode) {
      if (wubu_b200_gen_set_forward_only(ctx->gen, mode) != 0) {
        fail("generator: forward-only mode failed");
        goto out;
      }
      ctx->forward_only = mode;
    }
  }
  if (ctx->n_out > max_samples) {
    fail("generator: max_samples is smaller than the output");
    goto out;
  }
  if (gather_params(ctx, model, 0, &fp) != 0) goto out;
  if (ctx->model != model || ctx->fingerprint != fp) {
    if (gather_params(ctx, model, 1, NULL) != 0 || wubu_b200_gen_set_params(ctx->gen, ctx->flat) != 0) {
      fail("generator: weight upload failed");
      goto out;
    }
    ctx->model = model;
    ctx->fingerprint = fp;
  }
  if (!inject_noise) {
    const size_t nz = (size_t)ctx->n_out * (size_t)(cfg.harmonic_num + 1);
    if (!ctx->zeros && !(ctx->zeros = (float *)calloc(nz, sizeof(float)))) {
      fail("out of host memory");
      goto out;
    }
    noise = ctx->zeros;
  }
  if (wubu_b200_gen_upload(ctx->gen, z, nsff0, cfg.gin_channels ? g : NULL, noise, NULL) != 0 ||
      wubu_b200_gen_forward(ctx->gen, ++calls, out_audio) != 0) {
    fail("generator: forward failed");
    goto out;
  }
  rc = ctx->n_out;
out:
  pthread_mutex_unlock(&mu);
  return rc;
}
