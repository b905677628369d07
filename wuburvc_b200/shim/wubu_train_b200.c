/* wubu_train_b200.c — binds src/wubu_train.h's CUDA entry points to libwuburvc_b200.so */
#include "wubu_train.h"
#include "wuburvc_b200.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>

struct TrainCacheCuda { WubuB200Gen *gen; int frames; float *flat; long long total; };

static WubuB200GenConfig decoder_config(const WuBuRVCModel *m) {
  WubuB200GenConfig c = {0};
  c.sample_rate = 40000; c.n_ups = 4; c.initial_channel = 512; c.in_channels = 192;
  for (int L = 0; L < 4; L++) { c.upsample_rates[L] = m->upsample_rates[L]; c.upsample_kernels[L] = m->upsample_kernel_sizes[L]; }
  c.n_kernels = 3; c.n_dilations = 3;
  int k[3] = {3, 7, 11};
  for (int j = 0; j < 3; j++) { c.resblock_kernels[j] = k[j]; for (int p = 0; p < 3; p++) c.resblock_dilations[j][p] = 1 + 2 * p; }
  c.lrelu_slope = 0.1f; c.final_slope = 0.1f;           /* src/wubu_train.c:605-620 */
  c.gin_channels = 0; c.nsf = 0; c.weight_norm = 0;     /* the reference trains the decoder only */
  return c;
}

TrainCacheCuda *wubu_train_cache_alloc_cuda(void) { return calloc(1, sizeof(TrainCacheCuda)); }
void wubu_train_cache_free_cuda(TrainCacheCuda *c) { if (c) { wubu_b200_gen_destroy(c->gen); free(c->flat); free(c); } }

/* registry <-> flat buffer, by name */
static void sync_params(TrainCacheCuda *c, WuBuTrainRegistry *reg, const WubuB200GenConfig *cfg, int to_dev) {
  char name[160]; int shape[3]; long long off, n;
  int np = wubu_b200_gen_param_count(cfg);
  if (!to_dev) wubu_b200_gen_get_params(c->gen, c->flat);
  for (int i = 0; i < np; i++) {
    wubu_b200_gen_param_info(cfg, i, name, sizeof name, shape, &off, &n);
    int r = wubu_train_registry_find(reg, name);
    if (r < 0) continue;
    if (to_dev) memcpy(c->flat + off, reg->params[r].data, n * sizeof(float));
    else memcpy(reg->params[r].data, c->flat + off, n * sizeof(float));
  }
  if (to_dev) wubu_b200_gen_set_params(c->gen, c->flat);
}

int wubu_train_step_cuda(WuBuRVCModel *model, WuBuTrainRegistry *reg, WuBuAdamW *opt,
                         const float *mel_in, int n_frames, const float *wav, int n_samples,
                         float *loss_out, int epoch) {
  /* One context per process, like g_wcache.  Weights and AdamW state stay on the device between
   * calls with the same frame count and are written back to the registry after every step; a host
   * that edits the registry's weights in between must free the context (or change n_frames) so the
   * next call reloads them.  WuBuAdamW is opaque to this file: the hyper-parameters are the ones
   * every reference caller creates it with (lr 1e-3, betas 0.9 / 0.999, eps 1e-8, weight decay
   * 0.01; src/tt_train_demo.c:68, src/test_train_cuda.c:131). */
  static TrainCacheCuda *c;
  WubuB200GenConfig cfg = decoder_config(model);
  (void)opt; (void)epoch;
  if (!c || c->frames != n_frames) {
    if (c) wubu_train_cache_free_cuda(c);
    c = wubu_train_cache_alloc_cuda();
    WubuB200TrainOptions o = {1, n_frames, 0, 1e-3f, 0.9f, 0.999f, 1e-8f, 1e-2f, 0};
    c->gen = wubu_b200_gen_create(&cfg, &o);
    c->frames = n_frames;
    c->total = wubu_b200_gen_param_total(&cfg);
    c->flat = calloc(c->total, sizeof(float));
    if (!c->gen) return -1;
    sync_params(c, reg, &cfg, 1);
  }
  int T = wubu_b200_gen_samples(c->gen);
  float *audio = malloc(T * sizeof(float)), *d = malloc(T * sizeof(float));
  float *zero = calloc(T, sizeof(float));
  wubu_b200_gen_upload(c->gen, mel_in, NULL, NULL, NULL, zero);
  wubu_b200_gen_forward(c->gen, 0, audio);
  int n = n_samples < T ? n_samples : T;
  float mse = wubu_mse_loss(audio, wav, n);
  /* the reference step's spectral term (src/wubu_train.c:1151-1176), its gradient taken on the GPU:
   * weight WUBU_SPECTRAL_WEIGHT (default 1), rescaled to half the MSE gradient's RMS */
  float weight = getenv("WUBU_SPECTRAL_WEIGHT") ? (float)atof(getenv("WUBU_SPECTRAL_WEIGHT")) : 1.0f;
  float spec = 0.0f, *ds = NULL;
  if (weight > 0.0f && n > 128 && (ds = malloc(n * sizeof(float))) != NULL) {
    if (wubu_b200_stft_loss_grad_host(audio, wav, 1, n, 3, ds, &spec) == 0) {
      float ss = 0.0f;
      for (int i = 0; i < n; i++) ss += ds[i] * ds[i];
      float rms = sqrtf(ss / (float)n);
      float k = (rms > 1e-9f && mse > 1e-12f) ? weight * 0.5f * (2.0f / (float)n) * sqrtf(mse) / rms : 0.0f;
      for (int i = 0; i < n; i++) ds[i] *= k;
    } else {
      free(ds); ds = NULL; spec = 0.0f;
    }
  }
  float total = mse + spec;
  for (int i = 0; i < T; i++) d[i] = i < n ? 2.f * (audio[i] - wav[i]) / (float)n + (ds ? ds[i] : 0.f) : 0.f;
  wubu_b200_gen_upload(c->gen, mel_in, NULL, NULL, NULL, d);
  int rc = wubu_b200_gen_backward(c->gen) || wubu_b200_gen_adamw(c->gen);
  sync_params(c, reg, &cfg, 0);             /* weights back on the host: synthesis-ready */
  if (loss_out) *loss_out = total;
  model->last_loss = total;
  free(audio); free(d); free(zero); free(ds);
  return rc ? -1 : (total < 0.1f ? 1 : 0);
}
