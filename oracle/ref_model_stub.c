/* ref_model_stub.c — TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * Stands in for the reference's model-file loader (wubu_rvc_load_model / wubu_rvc_load_weights /
 * wubu_rvc_model_free, src/wubu_rvc_parity.c) so the reference's own CUDA A/B program,
 * src/test_train_cuda.c, can be built unmodified against the drop-in shim and run without the
 * Windows-path .pth files it names.  The model is a seeded synthetic 40 kHz decoder laid out as the
 * reference's loader leaves a real one: RVCTensor entries named like the checkpoint
 * (dec.conv_pre.*, dec.ups.L.bias, dec.resblocks.R.convs{1,2}.P.{weight_v,bias} holding the
 * de-normalised weights, dec.conv_post.weight) and model->hifi_upsample_denorm[L] for the
 * upsampling weights (src/wubu_rvc_weights.c:141-191).  Weights ~ N(0, 0.01), biases 0.
 * Built by oracle/Makefile together with src/test_train_cuda.c into oracle/_ref/.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "wubu_rvc_parity.h"

static uint64_t g_lcg = 0x2545F4914F6CDD1Dull;

static float uniform01(void) {
  g_lcg = g_lcg * 6364136223846793005ull + 1442695040888963407ull;
  return ((float)(g_lcg >> 40) + 0.5f) / 16777216.0f;
}

static float normal(float std) {
  const float u1 = uniform01(), u2 = uniform01();
  return std * sqrtf(-2.0f * logf(u1)) * cosf(6.28318530718f * u2);
}

static float *filled(size_t n, float std) {
  float *p = (float *)malloc(n * sizeof(float));
  if (!p) return NULL;
  for (size_t i = 0; i < n; i++) p[i] = std > 0.0f ? normal(std) : 0.0f;
  return p;
}

static int add_tensor(WuBuRVCModel *m, const char *name, int nd, int d0, int d1, int d2, float std) {
  RVCTensor *t = &m->tensors[m->n_tensors];
  snprintf(t->name, sizeof(t->name), "%s", name);
  t->n_dims = nd;
  t->dims[0] = d0;
  t->dims[1] = nd > 1 ? d1 : 1;
  t->dims[2] = nd > 2 ? d2 : 1;
  t->dims[3] = 1;
  t->data = filled((size_t)d0 * (nd > 1 ? d1 : 1) * (nd > 2 ? d2 : 1), std);
  if (!t->data) return -1;
  m->n_tensors++;
  return 0;
}

WuBuRVCModel *wubu_rvc_load_model(const char *path) {
  (void)path;
  static const int rates[4] = {10, 10, 2, 2}, kers[4] = {16, 16, 4, 4}, rk[3] = {3, 7, 11};
  WuBuRVCModel *m = (WuBuRVCModel *)calloc(1, sizeof(WuBuRVCModel));
  if (!m) return NULL;
  m->tensors = (RVCTensor *)calloc(256, sizeof(RVCTensor));
  if (!m->tensors) {
    free(m);
    return NULL;
  }
  g_lcg = 0x2545F4914F6CDD1Dull;
  m->sample_rate = 40000;
  m->n_upsample_layers = 4;
  int rc = add_tensor(m, "dec.conv_pre.weight", 3, 512, 192, 7, 0.01f);
  rc |= add_tensor(m, "dec.conv_pre.bias", 1, 512, 0, 0, 0.0f);
  char name[128];
  for (int L = 0; L < 4; L++) {
    const int cin = 512 >> L, c = 512 >> (L + 1);
    m->upsample_rates[L] = rates[L];
    m->upsample_kernel_sizes[L] = kers[L];
    m->hifi_upsample_denorm_len[L] = cin * c * kers[L];
    m->hifi_upsample_denorm[L] = filled((size_t)m->hifi_upsample_denorm_len[L], 0.01f);
    if (!m->hifi_upsample_denorm[L]) rc = -1;
    snprintf(name, sizeof name, "dec.ups.%d.bias", L);
    rc |= add_tensor(m, name, 1, c, 0, 0, 0.0f);
    for (int j = 0; j < 3; j++)
      for (int ct = 1; ct <= 2; ct++)
        for (int p = 0; p < 3; p++) {
          snprintf(name, sizeof name, "dec.resblocks.%d.convs%d.%d.weight_v", L * 3 + j, ct, p);
          rc |= add_tensor(m, name, 3, c, c, rk[j], 0.01f);
          snprintf(name, sizeof name, "dec.resblocks.%d.convs%d.%d.bias", L * 3 + j, ct, p);
          rc |= add_tensor(m, name, 1, c, 0, 0, 0.0f);
        }
  }
  rc |= add_tensor(m, "dec.conv_post.weight", 3, 1, 32, 7, 0.01f);
  m->loaded = 1;
  if (rc) {
    wubu_rvc_model_free(m);
    return NULL;
  }
  return m;
}

int wubu_rvc_load_weights(WuBuRVCModel *model, const char *path) {
  (void)path;
  return model ? 0 : -1;
}

void wubu_rvc_model_free(WuBuRVCModel *m) {
  if (!m) return;
  for (int i = 0; i < m->n_tensors; i++) free(m->tensors[i].data);
  free(m->tensors);
  for (int L = 0; L < 4; L++) free(m->hifi_upsample_denorm[L]);
  free(m);
}
