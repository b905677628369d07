/* ref_harness.c — TEST INFRASTRUCTURE ONLY (never linked into the product).
 *
 * Drives the reference CPU generator trainer, compiled from its own source
 * file src/wubu_train.c (included below, not copied), so the tests and the
 * bench's CPU arm can call the static decoder_forward / decoder_backward
 * with an injected upstream gradient dL/dy:
 *   - decoder_forward   src/wubu_train.c:789-939 (cached forward)
 *   - decoder_backward  src/wubu_train.c:955-1097
 *   - wubu_adamw_step   src/wubu_train.c:90-117
 *   - registry build    src/wubu_train.c:131-210 (parameter order/names)
 * The model struct is built in memory (no weight file): RVCTensor entries for
 * conv_pre / resblocks / conv_post and model->hifi_upsample_denorm[] for the
 * upsampling ConvTranspose weights, exactly what the reference trainer reads.
 *
 * Built by oracle/Makefile into oracle/_ref/libwubu_ref.so.
 */
#include "wubu_train.c"

#include <omp.h>

typedef struct {
    WuBuRVCModel *model;
    WuBuTrainRegistry reg;
    int reg_built;
    WuBuAdamW *opt;
    DecCache cache;
    int have_cache;
} RefH;

void *refh_create(int max_tensors) {
    RefH *h = (RefH *)calloc(1, sizeof(RefH));
    if (!h) return NULL;
    h->model = (WuBuRVCModel *)calloc(1, sizeof(WuBuRVCModel));
    if (!h->model) { free(h); return NULL; }
    h->model->tensors = (RVCTensor *)calloc((size_t)max_tensors, sizeof(RVCTensor));
    if (!h->model->tensors) { free(h->model); free(h); return NULL; }
    h->model->n_tensors = 0;
    return h;
}

/* Adds a named tensor (data copied). Returns its index or -1. */
int refh_add_tensor(void *hp, const char *name, const float *data, int n_dims, const int *dims) {
    RefH *h = (RefH *)hp;
    WuBuRVCModel *m = h->model;
    RVCTensor *t = &m->tensors[m->n_tensors];
    size_t n = 1;
    for (int d = 0; d < n_dims; d++) n *= (size_t)dims[d];
    snprintf(t->name, sizeof(t->name), "%s", name);
    t->data = (float *)malloc(n * sizeof(float));
    if (!t->data) return -1;
    memcpy(t->data, data, n * sizeof(float));
    t->n_dims = n_dims;
    for (int d = 0; d < 4; d++) t->dims[d] = d < n_dims ? dims[d] : 1;
    return m->n_tensors++;
}

/* ConvTranspose weight [C_in][C_out][k] (already de-normalised) for stage L. */
int refh_set_ups(void *hp, int L, const float *w, int n, int rate, int k) {
    RefH *h = (RefH *)hp;
    WuBuRVCModel *m = h->model;
    m->hifi_upsample_denorm[L] = (float *)malloc((size_t)n * sizeof(float));
    if (!m->hifi_upsample_denorm[L]) return -1;
    memcpy(m->hifi_upsample_denorm[L], w, (size_t)n * sizeof(float));
    m->hifi_upsample_denorm_len[L] = n;
    m->upsample_rates[L] = rate;
    m->upsample_kernel_sizes[L] = k;
    if (m->n_upsample_layers < L + 1) m->n_upsample_layers = L + 1;
    return 0;
}

/* Builds the training registry and the AdamW state. Returns the entry count. */
int refh_finalize(void *hp, float lr, float b1, float b2, float eps, float wd) {
    RefH *h = (RefH *)hp;
    h->model->loaded = 1;
    memset(&h->reg, 0, sizeof(h->reg));
    int n = wubu_train_registry_build(h->model, &h->reg);
    if (n <= 0) return -1;
    h->reg_built = 1;
    h->opt = wubu_adamw_create(n, lr, b1, b2, eps, wd);
    if (!h->opt) return -1;
    for (int i = 0; i < n; i++)
        if (wubu_adamw_init_param(h->opt, i, h->reg.params[i].n) != 0) return -1;
    return n;
}

int refh_reg_count(void *hp) { return ((RefH *)hp)->reg.count; }
const char *refh_reg_name(void *hp, int i) { return ((RefH *)hp)->reg.params[i].name; }
int refh_reg_size(void *hp, int i) { return ((RefH *)hp)->reg.params[i].n; }

/* Copies registry data (which=0) or grads (which=1) into a flat buffer in
 * registry order. Returns the number of floats written. */
long refh_reg_gather(void *hp, int which, float *out) {
    RefH *h = (RefH *)hp;
    long off = 0;
    for (int i = 0; i < h->reg.count; i++) {
        const float *src = which ? h->reg.params[i].grad : h->reg.params[i].data;
        memcpy(out + off, src, (size_t)h->reg.params[i].n * sizeof(float));
        off += h->reg.params[i].n;
    }
    return off;
}

/* Forward only (decoder_forward). Returns samples or -1. */
int refh_forward(void *hp, const float *mel, int n_frames, float *audio, int max_samples) {
    RefH *h = (RefH *)hp;
    if (h->have_cache) { decoder_cache_free(&h->cache); h->have_cache = 0; }
    memset(&h->cache, 0, sizeof(h->cache));
    int n = decoder_forward(h->model, mel, n_frames, audio, max_samples, &h->cache);
    if (n > 0) h->have_cache = 1;
    else decoder_cache_free(&h->cache);
    return n;
}

/* Backward from the cached forward with an explicit dL/d(audio); grads are
 * zeroed first, as in wubu_train_step (src/wubu_train.c:1195). */
int refh_backward(void *hp, const float *mel, const float *d_audio) {
    RefH *h = (RefH *)hp;
    if (!h->have_cache) return -1;
    wubu_train_registry_zero_grads(&h->reg);
    decoder_backward(h->model, &h->cache, mel, d_audio, &h->reg, NULL);
    return 0;
}

/* AdamW over every registry entry in order (src/wubu_train.c:1199-1200). */
int refh_adamw(void *hp) {
    RefH *h = (RefH *)hp;
    for (int i = 0; i < h->reg.count; i++)
        wubu_adamw_step(h->opt, i, h->reg.params[i].data, h->reg.params[i].grad);
    return 0;
}

/* Copies a flat buffer in registry order into the registry's gradients (for applying the
 * reference's own AdamW to gradients computed elsewhere).  Returns the number of floats read. */
long refh_reg_set_grads(void *hp, const float *in) {
  RefH *h = (RefH *)hp;
  long off = 0;
  for (int i = 0; i < h->reg.count; i++) {
    memcpy(h->reg.params[i].grad, in + off, (size_t)h->reg.params[i].n * sizeof(float));
    off += h->reg.params[i].n;
  }
  return off;
}

/* Model config field the reference's inference generator reads (src/wubu_rvc_real.c:1420). */
void refh_set_sample_rate(void *hp, int sr) { ((RefH *)hp)->model->sample_rate = sr; }

int refh_threads(void) { return omp_get_max_threads(); }
/* Thread count of the reference's OpenMP regions (its reductions, e.g. wubu_mse_loss, then run in a
 * fixed order when 1). */
void refh_set_threads(int n) { omp_set_num_threads(n); }

/* The reference's own objects, for a caller that drives the reference's public entry points
 * (e.g. wubu_train_step_cuda through a drop-in back-end) on this model. */
void *refh_model(void *hp) { return ((RefH *)hp)->model; }
void *refh_registry(void *hp) { return &((RefH *)hp)->reg; }
void *refh_optimizer(void *hp) { return ((RefH *)hp)->opt; }

void refh_free(void *hp) {
    RefH *h = (RefH *)hp;
    if (!h) return;
    if (h->have_cache) decoder_cache_free(&h->cache);
    if (h->opt) wubu_adamw_free(h->opt);
    if (h->reg_built) wubu_train_registry_free(&h->reg);
    for (int i = 0; i < h->model->n_tensors; i++) free(h->model->tensors[i].data);
    free(h->model->tensors);
    for (int L = 0; L < 4; L++) free(h->model->hifi_upsample_denorm[L]);
    free(h->model);
    free(h);
}
