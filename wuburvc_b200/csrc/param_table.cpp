// param_table.cpp — parameter table and deterministic initialisation (host only).
#include "param_table.h"

#include <cmath>
#include <cstring>

namespace wb {

bool config_valid(const WubuB200GenConfig& c) {
  if (c.n_ups != 4 || c.n_kernels < 1 || c.n_kernels > 3 || c.n_dilations < 1 || c.n_dilations > 3) return false;
  if (c.initial_channel != 512 || c.in_channels < 32 || c.in_channels % 32) return false;
  if (c.gin_channels < 0 || c.harmonic_num < 0 || c.harmonic_num > 8) return false;
  for (int L = 0; L < 4; ++L) {
    const int u = c.upsample_rates[L], k = c.upsample_kernels[L];
    if (u < 1 || u > 12 || k < u || (k - u) % 2 || (k - u) / 2 >= u) return false;
  }
  for (int j = 0; j < c.n_kernels; ++j) {
    const int k = c.resblock_kernels[j];
    if (k < 1 || k > 11 || k % 2 == 0) return false;
    for (int p = 0; p < c.n_dilations; ++p)
      if (c.resblock_dilations[j][p] < 1) return false;
  }
  return c.activation == 0 || c.activation == 1;
}

static int noise_kernel(const WubuB200GenConfig& c, int L) {
  if (L + 1 >= c.n_ups) return 1;
  int s = 1;
  for (int i = L + 1; i < c.n_ups; ++i) s *= c.upsample_rates[i];
  return 2 * s;
}

ParamTable build_param_table(const WubuB200GenConfig& c) {
  ParamTable t;
  auto add = [&](const std::string& name, int kind, int d0, int d1, int d2) {
    ParamEntry p;
    p.name = name;
    p.kind = kind;
    p.shape[0] = d0; p.shape[1] = d1; p.shape[2] = d2;
    p.n = (long long)d0 * d1 * d2;
    p.off = t.total;
    t.total += (p.n + 63) / 64 * 64;
    // GEMM-fed convolutions are stored tap-major on the device
    const bool ups = name.rfind("dec.ups.", 0) == 0;
    const bool gemm_conv = name.rfind("dec.resblocks.", 0) == 0 || name == "dec.conv_pre.weight";
    if (kind == P_CONVT_W || (kind == P_WN_V && ups)) p.internal = 2;
    else if ((kind == P_CONV_W || kind == P_WN_V) && gemm_conv) p.internal = 1;
    t.e.push_back(p);
  };
  const bool snake = c.activation == 1;
  const int C0 = c.initial_channel;
  const int Clast = C0 >> c.n_ups;
  // backward-completion order: conv_post, stages 3..0, conv_pre, cond, source
  add("dec.conv_post.weight", P_CONV_W, 1, Clast, 7);
  if (snake) add("dec.post_act.alpha", P_ALPHA, Clast, 1, 1);
  for (int L = c.n_ups - 1; L >= 0; --L) {
    const int C = C0 >> (L + 1);
    for (int j = 0; j < c.n_kernels; ++j) {
      const int R = L * c.n_kernels + j, kk = c.resblock_kernels[j];
      for (int cp = c.n_dilations - 1; cp >= 0; --cp)
        for (int ct = 2; ct >= 1; --ct) {
          const std::string base = "dec.resblocks." + std::to_string(R) + ".convs" + std::to_string(ct) + "." +
                                   std::to_string(cp);
          if (c.weight_norm) {
            add(base + ".weight_g", P_WN_G, C, 1, 1);
            add(base + ".weight_v", P_WN_V, C, C, kk);
          } else {
            add(base + ".weight_v", P_CONV_W, C, C, kk);
          }
          add(base + ".bias", P_BIAS, C, 1, 1);
          if (snake)
            add("dec.resblocks." + std::to_string(R) + ".alpha" + std::to_string(ct) + "." + std::to_string(cp),
                P_ALPHA, C, 1, 1);
        }
    }
    if (c.nsf) {
      add("dec.noise_convs." + std::to_string(L) + ".weight", P_CONV_W, C, 1, noise_kernel(c, L));
      add("dec.noise_convs." + std::to_string(L) + ".bias", P_BIAS, C, 1, 1);
    }
    const int Cin = C0 >> L;
    const std::string ub = "dec.ups." + std::to_string(L);
    if (c.weight_norm) {
      add(ub + ".weight_g", P_WN_G, Cin, 1, 1);
      add(ub + ".weight_v", P_WN_V, Cin, C, c.upsample_kernels[L]);
    } else {
      add(ub + ".weight", P_CONVT_W, Cin, C, c.upsample_kernels[L]);
    }
    add(ub + ".bias", P_BIAS, C, 1, 1);
    if (snake) add("dec.ups_act." + std::to_string(L) + ".alpha", P_ALPHA, Cin, 1, 1);
  }
  add("dec.conv_pre.weight", P_CONV_W, C0, c.in_channels, 7);
  add("dec.conv_pre.bias", P_BIAS, C0, 1, 1);
  if (c.gin_channels > 0) {
    add("dec.cond.weight", P_CONV_W, C0, c.gin_channels, 1);
    add("dec.cond.bias", P_BIAS, C0, 1, 1);
  }
  if (c.nsf) {
    add("dec.m_source.l_linear.weight", P_LIN_W, 1, c.harmonic_num + 1, 1);
    add("dec.m_source.l_linear.bias", P_LIN_B, 1, 1, 1);
  }
  return t;
}

void to_internal(const ParamEntry& p, const float* ref, float* dev) {
  const int d0 = p.shape[0], d1 = p.shape[1], k = p.shape[2];
  if (p.internal == 0) {
    memcpy(dev, ref, sizeof(float) * (size_t)p.n);
  } else if (p.internal == 1) {  // ref [Co][Ci][k] -> [k][Co][Ci]
    for (int o = 0; o < d0; ++o)
      for (int i = 0; i < d1; ++i)
        for (int t = 0; t < k; ++t) dev[((size_t)t * d0 + o) * d1 + i] = ref[((size_t)o * d1 + i) * k + t];
  } else {  // ref [Ci][Co][k] -> [k][Co][Ci]
    for (int i = 0; i < d0; ++i)
      for (int o = 0; o < d1; ++o)
        for (int t = 0; t < k; ++t) dev[((size_t)t * d1 + o) * d0 + i] = ref[((size_t)i * d1 + o) * k + t];
  }
}

void to_reference(const ParamEntry& p, const float* dev, float* ref) {
  const int d0 = p.shape[0], d1 = p.shape[1], k = p.shape[2];
  if (p.internal == 0) {
    memcpy(ref, dev, sizeof(float) * (size_t)p.n);
  } else if (p.internal == 1) {
    for (int o = 0; o < d0; ++o)
      for (int i = 0; i < d1; ++i)
        for (int t = 0; t < k; ++t) ref[((size_t)o * d1 + i) * k + t] = dev[((size_t)t * d0 + o) * d1 + i];
  } else {
    for (int i = 0; i < d0; ++i)
      for (int o = 0; o < d1; ++o)
        for (int t = 0; t < k; ++t) ref[((size_t)i * d1 + o) * k + t] = dev[((size_t)t * d1 + o) * d0 + i];
  }
}

// counter-based generator shared with the device source-noise generator (splitmix64 finaliser)
static unsigned long long mix64(unsigned long long x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
static void counter_u2(unsigned long long seed, unsigned long long stream, unsigned long long idx, double& u1,
                       double& u2) {
  const unsigned long long key = mix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull);
  const unsigned long long h = mix64(key ^ (idx * 0x9E3779B97F4A7C15ull));
  u1 = (double)((h >> 40) + 1ull) / 16777216.0;
  u2 = (double)(((h >> 8) & 0xFFFFFFull) + 1ull) / 16777216.0;
}

void init_params(const WubuB200GenConfig& c, const ParamTable& t, unsigned long long seed, float* flat) {
  (void)c;
  memset(flat, 0, sizeof(float) * (size_t)t.total);
  const double two_pi = 6.283185307179586476925286766559;
  for (size_t i = 0; i < t.e.size(); ++i) {
    const ParamEntry& p = t.e[i];
    float* d = flat + p.off;
    const unsigned long long stream = 1000ull + i;
    switch (p.kind) {
      case P_CONV_W:
      case P_CONVT_W:
      case P_WN_V:
        for (long long q = 0; q < p.n; ++q) {
          double u1, u2;
          counter_u2(seed, stream, (unsigned long long)q, u1, u2);
          d[q] = (float)(0.01 * std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2));
        }
        break;
      case P_ALPHA:
        for (long long q = 0; q < p.n; ++q) d[q] = 1.f;
        break;
      case P_LIN_W:
        for (long long q = 0; q < p.n; ++q) {
          double u1, u2;
          counter_u2(seed, stream, (unsigned long long)q, u1, u2);
          d[q] = (float)((2.0 * u1 - 1.0) / 3.0);
        }
        break;
      default:
        break;
    }
  }
  // g = ||v|| per dim-0 row (so W = v at init)
  for (size_t i = 0; i < t.e.size(); ++i) {
    const ParamEntry& p = t.e[i];
    if (p.kind != P_WN_G) continue;
    const std::string vn = p.name.substr(0, p.name.size() - 1) + "v";
    const int vi = t.find(vn);
    if (vi < 0) continue;
    const ParamEntry& v = t.e[vi];
    const long long per = v.n / v.shape[0];
    for (int r = 0; r < v.shape[0]; ++r) {
      double s = 0;
      for (long long q = 0; q < per; ++q) {
        const double x = flat[v.off + r * per + q];
        s += x * x;
      }
      flat[p.off + r] = (float)std::sqrt(s);
    }
  }
}

}  // namespace wb

using namespace wb;

extern "C" {

int wubu_b200_gen_param_count(const WubuB200GenConfig* cfg) {
  if (!cfg || !config_valid(*cfg)) return WUBU_B200_ERR_ARG;
  return (int)build_param_table(*cfg).e.size();
}

long long wubu_b200_gen_param_total(const WubuB200GenConfig* cfg) {
  if (!cfg || !config_valid(*cfg)) return WUBU_B200_ERR_ARG;
  return build_param_table(*cfg).total;
}

int wubu_b200_gen_param_info(const WubuB200GenConfig* cfg, int index, char* name, int name_cap, int* shape3,
                             long long* offset, long long* numel) {
  if (!cfg || !config_valid(*cfg)) return WUBU_B200_ERR_ARG;
  ParamTable t = build_param_table(*cfg);
  if (index < 0 || index >= (int)t.e.size()) return WUBU_B200_ERR_ARG;
  const ParamEntry& p = t.e[index];
  if (name && name_cap > 0) {
    strncpy(name, p.name.c_str(), (size_t)name_cap - 1);
    name[name_cap - 1] = 0;
  }
  if (shape3)
    for (int i = 0; i < 3; ++i) shape3[i] = p.shape[i];
  if (offset) *offset = p.off;
  if (numel) *numel = p.n;
  return p.kind;
}

int wubu_b200_gen_init_params(const WubuB200GenConfig* cfg, unsigned long long seed, float* host_flat) {
  if (!cfg || !host_flat || !config_valid(*cfg)) return WUBU_B200_ERR_ARG;
  ParamTable t = build_param_table(*cfg);
  init_params(*cfg, t, seed, host_flat);
  return WUBU_B200_OK;
}

}  // extern "C"
