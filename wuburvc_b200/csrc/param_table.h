// param_table.h — the generator's trainable tensors, their flat-buffer offsets and init.
#pragma once
#include <string>
#include <vector>

#include "../../include/wuburvc_b200.h"

namespace wb {

enum ParamKind { P_CONV_W = 0, P_CONVT_W, P_WN_G, P_WN_V, P_BIAS, P_ALPHA, P_LIN_W, P_LIN_B };

struct ParamEntry {
  std::string name;
  int kind;
  int shape[3];
  long long off, n;
};

struct ParamTable {
  std::vector<ParamEntry> e;
  long long total = 0;
  int find(const std::string& name) const {
    for (size_t i = 0; i < e.size(); ++i)
      if (e[i].name == name) return (int)i;
    return -1;
  }
};

bool config_valid(const WubuB200GenConfig& c);
ParamTable build_param_table(const WubuB200GenConfig& c);
void init_params(const WubuB200GenConfig& c, const ParamTable& t, unsigned long long seed, float* flat);

}  // namespace wb
