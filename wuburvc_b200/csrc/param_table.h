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
  // Device storage order of the tensor: 0 = reference layout, 1 = Conv1d weight stored tap-major
  // [k][C_out][C_in], 2 = ConvTranspose1d weight stored tap-major [k][C_out][C_in].  Tap-major is the
  // order the weight-gradient GEMM produces; the host API converts at set/get.
  int internal = 0;
};

// reference layout <-> device storage layout of one tensor
void to_internal(const ParamEntry& p, const float* ref, float* dev);
void to_reference(const ParamEntry& p, const float* dev, float* ref);

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
