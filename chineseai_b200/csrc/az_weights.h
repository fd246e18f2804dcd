// az_weights.h - host weights of the AZ-NNUE evaluator, shared by the host
// code (az_host.cpp) and the device model (az.cu).
#pragma once

#include <vector>

#include "../../include/cnnue.h"

// The 22 fp32 tensors of az_weight_tensors! (src/az.rs:241-278) in that order,
// and the quantised tables the reference derives from them at load time
// (src/az.rs:2201-2342), indexed by CNNUE_AZ_Q_*.
struct cnnue_az_weights {
  int64_t hidden = 0;
  std::vector<float> t[CNNUE_AZ_TENSORS];
  std::vector<int8_t> q8[4];    // POLICY_FEATURE, POLICY_MOVE, POLICY_SPARSE, VALUE_THREAT
  std::vector<int32_t> q32[2];  // MOVED_DELTA, CAPTURE
  float scale[4] = {1.f, 1.f, 1.f, 1.f};
  int value_threat_active = 0;
  int policy_tactical_active = 0;
  // fill_policy_piece_square_scores (src/az.rs:2189-2199): input_hidden row
  // prefix . policy_consequence_output, one score per piece-square feature.
  std::vector<float> ps_scores;
};

namespace cnnue {
namespace az {
// Tensor positions in cnnue_az_weights::t.
enum Tensor {
  kInputHidden = 0,
  kInputPiece = 1,
  kInputRank = 2,
  kInputFile = 3,
  kInputKingPiece = 4,
  kRuleContext = 5,
  kHiddenBias = 6,
  kValueHeadHidden = 7,
  kValueHeadBias = 8,
  kValueHeadOutput = 9,
};
}  // namespace az
}  // namespace cnnue
