// The RoPE inverse-frequency table of a model (decode_ctx.cu), shared by the
// single-sequence and batched contexts.
#pragma once

#include <vector>

#include "lcr_b200.h"

namespace lcrb {

// inv_freq[i] = theta^(-2i / head_dim) in double, llama3 band scaling when
// the model has it, rounded to float (src/config.cpp:223-259).
std::vector<float> rope_inv_freq(const lcr_model_desc& d);

}  // namespace lcrb
