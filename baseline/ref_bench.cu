// Times the reference runtime's own Model (src/model.h of
// mohamadmsalman82/llama-cuda-runtime) on a checkpoint directory, the way its
// llama-run --bench loop does (src/main.cu:420-466): warm-up passes, one
// prefill of the prompt, then greedy steps of sample + decode, with the
// decode time summed from the Model's own per-step GPU timer
// (ForwardStats::last_decode_ms). The prompt is token ids (no tokenizer on
// this path). Prints one JSON object; --logits-out writes the fp32 logits
// after the prompt.
//
//   ref_bench --model DIR --prompt IDS.bin --steps N --max-seq S
//             [--paged] [--warmup W] [--logits-out FILE]
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "model.h"

namespace {

std::vector<int> read_ids(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  std::vector<int> ids;
  int32_t v;
  while (f.read(reinterpret_cast<char*>(&v), sizeof v)) ids.push_back(v);
  return ids;
}

}  // namespace

int main(int argc, char** argv) {
  std::string model_dir, prompt_path, logits_out;
  int steps = 64, max_seq = 512, warmup = 1;
  bool paged = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() { return std::string(i + 1 < argc ? argv[++i] : ""); };
    if (a == "--model") model_dir = next();
    else if (a == "--prompt") prompt_path = next();
    else if (a == "--steps") steps = std::atoi(next().c_str());
    else if (a == "--max-seq") max_seq = std::atoi(next().c_str());
    else if (a == "--warmup") warmup = std::atoi(next().c_str());
    else if (a == "--paged") paged = true;
    else if (a == "--logits-out") logits_out = next();
  }
  const std::vector<int> prompt = read_ids(prompt_path);
  if (model_dir.empty() || prompt.empty()) {
    std::fprintf(stderr, "usage: ref_bench --model DIR --prompt IDS.bin [--steps N] [--max-seq S]\n");
    return 2;
  }
  try {
    lcr::Model::Options opt;
    opt.max_seq = max_seq;
    opt.kv_layout = paged ? lcr::KvLayout::kPaged : lcr::KvLayout::kContiguous;
    const auto t0 = std::chrono::steady_clock::now();
    lcr::Model model(model_dir, opt);
    const double load_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    for (int i = 0; i < warmup; ++i) {
      const float* warm = model.prefill(prompt);
      model.decode(model.sample(warm, 0.0f, 0, 1.0f, 0.0f));
      model.reset();
    }
    const float* logits = model.prefill(prompt);
    const double prefill_ms = model.stats().last_prefill_ms;
    if (!logits_out.empty()) {
      const std::vector<float> host = model.logits_to_host(logits);
      std::ofstream(logits_out, std::ios::binary)
          .write(reinterpret_cast<const char*>(host.data()), static_cast<std::streamsize>(host.size() * 4));
    }
    std::vector<int> ids;
    double decode_ms = 0.0;
    const auto w0 = std::chrono::steady_clock::now();
    for (int s = 0; s < steps; ++s) {
      const int token = model.sample(logits, 0.0f, 0, 1.0f, 0.0f);
      ids.push_back(token);
      logits = model.decode(token);
      decode_ms += model.stats().last_decode_ms;
    }
    const double wall_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - w0).count();
    std::printf("{\"load_ms\": %.1f, \"prompt_tokens\": %zu, \"prefill_ms\": %.3f, \"decode_steps\": %d, "
                "\"decode_ms\": %.3f, \"decode_tokens_per_s\": %.2f, \"loop_wall_ms\": %.3f, "
                "\"loop_tokens_per_s\": %.2f, \"weight_bytes_per_token\": %zu, \"kv_bytes_per_position\": %zu, "
                "\"final_position\": %d, \"ids\": [",
                load_ms, prompt.size(), prefill_ms, steps, decode_ms, steps / (decode_ms / 1e3), wall_ms,
                steps / (wall_ms / 1e3), model.stats().weight_bytes_per_token,
                model.stats().kv_bytes_per_position, model.position());
    for (size_t i = 0; i < ids.size(); ++i) std::printf("%s%d", i ? ", " : "", ids[i]);
    std::printf("]}\n");
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ref_bench: %s\n", e.what());
    return 1;
  }
  return 0;
}
