// Drives dsb::rt (include/dsb/runtime.hpp) the way a ds::rt caller would:
//   rt_demo tok <tokenizer.json> <text>          encode + decode, no GPU
//   rt_demo load <model_dir>                     load_model (needs a GPU)
//   rt_demo gen <model_dir> <ids,...> <n> [temperature top_k top_p seed]
//   rt_demo batch <model_dir> <ids,...> <ids,...> <n>   two prompts together
// Prints one line per result; exit status 1 with "error <code>: <what>".
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "dsb/runtime.hpp"

namespace rt = dsb::rt;

static std::vector<std::int32_t> parse_ids(const std::string& csv) {
  std::vector<std::int32_t> v;
  size_t i = 0;
  while (i < csv.size()) {
    size_t j = csv.find(',', i);
    if (j == std::string::npos) j = csv.size();
    v.push_back((std::int32_t)std::atoi(csv.substr(i, j - i).c_str()));
    i = j + 1;
  }
  return v;
}

int main(int argc, char** argv) {
  try {
    const std::string cmd = argc > 1 ? argv[1] : "";
    if (cmd == "tok" && argc == 4) {
      const rt::Tokenizer tok = rt::Tokenizer::load_from_file(argv[2]);
      const std::vector<std::int32_t> ids = tok.encode(argv[3]);
      std::printf("ids");
      for (std::int32_t id : ids) std::printf(" %d", id);
      std::printf("\ntext %s\n", tok.decode(ids, false).c_str());
      return 0;
    }
    if (cmd == "load" && argc == 3) {
      auto model = rt::load_model(argv[2]);
      std::printf("vocab %d\n", model->info().vocab_size);
      return 0;
    }
    if (cmd == "gen" && (argc == 5 || argc == 9)) {
      auto model = rt::load_model(argv[2]);
      rt::ModelExecutor ex(model, rt::RunConfig{0, 256, false});
      rt::GenerationConfig g;
      g.max_new_tokens = std::atoi(argv[4]);
      if (argc == 9) {
        g.temperature = (float)std::atof(argv[5]);
        g.top_k = std::atoi(argv[6]);
        g.top_p = (float)std::atof(argv[7]);
        g.seed = (std::uint32_t)std::atoi(argv[8]);
      }
      const std::vector<std::int32_t> prompt = parse_ids(argv[3]);
      const std::vector<std::int32_t> ids = ex.generate(prompt, g);
      std::printf("ids");
      for (std::int32_t id : ids) std::printf(" %d", id);
      std::printf("\nposition %zu\n", ex.position());
      // the executor's own step API after a reset: prefill, then decode_next
      ex.reset();
      const rt::StepResult first = ex.prefill(prompt);
      const rt::StepResult second = ex.decode_next(first.greedy_token_id);
      std::printf("steps %d %d %zu\n", first.greedy_token_id, second.greedy_token_id, ex.position());
      return 0;
    }
    if (cmd == "batch" && argc == 6) {
      // batch <model_dir> <ids,...> <ids,...> <n>: two prompts generated together, greedy
      auto model = rt::load_model(argv[2]);
      rt::BatchSession batch(model, 2, 256);
      const std::vector<int> seqs = {batch.add(), batch.add()};
      rt::GenerationConfig g;
      g.max_new_tokens = std::atoi(argv[5]);
      const auto out = batch.generate(seqs, {parse_ids(argv[3]), parse_ids(argv[4])}, g);
      for (const auto& ids : out) {
        std::printf("ids");
        for (std::int32_t id : ids) std::printf(" %d", id);
        std::printf("\n");
      }
      return 0;
    }
    std::fprintf(stderr, "usage: rt_demo tok|load|gen|batch ...\n");
    return 2;
  } catch (const rt::Error& e) {
    std::fprintf(stderr, "error %d: %s\n", e.code(), e.what());
    return 1;
  }
}
