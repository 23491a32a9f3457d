// The reference engine's own runtime (ds::rt::generate, ModelExecutor, the
// package descriptor's host functions) driving the B200 package.  Built by
// oracle/Makefile against the reference's headers and its compiled sources
// (oracle/_ref/libds_ref.so), plus deepseek_cpp_infer_b200/refapi and
// libdsb.so.  Test infrastructure: tests/test_ref_dropin.py runs it.
//
//   ds_dropin_demo info <model_dir>                 package id + print_config
//   ds_dropin_demo gen  <model_dir> <ids,...> <n>   ds::rt::generate and ModelExecutor
//   ds_dropin_demo cpu  <model_dir>                 a CPU-backend session (an error)
#include "b200_package.h"

#include "ds/hf/config.h"
#include "ds/runtime/model.h"
#include "ds/runtime/model_executor.h"

#include <cstdio>
#include <cstdlib>
#include <exception>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

namespace {

std::vector<std::int32_t> parse_ids(const std::string& s) {
  std::vector<std::int32_t> ids;
  std::stringstream ss(s);
  std::string tok;
  while (std::getline(ss, tok, ',')) ids.push_back(static_cast<std::int32_t>(std::stol(tok)));
  return ids;
}

void print_ids(const char* key, const std::vector<std::int32_t>& ids) {
  std::cout << key;
  for (auto id : ids) std::cout << ' ' << id;
  std::cout << '\n';
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 3) {
    std::cerr << "usage: ds_dropin_demo info|gen|cpu <model_dir> [ids n]\n";
    return 2;
  }
  const std::string cmd = argv[1], dir = argv[2];
  try {
    const auto& pkg = ds::models::b200::package_descriptor();
    const auto cfg = ds::hf::load_config_json(dir + "/config.json");
    if (!pkg.matches(cfg)) throw std::runtime_error("package does not match " + cfg.model_type);
    if (cmd == "info") {
      std::cout << "package " << pkg.package_id << '\n';
      pkg.print_config(std::cout, cfg);
      return 0;
    }
    auto model = pkg.load(dir, cfg);  // the descriptor's load: the B200 model
    if (cmd == "cpu") {
      ds::rt::RunConfig rc;  // the reference's default backend, CPU
      model->create_session(rc);
      return 0;
    }
    if (cmd != "gen" || argc < 5) throw std::runtime_error("bad command");
    const auto prompt = parse_ids(argv[3]);
    ds::rt::GenerationConfig g;
    g.max_new_tokens = std::atoi(argv[4]);
    ds::rt::RunConfig rc;
    rc.backend = ds::rt::BackendKind::CUDA;
    rc.max_seq = 256;
    // the reference's free generate on a session of the model
    auto session = model->create_session(rc);
    print_ids("ids", ds::rt::generate(*model, *session, prompt, g));
    std::cout << "position " << session->position() << '\n';
    // the reference's ModelExecutor: generate, then prefill + decode_next
    ds::rt::ModelExecutor exec(model, rc);
    print_ids("exec", exec.generate(prompt, g));
    exec.reset();
    const auto first = exec.prefill(prompt);
    const auto second = exec.decode_next(first.greedy_token_id);
    std::cout << "steps " << first.greedy_token_id << ' ' << second.greedy_token_id << ' ' << exec.position() << '\n';
    std::cout << "backends " << model->info().supports_backend(ds::rt::BackendKind::CUDA) << ' '
              << model->info().supports_backend(ds::rt::BackendKind::CPU) << '\n';
    // an empty forward fails as the reference's does
    try {
      model->forward(*session, ds::rt::ForwardInput{});
      std::cout << "empty ok\n";
    } catch (const std::exception& e) {
      std::cout << "empty error " << e.what() << '\n';
    }
    return 0;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << '\n';
    return 1;
  }
}
