// ds_chat_b200: the reference's command-line front end (src/main.cpp:22-306,
// `ds_chat <model_dir> [info|verify|strict|load|run|generate] [options]`)
// over libdsb.so's C ABI, plus a decode-throughput `bench` subcommand.
//
//   info      config, tokenizer, index and shards of the model directory
//   verify    open the checkpoint (index, every shard header, byte ranges)
//             and check the tensors every layer needs
//   strict    verify, then the dense / MoE layer map
//   load      upload every decode tensor to the GPU and finalize the model
//   run       prefill the prompt, print the next-token prediction
//   generate  prefill, then decode up to --max-new-tokens ids (greedy, or
//             sampled when --temperature, --top-k or --top-p is above 0)
//   bench     decode throughput: --batch sequences of --prompt-len random
//             ids prefilled, then --steps greedy decode steps timed
//
// Output lines and error handling follow the reference ("fatal: <message>"
// on stderr, exit status 1).

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "dsb/dsb.h"

namespace {

struct Options {
  std::string prompt, prompt_ids;
  int max_new_tokens = 32;
  long max_seq = 0;
  float temperature = 0.0f, top_p = 0.0f;
  int top_k = 0;
  unsigned seed = 0;
  int device = 0, batch = 32, prompt_len = 512, steps = 32;
};

[[noreturn]] void usage() {
  throw std::runtime_error(
      "usage: ds_chat_b200 <model_dir> [info|verify|strict|load|run|generate|bench] [options]\n"
      "  info:     print config, tokenizer, index and shard list\n"
      "  verify:   open the checkpoint (index, shard headers, byte ranges) (default)\n"
      "  strict:   verify + print the dense/MoE layer map from the tensor names\n"
      "  load:     upload every tensor to the GPU and finalize the model\n"
      "  run:      prefill the prompt and print the next-token prediction\n"
      "  generate: autoregressive decode\n"
      "  bench:    decode throughput of --batch sequences\n"
      "options:\n"
      "  --prompt <text>  --prompt-ids <id0,id1,...>  --max-new-tokens <n>  --max-seq <n>\n"
      "  --temperature <float>  --top-k <int>  --top-p <float>  --seed <int>  --device <int>\n"
      "  --batch <n>  --prompt-len <n>  --steps <n>   (bench)");
}

long to_long(const std::string& key, const std::string& v) {
  char* end = nullptr;
  const long x = std::strtol(v.c_str(), &end, 10);
  if (v.empty() || *end != '\0') throw std::runtime_error("bad value for " + key + ": " + v);
  return x;
}

float to_float(const std::string& key, const std::string& v) {
  char* end = nullptr;
  const float x = std::strtof(v.c_str(), &end);
  if (v.empty() || *end != '\0') throw std::runtime_error("bad value for " + key + ": " + v);
  return x;
}

Options parse_options(int argc, char** argv, int first) {
  Options o;
  for (int i = first; i < argc; ++i) {
    const std::string key = argv[i];
    if (i + 1 >= argc) throw std::runtime_error("missing value for " + key);
    const std::string v = argv[++i];
    if (key == "--prompt") o.prompt = v;
    else if (key == "--prompt-ids") o.prompt_ids = v;
    else if (key == "--max-new-tokens") o.max_new_tokens = (int)to_long(key, v);
    else if (key == "--max-seq") o.max_seq = to_long(key, v);
    else if (key == "--temperature") o.temperature = to_float(key, v);
    else if (key == "--top-k") o.top_k = (int)to_long(key, v);
    else if (key == "--top-p") o.top_p = to_float(key, v);
    else if (key == "--seed") o.seed = (unsigned)to_long(key, v);
    else if (key == "--device") o.device = (int)to_long(key, v);
    else if (key == "--batch") o.batch = (int)to_long(key, v);
    else if (key == "--prompt-len") o.prompt_len = (int)to_long(key, v);
    else if (key == "--steps") o.steps = (int)to_long(key, v);
    else throw std::runtime_error("unknown option: " + key);
  }
  return o;
}

bool file_exists(const std::string& p) {
  FILE* f = std::fopen(p.c_str(), "rb");
  if (f == nullptr) return false;
  std::fclose(f);
  return true;
}

void ck(int rc, const char* what) {
  if (rc != DSB_OK) throw std::runtime_error(std::string(what) + ": " + dsb_checkpoint_error());
}

void tk(int rc, const char* what) {
  if (rc != DSB_OK) throw std::runtime_error(std::string(what) + ": " + dsb_tokenizer_error());
}

// Owners of the library handles (destroyed in reverse order of creation).
struct Session {
  dsb_checkpoint* ckpt = nullptr;
  dsb_tokenizer* tok = nullptr;
  dsb_ctx* ctx = nullptr;
  dsb_model* model = nullptr;
  dsb_kvcache* kv = nullptr;
  ~Session() {
    if (kv) dsb_kvcache_destroy(kv);
    if (model) dsb_model_destroy(model);
    if (ctx) dsb_ctx_destroy(ctx);
    if (tok) dsb_tokenizer_destroy(tok);
    if (ckpt) dsb_checkpoint_close(ckpt);
  }
  void check(int rc, const char* what) const {
    if (rc != DSB_OK)
      throw std::runtime_error(std::string(what) + ": " + (ctx ? dsb_last_error(ctx) : "no context"));
  }
};

void print_config(const dsb_model_config& c) {
  std::printf("Loaded config:\n  family: deepseek\n  layers: %d\n  hidden: %d\n  heads: %d\n  vocab: %d\n"
              "  max_pos: %d\n  rope_theta: %g\n  n_experts: %d\n  n_shared_experts: %d\n  moe_top_k: %d\n"
              "  q_lora_rank: %d\n  kv_lora_rank: %d\n  qk_nope_head_dim: %d\n  qk_rope_head_dim: %d\n"
              "  v_head_dim: %d\n  scoring: %s (n_group %d, topk_group %d)\n  weights: %s\n",
              c.num_hidden_layers, c.hidden_size, c.num_attention_heads, c.vocab_size, c.max_position_embeddings,
              c.rope_theta, c.n_routed_experts, c.n_shared_experts, c.num_experts_per_tok, c.q_lora_rank,
              c.kv_lora_rank, c.qk_nope_head_dim, c.qk_rope_head_dim, c.v_head_dim,
              c.scoring_func == DSB_SCORE_SIGMOID ? "sigmoid" : "softmax", c.n_group, c.topk_group,
              c.weights_fp8 ? "block-scaled fp8" : "bf16/f32");
}

// inspect_index (src/models/deepseek/package.cpp:58-120): the tensors every
// layer needs, "dense" / "MoE" per layer from the experts' presence.  Unlike
// the reference, a q_lora layer (q_a_proj, q_a_layernorm, q_b_proj) stands in
// for q_proj and shared experts are required only when the config has some.
std::vector<std::string> layer_map(const dsb_checkpoint* ckpt, const dsb_model_config& c) {
  auto has = [&](const std::string& name) {
    int idx = -1;
    ck(dsb_checkpoint_find(ckpt, name.c_str(), &idx), "find");
    return idx >= 0;
  };
  auto require = [&](const std::string& name) {
    if (!has(name)) throw std::runtime_error("missing tensor in index: " + name);
  };
  require("lm_head.weight");
  require("model.embed_tokens.weight");
  require("model.norm.weight");
  std::vector<std::string> kinds;
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    const std::string base = "model.layers." + std::to_string(i) + ".", attn = base + "self_attn.", mlp = base + "mlp.";
    for (const char* n : {"input_layernorm.weight", "post_attention_layernorm.weight"}) require(base + n);
    for (const char* n : {"o_proj.weight", "kv_a_layernorm.weight", "kv_a_proj_with_mqa.weight", "kv_b_proj.weight"})
      require(attn + n);
    if (!has(attn + "q_proj.weight"))
      for (const char* n : {"q_a_proj.weight", "q_a_layernorm.weight", "q_b_proj.weight"}) require(attn + n);
    const bool moe = has(mlp + "experts.0.gate_proj.weight");
    kinds.push_back(moe ? "MoE" : "dense");
    if (!moe) {
      for (const char* n : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"}) require(mlp + n);
      continue;
    }
    require(mlp + "gate.weight");
    if (c.n_shared_experts > 0)
      for (const char* n : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"})
        require(mlp + "shared_experts." + n);
    for (int e : {0, c.n_routed_experts - 1})
      for (const char* n : {"gate_proj.weight", "up_proj.weight", "down_proj.weight"})
        require(mlp + "experts." + std::to_string(e) + "." + n);
  }
  return kinds;
}

std::vector<int32_t> parse_ids(const std::string& csv) {
  std::vector<int32_t> out;
  size_t i = 0;
  while (i <= csv.size()) {
    size_t j = csv.find(',', i);
    if (j == std::string::npos) j = csv.size();
    const std::string t = csv.substr(i, j - i);
    if (!t.empty()) out.push_back((int32_t)to_long("--prompt-ids", t));
    i = j + 1;
  }
  return out;
}

// Create the context and model, upload the checkpoint, and a cache for
// max_seqs sequences of max_seq positions.
void load_model(Session& s, const Options& o, const dsb_model_config& cfg, int max_seqs, long max_seq) {
  if (dsb_ctx_create(o.device, &s.ctx) != DSB_OK) throw std::runtime_error("dsb_ctx_create: no usable CUDA device");
  s.check(dsb_model_create(s.ctx, &cfg, &s.model), "dsb_model_create");
  int up = 0, skipped = 0;
  s.check(dsb_model_upload_checkpoint(s.model, s.ckpt, &up, &skipped), "dsb_model_upload_checkpoint");
  s.check(dsb_model_finalize(s.model), "dsb_model_finalize");
  std::printf("Uploaded tensors: %d (skipped %d)\n", up, skipped);
  if (max_seqs > 0) {
    const long pages = (max_seq + 63) / 64;
    s.check(dsb_kvcache_create(s.ctx, s.model, pages * max_seqs, max_seqs, (int)pages, &s.kv), "dsb_kvcache_create");
  }
}

// Prompt rows [0, n) of sequence `seq` through dsb_prefill in chunks; the
// greedy id after the last row.
int32_t prefill(Session& s, int seq, const int32_t* ids, size_t n) {
  int32_t next = -1;
  for (size_t c = 0; c < n; c += DSB_PREFILL_MAX_TOKENS) {
    const int m = (int)std::min<size_t>(DSB_PREFILL_MAX_TOKENS, n - c);
    std::vector<int32_t> sid((size_t)m, seq);
    int n_seq = 0;
    s.check(dsb_prefill(s.ctx, s.model, s.kv, sid.data(), ids + c, m, nullptr, &next, &n_seq), "dsb_prefill");
  }
  return next;
}

std::string decode_one(const dsb_tokenizer* tok, int32_t id) {
  size_t len = 0;
  if (dsb_tokenizer_decode(tok, &id, 1, 1, nullptr, 0, &len) != DSB_OK && len == 0) tk(DSB_EINVAL, "decode");
  std::string s(len, '\0');
  tk(dsb_tokenizer_decode(tok, &id, 1, 1, s.empty() ? nullptr : &s[0], s.size(), &len), "decode");
  return s;
}

int main_impl(int argc, char** argv) {
  if (argc < 2) usage();
  const std::string dir = argv[1];
  const std::string cmd = argc >= 3 ? argv[2] : "verify";
  if (!file_exists(dir + "/config.json")) throw std::runtime_error("missing config.json in model_dir: " + dir + "/config.json");
  Session s;
  ck(dsb_checkpoint_open(dir.c_str(), &s.ckpt), "checkpoint");
  dsb_model_config cfg{};
  ck(dsb_checkpoint_config(s.ckpt, &cfg), "config");
  const std::string tok_path = dir + "/tokenizer.json";
  const bool has_tok = file_exists(tok_path);
  int n_tensors = 0;
  ck(dsb_checkpoint_num_tensors(s.ckpt, &n_tensors), "tensors");

  if (cmd == "info") {
    print_config(cfg);
    std::printf("Tokenizer: %s (%s)\n", has_tok ? "OK" : "MISSING", tok_path.c_str());
    std::printf("Index: %s\n", file_exists(dir + "/model.safetensors.index.json") ? "OK" : "(none)");
    std::printf("Tensors: %d\n", n_tensors);
    return 0;
  }
  if (cmd == "verify" || cmd == "strict") {
    print_config(cfg);
    if (!has_tok) std::printf("warn: tokenizer.json missing: %s\n", tok_path.c_str());
    const std::vector<std::string> kinds = layer_map(s.ckpt, cfg);
    std::printf("Index OK (required tensor keys present). keys=%d\n", n_tensors);
    if (cmd == "strict") {
      int moe = 0;
      std::printf("Layer map (from index):\n");
      for (size_t li = 0; li < kinds.size(); ++li) {
        std::printf("  layer %zu: %s\n", li, kinds[li].c_str());
        moe += kinds[li] == "MoE";
      }
      std::printf("MoE layers: %d/%d\n", moe, cfg.num_hidden_layers);
    }
    uint64_t bytes = 0;
    for (int i = 0; i < n_tensors; ++i) {
      dsb_tensor_info t;
      ck(dsb_checkpoint_tensor(s.ckpt, i, &t), "tensor");
      bytes += t.nbytes;
    }
    std::printf("OK (parsed headers). total_tensors=%d bytes=%llu\n", n_tensors, (unsigned long long)bytes);
    return 0;
  }

  const Options o = parse_options(argc, argv, 3);
  if (cmd == "load") {
    load_model(s, o, cfg, 0, 0);
    std::printf("OK\n");
    return 0;
  }
  if (cmd == "bench") {
    if (o.batch <= 0 || o.prompt_len <= 0 || o.steps <= 0) throw std::runtime_error("bench needs positive sizes");
    const long max_seq = (long)o.prompt_len + o.steps + 1;
    if (max_seq > cfg.max_position_embeddings) throw std::runtime_error("bench sequence exceeds max_position_embeddings");
    load_model(s, o, cfg, o.batch, max_seq);
    std::mt19937 rng(o.seed ? o.seed : 1u);
    std::uniform_int_distribution<int32_t> pick(0, cfg.vocab_size - 1);
    std::vector<int32_t> seqs((size_t)o.batch), toks((size_t)o.batch), next((size_t)o.batch);
    const auto t0 = std::chrono::steady_clock::now();
    for (int b = 0; b < o.batch; ++b) {
      s.check(dsb_kvcache_alloc_seq(s.kv, &seqs[(size_t)b]), "dsb_kvcache_alloc_seq");
      std::vector<int32_t> p((size_t)o.prompt_len);
      for (auto& x : p) x = pick(rng);
      toks[(size_t)b] = prefill(s, seqs[(size_t)b], p.data(), p.size());
    }
    const auto t1 = std::chrono::steady_clock::now();
    for (int i = 0; i < o.steps; ++i) {
      s.check(dsb_decode_step(s.ctx, s.model, s.kv, seqs.data(), toks.data(), o.batch, nullptr, next.data()),
              "dsb_decode_step");
      toks.swap(next);
    }
    const auto t2 = std::chrono::steady_clock::now();
    const double pre = std::chrono::duration<double>(t1 - t0).count(), dec = std::chrono::duration<double>(t2 - t1).count();
    std::printf("Prefill: %d x %d tokens in %.3f s (%.0f tokens/s)\n", o.batch, o.prompt_len, pre,
                (double)o.batch * o.prompt_len / pre);
    std::printf("Decode: %d steps of %d sequences in %.3f s: %.3f ms/step, %.0f tokens/s\n", o.steps, o.batch, dec,
                1e3 * dec / o.steps, (double)o.batch * o.steps / dec);
    return 0;
  }
  if (cmd != "run" && cmd != "generate") usage();

  // resolve_prompt_ids / resolve_max_seq (src/main.cpp:104-141)
  std::vector<int32_t> prompt;
  if (has_tok) tk(dsb_tokenizer_load(tok_path.c_str(), &s.tok), "tokenizer");
  if (!o.prompt_ids.empty()) {
    prompt = parse_ids(o.prompt_ids);
  } else {
    if (o.prompt.empty()) throw std::runtime_error("run/generate requires --prompt or --prompt-ids");
    if (!has_tok) throw std::runtime_error("tokenizer.json is required to encode --prompt; use --prompt-ids instead");
    size_t n = 0;
    prompt.resize(o.prompt.size() + 1);
    tk(dsb_tokenizer_encode(s.tok, o.prompt.data(), o.prompt.size(), prompt.data(), prompt.size(), &n), "encode");
    prompt.resize(n);
  }
  if (prompt.empty()) throw std::runtime_error("prompt resolved to zero token ids");
  for (int32_t id : prompt)
    if (id < 0 || id >= cfg.vocab_size) throw std::runtime_error("prompt id out of range: " + std::to_string(id));
  const bool gen = cmd == "generate";
  long required = (long)prompt.size() + (gen && o.max_new_tokens > 0 ? o.max_new_tokens : 0);
  if (required > cfg.max_position_embeddings)
    throw std::runtime_error("requested sequence exceeds model max_position_embeddings");
  if (o.max_seq != 0 && o.max_seq < required)
    throw std::runtime_error("--max-seq is smaller than the requested prompt/generation length");
  if (o.max_seq > cfg.max_position_embeddings) throw std::runtime_error("--max-seq exceeds model max_position_embeddings");
  const long max_seq = o.max_seq != 0 ? o.max_seq : required;

  load_model(s, o, cfg, 1, max_seq);
  int seq = 0;
  s.check(dsb_kvcache_alloc_seq(s.kv, &seq), "dsb_kvcache_alloc_seq");
  if (!gen) {
    const int32_t next = prefill(s, seq, prompt.data(), prompt.size());
    std::printf("Prompt tokens: %zu\nNext token id: %d\n", prompt.size(), next);
    if (s.tok) std::printf("Next token text: %s\n", decode_one(s.tok, next).c_str());
    return 0;
  }
  // the prompt but its last token by prefill; generation feeds the last one
  if (prompt.size() > 1) prefill(s, seq, prompt.data(), prompt.size() - 1);
  int32_t eos = -1;
  if (s.tok) tk(dsb_tokenizer_info(s.tok, nullptr, nullptr, &eos, nullptr), "tokenizer");
  const dsb_sampling smp{o.temperature, o.top_k, o.top_p, o.seed};
  const int32_t offs[2] = {0, 1};
  std::vector<int32_t> out((size_t)std::max(1, o.max_new_tokens));
  int32_t count = 0;
  s.check(dsb_generate_sampled(s.ctx, s.model, s.kv, &seq, 1, &prompt.back(), offs, o.max_new_tokens, eos, &smp,
                               out.data(), &count),
          "dsb_generate_sampled");
  std::printf("Generated ids:");
  for (int i = 0; i < count; ++i) std::printf(" %d", out[(size_t)i]);
  std::printf("\n");
  if (s.tok) {
    std::string text;
    for (int i = 0; i < count; ++i) text += decode_one(s.tok, out[(size_t)i]);
    std::printf("Generated text: %s\n", text.c_str());
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc == 2 && (std::string(argv[1]) == "-h" || std::string(argv[1]) == "--help")) {
    try {
      usage();
    } catch (const std::exception& e) {
      std::printf("%s\n", e.what());
    }
    return 0;
  }
  try {
    return main_impl(argc, argv);
  } catch (const std::exception& e) {
    std::fflush(stdout);
    std::fprintf(stderr, "fatal: %s\n", e.what());
    return 1;
  }
}
