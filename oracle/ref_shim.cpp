// C entry points over the reference's own CPU implementation.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile together with the
// reference's unmodified sources (read in place, never copied) into
// oracle/_ref/libds_ref.so.  The tests use it to pin the C restatement in
// oracle/oracle.c and to generate the golden fixtures under tests/golden/;
// bench.py's reference arm may time it.  Nothing in the product links it.
//
// Every function returns 0 on success and -1 when the reference threw.

#include "ds/core/math.h"
#include "ds/core/ops.h"
#include "ds/core/rope.h"
#include "ds/core/sampler.h"
#include "ds/hf/config.h"
#include "ds/hf/model_loader.h"
#include "ds/models/deepseek/config.h"
#include "ds/models/deepseek/mla.h"
#include "ds/models/deepseek/model.h"
#include "ds/models/deepseek/ops.h"
#include "ds/models/deepseek/weights.h"
#include "ds/runtime/model.h"
#include "ds/runtime/tokenizer.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <memory>
#include <random>
#include <string>
#include <vector>

namespace {

ds::hf::TensorSlice f32_slice(const std::string& name, std::vector<std::int64_t> shape, const float* data) {
  ds::hf::TensorSlice t;
  t.name = name;
  t.dtype = ds::hf::DType::F32;
  std::size_t n = 1;
  for (auto d : shape) n *= static_cast<std::size_t>(d);
  t.shape = std::move(shape);
  t.data = reinterpret_cast<const std::uint8_t*>(data);
  t.nbytes = n * sizeof(float);
  t.shard_path = "in-memory";
  return t;
}

}  // namespace

extern "C" {

// Model hyper-parameters passed from the tests (mirrors ds::hf::DeepSeekConfig).
struct ref_config {
  int hidden_size, intermediate_size, num_hidden_layers, num_attention_heads;
  int vocab_size, max_position_embeddings;
  int n_experts, n_shared_experts, moe_top_k, moe_intermediate_size;
  int q_lora_rank, kv_lora_rank, qk_nope_head_dim, qk_rope_head_dim, v_head_dim;
  int norm_topk_prob;
  float rms_norm_eps, rope_theta, routed_scaling_factor;
};

static ds::hf::DeepSeekConfig to_cfg(const ref_config* c) {
  ds::hf::DeepSeekConfig cfg;
  cfg.model_type = "deepseek_v2";
  cfg.hidden_size = c->hidden_size;
  cfg.intermediate_size = c->intermediate_size;
  cfg.num_hidden_layers = c->num_hidden_layers;
  cfg.num_attention_heads = c->num_attention_heads;
  cfg.num_key_value_heads = c->num_attention_heads;
  cfg.vocab_size = c->vocab_size;
  cfg.max_position_embeddings = c->max_position_embeddings;
  cfg.n_experts = c->n_experts;
  cfg.n_shared_experts = c->n_shared_experts;
  cfg.moe_top_k = c->moe_top_k;
  cfg.moe_intermediate_size = c->moe_intermediate_size;
  cfg.q_lora_rank = c->q_lora_rank;
  cfg.kv_lora_rank = c->kv_lora_rank;
  cfg.qk_nope_head_dim = c->qk_nope_head_dim;
  cfg.qk_rope_head_dim = c->qk_rope_head_dim;
  cfg.v_head_dim = c->v_head_dim;
  cfg.norm_topk_prob = c->norm_topk_prob != 0;
  cfg.rms_norm_eps = c->rms_norm_eps;
  cfg.rope_theta = c->rope_theta;
  cfg.routed_scaling_factor = c->routed_scaling_factor;
  return cfg;
}

__attribute__((visibility("default"))) float ref_dot_f32(const float* a, const float* b, std::size_t n) {
  return ds::core::dot_f32(a, b, n);
}

__attribute__((visibility("default"))) void ref_rmsnorm_f32(const float* x, const float* w, std::size_t n, float eps,
                                                            float* y) {
  ds::core::rmsnorm_f32(x, w, n, eps, y);
}

__attribute__((visibility("default"))) int ref_rope_inplace_f32(float* x, std::size_t dim, std::size_t pos,
                                                                float theta) {
  try {
    ds::core::rope_inplace_f32(x, dim, pos, theta);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

__attribute__((visibility("default"))) int ref_softmax_f32(float* x, std::size_t n) {
  try {
    ds::core::softmax_f32(x, n);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

__attribute__((visibility("default"))) std::int64_t ref_argmax_f32(const float* x, std::size_t n) {
  return static_cast<std::int64_t>(ds::core::argmax_f32(x, n));
}

// ds::rt::linear on an in-memory f32 weight [out, in].
__attribute__((visibility("default"))) int ref_linear_f32(const float* w, const float* x, std::size_t in, float* y,
                                                          std::size_t out) {
  try {
    auto t = f32_slice("w", {static_cast<std::int64_t>(out), static_cast<std::int64_t>(in)}, w);
    ds::rt::linear(t, x, in, y, out);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// mla_decode_step for positions 0..T-1 of a fresh cache (no q-LoRA).
__attribute__((visibility("default"))) int ref_mla_seq(const ref_config* c, const float* w_q, const float* w_kva,
                                                       const float* w_kva_norm, const float* w_kvb, const float* w_o,
                                                       const float* hidden, int T, float* out) {
  try {
    const auto cfg = to_cfg(c);
    const std::int64_t D = cfg.hidden_size, H = cfg.num_attention_heads;
    const std::int64_t qh = cfg.qk_nope_head_dim + cfg.qk_rope_head_dim;
    const std::int64_t R = cfg.kv_lora_rank, P = cfg.qk_rope_head_dim;
    const std::int64_t V = cfg.v_head_dim, nope = cfg.qk_nope_head_dim;
    auto tq = f32_slice("q_proj", {H * qh, D}, w_q);
    auto tkva = f32_slice("kv_a_proj_with_mqa", {R + P, D}, w_kva);
    auto tkvb = f32_slice("kv_b_proj", {H * (nope + V), R}, w_kvb);
    auto to = f32_slice("o_proj", {D, H * V}, w_o);
    auto tnorm = f32_slice("kv_a_layernorm", {R}, w_kva_norm);
    ds::rt::AttentionWeights attn;
    attn.q_proj.weight = &tq;
    attn.kv_a_proj_with_mqa.weight = &tkva;
    attn.kv_a_layernorm.weight = &tnorm;
    attn.kv_a_layernorm.f32.assign(w_kva_norm, w_kva_norm + R);
    attn.kv_b_proj.weight = &tkvb;
    attn.o_proj.weight = &to;
    attn.use_q_lora = false;
    ds::rt::MLACache cache;
    cache.init(static_cast<std::size_t>(T), static_cast<std::size_t>(H), static_cast<std::size_t>(qh),
               static_cast<std::size_t>(V));
    for (int pos = 0; pos < T; ++pos) {
      ds::rt::mla_decode_step(cfg, attn, hidden + static_cast<std::int64_t>(pos) * D, static_cast<std::size_t>(pos),
                              &cache, out + static_cast<std::int64_t>(pos) * D, ds::rt::BackendKind::CPU);
    }
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// moe_step for T independent tokens: gate [E, D], experts gate/up [E, I, D],
// down [E, D, I], optional shared gate/up [Is, D], down [D, Is].
__attribute__((visibility("default"))) int ref_moe_tokens(const ref_config* c, const float* w_gate,
                                                          const float* e_gate, const float* e_up, const float* e_down,
                                                          const float* s_gate, const float* s_up, const float* s_down,
                                                          int shared_inter, const float* x, int T, float* out) {
  try {
    const auto cfg = to_cfg(c);
    const std::int64_t D = cfg.hidden_size, E = cfg.n_experts, I = cfg.moe_intermediate_size;
    std::vector<ds::hf::TensorSlice> slices;
    slices.reserve(static_cast<std::size_t>(3 * E + 4));
    slices.push_back(f32_slice("gate", {E, D}, w_gate));
    ds::rt::MoEWeights moe;
    moe.gate.weight = &slices.back();
    for (std::int64_t e = 0; e < E; ++e) {
      slices.push_back(f32_slice("g", {I, D}, e_gate + e * I * D));
      const auto* g = &slices.back();
      slices.push_back(f32_slice("u", {I, D}, e_up + e * I * D));
      const auto* u = &slices.back();
      slices.push_back(f32_slice("d", {D, I}, e_down + e * D * I));
      const auto* d = &slices.back();
      ds::rt::ExpertWeights ew;
      ew.ffn.gate_proj.weight = g;
      ew.ffn.up_proj.weight = u;
      ew.ffn.down_proj.weight = d;
      moe.experts.push_back(ew);
    }
    if (s_gate != nullptr) {
      const std::int64_t Is = shared_inter;
      slices.push_back(f32_slice("sg", {Is, D}, s_gate));
      moe.shared_experts.gate_proj.weight = &slices.back();
      slices.push_back(f32_slice("su", {Is, D}, s_up));
      moe.shared_experts.up_proj.weight = &slices.back();
      slices.push_back(f32_slice("sd", {D, Is}, s_down));
      moe.shared_experts.down_proj.weight = &slices.back();
    }
    for (int t = 0; t < T; ++t) {
      ds::rt::moe_step(ds::rt::BackendKind::CPU, cfg, moe, x + static_cast<std::int64_t>(t) * D,
                       static_cast<std::size_t>(D), out + static_cast<std::int64_t>(t) * D);
    }
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// A whole in-memory model: tensors named as in the HF checkpoint.
struct ref_model {
  ds::hf::DeepSeekConfig cfg;
  std::vector<std::vector<float>> storage;
  std::unique_ptr<ds::rt::DeepSeekModel> model;
  std::unique_ptr<ds::rt::ModelSession> session;
};

__attribute__((visibility("default"))) void* ref_model_create(const ref_config* c, int n_tensors, const char** names,
                                                              const int* ndims, const std::int64_t* shapes,
                                                              const float** datas) {
  try {
    auto m = std::make_unique<ref_model>();
    m->cfg = to_cfg(c);
    ds::hf::LoadedModel loaded;
    loaded.model_dir = "in-memory";
    const std::int64_t* sp = shapes;
    m->storage.resize(static_cast<std::size_t>(n_tensors));
    for (int i = 0; i < n_tensors; ++i) {
      std::vector<std::int64_t> shape(sp, sp + ndims[i]);
      sp += ndims[i];
      std::size_t n = 1;
      for (auto d : shape) n *= static_cast<std::size_t>(d);
      m->storage[static_cast<std::size_t>(i)].assign(datas[i], datas[i] + n);
      loaded.tensors.emplace(names[i], f32_slice(names[i], shape, m->storage[static_cast<std::size_t>(i)].data()));
    }
    m->model = std::make_unique<ds::rt::DeepSeekModel>(m->cfg, std::move(loaded));
    ds::rt::RunConfig rc;
    rc.backend = ds::rt::BackendKind::CPU;
    rc.max_seq = static_cast<std::size_t>(m->cfg.max_position_embeddings);
    m->session = m->model->create_session(rc);
    return m.release();
  } catch (const std::exception&) {
    return nullptr;
  }
}

__attribute__((visibility("default"))) void ref_model_destroy(void* h) { delete static_cast<ref_model*>(h); }

__attribute__((visibility("default"))) void ref_model_reset(void* h) { static_cast<ref_model*>(h)->session->reset(); }

// forward({token}) once: logits [vocab] and the greedy id.
__attribute__((visibility("default"))) int ref_model_step(void* h, std::int32_t token, float* logits,
                                                          std::int32_t* greedy) {
  try {
    auto* m = static_cast<ref_model*>(h);
    auto out = m->model->forward(*m->session, ds::rt::ForwardInput{{token}});
    if (logits != nullptr) std::memcpy(logits, out.logits.data(), out.logits.size() * sizeof(float));
    *greedy = out.greedy_token_id;
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// ds::rt::generate with greedy decoding from a fresh session.
__attribute__((visibility("default"))) int ref_model_generate(void* h, const std::int32_t* prompt, int n_prompt,
                                                              int n_new, std::int32_t* out_ids) {
  try {
    auto* m = static_cast<ref_model*>(h);
    m->session->reset();
    ds::rt::GenerationConfig g;
    g.max_new_tokens = n_new;
    std::vector<std::int32_t> p(prompt, prompt + n_prompt);
    auto ids = ds::rt::generate(*m->model, *m->session, p, g);
    for (std::size_t i = 0; i < ids.size(); ++i) out_ids[i] = ids[i];
    return static_cast<int>(ids.size()) == n_new ? 0 : -1;
  } catch (const std::exception&) {
    return -1;
  }
}

// The reference's loader on a model directory: parse_deepseek_config over
// load_config_json(dir/config.json), and load_model_dir's tensor views, as
// text ("cfg <field> <value>" lines, then "t <name> <dtype> <nbytes> <dims>"
// per tensor in name order; dtype is the reference's DType enum value).
// Returns the text length, or -1 with the exception message in buf.
__attribute__((visibility("default"))) int ref_checkpoint_summary(const char* dir, char* buf, int len) {
  std::string text;
  int rc = 0;
  try {
    const std::string d(dir);
    const auto cfg = ds::hf::parse_deepseek_config(ds::hf::load_config_json(d + "/config.json"));
    // snprintf, not iostreams: this library is loaded into Python by ctypes
    char line[512];
    auto put_i = [&](const char* k, long long v) {
      std::snprintf(line, sizeof line, "cfg %s %lld\n", k, v);
      text += line;
    };
    auto put_f = [&](const char* k, double v) {
      std::snprintf(line, sizeof line, "cfg %s %.9g\n", k, v);
      text += line;
    };
    put_i("hidden_size", cfg.hidden_size);
    put_i("intermediate_size", cfg.intermediate_size);
    put_i("num_hidden_layers", cfg.num_hidden_layers);
    put_i("num_attention_heads", cfg.num_attention_heads);
    put_i("vocab_size", cfg.vocab_size);
    put_i("max_position_embeddings", cfg.max_position_embeddings);
    put_i("n_routed_experts", cfg.n_experts);
    put_i("n_shared_experts", cfg.n_shared_experts);
    put_i("num_experts_per_tok", cfg.moe_top_k);
    put_i("moe_intermediate_size", cfg.moe_intermediate_size);
    put_i("first_k_dense_replace", cfg.first_k_dense_replace);
    put_i("norm_topk_prob", cfg.norm_topk_prob ? 1 : 0);
    put_i("q_lora_rank", cfg.q_lora_rank);
    put_i("kv_lora_rank", cfg.kv_lora_rank);
    put_i("qk_nope_head_dim", cfg.qk_nope_head_dim);
    put_i("qk_rope_head_dim", cfg.qk_rope_head_dim);
    put_i("v_head_dim", cfg.v_head_dim);
    text += "cfg scoring_func " + cfg.scoring_func + "\n";
    put_f("rms_norm_eps", cfg.rms_norm_eps);
    put_f("rope_theta", cfg.rope_theta);
    put_f("routed_scaling_factor", cfg.routed_scaling_factor);
    const auto m = ds::hf::load_model_dir(d);
    std::vector<std::string> names;
    for (const auto& kv : m.tensors) names.push_back(kv.first);
    std::sort(names.begin(), names.end());
    for (const auto& n : names) {
      const auto& t = m.tensors.at(n);
      std::snprintf(line, sizeof line, " %d %zu", static_cast<int>(t.dtype), t.nbytes);
      text += "t " + n + line;
      for (auto x : t.shape) {
        std::snprintf(line, sizeof line, " %lld", static_cast<long long>(x));
        text += line;
      }
      text += "\n";
    }
  } catch (const std::exception& e) {
    text = e.what();
    rc = -1;
  }
  if (len <= 0) return -1;
  const int n = static_cast<int>(std::min<std::size_t>(text.size(), static_cast<std::size_t>(len - 1)));
  std::memcpy(buf, text.data(), static_cast<std::size_t>(n));
  buf[n] = 0;
  return rc == 0 ? n : -1;
}

// ds::core::Sampler (src/core/sampler.cpp:23-77) with a fixed seed: n calls
// of sample() on the same logits row.
__attribute__((visibility("default"))) int ref_sampler_draws(const float* logits, int V, float temperature, int top_k,
                                                             float top_p, std::uint32_t seed, int n, std::int32_t* out) {
  try {
    ds::core::Sampler sm(ds::core::SamplerConfig{temperature, top_k, top_p, seed});
    const std::vector<float> row(logits, logits + V);
    for (int i = 0; i < n; ++i) out[i] = sm.sample(row);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// The uniform draws such a Sampler makes, one per sample() call: a
// std::mt19937 seeded with `seed` through a fresh
// std::uniform_real_distribution<float>(0, 1) each time (sampler.cpp:21, 69-70).
__attribute__((visibility("default"))) int ref_sampler_uniforms(std::uint32_t seed, int n, float* out) {
  std::mt19937 rng(seed);
  for (int i = 0; i < n; ++i) {
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    out[i] = dist(rng);
  }
  return 0;
}

// ds::rt::Tokenizer (src/runtime/tokenizer.cpp) loaded from `path`: encode
// text[0, len) into ids[0, cap); returns the id count, or -1 with the
// exception message in msg.
__attribute__((visibility("default"))) int ref_tokenizer_encode(const char* path, const char* text, int len,
                                                                std::int32_t* ids, int cap, char* msg, int msg_len) {
  try {
    const auto tok = ds::rt::Tokenizer::load_from_file(path);
    const auto v = tok.encode(std::string(text, text + len));
    for (std::size_t i = 0; i < v.size() && static_cast<int>(i) < cap; ++i) ids[i] = v[i];
    return static_cast<int>(v.size());
  } catch (const std::exception& e) {
    std::snprintf(msg, static_cast<std::size_t>(msg_len), "%s", e.what());
    return -1;
  }
}

// Tokenizer::decode of ids[0, n) into out[0, cap); returns the byte count, or -1.
__attribute__((visibility("default"))) int ref_tokenizer_decode(const char* path, const std::int32_t* ids, int n,
                                                                int skip_special, char* out, int cap) {
  try {
    const auto tok = ds::rt::Tokenizer::load_from_file(path);
    const auto s = tok.decode(std::vector<std::int32_t>(ids, ids + n), skip_special != 0);
    std::memcpy(out, s.data(), std::min<std::size_t>(s.size(), static_cast<std::size_t>(cap)));
    return static_cast<int>(s.size());
  } catch (const std::exception&) {
    return -1;
  }
}

}  // extern "C"
