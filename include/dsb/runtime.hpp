// dsb/runtime.hpp - the reference's C++ runtime API (namespace ds::rt:
// include/ds/runtime/model.h, model_executor.h, backend.h, model_factory.h,
// tokenizer.h) over libdsb.so's C ABI, header-only, C++17.
//
// The same names and meanings, so a caller of ds::rt switches with
// `namespace rt = dsb::rt;` and a link against libdsb.so:
//   load_model(dir)                  -> shared_ptr<const Model> (ds::rt::load_model)
//   Model::info / create_session / forward
//   ModelSession::reset / position
//   generate(model, session, prompt, GenerationConfig, tokenizer, pieces)
//   ModelExecutor: prefill / decode_next / generate / reset / position
//   Tokenizer::load_from_file / encode / decode / metadata
// plus BatchSession, the batched session the reference does not have.
// Differences: the backend is always the B200 path (RunConfig carries a CUDA
// device instead of a BackendKind), and failures throw dsb::rt::Error (a
// std::runtime_error carrying the DSB_E* code) where the reference throws
// std::runtime_error.  Sampling draws its uniforms from std::mt19937(seed)
// (std::random_device when seed is 0) exactly as ds::core::Sampler does and
// picks the id on the device (dsb_decode_step_sampled).
//
// A Model owns one dsb_ctx: use a Model and its sessions from one thread.

#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "dsb/dsb.h"

namespace dsb {
namespace rt {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& what) : std::runtime_error(what), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

struct ModelInfo {
  std::string family_id = "deepseek";
  std::int32_t vocab_size = 0;
  std::int32_t max_position_embeddings = 0;
  bool weights_fp8 = false;
};

// ds::rt::RunConfig with the backend fixed to this library's GPU path.
struct RunConfig {
  int device = 0;
  std::size_t max_seq = 0;  // 0: max_position_embeddings
  bool verbose = false;
};

struct GenerationConfig {
  std::int32_t max_new_tokens = 1;
  float temperature = 0.0f;
  std::int32_t top_k = 0;
  float top_p = 0.0f;
  std::uint32_t seed = 0;
};

struct ForwardInput {
  std::vector<std::int32_t> token_ids;
};

struct ForwardOutput {
  std::vector<float> logits;
  std::int32_t greedy_token_id = 0;
  std::size_t position_after = 0;
};

struct StepResult {
  std::vector<float> logits;
  std::int32_t greedy_token_id = 0;
};

struct TokenizerMetadata {
  std::int32_t bos_token_id = -1;
  std::int32_t eos_token_id = -1;
  std::int32_t unk_token_id = -1;
};

class Tokenizer {
 public:
  Tokenizer() = default;
  static Tokenizer load_from_file(const std::string& path) {
    Tokenizer t;
    dsb_tokenizer* h = nullptr;
    const int rc = dsb_tokenizer_load(path.c_str(), &h);
    if (rc != DSB_OK) throw Error(rc, dsb_tokenizer_error());
    t.h_.reset(h, [](dsb_tokenizer* p) { dsb_tokenizer_destroy(p); });
    dsb_tokenizer_info(h, nullptr, &t.meta_.bos_token_id, &t.meta_.eos_token_id, &t.meta_.unk_token_id);
    return t;
  }
  bool empty() const { return !h_; }
  const TokenizerMetadata& metadata() const { return meta_; }
  std::vector<std::int32_t> encode(const std::string& text) const {
    std::vector<std::int32_t> ids(text.size() + 1);
    std::size_t n = 0;
    const int rc = dsb_tokenizer_encode(handle(), text.data(), text.size(), ids.data(), ids.size(), &n);
    if (rc != DSB_OK) throw Error(rc, dsb_tokenizer_error());
    ids.resize(n);
    return ids;
  }
  std::string decode(const std::vector<std::int32_t>& ids, bool skip_special_tokens = true) const {
    std::size_t len = 0;
    int rc = dsb_tokenizer_decode(handle(), ids.data(), ids.size(), skip_special_tokens ? 1 : 0, nullptr, 0, &len);
    if (rc != DSB_OK && len == 0) throw Error(rc, dsb_tokenizer_error());
    std::string s(len, '\0');
    rc = dsb_tokenizer_decode(handle(), ids.data(), ids.size(), skip_special_tokens ? 1 : 0, len ? &s[0] : nullptr,
                              s.size(), &len);
    if (rc != DSB_OK) throw Error(rc, dsb_tokenizer_error());
    return s;
  }

 private:
  const dsb_tokenizer* handle() const {
    if (!h_) throw Error(DSB_EINVAL, "tokenizer not loaded");
    return h_.get();
  }
  std::shared_ptr<dsb_tokenizer> h_;
  TokenizerMetadata meta_;
};

namespace detail {

// The device context and model a Model and its sessions share.
struct ModelState {
  dsb_ctx* ctx = nullptr;
  dsb_model* model = nullptr;
  dsb_model_config cfg{};
  ~ModelState() {
    if (model) dsb_model_destroy(model);
    if (ctx) dsb_ctx_destroy(ctx);
  }
  void check(int rc, const char* what) const {
    if (rc != DSB_OK) throw Error(rc, std::string(what) + ": " + dsb_last_error(ctx));
  }
};

}  // namespace detail

class Model;
class ModelSession;
class BatchSession;
inline std::vector<std::int32_t> generate(const Model& model, ModelSession& session,
                                          const std::vector<std::int32_t>& prompt_ids, const GenerationConfig& gen_cfg,
                                          const Tokenizer* tokenizer = nullptr,
                                          std::vector<std::string>* text_pieces = nullptr);

// One sequence's paged KV cache (ds::rt::ModelSession).
class ModelSession {
 public:
  ~ModelSession() {
    if (kv_) dsb_kvcache_destroy(kv_);
  }
  ModelSession(const ModelSession&) = delete;
  ModelSession& operator=(const ModelSession&) = delete;
  void reset() {
    st_->check(dsb_kvcache_free_seq(kv_, seq_), "dsb_kvcache_free_seq");
    st_->check(dsb_kvcache_alloc_seq(kv_, &seq_), "dsb_kvcache_alloc_seq");
    pos_ = 0;
  }
  std::size_t position() const { return pos_; }
  std::size_t max_seq() const { return max_seq_; }

 private:
  friend class Model;
  friend std::vector<std::int32_t> generate(const Model&, ModelSession&, const std::vector<std::int32_t>&,
                                            const GenerationConfig&, const Tokenizer*, std::vector<std::string>*);
  ModelSession(std::shared_ptr<detail::ModelState> st, std::size_t max_seq) : st_(std::move(st)), max_seq_(max_seq) {
    const int64_t pages = (int64_t)((max_seq_ + 63) / 64);
    st_->check(dsb_kvcache_create(st_->ctx, st_->model, pages, 1, (int)pages, &kv_), "dsb_kvcache_create");
    st_->check(dsb_kvcache_alloc_seq(kv_, &seq_), "dsb_kvcache_alloc_seq");
  }
  std::shared_ptr<detail::ModelState> st_;
  dsb_kvcache* kv_ = nullptr;
  int seq_ = -1;
  std::size_t pos_ = 0, max_seq_ = 0;
};

// A device-resident model (ds::rt::Model).
class Model {
 public:
  // ds::rt::load_model: a Hugging Face directory (config.json + safetensors)
  // uploaded to `device`.
  static std::shared_ptr<const Model> load(const std::string& model_dir, int device = 0) {
    dsb_checkpoint* ck = nullptr;
    int rc = dsb_checkpoint_open(model_dir.c_str(), &ck);
    if (rc != DSB_OK) throw Error(rc, dsb_checkpoint_error());
    std::unique_ptr<dsb_checkpoint, int (*)(dsb_checkpoint*)> ck_owner(ck, dsb_checkpoint_close);
    auto st = std::make_shared<detail::ModelState>();
    dsb_checkpoint_config(ck, &st->cfg);
    rc = dsb_ctx_create(device, &st->ctx);
    if (rc != DSB_OK) throw Error(rc, "dsb_ctx_create: no usable CUDA device " + std::to_string(device));
    st->check(dsb_model_create(st->ctx, &st->cfg, &st->model), "dsb_model_create");
    st->check(dsb_model_upload_checkpoint(st->model, ck, nullptr, nullptr), "dsb_model_upload_checkpoint");
    st->check(dsb_model_finalize(st->model), "dsb_model_finalize");
    std::shared_ptr<Model> m(new Model());
    m->st_ = std::move(st);
    m->info_.vocab_size = m->st_->cfg.vocab_size;
    m->info_.max_position_embeddings = m->st_->cfg.max_position_embeddings;
    m->info_.weights_fp8 = m->st_->cfg.weights_fp8 != 0;
    return m;
  }

  const ModelInfo& info() const { return info_; }

  std::unique_ptr<ModelSession> create_session(const RunConfig& run_cfg) const {
    const std::size_t limit = (std::size_t)std::max(1, info_.max_position_embeddings);
    const std::size_t max_seq = run_cfg.max_seq ? run_cfg.max_seq : limit;
    if (max_seq > limit) throw Error(DSB_EINVAL, "max_seq exceeds model max_position_embeddings");
    return std::unique_ptr<ModelSession>(new ModelSession(st_, max_seq));
  }

  // DeepSeekModel::forward: every input token in order (a prompt as one
  // batched prefill), the logits and greedy id after the last.
  ForwardOutput forward(ModelSession& s, const ForwardInput& input) const {
    const std::vector<std::int32_t>& ids = input.token_ids;
    if (ids.empty()) throw Error(DSB_EINVAL, "forward: empty input");
    if (s.pos_ + ids.size() > s.max_seq_) throw Error(DSB_EINVAL, "forward: sequence exceeds max_seq");
    ForwardOutput out;
    out.logits.assign((std::size_t)info_.vocab_size, 0.0f);
    if (ids.size() == 1) {
      st_->check(dsb_decode_step(st_->ctx, st_->model, s.kv_, &s.seq_, ids.data(), 1, out.logits.data(),
                                 &out.greedy_token_id),
                 "dsb_decode_step");
    } else {
      for (std::size_t c = 0; c < ids.size(); c += DSB_PREFILL_MAX_TOKENS) {
        const int n = (int)std::min<std::size_t>(DSB_PREFILL_MAX_TOKENS, ids.size() - c);
        const std::vector<std::int32_t> sid((std::size_t)n, s.seq_);
        int n_seq = 0;
        st_->check(dsb_prefill(st_->ctx, st_->model, s.kv_, sid.data(), ids.data() + c, n, out.logits.data(),
                               &out.greedy_token_id, &n_seq),
                   "dsb_prefill");
      }
    }
    s.pos_ += ids.size();
    out.position_after = s.pos_;
    return out;
  }

 private:
  friend std::vector<std::int32_t> generate(const Model&, ModelSession&, const std::vector<std::int32_t>&,
                                            const GenerationConfig&, const Tokenizer*, std::vector<std::string>*);
  friend class BatchSession;
  Model() = default;
  std::shared_ptr<detail::ModelState> st_;
  ModelInfo info_;
};

inline std::shared_ptr<const Model> load_model(const std::string& model_dir, int device = 0) {
  return Model::load(model_dir, device);
}

// ds::rt::generate (src/runtime/model.cpp:14-49): forward the prompt, then
// feed back each next id until max_new_tokens or the tokenizer's eos; the
// next id is greedy unless temperature, top_k or top_p is above 0, then it
// is sampled on the device with the Sampler's draw stream.
inline std::vector<std::int32_t> generate(const Model& model, ModelSession& session,
                                          const std::vector<std::int32_t>& prompt_ids, const GenerationConfig& gen_cfg,
                                          const Tokenizer* tokenizer, std::vector<std::string>* text_pieces) {
  if (gen_cfg.max_new_tokens <= 0) return {};
  if (prompt_ids.empty()) throw Error(DSB_EINVAL, "generate: empty prompt");
  const bool sampling = gen_cfg.temperature > 0.0f || gen_cfg.top_k > 0 || gen_cfg.top_p > 0.0f;
  const detail::ModelState& st = *model.st_;
  std::mt19937 rng;
  if (sampling) {
    if (gen_cfg.seed != 0) {
      rng.seed(gen_cfg.seed);
    } else {
      std::random_device rd;
      rng.seed(rd());
    }
  }
  const dsb_sampling smp{gen_cfg.temperature, gen_cfg.top_k, gen_cfg.top_p, gen_cfg.seed};
  // the id after feeding `ids`: the forward's greedy id, or a sampled one
  // (all but the last token by forward, the last through the sampled step)
  auto next_after = [&](const std::vector<std::int32_t>& ids) -> std::int32_t {
    if (!sampling) return model.forward(session, ForwardInput{ids}).greedy_token_id;
    if (ids.size() > 1) model.forward(session, ForwardInput{std::vector<std::int32_t>(ids.begin(), ids.end() - 1)});
    if (session.pos_ + 1 > session.max_seq_) throw Error(DSB_EINVAL, "generate: sequence exceeds max_seq");
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    const float u = dist(rng);
    std::int32_t id = 0;
    st.check(dsb_decode_step_sampled(st.ctx, st.model, session.kv_, &session.seq_, &ids.back(), 1, &smp, &u, nullptr,
                                     &id),
             "dsb_decode_step_sampled");
    session.pos_ += 1;
    return id;
  };
  const std::int32_t eos = tokenizer != nullptr && !tokenizer->empty() ? tokenizer->metadata().eos_token_id : -1;
  std::vector<std::int32_t> generated;
  std::int32_t next = next_after(prompt_ids);
  for (std::int32_t i = 0; i < gen_cfg.max_new_tokens; ++i) {
    generated.push_back(next);
    if (text_pieces != nullptr && tokenizer != nullptr && !tokenizer->empty())
      text_pieces->push_back(tokenizer->decode({next}));
    if (eos >= 0 && next == eos) break;
    if (i + 1 < gen_cfg.max_new_tokens) next = next_after({next});
  }
  return generated;
}

// The batched session the reference lacks: one paged cache shared by up to
// max_seqs sequences, stepped together (dsb_decode_step / dsb_prefill /
// dsb_generate).  Sequence ids come from add() and return through release().
class BatchSession {
 public:
  BatchSession(std::shared_ptr<const Model> model, int max_seqs, std::size_t max_seq)
      : model_(std::move(model)), st_(model_->st_) {
    if (max_seqs <= 0 || max_seq == 0 || max_seq > (std::size_t)std::max(1, model_->info().max_position_embeddings))
      throw Error(DSB_EINVAL, "BatchSession: bad sizes");
    const int64_t pages = (int64_t)((max_seq + 63) / 64);
    st_->check(dsb_kvcache_create(st_->ctx, st_->model, pages * max_seqs, max_seqs, (int)pages, &kv_),
               "dsb_kvcache_create");
  }
  ~BatchSession() {
    if (kv_) dsb_kvcache_destroy(kv_);
  }
  BatchSession(const BatchSession&) = delete;
  BatchSession& operator=(const BatchSession&) = delete;

  int add() {
    int seq = -1;
    st_->check(dsb_kvcache_alloc_seq(kv_, &seq), "dsb_kvcache_alloc_seq");
    return seq;
  }
  void release(int seq) { st_->check(dsb_kvcache_free_seq(kv_, seq), "dsb_kvcache_free_seq"); }
  std::size_t position(int seq) const {
    int len = 0;
    st_->check(dsb_kvcache_seq_len(kv_, seq, &len), "dsb_kvcache_seq_len");
    return (std::size_t)len;
  }

  // One token for each of the given (distinct) sequences; their greedy ids.
  std::vector<std::int32_t> step(const std::vector<int>& seqs, const std::vector<std::int32_t>& tokens) {
    if (seqs.size() != tokens.size() || seqs.empty()) throw Error(DSB_EINVAL, "BatchSession::step: bad arguments");
    std::vector<std::int32_t> next(seqs.size());
    st_->check(dsb_decode_step(st_->ctx, st_->model, kv_, seqs.data(), tokens.data(), (int)seqs.size(), nullptr,
                               next.data()),
               "dsb_decode_step");
    return next;
  }

  // ds::rt::generate for every sequence at once: prompts[i] continues
  // sequence seqs[i]; the generated ids per sequence (stopping at eos_id
  // when >= 0).
  std::vector<std::vector<std::int32_t>> generate(const std::vector<int>& seqs,
                                                  const std::vector<std::vector<std::int32_t>>& prompts,
                                                  const GenerationConfig& gen_cfg, std::int32_t eos_id = -1) {
    if (seqs.size() != prompts.size() || seqs.empty()) throw Error(DSB_EINVAL, "BatchSession::generate: bad arguments");
    const int B = (int)seqs.size(), n = std::max(0, gen_cfg.max_new_tokens);
    std::vector<std::int32_t> flat, offsets(1, 0);
    for (const auto& p : prompts) {
      flat.insert(flat.end(), p.begin(), p.end());
      offsets.push_back((std::int32_t)flat.size());
    }
    std::vector<std::int32_t> out((std::size_t)B * (std::size_t)std::max(1, n)), counts((std::size_t)B);
    const dsb_sampling smp{gen_cfg.temperature, gen_cfg.top_k, gen_cfg.top_p, gen_cfg.seed};
    st_->check(dsb_generate_sampled(st_->ctx, st_->model, kv_, seqs.data(), B, flat.data(), offsets.data(), n, eos_id,
                                    &smp, out.data(), counts.data()),
               "dsb_generate_sampled");
    std::vector<std::vector<std::int32_t>> res((std::size_t)B);
    for (int b = 0; b < B; ++b)
      res[(std::size_t)b].assign(out.begin() + (std::ptrdiff_t)b * std::max(1, n),
                                 out.begin() + (std::ptrdiff_t)b * std::max(1, n) + counts[(std::size_t)b]);
    return res;
  }

 private:
  std::shared_ptr<const Model> model_;
  std::shared_ptr<detail::ModelState> st_;
  dsb_kvcache* kv_ = nullptr;
};

// ds::rt::ModelExecutor: one model and one session.
class ModelExecutor {
 public:
  ModelExecutor(std::shared_ptr<const Model> model, RunConfig run_cfg)
      : model_(std::move(model)), session_(model_->create_session(run_cfg)) {}
  void reset() {
    session_->reset();
    pos_ = 0;
  }
  std::size_t position() const { return pos_; }
  const ModelInfo& info() const { return model_->info(); }
  StepResult prefill(const std::vector<std::int32_t>& prompt_ids) { return step(prompt_ids); }
  StepResult decode_next(std::int32_t token_id) { return step({token_id}); }
  std::vector<std::int32_t> generate(const std::vector<std::int32_t>& prompt_ids, const GenerationConfig& gen_cfg,
                                     const Tokenizer* tokenizer = nullptr,
                                     std::vector<std::string>* text_pieces = nullptr) {
    auto ids = rt::generate(*model_, *session_, prompt_ids, gen_cfg, tokenizer, text_pieces);
    pos_ = session_->position();
    return ids;
  }

 private:
  StepResult step(const std::vector<std::int32_t>& ids) {
    ForwardOutput out = model_->forward(*session_, ForwardInput{ids});
    pos_ = out.position_after;
    return StepResult{std::move(out.logits), out.greedy_token_id};
  }
  std::shared_ptr<const Model> model_;
  std::unique_ptr<ModelSession> session_;
  std::size_t pos_ = 0;
};

}  // namespace rt
}  // namespace dsb
