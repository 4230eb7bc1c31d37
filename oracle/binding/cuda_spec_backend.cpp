// CudaSpecBackend: see cuda_spec_backend.hpp.
#include "cuda_spec_backend.hpp"

#include <algorithm>
#include <stdexcept>

#include "core/tensor.hpp"
#include "nn/layer.hpp"

CudaSpecBackend::CudaSpecBackend(const specdec_config &cfg, int device) : cfg_(cfg), device_(device) {
  if (cfg_.draft_shares_target)
    throw std::runtime_error("CudaSpecBackend: the reference's draft is its own decoder (draft_shares_target = 0)");
}

CudaSpecBackend::~CudaSpecBackend() { specdec_destroy(h_); }

void CudaSpecBackend::check(int rc) const {
  if (rc != SPECDEC_OK) throw std::runtime_error(specdec_last_error(h_));  // the reference's error type
}

specdec_handle *CudaSpecBackend::handle(bool int8_kv) {
  if (h_ && int8_kv == int8_kv_) return h_;
  // quantized_cache selects the cache type, fixed per handle: a call that
  // asks for the other one gets a new handle (and a new upload)
  specdec_destroy(h_);
  h_ = nullptr;
  specdec_config c = cfg_;
  c.kv_dtype = int8_kv ? SPECDEC_INT8 : cfg_.kv_dtype;
  if (specdec_create(&c, device_, &h_) != SPECDEC_OK)
    throw std::runtime_error(std::string("specdec_create: ") + specdec_last_error(nullptr));
  int8_kv_ = int8_kv;
  uploaded_ = draft_uploaded_ = false;
  return h_;
}

// parameters() in order, the pattern of tests/nn/gqa_test.cpp:56-62 in reverse.
void CudaSpecBackend::upload(TransformerDecoder *m, int role) {
  auto ps = m->parameters();
  std::vector<std::vector<float>> host;
  host.reserve(ps.size());
  for (auto &p : ps) host.push_back(p->to_host());
  std::vector<const float *> ptrs;
  std::vector<int64_t> numels;
  for (auto &v : host) {
    ptrs.push_back(v.data());
    numels.push_back(static_cast<int64_t>(v.size()));
  }
  check(specdec_load_params(h_, role, static_cast<int>(ptrs.size()), ptrs.data(), numels.data()));
}

bool CudaSpecBackend::generate_speculative(TransformerDecoder *target, TransformerDecoder *draft,
                                           const std::vector<size_t> &prompt, size_t max_new_tokens,
                                           size_t lookahead, float temperature, size_t top_k, float top_p,
                                           unsigned int seed, bool quantized_cache, std::vector<size_t> *out) {
  handle(quantized_cache);
  if (!uploaded_) {
    upload(target, SPECDEC_TARGET);
    uploaded_ = true;
    draft_uploaded_ = false;
  }
  if (!draft_uploaded_) {
    upload(draft, SPECDEC_DRAFT);
    draft_uploaded_ = true;
  }
  std::vector<int32_t> p(prompt.begin(), prompt.end());
  std::vector<int32_t> o(prompt.size() + std::max<size_t>(1, max_new_tokens));
  specdec_gen_params gp{};
  gp.max_new_tokens = static_cast<int32_t>(max_new_tokens);
  gp.lookahead = static_cast<int32_t>(lookahead);
  gp.temperature = temperature;
  gp.top_k = static_cast<int32_t>(top_k);
  gp.top_p = top_p;
  gp.rng_mode = SPECDEC_RNG_MT19937;      // the reference's std::mt19937 gen(seed)
  gp.seed = seed;
  gp.draft_catchup = SPECDEC_CATCHUP_REF; // the reference's draft catch-up (src/nn/layer.cpp:1632-1655)
  check(specdec_generate(h_, &gp, p.data(), 1, static_cast<int>(p.size()), o.data(), nullptr));
  last_launches_ = specdec_last_launch_count(h_);
  out->assign(o.begin(), o.end());
  return true;
}

bool CudaSpecBackend::generate_advanced(TransformerDecoder *target, const std::vector<size_t> &prompt,
                                        size_t max_new_tokens, float temperature, size_t top_k, float top_p,
                                        unsigned int seed, std::vector<size_t> *out) {
  handle(int8_kv_);
  if (!uploaded_) {
    upload(target, SPECDEC_TARGET);
    uploaded_ = true;
    draft_uploaded_ = false;
  }
  std::vector<int32_t> p(prompt.begin(), prompt.end());
  std::vector<int32_t> o(prompt.size() + max_new_tokens);
  specdec_gen_params gp{};
  gp.max_new_tokens = static_cast<int32_t>(max_new_tokens);
  gp.temperature = temperature;
  gp.top_k = static_cast<int32_t>(top_k);
  gp.top_p = top_p;
  gp.rng_mode = SPECDEC_RNG_MT19937;
  gp.seed = seed;
  check(specdec_generate_ar(h_, &gp, p.data(), 1, static_cast<int>(p.size()), o.data(), nullptr));
  last_launches_ = specdec_last_launch_count(h_);
  out->assign(o.begin(), o.end());
  return true;
}

bool cuda_spec_dispatch_speculative(TransformerDecoder *target, ExecutionBackend *backend,
                                    TransformerDecoder *draft, const std::vector<size_t> &prompt,
                                    size_t max_new_tokens, size_t lookahead, float temperature, size_t top_k,
                                    float top_p, unsigned int seed, bool quantized_cache, std::vector<size_t> *out) {
  auto *be = dynamic_cast<CudaSpecBackend *>(backend);  // the idiom of src/nn/layer.cpp:506, 546
  if (!be) return false;
  return be->generate_speculative(target, draft, prompt, max_new_tokens, lookahead, temperature, top_k, top_p, seed,
                                  quantized_cache, out);
}

bool cuda_spec_dispatch_advanced(TransformerDecoder *target, ExecutionBackend *backend,
                                 const std::vector<size_t> &prompt, size_t max_new_tokens, float temperature,
                                 size_t top_k, float top_p, unsigned int seed, bool use_kv_cache,
                                 std::vector<size_t> *out) {
  auto *be = dynamic_cast<CudaSpecBackend *>(backend);
  // use_kv_cache = false recomputes the whole window each step: host path
  if (!be || !use_kv_cache) return false;
  return be->generate_advanced(target, prompt, max_new_tokens, temperature, top_k, top_p, seed, out);
}
