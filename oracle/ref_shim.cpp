// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// A thin extern "C" shim over the UNMODIFIED reference library
// (islhkafaa/neural-network), compiled from the reference's own sources by
// oracle/Makefile into oracle/_ref/libnnref.so.  It lets the pytest suite and
// bench.py's reference arm drive the reference's public C++ API from Python:
//
//   * TransformerDecoder construction (include/nn/layer.hpp:298-303),
//   * seeded weight injection through parameters() + copy_from_host, the same
//     pattern the reference's own tests use (tests/nn/gqa_test.cpp:56-62),
//   * TransformerDecoder::forward (src/nn/layer.cpp:1161-1193),
//   * generate / generate_advanced / generate_speculative
//     (src/nn/layer.cpp:1195-1661),
//   * Layer::save_weights / load_weights, the NETW v1 parameter file
//     (src/nn/layer.cpp:463-469, src/core/serialization.cpp:8-107),
//   * Tensor::rope (src/core/tensor.cpp:1126-1166) and the QuantizedDense
//     per-channel int8 quantiser (src/nn/quantization.cpp:7-66).
//
// Every entry returns 0 on success and -1 when the reference threw; the
// message is then available from nnref_last_error().
//
// Built with NNREF_CUDA (oracle/_ref/libnnref_cuda.so, the reference library
// with the B200 dispatch of oracle/binding/) it also makes decoders on a
// CudaSpecBackend, so the same calls reach libspecdec_b200.so.
#include "core/tensor.hpp"
#include "nn/layer.hpp"
#include "nn/quantization.hpp"
#ifdef NNREF_CUDA
#include "cuda_spec_backend.hpp"
#endif

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {
thread_local std::string g_err;

struct RefModel {
  std::unique_ptr<TransformerDecoder> dec;
  std::vector<std::shared_ptr<Tensor>> params;
  size_t vocab = 0;
};

template <class F> int guard(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return -1;
  } catch (...) {
    g_err = "unknown exception";
    return -1;
  }
}

std::vector<size_t> to_tokens(const int64_t *p, size_t n) {
  std::vector<size_t> v(n);
  for (size_t i = 0; i < n; ++i) v[i] = static_cast<size_t>(p[i]);
  return v;
}

void copy_out(const std::vector<size_t> &v, int64_t *out, size_t cap,
              size_t *n_out) {
  size_t n = v.size() < cap ? v.size() : cap;
  for (size_t i = 0; i < n; ++i) out[i] = static_cast<int64_t>(v[i]);
  if (n_out) *n_out = v.size();
}
} // namespace

extern "C" {

const char *nnref_last_error() { return g_err.c_str(); }

void *nnref_decoder_new(size_t vocab, size_t d_model, size_t n_heads,
                        size_t d_ff, size_t n_layers, size_t max_seq_len) {
  RefModel *m = nullptr;
  int rc = guard([&] {
    auto rm = std::make_unique<RefModel>();
    rm->dec = std::make_unique<TransformerDecoder>(vocab, d_model, n_heads,
                                                   d_ff, n_layers, max_seq_len);
    rm->params = rm->dec->parameters();
    rm->vocab = vocab;
    m = rm.release();
  });
  return rc == 0 ? m : nullptr;
}

void nnref_decoder_free(void *h) { delete static_cast<RefModel *>(h); }

#ifdef NNREF_CUDA
// A CudaSpecBackend for decoders of the given target / draft shapes (the
// fields of specdec_config after draft_shares_target are taken as given).
void *nnref_cuda_backend_new(const specdec_config *cfg, int device) {
  CudaSpecBackend *be = nullptr;
  int rc = guard([&] { be = new CudaSpecBackend(*cfg, device); });
  return rc == 0 ? be : nullptr;
}
void nnref_cuda_backend_free(void *be) { delete static_cast<CudaSpecBackend *>(be); }
long long nnref_cuda_backend_launches(void *be) { return static_cast<CudaSpecBackend *>(be)->last_launches(); }

// TransformerDecoder constructed on the backend (include/nn/layer.hpp:301-303).
void *nnref_decoder_new_on(void *be, size_t vocab, size_t d_model, size_t n_heads, size_t d_ff, size_t n_layers,
                           size_t max_seq_len) {
  RefModel *m = nullptr;
  int rc = guard([&] {
    auto rm = std::make_unique<RefModel>();
    rm->dec = std::make_unique<TransformerDecoder>(vocab, d_model, n_heads, d_ff, n_layers, max_seq_len,
                                                   static_cast<CudaSpecBackend *>(be));
    rm->params = rm->dec->parameters();
    rm->vocab = vocab;
    m = rm.release();
  });
  return rc == 0 ? m : nullptr;
}
#endif

int nnref_num_params(void *h) {
  return static_cast<int>(static_cast<RefModel *>(h)->params.size());
}

size_t nnref_param_numel(void *h, int i) {
  auto *m = static_cast<RefModel *>(h);
  return count_elements(m->params.at(static_cast<size_t>(i))->shape());
}

int nnref_set_param(void *h, int i, const float *data, size_t n) {
  return guard([&] {
    auto *m = static_cast<RefModel *>(h);
    auto &t = m->params.at(static_cast<size_t>(i));
    if (count_elements(t->shape()) != n)
      throw std::runtime_error("nnref_set_param: element count mismatch");
    t->copy_from_host(std::vector<float>(data, data + n));
  });
}

int nnref_get_param(void *h, int i, float *data, size_t n) {
  return guard([&] {
    auto *m = static_cast<RefModel *>(h);
    auto v = m->params.at(static_cast<size_t>(i))->to_host();
    if (v.size() != n)
      throw std::runtime_error("nnref_get_param: element count mismatch");
    std::memcpy(data, v.data(), n * sizeof(float));
  });
}

// requires_grad selects the reference's attention path: with every parameter
// grad-free the fused ThreadPool kernel runs (src/nn/layer.cpp:811-952), as it
// does for QuantizedDense models; with the constructor default (true) the
// unfused bmm/softmax path runs (src/nn/layer.cpp:953-990).
void nnref_set_requires_grad(void *h, int flag) {
  auto *m = static_cast<RefModel *>(h);
  for (auto &t : m->params) t->set_requires_grad(flag != 0);
}

// Plain forward over one sequence without a cache; logits is [S, V].
int nnref_forward(void *h, const int64_t *tokens, size_t S, float *logits) {
  return guard([&] {
    auto *m = static_cast<RefModel *>(h);
    std::vector<float> in(S);
    for (size_t i = 0; i < S; ++i) in[i] = static_cast<float>(tokens[i]);
    auto t = std::make_shared<Tensor>(Shape{1, S}, in);
    // Inference: Dropout off, as generate*() do (src/nn/layer.cpp:1389-1392).
    m->dec->set_training(false);
    auto out = m->dec->forward(t)->to_host();
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
  });
}

int nnref_generate(void *h, const int64_t *prompt, size_t S, size_t max_new,
                   int64_t *out, size_t cap, size_t *n_out) {
  return guard([&] {
    auto *m = static_cast<RefModel *>(h);
    copy_out(m->dec->generate(to_tokens(prompt, S), max_new), out, cap, n_out);
  });
}

int nnref_generate_advanced(void *h, const int64_t *prompt, size_t S,
                            size_t max_new, float temperature, size_t top_k,
                            float top_p, unsigned seed, int use_kv_cache,
                            int64_t *out, size_t cap, size_t *n_out) {
  return guard([&] {
    auto *m = static_cast<RefModel *>(h);
    copy_out(m->dec->generate_advanced(to_tokens(prompt, S), max_new,
                                       temperature, top_k, top_p, seed,
                                       use_kv_cache != 0),
             out, cap, n_out);
  });
}

int nnref_generate_speculative(void *target, void *draft, const int64_t *prompt,
                               size_t S, size_t max_new, size_t lookahead,
                               float temperature, size_t top_k, float top_p,
                               unsigned seed, int quantized_cache, int64_t *out,
                               size_t cap, size_t *n_out) {
  return guard([&] {
    auto *t = static_cast<RefModel *>(target);
    auto *d = static_cast<RefModel *>(draft);
    copy_out(t->dec->generate_speculative(
                 d->dec.get(), to_tokens(prompt, S), max_new, lookahead,
                 temperature, top_k, top_p, seed, quantized_cache != 0),
             out, cap, n_out);
  });
}

// Layer::save_weights / Layer::load_weights of the decoder.
int nnref_save_weights(void *h, const char *path) {
  return guard([&] { static_cast<RefModel *>(h)->dec->save_weights(path); });
}
int nnref_load_weights(void *h, const char *path) {
  return guard([&] { static_cast<RefModel *>(h)->dec->load_weights(path); });
}

// Tensor::rope on a [B, H, S, D] tensor at offset S_past.
int nnref_rope(const float *in, size_t B, size_t H, size_t S, size_t D,
               size_t S_past, float *out) {
  return guard([&] {
    size_t n = B * H * S * D;
    auto t = std::make_shared<Tensor>(Shape{B, H, S, D},
                                      std::vector<float>(in, in + n));
    auto r = t->rope(S_past)->to_host();
    std::memcpy(out, r.data(), n * sizeof(float));
  });
}

// QuantizedDense(INT8) over a [in, out] weight: per-output-channel scales,
// int8 codes and the dequantised weight the reference multiplies with.
int nnref_quantize_int8(const float *w, size_t in_f, size_t out_f,
                        float *scales, int8_t *q, float *dequant) {
  return guard([&] {
    auto base = std::make_shared<Dense>(in_f, out_f);
    base->parameters()[0]->copy_from_host(
        std::vector<float>(w, w + in_f * out_f));
    QuantizationConfig cfg{QuantizationType::INT8};
    QuantizedDense qd(base, cfg);
    auto s = qd.scales()->to_host();
    std::memcpy(scales, s.data(), out_f * sizeof(float));
    const auto &pk = qd.packed_weights();
    for (size_t i = 0; i < in_f * out_f; ++i)
      q[i] = static_cast<int8_t>(pk[i]);
    auto dq = qd.dequantize_weight()->to_host();
    std::memcpy(dequant, dq.data(), dq.size() * sizeof(float));
  });
}

} // extern "C"
