// The reference-side binding of the B200 speculative-decoding library: what a
// maintainer of islhkafaa/neural-network adds to route
// TransformerDecoder::generate_speculative (include/nn/layer.hpp:318-323) and
// generate_advanced with the KV cache (layer.hpp:312-317) to the device, with
// the public API unchanged.  Test infrastructure here: oracle/Makefile builds
// it with a copy of src/nn/layer.cpp into which oracle/bind_reference.py
// inserts the two dispatch calls below, against the reference's own headers.
//
// A model is put on the device by constructing it on a CudaSpecBackend (the
// ExecutionBackend* every layer constructor takes, layer.hpp:301-303).  The
// backend subclasses CpuBackend, so every tensor op outside the speculative
// path still runs on the host as before; the speculative path itself runs in
// libspecdec_b200.so through the C ABI of include/specdec.h.
#pragma once

#include <cstddef>
#include <memory>
#include <string>
#include <vector>

#include "backend/cpu_backend.hpp"
#include "specdec.h"

class TransformerDecoder;

class CudaSpecBackend : public CpuBackend {
public:
  // `cfg` gives the shapes of the target and draft decoders that will be
  // built on this backend (the reference's draft is its own decoder, so
  // draft_shares_target must be 0); the handle is created on first use, with
  // kv_dtype INT8 when a call asks for the quantized cache.
  CudaSpecBackend(const specdec_config &cfg, int device);
  ~CudaSpecBackend() override;
  // Weights are uploaded before the first call; after the caller changes
  // them (training, load_weights), mark them stale.
  void invalidate_weights() { uploaded_ = false; }
  // Device launches of the last generate call (0: the call stayed on the host).
  long long last_launches() const { return last_launches_; }

  bool generate_speculative(TransformerDecoder *target, TransformerDecoder *draft, const std::vector<size_t> &prompt,
                            size_t max_new_tokens, size_t lookahead, float temperature, size_t top_k, float top_p,
                            unsigned int seed, bool quantized_cache, std::vector<size_t> *out);
  bool generate_advanced(TransformerDecoder *target, const std::vector<size_t> &prompt, size_t max_new_tokens,
                         float temperature, size_t top_k, float top_p, unsigned int seed, std::vector<size_t> *out);

private:
  specdec_handle *handle(bool int8_kv);
  void upload(TransformerDecoder *m, int role);
  void check(int rc) const;

  specdec_config cfg_;
  int device_;
  bool int8_kv_ = false;
  bool uploaded_ = false;
  bool draft_uploaded_ = false;
  long long last_launches_ = 0;
  specdec_handle *h_ = nullptr;
};

// The calls bind_reference.py inserts at the top of the two methods: they
// return true with the tokens in *out when the model lives on a
// CudaSpecBackend, false (the method continues on the host) otherwise.
bool cuda_spec_dispatch_speculative(TransformerDecoder *target, ExecutionBackend *backend,
                                    TransformerDecoder *draft, const std::vector<size_t> &prompt,
                                    size_t max_new_tokens, size_t lookahead, float temperature, size_t top_k,
                                    float top_p, unsigned int seed, bool quantized_cache, std::vector<size_t> *out);
bool cuda_spec_dispatch_advanced(TransformerDecoder *target, ExecutionBackend *backend,
                                 const std::vector<size_t> &prompt, size_t max_new_tokens, float temperature,
                                 size_t top_k, float top_p, unsigned int seed, bool use_kv_cache,
                                 std::vector<size_t> *out);
