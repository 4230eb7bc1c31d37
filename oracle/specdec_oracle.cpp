// TEST INFRASTRUCTURE ONLY — the CPU checker for the B200 speculative-decoding
// path.  Nothing in the product library links, loads or calls this file; only
// tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it.
//
// A plain-C++ restatement of the reference's speculative-decoding hot path
// (islhkafaa/neural-network), written from its behaviour:
//
//   forward ............ TransformerDecoder::forward      src/nn/layer.cpp:1161-1193
//   decoder layer ...... TransformerDecoderLayer::forward src/nn/layer.cpp:1097-1114
//   attention + cache .. MultiHeadAttention::forward      src/nn/layer.cpp:593-994
//   int8 KV ............ quantize_kv lambda                src/nn/layer.cpp:635-665
//   RoPE ............... Tensor::rope                      src/core/tensor.cpp:1126-1166
//   LayerNorm .......... LayerNorm::forward                src/nn/layer.cpp:242-261
//   SwiGLU ............. SwiGLU::forward                   src/nn/layer.cpp:1704-1710
//   int8 weights ....... QuantizedDense                    src/nn/quantization.cpp:7-147
//   get_probs .......... lambda                            src/nn/layer.cpp:1410-1491
//   sample_token ....... lambda                            src/nn/layer.cpp:1493-1498
//   spec-decode loop ... generate_speculative              src/nn/layer.cpp:1382-1661
//   AR comparator ...... generate_advanced                 src/nn/layer.cpp:1240-1380
//
// Extensions the reference does not have (each is a switch; the defaults are the
// reference's behaviour):
//   * batch: B independent batch-1 requests (request b seeded with seed + b);
//   * rng_mode 1: a host-supplied uniform table u[b][round][slot] replaces the
//     std::mt19937 stream (slot j < k: draft sample j; slot k + j: acceptance
//     draw j; slot 2k: residual or bonus sample; round 0 slot 2k: first token);
//     a sample is then the first i whose fp64 running sum exceeds u * total;
//   * catchup 1: the draft cache is rolled back consistently (the reference
//     feeds the recovered token to the draft twice after a rejection,
//     src/nn/layer.cpp:1632-1642 then 1542);
//   * act_bf16: activations rounded to bf16 at the points where the CUDA kernels
//     store them (embedding out, q, attention out, each residual sum, each
//     LayerNorm out, FFN hidden); kv_mode 1 stores K/V as bf16;
//   * arch 1 ("cfg"): pre-LN, GELU (erf form) FFN, learned positional embedding,
//     final LayerNorm; parameter order is this file's own (no reference twin).
//
// The uniform and sampling conventions of std::mt19937 / discrete_distribution /
// uniform_real_distribution are the C++ standard library's (libstdc++ of GCC
// 13.3 on this image); this file calls them directly, as the reference does.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;

// ---------------------------------------------------------------------------
// bf16 round-to-nearest-even, as include/core/dtype.hpp:83-96 (bias 0x7fff+lsb).
inline float bf16_round(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {  // inf / nan: truncate
    u &= 0xffff0000u;
  } else {
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    u &= 0xffff0000u;
  }
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

struct ModelCfg {
  int32_t vocab, d_model, n_heads, n_kv_heads, d_ff, n_layers, max_seq_len;
  int32_t arch;  // 0 = reference TransformerDecoder, 1 = cfg variant
};

struct Numerics {
  int32_t act_bf16;
  int32_t kv_mode;  // 0 fp32, 1 bf16, 2 int8 per (head, position)
};

struct Dense {
  int in = 0, out = 0;
  std::vector<float> w;  // [in, out] row-major, the reference layout (layer.cpp:153)
  std::vector<float> b;  // [out]
};

struct Layer {
  Dense q, k, v, o;          // attention projections
  Dense gate, up, down;      // ref arch (SwiGLU)
  Dense fc1, fc2;            // cfg arch (GELU)
  std::vector<float> n1g, n1b, n2g, n2b;
};

struct Model {
  ModelCfg c{};
  std::vector<float> emb;   // [V, d]
  std::vector<float> pos;   // [max_seq, d] (cfg)
  std::vector<Layer> layers;
  std::vector<float> nfg, nfb;  // final LN (cfg)
  Dense head;
  std::vector<std::pair<float *, size_t>> params;  // parameters() order
};

void init_dense(Dense &d, int in, int out) {
  d.in = in;
  d.out = out;
  d.w.assign(static_cast<size_t>(in) * out, 0.f);
  d.b.assign(out, 0.f);
}

void build_params(Model &m) {
  auto &p = m.params;
  p.clear();
  auto add = [&](std::vector<float> &v) { p.emplace_back(v.data(), v.size()); };
  auto addd = [&](Dense &d) { add(d.w); add(d.b); };
  add(m.emb);
  if (m.c.arch == 1) add(m.pos);
  for (auto &L : m.layers) {
    if (m.c.arch == 0) {
      // TransformerDecoderLayer::parameters (layer.cpp:1079-1090): attn, ffn, n1, n2
      addd(L.q); addd(L.k); addd(L.v); addd(L.o);
      addd(L.gate); addd(L.up); addd(L.down);
      add(L.n1g); add(L.n1b); add(L.n2g); add(L.n2b);
    } else {
      add(L.n1g); add(L.n1b);
      addd(L.q); addd(L.k); addd(L.v); addd(L.o);
      add(L.n2g); add(L.n2b);
      addd(L.fc1); addd(L.fc2);
    }
  }
  if (m.c.arch == 1) { add(m.nfg); add(m.nfb); }
  addd(m.head);
}

Model *new_model(const ModelCfg &c) {
  if (c.d_model % c.n_heads) throw std::runtime_error("embed_dim must be divisible by num_heads");
  int hkv = c.n_kv_heads ? c.n_kv_heads : c.n_heads;
  if (c.n_heads % hkv) throw std::runtime_error("num_heads must be divisible by num_kv_heads");
  if ((c.d_model / c.n_heads) % 2) throw std::runtime_error("rope: head dimension D must be even");
  auto m = std::make_unique<Model>();
  m->c = c;
  m->c.n_kv_heads = hkv;
  int d = c.d_model, D = d / c.n_heads;
  m->emb.assign(static_cast<size_t>(c.vocab) * d, 0.f);
  if (c.arch == 1) m->pos.assign(static_cast<size_t>(c.max_seq_len) * d, 0.f);
  m->layers.resize(c.n_layers);
  for (auto &L : m->layers) {
    init_dense(L.q, d, d);
    init_dense(L.k, d, hkv * D);
    init_dense(L.v, d, hkv * D);
    init_dense(L.o, d, d);
    if (c.arch == 0) {
      init_dense(L.gate, d, c.d_ff);
      init_dense(L.up, d, c.d_ff);
      init_dense(L.down, c.d_ff, d);
    } else {
      init_dense(L.fc1, d, c.d_ff);
      init_dense(L.fc2, c.d_ff, d);
    }
    L.n1g.assign(d, 1.f); L.n1b.assign(d, 0.f);
    L.n2g.assign(d, 1.f); L.n2b.assign(d, 0.f);
  }
  if (c.arch == 1) { m->nfg.assign(d, 1.f); m->nfb.assign(d, 0.f); }
  init_dense(m->head, d, c.vocab);
  build_params(*m);
  return m.release();
}

// QuantizedDense(INT8) (quantization.cpp:40-66 and 89-103): per-output-column
// scale max|W[:,c]|/127 (0 -> 1), q = clamp(round(W/s), +-127); the forward then
// multiplies by the dequantised weight q*s (quantization.cpp:127-147).
void quantize_dense(Dense &d) {
  std::vector<float> s(d.out, 1.f);
  for (int c = 0; c < d.out; ++c) {
    float mx = 0.f;
    for (int r = 0; r < d.in; ++r) mx = std::max(mx, std::abs(d.w[static_cast<size_t>(r) * d.out + c]));
    float sc = mx / 127.0f;
    s[c] = (sc == 0.0f) ? 1.0f : sc;
  }
  for (int r = 0; r < d.in; ++r)
    for (int c = 0; c < d.out; ++c) {
      size_t i = static_cast<size_t>(r) * d.out + c;
      float q = std::round(d.w[i] / s[c]);
      q = std::max(-127.0f, std::min(127.0f, q));
      d.w[i] = static_cast<float>(static_cast<int8_t>(q)) * s[c];
    }
}

// ---------------------------------------------------------------------------
// Per-request KV cache: [layer][head_kv][position][D], fixed capacity.
struct Cache {
  int len = 0;
  int cap = 0;
  std::vector<std::vector<float>> k, v;              // fp32 / bf16-rounded values
  std::vector<std::vector<int8_t>> kq, vq;           // int8 mode
  std::vector<std::vector<float>> ks, vs;            // int8 scales [hkv][pos]
};

void cache_init(Cache &c, const Model &m, int cap, int kv_mode) {
  int D = m.c.d_model / m.c.n_heads, hkv = m.c.n_kv_heads, L = m.c.n_layers;
  c.len = 0;
  c.cap = cap;
  size_t n = static_cast<size_t>(hkv) * cap * D;
  c.k.assign(L, std::vector<float>(kv_mode == 2 ? 0 : n, 0.f));
  c.v.assign(L, std::vector<float>(kv_mode == 2 ? 0 : n, 0.f));
  if (kv_mode == 2) {
    c.kq.assign(L, std::vector<int8_t>(n, 0));
    c.vq.assign(L, std::vector<int8_t>(n, 0));
    c.ks.assign(L, std::vector<float>(static_cast<size_t>(hkv) * cap, 1.f));
    c.vs.assign(L, std::vector<float>(static_cast<size_t>(hkv) * cap, 1.f));
  }
}

// y[S, out] = x[S, in] . W + b  (Dense::forward, layer.cpp:162-171: matmul then add)
void dense_fwd(const Dense &d, const float *x, int S, float *y) {
  std::vector<float> acc(d.out);
  for (int r = 0; r < S; ++r) {
    std::fill(acc.begin(), acc.end(), 0.f);
    const float *xr = x + static_cast<size_t>(r) * d.in;
    for (int k = 0; k < d.in; ++k) {
      float xv = xr[k];
      const float *wr = d.w.data() + static_cast<size_t>(k) * d.out;
      for (int n = 0; n < d.out; ++n) acc[n] += xv * wr[n];
    }
    float *yr = y + static_cast<size_t>(r) * d.out;
    for (int n = 0; n < d.out; ++n) yr[n] = acc[n] + d.b[n];
  }
}

// LayerNorm::forward (layer.cpp:242-261): mean, diff, biased var, / sqrt(var+eps).
void layernorm(const float *x, int S, int d, const std::vector<float> &g,
               const std::vector<float> &b, float *y) {
  const float eps = 1e-5f;
  float N = static_cast<float>(d);
  for (int r = 0; r < S; ++r) {
    const float *xr = x + static_cast<size_t>(r) * d;
    float *yr = y + static_cast<size_t>(r) * d;
    float s = 0.f;
    for (int i = 0; i < d; ++i) s += xr[i];
    float mean = s / N;
    float v = 0.f;
    for (int i = 0; i < d; ++i) { float df = xr[i] - mean; v += df * df; }
    float var = v / N;
    float sd = std::sqrt(var + eps);
    for (int i = 0; i < d; ++i) yr[i] = ((xr[i] - mean) / sd) * g[i] + b[i];
  }
}

inline void round_vec(float *p, size_t n, bool on) {
  if (!on) return;
  for (size_t i = 0; i < n; ++i) p[i] = bf16_round(p[i]);
}

// Tensor::rope (tensor.cpp:1144-1163): interleaved pairs (2j, 2j+1) rotated by
// m * 10000^(-2j/D), all in fp32 with std::pow / std::cos / std::sin.
void rope_row(float *v, int D, int m_pos) {
  float m = static_cast<float>(m_pos);
  for (int j = 0; j < D / 2; ++j) {
    float theta = std::pow(10000.0f, -2.0f * static_cast<float>(j) / static_cast<float>(D));
    float omega = m * theta;
    float c = std::cos(omega), s = std::sin(omega);
    float xe = v[2 * j], xo = v[2 * j + 1];
    v[2 * j] = xe * c - xo * s;
    v[2 * j + 1] = xe * s + xo * c;
  }
}

// quantize_kv (layer.cpp:635-665) for one [D] row.
void quant_kv_row(const float *src, int D, int8_t *q, float *scale) {
  float mx = 0.f;
  for (int d = 0; d < D; ++d) mx = std::max(mx, std::abs(src[d]));
  float s = mx / 127.0f;
  if (s == 0.0f) s = 1.0f;
  *scale = s;
  float inv = 1.0f / s;
  for (int d = 0; d < D; ++d) {
    float qv = std::round(src[d] * inv);
    qv = std::max(-127.0f, std::min(127.0f, qv));
    q[d] = static_cast<int8_t>(qv);
  }
}

// One forward over S new tokens of one request at positions cache.len ... (+S-1).
// Appends K/V, returns logits [S, V].  Throws like layer.cpp:1176-1179 when the
// cache capacity would be exceeded.
void forward(const Model &m, const Numerics &nm, Cache &cache, const int64_t *tok,
             int S, std::vector<float> &logits) {
  const ModelCfg &c = m.c;
  const int d = c.d_model, H = c.n_heads, hkv = c.n_kv_heads, D = d / H, F = c.d_ff;
  const int grp = H / hkv;
  const int S_past = cache.len;
  const bool bf = nm.act_bf16 != 0;
  if (S_past + S > cache.cap)
    throw std::runtime_error("Sequence length S plus past cached length exceeds max_seq_len");

  std::vector<float> x(static_cast<size_t>(S) * d);
  // Embedding (cpu_backend.cpp:998-1033): out-of-range ids read row 0.
  for (int s = 0; s < S; ++s) {
    int64_t id = tok[s];
    if (id < 0 || id >= c.vocab) id = 0;
    std::memcpy(&x[static_cast<size_t>(s) * d], &m.emb[static_cast<size_t>(id) * d], d * sizeof(float));
    if (c.arch == 1)
      for (int i = 0; i < d; ++i) x[static_cast<size_t>(s) * d + i] += m.pos[static_cast<size_t>(S_past + s) * d + i];
  }
  round_vec(x.data(), x.size(), bf);

  std::vector<float> q(static_cast<size_t>(S) * d), kk(static_cast<size_t>(S) * hkv * D),
      vv(static_cast<size_t>(S) * hkv * D), att(static_cast<size_t>(S) * d),
      tmp(static_cast<size_t>(S) * d), h1(static_cast<size_t>(S) * d), x1(static_cast<size_t>(S) * d),
      ga(static_cast<size_t>(S) * F), up(static_cast<size_t>(S) * F), y(static_cast<size_t>(S) * d);
  std::vector<float> scores;
  const float scale = std::sqrt(static_cast<float>(D));

  for (int l = 0; l < c.n_layers; ++l) {
    const Layer &L = m.layers[l];
    const float *ain = x.data();
    if (c.arch == 1) {  // pre-LN
      layernorm(x.data(), S, d, L.n1g, L.n1b, x1.data());
      round_vec(x1.data(), x1.size(), bf);
      ain = x1.data();
    }
    dense_fwd(L.q, ain, S, q.data());
    dense_fwd(L.k, ain, S, kk.data());
    dense_fwd(L.v, ain, S, vv.data());
    for (int s = 0; s < S; ++s) {
      for (int h = 0; h < H; ++h) rope_row(&q[static_cast<size_t>(s) * d + h * D], D, S_past + s);
      for (int h = 0; h < hkv; ++h) rope_row(&kk[static_cast<size_t>(s) * hkv * D + h * D], D, S_past + s);
    }
    round_vec(q.data(), q.size(), bf);
    // KV append at positions S_past + s (layer.cpp:667-809).
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < hkv; ++h) {
        size_t dst = (static_cast<size_t>(h) * cache.cap + S_past + s) * D;
        const float *ks = &kk[static_cast<size_t>(s) * hkv * D + h * D];
        const float *vs = &vv[static_cast<size_t>(s) * hkv * D + h * D];
        if (nm.kv_mode == 2) {
          quant_kv_row(ks, D, &cache.kq[l][dst], &cache.ks[l][static_cast<size_t>(h) * cache.cap + S_past + s]);
          quant_kv_row(vs, D, &cache.vq[l][dst], &cache.vs[l][static_cast<size_t>(h) * cache.cap + S_past + s]);
        } else {
          for (int e = 0; e < D; ++e) {
            cache.k[l][dst + e] = nm.kv_mode == 1 ? bf16_round(ks[e]) : ks[e];
            cache.v[l][dst + e] = nm.kv_mode == 1 ? bf16_round(vs[e]) : vs[e];
          }
        }
      }
    // Causal attention, fused-path arithmetic (layer.cpp:859-948).
    const int S_tot = S_past + S;
    scores.resize(S_tot);
    for (int s = 0; s < S; ++s)
      for (int h = 0; h < H; ++h) {
        int hk = h / grp;
        const float *qr = &q[static_cast<size_t>(s) * d + h * D];
        float mx = -std::numeric_limits<float>::infinity();
        int last = S_past + s;  // mask j > S_past + i
        for (int j = 0; j <= last; ++j) {
          size_t base = (static_cast<size_t>(hk) * cache.cap + j) * D;
          float dot = 0.f;
          if (nm.kv_mode == 2) {
            float ksc = cache.ks[l][static_cast<size_t>(hk) * cache.cap + j];
            for (int e = 0; e < D; ++e) dot += qr[e] * (static_cast<float>(cache.kq[l][base + e]) * ksc);
          } else {
            for (int e = 0; e < D; ++e) dot += qr[e] * cache.k[l][base + e];
          }
          float sc = dot / scale;
          scores[j] = sc;
          if (sc > mx) mx = sc;
        }
        float sum = 0.f;
        for (int j = 0; j <= last; ++j) { float e = std::exp(scores[j] - mx); scores[j] = e; sum += e; }
        float inv = 1.0f / sum;
        for (int j = 0; j <= last; ++j) scores[j] *= inv;
        float *orow = &att[static_cast<size_t>(s) * d + h * D];
        for (int e = 0; e < D; ++e) {
          float acc = 0.f;
          for (int j = 0; j <= last; ++j) {
            if (scores[j] == 0.0f) continue;
            size_t base = (static_cast<size_t>(hk) * cache.cap + j) * D;
            float vvv = nm.kv_mode == 2
                            ? static_cast<float>(cache.vq[l][base + e]) * cache.vs[l][static_cast<size_t>(hk) * cache.cap + j]
                            : cache.v[l][base + e];
            acc += scores[j] * vvv;
          }
          orow[e] = acc;
        }
      }
    round_vec(att.data(), att.size(), bf);
    dense_fwd(L.o, att.data(), S, tmp.data());
    if (c.arch == 0) {
      // x1 = norm1(x + attn) ; x = norm2(x1 + ffn(x1))   (layer.cpp:1097-1114)
      for (size_t i = 0; i < h1.size(); ++i) h1[i] = x[i] + tmp[i];
      round_vec(h1.data(), h1.size(), bf);
      layernorm(h1.data(), S, d, L.n1g, L.n1b, x1.data());
      round_vec(x1.data(), x1.size(), bf);
      dense_fwd(L.gate, x1.data(), S, ga.data());
      dense_fwd(L.up, x1.data(), S, up.data());
      // SwiGLU (layer.cpp:1704-1710): gate * sigmoid(gate) * up; sigmoid = 1/(1+exp(-x))
      for (size_t i = 0; i < ga.size(); ++i) {
        float g = ga[i];
        float sg = 1.0f / (1.0f + std::exp(-g));
        ga[i] = (g * sg) * up[i];
      }
      round_vec(ga.data(), ga.size(), bf);
      dense_fwd(L.down, ga.data(), S, tmp.data());
      for (size_t i = 0; i < h1.size(); ++i) h1[i] = x1[i] + tmp[i];
      round_vec(h1.data(), h1.size(), bf);
      layernorm(h1.data(), S, d, L.n2g, L.n2b, x.data());
      round_vec(x.data(), x.size(), bf);
    } else {
      for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + tmp[i];
      round_vec(x.data(), x.size(), bf);
      layernorm(x.data(), S, d, L.n2g, L.n2b, x1.data());
      round_vec(x1.data(), x1.size(), bf);
      dense_fwd(L.fc1, x1.data(), S, ga.data());
      for (size_t i = 0; i < ga.size(); ++i) {
        float g = ga[i];
        ga[i] = 0.5f * g * (1.0f + std::erf(g * 0.70710678118654752f));
      }
      round_vec(ga.data(), ga.size(), bf);
      dense_fwd(L.fc2, ga.data(), S, tmp.data());
      for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + tmp[i];
      round_vec(x.data(), x.size(), bf);
    }
  }
  const float *hin = x.data();
  if (c.arch == 1) {
    layernorm(x.data(), S, d, m.nfg, m.nfb, x1.data());
    round_vec(x1.data(), x1.size(), bf);
    hin = x1.data();
  }
  logits.resize(static_cast<size_t>(S) * c.vocab);
  dense_fwd(m.head, hin, S, logits.data());
  cache.len = S_past + S;
}

// KVCache::truncate (layer.cpp:67-149): only ever shortens.
inline void truncate(Cache &c, int len) {
  if (len < c.len) c.len = len;
}

// ---------------------------------------------------------------------------
// get_probs (layer.cpp:1410-1491).
std::vector<float> get_probs(const float *logits, int V, float T, int top_k, float top_p) {
  std::vector<float> probs(V, 0.f);
  if (T <= 0.0f) {
    float mx = logits[0];
    int am = 0;
    for (int v = 1; v < V; ++v)
      if (logits[v] > mx) { mx = logits[v]; am = v; }
    probs[am] = 1.0f;
    return probs;
  }
  std::vector<float> sl(logits, logits + V);
  for (int v = 0; v < V; ++v) sl[v] /= T;
  float mx = sl[0];
  for (int v = 1; v < V; ++v)
    if (sl[v] > mx) mx = sl[v];
  float sum = 0.f;
  for (int v = 0; v < V; ++v) { probs[v] = std::exp(sl[v] - mx); sum += probs[v]; }
  for (int v = 0; v < V; ++v) probs[v] /= sum;
  std::vector<std::pair<float, size_t>> ip(V);
  for (int v = 0; v < V; ++v) ip[v] = {probs[v], static_cast<size_t>(v)};
  std::sort(ip.begin(), ip.end(), [](const auto &a, const auto &b) { return a.first > b.first; });
  if (top_k > 0 && top_k < V)
    for (int i = top_k; i < V; ++i) ip[i].first = 0.0f;
  if (top_p > 0.0f && top_p < 1.0f) {
    float cum = 0.f;
    bool cut = false;
    for (int i = 0; i < V; ++i) {
      if (cut) ip[i].first = 0.0f;
      else { cum += ip[i].first; if (cum >= top_p) cut = true; }
    }
  }
  float fs = 0.f;
  for (int v = 0; v < V; ++v) fs += ip[v].first;
  std::vector<float> out(V, 0.f);
  if (fs <= 0.0f) out[ip[0].second] = 1.0f;
  else
    for (int v = 0; v < V; ++v) out[ip[v].second] = ip[v].first / fs;
  return out;
}

inline int argmax_first(const float *p, int V) {
  int am = 0;
  float mx = p[0];
  for (int v = 1; v < V; ++v)
    if (p[v] > mx) { mx = p[v]; am = v; }
  return am;
}

// Uniform sources.  Mode 0 is the reference's std::mt19937 stream; mode 1 reads
// a host table.  `margin` records how close a decision came to flipping, so the
// parity tests can tell near-ties from real mismatches.
struct Rng {
  int mode = 0;
  std::mt19937 gen;
  const float *table = nullptr;  // this request's [n_rounds][2k+1]
  int n_rounds = 0, slots = 0;

  float table_u(int round, int slot) const {
    if (round >= n_rounds) throw std::runtime_error("uniform table too short");
    return table[static_cast<size_t>(round) * slots + slot];
  }
};

// sample_token (layer.cpp:1493-1498).  Mode 1: first i with fp64 running sum
// C_i > u * C_{V-1}.
int sample(Rng &rng, const std::vector<float> &p, int round, int slot, double *margin) {
  const int V = static_cast<int>(p.size());
  if (rng.mode == 0) {
    std::vector<double> np(p.begin(), p.end());
    std::discrete_distribution<size_t> dist(np.begin(), np.end());
    // margin: distance of the drawn uniform from the nearest CDF boundary needs
    // the uniform itself; replay the draw on a copy of the engine.
    std::mt19937 probe = rng.gen;
    size_t tok = dist(rng.gen);
    if (margin) {
      double u = std::generate_canonical<double, std::numeric_limits<double>::digits>(probe);
      double tot = 0.0;
      for (double x : np) tot += x;
      double cum = 0.0, best = 1e300;
      for (int i = 0; i < V; ++i) {
        cum += np[i] / tot;
        best = std::min(best, std::abs(cum - u));
      }
      *margin = std::min(*margin, best);
    }
    return static_cast<int>(tok);
  }
  double u = rng.table_u(round, slot);
  double tot = 0.0;
  for (int i = 0; i < V; ++i) tot += static_cast<double>(p[i]);
  double thr = u * tot;
  double cum = 0.0;
  int pick = -1, last_nz = 0;
  double best = 1e300;
  for (int i = 0; i < V; ++i) {
    if (p[i] > 0.f) last_nz = i;
    cum += static_cast<double>(p[i]);
    best = std::min(best, std::abs(cum - thr) / (tot > 0 ? tot : 1.0));
    if (pick < 0 && cum > thr) pick = i;
  }
  if (margin) *margin = std::min(*margin, best);
  return pick < 0 ? last_nz : pick;
}

float accept_uniform(Rng &rng, int round, int slot) {
  if (rng.mode == 0) {
    std::uniform_real_distribution<float> ud(0.0f, 1.0f);
    return ud(rng.gen);
  }
  return rng.table_u(round, slot);
}

struct SpecParams {
  int32_t max_new, lookahead;
  float temperature;
  int32_t top_k;
  float top_p;
  int32_t rng_mode;
  uint32_t seed;
  const float *uniforms;  // [B][n_rounds][2k+1]
  int32_t n_rounds;
  int32_t catchup;        // 0 = reference behaviour, 1 = consistent rollback
  Numerics num;
  int32_t cache_cap;      // 0 -> the model's max_seq_len
};

// Per-request statistics: [rounds, drafted, accepted, rejections].
void spec_one(const Model &tgt, const Model &dft, const SpecParams &sp, const int64_t *prompt,
              int S, int b, int64_t *out, int64_t *stats, double *margins) {
  const int V = tgt.c.vocab;
  const int k = sp.lookahead;
  const float T = sp.temperature;
  Rng rng;
  rng.mode = sp.rng_mode;
  rng.gen.seed(sp.seed + static_cast<uint32_t>(b));
  rng.slots = 2 * k + 1;
  rng.n_rounds = sp.n_rounds;
  if (sp.rng_mode == 1) rng.table = sp.uniforms + static_cast<size_t>(b) * sp.n_rounds * rng.slots;

  Cache tc, dc;
  cache_init(tc, tgt, sp.cache_cap ? sp.cache_cap : tgt.c.max_seq_len, sp.num.kv_mode);
  cache_init(dc, dft, sp.cache_cap ? sp.cache_cap : dft.c.max_seq_len, sp.num.kv_mode);

  std::vector<int64_t> gen(prompt, prompt + S);
  std::vector<float> tl, dl;
  forward(tgt, sp.num, tc, prompt, S, tl);
  forward(dft, sp.num, dc, prompt, S, dl);

  double mg = 1e300;
  auto tok_margin = [&](const float *lg) {
    // greedy: gap between the top two logits, relative to the top one
    float a = -INFINITY, bb = -INFINITY;
    for (int v = 0; v < V; ++v) {
      if (lg[v] > a) { bb = a; a = lg[v]; }
      else if (lg[v] > bb) bb = lg[v];
    }
    return static_cast<double>(a - bb) / std::max(1e-30, static_cast<double>(std::abs(a)));
  };
  auto note = [&](size_t idx) {
    if (margins && idx < static_cast<size_t>(sp.max_new)) margins[idx] = mg;
    mg = 1e300;
  };

  const float *last_row = &tl[static_cast<size_t>(S - 1) * V];
  auto p0 = get_probs(last_row, V, T, sp.top_k, sp.top_p);
  if (T <= 0.0f) mg = std::min(mg, tok_margin(last_row));
  int first = sample(rng, p0, 0, 2 * k, T > 0 ? &mg : nullptr);
  gen.push_back(first);
  note(0);
  int ngen = 1;
  int64_t rounds = 0, drafted = 0, accepted_n = 0, rejections = 0;

  while (ngen < sp.max_new) {
    int M = std::min(k, sp.max_new - ngen);
    if (M == 0) break;
    int round = static_cast<int>(rounds) + 1;
    rounds++;
    int t_start = tc.len, d_start = dc.len;
    std::vector<int64_t> cand;
    std::vector<std::vector<float>> qs;
    std::vector<double> qmarg;
    for (int j = 0; j < M; ++j) {
      int64_t in = (j == 0) ? gen.back() : cand.back();
      forward(dft, sp.num, dc, &in, 1, dl);
      auto q = get_probs(dl.data(), V, T, sp.top_k, sp.top_p);
      double m1 = 1e300;
      if (T <= 0.0f) m1 = tok_margin(dl.data());
      int c = sample(rng, q, round, j, T > 0 ? &m1 : nullptr);
      qmarg.push_back(m1);
      cand.push_back(c);
      qs.push_back(std::move(q));
    }
    drafted += M;
    std::vector<int64_t> tin(M + 1);
    tin[0] = gen.back();
    for (int i = 0; i < M; ++i) tin[i + 1] = cand[i];
    forward(tgt, sp.num, tc, tin.data(), M + 1, tl);
    std::vector<std::vector<float>> ps(M + 1);
    for (int i = 0; i <= M; ++i) ps[i] = get_probs(&tl[static_cast<size_t>(i) * V], V, T, sp.top_k, sp.top_p);

    bool all = true;
    int rj = 0;
    for (int j = 0; j < M; ++j) {
      int x = static_cast<int>(cand[j]);
      float q = qs[j][x], p = ps[j][x];
      bool acc;
      mg = std::min(mg, qmarg[j]);
      if (T <= 0.0f) {
        mg = std::min(mg, tok_margin(&tl[static_cast<size_t>(j) * V]));
        acc = (x == argmax_first(ps[j].data(), V));
      } else {
        float r = accept_uniform(rng, round, k + j);
        acc = (r * q < p);
        mg = std::min(mg, static_cast<double>(std::abs(r * q - p)));
      }
      if (acc) {
        gen.push_back(x);
        note(static_cast<size_t>(ngen));
        ngen++;
        accepted_n++;
      } else {
        all = false;
        rj = j;
        break;
      }
    }
    if (!all) {
      rejections++;
      std::vector<float> pr(V, 0.f);
      float sr = 0.f;
      for (int v = 0; v < V; ++v) { pr[v] = std::max(0.0f, ps[rj][v] - qs[rj][v]); sr += pr[v]; }
      int rec;
      if (T <= 0.0f) mg = std::min(mg, tok_margin(&tl[static_cast<size_t>(rj) * V]));
      if (sr <= 0.0f) rec = sample(rng, ps[rj], round, 2 * k, T > 0 ? &mg : nullptr);
      else {
        for (int v = 0; v < V; ++v) pr[v] /= sr;
        rec = sample(rng, pr, round, 2 * k, T > 0 ? &mg : nullptr);
      }
      gen.push_back(rec);
      note(static_cast<size_t>(ngen));
      ngen++;
      truncate(tc, t_start + rj + 1);
      truncate(dc, d_start + rj + 1);
      if (sp.catchup == 0) {
        int64_t in = rec;  // layer.cpp:1639-1642
        forward(dft, sp.num, dc, &in, 1, dl);
      }
    } else if (ngen < sp.max_new) {
      if (T <= 0.0f) mg = std::min(mg, tok_margin(&tl[static_cast<size_t>(M) * V]));
      int fin = sample(rng, ps[M], round, 2 * k, T > 0 ? &mg : nullptr);
      gen.push_back(fin);
      note(static_cast<size_t>(ngen));
      ngen++;
      int64_t in = cand[M - 1];  // layer.cpp:1649-1653
      forward(dft, sp.num, dc, &in, 1, dl);
    }
  }
  std::copy(gen.begin(), gen.end(), out);
  if (stats) {
    stats[0] = rounds;
    stats[1] = drafted;
    stats[2] = accepted_n;
    stats[3] = rejections;
  }
}

// ---------------------------------------------------------------------------
// Tree speculation (no counterpart in the reference).  Per round the draft
// expands a token tree level by level: every node at depth l < L gets the
// branch[l] most likely next tokens of the draft as children (largest
// logits, ties to the lower id).  The target scores every node; acceptance
// walks from the root, trying a node's children in rank order as point-mass
// proposals: greedy accepts the child equal to the target's argmax; sampled
// accepts child c when u < p(c) and otherwise sets p(c) = 0 and renormalises
// p, which samples exactly from p.  When no child is accepted the token is
// drawn from the remaining p; after an accepted leaf a bonus token is drawn
// from the leaf's p.  Here each node's logits come from running the model on
// the committed sequence plus the node's path (what an ancestor-masked tree
// forward computes).  Uniform slots per round: depth * bmax + rank for the
// test of a child, L * bmax for the drawn token.
struct TreeParams {
  int32_t depth;
  int32_t branch[8];
};

int tree_nodes(const TreeParams &tp) {
  int n = 0, level = 1;
  for (int l = 0; l < tp.depth; ++l) {
    level *= tp.branch[l];
    n += level;
  }
  return n;
}

// the `b` largest logits (ties to the lower id), best first
std::vector<int> top_b(const float *lg, int V, int b, double *margin) {
  std::vector<int> idx(V);
  for (int v = 0; v < V; ++v) idx[v] = v;
  std::stable_sort(idx.begin(), idx.end(), [&](int x, int y) { return lg[x] > lg[y]; });
  idx.resize(b);
  if (margin && b < V) {
    std::vector<float> srt(lg, lg + V);
    std::sort(srt.begin(), srt.end(), std::greater<float>());
    const double gap = static_cast<double>(srt[b - 1] - srt[b]) / std::max(1e-30, static_cast<double>(std::abs(srt[b - 1])));
    *margin = std::min(*margin, gap);
  }
  return idx;
}

void tree_one(const Model &tgt, const Model &dft, const SpecParams &sp, const TreeParams &tp, const int64_t *prompt,
              int S, int b, int64_t *out, int64_t *stats, double *margins) {
  const int V = tgt.c.vocab;
  const float T = sp.temperature;
  const int L = tp.depth;
  int bmax = 1;
  for (int l = 0; l < L; ++l) bmax = std::max(bmax, tp.branch[l]);
  const int nslots = L * bmax + 1;
  Rng rng;
  rng.mode = sp.rng_mode;
  rng.gen.seed(sp.seed + static_cast<uint32_t>(b));
  rng.slots = nslots;
  rng.n_rounds = sp.n_rounds;
  if (sp.rng_mode == 1) rng.table = sp.uniforms + static_cast<size_t>(b) * sp.n_rounds * nslots;

  Cache tc, dc;
  cache_init(tc, tgt, sp.cache_cap ? sp.cache_cap : tgt.c.max_seq_len, sp.num.kv_mode);
  cache_init(dc, dft, sp.cache_cap ? sp.cache_cap : dft.c.max_seq_len, sp.num.kv_mode);
  std::vector<int64_t> gen(prompt, prompt + S);
  std::vector<float> tl, dl;
  forward(tgt, sp.num, tc, prompt, S, tl);
  forward(dft, sp.num, dc, prompt, S, dl);

  double mg = 1e300;
  auto tok_margin = [&](const float *lg) {
    float a = -INFINITY, bb = -INFINITY;
    for (int v = 0; v < V; ++v) {
      if (lg[v] > a) { bb = a; a = lg[v]; }
      else if (lg[v] > bb) bb = lg[v];
    }
    return static_cast<double>(a - bb) / std::max(1e-30, static_cast<double>(std::abs(a)));
  };
  auto note = [&](size_t idx) {
    if (margins && idx < static_cast<size_t>(sp.max_new)) margins[idx] = mg;
    mg = 1e300;
  };
  const float *last_row = &tl[static_cast<size_t>(S - 1) * V];
  auto p0 = get_probs(last_row, V, T, sp.top_k, sp.top_p);
  if (T <= 0.0f) mg = std::min(mg, tok_margin(last_row));
  gen.push_back(sample(rng, p0, 0, L * bmax, T > 0 ? &mg : nullptr));
  note(0);
  int ngen = 1;
  int64_t rounds = 0, drafted = 0, accepted_n = 0, rejections = 0;

  // tree structure (BFS order): node j's parent and depth
  const int N = tree_nodes(tp);
  std::vector<int> parent(N), depth(N), first_child(N + 1, -1);
  {
    int base = 0, prev_base = -1, level = 1;
    for (int l = 0; l < L; ++l) {
      const int nl = level * tp.branch[l];
      for (int i = 0; i < nl; ++i) {
        parent[base + i] = l == 0 ? -1 : prev_base + i / tp.branch[l];
        depth[base + i] = l + 1;
      }
      prev_base = base;
      base += nl;
      level = nl;
    }
  }
  while (ngen < sp.max_new) {
    const int round = static_cast<int>(++rounds);
    const int Leff = std::min(L, sp.max_new - ngen);
    const int64_t root = gen.back();
    // draft expansion: caches after root + path, per node
    std::vector<int64_t> tok(N);
    std::vector<Cache> dcs(N + 1);  // [N] = after the root
    dcs[N] = dc;
    forward(dft, sp.num, dcs[N], &root, 1, dl);
    std::vector<std::vector<float>> dlog(N + 1);
    dlog[N] = dl;
    int base = 0, level = 1;
    for (int l = 0; l < L; ++l) {
      const int nl = level * tp.branch[l];
      for (int i = 0; i < nl; ++i) {
        const int j = base + i;
        const int par = parent[j] < 0 ? N : parent[j];
        const int rank = i % tp.branch[l];
        if (rank == 0) {
          double m1 = 1e300;
          auto kids = top_b(dlog[par].data(), V, tp.branch[l], &m1);
          mg = std::min(mg, m1);
          for (int r = 0; r < tp.branch[l]; ++r) tok[j + r] = kids[r];
        }
        if (l + 1 < L) {  // leaves are not fed to the draft
          dcs[j] = dcs[par];
          forward(dft, sp.num, dcs[j], &tok[j], 1, dl);
          dlog[j] = dl;
        }
      }
      base += nl;
      level = nl;
    }
    drafted += N;
    // target scores: root and every node
    std::vector<std::vector<float>> tlog(N + 1);
    std::vector<Cache> tcs(N + 1);
    tcs[N] = tc;
    forward(tgt, sp.num, tcs[N], &root, 1, tl);
    tlog[N] = tl;
    for (int j = 0; j < N; ++j) {
      const int par = parent[j] < 0 ? N : parent[j];
      tcs[j] = tcs[par];
      forward(tgt, sp.num, tcs[j], &tok[j], 1, tl);
      tlog[j] = tl;
    }
    tcs.clear();
    dcs.clear();
    // acceptance walk
    int node = N, d = 0, child0 = 0, nb = tp.branch[0];  // root's children start at node 0
    std::vector<int64_t> path;
    bool rejected = false;
    int out_tok = -1;
    auto children_of = [&](int nd, int dd, int &c0, int &cnt) {
      cnt = tp.branch[dd];
      if (nd == N) { c0 = 0; return; }
      // BFS: children of node nd (depth dd) start at level_base(dd+1) + (nd - level_base(dd)) * branch[dd]
      int lb = 0, lv = 1, lb_next = 0;
      for (int l = 0; l < dd; ++l) { lv *= tp.branch[l]; if (l + 1 < dd) lb += lv; }
      lb_next = lb + lv;
      c0 = lb_next + (nd - lb) * tp.branch[dd];
    };
    while (d < Leff) {
      int c0, cnt;
      children_of(node, d, c0, cnt);
      (void)child0; (void)nb;
      const float *lg = tlog[node].data();
      int acc = -1;
      if (T <= 0.0f) {
        mg = std::min(mg, tok_margin(lg));
        const int am = argmax_first(lg, V);
        for (int r = 0; r < cnt; ++r)
          if (tok[c0 + r] == am) { acc = c0 + r; break; }
        if (acc < 0) out_tok = am;
      } else {
        auto p = get_probs(lg, V, T, sp.top_k, sp.top_p);
        for (int r = 0; r < cnt && acc < 0; ++r) {
          const int c = static_cast<int>(tok[c0 + r]);
          const float u = accept_uniform(rng, round, d * bmax + r);
          mg = std::min(mg, static_cast<double>(std::abs(u - p[c])));
          if (u < p[c]) {
            acc = c0 + r;
          } else {
            p[c] = 0.0f;
            float s = 0.f;
            for (int v = 0; v < V; ++v) s += p[v];
            if (s > 0.f)
              for (int v = 0; v < V; ++v) p[v] /= s;
          }
        }
        if (acc < 0) out_tok = sample(rng, p, round, L * bmax, &mg);
      }
      if (acc < 0) {
        rejected = true;
        break;
      }
      path.push_back(tok[acc]);
      gen.push_back(tok[acc]);
      note(static_cast<size_t>(ngen));
      ngen++;
      accepted_n++;
      node = acc;
      d++;
    }
    if (rejected) {
      rejections++;
      gen.push_back(out_tok);
      note(static_cast<size_t>(ngen));
      ngen++;
    } else if (ngen < sp.max_new) {
      const float *lg = tlog[node].data();
      int fin;
      if (T <= 0.0f) {
        mg = std::min(mg, tok_margin(lg));
        fin = argmax_first(lg, V);
      } else {
        auto p = get_probs(lg, V, T, sp.top_k, sp.top_p);
        fin = sample(rng, p, round, L * bmax, &mg);
      }
      gen.push_back(fin);
      note(static_cast<size_t>(ngen));
      ngen++;
    }
    // commit root + accepted path to both caches
    std::vector<int64_t> commit(1, root);
    commit.insert(commit.end(), path.begin(), path.end());
    forward(tgt, sp.num, tc, commit.data(), static_cast<int>(commit.size()), tl);
    forward(dft, sp.num, dc, commit.data(), static_cast<int>(commit.size()), dl);
  }
  std::copy(gen.begin(), gen.end(), out);
  if (stats) {
    stats[0] = rounds;
    stats[1] = drafted;
    stats[2] = accepted_n;
    stats[3] = rejections;
  }
}

template <class F> int guard(F &&f) {
  try {
    f();
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return -1;
  }
}

}  // namespace

extern "C" {

const char *oc_last_error() { return g_err.c_str(); }

void *oc_model_new(const ModelCfg *c) {
  Model *m = nullptr;
  guard([&] { m = new_model(*c); });
  return m;
}
void oc_model_free(void *m) { delete static_cast<Model *>(m); }
int oc_model_num_params(void *m) { return static_cast<int>(static_cast<Model *>(m)->params.size()); }
int64_t oc_model_param_numel(void *m, int i) {
  return static_cast<int64_t>(static_cast<Model *>(m)->params.at(i).second);
}
int oc_model_set_param(void *mp, int i, const float *data, int64_t n) {
  return guard([&] {
    auto &p = static_cast<Model *>(mp)->params.at(i);
    if (static_cast<int64_t>(p.second) != n) throw std::runtime_error("oc_model_set_param: numel mismatch");
    std::memcpy(p.first, data, n * sizeof(float));
  });
}
int oc_model_get_param(void *mp, int i, float *data, int64_t n) {
  return guard([&] {
    auto &p = static_cast<Model *>(mp)->params.at(i);
    if (static_cast<int64_t>(p.second) != n) throw std::runtime_error("oc_model_get_param: numel mismatch");
    std::memcpy(data, p.first, n * sizeof(float));
  });
}
// Replaces every Dense weight (attention, FFN and lm_head) by its int8
// dequantisation q*s, exactly the matrix QuantizedDense multiplies with.
int oc_model_quantize_int8(void *mp) {
  return guard([&] {
    auto *m = static_cast<Model *>(mp);
    for (auto &L : m->layers) {
      for (Dense *d : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down, &L.fc1, &L.fc2})
        if (!d->w.empty()) quantize_dense(*d);
    }
    quantize_dense(m->head);
  });
}

// Full forward of one sequence without reuse of a cache; logits [S, V].
int oc_forward(void *mp, const Numerics *nm, const int64_t *tokens, int S, float *logits) {
  return guard([&] {
    auto *m = static_cast<Model *>(mp);
    Cache c;
    cache_init(c, *m, std::max(S, 1), nm->kv_mode);
    std::vector<float> lg;
    forward(*m, *nm, c, tokens, S, lg);
    std::memcpy(logits, lg.data(), lg.size() * sizeof(float));
  });
}

// Chunked forward through a cache: chunk sizes in `chunks` (sum = S); the logits
// of every chunk are concatenated into [S, V].  Exercises cache reuse exactly as
// prefill + decode steps do.
int oc_forward_chunked(void *mp, const Numerics *nm, const int64_t *tokens, const int32_t *chunks,
                       int n_chunks, float *logits) {
  return guard([&] {
    auto *m = static_cast<Model *>(mp);
    int S = 0;
    for (int i = 0; i < n_chunks; ++i) S += chunks[i];
    Cache c;
    cache_init(c, *m, std::max(S, 1), nm->kv_mode);
    std::vector<float> lg;
    int off = 0;
    for (int i = 0; i < n_chunks; ++i) {
      forward(*m, *nm, c, tokens + off, chunks[i], lg);
      std::memcpy(logits + static_cast<size_t>(off) * m->c.vocab, lg.data(), lg.size() * sizeof(float));
      off += chunks[i];
    }
  });
}

// B independent requests with equal prompt length S; out [B][S + max_new].
// stats [B][4] = rounds, drafted, accepted drafts, rejections.  margins
// [B][max_new] (optional) = the smallest decision margin seen while producing
// each new token (greedy: relative top-2 logit gap; sampled: |r*q - p| and the
// distance of the uniform to the nearest CDF boundary).
int oc_generate_speculative(void *tgt, void *dft, const SpecParams *sp, const int64_t *prompts,
                            int B, int S, int64_t *out, int64_t *stats, double *margins,
                            int n_threads) {
  return guard([&] {
    auto *t = static_cast<Model *>(tgt);
    auto *d = static_cast<Model *>(dft);
    if (t->c.vocab != d->c.vocab) throw std::runtime_error("target and draft vocab differ");
    const size_t row = static_cast<size_t>(S) + sp->max_new;
    std::vector<std::string> errs(B);
    auto work = [&](int b) {
      try {
        spec_one(*t, *d, *sp, prompts + static_cast<size_t>(b) * S, S, b, out + b * row,
                 stats ? stats + 4 * b : nullptr, margins ? margins + static_cast<size_t>(b) * sp->max_new : nullptr);
      } catch (const std::exception &e) {
        errs[b] = e.what();
      }
    };
    int nt = n_threads > 0 ? n_threads : static_cast<int>(std::thread::hardware_concurrency());
    nt = std::max(1, std::min(nt, B));
    std::vector<std::thread> th;
    for (int w = 0; w < nt; ++w)
      th.emplace_back([&, w] {
        for (int b = w; b < B; b += nt) work(b);
      });
    for (auto &x : th) x.join();
    for (auto &e : errs)
      if (!e.empty()) throw std::runtime_error(e);
  });
}

// Tree speculation for B requests (tree_one), threads over requests.
int oc_generate_tree(void *tgt, void *dft, const SpecParams *sp, const TreeParams *tp, const int64_t *prompts, int B,
                     int S, int64_t *out, int64_t *stats, double *margins, int n_threads) {
  return guard([&] {
    auto *t = static_cast<Model *>(tgt);
    auto *d = static_cast<Model *>(dft);
    if (t->c.vocab != d->c.vocab) throw std::runtime_error("target and draft vocab differ");
    if (tp->depth < 1 || tp->depth > 8) throw std::runtime_error("tree depth must be 1..8");
    for (int l = 0; l < tp->depth; ++l)
      if (tp->branch[l] < 1 || tp->branch[l] > t->c.vocab) throw std::runtime_error("bad tree branching");
    const size_t row = static_cast<size_t>(S) + sp->max_new;
    std::vector<std::string> errs(B);
    auto work = [&](int b) {
      try {
        tree_one(*t, *d, *sp, *tp, prompts + static_cast<size_t>(b) * S, S, b, out + b * row,
                 stats ? stats + 4 * b : nullptr, margins ? margins + static_cast<size_t>(b) * sp->max_new : nullptr);
      } catch (const std::exception &e) {
        errs[b] = e.what();
      }
    };
    int nt = n_threads > 0 ? n_threads : static_cast<int>(std::thread::hardware_concurrency());
    nt = std::max(1, std::min(nt, B));
    std::vector<std::thread> th;
    for (int w = 0; w < nt; ++w)
      th.emplace_back([&, w] {
        for (int b = w; b < B; b += nt) work(b);
      });
    for (auto &x : th) x.join();
    for (auto &e : errs)
      if (!e.empty()) throw std::runtime_error(e);
  });
}

// generate_advanced with the KV cache (layer.cpp:1240-1380), batch 1.
int oc_generate_advanced(void *mp, const Numerics *nm, const int64_t *prompt, int S, int max_new,
                         float T, int top_k, float top_p, uint32_t seed, int64_t *out) {
  return guard([&] {
    auto *m = static_cast<Model *>(mp);
    const int V = m->c.vocab;
    std::mt19937 gen(seed);
    Cache c;
    cache_init(c, *m, m->c.max_seq_len, nm->kv_mode);
    std::vector<int64_t> g(prompt, prompt + S);
    std::vector<float> lg;
    for (int step = 0; step < max_new; ++step) {
      if (step == 0) forward(*m, *nm, c, prompt, S, lg);
      else { int64_t in = g.back(); forward(*m, *nm, c, &in, 1, lg); }
      int rows = static_cast<int>(lg.size() / V);
      const float *row = &lg[static_cast<size_t>(rows - 1) * V];
      int next;
      if (T <= 0.0f) next = argmax_first(row, V);
      else {
        auto p = get_probs(row, V, T, top_k, top_p);
        std::vector<double> np(p.begin(), p.end());
        std::discrete_distribution<size_t> dist(np.begin(), np.end());
        next = static_cast<int>(dist(gen));
      }
      g.push_back(next);
    }
    std::copy(g.begin(), g.end(), out);
  });
}

// generate_advanced (src/nn/layer.cpp:1239-1380, use_kv_cache = true) for B
// independent requests with the uniform sources of the speculative path:
// request b draws from mt19937(seed + b) (rng_mode 0) or from
// uniforms[b][step][0] (rng_mode 1, n_rounds >= max_new rows of one slot).
// margins[b][step]: the decision margin of each token (greedy: relative top-2
// logit gap; sampled: distance of the uniform to a CDF boundary).
int oc_generate_ar(void *mp, const Numerics *nm, const int64_t *prompts, int B, int S, int max_new, float T,
                   int top_k, float top_p, int rng_mode, uint32_t seed, const float *uniforms, int n_rounds,
                   int64_t *out, double *margins) {
  return guard([&] {
    auto *m = static_cast<Model *>(mp);
    const int V = m->c.vocab;
    for (int b = 0; b < B; ++b) {
      Rng rng;
      rng.mode = rng_mode;
      rng.gen.seed(seed + static_cast<uint32_t>(b));
      rng.slots = 1;
      rng.n_rounds = n_rounds;
      if (rng_mode == 1) rng.table = uniforms + static_cast<size_t>(b) * n_rounds;
      Cache c;
      cache_init(c, *m, m->c.max_seq_len, nm->kv_mode);
      const int64_t *prompt = prompts + static_cast<size_t>(b) * S;
      std::vector<int64_t> g(prompt, prompt + S);
      std::vector<float> lg;
      for (int step = 0; step < max_new; ++step) {
        double mg = 1e300;
        if (step == 0) forward(*m, *nm, c, prompt, S, lg);
        else { int64_t in = g.back(); forward(*m, *nm, c, &in, 1, lg); }
        const int rows = static_cast<int>(lg.size() / V);
        const float *row = &lg[static_cast<size_t>(rows - 1) * V];
        int next;
        if (T <= 0.0f) {
          next = argmax_first(row, V);
          float a = -INFINITY, bb = -INFINITY;
          for (int v = 0; v < V; ++v) {
            if (row[v] > a) { bb = a; a = row[v]; }
            else if (row[v] > bb) bb = row[v];
          }
          mg = std::min(mg, static_cast<double>(a - bb) / std::max(1e-30, static_cast<double>(std::abs(a))));
        } else {
          next = sample(rng, get_probs(row, V, T, top_k, top_p), step, 0, &mg);
        }
        g.push_back(next);
        if (margins) margins[static_cast<size_t>(b) * max_new + step] = mg;
      }
      std::copy(g.begin(), g.end(), out + static_cast<size_t>(b) * (S + max_new));
    }
  });
}

// get_probs + sample on one logits row, for unit tests of the sampler alone.
int oc_get_probs(const float *logits, int V, float T, int top_k, float top_p, float *probs) {
  return guard([&] {
    auto p = get_probs(logits, V, T, top_k, top_p);
    std::memcpy(probs, p.data(), V * sizeof(float));
  });
}

int oc_rope(const float *in, int rows, int D, const int32_t *pos, float *out) {
  return guard([&] {
    for (int r = 0; r < rows; ++r) {
      std::memcpy(out + static_cast<size_t>(r) * D, in + static_cast<size_t>(r) * D, D * sizeof(float));
      rope_row(out + static_cast<size_t>(r) * D, D, pos[r]);
    }
  });
}

// The first n outputs of std::mt19937 seeded with `seed`.
void oc_mt19937(uint32_t seed, int n, uint32_t *out) {
  std::mt19937 g(seed);
  for (int i = 0; i < n; ++i) out[i] = static_cast<uint32_t>(g());
}

}  // extern "C"
