// TEST INFRASTRUCTURE — CPU oracle for the ragged hybrid-Qwen decode step.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
// load this library; the product library never links or calls it.
//
// This file restates, in FP64 scalar C++, the reference's per-layer math:
//   quantized affine projection / embedding  native/projection_reference.h:8-30
//   RMSNorm, SiLU, partial RoPE              native/operator_reference.h:9-18
//   Gated-DeltaNet conv + recurrence         native/operator_reference.h:19-45
//   softmax routing + renormalisation        native/operator_reference.h:47-57
//   causal GQA attention                     native/attention_reference.h:8-21
//   layer wiring and state layout            native/qwen_model.inc:75-206,268-373
//   total-order greedy selection             native/selection.h:3-12, src/serving/choices.rs:65-79
//   speculative accept plan                  src/serving/native_speculative.rs:74-128
// plus the ragged packing and token->expert sort rules this project defines
// (the reference has no ragged batch; its sort is mx::argsort, qwen_model.inc:81).
//
// Parity status: the scalar operators are pinned against the reference's own
// oracle headers and judge known-answer vectors (tests/golden). The whole-model
// forward has no archived reference output (the reference's tiny-model test
// compares MLX CPU vs GPU only, src/serving/qwen_tests.rs:256-310): it is a
// composition of pinned operators following qwen_model.inc's wiring.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../include/qwen_b200.h"
#include "synth.h"

namespace {

thread_local std::string g_error;
double g_routing_slack = 2e-3;

// Error-analysis knobs (default 0 = exact FP64). Each bit rounds one class of
// values the way a 16-bit device datapath stores them, so the contribution of
// each rounding to the end-to-end error can be measured on the CPU:
//   1 dequantised weights of the projections (scale*q + bias, one rounding)
//   2 projection input activations
//   4 attention K / V cache entries
//   8 attention queries and the unnormalised softmax weights of P.V
//   256: the 16-bit type is IEEE half instead of bfloat16
int g_emulate = 0;

double round16(double v) {
  if (g_emulate & 256) return double(float(_Float16(float(v))));
  return double(synth::bf16_to_float(synth::bf16_rne(float(v))));
}

template <class F>
int guarded(F f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
  } catch (...) {
    g_error = "unknown oracle exception";
  }
  return -1;
}

int worker_count() {
  unsigned n = std::thread::hardware_concurrency();
  return int(n ? std::min(n, 64u) : 1u);
}

template <class F>
void parallel_for(size_t n, F f, size_t min_chunk = 1) {
  int workers = worker_count();
  if (n < 2 * min_chunk || workers == 1) {
    f(size_t(0), n);
    return;
  }
  size_t chunk = std::max(min_chunk, (n + workers - 1) / workers);
  std::vector<std::thread> pool;
  for (size_t b = 0; b < n; b += chunk) pool.emplace_back(f, b, std::min(n, b + chunk));
  for (auto& t : pool) t.join();
}

// ---------------------------------------------------------------- operators --

double sigmoid(double x) {
  if (x >= 0) return 1. / (1. + std::exp(-x));
  double e = std::exp(x);
  return e / (1. + e);
}
double silu(double x) { return x * sigmoid(x); }

// RMSNorm over rows of `width` (operator_reference.h:11-14); weight empty = 1.
void rms_rows(const double* x, double* y, size_t rows, size_t width, const float* weight,
              double eps) {
  for (size_t r = 0; r < rows; ++r) {
    double sq = 0;
    for (size_t c = 0; c < width; ++c) sq += x[r * width + c] * x[r * width + c];
    double inv = 1. / std::sqrt(sq / double(width) + eps);
    for (size_t c = 0; c < width; ++c)
      y[r * width + c] = x[r * width + c] * inv * (weight ? double(weight[c]) : 1.);
  }
}

// Non-traditional (rotate-half) RoPE on the first `rotary` dims of one head
// vector (operator_reference.h:15-18): angle = pos * theta^(-2j/rotary).
void rope_vec(double* v, int rotary, double pos, double theta) {
  for (int j = 0; j < rotary / 2; ++j) {
    double angle = pos * std::pow(theta, -2. * j / rotary);
    double c = std::cos(angle), s = std::sin(angle);
    double a = v[j], b = v[j + rotary / 2];
    v[j] = a * c - b * s;
    v[j + rotary / 2] = a * s + b * c;
  }
}

// IEEE total-order key (selection.h:3-12): -0 < +0, NaN ordered by bits.
uint32_t total_key(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}

// ------------------------------------------------------------ weight tensors --

// A 4-bit g64 matrix [rows, cols], generated lazily in 128-row blocks with the
// synthetic generator (synth.h). Dequantized on the fly in FP64.
struct QTensor {
  std::string name;
  size_t rows = 0, cols = 0;
  uint64_t key = 0;
  std::mutex mu;
  struct Block {
    std::vector<uint32_t> packed;    // 128 * cols/8
    std::vector<float> scale, bias;  // 128 * cols/64 (bf16 widened)
  };
  std::unordered_map<size_t, std::unique_ptr<Block>> blocks;
  // Replacement data in any reference quantization (bits 2..8, group 32/64/128;
  // a checkpoint module with a quantization override): rows of LSB-first
  // `bits`-bit values, float scales and biases per group.
  struct Override {
    int bits = 4, group = 64;
    std::vector<uint32_t> packed;
    std::vector<float> scale, bias;
  };
  std::unique_ptr<Override> ov;

  const Block& block(size_t b) {
    {
      std::lock_guard<std::mutex> lock(mu);
      auto it = blocks.find(b);
      if (it != blocks.end()) return *it->second;
    }
    auto blk = std::make_unique<Block>();
    size_t words = cols / 8, groups = cols / 64;
    blk->packed.assign(128 * words, 0);
    blk->scale.assign(128 * groups, 0.f);
    blk->bias.assign(128 * groups, 0.f);
    std::vector<float> w(64);
    uint8_t q[64];
    for (size_t r = 0; r < 128; ++r) {
      size_t row = b * 128 + r;
      if (row >= rows) break;
      for (size_t g = 0; g < groups; ++g) {
        for (int i = 0; i < 64; ++i) w[i] = synth::normal(key, row * cols + g * 64 + i, 0.02f);
        uint16_t sb, bb;
        synth::quantize_group(w.data(), q, &sb, &bb);
        blk->scale[r * groups + g] = synth::bf16_to_float(sb);
        blk->bias[r * groups + g] = synth::bf16_to_float(bb);
        for (int i = 0; i < 64; ++i)
          blk->packed[r * words + (g * 64 + i) / 8] |= uint32_t(q[i]) << (4 * ((g * 64 + i) % 8));
      }
    }
    std::lock_guard<std::mutex> lock(mu);
    auto it = blocks.find(b);
    if (it != blocks.end()) return *it->second;  // another thread won the race
    auto& ref = *blk;
    blocks.emplace(b, std::move(blk));
    return ref;
  }
  void ensure(size_t row0, size_t n) {
    if (ov) return;
    size_t b0 = row0 / 128, b1 = (row0 + n - 1) / 128;
    parallel_for(b1 - b0 + 1, [&](size_t b, size_t e) {
      for (size_t i = b; i < e; ++i) block(b0 + i);
    });
  }
  // Dequantized row (native/projection_reference.h:74 element formula).
  // `projection`: the row feeds a projection (emulation bit 1 may round it).
  void row(size_t r, double* out, bool projection = false) {
    const bool rnd = projection && (g_emulate & 1);
    if (ov) {  // native/projection_reference.h:8-22 with the override's bits and group
      const size_t words = cols * ov->bits / 32, groups = cols / ov->group;
      const uint32_t* rw = &ov->packed[r * words];
      for (size_t c = 0; c < cols; ++c) {
        const size_t bit = c * ov->bits, w = bit / 32;
        const unsigned sh = unsigned(bit % 32);
        uint64_t v = rw[w];
        if (sh + ov->bits > 32) v |= uint64_t(rw[w + 1]) << 32;
        const unsigned q = unsigned(v >> sh) & ((1u << ov->bits) - 1u);
        const size_t g = r * groups + c / ov->group;
        out[c] = double(ov->scale[g]) * q + double(ov->bias[g]);
        if (rnd) out[c] = round16(out[c]);
      }
      return;
    }
    const Block& blk = block(r / 128);
    size_t lr = r % 128, words = cols / 8, groups = cols / 64;
    for (size_t c = 0; c < cols; ++c) {
      unsigned q = (blk.packed[lr * words + c / 8] >> (4 * (c % 8))) & 15u;
      out[c] = double(blk.scale[lr * groups + c / 64]) * q + double(blk.bias[lr * groups + c / 64]);
      if (rnd) out[c] = round16(out[c]);
    }
  }
  // y[t][o] = sum_c x[t][c] * W[row0+o][c], for o < n_out.
  void project(const double* x, size_t n_tok, size_t row0, size_t n_out, double* y) {
    if (row0 + n_out > rows) throw std::invalid_argument("projection rows out of range: " + name);
    ensure(row0, n_out);
    std::vector<double> xr;
    if (g_emulate & 2) {
      xr.assign(x, x + n_tok * cols);
      for (auto& v : xr) v = round16(v);
      x = xr.data();
    }
    parallel_for(
        n_out,
        [&](size_t b, size_t e) {
          std::vector<double> w(cols);
          for (size_t o = b; o < e; ++o) {
            row(row0 + o, w.data(), true);
            for (size_t t = 0; t < n_tok; ++t) {
              double s = 0;
              const double* xt = x + t * cols;
              for (size_t c = 0; c < cols; ++c) s += xt[c] * w[c];
              y[t * n_out + o] = s;
            }
          }
        },
        64);
  }
};

struct Model {
  rs_qwen_config c{};
  uint64_t seed = 0;
  bool mtp = false;
  std::map<std::string, std::unique_ptr<QTensor>> q;
  std::map<std::string, std::vector<float>> v;

  QTensor& Q(const std::string& n) {
    auto it = q.find(n);
    if (it == q.end()) throw std::invalid_argument("oracle: missing matrix " + n);
    return *it->second;
  }
  const std::vector<float>& V(const std::string& n) const {
    auto it = v.find(n);
    if (it == v.end()) throw std::invalid_argument("oracle: missing vector " + n);
    return it->second;
  }
  void add_q(const std::string& n, size_t rows, size_t cols) {
    if (cols % 64) throw std::invalid_argument("oracle: width not a multiple of 64: " + n);
    auto t = std::make_unique<QTensor>();
    t->name = n;
    t->rows = rows;
    t->cols = cols;
    t->key = synth::tensor_key(seed, synth::tensor_id(n));
    q[n] = std::move(t);
  }
  void add_gain(const std::string& n, size_t len) { v[n].assign(len, 1.0f); }
  void add_normal(const std::string& n, size_t len) {
    uint64_t key = synth::tensor_key(seed, synth::tensor_id(n));
    auto& x = v[n];
    x.resize(len);
    for (size_t i = 0; i < len; ++i) x[i] = synth::normal(key, i, 0.02f);
  }
  void add_attention(const std::string& p) {
    size_t H = c.hidden, d = c.head_dim;
    add_q(p + ".self_attn.q_proj", size_t(c.q_heads) * 2 * d, H);
    add_q(p + ".self_attn.k_proj", size_t(c.kv_heads) * d, H);
    add_q(p + ".self_attn.v_proj", size_t(c.kv_heads) * d, H);
    add_gain(p + ".self_attn.q_norm.weight", d);
    add_gain(p + ".self_attn.k_norm.weight", d);
    add_q(p + ".self_attn.o_proj", H, size_t(c.q_heads) * d);
  }
  void add_moe(const std::string& p) {
    size_t H = c.hidden, E = c.experts, I = c.intermediate, S = c.shared;
    add_q(p + ".mlp.gate", E, H);
    add_q(p + ".mlp.switch_mlp.gate_proj", E * I, H);
    add_q(p + ".mlp.switch_mlp.up_proj", E * I, H);
    add_q(p + ".mlp.switch_mlp.down_proj", E * H, I);
    add_q(p + ".mlp.shared_expert.gate_proj", S, H);
    add_q(p + ".mlp.shared_expert.up_proj", S, H);
    add_q(p + ".mlp.shared_expert.down_proj", H, S);
    add_q(p + ".mlp.shared_expert_gate", 1, H);
  }
  void build() {
    size_t H = c.hidden;
    size_t kd = size_t(c.key_heads) * c.key_dim, vd = size_t(c.value_heads) * c.value_dim;
    size_t cd = 2 * kd + vd;
    add_q("language_model.model.embed_tokens", c.vocab, H);
    add_q("language_model.lm_head", c.vocab, H);
    add_gain("language_model.model.norm.weight", H);
    for (int i = 0; i < c.layers; ++i) {
      std::string p = "language_model.model.layers." + std::to_string(i);
      add_gain(p + ".input_layernorm.weight", H);
      add_gain(p + ".post_attention_layernorm.weight", H);
      if ((i + 1) % c.interval == 0) {
        add_attention(p);
      } else {
        std::string g = p + ".linear_attn";
        add_q(g + ".in_proj_qkv", cd, H);
        add_q(g + ".in_proj_z", vd, H);
        add_q(g + ".in_proj_a", c.value_heads, H);
        add_q(g + ".in_proj_b", c.value_heads, H);
        add_normal(g + ".conv1d.weight", cd * size_t(c.conv));
        add_normal(g + ".A_log", c.value_heads);
        add_normal(g + ".dt_bias", c.value_heads);
        add_gain(g + ".norm.weight", c.value_dim);
        add_q(g + ".out_proj", H, vd);
      }
      add_moe(p);
    }
    if (mtp) {
      std::string m = "language_model.mtp";
      add_gain(m + ".pre_fc_norm_embedding.weight", H);
      add_gain(m + ".pre_fc_norm_hidden.weight", H);
      add_q(m + ".fc", H, 2 * H);
      add_gain(m + ".layers.0.input_layernorm.weight", H);
      add_gain(m + ".layers.0.post_attention_layernorm.weight", H);
      add_attention(m + ".layers.0");
      add_moe(m + ".layers.0");
      add_gain(m + ".norm.weight", H);
    }
  }
};

// -------------------------------------------------------------- layer math --

struct Forward {
  Model& m;
  const rs_qwen_config& c;
  size_t H, kd, vd, cd;
  const int32_t* forced = nullptr;  // [moe layer][T][top] or null
  size_t forced_count = 0;
  size_t moe_index = 0;
  int32_t* routed_out = nullptr;  // optional capture, same layout
  explicit Forward(Model& mm) : m(mm), c(mm.c) {
    H = c.hidden;
    kd = size_t(c.key_heads) * c.key_dim;
    vd = size_t(c.value_heads) * c.value_dim;
    cd = 2 * kd + vd;
  }

  // MoE block (qwen_model.inc:75-100): softmax router, top-k, renormalised
  // weights, SwiGLU experts, plus sigmoid-gated shared expert.
  // Top-k rule: larger logit first, lower expert id on equal logits.
  void moe(const std::string& p, const double* h, size_t T, double* y) {
    size_t E = c.experts, K = c.top, I = c.intermediate, S = c.shared;
    std::vector<double> logits(T * E), sg(T);
    m.Q(p + ".mlp.gate").project(h, T, 0, E, logits.data());
    m.Q(p + ".mlp.shared_expert_gate").project(h, T, 0, 1, sg.data());
    std::vector<double> sh_g(T * S), sh_u(T * S), act(T * S), sh_out(T * H);
    m.Q(p + ".mlp.shared_expert.gate_proj").project(h, T, 0, S, sh_g.data());
    m.Q(p + ".mlp.shared_expert.up_proj").project(h, T, 0, S, sh_u.data());
    for (size_t i = 0; i < T * S; ++i) act[i] = silu(sh_g[i]) * sh_u[i];
    m.Q(p + ".mlp.shared_expert.down_proj").project(act.data(), T, 0, H, sh_out.data());
    std::vector<double> eg(I), eu(I), ea(I), ed(H);
    for (size_t t = 0; t < T; ++t) {
      const double* lt = &logits[t * E];
      double peak = *std::max_element(lt, lt + E);
      std::vector<int32_t> sel(K);
      if (forced) {
        if ((moe_index + 1) * T * K > forced_count) throw std::invalid_argument("forced routing too short");
        for (size_t j = 0; j < K; ++j) sel[j] = forced[(moe_index * T + t) * K + j];
        // The forced selection must be a top-k of the FP64 logits up to a
        // small slack (near-ties may legitimately differ in fp32).
        double lo = INFINITY;
        std::vector<bool> seen(E, false);
        for (size_t j = 0; j < K; ++j) {
          if (sel[j] < 0 || size_t(sel[j]) >= E || seen[sel[j]])
            throw std::invalid_argument("forced routing invalid membership");
          seen[sel[j]] = true;
          lo = std::min(lo, lt[sel[j]]);
        }
        for (size_t e = 0; e < E; ++e)
          if (!seen[e] && lt[e] > lo + g_routing_slack * (1. + std::abs(lo)))
            throw std::runtime_error("forced routing is not a top-k of the oracle logits");
      } else {
        std::vector<int32_t> order(E);
        for (size_t e = 0; e < E; ++e) order[e] = int32_t(e);
        std::stable_sort(order.begin(), order.end(),
                         [&](int32_t a, int32_t b) { return lt[a] > lt[b]; });
        for (size_t j = 0; j < K; ++j) sel[j] = order[j];
      }
      if (routed_out)
        for (size_t j = 0; j < K; ++j) routed_out[(moe_index * T + t) * K + j] = sel[j];
      double denom = 0;
      for (size_t j = 0; j < K; ++j) denom += std::exp(lt[sel[j]] - peak);
      double* yt = y + t * H;
      for (size_t i = 0; i < H; ++i) yt[i] = 0;
      for (size_t j = 0; j < K; ++j) {
        double w = std::exp(lt[sel[j]] - peak) / denom;
        size_t e = size_t(sel[j]);
        m.Q(p + ".mlp.switch_mlp.gate_proj").project(h + t * H, 1, e * I, I, eg.data());
        m.Q(p + ".mlp.switch_mlp.up_proj").project(h + t * H, 1, e * I, I, eu.data());
        for (size_t i = 0; i < I; ++i) ea[i] = silu(eg[i]) * eu[i];
        m.Q(p + ".mlp.switch_mlp.down_proj").project(ea.data(), 1, e * H, H, ed.data());
        for (size_t i = 0; i < H; ++i) yt[i] += w * ed[i];
      }
      double gate = sigmoid(sg[t]);
      for (size_t i = 0; i < H; ++i) yt[i] += gate * sh_out[t * H + i];
    }
    ++moe_index;
  }

  // Gated attention layer (qwen_model.inc:101-153) for T tokens at `offset`,
  // K/V caches [kv][ctx][d] in FP64 (rows < offset hold the prefix).
  void attention(const std::string& p, const double* h, size_t T, size_t offset, double* Kc,
                 double* Vc, size_t ctx, double* y) {
    size_t Hq = c.q_heads, Hk = c.kv_heads, d = c.head_dim;
    std::vector<double> qg(T * Hq * 2 * d), k(T * Hk * d), v(T * Hk * d);
    m.Q(p + ".self_attn.q_proj").project(h, T, 0, Hq * 2 * d, qg.data());
    m.Q(p + ".self_attn.k_proj").project(h, T, 0, Hk * d, k.data());
    m.Q(p + ".self_attn.v_proj").project(h, T, 0, Hk * d, v.data());
    const auto& qn = m.V(p + ".self_attn.q_norm.weight");
    const auto& kn = m.V(p + ".self_attn.k_norm.weight");
    std::vector<double> q(T * Hq * d), gate(T * Hq * d), tmp(d);
    for (size_t t = 0; t < T; ++t)
      for (size_t hh = 0; hh < Hq; ++hh) {
        const double* src = &qg[(t * Hq + hh) * 2 * d];
        rms_rows(src, &q[(t * Hq + hh) * d], 1, d, qn.data(), c.epsilon);
        for (size_t i = 0; i < d; ++i) gate[(t * Hq + hh) * d + i] = src[d + i];
        rope_vec(&q[(t * Hq + hh) * d], c.rope_dims, double(offset + t), c.theta);
        if (g_emulate & 8)
          for (size_t i = 0; i < d; ++i) q[(t * Hq + hh) * d + i] = round16(q[(t * Hq + hh) * d + i]);
      }
    for (size_t t = 0; t < T; ++t)
      for (size_t g = 0; g < Hk; ++g) {
        rms_rows(&k[(t * Hk + g) * d], tmp.data(), 1, d, kn.data(), c.epsilon);
        rope_vec(tmp.data(), c.rope_dims, double(offset + t), c.theta);
        if (offset + t >= ctx) throw std::invalid_argument("oracle context overflow");
        for (size_t i = 0; i < d; ++i) {
          Kc[(g * ctx + offset + t) * d + i] = (g_emulate & 4) ? round16(tmp[i]) : tmp[i];
          Vc[(g * ctx + offset + t) * d + i] = (g_emulate & 4) ? round16(v[(t * Hk + g) * d + i]) : v[(t * Hk + g) * d + i];
        }
      }
    // attention_reference.h:8-21, bottom-right causal window.
    std::vector<double> o(T * Hq * d);
    size_t group = Hq / Hk;
    double scale = 1. / std::sqrt(double(d));
    for (size_t hh = 0; hh < Hq; ++hh)
      for (size_t t = 0; t < T; ++t) {
        size_t g = hh / group, visible = offset + t + 1;
        std::vector<double> sc(visible);
        double peak = -INFINITY;
        for (size_t j = 0; j < visible; ++j) {
          double dot = 0;
          for (size_t i = 0; i < d; ++i) dot += q[(t * Hq + hh) * d + i] * Kc[(g * ctx + j) * d + i];
          sc[j] = dot * scale;
          peak = std::max(peak, sc[j]);
        }
        double tot = 0;
        for (auto& s : sc) { s = std::exp(s - peak); tot += s; }
        if (g_emulate & 8)
          for (auto& s : sc) s = round16(s);  // P enters P.V as 16-bit; the sum stays exact
        for (size_t i = 0; i < d; ++i) {
          double acc = 0;
          for (size_t j = 0; j < visible; ++j) acc += sc[j] / tot * Vc[(g * ctx + j) * d + i];
          o[(t * Hq + hh) * d + i] = acc * sigmoid(gate[(t * Hq + hh) * d + i]);
        }
      }
    m.Q(p + ".self_attn.o_proj").project(o.data(), T, 0, H, y);
  }

  // Gated-DeltaNet layer (qwen_model.inc:154-206, operator_reference.h:19-45).
  // conv_state [(K-1)][cd], S [hv][dv][dk]; both updated in place.
  void deltanet(const std::string& p, const double* h, size_t T, double* conv_state, double* S,
                double* y) {
    size_t hv = c.value_heads, hk = c.key_heads, dk = c.key_dim, dv = c.value_dim, K = c.conv;
    std::string g = p + ".linear_attn";
    std::vector<double> qkv(T * cd), z(T * vd), a(T * hv), b(T * hv);
    m.Q(g + ".in_proj_qkv").project(h, T, 0, cd, qkv.data());
    m.Q(g + ".in_proj_z").project(h, T, 0, vd, z.data());
    m.Q(g + ".in_proj_a").project(h, T, 0, hv, a.data());
    m.Q(g + ".in_proj_b").project(h, T, 0, hv, b.data());
    const auto& cw = m.V(g + ".conv1d.weight");
    const auto& alog = m.V(g + ".A_log");
    const auto& dt = m.V(g + ".dt_bias");
    const auto& nw = m.V(g + ".norm.weight");
    // stream = [conv_state rows; qkv rows]
    std::vector<double> stream((K - 1 + T) * cd);
    std::copy(conv_state, conv_state + (K - 1) * cd, stream.begin());
    std::copy(qkv.begin(), qkv.end(), stream.begin() + (K - 1) * cd);
    std::vector<double> act(T * cd);
    for (size_t t = 0; t < T; ++t)
      for (size_t ch = 0; ch < cd; ++ch) {
        double val = 0;
        for (size_t tap = 0; tap < K; ++tap) val += stream[(t + tap) * cd + ch] * cw[ch * K + tap];
        act[t * cd + ch] = silu(val);
      }
    std::copy(stream.begin() + T * cd, stream.end(), conv_state);
    std::vector<double> o(T * vd), qh(dk), kh(dk);
    for (size_t t = 0; t < T; ++t)
      for (size_t head = 0; head < hv; ++head) {
        size_t kh_idx = head / (hv / hk);
        double qs = 0, ks = 0;
        for (size_t j = 0; j < dk; ++j) {
          qh[j] = act[t * cd + kh_idx * dk + j];
          kh[j] = act[t * cd + kd + kh_idx * dk + j];
          qs += qh[j] * qh[j];
          ks += kh[j] * kh[j];
        }
        double qi = 1. / (std::sqrt(qs / dk + 1e-6) * dk);
        double ki = 1. / (std::sqrt(ks / dk + 1e-6) * std::sqrt(double(dk)));
        for (size_t j = 0; j < dk; ++j) { qh[j] *= qi; kh[j] *= ki; }
        double logit = a[t * hv + head] + dt[head];
        double sp = std::max(logit, 0.) + std::log1p(std::exp(-std::abs(logit)));
        double decay = std::exp(-std::exp(double(alog[head])) * sp);
        double beta = sigmoid(b[t * hv + head]);
        for (size_t r = 0; r < dv; ++r) {
          double* row = S + (head * dv + r) * dk;
          double mem = 0;
          for (size_t j = 0; j < dk; ++j) { row[j] *= decay; mem += row[j] * kh[j]; }
          double delta = (act[t * cd + 2 * kd + head * dv + r] - mem) * beta, rd = 0;
          for (size_t j = 0; j < dk; ++j) { row[j] += delta * kh[j]; rd += row[j] * qh[j]; }
          o[t * vd + head * dv + r] = rd;
        }
      }
    // y = rms(o per head, norm.weight) * silu(z) -> out_proj (qwen_model.inc:203-205)
    std::vector<double> gated(T * vd);
    for (size_t t = 0; t < T; ++t)
      for (size_t head = 0; head < hv; ++head) {
        rms_rows(&o[t * vd + head * dv], &gated[t * vd + head * dv], 1, dv, nw.data(), c.epsilon);
        for (size_t r = 0; r < dv; ++r)
          gated[t * vd + head * dv + r] *= silu(z[t * vd + head * dv + r]);
      }
    m.Q(g + ".out_proj").project(gated.data(), T, 0, H, y);
  }

  void embed(const uint32_t* tokens, size_t T, double* x) {
    auto& e = m.Q("language_model.model.embed_tokens");
    for (size_t t = 0; t < T; ++t) {
      if (tokens[t] >= uint32_t(c.vocab)) throw std::invalid_argument("token outside vocabulary");
      e.row(tokens[t], x + t * H);
    }
  }
};

size_t state_count(const rs_qwen_config& c) {
  size_t full = c.layers / c.interval, lin = c.layers - full;
  size_t cd = 2 * size_t(c.key_heads) * c.key_dim + size_t(c.value_heads) * c.value_dim;
  return lin * (size_t(c.conv - 1) * cd + size_t(c.value_heads) * c.value_dim * c.key_dim) +
         full * 2 * size_t(c.kv_heads) * size_t(c.context) * c.head_dim;
}

void validate(const rs_qwen_config& c) {
  if (c.hidden <= 0 || c.layers <= 0 || c.vocab <= 0 || c.interval <= 0 || c.layers % c.interval ||
      c.q_heads % c.kv_heads || c.value_heads % c.key_heads || c.conv < 2 || c.top > c.experts ||
      c.rope_dims <= 0 || c.rope_dims > c.head_dim || c.rope_dims % 2 || c.context <= 0)
    throw std::invalid_argument("oracle: model geometry");
}

}  // namespace

extern "C" {

const char* orc_last_error() { return g_error.c_str(); }

// Slack (relative to 1+|logit|) allowed when a forced expert selection is
// checked against the oracle's own FP64 router logits.
void orc_set_routing_slack(double slack) { g_routing_slack = slack; }

// Error-analysis knobs (bits documented at g_emulate); 0 restores exact FP64.
void orc_set_emulation(int bits) { g_emulate = bits; }

size_t orc_state_count(const rs_qwen_config* c) { return state_count(*c); }

// Build a lazily generated synthetic model (same tensors and bytes as
// rs_qwen_weights_synthetic).
void* orc_model_create(const rs_qwen_config* config, uint64_t seed, int with_mtp) {
  Model* m = nullptr;
  if (guarded([&] {
        validate(*config);
        auto mm = std::make_unique<Model>();
        mm->c = *config;
        mm->seed = seed;
        mm->mtp = with_mtp != 0;
        mm->build();
        m = mm.release();
      }))
    return nullptr;
  return m;
}
void orc_model_destroy(void* m) { delete static_cast<Model*>(m); }

// Canonical bytes of a quantized tensor rows [row0, row0+n): packed uint32
// [n][cols/8], scales/biases float [n][cols/64].
int orc_model_qrows(void* model, const char* name, size_t row0, size_t n, uint32_t* packed,
                    float* scales, float* biases) {
  return guarded([&] {
    auto& t = static_cast<Model*>(model)->Q(name);
    if (row0 + n > t.rows) throw std::invalid_argument("qrows range");
    size_t words = t.cols / 8, groups = t.cols / 64;
    for (size_t r = 0; r < n; ++r) {
      size_t row = row0 + r;
      const auto& b = t.block(row / 128);
      size_t lr = row % 128;
      if (packed) std::memcpy(packed + r * words, &b.packed[lr * words], words * 4);
      if (scales) std::memcpy(scales + r * groups, &b.scale[lr * groups], groups * 4);
      if (biases) std::memcpy(biases + r * groups, &b.bias[lr * groups], groups * 4);
    }
  });
}
// Replaces a matrix's synthetic data with rows in another quantization
// (bits 2..8, group 32/64/128): packed [rows][cols*bits/32] LSB-first words,
// scales / biases [rows][cols/group] (values as loaded, widened to float).
int orc_model_override(void* model, const char* name, int bits, int group, const uint32_t* packed,
                       const float* scales, const float* biases) {
  return guarded([&] {
    auto& t = static_cast<Model*>(model)->Q(name);
    if (bits < 2 || bits > 8 || bits == 7 || (group != 32 && group != 64 && group != 128) || t.cols % group ||
        (t.cols * bits) % 32)
      throw std::invalid_argument("override quantization");
    auto ov = std::make_unique<QTensor::Override>();
    ov->bits = bits;
    ov->group = group;
    const size_t words = t.cols * bits / 32, groups = t.cols / group;
    ov->packed.assign(packed, packed + t.rows * words);
    ov->scale.assign(scales, scales + t.rows * groups);
    ov->bias.assign(biases, biases + t.rows * groups);
    t.ov = std::move(ov);
  });
}

int orc_model_vector(void* model, const char* name, float* out, size_t count) {
  return guarded([&] {
    const auto& v = static_cast<Model*>(model)->V(name);
    if (count != v.size()) throw std::invalid_argument("vector length");
    std::memcpy(out, v.data(), count * 4);
  });
}

// Mirrors rs_qwen_forward (native/qwen_model.inc:375-377) for one sequence:
// count tokens at `offset`, old_state (state_count floats, ignored when
// offset == 0), new_state out, logits out for EVERY input token
// (count*vocab, position-major), hidden out (count*hidden post-final-norm,
// nullable). forced_routing: [moe layers][count][top] or null; routed:
// capture of the routing used (same layout), nullable.
int orc_forward(void* model, const uint32_t* tokens, size_t count, size_t offset,
                const float* old_state, float* new_state, double* logits, double* hidden,
                const int32_t* forced_routing, size_t forced_count, int32_t* routed) {
  return guarded([&] {
    Model& m = *static_cast<Model*>(model);
    const auto& c = m.c;
    if (!count || offset + count > size_t(c.context)) throw std::invalid_argument("oracle forward capacity");
    Forward f(m);
    f.forced = forced_routing;
    f.forced_count = forced_count;
    f.routed_out = routed;
    size_t H = c.hidden, T = count, ctx = c.context, d = c.head_dim, Hk = c.kv_heads;
    size_t convn = size_t(c.conv - 1) * f.cd, sn = size_t(c.value_heads) * c.value_dim * c.key_dim;
    std::vector<double> x(T * H), h(T * H), r(T * H);
    f.embed(tokens, T, x.data());
    size_t rd = 0, wr = 0;
    for (int layer = 0; layer < c.layers; ++layer) {
      std::string p = "language_model.model.layers." + std::to_string(layer);
      rms_rows(x.data(), h.data(), T, H, m.V(p + ".input_layernorm.weight").data(), c.epsilon);
      if ((layer + 1) % c.interval == 0) {
        std::vector<double> K(Hk * ctx * d, 0.), V(Hk * ctx * d, 0.);
        if (offset) {
          for (size_t i = 0; i < K.size(); ++i) K[i] = old_state[rd + i];
          for (size_t i = 0; i < V.size(); ++i) V[i] = old_state[rd + K.size() + i];
        }
        rd += 2 * K.size();
        f.attention(p, h.data(), T, offset, K.data(), V.data(), ctx, r.data());
        for (size_t i = 0; i < K.size(); ++i) new_state[wr + i] = float(K[i]);
        for (size_t i = 0; i < V.size(); ++i) new_state[wr + K.size() + i] = float(V[i]);
        wr += 2 * K.size();
      } else {
        std::vector<double> conv(convn, 0.), S(sn, 0.);
        if (offset) {
          for (size_t i = 0; i < convn; ++i) conv[i] = old_state[rd + i];
          for (size_t i = 0; i < sn; ++i) S[i] = old_state[rd + convn + i];
        }
        rd += convn + sn;
        f.deltanet(p, h.data(), T, conv.data(), S.data(), r.data());
        for (size_t i = 0; i < convn; ++i) new_state[wr + i] = float(conv[i]);
        for (size_t i = 0; i < sn; ++i) new_state[wr + convn + i] = float(S[i]);
        wr += convn + sn;
      }
      for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
      rms_rows(x.data(), h.data(), T, H, m.V(p + ".post_attention_layernorm.weight").data(),
               c.epsilon);
      f.moe(p, h.data(), T, r.data());
      for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
    }
    rms_rows(x.data(), h.data(), T, H, m.V("language_model.model.norm.weight").data(), c.epsilon);
    if (hidden) std::copy(h.begin(), h.end(), hidden);
    if (logits) m.Q("language_model.lm_head").project(h.data(), T, 0, c.vocab, logits);
  });
}

// MTP draft head (native/qwen_mtp.inc:157-171) for `count` tokens at draft
// position `offset`: x = fc(concat(rms(embed(tok)), rms(hidden))) -> attention
// layer with its own KV (kv_state [2][kv][context][d] in/out) -> MoE -> norm.
// Outputs logits of every row through the target lm_head and the post-norm
// hidden rows.
int orc_mtp_forward(void* model, const uint32_t* tokens, size_t count, size_t offset,
                    const double* target_hidden, double* kv_state, double* logits,
                    double* hidden_out, const int32_t* forced_routing, size_t forced_count) {
  return guarded([&] {
    Model& m = *static_cast<Model*>(model);
    if (!m.mtp) throw std::invalid_argument("oracle model has no MTP head");
    const auto& c = m.c;
    size_t H = c.hidden, T = count, ctx = c.context, d = c.head_dim, Hk = c.kv_heads;
    Forward f(m);
    f.forced = forced_routing;
    f.forced_count = forced_count;
    std::string mp = "language_model.mtp";
    std::vector<double> e(T * H), en(T * H), hn(T * H), cat(T * 2 * H), x(T * H), h(T * H),
        r(T * H);
    f.embed(tokens, T, e.data());
    rms_rows(e.data(), en.data(), T, H, m.V(mp + ".pre_fc_norm_embedding.weight").data(), c.epsilon);
    rms_rows(target_hidden, hn.data(), T, H, m.V(mp + ".pre_fc_norm_hidden.weight").data(),
             c.epsilon);
    for (size_t t = 0; t < T; ++t)
      for (size_t i = 0; i < H; ++i) {
        cat[t * 2 * H + i] = en[t * H + i];
        cat[t * 2 * H + H + i] = hn[t * H + i];
      }
    m.Q(mp + ".fc").project(cat.data(), T, 0, H, x.data());
    std::string p = mp + ".layers.0";
    rms_rows(x.data(), h.data(), T, H, m.V(p + ".input_layernorm.weight").data(), c.epsilon);
    f.attention(p, h.data(), T, offset, kv_state, kv_state + Hk * ctx * d, ctx, r.data());
    for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
    rms_rows(x.data(), h.data(), T, H, m.V(p + ".post_attention_layernorm.weight").data(),
             c.epsilon);
    f.moe(p, h.data(), T, r.data());
    for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
    rms_rows(x.data(), h.data(), T, H, m.V(mp + ".norm.weight").data(), c.epsilon);
    if (hidden_out) std::copy(h.begin(), h.end(), hidden_out);
    if (logits) m.Q("language_model.lm_head").project(h.data(), T, 0, c.vocab, logits);
  });
}

// ------------------------------------------------------- standalone kernels --

// Scalar affine projection (native/projection_reference.h:8-22), any bits in
// {2,3,4,5,6,8} and groups {32,64,128}; rows of packed are LSB-first bitstreams.
int orc_projection(const float* x, const uint32_t* packed, const float* scales,
                   const float* biases, size_t rows, size_t outputs, size_t width, int group,
                   int bits, double* y) {
  return guarded([&] {
    if (!rows || !outputs || !width || (group != 32 && group != 64 && group != 128) ||
        (bits != 2 && bits != 3 && bits != 4 && bits != 5 && bits != 6 && bits != 8) ||
        width % size_t(group))
      throw std::invalid_argument("projection oracle geometry");
    size_t words = width * bits / 32, groups = width / group;
    for (size_t o = 0; o < outputs; ++o)
      for (size_t r = 0; r < rows; ++r) {
        double s = 0;
        for (size_t col = 0; col < width; ++col) {
          size_t bit = col * bits, word = bit / 32;
          unsigned shift = bit % 32;
          uint64_t val = packed[o * words + word];
          if (shift + bits > 32) val |= uint64_t(packed[o * words + word + 1]) << 32;
          unsigned q = unsigned(val >> shift) & ((1u << bits) - 1);
          size_t g = o * groups + col / group;
          s += double(x[r * width + col]) * (double(scales[g]) * q + double(biases[g]));
        }
        y[r * outputs + o] = s;
      }
  });
}

int orc_rms(const float* x, const float* weight, size_t rows, size_t width, double eps,
            double* y) {
  return guarded([&] {
    std::vector<double> xd(x, x + rows * width);
    rms_rows(xd.data(), y, rows, width, weight, eps);
  });
}

int orc_silu(const float* x, size_t n, double* y) {
  return guarded([&] {
    for (size_t i = 0; i < n; ++i) y[i] = silu(x[i]);
  });
}

// x: [heads][tokens][dim] (operator_reference.h:15-18 layout).
int orc_rope(const float* x, int heads, int tokens, int dim, int rotary, int offset, double theta,
             double* y) {
  return guarded([&] {
    for (int h = 0; h < heads; ++h)
      for (int t = 0; t < tokens; ++t) {
        double* v = y + (size_t(h) * tokens + t) * dim;
        for (int i = 0; i < dim; ++i) v[i] = x[(size_t(h) * tokens + t) * dim + i];
        rope_vec(v, rotary, double(offset + t), theta);
      }
  });
}

// Gated delta rule with causal conv (operator_reference.h:19-45 argument
// order): outputs activated [T][channels], history [(K-1)][channels],
// output [T][hv*dv], state [hv][dv][dk].
int orc_delta(const float* qkv, const float* history, const float* conv, const float* a,
              const float* b, const float* alog, const float* dt, const float* initial,
              int tokens, int hk, int hv, int dk, int dv, int kernel, double* activated,
              double* history_out, double* output, double* state) {
  return guarded([&] {
    size_t kd = size_t(hk) * dk, vd = size_t(hv) * dv, ch = 2 * kd + vd;
    std::vector<double> stream(size_t(kernel - 1 + tokens) * ch);
    for (size_t i = 0; i < size_t(kernel - 1) * ch; ++i) stream[i] = history[i];
    for (size_t i = 0; i < size_t(tokens) * ch; ++i) stream[size_t(kernel - 1) * ch + i] = qkv[i];
    for (size_t i = 0; i < size_t(hv) * dv * dk; ++i) state[i] = initial[i];
    for (int t = 0; t < tokens; ++t)
      for (size_t c = 0; c < ch; ++c) {
        double v = 0;
        for (int tap = 0; tap < kernel; ++tap) v += stream[(size_t(t) + tap) * ch + c] * conv[c * kernel + tap];
        activated[size_t(t) * ch + c] = silu(v);
      }
    for (size_t i = 0; i < size_t(kernel - 1) * ch; ++i) history_out[i] = stream[size_t(tokens) * ch + i];
    std::vector<double> qh(dk), kh(dk);
    for (int t = 0; t < tokens; ++t)
      for (int head = 0; head < hv; ++head) {
        int key = head / (hv / hk);
        double qs = 0, ks = 0;
        for (int j = 0; j < dk; ++j) {
          qh[j] = activated[size_t(t) * ch + size_t(key) * dk + j];
          kh[j] = activated[size_t(t) * ch + kd + size_t(key) * dk + j];
          qs += qh[j] * qh[j];
          ks += kh[j] * kh[j];
        }
        double qi = 1. / (std::sqrt(qs / dk + 1e-6) * dk), ki = 1. / (std::sqrt(ks / dk + 1e-6) * std::sqrt(double(dk)));
        for (int j = 0; j < dk; ++j) { qh[j] *= qi; kh[j] *= ki; }
        double logit = double(a[size_t(t) * hv + head]) + dt[head];
        double sp = std::max(logit, 0.) + std::log1p(std::exp(-std::abs(logit)));
        double decay = std::exp(-std::exp(double(alog[head])) * sp), beta = sigmoid(b[size_t(t) * hv + head]);
        for (int r = 0; r < dv; ++r) {
          double* row = state + (size_t(head) * dv + r) * dk;
          double mem = 0;
          for (int j = 0; j < dk; ++j) { row[j] *= decay; mem += row[j] * kh[j]; }
          double delta = (activated[size_t(t) * ch + 2 * kd + size_t(head) * dv + r] - mem) * beta, rd = 0;
          for (int j = 0; j < dk; ++j) { row[j] += delta * kh[j]; rd += row[j] * qh[j]; }
          output[size_t(t) * vd + size_t(head) * dv + r] = rd;
        }
      }
  });
}

// Causal GQA over a bottom-right window (attention_reference.h:8-21):
// q [heads][tokens][dim], k/v [kv_heads][offset+tokens][dim].
int orc_attention(const float* q, const float* k, const float* v, int heads, int kv_heads,
                  int tokens, int offset, int dim, double* out) {
  return guarded([&] {
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || tokens <= 0 || offset < 0 || dim <= 0)
      throw std::invalid_argument("attention oracle geometry");
    size_t n = size_t(offset) + tokens;
    for (int h = 0; h < heads; ++h)
      for (int row = 0; row < tokens; ++row) {
        int kh = h / (heads / kv_heads);
        size_t visible = size_t(offset) + row + 1;
        std::vector<double> sc(visible);
        double peak = -INFINITY;
        for (size_t j = 0; j < visible; ++j) {
          double dot = 0;
          for (int z = 0; z < dim; ++z) dot += double(q[(size_t(h) * tokens + row) * dim + z]) * k[(kh * n + j) * dim + z];
          sc[j] = dot / std::sqrt(double(dim));
          peak = std::max(peak, sc[j]);
        }
        double tot = 0;
        for (auto& s : sc) { s = std::exp(s - peak); tot += s; }
        for (int z = 0; z < dim; ++z) {
          double e = 0;
          for (size_t j = 0; j < visible; ++j) e += sc[j] / tot * v[(kh * n + j) * dim + z];
          out[(size_t(h) * tokens + row) * dim + z] = e;
        }
      }
  });
}

// Routing probabilities and renormalised weights for a GIVEN selection
// (operator_reference.h:47-57): validates that the selection is a top-k.
int orc_routing(const float* logits, const int32_t* selected, int rows, int experts, int top,
                double* probabilities, double* weights) {
  return guarded([&] {
    for (int r = 0; r < rows; ++r) {
      const float* lv = logits + size_t(r) * experts;
      double peak = *std::max_element(lv, lv + experts), tot = 0;
      for (int e = 0; e < experts; ++e) tot += std::exp(double(lv[e]) - peak);
      for (int e = 0; e < experts; ++e) probabilities[size_t(r) * experts + e] = std::exp(double(lv[e]) - peak) / tot;
      std::vector<bool> seen(experts, false);
      double lo = INFINITY, w = 0;
      for (int j = 0; j < top; ++j) {
        int id = selected[r * top + j];
        if (id < 0 || id >= experts || seen[id]) throw std::invalid_argument("invalid routing membership");
        seen[id] = true;
        lo = std::min(lo, double(lv[id]));
        w += std::exp(double(lv[id]) - peak);
      }
      for (int e = 0; e < experts; ++e)
        if (!seen[e] && lv[e] > lo) throw std::invalid_argument("non-top-k routing membership");
      for (int j = 0; j < top; ++j) weights[r * top + j] = std::exp(double(lv[selected[r * top + j]]) - peak) / w;
    }
  });
}

// Top-k selection rule used by the CUDA router: by fp32 logit descending,
// lower expert id first on equal logits (total order, -0 < +0).
int orc_topk(const float* logits, size_t rows, size_t experts, size_t top, int32_t* idx) {
  return guarded([&] {
    for (size_t r = 0; r < rows; ++r) {
      std::vector<int32_t> order(experts);
      for (size_t e = 0; e < experts; ++e) order[e] = int32_t(e);
      const float* lv = logits + r * experts;
      std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
        return total_key(lv[a]) > total_key(lv[b]);
      });
      for (size_t j = 0; j < top; ++j) idx[r * top + j] = order[j];
    }
  });
}

// Greedy selection (selection.h:3-12, choices.rs:65-79): IEEE total order,
// lowest index on ties. Returns -1 (error) on a non-finite value.
int64_t orc_argmax(const float* logits, size_t n) {
  if (!n) return -1;
  size_t best = 0;
  uint32_t bk = total_key(logits[0]);
  for (size_t i = 0; i < n; ++i) {
    if (!std::isfinite(logits[i])) return -1;
    uint32_t k = total_key(logits[i]);
    if (k > bk) { bk = k; best = i; }
  }
  return int64_t(best);
}

// Constrained greedy selection (src/serving/choices.rs:65-98, `select` with
// an allowed set): every logit of the row must be finite; the winner is the
// allowed id with the largest logit on the total order, the lowest id on
// ties; ids may repeat or come in any order. Returns the id, or -1 with an
// error for a non-finite row, an id outside the row, or an empty set.
int64_t orc_select(const float* logits, size_t n, const uint32_t* allowed, size_t n_allowed) {
  g_error.clear();
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(logits[i])) {
      g_error = "invalid logits";
      return -1;
    }
  int64_t winner = -1;
  for (size_t k = 0; k < n_allowed; ++k) {
    const uint32_t id = allowed[k];
    if (id >= n) {
      g_error = "invalid legal token";
      return -1;
    }
    if (winner < 0) {
      winner = id;
      continue;
    }
    const uint32_t a = total_key(logits[id]), b = total_key(logits[winner]);
    if (a > b || (a == b && int64_t(id) < winner)) winner = id;
  }
  if (winner < 0) g_error = "empty legal token set";
  return winner;
}

// Stable token->expert counting sort. Input: expert id of each flat
// assignment (token-major, slot-minor), n_assign entries, ids < n_experts.
// Output: counts[n_experts], offsets[n_experts+1] (exclusive prefix),
// perm[n_assign] (sorted position -> flat assignment), inv[n_assign].
int orc_expert_sort(const int32_t* ids, size_t n_assign, size_t n_experts, int32_t* counts,
                    int32_t* offsets, int32_t* perm, int32_t* inv) {
  return guarded([&] {
    std::vector<int32_t> cnt(n_experts, 0);
    for (size_t i = 0; i < n_assign; ++i) {
      if (ids[i] < 0 || size_t(ids[i]) >= n_experts) throw std::invalid_argument("expert id range");
      ++cnt[ids[i]];
    }
    offsets[0] = 0;
    for (size_t e = 0; e < n_experts; ++e) {
      counts[e] = cnt[e];
      offsets[e + 1] = offsets[e] + cnt[e];
    }
    std::vector<int32_t> cursor(offsets, offsets + n_experts);
    for (size_t i = 0; i < n_assign; ++i) {
      int32_t pos = cursor[ids[i]]++;
      perm[pos] = int32_t(i);
      inv[i] = pos;
    }
  });
}

// Ragged packing. Per sequence s: position, count, parent block-table row
// (-1 = none), child row, number of parent pages kept (n_shared), offset and
// number of freshly allocated pages in new_pages. Outputs cu_seqlens[n+1],
// token_seq[T], token_pos[T], child rows written into block_table
// (row-major, `row_stride` entries per row; the caller passes the current
// table which is updated in place), slot_mapping[T] = page*page_size + pos%page_size.
int orc_pack_ragged(size_t n_seq, const int32_t* position, const int32_t* count,
                    const int32_t* parent_row, const int32_t* child_row,
                    const int32_t* n_shared, const int32_t* new_off, const int32_t* n_new,
                    const int32_t* new_pages, int32_t page_size, int32_t* block_table,
                    size_t row_stride, int32_t* cu_seqlens, int32_t* token_seq,
                    int32_t* token_pos, int64_t* slot_mapping) {
  return guarded([&] {
    cu_seqlens[0] = 0;
    for (size_t s = 0; s < n_seq; ++s) cu_seqlens[s + 1] = cu_seqlens[s] + count[s];
    for (size_t s = 0; s < n_seq; ++s) {
      int32_t* child = block_table + size_t(child_row[s]) * row_stride;
      std::vector<int32_t> row(size_t(n_shared[s] + n_new[s]));
      for (int32_t j = 0; j < n_shared[s]; ++j) {
        if (parent_row[s] < 0) throw std::invalid_argument("shared pages without parent");
        row[j] = block_table[size_t(parent_row[s]) * row_stride + j];
      }
      for (int32_t j = 0; j < n_new[s]; ++j) row[n_shared[s] + j] = new_pages[new_off[s] + j];
      if (row.size() > row_stride) throw std::invalid_argument("block table row overflow");
      for (size_t j = 0; j < row.size(); ++j) child[j] = row[j];
      for (int32_t i = 0; i < count[s]; ++i) {
        int32_t t = cu_seqlens[s] + i, pos = position[s] + i;
        token_seq[t] = int32_t(s);
        token_pos[t] = pos;
        int32_t page = child[pos / page_size];
        slot_mapping[t] = int64_t(page) * page_size + pos % page_size;
      }
    }
  });
}

// Speculative accept plan (src/serving/native_speculative.rs:74-128) over
// winners already computed: initial = argmax after the parent, rows[i] =
// argmax of verifier row i. Returns emitted count; writes emitted tokens,
// accepted, terminal.
int orc_accept(uint32_t initial, const uint32_t* draft, const uint32_t* rows, size_t n_draft,
               const uint32_t* eos, size_t n_eos, size_t remaining, uint32_t* emitted,
               uint32_t* n_emitted, uint32_t* accepted, uint32_t* terminal) {
  return guarded([&] {
    if (n_draft > 8 || n_draft > remaining || remaining == 0)
      throw std::invalid_argument("greedy draft/rows/context geometry");
    auto is_eos = [&](uint32_t t) { return std::find(eos, eos + n_eos, t) != eos + n_eos; };
    size_t ne = 0, acc = 0;
    bool term = false;
    for (size_t i = 0; i < n_draft; ++i) {
      uint32_t target = i == 0 ? initial : rows[i - 1];
      emitted[ne++] = target;
      term = is_eos(target);
      if (draft[i] != target || term) {
        acc += draft[i] == target;
        *n_emitted = uint32_t(ne);
        *accepted = uint32_t(acc);
        *terminal = term;
        return;
      }
      ++acc;
    }
    if (ne < remaining) {
      uint32_t bonus = n_draft ? rows[n_draft - 1] : initial;
      emitted[ne++] = bonus;
      term = is_eos(bonus);
    }
    *n_emitted = uint32_t(ne);
    *accepted = uint32_t(acc);
    *terminal = term;
  });
}

}  // extern "C"
