// TEST INFRASTRUCTURE — C ABI over the reference's OWN scalar oracle headers.
//
// Compiled only by oracle/Makefile (target `ref`) against the reference tree
// (REF=<reference checkout>/native) into oracle/_ref/libref_oracle.so; no
// reference source is copied into this repository. Used to pin the in-repo
// restatement (qwen_oracle.cpp) and to generate tests/golden fixtures.
// Wrapped headers: native/operator_reference.h, native/projection_reference.h,
// native/attention_reference.h.
#include <cstring>
#include <string>
#include <vector>
#include "operator_reference.h"
#include "projection_reference.h"
#include "attention_reference.h"

namespace {
thread_local std::string err;
template <class F> int run(F f) {
  try { f(); return 0; } catch (const std::exception& e) { err = e.what(); } catch (...) { err = "unknown"; }
  return -1;
}
std::vector<float> vec(const float* p, size_t n) { return std::vector<float>(p, p + n); }
void put(const std::vector<double>& v, double* out) { std::memcpy(out, v.data(), v.size() * sizeof(double)); }
}

extern "C" {
const char* ref_last_error() { return err.c_str(); }
int ref_rms(const float* x, size_t n, const float* w, size_t nw, size_t width, double eps, double* y) {
  return run([&] { put(scalar_reference::rms(vec(x, n), vec(w, nw), width, eps), y); });
}
int ref_silu(const float* x, size_t n, double* y) { return run([&] { put(scalar_reference::silu(vec(x, n)), y); }); }
int ref_rope(const float* x, int heads, int tokens, int dim, int rotary, int offset, double theta, double* y) {
  return run([&] { put(scalar_reference::rope(vec(x, size_t(heads) * tokens * dim), heads, tokens, dim, rotary, offset, theta), y); });
}
int ref_delta(const float* qkv, const float* history, const float* conv, const float* a, const float* b,
              const float* alog, const float* dt, const float* initial, int tokens, int hk, int hv, int dk,
              int dv, int kernel, double* activated, double* history_out, double* output, double* state) {
  return run([&] {
    size_t kd = size_t(hk) * dk, vd = size_t(hv) * dv, ch = 2 * kd + vd;
    auto r = scalar_reference::delta(vec(qkv, size_t(tokens) * ch), vec(history, size_t(kernel - 1) * ch),
                                     vec(conv, ch * kernel), vec(a, size_t(tokens) * hv), vec(b, size_t(tokens) * hv),
                                     vec(alog, hv), vec(dt, hv), vec(initial, size_t(hv) * dv * dk), tokens, hk, hv,
                                     dk, dv, kernel);
    put(r.activated, activated); put(r.history, history_out); put(r.output, output); put(r.state, state);
  });
}
int ref_routing(const float* logits, const int* selected, int rows, int experts, int top, double* probs, double* weights) {
  return run([&] {
    auto r = scalar_reference::routing(vec(logits, size_t(rows) * experts),
                                       std::vector<int32_t>(selected, selected + size_t(rows) * top), rows, experts, top);
    put(r.probabilities, probs); put(r.weights, weights);
  });
}
int ref_projection(const float* x, const uint32_t* packed, const float* scales, const float* biases, size_t rows,
                   size_t outputs, size_t width, int group, int bits, double* y) {
  return run([&] {
    size_t words = width * bits / 32, groups = width / group;
    put(projection_reference(vec(x, rows * width), std::vector<uint32_t>(packed, packed + outputs * words),
                             vec(scales, outputs * groups), vec(biases, outputs * groups), rows, outputs, width, group, bits), y);
  });
}
int ref_attention(const float* q, const float* k, const float* v, int heads, int kv_heads, int tokens, int offset,
                  int dim, double* out) {
  return run([&] {
    size_t n = size_t(offset) + tokens;
    put(attention_reference(vec(q, size_t(heads) * tokens * dim), vec(k, size_t(kv_heads) * n * dim),
                            vec(v, size_t(kv_heads) * n * dim), heads, kv_heads, tokens, offset, dim), out);
  });
}
}
