// Training checkpoints in Spar's SPARCKPT v1 format (src/checkpoint/checkpoint.cpp:18-475), so a
// Spar build can resume from a checkpoint written by this runtime and the reverse.
//
// Format (little-endian stream): "SPARCKPT", u32 version 1, u32 endian marker 0x01020304;
// DecoderConfig (u64 vocab, model_dim, hidden_dim, layers, query heads, kv heads; u8 dtype tag
// (1 = float32); bool attention_bias, mlp_bias; f64 norm_epsilon, rope_theta; bool qk_norm; f64
// qk_norm_epsilon); u64 global_step, tokens_seen; u64 RNG state; f64 AdamW learning rate, beta1,
// beta2, epsilon, weight_decay; u64 count + per parameter (named_parameters order): string name
// (u32 length + bytes), u8 dtype, bool requires_grad, u32 rank + u64 dims, u64 payload bytes,
// zero padding to the next 64-byte offset, the row-major values; u64 count + per parameter: name,
// bool has_state, [u64 step, u64 payload bytes, padded first moment, padded second moment].
// Readers reject any mismatch (magic, version, marker, config, names, shapes, byte counts, non-zero
// padding, trailing data).
//
// Host-only code: the entry points here take host arrays (one per named tensor, contiguous
// row-major, in named-parameter order) and need no GPU; the training runtime stages its device
// arenas through them (spar_b200_lm_{save,load}_checkpoint in trainer.cu).
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "checkpoint.h"

namespace spar_b200 {

namespace {

constexpr char kMagic[8] = {'S', 'P', 'A', 'R', 'C', 'K', 'P', 'T'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kEndianMarker = 0x01020304u;
constexpr uint64_t kAlign = 64;
constexpr uint8_t kFloat32 = 1;

class Out {
 public:
  explicit Out(const std::string& path) : f_(path, std::ios::binary | std::ios::trunc) {}
  bool ok() const { return static_cast<bool>(f_); }
  void bytes(const void* p, uint64_t n) {
    f_.write(static_cast<const char*>(p), static_cast<std::streamsize>(n));
    pos_ += n;
  }
  void u8(uint8_t v) { bytes(&v, 1); }
  void u32(uint32_t v) {
    uint8_t b[4];
    for (int i = 0; i < 4; ++i) b[i] = static_cast<uint8_t>(v >> (8 * i));
    bytes(b, 4);
  }
  void u64(uint64_t v) {
    uint8_t b[8];
    for (int i = 0; i < 8; ++i) b[i] = static_cast<uint8_t>(v >> (8 * i));
    bytes(b, 8);
  }
  void f64(double v) {
    uint64_t u;
    std::memcpy(&u, &v, 8);
    u64(u);
  }
  void str(const std::string& s) {
    u32(static_cast<uint32_t>(s.size()));
    bytes(s.data(), s.size());
  }
  void pad() {
    static const char zeros[kAlign] = {};
    bytes(zeros, (kAlign - pos_ % kAlign) % kAlign);
  }
  // float32 values, little-endian (this library only builds for little-endian hosts)
  void payload(const float* v, uint64_t n) {
    pad();
    bytes(v, n * 4);
  }
  bool close() {
    f_.flush();
    const bool good = static_cast<bool>(f_);
    f_.close();
    return good;
  }

 private:
  std::ofstream f_;
  uint64_t pos_ = 0;
};

class In {
 public:
  explicit In(const std::string& path) : f_(path, std::ios::binary) {}
  bool ok() const { return ok_ && static_cast<bool>(f_); }
  void bytes(void* p, uint64_t n) {
    if (!ok_) return;
    f_.read(static_cast<char*>(p), static_cast<std::streamsize>(n));
    if (static_cast<uint64_t>(f_.gcount()) != n) ok_ = false;
    pos_ += n;
  }
  uint8_t u8() {
    uint8_t v = 0;
    bytes(&v, 1);
    return v;
  }
  bool boolean() {
    const uint8_t v = u8();
    if (v > 1) ok_ = false;
    return v == 1;
  }
  uint32_t u32() {
    uint8_t b[4] = {};
    bytes(b, 4);
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) v |= static_cast<uint32_t>(b[i]) << (8 * i);
    return v;
  }
  uint64_t u64() {
    uint8_t b[8] = {};
    bytes(b, 8);
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(b[i]) << (8 * i);
    return v;
  }
  double f64() {
    const uint64_t u = u64();
    double v;
    std::memcpy(&v, &u, 8);
    return v;
  }
  std::string str() {
    const uint32_t n = u32();
    if (n > (1u << 20)) {
      ok_ = false;
      return {};
    }
    std::string s(n, '\0');
    bytes(&s[0], n);
    return s;
  }
  void pad() {
    char b[kAlign];
    const uint64_t n = (kAlign - pos_ % kAlign) % kAlign;
    bytes(b, n);
    for (uint64_t i = 0; i < n && ok_; ++i)
      if (b[i] != 0) ok_ = false;
  }
  void payload(float* v, uint64_t n) {
    pad();
    bytes(v, n * 4);
  }
  bool at_end() {
    char c;
    f_.read(&c, 1);
    return f_.gcount() == 0;
  }
  void fail() { ok_ = false; }

 private:
  std::ifstream f_;
  uint64_t pos_ = 0;
  bool ok_ = true;
};

SparCudaStatus bad() { return {1, 0}; }

}  // namespace

// Writes the checkpoint of `c` (family 1) from host arrays (m / v unused when adam_step == 0).
SparCudaStatus checkpoint_write(const char* path, const SparB200LMConfig& c,
                                const SparB200Checkpoint& meta, const float* const* values,
                                const float* const* m, const float* const* v) {
  std::vector<CkptTensor> ts;
  if (!path || !values || !checkpoint_tensors(c, ts)) return bad();
  if (meta.adam_step && (!m || !v)) return bad();
  const std::string tmp = std::string(path) + ".tmp";
  {
    Out o(tmp);
    if (!o.ok()) return {2, 0};
    o.bytes(kMagic, 8);
    o.u32(kVersion);
    o.u32(kEndianMarker);
    o.u64(c.vocab_size);
    o.u64(c.model_dim);
    o.u64(c.hidden_dim);
    o.u64(c.num_layers);
    o.u64(c.num_heads);
    o.u64(c.num_kv_heads ? c.num_kv_heads : c.num_heads);
    o.u8(kFloat32);
    o.u8(0);  // attention_bias
    o.u8(0);  // mlp_bias
    o.f64(c.norm_epsilon);
    o.f64(c.rope_theta);
    o.u8(c.qk_norm ? 1 : 0);
    o.f64(c.qk_norm_epsilon);
    o.u64(meta.global_step);
    o.u64(meta.tokens_seen);
    o.u64(meta.rng_state);
    o.f64(meta.learning_rate);
    o.f64(c.beta1);
    o.f64(c.beta2);
    o.f64(c.adam_epsilon);
    o.f64(c.weight_decay);
    o.u64(ts.size());
    for (size_t i = 0; i < ts.size(); ++i) {
      o.str(ts[i].name);
      o.u8(kFloat32);
      o.u8(1);  // requires_grad
      o.u32(static_cast<uint32_t>(ts[i].shape.size()));
      for (uint64_t dim : ts[i].shape) o.u64(dim);
      o.u64(ts[i].numel() * 4);
      o.payload(values[i], ts[i].numel());
    }
    o.u64(ts.size());
    for (size_t i = 0; i < ts.size(); ++i) {
      o.str(ts[i].name);
      o.u8(meta.adam_step ? 1 : 0);
      if (!meta.adam_step) continue;
      o.u64(meta.adam_step);
      o.u64(ts[i].numel() * 4);
      o.payload(m[i], ts[i].numel());
      o.payload(v[i], ts[i].numel());
    }
    if (!o.close()) {
      std::remove(tmp.c_str());
      return {2, 0};
    }
  }
  if (std::rename(tmp.c_str(), path) != 0) {
    std::remove(tmp.c_str());
    return {2, 0};
  }
  return {0, 0};
}

// Reads a checkpoint written for config `c` into host arrays (layout as checkpoint_write);
// meta receives progress, RNG state, learning rate and the AdamW step (0: no optimizer state,
// m / v zero-filled). Code 1 on any format or config mismatch.
SparCudaStatus checkpoint_read(const char* path, const SparB200LMConfig& c,
                               SparB200Checkpoint& meta, float* const* values, float* const* m,
                               float* const* v) {
  std::vector<CkptTensor> ts;
  if (!path || !values || !m || !v || !checkpoint_tensors(c, ts)) return bad();
  In in(path);
  if (!in.ok()) return {2, 0};
  char magic[8] = {};
  in.bytes(magic, 8);
  if (std::memcmp(magic, kMagic, 8) != 0 || in.u32() != kVersion || in.u32() != kEndianMarker)
    return bad();
  const uint64_t kvh = c.num_kv_heads ? c.num_kv_heads : c.num_heads;
  const bool cfg_ok = in.u64() == c.vocab_size && in.u64() == c.model_dim &&
                      in.u64() == c.hidden_dim && in.u64() == c.num_layers &&
                      in.u64() == c.num_heads && in.u64() == kvh && in.u8() == kFloat32 &&
                      !in.boolean() && !in.boolean() && in.f64() == c.norm_epsilon &&
                      in.f64() == c.rope_theta && in.boolean() == (c.qk_norm != 0) &&
                      in.f64() == c.qk_norm_epsilon;
  if (!cfg_ok || !in.ok()) return bad();
  meta.global_step = in.u64();
  meta.tokens_seen = in.u64();
  meta.rng_state = in.u64();
  meta.learning_rate = in.f64();
  // The runtime's AdamW hyper-parameters are part of its config: they must match.
  if (in.f64() != c.beta1 || in.f64() != c.beta2 || in.f64() != c.adam_epsilon ||
      in.f64() != c.weight_decay || !in.ok())
    return bad();
  std::map<std::string, size_t> index;
  for (size_t i = 0; i < ts.size(); ++i) index[ts[i].name] = i;
  if (in.u64() != ts.size()) return bad();
  std::set<std::string> seen;
  for (size_t k = 0; k < ts.size() && in.ok(); ++k) {
    const std::string name = in.str();
    const auto it = index.find(name);
    if (it == index.end() || !seen.insert(name).second) return bad();
    const CkptTensor& t = ts[it->second];
    if (in.u8() != kFloat32) return bad();
    in.boolean();  // requires_grad: every parameter of this runtime trains
    const uint32_t rank = in.u32();
    if (rank != t.shape.size()) return bad();
    for (uint64_t dim : t.shape)
      if (in.u64() != dim) return bad();
    if (in.u64() != t.numel() * 4) return bad();
    in.payload(values[it->second], t.numel());
  }
  if (!in.ok() || in.u64() != ts.size()) return bad();
  seen.clear();
  uint64_t step = 0;
  bool any = false, all = true;
  for (size_t k = 0; k < ts.size() && in.ok(); ++k) {
    const std::string name = in.str();
    const auto it = index.find(name);
    if (it == index.end() || !seen.insert(name).second) return bad();
    const CkptTensor& t = ts[it->second];
    if (!in.boolean()) {
      all = false;
      std::memset(m[it->second], 0, t.numel() * 4);
      std::memset(v[it->second], 0, t.numel() * 4);
      continue;
    }
    const uint64_t s = in.u64();
    if (s == 0 || (any && s != step)) return bad();  // one AdamW step counter in this runtime
    step = s;
    any = true;
    if (in.u64() != t.numel() * 4) return bad();
    in.payload(m[it->second], t.numel());
    in.payload(v[it->second], t.numel());
  }
  if (!in.ok() || (any && !all) || !in.at_end()) return bad();
  meta.adam_step = step;
  return {0, 0};
}

}  // namespace spar_b200

using namespace spar_b200;

extern "C" SparCudaStatus spar_b200_checkpoint_write(const char* path,
                                                     const SparB200LMConfig* config,
                                                     const SparB200Checkpoint* meta,
                                                     const float* const* values,
                                                     const float* const* first_moments,
                                                     const float* const* second_moments) {
  if (!config || !meta) return bad();
  return checkpoint_write(path, *config, *meta, values, first_moments, second_moments);
}

extern "C" SparCudaStatus spar_b200_checkpoint_read(const char* path,
                                                    const SparB200LMConfig* config,
                                                    SparB200Checkpoint* meta, float* const* values,
                                                    float* const* first_moments,
                                                    float* const* second_moments) {
  if (!config || !meta) return bad();
  return checkpoint_read(path, *config, *meta, values, first_moments, second_moments);
}
