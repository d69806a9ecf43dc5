// C API over the reference's public C++ API (bzzling/spar), compiled together with the reference
// sources by oracle/make_ref.py. TEST INFRASTRUCTURE: used to pin the numpy oracle (golden
// fixtures) and as the CPU baseline; never part of the product.
//
// LayerNorm and GELU do not exist in Spar; they are composed from Spar ops exactly as the
// oracle documents (mean/subtract/square/mean/add_scalar/sqrt/divide/multiply/add, and
// x * sigmoid(2*sqrt(2/pi)*(x + 0.044715 x^3))). The decoder uses Spar's own Embedding,
// SelfAttention (bias, RoPE) and Linear modules, Spar's autograd, LM cross-entropy,
// clip_grad_norm, AdamW and warmup-cosine schedule.
#include "spar.hpp"
#ifdef SPAR_B200_FUSED
#include "spar.b200.hpp"  // the product's fused differentiable operations (drop-in build only)
#endif

#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

using namespace spar;

namespace {

thread_local std::string g_error;

using dim = Shape::dimension_type;

Tensor from_host(const float* data, std::vector<dim> shape, bool grad) {
  Tensor t{Shape{std::move(shape)}, DType::Float32};
  auto s = t.span<float>();
  std::memcpy(s.data(), data, s.size() * sizeof(float));
  if (grad) t.set_requires_grad(true);
  return t;
}

Tensor ids_from_host(const int32_t* data, std::vector<dim> shape) {
  Tensor t{Shape{std::move(shape)}, DType::Int32};
  auto s = t.span<int32_t>();
  std::memcpy(s.data(), data, s.size() * sizeof(int32_t));
  return t;
}

// device < 0: the CPU; otherwise Device::cuda(device) (builds with SPAR_ENABLE_CUDA=1).
Device device_of(int64_t device) {
  return device < 0 ? Device::cpu() : Device::cuda(static_cast<std::int32_t>(device));
}

// The value of a one-element float tensor on any device.
float scalar_of(const Tensor& t) {
  const Tensor c = t.detach().to(Device::cpu());
  return c.span<float>()[0];
}

void to_host(const Tensor& t, float* out) {
  const Tensor c = t.detach().to(Device::cpu()).contiguous();
  auto s = std::as_const(c).span<float>();
  std::memcpy(out, s.data(), s.size() * sizeof(float));
}

Tensor layer_norm(const Tensor& x, const Tensor& gamma, const Tensor& beta, double eps) {
  const std::size_t axis = x.rank() - 1;
  const Tensor mu = mean(x, axis, true);
  const Tensor xc = subtract(x, mu);
  const Tensor var = mean(square(xc), axis, true);
  const Tensor den = sqrt(add_scalar(var, eps));
  return add(multiply(divide(xc, den), gamma), beta);
}

Tensor gelu(const Tensor& x) {
  const Tensor x3 = multiply(multiply(x, x), x);
  const Tensor u = multiply_scalar(add(x, multiply_scalar(x3, 0.044715)), 1.5957691216057308);
  return multiply(x, sigmoid(u));
}

Tensor weighted_sum(const Tensor& y, const float* w) {
  std::vector<dim> shape(y.shape().dimensions().begin(), y.shape().dimensions().end());
  return sum(multiply(y, from_host(w, shape, false)));
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}

struct Block {
  nn::Parameter ln1_g, ln1_b;
  nn::SelfAttention attn;
  nn::Parameter ln2_g, ln2_b;
  nn::Linear up, down;
  Block(std::size_t d, std::size_t f, std::size_t h, double theta, Random& rng)
      : ln1_g{ones(Shape{dim(d)}, DType::Float32)}, ln1_b{zeros(Shape{dim(d)}, DType::Float32)},
        attn{d, h, h, DType::Float32, rng, true, theta},
        ln2_g{ones(Shape{dim(d)}, DType::Float32)}, ln2_b{zeros(Shape{dim(d)}, DType::Float32)},
        up{d, f, DType::Float32, rng, true}, down{f, d, DType::Float32, rng, true} {}
};

struct Model {
  nn::Embedding embedding;
  std::vector<Block> blocks;
  nn::Parameter lnf_g, lnf_b;
  double eps;
  Model(std::size_t v, std::size_t d, std::size_t f, std::size_t layers, std::size_t h,
        double theta, double eps_, Random& rng)
      : embedding{v, d, DType::Float32, rng}, lnf_g{ones(Shape{dim(d)}, DType::Float32)},
        lnf_b{zeros(Shape{dim(d)}, DType::Float32)}, eps{eps_} {
    blocks.reserve(layers);
    for (std::size_t i = 0; i < layers; ++i) blocks.emplace_back(d, f, h, theta, rng);
  }
  // Named-parameter order (src/nn/parameters.cpp:51-132 with LayerNorm weight+bias).
  std::vector<nn::Parameter> parameters() {
    std::vector<nn::Parameter> p{embedding.weight()};
    for (Block& b : blocks) {
      p.push_back(b.ln1_g);
      p.push_back(b.ln1_b);
      for (nn::Linear* l : {&b.attn.q_proj(), &b.attn.k_proj(), &b.attn.v_proj(), &b.attn.out_proj()}) {
        p.push_back(l->weight());
        p.push_back(*l->bias());
      }
      p.push_back(b.ln2_g);
      p.push_back(b.ln2_b);
      for (nn::Linear* l : {&b.up, &b.down}) {
        p.push_back(l->weight());
        p.push_back(*l->bias());
      }
    }
    p.push_back(lnf_g);
    p.push_back(lnf_b);
    return p;
  }
#ifdef SPAR_B200_FUSED
  // The same decoder with the product's fused operations recorded on Spar's tape: LayerNorm,
  // the MLP's up projection + bias + GELU, and (in the caller) the LM cross-entropy. Every
  // up-projection weight and LayerNorm gain passes through b200::grad_ready with `hook`.
  Tensor logits_fused(const Tensor& ids,
                      const std::function<void(int, const Tensor&)>& hook) {
    int slot = 0;
    auto ready = [&](const nn::Parameter& p) {
      const int id = slot++;
      // The hook is copied into the node: the node's backward runs after this call returns.
      return b200::grad_ready(p.tensor(), [id, hook](const Tensor& g) { hook(id, g); });
    };
    Tensor h = embedding.forward(ids);
    for (Block& b : blocks) {
      const Tensor a1 = b200::layer_norm(h, ready(b.ln1_g), b.ln1_b.tensor(), eps);
      const Tensor h1 = add(h, b.attn.forward(a1));
      const Tensor a2 = b200::layer_norm(h1, ready(b.ln2_g), b.ln2_b.tensor(), eps);
      const Tensor g = b200::linear_gelu(a2, ready(b.up.weight()), b.up.bias()->tensor());
      h = add(h1, b.down.forward(g));
    }
    const Tensor hf = b200::layer_norm(h, lnf_g.tensor(), lnf_b.tensor(), eps);
    return matmul(hf, embedding.weight().tensor().transpose(0, 1));
  }
#endif
  Tensor logits(const Tensor& ids) {
    Tensor h = embedding.forward(ids);
    for (Block& b : blocks) {
      const Tensor h1 = add(h, b.attn.forward(layer_norm(h, b.ln1_g.tensor(), b.ln1_b.tensor(), eps)));
      const Tensor a2 = layer_norm(h1, b.ln2_g.tensor(), b.ln2_b.tensor(), eps);
      h = add(h1, b.down.forward(gelu(b.up.forward(a2))));
    }
    const Tensor hf = layer_norm(h, lnf_g.tensor(), lnf_b.tensor(), eps);
    return matmul(hf, embedding.weight().tensor().transpose(0, 1));
  }
};

void load(nn::Parameter& p, const float* src) {
  Tensor values = p.tensor().detach();
  auto s = values.span<float>();
  std::memcpy(s.data(), src, s.size() * sizeof(float));
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

// Composed LayerNorm forward + backward of sum(y * dy).
int ref_layernorm(const float* x, const float* gamma, const float* beta, const float* dy,
                  int64_t rows, int64_t cols, double eps, float* y, float* dx, float* dgamma,
                  float* dbeta) {
  return guarded([&] {
    Tensor tx = from_host(x, {rows, cols}, true);
    Tensor tg = from_host(gamma, {cols}, true);
    Tensor tb = from_host(beta, {cols}, true);
    Tensor out = layer_norm(tx, tg, tb, eps);
    to_host(out, y);
    Tensor loss = weighted_sum(out, dy);
    loss.backward();
    to_host(tx.grad(), dx);
    to_host(tg.grad(), dgamma);
    to_host(tb.grad(), dbeta);
  });
}

// nn::RMSNorm (src/nn/rmsnorm.cpp:40-53) with the given weight; dx, dweight for upstream dy.
int ref_rmsnorm(const float* x, const float* weight, const float* dy, int64_t rows, int64_t cols,
                double eps, float* y, float* dx, float* dweight) {
  return guarded([&] {
    nn::RMSNorm norm{static_cast<std::size_t>(cols), DType::Float32, eps};
    load(norm.weight(), weight);
    Tensor tx = from_host(x, {rows, cols}, true);
    Tensor out = norm.forward(tx);
    to_host(out, y);
    Tensor loss = weighted_sum(out, dy);
    loss.backward();
    to_host(tx.grad(), dx);
    to_host(norm.weight().tensor().grad(), dweight);
  });
}

// nn::swiglu (src/nn/functional.cpp:9-11): h = silu(gate) * value; d gate, d value for dh.
int ref_swiglu(const float* gate, const float* value, const float* dh, int64_t n, float* h,
               float* dgate, float* dvalue) {
  return guarded([&] {
    Tensor tg = from_host(gate, {n}, true);
    Tensor tv = from_host(value, {n}, true);
    Tensor out = nn::swiglu(tg, tv);
    to_host(out, h);
    Tensor loss = weighted_sum(out, dh);
    loss.backward();
    to_host(tg.grad(), dgate);
    to_host(tv.grad(), dvalue);
  });
}

// nn::scaled_dot_product_attention (src/nn/attention.cpp:121-135), causal, with key / value of
// kv_heads heads (repeat_kv_heads inside): q [b, heads, t, dh], k / v [b, kv_heads, t, dh].
int ref_attention(const float* q, const float* k, const float* v, const float* d_out, int64_t b,
                  int64_t heads, int64_t kv_heads, int64_t t, int64_t dh, float* out, float* dq,
                  float* dk, float* dv) {
  return guarded([&] {
    Tensor tq = from_host(q, {b, heads, t, dh}, true);
    Tensor tk = from_host(k, {b, kv_heads, t, dh}, true);
    Tensor tv = from_host(v, {b, kv_heads, t, dh}, true);
    Tensor o = nn::scaled_dot_product_attention(tq, tk, tv, true);
    to_host(o, out);
    Tensor loss = weighted_sum(o, d_out);
    loss.backward();
    to_host(tq.grad(), dq);
    to_host(tk.grad(), dk);
    to_host(tv.grad(), dv);
  });
}

int ref_gelu(const float* x, const float* dy, int64_t n, float* y, float* dx) {
  return guarded([&] {
    Tensor tx = from_host(x, {n}, true);
    Tensor out = gelu(tx);
    to_host(out, y);
    Tensor loss = weighted_sum(out, dy);
    loss.backward();
    to_host(tx.grad(), dx);
  });
}

// scores [batch, t, t] -> P = softmax(scale * s + causal mask, axis 2); dS for upstream dp.
int ref_causal_softmax(const float* s, const float* dp, int64_t batch, int64_t t, double scale,
                       float* p, float* ds) {
  return guarded([&] {
    Tensor ts = from_host(s, {batch, t, t}, true);
    Tensor mask = zeros(Shape{t, t}, DType::Float32);
    auto mv = mask.span<float>();
    for (int64_t i = 0; i < t; ++i)
      for (int64_t j = i + 1; j < t; ++j) mv[i * t + j] = -std::numeric_limits<float>::infinity();
    Tensor probs = softmax(add(multiply_scalar(ts, scale), mask), 2);
    to_host(probs, p);
    Tensor loss = weighted_sum(probs, dp);
    loss.backward();
    to_host(ts.grad(), ds);
  });
}

// seq == 0: loss::cross_entropy over [rows, classes]; seq > 1: language_model_cross_entropy
// over [rows/seq, seq, classes] with targets = the id tensor. Mean reduction.
int ref_cross_entropy(const float* logits, const int32_t* targets, int64_t rows, int64_t classes,
                      int64_t seq, float* loss_out, float* dlogits) {
  return guarded([&] {
    Tensor z = seq ? from_host(logits, {rows / seq, seq, classes}, true)
                   : from_host(logits, {rows, classes}, true);
    Tensor loss = seq ? loss::language_model_cross_entropy(z, ids_from_host(targets, {rows / seq, seq}))
                      : loss::cross_entropy(z, ids_from_host(targets, {rows}));
    *loss_out = std::as_const(loss).span<float>()[0];
    loss.backward();
    to_host(z.grad(), dlogits);
  });
}

int ref_matmul(const float* a, const float* b, const float* dc, int64_t m, int64_t k, int64_t n,
               float* c, float* da, float* db) {
  return guarded([&] {
    Tensor ta = from_host(a, {m, k}, true);
    Tensor tb = from_host(b, {k, n}, true);
    Tensor out = matmul(ta, tb);
    to_host(out, c);
    Tensor loss = weighted_sum(out, dc);
    loss.backward();
    to_host(ta.grad(), da);
    to_host(tb.grad(), db);
  });
}

// `steps` consecutive clip_grad_norm + AdamW steps on one parameter with a fixed gradient.
int ref_adamw(float* p, const float* g, float* m_out, float* v_out, int64_t n, int64_t steps,
              double lr, double beta1, double beta2, double eps, double wd, double max_norm,
              double* norm_out) {
  return guarded([&] {
    nn::Parameter param{from_host(p, {n}, false)};
    optim::AdamW opt{{param}, lr, beta1, beta2, eps, wd};
    std::vector<nn::Parameter> list{param};
    for (int64_t s = 0; s < steps; ++s) {
      param.zero_grad();
      Tensor loss = weighted_sum(param.tensor(), g);  // d loss / d p = g
      loss.backward();
      if (max_norm >= 0) *norm_out = training::clip_grad_norm(list, max_norm).total_norm;
      opt.step();
    }
    to_host(param.tensor(), p);
    const auto state = opt.parameter_state(param);
    to_host(state->first_moment, m_out);
    to_host(state->second_moment, v_out);
  });
}

double ref_warmup_cosine(double peak, double minimum, uint64_t warmup, uint64_t decay,
                         uint64_t step) {
  return training::warmup_cosine_learning_rate({peak, minimum, warmup, decay}, step);
}

// apply_rope on x [outer, t, d] (forward), then its backward of sum(out * dy).
int ref_rope(const float* x, const float* dy, int64_t outer, int64_t t, int64_t d, double theta,
             float* out, float* dx) {
  return guarded([&] {
    Tensor tx = from_host(x, {outer, t, d}, true);
    Tensor r = nn::apply_rope(tx, 0, theta);
    to_host(r, out);
    Tensor loss = weighted_sum(r, dy);
    loss.backward();
    to_host(tx.grad(), dx);
  });
}

// One optimiser step of the LN/GELU decoder: `micro` micro-batches of ids [batch, t] each,
// mean-of-micro-batch-means loss, Spar backward, clip_grad_norm, AdamW. params/grads/out_params
// are arrays of pointers in named-parameter order (embedding, per block: ln1 w/b, q/k/v/out
// w/b, ln2 w/b, up w/b, down w/b; final ln w/b). grads are the pre-clip gradients.
// `device` (last argument): < 0 runs on the CPU, otherwise the parameters are moved to
// Device::cuda(device) (nn::move_to) and the whole step runs through Spar's CUDA backend.
int ref_lm_step(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads, int64_t batch,
                int64_t t, int64_t micro, double eps, double theta, const float* const* params,
                const int32_t* ids, double lr, double beta1, double beta2, double adam_eps,
                double wd, double max_norm, float* loss_out, double* norm_out, float** grads,
                float** out_params, int64_t device) {
  return guarded([&] {
    Random rng{1};
    Model model(vocab, d, f, layers, heads, theta, eps, rng);
    std::vector<nn::Parameter> ps = model.parameters();
    for (std::size_t i = 0; i < ps.size(); ++i) load(ps[i], params[i]);
    const Device dev = device_of(device);
    nn::move_to(std::span<nn::Parameter>{ps}, dev);
    double total = 0.0;
    for (int64_t mi = 0; mi < micro; ++mi) {
      Tensor tid = ids_from_host(ids + mi * batch * t, {batch, t}).to(dev);
      Tensor loss = loss::language_model_cross_entropy(model.logits(tid), tid);
      total += scalar_of(loss);
      Tensor scaled = multiply_scalar(loss, 1.0 / static_cast<double>(micro));
      scaled.backward();
    }
    *loss_out = static_cast<float>(total / static_cast<double>(micro));
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].grad(), grads[i]);
    *norm_out = training::clip_grad_norm(ps, max_norm).total_norm;
    optim::AdamW opt{ps, lr, beta1, beta2, adam_eps, wd};
    opt.step();
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].tensor(), out_params[i]);
  });
}

// Spar's own decoder (nn::DecoderLM, src/nn/decoder.cpp: RMSNorm, RoPE self-attention with
// num_kv_heads key/value heads and optional q/k RMSNorm, SwiGLU MLP, no biases, tied logits).
nn::DecoderConfig spar_config(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads,
                              int64_t kv_heads, int64_t qk_norm, double eps, double theta) {
  nn::DecoderConfig c;
  c.vocab_size = static_cast<std::size_t>(vocab);
  c.model_dim = static_cast<std::size_t>(d);
  c.hidden_dim = static_cast<std::size_t>(f);
  c.num_layers = static_cast<std::size_t>(layers);
  c.num_query_heads = static_cast<std::size_t>(heads);
  c.num_kv_heads = static_cast<std::size_t>(kv_heads);
  c.norm_epsilon = eps;
  c.rope_theta = theta;
  c.qk_norm = qk_norm != 0;
  return c;
}

// Name and element count of named parameter `index` of that decoder (named_parameters order).
int ref_spar_param_info(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads,
                        int64_t kv_heads, int64_t qk_norm, int64_t index, char* name,
                        int64_t capacity, int64_t* numel) {
  return guarded([&] {
    Random rng{1};
    nn::DecoderLM model{spar_config(vocab, d, f, layers, heads, kv_heads, qk_norm, 1e-5, 1e4), rng};
    const auto named = nn::named_parameters(model);
    if (index < 0) {
      *numel = static_cast<int64_t>(named.size());
      return;
    }
    const auto& np = named.at(static_cast<std::size_t>(index));
    std::snprintf(name, static_cast<std::size_t>(capacity), "%s", np.name.c_str());
    *numel = static_cast<int64_t>(np.parameter.tensor().numel());
  });
}

// One optimiser step of nn::DecoderLM: as ref_lm_step (micro-batches, mean loss, backward,
// clip_grad_norm, AdamW), parameters in named_parameters order.
int ref_spar_lm_step(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads,
                     int64_t kv_heads, int64_t qk_norm, int64_t batch, int64_t t, int64_t micro,
                     double eps, double theta, const float* const* params, const int32_t* ids,
                     double lr, double beta1, double beta2, double adam_eps, double wd,
                     double max_norm, float* loss_out, double* norm_out, float** grads,
                     float** out_params, int64_t device) {
  return guarded([&] {
    Random rng{1};
    nn::DecoderLM model{spar_config(vocab, d, f, layers, heads, kv_heads, qk_norm, eps, theta), rng};
    std::vector<nn::Parameter> ps;
    for (auto& np : nn::named_parameters(model)) ps.push_back(np.parameter);
    for (std::size_t i = 0; i < ps.size(); ++i) load(ps[i], params[i]);
    const Device dev = device_of(device);
    nn::move_to(model, dev);
    double total = 0.0;
    for (int64_t mi = 0; mi < micro; ++mi) {
      Tensor tid = ids_from_host(ids + mi * batch * t, {batch, t}).to(dev);
      Tensor loss = loss::language_model_cross_entropy(model.forward(tid), tid);
      total += scalar_of(loss);
      Tensor scaled = multiply_scalar(loss, 1.0 / static_cast<double>(micro));
      scaled.backward();
    }
    *loss_out = static_cast<float>(total / static_cast<double>(micro));
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].grad(), grads[i]);
    *norm_out = training::clip_grad_norm(ps, max_norm).total_norm;
    optim::AdamW opt{ps, lr, beta1, beta2, adam_eps, wd};
    opt.step();
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].tensor(), out_params[i]);
  });
}

// checkpoint::save_training_checkpoint of nn::DecoderLM with the given parameters, an AdamW whose
// every parameter state is (m, v, adam_step) (none when adam_step == 0), a Random at rng_state.
int ref_spar_ckpt_save(const char* path, int64_t vocab, int64_t d, int64_t f, int64_t layers,
                       int64_t heads, int64_t kv_heads, int64_t qk_norm, double eps, double theta,
                       double qk_eps, const float* const* params, const float* const* m,
                       const float* const* v, uint64_t adam_step, uint64_t global_step,
                       uint64_t tokens, uint64_t rng_state, double lr, double beta1, double beta2,
                       double adam_eps, double wd) {
  return guarded([&] {
    Random rng{1};
    nn::DecoderConfig c = spar_config(vocab, d, f, layers, heads, kv_heads, qk_norm, eps, theta);
    c.qk_norm_epsilon = qk_eps;
    nn::DecoderLM model{c, rng};
    std::vector<nn::Parameter> ps;
    for (auto& np : nn::named_parameters(model)) ps.push_back(np.parameter);
    for (std::size_t i = 0; i < ps.size(); ++i) load(ps[i], params[i]);
    optim::AdamW opt{ps, lr, beta1, beta2, adam_eps, wd};
    if (adam_step)
      for (std::size_t i = 0; i < ps.size(); ++i) {
        const auto shape = ps[i].tensor().shape();
        std::vector<dim> dims(shape.dimensions().begin(), shape.dimensions().end());
        opt.set_parameter_state(ps[i], optim::AdamWParameterState{from_host(m[i], dims, false),
                                                                  from_host(v[i], dims, false),
                                                                  adam_step});
      }
    Random random{0};
    random.set_state(rng_state);
    checkpoint::save_training_checkpoint(path, model, opt, random, {global_step, tokens});
  });
}

// checkpoint::load_training_checkpoint: parameters, moments (zero without state), the AdamW step
// of the first parameter, progress, RNG state and learning rate.
int ref_spar_ckpt_load(const char* path, float** params, float** m, float** v,
                       uint64_t* adam_step, uint64_t* global_step, uint64_t* tokens,
                       uint64_t* rng_state, double* lr) {
  return guarded([&] {
    auto loaded = checkpoint::load_training_checkpoint(path);
    const auto named = nn::named_parameters(loaded.model);
    *adam_step = 0;
    for (std::size_t i = 0; i < named.size(); ++i) {
      to_host(named[i].parameter.tensor(), params[i]);
      const auto st = loaded.optimizer.parameter_state(named[i].parameter);
      const std::size_t n = named[i].parameter.tensor().numel();
      if (st) {
        to_host(st->first_moment, m[i]);
        to_host(st->second_moment, v[i]);
        if (i == 0) *adam_step = st->step;
      } else {
        std::memset(m[i], 0, n * sizeof(float));
        std::memset(v[i], 0, n * sizeof(float));
      }
    }
    *global_step = loaded.progress.global_step;
    *tokens = loaded.progress.tokens_seen;
    *rng_state = loaded.random.state();
    *lr = loaded.optimizer.learning_rate();
  });
}

// data::LMBatchIterator over data::WindowDataset of the TokenizedCorpus of `ndocs` documents
// (bytes `docs`, lengths `lens`) under the byte-level ByteBPETokenizer: the packed corpus tokens
// (tokens_out, *token_count) and every batch of `epochs` epochs, rows concatenated in batches_out
// ([sum rows, seq] int32), rows per batch in rows_out, *n_batches batches.
int ref_batches(const char* docs, const int64_t* lens, int64_t ndocs, int64_t seq, int64_t stride,
                int64_t batch, int64_t shuffle, uint64_t seed, int64_t drop_last, int64_t epochs,
                int32_t* tokens_out, int64_t* token_count, int32_t* batches_out, int64_t* rows_out,
                int64_t* n_batches) {
  return guarded([&] {
    std::vector<std::string> documents;
    const char* p = docs;
    for (int64_t i = 0; i < ndocs; ++i) {
      documents.emplace_back(p, static_cast<std::size_t>(lens[i]));
      p += lens[i];
    }
    tokenizer::ByteBPETokenizer tok;
    data::TokenizedCorpus corpus{documents, tok};
    const auto toks = corpus.tokens();
    for (std::size_t i = 0; i < toks.size(); ++i) tokens_out[i] = static_cast<int32_t>(toks[i]);
    *token_count = static_cast<int64_t>(toks.size());
    data::WindowDataset windows{corpus, {static_cast<std::size_t>(seq), static_cast<std::size_t>(stride)}};
    data::BatchConfig bc{static_cast<std::size_t>(batch), DType::Int32, shuffle != 0, seed,
                         drop_last != 0};
    data::LMBatchIterator it{windows, bc};
    int64_t nb = 0, row = 0;
    for (int64_t e = 0; e < epochs; ++e) {
      if (e > 0) it.next_epoch();
      while (auto b = it.next_batch()) {
        const auto v = std::as_const(*b).span<int32_t>();
        std::memcpy(batches_out + row * seq, v.data(), v.size() * sizeof(int32_t));
        rows_out[nb++] = b->shape()[0];
        row += b->shape()[0];
      }
    }
    *n_batches = nb;
  });
}

// data::split_documents: validation indices then training indices into `out`.
int ref_split_documents(int64_t count, int64_t validation, uint64_t seed, int64_t* out) {
  return guarded([&] {
    const auto split = data::split_documents(static_cast<std::size_t>(count),
                                             static_cast<std::size_t>(validation), seed);
    std::size_t k = 0;
    for (std::size_t i : split.validation_indices) out[k++] = static_cast<int64_t>(i);
    for (std::size_t i : split.train_indices) out[k++] = static_cast<int64_t>(i);
  });
}

// Seconds for `iters` training steps (forward, loss, backward, clip, AdamW) of a one-block
// decoder with the given dimensions on [1, t] token ids: the bounded CPU-baseline sample.
double ref_train_sample_seconds(int64_t vocab, int64_t d, int64_t f, int64_t heads, int64_t t,
                                int64_t iters) {
  double seconds = -1.0;
  guarded([&] {
    Random rng{7};
    Model model(vocab, d, f, 1, heads, 10000.0, 1e-5, rng);
    std::vector<nn::Parameter> ps = model.parameters();
    optim::AdamW opt{ps, 3e-4, 0.9, 0.95, 1e-8, 0.1};
    Tensor tid{Shape{1, t}, DType::Int32};
    auto s = tid.span<int32_t>();
    for (int64_t i = 0; i < t; ++i) s[i] = static_cast<int32_t>((i * 7919) % vocab);
    const auto t0 = std::chrono::steady_clock::now();
    for (int64_t it = 0; it < iters; ++it) {
      for (auto& p : ps) p.zero_grad();
      Tensor loss = loss::language_model_cross_entropy(model.logits(tid), tid);
      loss.backward();
      (void)training::clip_grad_norm(ps, 1.0);
      opt.step();
    }
    seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  });
  return seconds;
}

#ifdef SPAR_B200_FUSED
// ref_lm_step with the product's fused operations (logits_fused + b200::language_model_cross_
// entropy) on Device::cuda(device), through Spar's own autograd, clip and AdamW. hook_calls[i]
// and hook_norms[i] report how often grad_ready slot i fired and the norm of the gradient it saw
// (slots: per block ln1 gain, ln2 gain, up-projection weight); hook_order lists the slots in
// firing order (3 * layers * micro entries).
int ref_lm_step_fused(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads,
                      int64_t batch, int64_t t, int64_t micro, double eps, double theta,
                      const float* const* params, const int32_t* ids, double lr, double beta1,
                      double beta2, double adam_eps, double wd, double max_norm, float* loss_out,
                      double* norm_out, float** grads, float** out_params, int64_t device,
                      int64_t* hook_calls, double* hook_norms, int64_t* hook_order) {
  return guarded([&] {
    Random rng{1};
    Model model(vocab, d, f, layers, heads, theta, eps, rng);
    std::vector<nn::Parameter> ps = model.parameters();
    for (std::size_t i = 0; i < ps.size(); ++i) load(ps[i], params[i]);
    const Device dev = device_of(device);
    nn::move_to(std::span<nn::Parameter>{ps}, dev);
    const int64_t slots = 3 * layers;
    for (int64_t i = 0; i < slots; ++i) hook_calls[i] = 0;
    int64_t fired = 0;
    auto hook = [&](int id, const Tensor& g) {
      ++hook_calls[id];
      hook_order[fired++] = id;
      const Tensor c = g.detach().to(Device::cpu()).contiguous();
      double s = 0.0;
      for (float v : std::as_const(c).span<float>()) s += static_cast<double>(v) * v;
      hook_norms[id] = std::sqrt(s);
    };
    double total = 0.0;
    for (int64_t mi = 0; mi < micro; ++mi) {
      Tensor tid = ids_from_host(ids + mi * batch * t, {batch, t}).to(dev);
      Tensor loss = b200::language_model_cross_entropy(model.logits_fused(tid, hook), tid);
      total += scalar_of(loss);
      Tensor scaled = multiply_scalar(loss, 1.0 / static_cast<double>(micro));
      scaled.backward();
    }
    *loss_out = static_cast<float>(total / static_cast<double>(micro));
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].grad(), grads[i]);
    *norm_out = training::clip_grad_norm(ps, max_norm).total_norm;
    optim::AdamW opt{ps, lr, beta1, beta2, adam_eps, wd};
    opt.step();
    for (std::size_t i = 0; i < ps.size(); ++i) to_host(ps[i].tensor(), out_params[i]);
  });
}
#endif

// Seconds per training step (forward, LM loss, backward, clip, AdamW) of the LN/GELU decoder
// with N(0, 0.02) weights on [batch, t] ids, on `device` (< 0: CPU), after `warmup` untimed
// steps, averaged over `iters` steps. Each step ends with the loss read back to the host. Used to
// time the reference's own GPU path (reported beside the product's numbers, never a parity
// check).
double ref_lm_step_seconds(int64_t vocab, int64_t d, int64_t f, int64_t layers, int64_t heads,
                           int64_t batch, int64_t t, int64_t warmup, int64_t iters,
                           int64_t device) {
  double seconds = -1.0;
  guarded([&] {
    Random rng{11};
    Model model(vocab, d, f, layers, heads, 10000.0, 1e-5, rng);
    std::vector<nn::Parameter> ps = model.parameters();
    const Device dev = device_of(device);
    nn::move_to(std::span<nn::Parameter>{ps}, dev);
    optim::AdamW opt{ps, 3e-4, 0.9, 0.95, 1e-8, 0.1};
    Tensor host_ids{Shape{batch, t}, DType::Int32};
    auto s = host_ids.span<int32_t>();
    for (int64_t i = 0; i < batch * t; ++i) s[i] = static_cast<int32_t>((i * 7919 + 13) % vocab);
    const Tensor tid = host_ids.to(dev);
    auto one = [&] {
      for (auto& p : ps) p.zero_grad();
      Tensor loss = loss::language_model_cross_entropy(model.logits(tid), tid);
      loss.backward();
      (void)training::clip_grad_norm(ps, 1.0);
      opt.step();
      (void)scalar_of(loss);
    };
    for (int64_t i = 0; i < warmup; ++i) one();
    const auto t0 = std::chrono::steady_clock::now();
    for (int64_t i = 0; i < iters; ++i) one();
    seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() /
              static_cast<double>(iters);
  });
  return seconds;
}

// Seconds per Spar matmul (forward only, the cuda_blas seam on a CUDA device) of [m, k] x [k, n]
// fp32 N(0, 1) operands, averaged over `iters` calls after one warm-up call.
double ref_matmul_seconds(int64_t m, int64_t k, int64_t n, int64_t iters, int64_t device) {
  double seconds = -1.0;
  guarded([&] {
    const Device dev = device_of(device);
    auto pattern = [](Tensor t) {  // deterministic values spread over [-0.5, 0.5)
      auto v = t.span<float>();
      for (std::size_t i = 0; i < v.size(); ++i)
        v[i] = static_cast<float>((i * 2654435761ull) % 1000003ull) / 1000003.0f - 0.5f;
      return t;
    };
    Tensor a = pattern(Tensor{Shape{m, k}, DType::Float32}).to(dev);
    Tensor b = pattern(Tensor{Shape{k, n}, DType::Float32}).to(dev);
    (void)matmul(a, b);
    const auto t0 = std::chrono::steady_clock::now();
    for (int64_t i = 0; i < iters; ++i) (void)matmul(a, b);
    seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() /
              static_cast<double>(iters);
  });
  return seconds;
}

}  // extern "C"
