"""CPU restatement of Spar's Transformer training hot path (numpy). TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg may import it. The product path (libspar_b200.so) never calls it.

Every function restates the reference algorithm it cites (paths relative to the bzzling/spar
source tree). Parity of this restatement is pinned against the reference itself: the reference's
own sources are compiled by oracle/make_ref.py into oracle/_ref/libspar_ref.so and
tests/golden/make_golden.py stores its outputs as fixtures (tests/golden/*.npz), which
tests/test_oracle.py compares with this module.

Spar has no LayerNorm and no GELU op; BASELINE's pre-LN/GELU model composes them from Spar ops:
  LayerNorm = mean -> subtract -> square -> mean -> add_scalar(eps) -> sqrt -> divide
              -> multiply(gamma) -> add(beta)   (the RMSNorm pattern of src/nn/rmsnorm.cpp:50-52)
  GELU      = x * sigmoid(2*sqrt(2/pi) * (x + 0.044715 x^3))   (src/ops/unary.cpp:137-148)
Functions take a `dtype` (np.float32 mirrors the reference's fp32 path; np.float64 is the
secondary truth used to attribute error).
"""
from __future__ import annotations

import math

import numpy as np

# ------------------------------------------------------------------------------ RNG
MASK64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


def splitmix64(counters: np.ndarray) -> np.ndarray:
    """Output of Random::next_u64 (src/core/random.cpp:22-28) for state = counters * GOLDEN + seed,
    i.e. the i-th draw of a generator seeded with `seed` is splitmix64(seed + (i + 1) * GOLDEN)."""
    z = counters.astype(np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


class Random:
    """Vectorised Spar Random (src/core/random.cpp:12-38): SplitMix64 with a counter state."""

    def __init__(self, seed: int):
        self.state = seed & MASK64

    def next_u64(self, n: int) -> np.ndarray:
        idx = np.arange(1, n + 1, dtype=np.uint64)
        with np.errstate(over="ignore"):
            states = np.uint64(self.state) + idx * np.uint64(GOLDEN)
        self.state = (self.state + n * GOLDEN) & MASK64
        return splitmix64(states)

    def uniform_double(self, n: int) -> np.ndarray:
        """random.cpp:35-38: (next_u64 >> 11) / 2^53."""
        return (self.next_u64(n) >> np.uint64(11)).astype(np.float64) / 9007199254740992.0

    def normal(self, n: int, std: float) -> np.ndarray:
        """Harness-defined N(0, std) (Spar has no normal sampler): Box-Muller on two
        uniform_double draws per value, z = sqrt(-2 ln(1 - u1)) cos(2 pi u2), rounded to fp32."""
        u = self.uniform_double(2 * n).reshape(n, 2)
        z = np.sqrt(-2.0 * np.log1p(-u[:, 0])) * np.cos(2.0 * np.pi * u[:, 1])
        return (z * std).astype(np.float32)

    def bounded(self, n: int, bound: int) -> np.ndarray:
        """bounded_index (src/data/batch_iterator.cpp:22-32): rejection of values below
        (2^64 - bound) % bound, then value % bound."""
        threshold = ((1 << 64) - bound) % bound
        out = np.empty(n, dtype=np.int64)
        filled = 0
        while filled < n:
            v = self.next_u64(1)[0] if threshold else None
            if threshold:
                if int(v) < threshold:
                    continue
                out[filled] = int(v) % bound
                filled += 1
            else:
                vals = self.next_u64(n - filled)
                out[filled:] = (vals % np.uint64(bound)).astype(np.int64)
                filled = n
        return out


# ------------------------------------------------------------------------------ LayerNorm
def layer_norm_forward(x, gamma, beta, eps=1e-5, dtype=np.float32):
    """Composed LayerNorm over the last axis (see module docstring); returns y, mean, rstd.
    mean/var are mean over the axis (src/ops/reduction.cpp:282-311), divide by
    sqrt(var + eps) (unary.cpp:125, scalar.cpp:63, elementwise.cpp:173)."""
    x = np.asarray(x, dtype)
    mean = x.mean(axis=-1, keepdims=True, dtype=dtype)
    xc = x - mean
    var = (xc * xc).mean(axis=-1, keepdims=True, dtype=dtype)
    denom = np.sqrt(var + dtype(eps))
    y = xc / denom * np.asarray(gamma, dtype) + np.asarray(beta, dtype)
    return y.astype(dtype), mean[..., 0].astype(dtype), (1.0 / denom[..., 0]).astype(dtype)


def layer_norm_backward(dy, x, gamma, eps=1e-5, dtype=np.float64):
    """Closed form of the composed chain's reverse-mode gradient (src/autograd/autograd.cpp:
    201-265 sweeping the ops above): returns dx, dgamma, dbeta."""
    x = np.asarray(x, dtype)
    dy = np.asarray(dy, dtype)
    g = np.asarray(gamma, dtype)
    mean = x.mean(axis=-1, keepdims=True)
    xc = x - mean
    var = (xc * xc).mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(var + eps)
    xhat = xc * rstd
    gy = dy * g
    dx = rstd * (gy - gy.mean(axis=-1, keepdims=True) - xhat * (gy * xhat).mean(axis=-1, keepdims=True))
    red = tuple(range(dy.ndim - 1))
    return dx, (dy * xhat).sum(axis=red), dy.sum(axis=red)


# ------------------------------------------------------------------------------ RMSNorm
def rms_norm_forward(x, weight, eps=1e-5, dtype=np.float32):
    """nn::RMSNorm::forward (src/nn/rmsnorm.cpp:40-53): mean(square(x)) over the last axis,
    add_scalar(eps), sqrt, divide, multiply(weight); returns y and rstd = 1 / sqrt(ms + eps)."""
    x = np.asarray(x, dtype)
    ms = (x * x).mean(axis=-1, keepdims=True, dtype=dtype)
    denom = np.sqrt(ms + dtype(eps))
    y = x / denom * np.asarray(weight, dtype)
    return y.astype(dtype), (1.0 / denom[..., 0]).astype(dtype)


def rms_norm_backward(dy, x, weight, eps=1e-5, dtype=np.float64):
    """Closed form of the reverse-mode sweep over the chain above: with xhat = x * rstd and
    g = dy * weight, dx = rstd * (g - xhat * mean(g * xhat)), dweight = sum_rows dy * xhat."""
    x = np.asarray(x, dtype)
    dy = np.asarray(dy, dtype)
    rstd = 1.0 / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps)
    xhat = x * rstd
    gy = dy * np.asarray(weight, dtype)
    dx = rstd * (gy - xhat * (gy * xhat).mean(axis=-1, keepdims=True))
    return dx, (dy * xhat).sum(axis=tuple(range(dy.ndim - 1)))


# ------------------------------------------------------------------------------ GELU
def stable_sigmoid(v):
    """src/ops/unary.cpp:55-61."""
    v = np.asarray(v)
    out = np.empty_like(v)
    pos = v >= 0
    out[pos] = 1.0 / (1.0 + np.exp(-v[pos]))
    e = np.exp(v[~pos])
    out[~pos] = e / (1.0 + e)
    return out


GELU_A = 1.5957691216057308  # 2*sqrt(2/pi)
GELU_B = 0.044715


def gelu_forward(x, dtype=np.float32):
    x = np.asarray(x, dtype)
    u = (x + (x * x * x) * dtype(GELU_B)) * dtype(GELU_A)
    return (x * stable_sigmoid(u)).astype(dtype)


def gelu_derivative(x, dtype=np.float64):
    x = np.asarray(x, dtype)
    u = (x + (x * x * x) * GELU_B) * GELU_A
    s = stable_sigmoid(u)
    return s + x * s * (1.0 - s) * GELU_A * (1.0 + 3.0 * GELU_B * x * x)


# ------------------------------------------------------------------------------ SwiGLU
def swiglu_forward(gate, value, dtype=np.float32):
    """nn::swiglu (src/nn/functional.cpp:9-11): silu(gate) * value, silu(x) = x * sigmoid(x)
    with the stable sigmoid (src/ops/unary.cpp:55-61, 150-152)."""
    g = np.asarray(gate, dtype)
    return (g * stable_sigmoid(g) * np.asarray(value, dtype)).astype(dtype)


def swiglu_backward(dh, gate, value, dtype=np.float64):
    """d gate = dh * value * (s + gate * s * (1 - s)), d value = dh * gate * s, s = sigmoid(gate)
    (silu's local derivative, src/ops/unary.cpp:155-160, through multiply's backward)."""
    g = np.asarray(gate, dtype)
    v = np.asarray(value, dtype)
    d = np.asarray(dh, dtype)
    sg = stable_sigmoid(g)
    return d * v * (sg + g * (sg * (1.0 - sg))), d * (g * sg)


# ------------------------------------------------------------------------------ softmax
def causal_softmax_forward(s, scale, dtype=np.float32):
    """attention.cpp:128-134: multiply_scalar(scores, scale) + causal_mask (:96-118) then
    softmax over the last axis (src/ops/softmax.cpp:42-108). Returns P with zeros above the
    diagonal."""
    s = np.asarray(s, dtype) * dtype(scale)
    t = s.shape[-1]
    mask = np.triu(np.ones((t, t), dtype=bool), 1)
    s = np.where(mask, -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(dtype)


def causal_softmax_backward(dp, p, scale, dtype=np.float64):
    """softmax.cpp:110-150 (P * (g - sum(g * P))) then the scalar-multiply backward."""
    dp = np.asarray(dp, dtype)
    p = np.asarray(p, dtype)
    t = p.shape[-1]
    mask = np.tril(np.ones((t, t), dtype=bool))
    dp = np.where(mask, dp, 0.0)
    dot = (dp * p).sum(axis=-1, keepdims=True)
    return np.where(mask, p * (dp - dot) * scale, 0.0)


def attention_forward_backward(qkv, heads, dctx=None, dtype=np.float64, kv_heads=None):
    """Causal self-attention over a packed projection buffer qkv [B, T, (H + 2 KVH) dh] (Q | K | V,
    head h at columns h*dh of each part; KVH = kv_heads, default H): scaled_dot_product_attention
    (src/nn/attention.cpp:121-135: matmul(Q, K^T) * 1/sqrt(dh), + causal_mask, softmax over keys,
    matmul(P, V)) after repeat_kv_heads (:77-94: kv head j serves query heads j*G .. j*G+G-1,
    G = H / KVH) and, given dctx [B, T, H dh], the autograd backward of that chain (matmul
    backward, softmax backward src/ops/softmax.cpp:110-150, scalar-multiply backward; the repeat's
    backward sums each group's dK / dV). Returns (ctx, dqkv or None)."""
    qkv = np.asarray(qkv, dtype)
    kvh = heads if kv_heads is None else kv_heads
    b, t, width = qkv.shape
    dh = width // (heads + 2 * kvh)
    d, dk_w = heads * dh, kvh * dh
    group = heads // kvh
    scale = 1.0 / math.sqrt(dh)

    def split(x, n):  # [B, T, n dh] -> [B, n, T, dh]
        return x.reshape(b, t, n, dh).transpose(0, 2, 1, 3)

    def merge(x):
        return x.transpose(0, 2, 1, 3).reshape(b, t, -1)

    def repeat(x):  # repeat_kv_heads: [B, KVH, T, dh] -> [B, H, T, dh]
        return np.repeat(x, group, axis=1)

    def group_sum(x):  # backward of repeat: [B, H, T, dh] -> [B, KVH, T, dh]
        return x.reshape(b, kvh, group, t, dh).sum(axis=2)

    q = split(qkv[..., :d], heads)
    k = repeat(split(qkv[..., d:d + dk_w], kvh))
    v = repeat(split(qkv[..., d + dk_w:], kvh))
    mask = np.triu(np.ones((t, t), dtype=bool), 1)
    s = np.where(mask, -np.inf, (q @ k.transpose(0, 1, 3, 2)) * scale)
    e = np.exp(s - s.max(-1, keepdims=True))
    pr = e / e.sum(-1, keepdims=True)
    ctx = merge(pr @ v)
    if dctx is None:
        return ctx, None
    do = split(np.asarray(dctx, dtype), heads)
    dp = do @ v.transpose(0, 1, 3, 2)
    dv = pr.transpose(0, 1, 3, 2) @ do
    ds = pr * (dp - (dp * pr).sum(-1, keepdims=True)) * scale
    dq = ds @ k
    dk = ds.transpose(0, 1, 3, 2) @ q
    return ctx, np.concatenate([merge(dq), merge(group_sum(dk)), merge(group_sum(dv))], axis=-1)


# ------------------------------------------------------------------------------ cross-entropy
def lm_targets(ids):
    """language_model_cross_entropy target/row selection (src/loss/cross_entropy.cpp:198-209):
    rows b*T + t for t < T-1 with targets ids[b, t+1]."""
    b, t = ids.shape
    rows = (np.arange(b)[:, None] * t + np.arange(t - 1)[None, :]).reshape(-1)
    targets = ids[:, 1:].reshape(-1)
    return rows, targets


def cross_entropy_forward_backward(logits, targets, rows=None, dtype=np.float64):
    """log_softmax (softmax.cpp:342-404) + NLL gather (cross_entropy.cpp:52-64) + mean; the
    gradient of the mean loss is (exp(logp) - onehot)/N on selected rows (nll_gradient :66-78,
    log_softmax_gradient softmax.cpp:406-444). Returns (mean loss, per-row loss, dlogits)."""
    z = np.asarray(logits).reshape(-1, logits.shape[-1])
    if rows is None:
        rows = np.arange(z.shape[0])
    rows = np.asarray(rows)
    # One working copy of the selected rows, shifted by the row maximum, exponentiated in place
    # (large vocabularies: a single [rows, V] float64 array instead of several).
    d = np.zeros((z.shape[0], z.shape[1]), dtype)
    w = z[rows].astype(dtype)
    w -= w.max(axis=-1, keepdims=True)
    shifted_target = w[np.arange(len(rows)), targets].copy()
    np.exp(w, out=w)
    total = w.sum(axis=-1)
    n = len(rows)
    row_loss = np.zeros(z.shape[0], dtype)
    row_loss[rows] = np.log(total) - shifted_target  # -log softmax at the target
    w *= (1.0 / n) / total[:, None]
    d[rows] = w
    d[rows, targets] -= 1.0 / n
    return row_loss[rows].mean(), row_loss, d


# ------------------------------------------------------------------------------ optimiser
def global_grad_norm(grads):
    """src/training/gradients.cpp:105-137 (double accumulation; the scaled sum of squares of
    :28-88 only guards overflow)."""
    s = 0.0
    finite = True
    for g in grads:
        g64 = np.asarray(g, np.float64)
        finite = finite and bool(np.isfinite(g64).all())
        s += float(np.dot(g64.ravel(), g64.ravel()))
    return math.sqrt(s) if finite else math.nan


def clip_factor(norm, max_norm):
    """clip_grad_norm (gradients.cpp:176-190): error on non-finite, scale when norm > max."""
    if not math.isfinite(norm):
        raise RuntimeError("Cannot clip nonfinite gradients")
    if norm == 0.0 or norm <= max_norm:
        return 1.0
    return max_norm / norm


def adamw_update(p, g, m, v, step, lr, beta1, beta2, eps, weight_decay, clip=1.0):
    """AdamW::update_values (src/optim/adamw.cpp:37-63): double math, fp32 storage; gradient
    first scaled as scale_gradients does (gradients.cpp:139-174). Returns new (p, m, v)."""
    g = np.asarray(g, np.float32)
    if clip != 1.0:
        g = (g.astype(np.float64) * clip).astype(np.float32)
    gd = g.astype(np.float64)
    c1 = 1.0 - beta1 ** step
    c2 = 1.0 - beta2 ** step
    m = (beta1 * np.asarray(m, np.float64) + (1.0 - beta1) * gd).astype(np.float32)
    v = (beta2 * np.asarray(v, np.float64) + (1.0 - beta2) * gd * gd).astype(np.float32)
    mc = m.astype(np.float64) / c1
    vc = v.astype(np.float64) / c2
    p = (np.asarray(p, np.float64) * (1.0 - lr * weight_decay) - lr * mc / (np.sqrt(vc) + eps))
    return p.astype(np.float32), m, v


def warmup_cosine(peak, minimum, warmup, decay, step):
    """training::warmup_cosine_learning_rate (src/training/schedule.cpp:9-38)."""
    if step < warmup:
        return peak * ((step + 1) / warmup)  # progress first, as schedule.cpp:25-27
    idx = step - warmup
    if idx >= decay or decay == 1:
        return minimum
    return minimum + 0.5 * (peak - minimum) * (1.0 + math.cos(math.pi * idx / (decay - 1)))


# ------------------------------------------------------------------------------ RoPE
def rope_table(t, d, theta=10000.0, start=0):
    """Angles of rotate() (src/nn/rope.cpp:35-66): pos * theta^(-2i/D) in double, cos/sin
    rounded to fp32. Returns cos, sin arrays [t, d/2]."""
    pos = (start + np.arange(t, dtype=np.float64))[:, None]
    expo = -2.0 * np.arange(d // 2, dtype=np.float64)[None, :] / d
    ang = pos * np.power(theta, expo)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope_apply(x, cos, sin, inverse=False):
    """x [..., T, D]: pairs (2i, 2i+1) rotated (rope.cpp:55-62)."""
    s = -sin if inverse else sin
    a = x[..., 0::2]
    b = x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = a * cos - b * s
    out[..., 1::2] = a * s + b * cos
    return out


# ------------------------------------------------------------------------------ LM
def parameter_names(num_layers):
    """Names in nn::named_parameters order (src/nn/parameters.cpp:51-132) for the LN/GELU
    decoder (Linear weights [in, out], src/nn/linear.cpp:33-35)."""
    names = ["token_embedding.weight"]
    for i in range(num_layers):
        p = f"blocks.{i}."
        names += [p + "attention_norm.weight", p + "attention_norm.bias"]
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            names += [p + f"attention.{proj}.weight", p + f"attention.{proj}.bias"]
        names += [p + "mlp_norm.weight", p + "mlp_norm.bias"]
        for proj in ("up_proj", "down_proj"):
            names += [p + f"mlp.{proj}.weight", p + f"mlp.{proj}.bias"]
    names += ["final_norm.weight", "final_norm.bias"]
    return names


def parameter_shapes(cfg):
    v, d, f, layers = cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"]
    shapes = {}
    for name in parameter_names(layers):
        if name == "token_embedding.weight":
            shapes[name] = (v, d)
        elif name.endswith("norm.weight") or name.endswith("norm.bias"):
            shapes[name] = (d,)
        elif "up_proj" in name:
            shapes[name] = (d, f) if name.endswith("weight") else (f,)
        elif "down_proj" in name:
            shapes[name] = (f, d) if name.endswith("weight") else (d,)
        else:
            shapes[name] = (d, d) if name.endswith("weight") else (d,)
    return shapes


def init_parameters(cfg, seed, std=0.02):
    """BASELINE init: weight matrices and the embedding N(0, std) drawn in parameter order from
    one Random(seed) stream; LayerNorm gamma = 1, beta = 0; biases 0 (Linear bias init,
    linear.cpp:40-42)."""
    rng = Random(seed)
    params = {}
    for name, shape in parameter_shapes(cfg).items():
        if len(shape) == 2:
            params[name] = rng.normal(int(np.prod(shape)), std).reshape(shape)
        elif name.endswith("norm.weight"):
            params[name] = np.ones(shape, np.float32)
        else:
            params[name] = np.zeros(shape, np.float32)
    return params


def spar_family_shapes(cfg):
    """Shapes of nn::DecoderLM's named parameters (src/nn/parameters.cpp:61-108, Linear weights
    [in, out], linear.cpp:33-35) in order, for cfg {vocab, dim, hidden, layers, heads, kv_heads,
    qk_norm}."""
    v, d, f, n_l, h = cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"]
    kvh = cfg.get("kv_heads") or h
    dh = d // h
    shapes = {"token_embedding.weight": (v, d)}
    for i in range(n_l):
        p = f"blocks.{i}."
        shapes[p + "attention_norm.weight"] = (d,)
        shapes[p + "attention.q_proj.weight"] = (d, h * dh)
        shapes[p + "attention.k_proj.weight"] = (d, kvh * dh)
        shapes[p + "attention.v_proj.weight"] = (d, kvh * dh)
        shapes[p + "attention.out_proj.weight"] = (d, d)
        if cfg.get("qk_norm"):
            shapes[p + "attention.q_norm.weight"] = (dh,)
            shapes[p + "attention.k_norm.weight"] = (dh,)
        shapes[p + "mlp_norm.weight"] = (d,)
        shapes[p + "mlp.gate_proj.weight"] = (d, f)
        shapes[p + "mlp.up_proj.weight"] = (d, f)
        shapes[p + "mlp.down_proj.weight"] = (f, d)
    shapes["final_norm.weight"] = (d,)
    return shapes


def spar_family_parameters(cfg, seed, std=0.02, norm_std=0.1):
    """Test parameters for nn::DecoderLM: matrices N(0, std), norm weights 1 + N(0, norm_std),
    drawn in named-parameter order from one Random(seed) stream."""
    rng = Random(seed)
    out = {}
    for name, shape in spar_family_shapes(cfg).items():
        n = int(np.prod(shape))
        if len(shape) == 2:
            out[name] = rng.normal(n, std).reshape(shape)
        else:
            out[name] = (1.0 + rng.normal(n, norm_std)).astype(np.float32).reshape(shape)
    return out


def lm_forward_backward(params, ids, cfg, dtype=np.float64):
    """One forward + backward of the pre-LN decoder (DecoderLM::forward, src/nn/decoder.cpp:
    73-90; TransformerBlock::forward, transformer.cpp:53-69; SelfAttention::forward,
    attention.cpp:188-225 with RoPE; LN/GELU MLP) and the LM cross-entropy
    (cross_entropy.cpp:176-214). Returns (loss, grads dict)."""
    v, d, hdim, layers, heads = cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"]
    eps = cfg.get("eps", 1e-5)
    b, t = ids.shape
    dh = d // heads
    scale = 1.0 / math.sqrt(dh)
    P = {k: np.asarray(val, dtype) for k, val in params.items()}
    cos, sin = rope_table(t, dh, cfg.get("rope_theta", 10000.0))
    cos = cos.astype(dtype)
    sin = sin.astype(dtype)
    E = P["token_embedding.weight"]
    h = E[ids.reshape(-1)]
    cache = []

    def ln(x, g, bb):
        mean = x.mean(-1, keepdims=True)
        xc = x - mean
        rstd = 1.0 / np.sqrt((xc * xc).mean(-1, keepdims=True) + eps)
        return xc * rstd * g + bb

    def heads_of(x):  # [BT, d] -> [B, H, T, dh]
        return x.reshape(b, t, heads, dh).transpose(0, 2, 1, 3)

    def merge(x):  # [B, H, T, dh] -> [BT, d]
        return x.transpose(0, 2, 1, 3).reshape(b * t, d)

    mask = np.triu(np.ones((t, t), dtype=bool), 1)
    for i in range(layers):
        pre = f"blocks.{i}."
        x = h
        a = ln(x, P[pre + "attention_norm.weight"], P[pre + "attention_norm.bias"])
        q = a @ P[pre + "attention.q_proj.weight"] + P[pre + "attention.q_proj.bias"]
        k = a @ P[pre + "attention.k_proj.weight"] + P[pre + "attention.k_proj.bias"]
        vv = a @ P[pre + "attention.v_proj.weight"] + P[pre + "attention.v_proj.bias"]
        qh = rope_apply(heads_of(q), cos, sin)
        kh = rope_apply(heads_of(k), cos, sin)
        vh = heads_of(vv)
        s = np.where(mask, -np.inf, (qh @ kh.transpose(0, 1, 3, 2)) * scale)
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr = pr / pr.sum(-1, keepdims=True)
        ctx = merge(pr @ vh)
        o = ctx @ P[pre + "attention.out_proj.weight"] + P[pre + "attention.out_proj.bias"]
        h1 = x + o
        a2 = ln(h1, P[pre + "mlp_norm.weight"], P[pre + "mlp_norm.bias"])
        u = a2 @ P[pre + "mlp.up_proj.weight"] + P[pre + "mlp.up_proj.bias"]
        g = u * stable_sigmoid((u + u * u * u * GELU_B) * GELU_A)
        mm = g @ P[pre + "mlp.down_proj.weight"] + P[pre + "mlp.down_proj.bias"]
        h = h1 + mm
        cache.append((x, a, qh, kh, vh, pr, ctx, h1, a2, u, g))
    hf = ln(h, P["final_norm.weight"], P["final_norm.bias"])
    logits = hf @ E.T
    rows, targets = lm_targets(ids)
    loss, _, dlogits = cross_entropy_forward_backward(logits, targets, rows, dtype)

    grads = {name: np.zeros_like(val) for name, val in P.items()}
    grads["token_embedding.weight"] += dlogits.T @ hf
    dhf = dlogits @ E
    dres, dgf, dbf = layer_norm_backward(dhf, h, P["final_norm.weight"], eps, dtype)
    grads["final_norm.weight"] += dgf
    grads["final_norm.bias"] += dbf
    for i in reversed(range(layers)):
        pre = f"blocks.{i}."
        x, a, qh, kh, vh, pr, ctx, h1, a2, u, g = cache[i]
        dm = dres
        grads[pre + "mlp.down_proj.weight"] += g.T @ dm
        grads[pre + "mlp.down_proj.bias"] += dm.sum(0)
        dg = dm @ P[pre + "mlp.down_proj.weight"].T
        du = dg * gelu_derivative(u, dtype)
        grads[pre + "mlp.up_proj.weight"] += a2.T @ du
        grads[pre + "mlp.up_proj.bias"] += du.sum(0)
        da2 = du @ P[pre + "mlp.up_proj.weight"].T
        dx2, dg2, db2 = layer_norm_backward(da2, h1, P[pre + "mlp_norm.weight"], eps, dtype)
        grads[pre + "mlp_norm.weight"] += dg2
        grads[pre + "mlp_norm.bias"] += db2
        dh1 = dres + dx2
        grads[pre + "attention.out_proj.weight"] += ctx.T @ dh1
        grads[pre + "attention.out_proj.bias"] += dh1.sum(0)
        dctx = heads_of(dh1 @ P[pre + "attention.out_proj.weight"].T)
        dpr = dctx @ vh.transpose(0, 1, 3, 2)
        dvh = pr.transpose(0, 1, 3, 2) @ dctx
        ds = pr * (dpr - (dpr * pr).sum(-1, keepdims=True)) * scale
        dqh = rope_apply(ds @ kh, cos, sin, inverse=True)
        dkh = rope_apply(ds.transpose(0, 1, 3, 2) @ qh, cos, sin, inverse=True)
        dq, dk, dv = merge(dqh), merge(dkh), merge(dvh)
        da = np.zeros_like(a)
        for proj, dy in (("q_proj", dq), ("k_proj", dk), ("v_proj", dv)):
            grads[pre + f"attention.{proj}.weight"] += a.T @ dy
            grads[pre + f"attention.{proj}.bias"] += dy.sum(0)
            da += dy @ P[pre + f"attention.{proj}.weight"].T
        dx1, dg1, db1 = layer_norm_backward(da, x, P[pre + "attention_norm.weight"], eps, dtype)
        grads[pre + "attention_norm.weight"] += dg1
        grads[pre + "attention_norm.bias"] += db1
        dres = dh1 + dx1
    np.add.at(grads["token_embedding.weight"], ids.reshape(-1), dres)
    return float(loss), grads


def spar_lm_forward_backward(params, ids, cfg, dtype=np.float64):
    """One forward + backward of Spar's own nn::DecoderLM (decoder.cpp:73-90; TransformerBlock
    transformer.cpp:53-69 with RMSNorm pre-norms; SelfAttention attention.cpp:188-225 without
    biases, num_kv_heads key/value heads repeated over query groups (repeat_kv_heads :77-94), q /
    k RMSNorm(head_dim) before RoPE when qk_norm; SwiGLUMLP mlp.cpp:33-46: down(silu(gate) * up);
    final RMSNorm, tied logits) and the LM cross-entropy. Returns (loss, grads dict)."""
    v, d, f, layers, heads = cfg["vocab"], cfg["dim"], cfg["hidden"], cfg["layers"], cfg["heads"]
    kvh = cfg.get("kv_heads") or heads
    eps, qeps = cfg.get("eps", 1e-5), cfg.get("qk_eps", 1e-6)
    qk = bool(cfg.get("qk_norm"))
    b, t = ids.shape
    dh = d // heads
    group = heads // kvh
    scale = 1.0 / math.sqrt(dh)
    P = {k: np.asarray(val, dtype) for k, val in params.items()}
    cos, sin = rope_table(t, dh, cfg.get("rope_theta", 10000.0))
    cos, sin = cos.astype(dtype), sin.astype(dtype)
    E = P["token_embedding.weight"]
    h = E[ids.reshape(-1)]

    def rms(x, w, e):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + e) * w

    def heads_of(x, n):  # [BT, n dh] -> [B, n, T, dh]
        return x.reshape(b, t, n, dh).transpose(0, 2, 1, 3)

    def merge(x):  # [B, n, T, dh] -> [BT, n dh]
        return x.transpose(0, 2, 1, 3).reshape(b * t, -1)

    mask = np.triu(np.ones((t, t), dtype=bool), 1)
    cache = []
    for i in range(layers):
        pre = f"blocks.{i}."
        x = h
        a = rms(x, P[pre + "attention_norm.weight"], eps)
        qr = heads_of(a @ P[pre + "attention.q_proj.weight"], heads)
        kr = heads_of(a @ P[pre + "attention.k_proj.weight"], kvh)
        vh = heads_of(a @ P[pre + "attention.v_proj.weight"], kvh)
        qn = rms(qr, P[pre + "attention.q_norm.weight"], qeps) if qk else qr
        kn = rms(kr, P[pre + "attention.k_norm.weight"], qeps) if qk else kr
        qh, kh = rope_apply(qn, cos, sin), rope_apply(kn, cos, sin)
        kx, vx = np.repeat(kh, group, axis=1), np.repeat(vh, group, axis=1)
        sc = np.where(mask, -np.inf, (qh @ kx.transpose(0, 1, 3, 2)) * scale)
        pr = np.exp(sc - sc.max(-1, keepdims=True))
        pr = pr / pr.sum(-1, keepdims=True)
        ctx = merge(pr @ vx)
        h1 = x + ctx @ P[pre + "attention.out_proj.weight"]
        a2 = rms(h1, P[pre + "mlp_norm.weight"], eps)
        gate = a2 @ P[pre + "mlp.gate_proj.weight"]
        up = a2 @ P[pre + "mlp.up_proj.weight"]
        hid = swiglu_forward(gate, up, dtype)
        h = h1 + hid @ P[pre + "mlp.down_proj.weight"]
        cache.append((x, a, qr, kr, qh, kh, vh, kx, vx, pr, ctx, h1, a2, gate, up, hid))
    hf = rms(h, P["final_norm.weight"], eps)
    logits = hf @ E.T
    rows, targets = lm_targets(ids)
    loss, _, dlogits = cross_entropy_forward_backward(logits, targets, rows, dtype)

    grads = {name: np.zeros_like(val) for name, val in P.items()}
    grads["token_embedding.weight"] += dlogits.T @ hf
    dres, dwf = rms_norm_backward(dlogits @ E, h, P["final_norm.weight"], eps, dtype)
    grads["final_norm.weight"] += dwf
    group_sum = lambda z: z.reshape(b, kvh, group, t, dh).sum(axis=2)  # noqa: E731
    for i in reversed(range(layers)):
        pre = f"blocks.{i}."
        x, a, qr, kr, qh, kh, vh, kx, vx, pr, ctx, h1, a2, gate, up, hid = cache[i]
        grads[pre + "mlp.down_proj.weight"] += hid.T @ dres
        dgate, dup = swiglu_backward(dres @ P[pre + "mlp.down_proj.weight"].T, gate, up, dtype)
        grads[pre + "mlp.gate_proj.weight"] += a2.T @ dgate
        grads[pre + "mlp.up_proj.weight"] += a2.T @ dup
        da2 = dgate @ P[pre + "mlp.gate_proj.weight"].T + dup @ P[pre + "mlp.up_proj.weight"].T
        dx2, dw2 = rms_norm_backward(da2, h1, P[pre + "mlp_norm.weight"], eps, dtype)
        grads[pre + "mlp_norm.weight"] += dw2
        dh1 = dres + dx2
        grads[pre + "attention.out_proj.weight"] += ctx.T @ dh1
        dctx = heads_of(dh1 @ P[pre + "attention.out_proj.weight"].T, heads)
        dpr = dctx @ vx.transpose(0, 1, 3, 2)
        dvh = group_sum(pr.transpose(0, 1, 3, 2) @ dctx)
        ds = pr * (dpr - (dpr * pr).sum(-1, keepdims=True)) * scale
        dqn = rope_apply(ds @ kx, cos, sin, inverse=True)
        dkn = rope_apply(group_sum(ds.transpose(0, 1, 3, 2) @ qh), cos, sin, inverse=True)
        if qk:
            dqr, dwq = rms_norm_backward(dqn, qr, P[pre + "attention.q_norm.weight"], qeps, dtype)
            dkr, dwk = rms_norm_backward(dkn, kr, P[pre + "attention.k_norm.weight"], qeps, dtype)
            grads[pre + "attention.q_norm.weight"] += dwq
            grads[pre + "attention.k_norm.weight"] += dwk
        else:
            dqr, dkr = dqn, dkn
        da = np.zeros_like(a)
        for proj, dy in (("q_proj", merge(dqr)), ("k_proj", merge(dkr)), ("v_proj", merge(dvh))):
            grads[pre + f"attention.{proj}.weight"] += a.T @ dy
            da += dy @ P[pre + f"attention.{proj}.weight"].T
        dx1, dw1 = rms_norm_backward(da, x, P[pre + "attention_norm.weight"], eps, dtype)
        grads[pre + "attention_norm.weight"] += dw1
        dres = dh1 + dx1
    np.add.at(grads["token_embedding.weight"], ids.reshape(-1), dres)
    return float(loss), grads


def lm_train_step(params, moments, ids_list, cfg, step, lr, opt, dtype=np.float64):
    """One optimiser step with gradient accumulation over the micro-batches in ids_list: grads
    summed over micro-steps of the per-micro-batch mean loss divided by the micro-step count,
    then clip + AdamW on every parameter (decoupled decay on all, adamw.cpp:83-170).
    Returns (mean loss, grads, new params, new moments)."""
    n = len(ids_list)
    total = None
    loss_sum = 0.0
    for ids in ids_list:
        loss, grads = lm_forward_backward(params, ids, cfg, dtype)
        loss_sum += loss
        if total is None:
            total = {k: g / n for k, g in grads.items()}
        else:
            for k in total:
                total[k] += grads[k] / n
    norm = global_grad_norm([total[k].astype(np.float32) for k in total])
    clip = clip_factor(norm, opt["max_grad_norm"]) if opt["max_grad_norm"] >= 0 else 1.0
    new_p, new_m = {}, {}
    for k in params:
        m, v = moments.get(k, (np.zeros_like(params[k]), np.zeros_like(params[k])))
        new_p[k], m2, v2 = adamw_update(params[k], total[k].astype(np.float32), m, v, step, lr,
                                        opt["beta1"], opt["beta2"], opt["eps"],
                                        opt["weight_decay"], clip)
        new_m[k] = (m2, v2)
    return loss_sum / n, total, new_p, new_m
