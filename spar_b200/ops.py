"""Tensor-level wrappers over the spar_b200 C ABI.

These mirror the reference's tensor-level backend wrappers (src/backend/cuda_ops.cppm: validate,
allocate the output, call the C entry point, turn a non-zero status into an exception) for the
fused hot-path kernels. torch tensors are only used as device buffers; every computation runs in
libspar_b200.so on torch's current stream.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import SparB200Gemm, SparB200TensorSlice, call

TF32, TF32X3 = 0, 1
EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_GELU_BWD, EPI_BIAS_ADD = 0, 1, 2, 3, 4
CAUSAL_NONE, CAUSAL_LOWER, CAUSAL_K_UPTO, CAUSAL_K_FROM = 0, 1, 2, 3
NORM_STATE_DOUBLES = 1024


def _dev(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("spar_b200 ops take CUDA tensors")
    return t.device.index


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 tensor")
    return t


def _ptr(t):
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------------------------- LayerNorm
def layer_norm_forward(x, gamma, beta, eps: float = 1e-5):
    _f32(x, "x")
    cols = x.shape[-1]
    rows = x.numel() // cols
    y = torch.empty_like(x)
    mean = torch.empty(rows, device=x.device, dtype=torch.float32)
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    call("spar_b200_layernorm_forward", y.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
         x.data_ptr(), _f32(gamma, "gamma").data_ptr(), _f32(beta, "beta").data_ptr(), rows, cols,
         eps, _dev(x), _stream(x))
    return y, mean, rstd


def layer_norm_backward(dy, x, gamma, mean, rstd, dgamma=None, dbeta=None, dx=None,
                        accumulate_params=False, accumulate_dx=False):
    cols = x.shape[-1]
    rows = x.numel() // cols
    dx = torch.empty_like(x) if dx is None else dx
    dgamma = torch.empty(cols, device=x.device, dtype=torch.float32) if dgamma is None else dgamma
    dbeta = torch.empty(cols, device=x.device, dtype=torch.float32) if dbeta is None else dbeta
    call("spar_b200_layernorm_backward", dx.data_ptr(), dgamma.data_ptr(), dbeta.data_ptr(),
         _f32(dy, "dy").data_ptr(), _f32(x, "x").data_ptr(), gamma.data_ptr(), mean.data_ptr(),
         rstd.data_ptr(), rows, cols, int(accumulate_params), int(accumulate_dx), _dev(x),
         _stream(x))
    return dx, dgamma, dbeta


# ------------------------------------------------------------------------------- RMSNorm
def rms_norm_forward(x, weight, eps: float = 1e-5):
    _f32(x, "x")
    cols = x.shape[-1]
    rows = x.numel() // cols
    y = torch.empty_like(x)
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    call("spar_b200_rmsnorm_forward", y.data_ptr(), rstd.data_ptr(), x.data_ptr(),
         _f32(weight, "weight").data_ptr(), rows, cols, eps, _dev(x), _stream(x))
    return y, rstd


def rms_norm_backward(dy, x, weight, rstd, dweight=None, dx=None, accumulate_params=False,
                      accumulate_dx=False):
    cols = x.shape[-1]
    rows = x.numel() // cols
    dx = torch.empty_like(x) if dx is None else dx
    dweight = torch.empty(cols, device=x.device, dtype=torch.float32) if dweight is None else dweight
    call("spar_b200_rmsnorm_backward", dx.data_ptr(), dweight.data_ptr(), _f32(dy, "dy").data_ptr(),
         _f32(x, "x").data_ptr(), weight.data_ptr(), rstd.data_ptr(), rows, cols,
         int(accumulate_params), int(accumulate_dx), _dev(x), _stream(x))
    return dx, dweight


def head_rms_norm_forward(x, heads: int, head_dim: int, weight, eps: float = 1e-5, out=None):
    """qk-norm over the first heads * head_dim columns of each row of x (a 2-D view whose rows
    may be strided, e.g. qkv[:, 0:d] for q); out=x normalises in place."""
    tokens, _, ld = _rows_view(x, "x")
    if out is None:  # same row stride as x
        out = torch.empty(tokens, ld, device=x.device)[:, :heads * head_dim]
    y = out
    if y.stride(0) != ld:
        raise ValueError("out must have the row stride of x")
    rstd = torch.empty(tokens * heads, device=x.device, dtype=torch.float32)
    call("spar_b200_head_rmsnorm_forward", y.data_ptr(), x.data_ptr(), ld, tokens, heads, head_dim,
         _f32(weight, "weight").data_ptr(), rstd.data_ptr(), eps, _dev(x), _stream(x))
    return y, rstd


def head_rms_norm_backward(dy, x, heads: int, head_dim: int, weight, rstd, dweight=None,
                           out=None, accumulate_params=False):
    tokens, _, ld = _rows_view(x, "x")
    if dy.stride(0) != ld:
        raise ValueError("dy must have the row stride of x")
    dx = torch.empty(tokens, ld, device=x.device)[:, :heads * head_dim] if out is None else out
    dweight = torch.empty(head_dim, device=x.device) if dweight is None else dweight
    call("spar_b200_head_rmsnorm_backward", dx.data_ptr(), dweight.data_ptr(), dy.data_ptr(),
         x.data_ptr(), ld, tokens, heads, head_dim, weight.data_ptr(), rstd.data_ptr(),
         int(accumulate_params), _dev(x), _stream(x))
    return dx, dweight


# ------------------------------------------------------------------------------- SwiGLU
def _rows_view(t, name):
    """(rows, cols, row stride) of a 2-D float32 tensor whose rows may be strided (a column
    slice of a wider matrix)."""
    if t.dtype != torch.float32 or t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D float32 tensor with unit column stride")
    return t.shape[0], t.shape[1], t.stride(0)


def swiglu_forward(gate, value, out=None):
    rows, cols, ldg = _rows_view(gate, "gate")
    _, _, ldv = _rows_view(value, "value")
    h = torch.empty(rows, cols, device=gate.device, dtype=torch.float32) if out is None else out
    call("spar_b200_swiglu_forward", h.data_ptr(), _rows_view(h, "h")[2], gate.data_ptr(), ldg,
         value.data_ptr(), ldv, rows, cols, _dev(gate), _stream(gate))
    return h


def swiglu_backward(dh, gate, value, dgate=None, dvalue=None):
    rows, cols, ldg = _rows_view(gate, "gate")
    _, _, ldv = _rows_view(value, "value")
    _, _, lddh = _rows_view(dh, "dh")
    new = lambda: torch.empty(rows, cols, device=gate.device, dtype=torch.float32)  # noqa: E731
    dgate = new() if dgate is None else dgate
    dvalue = new() if dvalue is None else dvalue
    call("spar_b200_swiglu_backward", dgate.data_ptr(), _rows_view(dgate, "dgate")[2],
         dvalue.data_ptr(), _rows_view(dvalue, "dvalue")[2], dh.data_ptr(), lddh,
         gate.data_ptr(), ldg, value.data_ptr(), ldv, rows, cols, _dev(gate), _stream(gate))
    return dgate, dvalue


# ------------------------------------------------------------------------------- GELU
def gelu_forward(x):
    y = torch.empty_like(_f32(x, "x"))
    call("spar_b200_gelu_forward", y.data_ptr(), x.data_ptr(), x.numel(), _dev(x), _stream(x))
    return y


def gelu_backward(dy, x):
    dx = torch.empty_like(_f32(x, "x"))
    call("spar_b200_gelu_backward", dx.data_ptr(), _f32(dy, "dy").data_ptr(), x.data_ptr(),
         x.numel(), _dev(x), _stream(x))
    return dx


# ------------------------------------------------------------------------------- softmax
def causal_softmax_forward(s, scale: float, zero_fill_block: int = 0, out=None):
    _f32(s, "scores")
    t = s.shape[-1]
    batch = s.numel() // (t * t)
    p = torch.empty_like(s) if out is None else out
    call("spar_b200_causal_softmax_forward", p.data_ptr(), s.data_ptr(), batch, t, t, scale,
         zero_fill_block, _dev(s), _stream(s))
    return p


def causal_softmax_backward(dp, p, scale: float, zero_fill_block: int = 0, out=None):
    t = p.shape[-1]
    batch = p.numel() // (t * t)
    ds = torch.empty_like(p) if out is None else out
    call("spar_b200_causal_softmax_backward", ds.data_ptr(), _f32(dp, "dp").data_ptr(),
         _f32(p, "p").data_ptr(), batch, t, t, scale, zero_fill_block, _dev(p), _stream(p))
    return ds


# ------------------------------------------------------------------------------- attention
def attention_forward(qkv, heads: int, kv_heads: int | None = None):
    """Fused causal attention over the packed projection buffer qkv [batch, seq, (H + 2 KVH) dh]
    (KVH = kv_heads, default H: grouped-query attention when smaller).

    Returns (ctx [batch, seq, H dh], row_max [batch, heads, seq], row_inv [batch, heads, seq])."""
    _f32(qkv, "qkv")
    kvh = heads if kv_heads is None else kv_heads
    batch, seq, width = qkv.shape
    dh = width // (heads + 2 * kvh)
    ctx = torch.empty(batch, seq, heads * dh, device=qkv.device, dtype=torch.float32)
    row_max = torch.empty(batch, heads, seq, device=qkv.device, dtype=torch.float32)
    row_inv = torch.empty_like(row_max)
    call("spar_b200_attention_forward_gqa", qkv.data_ptr(), ctx.data_ptr(), row_max.data_ptr(),
         row_inv.data_ptr(), batch, seq, heads, kvh, dh, _dev(qkv), _stream(qkv))
    return ctx, row_max, row_inv


def attention_backward(dctx, qkv, ctx, row_max, row_inv, heads: int, rope_table=None,
                       kv_heads: int | None = None):
    """dqkv (the layout of qkv) of the fused causal attention (q, k parts rotated back by the RoPE
    table when one is given; dK / dV summed over each key/value head's query group)."""
    kvh = heads if kv_heads is None else kv_heads
    batch, seq, width = qkv.shape
    dh = width // (heads + 2 * kvh)
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(batch, heads, seq, device=qkv.device, dtype=torch.float32)
    call("spar_b200_attention_backward_gqa", _f32(qkv, "qkv").data_ptr(),
         _f32(ctx, "ctx").data_ptr(), _f32(dctx, "dctx").data_ptr(),
         _f32(row_max, "row_max").data_ptr(), _f32(row_inv, "row_inv").data_ptr(),
         delta.data_ptr(), dqkv.data_ptr(), batch, seq, heads, kvh, dh, _ptr(rope_table),
         _dev(qkv), _stream(qkv))
    return dqkv


def attention_error(device: int = 0, clear: bool = True) -> int:
    return _lib.load().spar_b200_attention_error(device, int(clear))


# ------------------------------------------------------------------------------- cross-entropy
def cross_entropy_forward_backward(logits, targets, sequence_length: int = 0,
                                   grad_scale: float | None = None, in_place: bool = False):
    """Returns (per-row loss, dlogits, invalid flag tensor)."""
    _f32(logits, "logits")
    classes = logits.shape[-1]
    rows = logits.numel() // classes
    if targets.dtype != torch.int32:
        raise ValueError("targets must be int32")
    if grad_scale is None:
        n = rows if sequence_length == 0 else rows // sequence_length * (sequence_length - 1)
        grad_scale = 1.0 / n
    loss = torch.empty(rows, device=logits.device, dtype=torch.float32)
    dlogits = logits if in_place else torch.empty_like(logits)
    invalid = torch.zeros(1, device=logits.device, dtype=torch.int32)
    call("spar_b200_cross_entropy_forward_backward", loss.data_ptr(), dlogits.data_ptr(),
         logits.data_ptr(), targets.contiguous().data_ptr(), rows, classes, classes,
         sequence_length, grad_scale, invalid.data_ptr(), _dev(logits), _stream(logits))
    return loss, dlogits, invalid


def total_sum(values):
    out = torch.empty(1, device=values.device, dtype=torch.float32)
    call("spar_b200_sum", out.data_ptr(), _f32(values, "values").data_ptr(), values.numel(),
         _dev(values), _stream(values))
    return out


# ------------------------------------------------------------------------------- AdamW
def _slices(params, grads, ms, vs):
    arr = (SparB200TensorSlice * len(params))()
    for j, (pp, g, m, v) in enumerate(zip(params, grads, ms, vs)):
        arr[j] = SparB200TensorSlice(_ptr(pp), _ptr(g), _ptr(m), _ptr(v), g.numel())
    return arr


def grad_norm_squared(grads, norm_state=None):
    dev = grads[0].device
    if norm_state is None:
        norm_state = torch.zeros(NORM_STATE_DOUBLES, device=dev, dtype=torch.float64)
    arr = _slices([None] * len(grads), grads, [None] * len(grads), [None] * len(grads))
    call("spar_b200_grad_norm_squared", norm_state.data_ptr(), arr, len(grads), dev.index,
         _stream(grads[0]))
    return norm_state


def adamw_clipped(params, grads, first_moments, second_moments, norm_state, *, lr, beta1=0.9,
                  beta2=0.999, eps=1e-8, weight_decay=0.01, step=1, max_norm=-1.0):
    dev = params[0].device
    flag = torch.zeros(1, device=dev, dtype=torch.int32)
    arr = _slices(params, grads, first_moments, second_moments)
    call("spar_b200_adamw_clipped", arr, len(params), norm_state.data_ptr(), max_norm, lr, beta1,
         beta2, eps, weight_decay, step, flag.data_ptr(), dev.index, _stream(params[0]))
    return flag


# ------------------------------------------------------------------------------- embedding
def embedding_forward(weight, ids):
    vocab, dim = weight.shape
    out = torch.empty(ids.numel(), dim, device=weight.device, dtype=torch.float32)
    invalid = torch.zeros(1, device=weight.device, dtype=torch.int32)
    call("spar_b200_embedding_forward", out.data_ptr(), _f32(weight, "weight").data_ptr(),
         ids.contiguous().data_ptr(), ids.numel(), vocab, dim, invalid.data_ptr(),
         _dev(weight), _stream(weight))
    return out, invalid


def embedding_backward(grad_weight, grad_out, ids):
    vocab, dim = grad_weight.shape
    lib = _lib.load()
    nbytes = lib.spar_b200_embedding_backward_scratch_bytes(ids.numel(), vocab)
    scratch = torch.empty(max(nbytes, 16), device=grad_weight.device, dtype=torch.uint8)
    call("spar_b200_embedding_backward", grad_weight.data_ptr(), _f32(grad_out, "grad").data_ptr(),
         ids.contiguous().data_ptr(), ids.numel(), vocab, dim, scratch.data_ptr(),
         _dev(grad_weight), _stream(grad_weight))
    return grad_weight


def column_sum(x, out=None, accumulate=False):
    rows, cols = x.shape
    out = torch.empty(cols, device=x.device, dtype=torch.float32) if out is None else out
    call("spar_b200_column_sum", out.data_ptr(), _f32(x, "x").data_ptr(), rows, cols, cols,
         int(accumulate), _dev(x), _stream(x))
    return out


def rope_table(t: int, d: int, theta: float = 10000.0, start: int = 0, device=None):
    table = torch.empty(t, d // 2, 2, device=device, dtype=torch.float32)
    call("spar_b200_rope_table", table.data_ptr(), t, d, theta, start, table.device.index,
         torch.cuda.current_stream(table.device).cuda_stream)
    return table


def rope_apply_(x, table, batch: int, t: int, heads: int, d: int, ld: int, inverse=False):
    call("spar_b200_rope_apply", x.data_ptr(), table.data_ptr(), batch, t, heads, d, ld,
         int(inverse), _dev(x), _stream(x))
    return x


# ------------------------------------------------------------------------------- GEMM
def gemm_desc(m, n, k, a, lda, b, ldb, c, ldc, *, a_t=False, b_t=False, alpha=1.0,
              accumulate=False, epilogue=EPI_NONE, bias=None, aux=None, ldaux=0,
              precision=TF32, causal=CAUSAL_NONE, batch=(1, 1), a_bs=(0, 0), b_bs=(0, 0),
              c_bs=(0, 0), round_output=False, rope=None, column_partials=None) -> SparB200Gemm:
    """rope = (table, seq, dim, cols) applies RoPE to columns < cols in the epilogue;
    column_partials = a device pointer to [ceil(m / 32), n] floats for per-32-row column sums."""
    g = SparB200Gemm()
    g.round_output = int(round_output)
    g.column_partials = column_partials
    if rope is not None:
        g.rope_table, g.rope_seq, g.rope_dim, g.rope_cols = rope[0].data_ptr(), *rope[1:]
    g.m, g.n, g.k = m, n, k
    g.batch[0], g.batch[1] = batch
    g.a, g.lda, g.a_transposed = a, lda, int(a_t)
    g.a_batch_stride[0], g.a_batch_stride[1] = a_bs
    g.b, g.ldb, g.b_transposed = b, ldb, int(b_t)
    g.b_batch_stride[0], g.b_batch_stride[1] = b_bs
    g.c, g.ldc = c, ldc
    g.c_batch_stride[0], g.c_batch_stride[1] = c_bs
    g.alpha, g.accumulate, g.epilogue = alpha, int(accumulate), epilogue
    g.bias, g.aux, g.ldaux = bias, aux, ldaux
    g.precision, g.causal = precision, causal
    return g


def gemm_run(desc: SparB200Gemm, device: int, stream: int) -> None:
    call("spar_b200_gemm", ctypes.byref(desc), device, stream)


def matmul(a, b, *, a_t=False, b_t=False, out=None, alpha=1.0, accumulate=False,
           epilogue=EPI_NONE, bias=None, aux=None, precision=TF32, round_output=False, rope=None,
           column_partials=None):
    """C = alpha * op(a) @ op(b) (+ epilogue) for 2-D row-major float32 tensors.

    op(a) = a.T when a_t (a stored [k, m]); op(b) = b.T when b_t (b stored [n, k]).
    column_partials: optional float32 tensor [ceil(m / 32), n] receiving per-32-row-block column
    sums of the epilogue output (its rows sum to the column sums of the result).
    """
    _f32(a, "a")
    _f32(b, "b")
    m, k = (a.shape[1], a.shape[0]) if a_t else a.shape
    k2, n = (b.shape[1], b.shape[0]) if b_t else b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    c = torch.empty(m, n, device=a.device, dtype=torch.float32) if out is None else out
    desc = gemm_desc(m, n, k, a.data_ptr(), a.shape[1], b.data_ptr(), b.shape[1], c.data_ptr(),
                     c.shape[1], a_t=a_t, b_t=b_t, alpha=alpha, accumulate=accumulate,
                     epilogue=epilogue, bias=_ptr(bias), aux=_ptr(aux),
                     ldaux=(aux.shape[1] if aux is not None else 0), precision=precision,
                     round_output=round_output, rope=rope,
                     column_partials=_ptr(column_partials))
    gemm_run(desc, _dev(a), _stream(a))
    return c


def gemm_error(device: int = 0, clear: bool = True) -> int:
    return _lib.load().spar_b200_gemm_error(device, int(clear))
