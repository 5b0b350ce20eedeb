"""Operator ABI calls (include/eg2_ops.h) on torch CUDA tensors.

Each function fills the parameter struct with device pointers and enqueues the
operator on the current torch stream; a non-zero return code raises.  torch is
only the allocator and stream provider here.
"""
from __future__ import annotations

import ctypes as C

from . import _lib


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call(name, struct, *extra):
    fn = getattr(_lib.load(), name)
    rc = fn(C.byref(struct), *extra, _stream())
    if rc:
        raise RuntimeError(f"{name} failed with CUDA error {rc}")


# ---- kernels/abi.h operators (reference semantics) ----
def gather(out, weight, ids, n):
    _call("eg2_launch_gather", _lib.EgGather(_p(out), _p(weight), _p(ids), n))


def mm(out, x, weight, n, k, m, type_):
    _call("eg2_launch_mm", _lib.EgMM(_p(out), _p(x), _p(weight), n, k, m, type_))


def norm(out, x, weight, rows, d, scale=1.0):
    _call("eg2_launch_norm", _lib.EgNorm(_p(out), _p(x), _p(weight), rows, d, scale))


def rope(x, table, n, heads, d):
    _call("eg2_launch_rope", _lib.EgRope(_p(x), _p(table), n, heads, d))


def attention(out, q, k, v, bounds, n, window, d):
    _call("eg2_launch_attention", _lib.EgAttention(_p(out), _p(q), _p(k), _p(v), _p(bounds), n, window), C.c_uint(d))


def element(out, x, other, n, mode, layer=0, scale=1.0):
    _call("eg2_launch_element", _lib.EgElement(_p(out), _p(x), _p(other), n, mode, layer, scale))


def pool(out, x, offsets, batch):
    _call("eg2_launch_pool", _lib.EgPool(_p(out), _p(x), _p(offsets), batch))


def norm_residual(out, x, weight, rows, d, scale):
    _call("eg2_launch_norm_residual", _lib.EgNormResidual(_p(out), _p(x), _p(weight), rows, d, scale))


def norm_rope(x, weight, table, rows, d, heads):
    _call("eg2_launch_norm_rope", _lib.EgNormRope(_p(x), _p(weight), _p(table), rows, d, heads))


# ---- fused executor operators ----
def embed(x, x_hi, x_lo, token_embd, ids, n):
    _call("eg2_launch_embed", _lib.EgEmbed(_p(x), _p(x_hi), _p(x_lo), _p(token_embd), _p(ids), n))


def ple_proj(ple, x_hi, x_lo, weight, norm_w, n):
    _call("eg2_launch_ple_proj", _lib.EgPleProj(_p(ple), _p(x_hi), _p(x_lo), _p(weight), _p(norm_w), n))


def norm_quant(q, scale, scale_stride, x, weight, rows, width, y=None, tier=0):
    _call("eg2_launch_norm_quant", _lib.EgNormQuant(_p(q), _p(scale), scale_stride, _p(y), _p(x), _p(weight),
                                                    rows, width, tier))


def q8_mm(out, xq, xs, xs_stride, wq, ws, n, k, m, exact=False):
    _call("eg2_launch_q8_mm", _lib.EgQ8MM(_p(out), _p(xq), _p(xs), xs_stride, _p(wq), _p(ws), n, k, m, int(exact)))


def q8_geglu(q, scale, scale_stride, xq, xs, xs_stride, wq, ws, n, k, m, exact=False, tier=0):
    _call("eg2_launch_q8_geglu", _lib.EgQ8GeGLU(_p(q), _p(scale), scale_stride, _p(xq), _p(xs), xs_stride, _p(wq),
                                                _p(ws), n, k, m, int(exact), tier))


def qkv_post(q, k, v, qkv, q_norm, k_norm, rope_cos, rope_sin, pos, n, d):
    _call("eg2_launch_qkv_post", _lib.EgQkvPost(_p(q), _p(k), _p(v), _p(qkv), _p(q_norm), _p(k_norm),
                                                _p(rope_cos), _p(rope_sin), _p(pos), n, d))


def attention_exact(out, q, k, v, bounds, n, d, window):
    """fp32 attention in the reference CPU graph's scalar order (parity mode)."""
    _call("eg2_launch_attention_exact", _lib.EgAttention(_p(out), _p(q), _p(k), _p(v), _p(bounds), n, window), d)


def attention_f16(out, q, k, v, bounds, n, d, window):
    _call("eg2_launch_attention_f16", _lib.EgAttentionF16(_p(out), _p(q), _p(k), _p(v), _p(bounds), n, d, window))


def attention_tc(out, q, k, v, bounds, n, window, d=256):
    """attention_f16 on the tcgen05 tensor cores (d = 256 or 512, n <= 8192)."""
    _call("eg2_launch_attention_tc", _lib.EgAttentionF16(_p(out), _p(q), _p(k), _p(v), _p(bounds), n, d, window))


def attention_tc_q8(q, qscale, scale_stride, qh, k, v, bounds, n, window, tier=0, d=256):
    """attention_tc with its output rows quantized to Q8_0 in the epilogue."""
    _call("eg2_launch_attention_tc_q8", _lib.EgAttentionQ8(_p(q), _p(qscale), scale_stride, _p(qh), _p(k), _p(v),
                                                           _p(bounds), n, window, tier, d))


def post_add(x, h, weight, scale, q, qscale, scale_stride, next_weight, rows, tier=0):
    _call("eg2_launch_post_add", _lib.EgPostAdd(_p(x), _p(h), _p(weight), _p(scale), _p(q), _p(qscale),
                                                scale_stride, _p(next_weight), rows, tier))


def gate_quant(q, scale, scale_stride, x, other, rows, width, other_stride, other_offset, tier=0):
    _call("eg2_launch_gate_quant", _lib.EgGateQuant(_p(q), _p(scale), scale_stride, _p(x), _p(other), rows, width,
                                                    other_stride, other_offset, tier))


def gelu_mul(g, u, n, tier=0):
    """g[:n] = gelu_tanh(g[:n]) * u[:n] in place (u None: gelu only)."""
    _call("eg2_launch_gelu_mul", _lib.EgGeluMul(_p(g), _p(u), n, tier))


def pool_l2(out, y, offsets, batch, width):
    _call("eg2_launch_pool_l2", _lib.EgPoolL2(_p(out), _p(y), _p(offsets), batch, width))


def repack_q8(blocks, rows, k, codes, scales):
    rc = _lib.load().eg2_repack_q8(_p(blocks), rows, k, _p(codes), _p(scales), _stream())
    if rc:
        raise RuntimeError(f"eg2_repack_q8 failed with CUDA error {rc}")


def read_error() -> int:
    return int(_lib.load().eg2_read_error())


def clear_error():
    _lib.load().eg2_clear_error()


def selftest_wait_timeout(stream=None):
    """Enqueue a kernel whose bounded wait runs out (sets the error word)."""
    rc = _lib.load().eg2_selftest_wait_timeout(C.c_void_p(stream) if stream is not None else _stream())
    if rc:
        raise RuntimeError(f"eg2_selftest_wait_timeout failed with CUDA error {rc}")
