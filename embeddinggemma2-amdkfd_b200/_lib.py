"""ctypes binding of libeg2_b200.so (the C ABI declared in include/*.h).

The library is built in-tree (build.py).  There is no fallback: if it is
missing or does not load, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libeg2_b200.so")

vp, i32, u32, sz, f32, cstr, b = (C.c_void_p, C.c_int, C.c_uint, C.c_size_t, C.c_float, C.c_char_p,
                                  C.c_bool)

# name -> (restype, argtypes); every function include/*.h declares.
SIGNATURES = {
    # include/eg2_gguf.h
    "eg2_gguf_open": (b, [vp, cstr, cstr, sz]),
    "eg2_gguf_close": (None, [vp]),
    "eg2_gguf_struct_size": (sz, []),
    # include/eg2_executor.h
    "ei_gemma2_kfd_create": (vp, [vp, cstr, sz]),
    "ei_gemma2_kfd_create_on": (vp, [vp, i32, cstr, sz]),
    "eg2_b200_create": (vp, [vp, i32, u32, cstr, sz]),
    "ei_gemma2_kfd_free": (None, [vp]),
    "ei_gemma2_kfd_batch": (b, [vp, vp, vp, sz, vp, cstr, sz]),
    "eg2_b200_prepare": (i32, [vp, u32, cstr, sz]),
    # the reference's CUDA executor ABI (include/gemma2_cuda.h)
    "ei_gemma2_cuda_create": (vp, [vp, cstr, sz]),
    "ei_gemma2_cuda_create_on": (vp, [vp, i32, cstr, sz]),
    "ei_gemma2_cuda_device_count": (i32, []),
    "ei_gemma2_cuda_device": (i32, [vp]),
    "ei_gemma2_cuda_free": (None, [vp]),
    "ei_gemma2_cuda_clone": (vp, [vp, b, cstr, sz]),
    "ei_gemma2_cuda_batch": (b, [vp, vp, vp, sz, vp, cstr, sz]),
    "ei_gemma2_cuda_embed_inputs": (b, [vp, vp, sz, vp, cstr, sz]),
    "ei_gemma2_cuda_vision": (b, [vp, vp, vp, i32, i32, vp, vp, cstr, sz]),
    "ei_gemma2_cuda_audio": (b, [vp, vp, vp, i32, vp, vp, cstr, sz]),
    "eg2_b200_validate": (b, [vp, vp, sz, cstr, sz]),
    "eg2_b200_stage": (b, [vp, vp, vp, sz, cstr, sz]),
    "eg2_b200_launch": (b, [vp, i32, cstr, sz]),
    "eg2_b200_finish": (b, [vp, vp, cstr, sz]),
    "eg2_b200_submit": (i32, [vp, vp, vp, sz, cstr, sz]),
    "eg2_b200_collect": (b, [vp, i32, vp, cstr, sz]),
    "eg2_b200_validate_rows": (b, [vp, vp, sz, cstr, sz]),
    "eg2_b200_batch_rows": (b, [vp, vp, vp, sz, vp, cstr, sz]),
    "eg2_b200_stage_rows": (b, [vp, vp, vp, sz, cstr, sz]),
    "eg2_b200_submit_rows": (i32, [vp, vp, vp, sz, cstr, sz]),
    "eg2_b200_forward_layers": (b, [vp, vp, vp, vp, sz, i32, i32, vp, cstr, sz]),
    "eg2_b200_normalize_prefix": (b, [vp, i32]),
    "eg2_b200_stream": (vp, [vp]),
    "eg2_b200_kernels_per_wave": (i32, [vp]),
    "eg2_b200_profile": (i32, [vp, vp, vp, i32]),
    "eg2_b200_device": (i32, [vp]),
    # include/eg2_ops.h
    "eg2_launch_gather": (i32, [vp, vp]),
    "eg2_launch_mm": (i32, [vp, vp]),
    "eg2_launch_norm": (i32, [vp, vp]),
    "eg2_launch_rope": (i32, [vp, vp]),
    "eg2_launch_attention": (i32, [vp, u32, vp]),
    "eg2_launch_element": (i32, [vp, vp]),
    "eg2_launch_pool": (i32, [vp, vp]),
    "eg2_launch_norm_residual": (i32, [vp, vp]),
    "eg2_launch_norm_rope": (i32, [vp, vp]),
    "eg2_launch_embed": (i32, [vp, vp]),
    "eg2_launch_ple_proj": (i32, [vp, vp]),
    "eg2_launch_norm_quant": (i32, [vp, vp]),
    "eg2_launch_q8_mm": (i32, [vp, vp]),
    "eg2_launch_q8_geglu": (i32, [vp, vp]),
    "eg2_launch_qkv_post": (i32, [vp, vp]),
    "eg2_launch_attention_f16": (i32, [vp, vp]),
    "eg2_launch_attention_tc": (i32, [vp, vp]),
    "eg2_launch_attention_tc_q8": (i32, [vp, vp]),
    "eg2_launch_attention_exact": (i32, [vp, u32, vp]),
    "eg2_launch_post_add": (i32, [vp, vp]),
    "eg2_launch_gate_quant": (i32, [vp, vp]),
    "eg2_launch_gelu_mul": (i32, [vp, vp]),
    "eg2_launch_pool_l2": (i32, [vp, vp]),
    "eg2_repack_q8": (i32, [vp, u32, u32, vp, vp, vp]),
    "eg2_read_error": (i32, []),
    "eg2_clear_error": (None, []),
    "eg2_selftest_wait_timeout": (i32, [vp]),
}

_lib = None


def load() -> C.CDLL:
    """Load the library once; raise if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python embeddinggemma2-amdkfd_b200/build.py`")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


# ---- operator ABI structs (include/eg2_ops.h), same field order and types ----
P = C.c_void_p


class EgGather(C.Structure):
    _fields_ = [("out", P), ("weight", P), ("ids", P), ("n", u32)]


class EgMM(C.Structure):
    _fields_ = [("out", P), ("x", P), ("weight", P), ("n", u32), ("k", u32), ("m", u32), ("type", u32)]


class EgNorm(C.Structure):
    _fields_ = [("out", P), ("x", P), ("weight", P), ("rows", u32), ("d", u32), ("scale", f32)]


class EgRope(C.Structure):
    _fields_ = [("x", P), ("table", P), ("n", u32), ("heads", u32), ("d", u32)]


class EgAttention(C.Structure):
    _fields_ = [("out", P), ("q", P), ("k", P), ("v", P), ("bounds", P), ("n", u32), ("window", u32)]


class EgElement(C.Structure):
    _fields_ = [("out", P), ("x", P), ("other", P), ("n", u32), ("mode", u32), ("layer", u32), ("scale", f32)]


class EgPool(C.Structure):
    _fields_ = [("out", P), ("x", P), ("offsets", P), ("batch", u32)]


class EgNormResidual(C.Structure):
    _fields_ = [("out", P), ("x", P), ("weight", P), ("rows", u32), ("d", u32), ("scale", f32)]


class EgNormRope(C.Structure):
    _fields_ = [("x", P), ("weight", P), ("table", P), ("rows", u32), ("d", u32), ("heads", u32)]


class EgEmbed(C.Structure):
    _fields_ = [("x", P), ("x_hi", P), ("x_lo", P), ("token_embd", P), ("ids", P), ("n", u32)]


class EgPleProj(C.Structure):
    _fields_ = [("ple", P), ("x_hi", P), ("x_lo", P), ("weight", P), ("norm", P), ("n", u32)]


class EgNormQuant(C.Structure):
    _fields_ = [("q", P), ("scale", P), ("scale_stride", u32), ("y", P), ("x", P), ("weight", P),
                ("rows", u32), ("width", u32), ("tier", u32)]


class EgQ8MM(C.Structure):
    _fields_ = [("out", P), ("xq", P), ("xs", P), ("xs_stride", u32), ("wq", P), ("ws", P),
                ("n", u32), ("k", u32), ("m", u32), ("exact", u32)]


class EgQ8GeGLU(C.Structure):
    _fields_ = [("q", P), ("scale", P), ("scale_stride", u32), ("xq", P), ("xs", P), ("xs_stride", u32), ("wq", P),
                ("ws", P), ("n", u32), ("k", u32), ("m", u32), ("exact", u32), ("tier", u32)]


class EgQkvPost(C.Structure):
    _fields_ = [("q", P), ("k", P), ("v", P), ("qkv", P), ("q_norm", P), ("k_norm", P),
                ("rope_cos", P), ("rope_sin", P), ("pos", P), ("n", u32), ("d", u32)]


class EgAttentionF16(C.Structure):
    _fields_ = [("out", P), ("q", P), ("k", P), ("v", P), ("bounds", P), ("n", u32), ("d", u32),
                ("window", u32)]


class EgAttentionQ8(C.Structure):
    _fields_ = [("q", P), ("qscale", P), ("scale_stride", u32), ("qh", P), ("k", P), ("v", P), ("bounds", P),
                ("n", u32), ("window", u32), ("tier", u32), ("d", u32)]


class EgPostAdd(C.Structure):
    _fields_ = [("x", P), ("h", P), ("weight", P), ("scale", P), ("q", P), ("qscale", P),
                ("scale_stride", u32), ("next_weight", P), ("rows", u32), ("tier", u32)]


class EgGateQuant(C.Structure):
    _fields_ = [("q", P), ("scale", P), ("scale_stride", u32), ("x", P), ("other", P), ("rows", u32),
                ("width", u32), ("other_stride", u32), ("other_offset", u32), ("tier", u32)]


class EgGeluMul(C.Structure):
    _fields_ = [("g", P), ("u", P), ("n", C.c_uint64), ("tier", u32)]


class EgPoolL2(C.Structure):
    _fields_ = [("out", P), ("y", P), ("offsets", P), ("batch", u32), ("width", u32)]


STRUCTS = {c.__name__: c for c in (EgGather, EgMM, EgNorm, EgRope, EgAttention, EgElement, EgPool, EgNormResidual,
                                   EgNormRope, EgEmbed, EgPleProj, EgNormQuant, EgQ8MM, EgQ8GeGLU, EgQkvPost, EgAttentionF16,
                                   EgPostAdd, EgGateQuant, EgGeluMul, EgPoolL2)}
