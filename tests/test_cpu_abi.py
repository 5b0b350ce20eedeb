"""The C-ABI boundary without a GPU: the library loads, exports every symbol the
headers declare, its structs have the C layout, and the host-side entry points
(GGUF loader, wave validation) behave like the reference's."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, REF_ROOT

INCLUDE = os.path.join(ROOT, "include")
REF_GGUF_H = os.path.join(REF_ROOT, "vendor", "embeddinggemma.c", "src", "gguf.h")


def _declared_functions():
    names = []
    for h in sorted(os.listdir(INCLUDE)):
        src = open(os.path.join(INCLUDE, h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", src, flags=re.M):
            if m.group(1) not in ("if", "defined"):
                names.append(m.group(1))
    return names


def test_headers_declare_what_the_binding_binds():
    declared = set(_declared_functions())
    from importlib import import_module
    sigs = import_module("embeddinggemma2-amdkfd_b200._lib").SIGNATURES
    assert declared == set(sigs), (declared ^ set(sigs))
    assert {"ei_gemma2_kfd_create", "ei_gemma2_kfd_free", "ei_gemma2_kfd_batch"} <= declared


def test_library_exports_every_declared_symbol(eg2):
    lib = eg2._lib.load()  # raises if the .so is missing: there is no fallback
    out = subprocess.run(["nm", "-D", "--defined-only", eg2._lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    for name in _declared_functions():
        assert name in exported, name
        assert getattr(lib, name) is not None


def _c_layout(tmp_path, structs, header):
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{header}"', "int main(void) {"]
    for sname, cls in structs.items():
        lines.append(f'printf("%s size %zu\\n", "{sname}", sizeof({sname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("%s.%s %zu\\n", "{sname}", "{fname}", offsetof({sname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", INCLUDE, str(src), "-o", str(exe)], check=True)
    return dict(l.rsplit(" ", 1) for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                            check=True).stdout.splitlines())


def test_ctypes_structs_have_the_c_layout(eg2, tmp_path):
    structs = eg2._lib.STRUCTS
    got = _c_layout(tmp_path, structs, "eg2_ops.h")
    for sname, cls in structs.items():
        assert int(got[f"{sname} size"]) == C.sizeof(cls), sname
        for fname, _ in cls._fields_:
            assert int(got[f"{sname}.{fname}"]) == getattr(cls, fname).offset, (sname, fname)


def test_operator_structs_match_reference_abi(tmp_path):
    """Part 1 of eg2_ops.h is kernels/abi.h's nine structs byte for byte."""
    ref = os.path.join(REF_ROOT, "kernels", "abi.h")
    if not os.path.exists(ref):
        pytest.skip("reference sources not present")
    names = ["EgGather", "EgMM", "EgNorm", "EgRope", "EgAttention", "EgElement", "EgPool", "EgNormResidual",
             "EgNormRope"]
    prog = ["#include <stdio.h>", "#include <stddef.h>", "#include <stdint.h>", "#include HDR", "int main(void){"]
    prog += [f'printf("{n} %zu\\n", sizeof({n}));' for n in names] + ["return 0;}"]
    (tmp_path / "s.c").write_text("\n".join(prog))
    outs = []
    for hdr in (f'"{ref}"', '"eg2_ops.h"'):
        exe = tmp_path / f"s{len(outs)}"
        subprocess.run(["gcc", "-std=c11", "-I", INCLUDE, f"-DHDR={hdr}", str(tmp_path / "s.c"), "-o", str(exe)],
                       check=True)
        outs.append(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert outs[0] == outs[1]


def test_gguf_struct_is_layout_identical_to_reference(eg2, tmp_path):
    """ei_gemma2_kfd_create receives the reference loader's ei_gguf: same size and
    field offsets whether the reference's gguf.h or ours defines it."""
    if not os.path.exists(REF_GGUF_H):
        pytest.skip("reference sources not present")
    fields = {"ei_gguf": ["map", "map_len", "version", "n_kv", "n_tensors", "alignment", "data_off", "kv",
                          "tensors"],
              "ei_tensor": ["name", "n_dims", "ne", "type", "offset", "data", "n_bytes"],
              "ei_kv": ["key", "type", "v", "arr_type", "arr_n", "arr_data"]}
    prog = ["#include <stdio.h>", "#include <stddef.h>", "#include HDR", "int main(void){"]
    for s, fs in fields.items():
        prog.append(f'printf("{s} %zu\\n", sizeof({s}));')
        prog += [f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));' for f in fs]
    prog.append("return 0;}")
    (tmp_path / "g.c").write_text("\n".join(prog))
    outs = []
    for hdr in (f'"{REF_GGUF_H}"', '"eg2_gguf.h"'):
        exe = tmp_path / f"g{len(outs)}"
        subprocess.run(["gcc", "-std=c11", "-I", INCLUDE, f"-DHDR={hdr}", str(tmp_path / "g.c"), "-o", str(exe)],
                       check=True)
        outs.append(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert outs[0] == outs[1]
    assert f"ei_gguf {eg2._lib.load().eg2_gguf_struct_size()}\n" in outs[1]


class _Str(C.Structure):
    _fields_ = [("str", C.c_void_p), ("len", C.c_uint64)]


class _Tensor(C.Structure):
    _fields_ = [("name", _Str), ("n_dims", C.c_uint32), ("ne", C.c_uint64 * 4), ("type", C.c_uint32),
                ("offset", C.c_uint64), ("data", C.c_void_p), ("n_bytes", C.c_uint64)]


class _Gguf(C.Structure):
    _fields_ = [("map", C.c_void_p), ("map_len", C.c_size_t), ("version", C.c_uint32), ("n_kv", C.c_uint64),
                ("n_tensors", C.c_uint64), ("alignment", C.c_uint64), ("data_off", C.c_uint64),
                ("kv", C.c_void_p), ("tensors", C.POINTER(_Tensor))]


def test_gguf_loader_indexes_like_the_reader(eg2, model_baseline):
    """eg2_gguf_open's tensor table equals an independent numpy parse of the file."""
    import oracle
    lib = eg2._lib.load()
    assert lib.eg2_gguf_struct_size() == C.sizeof(_Gguf)
    g = _Gguf()
    err = C.create_string_buffer(256)
    assert lib.eg2_gguf_open(C.byref(g), model_baseline.encode(), err, 256), err.value
    try:
        ref = oracle.Gguf(model_baseline)
        assert g.version == 3 and g.n_tensors == len(ref.tensors)
        base = g.map
        for i in range(g.n_tensors):
            t = g.tensors[i]
            name = C.string_at(t.name.str, t.name.len).decode()
            ne, typ, data = ref.tensors[name]
            assert t.type == typ and t.n_bytes == data.nbytes, name
            assert list(t.ne[:t.n_dims]) == list(ne[:t.n_dims]), name
            assert t.data - base == g.data_off + t.offset, name
    finally:
        lib.eg2_gguf_close(C.byref(g))


def test_gguf_loader_rejects_bad_files(eg2, tmp_path, model_baseline):
    lib = eg2._lib.load()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(60))
    trunc = tmp_path / "trunc.gguf"
    with open(model_baseline, "rb") as f:
        trunc.write_bytes(f.read(4096))
    for path, msg in ((tmp_path / "missing.gguf", "cannot open"), (bad, "not a GGUF"), (trunc, "")):
        g = _Gguf()
        err = C.create_string_buffer(256)
        assert not lib.eg2_gguf_open(C.byref(g), str(path).encode(), err, 256)
        assert msg in err.value.decode() and err.value


def test_validate_uses_reference_messages(eg2):
    """gemma2_kfd.cpp:270-278, checked on the host before any upload."""
    ok = np.array([2, 5, 1], np.int32)
    eg2.validate(ok, np.array([0, 3], np.uint64))
    eg2.validate(np.array([2, 9, 1, 2, 1], np.int32), np.array([0, 3, 5], np.uint64))
    cases = [
        (ok, np.array([0, 0], np.uint64), "invalid KFD sequence offsets"),
        (ok, np.array([0, 3, 3], np.uint64), "invalid KFD sequence offsets"),
        (ok, np.array([1, 3], np.uint64), "KFD batch requires 1..2048 packed tokens and nonempty sequences"),
        (ok, np.array([0], np.uint64), "KFD batch requires 1..2048 packed tokens"),
        (np.full(2049, 5, np.int32), np.array([0, 2049], np.uint64), "1..2048 packed tokens"),
        (np.array([2, 262144, 1], np.int32), np.array([0, 3], np.uint64), "token ID out of range"),
        (np.array([2, -1, 1], np.int32), np.array([0, 3], np.uint64), "token ID out of range"),
    ]
    for ids, off, msg in cases:
        with pytest.raises(eg2.ExecutorError, match=re.escape(msg)):
            eg2.validate(ids, off)


def test_validate_rows_uses_reference_messages(eg2):
    """Soft-token waves (512-wide input rows instead of ids) take the offsets
    checks and messages of an ids wave; the rows themselves are not inspected."""
    rows = np.zeros((3, 512), np.float32)
    eg2.validate_rows(rows, np.array([0, 3], np.uint64))
    eg2.validate_rows(np.full((5, 512), np.nan, np.float32), np.array([0, 3, 5], np.uint64))
    cases = [
        (rows, np.array([0, 0], np.uint64), "invalid KFD sequence offsets"),
        (rows, np.array([1, 3], np.uint64), "KFD batch requires 1..2048 packed tokens and nonempty sequences"),
        (np.zeros((2049, 512), np.float32), np.array([0, 2049], np.uint64), "1..2048 packed tokens"),
        (np.zeros((0, 512), np.float32), np.array([0, 3], np.uint64), "1..2048 packed tokens"),
    ]
    for r, off, msg in cases:
        with pytest.raises(eg2.ExecutorError, match=re.escape(msg)):
            eg2.validate_rows(r, off)


def test_product_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "embeddinggemma2-amdkfd_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                src = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(import|from)\s+oracle", src, flags=re.M), f
                assert "eg2_oracle" not in src and "libeg2ref" not in src, f


def test_reference_engine_links_against_library():
    """The reference's engine.c, compiled unchanged with -DEI_ENABLE_KFD=1
    against include/ (gemma2_kfd.h forwards to eg2_executor.h), links with
    libeg2_b200.so: the three executor calls it makes are undefined in the
    engine object and defined by the library (oracle/Makefile engine_link)."""
    if not os.path.isdir(os.path.join(REF_ROOT, "vendor")):
        pytest.skip("reference sources not present")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "engine_link", f"REF_ROOT={REF_ROOT}"],
                   check=True)
    so = os.path.join(ROOT, "oracle", "_ref", "libeg2enginelink.so")
    needed = subprocess.run(["readelf", "-d", so], capture_output=True, text=True, check=True).stdout
    assert "[libeg2_b200.so]" in needed
    syms = subprocess.run(["nm", "-D", so], capture_output=True, text=True, check=True).stdout.split("\n")
    lib = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "embeddinggemma2-amdkfd_b200",
                                                                      "libeg2_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    for fn in ("ei_gemma2_kfd_create", "ei_gemma2_kfd_free", "ei_gemma2_kfd_batch"):
        assert any(l.split()[-2:] == ["U", fn] for l in syms if l.strip()), fn
        assert f" T {fn}" in lib, fn


def test_reference_server_cuda_build_links_against_library():
    """The reference's HTTP server built for its CUDA backend
    (-DEI_ENABLE_CUDA, server.c / engine.c / media.c unchanged) against
    include/gemma2_cuda.h takes every ei_gemma2_cuda_* call it makes -- create
    per device, clone per pipeline slot, batch, the media entry points -- from
    libeg2_b200.so (oracle/Makefile server)."""
    if not os.path.isdir(os.path.join(REF_ROOT, "vendor")):
        pytest.skip("reference sources not present")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "server", f"REF_ROOT={REF_ROOT}"], check=True)
    exe = os.path.join(ROOT, "oracle", "_ref", "eg2server_cuda")
    assert "[libeg2_b200.so]" in subprocess.run(["readelf", "-d", exe], capture_output=True, text=True,
                                                check=True).stdout
    undef = subprocess.run(["nm", "-u", exe], capture_output=True, text=True, check=True).stdout
    lib = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "embeddinggemma2-amdkfd_b200",
                                                                      "libeg2_b200.so")],
                         capture_output=True, text=True, check=True).stdout
    for fn in ("ei_gemma2_cuda_create", "ei_gemma2_cuda_create_on", "ei_gemma2_cuda_clone", "ei_gemma2_cuda_batch",
               "ei_gemma2_cuda_free", "ei_gemma2_cuda_device", "ei_gemma2_cuda_device_count",
               "ei_gemma2_cuda_embed_inputs", "ei_gemma2_cuda_vision", "ei_gemma2_cuda_audio"):
        assert f" U {fn}" in undef, fn
        assert f" T {fn}" in lib, fn
