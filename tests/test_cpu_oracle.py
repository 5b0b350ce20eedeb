"""The oracle pinned to the reference (CPU only, no GPU).

The checker every GPU parity test relies on is oracle/eg2_oracle.c, a C
restatement of the reference's scalar CPU tier
(vendor/embeddinggemma.c/src/gemma2_fast.c).  These tests pin it against the
golden fixtures that tests/golden/make_golden.py produced by running the
reference itself (oracle/_ref, compiled from the reference's own sources), and,
where that build is present, against the reference live.
"""
import hashlib
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN, ROOT, cosine, golden


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


@pytest.mark.parametrize("norm", ["baseline", "plus1"])
def test_synthetic_models_are_the_golden_ones(syn, norm):
    """The seeded GGUF writer reproduces, byte for byte, the files the goldens came from."""
    meta = json.load(open(os.path.join(GOLDEN, "golden_meta.json")))[norm]
    assert _sha256(syn.model_path(meta["seed"], norm)) == meta["gguf_sha256"]


@pytest.mark.parametrize("norm", ["baseline", "plus1"])
def test_port_is_bit_identical_to_reference_scalar_tier(port, syn, norm):
    """Config-0 wave: the restatement equals ei_gemma2_embed_batch_fast_ctx at the
    scalar tier (EI_GEMMA2_CPU_X86=scalar) bit for bit, on both weight models."""
    import oracle
    g = golden(f"golden_{norm}.npz")
    out = port.embed(oracle.Gguf(syn.model_path(1234, norm)), g["ids"], g["offsets"])
    assert out.dtype == np.float32 and out.shape == g["embed_scalar"].shape
    assert np.array_equal(out, g["embed_scalar"])


@pytest.fixture
def vnni_port(port):
    """The restatement in the float orders of the reference's default tier on
    an AVX-512 VNNI host; restored to the scalar loops afterwards."""
    port.set_order(port.ORDER_VNNI512)
    yield port
    port.set_order(port.ORDER_SCALAR)


@pytest.mark.parametrize("norm", ["baseline", "plus1"])
def test_port_vnni512_order_is_bit_identical_to_reference_best_tier(vnni_port, syn, norm):
    """Config-0 wave: with the VNNI-512 float orders (gemma2_fast_x86.c lane
    sums, x86 quantizer and GELU) the restatement equals the reference's
    default tier, recorded as vnni512+gemm512 in the fixture, bit for bit --
    on the plus-one model too, where the two tiers decorrelate entirely."""
    import oracle
    g = golden(f"golden_{norm}.npz")
    assert str(g["best_tier"]) == "vnni512+gemm512"
    out = vnni_port.embed(oracle.Gguf(syn.model_path(1234, norm)), g["ids"], g["offsets"],
                          quant_mode=vnni_port.ROUND_X86, gelu_mode=1)
    assert np.array_equal(out, g["embed_best"])


def test_port_vnni512_order_short_and_input_waves(vnni_port, syn):
    """Waves of at most 8 tokens (the reference's 4-row tile order) and of 9
    (its 512-bit GEMM), and the input-rows wave, at the default tier."""
    import oracle
    m = oracle.Gguf(syn.model_path(1234, "baseline"))
    g = golden("golden_short_baseline.npz")
    assert str(g["best_tier"]) == "vnni512+gemm512"
    for i in range(4):
        out = vnni_port.embed(m, g[f"ids{i}"], g[f"offsets{i}"], quant_mode=vnni_port.ROUND_X86, gelu_mode=1)
        assert np.array_equal(out, g[f"embed{i}"]), i
    g = golden("golden_inputs_baseline.npz")
    out = vnni_port.embed_inputs(m, g["inputs"], g["offsets"], quant_mode=vnni_port.ROUND_X86, gelu_mode=1)
    assert np.array_equal(out, g["embed_best"])


def test_port_input_rows_bit_identical_to_reference_scalar_tier(port, syn):
    """Media soft-token wave (512-wide input rows, ids NULL: gemma2_fast.c:940-941):
    the restatement equals the reference's scalar tier bit for bit."""
    import oracle
    g = golden("golden_inputs_baseline.npz")
    out = port.embed_inputs(oracle.Gguf(syn.model_path(1234, "baseline")), g["inputs"], g["offsets"])
    assert np.array_equal(out, g["embed_scalar"])


def test_port_x86_quantizer_matches_reference():
    """quantize_row_q8_0 of the x86 tiers (gemma2_fast_x86.c:211-234): codes and
    fp16 scale bits identical on 1024 seeded blocks."""
    import oracle
    oracle.build(ref=False)
    p = oracle.Port()
    g = golden("golden_ops.npz")
    q, s = p.quantize(g["q_in"], oracle.Port.ROUND_X86)
    assert np.array_equal(q, g["q_codes"])
    assert np.array_equal(s, g["q_scales"])


def test_port_x86_gelu_matches_reference():
    """The x86 tiers' exp-polynomial GELU times up (gemma2_fast_x86.c:308-325)."""
    import oracle
    oracle.build(ref=False)
    p = oracle.Port()
    g = golden("golden_ops.npz")
    assert np.array_equal(p.gelu_mul(g["gelu_g"], g["gelu_u"], mode=1), g["gelu_out"])


def test_reference_tier_floor_on_baseline_model():
    """The reference's own tiers agree on the BASELINE-distribution model only to
    a cosine floor; the end-to-end GPU tolerance is derived from this floor."""
    g = golden("golden_baseline.npz")
    c_best = cosine(g["embed_best"], g["embed_scalar"])
    c_graph = cosine(g["embed_reference_graph"], g["embed_scalar"])
    assert c_best.min() > 0.997 and c_graph.min() > 0.997
    for e in (g["embed_scalar"], g["embed_best"], g["embed_reference_graph"]):
        assert np.allclose(np.linalg.norm(e, axis=1), 1.0, atol=1e-5)


def test_plus1_model_is_chaotic_across_reference_tiers():
    """With 1 + N(0, 0.1) norm weights the reference's own tiers decorrelate:
    that model is for bit-exact checks only, never for a tolerance."""
    g = golden("golden_plus1.npz")
    assert cosine(g["embed_best"], g["embed_scalar"]).min() < 0.9


def test_port_matches_live_reference_scalar_tier(syn, tmp_path):
    """A fresh ragged wave through the reference (oracle/_ref) and the port.  The
    reference picks its tier once per process, so it runs in a child process."""
    import oracle
    lib = os.path.join(ROOT, "oracle", "_ref", "libeg2ref.so")
    if not os.path.exists(lib):
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    ids, off = syn.wave((3, 29, 1), seed=77)
    np.savez(tmp_path / "w.npz", ids=ids, off=off)
    code = ("import sys, numpy as np; sys.path[:0] = [%r, %r]; import oracle, importlib;"
            "syn = importlib.import_module('embeddinggemma2-amdkfd_b200.synthetic');"
            "w = np.load(%r); r = oracle.RefGraph(syn.model_path(1234, 'baseline'), 1);"
            "assert r.tier.startswith('scalar'), r.tier;"
            "np.save(%r, r.embed(w['ids'], w['off']))"
            % (ROOT, os.path.join(ROOT, "oracle"), str(tmp_path / "w.npz"), str(tmp_path / "ref.npy")))
    env = dict(os.environ, EI_GEMMA2_CPU_X86="scalar")
    subprocess.run([sys.executable, "-c", code], check=True, env=env, timeout=600)
    oracle.build(ref=False)
    out = oracle.Port().embed(oracle.Gguf(syn.model_path(1234, "baseline")), ids, off)
    assert np.array_equal(out, np.load(tmp_path / "ref.npy"))


def test_matryoshka_prefixes_match_reference(eg2):
    """normalize_prefix (the server's truncation, kernels.c:403-407) reproduces the
    reference's 128/256/512 prefixes of the config-2 embedding exactly."""
    g = golden("golden_long_baseline.npz")
    e = g["long_embed"][0]
    for d in (128, 256, 512):
        assert np.array_equal(eg2.normalize_prefix(e, d), g[f"long_prefix_{d}"])
    assert np.array_equal(eg2.normalize_prefix(e, 768), e)


def test_matryoshka_matches_reference_live(eg2, syn):
    """eg2_b200_normalize_prefix (host C) against the reference's own
    ei_embedding_normalize_prefix (oracle/_ref) on 200 random unit vectors,
    every supported width, bit for bit."""
    import oracle
    if not os.path.exists(oracle.REF_SO):
        pytest.skip("oracle/_ref not built")
    ref = oracle.RefGraph(syn.model_path(1234, "baseline"), 1)
    try:
        rng = np.random.default_rng(21)
        for _ in range(200):
            e = rng.standard_normal(768).astype(np.float32) * np.float32(rng.uniform(0.01, 3))
            e /= np.float32(np.linalg.norm(e))
            for d in (128, 256, 512, 768):
                assert np.array_equal(eg2.normalize_prefix(e, d), ref.normalize_prefix(e, d)), d
    finally:
        ref.close()


def test_device_expf_matches_c_library(tmp_path):
    """The expf the parity-mode attention evaluates (csrc/ref_expf.h, shared
    with the device code) equals the C library's expf -- which the reference's
    scalar attention calls -- on a strided sample of all float bit patterns
    in (-inf, 0] (the full range was checked when the header was written)."""
    src = tmp_path / "t.c"
    src.write_text(r"""
#include <stdio.h>
#include "ref_expf.h"
static const uint64_t tab[32] = {EG2_EXP2_TAB};
int main(void) {
    long long n = 0, bad = 0;
    for (uint64_t u = 0x80000000u; u <= 0xFF800000u; u += 97) {
        uint32_t b = (uint32_t)u; float x; memcpy(&x, &b, 4);
        ++n;
        float a = eg2_ref_expf(x, tab), r = expf(x);
        if (memcmp(&a, &r, 4) != 0) { if (bad < 3) printf("x=%a %a %a\n", x, a, r); ++bad; }
    }
    printf("%lld %lld\n", n, bad);
    return bad != 0;
}
""")
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-O2", "-std=c11", "-I", os.path.join(ROOT, "embeddinggemma2-amdkfd_b200", "csrc"), str(src),
                    "-o", str(exe), "-lm"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    n, bad = map(int, out.stdout.split()[-2:])
    assert n > 20_000_000 and bad == 0


def test_device_tanhf_matches_c_library(tmp_path):
    """The tanhf of the scalar-tier GELU (csrc/ref_tanhf.h, shared with the
    device code) equals the C library's tanhf -- which the reference's scalar
    tier calls -- on a strided sample of all finite floats of both signs (the
    full range was checked when the header was written)."""
    src = tmp_path / "t.c"
    src.write_text(r"""
#include <math.h>
#include <stdio.h>
#include "ref_tanhf.h"
int main(void) {
    long long n = 0, bad = 0;
    for (uint64_t u = 0; u < 0x7f800000u; u += 89) {
        for (int s = 0; s < 2; ++s) {
            float x = eg2_bitsf((uint32_t)u | (s ? 0x80000000u : 0u));
            ++n;
            if (eg2_fbits(eg2_ref_tanhf(x)) != eg2_fbits(tanhf(x))) ++bad;
        }
    }
    printf("%lld %lld\n", n, bad);
    return bad != 0;
}
""")
    exe = tmp_path / "t"
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-I",
                    os.path.join(ROOT, "embeddinggemma2-amdkfd_b200", "csrc"), str(src), "-o", str(exe), "-lm"],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    n, bad = map(int, out.stdout.split()[-2:])
    assert n > 40_000_000 and bad == 0


def _layer_errors(got, ref):
    """Per token: cosine and max |difference| of the L2-normalised rows."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    gn = got / np.linalg.norm(got, axis=1, keepdims=True)
    rn = ref / np.linalg.norm(ref, axis=1, keepdims=True)
    return float(cosine(got, ref).min()), float(np.abs(gn - rn).max())


def _teacher_forced_worst(port, syn, **variant):
    """Worst per-layer (cosine, max |diff|) of a perturbed restatement run one
    layer at a time from the unperturbed restatement's own layer inputs."""
    import oracle
    G = oracle.Gguf(syn.model_path(1234, "baseline"))
    ids, off = syn.wave((8, 17, 33, 64), seed=7)
    _, xl, ple = port.trace(G, ids, off)
    worst_cos, worst_abs = 1.0, 0.0
    try:
        port.set_variant(**variant)
        for l in range(24):
            c, a = _layer_errors(port.layer(G, l, xl[l], ple, off), xl[l + 1])
            worst_cos, worst_abs = min(worst_cos, c), max(worst_abs, a)
    finally:
        port.set_variant()
    return worst_cos, worst_abs


def test_requantization_floor_of_one_layer(port, syn):
    """The floor under any implementation in another float order: the
    restatement itself with only its GEMMs' block sums reversed (an fp32
    reordering like those between the reference's own x86 tiers) moves one
    layer's output, teacher-forced, by up to ~1.3e-3 on the L2-normalised rows
    -- a last-bit difference lands a few Q8_0 codes on the other side of a
    rounding boundary and the next GEMM carries it.  Cosine stays >= 0.99998.
    (tests/test_gpu_layers.py compares the fast path with this floor.)"""
    c, a = _teacher_forced_worst(port, syn, gemm_descending=True)
    print(f"reversed block order: worst layer cosine {c:.7f}, max |diff| {a:.2e}")
    assert c >= 0.99998
    assert 1e-3 < a < 2e-3  # above the north star's 1e-3: no other order can promise it per layer


def test_fp16_attention_operands_explain_fast_path_error(port, syn):
    """Rounding only q, k and v to fp16 before the attention (the fast path's
    tensor-core operands), everything else in the reference's order, moves one
    layer by ~3e-3 -- the fast path's measured per-layer error on the GPU
    (tests/test_gpu_layers.py), i.e. its excess over the reordering floor comes
    from its fp16 attention operands."""
    c, a = _teacher_forced_worst(port, syn, attention_fp16=True)
    print(f"fp16 q/k/v: worst layer cosine {c:.7f}, max |diff| {a:.2e}")
    assert c >= 0.9999
    assert 2.5e-3 < a < 4e-3
