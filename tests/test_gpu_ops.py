"""Operator parity on the GPU, through the C ABI (include/eg2_ops.h).

Part 1 ports the reference's operator test (tests/kernels.cpp:57-137): the
kernels/abi.h operators against CPU sums with its tolerances.  Part 2 checks
each fused executor operator against the CPU restatement of the reference
graph (oracle/eg2_oracle.c) on identical inputs: Q8 codes, scales and every
value the reference computes with exactly-rounded operations must match bit
for bit; tensor-core accumulations are compared within stated tolerances.
"""
import numpy as np
import pytest

from conftest import cosine

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ops(eg2):
    import importlib
    return importlib.import_module("embeddinggemma2-amdkfd_b200.ops")


def T(a, dtype=None):
    t = torch.from_numpy(np.array(a, copy=True))
    return t.to(DEV) if dtype is None else t.to(DEV, dtype)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f16_to_f32(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------------- Part 1
def test_abi_mm_types_and_sizes(ops):
    """tests/kernels.cpp:57-80: 4 weight types x n in {1,17,33,65}, k=64, m=35, 2e-5."""
    k, m = 64, 35
    for type_ in (0, 1, 8, 30):
        for n in (1, 17, 33, 65):
            x = ((np.arange(n * k) % 19) - 9).astype(np.float32) * np.float32(0.03125)
            w = ((np.arange(k * m) % 23) - 11).astype(np.float32) * np.float32(0.125)
            if type_ == 0:
                wb = w.view(np.uint8)
            elif type_ == 1:
                wb = w.astype(np.float16).view(np.uint8)
            elif type_ == 30:
                wb = (w.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
            else:
                blk = np.zeros((k * m // 32, 34), np.uint8)
                blk[:, 0], blk[:, 1] = 0, 0x30  # fp16 0.125
                z = np.arange(k * m).reshape(-1, 32)
                blk[:, 2:] = (((z % 23) - 11).astype(np.int8)).view(np.uint8)
                wb = blk.ravel()
            out = torch.zeros(n * m, device=DEV)
            ops.mm(out, T(x), T(wb), n, k, m, type_)
            ref = x.reshape(n, k).astype(np.float64) @ w.reshape(m, k).astype(np.float64).T
            np.testing.assert_allclose(host(out).reshape(n, m), ref, atol=2e-5, rtol=0)


def test_abi_norm(ops):
    """tests/kernels.cpp:81-91."""
    for d in (256, 512):
        w = (0.5 + (np.arange(d) % 7) * 0.1).astype(np.float32)
        x = np.sin(np.arange(3 * d, dtype=np.float32) * np.float32(0.13)).astype(np.float32)
        out = torch.zeros(3 * d, device=DEV)
        ops.norm(out, T(x), T(w), 3, d, 1.0)
        xr = x.reshape(3, d).astype(np.float64)
        ref = xr * w / np.sqrt((xr * xr).sum(1, keepdims=True) / d + 1e-6)
        np.testing.assert_allclose(host(out).reshape(3, d), ref, atol=2e-5, rtol=0)


def test_abi_fused_vs_unfused(ops):
    """tests/kernels.cpp:92-113: norm_residual == norm + element, norm_rope == norm + rope (2e-6)."""
    for d in (256, 512):
        w = (0.5 + (np.arange(d) % 7) * 0.1).astype(np.float32)
        i = np.arange(6 * d, dtype=np.float32)
        x = np.sin(i * np.float32(0.13)).astype(np.float32)
        res = np.cos(i * np.float32(0.17)).astype(np.float32)
        y, r1, r2 = torch.zeros(6 * d, device=DEV), T(res), T(res)
        ops.norm(y, T(x), T(w), 6, d, 1.0)
        ops.element(r1, r1, y, 6 * d, 0, 0, 0.7)
        ops.norm_residual(r2, T(x), T(w), 6, d, 0.7)
        np.testing.assert_allclose(host(r2), host(r1), atol=2e-6, rtol=0)
        table = np.zeros((3, d), np.float32)
        tz = np.outer(np.arange(3), np.arange(d // 2)).astype(np.float32) * np.float32(0.01)
        table[:, :d // 2], table[:, d // 2:] = np.cos(tz), np.sin(tz)
        y = torch.zeros(6 * d, device=DEV)
        xt = T(x)
        ops.norm(y, xt, T(w), 6, d, 1.0)
        ops.rope(y, T(table), 3, 2, d)
        ops.norm_rope(xt, T(w), T(table), 6, d, 2)
        np.testing.assert_allclose(host(xt), host(y), atol=2e-6, rtol=0)


def test_abi_attention(ops):
    """tests/kernels.cpp:114-137: GQA, two packed sequences, window 0/1 vs a double softmax."""
    bounds = np.array([[0, 3] if t < 3 else [3, 8] for t in range(8)], np.uint32).ravel()
    q = (np.sin(np.arange(8 * 2048, dtype=np.float32) * np.float32(0.07)) * np.float32(0.1)).astype(np.float32)
    k = (np.cos(np.arange(8 * 512, dtype=np.float32) * np.float32(0.11)) * np.float32(0.1)).astype(np.float32)
    v = np.sin(np.arange(8 * 512, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    for d in (256, 512):
        for window in (0, 1):
            out = torch.zeros(8 * 4 * d, device=DEV)
            ops.attention(out, T(q), T(k), T(v), T(bounds), 8, window, d)
            got = host(out)
            for t in range(8):
                for h in range(4):
                    lo, hi, kh = int(bounds[2 * t]), int(bounds[2 * t + 1]), h // (4 // (512 // d))
                    if window:
                        if t > window:
                            lo = max(lo, t - window)
                        hi = min(hi, t + window + 1)
                    qv = q[(t * 4 + h) * d:(t * 4 + h + 1) * d].astype(np.float64)
                    ks = np.stack([k[s * 512 + kh * d:s * 512 + kh * d + d] for s in range(lo, hi)]).astype(np.float64)
                    vs = np.stack([v[s * 512 + kh * d:s * 512 + kh * d + d] for s in range(lo, hi)]).astype(np.float64)
                    e = np.exp(ks @ qv)
                    ref = (e / e.sum()) @ vs
                    np.testing.assert_allclose(got[(t * 4 + h) * d:(t * 4 + h + 1) * d], ref, atol=2e-5, rtol=0)


# --------------------------------------------------------------------------- Part 2
def _rand_rows(rng, rows, width, scale=3.0):
    x = (rng.standard_normal((rows, width)) * rng.uniform(0.05, scale, (rows, 1))).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero block
    x[1, :32] = np.float32(0.5) * np.arange(32, dtype=np.float32)  # exact halves
    return x


def _check_q8(q_gpu, s_gpu, rows, width, stride, q_ref, d_ref):
    q_gpu = q_gpu.reshape(-1)[:rows * width].reshape(rows, width)
    np.testing.assert_array_equal(q_gpu, q_ref.reshape(rows, width))
    s = s_gpu.reshape(-1, stride)[: width // 32, :rows].T  # [rows][blocks]
    np.testing.assert_array_equal(s, f16_to_f32(d_ref).reshape(rows, width // 32))


TIERS = [0, 1]  # x86 tiers' quantizer/GELU (the fast path) and the scalar tier's (parity mode option)


def _round_mode(port, tier):
    return port.ROUND_SCALAR if tier else port.ROUND_X86


@pytest.mark.parametrize("tier", TIERS)
@pytest.mark.parametrize("width,weighted", [(512, True), (512, False), (1024, False), (2048, False)])
def test_norm_quant_bit_exact(ops, port, width, weighted, tier):
    rng = np.random.default_rng(width + weighted)
    rows, stride = 77, 96
    x = _rand_rows(rng, rows, width)
    w = (1.0 + 0.1 * rng.standard_normal(width)).astype(np.float32) if weighted else None
    ref = port.rms_rows(x, w) if weighted else x
    q_ref, d_ref = port.quantize(ref, _round_mode(port, tier))
    q = torch.zeros(rows * width, dtype=torch.int8, device=DEV)
    s = torch.zeros(width // 32 * stride, device=DEV)
    ops.norm_quant(q, s, stride, T(x), T(w) if weighted else None, rows, width, tier=tier)
    _check_q8(host(q), host(s), rows, width, stride, q_ref, d_ref)


def _q8_operands(rng, rows, k, pow2=False):
    q = rng.integers(-127, 128, size=(rows, k), dtype=np.int8)
    if pow2:
        d = np.float16(2.0) ** rng.integers(0, 3, size=(rows, k // 32)).astype(np.float16)
    else:
        d = (np.abs(rng.standard_normal((rows, k // 32))) * 0.01 + 1e-4).astype(np.float16)
    return q, d.view(np.uint16)


def _gpu_q8_mm(ops, xq, xd, wq, wd, stride, exact=False):
    n, k = xq.shape
    m = wq.shape[0]
    xs = np.zeros((k // 32, stride), np.float32)
    xs[:, :n] = f16_to_f32(xd).T
    ws = np.ascontiguousarray(f16_to_f32(wd).T)  # [k/32][m]
    out = torch.zeros(n * m, device=DEV)
    ops.q8_mm(out, T(xq), T(xs), stride, T(wq), T(ws), n, k, m, exact)
    return host(out).reshape(n, m)


SHAPES = [(130, 512, 2048), (2048, 512, 3072), (200, 1024, 512), (2048, 2048, 512),
          (77, 512, 768), (1, 512, 512), (257, 512, 4096), (2048, 512, 512)]


@pytest.mark.parametrize("n,k,m", SHAPES)
def test_q8_mm_exact_mode_bit_identical(ops, port, n, k, m):
    """exact=1 evaluates ((float)dot * dw) * dx and sum += in ascending block
    order like the reference's scalar tile (gemma2_fast.c:193-204), so the
    fp32 outputs are identical, not merely close."""
    rng = np.random.default_rng(n * 7 + k + m)
    xq, xd = _q8_operands(rng, n, k)
    wq, wd = _q8_operands(rng, m, k)
    got = _gpu_q8_mm(ops, xq, xd, wq, wd, ((n + 127) // 128) * 128, exact=True)
    np.testing.assert_array_equal(got, port.gemm_q8(wq, wd, xq, xd))


@pytest.mark.parametrize("n,k,m", SHAPES)
def test_q8_mm_fast_mode_within_tolerance(ops, port, n, k, m):
    """exact=0 fuses the last multiply-add: within 2e-6 of the output range."""
    rng = np.random.default_rng(n * 7 + k + m + 1)
    xq, xd = _q8_operands(rng, n, k)
    wq, wd = _q8_operands(rng, m, k)
    got = _gpu_q8_mm(ops, xq, xd, wq, wd, ((n + 127) // 128) * 128)
    ref = port.gemm_q8(wq, wd, xq, xd)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 2e-6, err


@pytest.mark.parametrize("n,k,m", [(150, 512, 2048), (64, 2048, 512), (300, 1024, 512)])
def test_q8_mm_int32_block_accumulators_exact(ops, port, n, k, m):
    """With power-of-two block scales every term and partial sum is an exact
    integer in fp32, so the output equals sum_b D_b * 2^e exactly: any error
    in an int32 block accumulator would show."""
    rng = np.random.default_rng(n + k + m)
    xq, xd = _q8_operands(rng, n, k, pow2=True)
    wq, wd = _q8_operands(rng, m, k, pow2=True)
    got = _gpu_q8_mm(ops, xq, xd, wq, wd, 512)
    got_exact = _gpu_q8_mm(ops, xq, xd, wq, wd, 512, exact=True)
    D = port.gemm_q8_blockdots(wq, xq).astype(np.int64)  # [n][m][kb]
    sc = (f16_to_f32(xd)[:, None, :] * f16_to_f32(wd)[None, :, :]).astype(np.int64)
    exact = (D * sc).sum(-1)
    assert np.abs(exact).max() < 2 ** 24
    np.testing.assert_array_equal(got.astype(np.int64), exact)
    np.testing.assert_array_equal(got_exact.astype(np.int64), exact)


@pytest.mark.parametrize("n,k,m,exact,tier", [(130, 512, 2048, False, 0), (2048, 512, 2048, False, 0),
                                              (77, 1024, 128, True, 1), (300, 512, 2048, True, 1)])
def test_q8_geglu_equals_unfused(ops, n, k, m, exact, tier):
    """The GeGLU GEMM (gate/up interleaved in 64-row chunks, gelu(gate) * up
    and Q8_0 in the epilogue) reproduces q8_mm(gate), q8_mm(up), gate_quant
    bit for bit."""
    rng = np.random.default_rng(n + k + m + exact)
    xq, xd = _q8_operands(rng, n, k)
    gq, gd = _q8_operands(rng, m, k)
    uq, ud = _q8_operands(rng, m, k)
    stride = (n + 127) // 128 * 128
    xs = np.zeros((k // 32, stride), np.float32)
    xs[:, :n] = f16_to_f32(xd).T
    # unfused reference path on the GPU
    gate = torch.from_numpy(_gpu_q8_mm(ops, xq, xd, gq, gd, stride, exact)).to(DEV)
    up = torch.from_numpy(_gpu_q8_mm(ops, xq, xd, uq, ud, stride, exact)).to(DEV)
    q_ref = torch.zeros(n * m, dtype=torch.int8, device=DEV)
    s_ref = torch.zeros(m // 32 * stride, device=DEV)
    ops.gate_quant(q_ref, s_ref, stride, gate.ravel(), up.ravel(), n, m, m, 0, tier=tier)
    # fused
    wq = np.zeros((2 * m, k), np.int8)
    wd = np.zeros((2 * m, k // 32), np.uint16)
    for c in range(m // 64):
        wq[128 * c:128 * c + 64], wd[128 * c:128 * c + 64] = gq[64 * c:64 * c + 64], gd[64 * c:64 * c + 64]
        wq[128 * c + 64:128 * c + 128], wd[128 * c + 64:128 * c + 128] = uq[64 * c:64 * c + 64], ud[64 * c:64 * c + 64]
    ws = np.ascontiguousarray(f16_to_f32(wd).T)
    q = torch.zeros(n * m, dtype=torch.int8, device=DEV)
    sc = torch.zeros(m // 32 * stride, device=DEV)
    ops.q8_geglu(q, sc, stride, T(xq), T(xs), stride, T(wq), T(ws), n, k, m, exact, tier=tier)
    np.testing.assert_array_equal(host(q), host(q_ref))
    np.testing.assert_array_equal(host(sc).reshape(-1, stride)[:, :n], host(s_ref).reshape(-1, stride)[:, :n])


@pytest.mark.parametrize("tier", TIERS)
@pytest.mark.parametrize("width,stride,offset", [(2048, 2048, 0), (512, 12288, 7 * 512)])
def test_gate_quant_bit_exact(ops, port, width, stride, offset, tier):
    """GELU-tanh gate then Q8_0; the scalar tier's GELU calls the C library's
    tanhf (restated exactly in csrc/ref_tanhf.h)."""
    rng = np.random.default_rng(width)
    rows = 65
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
    other = rng.standard_normal((rows, stride)).astype(np.float32)
    g = port.gelu_mul(x, other[:, offset:offset + width], mode=0 if tier else 1).reshape(rows, width)
    q_ref, d_ref = port.quantize(g, _round_mode(port, tier))
    qstride = 128
    q = torch.zeros(rows * width, dtype=torch.int8, device=DEV)
    s = torch.zeros(width // 32 * qstride, device=DEV)
    ops.gate_quant(q, s, qstride, T(x), T(other), rows, width, stride, offset, tier=tier)
    _check_q8(host(q), host(s), rows, width, qstride, q_ref, d_ref)


def _gelu_inputs(step):
    """Every step-th float bit pattern with |x| <= 6.5 (past it the GELU's inner
    argument is clamped), both signs, plus zeros, infinities, NaN, extremes."""
    mag = np.arange(0, 0x40D00001, step, dtype=np.uint32)
    x = np.concatenate([mag, mag | np.uint32(0x80000000)]).view(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e30, -1e30, 3.4e38, -3.4e38, 1e-45, -1e-45],
                       np.float32)
    x = np.concatenate([special, x])
    return x[: x.size - x.size % 8]


@pytest.mark.parametrize("tier,step", [(0, 61), (1, 4093)])
def test_gelu_mul_bit_exact(ops, port, tier, step):
    """GELU rows against the CPU restatement, bit for bit, over a dense sweep of
    the GELU's input range: tier 0 is the x86 rows' exp polynomial with IEEE
    division (here the branch-free division), tier 1 the tanhf form."""
    x = _gelu_inputs(step)
    u = np.random.default_rng(5).standard_normal(x.size).astype(np.float32)
    for uu in (u, None):
        ref = port.gelu_mul(x, uu, mode=0 if tier else 1)
        g = T(x)
        ops.gelu_mul(g, None if uu is None else T(uu), x.size, tier=tier)
        out = host(g)
        same = (out.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(out) & np.isnan(ref))
        assert same.all(), (x[~same][:8], out[~same][:8], ref[~same][:8])


def test_gelu_mul_rejects_partial_vector_on_x86_tier(ops):
    g = torch.zeros(12, device=DEV)
    with pytest.raises(RuntimeError):
        ops.gelu_mul(g, None, 12, tier=0)


def test_fdiv_markstein_equals_ieee_division(tmp_path):
    """The kernels' branch-free divisions equal IEEE division: the GELU's for
    every denominator it can produce, the PLE's division by sqrt(512) for every
    float, the Q8_0 quantizer's amax / 127 and 1 / d for every non-negative
    float (tests/cuda/fdiv_check.cu)."""
    import os
    import shutil
    import subprocess
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "fdiv_check")
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                    "-I", os.path.join(root, "embeddinggemma2-amdkfd_b200", "csrc"), "-o", exe,
                    os.path.join(root, "tests", "cuda", "fdiv_check.cu")], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.count(" 0 differ") == 4, r.stdout + r.stderr


@pytest.mark.parametrize("tier", TIERS)
@pytest.mark.parametrize("next_norm,scaled", [(True, False), (False, False), (True, True)])
def test_post_add_bit_exact(ops, port, next_norm, scaled, tier):
    rng = np.random.default_rng(3 + next_norm + 2 * scaled)
    rows, stride = 90, 128
    x = (rng.standard_normal((rows, 512)) * 2).astype(np.float32)
    h = (rng.standard_normal((rows, 512)) * 5).astype(np.float32)
    w = rng.normal(0, 0.1, 512).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    sc = np.array([0.73], np.float32)
    hn = port.rms_rows(h, w)
    x_ref = ((x + hn) * (sc[0] if scaled else np.float32(1.0))).astype(np.float32)
    nxt = port.rms_rows(x_ref, nw) if next_norm else x_ref
    q_ref, d_ref = port.quantize(nxt, _round_mode(port, tier))
    xt = T(x)
    q = torch.zeros(rows * 512, dtype=torch.int8, device=DEV)
    s = torch.zeros(16 * stride, device=DEV)
    ops.post_add(xt, T(h), T(w), T(sc) if scaled else None, q, s, stride, T(nw) if next_norm else None, rows,
                 tier=tier)
    np.testing.assert_array_equal(host(xt), x_ref)
    _check_q8(host(q), host(s), rows, 512, stride, q_ref, d_ref)


@pytest.mark.parametrize("d", [256, 512])
def test_qkv_post_bit_exact(ops, port, d):
    rng = np.random.default_rng(d)
    n, kv = 70, 512 // d
    qkv = (rng.standard_normal((n, 4 * d + 1024)) * 4).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    pos = rng.integers(0, 2048, n).astype(np.uint32)
    c, s = port.rope_tables(d)
    c, s = np.ascontiguousarray(c[:2048]), np.ascontiguousarray(s[:2048])

    def rope(r, p):
        a, b = r[:, : d // 2], r[:, d // 2:]
        cc, ss = c[p], s[p]
        return np.concatenate([a * cc - b * ss, a * ss + b * cc], 1).astype(np.float32)

    q_ref = np.stack([rope(port.rms_rows(qkv[:, h * d:(h + 1) * d], qn), pos) for h in range(4)], 1)
    k_ref = np.stack([rope(port.rms_rows(qkv[:, 4 * d + h * d:4 * d + (h + 1) * d], kn), pos) for h in range(kv)], 1)
    v_ref = np.stack([port.rms_rows(qkv[:, 4 * d + 512 + h * d:4 * d + 512 + (h + 1) * d], None) for h in range(kv)], 1)
    qo = torch.zeros(n * 4 * d, dtype=torch.float16, device=DEV)
    ko = torch.zeros(n * kv * d, dtype=torch.float16, device=DEV)
    vo = torch.zeros(n * kv * d, dtype=torch.float16, device=DEV)
    ops.qkv_post(qo, ko, vo, T(qkv), T(qn), T(kn), T(c), T(s), T(pos), n, d)
    np.testing.assert_array_equal(host(qo).reshape(q_ref.shape), q_ref.astype(np.float16))
    np.testing.assert_array_equal(host(ko).reshape(k_ref.shape), k_ref.astype(np.float16))
    np.testing.assert_array_equal(host(vo).reshape(v_ref.shape), v_ref.astype(np.float16))


def _bounds(lengths):
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    lo = np.concatenate([[off[i]] * lengths[i] for i in range(len(lengths))]).astype(np.uint32)
    hi = np.concatenate([[off[i + 1]] * lengths[i] for i in range(len(lengths))]).astype(np.uint32)
    return lo, hi


@pytest.mark.parametrize("d,window,lengths", [(256, 512, [10, 19, 35, 66]), (512, 0, [10, 19, 35, 66]),
                                              (256, 512, [1300, 3, 128]), (512, 0, [700, 129])])
def test_attention_f16_vs_reference_attention(ops, port, d, window, lengths):
    rng = np.random.default_rng(d + sum(lengths))
    n, kv = sum(lengths), 512 // d
    q = rng.standard_normal((n, 4, d)).astype(np.float16)
    k = (rng.standard_normal((n, kv, d)) * 0.1).astype(np.float16)
    v = rng.standard_normal((n, kv, d)).astype(np.float16)
    lo, hi = _bounds(lengths)
    ref = port.attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), lo, hi, kv, d, window)
    bounds = np.stack([lo, hi], 1).ravel()
    out = torch.zeros(n * 4 * d, device=DEV)
    ops.attention_f16(out, T(q), T(k), T(v), T(bounds), n, d, window)
    got = host(out).reshape(n, 4 * d)
    np.testing.assert_allclose(got, ref, atol=3e-3, rtol=0)
    assert cosine(got.ravel(), ref.ravel()) > 0.99999


def _attn_case(rng, lengths, kscale=0.1, d=256):
    n, kv = sum(lengths), 512 // d
    q = rng.standard_normal((n, 4, d)).astype(np.float16)
    k = (rng.standard_normal((n, kv, d)) * kscale * (256 / d) ** 0.5).astype(np.float16)
    v = rng.standard_normal((n, kv, d)).astype(np.float16)
    lo, hi = _bounds(lengths)
    return n, q, k, v, lo, hi


@pytest.mark.parametrize("d,window,lengths,kscale", [
    (256, 512, [10, 19, 35, 66], 0.1), (256, 512, [1300, 3, 128], 0.1), (256, 0, [700, 129], 0.1),
    (256, 512, [2048], 0.1), (256, 512, [1] * 5 + [64] * 20 + [63, 65, 127, 129], 0.1), (256, 0, [1500, 96], 0.1),
    # Scores of std ~16: nearly one-hot rows, frequent reference-maximum moves.
    (256, 512, [900, 77], 1.0),
    # Global layers: d = 512, one KV head, no window (and a window, for coverage).
    (512, 0, [10, 19, 35, 66], 0.1), (512, 0, [700, 129], 0.1), (512, 0, [2048], 0.1),
    (512, 0, [1] * 5 + [64] * 20 + [63, 65, 127, 129], 0.1), (512, 512, [1300, 3, 128], 0.1),
    (512, 0, [900, 77], 1.0)])
def test_attention_tc_vs_reference_attention(ops, port, d, window, lengths, kscale):
    """Tensor-core attention (fp16 P, fp32 TMEM accumulators) against the
    reference's fp32 attention_rows restated, same tolerance as attention_f16."""
    rng = np.random.default_rng(sum(lengths) + window + int(kscale * 10) + d)
    n, q, k, v, lo, hi = _attn_case(rng, lengths, kscale, d)
    ref = port.attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), lo, hi, 512 // d, d,
                         window)
    out = torch.full((n * 4 * d,), float("nan"), device=DEV)
    ops.attention_tc(out, T(q), T(k), T(v), T(np.stack([lo, hi], 1).ravel()), n, window, d)
    got = host(out).reshape(n, 4 * d)
    np.testing.assert_allclose(got, ref.reshape(n, 4 * d), atol=3e-3, rtol=0)
    assert cosine(got.ravel(), ref.ravel()) > 0.99999


@pytest.mark.parametrize("d,window", [(256, 512), (512, 0)])
def test_attention_tc_packed_equals_solo(ops, d, window):
    """A sequence's rows come out bit-identical wherever it sits in the packed
    wave: key blocks are aligned to each sequence's own start."""
    rng = np.random.default_rng(77)
    lengths = [37, 300, 129, 5, 700]
    n, q, k, v, lo, hi = _attn_case(rng, lengths, d=d)
    out = torch.zeros(n * 4 * d, device=DEV)
    ops.attention_tc(out, T(q), T(k), T(v), T(np.stack([lo, hi], 1).ravel()), n, window, d)
    packed = host(out).reshape(n, 4 * d)
    off = np.concatenate([[0], np.cumsum(lengths)])
    for i, L in enumerate(lengths):
        a, b = off[i], off[i + 1]
        slo, shi = _bounds([L])
        solo = torch.zeros(L * 4 * d, device=DEV)
        ops.attention_tc(solo, T(np.ascontiguousarray(q[a:b])), T(np.ascontiguousarray(k[a:b])),
                         T(np.ascontiguousarray(v[a:b])), T(np.stack([slo, shi], 1).ravel()), L, window, d)
        np.testing.assert_array_equal(host(solo).reshape(L, 4 * d), packed[a:b])


@pytest.mark.parametrize("tier", [0, 1])
@pytest.mark.parametrize("d,lengths", [(256, [128] * 16), (256, [1300, 3, 128, 37]), (512, [128] * 16),
                                       (512, [1300, 3, 128, 37])])
def test_attention_tc_q8_equals_row_quantizer(ops, d, lengths, tier):
    """The fused Q8_0 epilogue writes exactly the codes and scales the row
    quantizer (norm_quant, weight NULL) gives for the fp32 attention rows."""
    rng = np.random.default_rng(len(lengths) + tier + d)
    n, q, k, v, lo, hi = _attn_case(rng, lengths, d=d)
    window, w = (512 if d == 256 else 0), 4 * d
    b = T(np.stack([lo, hi], 1).ravel())
    qt, kt, vt = T(q), T(k), T(v)
    out = torch.zeros(n * w, device=DEV)
    ops.attention_tc(out, qt, kt, vt, b, n, window, d)
    stride = n + 5
    ref_q = torch.zeros(n * w, dtype=torch.int8, device=DEV)
    ref_s = torch.zeros(w // 32 * stride, device=DEV)
    ops.norm_quant(ref_q, ref_s, stride, out, None, n, w, tier=tier)
    got_q = torch.full((n * w,), 99, dtype=torch.int8, device=DEV)
    got_s = torch.zeros(w // 32 * stride, device=DEV)
    ops.attention_tc_q8(got_q, got_s, stride, qt, kt, vt, b, n, window, tier=tier, d=d)
    np.testing.assert_array_equal(host(got_q), host(ref_q))
    np.testing.assert_array_equal(host(got_s).reshape(w // 32, stride)[:, :n],
                                  host(ref_s).reshape(w // 32, stride)[:, :n])


def test_attention_tc_rejects_unsupported(ops):
    """d other than 256 / 512 and more than 8192 tokens are refused before any launch."""
    z = torch.zeros(16, device=DEV)
    with pytest.raises(RuntimeError):
        ops.attention_tc(z, z, z, z, z, 8193, 512)
    with pytest.raises(RuntimeError):
        ops.attention_tc(z, z, z, z, z, 10, 0, d=384)


@pytest.mark.parametrize("d,window,lengths", [(256, 512, [10, 700, 3]), (512, 0, [300, 64]), (256, 512, [1100])])
def test_attention_exact_bit_identical(ops, port, d, window, lengths):
    """Parity-mode attention: the reference's scalar loop order and the C
    library's expf rounding give outputs identical to the restatement."""
    rng = np.random.default_rng(d + sum(lengths) + 1)
    n, kv = sum(lengths), 512 // d
    q = (rng.standard_normal((n, 4, d)) * 0.3).astype(np.float32)
    k = (rng.standard_normal((n, kv, d)) * 0.3).astype(np.float32)
    v = rng.standard_normal((n, kv, d)).astype(np.float32)
    lo, hi = _bounds(lengths)
    ref = port.attention(q, k, v, lo, hi, kv, d, window)
    out = torch.zeros(n * 4 * d, device=DEV)
    ops.attention_exact(out, T(q), T(k), T(v), T(np.stack([lo, hi], 1).ravel()), n, d, window)
    np.testing.assert_array_equal(host(out).reshape(n, 4 * d), ref.reshape(n, 4 * d))


def test_embed_bit_exact(ops, model_baseline):
    import oracle
    g = oracle.Gguf(model_baseline)
    raw = np.asarray(g.raw("token_embd.weight"))
    rng = np.random.default_rng(1)
    ids = rng.integers(0, 262144, 300).astype(np.int32)
    blk = raw.reshape(262144, 16, 34)[ids]
    d = f16_to_f32(np.ascontiguousarray(blk[:, :, :2]).view(np.uint16)[..., 0])
    qv = np.ascontiguousarray(blk[:, :, 2:]).view(np.int8).astype(np.float32)
    ref = ((d[:, :, None] * qv) * np.float32(np.sqrt(np.float32(512)))).astype(np.float32).reshape(300, 512)
    x = torch.zeros(300 * 512, device=DEV)
    hi = torch.zeros(300 * 512, dtype=torch.bfloat16, device=DEV)
    lo = torch.zeros(300 * 512, dtype=torch.bfloat16, device=DEV)
    ops.embed(x, hi, lo, T(raw), T(ids), 300)
    np.testing.assert_array_equal(host(x).reshape(300, 512), ref)
    xr = torch.from_numpy(ref).to(DEV).ravel()
    assert torch.equal(hi, xr.to(torch.bfloat16))
    assert torch.equal(lo, (xr - xr.to(torch.bfloat16).float()).to(torch.bfloat16))


def test_ple_proj_vs_reference(ops, port, model_baseline):
    import oracle
    g = oracle.Gguf(model_baseline)
    rng = np.random.default_rng(2)
    n = 150
    x = rng.standard_normal((n, 512)).astype(np.float32)
    w_bits = np.asarray(g.raw("per_layer_model_proj.weight")).view(np.uint16).reshape(12288, 512)
    nw = np.array(g.f32("per_layer_proj_norm.weight"))
    ref = port.gemm_bf16(w_bits, x) / np.float32(np.sqrt(np.float32(512)))
    ref = port.rms_rows(ref.astype(np.float32).reshape(n * 24, 512), nw).reshape(n, 12288)
    xt = torch.from_numpy(x).to(DEV)
    hi = xt.to(torch.bfloat16)
    lo = (xt - hi.float()).to(torch.bfloat16)
    ple = torch.zeros(n * 12288, device=DEV)
    ops.ple_proj(ple, hi, lo, T(w_bits), T(nw), n)
    got = host(ple).reshape(n, 12288)
    np.testing.assert_allclose(got, ref, atol=5e-4, rtol=2e-4)


def _sum_squares_sse2(row):
    """kernels.c:35-39,82-93 order: two 4-lane float accumulators over
    8-element chunks, then (v0 + v2) + (v1 + v3), then a scalar tail."""
    sq = (row * row).astype(np.float32)
    n8 = sq.size // 8 * 8
    s0 = np.zeros(4, np.float32)
    s1 = np.zeros(4, np.float32)
    for c in range(0, n8, 8):
        s0 = (s0 + sq[c:c + 4]).astype(np.float32)
        s1 = (s1 + sq[c + 4:c + 8]).astype(np.float32)
    v = (s0 + s1).astype(np.float32)
    ss = np.float32(np.float32(v[0] + v[2]) + np.float32(v[1] + v[3]))
    for z in range(n8, sq.size):
        ss = np.float32(ss + sq[z])
    return ss


def _pool_l2_ref(y, off):
    sumsq = _sum_squares_sse2
    out = []
    for s in range(len(off) - 1):
        lo, hi = int(off[s]), int(off[s + 1])
        o = np.zeros(y.shape[1], np.float32)
        ln = np.float32(hi - lo)
        for t in range(lo, hi):
            o = (o + (y[t] / ln).astype(np.float32)).astype(np.float32)
        ss = sumsq(o)
        out.append((o * np.float32(np.float32(1) / np.sqrt(ss, dtype=np.float32))).astype(np.float32))
    return np.stack(out)


def test_pool_l2_bit_exact(ops):
    rng = np.random.default_rng(4)
    lengths = [10, 19, 35, 66, 1]
    off = np.concatenate([[0], np.cumsum(lengths)]).astype(np.uint32)
    y = rng.standard_normal((off[-1], 768)).astype(np.float32)
    out = torch.zeros(len(lengths) * 768, device=DEV)
    ops.pool_l2(out, T(y), T(off), len(lengths), 768)
    np.testing.assert_array_equal(host(out).reshape(len(lengths), 768), _pool_l2_ref(y, off))


def test_repack_q8(ops, model_baseline):
    import oracle
    g = oracle.Gguf(model_baseline)
    raw = np.asarray(g.raw("blk.3.ffn_down.weight"))
    q_ref, d_ref = g.q8("blk.3.ffn_down.weight")
    codes = torch.zeros(512 * 2048, dtype=torch.int8, device=DEV)
    scales = torch.zeros(64 * 512, device=DEV)
    ops.repack_q8(T(raw), 512, 2048, codes, scales)
    np.testing.assert_array_equal(host(codes).reshape(512, 2048), q_ref)
    np.testing.assert_array_equal(host(scales).reshape(64, 512).T, f16_to_f32(d_ref))
    assert ops.read_error() == 0
