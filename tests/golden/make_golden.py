"""Regenerate the committed golden fixtures from the reference's OWN CPU graph.

Runs where the reference tree exists ($REF_ROOT, or `reference` beside this
repository's root):

    make -C oracle ref port
    python tests/golden/make_golden.py

The reference's published goldens (vendor/embeddinggemma.c/testdata/
gemma2-goldens.json) need the real GGUF, which is not available offline, so the
fixtures pin the reference compiled from its own sources
(oracle/_ref/libeg2ref.so) on the seeded synthetic models of
embeddinggemma2-amdkfd_b200/synthetic.py:

* golden_<norm>.npz -- config-0 wave (4 sequences, bodies 8/17/33/64 + BOS/EOS)
  through ei_gemma2_embed_batch_fast_ctx at the scalar tier
  (EI_GEMMA2_CPU_X86=scalar, tier independent) and at the host's best x86 tier,
  plus the reference graph (ei_gemma2_embed) per sequence;
* golden_long_baseline.npz -- config 2 (1 x 2048) and a 2 x 128 wave at the best
  tier, and the Matryoshka prefixes {128, 256, 512} of config 2 as the server
  applies them (kernels.c:403-407);
* golden_ops.npz -- the reference's x86 Q8_0 quantizer and exp-polynomial GELU
  on seeded random rows (gemma2_fast_x86.c:211-234, 308-325);
* golden_inputs_baseline.npz -- a 3-sequence wave (5/12/23 rows) given as
  512-wide input rows (media soft tokens, ids NULL: gemma2_fast.c:940-941),
  seeded N(0, 1), at the scalar and the best tier
  (`python tests/golden/make_golden.py inputs` writes only this one);
* golden_wide_baseline.npz -- one 8192-token sequence (the CPU graph's wave
  limit, gemma2_fast.c:924) at the best tier
  (`python tests/golden/make_golden.py wide` writes only this one);
* golden_short_baseline.npz -- waves of 8, 7, 3 and 9 tokens at the best tier:
  on an AVX-512 VNNI host, waves of at most 8 tokens take the 4-row Q8 tile
  and longer ones the repacked 512-bit GEMM, two float orders
  (`python tests/golden/make_golden.py short` writes only this one).

Each scalar-tier run happens in a child process because the reference caches
its tier on first use.
"""
from __future__ import annotations

import hashlib
import importlib
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
OUT = os.path.dirname(os.path.abspath(__file__))
SEED = 1234
SHORT_WAVES = ((6,), (2, 1), (1,), (7,))  # 8, 7, 3 and 9 tokens with BOS/EOS


def _child(norm: str, what: str, out_path: str):
    import oracle as O
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    path = syn.model_path(SEED, norm)
    ref = O.RefGraph(path, 0)
    res = {"tier": np.array(ref.tier)}
    if what == "cfg0":
        ids, off = syn.wave(syn.CONFIG0_BODIES)
        res["ids"], res["offsets"] = ids, off
        res["embed"] = ref.embed(ids, off)
        res["embed_reference_graph"] = np.stack(
            [ref.embed_reference_graph(ids[off[s]:off[s + 1]]) for s in range(len(off) - 1)])
    elif what == "long":
        ids, off = syn.wave(syn.CONFIG2_BODIES, seed=21)
        res["long_ids"], res["long_offsets"] = ids, off
        e = ref.embed(ids, off)
        res["long_embed"] = e
        for dims in (128, 256, 512):
            res[f"long_prefix_{dims}"] = ref.normalize_prefix(e[0], dims)
        ids, off = syn.wave((126, 126), seed=22)
        res["w2x128_ids"], res["w2x128_offsets"] = ids, off
        res["w2x128_embed"] = ref.embed(ids, off)
    elif what == "inputs":
        rng = np.random.Generator(np.random.PCG64(31))
        off = np.array([0, 5, 17, 40], np.uint64)
        x = rng.standard_normal((40, 512)).astype(np.float32)
        res["inputs"], res["offsets"] = x, off
        res["embed"] = ref.embed_inputs(x, off)
    elif what == "short":
        # waves of at most 8 tokens take the reference's 4-row Q8 tile, longer
        # ones the repacked 512-bit GEMM (gemma2_fast.c:446-449)
        for i, lens in enumerate(SHORT_WAVES):
            ids, off = syn.wave(lens, seed=40 + i)
            res[f"ids{i}"], res[f"offsets{i}"], res[f"embed{i}"] = ids, off, ref.embed(ids, off)
    elif what == "wide":
        ids, off = syn.wave((8190,), seed=24)
        res["ids"], res["offsets"] = ids, off
        res["embed"] = ref.embed(ids, off)
    elif what == "ops":
        rng = np.random.Generator(np.random.PCG64(5))
        x = (rng.standard_normal(64 * 512) * rng.uniform(0.01, 10.0, 64 * 512)).astype(np.float32)
        x[:32] = 0.0  # an all-zero block
        x[32:64] = np.float32(0.5) * np.arange(32, dtype=np.float32)  # exact halves
        q, d = ref.quantize_x86(x)
        g = (rng.standard_normal(8 * 2048) * 3).astype(np.float32)
        u = rng.standard_normal(8 * 2048).astype(np.float32)
        res.update(q_in=x, q_codes=q, q_scales=d, gelu_g=g, gelu_u=u, gelu_out=ref.gelu_mul(g, u))
    np.savez(out_path, **res)


def run(norm, what, scalar):
    tmp = os.path.join(OUT, f".tmp_{norm}_{what}_{int(scalar)}.npz")
    env = dict(os.environ)
    if scalar:
        env["EI_GEMMA2_CPU_X86"] = "scalar"
    subprocess.run([sys.executable, __file__, "--child", norm, what, tmp], check=True, env=env)
    d = dict(np.load(tmp))
    os.remove(tmp)
    return d


def make_inputs():
    s = run("baseline", "inputs", True)
    b = run("baseline", "inputs", False)
    np.savez_compressed(os.path.join(OUT, "golden_inputs_baseline.npz"), inputs=s["inputs"], offsets=s["offsets"],
                        embed_scalar=s["embed"], embed_best=b["embed"], best_tier=b["tier"])


def make_short():
    b = run("baseline", "short", False)
    np.savez_compressed(os.path.join(OUT, "golden_short_baseline.npz"), best_tier=b.pop("tier"), **b)


def make_wide():
    b = run("baseline", "wide", False)
    np.savez_compressed(os.path.join(OUT, "golden_wide_baseline.npz"), ids=b["ids"], offsets=b["offsets"],
                        embed_best=b["embed"], best_tier=b["tier"])


def main():
    syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
    meta = {}
    for norm in ("baseline", "plus1"):
        path = syn.model_path(SEED, norm)
        sha = hashlib.sha256(open(path, "rb").read()).hexdigest()
        s = run(norm, "cfg0", True)
        b = run(norm, "cfg0", False)
        np.savez_compressed(os.path.join(OUT, f"golden_{norm}.npz"), ids=s["ids"], offsets=s["offsets"],
                            embed_scalar=s["embed"], embed_best=b["embed"], best_tier=b["tier"],
                            embed_reference_graph=s["embed_reference_graph"])
        meta[norm] = {"seed": SEED, "gguf_sha256": sha, "best_tier": str(b["tier"])}
    lg = run("baseline", "long", False)
    np.savez_compressed(os.path.join(OUT, "golden_long_baseline.npz"), **lg)
    ops = run("baseline", "ops", False)
    np.savez_compressed(os.path.join(OUT, "golden_ops.npz"), **ops)
    make_inputs()
    make_wide()
    make_short()
    with open(os.path.join(OUT, "golden_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(json.dumps(meta, indent=1))


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "--child":
        _child(sys.argv[2], sys.argv[3], sys.argv[4])
    elif len(sys.argv) > 1 and sys.argv[1] == "inputs":
        make_inputs()
    elif len(sys.argv) > 1 and sys.argv[1] == "wide":
        make_wide()
    elif len(sys.argv) > 1 and sys.argv[1] == "short":
        make_short()
    else:
        main()
