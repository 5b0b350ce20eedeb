"""The drop-in link, on the GPU: the reference's own engine (engine.c compiled
unchanged with -DEI_ENABLE_KFD=1 against include/, oracle/_ref/
libeg2enginelink.so) loads the seeded model with --backend kfd and serves
packed waves through ei_engine_embed_tokens_batch (engine.c:1021-1048), which
reaches ei_gemma2_kfd_batch in libeg2_b200.so.  Its embeddings must equal the
executor's own, bit for bit.  The engine runs in a child process: on a load
failure it exits the process (ei_die)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys, importlib
import numpy as np
sys.path.insert(0, {root!r}); sys.path.insert(0, {oracle!r})
import oracle
syn = importlib.import_module("embeddinggemma2-amdkfd_b200.synthetic")
link = oracle.EngineLink(syn.model_path(1234, "baseline", tokenizer=True))
res = {{"backend": link.backend}}
for i, lens in enumerate([(40, 7, 300, 126), (2046,), (9,)]):
    ids, off = syn.wave(lens, seed=12 + i)
    np.save({out!r} + f"/engine{{i}}.npy", link.embed(ids, off))
try:
    ids, off = syn.wave((1000, 1047), seed=20)
    link.embed(ids, off)
    res["over_limit"] = "accepted"
except RuntimeError as e:
    res["over_limit"] = str(e)
link.close()
json.dump(res, open({out!r} + "/engine.json", "w"))
"""


def test_reference_engine_serves_waves_through_the_executor(eg2, syn, tmp_path):
    import oracle
    if not os.path.exists(oracle.ENGINE_LINK_SO):
        pytest.skip("oracle/_ref/libeg2enginelink.so not built (make -C oracle engine_link)")
    code = CHILD.format(root=ROOT, oracle=os.path.join(ROOT, "oracle"), out=str(tmp_path))
    subprocess.run([sys.executable, "-c", code], check=True, timeout=600)
    res = json.load(open(tmp_path / "engine.json"))
    assert res["backend"] == "kfd"
    # 2049 packed tokens: the executor's message, passed through by the engine
    assert "1..2048 packed tokens" in res["over_limit"], res
    m = eg2.GGUFModel(syn.model_path(1234, "baseline"))  # same tensors, no tokenizer section
    ex = eg2.Gemma2Executor(m, 0)
    try:
        for i, lens in enumerate([(40, 7, 300, 126), (2046,), (9,)]):
            ids, off = syn.wave(lens, seed=12 + i)
            np.testing.assert_array_equal(np.load(tmp_path / f"engine{i}.npy"), ex.batch(ids, off))
    finally:
        ex.close()
        m.close()
