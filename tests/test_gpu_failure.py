"""Failure detection on the GPU without a fault (the reference's contract:
gemma2_kfd.cpp:190-214,270 -- a failed wait poisons the context, every later
call fails with "restart process before reuse").  The failure is a bounded wait
that nothing completes: the kernel records the error word after about 2 s and
returns, so the GPU stays usable."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(eg2):
    import importlib
    return importlib.import_module("embeddinggemma2-amdkfd_b200.ops")


def test_timed_out_wait_sets_error_word_and_device_stays_usable(ops):
    ops.clear_error()
    try:
        ops.selftest_wait_timeout()
        torch.cuda.synchronize()
        assert ops.read_error() == 1
    finally:
        ops.clear_error()
    assert ops.read_error() == 0
    # The device still computes: a weighted row norm + Q8_0 against numpy.
    x = torch.arange(2 * 512, dtype=torch.float32, device="cuda:0").reshape(2, 512) / 512.0
    q = torch.zeros(2 * 512, dtype=torch.int8, device="cuda:0")
    s = torch.zeros(16 * 2, device="cuda:0")
    ops.norm_quant(q, s, 2, x.ravel(), None, 2, 512)
    torch.cuda.synchronize()
    xs = x.cpu().numpy().reshape(2, 16, 32)
    amax = np.abs(xs).max(-1)
    codes = q.cpu().numpy().reshape(2, 16, 32).astype(np.int32)
    assert np.abs(codes).max() == 127
    assert np.all(np.abs(codes * (amax[..., None] / 127.0) - xs) <= amax[..., None] / 127.0)


def test_wave_after_timed_out_wait_fails_and_poisons_context(eg2, syn, model_baseline, ops):
    model = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(model, 0)
    ids, off = syn.wave((40, 9), seed=5)
    good = ex.batch(ids, off)
    ops.clear_error()
    try:
        ops.selftest_wait_timeout(ex.stream)  # ahead of the next wave on the executor's stream
        with pytest.raises(eg2.ExecutorError, match="timed out"):
            ex.batch(ids, off)
        with pytest.raises(eg2.ExecutorError, match="restart process before reuse"):
            ex.batch(ids, off)
    finally:
        ops.clear_error()
        ex.close()
    # A new context on the same GPU works and agrees with the first result.
    ex2 = eg2.Gemma2Executor(model, 0)
    try:
        np.testing.assert_array_equal(ex2.batch(ids, off), good)
    finally:
        ex2.close()
        model.close()


def test_poison_is_sticky_across_pipeline_slots(eg2, syn, model_baseline, ops):
    """Two waves in flight; the first fails.  Even with the device word reset
    in between, the second slot's collect and every later call report the
    poisoned context (gemma2_kfd.cpp:190-214,270): a later successful wait
    must not clear the poison."""
    model = eg2.GGUFModel(model_baseline)
    ex = eg2.Gemma2Executor(model, 0)
    ids, off = syn.wave((40, 9), seed=5)
    ex.batch(ids, off)
    ops.clear_error()
    try:
        ops.selftest_wait_timeout(ex.stream)
        a = ex.submit(ids, off)
        b = ex.submit(ids, off)
        with pytest.raises(eg2.ExecutorError, match="timed out"):
            ex.collect(a)
        ops.clear_error()
        with pytest.raises(eg2.ExecutorError, match="restart process before reuse"):
            ex.collect(b)
        with pytest.raises(eg2.ExecutorError, match="restart process before reuse"):
            ex.submit(ids, off)
        with pytest.raises(eg2.ExecutorError, match="restart process before reuse"):
            ex.batch(ids, off)
    finally:
        torch.cuda.synchronize()
        ops.clear_error()
        ex.close()
        model.close()
