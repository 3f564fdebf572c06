"""Failure detection without a GPU fault.

Every kernel wait in the library is bounded: after a limited number of
suspend-hinted mbarrier tests it records a timeout status and returns, and
the host reports NDL_ERR_TIMEOUT (103).  ndl_selftest_bounded_wait runs that
path on a phase that nothing completes; afterwards the context must still
compute correctly.  Host-side failures (context exhaustion) must leave the
engine unchanged and usable."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(pkg, cuda, ops, oracle):
    from needle_cs_b200._native import lib
    import torch

    assert lib().ndl_selftest_bounded_wait(2000) == 103
    assert "gave up" in lib().ndl_last_error().decode()
    # the device still works: a quantized linear stays bit-exact
    x = ops.synth_normal_f32(5, 9, 4 * 256).reshape(4, 256)
    w = ops.synth_int8(5, 10, 64 * 256).reshape(64, 256)
    sw = ops.synth_uniform_f16(5, 11, 64 * 8, 0.001, 0.02).reshape(64, 8)
    q, s = oracle.quantize_rows(x)
    y = ops.matmul_i8g32(torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda), torch.from_numpy(w).to(cuda),
                         torch.from_numpy(sw.view(np.int16)).to(cuda))
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), oracle.matmul_i8g32(q, s, w, sw))


def test_engine_reports_context_exhaustion_without_side_effects(pkg, cuda):
    from needle_cs_b200 import NeedleError
    from needle_cs_b200.engine import BatchedEngine, SyntheticDecoder

    eng = BatchedEngine(SyntheticDecoder(layers=1, seed=2), slots=2, context_length=64, chunk_size=64)
    eng.forward_batch(list(range(60)), [0] * 60, [59])
    with pytest.raises(NeedleError) as e:
        eng.forward_batch(list(range(8)), [0] * 8, [7])
    assert e.value.status == 3
    assert eng.slot_length(0) == 60  # the failed step changed nothing
    eng.forward_batch([1, 2], [0, 1], [0, 1])  # and the engine keeps working
    assert eng.slot_length(0) == 61 and eng.slot_length(1) == 1
    eng.close()

