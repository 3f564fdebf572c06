"""The library's float exponential (Ops.Exp, used by the attention softmax
and the SiLU gate) against the oracle's restatement of it."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_exp_equals_oracle_exp(pkg, oracle, cuda):
    """The exponential of the attention softmax and the SiLU gate: the
    device's Ops.Exp returns the oracle's bits on every input (the same IEEE
    steps on both sides), which keeps decoder logits bit-comparable through
    12 layers."""
    import torch

    from needle_cs_b200._native import call

    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-110.0, 95.0, 2_000_000), rng.uniform(-20.0, 0.0, 2_000_000),
                        rng.normal(0.0, 4.0, 1_000_000),
                        [np.nan, np.inf, -np.inf, 0.0, -0.0, 88.72, 89.0, -103.97, -104.0]]).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda)
    yd = torch.empty_like(xd)
    call("ndl_selftest_exp", xd.data_ptr(), x.size, yd.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = yd.cpu().numpy()
    ref = oracle.exp_simd(x)
    same = (got.view(np.int32) == ref.view(np.int32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all(), (x[~same][:5], got[~same][:5], ref[~same][:5])
