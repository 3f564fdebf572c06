"""Standalone paged decode attention (ndl_attention_paged) against the
oracle: bit-identical to its restatement of the reference's AVX2 attention
tier (Attention.GroupAvx2: scores, max, Ops.Exp, the four-way partial sums,
1 / total, fma accumulation of e * vs * v in position order, the final
scale).  The oracle keeps that tier within the reference's own tier-to-tier
bar of Scalar.AttentionHead, 3e-5 x peak |output|
(tests/Needle.Tests/KernelTests.cs:231-236; tests/test_exp_oracle.py).
"""
import numpy as np
import pytest
import torch

from attention_support import make_case, oracle_out

pytestmark = pytest.mark.gpu

LENGTHS = [1, 2, 63, 64, 65, 130, 511, 512, 513, 777, 1024, 1088]


def _run(ops, cuda, case, workspace=None):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.attention_paged(t(case["q_perm"]), t(case["QS"]), t(case["row_slot"]), t(case["row_pos"]),
                              t(case["page_table"]), t(case["pool"]), case["page_bytes"], case["layer"],
                              workspace=workspace, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("heads", [8, 2])
def test_paged_attention_matches_oracle(ops, oracle, cuda, heads):
    case = make_case(11 + heads, LENGTHS, heads)
    got = _run(ops, cuda, case)
    ref = oracle_out(oracle, case, LENGTHS)
    for r in range(len(LENGTHS)):
        assert np.array_equal(got[r], ref[r]), (LENGTHS[r], np.abs(got[r] - ref[r]).max() / np.abs(ref[r]).max())


def test_paged_attention_caller_workspace(ops, cuda):
    case = make_case(5, LENGTHS, 8)
    need = ops.attention_paged_workspace(len(LENGTHS), 8, 17)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    a = _run(ops, cuda, case)
    b = _run(ops, cuda, case, workspace=ws)
    assert np.array_equal(a, b)


def test_paged_attention_flags_bad_rows(ops, cuda):
    case = make_case(6, [10, 20], 2)
    case["row_pos"] = np.array([9, 17 * 64 + 5], np.int32)  # second row longer than the page table
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.attention_paged(t(case["q_perm"]), t(case["QS"]), t(case["row_slot"]), t(case["row_pos"]),
                        t(case["page_table"]), t(case["pool"]), case["page_bytes"], case["layer"], status=status)
    torch.cuda.synchronize()
    assert status.item() == 2


def test_paged_attention_on_a_second_device(ops, oracle, cuda):
    """One process driving two GPUs: the kernel's shared-memory attribute and
    the SM count are set up per device, so a call on device 1 after device 0
    launches with the same result."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    lengths = [40, 700, 1024]
    case = make_case(21, lengths, 8)
    ref = oracle_out(oracle, case, lengths)
    first = _run(ops, cuda, case)
    second_dev = torch.device("cuda:1")
    with torch.cuda.device(second_dev):
        second = _run(ops, second_dev, case)
    assert np.array_equal(first, second)
    assert np.array_equal(second, ref)
