"""The allocation-free attention entry point (ndl_attention_paged_noalloc).

It serves hosts that must not allocate while handling a request, such as a
frame-budgeted game or job thread or a zero-allocation serving loop, where a
cudaMalloc could block or synchronise the device.  Its partials live in a
fixed device array owned by the library instead of a workspace.

Checked through the C ABI against the regular entry point
(ndl_attention_paged) on the same inputs, for two calls in a row (the second
call reuses the array the first one left dirty), within the attention
tolerance the other tests use (5e-5 x peak |output|).  Collected last so a
failure here cannot hide the rest of the suite; it also passes on its own.
"""
import numpy as np
import pytest
import torch

from attention_support import make_case

pytestmark = pytest.mark.gpu

LENGTHS = [1, 64, 65, 300, 513, 1024, 1088, 7]


def _args(case, cuda):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    return dict(q=t(case["q_perm"]), qs=t(case["QS"]), row_slot=t(case["row_slot"]), row_pos=t(case["row_pos"]),
                page_table=t(case["page_table"]), pool=t(case["pool"]))


def _call(name, d, case, out, status, extra=()):
    from needle_cs_b200._native import call

    rows, heads = case["q_perm"].shape[:2]
    slots, max_pages = case["page_table"].shape
    call(name, d["q"].data_ptr(), d["qs"].data_ptr(), d["row_slot"].data_ptr(), d["row_pos"].data_ptr(), rows,
         heads, d["page_table"].data_ptr(), slots, max_pages, d["pool"].data_ptr(), case["page_bytes"],
         d["pool"].numel() // case["page_bytes"], case["layer"], out.data_ptr(), *extra, status.data_ptr(),
         torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_regular_entry_point_twice(pkg, cuda):
    case = make_case(29, LENGTHS, 8)
    d = _args(case, cuda)
    rows, heads = case["q_perm"].shape[:2]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    ref = torch.empty((rows, heads, 64), dtype=torch.float32, device=cuda)
    _call("ndl_attention_paged", d, case, ref, status, extra=(None, 0))
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for _ in range(2):
        out = torch.full((rows, heads, 64), float("nan"), dtype=torch.float32, device=cuda)
        _call("ndl_attention_paged_noalloc", d, case, out, status)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert status.item() == 0
        for r in range(rows):
            peak = np.abs(ref[r]).max()
            assert np.all(np.abs(got[r] - ref[r]) <= 5e-5 * peak), LENGTHS[r]


def test_noalloc_rejects_requests_beyond_its_buffer(pkg, cuda):
    from needle_cs_b200 import NeedleError

    case = make_case(3, [10, 20], 8)
    d = _args(case, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty((2, 8, 64), dtype=torch.float32, device=cuda)
    from needle_cs_b200._native import call

    # 4 MiB holds at most 15420 (row, head, chunk) partials of 272 bytes; the
    # request is refused on the host before any device memory is touched
    with pytest.raises(NeedleError) as e:
        call("ndl_attention_paged_noalloc", d["q"].data_ptr(), d["qs"].data_ptr(), d["row_slot"].data_ptr(),
             d["row_pos"].data_ptr(), 4096, 8, d["page_table"].data_ptr(), 2, 17, d["pool"].data_ptr(),
             case["page_bytes"], d["pool"].numel() // case["page_bytes"], case["layer"], out.data_ptr(),
             status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert e.value.status == 100
    assert "scratch" in str(e.value)
