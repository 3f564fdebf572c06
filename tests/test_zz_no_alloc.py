"""The allocation-free attention entry point (ndl_attention_paged_noalloc).

It serves hosts that must not allocate while handling a request, such as a
frame-budgeted game or job thread or a zero-allocation serving loop, where a
cudaMalloc could block or synchronise the device.  Its work list lives in a
fixed 4 MiB device array owned by the library instead of a workspace.

Checked through the C ABI against the regular entry point
(ndl_attention_paged) on the same inputs, for several calls in a row (each
call reuses the array the previous one left dirty), and against the CPU
oracle: bit-identical, as the attention tests require.  The size limit is
pinned at its edge.  Collected last so a failure here cannot hide the rest
of the suite; it also passes on its own.
"""
import numpy as np
import pytest
import torch

from attention_support import make_case, oracle_out

pytestmark = pytest.mark.gpu

LENGTHS = [1, 64, 65, 300, 513, 1024, 1088, 7]
SCRATCH_BYTES = 4 << 20


def _args(case, cuda):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    return dict(q=t(case["q_perm"]), qs=t(case["QS"]), row_slot=t(case["row_slot"]), row_pos=t(case["row_pos"]),
                page_table=t(case["page_table"]), pool=t(case["pool"]))


def _call(name, d, case, out, status, extra=()):
    from needle_cs_b200._native import call

    rows, heads = d["q"].shape[:2]
    slots, max_pages = d["page_table"].shape
    call(name, d["q"].data_ptr(), d["qs"].data_ptr(), d["row_slot"].data_ptr(), d["row_pos"].data_ptr(), rows,
         heads, d["page_table"].data_ptr(), slots, max_pages, d["pool"].data_ptr(), case["page_bytes"],
         d["pool"].numel() // case["page_bytes"], case["layer"], out.data_ptr(), *extra, status.data_ptr(),
         torch.cuda.current_stream().cuda_stream)


def _regular(d, case, cuda):
    rows, heads = d["q"].shape[:2]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    ref = torch.empty((rows, heads, 64), dtype=torch.float32, device=cuda)
    _call("ndl_attention_paged", d, case, ref, status, extra=(None, 0))
    torch.cuda.synchronize()
    assert status.item() == 0
    return ref.cpu().numpy()


def _noalloc(d, case, cuda):
    rows, heads = d["q"].shape[:2]
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.full((rows, heads, 64), 12345.0, dtype=torch.float32, device=cuda)
    _call("ndl_attention_paged_noalloc", d, case, out, status)
    torch.cuda.synchronize()
    return out.cpu().numpy(), status.item()


def test_noalloc_matches_regular_entry_point_twice(pkg, oracle, cuda):
    case = make_case(29, LENGTHS, 8)
    d = _args(case, cuda)
    ref = _regular(d, case, cuda)
    assert np.array_equal(ref, oracle_out(oracle, case, LENGTHS))
    free = []
    for _ in range(3):
        got, st = _noalloc(d, case, cuda)
        assert st == 0
        assert np.array_equal(got, ref)
        free.append(torch.cuda.mem_get_info()[0])
    # after the first call (which may load the library's module on this
    # device) the calls leave the device's free memory unchanged
    assert free[1] == free[2]


def test_noalloc_bad_page_gives_nan_not_the_last_result(pkg, cuda):
    """The array keeps the previous call's work records.  A row with a page
    outside the pool must not come out with the previous call's result: its
    heads are NaN with status 2, and the other rows are unaffected."""
    case = make_case(31, LENGTHS, 8)
    d = _args(case, cuda)
    first, st = _noalloc(d, case, cuda)
    assert st == 0
    bad_row = LENGTHS.index(1024)  # 16 pages; page 9 goes out of range
    pt = case["page_table"].copy()
    pt[bad_row, 9] = d["pool"].numel() // case["page_bytes"] + 5
    d["page_table"] = torch.from_numpy(pt).to(cuda)
    got, st = _noalloc(d, case, cuda)
    assert st == 2
    assert np.all(np.isnan(got[bad_row]))
    others = [r for r in range(len(LENGTHS)) if r != bad_row]
    assert np.array_equal(got[others], first[others])
    # a row with an out-of-range slot is skipped and NaN as well
    rs = case["row_slot"].copy()
    rs[0] = 1000
    d["page_table"] = torch.from_numpy(case["page_table"]).to(cuda)
    d["row_slot"] = torch.from_numpy(rs).to(cuda)
    got, st = _noalloc(d, case, cuda)
    assert st == 2
    assert np.all(np.isnan(got[0]))
    assert np.array_equal(got[1:], first[1:])


def _max_items(ops, heads, max_pages):
    """Largest row count whose workspace fits the 4 MiB array."""
    lo, hi = 1, 1 << 20
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if ops.attention_paged_workspace(mid, heads, max_pages) <= SCRATCH_BYTES:
            lo = mid
        else:
            hi = mid - 1
    return lo


def test_noalloc_limit_at_its_edge(pkg, ops, cuda):
    """Each row takes a work record of 16 bytes plus 4 per page-table column
    (rounded up to 16), and the counters 16 bytes more: with a one-page
    table 4 MiB holds 131071 rows.  That many run and equal the regular entry
    point; one more is refused on the host before any device work."""
    from needle_cs_b200 import NeedleError

    rows = _max_items(ops, 1, 1)
    assert rows == (SCRATCH_BYTES - 16) // 32
    assert ops.attention_paged_workspace(rows, 1, 1) <= SCRATCH_BYTES < ops.attention_paged_workspace(rows + 1, 1, 1)
    assert ops.attention_paged_workspace(512, 8, 128) <= SCRATCH_BYTES  # 512 rows at the widest table fit
    base = make_case(7, [1, 9, 33, 64, 17, 50, 2, 63], 1, max_pages=1)
    n = len(base["row_slot"])
    idx = np.arange(rows) % n
    case = dict(base, q_perm=base["q_perm"][idx], QS=base["QS"][idx], row_slot=base["row_slot"][idx],
                row_pos=base["row_pos"][idx])
    d = _args(case, cuda)
    ref = _regular(d, case, cuda)
    got, st = _noalloc(d, case, cuda)
    assert st == 0
    assert np.array_equal(got, ref)
    over = np.arange(rows + 1) % n
    case_over = dict(base, q_perm=base["q_perm"][over], QS=base["QS"][over], row_slot=base["row_slot"][over],
                     row_pos=base["row_pos"][over])
    d_over = _args(case_over, cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty((rows + 1, 1, 64), dtype=torch.float32, device=cuda)
    with pytest.raises(NeedleError) as e:
        _call("ndl_attention_paged_noalloc", d_over, case_over, out, status)
    assert e.value.status == 100
    assert "scratch" in str(e.value)
    torch.cuda.synchronize()
    assert status.item() == 0
