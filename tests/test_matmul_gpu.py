"""GPU parity of the quantizer and the I8G32 linear against the CPU oracle.

Bar: int8 values, fp32 scales, int32 accumulators and fp32 outputs all
bit-identical to the scalar definition (the kernels sum groups in the same
order with round-to-nearest operations and no FMA).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(ops, m, n, k, seed=0):
    x = ops.synth_normal_f32(seed, 1, m * k).reshape(m, k)
    w = ops.synth_int8(seed, 2, n * k).reshape(n, k)
    sw = ops.synth_uniform_f16(seed, 3, n * (k // 32), 0.001, 0.02).reshape(n, k // 32)
    return x, w, sw


@pytest.mark.parametrize("rows,cols", [(1, 512), (16, 512), (3, 48), (7, 100), (64, 2048), (5, 8192), (0, 16)])
def test_quantize_rows_bit_exact(ops, oracle, cuda, rows, cols):
    x = ops.synth_normal_f32(4, rows, max(rows * cols, 1))[:rows * cols].reshape(rows, cols)
    if rows:
        x[0, ::7] = 0.0
        x[-1, 3::11] = 1e-38
    q, s = ops.quantize_rows(torch.from_numpy(x).to(cuda))
    if rows == 0:
        return
    q_ref, s_ref = oracle.quantize_rows(x)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)


def test_quantize_conformance_edges(ops, oracle, cuda):
    """QuantizeInt8Bounds inputs (KernelConformanceTests.cs:1112-1135) + golden."""
    for n in (8, 32, 128):
        x = oracle.XorShift64(0x0DE0).fill_edges(n, 3.0)[None, :n]
        q, s = ops.quantize_rows(torch.from_numpy(np.ascontiguousarray(x)).to(cuda))
        q_ref, s_ref = oracle.quantize_rows(x)
        assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)
    x = np.float32([[-4, 0, 4, 0, 0, 0, 0, 0]])
    q, s = ops.quantize_rows(torch.from_numpy(x).to(cuda))
    assert q.cpu().numpy().tolist() == [[-127, 0, 127, 0, 0, 0, 0, 0]]
    assert abs(s.item() - 0.03149606) <= 1e-6
    zero = torch.zeros((2, 64), device=cuda)
    q, s = ops.quantize_rows(zero)
    assert s.cpu().tolist() == [1.0, 1.0] and int(q.abs().sum()) == 0


@pytest.mark.parametrize("m,n,k", [(1, 2048, 512), (16, 2048, 512), (5, 37, 96), (1, 8192, 512),
                                   (16, 512, 2048), (33, 1536, 512), (2, 64, 8192)])
def test_matmul_i8g32_bit_exact(ops, oracle, cuda, m, n, k):
    x, w, sw = _inputs(ops, m, n, k)
    q_ref, s_ref = oracle.quantize_rows(x)
    y_ref, acc_ref = oracle.matmul_i8g32(q_ref, s_ref, w, sw, want_acc=True)
    q = torch.from_numpy(q_ref).to(cuda)
    s = torch.from_numpy(s_ref).to(cuda)
    acc = torch.empty((m, n, k // 32), dtype=torch.int32, device=cuda)
    y = ops.matmul_i8g32(q, s, torch.from_numpy(w).to(cuda), torch.from_numpy(sw.view(np.int16)).to(cuda), acc=acc)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    assert np.array_equal(y.cpu().numpy(), y_ref)


@pytest.mark.parametrize("m,n,k", [(64, 2048, 512), (128, 1536, 512), (200, 512, 2048), (512, 4096, 512),
                                   (100, 96, 96), (129, 136, 160), (512, 8192, 512), (64, 8, 32),
                                   (96, 256, 4096), (96, 384, 192), (160, 640, 320), (300, 1000, 704),
                                   (512, 512, 512)])
def test_matmul_tcgen05_bit_exact(ops, oracle, cuda, m, n, k):
    """m >= 64 runs the tcgen05 kind::i8 GEMM: D and y identical to the oracle
    and to the GEMV (batch invariance across the two kernels)."""
    x, w, sw = _inputs(ops, m, n, k, seed=11)
    q_ref, s_ref = oracle.quantize_rows(x)
    y_ref, acc_ref = oracle.matmul_i8g32(q_ref, s_ref, w, sw, want_acc=True)
    q = torch.from_numpy(q_ref).to(cuda)
    s = torch.from_numpy(s_ref).to(cuda)
    wd, swd = torch.from_numpy(w).to(cuda), torch.from_numpy(sw.view(np.int16)).to(cuda)
    acc = torch.empty((m, n, k // 32), dtype=torch.int32, device=cuda)
    y = ops.matmul_i8g32(q, s, wd, swd, acc=acc)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), acc_ref)
    assert np.array_equal(y.cpu().numpy(), y_ref)
    # the first 16 rows through the GEMV give the same bits
    y16 = ops.matmul_i8g32(q[:16].contiguous(), s[:16].contiguous(), wd, swd)
    torch.cuda.synchronize()
    assert np.array_equal(y16.cpu().numpy(), y[:16].cpu().numpy())


@pytest.mark.parametrize("m", [4, 130, 512])
def test_matmul_residual_and_ldy(ops, oracle, cuda, m):
    n, k = 96, 256
    x, w, sw = _inputs(ops, m, n, k, seed=9)
    q_ref, s_ref = oracle.quantize_rows(x)
    y_ref = oracle.matmul_i8g32(q_ref, s_ref, w, sw)
    res = ops.synth_normal_f32(9, 77, m * n).reshape(m, n)
    big = torch.full((m, n + 32), 7.5, device=cuda)
    y = big[:, :n]
    resd = torch.from_numpy(res).to(cuda)
    # write into a strided view: the ABI takes ldy (device tensors kept alive across the call)
    from needle_cs_b200._native import call

    qd, sd = torch.from_numpy(q_ref).to(cuda), torch.from_numpy(s_ref).to(cuda)
    wd, swd = torch.from_numpy(w).to(cuda), torch.from_numpy(sw.view(np.int16)).to(cuda)
    call("ndl_matmul_i8g32", qd.data_ptr(), sd.data_ptr(), m, wd.data_ptr(), swd.data_ptr(), n, k,
         y.data_ptr(), n + 32, None, None, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(big[:, :n].cpu().numpy(), y_ref)
    assert torch.all(big[:, n:] == 7.5)  # untouched columns (MatMulTests.cs:115-137 contract)
    out = ops.matmul_i8g32(torch.from_numpy(q_ref).to(cuda), torch.from_numpy(s_ref).to(cuda),
                           torch.from_numpy(w).to(cuda), torch.from_numpy(sw.view(np.int16)).to(cuda), residual=resd)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), res + y_ref)


@pytest.mark.parametrize("m", [16, 96])
def test_matmul_batched_equals_single(ops, oracle, cuda, m):
    n, k, b = 256, 512, 3
    x, _, _ = _inputs(ops, m, n, k)
    q_ref, s_ref = oracle.quantize_rows(x)
    w = ops.synth_int8(5, 2, b * n * k).reshape(b, n, k)
    sw = ops.synth_uniform_f16(5, 3, b * n * (k // 32), 0.001, 0.02).reshape(b, n, k // 32)
    y = torch.empty((b, m, n), device=cuda)
    ops.matmul_i8g32_batched(torch.from_numpy(q_ref).to(cuda), torch.from_numpy(s_ref).to(cuda),
                             torch.from_numpy(w).to(cuda), torch.from_numpy(sw.view(np.int16)).to(cuda), y)
    torch.cuda.synchronize()
    for i in range(b):
        assert np.array_equal(y[i].cpu().numpy(), oracle.matmul_i8g32(q_ref, s_ref, w[i], sw[i]))


def test_matmul_rejects_bad_shapes(ops, cuda):
    from needle_cs_b200 import NeedleError

    q = torch.zeros((1, 48), dtype=torch.int8, device=cuda)
    with pytest.raises(NeedleError) as e:
        ops.matmul_i8g32(q, torch.ones(1, device=cuda), torch.zeros((8, 48), dtype=torch.int8, device=cuda),
                         torch.zeros((8, 1), dtype=torch.int16, device=cuda))
    assert e.value.status == 100


def test_synth_device_matches_host(ops, cuda):
    n = 100003
    d = torch.empty(n, dtype=torch.float32, device=cuda)
    ops.synth_normal_f32_device(3, 11, d, scale=0.5, first=17)
    assert np.array_equal(d.cpu().numpy(), ops.synth_normal_f32(3, 11, n, scale=0.5, first=17))
    h = torch.empty(n, dtype=torch.int16, device=cuda)
    ops.synth_normal_f16_device(3, 12, h, scale=0.02)
    assert np.array_equal(h.cpu().numpy().view(np.uint16), ops.synth_normal_f16(3, 12, n, scale=0.02))
    ops.synth_uniform_f16_device(3, 13, h, 0.001, 0.02)
    assert np.array_equal(h.cpu().numpy().view(np.uint16), ops.synth_uniform_f16(3, 13, n, 0.001, 0.02))
    i8 = torch.empty(n, dtype=torch.int8, device=cuda)
    ops.synth_int8_device(3, 14, i8)
    assert np.array_equal(i8.cpu().numpy(), ops.synth_int8(3, 14, n))
