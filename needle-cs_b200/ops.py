"""Tensor-level wrappers over the C ABI.

torch is plumbing here: device memory, the current CUDA stream and shape
bookkeeping.  All arithmetic happens in libneedle_b200.so.  Every wrapper
checks device, dtype and contiguity before handing raw pointers to the ABI.
"""
import numpy as np
import torch

from ._native import call, lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _dev(t, dtype, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t.data_ptr()


# ---------------------------------------------------------------- synth --

def synth_normal_f32(seed, stream, count, scale=1.0, first=0):
    out = np.empty(count, np.float32)
    lib().ndl_synth_normal_f32(seed, stream, first, count, scale, out.ctypes.data)
    return out


def synth_normal_f16(seed, stream, count, scale=1.0, first=0):
    out = np.empty(count, np.uint16)
    lib().ndl_synth_normal_f16(seed, stream, first, count, scale, out.ctypes.data)
    return out


def synth_uniform_f16(seed, stream, count, lo, hi, first=0):
    out = np.empty(count, np.uint16)
    lib().ndl_synth_uniform_f16(seed, stream, first, count, lo, hi, out.ctypes.data)
    return out


def synth_int8(seed, stream, count, first=0):
    out = np.empty(count, np.int8)
    lib().ndl_synth_int8(seed, stream, first, count, out.ctypes.data)
    return out


def synth_normal_f32_device(seed, stream, out, scale=1.0, first=0):
    call("ndl_synth_normal_f32_device", seed, stream, first, out.numel(), scale, _dev(out, torch.float32, "out"),
         _stream())


def synth_normal_f16_device(seed, stream, out, scale=1.0, first=0):
    call("ndl_synth_normal_f16_device", seed, stream, first, out.numel(), scale, _dev(out, torch.int16, "out"),
         _stream())


def synth_uniform_f16_device(seed, stream, out, lo, hi, first=0):
    call("ndl_synth_uniform_f16_device", seed, stream, first, out.numel(), lo, hi, _dev(out, torch.int16, "out"),
         _stream())


def synth_int8_device(seed, stream, out, first=0):
    call("ndl_synth_int8_device", seed, stream, first, out.numel(), _dev(out, torch.int8, "out"), _stream())


# -------------------------------------------------------------- kernels --

def quantize_rows(x, q=None, scales=None):
    """Per-row int8 quantizer (Quant.QuantizeInt8 per row)."""
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=torch.int8, device=x.device) if q is None else q
    scales = torch.empty(rows, dtype=torch.float32, device=x.device) if scales is None else scales
    call("ndl_quantize_rows", _dev(x, torch.float32, "x"), rows, cols, _dev(q, torch.int8, "q"),
         _dev(scales, torch.float32, "scales"), _stream())
    return q, scales


def rmsnorm_quantize(x, weight, q=None, scales=None):
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=torch.int8, device=x.device) if q is None else q
    scales = torch.empty(rows, dtype=torch.float32, device=x.device) if scales is None else scales
    call("ndl_rmsnorm_quantize", _dev(x, torch.float32, "x"), _dev(weight, torch.float32, "weight"), rows, cols,
         _dev(q, torch.int8, "q"), _dev(scales, torch.float32, "scales"), _stream())
    return q, scales


def matmul_i8g32(q, sa, w, sw, y=None, residual=None, acc=None):
    """I8G32 linear: y[t][n] = sa[t] * (fma chain over groups of half(sw[n][g]) * D[t][n][g]).

    q int8 [m,k], sa fp32 [m], w int8 [n,k], sw fp16 bits as int16 [n,k/32].
    """
    m, k = q.shape
    n = w.shape[0]
    y = torch.empty((m, n), dtype=torch.float32, device=q.device) if y is None else y
    res_ptr = _dev(residual, torch.float32, "residual") if residual is not None else None
    acc_ptr = _dev(acc, torch.int32, "acc") if acc is not None else None
    call("ndl_matmul_i8g32", _dev(q, torch.int8, "q"), _dev(sa, torch.float32, "sa"), m,
         _dev(w, torch.int8, "w"), _dev(sw, torch.int16, "sw"), n, k, _dev(y, torch.float32, "y"), y.stride(0),
         res_ptr, acc_ptr, _stream())
    return y


def matmul_i8g32_batched(q, sa, w, sw, y):
    """Batched I8G32 linear over weight sets w [B,n,k], sw [B,n,k/32] -> y [B,m,n]."""
    m, k = q.shape
    batch, n, _ = w.shape
    call("ndl_matmul_i8g32_batched", _dev(q, torch.int8, "q"), _dev(sa, torch.float32, "sa"), m,
         _dev(w, torch.int8, "w"), _dev(sw, torch.int16, "sw"), n, k, batch, n * k, n * (k // 32),
         _dev(y, torch.float32, "y"), n, m * n, _stream())
    return y


def cq_prepare(x, bits, values=None, scales=None, offsets=None):
    """Quant.Prepare for CQ weights: per (token, 128 columns) FWHT, int8
    quantize and plane reorder.  x fp32 [tokens, cols] -> (values int8
    [tokens, cols], scales and offsets fp32 [tokens, stride])."""
    tokens, cols = x.shape
    stride = ((cols // 128) + 7) & ~7
    values = torch.empty((tokens, cols), dtype=torch.int8, device=x.device) if values is None else values
    scales = torch.empty((tokens, stride), dtype=torch.float32, device=x.device) if scales is None else scales
    offsets = torch.empty((tokens, stride), dtype=torch.float32, device=x.device) if offsets is None else offsets
    call("ndl_cq_prepare", _dev(x, torch.float32, "x"), tokens, cols, bits, _dev(values, torch.int8, "values"),
         _dev(scales, torch.float32, "scales"), _dev(offsets, torch.float32, "offsets"), scales.stride(0),
         _stream())
    return values, scales, offsets


def cq_matmul(indices, norms, book_bytes, byte_scale, bits, values, scales, offsets, y=None):
    """MatMulRows on a CQ matrix: indices uint8 [rows, cols*bits/8], norms fp16
    bits as int16 [rows, cols/128], book_bytes the codebook's 16 level bytes
    (host); activations from cq_prepare -> y fp32 [tokens, rows]."""
    import ctypes

    rows = indices.shape[0]
    tokens, cols = values.shape
    y = torch.empty((tokens, rows), dtype=torch.float32, device=values.device) if y is None else y
    table = (ctypes.c_uint8 * 16).from_buffer_copy(bytes(book_bytes[:16]))
    call("ndl_cq_matmul", _dev(indices, torch.uint8, "indices"), _dev(norms, torch.int16, "norms"),
         ctypes.addressof(table), float(byte_scale), rows, cols, bits, _dev(values, torch.int8, "values"),
         _dev(scales, torch.float32, "scales"), _dev(offsets, torch.float32, "offsets"), scales.stride(0), tokens,
         _dev(y, torch.float32, "y"), y.stride(0), 0, rows, _stream())
    return y


def attention_paged_workspace(rows, heads, max_pages):
    return lib().ndl_attention_paged_workspace(rows, heads, max_pages)


def attention_paged(q8, qs, row_slot, row_pos, page_table, pool, page_bytes, layer, out=None, workspace=None,
                    status=None):
    """Paged int8 decode attention (ndl_attention_paged).

    q8 int8 [rows,heads,64] in the page K dim order, qs fp32 [rows,heads],
    row_slot/row_pos int32 [rows], page_table int32 [slots,max_pages],
    pool uint8 [num_pages*page_bytes]; out fp32 [rows,heads,64]."""
    rows, heads, _ = q8.shape
    slots, max_pages = page_table.shape
    out = torch.empty((rows, heads, 64), dtype=torch.float32, device=q8.device) if out is None else out
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (_dev(workspace, torch.uint8, "workspace"),
                                                             workspace.numel())
    call("ndl_attention_paged", _dev(q8, torch.int8, "q8"), _dev(qs, torch.float32, "qs"),
         _dev(row_slot, torch.int32, "row_slot"), _dev(row_pos, torch.int32, "row_pos"), rows, heads,
         _dev(page_table, torch.int32, "page_table"), slots, max_pages, _dev(pool, torch.uint8, "pool"), page_bytes,
         pool.numel() // page_bytes, layer, _dev(out, torch.float32, "out"), ws_ptr, ws_bytes,
         _dev(status, torch.int32, "status") if status is not None else None, _stream())
    return out
