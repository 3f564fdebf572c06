"""ctypes binding of libneedle_b200.so (the C ABI in include/needle_cuda.h).

The library is built in-tree (needle-cs_b200/lib/) by `make -C needle-cs_b200`.
There is no fallback: if the library is missing every call raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libneedle_b200.so")

c_int, c_float, c_size_t, c_u64, c_ll = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_longlong
c_void_p, c_char_p = ctypes.c_void_p, ctypes.c_char_p
c_u16 = ctypes.c_uint16

# name -> (restype, argtypes).  Device pointers and streams travel as void*.
SIGNATURES = {
    "ndl_version": (c_char_p, []),
    "ndl_status_string": (c_char_p, [c_int]),
    "ndl_last_error": (c_char_p, []),
    "ndl_device_count": (c_int, [ctypes.POINTER(c_int)]),
    "ndl_synth_normal_f32": (None, [c_u64, c_u64, c_u64, c_size_t, c_float, c_void_p]),
    "ndl_synth_normal_f16": (None, [c_u64, c_u64, c_u64, c_size_t, c_float, c_void_p]),
    "ndl_synth_uniform_f16": (None, [c_u64, c_u64, c_u64, c_size_t, c_float, c_float, c_void_p]),
    "ndl_synth_int8": (None, [c_u64, c_u64, c_u64, c_size_t, c_void_p]),
    "ndl_f32_to_f16": (c_u16, [c_float]),
    "ndl_f16_to_f32": (c_float, [c_u16]),
    "ndl_synth_normal_f32_device": (c_int, [c_u64, c_u64, c_u64, c_size_t, c_float, c_void_p, c_void_p]),
    "ndl_synth_normal_f16_device": (c_int, [c_u64, c_u64, c_u64, c_size_t, c_float, c_void_p, c_void_p]),
    "ndl_synth_uniform_f16_device": (c_int, [c_u64, c_u64, c_u64, c_size_t, c_float, c_float, c_void_p, c_void_p]),
    "ndl_synth_int8_device": (c_int, [c_u64, c_u64, c_u64, c_size_t, c_void_p, c_void_p]),
    "ndl_quantize_rows": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_rmsnorm_quantize": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_matmul_i8g32": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int,
                                 c_void_p, c_void_p, c_void_p]),
    "ndl_matmul_i8g32_batched": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_ll,
                                         c_ll, c_void_p, c_int, c_ll, c_void_p]),
    "ndl_attention_paged_workspace": (c_size_t, [c_int, c_int, c_int]),
    "ndl_attention_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int,
                                    c_void_p, c_size_t, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p,
                                    c_void_p]),
    "ndl_attention_paged_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int,
                                            c_int, c_void_p, c_size_t, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_engine_create": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_void_p)]),
    "ndl_engine_create_model": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_void_p)]),
    "ndl_whistle_create": (c_int, [c_void_p, c_int, ctypes.POINTER(c_void_p)]),
    "ndl_whistle_encode": (c_int, [c_void_p, c_void_p, c_int, ctypes.POINTER(c_int)]),
    "ndl_whistle_encode_device": (c_int, [c_void_p, c_void_p, c_int]),
    "ndl_whistle_frames": (c_int, [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "ndl_whistle_read": (c_int, [c_void_p, c_int, c_int, c_void_p, c_size_t, ctypes.POINTER(c_size_t)]),
    "ndl_whistle_stream": (c_void_p, [c_void_p]),
    "ndl_whistle_destroy": (c_int, [c_void_p]),
    "ndl_engine_destroy": (c_int, [c_void_p]),
    "ndl_engine_stream": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "ndl_engine_tensor": (c_int, [c_void_p, c_char_p, c_int, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
    "ndl_engine_read_tensor": (c_int, [c_void_p, c_char_p, c_int, c_void_p, c_size_t]),
    "ndl_engine_page_bytes": (c_int, [c_void_p, ctypes.POINTER(c_size_t)]),
    "ndl_engine_sync": (c_int, [c_void_p]),
    "ndl_slot_length": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int)]),
    "ndl_slot_reset": (c_int, [c_void_p, c_int]),
    "ndl_slot_mark": (c_int, [c_void_p, c_int]),
    "ndl_slot_rewind": (c_int, [c_void_p, c_int]),
    "ndl_slot_page": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_int)]),
    "ndl_slot_fill_synthetic": (c_int, [c_void_p, c_int, c_int, c_u64, c_u64]),
    "ndl_forward_batch": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int]),
    "ndl_batch_logits_row": (c_int, [c_void_p, c_int, c_void_p]),
    "ndl_sample_argmax": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_sample_topk": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_engine_set_mask": (c_int, [c_void_p, c_int, c_void_p, c_int]),
    "ndl_sample_argmax_slots": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "ndl_logits_sparse": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ndl_cq_prepare": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "ndl_cq_gather_rows": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_cq_matmul": (c_int, [c_void_p, c_void_p, c_void_p, ctypes.c_float, c_int, c_int, c_int, c_void_p, c_void_p,
                              c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p]),
    "ndl_engine_get_info": (c_int, [c_void_p, c_void_p]),
    "ndl_slot_set_memory": (c_int, [c_void_p, c_int, c_void_p, c_int]),
    "ndl_slot_fill_memory_synthetic": (c_int, [c_void_p, c_int, c_int, c_u64, c_u64]),
    "ndl_slot_attach_memory": (c_int, [c_void_p, c_int, c_int]),
    "ndl_slot_copy": (c_int, [c_void_p, c_int, c_int]),
    "ndl_slot_prefix_bytes": (c_int, [c_void_p, c_int, ctypes.POINTER(c_size_t)]),
    "ndl_slot_export_prefix": (c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    "ndl_slot_import_prefix": (c_int, [c_void_p, c_int, c_void_p, c_size_t]),
    "ndl_slot_share_prefix": (c_int, [c_void_p, c_int, c_int]),
    "ndl_engine_free_pages": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "ndl_engine_time_attention": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_float)]),
    "ndl_selftest_bounded_wait": (c_int, [c_int]),
    "ndl_selftest_exp": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_kt_quantize_int8": (c_float, [c_void_p, c_int, c_void_p]),
    "ndl_kt_argmax_masked": (c_int, [c_void_p, c_void_p, c_int, c_int]),
    "ndl_kt_best_probability": (c_float, [c_void_p, c_int, c_float]),
    "ndl_kt_matmul_rows": (None, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int]),
    "ndl_kt_prepare": (None, [c_void_p, c_int, c_int, c_int, c_void_p]),
    "ndl_kt_gather_row": (None, [c_void_p, c_int, c_void_p]),
    "ndl_kt_rms_fake_a8": (None, [c_void_p, c_int, c_void_p]),
    "ndl_kt_centered_rms_fake_a8": (None, [c_void_p, c_void_p, c_int, c_void_p]),
    "ndl_kt_gate_fake_a8": (None, [c_void_p, c_void_p, c_int]),
    "ndl_kt_post_norm_add": (None, [c_void_p, c_void_p, c_void_p, c_float, c_int]),
    "ndl_kt_combine_diff4": (None, [c_void_p, c_int, c_float, c_float, c_float, c_float, c_void_p, c_void_p, c_float, c_void_p]),
    "ndl_kt_mix4": (None, [c_void_p, c_int, c_float, c_float, c_float, c_float, c_void_p]),
    "ndl_kt_combine4": (None, [c_void_p, c_int, c_float, c_float, c_float, c_float, c_void_p, c_float, c_void_p]),
    "ndl_kt_taps3": (None, [c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_kt_sinkhorn4x4": (None, [c_void_p, c_void_p]),
    "ndl_kt_rope": (None, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ndl_kt_zero_centered_rms": (None, [c_void_p, c_void_p, c_int, c_void_p]),
    "ndl_kt_rms_unit": (None, [c_void_p, c_int, c_void_p]),
    "ndl_kt_softmax": (None, [c_void_p, c_int]),
    "ndl_kt_dot": (c_float, [c_void_p, c_void_p, c_int]),
    "ndl_kt_add_scaled": (None, [c_void_p, c_void_p, c_float, c_int]),
    "ndl_kt_scale_add": (None, [c_void_p, c_float, c_void_p, c_float, c_int]),
    "ndl_kt_multiply_accumulate": (None, [c_void_p, c_void_p, c_void_p, c_int]),
    "ndl_kt_fake_a8": (c_float, [c_void_p, c_int]),
    "ndl_kt_attention_tile": (None, [c_void_p]),
    "ndl_kt_merge_partials": (None, [c_void_p, c_int, c_int, c_void_p]),
    "ndl_kt_hadamard_mlp": (None, [c_void_p, c_void_p, c_void_p]),
    "ndl_hc_mix4": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_hc_combine4": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_hc_combine_diff4x4": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_hc_sinkhorn4x4": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_taps3": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "ndl_fake_a8_rows": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ndl_engram_hash": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ndl_engram_conv": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_engram_gate": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "ndl_conf_pool_update": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ndl_conf_logit": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_beam_search": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                                c_void_p, c_void_p]),
    "ndl_sched_create": (c_int, [c_void_p, c_void_p, c_void_p]),
    "ndl_sched_create_dry": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p]),
    "ndl_sched_destroy": (c_int, [c_void_p]),
    "ndl_sched_submit": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_int]),
    "ndl_sched_force": (c_int, [c_void_p, c_int, c_void_p, c_int]),
    "ndl_sched_step": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "ndl_sched_tokens": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "ndl_sched_pending": (c_int, [c_void_p, c_void_p, c_void_p]),
    "ndl_sched_last_plan": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ndl_engine_profile": (c_int, [c_void_p, c_int]),
    "ndl_engine_use_graphs": (c_int, [c_void_p, c_int]),
    "ndl_engine_use_pdl": (c_int, [c_void_p, c_int]),
    "ndl_engine_profile_read": (c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    "ndl_model_load": (c_int, [c_void_p, c_size_t, c_int, c_void_p]),
    "ndl_model_destroy": (c_int, [c_void_p]),
    "ndl_model_get_info": (c_int, [c_void_p, c_void_p]),
    "ndl_model_tensor_count": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "ndl_model_tensor_name": (c_int, [c_void_p, c_int, ctypes.POINTER(c_char_p), ctypes.POINTER(c_int)]),
    "ndl_model_get_tensor": (c_int, [c_void_p, c_char_p, c_int, c_void_p]),
    "ndl_model_read_host": (c_int, [c_void_p, c_char_p, c_int, c_void_p, c_size_t]),
    "ndl_model_tokenizer": (c_int, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_size_t)]),
    "ndl_engram_workspace": (c_size_t, [c_void_p, c_int]),
    "ndl_mlp_apply": (c_int, [c_void_p, c_int, c_void_p, c_int, c_float, c_void_p]),
    "ndl_engram_apply": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
}

PROF_CLASSES = ["prepare", "norm_quant", "gemm_qkv", "kv_write", "attention", "gemm_o", "gemm_gateup", "swiglu",
                "gemm_down", "head", "sample", "cross"]


class DecoderConfig(ctypes.Structure):
    """ndl_decoder_config."""
    _fields_ = [("layers", c_int), ("dim", c_int), ("heads", c_int), ("head_dim", c_int), ("ffn", c_int),
                ("vocab", c_int), ("rope_theta", c_float), ("seed", c_u64), ("cross", c_int)]


class EngineInfo(ctypes.Structure):
    """ndl_engine_info."""
    _fields_ = [("slots", c_int), ("capacity", c_int), ("vocab", c_int), ("max_rows", c_int), ("max_heads", c_int),
                ("layers", c_int), ("dim", c_int), ("heads", c_int)]


class BeamConfig(ctypes.Structure):
    """ndl_beam_config."""
    _fields_ = [("width", c_int), ("max_steps", c_int), ("eos", c_int), ("mask_special_023", c_int),
                ("length_penalty", c_float)]


class SchedConfig(ctypes.Structure):
    """ndl_sched_config."""
    _fields_ = [("max_rows", c_int), ("prefill_chunk", c_int)]


class SchedEvent(ctypes.Structure):
    """ndl_sched_event."""
    _fields_ = [("request", c_int), ("kind", c_int), ("token", c_int), ("status", c_int)]


class EngineConfig(ctypes.Structure):
    """ndl_engine_config."""
    _fields_ = [("device", c_int), ("slots", c_int), ("capacity", c_int), ("kv_pages", c_int), ("max_rows", c_int),
                ("max_heads", c_int)]


class NeedleError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"needle status {status}: {message}")
        self.status = status


_lib = None


def lib():
    """Load the native library once; raise loudly if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"needle_cs_b200 native library not built: {LIB_PATH} (run make -C needle-cs_b200)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status):
    if status != 0:
        raise NeedleError(status, lib().ndl_last_error().decode())
    return status


def call(name, *args):
    return check(getattr(lib(), name)(*args))
