"""ctypes binding of libcortex.so (declarations in include/cortex.h).

The library is the product: every call here goes through its C ABI, exactly
as the PHP host binds it with FFI::cdef (src/tensor_ffi_adapter.php:46-61).
There is no Python or CPU fallback; a missing library raises.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcortex.so")

PREC_FP32, PREC_TF32, PREC_BF16 = 0, 1, 2
HOST_PTRS, DEVICE_PTRS = 0, 1

c_int, c_float, c_double, c_void_p, c_char_p = (ctypes.c_int, ctypes.c_float, ctypes.c_double,
                                                ctypes.c_void_p, ctypes.c_char_p)
c_int_p = ctypes.POINTER(ctypes.c_int)
c_float_p = ctypes.POINTER(ctypes.c_float)


class SampleParams(ctypes.Structure):
    """snai_sample_params: which reference sampler and its constants."""

    _fields_ = [
        ("variant", c_int),
        ("temperature", c_double),
        ("rep_penalty", c_double),
        ("top_k", c_int),
        ("top_p", c_double),
        ("nan_guard", c_int),
    ]


# name -> (restype, argtypes); the full export list of include/cortex.h
SIGNATURES = {
    # reference boundary (core/cortex.nim FFI exports)
    "cortex_init": (c_void_p, [c_int, c_int, c_int, c_int, c_int]),
    "cortex_load_stream": (c_void_p, [c_char_p, c_int]),
    "cortex_forward": (None, [c_void_p, c_void_p, c_int, c_void_p]),
    "cortex_reset_cache": (None, [c_void_p]),
    "cortex_free": (None, [c_void_p]),
    "cortex_init_gpu": (None, []),
    "get_vocab_size": (c_int, [c_void_p]),
    "get_ctx_size": (c_int, [c_void_p]),
    "cortex_load_layer": (None, [c_void_p, c_int, c_int, c_void_p, c_int]),
    "cortex_extract_layer": (None, [c_void_p, c_int, c_int, c_void_p, c_int]),
    "cortex_load_adam_layer": (None, [c_void_p, c_int, c_int, ctypes.c_bool, c_void_p, c_int]),
    "cortex_extract_adam_layer": (None, [c_void_p, c_int, c_int, ctypes.c_bool, c_void_p, c_int]),
    "cortex_train_step": (c_float, [c_void_p, c_void_p, c_void_p, c_int, c_float]),
    # batched extension
    "cortex_last_error": (c_char_p, []),
    "cortex_load_stream_ex": (c_void_p, [c_char_p, c_int, c_int, c_int, c_int]),
    "cortex_init_ex": (c_void_p, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "cortex_num_slots": (c_int, [c_void_p]),
    "cortex_head_size": (c_int, [c_void_p]),
    "cortex_num_heads": (c_int, [c_void_p]),
    "cortex_seq_reset": (c_int, [c_void_p, c_void_p, c_int]),
    "cortex_seq_pos": (c_int, [c_void_p, c_int]),
    "cortex_forward_batch": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int]),
    "cortex_decode_batch": (c_int, [c_void_p, c_void_p, c_int, c_void_p, ctypes.POINTER(SampleParams),
                                    c_void_p, c_int]),
    "cortex_decode_steps": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, ctypes.POINTER(SampleParams),
                                    c_void_p, c_int]),
    "cortex_get_logits": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "cortex_sample": (c_int, [c_void_p, c_int, c_int, ctypes.c_longlong, c_void_p, c_int, c_void_p, c_void_p,
                              ctypes.POINTER(SampleParams), c_void_p, c_void_p]),
    "cortex_set_stream": (c_int, [c_void_p, c_void_p]),
    "cortex_synchronize": (c_int, [c_void_p]),
    "cortex_seq_rewind": (c_int, [c_void_p, c_void_p, c_int, c_int]),
    "cortex_profile_enable": (c_int, [c_void_p, c_int]),
    "cortex_profile_read": (c_int, [c_void_p, c_int, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(c_double),
                                    ctypes.POINTER(c_double), ctypes.POINTER(c_double)]),
    "cortex_forward_batch_noalloc": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int]),
    "cortex_group_load": (c_void_p, [c_char_p, c_int, c_int, c_void_p, c_int, c_int]),
    "cortex_group_free": (None, [c_void_p]),
    "cortex_group_size": (c_int, [c_void_p]),
    "cortex_group_engine": (c_void_p, [c_void_p, c_int]),
    "cortex_group_shard": (c_int, [c_void_p, c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "cortex_group_load_seconds": (c_double, [c_void_p]),
    "cortex_group_forward": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "cortex_group_decode_steps": (c_int, [c_void_p, c_int, c_void_p, ctypes.POINTER(SampleParams), c_void_p]),
    "cortex_merge_files": (c_int, [ctypes.POINTER(c_char_p), c_int, c_char_p, c_int]),
    "cortex_upscale_file": (c_int, [c_char_p, c_char_p, c_int, ctypes.c_ulonglong, c_int]),
    "cortex_average_states": (c_int, [ctypes.POINTER(c_void_p), c_int]),
    "cortex_group_average": (c_int, [c_void_p]),
    "cortex_tokenizer_load": (c_void_p, [c_char_p]),
    "cortex_tokenizer_free": (None, [c_void_p]),
    "cortex_tokenizer_vocab_size": (c_int, [c_void_p]),
    "cortex_tokenizer_encode": (c_int, [c_void_p, c_char_p, c_int, c_void_p, c_int]),
    "cortex_tokenizer_decode": (c_int, [c_void_p, c_void_p, c_int, c_int, c_char_p, c_int]),
    "cortex_selftest_wait_timeout": (c_int, [c_void_p, ctypes.c_longlong]),
    "cortex_kernel_launches": (ctypes.c_longlong, [c_void_p]),
    "cortex_train_grads": (c_int, [c_void_p, c_void_p, c_void_p, c_int, ctypes.POINTER(c_float)]),
    "cortex_train_apply": (c_int, [c_void_p, c_float, c_float]),
    "cortex_load_grad_layer": (None, [c_void_p, c_int, c_int, c_void_p, c_int]),
    "cortex_extract_grad_layer": (None, [c_void_p, c_int, c_int, c_void_p, c_int]),
    "cortex_train_info": (c_int, [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_float), ctypes.POINTER(c_float),
                                  ctypes.POINTER(c_int)]),
}

_lib = None
_lock = threading.Lock()


class CortexError(RuntimeError):
    pass


def load(path=None):
    """Loads libcortex.so (once) and declares every exported function."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise CortexError(f"{p} is not built; run `make -C snai_b200/csrc` or __graft_entry__.build()")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def last_error():
    return load().cortex_last_error().decode(errors="replace")


def check(rc, what="libcortex call"):
    if rc != 0:
        raise CortexError(f"{what} failed ({rc}): {last_error()}")
    return rc
