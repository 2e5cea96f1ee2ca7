"""ctypes mirror of include/hy_device_abi.h and include/hymt2_cuda.h."""
from __future__ import annotations

import ctypes as C

import numpy as np

QK_K = 256
MAX_BATCH = 16
GT_F32, GT_F16, GT_Q8_0, GT_Q4_K, GT_Q6_K, GT_Q2_0C, GT_STQ1_0 = 0, 1, 8, 12, 14, 40, 43

# q8k_block: qp[256] i8, d f32, sum i32, bsums[16] i16, pad[24], qs[256] i8  (576 B)
Q8K_DTYPE = np.dtype([("qp", np.int8, 256), ("d", np.float32), ("sum", np.int32), ("bsums", np.int16, 16),
                      ("pad", np.uint8, 24), ("qs", np.int8, 256)])
assert Q8K_DTYPE.itemsize == 576


def q8k_empty(n: int) -> np.ndarray:
    """n zeroed q8k blocks in a 64-byte aligned buffer."""
    raw = np.zeros(n * 576 + 64, dtype=np.uint8)
    off = (-raw.ctypes.data) % 64
    return raw[off:off + n * 576].view(Q8K_DTYPE)


class WeightT(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int), ("k", C.c_int), ("n", C.c_int), ("row_bytes", C.c_size_t),
                ("pk", C.c_void_p), ("ps", C.c_void_p), ("pshift", C.c_int), ("poff", C.c_int), ("gpu", C.c_void_p)]


class FusedLayer(C.Structure):
    _fields_ = [("wq", C.c_void_p), ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p), ("wg", C.c_void_p),
                ("wu", C.c_void_p), ("wd", C.c_void_p), ("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p)]


class FusedArgs(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("hdim", C.c_int), ("qdim", C.c_int), ("kvdim", C.c_int), ("ctx", C.c_int),
                ("rope_half", C.c_int), ("nt", C.c_int), ("pos0", C.c_int), ("eps", C.c_float),
                ("want_logits", C.c_int), ("layers", C.POINTER(FusedLayer)), ("outw", C.c_void_p),
                ("out_norm", C.c_void_p), ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p), ("h", C.c_void_p),
                ("logits", C.c_void_p)]


DESTROY = C.CFUNCTYPE(None, C.c_void_p)
UPLOAD = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.POINTER(WeightT))
RELEASE = C.CFUNCTYPE(None, C.c_void_p)
MATMUL = C.CFUNCTYPE(C.c_bool, C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int, C.c_void_p, C.c_int)
IS_SW = C.CFUNCTYPE(C.c_bool, C.c_void_p)
WEIGHT_OUT = C.CFUNCTYPE(C.c_void_p, C.c_void_p)
PREPARE = C.CFUNCTYPE(C.c_bool, C.c_void_p, C.POINTER(FusedArgs))
FORWARD = C.CFUNCTYPE(C.c_bool, C.c_void_p, C.POINTER(FusedArgs))


class DeviceOps(C.Structure):
    _fields_ = [("destroy_impl", DESTROY), ("upload", UPLOAD), ("release", RELEASE), ("matmul", MATMUL),
                ("is_software", IS_SW), ("weight_out", WEIGHT_OUT), ("fused_prepare", PREPARE),
                ("fused_forward", FORWARD)]


class ServeStats(C.Structure):
    _fields_ = [("steps", C.c_longlong), ("decode_tokens", C.c_longlong), ("prefill_tokens", C.c_longlong),
                ("prefix_hits", C.c_longlong), ("prefix_tokens", C.c_longlong), ("generated", C.c_longlong),
                ("shared_pages", C.c_longlong), ("copied_rows", C.c_longlong), ("evictions", C.c_longlong),
                ("active_seq_steps", C.c_longlong)]


# Every symbol include/hymt2_cuda.h declares, with its ctypes signature.
P, I, F, Z = C.c_void_p, C.c_int, C.c_float, C.c_size_t
SIGNATURES = {
    "hy_cuda_create": (P, [C.c_char_p, C.c_char_p, Z]),
    "hy_cuda_probe": (I, [C.c_char_p, I]),
    "hyc_create": (P, [I, C.c_char_p, Z]),
    "hyc_device_ops": (C.POINTER(DeviceOps), []),
    "hyc_last_error": (I, [P, C.c_char_p, I]),
    "hyc_stream": (P, [P]),
    "hyc_sync": (I, [P]),
    "hyc_set_embedding": (I, [P, P]),
    "hyc_generate": (I, [P, P, I, I, I, P, I, I, P]),
    "hyc_decode_begin": (I, [P, P, I, I, I, P, I, I]),
    "hyc_decode_steps": (I, [P, I]),
    "hyc_decode_steps_host": (I, [P, I, P]),
    "hyc_decode_resident": (I, [P, I, P, C.c_ulonglong]),
    "hyc_resident_go": (I, [P, I, I]),
    "hyc_resident_wait": (I, [P, I, P, C.c_ulonglong]),
    "hyc_decode_read": (I, [P, P, I]),
    "hyc_decode_rewind": (I, [P, I, I]),
    "hyc_host_alloc": (P, [Z]),
    "hyc_host_free": (None, [P]),
    "hyc_set_decode_mode": (I, [P, I]),
    "hyc_set_tc": (I, [P, I]),
    "hyc_set_stq_layout": (I, [P, I]),
    "hyc_tc_test": (I, [P, P, I, P, P, P, F, I, P]),
    "hyc_decode_path": (I, [P, C.c_char_p, I]),
    "hyc_wait_probe": (I, [P, C.c_ulonglong, P]),
    "hyc_batch_prepare": (I, [P, I, I, I, I]),
    "hyc_batch_forward": (I, [P, P, P, P, I, P, I, I, P, P]),
    "hyc_batch_kv_copy": (I, [P, I, I, I]),
    "hyc_batch_kv_read": (I, [P, I, I, I, P, P]),
    "hyc_serve": (I, [P, P, P, I, I, P, I, I, I, P, P, C.POINTER(ServeStats)]),
    "hyc_mega_timeline": (I, [P, P, I]),
    "hyc_quantize_q8k": (I, [P, P, I, I, P]),
    "hyc_block_ints": (I, [P, P, P, I, P]),
    "hyc_tc_block_ints": (I, [P, P, P, I, P]),
    "hyc_tp_init": (I, [P, I, I, I, P]),
    "hyc_tp_connect": (I, [P, P]),
    "hyc_dequant_row": (I, [P, P, I, P]),
    "hyc_matmul_f32": (I, [P, P, P, I, P]),
    "hyc_kv_read": (I, [P, I, I, P, P]),
    "hyc_rope_tables": (I, [F, F, I, I, I, P, P]),
    "hyc_launch_count": (C.c_longlong, [P]),
    "hyc_bench_op": (I, [P, I, I]),
    "hyc_gemv_test": (I, [P, P, I, P, P, P, F, I, I, P]),
    "hyc_debug_buffer": (I, [P, I, P, Z]),
    "hyc_gemv_multi_test": (I, [P, P, I, I, P, P, F, I, P]),
    "hyc_trace": (I, [P, I]),
    "hyc_trace_read": (I, [P, P, I]),
    "hyc_attention_decode_noalloc": (I, [P, I, I, I, I, P, F, P, P, P, P, P, P, P, P, C.c_char_p, I]),
    "hyc_attention_test": (I, [P, I, I, I, I, I, I, F, P, P, P, P, P, P, P, P]),
}


def bind(lib: C.CDLL) -> C.CDLL:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib
