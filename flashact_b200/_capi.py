"""ctypes binding of include/flashact.h (the in-tree libflashact.so). No torch types cross it."""
import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libflashact.so")

FA_OK, FA_ERR_INVALID, FA_ERR_CUDA, FA_ERR_TIMEOUT, FA_ERR_STATE, FA_ERR_UNSUPPORTED, FA_ERR_OOM = range(7)
STATUS_NAMES = {0: "FA_OK", 1: "FA_ERR_INVALID", 2: "FA_ERR_CUDA", 3: "FA_ERR_TIMEOUT", 4: "FA_ERR_STATE",
                5: "FA_ERR_UNSUPPORTED", 6: "FA_ERR_OOM"}
FA_MODEL_PI05, FA_MODEL_MOLMOACT2 = 0, 1
FA_WFMT_BF16, FA_WFMT_FP8, FA_WFMT_NVFP4 = 0, 1, 2
FA_DT_F32, FA_DT_BF16, FA_DT_F16 = 0, 1, 2
FA_KV_COMPACT_SPLIT_HALF, FA_KV_FLASHRT_INTERLEAVED = 0, 1

# Every function the header declares (checked by tests/test_capi.py against include/flashact.h).
EXPORTS = ["fa_create", "fa_pi05_load_weights", "fa_pi05_load_weights_q", "fa_ma2_load_weights", "fa_ma2_set_rope", "fa_set_modulation", "fa_bind_prefix_kv", "fa_bind_prefix_kv_masked", "fa_sample_actions",
           "fa_sync", "fa_set_stage_timing", "fa_get_stage_cycles", "fa_last_launch_count",
           "fa_set_fault_injection", "fa_debug_trace", "fa_pi05_modulations_noalloc", "fa_quantize_fp8_rows", "fa_quantize_nvfp4",
           "fa_last_error", "fa_destroy"]


class FaConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("num_layers", "width", "num_heads", "num_kv_heads", "head_dim", "mlp_dim",
                                           "horizon", "action_dim", "max_prefix", "max_batch", "num_steps",
                                           "valid_action_dim")]


class FaTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("dtype", ctypes.c_int)]


PI05_WEIGHT_FIELDS = ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "ln_in_w", "ln_in_b", "ln_post_w",
                      "ln_post_b", "norm_w", "norm_b", "time_in_w", "time_in_b", "time_out_w", "time_out_b", "ain_w",
                      "ain_b", "aout_w", "aout_b"]


class FaPi05Weights(ctypes.Structure):
    _fields_ = [(n, FaTensor) for n in PI05_WEIGHT_FIELDS]


MA2_WEIGHT_FIELDS = ["w_qkv", "b_qkv", "w_so", "b_so", "w_cq", "b_cq", "w_co", "b_co", "w_gate", "b_gate", "w_up",
                     "b_up", "w_down", "b_down", "ain_w", "ain_b", "aout_w", "aout_b"]


class FaQScale(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_void_p), ("tensor", ctypes.c_void_p)]


PI05_QUANT_FIELDS = ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"]


class FaPi05QScales(ctypes.Structure):
    _fields_ = [(n, FaQScale) for n in PI05_QUANT_FIELDS]


class FaMa2Weights(ctypes.Structure):
    _fields_ = [(n, FaTensor) for n in MA2_WEIGHT_FIELDS]


class FlashActError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def load_library(path: str = None) -> ctypes.CDLL:
    """Loads libflashact.so (or the build named by $FLASHACT_LIB, for A/B comparisons of two
    builds); raises (never falls back) when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("FLASHACT_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise FlashActError(FA_ERR_UNSUPPORTED, f"{path} missing: run `python -m flashact_b200.build`")
    lib = ctypes.CDLL(path)
    H, S, P, I = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int
    sig = {
        "fa_create": (S, [I, ctypes.POINTER(FaConfig), I, ctypes.POINTER(ctypes.c_void_p)]),
        "fa_pi05_load_weights": (S, [H, ctypes.POINTER(FaPi05Weights), I]),
        "fa_pi05_load_weights_q": (S, [H, ctypes.POINTER(FaPi05Weights), I, ctypes.POINTER(FaPi05QScales)]),
        "fa_ma2_load_weights": (S, [H, ctypes.POINTER(FaMa2Weights)]),
        "fa_ma2_set_rope": (S, [H, P, P]),
        "fa_set_modulation": (S, [H, P, P]),
        "fa_bind_prefix_kv": (S, [H, I, P, P, I, ctypes.POINTER(ctypes.c_int), I, P]),
        "fa_bind_prefix_kv_masked": (S, [H, I, P, P, I, P, I, P]),
        "fa_sample_actions": (S, [H, I, P, P, P]),
        "fa_sync": (S, [H, P]),
        "fa_set_stage_timing": (S, [H, I]),
        "fa_get_stage_cycles": (S, [H, ctypes.POINTER(ctypes.c_uint64), I]),
        "fa_last_launch_count": (I, [H]),
        "fa_set_fault_injection": (S, [H, I, ctypes.c_uint]),
        "fa_debug_trace": (S, [H, I, I, ctypes.POINTER(ctypes.c_ulonglong), I]),
        "fa_pi05_modulations_noalloc": (S, [ctypes.POINTER(FaPi05Weights), I, I, P, P, P]),
        "fa_quantize_fp8_rows": (S, [P, I, I, I, I, P, P, P]),
        "fa_quantize_nvfp4": (S, [P, I, I, I, I, P, P, P, P]),
        "fa_last_error": (ctypes.c_char_p, [H]),
        "fa_destroy": (None, [H]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    _lib = lib
    return lib


def check(lib, handle, status):
    if status != FA_OK:
        raise FlashActError(status, lib.fa_last_error(handle).decode(errors="replace"))
