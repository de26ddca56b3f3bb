"""ctypes binding of libpolarswitch_b200.so (the C ABI in include/polar_switch_b200.h).

Torch tensors are used only for device memory and the current CUDA stream; the
library receives raw pointers, sizes and scalars. There is no fallback: if the
library is missing or the device is not a B200, calls raise.
"""

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libpolarswitch_b200.so")

PS_OK = 0
PS_ERR_INVALID = -1
PS_ERR_CUDA = -2
PS_ERR_UNSUPPORTED = -3
PS_ERR_WORKSPACE = -4

PS_F16, PS_F32, PS_BF16, PS_F64 = 0, 1, 2, 3
DTYPE_CODES = {torch.float16: PS_F16, torch.float32: PS_F32, torch.bfloat16: PS_BF16, torch.float64: PS_F64}

# Every symbol include/polar_switch_b200.h declares.
EXPORTED = (
    "ps_version", "ps_last_error", "ps_get_status", "ps_set_wait_limit", "ps_selftest_wait",
    "ps_selftest_chain_wait",
    "ps_normalize_workspace_bytes", "ps_normalize", "ps_gram", "ps_square", "ps_sym_product",
    "ps_apply", "ps_add_diag", "ps_circuit_workspace_bytes", "ps_circuit",
    "ps_circuit_grouped_workspace_bytes", "ps_circuit_grouped", "ps_launch_count",
    "ps_profile_enable", "ps_profile_read", "ps_normalize_noalloc", "ps_set_cta_pairs", "ps_set_chain",
    "ps_set_fused_normalize", "ps_circuit_grouped_update", "ps_set_circuit_kernel",
    "ps_set_max_ctas", "ps_gns_workspace_bytes", "ps_gns", "ps_sumsq", "ps_scale_cast",
    "ps_gram_f32", "ps_muon_direction", "ps_muon_update", "ps_update_stats",
    "ps_circuit_grouped_push", "ps_circuit_grouped_signal", "ps_stream_wait_flag",
)


class PsStep(ctypes.Structure):
    """Mirror of `ps_step`: B[dst] = alpha*B[src]@B[src] + beta*B[add] + diag*I."""

    _fields_ = [("dst", ctypes.c_int32), ("src", ctypes.c_int32), ("add", ctypes.c_int32),
                ("alpha", ctypes.c_float), ("beta", ctypes.c_float), ("diag", ctypes.c_float)]


class PsProblem(ctypes.Structure):
    """Mirror of `ps_problem`: one (L, rows, cols) problem of a grouped circuit."""

    _fields_ = [("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int32), ("L", ctypes.c_int64),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("sL", ctypes.c_int64),
                ("sR", ctypes.c_int64), ("sC", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("y_dtype", ctypes.c_int32)]


class PsUpdate(ctypes.Structure):
    """Mirror of `ps_update`: a Muon update folded into a problem's last apply."""

    _fields_ = [("p", ctypes.c_void_p), ("p_dtype", ctypes.c_int32), ("decay", ctypes.c_float),
                ("alpha", ctypes.c_float)]


class NativeError(RuntimeError):
    """A C-ABI call returned an error status."""

    def __init__(self, name, code, message):
        super().__init__(f"{name} failed ({code}): {message}")
        self.code = code


_lock = threading.Lock()
_lib = None

_i64, _f32, _ptr, _int = ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_int

_SIGNATURES = {
    "ps_version": ([], _int),
    "ps_last_error": ([], ctypes.c_char_p),
    "ps_get_status": ([ctypes.POINTER(_int), _int], _int),
    "ps_set_wait_limit": ([ctypes.c_longlong], _int),
    "ps_selftest_wait": ([ctypes.c_longlong, _ptr], _int),
    "ps_selftest_chain_wait": ([_ptr, ctypes.c_int64, ctypes.c_longlong, _ptr], _int),
    "ps_normalize_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "ps_normalize": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _ptr, _i64, _i64,
                      _ptr, _i64, _ptr], _int),
    "ps_normalize_noalloc": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _ptr, _i64,
                              _i64, _ptr], _int),
    "ps_gram": ([_ptr, _ptr, _i64, _i64, _i64, _i64, _ptr], _int),
    "ps_square": ([_ptr, _ptr, _ptr, _i64, _i64, _f32, _f32, _f32, _ptr], _int),
    "ps_sym_product": ([_ptr, _ptr, _ptr, _ptr, _i64, _i64, _f32, _f32, _f32, _ptr], _int),
    "ps_apply": ([_ptr, _ptr, _ptr, _i64, _i64, _i64, _i64, _f32, _int, _i64, _ptr], _int),
    "ps_add_diag": ([_ptr, _ptr, _i64, _i64, _f32, _ptr], _int),
    "ps_circuit_workspace_bytes": ([_i64, _i64, _i64, _int], _i64),
    "ps_circuit": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _int, _int,
                    ctypes.POINTER(_f32), ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(PsStep),
                    _int, _f32, _ptr, _i64, _ptr], _int),
    "ps_launch_count": ([], ctypes.c_longlong),
    "ps_set_cta_pairs": ([_int], _int),
    "ps_set_chain": ([_int], _int),
    "ps_set_fused_normalize": ([_int], _int),
    "ps_set_circuit_kernel": ([_int], _int),
    "ps_set_max_ctas": ([_int], _int),
    "ps_gns_workspace_bytes": ([_i64, _i64, _i64], _i64),
    "ps_sumsq": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _ptr, _i64, _ptr], _int),
    "ps_scale_cast": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _f32, _ptr, _i64, _i64,
                       _ptr], _int),
    "ps_gram_f32": ([_ptr, _ptr, _i64, _i64, _i64, _i64, _ptr], _int),
    "ps_muon_direction": ([ctypes.POINTER(_ptr), ctypes.POINTER(_ptr), _int, _i64, _int, _f32, _int, _ptr,
                           _int, _ptr], _int),
    "ps_muon_update": ([ctypes.POINTER(_ptr), _int, _i64, _int, _ptr, _int, _f32, _f32, _ptr], _int),
    "ps_update_stats": ([_ptr, _int, _i64, _i64, _ptr, _ptr, _ptr, _ptr], _int),
    "ps_gns": ([_ptr, _int, _i64, _i64, _i64, _i64, _i64, _i64, _ptr, _int, _int, ctypes.POINTER(_f32),
                _int, ctypes.POINTER(ctypes.c_int32), _f32, _ptr, _i64, _ptr], _int),
    "ps_profile_enable": ([_int], _int),
    "ps_profile_read": ([_int, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_i64),
                         ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)], _int),
    "ps_circuit_grouped_workspace_bytes": ([ctypes.POINTER(PsProblem), _int, _int], _i64),
    "ps_circuit_grouped": ([ctypes.POINTER(PsProblem), _int, _int, ctypes.POINTER(_f32),
                            ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(PsStep), _int, _f32,
                            _ptr, _i64, _ptr], _int),
    "ps_circuit_grouped_update": ([ctypes.POINTER(PsProblem), ctypes.POINTER(PsUpdate), _int, _int,
                                   ctypes.POINTER(_f32), ctypes.POINTER(ctypes.c_int32),
                                   ctypes.POINTER(PsStep), _int, _f32, _ptr, _i64, _ptr], _int),
    "ps_circuit_grouped_push": ([ctypes.POINTER(PsProblem), _int, _int, ctypes.POINTER(_f32),
                                 ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(PsStep), _int, _f32,
                                 _ptr, _i64, _ptr, ctypes.POINTER(_ptr), _int, _int,
                                 ctypes.POINTER(ctypes.c_int32), _ptr], _int),
    "ps_circuit_grouped_signal": ([ctypes.POINTER(PsProblem), _int, _int, ctypes.POINTER(_f32),
                                   ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(PsStep), _int, _f32,
                                   _ptr, _i64, _int, ctypes.POINTER(ctypes.c_int32), _ptr, _ptr], _int),
    "ps_stream_wait_flag": ([_ptr, _ptr, ctypes.c_uint], _int),
}


def library_path():
    return _LIB_PATH


def load():
    """Load the shared library (once) and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise ImportError(
                    f"polar_switch native library not built: {_LIB_PATH} is missing "
                    "(run `python polar-switch_b200/build.py`)")
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def stream_wait_flag(stream, flag_ptr, value=1):
    """Make `stream` (a torch CUDA stream) wait until the 32-bit word at device
    address `flag_ptr` is >= value (ps_stream_wait_flag)."""
    check("ps_stream_wait_flag", load().ps_stream_wait_flag(ctypes.c_void_p(stream.cuda_stream),
                                                            ctypes.c_void_p(flag_ptr), value))


def check(name, code):
    if code != PS_OK:
        msg = load().ps_last_error().decode(errors="replace")
        raise NativeError(name, code, msg)


def stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def get_status(clear=False):
    """Device status word of the current device (0 = every bounded wait completed)."""
    s = ctypes.c_int(0)
    check("ps_get_status", load().ps_get_status(ctypes.byref(s), 1 if clear else 0))
    return s.value


def set_wait_limit(cycles):
    check("ps_set_wait_limit", load().ps_set_wait_limit(int(cycles)))


def selftest_wait(limit_cycles, device=None):
    check("ps_selftest_wait", load().ps_selftest_wait(int(limit_cycles), stream_ptr(device)))


PROFILE_KINDS = {"normalize": 0, "gram": 1, "square": 2, "apply": 3, "other": 4, "circuit": 5}


def launch_count():
    """Kernels launched by the library in this process so far."""
    return int(load().ps_launch_count())


def profile_enable(enable=True):
    check("ps_profile_enable", load().ps_profile_enable(1 if enable else 0))


def profile_read():
    """{kind: dict(ms, launches, flops, bytes)} for the launches recorded since profile_enable()."""
    out = {}
    lib = load()
    for name, k in PROFILE_KINDS.items():
        ms, n, fl, by = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_double()
        check("ps_profile_read", lib.ps_profile_read(k, ctypes.byref(ms), ctypes.byref(n),
                                                     ctypes.byref(fl), ctypes.byref(by)))
        out[name] = dict(ms=ms.value, launches=n.value, flops=fl.value, bytes=by.value)
    return out


def set_cta_pairs(mode):
    """GEMM kernel selection: 0/False one-CTA kernel, 1/True (default) CTA pairs for
    every product, 2 CTA pairs for squares with n <= 1024 only. Returns the previous
    mode (an int)."""
    rc = load().ps_set_cta_pairs(int(mode))
    if rc < 0:
        check("ps_set_cta_pairs", rc)
    return rc


def set_chain(mode):
    """Inner iterations of grouped circuits on CTA pairs: 1 (default) one chain launch
    per outer iteration, 0 one launch per inner iteration. Returns the previous mode."""
    rc = load().ps_set_chain(int(mode))
    if rc < 0:
        check("ps_set_chain", rc)
    return rc


def set_circuit_kernel(mode):
    """Grouped circuits on CTA pairs: 1 (default) one persistent launch for all stages, 0
    one launch per stage. Returns the previous mode."""
    rc = load().ps_set_circuit_kernel(int(mode))
    if rc < 0:
        check("ps_set_circuit_kernel", rc)
    return rc


def set_fused_normalize(mode):
    """Normalisation inside circuits: 1 one read of each contiguous input, 0 (default)
    two passes. Returns the previous mode."""
    rc = load().ps_set_fused_normalize(int(mode))
    if rc < 0:
        check("ps_set_fused_normalize", rc)
    return rc


def set_max_ctas(max_ctas):
    """Cap the CTAs of persistent GEMM grids (0 = all SMs); returns the previous cap."""
    rc = load().ps_set_max_ctas(int(max_ctas))
    if rc < 0:
        check("ps_set_max_ctas", rc)
    return rc
