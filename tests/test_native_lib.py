"""The C-ABI library loads without a GPU and exports every symbol that
include/*.h declares (no compute calls here)."""

import ctypes
import glob
import os
import re

from polar_switch import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names.update(re.findall(r"PS_API\s+[\w\s\*]+?\b(ps_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_all_declared_symbols():
    lib = _native.load()
    declared = declared_symbols()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_native.EXPORTED) == declared


def test_version_and_error_string_without_gpu():
    lib = _native.load()
    assert lib.ps_version() >= 100
    assert isinstance(lib.ps_last_error(), bytes)


def test_invalid_arguments_are_rejected_before_any_device_work():
    lib = _native.load()
    null = ctypes.c_void_p(0)
    assert lib.ps_gram(null, null, 1, 8, 8, 8, null) == _native.PS_ERR_INVALID
    assert b"null" in lib.ps_last_error()
    assert lib.ps_set_wait_limit(0) == _native.PS_ERR_INVALID
    coeffs = (ctypes.c_float * 3)(1.0, 0.0, 0.0)
    resets = (ctypes.c_int32 * 1)(0)
    ws = ctypes.c_void_p(256)
    # ps_gns: null pointers, a square shape and a bad iteration count are argument errors
    assert lib.ps_gns(null, 1, 1, 8, 16, 128, 16, 1, null, 1, 1, coeffs, 0, resets, 1e-7, ws, 1 << 20,
                      null) == _native.PS_ERR_INVALID
    assert lib.ps_gns(ws, 1, 1, 16, 16, 256, 16, 1, ws, 1, 1, coeffs, 0, resets, 1e-7, ws, 1 << 20,
                      null) == _native.PS_ERR_INVALID
    assert b"square" in lib.ps_last_error()
    assert lib.ps_gns(ws, 1, 1, 8, 16, 128, 16, 1, ws, 1, 0, coeffs, 0, resets, 1e-7, ws, 1 << 20,
                      null) == _native.PS_ERR_INVALID
    # ps_update_stats: null outputs, an empty batch and FP64 (not an update type) are argument errors
    assert lib.ps_update_stats(ws, _native.PS_F16, 2, 64, null, ws, ws, null) == _native.PS_ERR_INVALID
    assert b"null" in lib.ps_last_error()
    assert lib.ps_update_stats(ws, _native.PS_F16, 0, 64, ws, ws, ws, null) == _native.PS_ERR_INVALID
    assert lib.ps_update_stats(ws, _native.PS_F64, 2, 64, ws, ws, ws, null) == _native.PS_ERR_INVALID
    assert b"FP16, BF16 or FP32" in lib.ps_last_error()


def test_struct_layouts_match_header():
    # ps_step: 3 x int32 + 3 x float; ps_problem: pointers and int64 fields
    assert ctypes.sizeof(_native.PsStep) == 24
    assert ctypes.sizeof(_native.PsProblem) == 8 + 8 + 6 * 8 + 8 + 8
    # ps_update: pointer, int32 dtype, two floats (padded to 8-byte alignment)
    assert ctypes.sizeof(_native.PsUpdate) == 24


def test_host_side_knobs_round_trip_without_gpu():
    """Kernel-selection and scheduling knobs are host state: they validate their
    argument and return the previous setting, with no device present."""
    lib = _native.load()
    assert lib.ps_set_cta_pairs(3) == _native.PS_ERR_INVALID
    assert lib.ps_set_cta_pairs(-1) == _native.PS_ERR_INVALID
    prev = lib.ps_set_cta_pairs(2)
    assert prev == 1  # default: CTA pairs for every product
    assert lib.ps_set_cta_pairs(0) == 2
    assert lib.ps_set_cta_pairs(prev) == 0
    assert lib.ps_set_max_ctas(-5) == _native.PS_ERR_INVALID
    assert lib.ps_set_max_ctas(100) == 0
    assert lib.ps_set_max_ctas(0) == 100


def test_public_header_compiles_cleanly_as_c_and_cpp(tmp_path):
    """The ABI header is included by C and C++ consumers: it must compile with
    -Wall -Wextra -Werror in both languages (a stray comment opener inside a
    comment, for one, trips -Wcomment)."""
    import shutil
    import subprocess
    src = tmp_path / "use_header.c"
    src.write_text('#include "polar_switch_b200.h"\nint main(void) { return PS_OK; }\n')
    inc = os.path.join(ROOT, "include")
    for cc, extra in (("gcc", []), ("g++", ["-x", "c++"])):
        if shutil.which(cc) is None:
            continue
        r = subprocess.run([cc, "-Wall", "-Wextra", "-Werror", *extra, "-I", inc, "-c", str(src),
                            "-o", str(tmp_path / f"o_{cc}.o")], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_chain_knob_and_selftest_arguments_without_gpu():
    lib = _native.load()
    assert lib.ps_set_chain(2) == _native.PS_ERR_INVALID
    assert lib.ps_set_chain(-1) == _native.PS_ERR_INVALID
    prev = lib.ps_set_chain(0)
    assert prev == 1  # default: chain launches on
    assert lib.ps_set_chain(prev) == 0
    null = ctypes.c_void_p(0)
    assert lib.ps_selftest_chain_wait(null, 1 << 20, 1000, null) == _native.PS_ERR_INVALID
    assert lib.ps_selftest_chain_wait(ctypes.c_void_p(256), 1024, 1000, null) == _native.PS_ERR_WORKSPACE
    assert lib.ps_selftest_chain_wait(ctypes.c_void_p(256), 1 << 20, 0, null) == _native.PS_ERR_INVALID


def test_fused_normalize_knob_without_gpu():
    lib = _native.load()
    assert lib.ps_set_fused_normalize(2) == _native.PS_ERR_INVALID
    prev = lib.ps_set_fused_normalize(1)
    assert prev == 0  # default: two passes
    assert lib.ps_set_fused_normalize(prev) == 1


def test_circuit_kernel_knob_without_gpu():
    lib = _native.load()
    assert lib.ps_set_circuit_kernel(2) == _native.PS_ERR_INVALID
    prev = lib.ps_set_circuit_kernel(1)
    assert prev in (0, 1)
    assert lib.ps_set_circuit_kernel(prev) == 1


def test_push_arguments_without_gpu():
    """ps_circuit_grouped_push rejects bad peer lists and phase tables before
    touching a device."""
    lib = _native.load()
    null = ctypes.c_void_p(0)
    ws = ctypes.c_void_p(256)
    probs = (_native.PsProblem * 2)(
        _native.PsProblem(256, _native.PS_F32, 4, 256, 128, 256 * 128, 128, 1, 512, _native.PS_F16),
        _native.PsProblem(256, _native.PS_F32, 3, 128, 128, 128 * 128, 128, 1, 1024, _native.PS_F16))
    res = (ctypes.c_float * 1)(0.0)
    nst = (ctypes.c_int32 * 1)(1)
    steps = (_native.PsStep * 1)(_native.PsStep(1, 0, 0, 1.0, 0.0, 0.0))
    peers = (ctypes.c_void_p * 8)(*([4096] * 8))

    def call(n_peers, n_phases, ends, peer_list=peers, local=ws):
        return lib.ps_circuit_grouped_push(probs, 2, 1, res, nst, steps, 2, 1e-7, ws, 1 << 20, local,
                                           peer_list, n_peers, n_phases, ends, null)

    assert call(8, 1, None) == _native.PS_ERR_INVALID
    assert b"n_peers" in lib.ps_last_error()
    assert call(-1, 1, None) == _native.PS_ERR_INVALID
    assert call(1, 1, None, local=null) == _native.PS_ERR_INVALID
    odd = (ctypes.c_void_p * 1)(4097)
    assert call(1, 1, None, peer_list=odd) == _native.PS_ERR_INVALID
    assert b"misaligned" in lib.ps_last_error()
    assert call(1, 0, None) == _native.PS_ERR_INVALID
    assert call(1, 9, None) == _native.PS_ERR_INVALID
    assert call(1, 2, None) == _native.PS_ERR_INVALID
    bad_end = (ctypes.c_int32 * 4)(2, 3, 1, 3)   # problem 0 ends at 3, not its L = 4
    assert call(1, 2, bad_end) == _native.PS_ERR_INVALID
    assert b"phase_ends" in lib.ps_last_error()
    decreasing = (ctypes.c_int32 * 4)(3, 4, 2, 1)
    assert call(1, 2, decreasing) == _native.PS_ERR_INVALID
