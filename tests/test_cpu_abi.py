"""The C-ABI library loads without a GPU, exports every entry point declared
in include/intcrush_b200.h, and rejects bad arguments before touching CUDA."""

import ctypes
import os
import re

import pytest

from _pkg import load

L = load("_lib")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "intcrush_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ic_\w+)\s*\(", src, flags=re.M)))


def test_library_loads_and_exports_all_declared_symbols():
    lib = L.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared but not exported"
    assert set(names) <= set(L.SIGNATURES), "every declared entry point has a ctypes signature"


def test_version():
    assert L.lib().ic_version() >> 16 == 1


@pytest.mark.parametrize("call,code", [
    (lambda l: l.ic_gemm_a8(None, 4, 64, 64, None, 7, 8, 32, None, 1, 64, None, None, 0, None, None, None, 0, 8,
                            None), L.IC_ERR_ARG),
    (lambda l: l.ic_prep_quant(None, 9, 4, 64, 64, None, 0, 64, None, None, None, 0, None, None, None, None),
     L.IC_ERR_ARG),
    (lambda l: l.ic_prep_quant(ctypes.c_void_p(16), 0, 4, 64, 64, None, 48, 64, None, None, None, 0, None, None,
                               None, None), L.IC_ERR_ARG),
    (lambda l: l.ic_gemm_w4a16(None, 2, 4, 64, 64, None, 8, 32, 0, None, 0, 1, 64, None, 0, None, None, 0, 1.0,
                               None, 8, None), L.IC_ERR_UNSUPPORTED),
    (lambda l: l.ic_repack_int4(None, 4, 64, 32, None, 32, 5, None), L.IC_ERR_ARG),
    (lambda l: l.ic_lowrank_add(None, 4, 8, 8, None, None, 512, 1.0, None), L.IC_ERR_UNSUPPORTED),
    (lambda l: l.ic_lowrank_add_ex(None, 2, 4, 8, 8, None, None, 16, 1.0, None), L.IC_ERR_ARG),
    (lambda l: l.ic_lowrank_down_ex(None, 2, 4, 8, 8, None, 16, None, None), L.IC_ERR_ARG),
])
def test_argument_validation_without_gpu(call, code):
    lib = L.lib()
    assert call(lib) == code
    assert lib.ic_last_error().decode()


def _gemm_a8_args(K, G, group_size, w_kind=None):
    f = ctypes.c_void_p(256)   # aligned stand-in pointers: validation fails before any use
    return [f, 64, K, K, f, L.IC_W_INT4 if w_kind is None else w_kind, 128, K // 2, f, G, group_size, f, None, 0,
            None, None, f, L.IC_DTYPE_F16, 128, None]


@pytest.mark.parametrize("K,G,gs", [(1024, 2, 512), (2048, 2, 1024)])
def test_int4_group_scales_wider_than_256_rejected(K, G, gs):
    """A 512-wide INT4 group's int32 partial can exceed the exact range of
    the kernel's int -> float hand-off, so group_size > 256 is refused."""
    lib = L.lib()
    assert lib.ic_gemm_a8(*_gemm_a8_args(K, G, gs)) == L.IC_ERR_UNSUPPORTED
    assert b"group_size 128 or 256" in lib.ic_last_error()


def test_partial_last_group_rejected():
    """K = 640 with 256-wide groups leaves a half group at the end (G = 3):
    the kernel's accumulation units must be whole groups, so it is refused."""
    lib = L.lib()
    assert lib.ic_gemm_a8(*_gemm_a8_args(640, 3, 256)) == L.IC_ERR_UNSUPPORTED
    assert b"multiple of group_size / 128" in lib.ic_last_error()


def test_workspace_size_check_does_not_overflow():
    """splits * M * N = 16 * 2^30 * 2^30 wraps int64 to 0; it is still refused."""
    lib = L.lib()
    f = ctypes.c_void_p(256)
    M = N = 1 << 30
    st = lib.ic_gemm_a8_splitk(f, M, 2048, 2048, f, L.IC_W_INT8, N, 2048, f, 1, 2048, f, None, 0, None, None, f,
                               L.IC_DTYPE_F16, N, 16, f, 16, None)
    assert st in (L.IC_ERR_ARG, L.IC_ERR_UNSUPPORTED)
    assert lib.ic_last_error()


def test_zero_sized_calls_are_no_ops():
    lib = L.lib()
    assert lib.ic_prep_quant(None, 0, 0, 64, 64, None, 0, 64, None, None, None, 0, None, None, None, None) == L.IC_OK
    assert lib.ic_unpack_int4_to_int8(None, 0, 64, 32, None, None) == L.IC_OK


def _gemm_ex_args(act=0, residual=None, residual_dtype=0, ldr=0):
    f = ctypes.c_void_p(256)
    return [f, 64, 256, 256, f, L.IC_W_INT8, 128, 256, f, 1, 256, f, None, 0, None, None, act, residual,
            residual_dtype, ldr, f, L.IC_DTYPE_F16, 128, 1, None, 0, None]


def test_gemm_epilogue_arguments_validated():
    lib = L.lib()
    assert lib.ic_gemm_a8_ex(*_gemm_ex_args(act=4)) == L.IC_ERR_ARG
    assert b"activation" in lib.ic_last_error()
    f = ctypes.c_void_p(256)
    assert lib.ic_gemm_a8_ex(*_gemm_ex_args(residual=f, residual_dtype=L.IC_DTYPE_F16, ldr=64)) == L.IC_ERR_ARG
    assert lib.ic_gemm_a8_ex(*_gemm_ex_args(residual=f, residual_dtype=9, ldr=128)) == L.IC_ERR_ARG


def test_int8out_workspace_and_output_checks():
    lib = L.lib()
    f = ctypes.c_void_p(256)
    base = [f, 64, 256, 256, f, L.IC_W_INT8, 128, 256, f, 1, 256, f, None, 0, 0]
    # workspace must hold M*N values plus M row maxima
    assert lib.ic_gemm_a8_int8out(*base, f, 128, f, f, 64 * 128, None) == L.IC_ERR_ARG
    assert b"M*N + M" in lib.ic_last_error()
    assert lib.ic_gemm_a8_int8out(*base, f, 64, f, f, 64 * 129, None) == L.IC_ERR_ARG   # ldc < N
    assert lib.ic_gemm_a8_int8out(*base, None, 128, f, f, 64 * 129, None) == L.IC_ERR_ARG
    zero = [f, 0] + base[2:]
    assert lib.ic_gemm_a8_int8out(*zero, f, 128, f, f, 0, None) == L.IC_OK


def test_weight_requant_and_lokr_validation():
    lib = L.lib()
    f = ctypes.c_void_p(256)
    assert lib.ic_quantize_weight(f, 4, 64, 64, 3, f, 32, f, None) == L.IC_ERR_ARG
    assert lib.ic_quantize_weight(f, 4, 64, 64, 4, f, 31, f, None) == L.IC_ERR_ARG     # ldq < ceil(K/2)
    assert lib.ic_quantize_weight(f, 4, 64, 64, 8, f, 32, f, None) == L.IC_ERR_ARG     # ldq < K
    assert lib.ic_quantize_weight(None, 0, 64, 64, 8, None, 64, None, None) == L.IC_OK
    # out_l * out_k must be N and in_m * in_n must be K
    assert lib.ic_lokr_add(f, L.IC_DTYPE_F16, 4, 100, f, 64, 64, f, 4, 4, f, 24, 16, 1.0, f, 1 << 20,
                           None) == L.IC_ERR_ARG
    assert lib.ic_lokr_add(f, L.IC_DTYPE_F16, 4, 96, f, 512, 512, f, 4, 1, f, 24, 512, 1.0, f, 1 << 20,
                           None) == L.IC_ERR_UNSUPPORTED   # in_n > 256
    assert lib.ic_lokr_add(f, L.IC_DTYPE_F16, 4, 96, f, 64, 64, f, 4, 4, f, 24, 16, 1.0, f, 10,
                           None) == L.IC_ERR_ARG            # temp too small
