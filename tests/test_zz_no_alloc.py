"""The allocation-free split-K GEMM entry point (collected last on purpose).

``ic_gemm_a8_splitk_noalloc`` serves callers that cannot allocate device
memory while they run the GEMM -- a C or FFI host with no device allocator of
its own, a process whose device memory is already reserved by another
framework's pool, or a path where cudaMalloc is not allowed because it can
synchronise the device.  It keeps its split-K partials in a scratch array built
into the library instead of a caller workspace.

These tests call it through the C ABI and compare it with ``ic_gemm_a8_splitk``
(the same kernels with a torch-allocated workspace) on two calls in a row with
different inputs and shapes, so that a result left in the shared scratch by the
first call cannot hide a wrong second result.  They pass alone in a fresh
process (the first call sets up the scratch address) and after every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

import intcrush_oracle as O
from _pkg import load

L = load("_lib")

SCRATCH_FLOATS = 2097152   # IC_NOALLOC_SCRATCH_FLOATS in include/intcrush_b200.h


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _case(M, N, K, G, int4, seed, dev):
    rng = np.random.default_rng(seed)
    xq = rng.integers(-128, 128, (M, K)).astype(np.int8)
    wq = rng.integers(-8, 8, (N, K)).astype(np.int8) if int4 else rng.integers(-127, 128, (N, K)).astype(np.int8)
    w = O.pack_int4(wq) if int4 else wq
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return dict(xq=t(xq), w=t(w), s_w=t(rng.uniform(1e-3, 2e-2, (N, G)).astype(np.float32)),
                s_a=t(rng.uniform(1e-3, 5e-2, M).astype(np.float32)),
                bias=t((rng.standard_normal(N) * 0.02).astype(np.float16)), G=G, M=M, N=N, K=K,
                kind=L.IC_W_INT4 if int4 else L.IC_W_INT8)


def _call(c, splits, noalloc, stream):
    lib = L.lib()
    M, N, K, G = c["M"], c["N"], c["K"], c["G"]
    out = torch.empty(M, N, dtype=torch.float16, device=c["xq"].device)
    args = [_p(c["xq"]), M, K, c["xq"].stride(0), _p(c["w"]), c["kind"], N, c["w"].stride(0), _p(c["s_w"]), G,
            K // G if G > 1 else K, _p(c["s_a"]), _p(c["bias"]), L.IC_DTYPE_F16, None, None, _p(out),
            L.IC_DTYPE_F16, N, splits]
    if noalloc:
        st = lib.ic_gemm_a8_splitk_noalloc(*args, stream)
    else:
        ws = torch.empty(splits * M * N, dtype=torch.float32, device=out.device)
        st = lib.ic_gemm_a8_splitk(*args, _p(ws), ws.numel(), stream)
    return st, out


@pytest.mark.gpu
def test_noalloc_splitk_matches_workspace_entry_two_calls():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    # first call: W4A8 group scales, 4 parts; second: W8A8 per channel, 3 parts,
    # other sizes, so the scratch holds the first call's partials when it starts
    cases = [(_case(24, 640, 3072, 24, True, 1, dev), 4), (_case(7, 1152, 1536, 1, False, 2, dev), 3)]
    for c, splits in cases:
        st_a, out_a = _call(c, splits, noalloc=True, stream=stream)
        st_b, out_b = _call(c, splits, noalloc=False, stream=stream)
        torch.cuda.synchronize()
        assert st_a == L.IC_OK and st_b == L.IC_OK, L.lib().ic_last_error()
        ref = out_b.float().cpu().numpy().astype(np.float64)
        assert O.max_rel(out_a.float().cpu().numpy(), ref) <= 1e-6
        assert torch.isfinite(out_a.float()).all()


@pytest.mark.gpu
def test_noalloc_splitk_at_the_scratch_limit():
    """A call whose partials fill the built-in scratch exactly (4 * 64 * 8192 =
    2,097,152 floats) matches the workspace entry point; 65 tokens, one token
    past the limit, are refused."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    c = _case(64, 8192, 1024, 8, True, 5, dev)
    assert 4 * 64 * 8192 == SCRATCH_FLOATS
    for _ in range(2):
        st_a, out_a = _call(c, 4, noalloc=True, stream=stream)
        st_b, out_b = _call(c, 4, noalloc=False, stream=stream)
        torch.cuda.synchronize()
        assert st_a == L.IC_OK and st_b == L.IC_OK, L.lib().ic_last_error()
        assert O.max_rel(out_a.float().cpu().numpy(), out_b.float().cpu().numpy().astype(np.float64)) <= 1e-6
    over = _case(65, 8192, 1024, 8, True, 6, dev)
    st, _ = _call(over, 4, noalloc=True, stream=stream)
    assert st == L.IC_ERR_ARG
    assert b"exceeds the built-in scratch" in L.lib().ic_last_error()


def test_noalloc_splitk_rejects_oversize_before_any_work():
    """splits * M * N above the built-in scratch is refused up front (no GPU
    work is queued, so this runs without a device too)."""
    lib = L.lib()
    M, N, splits = 1024, 4096, 2          # 8 Mi floats > 2 Mi
    assert splits * M * N > SCRATCH_FLOATS
    st = lib.ic_gemm_a8_splitk_noalloc(ctypes.c_void_p(16), M, 3072, 3072, ctypes.c_void_p(16), L.IC_W_INT8, N,
                                       3072, ctypes.c_void_p(16), 1, 3072, ctypes.c_void_p(16), None, 0, None,
                                       None, ctypes.c_void_p(16), L.IC_DTYPE_F16, N, splits, None)
    assert st == L.IC_ERR_ARG
    assert b"exceeds the built-in scratch" in L.lib().ic_last_error()
