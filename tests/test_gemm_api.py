"""Argument checks of the GEMM C entry points, which run on the host before any CUDA call (so they need the built
extension but no GPU): out-of-range problem counts, null and misaligned operands, bad strides, an unknown issue
lane and an unknown SwiGLU tile choice all return cudaErrorInvalidValue (1); empty problems return success."""
import ctypes
import glob
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INVALID = 1  # cudaErrorInvalidValue


@pytest.fixture(scope="module")
def lib():
    found = glob.glob(os.path.join(ROOT, "rwkv_theseus_b200", "_C*.so"))
    if not found:
        pytest.skip("extension not built")
    import torch  # noqa: F401  (loads the libraries the extension links against)
    handle = ctypes.CDLL(found[0])
    vp, lg, it, fl = ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_float
    handle.rt_gemm_bf16_group.argtypes = [it, ctypes.POINTER(vp), lg, it, ctypes.POINTER(vp), lg, it,
                                          ctypes.POINTER(vp), lg, it, it, it, it, fl, it, vp, vp]
    handle.rt_gemm_bf16_group.restype = it
    handle.rt_gemm_set_lane.argtypes = [it]
    handle.rt_gemm_set_lane.restype = it
    handle.rt_gemm_swiglu_bf16.argtypes = [vp, lg, vp, vp, lg, vp, lg, it, it, it, it, vp, vp]
    handle.rt_gemm_swiglu_bf16.restype = it
    return handle


def _ptrs(*values):
    return (ctypes.c_void_p * len(values))(*values)


def _group(lib, G, A, B, C, lda=64, ldb=64, M=128, N=128, K=64):
    return lib.rt_gemm_bf16_group(G, A, lda, 0, B, ldb, 0, C, N, M, N, K, 0, 1.0, -1, None, None)


def test_group_count_and_pointers_are_checked(lib):
    good = 0x10000  # 16-byte aligned stand-in addresses: every call below returns before using them
    ok3 = _ptrs(good, good + 4096, good + 8192)
    assert _group(lib, 0, ok3, ok3, ok3) == INVALID
    assert _group(lib, 4, _ptrs(*[good] * 4), _ptrs(*[good] * 4), _ptrs(*[good] * 4)) == INVALID
    assert _group(lib, 2, _ptrs(good, None), ok3, ok3) == INVALID            # null A of problem 1
    assert _group(lib, 2, ok3, _ptrs(good, good + 8), ok3) == INVALID        # B of problem 1 not 16-byte aligned
    assert _group(lib, 2, ok3, ok3, _ptrs(good, None)) == INVALID            # null output
    assert _group(lib, 2, ok3, ok3, ok3, lda=60) == INVALID                  # row stride not a multiple of 8
    assert _group(lib, 2, ok3, ok3, ok3, M=0) == 0                           # empty problem: nothing to do


def test_lane_and_swiglu_choice_are_checked(lib):
    assert lib.rt_gemm_set_lane(2) == INVALID
    assert lib.rt_gemm_set_lane(-1) == INVALID
    assert lib.rt_gemm_set_lane(0) == 0
    good = 0x10000
    # an unknown tile choice (only 128 rows, or 256 rows via bit 17, exist)
    assert lib.rt_gemm_swiglu_bf16(good, 64, good, good, 64, good, 128, 256, 128, 64, 256, None, None) == INVALID
    assert lib.rt_gemm_swiglu_bf16(good, 64, good, good + 8, 64, good, 128, 256, 128, 64, -1, None, None) == INVALID
