"""Operator layer: every hot op has one CUDA implementation (sm_100a, in the
in-tree extension ``rwkv_theseus_b200._C``) and one plain PyTorch definition
(``ops.reference``) that serves as the CPU path for Gloo tests and as the fp32
oracle in numerics tests. Tensors on a CUDA device always take the extension;
if it is missing there, ``native()`` raises instead of falling back.
"""
import importlib

_NATIVE = None
_ERROR = None


def native():
    """Return the compiled extension module, raising if it cannot be imported."""
    global _NATIVE, _ERROR
    if _NATIVE is None:
        import torch  # noqa: F401  (loads libc10/libtorch before the extension)
        try:
            _NATIVE = importlib.import_module("rwkv_theseus_b200._C")
        except ImportError as exc:  # pragma: no cover - depends on the build
            _ERROR = exc
            raise RuntimeError(
                "rwkv_theseus_b200._C is not built; run `python setup.py build_ext --inplace` "
                "(or __graft_entry__.build()) before using CUDA tensors") from exc
    return _NATIVE


def available():
    try:
        native()
        return True
    except RuntimeError:
        return False
