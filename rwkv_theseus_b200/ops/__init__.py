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


def f32(t):
    """fp32 contiguous copy of a (frozen) parameter, cached on the tensor and refreshed when it is modified
    in place; fp32 inputs pass through. Keeps per-call dtype conversions of small weights off the GPU."""
    import torch
    if t.dtype == torch.float32 and t.is_contiguous():
        return t
    cached = getattr(t, "_rt_f32", None)
    if cached is None or cached[0] != t._version:
        cached = (t._version, t.detach().float().contiguous())
        t._rt_f32 = cached
    return cached[1]

