"""B200-native Parallel Layer Migration: distil every full-attention block of a
frozen Qwen3.5-family hybrid teacher into an independent RWKV7 TimeMix student.

Subpackages: ``models`` (teacher, student, runner, checkpoint IO), ``ops``
(CUDA-kernel operators with PyTorch oracles), ``parallel`` (topology and the
peer-memory gradient exchange), ``convert`` (manifest writer, Lightning PTH
export). The compiled kernels are the in-tree extension ``_C``.
"""
__version__ = "0.1.0"
