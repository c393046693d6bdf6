"""msgl -- Python access to libmsgl, the sm_100a kernels of the mini-sglang-cpp Qwen3 path.

``msgl.lib()`` returns the ctypes handle of the in-tree ``libmsgl.so`` (it raises if the library
is missing: there is no fallback). ``msgl.ops`` wraps each C-ABI entry point for torch CUDA
tensors (device memory and the current stream come from torch; all compute is libmsgl's).
"""
from ._lib import LIB_PATH, MsglError, check, header_symbols, lib  # noqa: F401
