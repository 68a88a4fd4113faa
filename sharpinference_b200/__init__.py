"""sharpinference_b200: B200 (sm_100a) backend for SharpInference's quantized
mat-vec / matrix-multiply instructions.

The product is the native library libsharpinfer_cuda.so (C ABI declared in
include/sharpinfer_cuda.h); `native` is its ctypes binding. Using the
package requires the built library and raises ImportError without it — there
is no CPU fallback. `sharpinference_b200.build` (the in-tree build step) is
importable before the library exists.
"""
from importlib import import_module

_EXPORTS = ("Context", "Buffer", "F32", "F16", "Q8_0", "Q4_K", "I32", "SiError", "ArgumentError", "NotSupportedError",
            "InstructionAdaptationError", "InvalidDataError", "CudaError")

__all__ = ["native", *_EXPORTS]


def __getattr__(name):
    if name == "native":
        return import_module(".native", __name__)
    if name in _EXPORTS:
        return getattr(import_module(".native", __name__), name)
    raise AttributeError(name)
