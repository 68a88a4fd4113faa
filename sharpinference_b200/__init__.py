"""sharpinference_b200: B200 (sm_100a) backend for SharpInference's quantized
mat-vec / matrix-multiply instructions.

The product is the native library libsharpinfer_cuda.so (C ABI declared in
include/sharpinfer_cuda.h); `native` is its ctypes binding. Importing the
package requires the built library; there is no CPU fallback.
"""
from . import native  # noqa: F401
from .native import (F16, F32, I32, Q4_K, Q8_0, Context, Buffer, SiError, ArgumentError, NotSupportedError,  # noqa: F401
                     InstructionAdaptationError, InvalidDataError, CudaError)

__all__ = ["native", "Context", "Buffer", "F32", "F16", "Q8_0", "Q4_K", "I32", "SiError", "ArgumentError",
           "NotSupportedError", "InstructionAdaptationError", "InvalidDataError", "CudaError"]
