"""B200-native GGUF weight preparation (dequantize + requantize) for LLiMa.

The CUDA kernels live in ``llima_b200/lib/libgguf_b200.so`` (built by
``llima_b200/build.py``) and are reached through the C ABI declared in
``include/gguf_b200.h``.  Importing this package does not touch the GPU; the
library is loaded on first use and a missing or unloadable library raises.
"""
__version__ = "0.1.0"
