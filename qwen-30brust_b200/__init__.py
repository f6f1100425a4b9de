"""B200-native decode engine for Qwen3-MoE GGUF models.

The directory name is not a Python identifier, so the package is loaded by path
and registered as ``qwen30brust_b200`` (``__graft_entry__.load_package()``).

Submodules:
  engine  ctypes bindings of the C ABI in include/qwen_cuda.h (libqwen_cuda.so)
  tools   quantizers and synthetic GGUF images (libqwen_tools.so)
  build   nvcc / g++ recipes for both libraries
"""
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
