"""B200 (sm_100a) FP8 E4M3 quantized-linear hot path of listenflow-fastest-whisper.

The package directory name is not a Python identifier; import it with
``importlib.import_module("listenflow-fastest-whisper_b200")``.

Modules:
  _native  ctypes binding of liblffw_b200.so (include/lffw_fp8.h)
  fp8      Q/DQ linear host API mirroring the reference's _Fp8Graph, plus the
           LayerNorm, attention and fp16 plugin calls; the TensorRT plugin
           creators are restated in the C ABI itself (lffw_plugin_*)
  scales   the reference's FP8 activation-scale file loader
  replicas one process per GPU: rank environment, batch shards, max-over-ranks
  build    in-tree nvcc build of liblffw_b200.so
"""

from . import _native  # noqa: F401
from ._native import NativeError, bundle_sha256, launch_count  # noqa: F401

__all__ = ["NativeError", "bundle_sha256", "launch_count"]
