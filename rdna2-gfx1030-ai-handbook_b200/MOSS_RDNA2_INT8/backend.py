"""Production MOSS INT8 eager export on B200 (drop-in for the reference's
production/MOSS_RDNA2_INT8/backend.py:1-204).

The same public functions and install protocol as rdna2_ops.comfy_int8,
with this module's own installation state and statistics (the reference
also keeps two independent copies).  The linear runs on the library's
rotation + quantize prologue and tcgen05 INT8 GEMM with the Kitchen
epilogue order (x_scale * w_scale, cast, then + bias in the output dtype).
"""
from rdna2_ops.comfy_int8 import KitchenInt8Binding, module_api

_binding = KitchenInt8Binding()
(int8_linear, install_backend, disable_backend, get_stats, reset_stats,
 _scoped) = module_api(_binding)
