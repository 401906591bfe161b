"""Python mirror of the lrrt interfaces on B200 (ctypes over the C ABIs).

``runtime`` wraps the lr_* calls (light-rocm-runtime include/lrrt/lrrt.h);
``qwen`` wraps the Qwen2 FP32 resident decode driver (include/lrrt_qwen.h).
The compute path is the sm_100a cubin loaded through lr_module_load_hsaco; this
package only moves arguments across the C ABI.
"""
from .native import LrrtError, check, driver, runtime  # noqa: F401
