"""B200-native AES-128-GCM seal/open engine for persistent KV-cache objects.

Drop-in for ConfKV's GPU seal path: the C-ABI in ``include/gpu_aesgcm_api.h``
(built in-tree as ``libgpu_aesgcm.so``) and the ctypes binding in
``confkv_b200.gpu_aesgcm`` with the reference's class names.
"""

from .gpu_aesgcm import (  # noqa: F401
    FRAME_OVERHEAD,
    IV_LEN,
    KEY_LEN,
    GpuAes128GcmKey,
    GpuAesGcmError,
    GpuAesGcmLibrary,
)
