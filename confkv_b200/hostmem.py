"""Pinned host memory that device code can address directly.

Under unified virtual addressing, memory from cudaHostAlloc (torch's
`pin_memory=True`) is mapped into every device's address space at the same
address, so a seal can write its frame straight into host memory: the
ciphertext crosses the host link while it is being produced and no separate
device-to-host copy follows. `device_mapped` checks that property on the
host before such a pointer is handed to a kernel.
"""

from __future__ import annotations


def device_mapped(ptr: int) -> bool:
    """True when `ptr` is host memory that device code reaches at the same
    address (cudaPointerGetAttributes: host type, devicePointer == ptr)."""
    try:
        from cuda.bindings import runtime as rt
    except ImportError:
        return False
    err, attr = rt.cudaPointerGetAttributes(ptr)
    if err != rt.cudaError_t.cudaSuccess:
        return False
    return attr.type == rt.cudaMemoryType.cudaMemoryTypeHost and int(attr.devicePointer) == int(ptr)
