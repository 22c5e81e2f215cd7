"""Batched seal / open of many device objects in one call each.

Wraps lmcache_gpu_aes128gcm_{seal,open}_batch_async (an extension of the
reference ABI: its callers enqueue one seal_async / open_async per object).
`DeviceBatch` owns the device descriptor array, the workspace and a pinned
staging buffer for up to `capacity` objects; torch supplies the memory and
the stream, the library does the work.

    batch = DeviceBatch(lib, capacity=4096, device=0)
    batch.seal(key, [(src_ptr, frame_ptr, P, frame_capacity, iv), ...], stream)
    batch.open(key, [(frame_ptr, out_ptr, P, frame_len, auth_ptr), ...], stream)
    batch.statuses()   # int32 per object on the device: 0 or -1 (skipped)
    batch.fault()      # device int32: nonzero if a work kernel gave up a bounded wait
"""

from __future__ import annotations

import torch

from .gpu_aesgcm import BatchItem, GpuAes128GcmKey, GpuAesGcmLibrary, pack_batch_items

ITEM_BYTES = 64
STATUS_OFFSET = BatchItem.status.offset
FAULT_OFFSET = 28   # LMCACHE_GPU_AESGCM_BATCH_FAULT_OFFSET: uint32 in the workspace


class DeviceBatch:
    def __init__(self, library: GpuAesGcmLibrary, capacity: int, device: int | torch.device = 0):
        if capacity <= 0:
            raise ValueError("capacity must be positive")
        self.library = library
        self.capacity = int(capacity)
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.workspace_bytes = library.batch_workspace_size(self.capacity)
        if self.workspace_bytes == 0:
            raise ValueError("batch capacity above the library limit")
        self.workspace = torch.empty(self.workspace_bytes, dtype=torch.uint8, device=self.device)
        self.items = torch.empty(self.capacity * ITEM_BYTES, dtype=torch.uint8, device=self.device)
        self._staging = torch.empty(self.capacity * ITEM_BYTES, dtype=torch.uint8, pin_memory=True)
        self._copied = None   # event after the last descriptor upload
        self.count = 0

    def _upload(self, entries, stream: torch.cuda.Stream) -> int:
        raw = pack_batch_items(entries)
        count = len(raw) // ITEM_BYTES
        if count > self.capacity:
            raise ValueError(f"{count} objects exceed the batch capacity {self.capacity}")
        if self._copied is not None:
            self._copied.synchronize()   # the staging buffer is free again
        if count:
            self._staging[:len(raw)].copy_(torch.frombuffer(bytearray(raw), dtype=torch.uint8))
            with torch.cuda.stream(stream):
                self.items[:len(raw)].copy_(self._staging[:len(raw)], non_blocking=True)
                self._copied = torch.cuda.Event()
                self._copied.record(stream)
        self.count = count
        return count

    def seal(self, key: GpuAes128GcmKey, entries, stream: torch.cuda.Stream | None = None) -> None:
        """entries: (src_ptr, dst_ptr, plaintext_len, dst_capacity, iv) per object."""
        stream = stream or torch.cuda.current_stream(self.device)
        count = self._upload(((s, d, p, c, 0, iv) for s, d, p, c, iv in entries), stream)
        key.seal_batch_async(items_ptr=self.items.data_ptr(), count=count, workspace_ptr=self.workspace.data_ptr(),
                             workspace_bytes=self.workspace_bytes, stream_ptr=stream.cuda_stream)

    def open(self, key: GpuAes128GcmKey, entries, stream: torch.cuda.Stream | None = None) -> None:
        """entries: (frame_ptr, dst_ptr, plaintext_len, frame_len, auth_ok_ptr) per object."""
        stream = stream or torch.cuda.current_stream(self.device)
        count = self._upload(((f, d, p, fl, a, None) for f, d, p, fl, a in entries), stream)
        key.open_batch_async(items_ptr=self.items.data_ptr(), count=count, workspace_ptr=self.workspace.data_ptr(),
                             workspace_bytes=self.workspace_bytes, stream_ptr=stream.cuda_stream)

    def statuses(self) -> torch.Tensor:
        """Per-object status of the last call (int32, device): 0 or -1."""
        view = self.items[:self.count * ITEM_BYTES].view(self.count, ITEM_BYTES)
        return view[:, STATUS_OFFSET:STATUS_OFFSET + 4].contiguous().view(torch.int32).reshape(-1)

    def fault(self) -> torch.Tensor:
        """Fault word of the last call (int32, device): 0 unless a work kernel
        gave up on one of its bounded internal waits (outputs then invalid)."""
        return self.workspace[FAULT_OFFSET:FAULT_OFFSET + 4].view(torch.int32).reshape(())
