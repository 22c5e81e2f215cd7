"""Device-buffer helpers for the GPU tests: every call goes through the C-ABI
via the ctypes binding (confkv_b200.gpu_aesgcm); torch only supplies device
memory and streams."""

from __future__ import annotations

import numpy as np
import torch

from confkv_b200.gpu_aesgcm import GpuAes128GcmKey


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def dev_bytes(data, offset: int = 0, extra: int = 0, fill: int = 0xCC) -> tuple[torch.Tensor, int]:
    """Copy `data` to the device at byte `offset` of a fresh buffer; returns
    (buffer, address of the first byte)."""
    arr = np.array(np.frombuffer(bytes(data), dtype=np.uint8)) if not isinstance(data, np.ndarray) \
        else np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    buf = torch.full((offset + arr.size + extra + 16,), fill, dtype=torch.uint8, device="cuda")
    if arr.size:
        buf[offset:offset + arr.size].copy_(torch.from_numpy(np.ascontiguousarray(arr)))
    return buf, buf.data_ptr() + offset


class GpuKey:
    def __init__(self, lib, key: bytes, device: int = 0):
        self.key = GpuAes128GcmKey(lib, key, device=device)
        self.stream = torch.cuda.Stream(device=device)

    def close(self):
        self.key.close()

    def seal(self, pt, iv: bytes, src_off: int = 0, dst_off: int = 0) -> bytes:
        pt_arr = np.frombuffer(bytes(pt), np.uint8) if not isinstance(pt, np.ndarray) else pt.view(np.uint8).reshape(-1)
        size = pt_arr.size
        src, src_ptr = dev_bytes(pt_arr, src_off)
        dst = torch.full((dst_off + size + 29 + 16,), 0xAB, dtype=torch.uint8, device="cuda")
        torch.cuda.current_stream().synchronize()
        self.key.seal_async(src_ptr=src_ptr, plaintext_len=size, dst_ptr=dst.data_ptr() + dst_off,
                            dst_capacity=size + 29, iv=iv, stream_ptr=self.stream.cuda_stream)
        self.stream.synchronize()
        out = to_host(dst)
        # bytes outside the frame must be untouched
        assert (out[:dst_off] == 0xAB).all() and (out[dst_off + size + 29:] == 0xAB).all()
        return out[dst_off:dst_off + size + 29].tobytes()

    def seal_tensor(self, src: torch.Tensor, iv: bytes, dst: torch.Tensor) -> None:
        nbytes = src.numel() * src.element_size()
        self.key.seal_async(src_ptr=src.data_ptr(), plaintext_len=nbytes, dst_ptr=dst.data_ptr(),
                            dst_capacity=dst.numel(), iv=iv, stream_ptr=self.stream.cuda_stream)

    def open(self, frame: bytes, plen: int, frame_off: int = 0, dst_off: int = 0, pad: int = 0) -> tuple[int, bytes]:
        fr = bytes(frame) + b"\xee" * pad
        src, src_ptr = dev_bytes(fr, frame_off)
        dst = torch.full((dst_off + plen + 16,), 0xCC, dtype=torch.uint8, device="cuda")
        auth = torch.full((1,), 7, dtype=torch.int32, device="cuda")
        torch.cuda.current_stream().synchronize()
        self.key.open_async(src_ptr=src_ptr, frame_len=len(fr), dst_ptr=dst.data_ptr() + dst_off,
                            plaintext_len=plen, auth_ok_ptr=auth.data_ptr(), stream_ptr=self.stream.cuda_stream)
        self.stream.synchronize()
        out = to_host(dst)
        assert (out[:dst_off] == 0xCC).all() and (out[dst_off + plen:] == 0xCC).all()
        return int(auth.item()), out[dst_off:dst_off + plen].tobytes()
