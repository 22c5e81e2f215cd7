"""Test-only stand-in for lmcache.v1.distributed.serde.async_processor:
worker-thread processor with submit_* / query_*_result (None while pending,
True on success, False on failure), as exercised by
test_native_async_serde.py:189-289."""

import itertools
import threading
from concurrent.futures import ThreadPoolExecutor

from .base import SerdeProcessor


class AsyncSerdeProcessor(SerdeProcessor):
    def __init__(self, serializer, deserializer, max_workers: int = 1):
        self.serializer = serializer
        self.deserializer = deserializer
        self._pool = ThreadPoolExecutor(max_workers=max(1, int(max_workers)))
        self._ids = itertools.count(1)
        self._tasks = {}
        self._lock = threading.Lock()

    def estimate_serialized_size(self, layout_desc) -> int:
        return self.serializer.estimate_serialized_size(layout_desc)

    def _submit(self, fn, srcs, dsts, keys):
        def run():
            for s, d, k in zip(srcs, dsts, keys, strict=True):
                fn(s, d, k)
            return True

        tid = next(self._ids)
        with self._lock:
            self._tasks[tid] = self._pool.submit(run)
        return tid

    def _query(self, tid):
        with self._lock:
            fut = self._tasks.get(tid)
        if fut is None or not fut.done():
            return None
        with self._lock:
            self._tasks.pop(tid, None)
        return fut.exception() is None

    def submit_serialize(self, srcs, dsts, keys):
        return self._submit(self.serializer.serialize, srcs, dsts, keys)

    def submit_deserialize(self, srcs, dsts, keys):
        return self._submit(self.deserializer.deserialize, srcs, dsts, keys)

    def query_serialize_result(self, tid):
        return self._query(tid)

    def query_deserialize_result(self, tid):
        return self._query(tid)

    def close(self):
        self._pool.shutdown(wait=True)
