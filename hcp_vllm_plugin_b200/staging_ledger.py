"""Worker-side bookkeeping of ``HcpRingKvConnector``, in four small parts.

The behaviour is the reference connector's contract
(``hcp_vllm_plugin/ring_connector.py:144-170, 594-604, 939-997``): a staged
prefix chunk stays staged while any in-flight request still reads it; a
request's prefix layers are staged in model order at most a window of layers
ahead of the layer its forward consumed last; a chunk whose ready marker is
absent is looked for again only after the poll interval; a decode-ring
request keeps its ring slot until it finishes.

* :class:`ChunkLedger` - which chunks each request holds, and the count of
  holders per chunk; the last holder's release drops the chunk's staging.
* :class:`LayerFeed` - one request's staging thread and the per-layer
  hand-off to the forward.
* :class:`ReadinessCache` - ready-marker lookups, rate-limited per chunk.
* :class:`DecodeSlotPool` - the decode ring's request slots.
"""

from __future__ import annotations

import os
import threading
import time
from collections import Counter, deque
from typing import Any, Callable

from .ring_backend import drop_chunk_kv, map_request_peer, unmap_request_peer


class ChunkLedger:
    """Holds of in-flight requests on staged prefix chunks.

    ``hold`` binds the request's first block id to its ordered chunk list in
    the backend's registry (the lookup the backend's ``forward`` makes) and
    counts one holder per chunk; ``release`` undoes both, and drops a chunk's
    staged K/V from the backend when its count reaches zero."""

    def __init__(self):
        self._holds: dict[str, tuple[int, tuple[str, ...]]] = {}
        self._holders: Counter[str] = Counter()

    def hold(self, req_id: str, first_block_id: int, chunks: list[str]) -> None:
        if req_id in self._holds:
            raise RuntimeError(f"request {req_id} already holds staged chunks")
        map_request_peer(first_block_id, list(chunks))
        self._holds[req_id] = (first_block_id, tuple(chunks))
        self._holders.update(chunks)

    def release(self, req_id: str) -> bool:
        """Release ``req_id``'s hold; False when it held nothing."""
        entry = self._holds.pop(req_id, None)
        if entry is None:
            return False
        first_block_id, chunks = entry
        unmap_request_peer(first_block_id)
        for ck in chunks:
            self._holders[ck] -= 1
            if self._holders[ck] <= 0:
                del self._holders[ck]
                drop_chunk_kv(ck)
        return True

    def request_of_block(self, first_block_id: int) -> str | None:
        return next((rid for rid, (fb, _) in self._holds.items() if fb == first_block_id), None)

    def requests(self) -> list[str]:
        return list(self._holds)

    def holder_counts(self) -> dict[str, int]:
        return dict(self._holders)

    def release_all(self) -> None:
        for rid in list(self._holds):
            self.release(rid)
        for ck in list(self._holders):
            drop_chunk_kv(ck)
        self._holders.clear()


class LayerFeed:
    """One request's prefix staging, run on its own thread.

    ``stage(layer_name)`` (given to :meth:`start`) stages every prefix chunk
    of one layer and returns ``(tokens per chunk, completion event or None)``.
    The thread calls it for the layers in model order, each only once the
    forward has consumed the layer ``window`` places before it; the forward
    side calls :meth:`wait` before a layer's attention and :meth:`consumed`
    after.  The first error ends the thread and is raised by :meth:`wait`;
    a staged prefix whose total length is not ``expected_total`` is an
    error."""

    def __init__(self, req_id: str, layers: list[str], chunks: list[str], expected_total: int, window: int):
        self.req_id = req_id
        self.layers = list(layers)
        self.chunks = list(chunks)
        self.expected_total = expected_total
        self.window = max(1, window)
        self._staged = {ln: threading.Event() for ln in self.layers}
        self._device_done: dict[str, Any] = {}
        self._consumed = -1
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.error: BaseException | None = None

    def start(self, stage: Callable[[str], tuple[dict[str, int], Any]], init: Callable[[], None] | None = None):
        self._thread = threading.Thread(target=self._run, args=(stage, init), daemon=True)
        self._thread.start()

    def _run(self, stage, init) -> None:
        try:
            if init is not None:
                init()
            tokens: dict[str, int] = {}
            for i, layer_name in enumerate(self.layers):
                while not self._stop.is_set() and self._consumed < i - self.window:
                    time.sleep(0.0005)
                if self._stop.is_set():
                    return
                lens, done = stage(layer_name)
                tokens.update(lens)
                if done is not None:
                    self._device_done[layer_name] = done
                self._staged[layer_name].set()
            if sum(tokens.values()) != self.expected_total:
                raise RuntimeError(f"HcpRingKvConnector: staged prefix length {sum(tokens.values())} != "
                                   f"expected external prefix {self.expected_total} (chunks={self.chunks})")
        except BaseException as e:  # noqa: BLE001 - raised on the forward's thread by wait()
            self.error = e
            for ev in self._staged.values():
                ev.set()

    def covers(self, layer_name: str) -> bool:
        return layer_name in self._staged

    def wait(self, layer_name: str):
        """Block until ``layer_name`` is staged; returns its device-side
        completion event (or None), raises the thread's error."""
        self._staged[layer_name].wait()
        if self.error is not None:
            raise RuntimeError(f"HcpRingKvConnector: prefill stream for req {self.req_id} failed") from self.error
        return self._device_done.get(layer_name)

    def consumed(self, layer_idx: int) -> None:
        self._consumed = max(self._consumed, layer_idx)

    def join(self) -> None:
        if self._thread is not None:
            self._thread.join()

    def stop(self) -> None:
        self._stop.set()
        self.join()


class ReadinessCache:
    """Ready-marker lookups: a chunk seen ready stays ready; an absent one is
    looked for again only ``interval`` seconds after the last look."""

    def __init__(self, interval: float, exists: Callable[[str], bool] = os.path.exists,
                 clock: Callable[[], float] = time.monotonic):
        self.interval = interval
        self._exists = exists
        self._clock = clock
        self._ready: set[str] = set()
        self._next_look: dict[str, float] = {}

    def is_ready(self, key: str, marker_path: str) -> bool:
        if key in self._ready:
            return True
        now = self._clock()
        if now < self._next_look.get(key, 0.0):
            return False
        if self._exists(marker_path):
            self._ready.add(key)
            self._next_look.pop(key, None)
            return True
        self._next_look[key] = now + self.interval
        return False

    def look_again_now(self) -> None:
        self._next_look.clear()


class DecodeSlotPool:
    """The decode ring's request slots: taken lowest-free-first at a
    request's prefill, given back when the request finishes."""

    def __init__(self, slots: int):
        self.slots = slots
        self.free: deque[int] = deque(range(slots))
        self._taken: dict[str, tuple[int, int]] = {}   # req -> (slot, first block id)

    def take(self, req_id: str, first_block_id: int) -> int:
        if req_id in self._taken:
            raise RuntimeError(f"HcpRingKvConnector: request {req_id} already holds decode ring slot "
                               f"{self._taken[req_id][0]}")
        if not self.free:
            raise RuntimeError(f"HcpRingKvConnector: all {self.slots} decode ring slots are in use "
                               "(ring_decode_slots)")
        slot = self.free.popleft()
        self._taken[req_id] = (slot, first_block_id)
        return slot

    def give_back(self, req_id: str) -> int | None:
        """The request's first block id, or None if it held no slot."""
        entry = self._taken.pop(req_id, None)
        if entry is None:
            return None
        self.free.append(entry[0])
        return entry[1]

    def holders(self) -> list[str]:
        return list(self._taken)
