"""Base-worker wire protocol and deadline-driven fallback.

The reference hands the base ("host") partial sums of row tiles to remote workers and
takes them back in CRC-framed packets (src/phone_ffn_loopback.py:29-92); a tile whose
answer misses the step deadline, or arrives corrupted, is recomputed on the GPU's exact
full path instead (:155-197). This module keeps that contract, frame for frame:

    header  "!4sBB8I": magic b"PFFN", version 1, kind (1 request, 2 response), run_id,
            step_id, block_id, tile_id, row_start, row_count, payload length, CRC-32
            of the payload (zlib polynomial); then the payload.

and connects it to this library: a response payload is the tile's base sums as
little-endian f32 [tokens, row_count] (``base_payload`` / ``assemble_base``), which land
in the pinned base buffer that ``ffnrm_ffn_forward_host`` streams to the GPU, and the
fallback tile ids become the ``fallback_tiles`` mask of the same call.
"""
from __future__ import annotations

import struct
import time
import zlib
from concurrent.futures import ThreadPoolExecutor, as_completed
from dataclasses import dataclass
from typing import Callable, Iterable

import numpy as np

MAGIC = b"PFFN"
VERSION = 1
REQUEST = 1
RESPONSE = 2
HEADER = struct.Struct("!4sBB8I")


class ProtocolError(ValueError):
    """A frame is malformed or fails its integrity check."""


@dataclass(frozen=True)
class Frame:
    kind: int
    run_id: int
    step_id: int
    block_id: int
    tile_id: int
    row_start: int
    row_count: int
    payload: bytes

    def encode(self) -> bytes:
        crc = zlib.crc32(self.payload) & 0xFFFFFFFF
        return HEADER.pack(MAGIC, VERSION, self.kind, self.run_id, self.step_id, self.block_id, self.tile_id,
                           self.row_start, self.row_count, len(self.payload), crc) + self.payload

    @classmethod
    def decode(cls, packet: bytes) -> "Frame":
        if len(packet) < HEADER.size:
            raise ProtocolError("short frame")
        magic, version, kind, run_id, step_id, block_id, tile_id, row_start, row_count, n, crc = \
            HEADER.unpack_from(packet)
        if magic != MAGIC or version != VERSION:
            raise ProtocolError("unsupported frame header")
        payload = bytes(packet[HEADER.size:])
        if n != len(payload):
            raise ProtocolError("payload length mismatch")
        if zlib.crc32(payload) & 0xFFFFFFFF != crc:
            raise ProtocolError("payload checksum mismatch")
        if kind not in (REQUEST, RESPONSE):
            raise ProtocolError("unknown frame kind")
        return cls(kind, run_id, step_id, block_id, tile_id, row_start, row_count, payload)


@dataclass(frozen=True)
class DispatchResult:
    responses: tuple          # response frames, ordered by tile id
    fallback_tiles: tuple     # tile ids handed to the GPU's exact path, ascending
    deadline_misses: int      # number of fallback tiles
    protocol_errors: int      # responses that failed to decode or whose worker raised


class BaseWorker:
    """A worker that owns rows [row_start, row_start + row_count) and answers requests
    for tiles inside them with ``compute(request) -> payload`` (after ``delay_ms``)."""

    def __init__(self, worker_id: int, row_start: int, row_count: int, compute: Callable[[Frame], bytes],
                 delay_ms: float = 0.0):
        if worker_id < 0 or row_start < 0 or row_count <= 0:
            raise ValueError("invalid worker shard")
        self.worker_id, self.row_start, self.row_count = worker_id, row_start, row_count
        self.compute, self.delay_ms = compute, max(0.0, delay_ms)

    def accepts(self, request: Frame) -> bool:
        return (request.kind == REQUEST and request.row_start >= self.row_start
                and request.row_start + request.row_count <= self.row_start + self.row_count)

    def handle(self, request: Frame) -> Frame:
        if not self.accepts(request):
            raise ProtocolError(f"worker {self.worker_id} rejected row shard")
        if self.delay_ms:
            time.sleep(self.delay_ms / 1000.0)
        return Frame(RESPONSE, request.run_id, request.step_id, request.block_id, request.tile_id,
                     request.row_start, request.row_count, bytes(self.compute(request)))


class BaseCluster:
    """Sends each tile request to the worker that owns its rows, concurrently, and
    collects the answers until the deadline; tiles without an owner, late tiles and
    tiles whose answer fails to decode go to the exact fallback list."""

    def __init__(self, workers: Iterable[BaseWorker]):
        self.workers = tuple(workers)
        if not self.workers:
            raise ValueError("at least one worker is required")

    def dispatch(self, requests: Iterable[Frame], deadline_ms: float) -> DispatchResult:
        requests = tuple(requests)
        if any(r.kind != REQUEST for r in requests):
            raise ProtocolError("dispatch accepts request frames only")
        if deadline_ms <= 0:
            raise ValueError("deadline_ms must be positive")
        t0 = time.monotonic()
        responses, fallback, errors = [], [], 0
        pool = ThreadPoolExecutor(max_workers=len(self.workers))
        try:
            pending = {}
            for r in requests:
                w = next((w for w in self.workers if w.accepts(r)), None)
                if w is None:
                    fallback.append(r.tile_id)
                else:
                    pending[pool.submit(w.handle, r)] = r
            try:
                for fut in as_completed(pending, timeout=max(0.0, deadline_ms / 1e3 - (time.monotonic() - t0))):
                    r = pending.pop(fut)
                    if time.monotonic() - t0 > deadline_ms / 1e3:
                        fallback.append(r.tile_id)
                        continue
                    try:
                        # a transport would decode a wire packet here: round-trip the codec
                        responses.append(Frame.decode(fut.result().encode()))
                    except Exception:
                        errors += 1
                        fallback.append(r.tile_id)
            except TimeoutError:
                pass
            fallback.extend(r.tile_id for r in pending.values())  # still running at the deadline
        finally:
            pool.shutdown(wait=False, cancel_futures=True)
        responses.sort(key=lambda f: f.tile_id)
        fallback.sort()
        return DispatchResult(tuple(responses), tuple(fallback), len(fallback), errors)


def tile_requests(rows: int, tile_rows: int, run_id: int = 0, step_id: int = 0, block_id: int = 0,
                  descriptor: bytes = b"") -> list[Frame]:
    """One request per row tile of a projection (the last tile may be short)."""
    return [Frame(REQUEST, run_id, step_id, block_id, t, t * tile_rows, min(tile_rows, rows - t * tile_rows), descriptor)
            for t in range(-(-rows // tile_rows))]


def base_payload(base: np.ndarray) -> bytes:
    """Base sums of one tile, f32 [tokens, row_count], as a little-endian payload."""
    return np.ascontiguousarray(base, dtype="<f4").tobytes()


def assemble_base(result: DispatchResult, out: np.ndarray, tile_rows: int) -> np.ndarray:
    """Write every response's base tile into ``out`` [tokens, rows] (f32, e.g. pinned)
    and return the fallback mask, one byte per tile (nonzero = exact GPU path)."""
    tokens, rows = out.shape
    mask = np.zeros(-(-rows // tile_rows), dtype=np.uint8)
    for f in result.responses:
        if f.row_start + f.row_count > rows or f.row_start % tile_rows:
            raise ProtocolError("response rows outside the tile grid")
        tile = np.frombuffer(f.payload, dtype="<f4")
        if tile.size != tokens * f.row_count:
            raise ProtocolError("response payload does not hold the tile's base sums")
        out[:, f.row_start:f.row_start + f.row_count] = tile.reshape(tokens, f.row_count)
    for t in result.fallback_tiles:
        mask[t] = 1
    return mask
