"""Host-side mirror of the reference's ``marketforge::cuda`` head interface.

Same names, argument meaning and error behaviour as
``include/marketforge/cuda/greedy.hpp`` (plus the boundary types of
``device_buffer.hpp`` / ``cuda_stream.hpp`` / ``core/status.hpp``), calling
the CUDA kernels through the C-ABI in ``include/mf_head.h``.  Buffers may be
:class:`DeviceBuffer` objects or CUDA ``torch.Tensor`` s (their byte size is
``numel * element_size``); streams may be :class:`CudaStream`,
``torch.cuda.Stream`` or a raw ``cudaStream_t`` integer.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional, Union

from ._lib import lib

INVALID_TOKEN_ID = 0xFFFFFFFF
"""``restricted_greedy_invalid_token_id`` (greedy.hpp:11-12)."""


class ErrorCode(enum.IntEnum):
    """``marketforge::ErrorCode`` (include/marketforge/core/status.hpp:7-31)."""

    ok = 0
    invalid_argument = 1
    unsupported_dtype = 2
    invalid_shape = 3
    invalid_model = 4
    arithmetic_overflow = 5
    invalid_alignment = 6
    allocation_failed = 7
    insufficient_memory = 8
    insufficient_resources = 9
    io_error = 10
    invalid_format = 11
    invalid_utf8 = 12
    invalid_json = 13
    duplicate_key = 14
    resource_limit = 15
    truncated_data = 16
    invalid_tensor = 17
    missing_tensor = 18
    unexpected_tensor = 19
    hash_mismatch = 20
    cuda_backend_failure = 21
    cuda_runtime_failure = 22


@dataclass(frozen=True)
class Status:
    """``marketforge::Status`` (status.hpp:33-49)."""

    code: ErrorCode = ErrorCode.ok
    detail: int = 0

    def ok(self) -> bool:
        return self.code == ErrorCode.ok

    @staticmethod
    def success() -> "Status":
        return Status()

    @staticmethod
    def failure(code: ErrorCode, detail: int = 0) -> "Status":
        return Status(ErrorCode(code), detail)


def _status(s) -> Status:
    return Status(ErrorCode(s.code), int(s.detail))


class CudaStream:
    """``marketforge::cuda::CudaStream`` (cuda_stream.hpp:19-41): a
    non-blocking stream (src/cuda/cuda_stream.cu:13)."""

    def __init__(self, stream=None):
        import torch

        self._stream = stream if stream is not None else torch.cuda.Stream()

    @staticmethod
    def create() -> "CudaStream":
        return CudaStream()

    def handle(self) -> int:
        return int(self._stream.cuda_stream)

    @property
    def torch_stream(self):
        return self._stream

    def synchronize(self) -> Status:
        self._stream.synchronize()
        return Status.success()


class DeviceBuffer:
    """``marketforge::cuda::DeviceBuffer`` (device_buffer.hpp:20-56): an exact
    byte-sized device allocation (torch's caching allocator underneath)."""

    def __init__(self, tensor=None):
        self._t = tensor

    @staticmethod
    def allocate(byte_count: int) -> "DeviceBuffer":
        import torch

        if byte_count == 0:
            return DeviceBuffer()
        return DeviceBuffer(torch.empty(int(byte_count), dtype=torch.uint8, device="cuda"))

    def size_bytes(self) -> int:
        return 0 if self._t is None else self._t.numel() * self._t.element_size()

    def address(self) -> int:
        return 0 if self._t is None else int(self._t.data_ptr())

    @property
    def tensor(self):
        return self._t

    def view(self, dtype):
        return self._t.view(dtype)

    def copy_from_host_async(self, source, byte_count: int, offset: int, stream) -> Status:
        return _copy(self, source, byte_count, offset, stream, to_device=True)

    def copy_to_host_async(self, destination, byte_count: int, offset: int, stream) -> Status:
        return _copy(self, destination, byte_count, offset, stream, to_device=False)


def _copy(buf: DeviceBuffer, host, byte_count, offset, stream, to_device) -> Status:
    # src/cuda/device_buffer.cu:13-31 validation order
    import torch

    h = _stream_handle(stream)
    if h == 0 or (byte_count != 0 and host is None):
        return Status.failure(ErrorCode.invalid_argument)
    if offset + byte_count > buf.size_bytes():
        return Status.failure(ErrorCode.invalid_argument)
    if byte_count == 0:
        return Status.success()
    host_t = host if isinstance(host, torch.Tensor) else torch.from_numpy(host)
    host_bytes = host_t.reshape(-1).view(torch.uint8)[:byte_count]
    dev = buf.tensor[offset:offset + byte_count]
    with torch.cuda.stream(_torch_stream(stream)):
        if to_device:
            dev.copy_(host_bytes, non_blocking=True)
        else:
            host_bytes.copy_(dev, non_blocking=True)
    return Status.success()


Buffer = Union[DeviceBuffer, "torch.Tensor", None]  # noqa: F821


def _addr(b: Buffer) -> int:
    if b is None:
        return 0
    if isinstance(b, DeviceBuffer):
        return b.address()
    return int(b.data_ptr())


def _size(b: Buffer) -> int:
    if b is None:
        return 0
    if isinstance(b, DeviceBuffer):
        return b.size_bytes()
    return b.numel() * b.element_size()


def _stream_handle(s) -> int:
    if s is None:
        return 0
    if isinstance(s, CudaStream):
        return s.handle()
    if isinstance(s, int):
        return s
    return int(s.cuda_stream)


def _torch_stream(s):
    import torch

    if isinstance(s, CudaStream):
        return s.torch_stream
    if isinstance(s, int):
        return torch.cuda.ExternalStream(s)
    return s


def _pb(b: Buffer):
    return ctypes.c_void_p(_addr(b) or None), ctypes.c_uint64(_size(b))


def _sp(s):
    h = _stream_handle(s)
    return ctypes.c_void_p(h or None)


# ---- reference-signature functions (greedy.hpp:17-49) ----------------------

def greedy_select_f16(logits: Buffer, token_ids: Buffer, rows: int, vocabulary_size: int,
                      stream) -> Status:
    """greedy.hpp:17-21: argmax per row of fp16 logits[rows, V]."""
    return _status(lib.mf_greedy_select_f16(*_pb(logits), *_pb(token_ids), rows,
                                            vocabulary_size, _sp(stream)))


def restricted_greedy_select_f16(logits: Buffer, allowed_token_ids: Buffer,
                                 allowed_token_counts: Buffer, token_ids: Buffer, rows: int,
                                 vocabulary_size: int, maximum_allowed_tokens: int,
                                 stream) -> Status:
    """greedy.hpp:29-33: masked argmax over a padded candidate table."""
    return _status(lib.mf_restricted_greedy_select_f16(
        *_pb(logits), *_pb(allowed_token_ids), *_pb(allowed_token_counts), *_pb(token_ids),
        rows, vocabulary_size, maximum_allowed_tokens, _sp(stream)))


def restricted_output_head_f16(hidden: Buffer, embedding: Buffer, allowed_token_ids: Buffer,
                               allowed_token_counts: Buffer, token_ids: Buffer, rows: int,
                               hidden_size: int, vocabulary_size: int,
                               maximum_allowed_tokens: int, stream) -> Status:
    """greedy.hpp:43-49: fused tied projection + restricted argmax."""
    return _status(lib.mf_restricted_output_head_f16(
        *_pb(hidden), *_pb(embedding), *_pb(allowed_token_ids), *_pb(allowed_token_counts),
        *_pb(token_ids), rows, hidden_size, vocabulary_size, maximum_allowed_tokens,
        _sp(stream)))


# ---- ragged CSR head and device DFA (new batched launch path) -------------

def head_workspace_bytes(rows: int) -> int:
    return int(lib.mf_head_workspace_bytes(rows))


def dfa_workspace_bytes(batch: int) -> int:
    return int(lib.mf_dfa_workspace_bytes(batch))


def restricted_output_head_csr_f16(hidden: Buffer, embedding: Buffer, offsets: Buffer,
                                   ids: Buffer, token_ids: Buffer, scores: Optional[Buffer],
                                   workspace: Buffer, rows: int, hidden_size: int,
                                   vocabulary_size: int, stream) -> Status:
    """Ragged head: row r's candidates are ids[offsets[r]:offsets[r+1]]."""
    return _status(lib.mf_head_restricted_csr_f16(
        *_pb(hidden), *_pb(embedding), *_pb(offsets), *_pb(ids), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocabulary_size, _sp(stream)))


LAUNCH_OVERLAP_PREVIOUS = 1
"""``restricted_output_head_csr_f16_ex`` flag: the launch may overlap the tail
of the previous kernel on the stream, which must not write this call's
inputs (consecutive head calls on independent batches)."""


def restricted_output_head_csr_f16_ex(hidden: Buffer, embedding: Buffer, offsets: Buffer,
                                      ids: Buffer, token_ids: Buffer, scores: Optional[Buffer],
                                      workspace: Buffer, rows: int, hidden_size: int,
                                      vocabulary_size: int, launch_flags: int, stream) -> Status:
    """``restricted_output_head_csr_f16`` with launch options
    (``LAUNCH_OVERLAP_PREVIOUS``)."""
    return _status(lib.mf_head_restricted_csr_f16_ex(
        *_pb(hidden), *_pb(embedding), *_pb(offsets), *_pb(ids), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocabulary_size, launch_flags, _sp(stream)))


def restricted_output_head_csr_u16ids_f16_ex(hidden: Buffer, embedding: Buffer, offsets: Buffer,
                                             ids: Buffer, token_ids: Buffer,
                                             scores: Optional[Buffer], workspace: Buffer, rows: int,
                                             hidden_size: int, vocabulary_size: int,
                                             launch_flags: int, stream) -> Status:
    """``restricted_output_head_csr_f16_ex`` with the candidate ids as uint16
    (vocabularies of at most 65,536 ids): half the bytes to move per batch."""
    return _status(lib.mf_head_restricted_csr_u16ids_f16_ex(
        *_pb(hidden), *_pb(embedding), *_pb(offsets), *_pb(ids), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocabulary_size, launch_flags, _sp(stream)))


NOALLOC_MAX_ROWS = 65536
"""Largest batch ``restricted_output_head_csr_f16_noalloc`` accepts."""


def restricted_output_head_csr_f16_noalloc(hidden: Buffer, embedding: Buffer, offsets: Buffer,
                                           ids: Buffer, token_ids: Buffer,
                                           scores: Optional[Buffer], rows: int, hidden_size: int,
                                           vocabulary_size: int, stream) -> Status:
    """The ragged head without a workspace argument, for callers that cannot
    allocate device memory: the library keeps a fixed scratch array per GPU
    (up to NOALLOC_MAX_ROWS rows).  Calls sharing a device must not overlap
    on the GPU; make the first call on a device before any stream capture."""
    return _status(lib.mf_head_restricted_csr_f16_noalloc(
        *_pb(hidden), *_pb(embedding), *_pb(offsets), *_pb(ids), *_pb(token_ids), *_pb(scores),
        rows, hidden_size, vocabulary_size, _sp(stream)))


def restricted_output_head_csr_rmsnorm_f16(hidden: Buffer, gamma: Buffer, eps: float,
                                           embedding: Buffer, offsets: Buffer, ids: Buffer,
                                           token_ids: Buffer, scores: Optional[Buffer],
                                           workspace: Buffer, rows: int, hidden_size: int,
                                           vocabulary_size: int, stream) -> Status:
    """Ragged head with the final RMSNorm fused in front (hidden = the last
    layer's un-normalised rows, gamma = the norm weight)."""
    return _status(lib.mf_head_restricted_csr_rmsnorm_f16(
        *_pb(hidden), *_pb(gamma), float(eps), *_pb(embedding), *_pb(offsets), *_pb(ids),
        *_pb(token_ids), *_pb(scores), *_pb(workspace), rows, hidden_size, vocabulary_size,
        _sp(stream)))


def dfa_head_step_f16(hidden: Buffer, embedding: Buffer, state_offsets: Buffer,
                      arc_tokens: Buffer, arc_next: Buffer, states_in: Buffer,
                      states_out: Buffer, tokens: Buffer, scores: Optional[Buffer],
                      workspace: Buffer, batch: int, num_states: int, hidden_size: int,
                      vocabulary_size: int, stream) -> Status:
    """One device step: allowed-set lookup, restricted head, DFA advance."""
    return _status(lib.mf_dfa_head_step_f16(
        *_pb(hidden), *_pb(embedding), *_pb(state_offsets), *_pb(arc_tokens), *_pb(arc_next),
        *_pb(states_in), *_pb(states_out), *_pb(tokens), *_pb(scores), *_pb(workspace),
        batch, num_states, hidden_size, vocabulary_size, _sp(stream)))


def dfa_head_step_rmsnorm_f16(hidden: Buffer, gamma: Buffer, eps: float, embedding: Buffer,
                              state_offsets: Buffer, arc_tokens: Buffer, arc_next: Buffer,
                              states_in: Buffer, states_out: Buffer, tokens: Buffer,
                              scores: Optional[Buffer], workspace: Buffer, batch: int,
                              num_states: int, hidden_size: int, vocabulary_size: int,
                              stream) -> Status:
    """One device step with the final RMSNorm fused in front (hidden = the
    last layer's un-normalised rows, gamma = the norm weight)."""
    return _status(lib.mf_dfa_head_step_rmsnorm_f16(
        *_pb(hidden), *_pb(gamma), float(eps), *_pb(embedding), *_pb(state_offsets),
        *_pb(arc_tokens), *_pb(arc_next), *_pb(states_in), *_pb(states_out), *_pb(tokens),
        *_pb(scores), *_pb(workspace), batch, num_states, hidden_size, vocabulary_size,
        _sp(stream)))


def dfa_decode_f16(hidden: Buffer, embedding: Buffer, state_offsets: Buffer, arc_tokens: Buffer,
                   arc_next: Buffer, state_trace: Buffer, token_trace: Buffer,
                   score_trace: Optional[Buffer], workspace: Buffer, steps: int, batch: int,
                   num_states: int, hidden_size: int, vocabulary_size: int, stream) -> Status:
    """``steps`` DFA head steps back to back, no host synchronisation."""
    return _status(lib.mf_dfa_decode_f16(
        *_pb(hidden), *_pb(embedding), *_pb(state_offsets), *_pb(arc_tokens), *_pb(arc_next),
        *_pb(state_trace), *_pb(token_trace), *_pb(score_trace), *_pb(workspace), steps, batch,
        num_states, hidden_size, vocabulary_size, _sp(stream)))


# ---- dense full-vocabulary head (tcgen05) ---------------------------------

def dense_workspace_bytes(rows: int) -> int:
    return int(lib.mf_dense_workspace_bytes(rows))


def dense_head_f16(hidden: Buffer, embedding: Buffer, keys: Optional[Buffer],
                   token_ids: Optional[Buffer], scores: Optional[Buffer], workspace: Buffer,
                   rows: int, hidden_size: int, vocab_rows: int, vocab_begin: int,
                   stream) -> Status:
    """Full-vocabulary greedy head over one vocabulary shard (replaces
    linear_f16 + greedy_select_f16): packed keys and/or ids and scores."""
    return _status(lib.mf_dense_head_f16(
        *_pb(hidden), *_pb(embedding), *_pb(keys), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocab_rows, vocab_begin, _sp(stream)))


def dense_head_f16_ex(hidden: Buffer, embedding: Buffer, keys: Optional[Buffer],
                      token_ids: Optional[Buffer], scores: Optional[Buffer], workspace: Buffer,
                      rows: int, hidden_size: int, vocab_rows: int, vocab_begin: int,
                      launch_flags: int, stream) -> Status:
    """``dense_head_f16`` with launch options (``LAUNCH_OVERLAP_PREVIOUS``)."""
    return _status(lib.mf_dense_head_f16_ex(
        *_pb(hidden), *_pb(embedding), *_pb(keys), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocab_rows, vocab_begin, launch_flags, _sp(stream)))


def decode_keys(keys: Buffer, token_ids: Buffer, scores: Optional[Buffer], rows: int,
                stream) -> Status:
    """Packed keys (after a cross-shard max) -> ids and scores."""
    return _status(lib.mf_decode_keys(*_pb(keys), *_pb(token_ids), *_pb(scores), rows,
                                      _sp(stream)))


IPC_HANDLE_BYTES = 64


def exchange_bytes(rows: int, world: int) -> int:
    """Bytes of one rank's exchange buffer for ``dense_head_sharded_f16``."""
    return int(lib.mf_exchange_bytes(rows, world))


def exchange_broken(buffer) -> int:
    """1 once a sharded call on this rank's exchange buffer (a device tensor
    or address) gave up on a peer or saw a peer fail, else 0.  A broken
    buffer gives every row the sentinel until new buffers are made.  Reads
    the word synchronously."""
    ptr = buffer.data_ptr() if hasattr(buffer, "data_ptr") else int(buffer)
    out = ctypes.c_uint32()
    st = _status(lib.mf_exchange_broken(ctypes.c_void_p(ptr), ctypes.byref(out)))
    if not st.ok():
        raise RuntimeError(f"mf_exchange_broken failed: {st}")
    return int(out.value)


def dense_head_sharded_f16(hidden: Buffer, embedding: Buffer, keys: Optional[Buffer],
                           token_ids: Optional[Buffer], scores: Optional[Buffer],
                           workspace: Buffer, rows: int, hidden_size: int, vocab_rows: int,
                           vocab_begin: int, exchange, stream, launch_flags: int = 0) -> Status:
    """Vocabulary shards on several GPUs merged inside the dense kernel: every
    rank calls this on its own shard (``vocab_begin`` = the shard's first id)
    and gets the global ids / scores / keys.  ``exchange`` is a
    ``VocabShardExchange`` (or any object with ``ptrs``, ``nbytes``,
    ``world`` and ``rank``)."""
    arr = (ctypes.c_void_p * len(exchange.ptrs))(*exchange.ptrs)
    return _status(lib.mf_dense_head_sharded_f16(
        *_pb(hidden), *_pb(embedding), *_pb(keys), *_pb(token_ids), *_pb(scores),
        *_pb(workspace), rows, hidden_size, vocab_rows, vocab_begin, arr, exchange.nbytes,
        exchange.world, exchange.rank, launch_flags, _sp(stream)))


class VocabShardExchange:
    """The exchange buffers of ``dense_head_sharded_f16``: this rank allocates
    its own (``mf_exchange_alloc``), the 64-byte CUDA IPC handles are
    all-gathered (``all_gather(bytes) -> list[bytes]``, by default
    ``torch.distributed.all_gather_object`` on ``group``) and every peer's
    buffer is mapped here (``mf_exchange_open_peer``).  One process per GPU;
    the current device must be this rank's GPU."""

    def __init__(self, rows: int, world: int = None, rank: int = None, group=None,
                 all_gather=None):
        if world is None or rank is None:
            import torch.distributed as dist

            world, rank = dist.get_world_size(group), dist.get_rank(group)
        if all_gather is None:
            import torch.distributed as dist

            def all_gather(b: bytes):
                out = [None] * world
                dist.all_gather_object(out, b, group=group)
                return out
        self.world, self.rank, self.rows = int(world), int(rank), int(rows)
        self.nbytes = exchange_bytes(rows, world)
        own, handle = ctypes.c_void_p(), ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        st = _status(lib.mf_exchange_alloc(ctypes.byref(own), self.nbytes, handle))
        if not st.ok():
            raise RuntimeError(f"mf_exchange_alloc failed: {st}")
        self._own = own.value
        self._opened = []
        handles = all_gather(handle.raw)
        ptrs = []
        try:
            for q, h in enumerate(handles):
                if q == self.rank:
                    ptrs.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                st = _status(lib.mf_exchange_open_peer(ctypes.create_string_buffer(h, len(h)),
                                                       ctypes.byref(peer)))
                if not st.ok():
                    raise RuntimeError(f"mf_exchange_open_peer({q}) failed: {st}")
                self._opened.append(peer.value)
                ptrs.append(peer.value)
        except Exception:
            self.close()
            raise
        self.ptrs = ptrs

    def close(self) -> None:
        for p in self._opened:
            lib.mf_exchange_close_peer(p)
        self._opened = []
        if self._own:
            lib.mf_exchange_free(self._own)
            self._own = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


KEY_SIGN_FLIP = 1 << 63
"""XOR with this maps the unsigned key order onto signed int64 order, so a
signed MAX all-reduce (NCCL / torch.distributed) merges keys correctly."""


class RaggedHead:
    """Owns the workspace for repeated ragged-head calls on one stream.

    ``embedding`` stays resident; each ``__call__`` takes a batch of hidden
    rows and its CSR allowed sets (device tensors) and returns
    ``(token_ids, scores)`` device tensors.
    """

    def __init__(self, embedding, max_rows: int, stream=None):
        import torch

        self.embedding = embedding
        self.vocab, self.hidden_size = int(embedding.shape[0]), int(embedding.shape[1])
        self.max_rows = int(max_rows)
        self.workspace = torch.zeros(head_workspace_bytes(self.max_rows), dtype=torch.uint8,
                                     device=embedding.device)
        self.stream = stream

    def __call__(self, hidden, offsets, ids, out_ids=None, out_scores=None):
        import torch

        rows = int(hidden.shape[0])
        if rows > self.max_rows:
            raise ValueError(f"batch of {rows} rows exceeds max_rows={self.max_rows}")
        if out_ids is None:
            out_ids = torch.empty(rows, dtype=torch.int32, device=hidden.device)
        if out_scores is None:
            out_scores = torch.empty(rows, dtype=torch.float32, device=hidden.device)
        ws = self.workspace[: head_workspace_bytes(rows)]
        stream = self.stream if self.stream is not None else torch.cuda.current_stream()
        st = restricted_output_head_csr_f16(hidden, self.embedding, offsets, ids, out_ids,
                                            out_scores, ws, rows, self.hidden_size, self.vocab,
                                            stream)
        if not st.ok():
            raise RuntimeError(f"restricted head failed: {st}")
        return out_ids, out_scores


class HostPipeline:
    """Restricted head over batches that live in host memory (native
    ``mf_pipeline_*``): each ``submit`` copies one batch (hidden rows, CSR
    offsets, CSR ids) from pinned host memory to the device, runs the ragged
    head and copies ids and scores back into pinned host memory, in order on
    the stream of the next of ``depth`` slots (each slot has its own device
    buffers and workspace), so batches on different slots overlap.  Host
    tensors must stay untouched until ``wait(ticket)`` returns.
    """

    def __init__(self, embedding, max_rows: int, max_ids: int, depth: int = 6, device=None):
        self.embedding = embedding  # keeps the device table alive
        self.vocab, self.hidden_size = int(embedding.shape[0]), int(embedding.shape[1])
        self._p = ctypes.c_void_p()
        self._ticket = ctypes.c_uint64()
        self._ticket_ref = ctypes.byref(self._ticket)
        st = _status(lib.mf_pipeline_create(ctypes.byref(self._p), *_pb(embedding), self.vocab,
                                            self.hidden_size, int(max_rows), int(max_ids),
                                            int(depth)))
        if not st.ok():
            raise RuntimeError(f"mf_pipeline_create failed: {st}")

    def depth(self) -> int:
        """Number of slots (batches in flight)."""
        return int(lib.mf_pipeline_depth(self._p))

    def stream(self, slot: int) -> int:
        """cudaStream_t of slot ``slot`` (copy in, head, copy out in order)."""
        return int(lib.mf_pipeline_stream(self._p, slot) or 0)

    def submit(self, hidden, offsets, ids, out_ids, out_scores=None) -> int:
        """hidden fp16 [rows, H], offsets int32 [rows + 1], ids int32 [total],
        out_ids int32 [rows], out_scores float32 [rows] or None: pinned host
        tensors.  Returns the batch's ticket."""
        return self.submit_ptrs(hidden.data_ptr(), hidden.shape[0], offsets.data_ptr(),
                                ids.data_ptr(), ids.shape[0], out_ids.data_ptr(),
                                out_scores.data_ptr() if out_scores is not None else None)

    def submit_ptrs(self, hidden: int, rows: int, offsets: int, ids: int, total_ids: int,
                    out_ids: int, out_scores) -> int:
        """``submit`` with raw host addresses (for callers that keep their own
        pinned buffers)."""
        s = lib.mf_pipeline_submit(self._p, hidden, rows, offsets, ids or None, total_ids,
                                   out_ids, out_scores, self._ticket_ref)
        if s.code:
            raise RuntimeError(f"mf_pipeline_submit failed: {_status(s)}")
        return self._ticket.value

    @staticmethod
    def pack(hidden, offsets, ids, u16_ids: bool = False):
        """One pinned uint8 host buffer holding hidden fp16 [rows, H], offsets
        int32 [rows + 1] and ids int32 [total] back to back (the layout of
        ``submit_packed``); with ``u16_ids`` the ids as uint16 (the layout of
        ``submit_packed(..., u16_ids=True)``, vocabularies of at most 65,536)."""
        import numpy as np
        import torch

        if u16_ids:
            a = np.asarray(ids)
            if a.size and (a.min() < 0 or a.max() > 0xFFFF):
                raise ValueError("ids outside [0, 65535] do not fit uint16")
            ids = torch.from_numpy(a.astype(np.uint16).view(np.int16))
        parts = [torch.as_tensor(x).contiguous().view(torch.uint8).reshape(-1)
                 for x in (hidden, offsets, ids)]
        buf = torch.empty(sum(p.numel() for p in parts), dtype=torch.uint8).pin_memory()
        at = 0
        for part in parts:
            buf[at:at + part.numel()] = part
            at += part.numel()
        return buf

    def submit_packed_ptrs(self, batch: int, batch_bytes: int, rows: int, total_ids: int,
                           out: int, u16_ids: bool = False) -> int:
        """One packed batch (see ``pack``) at host address ``batch``; ``out``
        receives ids u32 [rows] then scores f32 [rows].  One H2D and one D2H
        copy per batch."""
        f = lib.mf_pipeline_submit_packed_u16ids if u16_ids else lib.mf_pipeline_submit_packed
        s = f(self._p, batch, batch_bytes, rows, total_ids, out, self._ticket_ref)
        if s.code:
            raise RuntimeError(f"mf_pipeline_submit_packed failed: {_status(s)}")
        return self._ticket.value

    def submit_packed(self, batch, rows: int, total_ids: int, out, u16_ids: bool = False) -> int:
        """``batch`` from ``pack`` (with the same ``u16_ids``); ``out`` a pinned
        host tensor of 8 * rows bytes."""
        return self.submit_packed_ptrs(batch.data_ptr(), batch.numel() * batch.element_size(),
                                       rows, total_ids, out.data_ptr(), u16_ids)

    def wait(self, ticket: int) -> None:
        st = _status(lib.mf_pipeline_wait(self._p, ticket))
        if not st.ok():
            raise RuntimeError(f"mf_pipeline_wait failed: {st}")

    def synchronize(self) -> None:
        st = _status(lib.mf_pipeline_synchronize(self._p))
        if not st.ok():
            raise RuntimeError(f"mf_pipeline_synchronize failed: {st}")

    def close(self) -> None:
        if self._p:
            lib.mf_pipeline_destroy(self._p)
            self._p = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
