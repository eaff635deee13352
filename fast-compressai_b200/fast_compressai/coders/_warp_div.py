"""Native module of the ``warp_div`` coder.

Drop-in for the reference's pybind extension ``fast_compressai.coders._warp_div``
(coders/cuda/ans_gpu.cpp:25-30): the same two callables with the same tuple
contract, implemented over the C ABI of ``_lib/libfcai_b200.so``
(include/fcai_warp_div.h).  Work is enqueued on the current CUDA stream of
the tensors' device.

    encode_warp_div(symbols, indexes, cdfs, cdf_sizes, offsets, P)
        -> (packed u8 [header_bytes + 128*sum(rounds)], max_rounds u32 [B, K],
            header_bytes i64 CPU [1], chunk_len i32 CPU [1], P i32 CPU [1])
    decode_warp_div(packed, max_rounds, header_bytes_cpu, chunk_len_cpu, P_cpu,
                    indexes, cdfs, cdf_sizes, offsets) -> int32 [B, N]

Failures raise ``RuntimeError`` (the reference raises it from TORCH_CHECK).
"""

from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass

import torch

from .. import _native

_WS_LOCK = threading.Lock()
_WORKSPACES: dict[tuple, torch.Tensor] = {}
_LANES = 32
_MAX_SYMBOL_WORDS = 10


def _ptr(t: torch.Tensor | None):
    # the native functions declare their argtypes, so an int address passes
    return None if t is None else t.data_ptr()


def workspace(kind: str, device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Cached device workspace per (kind, device, stream); control block zeroed on allocation."""
    key = (kind, device.index, stream)
    with _WS_LOCK:
        ws = _WORKSPACES.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            ws[:256].zero_()
            _WORKSPACES[key] = ws
        return ws


def release_workspaces() -> None:
    """Drop every cached workspace (e.g. before freeing device memory)."""
    with _WS_LOCK:
        _WORKSPACES.clear()


@dataclass(frozen=True)
class EncodeResult:
    packed: torch.Tensor
    max_rounds: torch.Tensor
    header_bytes: int
    chunk_len: int
    p_ch: int
    index_layout_is_channel: bool


def _plan(B: int, N: int, C: int, P: int) -> _native.WarpDivPlan:
    plan = _native.WarpDivPlan()
    _native.check(_native.lib().fcai_warp_div_plan_create(B, N, C, P, ctypes.byref(plan)))
    return plan


def _check_encode_inputs(symbols, indexes, cdfs, cdf_sizes, offsets) -> None:
    # coders/cuda/warp_ans_kernel_v2.cu:188-192
    tensors = [t for t in (symbols, indexes, cdfs, cdf_sizes, offsets) if t is not None]
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors):
        raise RuntimeError("CUDA required")
    if any(t.device != symbols.device for t in tensors):
        raise RuntimeError("all coder tensors must share a CUDA device")
    if any(t.dtype != torch.int32 for t in tensors):
        raise RuntimeError("all coder inputs must be int32")
    if not all(t.is_contiguous() for t in tensors):
        raise RuntimeError("all coder inputs must be contiguous")
    if (symbols.dim() != 2 or (indexes is not None and indexes.shape != symbols.shape) or cdfs.dim() != 2
            or cdf_sizes.dim() != 1 or offsets.dim() != 1):
        raise RuntimeError("invalid coder input ranks/shapes")
    if cdf_sizes.numel() != cdfs.shape[0] or offsets.numel() != cdfs.shape[0]:
        raise RuntimeError("CDF metadata length mismatch")


def _encode_sizes(B: int, N: int, C: int, P: int) -> tuple[int, int]:
    """(K, first workspace size): one staged word per symbol per lane covers
    any practical table; an encode that needs more reports the exact size."""
    plan = _plan(B, N, C, int(P))
    K = plan.chunks
    chunks = B * K
    lane_symbols = (plan.chunk_len + _LANES - 1) // _LANES
    rows_worst = _MAX_SYMBOL_WORDS * lane_symbols + 2
    fixed = plan.encode_workspace_bytes - chunks * rows_worst * _LANES * 4
    return K, fixed + chunks * min(rows_worst, lane_symbols + 4) * _LANES * 4


def _pack(B: int, N: int, C: int, P: int, ws: torch.Tensor, max_rounds: torch.Tensor, info, stream: int,
          dev: torch.device) -> EncodeResult:
    packed = torch.empty(int(info.packed_bytes), dtype=torch.uint8, device=dev)
    _native.check(_native.lib().fcai_warp_div_encode_pack(_ptr(ws), ws.numel(), B, N, C, int(P), _ptr(packed),
                                                          packed.numel(), stream))
    _native.count_launches(1)
    return EncodeResult(packed, max_rounds, int(info.header_bytes), int(info.chunk_len), int(info.p_ch),
                        bool(info.index_layout_is_channel))


def _run_encode(B: int, N: int, C: int, P: int, dev: torch.device, call) -> EncodeResult:
    """Workspace sizing, the encode call (retried once with the exact staging
    need if the first workspace was short), payload allocation and pack."""
    lib = _native.lib()
    with _native.on_device(dev):
        stream = _native.stream_handle(dev)
        K, nbytes = _encode_sizes(B, N, C, P)
        max_rounds = torch.empty((B, K), dtype=torch.uint32, device=dev)
        info = _native.WarpDivEncodeInfo()
        for attempt in range(2):
            ws = workspace("encode", dev, stream, nbytes)
            rc = call(lib, ws, max_rounds, info, stream)
            _native.count_launches(1)  # the encode (its last CTA also writes the status words to the host)
            if rc == _native.FCAI_ERR_WORKSPACE and attempt == 0 and info.required_workspace_bytes > ws.numel():
                nbytes = info.required_workspace_bytes
                continue
            _native.check(rc)
            break
        return _pack(B, N, C, P, ws, max_rounds, info, stream, dev)


@dataclass
class PendingEncode:
    """An encode enqueued by encode_latent_submit, awaiting encode_finish."""
    B: int
    N: int
    C: int
    P: int
    dev: torch.device
    stream: int
    ws: torch.Tensor
    max_rounds: torch.Tensor
    inputs: tuple  # (y, medians, cdfs, cdf_sizes, offsets): kept until the finish
    done: bool = False


def encode_latent_submit(y: torch.Tensor, medians: torch.Tensor, cdfs: torch.Tensor, cdf_sizes: torch.Tensor,
                         offsets: torch.Tensor, P: int) -> PendingEncode:
    """Enqueue encode_latent's work on the current stream and return at once;
    encode_finish returns its EncodeResult.  The caller may enqueue other
    work on the stream in between (not another encode)."""
    _check_latent(y, medians, cdfs, cdf_sizes, offsets)
    B = int(y.shape[0])
    N = int(y.numel() // max(B, 1))
    C, L = (int(v) for v in cdfs.shape)
    if B <= 0 or N <= 0 or y.shape[1] != C:
        raise RuntimeError("latent channels must equal the CDF count")
    dev = y.device
    with _native.on_device(dev):
        stream = _native.stream_handle(dev)
        K, nbytes = _encode_sizes(B, N, C, P)
        max_rounds = torch.empty((B, K), dtype=torch.uint32, device=dev)
        ws = workspace("encode", dev, stream, nbytes)
        rc = _native.lib().fcai_warp_div_encode_latent_submit(
            _ptr(y), _ptr(medians), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes), _ptr(offsets), int(P), _ptr(ws),
            ws.numel(), _ptr(max_rounds), stream)
        if rc:
            _native.check(rc)
        _native.count_launches(1)
    return PendingEncode(B, N, C, int(P), dev, stream, ws, max_rounds, (y, medians, cdfs, cdf_sizes, offsets))


def encode_finish(pending: PendingEncode) -> EncodeResult:
    """Wait for a submitted encode (only), then allocate and pack its payload
    on the stream it was submitted on.  A staging overflow repeats the encode
    synchronously with the workspace it needs."""
    if pending.done:
        raise RuntimeError("this encode was already finished")
    pending.done = True
    p = pending
    with _native.on_device(p.dev):
        info = _native.WarpDivEncodeInfo()
        rc = _native.lib().fcai_warp_div_encode_finish(p.B, p.N, p.C, p.P, p.ws.numel(), ctypes.byref(info), p.stream)
        if rc == _native.FCAI_ERR_WORKSPACE:
            with torch.cuda.stream(torch.cuda.ExternalStream(p.stream, device=p.dev)):
                return encode_latent(*p.inputs, p.P)
        _native.check(rc)
        return _pack(p.B, p.N, p.C, p.P, p.ws, p.max_rounds, info, p.stream, p.dev)


def encode(symbols: torch.Tensor, indexes: torch.Tensor | None, cdfs: torch.Tensor, cdf_sizes: torch.Tensor,
           offsets: torch.Tensor, P: int) -> EncodeResult:
    """Encode; ``indexes=None`` means the channel layout ``index = i // (N // C)``."""
    _check_encode_inputs(symbols, indexes, cdfs, cdf_sizes, offsets)
    B, N = (int(v) for v in symbols.shape)
    C, L = (int(v) for v in cdfs.shape)
    if B <= 0 or N <= 0 or C <= 0 or L < 2:
        raise RuntimeError("empty/invalid coder input dimensions")

    def call(lib, ws, max_rounds, info, stream):
        return lib.fcai_warp_div_encode(_ptr(symbols), _ptr(indexes), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes),
                                        _ptr(offsets), int(P), _ptr(ws), ws.numel(), _ptr(max_rounds),
                                        ctypes.byref(info), stream)

    return _run_encode(B, N, C, P, symbols.device, call)


def _check_latent(y: torch.Tensor, medians: torch.Tensor, cdfs, cdf_sizes, offsets) -> None:
    if not (isinstance(y, torch.Tensor) and y.is_cuda and y.dtype == torch.float32 and y.is_contiguous()):
        raise RuntimeError("latent must be a contiguous CUDA float32 tensor [B, C, ...]")
    if not (isinstance(medians, torch.Tensor) and medians.dtype == torch.float32 and medians.is_contiguous()
            and medians.numel() == cdfs.shape[0] and medians.device == y.device):
        raise RuntimeError("medians must be a contiguous float32 [C] tensor on the latent's device")
    # the table checks of _check_encode_inputs, without a symbols tensor
    tables = (cdfs, cdf_sizes, offsets)
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in tables):
        raise RuntimeError("CUDA required")
    if any(t.device != y.device for t in tables):
        raise RuntimeError("all coder tensors must share a CUDA device")
    if any(t.dtype != torch.int32 for t in tables):
        raise RuntimeError("all coder inputs must be int32")
    if not all(t.is_contiguous() for t in tables):
        raise RuntimeError("all coder inputs must be contiguous")
    if cdfs.dim() != 2 or cdf_sizes.dim() != 1 or offsets.dim() != 1:
        raise RuntimeError("invalid coder input ranks/shapes")
    if cdf_sizes.numel() != cdfs.shape[0] or offsets.numel() != cdfs.shape[0]:
        raise RuntimeError("CDF metadata length mismatch")


def encode_latent(y: torch.Tensor, medians: torch.Tensor, cdfs: torch.Tensor, cdf_sizes: torch.Tensor,
                  offsets: torch.Tensor, P: int) -> EncodeResult:
    """Quantize (``rint(y - median)``) and encode the latent y [B, C, ...] in one kernel."""
    _check_latent(y, medians, cdfs, cdf_sizes, offsets)
    B = int(y.shape[0])
    N = int(y.numel() // max(B, 1))
    C, L = (int(v) for v in cdfs.shape)
    if B <= 0 or N <= 0 or y.shape[1] != C:
        raise RuntimeError("latent channels must equal the CDF count")

    def call(lib, ws, max_rounds, info, stream):
        return lib.fcai_warp_div_encode_latent(_ptr(y), _ptr(medians), B, N, _ptr(cdfs), C, L, _ptr(cdf_sizes),
                                               _ptr(offsets), int(P), _ptr(ws), ws.numel(), _ptr(max_rounds),
                                               ctypes.byref(info), stream)

    return _run_encode(B, N, C, P, y.device, call)


def decode_latent(packed: torch.Tensor, max_rounds: torch.Tensor, header_bytes: int, chunk_len: int,
                  cdfs: torch.Tensor, cdf_sizes: torch.Tensor, offsets: torch.Tensor, medians: torch.Tensor,
                  out: torch.Tensor, check: bool = True) -> torch.Tensor:
    """Decode into the dequantised fp32 latent ``out`` [B, C, ...] (``symbol + median``).

    check=True waits for the GPU and raises on an inconsistent payload;
    check=False returns at once (for payloads whose header is known to agree
    with ``max_rounds``; a damaged body then decodes to unspecified values,
    every read staying in bounds)."""
    if not (out.is_cuda and out.dtype == torch.float32 and out.is_contiguous()):
        raise RuntimeError("output latent must be a contiguous CUDA float32 tensor")
    _check_latent(out, medians, cdfs, cdf_sizes, offsets)
    if packed.dtype != torch.uint8 or not packed.is_contiguous() or packed.device != out.device:
        raise RuntimeError("packed payload must be contiguous uint8 on the latent's device")
    B = int(out.shape[0])
    N = int(out.numel() // B)
    C, L = (int(v) for v in cdfs.shape)
    if max_rounds.dim() != 2 or max_rounds.shape[0] != B or not max_rounds.is_contiguous():
        raise RuntimeError("max_rounds dim0 mismatch")
    K = int(max_rounds.shape[1])
    dev = out.device
    with _native.on_device(dev):
        stream = _native.stream_handle(dev)
        nbytes = 256 + ((B * K * 8 + 255) // 256) * 256
        ws = workspace("decode", dev, stream, nbytes)
        rc = _native.lib().fcai_warp_div_decode_latent(
            _ptr(packed), packed.numel(), _ptr(max_rounds), K, int(header_bytes), int(chunk_len), B, N, _ptr(cdfs),
            C, L, _ptr(cdf_sizes), _ptr(offsets), _ptr(medians), _ptr(out), _ptr(ws), ws.numel(), 1 if check else 0,
            stream)
        # the prep kernel runs for checked decodes and for many chunks
        _native.count_launches(2 if check or B * K > _native.INLINE_OFFSET_CHUNKS else 1)
        if rc:
            _native.check(rc)
    return out


def decode(packed: torch.Tensor, max_rounds: torch.Tensor, header_bytes: int, chunk_len: int,
           indexes: torch.Tensor | None, cdfs: torch.Tensor, cdf_sizes: torch.Tensor, offsets: torch.Tensor,
           batch: int | None = None, symbols_per_batch: int | None = None,
           out: torch.Tensor | None = None, return_layout: bool = False):
    """Decode; ``indexes=None`` means the channel layout (then give batch/symbols_per_batch).

    With ``return_layout`` returns ``(symbols, indexes_are_channel_layout)``."""
    # coders/cuda/warp_ans_kernel.cu:483-487
    tensors = [t for t in (packed, max_rounds, indexes, cdfs, cdf_sizes, offsets) if t is not None]
    if not all(isinstance(t, torch.Tensor) and t.is_cuda for t in tensors):
        raise RuntimeError("CUDA required")
    if any(t.device != packed.device for t in tensors):
        raise RuntimeError("all decode tensors must share a CUDA device")
    if any(t.dtype != torch.int32 for t in (indexes, cdfs, cdf_sizes, offsets) if t is not None):
        raise RuntimeError("indexes/CDF metadata must be int32")
    if packed.dtype != torch.uint8:
        raise RuntimeError("expected scalar type Byte for the packed payload")
    if not all(t.is_contiguous() for t in tensors):
        raise RuntimeError("decode tensors must be contiguous")
    if ((indexes is not None and indexes.dim() != 2) or cdfs.dim() != 2 or cdf_sizes.dim() != 1
            or offsets.dim() != 1 or max_rounds.dim() != 2):
        raise RuntimeError("invalid decode tensor ranks")
    if indexes is not None:
        B, N = (int(v) for v in indexes.shape)
    else:
        B, N = int(batch), int(symbols_per_batch)
    C, L = (int(v) for v in cdfs.shape)
    if max_rounds.shape[0] != B:
        raise RuntimeError("max_rounds dim0 mismatch")
    K = int(max_rounds.shape[1])
    rounds32 = max_rounds if max_rounds.dtype in (torch.int32, torch.uint32) else max_rounds.to(torch.int32)
    dev = packed.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        if out is None:
            out = torch.empty((B, N), dtype=torch.int32, device=dev)
        nbytes = 256 + ((B * K * 8 + 255) // 256) * 256
        ws = workspace("decode", dev, stream, nbytes)
        layout = ctypes.c_int32(1)
        rc = _native.lib().fcai_warp_div_decode(
            _ptr(packed), packed.numel(), _ptr(rounds32), K, int(header_bytes), int(chunk_len), _ptr(indexes), B,
            N, _ptr(cdfs), C, L, _ptr(cdf_sizes), _ptr(offsets), _ptr(out), _ptr(ws), ws.numel(), 1,
            ctypes.byref(layout), ctypes.c_void_p(stream))
        _native.count_launches(2)
        _native.check(rc)
    return (out, bool(layout.value)) if return_layout else out


def encode_warp_div(symbols_bxn, indexes_bxn, cdfs_mxl, cdf_sizes_m, offsets_m, P):
    """Reference contract: coders/cuda/ans_gpu.cpp:26-27."""
    try:
        r = encode(symbols_bxn, indexes_bxn, cdfs_mxl, cdf_sizes_m, offsets_m, int(P))
    except _native.NativeCallError as exc:
        raise RuntimeError(str(exc)) from exc
    return (
        r.packed,
        r.max_rounds,
        torch.tensor([r.header_bytes], dtype=torch.int64),
        torch.tensor([r.chunk_len], dtype=torch.int32),
        torch.tensor([r.p_ch], dtype=torch.int32),
    )


def decode_warp_div(packed_u8, max_rounds_u32, header_bytes_cpu, chunk_len_cpu, P_cpu, indexes_bxn, cdfs_mxl,
                    cdf_sizes_m, offsets_m):
    """Reference contract: coders/cuda/ans_gpu.cpp:28-29 (P is not used, as there)."""
    del P_cpu
    try:
        return decode(packed_u8, max_rounds_u32, int(header_bytes_cpu[0]), int(chunk_len_cpu[0]), indexes_bxn,
                      cdfs_mxl, cdf_sizes_m, offsets_m)
    except _native.NativeCallError as exc:
        raise RuntimeError(str(exc)) from exc
