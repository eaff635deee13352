"""WarpDivPayload.to_bytes / from_bytes: a device-independent byte form of
the payload (the reference keeps payloads device-local only: README.md:56,106
and the invariants of coders/warp_div.py:34-67).

CPU tests check that damaged containers are refused before any device work:
wrong magic, wrong container version, truncation and excess bytes, a wrong
payload format version, a header round table that is not a count.  GPU
tests round-trip payloads through bytes: on the same device, in a fresh
process (no pointer or cache of this process survives) and, with two
GPUs, from cuda:0 to cuda:1; the fingerprint and every field survive, and
a corrupted header word in the bytes is caught by the decode.
"""

from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

from fast_compressai.coders import WarpDivBackend, WarpDivPayload
from fast_compressai.coders.errors import CoderInputError
from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables

ROOT = Path(__file__).resolve().parents[1]
META = 4 + 7 * 4 + 2 * 8 + 4 + 32  # container header bytes


def _case(B=2, C=24, HW=40, P=4, seed=5):
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=seed)
    sym = laplacian_symbols(B, C, HW, scales, seed=seed + 1, escape_rate=0.01)
    return sym, channel_indexes(B, C, HW), cdfs, sizes, offs, P


def _container(packed, *, B, N, C, P, chunk_len, header_bytes, fingerprint=None, version=1, fmt=1):
    fp = bytes.fromhex(fingerprint) if fingerprint else bytes(32)
    return (b"FCWD" + np.array([version, fmt, B, N, C, P, chunk_len], dtype="<u4").tobytes()
            + np.array([header_bytes, packed.size], dtype="<u8").tobytes()
            + np.array([1 if fingerprint else 0], dtype="<u4").tobytes() + fp + packed.tobytes())


@pytest.fixture(scope="module")
def cpu_container():
    sym, idx, cdfs, sizes, offs, P = _case()
    packed, rounds, hb, chunk_len = O.warp_div_encode(sym, None, cdfs, sizes, offs, P)
    B, N = sym.shape
    kw = dict(B=B, N=N, C=cdfs.shape[0], P=P, chunk_len=chunk_len, header_bytes=hb)
    return packed, kw


def test_container_layout_is_what_to_bytes_documents(cpu_container):
    packed, kw = cpu_container
    data = _container(packed, **kw)
    assert len(data) == META + packed.size and data[:4] == b"FCWD"
    assert data[META:] == packed.tobytes()


@pytest.mark.parametrize("damage", ["magic", "container_version", "truncated", "excess", "format_version",
                                    "negative_rounds", "short_header"])
def test_damaged_containers_are_refused(cpu_container, damage):
    packed, kw = cpu_container
    data = bytearray(_container(packed, **kw))
    if damage == "magic":
        data[:4] = b"FCWX"
        match = "not a serialized"
    elif damage == "container_version":
        data = bytearray(_container(packed, version=2, **kw))
        match = "container version"
    elif damage == "truncated":
        data = data[:-1]
        match = "truncated"
    elif damage == "excess":
        data += b"\0"
        match = "truncated"
    elif damage == "format_version":
        data = bytearray(_container(packed, fmt=2, **kw))
        match = "unsupported warp_div payload format"
    elif damage == "negative_rounds":
        struct = np.frombuffer(data, dtype=np.uint8)
        struct[META + 32 + 3] = 0x80  # round count of chunk 0 read as int32 < 0
        match = "round counts are invalid"
    else:
        data = data[:META - 8]
        match = "not a serialized"
    with pytest.raises(CoderInputError, match=match):
        WarpDivPayload.from_bytes(bytes(data), device="cpu")


def _gpu_payload(device):
    sym, idx, cdfs, sizes, offs, P = _case()
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in (sym, idx, cdfs, sizes, offs)]
    payload = WarpDivBackend().encode(*t, p_ch=P)
    return payload, t


def _fields(p):
    return (p.header_bytes, p.chunk_len, p.p_ch, p.batch, p.symbols_per_batch, p.cdf_count, p.coding_fingerprint,
            p.format_id, p.format_version)


@pytest.mark.gpu
def test_round_trip_on_the_same_device(cuda_device):
    payload, (sym, idx, cdfs, sizes, offs) = _gpu_payload(cuda_device)
    data = payload.to_bytes()
    assert isinstance(data, bytes) and len(data) == META + payload.packed.numel()
    back = WarpDivPayload.from_bytes(data, device=cuda_device)
    assert back.coding_fingerprint is not None and len(back.coding_fingerprint) == 64
    assert _fields(back) == _fields(payload)
    assert torch.equal(back.packed, payload.packed) and torch.equal(back.max_rounds, payload.max_rounds)
    assert torch.equal(WarpDivBackend().decode(back, idx, cdfs, sizes, offs), sym)
    # the bytes equal the CPU oracle's payload after the container header
    want = O.warp_div_encode(sym.cpu().numpy(), None, cdfs.cpu().numpy(), sizes.cpu().numpy(), offs.cpu().numpy(),
                             payload.p_ch)[0]
    assert data[META:] == want.tobytes()


@pytest.mark.gpu
def test_corrupted_header_word_is_caught_by_the_decode(cuda_device):
    payload, (sym, idx, cdfs, sizes, offs) = _gpu_payload(cuda_device)
    data = bytearray(payload.to_bytes())
    data[META + 4] ^= 0x01  # header word h1 (chunk_len)
    back = WarpDivPayload.from_bytes(bytes(data), device=cuda_device)
    with pytest.raises(CoderInputError, match="header is inconsistent"):
        WarpDivBackend().decode(back, idx, cdfs, sizes, offs)


@pytest.mark.gpu
def test_fingerprint_mismatch_after_the_trip_is_refused(cuda_device):
    payload, (sym, idx, cdfs, sizes, offs) = _gpu_payload(cuda_device)
    back = WarpDivPayload.from_bytes(payload.to_bytes(), device=cuda_device)
    other = cdfs.clone()
    other[0, 1] -= 1  # another (still valid) table
    with pytest.raises(CoderInputError, match="do not match"):
        WarpDivBackend().decode(back, idx, other, sizes, offs)


_RESTORE = textwrap.dedent("""
    import sys
    sys.path[:0] = [sys.argv[1], sys.argv[1] + "/fast-compressai_b200"]
    import numpy as np, torch
    from fast_compressai.coders import WarpDivBackend, WarpDivPayload
    z = np.load(sys.argv[2])
    dev = torch.device(sys.argv[3])
    back = WarpDivPayload.from_bytes(z["data"].tobytes(), device=dev)
    t = [torch.from_numpy(z[k]).to(dev) for k in ("idx", "cdfs", "sizes", "offs")]
    dec = WarpDivBackend().decode(back, *t)
    assert back.coding_fingerprint == str(z["fingerprint"]), "fingerprint changed"
    assert np.array_equal(dec.cpu().numpy(), z["sym"]), "decoded symbols differ"
    print("restored ok")
""")


@pytest.mark.gpu
def test_restore_in_a_fresh_process(cuda_device, tmp_path):
    payload, (sym, idx, cdfs, sizes, offs) = _gpu_payload(cuda_device)
    f = tmp_path / "payload.npz"
    np.savez(f, data=np.frombuffer(payload.to_bytes(), dtype=np.uint8), sym=sym.cpu().numpy(),
             idx=idx.cpu().numpy(), cdfs=cdfs.cpu().numpy(), sizes=sizes.cpu().numpy(), offs=offs.cpu().numpy(),
             fingerprint=np.array(payload.coding_fingerprint))
    proc = subprocess.run([sys.executable, "-c", _RESTORE, str(ROOT), str(f), "cuda:0"], capture_output=True,
                          text=True, timeout=600, env=dict(os.environ))
    assert proc.returncode == 0 and "restored ok" in proc.stdout, proc.stderr[-2000:]


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_restore_on_a_second_gpu():
    payload, (sym, idx, cdfs, sizes, offs) = _gpu_payload(torch.device("cuda:0"))
    d1 = torch.device("cuda:1")
    back = WarpDivPayload.from_bytes(payload.to_bytes(), device=d1)
    assert back.packed.device == d1 and back.max_rounds.device == d1
    dec = WarpDivBackend().decode(back, *(t.to(d1) for t in (idx, cdfs, sizes, offs)))
    assert dec.device == d1 and torch.equal(dec.cpu(), sym.cpu())
