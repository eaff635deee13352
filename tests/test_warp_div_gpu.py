"""GPU parity tests of the warp_div coder through the C ABI.

Every payload is compared byte for byte with the CPU oracle (pad bytes
included: both write zeros), and every decode with the original symbols.
Sizes the oracle finishes in seconds are compared directly; the full
BASELINE config-3 shapes are checked through size-independent properties
(round trip, payload length = header + 128 * sum(rounds), header words).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fast_compressai.coders import _warp_div as ext
from fast_compressai.coders.errors import CoderInputError
from fast_compressai.coders.warp_div import WarpDivBackend, WarpDivPayload
from oracle import oracle as O
from tests.coder_inputs import channel_indexes, laplacian_symbols, laplacian_tables, small_tables

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _compare(sym, idx, cdfs, sizes, offs, P, device, explicit=True):
    ref_packed, ref_mr, ref_hb, ref_cl = O.warp_div_encode(sym, idx, cdfs, sizes, offs, P)
    t = [_dev(a, device) for a in (sym, idx, cdfs, sizes, offs)]
    r = ext.encode(t[0], t[1] if explicit else None, t[2], t[3], t[4], P)
    torch.cuda.synchronize()
    assert r.header_bytes == ref_hb and r.chunk_len == ref_cl and r.p_ch == P
    assert np.array_equal(r.max_rounds.cpu().numpy(), ref_mr)
    got = r.packed.cpu().numpy()
    assert got.size == ref_packed.size
    assert np.array_equal(got, ref_packed), f"first diff at byte {np.argmax(got != ref_packed)}"
    dec = ext.decode(r.packed, r.max_rounds, r.header_bytes, r.chunk_len, t[1] if explicit else None, t[2], t[3],
                     t[4], batch=sym.shape[0], symbols_per_batch=sym.shape[1])
    assert np.array_equal(dec.cpu().numpy(), sym)
    return r


@pytest.mark.parametrize("P", [1, 2, 4])
def test_reference_known_answer_cases(cuda_device, P):
    # tests/gpu/test_warp_div_cuda.py:18-38 of the reference
    cdfs, sizes, offs = small_tables()
    idx = np.array([[0, 1, 2, 3] * 16], dtype=np.int32)
    for sym in ([0, 1, 2, 3] * 16, [-100, 100, -101, 102] * 16):
        _compare(np.array([sym], dtype=np.int32), idx, cdfs, sizes, offs, P, cuda_device)


@pytest.mark.parametrize(
    "B,C,HW,P,esc",
    [(1, 12, 16, 4, 0.0), (2, 12, 16, 5, 0.02), (2, 12, 16, 12, 0.0), (3, 7, 33, 3, 0.05), (1, 4, 1, 1, 0.3),
     (4, 16, 100, 16, 0.0), (2, 192, 48, 4, 0.001), (2, 192, 48, 192, 0.0), (1, 5, 7, 2, 0.5),
     (2, 320, 64, 8, 0.0), (1, 3, 1000, 1, 0.01),
     # >= 148 chunk groups: decode CTAs of 5 and 7 decoding warps plus staging-only warps
     (5, 192, 32, 1, 0.01), (7, 160, 16, 1, 0.0)],
)
def test_payload_bit_exact_vs_oracle(cuda_device, B, C, HW, P, esc):
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=C + P)
    sym = laplacian_symbols(B, C, HW, scales, seed=B + HW, escape_rate=esc)
    idx = channel_indexes(B, C, HW)
    r1 = _compare(sym, idx, cdfs, sizes, offs, P, cuda_device, explicit=True)
    r2 = _compare(sym, idx, cdfs, sizes, offs, P, cuda_device, explicit=False)
    assert r1.index_layout_is_channel and r2.index_layout_is_channel


def test_arbitrary_indexes_and_short_rows(cuda_device):
    rng = np.random.default_rng(9)
    cdfs, sizes, offs, _ = laplacian_tables(6, seed=7)
    sizes = sizes.copy()
    sizes[2] = 10
    cdfs[2, 9] = 65536
    cdfs[2, 10:] = 0
    sym = rng.integers(-40, 40, size=(3, 6 * 50)).astype(np.int32)
    idx = rng.integers(0, 6, size=(3, 6 * 50)).astype(np.int32)
    r = _compare(sym, idx, cdfs, sizes, offs, 4, cuda_device)
    assert not r.index_layout_is_channel


@pytest.mark.parametrize("B,C,HW,P", [(32767, 4, 1, 4), (1, 46340, 1, 1)])
def test_largest_batch_and_channel_counts(cuda_device, B, C, HW, P):
    # the largest batch the reference's decode accepts (its header compares
    # batch << 16 as int32) and a channel count at the N * C < 2^31 limit:
    # tens of thousands of one-chunk groups through the persistent grids
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=3)
    sym = laplacian_symbols(B, C, HW, scales, seed=4, escape_rate=0.01)
    r = _compare(sym, channel_indexes(B, C, HW), cdfs, sizes, offs, P, cuda_device, explicit=False)
    assert r.max_rounds.shape == (B, (C + P - 1) // P)


@pytest.mark.parametrize("B,C,HW,P,esc", [(3, 40, 97, 8, 0.02), (2, 24, 256, 3, 0.0), (2, 96, 64, 48, 0.01),
                                          (4, 10, 33, 1, 0.05)])
def test_mixed_indexes_fast_and_checked_paths(cuda_device, B, C, HW, P, esc):
    # mostly the channel layout (vote-checked fast batches) with scattered
    # positions naming another row, inside the chunk's group or outside it
    # (rows read from global memory), escapes included
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=C * P)
    sym = laplacian_symbols(B, C, HW, scales, seed=HW, escape_rate=esc)
    idx = channel_indexes(B, C, HW).copy()
    rng = np.random.default_rng(B * C + HW)
    pos = rng.random(idx.shape) < 0.01
    idx[pos] = rng.integers(0, C, size=int(pos.sum()))
    near = rng.random(idx.shape) < 0.01
    idx[near] = np.minimum(C - 1, idx[near] + 1)
    r = _compare(sym, idx, cdfs, sizes, offs, P, cuda_device)
    assert not r.index_layout_is_channel


def test_extreme_symbol_values(cuda_device):
    cdfs, sizes, offs = small_tables()
    big = np.array([[2**31 - 1, -(2**31), 2**30 - 7, -(2**30) + 3] * 8], dtype=np.int32)
    idx = np.array([[0, 1, 2, 3] * 8], dtype=np.int32)
    ref_packed, ref_mr, hb, cl = O.warp_div_encode(big, idx, cdfs, sizes, offs, 1)
    t = [_dev(a, cuda_device) for a in (big, idx, cdfs, sizes, offs)]
    r = ext.encode(*t, 1)
    assert np.array_equal(r.packed.cpu().numpy(), ref_packed)
    dec = ext.decode(r.packed, r.max_rounds, r.header_bytes, r.chunk_len, t[1], t[2], t[3], t[4]).cpu().numpy()
    assert np.array_equal(dec, O.warp_div_decode(ref_packed, ref_mr, hb, cl, idx, cdfs, sizes, offs))


def test_latent_entry_points_match_symbol_path(cuda_device):
    B, C, H, W = 2, 12, 5, 7
    torch.manual_seed(3)
    y = (torch.randn(B, C, H, W, device=cuda_device) * 6).contiguous()
    y[0, 0, 0, :4] = torch.tensor([0.5, 1.5, -0.5, -2.5])  # ties round to even
    med = (torch.randn(C, device=cuda_device) * 0.3).contiguous()
    cdfs, sizes, offs, _ = laplacian_tables(C, seed=2, lo=-8, hi=8)
    cdfs_t, sizes_t, offs_t = (_dev(a, cuda_device) for a in (cdfs, sizes, offs))
    sym = torch.round(y - med.reshape(1, C, 1, 1)).int().reshape(B, -1).contiguous()
    a = ext.encode(sym, None, cdfs_t, sizes_t, offs_t, 3)
    b = ext.encode_latent(y, med, cdfs_t, sizes_t, offs_t, 3)
    assert torch.equal(a.packed, b.packed) and torch.equal(a.max_rounds, b.max_rounds)
    out = torch.empty_like(y)
    ext.decode_latent(b.packed, b.max_rounds, b.header_bytes, b.chunk_len, cdfs_t, sizes_t, offs_t, med, out)
    expect = sym.reshape(B, C, H, W).float() + med.reshape(1, C, 1, 1)
    assert torch.equal(out, expect)


def test_workspace_retry_path(cuda_device):
    # escapes everywhere need far more staging than the first workspace guess
    cdfs, sizes, offs = small_tables()
    rng = np.random.default_rng(1)
    sym = rng.integers(2**28, 2**29, size=(2, 4 * 256)).astype(np.int32)  # 8-nibble escapes
    idx = np.tile(np.repeat(np.arange(4, dtype=np.int32), 256), (2, 1))
    ext.release_workspaces()
    _compare(sym, idx, cdfs, sizes, offs, 1, cuda_device)


def test_config3_shapes_round_trip(cuda_device):
    # 64 x 192 x 32 x 48 symbols, P swept
    B, C, HW = 64, 192, 32 * 48
    cdfs, sizes, offs, scales = laplacian_tables(C, seed=0)
    sym = _dev(laplacian_symbols(B, C, HW, scales, seed=0), cuda_device)
    cdfs_t, sizes_t, offs_t = (_dev(a, cuda_device) for a in (cdfs, sizes, offs))
    for P in (1, 2, 4, 8, 16, 48, 192):
        r = ext.encode(sym, None, cdfs_t, sizes_t, offs_t, P)
        K = (C + P - 1) // P
        assert r.max_rounds.shape == (B, K)
        rounds = r.max_rounds.to(torch.int64)
        assert int(rounds.min()) >= 2
        assert r.packed.numel() == r.header_bytes + 128 * int(rounds.sum())
        hdr = r.packed[:32].cpu().numpy().view(np.uint32)
        assert hdr[0] == C * HW and hdr[1] == P * HW and hdr[2] == (K | (B << 16))
        dec = ext.decode(r.packed, r.max_rounds, r.header_bytes, r.chunk_len, None, cdfs_t, sizes_t, offs_t,
                         batch=B, symbols_per_batch=C * HW)
        assert torch.equal(dec, sym), P
    # one image of the batch against the oracle, bytes of its chunks
    one = sym[:1].cpu().numpy()
    ref_packed, _, hb, _ = O.warp_div_encode(one, None, cdfs, sizes, offs, 4)
    r = ext.encode(sym[:1].contiguous(), None, cdfs_t, sizes_t, offs_t, 4)
    assert np.array_equal(r.packed.cpu().numpy(), ref_packed)


def _backend_case(device):
    cdfs, sizes, offs, scales = laplacian_tables(12, seed=5)
    sym = laplacian_symbols(2, 12, 16, scales, seed=6, escape_rate=0.02)
    idx = channel_indexes(2, 12, 16)
    t = [_dev(a, device) for a in (sym, idx, cdfs, sizes, offs)]
    return t


def test_backend_round_trip_and_payload_contract(cuda_device):
    sym, idx, cdfs, sizes, offs = _backend_case(cuda_device)
    be = WarpDivBackend()
    payload = be.encode(sym, idx, cdfs, sizes, offs, p_ch=5)
    assert isinstance(payload, WarpDivPayload)
    assert payload.format_id == "warpans-v2-warp-div-v1-decode" and payload.p_ch == 5
    assert payload.max_rounds.dtype == torch.uint32 and payload.max_rounds.shape == (2, 3)
    assert len(payload.coding_fingerprint) == 64
    assert torch.equal(be.decode(payload, idx, cdfs, sizes, offs), sym)
    # the reference's tuple contract
    packed, mr, hb, cl, p = ext.encode_warp_div(sym, idx, cdfs, sizes, offs, 5)
    assert torch.equal(packed, payload.packed) and int(hb[0]) == payload.header_bytes and int(p[0]) == 5
    assert hb.device.type == "cpu" and cl.dtype == torch.int32
    out = ext.decode_warp_div(packed, mr, hb, cl, p, idx, cdfs, sizes, offs)
    assert torch.equal(out, sym)


def test_backend_rejections(cuda_device):
    # negative cases of tests/gpu/test_factorized_gaans.py:120-143 of the reference, at the backend
    from dataclasses import replace

    sym, idx, cdfs, sizes, offs = _backend_case(cuda_device)
    be = WarpDivBackend()
    payload = be.encode(sym, idx, cdfs, sizes, offs, p_ch=4)
    with pytest.raises(CoderInputError, match="match"):
        replace(payload, p_ch=3, chunk_len=48)
    with pytest.raises(CoderInputError, match="match"):
        be.decode(replace(payload, coding_fingerprint="0" * 64), idx, cdfs, sizes, offs)
    bad = payload.packed.clone()
    bad[0] ^= 1
    with pytest.raises(CoderInputError, match="header"):
        be.decode(replace(payload, packed=bad), idx, cdfs, sizes, offs)
    bad = payload.packed.clone()
    bad[32] ^= 1  # round table entry of chunk 0
    with pytest.raises(CoderInputError, match="round counts"):
        be.decode(replace(payload, packed=bad), idx, cdfs, sizes, offs)
    with pytest.raises(CoderInputError, match="length does not match"):
        replace(payload, packed=payload.packed[:-128].contiguous())
    wrong = idx.clone()
    wrong[0, 0] = 12
    with pytest.raises(CoderInputError, match="outside the CDF table range"):
        be.encode(sym, wrong, cdfs, sizes, offs, p_ch=4)
    with pytest.raises(CoderInputError, match="outside the CDF table range"):
        be.decode(payload, wrong, cdfs, sizes, offs)
    with pytest.raises(CoderInputError):
        be.encode(sym, idx, cdfs, sizes, offs, p_ch=13)
    bad_sizes = sizes.clone()
    bad_sizes[0] = cdfs.shape[1] + 1
    with pytest.raises(CoderInputError, match="CDF table invalid"):
        be.encode(sym, idx, cdfs, bad_sizes, offs, p_ch=4)


def test_corrupt_body_is_reported_not_read_out_of_bounds(cuda_device):
    sym, idx, cdfs, sizes, offs = _backend_case(cuda_device)
    be = WarpDivBackend()
    payload = be.encode(sym, idx, cdfs, sizes, offs, p_ch=2)
    rng = np.random.default_rng(0)
    for trial in range(20):
        body = payload.packed.clone()
        n = body.numel() - payload.header_bytes
        pos = payload.header_bytes + torch.from_numpy(rng.integers(0, n, size=8)).to(cuda_device)
        body[pos] = torch.from_numpy(rng.integers(0, 256, size=8).astype(np.uint8)).to(cuda_device)
        corrupted = WarpDivPayload(body, payload.max_rounds, payload.header_bytes, payload.chunk_len, payload.p_ch,
                                   payload.batch, payload.symbols_per_batch, payload.cdf_count, None)
        try:
            out = be.decode(corrupted, idx, cdfs, sizes, offs)
        except CoderInputError as exc:
            assert "inconsistent" in str(exc)
        else:
            assert out.shape == sym.shape
    torch.cuda.synchronize()


@pytest.mark.parametrize("nbytes,offset", [(1, 0), (15, 3), (4096, 0), (100003, 5), (3 << 20, 0)])
def test_payload_copy_kernel_round_trip(cuda_device, nbytes, offset):
    # fcai_payload_copy_async moves bytes between device memory and pinned
    # mapped host memory with SM loads / stores (16-byte path plus a byte
    # tail, unaligned starts included), in both directions
    from fast_compressai.coders.warp_div import _kernel_copy

    rng = np.random.default_rng(nbytes)
    data = torch.from_numpy(rng.integers(0, 256, size=nbytes + offset, dtype=np.uint8))
    host_src = data.pin_memory()[offset:]
    dev = torch.empty(nbytes, dtype=torch.uint8, device=cuda_device)
    assert _kernel_copy(dev, host_src)
    host_dst = torch.zeros(nbytes + offset, dtype=torch.uint8).pin_memory()[offset:]
    assert _kernel_copy(host_dst, dev)
    torch.cuda.synchronize()
    assert torch.equal(dev.cpu(), data[offset:])
    assert torch.equal(host_dst, data[offset:])
    # pageable host memory is not mapped: refused, nothing launched
    assert not _kernel_copy(dev, data[offset:].clone())


def test_payload_through_host_memory_without_copy_engines(cuda_device):
    # packed_to_host and from_host_packed(non_blocking=True) carry a payload
    # down and back up with the payload kernel; max_rounds is then a view of
    # the uploaded header, the result decodes like the original, and it is
    # marked consistent (asynchronous decode)
    from fast_compressai.coders.warp_div import _is_consistent

    sym, idx, cdfs, sizes, offs = _backend_case(cuda_device)
    be = WarpDivBackend()
    payload = be.encode(sym, idx, cdfs, sizes, offs, p_ch=2)
    buf = torch.empty(payload.packed.numel() + 64, dtype=torch.uint8).pin_memory()
    host = payload.packed_to_host(buf)
    torch.cuda.synchronize()
    assert host.data_ptr() == buf.data_ptr() and torch.equal(host, payload.packed.cpu())
    q = WarpDivPayload.from_host_packed(host, batch=payload.batch, symbols_per_batch=payload.symbols_per_batch,
                                        cdf_count=payload.cdf_count, p_ch=payload.p_ch, chunk_len=payload.chunk_len,
                                        header_bytes=payload.header_bytes,
                                        coding_fingerprint=payload.coding_fingerprint, device=cuda_device,
                                        non_blocking=True)
    assert torch.equal(q.packed, payload.packed)
    assert q.max_rounds.dtype == torch.uint32 and torch.equal(q.max_rounds.cpu(), payload.max_rounds.cpu())
    assert _is_consistent(q)
    assert torch.equal(be.decode(q, idx, cdfs, sizes, offs), sym)
    with pytest.raises(CoderInputError):
        payload.packed_to_host(torch.empty(4, dtype=torch.uint8))
