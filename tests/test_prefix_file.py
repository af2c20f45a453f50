"""Prefix-state snapshot file (format v3): the reference's own persistence tests transcribed
(src/server/prefix_persist.zig:443-639) against the library's host reader/writer (CPU), plus a
GPU restore of a file image from pinned memory into the paged cache (bit-exact vs the oracle)
and the snapshot back into an identical file."""
import numpy as np
import pytest

from _util import NKV, D, PAGE, dev, host_u16

FP = 0x1234_5678_9ABC_DEF0


@pytest.fixture(scope="module")
def capi():
    from peregrine_b200 import build, capi as c
    build.build()
    return c


def _image(capi, fixtures, count, next_token=4242, hidden_fill=None):
    """File image with the fill pattern of the reference round-trip test: per layer in model
    order, linear -> conv=fill, recur=fill+1; full -> K=fill, V=fill+1; fill += 2 (u8)."""
    lay = capi.prefix_file_layout(count)
    img = np.zeros(lay.total_bytes, np.uint8)
    img[lay.tokens:lay.tokens + 4 * count] = np.arange(100, 100 + count, dtype=np.uint32).view(np.uint8)
    fill = fixtures["persist"]["fill_start"]
    li = fi = 0
    for is_lin in fixtures["topology"]["is_linear"]:
        if is_lin:
            img[lay.conv[li]:lay.recur[li]] = fill
            end = lay.recur[li] + 32 * 128 * 128 * 4
            img[lay.recur[li]:end] = (fill + 1) & 0xFF
            li += 1
        else:
            kv = 4 * count * 256 * 2
            img[lay.k_runs[fi]:lay.k_runs[fi] + kv] = fill
            img[lay.v_runs[fi]:lay.v_runs[fi] + kv] = (fill + 1) & 0xFF
            fi += 1
        fill = (fill + 2) & 0xFF
    if hidden_fill is not None:
        img[lay.hidden:] = hidden_fill
    capi.prefix_file_header(img.ctypes.data, img.nbytes, FP, count, next_token, True,
                            hidden_fill is not None)
    return img, lay


def test_layout_matches_expected_file_bytes(capi, fixtures):
    # prefix_persist.zig:443-455 (16153 tokens) and the 7-token round-trip file
    t = fixtures["topology"]
    for n in (fixtures["persist"]["expected_file_bytes_token_count"], 7):
        conv = (t["conv_k"] - 1) * t["conv_dim"] * 4
        recur = t["hv"] * t["dv"] * t["dk"] * 4
        kv = NKV * n * D * 2
        expected = 48 + n * 4 + 24 * (conv + recur) + 8 * 2 * kv + n * t["hidden"] * 2
        assert capi.prefix_file_layout(n).total_bytes == expected


def test_round_trip_and_validation(capi, fixtures, tmp_path):
    from peregrine_b200.capi import PgcError
    count = fixtures["persist"]["roundtrip_token_count"]
    img, lay = _image(capi, fixtures, count)
    path = tmp_path / "prefix-state.bin"
    capi.prefix_file_write(path, img.ctypes.data, img.nbytes)
    assert path.read_bytes()[:8] == b"PRGPFXS1" and path.stat().st_size == lay.total_bytes
    info = capi.prefix_file_inspect(path, FP, 8192, 64)
    assert (info.token_count, info.next_token, info.next_token_valid, info.hidden_valid) == (count, 4242, 1, 0)
    back = np.zeros_like(img)
    capi.prefix_file_read(path, FP, 8192, 64, back.ctypes.data, back.nbytes)
    assert np.array_equal(back, img)
    # every full-attention run holds its layer's fill byte (fullCacheRuns order)
    fill = fixtures["persist"]["fill_start"]
    fi = 0
    for is_lin in fixtures["topology"]["is_linear"]:
        if not is_lin:
            assert (back[lay.k_runs[fi]:lay.v_runs[fi]] == fill).all()
            fi += 1
        fill = (fill + 2) & 0xFF
    # rejected files (load() returns null; the caller cold-prefills)
    for args in [(FP + 1, 8192, 64), (FP, 100, 64), (FP, 8192, count - 1)]:
        with pytest.raises(PgcError, match="FORMAT"):
            capi.prefix_file_inspect(path, *args)
    trunc = tmp_path / "trunc.bin"
    trunc.write_bytes(path.read_bytes()[:-1])
    with pytest.raises(PgcError, match="FORMAT"):
        capi.prefix_file_inspect(trunc, FP, 8192, 64)
    bad = tmp_path / "bad.bin"
    raw = bytearray(path.read_bytes())
    raw[0] ^= 0xFF
    bad.write_bytes(bytes(raw))
    with pytest.raises(PgcError, match="FORMAT"):
        capi.prefix_file_inspect(bad, FP, 8192, 64)
    with pytest.raises(PgcError, match="FILE"):
        capi.prefix_file_inspect(tmp_path / "missing.bin", FP, 8192, 64)


def test_hidden_section_flags(capi, fixtures, tmp_path):
    # prefix_persist.zig:543-639: real hidden rows round-trip with hidden_valid set; a file from
    # a non-MTP run carries a zero-filled section with the flag clear
    img, lay = _image(capi, fixtures, 5, hidden_fill=0x5A)
    p = tmp_path / "h.bin"
    capi.prefix_file_write(p, img.ctypes.data, img.nbytes)
    info = capi.prefix_file_inspect(p, FP, 8192, 64)
    assert info.hidden_valid == 1
    assert (np.frombuffer(p.read_bytes(), np.uint8)[lay.hidden:] == 0x5A).all()
    img2, lay2 = _image(capi, fixtures, 5)
    p2 = tmp_path / "h2.bin"
    capi.prefix_file_write(p2, img2.ctypes.data, img2.nbytes)
    assert capi.prefix_file_inspect(p2, FP, 8192, 64).hidden_valid == 0
    assert (np.frombuffer(p2.read_bytes(), np.uint8)[lay2.hidden:] == 0).all()


@pytest.mark.gpu
def test_restore_file_into_pages_and_snapshot_back(cuda, oracle, tmp_path):
    """A v3 image in pinned host memory -> paged K/V (pgc_kv_restore_dense reads the runs with
    src_stride = count, straight over the host link) -> bit-exact vs the oracle -> snapshot back
    into a fresh image (pgc_kv_snapshot_dense) -> the same file bytes."""
    import torch
    count = 1001  # odd: the K/V runs of the file are only 4-byte aligned
    lay = cuda.prefix_file_layout(count)
    rng = np.random.default_rng(0)
    img = torch.from_numpy(rng.integers(0, 255, lay.total_bytes, dtype=np.uint8)).pin_memory()
    cuda.prefix_file_header(img.data_ptr(), lay.total_bytes, FP, count, 7, True, True)
    img.numpy()[lay.tokens:lay.tokens + 4 * count] = np.arange(count, dtype=np.uint32).view(np.uint8)
    path = tmp_path / "state.bin"
    cuda.prefix_file_write(path, img.data_ptr(), lay.total_bytes)
    loaded = torch.empty(lay.total_bytes, dtype=torch.uint8).pin_memory()
    cuda.prefix_file_read(path, FP, 50000, 65536, loaded.data_ptr(), lay.total_bytes)
    npages = (count + PAGE - 1) // PAGE + 9
    table = rng.permutation(npages).astype(np.int32)
    kv_elems = 4 * count * 256
    out_img = loaded.clone().pin_memory()  # header, tokens, linear states, hidden rows
    for f in range(8):  # K/V runs are re-created by the snapshot below
        out_img.numpy()[lay.k_runs[f]:lay.v_runs[f] + 2 * 4 * count * 256] = 0
    for f in range(8):
        kp = torch.zeros((npages, NKV, PAGE, D), dtype=torch.int16, device="cuda")
        vp = torch.zeros_like(kp)
        kd = loaded.data_ptr() + lay.k_runs[f]
        vd = loaded.data_ptr() + lay.v_runs[f]
        from peregrine_b200.capi import check, lib
        tbl = dev(table)  # keep the table alive until the kernels have run
        check(lib().pgc_kv_restore_dense(kd, vd, count, 0, kp.data_ptr(), vp.data_ptr(), npages,
                                         tbl.data_ptr(), npages, 0, count, None),
              "restore")
        torch.cuda.synchronize()
        k_np = loaded.numpy()[lay.k_runs[f]:lay.k_runs[f] + 2 * kv_elems].view(np.uint16)
        v_np = loaded.numpy()[lay.v_runs[f]:lay.v_runs[f] + 2 * kv_elems].view(np.uint16)
        ok_ = np.zeros((npages, NKV, PAGE, D), np.uint16)
        ov_ = np.zeros_like(ok_)
        assert oracle.kv_restore_dense(np.ascontiguousarray(k_np), np.ascontiguousarray(v_np),
                                       count, 0, ok_, ov_, table, 0, count) == 0
        assert np.array_equal(host_u16(kp), ok_) and np.array_equal(host_u16(vp), ov_)
        check(lib().pgc_kv_snapshot_dense(kp.data_ptr(), vp.data_ptr(), npages, tbl.data_ptr(),
                                          npages, 0, out_img.data_ptr() + lay.k_runs[f],
                                          out_img.data_ptr() + lay.v_runs[f], count, 0, count, None),
              "snapshot")
        torch.cuda.synchronize()
    path2 = tmp_path / "state2.bin"
    cuda.prefix_file_write(path2, out_img.data_ptr(), lay.total_bytes)
    assert path2.read_bytes() == path.read_bytes()
