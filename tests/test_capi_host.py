"""C-ABI library checks that need no GPU: it loads, exports every symbol the headers declare,
and its host-only functions agree with the oracle and the reference's golden values."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from peregrine_b200 import build, capi
    build.build()
    return capi


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(pgc_\w+)\s*\(", text))
    return names


def test_exports_every_declared_symbol(lib):
    declared = _declared_symbols()
    assert len(declared) >= 15
    handle = lib.lib()
    missing = [n for n in sorted(declared) if not hasattr(handle, n)]
    assert not missing, missing
    assert set(lib.SIGNATURES) >= declared


def test_status_strings(lib):
    h = lib.lib()
    assert h.pgc_status_string(0) == b"ok"
    for code in range(-12, 0):
        assert h.pgc_status_string(code) != b"unknown status"
    assert h.pgc_version() >= 100


def test_stride_matches_golden(lib, fixtures):
    from peregrine_b200.capi import PgcError
    for max_seq, expected in fixtures["stride_cases"]:
        if expected is None:
            with pytest.raises(PgcError):
                lib.full_cache_stride_for_max_seq(max_seq)
        else:
            assert lib.full_cache_stride_for_max_seq(max_seq) == expected


def test_rope_table_bit_identical_to_oracle(lib, oracle):
    a = lib.rope_table(70000)
    b = oracle.rope_table(70000)
    assert a.view(np.uint32).tobytes() == b.view(np.uint32).tobytes()


def test_nccl_setup_host_side(lib):
    """The NCCL entry points load NCCL at run time; argument errors need no GPU, and a unique
    id (a host-side bootstrap handle) comes back as 128 bytes when NCCL is in the process."""
    import ctypes as C
    h = lib.lib()
    comm = C.c_void_p()
    assert h.pgc_nccl_comm_init(2, 2, None, C.byref(comm)) == lib.STATUS_INVALID
    assert h.pgc_nccl_get_unique_id(None) == lib.STATUS_INVALID
    assert h.pgc_nccl_comm_destroy(None) == lib.STATUS_INVALID
    import torch  # noqa: F401  (brings torch's libnccl.so.2 into the process)
    uid = (C.c_uint8 * 128)()
    st = h.pgc_nccl_get_unique_id(uid)
    assert st in (0, -12)
    if st == 0:
        assert any(bytes(uid))
