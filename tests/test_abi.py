"""The C-ABI library loads (no GPU needed to load it) and exports every symbol
include/channel_cuda.h declares; the ctypes table covers the same set."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "channel_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ch_[a-z0-9_]+)\s*\(", text)) - {"ch_progress_fn"})


def test_header_symbols_exported():
    from channel_b200 import _lib
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) > 40
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from channel_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_api_version_and_bad_args():
    from channel_b200 import _lib
    lib = _lib.load()
    assert lib.ch_api_version() == 2
    # host-only validation paths: no device touched
    assert lib.ch_ctx_create(0, None) == _lib.CH_EINVAL
    assert b"NULL" in lib.ch_last_error()
    assert lib.ch_q4_tile_bytes(32, 128) == 2 * 2 * 576
    assert lib.ch_q8_tile_bytes(32, 64) == 2 * 2 * 576
    assert lib.ch_tensor_seed(3, 1, 4) == lib.ch_tensor_seed(3, 1, 4)


def test_tensor_seed_matches_oracle(oracle):
    from channel_b200 import _lib
    lib = _lib.load()
    for s, l, t in [(0, 0, 0), (3, 47, 6), (2**40 + 5, 3, 21)]:
        assert lib.ch_tensor_seed(s, l, t) == oracle.tensor_seed(s, l, t)
