"""The C-ABI library loads on a host without a GPU, exports every entry point
declared in include/prismkv_b200.h, and rejects bad arguments on the host
(negative return codes, as the reference's native launchers do,
kernels/ppu_8b/av_tuned.cu:63)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "prismkv_b200.h"


@pytest.fixture(scope="module")
def lib():
    from prismkv_b200 import build as b
    b.build()
    from prismkv_b200 import native
    return native


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|size_t)\s+(pk_\w+)\s*\(", text, re.M)))


def test_header_declares_the_path(lib):
    names = declared_symbols()
    for required in ["pk_route_qact", "pk_route_moments", "pk_union", "pk_sparse_av", "pk_lse_merge",
                     "pk_build_index", "pk_append_index", "pk_summarize", "pk_key_center"]:
        assert required in names


def test_every_declared_symbol_is_exported_and_bound(lib):
    L = ctypes.CDLL(str(lib.LIB_PATH))
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert name in lib.SIGNATURES, f"{name} has no binding signature"


def test_facts(lib):
    assert lib.query("pk_version") // 100 == 100
    assert lib.query("pk_supported_head_dim", 128) == 1
    assert lib.query("pk_supported_head_dim", 96) == 0


def test_workspace_sizes(lib):
    a = lib.query("pk_route_qact_workspace_bytes", 32, 4, 16384, 32)
    assert a >= 32 * 4 * 16384 * 4
    assert lib.query("pk_sparse_av_workspace_bytes", 32, 4, 128, 16) >= 32 * 4 * 16 * 130 * 4
    assert lib.query("pk_build_ids_capacity", 8192, 2048, 8, 0.0, 0) >= 8192 * 8
    assert lib.query("pk_build_workspace_bytes", 8, 8192, 2048, 8, 1 << 20) > 8 * 8192 * 8 * 8


def raw(lib, name, *args):
    fn = getattr(lib.lib(), name)
    return fn(*args)


def test_argument_errors_are_negative(lib):
    # U = 0, head dim 64, zero scale: rejected before any launch.
    qa = "pk_route_qact"
    assert raw(lib, qa, 1, 1, 0, 0, 1, 1, 0, 0, 1.0, 1, 0, 4, 128, 64, 8, 1, 1 << 20, 1, 1, 32, 0, 0, 0) < 0
    assert raw(lib, qa, 1, 1, 0, 1, 1, 1, 0, 0, 1.0, 1, 1, 4, 64, 64, 8, 1, 1 << 20, 1, 1, 32, 0, 0, 0) == -2
    assert raw(lib, qa, 1, 1, 0, 1, 1, 1, 0, 0, 0.0, 1, 1, 4, 128, 64, 8, 1, 1 << 20, 1, 1, 32, 0, 0, 0) < 0
    assert raw(lib, qa, 1, 1, 0, 1, 1, 1, 0, 0, 1.0, 1, 1, 4, 128, 64, 8, 1, 16, 1, 1, 32, 0, 0, 0) == -3
    assert raw(lib, "pk_sae_prepare", 1, 64, 64, 1, 1, 0) == -2
    assert raw(lib, "pk_sparse_av", 1, 1, 1, 1, 1, 0, 0, 64, 1, 1, 1, 1, 1, 1, 4, 64, 1, 0, 0, 1, 0, 0) == -2
    assert raw(lib, "pk_sparse_av", 1, 1, 1, 1, 1, 0, 0, 128, 1, 1, 1, 1, 1, 1, 17, 128, 1, 0, 0, 1, 0, 0) == -1
    assert raw(lib, "pk_union", 0, 0, 0, 0, 0, 0, 1, 0, 0, 1, 8, 64, 0, 0, 0, 0, 0, 0, 0, 0) == -1
    assert raw(lib, "pk_lse_merge", 1, 0, 4, 128, 1, 1, 0) == -1
    assert raw(lib, "pk_build_index", 1, 1, 0, 128, 1, 1.0, 1, 1, 0, 0, 1, 100, 128, 64, 8, 0, 0.0, 0, 1, 1, 1, 10,
               1, 1, 1 << 30, 1, 0) == -1  # ids_stride below capacity


def test_missing_library_fails_loudly(lib, monkeypatch, tmp_path):
    monkeypatch.setattr(lib, "LIB_PATH", tmp_path / "absent.so")
    monkeypatch.setattr(lib, "_lib", None)
    with pytest.raises(lib.NativeError):
        lib.lib()


def test_other_head_dims_refused_before_any_launch():
    """Every kernel is built for head_dim 128; the Python layer refuses any
    other head dimension with a clear error before reaching the library."""
    import torch
    import prismkv_b200 as pk
    keys = torch.zeros(8, 256)
    sae = pk.SAEParams(torch.zeros(16, 256), torch.zeros(16), key_mean=2, query_topk=2)
    with pytest.raises(ValueError, match="head_dim 256"):
        pk.build_index(keys, sae, 1.0)
    with pytest.raises(ValueError, match="head_dim 256"):
        pk.attend(torch.zeros(4, 256), torch.zeros(8, 256), torch.zeros(8, 256), torch.zeros(0, dtype=torch.long), 8)
