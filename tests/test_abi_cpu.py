"""The C ABI without a GPU: the shared library loads, exports every entry
point declared in include/*.h, the ctypes table binds exactly those, and the
host-side parts (scratch sizing, argument validation, error messages) behave
as documented.  No call here reaches a kernel launch."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tinybatch_b200 import _native as N

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    if not N.lib_path().exists():
        from tinybatch_b200 import build
        build.build()
    return N.load()


def _declared() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^(?:int|size_t|const char\*)\s+(tb_[a-z0-9_]+)\(", text, re.M))
    return names


def test_every_declared_symbol_is_exported(lib):
    declared = _declared()
    assert len(declared) >= 20
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    assert set(N.exported_symbols()) == _declared()


def test_host_only_entry_points(lib):
    assert lib.tb_version() == 1
    # split-K scratch: 64 KiB of counters + fp32 partial tiles
    assert lib.tb_gemm_scratch_bytes(128, 5120, 256, 6) == (64 << 10) + 20 * 6 * 256 * 128 * 4
    assert lib.tb_gemm_scratch_bytes(128, 5120, 256, 1) == 0
    # split-KV scratch: 64 KiB of counters + partial outputs + log-sum-exps
    assert lib.tb_attention_scratch_bytes(4, 8, 128, 4096, 4096) == 0
    b = lib.tb_attention_scratch_bytes(4, 8, 128, 4096, 512)
    rows = 4 * 8 * 8 * 16
    assert b == (64 << 10) + -(-rows * 128 * 4 // 256) * 256 + -(-rows * 4 // 256) * 256


@pytest.mark.parametrize("call,needle", [
    (lambda lib: lib.tb_linear(None, 0, None, 0, 128, 512, 512, None, 0, 0, 0.0, 0.0, None, 512,
                               1, 100, 1, None, 0, None), "bn must be"),
    (lambda lib: lib.tb_qkv_rope_kv(None, 0, None, 0, None, 8, 256, 4, 2, 48, None, 0, 0, 0.0,
                                    0.0, None, None, 16, None, None, None, 0, None, 16, 128, 1,
                                    None, 0, None), "multiple of head_dim"),
    (lambda lib: lib.tb_gate_up_swiglu(None, 0, None, 0, 8, 256, 100, None, 0, 0, 0.0, 0.0,
                                       None, 128, 128, 1, None, 0, None), "n_feat"),
    (lambda lib: lib.tb_paged_attention_decode(None, 0, None, 0, None, 1, 8, 2, 64, 16, None, 1,
                                               None, None, None, None, 1, 100, 500, None, 0,
                                               None), "split_tokens"),
    (lambda lib: lib.tb_argmax_vocab_parallel(None, None, 512, 8, 256, 0, None, 3, None),
     "communicator"),
    (lambda lib: lib.tb_row_linear_allreduce_residual(
        None, 0, None, 0, 8, 512, 512, None, 0, None, None, 0, None, 0, None, None, None, 0,
        None, 0, 0, None, 128, 1, None), "communicator"),
    (lambda lib: lib.tb_linear_static_scratch(None, 0, None, 0, 128, 512, 512, None, 0, 0, 0.0,
                                              0.0, None, 512, 1, 100, 1, None), "bn must be"),
])
def test_argument_errors_are_reported(lib, call, needle):
    rc = call(lib)
    assert rc in (1, 4)          # TB_ERR_ARG / TB_ERR_STATE
    msg = lib.tb_last_error().decode()
    assert needle in msg, msg
