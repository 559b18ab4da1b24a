"""The C-ABI library loads without a GPU and exports every entry point include/specdec_b200.h declares; the
Python binding declares exactly those."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER_FUNCTIONS = sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(specdec_\w+)\s*\(",
                                         "\n".join(p.read_text() for p in (ROOT / "include").glob("*.h")),
                                         flags=re.M)))


def test_header_declares_entry_points():
    assert "specdec_accept" in HEADER_FUNCTIONS and "specdec_last_error" in HEADER_FUNCTIONS


@pytest.fixture(scope="module")
def lib():
    from nanovllm_b200 import _lib
    return _lib.load()


@pytest.mark.parametrize("name", HEADER_FUNCTIONS)
def test_library_exports_declared_symbol(lib, name):
    assert hasattr(lib, name)


def test_binding_matches_header():
    from nanovllm_b200 import _lib
    assert sorted(_lib.SIGNATURES) == HEADER_FUNCTIONS


def test_host_queries_run_without_a_gpu(lib):
    assert lib.specdec_version() >= 1
    assert lib.specdec_sampler_workspace_bytes(512) > 0
    assert lib.specdec_last_error() is not None
