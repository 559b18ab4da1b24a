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


def test_accept_workspace_adds_the_noise_codes(lib):
    """The accept's workspace with room for the tail race's noise codes: the sampler workspace plus 2 bytes per
    element of the [B, V] noise, rounded to 256 bytes; 0 for sizes that are not positive."""
    for T, B, V in [(512, 64, 151936), (1, 1, 7), (16384, 1024, 1000)]:
        codes = (B * V * 2 + 255) // 256 * 256
        assert lib.specdec_accept_workspace_bytes(T, B, V) == lib.specdec_sampler_workspace_bytes(T) + codes
    assert lib.specdec_accept_workspace_bytes(0, 64, 151936) == 0
    assert lib.specdec_accept_workspace_bytes(512, 0, 151936) == 0
    assert lib.specdec_accept_workspace_bytes(512, 64, -1) == 0


def _attention_multi(lib, outs, num_outs):
    """specdec_paged_attention_multi with plausible (never dereferenced) addresses: only the host validation
    runs, so a call must be rejected before any CUDA call."""
    import ctypes
    fake = 1 << 20
    arr = (ctypes.c_void_p * max(len(outs), 1))(*(outs or [0]))
    return lib.specdec_paged_attention_multi(fake, 8, 4096, 32, 8, 128, fake, fake, 256, 256, fake, fake, None, 0,
                                             1, fake, 1, 8, 0.088, 1, arr, num_outs, 4096, fake, 1 << 24, fake, 0,
                                             None)


@pytest.mark.parametrize("outs,num_outs", [([1 << 20], 0), ([1 << 20] * 9, 9), ([(1 << 20) + 1], 1),
                                           ([1 << 20, 0], 2)])
def test_multi_destination_attention_rejects_bad_destinations_on_the_host(lib, outs, num_outs):
    assert _attention_multi(lib, outs, num_outs) == 1            # kInvalidArgument, nothing launched
    assert b"destination" in lib.specdec_last_error()


@pytest.mark.parametrize("world,rank,timeout_ns,flag_off,epoch_off", [
    (9, 0, 10**9, 0, 0), (2, 2, 10**9, 0, 0), (2, 0, 0, 0, 0), (2, 0, 10**9, 2, 0), (2, 0, 10**9, 0, 2)])
def test_peer_barrier_rejects_bad_arguments_on_the_host(lib, world, rank, timeout_ns, flag_off, epoch_off):
    import ctypes
    fake = 1 << 20
    flags = (ctypes.c_void_p * 8)(*[fake + flag_off] * 8)
    assert lib.specdec_peer_barrier(flags, world, rank, fake + epoch_off, timeout_ns, fake, None) == 1
