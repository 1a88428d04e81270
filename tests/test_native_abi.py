"""The C-ABI library loads (no GPU needed) and exports every entry point that
include/tiny_infra_b200.h declares; the ctypes binding covers each of them."""
import os
import re
import subprocess

import pytest

from tests.conftest import REPO

HEADER = os.path.join(REPO, "include", "tiny_infra_b200.h")


def declared_symbols() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(ti_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def native():
    from tiny_infra_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        from tiny_infra_b200 import build
        build.build()
    return _native


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {"ti_paged_attention_decode", "ti_rope_inplace", "ti_swiglu", "ti_rmsnorm",
            "ti_last_error"} <= syms


def test_library_exports_every_declared_symbol(native):
    lib = native.lib()
    for name in sorted(declared_symbols()):
        assert hasattr(lib, name), name
        assert name in native.SIGNATURES, f"ctypes binding misses {name}"
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (ti_[a-z0-9_]+)\b", out))
    assert declared_symbols() <= exported


def test_library_calls_without_gpu(native):
    """Host-only entry points answer without touching a device."""
    lib = native.lib()
    assert lib.ti_version() >= 1
    assert lib.ti_launch_count() >= 0
    assert lib.ti_paged_attention_workspace_bytes(256, 14, 2, 64, 128, 16) > 0
    # argument validation happens before any CUDA call
    rc = lib.ti_swiglu(None, None, 4, 12, 0, None)
    assert rc != 0 and lib.ti_last_error()
    rc = lib.ti_paged_attention_decode(None, 0, None, 0, None, None, 1, None, 0, None, None, 1,
                                       14, 2, 64, 16, 4, 0, 0, None, 0, None)
    assert rc == 1 and b"null" in lib.ti_last_error()
    # attention plan: size query and argument checks
    assert lib.ti_paged_attention_plan_bytes(256) > lib.ti_paged_attention_plan_bytes(8) > 0
    rc = lib.ti_paged_attention_plan(None, 0, None, None, 4, 14, 2, 64, 8, 100, None, 0, None)
    assert rc == 1 and b"null" in lib.ti_last_error()
    rc = lib.ti_paged_attention_decode_planned(None, 0, None, 0, None, None, 1, None, 0, None,
                                               None, 1, 14, 2, 64, 16, 4, 0, None, 0, None, None)
    assert rc == 1 and b"null" in lib.ti_last_error()
    # SwiGLU16 gate/up GEMM: N must be a multiple of 16 (checked before any CUDA call; the
    # operand addresses are never dereferenced)
    fake = 1 << 20
    rc = lib.ti_gemm(native.TI_EPI_SWIGLU16, fake, 896, fake, 896, 256, 9720, 896, fake,
                     4864, None, None, None, native.TI_DTYPE_BF16, 0, 1, None)
    assert rc != 0 and b"N % 16" in lib.ti_last_error()


def test_attention_workspace_follows_kernel_choice(native):
    """The size query mirrors the kernel choice: sequences of at most 32 blocks whose units (a
    sequence's pair of kv heads) fit one wave of CTAs run one CTA per unit and need no split-K
    slots, so the size does not grow with the table width; one block more per sequence, or one
    unit more than the 148 SMs, and the split-K slots appear."""
    lib = native.lib()

    def ws(batch, max_blocks):
        return lib.ti_paged_attention_workspace_bytes(batch, 14, 2, 64, max_blocks, 0)

    assert ws(8, 16) == ws(8, 32)
    assert ws(8, 33) > 4 * ws(8, 32)
    assert ws(149, 32) > 4 * ws(148, 32)
