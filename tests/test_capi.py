"""The C ABI without a GPU: libbasal200.so loads, exports every entry point include/basal200.h declares, and the
ctypes binding declares exactly those; status strings and argument checks that return before any device work."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "basal200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(basal200_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from basal_b200 import _lib
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 17
    for n in names:
        assert hasattr(lib, n), n


def test_binding_covers_the_header():
    from basal_b200 import _lib
    bound = set(_lib.SIGNATURES) | {"basal200_status_string", "basal200_version", "basal200_device_faults",
                                    "basal200_block_gemm_workspace_bytes", "basal200_block_linear_glu_workspace_bytes",
                                    "basal200_block_linear_residual_workspace_bytes"}
    assert bound == set(declared())


def test_status_strings_and_version(lib):
    assert lib.basal200_version() >= 1
    assert lib.basal200_status_string(0) == b"ok"
    assert b"shape" in lib.basal200_status_string(2)
    assert lib.basal200_status_string(99) == b"unknown status"


def test_argument_checks_before_device_work(lib):
    """Sizes the format cannot take are refused before the library touches a device (status codes, no exit)."""
    null = ctypes.c_void_p(0)
    # K not a multiple of 128
    assert lib.basal200_fp8_act_quant(null, 0, 4, 100, null, null, null) == 2
    # negative M
    assert lib.basal200_int8_act_quant(null, 0, -1, 128, null, null, null) == 1
    # M = 0 is an empty success
    assert lib.basal200_fp8_act_quant(null, 0, 0, 256, null, null, null) == 0
    assert lib.basal200_fp8_block_gemm(null, null, null, null, null, null, 0, 0, 256, 256, null, 0, null) == 0
    # N not a multiple of 128
    assert lib.basal200_fp8_block_gemm(null, null, null, null, null, null, 0, 4, 200, 256, null, 0, null) == 2
    # NVFP4: K % 64
    assert lib.basal200_nvfp4_act_quant(null, 0, null, 4, 96, null, null, null) == 2
    # column-parallel GEMM with gathered outputs: no output buffer; a shard past the full width; fp32 output
    outs = (ctypes.c_void_p * 2)(None, None)
    gather = lib.basal200_fp8_block_gemm_gather
    assert gather(null, null, null, null, outs, 0, 0, 256, 0, 4, 128, 256, null, null) == 1
    assert gather(null, null, null, null, outs, 2, 256, 256, 0, 4, 128, 256, null, null) == 2
    assert gather(null, null, null, null, outs, 2, 0, 256, 2, 4, 128, 256, null, null) == 4
    assert gather(null, null, null, null, outs, 2, 0, 256, 0, 0, 128, 256, null, null) == 0
    # gated linear: an unknown activation; I not a multiple of 128; fp32 activations; M = 0 is an empty success
    glu = lib.basal200_fp8_block_linear_glu
    assert glu(null, 0, null, null, null, 4, 256, 256, 3, null, null, null, 0, null) == 1
    assert glu(null, 0, null, null, null, 4, 200, 256, 1, null, null, null, 0, null) == 2
    assert lib.basal200_int8_block_linear_glu(null, 2, null, null, null, 4, 256, 256, 2, null, null, null, 0, null) == 4
    assert glu(null, 0, null, null, null, 0, 256, 256, 1, null, null, null, 0, null) == 0
    gws = lib.basal200_block_linear_glu_workspace_bytes
    assert gws(16, 6144, 2048) == 16 * 12288 * 2 and gws(65, 6144, 2048) == 0
    assert gws(16, 1024, 2048) == 16 * 2048 * 2 + 16 * 2048 * 16 * 4  # plus the split products
    # residual linear: N not a multiple of 128; fp32 activations; M = 0 is an empty success
    rl = lib.basal200_fp8_block_linear_residual
    assert rl(null, 0, null, null, null, null, null, 4, 200, 256, null, null, null, 0, null) == 2
    assert rl(null, 2, null, null, null, null, null, 4, 256, 256, null, null, null, 0, null) == 4
    assert rl(null, 0, null, null, null, null, null, 0, 256, 256, null, null, null, 0, null) == 0
    assert lib.basal200_block_linear_residual_workspace_bytes(16, 2048, 2048) == 16 * 2048 * 2 + 16 * 2048 * 16 * 4
    # readout: Kmax beyond 1024
    assert lib.basal200_code_probs(null, 1, 1, null, null, 2000, null, null) == 8
    # the allocation-free linear: one row past its array's limit is refused before any pointer is looked at or any
    # device call is made (null pointers here); M = 0 is an empty success
    noalloc = lib.basal200_fp8_block_linear_noalloc
    limit = 1 << 24  # BASAL200_NOALLOC_MAX_ELEMS
    assert noalloc(null, 0, null, null, null, null, limit // 2048 + 1, 256, 2048, null) == 8
    assert noalloc(null, 0, null, null, null, null, 1, 256, limit + 128, null) == 8
    assert noalloc(null, 0, null, null, null, null, 0, 256, 2048, null) == 0
    assert b"limit" in lib.basal200_status_string(8)


def test_split_workspace_sizes(lib):
    """The few-rows GEMM asks for a workspace only where spreading its slices over the SMs pays: M <= 64, weights of
    at most 64 tiles of 128 rows, at least 2 slices, products of at most 32 MiB (4 bytes per token, output, slice)."""
    ws = lib.basal200_block_gemm_workspace_bytes
    assert ws(16, 2048, 2048) == 16 * 2048 * 16 * 4
    assert ws(64, 2048, 6144) == 64 * 2048 * 48 * 4
    assert ws(1, 8192, 2048) == 8192 * 16 * 4
    assert ws(1, 12288, 2048) == 0          # 96 tiles
    assert ws(65, 2048, 2048) == 0          # the large-M kernel
    assert ws(16, 8320, 2048) == 0          # 65 tiles
    assert ws(16, 2048, 128) == 0           # one slice: nothing to spread
    assert ws(64, 8192, 6144) == 0          # 96 MiB of products
    assert ws(16, 200, 2048) == 0 and ws(0, 2048, 2048) == 0 and ws(16, 2048, 8320) == 0


def test_header_is_plain_c():
    """The header compiles as C (no torch or C++ types in the signatures)."""
    import shutil
    import subprocess
    import tempfile
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no gcc")
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.c")
        with open(src, "w") as f:
            f.write("#include \"basal200.h\"\nint (*probe)(void) = basal200_version;\n")
        subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), "-c", src, "-o",
                        os.path.join(d, "t.o")], check=True)
