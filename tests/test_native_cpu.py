"""CPU checks of the native boundary: the C-ABI library loads and exports
every symbol include/gdsq.h declares, the binding exports every op name of
the reference module, and argument validation fails cleanly without
touching a GPU."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

import gdsllm_b200
from gdsllm_b200._native import GdsqError, check, lib

ROOT = Path(__file__).resolve().parents[1]

# Every name the reference binding registers (gdsllm/runtime/gds_bindings.cpp:516-615).
REFERENCE_OPS = ["init", "shutdown", "is_driver_open", "GdsBufferHandle", "load_file",
                 "load_file_region", "load_expert", "view_tensor", "load_tensor", "dequant_gguf",
                 "fused_dequant_gemv", "dequant_affine_q4", "fused_affine_q4_gemv"]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"GDSQ_API\s+[\w\s\*]+?\b(gdsq_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 11
    l = lib()
    for s in syms:
        assert hasattr(l, s), f"{s} declared in include/ but not exported"


def test_exported_symbols_are_exactly_the_declared_ones():
    import subprocess
    from gdsllm_b200.build import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if l.split()[-1].startswith("gdsq_"))
    assert exported == declared_symbols()


def test_binding_has_the_reference_op_names():
    m = gdsllm_b200.ext()
    for name in REFERENCE_OPS:
        assert hasattr(m, name), name
    assert m.backend == "gdsq-sm100a"


def test_install_as_reference_module():
    import sys
    mod = gdsllm_b200.install_as_reference_module("gdsq_test_alias.gds_io_ext")
    assert sys.modules["gdsq_test_alias.gds_io_ext"] is mod
    del sys.modules["gdsq_test_alias.gds_io_ext"]


def test_status_strings():
    l = lib()
    assert l.gdsq_status_string(0) == b"ok"
    assert l.gdsq_status_string(2) == b"misaligned pointer"
    assert l.gdsq_version() >= 100


# Validation happens before any CUDA call, so these run without a GPU.
FAKE = 0x10000  # never dereferenced


@pytest.mark.parametrize("call,fragment", [
    (lambda l: l.gdsq_fused_q4_0_gemv(FAKE, FAKE, FAKE, 8, 48, 1, None), b"multiple of 32"),
    (lambda l: l.gdsq_fused_q8_0_gemv(FAKE, FAKE, FAKE, 8, 64, 0, None), b"batch 0"),
    (lambda l: l.gdsq_fused_q8_0_gemv(FAKE, FAKE, FAKE, 8, 64, 17, None), b"batch 17"),
    (lambda l: l.gdsq_fused_q4_0_gemv(FAKE, FAKE, FAKE, -1, 64, 1, None), b"negative"),
    (lambda l: l.gdsq_fused_affine_q4_gemv(FAKE, FAKE, FAKE, FAKE, FAKE, 8, 100, 12, 1, None), b"multiple of 8"),
    (lambda l: l.gdsq_fused_affine_q4_gemv(FAKE, FAKE, FAKE, FAKE, FAKE, 8, 96, 64, 1, None), b"not a multiple"),
    (lambda l: l.gdsq_fused_q4_0_gemv(None, FAKE, FAKE, 8, 64, 1, None), b"null"),
    (lambda l: l.gdsq_dequant_affine_q4(FAKE, FAKE, FAKE, FAKE, 100, 64, 32, None), b"whole number of rows"),
])
def test_invalid_arguments_are_rejected(call, fragment):
    l = lib()
    st = call(l)
    assert st == 1, st
    assert fragment in l.gdsq_last_error()
    with pytest.raises(GdsqError):
        check(st)


@pytest.mark.parametrize("call", [
    lambda l: l.gdsq_fused_q4_0_gemv(FAKE + 1, FAKE, FAKE, 8, 64, 1, None),
    lambda l: l.gdsq_fused_q4_0_gemv(FAKE, FAKE, FAKE + 1, 8, 64, 1, None),
    lambda l: l.gdsq_fused_affine_q4_gemv(FAKE + 2, FAKE, FAKE, FAKE, FAKE, 8, 128, 128, 1, None),
    lambda l: l.gdsq_dequant_q4_0(FAKE + 1, FAKE, 4, None),
    lambda l: l.gdsq_dequant_affine_q4(FAKE + 2, FAKE, FAKE, FAKE, 128, 128, 128, None),
])
def test_misaligned_pointers_are_rejected(call):
    assert call(lib()) == 2


def _arr(ctype, vals):
    import ctypes
    return (ctype * len(vals))(*vals)


def _moe_gate_up(l, top_k=4, group=128, first=0, count=8, total=8, shared=None):
    sh = shared if shared is not None else [None] * 6
    return l.gdsq_moe_affine_q4_gate_up(*([FAKE] * 6), *sh, FAKE, FAKE, FAKE, 1, top_k, 512, 1024, group, first, count,
                                        total, None)


@pytest.mark.parametrize("call,fragment", [
    (lambda l: l.gdsq_fused_gemv_group(7, 2, _arr(ctypes_vp(), [FAKE, FAKE]), _arr(ctypes_int(), [8, 8]),
                                       _arr(ctypes_vp(), [FAKE, FAKE]), FAKE, 256, 1, None), b"gguf_type"),
    (lambda l: l.gdsq_fused_gemv_group(0, 5, _arr(ctypes_vp(), [FAKE] * 5), _arr(ctypes_int(), [8] * 5),
                                       _arr(ctypes_vp(), [FAKE] * 5), FAKE, 256, 1, None), b"count 5"),
    (lambda l: _moe_gate_up(l, top_k=65), b"top_k"),
    (lambda l: _moe_gate_up(l, group=12), b"group_size"),
    (lambda l: _moe_gate_up(l, first=4, count=8, total=8), b"resident experts"),
    (lambda l: _moe_gate_up(l, shared=[FAKE, None, None, None, None, None]), b"all given or all null"),
    (lambda l: l.gdsq_moe_affine_q4_down(*([FAKE] * 3), None, None, None, FAKE, FAKE, FAKE, None, FAKE, 1, 4, 1024,
                                         512, 128, 0, 8, 8, 8, None), b"unknown flags"),
    (lambda l: l.gdsq_moe_route(FAKE, 1, 8, 9, None, None, 0, FAKE, FAKE, None, None), b"top_k"),
    (lambda l: l.gdsq_moe_route(FAKE, 1, 5000, 10, None, None, 0, FAKE, FAKE, None, None), b"experts"),
    (lambda l: l.gdsq_allreduce_sum_f16(FAKE, FAKE, 8192, _arr(ctypes_vp(), [FAKE] * 9),
                                        _arr(ctypes_vp(), [FAKE] * 9), 8192, 0, 9, None), b"world 9"),
    (lambda l: l.gdsq_allreduce_sum_f16(FAKE, FAKE, 12, _arr(ctypes_vp(), [FAKE, FAKE]),
                                        _arr(ctypes_vp(), [FAKE, FAKE]), 8192, 0, 2, None), b"multiple of 8"),
    (lambda l: l.gdsq_allreduce_sum_f16(FAKE, FAKE, 16384, _arr(ctypes_vp(), [FAKE, FAKE]),
                                        _arr(ctypes_vp(), [FAKE, FAKE]), 8192, 1, 2, None), b"capacity"),
    (lambda l: l.gdsq_allreduce_sum_words(5, FAKE, FAKE, 64, _arr(ctypes_vp(), [FAKE, FAKE]), FAKE, 64, 0, 2,
                                          None), b"elem_type"),
    (lambda l: l.gdsq_allreduce_sum_words(1, FAKE, FAKE, 64, _arr(ctypes_vp(), [FAKE] * 9), FAKE, 64, 0, 9,
                                          None), b"world 9"),
    (lambda l: l.gdsq_allreduce_sum_words(1, FAKE, FAKE, 65, _arr(ctypes_vp(), [FAKE, FAKE]), FAKE, 64, 0, 2,
                                          None), b"capacity"),
    (lambda l: l.gdsq_allreduce_sum_words(1, FAKE, FAKE, 40000, _arr(ctypes_vp(), [FAKE, FAKE]), FAKE, 40000, 0,
                                          2, None), b"32768"),
    (lambda l: l.gdsq_fused_gemv_allreduce(2, FAKE, FAKE, FAKE, 4096, 4096, _arr(ctypes_vp(), [FAKE, FAKE]),
                                           _arr(ctypes_vp(), [FAKE, FAKE]), 4096, 0, 2, None), b"gguf_type"),
    (lambda l: l.gdsq_fused_gemv_allreduce(0, FAKE, FAKE, FAKE, 4096, 4096, _arr(ctypes_vp(), [FAKE] * 9),
                                           _arr(ctypes_vp(), [FAKE] * 9), 4096, 0, 9, None), b"world 9"),
    (lambda l: l.gdsq_fused_gemv_allreduce(0, FAKE, FAKE, FAKE, 4100, 4096, _arr(ctypes_vp(), [FAKE, FAKE]),
                                           _arr(ctypes_vp(), [FAKE, FAKE]), 4096, 1, 2, None), b"exchange buffer"),
])
def test_invalid_arguments_of_the_additive_entry_points(call, fragment):
    """The grouped GEMV, MoE and all-reduce entry points reject bad arguments
    before any CUDA call."""
    l = lib()
    st = call(l)
    assert st == 1, (st, l.gdsq_last_error())
    assert fragment in l.gdsq_last_error(), l.gdsq_last_error()


def ctypes_vp():
    import ctypes
    return ctypes.c_void_p


def ctypes_int():
    import ctypes
    return ctypes.c_int


def test_empty_work_is_a_no_op():
    l = lib()
    assert l.gdsq_dequant_q4_0(None, None, 0, None) == 0
    assert l.gdsq_fused_q4_0_gemv(None, None, None, 0, 64, 1, None) == 0


# Mangled names of the reference's launchers, as g++ produces them from
# gdsllm/runtime/fused_gemv.h, gguf_dequant.h and affine_q4_dequant.h.
REFERENCE_LAUNCHERS = [
    "_Z19launch_dequant_q4_0PKvP6__halfmP11CUstream_st",
    "_Z19launch_dequant_q8_0PKvP6__halfmP11CUstream_st",
    "_Z22launch_fused_q4_0_gemvPKvPK6__halfPS1_iiP11CUstream_st",
    "_Z22launch_fused_q8_0_gemvPKvPK6__halfPS1_iiP11CUstream_st",
    "_Z24launch_dequant_affine_q4PKjPK6__halfS3_PS1_miiP11CUstream_st",
    "_Z27launch_fused_affine_q4_gemvPKjPK6__halfS3_S3_PS1_iiiP11CUstream_st",
]


def test_reference_launcher_abi_is_exported():
    import subprocess
    from gdsllm_b200.build import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines()}
    for name in REFERENCE_LAUNCHERS:
        assert name in exported, name


def test_cpp_caller_links_against_reference_abi(tmp_path):
    """A C++ translation unit written against include/gdsq_reference_abi.h
    (the reference's launcher declarations) links with libgdsq.so."""
    import subprocess
    from gdsllm_b200.build import BUILD
    src = tmp_path / "caller.cpp"
    src.write_text(
        '#include "gdsq_reference_abi.h"\n'
        "int main() {\n"
        "  void* f[] = {(void*)&launch_fused_q4_0_gemv, (void*)&launch_fused_q8_0_gemv,\n"
        "               (void*)&launch_dequant_q4_0, (void*)&launch_dequant_q8_0,\n"
        "               (void*)&launch_dequant_affine_q4, (void*)&launch_fused_affine_q4_gemv};\n"
        "  return f[0] == nullptr;\n"
        "}\n")
    exe = tmp_path / "caller"
    subprocess.run(["g++", str(src), "-o", str(exe), f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
                    f"-L{BUILD}", "-lgdsq", f"-Wl,-rpath,{BUILD}", "-Wl,--unresolved-symbols=ignore-in-shared-libs"],
                   check=True, capture_output=True)
    assert exe.exists()
