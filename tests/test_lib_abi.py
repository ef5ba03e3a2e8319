"""The C-ABI library loads without a GPU and exports every declared symbol."""
import os
import re
import subprocess

import pytest

from heterocache_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "heterocache_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(hc_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def built():
    import __graft_entry__
    __graft_entry__.build()
    return _lib.library_path()


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ("hc_prefill_keep", "hc_prefill_select", "hc_pivot_init", "hc_decode_append", "hc_flash_decode",
              "hc_drift_check", "hc_retrieve", "hc_retrieve_delta"):
        assert n in names


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (hc_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_ctypes_signatures_cover_the_header(built):
    assert sorted(_lib.SIGNATURES) == declared_functions()
    lib = _lib.lib()
    assert lib.hc_abi_version() == 1
    assert lib.hc_status_string(3) == b"decode free list exhausted"


def test_argument_validation_needs_no_gpu(built):
    """Bad arguments are rejected on the host before any CUDA call."""
    lib = _lib.lib()
    # unsupported dtype / head_dim / window / kernel size
    assert lib.hc_flash_decode(9, 1, 8, 4, 128, None, 0, 0, None, None, 1, None, 1, None, 0.0, None, 0,
                               None, 0, None, None) == 2
    assert lib.hc_flash_decode(1, 1, 8, 4, 64, None, 0, 0, None, None, 1, None, 1, None, 0.0, None, 0,
                               None, 0, None, None) == 1
    assert lib.hc_prefill_select(1, 1, 8, 4, 100, 128, 5, 200, 0, 5, None, 0, 0, 0, None, None, 0, 0, 0, 0, 0, 0,
                                 None, 0, None, None, 1, None, 1, None, None, None, None, 0, None, None) == 1
    assert lib.hc_drift_check(1, 8, 4, 128, 9, 1000, 0, 5, 10, 0.5, None, 0, 0, None, 1, None, 4, 1, None,
                              None, None, 1, None, None, None, None, None, None, None, None, 0, None, None) == 8
    # the entry point without a workspace checks rows and groups first, with
    # the same codes as hc_flash_decode (8 = unsupported configuration)
    assert lib.hc_flash_decode_noalloc(1, 1000, 8, 4, 128, None, 0, 0, None, None, 1, None, 1, None, 0.0, None,
                                       None, None) == 8
    assert lib.hc_flash_decode_noalloc(1, 1, 8, 16, 128, None, 0, 0, None, None, 1, None, 1, None, 0.0, None,
                                       None, None) == 8
    # SnapKV: the window must leave positions to select from, and the
    # capacity must hold the window (the reference's topk would fail)
    snap = (None, 0, 0, 0, None, None, 0, 0, 0, 0, 0, 0, None, None, None, None, None, 0, None, None)
    assert lib.hc_snapkv_update_kv(1, 1, 4, 100, 128, 100, 0, 5, 100, *snap) == 1
    assert lib.hc_snapkv_update_kv(1, 1, 4, 100, 128, 8, 0, 5, 7, *snap) == 1
    assert lib.hc_snapkv_update_kv(1, 1, 4, 100, 128, 8, 0, 4, 50, *snap) == 1
    # nothing to do is not an error
    assert lib.hc_retrieve(1, 8, 128, 0, None, None, None, 0, None, None, 0, None, None, 0, 0, None, None, 1,
                           None, 1, None, None) == 0
    assert lib.hc_retrieve_delta(1, 8, 128, 0, None, None, None, None, None, 0, None, None, 0, None, 0, None, None,
                                 0, 0, None, None, 1, None, 1, None, None, None, 0, None, None) == 0
    # misaligned staging area
    assert lib.hc_retrieve_delta(1, 8, 128, 1, None, None, None, None, None, 1, None, None, 1, None, 1, None, None,
                                 0, 0, None, None, 1, None, 1, 8, None, None, 1, None, None) == 1
    # prefill attention: 16-bit only, head_dim 128, KV heads dividing the
    # query heads, aligned pointers; an empty prompt is not an error
    pa = (None, 8, 8, 8, None, 8, 8, 8, None, 8, 8, 8, 0.0, None, 8, 8, 8, None, None)
    assert lib.hc_prefill_attention(0, 1, 8, 8, 16, 128, *pa) == 8
    assert lib.hc_prefill_attention(1, 1, 8, 8, 16, 64, *pa) == 1
    assert lib.hc_prefill_attention(1, 1, 8, 3, 16, 128, *pa) == 1
    assert lib.hc_prefill_attention(1, 1, 8, 8, 0, 128, *pa) == 0
    assert lib.hc_prefill_attention(1, 1, 8, 8, 16, 128, 8, 8, 8, 8, *pa[4:]) == 1
    # workspace sizes are pure host arithmetic
    assert lib.hc_prefill_select_workspace_size(1, 1, 5, 32768, 4, 1) > 0
    assert lib.hc_flash_decode_workspace_size(1, 8, 4, 128) > 0


def declared_parameters():
    """Parameter types of every declared entry point, in order."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"^\s*(?:const\s+)?\w+\**\s+\**(hc_\w+)\s*\(([^)]*)\)\s*;", src, flags=re.M):
        params = [p.strip() for p in m.group(2).split(",") if p.strip()]
        out[m.group(1)] = [] if params == ["void"] else params
    return out


def _ctype_for(param: str):
    """The ctypes type a C parameter declaration maps to."""
    from ctypes import c_double, c_float, c_int, c_int64, c_size_t, c_ulonglong, c_void_p
    decl = param.rsplit(" ", 1)[0] if " " in param else param
    if "*" in param:
        return c_void_p
    return {"int": c_int, "int64_t": c_int64, "long long": c_int64, "size_t": c_size_t, "float": c_float,
            "double": c_double, "unsigned long long": c_ulonglong}[decl.strip()]


def test_ctypes_argument_lists_match_the_header_declarations():
    """Every entry point's ctypes argument list has the header's parameter
    count and types (a drift between the two would pass wrong arguments)."""
    from ctypes import c_int64, c_longlong
    params = declared_parameters()
    assert sorted(params) == declared_functions()
    for name, (_, argtypes) in _lib.SIGNATURES.items():
        want = [_ctype_for(p) for p in params[name]]
        assert len(argtypes) == len(want), (name, len(argtypes), len(want))
        for i, (got, exp) in enumerate(zip(argtypes, want)):
            same = got is exp or {got, exp} <= {c_int64, c_longlong}
            assert same, (name, i, params[name][i], got, exp)


def test_drift_job_struct_matches_the_header(tmp_path):
    """The ctypes mirror of hc_drift_job has the C struct's size and field
    offsets (gcc compiles the header and prints them)."""
    import ctypes
    fields = [f for f, _ in _lib.DriftJob._fields_]
    prog = tmp_path / "layout.c"
    prog.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"heterocache_b200.h\"\n"
                    "int main(void) {\n  printf(\"%zu\\n\", sizeof(hc_drift_job));\n"
                    + "".join(f"  printf(\"%zu\\n\", offsetof(hc_drift_job, {f}));\n" for f in fields)
                    + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got[0] == ctypes.sizeof(_lib.DriftJob)
    assert got[1:] == [getattr(_lib.DriftJob, f).offset for f in fields]


def test_drift_batch_validation_needs_no_gpu(built):
    """hc_drift_check_batch rejects bad sizes and descriptors on the host."""
    lib = _lib.lib()
    jobs = (_lib.DriftJob * 2)()
    args = (0, 5, 10, 0.5)
    # more than 7 steps: unsupported; no jobs: nothing to do
    assert lib.hc_drift_check_batch(1, 8, 4, 128, 9, 1000, *args, jobs, 2, 0, None, 0, None, None) == 8
    assert lib.hc_drift_check_batch(1, 8, 4, 128, 5, 1000, *args, jobs, 0, 0, None, 0, None, None) == 0
    # null descriptors (no pool, no page table) and a misaligned query buffer
    assert lib.hc_drift_check_batch(1, 8, 4, 128, 5, 1000, *args, jobs, 2, 0, None, 0, None, None) == 1
    for j in jobs:
        j.qbuf, j.k_pool, j.block_table, j.n_pool_blocks, j.max_blocks = 256, 512, 1024, 4, 4
        j.pivot_head, j.max_len, j.trigger, j.retrieve_positions, j.ref_positions = 7, 10, 64, 128, 192
    jobs[0].ref_bitmap, jobs[1].ref_bitmap = 4096, 8192
    jobs[1].qbuf = 264
    assert lib.hc_drift_check_batch(1, 8, 4, 128, 5, 1000, *args, jobs, 2, 0, None, 0, None, None) == 1
    jobs[1].qbuf = 256
    # a pivot head outside the layer, a retrieval longer than the context,
    # a page table too short for the context, a shared reference bitmap
    for field, bad in (("pivot_head", 8), ("max_len", 1001), ("max_blocks", 3), ("ref_bitmap", 4096)):
        good = getattr(jobs[1], field)
        setattr(jobs[1], field, bad)
        assert lib.hc_drift_check_batch(1, 8, 4, 128, 5, 1000, *args, jobs, 2, 0, None, 0, None, None) == 1, field
        setattr(jobs[1], field, good)
    # jobs per launch: capped where a launch's shared memory runs out
    assert lib.hc_drift_check_batch_per_launch(1, 32, 5, 131072, 4, 0) == 8
    assert 1 < lib.hc_drift_check_batch_per_launch(1, 32, 5, 131072, 4, 16) < 16
    assert lib.hc_drift_check_batch_per_launch(1, 3, 5, 4096, 4, 0) == 3
    assert lib.hc_drift_check_batch_workspace_size(1, 32, 5, 131072, 4, 0) > 0
