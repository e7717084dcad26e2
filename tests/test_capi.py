"""The C-ABI library loads, exports every symbol include/asterq.h declares, and
rejects bad arguments with a status (host-side validation, no GPU needed)."""
from __future__ import annotations

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from asterq import _lib

REPO = Path(__file__).resolve().parent.parent


def declared_functions() -> set[str]:
    text = (REPO / "include" / "asterq.h").read_text()
    return set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(asterq_\w+)\s*\(", text, flags=re.M))


def test_header_matches_binding():
    assert declared_functions() == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.lib_path())], capture_output=True, text=True)
    if out.returncode == 0:
        for name in declared_functions():
            assert re.search(rf"\bT {name}\b", out.stdout), name


def test_version_and_error_string():
    lib = _lib.load()
    assert lib.asterq_version() == 1
    assert isinstance(lib.asterq_last_error(), bytes)


def test_struct_layout_matches_header():
    # sizes of the C struct: 6 int32 + 2 float + 3 int64 + 4 int32 + 14 pointers + int64 + 2 pointers + 2 int32
    # + the workers pointer + 2 int32 + the unit_jobs pointer + the int64 wait limit + the plan_counts pointer
    # + the RoPE scheme int32 (+ padding) and the cold_rope_scales pointer
    size = 6 * 4 + 2 * 4 + 3 * 8 + 4 * 4 + 14 * 8 + 8 + 8 + 8 + 2 * 4 + 8 + 2 * 4 + 8 + 8 + 8 + 8 + 8
    assert ctypes.sizeof(_lib.DecodeParams) == size
    assert _lib.DecodeParams.workers.offset == size - 56
    assert _lib.DecodeParams.wait_limit_cycles.offset == size - 32
    assert _lib.DecodeParams.plan_counts.offset == size - 24
    assert _lib.DecodeParams.rope_scheme.offset == size - 16
    assert _lib.DecodeParams.cold_rope_scales.offset == size - 8
    # asterq_batch_desc: 6 int32 + 7 pointers + the cold tile int32 (+ padding); asterq_plan_buffers:
    # 3 int32 (+ padding) + 8 pointers
    assert ctypes.sizeof(_lib.BatchDesc) == 6 * 4 + 7 * 8 + 8
    assert ctypes.sizeof(_lib.PlanBuffers) == 16 + 8 * 8 and _lib.PlanBuffers.tiles.offset == 16


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_ctypes_mirrors_match_the_c_compiler(tmp_path):
    """Every field offset and struct size of the ctypes mirrors equals what a C compiler lays out
    from include/asterq.h."""
    structs = {"asterq_decode_params": _lib.DecodeParams, "asterq_batch_desc": _lib.BatchDesc,
               "asterq_plan_buffers": _lib.PlanBuffers}
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "asterq.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    include = Path(__file__).resolve().parent.parent / "include"
    subprocess.run(["gcc", "-std=c11", "-I", str(include), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, fname, value = line.split()
        got[(cname, fname)] = int(value)
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def test_quantize_rejects_bad_sizes_without_touching_the_gpu():
    lib = _lib.load()
    st = lib.asterq_quantize(None, _lib.DTYPE_BF16, -1, 512, 512, _lib.SCHEME_HADAMARD_INT4, 64, None, None, None)
    assert st == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert b"bad sizes" in lib.asterq_last_error()
    st = lib.asterq_quantize(None, _lib.DTYPE_BF16, 4, 512, 100, _lib.SCHEME_HADAMARD_INT4, 64, None, None, None)
    assert st == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    # zero tokens is a valid no-op
    assert lib.asterq_quantize(None, _lib.DTYPE_BF16, 0, 512, 512, 0, 64, None, None, None) == _lib.ASTERQ_OK
    st = lib.asterq_fwht(None, None, 4, 48, None)
    assert st == _lib.ASTERQ_ERR_INVALID_ARGUMENT


def test_combine_ranks_rejects_bad_arguments_without_touching_the_gpu():
    lib = _lib.load()
    f32 = _lib.DTYPE_F32
    assert lib.asterq_splitkv_combine_ranks(None, 2, 1, None, 256, None, f32, None) == _lib.ASTERQ_ERR_UNSUPPORTED
    assert lib.asterq_splitkv_combine_ranks(None, 0, 1, None, 512, None, f32, None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_splitkv_combine_ranks(None, 2, -1, None, 512, None, f32, None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_splitkv_combine_ranks(None, 2, 1, None, 512, None, f32, None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert b"null pointer" in lib.asterq_last_error()
    assert lib.asterq_splitkv_combine_ranks(16, 2, 1, 16, 512, 16, 7, None) == _lib.ASTERQ_ERR_UNSUPPORTED
    assert lib.asterq_splitkv_combine_ranks(8, 2, 1, 16, 512, 16, f32, None) == _lib.ASTERQ_ERR_MISALIGNED
    # no row blocks is a valid no-op
    assert lib.asterq_splitkv_combine_ranks(None, 2, 0, None, 512, None, f32, None) == _lib.ASTERQ_OK


def _params(**kw) -> _lib.DecodeParams:
    p = _lib.DecodeParams()
    p.n_heads, p.latent_dim, p.rope_dim, p.group_size, p.page_tokens = 16, 512, 64, 64, 512
    p.out_dtype = _lib.DTYPE_F32
    p.softmax_scale = 1.0
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize(
    "kw,status",
    [
        (dict(latent_dim=256), _lib.ASTERQ_ERR_UNSUPPORTED),
        (dict(rope_dim=32), _lib.ASTERQ_ERR_UNSUPPORTED),
        (dict(page_tokens=100), _lib.ASTERQ_ERR_UNSUPPORTED),
        (dict(page_tokens=0), _lib.ASTERQ_ERR_UNSUPPORTED),
        (dict(out_dtype=_lib.DTYPE_F16), _lib.ASTERQ_ERR_UNSUPPORTED),
        (dict(n_heads=0), _lib.ASTERQ_ERR_INVALID_ARGUMENT),
        (dict(n_items=3), _lib.ASTERQ_ERR_INVALID_ARGUMENT),  # null tables
        (dict(n_slots=2, n_items=0), _lib.ASTERQ_ERR_WORKSPACE),
        (dict(n_items=1, items=8, tiles=16, q_lat=16, q_rope=16, out=16), _lib.ASTERQ_ERR_MISALIGNED),
        (dict(n_workers=4), _lib.ASTERQ_ERR_INVALID_ARGUMENT),  # a worker count without a workers table
        (dict(n_workers=-1), _lib.ASTERQ_ERR_INVALID_ARGUMENT),
        (dict(n_workers=1, workers=18), _lib.ASTERQ_ERR_MISALIGNED),
        (dict(unit_jobs=6), _lib.ASTERQ_ERR_MISALIGNED),
        (dict(n_combine_total=-1), _lib.ASTERQ_ERR_INVALID_ARGUMENT),
    ],
)
def test_decode_validation(kw, status):
    lib = _lib.load()
    p = _params(**kw)
    assert lib.asterq_latent_decode(ctypes.byref(p), None) == status
    assert lib.asterq_last_error()


def test_decode_noop_and_workspace_query():
    lib = _lib.load()
    p = _params()
    assert lib.asterq_latent_decode(ctypes.byref(p), None) == _lib.ASTERQ_OK
    p.n_slots = 3
    assert lib.asterq_decode_workspace_bytes(ctypes.byref(p)) == 3 * 16 * 514 * 4
    # + the prepared query blocks and one counter per unit (fused combine), rounded to 16 bytes
    p.n_units = 5
    assert lib.asterq_decode_workspace_bytes(ctypes.byref(p)) == 3 * 16 * 514 * 4 + 5 * 37376 + 32


def test_plan_workspace_matches_the_library():
    from asterq.plan import SequenceLayout, build_plan

    lib = _lib.load()
    seqs = [SequenceLayout(cold=[(i, 0, 512)] * (4 * i + 1), hot=[(i, 0, 200)], q_start=i, q_len=1 + (i % 3))
            for i in range(9)]
    for kw in (dict(), dict(n_sms=8), dict(persistent=False)):
        plan = build_plan(seqs, 16, **kw)
        p = _params(n_slots=plan.n_slots, n_units=plan.n_units)
        assert lib.asterq_decode_workspace_bytes(ctypes.byref(p)) == plan.workspace_bytes


def test_check_maps_status_to_exception_types():
    lib = _lib.load()
    lib.asterq_fwht(None, None, 1, 3, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.ASTERQ_ERR_INVALID_ARGUMENT)
    with pytest.raises(_lib.AsterqError):
        _lib.check(_lib.ASTERQ_ERR_UNSUPPORTED)


def test_plan_and_append_reject_bad_arguments_without_touching_the_gpu():
    lib = _lib.load()
    d = _lib.BatchDesc()
    d.n_seqs, d.n_heads, d.page_tokens, d.n_workers = 2, 16, 512, 148
    b = _lib.PlanBuffers()
    assert lib.asterq_plan_batch(None, ctypes.byref(b), None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert b"null sequence table" in lib.asterq_last_error()
    for name in ("n_cold_pages", "cold_pages", "cold_page_tokens", "hot_tokens", "hot_pages", "q_len", "q_start"):
        setattr(d, name, 16)
    d.max_cold_pages, d.max_hot_pages = 4, 4
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert b"null plan buffer" in lib.asterq_last_error()
    for name in ("tiles", "units", "items", "combine", "unit_jobs", "workers", "counts", "scratch"):
        setattr(b, name, 32)
    b.items = 40
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_MISALIGNED
    d.page_tokens = 100
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_UNSUPPORTED
    assert lib.asterq_plan_scratch_bytes(ctypes.byref(d), -1, 4, 4) == 0
    d.page_tokens = 512
    d.n_workers = 0
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_plan_scratch_bytes(ctypes.byref(d), 4, 4, 4) == 0
    d.n_workers = 148
    d.cold_tile_tokens = 32  # cold tiles of 0 (= 128), 64 or 128 tokens only
    assert lib.asterq_plan_batch(ctypes.byref(d), ctypes.byref(b), None) == _lib.ASTERQ_ERR_UNSUPPORTED
    assert b"cold_tile_tokens" in lib.asterq_last_error()
    d.cold_tile_tokens = 0
    # scratch: tile costs, segment and per-unit prefix arrays (int64), per-boundary and per-item int32
    n_segs = 2 * (4 + 2)
    want = 8 * (10 + 1 + n_segs + 1 + 2 + 1 + 6 * (3 + 1) + 148 + 1) + 4 * (3 * 148 + 5)
    assert lib.asterq_plan_scratch_bytes(ctypes.byref(d), 10, 3, 5) == want
    # append: null and misaligned arrays
    assert lib.asterq_batch_append(ctypes.byref(d), None, 16, 16, 2, 16, 16, 8, None, None) == \
        _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_batch_append(ctypes.byref(d), 16, 16, 16, -1, 16, 16, 8, None, None) == \
        _lib.ASTERQ_ERR_INVALID_ARGUMENT
    assert lib.asterq_batch_append(ctypes.byref(d), 16, 16, 24, 2, 16, 16, 8, None, None) == _lib.ASTERQ_ERR_MISALIGNED
    d.n_seqs = 0  # nothing to append is a valid no-op
    assert lib.asterq_batch_append(ctypes.byref(d), None, None, None, 0, None, None, 0, None, None) == _lib.ASTERQ_OK
