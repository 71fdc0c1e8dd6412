"""The C-ABI library loads on a CPU host, exports every symbol the header declares, and
the structs the host passes by value have the header's layout."""

import ctypes
import re
from pathlib import Path

import pytest

from oscar_new_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "oscar_b200.h").read_text()
    return sorted(set(re.findall(r"^(?:int|int64_t) (oscar_\w+)\(", text, flags=re.M)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.exported_symbols())


def test_library_loads_and_exports_every_symbol():
    handle = _lib.lib()
    for name in declared_symbols():
        assert hasattr(handle, name), name
    assert handle.oscar_version() == 100


def test_invalid_arguments_are_rejected_without_launch():
    handle = _lib.lib()
    geo = _lib.Geometry(kv_heads=4, group=6, head_dim=128, block_tokens=768, kernel_block=128, slot_bytes=160,
                        vector_bytes=68, sink=4, recent=128, ring=129, table_stride=8, query_tile=4,
                        page_bytes=768 * 4 * 256 * 2)
    clip = _lib.Clip(enabled=0, mode=0, asc_lo=0, asc_hi=0, weight=0.0, factor=1.0)
    # head_dim != 256 is refused before any device work
    assert handle.oscar_store_int2(None, None, 4, None, None, None, geo, clip, clip, None) == 1
    assert handle.oscar_jacobi_rotations(None, 1, 0, 1e-6, None, None, None, None) == 1
    assert handle.oscar_jacobi_rotations(None, (1 << 20) + 1, 12, 1e-6, None, None, None, None) == 1
    assert handle.oscar_jacobi_rotations(None, 0, 12, 1e-6, None, None, None, None) == 0  # nothing to do
    assert handle.oscar_rotate(None, 0, 1, 0, 0, 1, None, 0, 0, None, None) == 1


def test_metadata_staging_rejects_inconsistent_steps_without_launch():
    """oscar_stage_step_metadata checks the step against the arena before any device
    work: more requests / tokens / columns than the arena holds, missing sources."""
    h = _lib.lib()
    fake = 1 << 20  # never dereferenced: every call below is refused first
    args = dict(qs=fake, sl=fake, tb=fake, ts=40, sm=fake, nr=3, nt=3, cc=17, tile=4, arena=fake, mr=5, cols=39,
                cap=19, so=fake, scap=40)

    def call(**kw):
        a = {**args, **kw}
        return h.oscar_stage_step_metadata(a["qs"], a["sl"], a["tb"], a["ts"], a["sm"], a["nr"], a["nt"], a["cc"],
                                           a["tile"], a["arena"], a["mr"], a["cols"], a["cap"], a["so"], a["scap"],
                                           None)

    assert call(nr=6) == 1              # more requests than the arena
    assert call(nt=41) == 1             # more tokens than the slot buffer
    assert call(cc=40) == 1             # more columns than the table
    assert call(qs=None) == 1           # requests without query starts
    assert call(sm=None) == 1           # tokens without a slot mapping
    assert call(ts=10) == 1             # a source row shorter than the columns copied
    assert call(arena=None) == 1
    assert call(tile=0) == 1
    offsets = (ctypes.c_int64 * 5)()
    assert h.oscar_step_arena_layout(0, 39, 19, ctypes.addressof(offsets)) == 1
    assert h.oscar_step_arena_layout(5, 39, 19, ctypes.addressof(offsets)) == 0
    assert list(offsets) == [4, 12, 20, 216, 256]


def test_sst_weights_reject_keys_that_are_not_16_byte_rows():
    """The SST entry points read key rows as 16-byte vectors: a key pointer off a 16-byte
    boundary or strides that are not multiples of 8 elements are refused before any
    device work (the pointers here are host placeholders and are never dereferenced)."""
    handle = _lib.lib()
    buf = (ctypes.c_char * 256)()
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    ok_ptr, off_ptr = base, base + 2
    for fn in (handle.oscar_sst_weights, handle.oscar_sst_weights_per_head):
        assert fn(off_ptr, 1, 1, 256, 256, ok_ptr, ok_ptr, ok_ptr, None) == 1
        assert fn(ok_ptr, 1, 1, 260, 256, ok_ptr, ok_ptr, ok_ptr, None) == 1
        assert fn(ok_ptr, 1, 1, 256, 260, ok_ptr, ok_ptr, ok_ptr, None) == 1
        assert fn(ok_ptr, 0, 1, 260, 260, ok_ptr, ok_ptr, ok_ptr, None) == 0  # nothing to do
    split = handle.oscar_sst_weights_split  # pre-split covariances, nullable status word
    assert split(off_ptr, 1, 1, 256, 256, ok_ptr, ok_ptr, ok_ptr, None, None) == 1
    assert split(ok_ptr, 1, 1, 260, 256, ok_ptr, ok_ptr, ok_ptr, None, None) == 1
    assert split(ok_ptr, 1, 0, 256, 256, ok_ptr, ok_ptr, ok_ptr, None, None) == 1
    assert split(ok_ptr, 0, 1, 260, 260, ok_ptr, ok_ptr, ok_ptr, None, None) == 0
    assert handle.oscar_split_bf16x3(ok_ptr, -1, ok_ptr, None) == 1
    assert handle.oscar_split_bf16x3(ok_ptr, 1, off_ptr, None) == 1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_PATH", tmp_path / "liboscar_b200.so")
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="not built"):
        _lib.lib()


@pytest.mark.parametrize("status,text", [(1, "invalid argument"), (2, "launch error"), (3, "unsupported"),
                                         (4, "device wait timeout")])
def test_nonzero_status_raises_with_its_name(status, text):
    with pytest.raises(RuntimeError, match=f"^oscar_store_int2 failed: {text}$"):
        _lib.check(status, "oscar_store_int2")
    _lib.check(0, "oscar_store_int2")


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """sizeof / offsetof of oscar_geometry and oscar_clip as gcc lays them out from the
    header, against the ctypes structures the host passes by value."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    fields = {"oscar_geometry": _lib.Geometry, "oscar_clip": _lib.Clip}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "oscar_b200.h"', "int main(void) {"]
    for cname, cls in fields.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                              check=True).stdout.splitlines())
    for cname, cls in fields.items():
        assert int(got[f"{cname} size"]) == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert int(got[f"{cname} {fname}"]) == getattr(cls, fname).offset, (cname, fname)


def _ctype_of(param: str):
    """ctypes class of one C parameter declaration of the header."""
    p = " ".join(param.replace("const ", "").split())
    if "*" in p:
        return ctypes.c_void_p
    kind = p.rsplit(" ", 1)[0] if " " in p else p
    return {"int32_t": ctypes.c_int32, "uint32_t": ctypes.c_uint32, "int64_t": ctypes.c_int64, "float": ctypes.c_float,
            "oscar_geometry": _lib.Geometry, "oscar_clip": _lib.Clip, "void": None}[kind]


def test_binding_argument_types_follow_the_header_prototypes():
    text = (ROOT / "include" / "oscar_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    protos = re.findall(r"^(int|int64_t) (oscar_\w+)\((.*?)\);", text, flags=re.M | re.S)
    assert protos
    for ret, name, params in protos:
        want = [t for t in (_ctype_of(x) for x in params.split(",")) if t is not None]
        got = _lib._SIGNATURES[name]
        assert len(got) == len(want), (name, len(got), len(want))
        for i, (g, w) in enumerate(zip(got, want)):
            assert g is w, (name, i, g, w)
        assert _lib._RESTYPES.get(name, ctypes.c_int) is (ctypes.c_int64 if ret == "int64_t" else ctypes.c_int), name


def test_sst_preparation_refuses_host_tensors_and_foreign_parts():
    """The tensor-core SST path is device-only, and its prepared covariances must be the
    [h, 3, 256, 256] bf16 split of the same covariances (checked before any launch)."""
    import torch

    from oscar_new_b200 import calibration_kernels as ck

    with pytest.raises(RuntimeError, match="CUDA"):
        ck.prepare_sst_covariances(torch.zeros(2, 256, 256))
    with pytest.raises(RuntimeError, match="CUDA"):
        ck.sst_weights_per_head(torch.zeros(4, 2, 256, dtype=torch.bfloat16), torch.zeros(2, 256, 256),
                                torch.zeros(2), prepared=torch.zeros(2, 3, 256, 256, dtype=torch.bfloat16))
