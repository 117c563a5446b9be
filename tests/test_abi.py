"""The C-ABI library loads and exports every entry point include/kq.h declares. No compute: these
run without a GPU."""
import ctypes
import os
import re
import subprocess

import oracle

import kernite_b200 as kb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions() -> set[str]:
    names = set()
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(kq_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    L = kb.lib()
    declared = header_functions()
    assert declared, "no declarations found in include/"
    missing = [n for n in sorted(declared) if not hasattr(L, n)]
    assert not missing, missing


def test_python_binding_lists_every_declared_symbol():
    assert header_functions() == set(kb.EXPORTS)


def test_stream_key_matches_oracle():
    for seed, t in [(0, 0), (1234, 7), (2**63 + 5, 99)]:
        assert kb.stream_key(seed, t) == oracle.stream_key(seed, t)


def test_last_error_is_a_string():
    assert isinstance(kb.last_error(), str)


def test_ctx_create_rejects_null_out():
    L = kb.lib()
    rc = L.kq_ctx_create(0, None)
    assert rc == kb.KQ_E_INVALID
    assert "kq_ctx_create" in kb.last_error()


def test_entry_points_reject_null_ctx():
    L = kb.lib()
    assert L.kq_matvec_q4k(None, 0, 0, 0, 1, 256, 1, None) == kb.KQ_E_INVALID
    for name in ("kq_dequant_q4k", "kq_dequant_q5k", "kq_dequant_q6k", "kq_dequant_q2k",
                 "kq_dequant_q3k", "kq_dequant_q8_0"):
        assert getattr(L, name)(None, 0, 0, 1, None) == kb.KQ_E_INVALID, name
    for name in ("kq_fill_q5k", "kq_fill_q6k"):
        assert getattr(L, name)(None, 0, 0, 1, 0, None) == kb.KQ_E_INVALID, name
    assert L.kq_fill_q4k(None, 0, 0, 1, 0, None) == kb.KQ_E_INVALID
    d = kb.KqMatvecDesc()
    assert L.kq_matvec(None, ctypes.byref(d), None) == kb.KQ_E_INVALID


def test_desc_layout_matches_header(tmp_path):
    # the C compiler's layout of kq_matvec_desc against the ctypes mirror
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "kq.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu\\n", sizeof(kq_matvec_desc),'
        ' offsetof(kq_matvec_desc, y), offsetof(kq_matvec_desc, prologue),'
        ' offsetof(kq_matvec_desc, eps), offsetof(kq_matvec_desc, flags));return 0;}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    D = kb.KqMatvecDesc
    assert got == [ctypes.sizeof(D), D.y.offset, D.prologue.offset, D.eps.offset, D.flags.offset]


def test_module_image_is_an_sm100a_cubin():
    import struct

    img = kb.module_image()
    assert img[:4] == b"\x7fELF" and len(img) > 100_000
    # ELF64 header: e_machine at 18 is EM_CUDA (190); the CUDA ELF's e_flags hold the SM (100)
    assert img[4] == 2 and struct.unpack_from("<H", img, 18)[0] == 190
    flags = struct.unpack_from("<I", img, 48)[0]
    assert (flags & 0xFF) == 100 or ((flags >> 8) & 0xFF) == 100, hex(flags)


def test_launch_struct_layout_matches_header(tmp_path):
    src = tmp_path / "launch.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "kq.h"\n'
        'int main(void){printf("%zu %zu %zu %zu %zu\\n", sizeof(kq_launch), offsetof(kq_launch, grid),'
        ' offsetof(kq_launch, shared_bytes), offsetof(kq_launch, params), sizeof(kq_chain_job));return 0;}\n')
    exe = tmp_path / "launch"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    L = kb.KqLaunch
    assert got == [ctypes.sizeof(L), L.grid.offset, L.shared_bytes.offset, L.params.offset,
                   ctypes.sizeof(kb.KqChainJob)]
