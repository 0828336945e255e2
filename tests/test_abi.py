"""The C ABI library: it loads, exports every symbol the header declares, and
the ctypes descriptor layouts match the C structs (CPU only, no compute)."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from commitllm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vcommit.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^VC_API\s+\w+\s+(vc_\w+)\(", text, flags=re.M)))


def test_header_declares_the_binding_symbols():
    assert header_symbols() == sorted(_lib.SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    lib = _lib.lib()
    for s in header_symbols():
        assert hasattr(lib, s), s
    assert lib.vc_abi_version() == 2


def test_last_error_is_empty_before_any_failure():
    assert isinstance(_lib.last_error(), str)


def _c_layout(struct, fields):
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"vcommit.h\"\nint main(void){\n"
    src += f'printf("%zu\\n", sizeof({struct}));\n'
    for f in fields:
        src += f'printf("%zu\\n", offsetof({struct}, {f}));\n'
    src += "return 0;}\n"
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "l.c")
        exe = os.path.join(d, "l")
        open(c, "w").write(src)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    return [int(x) for x in out]


@pytest.mark.parametrize("cls,cname", [(_lib.KvDesc, "vc_kv_desc"), (_lib.TraceDesc, "vc_trace_desc"),
                                      (_lib.KvtDesc, "vc_kvt_desc")])
def test_struct_layouts_match_header(cls, cname):
    names = [f[0] for f in cls._fields_]
    want = _c_layout(cname, names)
    assert want[0] == ctypes.sizeof(cls)
    assert want[1:] == [getattr(cls, n).offset for n in names]
