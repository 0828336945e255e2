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


# ---------------------------------------------------------------------------
# The Rust binding of INTEGRATION.md, translated to C and checked against the header
# ---------------------------------------------------------------------------

_RS_BASE = {"i32": "int32_t", "i64": "int64_t", "u32": "uint32_t", "u8": "uint8_t", "i8": "int8_t", "f32": "float",
            "f64": "double", "usize": "size_t", "c_void": "void", "c_char": "char", "VcCtx": "vc_ctx",
            "VcTreeSet": "vc_tree_set", "VcKvDesc": "vc_kv_desc", "VcTraceDesc": "vc_trace_desc",
            "VcKvtDesc": "vc_kvt_desc"}


def _rs_to_c(t: str) -> str:
    """Rust FFI type -> C type; ``*const T`` is a pointer to const T (postfix const)."""
    t = t.strip()
    if t.startswith("*const "):
        return _rs_to_c(t[len("*const "):]) + " const*"
    if t.startswith("*mut "):
        return _rs_to_c(t[len("*mut "):]) + "*"
    return _RS_BASE[t]


def _rust_block():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return re.search(r"```rust\n(.*?)```", text, flags=re.S).group(1)


def _rust_structs(src):
    out = {}
    for name, body in re.findall(r"#\[repr\(C\)\]\s*pub struct (\w+) \{(.*?)\}", src, flags=re.S):
        fields = re.findall(r"pub (\w+): ([^,]+?)\s*(?:,|$)", body, flags=re.M)
        if fields:
            out[name] = fields
    return out


def _rust_fns(src):
    block = re.search(r'extern "C" \{(.*?)\n\}', src, flags=re.S).group(1)
    fns = []
    for name, args, ret in re.findall(r"fn (\w+)\((.*?)\)\s*->\s*(\w+);", block, flags=re.S):
        params = [tuple(x.strip() for x in a.split(":", 1)) for a in re.split(r",\s*", " ".join(args.split())) if a]
        fns.append((name, params, ret))
    return fns


def test_rust_binding_covers_every_export():
    fns = {f[0] for f in _rust_fns(_rust_block())}
    assert fns == set(header_symbols()) - {"vc_int_peak", "vc_wait_probe"}


def test_rust_binding_matches_header_and_fails_closed(tmp_path):
    """Every declaration of the Rust block, translated to C, is redeclared after
    including vcommit.h (a type mismatch does not compile), every struct's size
    and field offsets equal the header's, and every call with NULL arguments
    returns VC_EINVAL (the context / tree-set destructors and counters: their no-op)."""
    src = _rust_block()
    lines = ["#include <stddef.h>", "#include <stdio.h>", "#include <stdint.h>", '#include "vcommit.h"']
    for name, fields in _rust_structs(src).items():
        cname = _RS_BASE[name]
        lines.append(f"struct rs_{name} {{")
        lines += [f"  {_rs_to_c(t)} {f};" for f, t in fields]
        lines.append("};")
        lines.append(f"_Static_assert(sizeof(struct rs_{name}) == sizeof({cname}), \"{name} size\");")
        for f, _t in fields:
            lines.append(f"_Static_assert(offsetof(struct rs_{name}, {f}) == offsetof({cname}, {f}), "
                         f"\"{name}.{f} offset\");")
    fns = _rust_fns(src)
    for name, params, ret in fns:
        args = ", ".join(f"{_rs_to_c(t)} {p}" for p, t in params) or "void"
        lines.append(f"{_RS_BASE[ret]} {name}({args});")
    lines.append("int main(void) {")
    for name, params, _ret in fns:
        call_args = ", ".join("0" if not t.startswith("*") else "NULL" for _p, t in params)
        lines.append(f'  printf("{name} %lld\\n", (long long){name}({call_args}));')
    lines += ["  return 0;", "}"]
    c = tmp_path / "rs_binding.c"
    c.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "rs_binding"
    libdir = os.path.dirname(_lib.lib()._name)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(c), "-o", str(exe),
                    "-L", libdir, "-lvcommit", f"-Wl,-rpath,{libdir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = dict(l.split() for l in out if l)
    want_zero = {"vc_ctx_destroy", "vc_tree_set_free", "vc_tree_set_count"}
    for name, _params, _ret in fns:
        if name == "vc_abi_version":
            assert int(got[name]) == 2
        elif name == "vc_last_error":
            assert int(got[name]) >= 0
        elif name in want_zero:
            assert int(got[name]) == 0, name
        else:
            assert int(got[name]) == _lib.VC_EINVAL, (name, got[name])
