"""The Rust glm-cuda backend (rust/glm-cuda-sm100) against the C ABI it binds.

No Rust toolchain exists here, so the crate is checked as text: every C
prototype of include/glmaxx_kernel.h has a `pub fn` of the same name and
parameter count in ffi.rs (and the reverse), every bound name is exported by
libglmaxx_sm100.so, and every repr(C) struct of abi.rs has the C struct's fields
in the same order with the same widths (so the same offsets and size)."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include/glmaxx_kernel.h"
CRATE = ROOT / "rust/glm-cuda-sm100/src"
LIB = ROOT / "glmaxx_b200/libglmaxx_sm100.so"

C_WIDTH = {"uint32_t": 4, "int32_t": 4, "float": 4, "uint64_t": 8}
RUST_WIDTH = {"u32": 4, "i32": 4, "f32": 4, "u64": 8}
STRUCTS = {"glmaxx_router_descriptor": "RouterDescriptor",
           "glmaxx_moe_exl3_experts": "MoeExl3Experts",
           "glmaxx_moe_layer_descriptor": "MoeLayerDescriptor",
           "glmaxx_moe_finish_descriptor": "MoeFinishDescriptor",
           "glmaxx_moe_peer_descriptor": "MoePeerDescriptor",
           "glmaxx_moe_ep_descriptor": "MoeEpDescriptor"}


def _strip_c(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def _c_prototypes():
    s = _strip_c(HEADER.read_text())
    out = {}
    for m in re.finditer(r"\n(?:const )?[\w ]+?\*?\s*(glmaxx_\w+)\s*\(([^;]*?)\);", s):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def _rust_fns():
    s = (CRATE / "ffi.rs").read_text()
    out = {}
    for m in re.finditer(r"pub fn (glmaxx_\w+)\s*\((.*?)\)\s*(?:->[^;]*)?;", s, flags=re.S):
        params = [p for p in m.group(2).replace("\n", " ").split(",") if p.strip()]
        out[m.group(1)] = len(params)
    return out


def _c_fields(name):
    s = _strip_c(HEADER.read_text())
    body = re.search(r"struct (?:alignas\(16\) )?%s \{(.*?)\};" % name, s, flags=re.S).group(1)
    fields = []
    for ty, field, arr in re.findall(r"(\w+)\s+(\w+)(?:\[(\d+)\])?;", body):
        fields.append((field, C_WIDTH[ty] * (int(arr) if arr else 1), C_WIDTH[ty]))
    return fields


def _rust_fields(name):
    s = (CRATE / "abi.rs").read_text()
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, s, flags=re.S).group(1)
    fields = []
    for field, ty in re.findall(r"pub (\w+): ([^,]+),", body):
        ty = ty.strip()
        m = re.fullmatch(r"\[(\w+); (\d+)\]", ty)
        if m:
            fields.append((field, RUST_WIDTH[m.group(1)] * int(m.group(2)), RUST_WIDTH[m.group(1)]))
        else:
            fields.append((field, RUST_WIDTH[ty], RUST_WIDTH[ty]))
    return fields


def _layout(fields):
    off, offsets = 0, []
    for _, size, align in fields:
        off = (off + align - 1) // align * align
        offsets.append(off)
        off += size
    return offsets, (off + 15) // 16 * 16


def test_every_c_entry_point_is_bound_with_its_arity():
    c, r = _c_prototypes(), _rust_fns()
    assert len(c) >= 70
    assert set(c) == set(r), (sorted(set(c) - set(r)), sorted(set(r) - set(c)))
    for name, n in c.items():
        assert r[name] == n, (name, n, r[name])


def test_bound_names_are_exported_by_the_library():
    if not LIB.exists():
        pytest.skip("library not built")
    nm = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r"\b(glmaxx_\w+)\b", nm))
    missing = set(_rust_fns()) - exported
    assert not missing, sorted(missing)


@pytest.mark.parametrize("c_name,rust_name", sorted(STRUCTS.items()))
def test_struct_layouts_match(c_name, rust_name):
    cf, rf = _c_fields(c_name), _rust_fields(rust_name)
    assert [f[0] for f in cf] == [f[0] for f in rf]
    assert [f[1] for f in cf] == [f[1] for f in rf]
    c_off, c_size = _layout(cf)
    r_off, r_size = _layout(rf)
    assert c_off == r_off and c_size == r_size
    asserted = re.search(r"sizeof\(%s\) == (\d+)" % c_name, HEADER.read_text())
    if asserted:
        assert c_size == int(asserted.group(1))
    rust_assert = re.search(r"size_of::<%s>\(\) == (\d+)" % rust_name,
                            (CRATE / "abi.rs").read_text())
    assert rust_assert and int(rust_assert.group(1)) == r_size
