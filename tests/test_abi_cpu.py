"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, keeps the reference descriptor layouts and workspace formulas,
and rejects bad descriptors before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from glmaxx_b200 import abi

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "glmaxx_kernel.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(glmaxx_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = abi.load()
    names = declared_functions()
    assert len(names) >= 55
    for n in names:
        assert hasattr(lib, n), f"missing export {n}"
        assert n in abi.SIGNATURES, f"binding lacks {n}"


def test_descriptor_layouts():
    for cls, size in abi.EXPECTED_SIZES.items():
        assert ctypes.sizeof(cls) == size
        d = cls.new()
        assert ctypes.addressof(d) % 16 == 0 and d.struct_bytes == size


def test_abi_strings():
    assert abi.abi_string() == "glmaxx.sm100.nvfp4.routed_moe.v3"
    assert abi.load().glmaxx_exl3_kernel_abi().decode().startswith("glmaxx.sm100.exl3")


def _rust_workspace(a):  # crates/glm-cuda/src/abi.rs:454-479
    p = (a + 127) // 128 * 128
    return a * 6144 * 2 + p * 3072 + p * 384 + a * 4 + a * 1024 * 4 + 257 * 4


def _rust_grouped(a):  # abi.rs:481-494, 77-91
    p = (a + 127) // 128 * 128
    return _rust_workspace(a) - p * 384 + (a + 127 * min(a, 256)) * 384


def _rust_fc2(r, a):  # abi.rs:496-547
    p = (a + 127) // 128 * 128
    return p * 256 + p * 32 + a * 4 + a * 6144 * 4 + a * 6144 * 2 + r * 6144 * 4 + r * 8 * 4 + 4


def _rust_fc2_grouped(r, a):  # abi.rs:549-559
    p = (a + 127) // 128 * 128
    return _rust_fc2(r, a) - p * 32 + (a + 127 * min(a, 256)) * 32


@pytest.mark.parametrize("a", [1, 8, 127, 128, 129, 512, 2043, 65535])
def test_reference_workspace_formulas(a):
    L = abi.load()
    assert L.glmaxx_nvfp4_routed_fc1_workspace_bytes(a) == _rust_workspace(a)
    assert L.glmaxx_nvfp4_grouped_workspace_bytes(a) == _rust_grouped(a)
    rows = (a + 7) // 8
    assert L.glmaxx_nvfp4_routed_fc2_workspace_bytes(rows, a) == _rust_fc2(rows, a)
    assert L.glmaxx_nvfp4_grouped_fc2_workspace_bytes(rows, a) == _rust_fc2_grouped(rows, a)


def test_exl3_workspace_formula():
    L = abi.load()
    assert L.glmaxx_exl3_projection_workspace_bytes(8, 6144, 512) == 8 * (6144 + 512) * 2
    assert L.glmaxx_exl3_projection_workspace_bytes(0, 6144, 512) == 0


def test_launches_reject_null_and_bad_descriptors_without_a_device():
    L = abi.load()
    err = ctypes.c_int32(7)
    s = ctypes.c_void_p(1)
    assert L.glmaxx_nvfp4_routed_fc1_launch(None, s, ctypes.byref(err)) == -1
    assert L.glmaxx_nvfp4_routed_fc2_launch(None, s, ctypes.byref(err)) == -1
    assert L.glmaxx_moe_layer_launch(None, s, ctypes.byref(err)) == -1
    d = abi.Fc1Descriptor.new(abi_version=1)  # geometry missing
    assert L.glmaxx_nvfp4_routed_fc1_launch(ctypes.byref(d), s, ctypes.byref(err)) == -2
    assert err.value == 0
    m = abi.MoeLayerDescriptor.new(abi_version=3, tokens=64, hidden=6144, experts=256,
                                   local_intermediate=2048, top_k=8, groups=8, topk_groups=4,
                                   route_scale=2.5)
    assert L.glmaxx_moe_layer_launch(ctypes.byref(m), s, ctypes.byref(err)) == -2  # no pointers
    m.reserved0[1] = 1
    assert L.glmaxx_moe_layer_launch(ctypes.byref(m), s, ctypes.byref(err)) == -2
    x = abi.Exl3Descriptor.new(abi_version=1, projection=9)
    assert L.glmaxx_exl3_projection_launch(ctypes.byref(x), s, ctypes.byref(err)) == -2


def test_layer_workspace_grows_with_tokens():
    L = abi.load()

    def ws(t, path):
        d = abi.MoeLayerDescriptor.new(abi_version=3, tokens=t, hidden=6144, experts=256,
                                       local_intermediate=2048, top_k=8, groups=8,
                                       topk_groups=4, route_scale=2.5, path=path)
        return L.glmaxx_moe_layer_workspace_bytes(ctypes.byref(d))

    assert 0 < ws(8, 1) < ws(64, 1) < ws(8192, 2)
