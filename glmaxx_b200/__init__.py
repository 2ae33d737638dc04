"""B200-native (sm_100a) routed-MoE hot path of yatesdr/glmaxx.

The product is libglmaxx_sm100.so (glmaxx_b200/csrc, C ABI in
include/glmaxx_kernel.h); this package is its Python host side:
``abi`` (ctypes binding), ``moe`` (layer object), ``synth`` (seeded synthetic
workloads), ``tp`` (tensor-parallel sharding and the partial-sum all-reduce).
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
