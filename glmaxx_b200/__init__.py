"""B200-native (sm_100a) routed-MoE hot path of yatesdr/glmaxx.

The product is libglmaxx_sm100.so (glmaxx_b200/csrc; C ABI in
include/glmaxx_kernel.h and include/glmaxx_rank_file.h); this package is its
Python host side:

- ``abi``: ctypes binding of glmaxx_kernel.h;
- ``moe``: the rank-local routed-MoE layer object and the sparse-layer finish;
- ``graphs``: per-row-bucket CUDA graphs of the layer;
- ``peer``: the tensor-parallel peer finish over CUDA IPC mappings;
- ``rank_file``: the native .g5n rank-file reader, writer and layer loader;
- ``synth``: seeded synthetic weights and inputs of the benchmark configs;
- ``build``: the in-tree nvcc / g++ build of the library;
- ``profile_case``, ``peer_bench``: targets for ncu captures and reduce timing.
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
